"""The C++ host driver (index-tts2-metal_b200/cli/mtts_cfm.cpp, built on the
header-only shim include/itts_cfm.hpp) produces exactly what the C ABI
produces, and its --bench-cfm mode mirrors the reference CLI's report."""
from __future__ import annotations

import json
import subprocess
from pathlib import Path

import numpy as np
import pytest

import workloads as W

pytestmark = pytest.mark.gpu

CLI = Path(__file__).resolve().parent.parent / "index-tts2-metal_b200" / "lib" / "mtts_cfm"


def test_cli_cfm_matches_capi(ctx_unit, unit_bundle, tmp_path, rng):
    T, P, steps, cfg = 40, 9, 3, 0.7
    u = W.utterance(rng, T, P)
    pre = tmp_path / "in"
    for name, arr in (("noise", u.noise), ("prompt", u.prompt), ("cond", u.cond), ("style", u.style)):
        np.ascontiguousarray(arr, np.float32).tofile(f"{pre}.{name}.f32")
    out = tmp_path / "mel.f32"
    r = subprocess.run([str(CLI), "--cfm", str(unit_bundle), str(T), str(P), str(steps), str(cfg), str(pre), str(out)],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    mel = np.fromfile(out, np.float32).reshape(T, 80)
    ref = ctx_unit.run(u.noise, u.prompt, u.cond, u.style, steps, cfg)
    assert np.array_equal(mel, ref)


def test_cli_bench_cfm_report(unit_bundle):
    r = subprocess.run([str(CLI), "--bench-cfm", str(unit_bundle), "70", "2", "2"], capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stderr
    rep = json.loads(r.stdout)
    assert rep["stage"] == "bench_cfm" and rep["tokens"] == 70 and rep["steps"] == 2
    assert rep["ms_per_step"] > 0 and np.isfinite(rep["mel_checksum"])


def test_cli_rejects_bad_bundle(tmp_path):
    r = subprocess.run([str(CLI), "--bench-cfm", str(tmp_path / "nope"), "8", "1", "1"], capture_output=True, text=True,
                       timeout=120)
    assert r.returncode == 1 and "itts_cfm_create" in r.stderr


@pytest.mark.parametrize("sampled", [False, True])
def test_cli_gpt_matches_capi(gpt_bundle, tmp_path, sampled):
    """--gpt (generate-style positions, as the synthesis pipeline calls the
    decoder): the codes the C++ driver writes equal the C ABI's, greedy and
    sampled."""
    import itts_cfm

    P, steps = 7, 9
    prefix = np.random.default_rng(77).standard_normal((P, 1280)).astype(np.float32)
    pre, out = tmp_path / "prefix.f32", tmp_path / "codes.u32"
    prefix.tofile(pre)
    cfg = dict(seed=99, temperature=0.8, top_k=30, top_p=0.8, repetition_penalty=10.0)
    extra = [str(cfg[k]) for k in ("seed", "temperature", "top_k", "top_p", "repetition_penalty")] if sampled else []
    r = subprocess.run([str(CLI), "--gpt", str(gpt_bundle), str(P), str(steps), str(pre), str(out)] + extra,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr
    rep = json.loads(r.stdout)
    codes = np.fromfile(out, np.uint32).tolist()
    assert rep["codes"] == len(codes) and rep["stage"] == ("gpt_sampled" if sampled else "gpt_greedy")
    with itts_cfm.GptDecoder(gpt_bundle, device=0) as d:
        want = d.generate_sampled(prefix, steps, cfg, hf_positions=True)[0] if sampled else \
            d.generate(prefix, steps, hf_positions=True)[0]
    assert codes == want
