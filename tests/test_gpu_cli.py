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
