"""CPU-only tests: bundle format, host logic, the C-ABI library's exports, and
input generators. No kernel is launched here."""
from __future__ import annotations

import json
import re
from pathlib import Path

import numpy as np
import pytest

import mit2
import workloads as W

REPO = Path(__file__).resolve().parent.parent
HEADER = REPO / "include" / "itts_cfm.h"


def test_bundle_round_trip(tmp_path):
    man = mit2.write_bundle(tmp_path, [("a.weight", np.arange(12, dtype=np.float32).reshape(3, 4)),
                                       ("b.codes", np.arange(5, dtype=np.int32)),
                                       ("c.half", np.linspace(-1, 1, 7).astype(np.float16))])
    assert man["format"] == "MIT2" and man["version"] == 1
    assert all(t["offset"] % man["alignment"] == 0 for t in man["tensors"])
    raw = (tmp_path / "weights.bin").read_bytes()
    assert raw[:4] == b"MIT2" and int.from_bytes(raw[4:8], "little") == 1 and int.from_bytes(raw[8:12], "little") == 4096
    got = mit2.read_bundle(tmp_path, verify=True)
    np.testing.assert_array_equal(got["a.weight"], np.arange(12, dtype=np.float32).reshape(3, 4))
    np.testing.assert_array_equal(got["b.codes"], np.arange(5, dtype=np.int32))
    assert got["c.half"].dtype == np.float16


def test_bundle_checksum_detects_corruption(tmp_path):
    mit2.write_bundle(tmp_path, [("x", np.ones(8, np.float32))])
    man = json.loads((tmp_path / "manifest.json").read_text())
    off = man["tensors"][0]["offset"]
    with (tmp_path / "weights.bin").open("r+b") as f:
        f.seek(off)
        f.write(b"\x00\x00\x80\x7f")
    with pytest.raises(ValueError):
        mit2.read_bundle(tmp_path, verify=True)


def test_synthetic_bundle_is_deterministic_and_complete():
    a = mit2.make_dit_tensors(3, "baseline")
    b = mit2.make_dit_tensors(3, "baseline")
    assert [n for n, _ in a] == [n for n, _ in b]
    for (na, xa), (_, xb) in zip(a, b):
        assert xa.dtype == xb.dtype and np.array_equal(xa, xb), na
    names = {n for n, _ in a}
    for spec_name, shape, _ in mit2.dit_tensor_specs():
        assert mit2.PREFIX + spec_name in names
    d = dict(a)
    # weight-norm g = ||v_row|| * gain, gain ~ U(0.5, 1.5): the folded weight differs from v
    v = d[mit2.PREFIX + "final_layer.linear.weight_v"].astype(np.float32)
    g = d[mit2.PREFIX + "final_layer.linear.weight_g"].astype(np.float32).ravel()
    gain = g / np.sqrt((v * v).sum(1))
    assert gain.min() >= 0.499 and gain.max() <= 1.501 and gain.std() > 0.2
    w = d[mit2.PREFIX + "transformer.layers.0.attention.wqkv.weight"].astype(np.float32)
    assert abs(w.std() - 0.02) < 1e-3


def test_unit_init_scale():
    d = dict(mit2.make_dit_tensors(0, "unit"))
    w = d[mit2.PREFIX + "transformer.layers.3.feed_forward.w2.weight"].astype(np.float32)
    assert abs(w.std() - 1 / np.sqrt(1536)) < 2e-3
    pb = d[mit2.PREFIX + "transformer.layers.3.ffn_norm.project_layer.bias"].astype(np.float32)
    assert abs(pb[:512].mean() - 1.0) < 0.05 and abs(pb[512:].mean()) < 0.05


def test_header_exports_every_symbol():
    """libitts_cfm.so loads on a CPU-only host and exports every declared entry point."""
    import itts_cfm

    decl = set(re.findall(r"^\s*(?:[\w\s\*]+?)\b(itts_\w+)\s*\(", HEADER.read_text(), re.M))
    assert decl, "no declarations parsed"
    lib = itts_cfm.load()
    for name in sorted(decl):
        assert hasattr(lib, name), name
    assert decl == set(itts_cfm.EXPORTED)


def test_header_constants_match_python_binding():
    """Every numeric #define of the C header that the Python binding mirrors
    has the same value there (the header is the single source of truth)."""
    import itts_cfm

    text = HEADER.read_text()
    defines = {m.group(1): int(m.group(2), 0) for m in re.finditer(
        r"^#define\s+(ITTS_\w+)\s+(0x[0-9a-fA-F]+|\d+)u?\b", text, re.M)}
    defines.update({m.group(1): int(m.group(2)) for m in re.finditer(r"^\s*(ITTS_\w+)\s*=\s*(-?\d+)\s*,?", text, re.M)})
    mirrored = {
        "ITTS_NOALLOC_CONV5_MAX_ROWS": itts_cfm.NOALLOC_CONV5_MAX_ROWS,
        "ITTS_VOCODER_MAX_T": itts_cfm.VOCODER_MAX_T,
    }
    for name in ("ITTS_OK", "ITTS_EINVAL_SHAPE", "ITTS_EBUNDLE", "ITTS_ECUDA", "ITTS_ETIMEOUT", "ITTS_ECAP",
                 "ITTS_ENODEV", "ITTS_GEMM_PAIR", "ITTS_COMPONENT_CFM", "ITTS_COMPONENT_LENGTH_REGULATOR",
                 "ITTS_COMPONENT_BIGVGAN", "ITTS_COMPONENT_GPT", "ITTS_COMPONENT_ALL"):
        mirrored[name] = getattr(itts_cfm, name)
    for name in ("WIDTH", "VOCAB", "START", "STOP", "MAX_STEPS", "MAX_LEN", "HF_POSITIONS"):
        mirrored["ITTS_GPT_" + name] = getattr(itts_cfm, "GPT_" + name)
    for name, value in mirrored.items():
        assert name in defines, f"{name} is not #defined in the header"
        assert defines[name] == value, (name, defines[name], value)


def test_create_fails_loudly_without_gpu_or_bundle(tmp_path):
    """No CPU fallback: creation without a usable GPU (or bundle) returns an error code."""
    import itts_cfm

    with pytest.raises(itts_cfm.IttsError) as e:
        itts_cfm.Context(tmp_path / "missing", device=0)
    assert e.value.code in (itts_cfm.ITTS_ECUDA, itts_cfm.ITTS_ENODEV, itts_cfm.ITTS_EBUNDLE)


def test_bucket_len_policy():
    import itts_cfm

    assert itts_cfm.bucket_len(2) == 128
    assert itts_cfm.bucket_len(128) == 128
    assert itts_cfm.bucket_len(129) == 256
    assert itts_cfm.bucket_len(1500) == 1536
    assert itts_cfm.bucket_len(2049) == 2304
    for t in range(2, 5000, 37):
        b = itts_cfm.bucket_len(t)
        assert b >= t and itts_cfm.bucket_len(b) == b


def test_step_flops_matches_cost_model():
    import itts_cfm

    # 294.09e6 * T + 53,248 * T^2 per guided step (2 branches)
    for T in (400, 800, 4096):
        want = 2 * 2 * 73_523_200 * T + 2 * 13 * 4 * 512 * T * T
        assert abs(itts_cfm.step_flops(2, T) - want) / want < 1e-12
    assert abs(itts_cfm.step_flops(2, 800) - 269.35e9) / 269.35e9 < 1e-3


def test_workloads_deterministic():
    a = W.config_utterances(3, n=5)
    b = W.config_utterances(3, n=5)
    for x, y in zip(a, b):
        assert x.T == y.T and x.P == y.P and np.array_equal(x.noise, y.noise)
        assert 200 <= x.T <= 1500 and x.P <= x.T
    u = W.config_utterances(2)[0]
    assert u.T == 800 and u.P == 200 and u.cond.shape == (800, 512)
    vl, pl, noise, px, cond, style = W.pad_batch(a[:2], 1536)
    assert noise.shape == (2, 1536, 80) and np.all(noise[0, a[0].T:] == 0)
    assert np.array_equal(px[1, : a[1].P], a[1].prompt) and np.all(px[1, a[1].P:] == 0)


def test_vocoder_create_fails_loudly_without_gpu_or_bundle(tmp_path):
    """No CPU fallback for the vocoder either."""
    import itts_cfm

    with pytest.raises(itts_cfm.IttsError) as e:
        itts_cfm.Vocoder(tmp_path / "missing", device=0)
    assert e.value.code in (itts_cfm.ITTS_ECUDA, itts_cfm.ITTS_ENODEV, itts_cfm.ITTS_EBUNDLE)


def test_vocoder_flops_matches_layer_count():
    import itts_cfm

    def macs(T):
        m, t = T * 80 * 1536 * 7, T
        for cin, cout, k, s, _ in mit2.BIGVGAN_UPSAMPLERS:
            m += t * cin * cout * k
            t *= s
            m += sum(3 * 2 * t * cout * cout * kk for kk in mit2.BIGVGAN_RESBLOCK_KERNELS)
        return 2.0 * (m + t * 24 * 7)

    for T in (1, 3, 800):
        assert abs(itts_cfm.Vocoder.flops(T) - macs(T)) / macs(T) < 1e-12


def test_bigvgan_tensor_specs_complete():
    specs = mit2.bigvgan_tensor_specs()
    names = [n for n, _, _ in specs]
    assert len(names) == len(set(names)) == 783
    assert "bigvgan.resblocks.17.convs2.2.weight_v" in names and "bigvgan.conv_post.weight_v" in names
    f = mit2.kaiser_sinc_lowpass(0.25, 0.3)
    assert f.shape == (12,) and abs(float(f.sum()) - 1.0) < 1e-6 and np.allclose(f, f[::-1])


def test_condition_create_fails_loudly_without_gpu_or_bundle(tmp_path):
    import itts_cfm

    with pytest.raises(itts_cfm.IttsError) as e:
        itts_cfm.ConditionAssembler(tmp_path / "missing", device=0)
    assert e.value.code in (itts_cfm.ITTS_ECUDA, itts_cfm.ITTS_ENODEV, itts_cfm.ITTS_EBUNDLE)


def test_condition_flops_and_specs():
    import itts_cfm

    assert itts_cfm.ConditionAssembler.flops(175, 600) == 2.0 * (175 * 1024 * 512 + 4 * 600 * 512 * 512 * 3 + 600 * 512 * 512)
    names = [n for n, _, _ in mit2.length_regulator_tensor_specs()]
    assert len(names) == len(set(names)) == 20
    assert names[0] == "s2mel.net.length_regulator.content_in_proj.weight"


def test_gpt_create_fails_loudly_without_gpu_or_bundle(tmp_path):
    import itts_cfm

    with pytest.raises(itts_cfm.IttsError) as e:
        itts_cfm.GptDecoder(tmp_path / "missing", device=0)
    assert e.value.code in (itts_cfm.ITTS_ECUDA, itts_cfm.ITTS_ENODEV, itts_cfm.ITTS_EBUNDLE)


def test_gpt_specs_and_weight_bytes():
    import itts_cfm

    specs = mit2.gpt_tensor_specs()
    names = [n for n, _, _ in specs]
    assert len(names) == len(set(names)) == 24 * 12 + 8
    w = sum(int(np.prod(s)) for n, s, k in specs if k == "w")
    assert itts_cfm.GptDecoder.weight_bytes_per_token() == 2.0 * w  # every linear weight once per token


def test_make_noise_bit_exact_to_reference_golden(port_unit):
    """itts_make_noise (the product's x0 draw) equals the reference's
    make_deterministic_normal_noise bit for bit: its own outputs in
    tests/golden/kat_noise.npz, and the pinned oracle restatement at other
    seeds, temperatures and odd sizes."""
    import itts_cfm

    g = np.load(REPO / "tests" / "golden" / "kat_noise.npz")
    assert np.array_equal(itts_cfm.make_noise(5, 80, 1234), g["a"])
    assert np.array_equal(itts_cfm.make_noise(3, 7, 0), g["b"])
    for T, C, seed, temp in ((800, 80, 20240605, 0.8), (1, 1, 2**64 - 1, 1.0), (17, 3, 42, 1.3)):
        assert np.array_equal(itts_cfm.make_noise(T, C, seed, temp), port_unit.noise(T, C, seed, temp)), (T, C, seed)


def test_make_noise_rejects_bad_shapes():
    import itts_cfm

    for T, C in ((0, 80), (5, 0), (65537, 80), (4, itts_cfm.NOISE_MAX_CHANNELS + 1)):
        with pytest.raises(itts_cfm.IttsError) as e:
            itts_cfm.make_noise(T, C, 1)
        assert e.value.code == itts_cfm.ITTS_EINVAL_SHAPE
