"""Bundle contract gates and the cached-voice loader (host only, no GPU):
itts_inspect_voice_bundle / itts_inspect_model_bundle / itts_voice_load,
checked against the rules of the reference's --inspect-voice-bundle and
--inspect-model-bundle gates (docs/native_bundle.md:55-112 in the reference)."""
from __future__ import annotations

import json

import numpy as np
import pytest

import itts_cfm
import mit2


@pytest.fixture()
def voice(tmp_path):
    return mit2.make_voice_bundle(tmp_path / "voice", seed=3, prompt_tokens=37)


def _rewrite_manifest(d, fn):
    m = json.loads((d / "manifest.json").read_text())
    fn(m)
    (d / "manifest.json").write_text(json.dumps(m))


def test_voice_gate_accepts_synthetic_voice(voice):
    rc, rep = itts_cfm.inspect_voice_bundle(voice)
    assert rc == itts_cfm.ITTS_OK and rep["ok"] is True
    assert rep["prompt_tokens"] == rep["mel_frames"] == 37 and rep["spk_cond_tokens"] == 170
    assert rep["integrity"]["sha256_verified_count"] == 4
    assert [t["name"] for t in rep["required_tensors"]] == ["spk_cond_emb", "s2mel_style", "s2mel_prompt", "mel"]


def test_voice_load_matches_pipeline_layout(voice):
    t = dict(mit2.make_voice_tensors(3, 37))
    v = itts_cfm.voice_load(voice)
    assert v["P"] == 37
    assert np.array_equal(v["prompt_cond"], t["s2mel_prompt"][0])
    assert np.array_equal(v["style"], t["s2mel_style"][0])
    assert np.array_equal(v["prompt_mel"], t["mel"][0].T)  # [1,80,P] -> [P,80]
    v20 = itts_cfm.voice_load(voice, prompt_tokens=20)
    assert v20["P"] == 20 and np.array_equal(v20["prompt_mel"], t["mel"][0].T[:20])
    with pytest.raises(itts_cfm.IttsError):
        itts_cfm.voice_load(voice, prompt_tokens=38)


def test_voice_gate_rejects_corrupted_payload(voice):
    m = json.loads((voice / "manifest.json").read_text())
    rec = next(r for r in m["tensors"] if r["name"] == "s2mel_style")
    with (voice / "weights.bin").open("r+b") as f:
        f.seek(rec["offset"] + 5)
        b = f.read(1)
        f.seek(rec["offset"] + 5)
        f.write(bytes([b[0] ^ 0x40]))
    rc, rep = itts_cfm.inspect_voice_bundle(voice)
    assert rc == itts_cfm.ITTS_EBUNDLE and rep["ok"] is False and "sha256 mismatch: s2mel_style" in rep["error"]


@pytest.mark.parametrize("edit,msg", [
    (lambda m: [r.__setitem__("component", "s2mel") for r in m["tensors"] if r["name"] == "mel"], "component=voice"),
    (lambda m: [r.pop("sha256") for r in m["tensors"] if r["name"] == "spk_cond_emb"], "missing sha256"),
    (lambda m: m.__setitem__("tensors", [r for r in m["tensors"] if r["name"] != "s2mel_prompt"]), "missing tensor"),
])
def test_voice_gate_rejects_contract_violations(voice, edit, msg):
    _rewrite_manifest(voice, edit)
    rc, rep = itts_cfm.inspect_voice_bundle(voice)
    assert rc == itts_cfm.ITTS_EBUNDLE and msg in rep["error"], rep


def test_voice_gate_rejects_prompt_mel_mismatch_and_dtype(tmp_path):
    t = dict(mit2.make_voice_tensors(1, 12))
    t["mel"] = t["mel"][:, :, :11].copy()
    mit2.write_bundle(tmp_path / "a", list(t.items()))
    rc, rep = itts_cfm.inspect_voice_bundle(tmp_path / "a")
    assert rc == itts_cfm.ITTS_EBUNDLE and "prompt token count must match mel frame count" in rep["error"]
    t = dict(mit2.make_voice_tensors(1, 12))
    t["s2mel_style"] = t["s2mel_style"].astype(np.float16)
    mit2.write_bundle(tmp_path / "b", list(t.items()))
    rc, rep = itts_cfm.inspect_voice_bundle(tmp_path / "b")
    assert rc == itts_cfm.ITTS_EBUNDLE and "f32 dtype" in rep["error"]


def test_model_gate_per_component(unit_bundle, tmp_path):
    rc, rep = itts_cfm.inspect_model_bundle(unit_bundle, itts_cfm.ITTS_COMPONENT_CFM)
    assert rc == itts_cfm.ITTS_OK and rep["ok"] and rep["components"] == ["cfm_estimator"]
    assert rep["integrity"]["sha256_verified_count"] == rep["tensor_count"] == len(mit2.dit_tensor_specs())
    lr = mit2.make_condition_bundle(tmp_path / "lr", seed=0)
    rc, rep = itts_cfm.inspect_model_bundle(lr, itts_cfm.ITTS_COMPONENT_LENGTH_REGULATOR)
    assert rc == itts_cfm.ITTS_OK, rep
    # the estimator bundle holds no BigVGAN tensors
    rc, rep = itts_cfm.inspect_model_bundle(unit_bundle, itts_cfm.ITTS_COMPONENT_BIGVGAN)
    assert rc == itts_cfm.ITTS_EBUNDLE and "missing tensor: bigvgan.conv_pre.weight_v" in rep["error"]
    rc, rep = itts_cfm.inspect_model_bundle(unit_bundle, 0x100)
    assert rc == itts_cfm.ITTS_EBUNDLE and "component mask" in rep["error"]


def test_model_gate_gpt(gpt_bundle, unit_bundle):
    """The GPT decoder's sentinels (Conv1D weights [in, out]) on the
    synthetic GPT bundle, every payload's SHA-256 verified; missing from the
    estimator bundle."""
    rc, rep = itts_cfm.inspect_model_bundle(gpt_bundle, itts_cfm.ITTS_COMPONENT_GPT)
    assert rc == itts_cfm.ITTS_OK and rep["ok"] and rep["components"] == ["gpt"], rep
    assert rep["integrity"]["sha256_verified_count"] == rep["tensor_count"] == len(mit2.gpt_tensor_specs())
    rc, rep = itts_cfm.inspect_model_bundle(unit_bundle, itts_cfm.ITTS_COMPONENT_GPT)
    assert rc == itts_cfm.ITTS_EBUNDLE and "missing tensor: gpt." in rep["error"]


def test_model_gate_bigvgan(vocoder_bundle):
    rc, rep = itts_cfm.inspect_model_bundle(vocoder_bundle, itts_cfm.ITTS_COMPONENT_BIGVGAN)
    assert rc == itts_cfm.ITTS_OK, rep
    assert all(t["component"] == "bigvgan" for t in rep["required_tensors"])


def test_cli_gates(voice, unit_bundle, tmp_path):
    """mtts_cfm --inspect-voice-bundle / --inspect-model-bundle: JSON report, exit status."""
    import subprocess
    from pathlib import Path

    cli = Path(__file__).resolve().parent.parent / "index-tts2-metal_b200" / "lib" / "mtts_cfm"
    r = subprocess.run([str(cli), "--inspect-voice-bundle", str(voice)], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0 and json.loads(r.stdout)["ok"] is True
    r = subprocess.run([str(cli), "--inspect-model-bundle", str(unit_bundle), "cfm"], capture_output=True, text=True,
                       timeout=120)
    assert r.returncode == 0 and json.loads(r.stdout)["components"] == ["cfm_estimator"]
    r = subprocess.run([str(cli), "--inspect-model-bundle", str(unit_bundle), "bigvgan"], capture_output=True,
                       text=True, timeout=120)
    assert r.returncode == 1 and json.loads(r.stdout)["ok"] is False


def test_single_file_voice_bundle_equals_directory_form(tmp_path):
    """The one-file bundle form (weights stream + manifest + "MIT2VOIC" footer,
    the reference's runtime/bundle.cpp:153-200) passes the same gate with the
    same report and loads the same voice as the directory form."""
    d = mit2.make_voice_bundle(tmp_path / "voice_dir", seed=5, prompt_tokens=23)
    f = mit2.make_voice_bundle(tmp_path / "voice.mit2", seed=5, prompt_tokens=23, single_file=True)
    assert f.is_file()
    rc_d, rep_d = itts_cfm.inspect_voice_bundle(d)
    rc_f, rep_f = itts_cfm.inspect_voice_bundle(f)
    assert rc_d == rc_f == itts_cfm.ITTS_OK and rep_f["ok"] is True
    for k in ("prompt_tokens", "mel_frames", "spk_cond_tokens"):
        assert rep_f[k] == rep_d[k]
    vd, vf = itts_cfm.voice_load(d, 11), itts_cfm.voice_load(f, 11)
    for k in ("prompt_cond", "style", "prompt_mel"):
        assert np.array_equal(vd[k], vf[k])
    got = mit2.read_bundle(f, verify=True)
    want = mit2.read_bundle(d, verify=True)
    assert got.keys() == want.keys() and all(np.array_equal(got[k], want[k]) for k in got)


def _single_file_voice(tmp_path):
    return mit2.make_voice_bundle(tmp_path / "v.mit2", seed=6, prompt_tokens=9, single_file=True)


@pytest.mark.parametrize("damage,msg", [
    ("truncate", "footer magic"),
    ("manifest_past_end", "manifest exceeds"),
    ("tiny", "too small"),
    ("payload_flip", "sha256"),
])
def test_single_file_bundle_rejections(tmp_path, damage, msg):
    f = _single_file_voice(tmp_path)
    raw = bytearray(f.read_bytes())
    if damage == "truncate":
        raw = raw[:-5]
    elif damage == "manifest_past_end":
        off = int.from_bytes(raw[-24:-16], "little")
        raw[-16:-8] = (len(raw) - off).to_bytes(8, "little")
    elif damage == "tiny":
        raw = raw[:20]
    else:
        raw[4096 + 3] ^= 0x40  # inside the first payload (offsets are 4096-aligned)
    f.write_bytes(bytes(raw))
    rc, rep = itts_cfm.inspect_voice_bundle(f)
    assert rc == itts_cfm.ITTS_EBUNDLE and rep["ok"] is False
    assert msg in rep["error"].lower() or msg in json.dumps(rep).lower(), rep


def test_single_file_model_bundle_gate(tmp_path):
    f = tmp_path / "cfm.mit2"
    mit2.write_single_file_bundle(f, mit2.make_dit_tensors(0, "unit"))
    rc, rep = itts_cfm.inspect_model_bundle(f, itts_cfm.ITTS_COMPONENT_CFM)
    assert rc == itts_cfm.ITTS_OK and rep["ok"] is True, rep
