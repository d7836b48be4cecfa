"""Pin the CPU oracles (oracle/dit_oracle.c, oracle/bigvgan_oracle.c,
oracle/condition_oracle.c, oracle/gpt_oracle.py) to the reference's own CPU
functions through the committed golden vectors (tests/golden/, made by
tests/golden/make_golden.py from oracle/_ref). fp32 vs fp32 with a different
summation order: the reference's own unit tolerance ladder applies (1e-4
relative to the output scale)."""
from __future__ import annotations

import hashlib
from pathlib import Path

import numpy as np
import pytest

import oracle as O

GOLD = Path(__file__).resolve().parent / "golden"
REL = 1e-4


def _load(name):
    return dict(np.load(GOLD / f"{name}.npz"))


def _close(ref, got, rel=REL):
    ref = np.asarray(ref, np.float64)
    got = np.asarray(got, np.float64)
    scale = max(1.0, float(np.abs(ref).max()))
    err = float(np.abs(ref - got).max())
    assert err <= rel * scale, (err, scale)


def _sha(d: Path) -> str:
    h = hashlib.sha256()
    with (d / "weights.bin").open("rb") as f:
        for chunk in iter(lambda: f.read(1 << 22), b""):
            h.update(chunk)
    return h.hexdigest()


def test_bundles_match_golden_generator(unit_bundle, baseline_bundle):
    g = _load("kat_estimator_t6")
    assert _sha(unit_bundle) == str(g["weights_sha256"])
    assert _sha(baseline_bundle) == str(g["baseline_weights_sha256"])


def test_noise_bit_exact(port_unit):
    g = _load("kat_noise")
    assert np.array_equal(port_unit.noise(5, 80, 1234), g["a"])
    assert np.array_equal(port_unit.noise(3, 7, 0), g["b"])


def test_timestep_embedders(port_unit):
    g = _load("kat_tembed")
    for i, t in enumerate(g["t"]):
        _close(g["t1"][i], port_unit.timestep_embed(float(t), 0))
        _close(g["t2"][i], port_unit.timestep_embed(float(t), 1))


def test_estimator_selftest_inputs(port_unit, port_baseline):
    g = _load("kat_estimator_t6")
    args = (g["x"], g["prompt_x"], g["cond"], g["style"], float(g["t"]), g["mask"])
    _close(g["vel_unit"], port_unit.estimator(*args))
    _close(g["vel_baseline"], port_baseline.estimator(*args))


def test_estimator_random_t33(port_unit):
    g = _load("kat_estimator_t33")
    _close(g["vel"], port_unit.estimator(g["x"], g["prompt_x"], g["cond"], g["style"], float(g["t"]), g["mask"]))


def test_attention_core(port_unit):
    g = _load("kat_attention_t6")
    _close(g["l0_a"], port_unit.attention_layer(g["x"], g["mask_a"], 0))
    _close(g["l0_b"], port_unit.attention_layer(g["x"], g["mask_b"], 0))
    _close(g["l12_a"], port_unit.attention_layer(g["x"], g["mask_a"], 12))


def test_wavenet_global_cond(port_unit):
    g = _load("kat_wavenet_t6")
    _close(g["out"], port_unit.wavenet(g["x"], g["g"], g["mask"]))


def test_euler_sampler(port_unit):
    g = _load("kat_euler_t5")
    px = np.zeros((5, 80), np.float32)
    px[:2] = g["prompt"]
    _close(g["mel_3_cfg0"], port_unit.euler(g["noise"], px, g["cond"], g["style"], 2, 3, 0.0))
    _close(g["mel_25_cfg05"], port_unit.euler(g["noise"], px, g["cond"], g["style"], 2, 25, 0.5))


def test_euler_masked(port_unit):
    g = _load("kat_euler_masked")
    _close(g["mel"], port_unit.euler(g["noise"], g["prompt_x"], g["cond"], g["style"], 2, 2, 0.7, mask=g["mask"]))


def test_oracle_detects_planted_error(port_unit, unit_tensors):
    """A wrong weight in the oracle must break the pin (the check has teeth)."""
    g = _load("kat_estimator_t6")
    bad = dict(unit_tensors)
    k = "s2mel.net.cfm.estimator.transformer.layers.5.feed_forward.w2.weight"
    bad[k] = bad[k].copy()
    bad[k][3, :] *= 1.5
    wrong = O.PortOracle(bad)
    args = (g["x"], g["prompt_x"], g["cond"], g["style"], float(g["t"]), g["mask"])
    with pytest.raises(AssertionError):
        _close(g["vel_unit"], wrong.estimator(*args))


def test_weight_norm_gain_is_visible(port_unit, unit_tensors):
    """The synthetic bundles' weight-norm gains differ from ||v_row||, so a fold
    that drops g (W = v) or normalises along the wrong axis breaks the pin."""
    g = _load("kat_estimator_t6")
    args = (g["x"], g["prompt_x"], g["cond"], g["style"], float(g["t"]), g["mask"])
    for planted in ("drop_gain", "column_norm"):
        bad = dict(unit_tensors)
        for k in [k for k in bad if k.endswith("weight_g")]:
            v = bad[k[: -len("weight_g")] + "weight_v"].astype(np.float32)
            rows = v.reshape(v.shape[0], -1)
            if planted == "drop_gain":
                gain = np.sqrt((rows**2).sum(axis=1))
            else:
                gain = np.sqrt((rows**2).sum(axis=0)).mean() * np.ones(rows.shape[0], np.float32)
            bad[k] = gain.reshape(bad[k].shape).astype(np.float32)
        with pytest.raises(AssertionError):
            _close(g["vel_unit"], O.PortOracle(bad).estimator(*args))


def test_bigvgan_bundle_matches_golden_generator(vocoder_bundle):
    assert _sha(vocoder_bundle) == str(_load("kat_bigvgan")["weights_sha256"])


def test_bigvgan_activations(port_vocoder):
    g = _load("kat_bigvgan")
    _close(g["act_rb0"], port_vocoder.activation("bigvgan.resblocks.0.activations.0", g["x_act"]))
    _close(g["act_post"], port_vocoder.activation("bigvgan.activation_post", g["x_post"]))


def test_bigvgan_vocoder(port_vocoder):
    g = _load("kat_bigvgan")
    wave = port_vocoder.vocoder(g["mel"])
    assert wave.shape == (3 * 256,)
    _close(g["wave"], wave)


def test_bigvgan_oracle_detects_planted_error(vocoder_tensors):
    """A wrong resblock weight in the vocoder oracle must break the pin."""
    g = _load("kat_bigvgan")
    bad = dict(vocoder_tensors)
    k = "bigvgan.resblocks.4.convs2.1.weight_v"
    bad[k] = bad[k].copy()
    bad[k][5] *= -1.0
    with pytest.raises(AssertionError):
        _close(g["wave"], O.VocoderOracle(bad).vocoder(g["mel"]))


def test_length_regulator_bundle_matches_golden_generator(condition_bundle):
    assert _sha(condition_bundle) == str(_load("kat_length_regulator")["weights_sha256"])


def test_length_regulator(port_condition):
    g = _load("kat_length_regulator")
    _close(g["out7_11"], port_condition.length_regulator(g["x7"], 11))
    _close(g["out40_63"], port_condition.length_regulator(g["x40"], 63))


def test_condition_merge_places_prompt_rows_first(port_condition):
    g = _load("kat_length_regulator")
    prompt = np.random.default_rng(5).standard_normal((4, 512)).astype(np.float32)
    cond = port_condition.assemble(g["x7"], prompt, 11)
    assert cond.shape == (15, 512)
    assert np.array_equal(cond[:4], prompt)
    _close(g["out7_11"], cond[4:])


def test_gpt_bundle_matches_golden_generator(gpt_bundle):
    assert _sha(gpt_bundle) == str(_load("kat_gpt_decode")["weights_sha256"])


def test_gpt_greedy_decode(gpt_oracle):
    g = _load("kat_gpt_decode")
    codes, logits = gpt_oracle.greedy(g["prefix"], 3)
    assert codes == g["codes"].tolist()
    _close(g["last_logits"], logits[-1])


@pytest.mark.parametrize("name", ["ref_test", "production", "wide", "greedy_k1", "big_topp"])
def test_gpt_sampling_matches_reference(name):
    """The restated logits processors reproduce the reference's processed
    logits bit for bit (including which entries are -inf), and the restated
    SplitMix64 sampler its draws; "ref_test" is the reference's own known
    answer (processed[8] = 12, processed[9] = 14, draw 9)."""
    import gpt_oracle as G

    g = _load("kat_gpt_sampling")
    seed, t, k, p, pen, draws = g[f"{name}_config"].tolist()
    proc = G.sampling_processors(g[f"{name}_logits"], g[f"{name}_history"], t, int(k), p, pen)
    ref = g[f"{name}_processed"]
    assert np.array_equal(np.isfinite(proc), np.isfinite(ref))
    assert np.array_equal(proc[np.isfinite(ref)], ref[np.isfinite(ref)])
    rng = G.SplitMix64(int(seed))
    assert [G.sample_token(proc, rng) for _ in range(int(draws))] == g[f"{name}_tokens"].tolist()
    if name == "ref_test":
        assert ref[8] == 12.0 and ref[9] == 14.0 and g[f"{name}_tokens"][0] == 9


def test_gpt_greedy_decode_hf_positions(gpt_oracle):
    """hf_generate_positions = true, as the synthesis pipeline calls the
    decoder: step s > 0 takes position embedding s + 1."""
    g = _load("kat_gpt_decode_hf")
    codes, logits = gpt_oracle.greedy(g["prefix"], 3, hf_positions=True)
    assert codes == g["codes"].tolist()
    _close(g["last_logits"], logits[-1])
    plain = gpt_oracle.greedy(g["prefix"], 3)[1][-1]
    assert not np.allclose(plain, logits[-1])  # the flag changes the decode
