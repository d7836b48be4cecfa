"""The S2Mel-to-waveform chain (itts_pipeline_synthesize) on the GPU: equal,
bit for bit, to the stages called one by one through their own entry points,
and within the output gate of the CPU oracle chain (condition oracle ->
estimator/Euler oracle -> vocoder oracle)."""
from __future__ import annotations

import numpy as np
import pytest

import itts_cfm
import mit2
import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def voice(tmp_path_factory):
    return mit2.make_voice_bundle(tmp_path_factory.mktemp("voice"), seed=9, prompt_tokens=6)


@pytest.fixture(scope="module")
def pipe(unit_bundle, condition_bundle, vocoder_bundle):
    p = itts_cfm.Pipeline(unit_bundle, condition_bundle, vocoder_bundle, device=0)
    yield p
    p.close()


def _inputs(P, G, n_in, seed):
    rng = np.random.default_rng(seed)
    return rng.standard_normal((n_in, 1024)).astype(np.float32), rng.standard_normal((P + G, 80)).astype(np.float32)


def test_pipeline_equals_staged_calls(pipe, voice, unit_bundle, condition_bundle, vocoder_bundle):
    P, G, n_in = 6, 40, 12
    s_infer, noise = _inputs(P, G, n_in, 1)
    wave, mel = pipe.synthesize(voice, s_infer, G, noise, 3, 0.7)
    v = itts_cfm.voice_load(voice)
    with itts_cfm.ConditionAssembler(condition_bundle) as ca:
        cond = ca.assemble(s_infer, v["prompt_cond"], G)
    with itts_cfm.Context(unit_bundle) as ctx:
        mel_s = ctx.run(noise, v["prompt_mel"], cond, v["style"], 3, 0.7)
    with itts_cfm.Vocoder(vocoder_bundle) as voc:
        wave_s = voc.run(mel_s[P:])
    assert np.array_equal(mel, mel_s)
    assert np.array_equal(wave, wave_s)
    assert wave.shape == (G * 256,) and np.isfinite(wave).all() and np.abs(wave).max() <= 1.0
    assert np.all(mel[:P] == 0.0)


def test_pipeline_vs_oracle_chain(pipe, voice, port_unit, port_condition, port_vocoder):
    P, G, n_in = 6, 10, 4
    s_infer, noise = _inputs(P, G, n_in, 2)
    wave, mel = pipe.synthesize(voice, s_infer, G, noise, 2, 0.7)
    v = itts_cfm.voice_load(voice)
    cond = port_condition.assemble(s_infer, v["prompt_cond"], G)
    px = np.zeros((P + G, 80), np.float32)
    px[:P] = v["prompt_mel"]
    mel_ref = port_unit.euler(noise, px, cond, v["style"], P, 2, 0.7)
    c = O.compare(mel_ref, mel)
    assert c["cosine"] >= 0.999 and (c["max_abs"] <= 2e-2 or c["rel_l2"] <= 1e-2), c
    c = O.compare(port_vocoder.vocoder(mel_ref[P:]), wave)
    assert c["cosine"] >= 0.999 and (c["max_abs"] <= 2e-2 or c["rel_l2"] <= 1e-2), c


def test_pipeline_reports_stage_errors(pipe, voice, tmp_path):
    s_infer, noise = _inputs(6, 8, 3, 3)
    with pytest.raises(itts_cfm.IttsError) as e:
        pipe.synthesize(tmp_path / "no_voice", s_infer, 8, noise, 2, 0.7)
    assert e.value.code == itts_cfm.ITTS_EBUNDLE and "voice" in str(e.value)
    with pytest.raises(itts_cfm.IttsError) as e:
        pipe.synthesize(voice, s_infer, 0, noise, 2, 0.7)
    assert e.value.code == itts_cfm.ITTS_EINVAL_SHAPE


def test_pipeline_seeded_noise_form(pipe, voice):
    """itts_pipeline_synthesize_seeded draws x0 as the reference's pipeline
    does (make_deterministic_normal_noise(P + G, 80, seed, temperature)) and
    then equals the explicit-noise call bit for bit."""
    P, G, n_in = 6, 24, 7
    s_infer, _ = _inputs(P, G, n_in, 4)
    seed, temp = 20240605, 0.8
    wave_s, mel_s = pipe.synthesize_seeded(voice, s_infer, G, seed, temp, 3, 0.7)
    noise = itts_cfm.make_noise(P + G, 80, seed, temp)
    wave, mel = pipe.synthesize(voice, s_infer, G, noise, 3, 0.7)
    assert np.array_equal(mel_s, mel) and np.array_equal(wave_s, wave)
