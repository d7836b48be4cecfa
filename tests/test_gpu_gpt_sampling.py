"""Sampled GPT decode on the GPU (itts_gpt_generate_sampled) against the
reference's sampler.

The numpy restatement of the reference's logits processors and SplitMix64
sampler (oracle/gpt_oracle.py) is pinned bit for bit to the reference's own
compiled functions (tests/golden/kat_gpt_sampling.npz). Here the device
sampler is checked (1) exactly, on the GPU's own logits of a one-step decode,
and (2) against whole decodes of the numpy decoder + sampler: the logits
differ from the oracle's by ~1e-6 relative (summation order), far below the
sampling margins, so the codes must be identical."""
from __future__ import annotations

import numpy as np
import pytest

import gpt_oracle as G
import itts_cfm

pytestmark = pytest.mark.gpu

PRODUCTION = dict(seed=20240605, temperature=0.8, top_k=30, top_p=0.8, repetition_penalty=10.0)


@pytest.fixture(scope="module")
def dec(gpt_bundle):
    d = itts_cfm.GptDecoder(gpt_bundle, device=0)
    yield d
    d.close()


def test_one_step_draw_is_exact_on_device_logits(dec):
    """One decode step: the code must be the reference sampler's draw from
    the logits the GPU itself computed (history [8192], fresh stream)."""
    prefix = np.random.default_rng(21).standard_normal((5, 1280)).astype(np.float32)
    for cfg in (PRODUCTION, dict(seed=3, temperature=1.2, top_k=2048, top_p=0.5, repetition_penalty=1.0)):
        codes, logits = dec.generate_sampled(prefix, 1, cfg)
        proc = G.sampling_processors(logits, [8192], cfg["temperature"], cfg["top_k"], cfg["top_p"],
                                     cfg["repetition_penalty"])
        assert codes == [G.sample_token(proc, G.SplitMix64(cfg["seed"]))]


@pytest.mark.parametrize("cfg", [
    PRODUCTION,
    dict(seed=7, temperature=1.0, top_k=200, top_p=0.95, repetition_penalty=1.0),
    dict(seed=11, temperature=0.8, top_k=1, top_p=1.0, repetition_penalty=1.3),
    dict(seed=3, temperature=1.2, top_k=2048, top_p=0.5, repetition_penalty=1.0),
], ids=["production", "wide", "k1", "big_topp"])
def test_sampled_decode_matches_oracle(dec, gpt_oracle, cfg):
    """The synthesis pipeline's call shape: generate-style positions and a
    repetition history prefix (fake inputs of 1s then the start code)."""
    prefix = np.random.default_rng(31).standard_normal((8, 1280)).astype(np.float32)
    hist = [1] * 9 + [8192]
    want, logits = gpt_oracle.greedy(prefix, 12, hf_positions=True, sampling=cfg, history_prefix=hist)
    codes, last = dec.generate_sampled(prefix, 12, cfg, history=hist, hf_positions=True)
    assert codes == want
    ref = np.asarray(logits[-1], np.float64)
    assert np.linalg.norm(ref - last) / np.linalg.norm(ref) <= 1e-4


def test_sampled_decode_is_seeded(dec):
    prefix = np.random.default_rng(41).standard_normal((4, 1280)).astype(np.float32)
    a = dec.generate_sampled(prefix, 10, PRODUCTION)[0]
    b = dec.generate_sampled(prefix, 10, PRODUCTION)[0]
    c = dec.generate_sampled(prefix, 10, dict(PRODUCTION, seed=PRODUCTION["seed"] + 1))[0]
    g = dec.generate(prefix, 10)[0]  # a greedy call in between leaves the sampler state alone
    d = dec.generate_sampled(prefix, 10, PRODUCTION)[0]
    assert a == b == d and a != c and len(g) == 10


@pytest.mark.parametrize("bad", [dict(top_k=0), dict(top_k=4096), dict(temperature=0.0), dict(top_p=0.0),
                                 dict(top_p=1.5), dict(repetition_penalty=0.0)])
def test_sampling_config_rejected(dec, bad):
    x = np.zeros((2, 1280), np.float32)
    with pytest.raises(itts_cfm.IttsError) as e:
        dec.generate_sampled(x, 2, dict(PRODUCTION, **bad))
    assert e.value.code == itts_cfm.ITTS_EINVAL_SHAPE
