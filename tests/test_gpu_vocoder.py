"""BigVGAN vocoder on the GPU (itts_vocoder_*), against the reference.

The reference's own CPU vocoder (oracle/_ref) made the golden waveform of
tests/golden/kat_bigvgan.npz; the C restatement (oracle/bigvgan_oracle.c,
pinned to that golden) checks other lengths. The GPU path runs f16 operands
with fp32 accumulation through 6 upsampling stages and 54 resblock pairs, so
the gate is the north-star output gate: max-abs <= 2e-2 or rel-L2 <= 1e-2,
and cosine >= 0.999."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

import itts_cfm
import oracle as O

pytestmark = pytest.mark.gpu

GOLD = Path(__file__).resolve().parent / "golden"
MAX_ABS = 2e-2
REL_L2 = 1e-2
COS_MIN = 0.999


def _ok(ref, got):
    c = O.compare(ref, got)
    assert c["cosine"] >= COS_MIN and (c["max_abs"] <= MAX_ABS or c["rel_l2"] <= REL_L2), c
    return c


@pytest.fixture(scope="module")
def voc(vocoder_bundle):
    v = itts_cfm.Vocoder(vocoder_bundle, device=0)
    yield v
    v.close()


def test_vocoder_matches_reference_golden(voc):
    g = dict(np.load(GOLD / "kat_bigvgan.npz"))
    wave = voc.run(g["mel"])
    assert wave.shape == g["wave"].shape
    _ok(g["wave"], wave)


@pytest.mark.parametrize("T", [1, 2, 5, 33])
def test_vocoder_vs_oracle(voc, port_vocoder, T):
    rng = np.random.default_rng(100 + T)
    mel = rng.standard_normal((T, 80)).astype(np.float32)
    _ok(port_vocoder.vocoder(mel), voc.run(mel))


def test_vocoder_deterministic_and_bounded(voc):
    rng = np.random.default_rng(7)
    mel = rng.standard_normal((800, 80)).astype(np.float32)  # config-2 utterance length
    a = voc.run(mel)
    b = voc.run(mel)
    assert a.shape == (800 * 256,)
    assert np.isfinite(a).all()
    assert np.abs(a).max() <= 1.0
    assert np.array_equal(a, b)


def test_vocoder_is_causal_free_of_cross_utterance_state(voc):
    """A call depends only on its own mel: interleaving another length in
    between leaves the result bitwise unchanged (plans are per length)."""
    rng = np.random.default_rng(11)
    m1 = rng.standard_normal((40, 80)).astype(np.float32)
    m2 = rng.standard_normal((17, 80)).astype(np.float32)
    a = voc.run(m1)
    voc.run(m2)
    assert np.array_equal(a, voc.run(m1))


def test_vocoder_rejects_bad_lengths(voc):
    with pytest.raises(itts_cfm.IttsError) as e:
        voc.run(np.zeros((0, 80), np.float32))
    assert e.value.code == itts_cfm.ITTS_EINVAL_SHAPE
    with pytest.raises(ValueError):
        voc.run(np.zeros((4, 79), np.float32))
