"""Condition assembly on the GPU (itts_cond_*): the S2Mel length regulator and
the prompt/generated merge, against the reference.

The reference's own CPU length regulator (oracle/_ref) made
tests/golden/kat_length_regulator.npz (its self-test input 7 -> 11 frames and
a seeded 40 -> 63 case); the C restatement (oracle/condition_oracle.c,
pinned to that golden) checks a config-2-sized assembly. f16 operands with
fp32 accumulation through five convs and four GroupNorms: gate max-abs <=
2e-2 or rel-L2 <= 1e-2, cosine >= 0.999; the prompt rows are copied bit for
bit."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

import itts_cfm
import oracle as O

pytestmark = pytest.mark.gpu

GOLD = Path(__file__).resolve().parent / "golden"


def _ok(ref, got):
    c = O.compare(ref, got)
    assert c["cosine"] >= 0.999 and (c["max_abs"] <= 2e-2 or c["rel_l2"] <= 1e-2), c
    return c


@pytest.fixture(scope="module")
def ca(condition_bundle):
    c = itts_cfm.ConditionAssembler(condition_bundle, device=0)
    yield c
    c.close()


def test_length_regulator_matches_reference_golden(ca):
    g = dict(np.load(GOLD / "kat_length_regulator.npz"))
    _ok(g["out7_11"], ca.length_regulator(g["x7"], 11))
    _ok(g["out40_63"], ca.length_regulator(g["x40"], 63))


def test_condition_assembly_config2_size(ca, port_condition):
    """175 semantic frames -> 600 generated mel frames after a 200-row prompt."""
    rng = np.random.default_rng(21)
    s_infer = rng.standard_normal((175, 1024)).astype(np.float32)
    prompt = rng.standard_normal((200, 512)).astype(np.float32)
    got = ca.assemble(s_infer, prompt, 600)
    assert got.shape == (800, 512)
    assert np.array_equal(got[:200], prompt)
    _ok(port_condition.assemble(s_infer, prompt, 600), got)


@pytest.mark.parametrize("n_in,G", [(1, 1), (1, 9), (13, 5), (64, 64)])
def test_length_regulator_edge_shapes(ca, port_condition, n_in, G):
    """Single input frame, downsampling (n_in > G) and equal lengths."""
    x = np.random.default_rng(n_in * 100 + G).standard_normal((n_in, 1024)).astype(np.float32)
    _ok(port_condition.length_regulator(x, G), ca.length_regulator(x, G))


def test_condition_assembly_deterministic(ca):
    rng = np.random.default_rng(22)
    s_infer = rng.standard_normal((90, 1024)).astype(np.float32)
    prompt = rng.standard_normal((30, 512)).astype(np.float32)
    a = ca.assemble(s_infer, prompt, 300)
    assert np.isfinite(a).all()
    assert np.array_equal(a, ca.assemble(s_infer, prompt, 300))


def test_condition_rejects_bad_shapes(ca):
    with pytest.raises(itts_cfm.IttsError) as e:
        ca.length_regulator(np.zeros((4, 1024), np.float32), 0)
    assert e.value.code == itts_cfm.ITTS_EINVAL_SHAPE
    with pytest.raises(ValueError):
        ca.length_regulator(np.zeros((4, 1000), np.float32), 8)
