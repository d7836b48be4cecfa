"""GPT mel-code decoder on the GPU (itts_gpt_*): cached greedy decode against
the reference.

The reference's own compiled CPU decoder (run_gpt_kv_greedy_cpu, oracle/_ref)
made tests/golden/kat_gpt_decode.npz (a 4-row prefix, 3 steps, seed-0
synthetic bundle); the numpy restatement (oracle/gpt_oracle.py, pinned to that
golden) checks longer decodes, the stop code and the edge cases. The weights
are the bundle's f16 values exactly and everything else is fp32, so only the
summation order differs: codes must be identical and logits within rel-L2
1e-4 (measured ~1e-6)."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

import itts_cfm
import mit2

pytestmark = pytest.mark.gpu

GOLD = Path(__file__).resolve().parent / "golden"
STOP = 8193


def _close(ref, got, tol=1e-4):
    ref, got = np.asarray(ref, np.float64), np.asarray(got, np.float64)
    rel = np.linalg.norm(ref - got) / max(np.linalg.norm(ref), 1e-30)
    assert rel <= tol, rel
    return rel


@pytest.fixture(scope="module")
def dec(gpt_bundle):
    d = itts_cfm.GptDecoder(gpt_bundle, device=0)
    yield d
    d.close()


def test_decode_matches_reference_golden(dec):
    g = dict(np.load(GOLD / "kat_gpt_decode.npz"))
    codes, logits = dec.generate(g["prefix"], 3)
    assert codes == [int(c) for c in g["codes"]]
    _close(g["last_logits"], logits)


def test_decode_hf_positions_matches_reference_golden(dec, gpt_oracle):
    """The synthesis pipeline's call (hf_generate_positions = true): the
    reference's own golden, then a longer decode against the oracle."""
    g = dict(np.load(GOLD / "kat_gpt_decode_hf.npz"))
    codes, logits = dec.generate(g["prefix"], 3, hf_positions=True)
    assert codes == [int(c) for c in g["codes"]]
    _close(g["last_logits"], logits)
    prefix = np.random.default_rng(11).standard_normal((12, 1280)).astype(np.float32)
    want, ref = gpt_oracle.greedy(prefix, 10, hf_positions=True)
    codes, last = dec.generate(prefix, 10, hf_positions=True)
    assert codes == want
    _close(ref[-1], last)


def test_decode_matches_oracle_longer(dec, gpt_oracle):
    """A 24-row prefix and 12 steps (crosses the 8-step stop-flag chunk)."""
    prefix = np.random.default_rng(5).standard_normal((24, 1280)).astype(np.float32) * np.float32(0.5)
    want, logits = gpt_oracle.greedy(prefix, 12)
    codes, last = dec.generate(prefix, 12)
    assert codes == want
    _close(logits[-1], last)


@pytest.mark.parametrize("P,steps", [(0, 3), (1, 1), (9, 8), (3, 9)])
def test_decode_edge_lengths(dec, gpt_oracle, P, steps):
    """Empty prefix, a single step, exactly one chunk, one past a chunk."""
    prefix = np.random.default_rng(100 + P).standard_normal((P, 1280)).astype(np.float32)
    want, logits = gpt_oracle.greedy(prefix, steps)
    codes, last = dec.generate(prefix if P else None, steps)
    assert codes == want
    assert len(codes) == steps or codes[-1] == STOP
    _close(logits[-1], last)


def test_decode_is_deterministic_and_reusable(dec):
    prefix = np.random.default_rng(9).standard_normal((7, 1280)).astype(np.float32)
    a = dec.generate(prefix, 5)
    b = dec.generate(prefix[:3], 2)  # a different run in between resets the cache
    c = dec.generate(prefix, 5)
    assert a[0] == c[0] and np.array_equal(a[1], c[1])
    assert len(b[0]) == 2


def test_invalid_lengths_rejected(dec):
    x = np.zeros((4, 1280), np.float32)
    for steps in (0, 1819):
        with pytest.raises(itts_cfm.IttsError) as e:
            dec.generate(x, steps)
        assert e.value.code == itts_cfm.ITTS_EINVAL_SHAPE
    with pytest.raises(itts_cfm.IttsError) as e:
        dec.generate(np.zeros((4000, 1280), np.float32), 100)
    assert e.value.code == itts_cfm.ITTS_EINVAL_SHAPE


def test_stop_code_ends_decode(gpt_oracle, tmp_path_factory):
    """Raise the stop code's head bias so that the stop wins at a step k >= 1
    where its logit margin reaches a new minimum (seed 18: k = 6, mid-way
    through the first 8-step chunk): the decode returns
    the first k codes of the unmodified run followed by the stop code, and
    the kernels after it in the same chunk leave codes and logits alone."""
    prefix = np.random.default_rng(18).standard_normal((6, 1280)).astype(np.float32)
    want, logits = gpt_oracle.greedy(prefix, 8)
    assert STOP not in want
    d = [float(np.max(l) - l[STOP]) for l in logits]
    k = max(range(1, len(d)), key=lambda i: min(d[:i]) - d[i])  # widest window
    assert min(d[:k]) - d[k] > 0.05
    old = float(gpt_oracle.t["gpt.mel_head.bias"][STOP])
    new = float(np.float16(old + 0.5 * (d[k] + min(d[:k]))))
    shift = new - old
    assert d[k] < shift < min(d[:k])
    bundle = mit2.make_gpt_bundle(tmp_path_factory.mktemp("gpt_stop"), seed=0, stop_bias=new)
    with itts_cfm.GptDecoder(bundle, device=0) as dk:
        codes, last = dk.generate(prefix, 8)
    assert codes == want[:k] + [STOP]
    ref = logits[k].astype(np.float64)
    ref[STOP] += shift
    _close(ref, last)


@pytest.mark.parametrize("P,steps,sampled", [(1200, 6, False), (3000, 4, True)])
def test_batched_prefill_matches_row_by_row(gpt_bundle, P, steps, sampled, monkeypatch):
    """Long prefixes: the batched prefill (all rows per layer, fp32 GEMMs,
    causal attention over up to 3000 keys) against the row-by-row pass of
    the persistent decoder (itself checked against the oracle above): same
    codes, logits within rel-L2 1e-4."""
    prefix = np.random.default_rng(P).standard_normal((P, 1280)).astype(np.float32) * np.float32(0.5)
    cfg = dict(seed=5, temperature=0.8, top_k=30, top_p=0.8, repetition_penalty=10.0)

    def run():
        with itts_cfm.GptDecoder(gpt_bundle, device=0) as d:
            if sampled:
                return d.generate_sampled(prefix, steps, cfg, hf_positions=True)
            return d.generate(prefix, steps)

    monkeypatch.delenv("ITTS_GPT_PREFILL", raising=False)
    codes_b, logits_b = run()
    monkeypatch.setenv("ITTS_GPT_PREFILL", "rows")
    codes_r, logits_r = run()
    assert codes_b == codes_r
    _close(logits_r, logits_b)
