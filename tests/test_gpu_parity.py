"""Estimator and sampler parity: the CUDA path through the C-ABI against the
CPU oracle (oracle/dit_oracle.c, itself pinned to the reference's compiled CPU
functions by tests/golden/).

Gates: per-step velocity cosine >= 0.999; final mel
max-abs <= 2e-2 or relative L2 <= 1e-2. f16 GEMM operands with fp32
accumulation; the "unit" bundle makes every sub-path contribute O(1)."""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O
import workloads as W

pytestmark = pytest.mark.gpu

COS_MIN = 0.999
VEL_REL_L2 = 1e-2
MEL_MAX_ABS = 2e-2
MEL_REL_L2 = 1e-2


def _inputs(rng, B, T, P=0):
    x = rng.standard_normal((B, T, 80)).astype(np.float32)
    px = np.zeros((B, T, 80), np.float32)
    px[:, :P] = rng.standard_normal((B, P, 80))
    cond = rng.standard_normal((B, T, 512)).astype(np.float32)
    style = rng.standard_normal((B, 192)).astype(np.float32)
    return x, px, cond, style


def _vel_ok(ref, got):
    c = O.compare(ref, got)
    assert c["cosine"] >= COS_MIN and c["rel_l2"] <= VEL_REL_L2, c
    return c


@pytest.mark.parametrize("T,mask_tail", [(6, 2), (33, 0), (130, 7)])
def test_estimator_vs_oracle(ctx_unit, port_unit, rng, T, mask_tail):
    x, px, cond, style = _inputs(rng, 1, T, P=min(4, T // 3))
    mask = np.ones((1, T), np.uint32)
    if mask_tail:
        mask[0, T - mask_tail :] = 0
    vel = ctx_unit.estimator(x, px, cond, style, mask, t=0.37, branches=2)
    ref_c = port_unit.estimator(x[0], px[0], cond[0], style[0], 0.37, mask[0])
    ref_u = port_unit.estimator(x[0], np.zeros_like(px[0]), np.zeros_like(cond[0]), np.zeros_like(style[0]), 0.37, mask[0])
    _vel_ok(ref_c, vel[0, 0])
    _vel_ok(ref_u, vel[0, 1])


def test_estimator_batched_masks(ctx_unit, port_unit, rng):
    B, T = 3, 40
    x, px, cond, style = _inputs(rng, B, T, P=5)
    mask = np.ones((B, T), np.uint32)
    mask[1, 30:] = 0
    mask[2, ::3] = 0
    vel = ctx_unit.estimator(x, px, cond, style, mask, t=0.8, branches=2)
    for b in range(B):
        _vel_ok(port_unit.estimator(x[b], px[b], cond[b], style[b], 0.8, mask[b]), vel[b, 0])


def test_estimator_baseline_bundle(ctx_baseline, port_baseline, rng):
    T = 48
    x, px, cond, style = _inputs(rng, 1, T, P=10)
    mask = np.ones((1, T), np.uint32)
    vel = ctx_baseline.estimator(x, px, cond, style, mask, t=0.5, branches=2)
    _vel_ok(port_baseline.estimator(x[0], px[0], cond[0], style[0], 0.5, mask[0]), vel[0, 0])


def _mel_ok(ref, got):
    c = O.compare(ref, got)
    assert c["max_abs"] <= MEL_MAX_ABS or c["rel_l2"] <= MEL_REL_L2, c
    return c


@pytest.mark.parametrize("cfg,steps", [(0.7, 3), (0.0, 2)])
def test_sampler_vs_oracle(ctx_unit, port_unit, rng, cfg, steps):
    T, P = 24, 6
    u = W.utterance(rng, T, P)
    got = ctx_unit.run(u.noise, u.prompt, u.cond, u.style, steps, cfg)
    ref, trace = port_unit.euler(u.noise, u.prompt_x(), u.cond, u.style, P, steps, cfg, trace=True)
    _mel_ok(ref, got)
    assert np.all(got[:P] == 0.0)


def test_sampler_teacher_forced_velocity(ctx_unit, port_unit, rng):
    """Per-step guided velocity on the oracle's own trajectory (cosine >= 0.999)."""
    T, P, steps, cfg = 20, 4, 4, 0.7
    u = W.utterance(rng, T, P)
    x = u.noise.copy()
    x[:P] = 0
    t = np.float32(0.0)
    dt = np.float32(1.0) / np.float32(steps)
    mask = np.ones((1, T), np.uint32)
    px = u.prompt_x()
    for _ in range(steps):
        vel = ctx_unit.estimator(x[None], px[None], u.cond[None], u.style[None], mask, t=float(t), branches=2)
        guided = (1 + cfg) * vel[0, 0] - cfg * vel[0, 1]
        ref = port_unit.estimator(x, px, u.cond, u.style, float(t), mask[0])
        ref_u = port_unit.estimator(x, np.zeros_like(px), np.zeros_like(u.cond), np.zeros_like(u.style), float(t), mask[0])
        ref_g = (1 + cfg) * ref - cfg * ref_u
        _vel_ok(ref_g, guided)
        x = x + dt * ref_g
        x[:P] = 0
        t = np.float32(t + dt)


def test_padded_batch_vs_oracle(ctx_unit, port_unit, rng):
    """Padded batch: each utterance equals the masked sampler at the padded length."""
    utts = [W.utterance(rng, T, P) for T, P in ((40, 8), (29, 3), (17, 0))]
    Tp = 40
    vl, pl, noise, px, cond, style = W.pad_batch(utts, Tp)
    got = ctx_unit.run_padded(vl, pl, noise, px, cond, style, steps=2, cfg_rate=0.7)
    for b, u in enumerate(utts):
        mask = (np.arange(Tp) < u.T).astype(np.uint32)
        ref = port_unit.euler(noise[b], px[b], cond[b], style[b], u.P, 2, 0.7, mask=mask)
        _mel_ok(ref[: u.T], got[b, : u.T])


def test_run_batch_buckets_equal_padded(ctx_unit, rng):
    """itts_cfm_run_batch == itts_cfm_run_padded at the length each
    utterance's launch is padded to (the longest of its length class), bitwise;
    an utterance that is the longest of its class equals itts_cfm_run."""
    import itts_cfm

    utts = [W.utterance(rng, T, P) for T, P in ((100, 10), (140, 20), (60, 5))]
    outs = ctx_unit.run_batch([dict(noise=u.noise, prompt=u.prompt, cond=u.cond, style=u.style) for u in utts], 2, 0.7)
    lens = itts_cfm.batch_padded_lengths([u.T for u in utts], 0.7)
    assert lens == [100, 140, 100]
    for u, o, Tp in zip(utts, outs, lens):
        vl, pl, noise, px, cond, style = W.pad_batch([u], Tp)
        ref = ctx_unit.run_padded(vl, pl, noise, px, cond, style, 2, 0.7)[0, : u.T]
        assert np.array_equal(ref, o)
    assert np.array_equal(outs[1], ctx_unit.run(utts[1].noise, utts[1].prompt, utts[1].cond, utts[1].style, 2, 0.7))


def test_batch_invariance_and_determinism(ctx_unit, rng):
    """Rows never mix across sequences: an utterance alone and inside a batch
    give bitwise-identical mels; repeated runs are bitwise identical."""
    utts = [W.utterance(rng, 64, 8) for _ in range(3)]
    vl, pl, noise, px, cond, style = W.pad_batch(utts, 64)
    batch = ctx_unit.run_padded(vl, pl, noise, px, cond, style, 3, 0.7)
    again = ctx_unit.run_padded(vl, pl, noise, px, cond, style, 3, 0.7)
    assert np.array_equal(batch, again)
    for b, u in enumerate(utts):
        alone = ctx_unit.run(u.noise, u.prompt, u.cond, u.style, 3, 0.7)
        assert np.array_equal(alone, batch[b])


def test_reference_kat_sincos_estimator(ctx_unit, port_unit):
    """The reference's own estimator self-test inputs (T=6, t=0.37, mask 111100)."""
    T = 6
    i = np.arange(T * 80, dtype=np.float32)
    x = (np.sin(i * np.float32(0.021)) * np.float32(0.10) + np.cos((np.arange(T * 80) % 53).astype(np.float32) * np.float32(0.017)) * np.float32(0.04)).reshape(T, 80)
    px = (np.cos(i * np.float32(0.019)) * np.float32(0.08) + np.sin((np.arange(T * 80) % 47).astype(np.float32) * np.float32(0.023)) * np.float32(0.03)).reshape(T, 80)
    ic = np.arange(T * 512, dtype=np.float32)
    cond = (np.sin(ic * np.float32(0.010)) * np.float32(0.09) + np.cos((np.arange(T * 512) % 127).astype(np.float32) * np.float32(0.013)) * np.float32(0.05)).reshape(T, 512)
    style = np.cos(np.arange(192, dtype=np.float32) * np.float32(0.016)) * np.float32(0.20)
    mask = np.array([[1, 1, 1, 1, 0, 0]], np.uint32)
    vel = ctx_unit.estimator(x[None], px[None], cond[None], style[None], mask, t=0.37, branches=1)
    _vel_ok(port_unit.estimator(x, px, cond, style, 0.37, mask[0]), vel[0, 0])


def test_full_size_config2_single_step(ctx_baseline, port_baseline):
    """Config 2 size (T=800, P=200): one teacher-forced guided step vs the oracle."""
    u = W.config_utterances(2)[0]
    x = u.noise.copy()
    x[: u.P] = 0
    mask = np.ones((1, u.T), np.uint32)
    px = u.prompt_x()
    vel = ctx_baseline.estimator(x[None], px[None], u.cond[None], u.style[None], mask, t=0.0, branches=2)
    ref_c = port_baseline.estimator(x, px, u.cond, u.style, 0.0, mask[0])
    _vel_ok(ref_c, vel[0, 0])


def test_single_file_bundle_context(ctx_unit, unit_tensors, tmp_path, rng):
    """A context created from the one-file form of the bundle computes exactly
    what the directory form computes."""
    import itts_cfm
    import mit2

    f = tmp_path / "unit.mit2"
    mit2.write_single_file_bundle(f, mit2.make_dit_tensors(0, "unit"))
    T = 24
    x, px, cond, style = _inputs(rng, 1, T, P=4)
    mask = np.ones((1, T), np.uint32)
    with itts_cfm.Context(f, device=0) as one:
        got = one.estimator(x, px, cond, style, mask, t=0.3, branches=2)
    want = ctx_unit.estimator(x, px, cond, style, mask, t=0.3, branches=2)
    assert np.array_equal(got, want)
