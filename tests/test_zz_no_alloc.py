"""The allocation-free conv entry point (itts_op_conv5_noalloc) against the
context-based one (itts_op_conv5), through the C ABI.

Some callers cannot call cudaMalloc, for example a serving process whose
memory pool already holds the GPU's memory, or a real-time audio thread that
must not take cudaMalloc's device-wide synchronisation. For them the
reflect-padded staging rows of the k=5 conv live in a static device array
inside the library. This file is named so that pytest collects it last. It
passes alone in a fresh process and after the other tests.
"""
from __future__ import annotations

import pytest

import itts_cfm

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def _dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


def _reflect_index(T: int) -> list[int]:
    idx = []
    for j in range(-2, T + 2):
        s = j
        while s < 0 or s >= T:
            if s < 0:
                s = -s
            if s >= T:
                s = 2 * T - 2 - s
        idx.append(s)
    return idx


def _case(S: int, T: int, N: int, seed: int, dev):
    g = torch.Generator(device="cpu").manual_seed(seed)
    x = torch.randn(S, T, 512, generator=g).half()
    w = (torch.randn(N, 5 * 512, generator=g) / (512 * 5) ** 0.5).half()
    bias = torch.randn(N, generator=g).float()
    xp = x[:, _reflect_index(T), :].contiguous()
    return x.to(dev), xp.to(dev), w.to(dev), bias.to(dev)


def test_conv5_noalloc_matches_conv5_twice(ctx_unit):
    """Two calls in a row (a larger then a smaller problem, so the second one
    runs over scratch rows the first left behind; the first fills 16,032 of
    the 16,384 rows) each match itts_op_conv5 on
    the same data. Same kernel on the same padded rows: the bar is the conv
    test's tolerance (rel 1e-5, max abs 1e-3)."""
    dev = _dev()
    for S, T, N, seed in ((8, 2000, 1024, 11), (2, 77, 512, 12)):
        x, xp, w, bias = _case(S, T, N, seed, dev)
        want = torch.full((S * T, N), float("nan"), device=dev)
        ctx_unit.op_conv5(xp.data_ptr(), S, T, w.data_ptr(), bias.data_ptr(), want.data_ptr(), N)
        got = torch.full((S * T, N), float("nan"), device=dev)
        stream = torch.cuda.current_stream(dev).cuda_stream
        itts_cfm.conv5_noalloc(x.data_ptr(), S, T, w.data_ptr(), bias.data_ptr(), got.data_ptr(), N, stream)
        assert torch.isfinite(got).all()
        diff = (got.double() - want.double())
        rel = float(diff.norm() / want.double().norm())
        assert rel < 1e-5 and float(diff.abs().max()) < 1e-3, (S, T, rel)


def test_conv5_noalloc_rejects_beyond_scratch():
    """S*(T+4) above the static array's row count is refused before any GPU
    work, with ITTS_ECAP and a message naming the limit."""
    dev = _dev()
    T = 2000
    S = itts_cfm.NOALLOC_CONV5_MAX_ROWS // (T + 4) + 1
    x = torch.zeros(S * T, 512, device=dev, dtype=torch.float16)
    w = torch.zeros(512, 5 * 512, device=dev, dtype=torch.float16)
    out = torch.zeros(S * T, 512, device=dev)
    with pytest.raises(itts_cfm.IttsError) as ei:
        itts_cfm.conv5_noalloc(x.data_ptr(), S, T, w.data_ptr(), None, out.data_ptr(), 512)
    assert ei.value.code == itts_cfm.ITTS_ECAP
    assert str(itts_cfm.NOALLOC_CONV5_MAX_ROWS) in str(ei.value)


def test_conv5_noalloc_five_weight_tiles(ctx_unit):
    """N = 640 output channels (five 128-row weight tiles) against itts_op_conv5."""
    dev = _dev()
    S, T, N = 3, 131, 640
    x, xp, w, bias = _case(S, T, N, 13, dev)
    want = torch.full((S * T, N), float("nan"), device=dev)
    ctx_unit.op_conv5(xp.data_ptr(), S, T, w.data_ptr(), bias.data_ptr(), want.data_ptr(), N)
    got = torch.full((S * T, N), float("nan"), device=dev)
    itts_cfm.conv5_noalloc(x.data_ptr(), S, T, w.data_ptr(), bias.data_ptr(), got.data_ptr(), N)
    assert torch.isfinite(got).all()
    diff = got.double() - want.double()
    assert float(diff.norm() / want.double().norm()) < 1e-5 and float(diff.abs().max()) < 1e-3


@pytest.mark.parametrize("N", [80, 48, 720])
def test_conv5_noalloc_rejects_partial_weight_tiles(N):
    """N that is not a multiple of 128 is refused with ITTS_EINVAL_SHAPE before any GPU work."""
    dev = _dev()
    x = torch.zeros(2 * 16, 512, device=dev, dtype=torch.float16)
    w = torch.zeros(N, 5 * 512, device=dev, dtype=torch.float16)
    out = torch.zeros(2 * 16, N, device=dev)
    with pytest.raises(itts_cfm.IttsError) as ei:
        itts_cfm.conv5_noalloc(x.data_ptr(), 2, 16, w.data_ptr(), None, out.data_ptr(), N)
    assert ei.value.code == itts_cfm.ITTS_EINVAL_SHAPE
