"""Kernel-level parity on the GPU through the C-ABI op entry points, each
against a plain PyTorch fp32 computation of the same op on the same f16
inputs. Tolerances are stated per test."""
from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def _dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


def _rel_err(ref, got):
    ref = ref.double()
    got = got.double()
    return float((got - ref).norm() / max(ref.norm().item(), 1e-30)), float((got - ref).abs().max())


@pytest.mark.parametrize(
    "M,N,K,bn",
    [
        (1, 512, 512, 128),
        (127, 512, 512, 128),
        (128, 1536, 512, 128),
        (300, 3072, 512, 256),
        (1600, 512, 1536, 128),
        (1600, 80, 512, 80),
        (513, 512, 128, 128),
        (257, 512, 832, 128),
        (129, 512, 704, 64),
        (1000, 1024, 2560, 256),
        (1600, 512, 128, 64),
        (300, 512, 832, 64),
        (1600, 1536, 512, 192),
        (77, 1536, 512, 192),
    ],
)
def test_gemm_plain(ctx_unit, M, N, K, bn):
    dev = _dev()
    g = torch.Generator(device="cpu").manual_seed(M * 7 + N + K)
    a = torch.randn(M, K, generator=g).half().to(dev)
    b = (torch.randn(N, K, generator=g) / K**0.5).half().to(dev)
    bias = torch.randn(N, generator=g).float().to(dev)
    c = torch.full((M, N), float("nan"), device=dev)
    ctx_unit.op_gemm(a.data_ptr(), K, None, 0, 0, b.data_ptr(), K, bias.data_ptr(), c.data_ptr(), N, M, N, K, bn)
    ref = a.float() @ b.float().T + bias
    rel, mx = _rel_err(ref, c)
    # fp32 accumulation of exact f16 products: only summation order differs.
    assert rel < 1e-5 and mx < 1e-3, (rel, mx)


@pytest.mark.parametrize(
    "M,N,K,bn",
    [
        (128, 512, 512, 64),
        (1600, 512, 512, 64),
        (300, 1536, 512, 256),
        (1600, 3072, 512, 128),
        (257, 512, 832, 128),
        (129, 512, 704, 64),
        (1000, 1024, 2560, 256),
        (4096, 512, 1536, 256),
    ],
)
def test_gemm_pair(ctx_unit, M, N, K, bn):
    """CTA-pair form (clusters of 2, cta_group::2 MMA over 256-row tiles)."""
    import itts_cfm

    dev = _dev()
    g = torch.Generator(device="cpu").manual_seed(M * 11 + N + K)
    a = torch.randn(M, K, generator=g).half().to(dev)
    b = (torch.randn(N, K, generator=g) / K**0.5).half().to(dev)
    bias = torch.randn(N, generator=g).float().to(dev)
    c = torch.full((M, N), float("nan"), device=dev)
    ctx_unit.op_gemm(a.data_ptr(), K, None, 0, 0, b.data_ptr(), K, bias.data_ptr(), c.data_ptr(), N, M, N, K,
                     bn | itts_cfm.ITTS_GEMM_PAIR)
    ref = a.float() @ b.float().T + bias
    rel, mx = _rel_err(ref, c)
    assert rel < 1e-5 and mx < 1e-3, (rel, mx)


@pytest.mark.parametrize("bn", [64, 128, 128 | 0x10000])
def test_gemm_split_two_sources(ctx_unit, bn):
    """[x_normed(512) | x_mel(80)] @ W^T without a concat buffer (skip_linear shape)."""
    dev = _dev()
    M = 333
    g = torch.Generator(device="cpu").manual_seed(5)
    a0 = torch.randn(M, 512, generator=g).half().to(dev)
    a1 = torch.zeros(M, 128).half()
    a1[:, :80] = torch.randn(M, 80, generator=g).half()
    a1 = a1.to(dev)
    w = torch.zeros(512, 640).half()
    w[:, :592] = (torch.randn(512, 592, generator=g) / 592**0.5).half()
    w = w.to(dev)
    bias = torch.randn(512, generator=g).float().to(dev)
    c = torch.empty(M, 512, device=dev)
    # columns 80..127 of a1 and 592..639 of w are the zero padding of the 64-column k-blocks
    ctx_unit.op_gemm(a0.data_ptr(), 512, a1.data_ptr(), 128, 512, w.data_ptr(), 640, bias.data_ptr(), c.data_ptr(), 512,
                     M, 512, 640, bn)
    ref = torch.cat([a0, a1], 1).float() @ w.float().T + bias
    rel, mx = _rel_err(ref, c)
    assert rel < 1e-5 and mx < 1e-3, (rel, mx)


@pytest.mark.parametrize("S,T", [(1, 2), (2, 5), (3, 127), (2, 300)])
def test_conv5_reflect(ctx_unit, S, T):
    """Implicit-GEMM k=5 conv over reflect-padded rows vs torch conv1d(reflect)."""
    dev = _dev()
    g = torch.Generator(device="cpu").manual_seed(S * 1000 + T)
    x = torch.randn(S, T, 512, generator=g).half()
    w = (torch.randn(1024, 512, 5, generator=g) / (512 * 5) ** 0.5).half()
    bias = torch.randn(1024, generator=g).float()
    # reflect-padded rows [S, T+4, 512] (torch reflect == reference reflect_pad_1d for T >= 3)
    idx = []
    for j in range(-2, T + 2):
        s = j
        while s < 0 or s >= T:
            if s < 0:
                s = -s
            if s >= T:
                s = 2 * T - 2 - s
        idx.append(s)
    xp = x[:, idx, :].contiguous().to(dev)
    wt = w.permute(0, 2, 1).contiguous().reshape(1024, 2560).to(dev)  # [out][tap][in]
    out = torch.full((S * T, 1024), float("nan"), device=dev)
    ctx_unit.op_conv5(xp.data_ptr(), S, T, wt.data_ptr(), bias.to(dev).data_ptr(), out.data_ptr(), 1024)
    xpf = x[:, idx, :].float().permute(0, 2, 1)  # [S, 512, T+4]
    ref = torch.nn.functional.conv1d(xpf, w.float(), bias).permute(0, 2, 1).reshape(S * T, 1024)
    rel, mx = _rel_err(ref.to(dev), out)
    assert rel < 1e-5 and mx < 1e-3, (rel, mx)


@pytest.mark.parametrize("S,T,masked", [(1, 1, False), (2, 5, True), (3, 64, False), (2, 65, True), (2, 333, True),
                                         (1, 800, False), (2, 800, True), (20, 300, True), (40, 800, True),
                                         (1, 4096, False)])
def test_attention(ctx_unit, S, T, masked):
    dev = _dev()
    g = torch.Generator(device="cpu").manual_seed(S * 100 + T)
    qkv = torch.randn(S * T, 1536, generator=g)
    qkv[:, :512] *= 0.125
    qkv = qkv.half().to(dev)
    mask = torch.ones(S * T)
    if masked:
        mask = (torch.rand(S * T, generator=g) > 0.3).float()
        mask.view(S, T)[:, 0] = 1.0  # at least one live key per sequence
    mask = mask.to(dev)
    out = torch.full((S * T, 512), float("nan"), device=dev, dtype=torch.float16)
    ctx_unit.op_attention(qkv.data_ptr(), mask.data_ptr(), out.data_ptr(), S, T)
    q = qkv[:, :512].float().view(S, T, 8, 64).permute(0, 2, 1, 3)
    k = qkv[:, 512:1024].float().view(S, T, 8, 64).permute(0, 2, 1, 3)
    v = qkv[:, 1024:].float().view(S, T, 8, 64).permute(0, 2, 1, 3)
    sc = q @ k.transpose(-1, -2)
    sc = sc.masked_fill(mask.view(S, 1, 1, T) == 0, float("-inf"))
    ref = (torch.softmax(sc, -1) @ v).permute(0, 2, 1, 3).reshape(S * T, 512)
    rel, mx = _rel_err(ref, out.float())
    # P is rounded to f16 before PV and the output to f16: ~1e-3 relative.
    assert rel < 2e-3 and mx < 1e-2, (rel, mx)


@pytest.mark.parametrize("R", [1, 7, 1600])
def test_adarms(ctx_unit, R):
    dev = _dev()
    g = torch.Generator(device="cpu").manual_seed(R)
    x = (torch.randn(R, 512, generator=g) * 3).to(dev)
    wb = torch.randn(1024, generator=g).to(dev)
    gamma = torch.rand(512, generator=g).to(dev) + 0.5
    y = torch.empty(R, 512, device=dev, dtype=torch.float16)
    ctx_unit.op_adarms(x.data_ptr(), R, wb.data_ptr(), gamma.data_ptr(), y.data_ptr())
    inv = torch.rsqrt((x * x).mean(-1, keepdim=True) + 1e-5)
    ref = wb[:512] * (x * inv * gamma) + wb[512:]
    rel, mx = _rel_err(ref, y.float())
    assert rel < 1e-3, (rel, mx)
