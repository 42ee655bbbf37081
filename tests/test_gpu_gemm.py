"""The tensor-core float32 GEMM (tcgen05 kind::tf32 with the 3xTF32 split, C ABI mmk_gemm_tf32x3) against a float64
product, and the radial MLP layer built on it.

Tolerance: elementwise |C - C64| <= 1e-5 * (|A| . |B|^T), i.e. float32-level relative error of every dot product's
magnitude (a plain TF32 product is ~1e-3; float32 with K-term accumulation ~1e-7 .. 1e-5), and the largest error at
most 5x that of a float32 SIMT product (torch.matmul with TF32 off) on the same operands.
"""
import numpy as np
import pytest
import torch

from mace_mps_kernels_b200 import gemm

pytestmark = pytest.mark.gpu

REL = 1e-5

SHAPES = [
    (5218, 1280, 64),        # radial MLP last layer, configs[1] layer 2 (forward)
    (5218, 64, 1280),        # its input gradient
    (5218, 512, 64), (5218, 64, 512),
    (20000, 2176, 64),       # configs[4] layer 2
    (1, 64, 64), (127, 256, 32), (129, 260, 36), (300, 48, 100), (1000, 132, 4), (64, 16, 2176), (333, 200, 64),
    (1000, 64, 2176), (731294 // 64, 2176, 64),
]


def _check(C, A, B):
    A64, B64 = A.double().cpu(), B.double().cpu()
    ref = A64 @ B64.T
    mag = A64.abs() @ B64.abs().T
    err = (C.double().cpu() - ref).abs()
    worst = float((err / (mag + 1e-30)).max())
    assert worst <= REL, f'relative error {worst:.2e}'
    return worst


@pytest.mark.parametrize('M,N,K', SHAPES)
def test_gemm_matches_float64(cuda, M, N, K):
    g = torch.Generator(device='cpu').manual_seed(M * 7 + N * 3 + K)
    A = torch.randn(M, K, generator=g).to(cuda)
    B = torch.randn(N, K, generator=g).to(cuda)
    hi, lo = gemm.tf32_split(B)
    C = gemm.matmul_nt(A, hi, lo)
    torch.cuda.synchronize()
    mine = _check(C, A, B)
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        fp32 = (A.double().cpu() @ B.double().cpu().T - (A @ B.T).double().cpu()).abs().max()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    assert float((C.double().cpu() - A.double().cpu() @ B.double().cpu().T).abs().max()) <= 5 * float(fp32) + 1e-30, mine
    C2 = gemm.matmul_nt(A, hi, lo)                   # deterministic: the same bits again
    assert torch.equal(C, C2)
    assert gemm.status() == 0


def test_gemm_strided_operands(cuda):
    A = torch.randn(700, 96, device=cuda)[:, :64]    # row stride 96 floats
    B = torch.randn(320, 80, device=cuda)[:, :64]
    hi, lo = gemm.tf32_split(B.contiguous())
    out = torch.full((700, 400), float('nan'), device=cuda)
    gemm.matmul_nt(A, hi, lo, out=out[:, :320])
    _check(out[:, :320], A, B)
    assert torch.isnan(out[:, 320:]).all()           # nothing written past N in a strided output


def test_device_split_equals_host_split(cuda):
    x = torch.randn(100000) * torch.logspace(-20, 20, 100000)
    hi_h, lo_h = gemm.tf32_split_host(x)
    hi_d, lo_d = gemm.tf32_split(x.to(cuda))
    assert torch.equal(hi_h, hi_d.cpu()) and torch.equal(lo_h, lo_d.cpu())


@pytest.mark.parametrize('K,N', [(64, 1280), (64, 2176), (7, 96), (30, 33)])
def test_tensor_core_linear_fwd_bwd(cuda, K, N):
    W = torch.randn(K, N, device=cuda) / K ** 0.5
    op = gemm.TensorCoreLinear(W)
    x = torch.randn(3001, K, device=cuda, requires_grad=True)
    y = op(x)
    g = torch.randn_like(y)
    (gx,) = torch.autograd.grad(y, x, g)
    W64, x64, g64 = W.double().cpu(), x.detach().double().cpu(), g.double().cpu()
    assert y.shape == (3001, N) and gx.shape == (3001, K)
    assert float(((y.double().cpu() - x64 @ W64).abs() / (x64.abs() @ W64.abs() + 1e-30)).max()) <= REL
    assert float(((gx.double().cpu() - g64 @ W64.T).abs() / (g64.abs() @ W64.abs().T + 1e-30)).max()) <= REL
