"""Skinny-token GEMM (fast mode, M <= 128 rows: the decode step's projections)
through the C ABI against a plain PyTorch FP32 reference on the same BF16
operands.

The kernel streams the weights as the MMA's 128-row side, splits K over a
thread-block cluster of 1-16 CTAs and sums the partial tiles on chip in K order.
Tolerance: FP32 accumulation of BF16 products, so |C - ref| <= 1e-4 * (1 +
max|ref|) for the FP32 outputs; the SwiGLU output is BF16 (2^-8 relative) plus
the fast exponential: |h - ref| <= 1e-2 |ref| + 1e-3.
"""
import pytest
import torch

import n550_qwen3_bringup_handover_b200 as n5

pytestmark = pytest.mark.gpu

SHAPES = [            # (N, K): q/k/v, o, down, odd sizes
    (4096, 1024), (1024, 2048), (1024, 3072), (200, 520), (136, 40),
]


def operands(M, N, K, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    a = torch.randn((M, K), device="cuda", generator=g).to(torch.bfloat16)
    b = (torch.randn((N, K), device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    return a, b


def close_f32(c, ref):
    tol = 1e-4 * (1.0 + ref.abs().max().item())
    err = (c - ref).abs().max().item()
    assert err <= tol, (err, tol)


@pytest.fixture
def skinny_cs():
    """Sets the K-split cluster size for one test, restores automatic."""
    def set_cs(cs):
        n5.check(n5.lib().n550_gemm_skinny_config(cs))
    yield set_cs
    n5.lib().n550_gemm_skinny_config(0)


@pytest.mark.parametrize("M", [9, 16, 17, 32, 33, 64, 100, 128])
@pytest.mark.parametrize("N,K", SHAPES)
def test_skinny_gemm_f32(skinny_cs, M, N, K):
    """FP32-output GEMMs of 9-128 rows take the skinny GEMM by default (from 33
    rows in 64- and 128-column token tiles); above 32 rows also with the
    cluster size forced to 4."""
    a, b = operands(M, N, K, 100 + M + N + K)
    ref = a.float() @ b.float().T
    for cs in ((0, 4) if M > 32 else (0,)):
        skinny_cs(cs)
        c = n5.gemm(a, b)
        torch.cuda.synchronize()
        assert n5.device_status() == n5.OK
        close_f32(c, ref)


@pytest.mark.parametrize("cs,K", [(1, 512), (2, 1024), (3, 1024), (5, 576), (8, 3072), (16, 3072)])
def test_skinny_cluster_sizes_agree(skinny_cs, cs, K):
    """K splits over 1 to 16 CTAs per cluster (uneven ones included: 16 k-tiles
    over 3 CTAs, 9 over 5) give the reference result, and the same split twice
    gives the same bits."""
    M, N = 40, 1024
    a, b = operands(M, N, K, 7)
    skinny_cs(cs)
    c1 = n5.gemm(a, b)
    c2 = n5.gemm(a, b)
    torch.cuda.synchronize()
    assert n5.device_status() == n5.OK
    assert torch.equal(c1, c2)
    close_f32(c1, a.float() @ b.float().T)


@pytest.mark.parametrize("M", [12, 32, 128])
def test_skinny_residual(skinny_cs, M):
    skinny_cs(0 if M <= 32 else 8)
    N, K = 1024, 2048
    a, b = operands(M, N, K, 11)
    x0 = torch.randn((M, N), device="cuda")
    x = x0.clone()
    n5.gemm_residual(a, b, x)
    torch.cuda.synchronize()
    close_f32(x, x0 + a.float() @ b.float().T)


def test_skinny_residual_strided():
    """Strided x (ldx > N) and A rows inside a wider buffer: only the M x N
    block changes."""
    M, N, K = 24, 1024, 1024
    a_wide, b = operands(M, N, 2 * K, 12)
    a = a_wide[:, :K]
    xw = torch.randn((M, N + 64), device="cuda")
    x0 = xw.clone()
    n5.gemm_residual(a, b[:, :K].contiguous(), xw[:, :N])
    torch.cuda.synchronize()
    close_f32(xw[:, :N], x0[:, :N] + a.float() @ b[:, :K].float().T)
    assert torch.equal(xw[:, N:], x0[:, N:])


@pytest.mark.parametrize("M", [10, 32, 64, 128])
def test_skinny_swiglu(skinny_cs, M):
    skinny_cs(0 if M <= 32 else 4)
    N, K = 3072, 1024
    a, wg = operands(M, N, K, 21)
    _, wu = operands(M, N, K, 22)
    h = n5.gemm_swiglu(a, wg, wu)
    torch.cuda.synchronize()
    g = a.float() @ wg.float().T
    u = a.float() @ wu.float().T
    ref = torch.nn.functional.silu(g) * u
    err = (h.float() - ref).abs()
    assert (err <= 1e-2 * ref.abs() + 1e-3).all(), err.max().item()


def test_skinny_off_switch_agrees(skinny_cs):
    """-1 routes skinny M back to the split-K GEMM with partials in global
    memory; both agree within the FP32 tolerance."""
    M, N, K = 24, 4096, 1024
    a, b = operands(M, N, K, 31)
    on = n5.gemm(a, b)
    skinny_cs(-1)
    off = n5.gemm(a, b)
    torch.cuda.synchronize()
    close_f32(on, off)
