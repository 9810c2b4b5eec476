"""GPU parity of the GEMM against the oracle, through the C ABI.

exact mode: bit-identical to the AME golden semantics -- the 12 shipped
cases (with their row strides), BASELINE config 1 against the reference
generator's own output at K-block 16 and 32, and random/edge shapes against
the C oracle.
fast mode (tcgen05 / GEMV / CUDA-core paths): max|C - C_ref| / max|C_ref| <= 1e-4
against a binary64 reference of the same BF16 operands (FP32 accumulation of
K <= 3072 terms), and <= 2^-7 when C is rounded to BF16.
"""
import numpy as np
import pytest

import oracle
import n550_qwen3_bringup_handover_b200 as n5
from tests.conftest import bf16_bits, case_operands, to_dev_bf16

pytestmark = pytest.mark.gpu

CASE_IDS = ["001", "002", "003", "004", "005", "006", "007", "008",
            "009a", "009b", "010", "011"]

FAST_TOL = 1e-4
BF16_OUT_TOL = 2.0 ** -7


def exact_dev(a_bits, b_bits, M, N, K, lda, ldb, kb, dev):
    import torch
    a = to_dev_bf16(a_bits, dev)
    b = to_dev_bf16(b_bits, dev)
    c = torch.full((M, N), float("nan"), dtype=torch.float32, device=dev)  # dirty preset
    n5.gemm(a, b, mode=n5.MODE_EXACT, kblock=kb, out=c, M=M, N=N, K=K)
    torch.cuda.synchronize()
    assert n5.device_status() == n5.OK
    return c.cpu().numpy().view(np.uint32)


@pytest.mark.parametrize("cid", CASE_IDS)
def test_exact_shipped_cases(cuda, golden_cases, cid):
    a, b, M, N, K, lda, ldb, a_src = case_operands(golden_cases, cid)
    c = exact_dev(a, b, M, N, K, lda, ldb, 16, cuda)
    assert np.array_equal(c, golden_cases[f"{cid}/c_ref"])
    if f"{cid}/xor_ref" in golden_cases:
        assert int(np.bitwise_xor.reduce(c.ravel())) == int(golden_cases[f"{cid}/xor_ref"][0])


@pytest.mark.parametrize("cid", ["009a", "010", "011"])
def test_exact_fp32_activation_staging(cuda, golden_cases, cid):
    """Mixed cases: FP32 a_src rounded to BF16 RNE inside the kernel."""
    import torch
    a, b, M, N, K, lda, ldb, a_src = case_operands(golden_cases, cid)
    at = torch.from_numpy(np.ascontiguousarray(a_src)).to(cuda)
    bt = to_dev_bf16(b, cuda)
    c = n5.gemm(at, bt, mode=n5.MODE_EXACT, kblock=16, M=M, N=N, K=K)
    assert np.array_equal(c.cpu().numpy().view(np.uint32), golden_cases[f"{cid}/c_ref"])


@pytest.mark.parametrize("kb", [16, 32])
def test_exact_config1_vs_reference_generator(cuda, config1_golden, kb):
    M, K, N, seed = (int(v) for v in config1_golden["meta"])
    A = oracle.synth_normal_bf16((M, K), seed, 0x41, 1.0)
    B = oracle.synth_normal_bf16((N, K), seed, 0x42, 0.02)
    c = exact_dev(A, B, M, N, K, K, K, kb, cuda)
    assert np.array_equal(c, config1_golden[f"c_kb{kb}"])


EXACT_SHAPES = [(1, 1, 1), (7, 13, 17), (1, 1024, 2048), (65, 129, 33), (128, 64, 1024),
                (3, 200, 3072), (16, 1, 15), (0, 4, 8), (4, 0, 8), (5, 6, 0)]


@pytest.mark.parametrize("M,N,K", EXACT_SHAPES)
@pytest.mark.parametrize("kb", [16, 32])
def test_exact_random_shapes_vs_oracle(cuda, M, N, K, kb):
    A = oracle.synth_normal_bf16((M, K), 11 + M, 0x41, 1.0)
    B = oracle.synth_normal_bf16((N, K), 11 + N, 0x42, 0.02)
    c_ref, _ = oracle.gemm_ame_exact(A, B, kb, M=M, N=N, K=K, lda=max(K, 1), ldb=max(K, 1))
    if M == 0 or N == 0:
        return
    c = exact_dev(A, B, M, N, K, K, K, kb, cuda)
    assert np.array_equal(c, c_ref)


@pytest.mark.parametrize("M,sparse", [(37, False), (5, False), (5, True), (16, True)])
def test_exact_wide_dynamic_range_fallback(cuda, M, sparse):
    """Blocks whose products span > 53 bits take the integer fallback: every
    block, or (sparse) only the blocks holding a rare +-2^40 outlier, so that
    exact and fallback blocks alternate in one output. 37 rows run the 64 x 64
    tiles, 5 and 16 rows the one-output-per-thread tiles whose consecutive
    K-blocks are summed as independent chains."""
    rng = np.random.default_rng(3 + M)
    N, K = 41, 200
    if sparse:
        v = rng.standard_normal((M + N, K))
        hit = rng.random((M + N, K)) < 0.01
        v[hit] = np.sign(v[hit]) * 2.0 ** 40
    else:
        v = np.sign(rng.standard_normal((M + N, K))) * np.exp2(rng.uniform(-60, 60, (M + N, K)))
    bits = oracle.f32_to_bf16(v.astype(np.float32))
    A, B = bits[:M], bits[M:]
    for kb in (16, 32):
        c_ref, _ = oracle.gemm_ame_exact(A, B, kb)
        assert np.array_equal(exact_dev(A, B, M, N, K, K, K, kb, cuda), c_ref)


def test_exact_host_shim_qwen3_gemm(cuda):
    """qwen3_gemm over host buffers (FP32 A) in the default exact mode."""
    rng = np.random.default_rng(5)
    M, K, N = 4, 1024, 2048
    a = rng.uniform(-1, 1, (M, K)).astype(np.float32)
    b = oracle.synth_normal_bf16((N, K), 3, 0x42, 0.02)
    n5.set_gemm_mode(n5.MODE_EXACT, 16)
    c = n5.qwen3_gemm(a, b)
    assert np.array_equal(c, oracle.gemm_ame_exact_f32a(a, b, 16))
    # kernels_hwsim.c agrees here too (block sums exact in binary64)
    assert np.array_equal(c, oracle.gemm_hwsim(a, b))


def test_exact_host_shim_tile_major_layout(cuda):
    """qwen3_gemm with tile-major weights after qwen3_set_weight_layout(TILE)."""
    M, K, N = 3, 256, 384
    a = oracle.synth_normal_f32((M, K), 1, 0x41, 1.0)
    b = oracle.synth_normal_bf16((N, K), 1, 0x42, 0.02)
    tiled = b.reshape(N // 128, 128, K // 32, 32).transpose(0, 2, 1, 3).copy()
    try:
        assert n5.qwen3_set_weight_layout(n5.LAYOUT_TILE, 128, 32) == 0
        c_t = n5.qwen3_gemm(a, tiled.reshape(N, K))
        c_r = n5.qwen3_gemm_row(a, b)
    finally:
        n5.qwen3_set_weight_layout(n5.LAYOUT_ROW, 0, 0)
    ref = oracle.gemm_ame_exact_f32a(a, b, 16)
    assert np.array_equal(c_t, ref) and np.array_equal(c_r, ref)


def f64_ref(A_bits, B_bits):
    a = oracle.bf16_to_f32(A_bits).astype(np.float64)
    b = oracle.bf16_to_f32(B_bits).astype(np.float64)
    return a @ b.T


def rel_err(c, ref):
    return float(np.abs(c.astype(np.float64) - ref).max() / max(np.abs(ref).max(), 1e-30))


# test_kernels.c:74-90 shapes plus the model's projection shapes and tails
FAST_SHAPES = [(1, 1024, 2048), (1, 1024, 1024), (1, 2048, 1024), (1, 1024, 3072),
               (1, 3072, 1024), (4, 1024, 2048), (127, 1024, 1024), (128, 1024, 1024),
               (129, 1024, 1024), (8, 32, 128), (8, 64, 128), (8, 33, 128),
               (9, 1024, 4096), (300, 1024, 6144), (256, 3072, 1024), (1000, 2048, 1024),
               (64, 1024, 1000), (2, 1024, 151936)]


@pytest.mark.parametrize("M,K,N", FAST_SHAPES)
def test_fast_vs_f64_reference(cuda, M, K, N):
    import torch
    A = oracle.synth_normal_bf16((M, K), 21, 0x41, 1.0)
    B = oracle.synth_normal_bf16((N, K), 21, 0x42, 0.02)
    c = n5.gemm(to_dev_bf16(A, cuda), to_dev_bf16(B, cuda), mode=n5.MODE_FAST)
    torch.cuda.synchronize()
    assert n5.device_status() == n5.OK
    assert rel_err(c.cpu().numpy(), f64_ref(A, B)) <= FAST_TOL


@pytest.mark.parametrize("M,K,N", [(1, 1024, 2048), (256, 1024, 4096), (77, 3072, 1024)])
def test_fast_bf16_output(cuda, M, K, N):
    import torch
    A = oracle.synth_normal_bf16((M, K), 2, 0x41, 1.0)
    B = oracle.synth_normal_bf16((N, K), 2, 0x42, 0.02)
    c = n5.gemm(to_dev_bf16(A, cuda), to_dev_bf16(B, cuda), mode=n5.MODE_FAST,
                out_dtype=torch.bfloat16)
    got = oracle.bf16_to_f32(bf16_bits(c)).astype(np.float64)
    assert rel_err(got, f64_ref(A, B)) <= BF16_OUT_TOL


def test_fast_fp32_activations_are_staged_rne(cuda):
    import torch
    rng = np.random.default_rng(9)
    M, K, N = 200, 1024, 512
    a = rng.standard_normal((M, K)).astype(np.float32)
    B = oracle.synth_normal_bf16((N, K), 4, 0x42, 0.02)
    c = n5.gemm(torch.from_numpy(a).to(cuda), to_dev_bf16(B, cuda), mode=n5.MODE_FAST)
    assert rel_err(c.cpu().numpy(), f64_ref(oracle.f32_to_bf16(a), B)) <= FAST_TOL


def test_fast_strided_operands(cuda):
    import torch
    M, K, N = 130, 512, 260
    A = oracle.synth_normal_bf16((M, K + 64), 8, 0x41, 1.0)
    B = oracle.synth_normal_bf16((N, K + 32), 8, 0x42, 0.02)
    a = to_dev_bf16(A, cuda)
    b = to_dev_bf16(B, cuda)
    out = torch.zeros((M, N + 12), dtype=torch.float32, device=cuda)
    n5.gemm(a, b, mode=n5.MODE_FAST, out=out, M=M, N=N, K=K)
    ref = f64_ref(A[:, :K], B[:, :K])
    got = out.cpu().numpy()
    assert rel_err(got[:, :N], ref) <= FAST_TOL
    assert not got[:, N:].any()


def test_fast_host_shim(cuda):
    rng = np.random.default_rng(6)
    a = rng.uniform(-1, 1, (33, 1024)).astype(np.float32)
    b = oracle.synth_normal_bf16((3072, 1024), 6, 0x42, 0.02)
    try:
        n5.set_gemm_mode(n5.MODE_FAST)
        c = n5.qwen3_gemm(a, b)
    finally:
        n5.set_gemm_mode(n5.MODE_EXACT, 16)
    assert rel_err(c, f64_ref(oracle.f32_to_bf16(a), b)) <= FAST_TOL


@pytest.mark.parametrize("M,K,N", [(1, 2048, 1024), (300, 2048, 1024), (129, 3072, 1000), (64, 1024, 1024)])
def test_fused_residual_gemm(cuda, M, K, N):
    """x += A . B^T (qwen3_gemm then qwen3_op_residual_add)."""
    import torch
    A = oracle.synth_normal_bf16((M, K), 31, 0x41, 1.0)
    B = oracle.synth_normal_bf16((N, K), 31, 0x42, 0.02)
    x0 = oracle.synth_normal_f32((M, N), 31, 0x58, 1.0)
    x = torch.from_numpy(x0.copy()).to(cuda)
    n5.gemm_residual(to_dev_bf16(A, cuda), to_dev_bf16(B, cuda), x)
    ref = x0.astype(np.float64) + f64_ref(A, B)
    assert rel_err(x.cpu().numpy(), ref) <= FAST_TOL


@pytest.mark.parametrize("M,K,N,ld", [(2048, 1024, 1024, 1024), (1100, 2048, 1000, 1000),
                                      (1500, 3072, 1024, 1040)])
def test_residual_gemm_tma_add_is_exact(cuda, M, K, N, ld):
    """Large-M residual GEMMs reduce-add their tiles into x through the TMA:
    the result must be bit-identical to the FP32-output GEMM (same tiles, same
    accumulation order) added to x in FP32, and columns past N of a strided x
    must stay untouched."""
    import torch
    A = to_dev_bf16(oracle.synth_normal_bf16((M, K), 37, 0x41, 1.0), cuda)
    B = to_dev_bf16(oracle.synth_normal_bf16((N, K), 37, 0x42, 0.02), cuda)
    x0 = torch.from_numpy(oracle.synth_normal_f32((M, ld), 37, 0x58, 1.0)).to(cuda)
    c = n5.gemm(A, B, mode=n5.MODE_FAST)
    x = x0.clone()
    n5.gemm_residual(A, B, x[:, :N])
    torch.cuda.synchronize()
    assert torch.equal(x[:, :N], x0[:, :N] + c)
    assert torch.equal(x[:, N:], x0[:, N:])


@pytest.mark.parametrize("tile", [128, 256, 512])
@pytest.mark.parametrize("M,K,N,out", [(1100, 1024, 1000, "f32"), (2048, 2048, 1024, "resid"),
                                       (1500, 1024, 768, "swiglu"), (1024, 1024, 4096, "bf16"),
                                       (384, 3072, 1024, "f32")])
def test_tile_shapes(cuda, tile, M, K, N, out):
    """Every fast-GEMM tile shape -- 128- and 256-wide single-CTA tiles and
    256 x 256 tiles on 2-CTA clusters (forced with n550_gemm_tile_config) --
    on ragged M and N, for each epilogue, against binary64."""
    import torch
    A = oracle.synth_normal_bf16((M, K), 53, 0x41, 1.0)
    B = oracle.synth_normal_bf16((N, K), 53, 0x42, 0.02)
    dA, dB = to_dev_bf16(A, cuda), to_dev_bf16(B, cuda)
    try:
        n5.check(n5.lib().n550_gemm_tile_config(tile))
        if out == "swiglu":
            U = oracle.synth_normal_bf16((N, K), 53, 0x55, 0.02)
            h = n5.gemm_swiglu(dA, dB, to_dev_bf16(U, cuda))
            torch.cuda.synchronize()
            g, u = f64_ref(A, B), f64_ref(A, U)
            got = oracle.bf16_to_f32(bf16_bits(h)).astype(np.float64)
            assert rel_err(got, g / (1.0 + np.exp(-g)) * u) <= BF16_OUT_TOL
        elif out == "resid":
            x0 = oracle.synth_normal_f32((M, N), 53, 0x58, 1.0)
            x = torch.from_numpy(x0.copy()).to(cuda)
            n5.gemm_residual(dA, dB, x)
            torch.cuda.synchronize()
            assert rel_err(x.cpu().numpy(), x0.astype(np.float64) + f64_ref(A, B)) <= FAST_TOL
        elif out == "bf16":
            c = n5.gemm(dA, dB, mode=n5.MODE_FAST, out_dtype=torch.bfloat16)
            torch.cuda.synchronize()
            got = oracle.bf16_to_f32(bf16_bits(c)).astype(np.float64)
            assert rel_err(got, f64_ref(A, B)) <= BF16_OUT_TOL
        else:
            c = n5.gemm(dA, dB, mode=n5.MODE_FAST)
            torch.cuda.synchronize()
            assert rel_err(c.cpu().numpy(), f64_ref(A, B)) <= FAST_TOL
    finally:
        n5.lib().n550_gemm_tile_config(0)
    assert n5.device_status() == n5.OK


@pytest.mark.parametrize("M,K,N", [(300, 1024, 3072), (128, 1024, 200), (17, 1024, 64),
                                   (1, 1024, 3072), (3, 1024, 3072), (8, 1024, 200)])
def test_fused_swiglu_gemm(cuda, M, K, N):
    """h = silu(A . Wg^T) * (A . Wu^T) in BF16 (gate/up qwen3_gemm then qwen3_op_silu_mul);
    up to 8 rows through the one-launch SwiGLU GEMV."""
    A = oracle.synth_normal_bf16((M, K), 41, 0x41, 1.0)
    G = oracle.synth_normal_bf16((N, K), 41, 0x47, 0.02)
    U = oracle.synth_normal_bf16((N, K), 41, 0x55, 0.02)
    h = n5.gemm_swiglu(to_dev_bf16(A, cuda), to_dev_bf16(G, cuda), to_dev_bf16(U, cuda))
    g, u = f64_ref(A, G), f64_ref(A, U)
    ref = g / (1.0 + np.exp(-g)) * u
    got = oracle.bf16_to_f32(bf16_bits(h)).astype(np.float64)
    assert rel_err(got, ref) <= BF16_OUT_TOL
