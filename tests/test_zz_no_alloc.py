"""n550_gemm_f32a_noalloc: the fast-mode GEMM with FP32 activations for
callers that cannot allocate device memory (a fixed-arena runtime in the
reference's no-malloc style, or a host that must not let the call synchronise
the device). Its BF16 staging copy lives in a fixed array inside the library
instead of a per-call allocation.

Checked through the C ABI against the allocating entry point
n550_gemm(MODE_FAST, a_type = F32) and against a binary64 product on several
calls in a row (different shapes, so a stale array would show), within the
fast-mode GEMM tolerance of the other GEMM tests; and an over-limit call is
refused without writing C.
This file is collected last so that a failure here leaves every other test
already run; it also passes alone in a fresh process.
"""
import ctypes as C

import numpy as np
import pytest

import n550_qwen3_bringup_handover_b200 as n5
from tests.conftest import to_dev_bf16

pytestmark = pytest.mark.gpu

FAST_TOL = 1e-4            # same bound as tests/test_gemm_gpu.py
LIMIT_ELEMS = 4 << 20      # M * round_up(K, 8) the entry point accepts


def noalloc_fn():
    fn = n5.lib().n550_gemm_f32a_noalloc
    fn.restype = C.c_int
    fn.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_void_p, C.c_int,
                   C.c_int, C.c_int, C.c_int, C.c_int]
    return fn


def run_noalloc(a, b, out):
    M, K = a.shape
    N = b.shape[0]
    return noalloc_fn()(n5.stream_ptr(), C.c_void_p(a.data_ptr()), a.stride(0),
                        C.c_void_p(b.data_ptr()), b.stride(0), C.c_void_p(out.data_ptr()),
                        n5.F32 if out.dtype.is_floating_point and out.element_size() == 4 else n5.BF16,
                        out.stride(0), M, N, K)


def rel_err(got, ref):
    got = got.double().cpu().numpy()
    ref = ref.double().cpu().numpy()
    return float(np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30))


def f64_reference(a, b_bits):
    """Binary64 product of the BF16-rounded activations and the BF16 weights."""
    import oracle
    a16 = oracle.bf16_to_f32(oracle.f32_to_bf16(a.cpu().numpy())).astype(np.float64)
    return a16 @ oracle.bf16_to_f32(b_bits).astype(np.float64).T


def test_noalloc_matches_allocating_entry_point_twice(cuda):
    """Each route of the entry point on consecutive calls, smaller K after
    larger K so that stale staging contents would show: GEMV (5 rows), the
    CUDA-core kernel for a K that leaves the rows unaligned (17 x 1001, staged
    rows padded to 1008), the tile GEMM, the weight-streaming GEMM (9 rows),
    and the tile GEMM again. Each result is held to the fast-mode tolerance
    against binary64 and against n550_gemm."""
    import torch
    rng = np.random.default_rng(77)
    import oracle
    cases = [(5, 3072, 1024), (17, 1001, 256), (1024, 2048, 256), (9, 3072, 1024), (300, 1024, 768)]
    for M, K, N in cases:
        a = torch.from_numpy(rng.standard_normal((M, K)).astype(np.float32)).to(cuda)
        b_bits = oracle.synth_normal_bf16((N, K), M, 0x42, 0.02)
        b = to_dev_bf16(b_bits, cuda)
        want = n5.gemm(a, b, mode=n5.MODE_FAST)                    # allocating path
        got = torch.full((M, N), float("nan"), dtype=torch.float32, device=cuda)
        assert run_noalloc(a, b, got) == n5.OK
        torch.cuda.synchronize()
        assert n5.device_status() == n5.OK
        assert rel_err(got, want) <= FAST_TOL, (M, K, N)
        ref = f64_reference(a, b_bits)
        g = got.double().cpu().numpy()
        assert float(np.abs(g - ref).max() / np.abs(ref).max()) <= FAST_TOL, (M, K, N)
    # BF16 output through the same array
    M, K, N = 64, 1024, 512
    a = torch.from_numpy(rng.standard_normal((M, K)).astype(np.float32)).to(cuda)
    b_bits = oracle.synth_normal_bf16((N, K), 9, 0x42, 0.02)
    b = to_dev_bf16(b_bits, cuda)
    want = n5.gemm(a, b, mode=n5.MODE_FAST, out_dtype=torch.bfloat16)
    got = torch.empty((M, N), dtype=torch.bfloat16, device=cuda)
    assert run_noalloc(a, b, got) == n5.OK
    assert rel_err(got.float(), want.float()) <= 2.0 ** -7
    ref = f64_reference(a, b_bits)
    assert float(np.abs(got.double().cpu().numpy() - ref).max() / np.abs(ref).max()) <= 2.0 ** -7


def test_noalloc_refuses_sizes_beyond_the_array(cuda):
    import torch
    K = 1024
    M = LIMIT_ELEMS // K + 1
    a = torch.zeros((M, K), dtype=torch.float32, device=cuda)
    b = torch.zeros((8, K), dtype=torch.bfloat16, device=cuda)
    out = torch.full((M, 8), 7.0, dtype=torch.float32, device=cuda)
    assert run_noalloc(a, b, out) == n5.ERR_ARG
    torch.cuda.synchronize()
    assert bool((out == 7.0).all())
