"""Pins the oracle's C restatement against the reference's own C code built
in oracle/_ref (qwen3.c, kernels_scalar.c, kernels_hwsim.c, ops_scalar.c),
bit for bit. Skipped where oracle/_ref was not built (no reference checkout)."""
import numpy as np
import pytest

import oracle

needs_ref = pytest.mark.skipif(not (oracle.ref_available("scalar") and oracle.ref_available("hwsim")),
                               reason="oracle/_ref not built")

# test_kernels.c:74-90 plus odd shapes
SHAPES = [(1, 1024, 256), (4, 64, 128), (7, 33, 13), (3, 17, 5), (2, 3072, 64)]


@needs_ref
@pytest.mark.parametrize("M,K,N", SHAPES)
def test_gemm_restatements_bit_identical(M, K, N):
    rng = np.random.default_rng(M * 1000 + K + N)
    a = rng.uniform(-1, 1, (M, K)).astype(np.float32)
    b = oracle.f32_to_bf16(rng.uniform(-1, 1, (N, K)).astype(np.float32))
    assert np.array_equal(oracle.gemm_scalar(a, b).view(np.uint32),
                          oracle.ref_gemm("scalar", a, b).view(np.uint32))
    assert np.array_equal(oracle.gemm_hwsim(a, b).view(np.uint32),
                          oracle.ref_gemm("hwsim", a, b).view(np.uint32))


@needs_ref
def test_hwsim_equals_exact_kblock16_on_random_activations():
    """kernels_hwsim.c's double block sum is exact for these operands."""
    rng = np.random.default_rng(1)
    a = rng.standard_normal((8, 1024)).astype(np.float32)
    b = oracle.synth_normal_bf16((512, 1024), 1, 0x42, 0.02)
    assert np.array_equal(oracle.ref_gemm("hwsim", a, b).view(np.uint32),
                          oracle.gemm_ame_exact_f32a(a, b, 16).view(np.uint32))


@pytest.fixture(scope="module")
def blob():
    return oracle.qw3m_blob(seed=0, sigma=0.02)


@needs_ref
@pytest.mark.parametrize("kernel,kind", [("scalar", oracle.GEMM_SCALAR), ("hwsim", oracle.GEMM_HWSIM)])
def test_forward_restatement_bit_identical(blob, kernel, kind):
    toks = oracle.synth_tokens(4, 0, 0x544F4B)
    ref = oracle.RefModel(blob, kernel)
    om = oracle.OracleModel(blob, max_seq=64, gemm_kind=kind)
    r1, o1 = ref.forward_batch(toks, 0), om.forward_batch(toks, 0)
    assert np.array_equal(r1.view(np.uint32), o1.view(np.uint32))
    nxt = np.array([oracle.argmax(r1)], np.int32)
    r2, o2 = ref.forward_batch(nxt, 4), om.forward_batch(nxt, 4)
    assert np.array_equal(r2.view(np.uint32), o2.view(np.uint32))


def test_forward_restatement_rejects_bad_header():
    bad = np.zeros(300, np.uint8)
    with pytest.raises(RuntimeError):
        oracle.OracleModel(bad)
