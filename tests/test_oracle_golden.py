"""Pins the CPU oracle (test infrastructure) before it is trusted as the
checker: against the reference's shipped AME golden vectors, against the
reference generator's own output on BASELINE config 1, and against the
pure-Python Fraction restatement on adversarial small cases."""
import hashlib
import struct

import numpy as np
import pytest

import oracle
from oracle import ame_golden
from tests.conftest import case_operands

CASE_IDS = ["001", "002", "003", "004", "005", "006", "007", "008",
            "009a", "009b", "010", "011"]


@pytest.mark.parametrize("cid", CASE_IDS)
def test_oracle_matches_shipped_case_kblock16(golden_cases, cid):
    a, b, M, N, K, lda, ldb, _ = case_operands(golden_cases, cid)
    c, peak = oracle.gemm_ame_exact(a, b, 16, M=M, N=N, K=K, lda=lda, ldb=ldb)
    assert np.array_equal(c, golden_cases[f"{cid}/c_ref"])
    assert np.array_equal(peak, golden_cases[f"{cid}/c_peak"])
    if f"{cid}/xor_ref" in golden_cases:
        assert int(np.bitwise_xor.reduce(c.ravel())) == int(golden_cases[f"{cid}/xor_ref"][0])


def test_shipped_cases_pin_kblock16_not_32(golden_cases):
    """The generator as shipped says K_BLOCK=32; the shipped data disagrees."""
    mismatching = 0
    for cid in ("001", "004", "008"):
        a, b, M, N, K, lda, ldb, _ = case_operands(golden_cases, cid)
        c, _ = oracle.gemm_ame_exact(a, b, 32, M=M, N=N, K=K, lda=lda, ldb=ldb)
        mismatching += int((c != golden_cases[f"{cid}/c_ref"]).sum())
    assert mismatching > 0


@pytest.mark.parametrize("cid", ["001", "002", "003", "005", "006", "007", "008"])
def test_rng_restatement_rebuilds_case_inputs(golden_cases, cid):
    A, B = ame_golden.case_inputs(cid)
    M, N, K, lda, ldb, _ = (int(v) for v in golden_cases[f"{cid}/shape"])
    a = golden_cases[f"{cid}/a"][:, :K]
    b = golden_cases[f"{cid}/b"][:, :K]
    assert np.array_equal(np.array(A, np.uint16), a)
    assert np.array_equal(np.array(B, np.uint16), b)
    # row gaps are zero (40_gen_ame_vectors.py:197-209)
    assert not golden_cases[f"{cid}/a"][:, K:].any()


@pytest.mark.parametrize("kb", [16, 32])
def test_oracle_matches_reference_generator_config1(config1_golden, kb):
    M, K, N, seed = (int(v) for v in config1_golden["meta"])
    A = oracle.synth_normal_bf16((M, K), seed, 0x41, 1.0)
    B = oracle.synth_normal_bf16((N, K), seed, 0x42, 0.02)
    assert hashlib.sha256(A.tobytes()).digest() == config1_golden["a_sha256"].tobytes()
    assert hashlib.sha256(B.tobytes()).digest() == config1_golden["b_sha256"].tobytes()
    c, _ = oracle.gemm_ame_exact(A, B, kb)
    assert np.array_equal(c, config1_golden[f"c_kb{kb}"])


def test_hwsim_equals_generator_on_config1(config1_golden):
    M, K, N, seed = (int(v) for v in config1_golden["meta"])
    A = oracle.synth_normal_bf16((M, K), seed, 0x41, 1.0)
    B = oracle.synth_normal_bf16((N, K), seed, 0x42, 0.02)
    hw = oracle.gemm_hwsim(oracle.bf16_to_f32(A), B)
    assert np.array_equal(hw.view(np.uint32), config1_golden["c_kb16"])


def _bits(vals):
    return [ame_golden.f32_to_bf16_rne(v) for v in vals]


ADVERSARIAL = {
    # T1 of the generator docstring: 2^24 + 31 ones inside one block are exact
    "t1_wide_block": ([[2.0 ** 24] + [1.0] * 31], [[1.0] * 32]),
    # outliers and tiny values spanning > 53 bits inside one block
    "span": ([[6912.0, 1e-7, -6912.0, 3e-8] * 8], [[6912.0, 1e-6, 6912.0, 1.0] * 8]),
    # cancellation to exactly zero -> +0.0
    "cancel": ([[1.5, -1.5, 2.0 ** -100, -(2.0 ** -100)] * 8], [[1.0, 1.0, 1.0, 1.0] * 8]),
    # subnormal bf16 operands and products near the binary32 underflow
    "subnormal": ([[1e-39, -3e-39, 2.0 ** -126, 1e-20] * 8], [[1e-38, 2.0 ** -120, -1e-30, 1e-20] * 8]),
    # ties at the binary32 rounding point across blocks (T2/T3)
    "ties": ([[2.0 ** 24, 1.0, 1.0, 1.0] + [0.0] * 12 + [1.0] * 16], [[1.0] * 32]),
}


@pytest.mark.parametrize("name", sorted(ADVERSARIAL))
@pytest.mark.parametrize("kb", [16, 32])
def test_oracle_matches_fraction_restatement_adversarial(name, kb):
    a_rows, b_rows = ADVERSARIAL[name]
    A = [_bits(r) for r in a_rows]
    B = [_bits(r) for r in b_rows]
    K = len(A[0])
    C_ref, P_ref = ame_golden.ame_gemm_ref(A, B, len(A), len(B), K, kb)
    c, p = oracle.gemm_ame_exact(np.array(A, np.uint16), np.array(B, np.uint16), kb)
    assert np.array_equal(c, np.array(C_ref, np.uint32))
    assert np.allclose(p, np.array(P_ref, np.float32), rtol=0, atol=0)


def test_oracle_matches_fraction_restatement_random_wide_range():
    rng = np.random.default_rng(1234)
    M, N, K = 3, 5, 47
    mags = rng.uniform(-40, 40, size=(M + N, K))
    vals = np.sign(rng.standard_normal((M + N, K))) * np.exp2(mags)
    bits = oracle.f32_to_bf16(vals.astype(np.float32))
    A, B = bits[:M], bits[M:]
    for kb in (16, 32):
        C_ref, _ = ame_golden.ame_gemm_ref(A.tolist(), B.tolist(), M, N, K, kb)
        c, _ = oracle.gemm_ame_exact(A, B, kb)
        assert np.array_equal(c, np.array(C_ref, np.uint32))


def test_f32_to_bf16_matches_generator_rule():
    rng = np.random.default_rng(7)
    x = np.concatenate([rng.standard_normal(2000).astype(np.float32),
                        np.array([np.inf, -np.inf, 0.0, -0.0, 1e-40, 3.3895314e38], np.float32)])
    ours = oracle.f32_to_bf16(x)
    ref = np.array([ame_golden.f32_to_bf16_rne(float(v)) for v in x], np.uint16)
    assert np.array_equal(ours, ref)


def test_synthetic_generator_is_seeded_and_centred():
    a = oracle.synth_normal_f32(200000, 5, 9, 0.02)
    b = oracle.synth_normal_f32(200000, 5, 9, 0.02)
    assert np.array_equal(a, b)
    assert abs(a.mean()) < 2e-4 and abs(a.std() - 0.02) < 2e-4
    t = oracle.synth_tokens(10000, 0, 7)
    assert t.min() >= 0 and t.max() < 151936


def test_qw3m_blob_layout():
    size = oracle.lib().oracle_qw3m_size()
    assert size == 1_192_100_096
