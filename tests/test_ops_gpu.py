"""GPU parity of the non-GEMM ops against the oracle's restatement of
ops_scalar.c. FP32 ops: |got - ref| <= 1e-5 * max(1, |ref|) elementwise
(parallel reductions and CUDA libm differ from the sequential glibc ones in
the last bits); argmax and bf16 -> f32 are exact."""
import numpy as np
import pytest

import oracle
import n550_qwen3_bringup_handover_b200 as n5
from tests.conftest import to_dev_bf16

pytestmark = pytest.mark.gpu

TOL = 1e-5


def close(got, ref, tol=TOL):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return bool(np.all(np.abs(got - ref) <= tol * np.maximum(1.0, np.abs(ref))))


def test_rmsnorm_device_and_host(cuda):
    import torch
    x = oracle.synth_normal_f32((64, 1024), 1, 1, 1.0) * 3
    w = oracle.synth_normal_bf16(1024, 1, 2, 1.0)
    ref = oracle.rmsnorm(x, w)
    got = n5.rmsnorm(torch.from_numpy(x).to(cuda), to_dev_bf16(w, cuda)).cpu().numpy()
    assert close(got, ref)
    assert close(n5.qwen3_op_rmsnorm(x[3], w), ref[3])
    # BF16 output: RNE of the FP32 result, within one BF16 ulp at rounding ties
    gb = n5.rmsnorm(torch.from_numpy(x).to(cuda), to_dev_bf16(w, cuda), out_dtype=torch.bfloat16)
    gbf = gb.float().cpu().numpy()
    assert close(gbf, oracle.bf16_to_f32(oracle.f32_to_bf16(ref)), 2 ** -7)


@pytest.mark.parametrize("pos", [0, 1, 31, 511, 1151, 2047])
def test_rope_vs_reference(cuda, pos):
    import torch
    v = oracle.synth_normal_f32(16 * 128, pos, 3, 1.0)
    ref = oracle.rope(v, 16, pos)
    got = n5.rope(torch.from_numpy(v.copy()).to(cuda), 16, pos).cpu().numpy()
    assert close(got, ref, 2e-5)
    assert close(n5.qwen3_op_rope(v, 16, pos), ref, 2e-5)


def test_rope_rows_positions(cuda):
    import torch
    rows = 5
    v = oracle.synth_normal_f32((rows, 8 * 128), 4, 4, 1.0)
    got = n5.rope(torch.from_numpy(v.copy()).to(cuda), 8, 100).cpu().numpy()
    for r in range(rows):
        assert close(got[r], oracle.rope(v[r], 8, 100 + r), 2e-5)


def test_softmax_silu_residual_dot_axpy(cuda):
    import torch
    x = oracle.synth_normal_f32(3000, 5, 5, 4.0)
    y = oracle.synth_normal_f32(3000, 5, 6, 1.0)
    assert close(n5.qwen3_op_softmax(x), oracle.softmax(x))
    assert close(n5.softmax(torch.from_numpy(x.copy()).to(cuda)).cpu().numpy(), oracle.softmax(x))
    assert close(n5.qwen3_op_silu_mul(x, y), oracle.silu_mul(x, y))
    assert close(n5.silu_mul(torch.from_numpy(x.copy()).to(cuda), torch.from_numpy(y).to(cuda)).cpu().numpy(),
                 oracle.silu_mul(x, y))
    assert close(n5.qwen3_op_residual_add(x, y), x + y, 0)
    d = n5.qwen3_op_dot(x[:128], y[:128])
    assert abs(d - oracle.dot(x[:128], y[:128])) <= 1e-5 * max(1, abs(d))
    assert close(n5.qwen3_op_axpy(y, 0.375, x), oracle.axpy(y, 0.375, x), 0)


def test_bf16_to_f32_exact(cuda):
    import torch
    b = np.arange(0, 65536, 7, dtype=np.uint16)
    got = n5.qwen3_op_bf16_to_f32(b)
    ref = oracle.bf16_to_f32(b)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
    dev = n5.bf16_to_f32(to_dev_bf16(b, cuda)).cpu().numpy()
    assert np.array_equal(dev.view(np.uint32), ref.view(np.uint32))


def test_argmax_ties_take_lowest_index(cuda):
    import torch
    v = oracle.synth_normal_f32((4, 151936), 7, 7, 1.0)
    v[1, 5] = v[1, 150000] = v[1, 77777] = 99.0        # three-way tie
    v[2, :] = -3.0                                      # all equal -> 0
    v[3, 151935] = 50.0                                 # last element
    got = n5.argmax(torch.from_numpy(v).to(cuda)).cpu().numpy()
    ref = [oracle.argmax(r) for r in v]
    assert list(got) == ref == [ref[0], 5, 0, 151935]
    assert n5.qwen3_op_argmax(v[1]) == 5
