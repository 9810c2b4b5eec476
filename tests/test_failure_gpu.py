"""Failure detection without a GPU fault: every spin-wait of the library is
bounded; one that nothing completes gives up after its limit, records
N550_ERR_TIMEOUT in the device status word and returns, so the host learns
of it from n550_device_status() and the context stays usable. The wait here
is an mbarrier no thread arrives on (n550_check_wait_expiry), limited to a
few milliseconds; no kernel traps, faults or hangs."""
import numpy as np
import pytest

import oracle
import n550_qwen3_bringup_handover_b200 as n5
from tests.conftest import to_dev_bf16

pytestmark = pytest.mark.gpu


def test_expired_wait_reports_timeout_and_context_survives(cuda):
    import time
    import torch
    L = n5.lib()
    assert n5.device_status() == n5.OK
    t0 = time.perf_counter()
    # a polling and a sleeping wait, 4M cycles (~2 ms) each
    n5.check(L.n550_check_wait_expiry(n5.stream_ptr(), 4_000_000), "n550_check_wait_expiry")
    assert n5.device_status() == n5.ERR_TIMEOUT
    assert time.perf_counter() - t0 < 0.5           # both waits gave up near their limit
    assert n5.device_status() == n5.OK              # read once, then cleared
    # the context still runs kernels correctly: a GEMM against binary64
    M, K, N = 64, 1024, 2048
    A = oracle.synth_normal_bf16((M, K), 31, 0x41, 1.0)
    B = oracle.synth_normal_bf16((N, K), 31, 0x42, 0.02)
    c = n5.gemm(to_dev_bf16(A, cuda), to_dev_bf16(B, cuda), mode=n5.MODE_FAST)
    torch.cuda.synchronize()
    ref = oracle.bf16_to_f32(A).astype(np.float64) @ oracle.bf16_to_f32(B).astype(np.float64).T
    assert np.abs(c.cpu().numpy() - ref).max() <= 1e-4 * np.abs(ref).max()
    assert n5.device_status() == n5.OK


def test_expired_waits_on_two_streams(cuda):
    """Expiries enqueued on two streams are both reported through the one
    status word, which a single read clears."""
    import torch
    L = n5.lib()
    s1, s2 = torch.cuda.Stream(), torch.cuda.Stream()
    n5.check(L.n550_check_wait_expiry(n5.stream_ptr(s1), 2_000_000))
    n5.check(L.n550_check_wait_expiry(n5.stream_ptr(s2), 2_000_000))
    assert n5.device_status() == n5.ERR_TIMEOUT
    assert n5.device_status() == n5.OK
