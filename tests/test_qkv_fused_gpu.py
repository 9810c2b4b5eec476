"""Tensor-level parity of the fused q/k/v step of a decoder layer
(n550_qkv_rope_kv): qkv = x . [Wq;Wk;Wv]^T, per-head QK-norm (qwen3.c:287-292),
RoPE at each row's position (ops_scalar.c:21-35) and the BF16 K/V cache write
(qwen3.c:498-511), on every route the runtime takes -- the GEMV (1-8 rows),
the weight-streaming GEMM (9-32 rows), split-K partials with the row kernel
(33-1023 rows) and the tcgen05 tile GEMM with the fused epilogue (1024 rows
on; single-CTA 128- and 256-wide tiles and 256 x 256 CTA-pair tiles) -- at
positions up to 2047.

The reference values are the oracle's: the projection in binary64 rounded to
FP32 (the reference's GEMM output), then the C restatements of qwen3_op_rmsnorm
and qwen3_op_rope (oracle/ops_oracle.c, bit-identical to ops_scalar.c), so the
RoPE factors the kernels take from rope_sincos are checked against the C
library's sinf/cosf of the same FP32 angle. Tolerances: FP32 queries within
1e-4 of the row's max |value|; BF16 outputs within 2^-8 of each value plus
1e-4 of the max (one BF16 rounding of nearby FP32 values).
"""
import numpy as np
import pytest

import oracle
import n550_qwen3_bringup_handover_b200 as n5
from tests.conftest import bf16_bits, to_dev_bf16

pytestmark = pytest.mark.gpu

H, QKVD, QD, HD = 1024, 4096, 2048, 128
F32_TOL = 1e-4
MAX_LEN = 2048
LAYER = 5
SENTINEL = 0x7FC1          # a NaN pattern no write produces


def rows_and_positions(M, rng):
    """(seq, pos) per row, distinct pairs, positions spread over [0, 2048)
    and always including 2047."""
    n_slots = -(-M // MAX_LEN)
    seq = np.arange(M, dtype=np.int32) % n_slots
    pos = np.empty(M, np.int32)
    for s in range(n_slots):
        idx = np.nonzero(seq == s)[0]
        p = rng.permutation(MAX_LEN)[:len(idx)]
        if MAX_LEN - 1 not in p:
            p[0] = MAX_LEN - 1
        pos[idx] = p
    return seq, pos, n_slots


def oracle_rows(x_bits, w_bits, qn, kn, pos):
    """FP32 q [R, 2048], k [R, 1024], v [R, 1024] for the given rows."""
    qkv = (oracle.bf16_to_f32(x_bits).astype(np.float64) @
           oracle.bf16_to_f32(w_bits).astype(np.float64).T).astype(np.float32)
    q = np.empty((len(pos), QD), np.float32)
    k = np.empty((len(pos), 1024), np.float32)
    for r, p in enumerate(pos):
        qh = oracle.rmsnorm(qkv[r, :QD].reshape(16, HD), qn)
        kh = oracle.rmsnorm(qkv[r, QD:QD + 1024].reshape(8, HD), kn)
        q[r] = oracle.rope(qh.reshape(-1), 16, int(p))
        k[r] = oracle.rope(kh.reshape(-1), 8, int(p))
    return q, k, qkv[:, QD + 1024:]


def bf16_close(got_bits, ref):
    got = oracle.bf16_to_f32(got_bits).astype(np.float64)
    ref = ref.astype(np.float64)
    bound = 2.0 ** -8 * np.abs(ref) + F32_TOL * np.abs(ref).max()
    return bool((np.abs(got - ref) <= bound).all()), float(np.abs(got - ref).max())


@pytest.mark.parametrize("M,q_type,tile", [
    (2, "f32", 0), (3, "bf16", 0), (7, "f32", 0),   # GEMV + row kernel
    (16, "f32", 0), (32, "bf16", 0),            # weight-streaming GEMM, fused epilogue
    (100, "bf16", 0), (256, "f32", 0),          # split-K partials + row kernel
    (2048, "bf16", 128),                        # tile GEMM, 128-wide single-CTA tiles
    (12288, "bf16", 256),                       # 128 x 256 single-CTA tiles
    (12288, "bf16", 0),                         # automatic: 256 x 256 CTA pairs
    (4096, "bf16", 512),                        # pairs forced below their automatic range
])
def test_qkv_rope_kv_vs_oracle(cuda, M, q_type, tile):
    import torch
    rng = np.random.default_rng(M * 7 + tile)
    x_bits = oracle.synth_normal_bf16((M, H), M, 0x58, 1.0)
    w_bits = oracle.synth_normal_bf16((QKVD, H), 3, 0x57, 0.02)
    qn = oracle.f32_to_bf16(1.0 + 0.1 * oracle.synth_normal_f32(HD, 3, 0x51, 1.0))
    kn = oracle.f32_to_bf16(1.0 + 0.1 * oracle.synth_normal_f32(HD, 3, 0x52, 1.0))
    seq, pos, n_slots = rows_and_positions(M, rng)

    dev = cuda
    x = to_dev_bf16(x_bits, dev)
    w = to_dev_bf16(w_bits, dev)
    dqn, dkn = to_dev_bf16(qn, dev), to_dev_bf16(kn, dev)
    rope = torch.empty((MAX_LEN, 64, 2), dtype=torch.float32, device=dev)
    tseq = torch.from_numpy(seq).to(dev)
    tpos = torch.from_numpy(pos).to(dev)
    qdt = torch.float32 if q_type == "f32" else torch.bfloat16
    q = torch.full((M, QD), float("nan"), dtype=qdt, device=dev)
    shape = (n_slots, 28, 8, MAX_LEN, HD)
    kc = torch.full(shape, SENTINEL, dtype=torch.int16, device=dev)
    vc = torch.full(shape, SENTINEL, dtype=torch.int16, device=dev)
    L = n5.lib()
    vp = n5.C.c_void_p
    try:
        n5.check(L.n550_gemm_tile_config(tile))
        n5.check(L.n550_rope_table(n5.stream_ptr(), vp(rope.data_ptr()), MAX_LEN))
        n5.check(L.n550_qkv_rope_kv(
            n5.stream_ptr(), vp(x.data_ptr()), H, vp(w.data_ptr()), vp(dqn.data_ptr()),
            vp(dkn.data_ptr()), vp(rope.data_ptr()), vp(tseq.data_ptr()), vp(tpos.data_ptr()), M,
            vp(q.data_ptr()), n5.F32 if q_type == "f32" else n5.BF16, QD, vp(kc.data_ptr()),
            vp(vc.data_ptr()), MAX_LEN, LAYER), "n550_qkv_rope_kv")
        torch.cuda.synchronize()
    finally:
        L.n550_gemm_tile_config(0)
    assert n5.device_status() == n5.OK

    # exactly the M x 8 x 128 addressed cache elements were written, in each cache
    for c in (kc, vc):
        assert int((c != SENTINEL).sum()) == M * 8 * HD

    # oracle on a sample of rows (all of them for small M), the highest positions included
    if M <= 256:
        rows = np.arange(M)
    else:
        rows = np.unique(np.concatenate([np.arange(64), np.arange(M - 64, M),
                                         rng.choice(M, 96, replace=False),
                                         np.argsort(pos)[-32:]]))
    q_ref, k_ref, v_ref = oracle_rows(x_bits[rows], w_bits, qn, kn, pos[rows])
    if q_type == "f32":
        got = q.cpu().numpy()[rows].astype(np.float64)
        for r in range(len(rows)):
            err = np.abs(got[r] - q_ref[r]).max() / np.abs(q_ref[r]).max()
            assert err <= F32_TOL, (rows[r], pos[rows[r]], err)
    else:
        ok, worst = bf16_close(bf16_bits(q)[rows], q_ref)
        assert ok, worst
    kc_h = kc.view(torch.int16)[tseq.long(), LAYER, :, tpos.long(), :]     # [M, 8, 128]
    vc_h = vc.view(torch.int16)[tseq.long(), LAYER, :, tpos.long(), :]
    kb = kc_h.cpu().numpy().view(np.uint16)[rows].reshape(len(rows), -1)
    vb = vc_h.cpu().numpy().view(np.uint16)[rows].reshape(len(rows), -1)
    ok, worst = bf16_close(kb, k_ref)
    assert ok, ("K", worst)
    ok, worst = bf16_close(vb, v_ref)
    assert ok, ("V", worst)


def test_rope_table_vs_libm(cuda):
    """n550_rope_table (rope_sincos: Cody-Waite reduction by pi/2 and the
    hardware sine/cosine) against binary64 sin/cos of the same FP32 angle
    pos * inv_freq[i], inv_freq from powf as ops_scalar.c:24, positions up to
    40959 (Qwen3's trained context): absolute error <= 1e-6."""
    import torch
    n = 40960
    t = torch.empty((n, 64, 2), dtype=torch.float32, device=cuda)
    n5.check(n5.lib().n550_rope_table(n5.stream_ptr(), n5.C.c_void_p(t.data_ptr()), n))
    torch.cuda.synchronize()
    got = t.cpu().numpy().astype(np.float64)
    import ctypes
    libm = ctypes.CDLL("libm.so.6")            # the powf the library's host code calls
    libm.powf.restype = ctypes.c_float
    libm.powf.argtypes = [ctypes.c_float, ctypes.c_float]
    inv = np.array([np.float32(1.0) / np.float32(libm.powf(1e6, 2 * i / 128)) for i in range(64)],
                   np.float32)
    ang = (np.arange(n, dtype=np.float32)[:, None] * inv[None, :]).astype(np.float64)
    assert np.abs(got[..., 0] - np.cos(ang)).max() <= 1e-6
    assert np.abs(got[..., 1] - np.sin(ang)).max() <= 1e-6
