"""GQA causal attention through the C ABI (n550_attention_prefill / _decode)
against a plain PyTorch FP32 restatement of qwen3.c:374-436.

Tolerance: outputs are BF16 and the prefill kernel rounds the softmax
probabilities P to BF16 before the P.V product, so every element must satisfy
|out - ref| <= 2e-2 + 2e-2 |ref| and the mean absolute error must stay below
2e-3 (values ~N(0,1))."""
import pytest
import torch

import n550_qwen3_bringup_handover_b200 as n5

pytestmark = pytest.mark.gpu

SCALE = 0.08838834764831845          # qwen3.c:296
ATOL, RTOL, MEAN_TOL = 2e-2, 2e-2, 2e-3


def ref_attention(q, kc, vc, seq_ids, L, pos0s, layer):
    """q [n*L, >=2048]; pos0s: first query position per sequence."""
    n = len(seq_ids)
    out = torch.empty((n * L, 2048), dtype=torch.float32, device=q.device)
    qf = q[:, :2048].float().view(n, L, 16, 128)
    for i, sid in enumerate(seq_ids):
        p0 = pos0s[i]
        kv_len = p0 + L
        k = kc[sid, layer, :, :kv_len].float().repeat_interleave(2, dim=0)   # head h -> kv h//2
        v = vc[sid, layer, :, :kv_len].float().repeat_interleave(2, dim=0)
        s = torch.einsum("lhd,htd->hlt", qf[i], k) * SCALE
        qpos = p0 + torch.arange(L, device=q.device)
        mask = torch.arange(kv_len, device=q.device)[None, :] > qpos[:, None]
        s = s.masked_fill(mask[None], float("-inf"))
        o = torch.einsum("hlt,htd->lhd", torch.softmax(s, dim=-1), v)
        out[i * L:(i + 1) * L] = o.reshape(L, 2048)
    return out


def make_cache(n_slots, max_len, gen, poison_from=None):
    shape = (n_slots, 28, 8, max_len, 128)
    kc = torch.randn(shape, device="cuda", generator=gen).to(torch.bfloat16)
    vc = torch.randn(shape, device="cuda", generator=gen).to(torch.bfloat16)
    if poison_from is not None:
        # positions the kernel must not read (or must not let through)
        kc[:, :, :, poison_from:] = float("nan")
        vc[:, :, :, poison_from:] = float("nan")
    return kc, vc


def check_close(out, ref):
    o = out.float()
    err = (o - ref).abs()
    assert torch.isfinite(o).all()
    bad = err > ATOL + RTOL * ref.abs()
    assert not bad.any(), f"{int(bad.sum())} elements off, max err {err.max().item():.4g}"
    assert err.mean().item() < MEAN_TOL, err.mean().item()


@pytest.mark.parametrize("n_seqs,L,pos0,max_len,n_slots,qscale", [
    (2, 512, 0, 640, 3, 1.0),      # the prefill shape of the batched benchmark
    (3, 200, 0, 256, 4, 1.0),      # ragged last query block
    (2, 130, 64, 256, 3, 1.0),     # pos0 off the 128-key grid
    (1, 1, 37, 64, 1, 1.0),        # a single query
    (4, 128, 300, 512, 5, 1.0),    # chunked prefill: cached context longer than L
    (2, 384, 0, 384, 2, 8.0),      # peaked scores: exercises the running-max rescale
])
def test_prefill_matches_fp32_reference(n_seqs, L, pos0, max_len, n_slots, qscale):
    gen = torch.Generator(device="cuda").manual_seed(1000 + L + pos0)
    kc, vc = make_cache(n_slots, max_len, gen, poison_from=pos0 + L if pos0 + L < max_len else None)
    seq_ids = torch.randperm(n_slots, generator=torch.Generator().manual_seed(L))[:n_seqs]
    sid = seq_ids.to(torch.int32).cuda()
    # q rows live in a larger buffer whose extra rows are NaN: the kernel must
    # not read past row n_seqs * L
    qbuf = torch.full((n_seqs * L + 256, 2048), float("nan"), device="cuda", dtype=torch.bfloat16)
    qbuf[:n_seqs * L] = (torch.randn((n_seqs * L, 2048), device="cuda", generator=gen) * qscale).to(torch.bfloat16)
    q = qbuf[:n_seqs * L]
    layer = 11
    out = n5.attention_prefill(q, kc, vc, sid, L, pos0, layer)
    torch.cuda.synchronize()
    assert n5.device_status() == n5.OK
    ref = ref_attention(q, kc, vc, seq_ids.tolist(), L, [pos0] * n_seqs, layer)
    check_close(out, ref)


def test_prefill_strided_q_and_out():
    """q and out as column slices of wider rows (ldq, ldo > 2048)."""
    gen = torch.Generator(device="cuda").manual_seed(7)
    kc, vc = make_cache(2, 256, gen)
    L = 160
    wide_q = torch.randn((2 * L, 4096), device="cuda", generator=gen).to(torch.bfloat16)
    wide_o = torch.zeros((2 * L, 2048 + 512), device="cuda", dtype=torch.bfloat16)
    sid = torch.tensor([1, 0], dtype=torch.int32, device="cuda")
    n5.attention_prefill(wide_q, kc, vc, sid, L, 0, 3, out=wide_o)
    torch.cuda.synchronize()
    ref = ref_attention(wide_q, kc, vc, [1, 0], L, [0, 0], 3)
    check_close(wide_o[:, :2048], ref)
    assert (wide_o[:, 2048:] == 0).all()


def test_prefill_rejects_bad_arguments():
    kc = torch.zeros((1, 28, 8, 64, 128), device="cuda", dtype=torch.bfloat16)
    q = torch.zeros((64, 2048), device="cuda", dtype=torch.bfloat16)
    sid = torch.zeros(1, dtype=torch.int32, device="cuda")
    with pytest.raises(n5.N550Error):          # pos0 + L beyond max_len
        n5.attention_prefill(q, kc, kc, sid, 64, 1, 0)
    with pytest.raises(n5.N550Error):          # layer out of range
        n5.attention_prefill(q, kc, kc, sid, 64, 0, 28)


@pytest.mark.parametrize("split", [True, False])
def test_decode_matches_fp32_reference(split):
    gen = torch.Generator(device="cuda").manual_seed(99)
    n_slots, max_len = 6, 1100
    kc, vc = make_cache(n_slots, max_len, gen)
    seq_ids = [4, 0, 5, 2, 1]
    pos = [1099, 0, 63, 64, 517]
    q = torch.randn((len(seq_ids), 2048), device="cuda", generator=gen).to(torch.bfloat16)
    sid = torch.tensor(seq_ids, dtype=torch.int32, device="cuda")
    pt = torch.tensor(pos, dtype=torch.int32, device="cuda")
    out = n5.attention_decode(q, kc, vc, sid, pt, 20, split=split)
    torch.cuda.synchronize()
    assert n5.device_status() == n5.OK
    ref = ref_attention(q, kc, vc, seq_ids, 1, pos, 20)
    check_close(out, ref)


def test_prefill_agrees_with_decode_rows():
    """Query i of a prefill equals a decode at position pos0 + i."""
    gen = torch.Generator(device="cuda").manual_seed(5)
    kc, vc = make_cache(2, 384, gen)
    L = 300
    q = torch.randn((L, 2048), device="cuda", generator=gen).to(torch.bfloat16)
    sid = torch.tensor([1], dtype=torch.int32, device="cuda")
    pre = n5.attention_prefill(q, kc, vc, sid, L, 0, 0).float()
    rows = [0, 1, 127, 128, 255, 299]
    dq = q[rows].contiguous()
    dec = n5.attention_decode(dq, kc, vc, torch.tensor([1] * len(rows), dtype=torch.int32, device="cuda"),
                              torch.tensor(rows, dtype=torch.int32, device="cuda"), 0).float()
    torch.cuda.synchronize()
    err = (pre[rows] - dec).abs()
    assert (err <= ATOL + RTOL * dec.abs()).all(), err.max().item()
