"""Decode attention that finishes the raw q/k/v rows itself (QK-norm, RoPE and
the K/V write, qwen3.c:287-292 and 498-511, inside the attention kernel;
n550_qwen3_fused_attention_prep, default on) against the separate row kernel it
replaces: bit-identical logits, ids and KV-cache effects (a second decode step
reads the K/V the first one wrote) on the GEMV route (1-8 sequences, with
split-KV at long contexts), the split-K route (33-1023 sequences), in eager
steps and in the CUDA-graph loop."""
import numpy as np
import pytest

import oracle
import n550_qwen3_bringup_handover_b200 as n5

pytestmark = pytest.mark.gpu


def run(S, lens, fused, steps=3):
    import torch
    n5.check(n5.lib().n550_qwen3_fused_attention_prep(1 if fused else 0))
    L = max(lens)
    m = n5.Model(seed=0, max_seqs=S, max_len=L + steps + 8, max_tokens=max(S * L, 64))
    try:
        toks = oracle.synth_tokens(S * L, 5 + S, 0x544F4B).reshape(S, L)
        seq = torch.arange(S, dtype=torch.int32, device="cuda")
        nx = torch.empty(S, dtype=torch.int32, device="cuda")
        for s in range(S):                  # ragged contexts: one prefill per sequence
            t = torch.from_numpy(np.ascontiguousarray(toks[s, :lens[s]]).reshape(1, -1)).cuda()
            m.prefill(t, seq[s:s + 1], 0, None, nx[s:s + 1])
        tok = nx.clone()
        pos = torch.tensor(lens, dtype=torch.int32, device="cuda")
        out = []
        for _ in range(2):
            lg = torch.empty((S, 151936), dtype=torch.float32, device="cuda")
            m.decode(tok, seq, pos, lg, nx)
            torch.cuda.synchronize()
            out.append(lg.cpu().numpy())
            tok = nx.clone()
            pos = pos + 1
        ids = torch.zeros((steps, S), dtype=torch.int32, device="cuda")
        m.decode_steps(tok, seq, pos, steps, ids, use_graph=True)
        torch.cuda.synchronize()
        out.append(ids.cpu().numpy())
        return out
    finally:
        m.close()


@pytest.mark.parametrize("S,lens", [(1, [40]), (3, [1500, 70, 900]), (48, [24] * 48)])
def test_fused_prep_bit_identical(cuda, S, lens):
    try:
        a = run(S, lens, True)
        b = run(S, lens, False)
    finally:
        n5.lib().n550_qwen3_fused_attention_prep(1)
    assert n5.device_status() == n5.OK
    for x, y in zip(a, b):
        assert np.array_equal(x, y)
