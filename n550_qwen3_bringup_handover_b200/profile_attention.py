"""Run one prefill forward of the random-init model on a bounded case (for
profilers): n_seqs sequences x seq_len tokens, weights + a small KV cache.

    python -m n550_qwen3_bringup_handover_b200.profile_attention --seqs 8 --len 512
"""
from __future__ import annotations

import argparse

import torch

import n550_qwen3_bringup_handover_b200 as n5


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--seqs", type=int, default=8)
    ap.add_argument("--len", type=int, default=512)
    ap.add_argument("--iters", type=int, default=2)
    a = ap.parse_args()
    m = n5.Model(seed=0, max_seqs=a.seqs, max_len=a.len, max_tokens=a.seqs * a.len)
    tok = torch.from_numpy(n5.synth_tokens(a.seqs * a.len, 0, 0x544F4B).reshape(a.seqs, a.len)).cuda()
    seq = torch.arange(a.seqs, dtype=torch.int32, device="cuda")
    nxt = torch.empty(a.seqs, dtype=torch.int32, device="cuda")
    for _ in range(a.iters):
        m.prefill(tok, seq, 0, None, nxt)
    torch.cuda.synchronize()
    n5.check(n5.device_status(), "device status")
    print("ok", nxt[:4].tolist())
    m.close()


if __name__ == "__main__":
    main()
