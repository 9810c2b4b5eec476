"""Run greedy decode steps of the random-init model on a bounded case (for
profilers): n_seqs sequences with a ctx-token prefilled context, then `steps`
eager decode steps (one kernel sequence per step, no CUDA graph).

    python -m n550_qwen3_bringup_handover_b200.profile_decode --seqs 64 --ctx 1024 --steps 2
"""
from __future__ import annotations

import argparse

import torch

import n550_qwen3_bringup_handover_b200 as n5


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--seqs", type=int, default=64)
    ap.add_argument("--ctx", type=int, default=1024)
    ap.add_argument("--steps", type=int, default=2)
    a = ap.parse_args()
    m = n5.Model(seed=0, max_seqs=a.seqs, max_len=a.ctx + a.steps + 1, max_tokens=a.seqs * a.ctx)
    tok = torch.from_numpy(n5.synth_tokens(a.seqs * a.ctx, 0, 0x544F4B).reshape(a.seqs, a.ctx)).cuda()
    seq = torch.arange(a.seqs, dtype=torch.int32, device="cuda")
    nxt = torch.empty(a.seqs, dtype=torch.int32, device="cuda")
    m.prefill(tok, seq, 0, None, nxt)
    pos = torch.full((a.seqs,), a.ctx, dtype=torch.int32, device="cuda")
    for _ in range(a.steps):
        cur = nxt.clone()
        m.decode(cur, seq, pos, None, nxt)
        pos += 1
    torch.cuda.synchronize()
    n5.check(n5.device_status(), "device status")
    print("ok", nxt[:4].tolist())
    m.close()


if __name__ == "__main__":
    main()
