"""Run prefill forwards of the random-init model on a bounded case (for
profilers): n_seqs sequences x seq_len tokens, weights + a small KV cache.
With --time, report the device time per prefill (CUDA events over --iters
repeated calls after two warm-up calls; repeated calls replay a CUDA graph).

    python -m n550_qwen3_bringup_handover_b200.profile_attention --seqs 8 --len 512
    python -m n550_qwen3_bringup_handover_b200.profile_attention --seqs 8 --len 512 --iters 10 --time
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
    ap.add_argument("--time", action="store_true")
    a = ap.parse_args()
    m = n5.Model(seed=0, max_seqs=a.seqs, max_len=a.len, max_tokens=a.seqs * a.len)
    tok = torch.from_numpy(n5.synth_tokens(a.seqs * a.len, 0, 0x544F4B).reshape(a.seqs, a.len)).cuda()
    seq = torch.arange(a.seqs, dtype=torch.int32, device="cuda")
    nxt = torch.empty(a.seqs, dtype=torch.int32, device="cuda")
    if a.time:
        for _ in range(2):
            m.prefill(tok, seq, 0, None, nxt)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
    for _ in range(a.iters):
        m.prefill(tok, seq, 0, None, nxt)
    if a.time:
        e1.record()
    torch.cuda.synchronize()
    if a.time:
        ms = e0.elapsed_time(e1) / a.iters
        print(f"seqs={a.seqs} len={a.len}: {ms:.3f} ms per prefill, {a.seqs * a.len / ms * 1e3:.0f} tok/s")
    n5.check(n5.device_status(), "device status")
    print("ok", nxt[:4].tolist())
    m.close()


if __name__ == "__main__":
    main()
