"""Run the fast-mode GEMM on one shape a few times -- a bounded workload for
profilers (a few hundred MB on the device; operands larger than L2).

    python -m n550_qwen3_bringup_handover_b200.profile_gemm --M 16384 --N 4096 --K 1024
    python -m n550_qwen3_bringup_handover_b200.profile_gemm --M 16 --N 2048 --K 1024 --mode exact
"""
from __future__ import annotations

import argparse

import torch

import n550_qwen3_bringup_handover_b200 as n5


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--M", type=int, default=16384)
    ap.add_argument("--N", type=int, default=4096)
    ap.add_argument("--K", type=int, default=1024)
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--out", choices=["f32", "bf16", "resid", "swiglu"], default="f32")
    ap.add_argument("--bn", type=int, default=0, help="tile width 128/256 (0 = automatic)")
    ap.add_argument("--mode", choices=["fast", "exact"], default="fast")
    ap.add_argument("--kblock", type=int, default=16, help="exact mode: AME K-block")
    a = ap.parse_args()
    n5.check(n5.lib().n550_gemm_tile_config(a.bn), "n550_gemm_tile_config")
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev).manual_seed(0)
    A = torch.randn((a.M, a.K), device=dev, generator=g).to(torch.bfloat16)
    B = (torch.randn((a.N, a.K), device=dev, generator=g) * 0.02).to(torch.bfloat16)
    C = torch.zeros((a.M, a.N), device=dev,
                    dtype=torch.float32 if a.out in ("f32", "resid") else torch.bfloat16)
    if a.out == "swiglu":
        U = (torch.randn((a.N, a.K), device=dev, generator=g) * 0.02).to(torch.bfloat16)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    times = []
    for _ in range(a.iters):
        e0.record()
        if a.out == "resid":
            n5.gemm_residual(A, B, C)
        elif a.out == "swiglu":
            n5.gemm_swiglu(A, B, U, out=C)
        elif a.mode == "exact":
            n5.gemm(A, B, mode=n5.MODE_EXACT, kblock=a.kblock, out=C)
        else:
            n5.gemm(A, B, mode=n5.MODE_FAST, out=C)
        e1.record()
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1))
    n5.check(n5.device_status(), "device status")
    ms = min(times)
    flop = 2.0 * a.M * a.N * a.K * (2 if a.out == "swiglu" else 1)
    print(f"M={a.M} N={a.N} K={a.K} out={a.out} bn={a.bn} mode={a.mode}: {ms:.4f} ms, "
          f"{flop / ms / 1e9:.1f} TFLOP/s")


if __name__ == "__main__":
    main()
