"""Benchmark of the n550 Qwen3-0.6B hot path on B200 (driver contract).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl n550|reference]
    python -m torch.distributed.run --nproc-per-node N ... bench.py --gpus N

Headline ("batched prefill data-parallel"): 64 independent
sequences x 512 seeded random tokens through the random-init Qwen3-0.6B,
sequences sharded over the N ranks (strong scaling), BF16 weights replicated,
last-token logits and greedy next tokens gathered to rank 0 with NCCL. One
step = that whole job. metric = prefill+decode tok/s: `value` is the prefill
tokens per second of the job; the "decode" object reports BASELINE configs[4]
(256 sequences, 1024-token context in a BF16 KV cache, 128 greedy steps).

Inputs (weights 1.19 GB, activations, KV cache) are larger than the 126 MB L2,
so no flush between steps is needed (config.l2 says so).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

VOCAB = 151936
PREFILL_SEQS, PREFILL_LEN = 64, 512
DECODE_SEQS, DECODE_CTX, DECODE_STEPS = 256, 1024, 128
TOKEN_STREAM = 0x544F4B
# Qwen3-0.6B linear work per token: 28 x (q,k,v,o,gate,up,down) weights
LINEAR_PARAMS = 28 * (2048 * 1024 + 2 * 1024 * 1024 + 1024 * 2048 + 3 * 3072 * 1024)
WEIGHT_BYTES = 1_192_099_840
KV_BYTES_PER_POS = 28 * 8 * 128 * 2 * 2          # K and V, BF16, all layers


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "source": "fallback"}


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi sampling during the timed region (clocks and throttle reasons)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self):
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in getattr(self, "lines", []):
            f = [x.strip() for x in l.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ----------------------------------------------------------------------------- dist
def dist_setup(n_gpus):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n_gpus and world > 1:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}")
    return world, rank, local


def dist_init(world, local, backend):
    import datetime

    import torch
    import torch.distributed as dist
    if world > 1:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local) if backend == "nccl" else None)
    return dist


def max_over_ranks(x: float, world: int, device) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def shard(n_total: int, world: int, rank: int):
    """Rows [lo, hi) of n_total independent sequences that rank `rank` of
    `world` processes (equal contiguous shards, rank order)."""
    if n_total % world:
        raise SystemExit("sequence counts must divide by the number of GPUs")
    per = n_total // world
    return rank * per, (rank + 1) * per


def gather_rows(world: int, out, mine) -> None:
    """Rank-ordered gather of every rank's rows `mine` into `out` (all ranks);
    the only collective of the data-parallel path."""
    if world > 1:
        import torch.distributed as dist
        dist.all_gather_into_tensor(out, mine)


# ----------------------------------------------------------------------------- n550 arm
def run_n550(args, world, rank, local):
    import numpy as np
    import torch

    import n550_qwen3_bringup_handover_b200 as n5
    import ctypes as C

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = dist_init(world, local, "nccl")

    p_lo, p_hi = shard(PREFILL_SEQS, world, rank)
    d_lo, d_hi = shard(DECODE_SEQS, world, rank)
    ps, ds = p_hi - p_lo, d_hi - d_lo
    max_len = DECODE_CTX + DECODE_STEPS
    max_tokens = ps * PREFILL_LEN
    m = n5.Model(seed=0, max_seqs=max(ps, ds), max_len=max_len, max_tokens=max_tokens)

    # seeded synthetic tokens of the whole job; this rank's shard of sequences
    all_prompts = n5.synth_tokens(PREFILL_SEQS * PREFILL_LEN, 0, TOKEN_STREAM).reshape(PREFILL_SEQS, PREFILL_LEN)
    mine = np.ascontiguousarray(all_prompts[p_lo:p_hi])
    tok_host = torch.from_numpy(mine).pin_memory()
    tok_dev = tok_host.to(dev)
    seq_ids = torch.arange(ps, dtype=torch.int32, device=dev)
    logits = torch.empty((ps, VOCAB), dtype=torch.float32, device=dev)
    nxt = torch.empty(ps, dtype=torch.int32, device=dev)
    gathered_logits = torch.empty((PREFILL_SEQS, VOCAB), dtype=torch.float32, device=dev) if world > 1 else logits
    gathered_next = torch.empty(PREFILL_SEQS, dtype=torch.int32, device=dev) if world > 1 else nxt
    out_logits_host = torch.empty((PREFILL_SEQS, VOCAB), dtype=torch.float32).pin_memory()
    out_next_host = torch.empty(PREFILL_SEQS, dtype=torch.int32).pin_memory()
    stream = torch.cuda.current_stream(dev)

    def gather():
        gather_rows(world, gathered_logits, logits)
        gather_rows(world, gathered_next, nxt)

    def step_device():
        m.prefill(tok_dev, seq_ids, 0, logits, nxt)
        gather()

    # End to end: every step copies its tokens in from pinned host memory and
    # its gathered logits and next tokens out to pinned host memory (rank 0).
    # As in a serving loop the read-back of step i runs on a copy stream while
    # step i+1 computes, through two result buffers (device and host); the
    # timed region ends when the last read-back has landed.
    copy_stream = torch.cuda.Stream(dev)
    res_logits = [torch.empty((PREFILL_SEQS, VOCAB), dtype=torch.float32, device=dev) for _ in range(2)]
    res_next = [torch.empty(PREFILL_SEQS, dtype=torch.int32, device=dev) for _ in range(2)]
    host_logits = [out_logits_host, torch.empty_like(out_logits_host).pin_memory()]
    host_next = [out_next_host, torch.empty_like(out_next_host).pin_memory()]
    ev_ready = [torch.cuda.Event() for _ in range(2)]
    ev_copied = [torch.cuda.Event() for _ in range(2)]
    e2e_i = [0]

    def step_e2e():
        b = e2e_i[0] & 1
        e2e_i[0] += 1
        tok_dev.copy_(tok_host, non_blocking=True)
        m.prefill(tok_dev, seq_ids, 0, logits, nxt)
        stream.wait_event(ev_copied[b])              # buffer b's previous read-back is done
        if world > 1:
            gather_rows(world, res_logits[b], logits)
            gather_rows(world, res_next[b], nxt)
        else:
            res_logits[b].copy_(logits, non_blocking=True)
            res_next[b].copy_(nxt, non_blocking=True)
        if rank == 0:
            ev_ready[b].record(stream)
            copy_stream.wait_event(ev_ready[b])
            with torch.cuda.stream(copy_stream):
                host_logits[b].copy_(res_logits[b], non_blocking=True)
                host_next[b].copy_(res_next[b], non_blocking=True)
            ev_copied[b].record(copy_stream)

    def e2e_done():
        if rank == 0:
            for b in range(2):
                stream.wait_event(ev_copied[b])

    def timed(fn, steps, prof=False, finish=None):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize(dev)
        barrier(world)
        torch.cuda.synchronize(dev)
        if prof:
            n5.check(n5.lib().n550_qwen3_profile(m.handle, 1))
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            fn()
        if finish:
            finish()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        barrier(world)
        torch.cuda.synchronize(dev)
        ms = e0.elapsed_time(e1) / steps
        return max_over_ranks(ms, world, dev)

    K = args.steps
    # Headline: the prefill as a user repeats it (from the second identical
    # call the library replays a captured CUDA graph), no profiler attached.
    with ClockSampler(local) as clk:
        ms = timed(step_device, K)
    clocks = clk.summary()
    ms_e2e = timed(step_e2e, K, finish=e2e_done)
    # Per-kernel breakdown and the GEMM roofline: a separate eager pass with
    # CUDA events around every launch (not used for `value`).
    timed(step_device, K, prof=True)
    kind_ms = (C.c_double * 9)()
    kind_n = (C.c_int64 * 9)()
    n5.check(n5.lib().n550_qwen3_profile_read(m.handle, kind_ms, kind_n, 9))
    n5.check(n5.lib().n550_qwen3_profile(m.handle, 0))
    launches_per_step = sum(kind_n) / K

    total_tokens = PREFILL_SEQS * PREFILL_LEN
    value = total_tokens / (ms / 1000.0)
    e2e_value = total_tokens / (ms_e2e / 1000.0)

    # roofline of the dominant kernel: the tcgen05 projection GEMMs
    pk = peaks()
    tokens_rank = ps * PREFILL_LEN
    gemm_flops_step = 2.0 * LINEAR_PARAMS * tokens_rank
    gemm_ms = sum(kind_ms[k] for k in range(4)) / K
    gemm_launches = sum(kind_n[k] for k in range(4)) / K
    achieved_tflops = gemm_flops_step / (gemm_ms / 1000.0) / 1e12
    kinds = ["gemm_qkv", "gemm_o", "gemm_gateup", "gemm_down", "gemm_lmhead", "attention",
             "qknorm_rope_kv", "rmsnorm", "other"]
    breakdown = {k: round(kind_ms[i] / K, 4) for i, k in enumerate(kinds)}
    traffic = read_traffic_summary()

    decode = None
    if not args.no_decode:
        decode = run_decode(args, m, world, rank, dev, stream, ds, pk, timed)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(args.cpu_seconds)

    if rank == 0:
        line = {
            "metric": "Qwen3-0.6B tok/s prefill+decode @1/2/4/8 B200; GEMM % of BF16 TC peak",
            "value": round(value, 1), "unit": "tok/s", "n_gpus": world, "steps": K,
            "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: seeded random token ids, random-init weights ~N(0,0.02^2) (integer Irwin-Hall)",
            "config": {"workload": "configs[3] batched prefill DP: 64 seqs x 512 tokens, last-token logits gathered",
                       "model": "Qwen3-0.6B (random-init)", "global_batch": PREFILL_SEQS,
                       "seq_len": PREFILL_LEN, "parallelism": f"dp{world}",
                       "l2": "inputs larger than L2 (1.19 GB weights streamed per step); no flush"},
            "e2e": {"value": round(e2e_value, 1), "unit": "tok/s",
                    "h2d_bytes_per_step": int(tok_host.numel() * 4),
                    "d2h_bytes_per_step": int(PREFILL_SEQS * VOCAB * 4 + PREFILL_SEQS * 4)},
            "gpu_launches": int(round(launches_per_step * K)),
            "roofline": {"bound": "tensor", "kernel": "gemm_tc_kernel (q/k/v, o, gate-up, down)",
                         "achieved": round(achieved_tflops, 1),
                         "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                         "frac": round(achieved_tflops / pk["bf16_tflops"], 4),
                         "peak_source": pk["source"] + " (burst, MEASURED_PEAKS.json)",
                         # the GEMMs run back to back under the power cap inside the step:
                         # against the seconds-long cuBLAS loop as well
                         "frac_of_sustained": round(achieved_tflops / pk["bf16_tflops_sustained"], 4),
                         "launches_per_step": gemm_launches,
                         "traffic": traffic},
            "kernel_ms_per_step": breakdown,
            "clocks": clocks,
        }
        if decode:
            line["decode"] = decode
        if cpu:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    m.close()
    if world > 1:
        dist.destroy_process_group()


def run_decode(args, m, world, rank, dev, stream, ds, pk, timed):
    """256 sequences, 1024-token context, 128 greedy steps (sharded)."""
    import numpy as np
    import torch

    import n550_qwen3_bringup_handover_b200 as n5
    import ctypes as C

    ctx = n5.synth_tokens(DECODE_SEQS * DECODE_CTX, 1, TOKEN_STREAM).reshape(DECODE_SEQS, DECODE_CTX)
    d_lo, d_hi = shard(DECODE_SEQS, world, rank)
    mine = torch.from_numpy(np.ascontiguousarray(ctx[d_lo:d_hi])).to(dev)
    seq = torch.arange(ds, dtype=torch.int32, device=dev)
    nxt = torch.empty(ds, dtype=torch.int32, device=dev)
    m.prefill(mine, seq, 0, None, nxt)                 # untimed: fills the KV cache
    first = nxt.clone()
    pos = torch.full((ds,), DECODE_CTX, dtype=torch.int32, device=dev)
    ids = torch.empty((DECODE_STEPS, ds), dtype=torch.int32, device=dev)

    def job(use_graph=True):
        tok = first.clone()
        p = pos.clone()
        # each step is one replay of the captured decode step (all its kernels)
        m.decode_steps(tok, seq, p, DECODE_STEPS, ids, use_graph=use_graph)

    # one warm-up job (captures the graph), then time whole jobs (128 steps each)
    saved = args.warmup
    args.warmup = 1
    n_jobs = max(1, min(args.steps, 3))
    with ClockSampler(torch.cuda.current_device()) as clk:
        ms = timed(job, n_jobs)
    args.warmup = saved
    # per-kernel breakdown: one extra job launched eagerly with event timing
    torch.cuda.synchronize(dev)
    n5.check(n5.lib().n550_qwen3_profile(m.handle, 1))
    job(use_graph=False)
    kind_ms = (C.c_double * 9)()
    kind_n = (C.c_int64 * 9)()
    n5.check(n5.lib().n550_qwen3_profile_read(m.handle, kind_ms, kind_n, 9))
    n5.check(n5.lib().n550_qwen3_profile(m.handle, 0))
    launches_per_step = sum(kind_n) / DECODE_STEPS + 1          # + the advance kernel
    tokens = DECODE_SEQS * DECODE_STEPS
    # algorithmic HBM bytes per decode step on one rank: weights + KV read + KV write
    avg_ctx = DECODE_CTX + (DECODE_STEPS + 1) / 2.0
    bytes_step = WEIGHT_BYTES + ds * KV_BYTES_PER_POS * avg_ctx + ds * KV_BYTES_PER_POS
    step_ms = ms / DECODE_STEPS
    gbs = bytes_step / (step_ms / 1000.0) / 1e9
    attn_ms = kind_ms[5] / DECODE_STEPS
    kv_bytes = ds * KV_BYTES_PER_POS * avg_ctx
    return {"workload": "configs[4] batched decode DP: 256 seqs, 1024-token BF16 KV context, 128 greedy steps",
            "value": round(tokens / (ms / 1000.0), 1), "unit": "tok/s",
            "ms_per_job": round(ms, 3), "ms_per_step": round(step_ms, 4),
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": pk["hbm_gbs"],
                         "unit": "GB/s", "frac": round(gbs / pk["hbm_gbs"], 4),
                         "attention_kernel_gbs": round(kv_bytes / (attn_ms / 1000.0) / 1e9, 1)
                         if attn_ms > 0 else None},
            "launches_per_step": round(launches_per_step, 1), "cuda_graph": True,
            "kernel_ms_per_step_eager": {k: round(kind_ms[i] / DECODE_STEPS, 4) for i, k in enumerate(
                ["gemm_qkv", "gemm_o", "gemm_gateup", "gemm_down", "gemm_lmhead", "attention",
                 "qknorm_rope_kv", "rmsnorm", "other"])},
            "clocks": clk.summary()}


def read_traffic_summary():
    """DRAM bytes per GEMM launch from the committed ncu summary, if present."""
    p = ROOT / "profiles" / "gemm_tc_prefill_traffic.txt"
    if not p.exists():
        return None
    for l in p.read_text().splitlines():
        if l.startswith("traffic_bytes_per_launch="):
            try:
                return float(l.split("=", 1)[1])
            except ValueError:
                return None
    return None


# ----------------------------------------------------------------------------- CPU arms
def _cpu_worker(args):
    """One host core: the reference's own scalar forward (qwen3.c +
    kernels_scalar.c + ops_scalar.c in oracle/_ref, else the oracle's
    bit-identical restatement) prefilling `n_tok` tokens of sequence i."""
    i, n_tok, blob_path = args
    import numpy as np
    import oracle
    blob = np.memmap(blob_path, dtype=np.uint8, mode="r")
    blob = np.asarray(blob)
    toks = oracle.synth_tokens(PREFILL_SEQS * PREFILL_LEN, 0, TOKEN_STREAM)[i * PREFILL_LEN:i * PREFILL_LEN + n_tok]
    t0 = time.perf_counter()
    if oracle.ref_available("scalar"):
        m = oracle.RefModel(blob, "scalar")
        kind = "reference"
    else:
        m = oracle.OracleModel(blob, max_seq=PREFILL_LEN, gemm_kind=oracle.GEMM_SCALAR)
        kind = "port"
    m.forward_batch(toks, 0)
    return time.perf_counter() - t0, kind


def cpu_baseline(seconds_target=20.0, workers=None):
    """Timed sample of the reference CPU path on this host: every core prefills
    its own sequence (the reference runs one sequence per process)."""
    import multiprocessing as mp

    import numpy as np
    import oracle
    workers = workers or min(os.cpu_count() or 1, 16)
    n_tok = 32          # ~11 s of scalar work per core at ~2.6 GFLOP/s
    blob_path = Path("/dev/shm") / f"n550_qw3m_{os.getpid()}.bin"
    oracle.qw3m_blob(0, 0.02).tofile(blob_path)
    try:
        ctx = mp.get_context("spawn")
        t0 = time.perf_counter()
        with ctx.Pool(workers) as pool:
            res = pool.map(_cpu_worker, [(i % PREFILL_SEQS, n_tok, str(blob_path)) for i in range(workers)])
        wall = time.perf_counter() - t0
    finally:
        blob_path.unlink(missing_ok=True)
    compute = max(r[0] for r in res)
    kind = res[0][1]
    tok_s = workers * n_tok / compute
    return {"value": round(tok_s, 3), "unit": "tok/s", "cores": workers, "kind": kind,
            "sample": f"{workers} processes x {n_tok}-token prefill of one configs[3] sequence each "
                      f"(qwen3_forward_batch, scalar GEMM), {compute:.1f} s compute, {wall:.1f} s wall; "
                      f"per-token cost grows <2% from 32 to 512 tokens (attention), so this stands "
                      f"for the 512-token prefill"}


def run_reference(args, world, rank):
    """--impl reference: the reference's own CPU implementation of the path
    (qwen3.c + kernels_scalar.c + ops_scalar.c) on this host's cores, same
    metric/config; each step a bounded sample. Rank 0 only."""
    if rank != 0:
        return
    steps = []
    for _ in range(args.warmup):
        pass            # the CPU path has no warm-up state; keep the argument
    cpu = None
    for _ in range(max(1, min(args.steps, 2))):
        cpu = cpu_baseline(args.cpu_seconds)
        steps.append(cpu["value"])
    value = statistics.median(steps)
    cpu["value"] = round(value, 3)
    line = {
        "impl": "reference",
        "metric": "Qwen3-0.6B tok/s prefill+decode @1/2/4/8 B200; GEMM % of BF16 TC peak",
        "value": round(value, 3), "unit": "tok/s", "n_gpus": world, "steps": len(steps),
        "warmup": args.warmup, "ms_per_step": round(1000.0 * PREFILL_SEQS * PREFILL_LEN / value, 1),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: seeded random token ids, random-init weights",
        "config": {"workload": "configs[3] batched prefill DP: 64 seqs x 512 tokens (sampled)",
                   "model": "Qwen3-0.6B (random-init)", "global_batch": PREFILL_SEQS,
                   "seq_len": PREFILL_LEN, "parallelism": "host cores"},
        "cpu_baseline": cpu,
        "e2e": {"value": round(value, 3), "unit": "tok/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["n550", "reference"], default="n550")
    ap.add_argument("--no-decode", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=20.0)
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    world, rank, local = dist_setup(args.gpus)
    if args.impl == "reference":
        run_reference(args, world, rank)
        return
    run_n550(args, world, rank, local)


if __name__ == "__main__":
    main()
