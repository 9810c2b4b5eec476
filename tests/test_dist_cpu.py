"""bench.py's multi-rank host logic on CPU: two processes over the gloo backend
(the GPU runs use NCCL with the same calls). Covers the data-parallel path's
sequence sharding, the rank-ordered gather of outputs (its only collective),
the max over ranks of the step time, the barrier, and the reference arm's
rule that rank 0 alone runs and prints.
"""
import json
import os
import socket
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parent.parent


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def rank_main(rank: int, world: int, port: int, q) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    sys.path.insert(0, str(ROOT))
    import bench
    w, r, _ = bench.dist_setup(world)
    dist = bench.dist_init(w, r, "gloo")
    try:
        total, width = 64, 7
        rows = np.arange(total * width, dtype=np.int32).reshape(total, width)
        lo, hi = bench.shard(total, w, r)
        # stand-ins for the per-rank next tokens and logits
        mine_i = torch.from_numpy(rows[lo:hi] * 3 + 1)
        mine_f = torch.from_numpy(rows[lo:hi].astype(np.float32) * 0.5)
        out_i = torch.empty((total, width), dtype=torch.int32)
        out_f = torch.empty((total, width), dtype=torch.float32)
        bench.gather_rows(w, out_i, mine_i)
        bench.gather_rows(w, out_f, mine_f)
        gathered = bool(torch.equal(out_i, torch.from_numpy(rows * 3 + 1)) and
                        torch.equal(out_f, torch.from_numpy(rows.astype(np.float32) * 0.5)))
        slowest = bench.max_over_ranks(10.0 + 2.5 * r, w, torch.device("cpu"))
        bench.barrier(w)
        q.put(json.dumps({"rank": r, "lo": lo, "hi": hi, "gathered": gathered, "max": slowest}))
    finally:
        dist.destroy_process_group()


def test_two_ranks_shard_gather_and_time():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        res = sorted((json.loads(q.get(timeout=180)) for _ in procs), key=lambda d: d["rank"])
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert [p.exitcode for p in procs] == [0, 0]
    assert [(d["lo"], d["hi"]) for d in res] == [(0, 32), (32, 64)]
    assert all(d["gathered"] for d in res)
    assert all(d["max"] == 12.5 for d in res)


def test_shard_rejects_uneven_split():
    sys.path.insert(0, str(ROOT))
    import bench
    assert bench.shard(256, 8, 7) == (224, 256)
    with pytest.raises(SystemExit):
        bench.shard(64, 3, 0)


def test_reference_arm_prints_on_rank_zero_only():
    """Under torchrun with two ranks the reference arm's rank 1 exits 0 at once
    without output (rank 0 alone times the CPU reference)."""
    env = dict(os.environ, RANK="1", WORLD_SIZE="2", LOCAL_RANK="1", MASTER_ADDR="127.0.0.1")
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--gpus", "2",
                        "--steps", "1"], cwd=ROOT, env=env, capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip() == ""
