"""The data-parallel layer's host logic (n550_qwen3_bringup_handover_b200/dp.py)
on CPU: two processes over the gloo backend (the GPU runs use NCCL with the
same calls). Covers the sequence sharding, the rank-ordered gathers of outputs
(the path's only collectives: last-token rows and per-step ids), the max over
ranks of the step time, the barrier, and bench.py's reference-arm rule that
rank 0 alone runs and prints.
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
    from n550_qwen3_bringup_handover_b200 import dp
    import torch.distributed as dist
    w, r, _ = dp.init_process_group("gloo")
    try:
        assert dp.world_and_rank() == (w, r)
        total, width = 64, 7
        rows = np.arange(total * width, dtype=np.int32).reshape(total, width)
        lo, hi = dp.shard(total, w, r)
        # stand-ins for the per-rank next tokens and logits
        mine_i = torch.from_numpy(rows[lo:hi] * 3 + 1)
        mine_f = torch.from_numpy(rows[lo:hi].astype(np.float32) * 0.5)
        out_i = torch.empty((total, width), dtype=torch.int32)
        out_f = torch.empty((total, width), dtype=torch.float32)
        dp.gather_rows(out_i, mine_i)
        dp.gather_rows(out_f, mine_f)
        gathered = bool(torch.equal(out_i, torch.from_numpy(rows * 3 + 1)) and
                        torch.equal(out_f, torch.from_numpy(rows.astype(np.float32) * 0.5)))
        # per-step ids of each rank's sequences: [steps, local] -> [steps, total]
        steps = 5
        ids = np.arange(steps * total, dtype=np.int32).reshape(steps, total) * 7
        out_ids = torch.empty((steps, total), dtype=torch.int32)
        dp.gather_columns(out_ids, torch.from_numpy(np.ascontiguousarray(ids[:, lo:hi])))
        gathered = gathered and bool(torch.equal(out_ids, torch.from_numpy(ids)))
        slowest = dp.max_over_ranks(10.0 + 2.5 * r, torch.device("cpu"))
        dp.barrier()
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
    from n550_qwen3_bringup_handover_b200 import dp
    assert dp.shard(256, 8, 7) == (224, 256)
    with pytest.raises(ValueError):
        dp.shard(64, 3, 0)
    with pytest.raises(ValueError):
        dp.shard(64, 2, 2)


def test_single_process_helpers_are_copies():
    """Without a process group the gathers are plain copies and the max is the value."""
    sys.path.insert(0, str(ROOT))
    from n550_qwen3_bringup_handover_b200 import dp
    assert dp.world_and_rank() == (1, 0)
    a = torch.arange(12, dtype=torch.int32).reshape(3, 4)
    out = torch.empty_like(a)
    dp.gather_rows(out, a)
    assert torch.equal(out, a)
    out2 = torch.empty_like(a)
    dp.gather_columns(out2, a)
    assert torch.equal(out2, a)
    assert dp.max_over_ranks(3.5, torch.device("cpu")) == 3.5
    dp.barrier()


def test_reference_arm_prints_on_rank_zero_only():
    """Under torchrun with two ranks the reference arm's rank 1 exits 0 at once
    without output (rank 0 alone times the CPU reference)."""
    env = dict(os.environ, RANK="1", WORLD_SIZE="2", LOCAL_RANK="1", MASTER_ADDR="127.0.0.1")
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--gpus", "2",
                        "--steps", "1"], cwd=ROOT, env=env, capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip() == ""


def lost_rank_main(rank: int, world: int, port: int, q) -> None:
    """Rank 1 leaves between steps (after joining, before the gather); rank 0's
    gather must end with an error inside the process group's timeout."""
    import time
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    sys.path.insert(0, str(ROOT))
    from n550_qwen3_bringup_handover_b200 import dp
    w, r, _ = dp.init_process_group("gloo", timeout_s=10.0)
    dp.barrier()
    if r == 1:
        os._exit(0)                        # the lost peer: no cleanup, no more collectives
    t0 = time.monotonic()
    try:
        out = torch.empty((4, 3), dtype=torch.float32)
        dp.gather_rows(out, torch.ones((2, 3), dtype=torch.float32))
        q.put(json.dumps({"raised": False, "s": time.monotonic() - t0}))
    except Exception as e:                 # gloo reports the closed peer or the timeout
        q.put(json.dumps({"raised": True, "s": time.monotonic() - t0, "what": type(e).__name__}))
    os._exit(0)


def test_lost_rank_ends_the_gather_with_an_error():
    """A rank that exits between steps is detected on the host: the surviving
    rank's next collective raises (peer closed, or the short process-group
    timeout) instead of waiting for good."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=lost_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        res = json.loads(q.get(timeout=120))
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert res["raised"], res
    assert res["s"] < 60.0, res
