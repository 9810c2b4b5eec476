"""Data-parallel serving of independent sequences over the GPUs of one node.

The reference runs one sequence per process on one core (qwen3_forward_batch,
qwen3.c:455; qwen3_forward, qwen3.c:578). Here a job of many independent
sequences is split into equal contiguous shards, one per rank (one process
per GPU, torch.distributed over NCCL); every rank holds a full replica of the
BF16 weights and the KV cache of its own sequences, so the data path has no
collective at all. The one exchange is at the end of a call: the per-sequence
outputs (last-token logits, greedy ids) are gathered in rank order with one
all_gather_into_tensor per output, so every rank ends with the whole job's
rows.

    dp = DataParallel(n_seqs=64, max_len=512)          # after init_process_group()
    dp.prefill(my_tokens, logits_all, next_all)         # my_tokens: rows dp.lo:dp.hi

The helpers (shard, gather_rows, max_over_ranks, barrier) work with one
process too, where they reduce to a copy or nothing.
"""
from __future__ import annotations

import datetime
import os

from .model import Model


def world_and_rank(group=None):
    """(world size, rank) of the default process group, or (1, 0) without one."""
    import torch.distributed as dist
    if dist.is_available() and dist.is_initialized():
        return dist.get_world_size(group), dist.get_rank(group)
    return 1, 0


def init_process_group(backend: str = "nccl", timeout_s: float = 120.0):
    """One process per GPU from torchrun's environment (RANK, WORLD_SIZE,
    LOCAL_RANK, MASTER_ADDR/PORT): selects the local GPU and, for more than one
    rank, joins the process group with a short timeout so that ranks waiting
    for a lost peer end with an error. Returns (world, rank, local_rank)."""
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if backend == "nccl":
        torch.cuda.set_device(local)
    if world > 1 and not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group(
            backend, timeout=datetime.timedelta(seconds=timeout_s),
            device_id=torch.device("cuda", local) if backend == "nccl" else None)
    return world, rank, local


def shard(n_total: int, world: int, rank: int):
    """Rows [lo, hi) of n_total independent sequences that rank `rank` of
    `world` processes serves: equal contiguous shards in rank order."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of {world}")
    if n_total % world:
        raise ValueError(f"{n_total} sequences do not divide over {world} ranks")
    per = n_total // world
    return rank * per, (rank + 1) * per


def gather_rows(out, mine, group=None) -> None:
    """Rank-ordered gather of every rank's rows `mine` (same shape on every
    rank) into `out` (world x that many rows), on every rank."""
    world, _ = world_and_rank(group)
    if world > 1:
        import torch.distributed as dist
        dist.all_gather_into_tensor(out, mine, group=group)
    elif out.data_ptr() != mine.data_ptr():
        out.copy_(mine)


def gather_columns(out, mine, group=None) -> None:
    """Rank-ordered gather along the second axis: every rank's `mine`
    [steps, n] into out [steps, world * n] (per-step ids of each rank's
    sequences side by side), on every rank."""
    import torch
    world, _ = world_and_rank(group)
    if world == 1:
        if out.data_ptr() != mine.data_ptr():
            out.copy_(mine)
        return
    buf = torch.empty((world,) + tuple(mine.shape), dtype=mine.dtype, device=mine.device)
    gather_rows(buf, mine.unsqueeze(0).contiguous(), group)
    out.copy_(buf.permute(1, 0, 2).reshape(out.shape))


def max_over_ranks(x: float, device, group=None) -> float:
    """The largest x over the ranks (the job's time is its slowest rank's)."""
    world, _ = world_and_rank(group)
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())


def barrier(group=None) -> None:
    world, _ = world_and_rank(group)
    if world > 1:
        import torch.distributed as dist
        dist.barrier(group=group)


class DataParallel:
    """A job of n_seqs independent sequences over the process group's ranks.

    This rank serves rows [lo, hi) with its own Model replica (sequence slots
    0 .. hi - lo - 1; max_seqs reserves more slots for other work on the same
    replica); outputs are gathered to full-job tensors on every rank.
    """

    def __init__(self, n_seqs: int, max_len: int, max_tokens: int | None = None, *,
                 max_seqs: int | None = None, seed: int = 0, sigma: float = 0.02, blob=None,
                 group=None, **model_kw):
        import torch
        self.world, self.rank = world_and_rank(group)
        self.group = group
        self.n_seqs = n_seqs
        self.lo, self.hi = shard(n_seqs, self.world, self.rank)
        self.local = self.hi - self.lo
        self.device = torch.device("cuda", torch.cuda.current_device())
        self.model = Model(blob=blob, seed=seed, sigma=sigma,
                           max_seqs=max(max_seqs or self.local, self.local, 1), max_len=max_len,
                           max_tokens=max_tokens or self.local * max_len, **model_kw)
        self.seq_ids = torch.arange(self.local, dtype=torch.int32, device=self.device)
        self._lg = None
        self._nx = None

    def close(self):
        self.model.close()

    def _local_out(self, with_logits: bool):
        import torch
        if self._nx is None:
            self._nx = torch.empty(self.local, dtype=torch.int32, device=self.device)
        if with_logits and self._lg is None:
            self._lg = torch.empty((self.local, 151936), dtype=torch.float32, device=self.device)
        return (self._lg if with_logits else None), self._nx

    def prefill(self, tokens, logits_all=None, next_all=None, pos0: int = 0, stream=None):
        """Prefill this rank's rows `tokens` [hi - lo, L] (device int32) from
        position pos0; gather the last-token logits [n_seqs, 151936] (if
        given) and greedy next ids [n_seqs] of the whole job."""
        if self.world == 1:            # the job is this rank's rows: write in place
            nx = next_all if next_all is not None else self._local_out(False)[1]
            self.model.prefill(tokens, self.seq_ids, pos0, logits_all, nx, stream=stream)
            return logits_all, nx
        lg, nx = self._local_out(logits_all is not None)
        self.model.prefill(tokens, self.seq_ids, pos0, lg, nx, stream=stream)
        if logits_all is not None:
            gather_rows(logits_all, lg, self.group)
        if next_all is not None:
            gather_rows(next_all, nx, self.group)
        return lg, nx

    def decode_steps(self, tokens, pos, steps: int, ids_all=None, use_graph: bool = True,
                     stream=None):
        """`steps` greedy decode steps of this rank's rows (tokens, pos: device
        int32 [hi - lo], advanced in place); the chosen ids of the whole job
        are gathered into ids_all [steps, n_seqs] (if given)."""
        import torch
        ids = torch.empty((steps, self.local), dtype=torch.int32, device=self.device)
        self.model.decode_steps(tokens, self.seq_ids, pos, steps, ids, use_graph=use_graph,
                                stream=stream)
        if ids_all is not None:
            gather_columns(ids_all, ids, self.group)
        return ids
