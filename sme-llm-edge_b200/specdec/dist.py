"""Request sharding across ranks and the reductions of a timed multi-GPU run.

The speculative step shards by request: every rank (one process per GPU)
holds a full weight replica and a disjoint slice of the sequences, so the
data path needs no collective.  What crosses ranks is bookkeeping only: the
slice each rank owns, and after a timed run the slowest rank's device time
(max) and the tokens all ranks emitted (sum).

These helpers take a `torch.distributed`-style module or process group and a
device for the reduction tensors ("cuda:<local rank>" under NCCL, "cpu" under
gloo), so the same code runs in the benchmark and in CPU tests.
"""
from __future__ import annotations


def shard_range(n: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous slice [lo, hi) of n requests owned by `rank`; slices differ in
    size by at most one and cover 0..n-1 exactly once."""
    if world <= 0 or not 0 <= rank < world or n < 0:
        raise ValueError(f"bad shard: n={n} world={world} rank={rank}")
    base, extra = divmod(n, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def _reduce(dist, x: float, device: str, op) -> float:
    if dist is None:
        return float(x)
    import torch

    t = torch.tensor([float(x)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=op)
    return float(t.item())


def reduce_max(dist, x: float, device: str = "cpu") -> float:
    return _reduce(dist, x, device, None if dist is None else dist.ReduceOp.MAX)


def reduce_sum(dist, x: float, device: str = "cpu") -> float:
    return _reduce(dist, x, device, None if dist is None else dist.ReduceOp.SUM)


def step_throughput(dist, ms: float, tokens: float, device: str = "cpu") -> dict:
    """Whole-job throughput of a timed run: tokens of all ranks over the
    slowest rank's device time.  Every rank must call it (it is collective)."""
    ms_max = reduce_max(dist, ms, device)
    tok = reduce_sum(dist, tokens, device)
    return {"ms_max": ms_max, "tokens": tok, "value": tok / (ms_max / 1e3) if ms_max > 0 else 0.0}
