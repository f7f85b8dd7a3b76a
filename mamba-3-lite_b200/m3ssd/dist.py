"""Multi-GPU host logic for the operator: it has no collective of its own.

Every (b, h) sequence of the chunkwise SSD is independent (A is per head and nothing couples
sequences, models/ssd_complex.py:58-119), so a job spreads sequences over ranks and each rank
runs the operator on its own slice. The only communication is host orchestration: agreeing on
timings (max over ranks) and noticing a rank that failed.
"""
from __future__ import annotations

from datetime import timedelta


def head_shard(nheads: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous head range [start, stop) of `rank` when heads are split over `world` ranks.

    Heads are the sharding unit because dA (H,) then stays local to one rank. Earlier ranks take
    the remainder, so shard sizes differ by at most one.
    """
    if world <= 0 or not (0 <= rank < world):
        raise ValueError(f"bad rank {rank} of {world}")
    base, extra = divmod(nheads, world)
    start = rank * base + min(rank, extra)
    stop = start + base + (1 if rank < extra else 0)
    return start, stop


def shard_inputs(x, A, B_t, C_t, dt, world: int, rank: int):
    """Views of the five operator inputs restricted to this rank's heads."""
    h0, h1 = head_shard(A.shape[0], world, rank)
    return (x[:, :, h0:h1], A[h0:h1], B_t[:, :, h0:h1], C_t[:, :, h0:h1], dt[:, :, h0:h1])


def max_over_ranks(values, device=None):
    """Element-wise max of a list of floats over all ranks (timings: the slowest rank counts)."""
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(v) for v in values], dtype=torch.float64, device=device)
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def init_process_group(backend: str, timeout_s: float = 120.0, device=None):
    """Process group with a short timeout so ranks waiting on a failed peer end with an error."""
    import torch.distributed as dist
    kw = {"timeout": timedelta(seconds=timeout_s)}
    if device is not None:
        kw["device_id"] = device
    dist.init_process_group(backend, **kw)
