"""Row sharding across GPUs, one process per GPU.

Every row is an independent sampler (the reference keeps one ``Sampler`` per
sequence, sampler.h:165, and ``sample()`` touches nothing else), so a batch
splits into contiguous row blocks with no exchange while sampling.  Row r
keeps the RNG stream it has on one GPU (seed + r, counted over the whole
batch), so the sharded job draws exactly what the single-GPU job draws.  The
only collective is the gather of the int32 tokens (and, when asked, the RNG
states) to one rank, plus the max-over-ranks of the timed region.

The functions take a torch.distributed process group (NCCL on GPUs, gloo in
the CPU tests) and plain tensors; nothing here depends on the sampler
library.
"""
from typing import List, Optional, Tuple

import numpy as np


def row_block(rank: int, world: int, batch: int) -> Tuple[int, int]:
    """Rows [start, stop) of ``rank``: contiguous blocks of ceil(batch / world)
    rows (the last ones shorter or empty)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("rank outside [0, world)")
    per = -(-batch // world)
    start = min(rank * per, batch)
    return start, min(start + per, batch)


def row_seeds(seed: int, start: int, stop: int) -> np.ndarray:
    """xorshift64* states of rows [start, stop) of a batch seeded with
    ``seed``: seed + r for global row r (never 0, the generator's fixed point)."""
    s = (np.arange(start, stop, dtype=np.uint64) + np.uint64(seed & 0xFFFFFFFFFFFFFFFF))
    s[s == 0] = 1
    return s


def gather_rows(local, batch: int, world: int, rank: int, dst: int = 0, group=None):
    """Gathers every rank's row block of a per-row tensor (first dimension =
    rows, blocks as ``row_block``) into the whole batch on ``dst``; other
    ranks get None.  Blocks are padded to a common length for the collective."""
    import torch
    import torch.distributed as dist
    per = -(-batch // world)
    start, stop = row_block(rank, world, batch)
    n = stop - start
    if local.shape[0] != n:
        raise ValueError(f"rank {rank} holds {local.shape[0]} rows, its block has {n}")
    pad = torch.zeros((per,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    pad[:n] = local
    parts: Optional[List] = None
    if rank == dst:
        parts = [torch.empty_like(pad) for _ in range(world)]
    dist.gather(pad, gather_list=parts, dst=dst, group=group)
    if rank != dst:
        return None
    out = []
    for r in range(world):
        a, b = row_block(r, world, batch)
        out.append(parts[r][:b - a])
    return torch.cat(out, dim=0)


def max_over_ranks(value: float, device=None, group=None) -> float:
    """The largest of every rank's ``value`` (the timed region of a multi-GPU
    step is the slowest rank's)."""
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())
