"""Host side of the multi-GPU layout: every GPU runs a full replica of the
model on its own block of sequences, and nothing is exchanged inside a step
(sequences are independent).  After a timed region the ranks agree on the
slowest rank's device time and the total of generated tokens, and rank 0
gathers the per-rank figures.

One process per GPU (torchrun sets RANK / LOCAL_RANK / WORLD_SIZE).  These
helpers run unchanged on the gloo backend with CPU tensors, which is how they
are tested without GPUs.
"""
from __future__ import annotations

import os
from typing import List, Optional, Tuple


def replica_env() -> Tuple[int, int, int]:
    """(world, rank, local_rank) from the torchrun environment (1, 0, 0 alone)."""
    return (int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")),
            int(os.environ.get("LOCAL_RANK", "0")))


def sequence_slice(global_seqs: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous block [start, end) of the global sequence ids owned by a
    rank; blocks differ in size by at most one sequence."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    base, extra = divmod(global_seqs, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def step_totals(device_ms: float, tokens: int, device=None) -> Tuple[float, int]:
    """(max over ranks of device_ms, sum over ranks of tokens).  A no-op for a
    single process; every rank must call it (it is a collective)."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(device_ms), int(tokens)
    dev = device if device is not None else ("cuda" if dist.get_backend() == "nccl" else "cpu")
    mx = torch.tensor([float(device_ms)], dtype=torch.float64, device=dev)
    sm = torch.tensor([float(tokens)], dtype=torch.float64, device=dev)
    dist.all_reduce(mx, op=dist.ReduceOp.MAX)
    dist.all_reduce(sm, op=dist.ReduceOp.SUM)
    return float(mx.item()), int(round(sm.item()))


def gather_to_root(obj) -> Optional[List]:
    """Every rank's object, in rank order, on rank 0 (None elsewhere)."""
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return [obj]
    out = [None] * dist.get_world_size() if dist.get_rank() == 0 else None
    dist.gather_object(obj, out, dst=0)
    return out
