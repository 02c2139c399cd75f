"""Host logic of the multi-GPU jobs (one process per GPU; torch.distributed for the plumbing).

The op-chain shards only where acestep.cpp's work is independent (process-per-GPU replicas,
tools/ace-server.cpp:2118): the sequences of a DiT batch and the sequences of a batched LM
decode. Nothing here computes; these helpers decide which sequences a rank owns and move the
per-rank results, so that every rank ends a DiT step with the full batch of velocities in the
reference's slot order (conditional tracks 0..N-1, then their unconditional twins N..2N-1, the
CFG packing of dit-sampler.h:167-174), and a sharded job reports its time as the max over ranks.
"""
from __future__ import annotations


def dit_slots(n_seq: int, world: int, rank: int) -> list[int]:
    """The contiguous block of batch slots rank `rank` evaluates (n_seq = 2 * tracks with CFG)."""
    if world <= 0 or n_seq % world != 0:
        raise ValueError(f"{n_seq} sequences do not shard over {world} ranks")
    n = n_seq // world
    return list(range(rank * n, (rank + 1) * n))


def slot_tracks(slots: list[int], n_tracks: int) -> tuple[list[int], list[bool]]:
    """Track index of every slot and whether the slot is the unconditional twin (slot >= N)."""
    return [j % n_tracks for j in slots], [j >= n_tracks for j in slots]


def gather_rows(t_loc, world: int):
    """All ranks' `t_loc` (same shape) concatenated along dim 0 in rank order, on every rank.
    NCCL gathers into one tensor; other backends (gloo on the CPU) gather a list."""
    import torch
    import torch.distributed as dist
    if world == 1:
        return t_loc
    if dist.get_backend() == "nccl":
        out = torch.empty((world * t_loc.shape[0],) + tuple(t_loc.shape[1:]), dtype=t_loc.dtype, device=t_loc.device)
        dist.all_gather_into_tensor(out, t_loc.contiguous())
        return out
    parts = [torch.empty_like(t_loc) for _ in range(world)]
    dist.all_gather(parts, t_loc.contiguous())
    return torch.cat(parts, 0)


def max_over_ranks(value: float, world: int, device=None) -> float:
    """The job's time: the slowest rank's (every rank gets it)."""
    if world == 1:
        return float(value)
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
