"""Batch sharding of the policy-sampling path over GPUs, one process per GPU.

Chunks are independent: sampling has no cross-sample reduction and GroupNorm
is per sample, so a global batch splits into contiguous shards, one per rank,
with no collective inside the sampling loop.  DDPM noise stays shard-invariant
because sample b of a batched call with seed s draws from the Gaussian stream
of seed s + b (the reference's single-sample stream, diffusion.cc:193-231): a
rank whose shard starts at global index `offset` calls with seed + offset.
Collectives run only after the timed region: the maximum of the ranks' device
times and the all-gather of the actions.  `dist` is `torch.distributed` (NCCL
on GPUs, gloo in the CPU tests).
"""

from __future__ import annotations


def shard_range(global_batch: int, world: int, rank: int) -> tuple[int, int]:
    """(offset, size) of rank's contiguous shard; the first global_batch % world
    ranks take one extra chunk."""
    if world < 1 or not 0 <= rank < world or global_batch < 0:
        raise ValueError(f"invalid shard request: batch {global_batch}, world {world}, rank {rank}")
    base, extra = divmod(global_batch, world)
    size = base + (1 if rank < extra else 0)
    offset = rank * base + min(rank, extra)
    return offset, size


def shard_seed(seed: int, offset: int) -> int:
    """Seed of a rank's batched call, so that every sample keeps the seed of its
    global index (seed + index) whatever the number of ranks."""
    return (int(seed) + int(offset)) & 0xFFFFFFFFFFFFFFFF


def max_over_ranks(value: float, dist=None, device=None) -> float:
    """Maximum of a per-rank value (a device time) over all ranks."""
    if dist is None:
        return float(value)
    import torch

    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_rows(local, dist=None):
    """All-gather of every rank's rows (equal shard sizes), concatenated in rank
    order, i.e. in global batch order for contiguous shards."""
    if dist is None:
        return local
    import torch

    parts = [torch.empty_like(local) for _ in range(dist.get_world_size())]
    dist.all_gather(parts, local)
    return torch.cat(parts, dim=0)
