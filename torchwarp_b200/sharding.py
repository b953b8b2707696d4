"""Batch sharding of the alignment path over GPUs, one process per GPU.

Pairs are independent: the reference runs one CUDA block per pair
(hibana2077/torchwarp src/torchwarp/csrc/udtw_cuda.cu:3).  A data-parallel
job therefore splits the batch into contiguous shards, each rank runs the
forward and backward of its own pairs, and the only exchange is the gather
of the per-pair outputs (distances, penalties).  Gradients stay with the rank
that owns the pairs.  With the NCCL backend the tensors live on the rank's
GPU; with gloo (tests) on the CPU.
"""

import torch
import torch.distributed as dist


def shard_bounds(B, world, rank):
    """[start, stop) of rank's contiguous shard of B pairs; the first B % world
    ranks take one extra pair."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("rank {} outside a world of {}".format(rank, world))
    if B < 0:
        raise ValueError("negative batch {}".format(B))
    base, rem = divmod(B, world)
    start = rank * base + min(rank, rem)
    return start, start + base + (1 if rank < rem else 0)


def gather_pairs(local, B, group=None):
    """All-gather a per-pair tensor [B_rank, ...] from every rank into [B, ...]
    in rank order.  Shards may differ in size by one pair; they are padded to
    the largest for the collective and trimmed after it."""
    world = dist.get_world_size(group)
    sizes = [b - a for a, b in (shard_bounds(B, world, r) for r in range(world))]
    rank = dist.get_rank(group)
    if local.shape[0] != sizes[rank]:
        raise ValueError("rank {} holds {} pairs, its shard has {}".format(
            rank, local.shape[0], sizes[rank]))
    cap = max(sizes) if sizes else 0
    buf = local.new_zeros((cap,) + tuple(local.shape[1:]))
    buf[:local.shape[0]] = local
    parts = [torch.empty_like(buf) for _ in range(world)]
    dist.all_gather(parts, buf, group=group)
    return torch.cat([p[:n] for p, n in zip(parts, sizes)])
