"""Contiguous sample shards across ranks, and the rank-order fold of their
canonical partials.

eagle splits samples over MPI ranks and folds per-rank partials in rank order
(eagle/exec/RankPartition.h:222-241 of the eagle source tree; MPI_Allreduce is
avoided there because its combine order is unspecified). Here ranks are the GPUs of
one box under ``torch.distributed``: each rank holds one contiguous shard, runs
the until-done loop on it with no traffic to the others, reduces its shard to a
16-byte ``(hi, comp)`` partial, and the partials are all-gathered in rank order
(NCCL on GPUs, gloo on CPU) and folded by the canonical pairwise levels on the
device. A shard of ``4096 * 2^q`` samples is a subtree of the canonical tree
(eagle/reduce/canonical.h:30-32), so with a power-of-two rank count the folded
bits equal the one-device reduction of the concatenated shards.
"""

from __future__ import annotations

import ctypes

from . import _abi

LEAF = 4096


def shard_range(n: int, rank: int, world: int) -> tuple[int, int]:
    """``(begin, count)`` of rank ``rank``'s contiguous shard of ``n`` samples."""
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside [0, {world})")
    base, extra = divmod(n, world)
    begin = rank * base + min(rank, extra)
    return begin, base + (1 if rank < extra else 0)


def is_aligned_split(n: int, world: int) -> bool:
    """True when every shard is ``4096 * 2^q`` samples and ``world`` is a power of
    two: then the rank-order fold gives the bits of the whole (canonical.h:90-95)."""
    if world < 1 or world & (world - 1):
        return False
    if n % world:
        return False
    chunk = n // world
    return chunk >= LEAF and chunk & (chunk - 1) == 0


def gather_partials(local_pair, group=None):
    """All-gather each rank's ``(hi, comp)`` pair (a 2-element float64 tensor on the
    rank's device) into a ``2 * world`` tensor in rank order."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    out = torch.empty(2 * world, dtype=torch.float64, device=local_pair.device)
    dist.all_gather_into_tensor(out, local_pair.reshape(2).contiguous(), group=group)
    return out


def fold_partials(pairs, stream=None):
    """The canonical pairwise fold of ``pairs`` (a CUDA float64 tensor of m (hi, comp)
    pairs, chunk order) on the device: a 3-element tensor {hi, comp, value}."""
    import torch

    if not (pairs.is_cuda and pairs.dtype == torch.float64 and pairs.numel() % 2 == 0 and pairs.numel() >= 2):
        raise ValueError("fold_partials takes a CUDA float64 tensor of (hi, comp) pairs")
    m = pairs.numel() // 2
    work = torch.empty(2 * ((m + 511) // 512) + 2, dtype=torch.float64, device=pairs.device)
    out = torch.empty(3, dtype=torch.float64, device=pairs.device)
    s = (stream or torch.cuda.current_stream()).cuda_stream
    _abi.check(_abi.lib().eagle_backend_x_b200_combine_partials(pairs.data_ptr(), m, work.data_ptr(),
                                                                out.data_ptr(), s))
    return out
