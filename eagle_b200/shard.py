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

A compaction's survivors are ragged: rank r keeps ``c_r`` values, so its part of
the concatenated survivors starts at an arbitrary offset and its partial is no
subtree. :func:`compact_sum_sharded` makes the one exchange that needs: the
counts are all-gathered (offsets by prefix), every rank shares its first
``LEAF - 1`` survivors, each rank forms the partials of the leaves that START in
its part (completing its last leaf from the later ranks' heads), and the leaf
partials are all-gathered and joined by the canonical pairwise levels -- the bits
of the one-device canonical sum over the concatenated survivors. The compaction map
itself needs only the counts: :func:`compact_map_sharded` gives each rank its
survivors' global sample indices and where they start in the map over all shards.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass, field

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


@dataclass
class RaggedPlan:
    """Rank ``rank``'s share of the canonical tree over ragged survivors."""

    offset: int          # the rank's first survivor in the concatenation
    total: int           # all ranks' survivors
    first_leaf: int      # the first leaf starting in the rank's part
    leaves: int          # leaves starting in the rank's part
    local_start: int     # the first such leaf's start, in the rank's own survivors
    full_end: int        # local end of the leaves complete within the rank
    straddle: list = field(default_factory=list)  # (rank q, lo, hi): head pieces completing the last leaf
    straddle_len: int = 0  # elements of the straddling leaf (0: none)


def ragged_plan(counts, rank: int) -> RaggedPlan:
    """Which leaves of the canonical tree over the concatenation of every rank's
    survivors (``counts[q]`` on rank q, in rank order) rank ``rank`` forms, and the
    pieces of later ranks' heads its last leaf needs."""
    counts = [int(c) for c in counts]
    offsets = [0]
    for c in counts:
        offsets.append(offsets[-1] + c)
    total = offsets[-1]
    o, c = offsets[rank], counts[rank]
    plan = RaggedPlan(offset=o, total=total, first_leaf=0, leaves=0, local_start=0, full_end=0)
    if c == 0:
        return plan
    first = -(-o // LEAF)
    last = (o + c - 1) // LEAF
    if first > last:
        return plan  # every survivor here belongs to a leaf an earlier rank forms
    plan.first_leaf, plan.leaves = first, last - first + 1
    plan.local_start = first * LEAF - o
    end = min((last + 1) * LEAF, total)  # the last leaf's global end
    if end <= o + c:
        plan.full_end = end - o
        return plan
    plan.full_end = last * LEAF - o
    plan.straddle_len = end - last * LEAF
    for q in range(rank + 1, len(counts)):
        lo, hi = max(offsets[q], o + c), min(offsets[q + 1], end)
        if lo < hi:
            plan.straddle.append((q, lo - offsets[q], hi - offsets[q]))
        if offsets[q + 1] >= end:
            break
    return plan


def ragged_fold(kept, count: int, *, group=None, leaf_partials=None, combine=None):
    """The canonical sum over every rank's survivors ``kept[:count]`` (1-D float64
    tensors, any device), joined in rank order: ``(hi, comp, value)`` on every rank.
    ``leaf_partials`` maps a 1-D tensor to its ``(leaves, 2)`` partials and
    ``combine`` a ``(m, 2)`` tensor of pairs to ``(hi, comp, value)``; both default
    to this library's device entries."""
    import torch
    import torch.distributed as dist

    leaf_partials = leaf_partials or device_leaf_partials
    combine = combine or (lambda pairs: fold_partials(pairs.reshape(-1)))
    dev = kept.device
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    cnt = torch.tensor([int(count)], dtype=torch.int64, device=dev)
    gathered = [torch.zeros(1, dtype=torch.int64, device=dev) for _ in range(world)]
    dist.all_gather(gathered, cnt, group=group)
    counts = [int(g.item()) for g in gathered]
    total = sum(counts)
    if total == 0:
        return torch.zeros(3, dtype=torch.float64, device=dev)
    # every rank's first LEAF - 1 survivors
    head = torch.zeros(LEAF - 1, dtype=torch.float64, device=dev)
    h = min(int(count), LEAF - 1)
    head[:h] = kept[:h]
    heads = [torch.zeros(LEAF - 1, dtype=torch.float64, device=dev) for _ in range(world)]
    dist.all_gather(heads, head, group=group)
    plan = ragged_plan(counts, rank)
    pairs = []
    if plan.full_end > plan.local_start:
        pairs.append(leaf_partials(kept[plan.local_start:plan.full_end].contiguous()))
    if plan.straddle_len:
        parts = [kept[plan.full_end:int(count)]] + [heads[q][lo:hi] for q, lo, hi in plan.straddle]
        leaf = torch.cat(parts).contiguous()
        assert leaf.numel() == plan.straddle_len
        pairs.append(leaf_partials(leaf))
    mine = torch.cat(pairs) if pairs else torch.zeros((0, 2), dtype=torch.float64, device=dev)
    # all-gather the leaf partials, each rank's padded to the most any rank forms
    sizes = [ragged_plan(counts, q).leaves for q in range(world)]
    width = max(sizes)
    padded = torch.zeros((width, 2), dtype=torch.float64, device=dev)
    padded[:mine.shape[0]] = mine
    every = [torch.zeros((width, 2), dtype=torch.float64, device=dev) for _ in range(world)]
    dist.all_gather(every, padded, group=group)
    ordered = torch.cat([every[q][:sizes[q]] for q in range(world)]).contiguous()
    return combine(ordered)


def global_map(local_map, count: int, begin: int, *, group=None):
    """This rank's part of the compaction map over every rank's shard in rank order:
    ``(indices, offset, total)``. ``indices`` are ``local_map[:count]`` shifted by the
    shard's first sample ``begin`` (int64: eight shards of 2^28 pass int32), ``offset``
    is the survivors of the earlier ranks -- where this part starts in the
    concatenated map -- and ``total`` all ranks' survivors, from one all-gather of the
    counts (Compact.h:23-47's ascending map, per rank plus a rank base offset)."""
    import torch
    import torch.distributed as dist

    dev = local_map.device
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    cnt = torch.tensor([int(count)], dtype=torch.int64, device=dev)
    gathered = [torch.zeros(1, dtype=torch.int64, device=dev) for _ in range(world)]
    dist.all_gather(gathered, cnt, group=group)
    counts = [int(g.item()) for g in gathered]
    indices = local_map[:int(count)].to(torch.int64) + int(begin)
    return indices, sum(counts[:rank]), sum(counts)


def compact_map_sharded(mask, begin: int, *, drop: bool = True, group=None):
    """Compact this rank's shard (``mask`` holds samples ``[begin, begin + n)``) on its
    device and place the survivors in the map over every rank's shard:
    ``(indices, offset, total)`` as :func:`global_map` returns them."""
    from ._api import compact

    index_map, count = compact(mask, drop=drop)
    return global_map(index_map, int(count.item()), begin, group=group)


def device_leaf_partials(x):
    """``(leaves, 2)`` (hi, comp) leaf partials of a CUDA float64 tensor."""
    import torch

    n = x.numel()
    out = torch.empty(((n + LEAF - 1) // LEAF, 2), dtype=torch.float64, device=x.device)
    if n:
        _abi.check(_abi.lib().eagle_backend_x_b200_leaf_partials(x.data_ptr(), n, out.data_ptr(),
                                                                  torch.cuda.current_stream(x.device).cuda_stream))
    return out


def compact_sum_sharded(mask, values, *, drop: bool = False, group=None):
    """Compact each rank's shard and take the canonical sum of every rank's
    survivors as ONE concatenation in rank order: ``(hi, comp, value)`` on every
    rank, the bits of the one-device compact-then-sum of the concatenated shards."""
    from ._api import CompactSum

    cs = CompactSum(mask, values, drop=drop)
    cs.gather()
    count = int(cs.count.item())
    return ragged_fold(cs.kept, count, group=group)


class ShardedCompactSum:
    """The canonical sum of every rank's survivors as ONE concatenation in rank order,
    prepared once per shard and run with no host round trip and without writing the
    survivors out. Each call runs the fused compact-then-sum's front end on this rank's
    shard (``eagle_backend_x_b200_compact_sum_count``) and forms the rank's head block
    -- its first ``LEAF - 1`` survivors and its count (``_compact_sum_head``) -- then
    all-gathers the head blocks; sums every leaf of the concatenation that starts here
    straight from the values, the one running into the later ranks from their heads
    (``_compact_sum_leaves``, ``_compact_sum_straddle``, planned on the device from
    the gathered counts); all-gathers the partial blocks (the leaf partials and their
    number) and folds them in rank order (``eagle_backend_x_b200_ragged_fold``). Two
    collectives per call, each of a fixed number of bytes. Returns ``(hi, comp,
    value)`` on every rank: the bits of the one-device compact-then-sum of the
    concatenated shards."""

    def __init__(self, mask, values, *, drop: bool = False, group=None):
        import torch
        import torch.distributed as dist

        from ._api import CompactSum

        self.cs = CompactSum(mask, values, drop=drop)
        self.values = values
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        dev = mask.device
        n = mask.numel()
        self.cap = (n + LEAF - 1) // LEAF + 1
        self.block = torch.zeros(LEAF, dtype=torch.float64, device=dev)
        self.blocks = torch.zeros(self.world * LEAF, dtype=torch.float64, device=dev)
        self.partials = torch.zeros(2 * self.cap + 2, dtype=torch.float64, device=dev)
        self.all_partials = torch.zeros(self.world * (2 * self.cap + 2), dtype=torch.float64, device=dev)
        self.work = torch.zeros(2 * ((self.world * self.cap + 511) // 512) + 2, dtype=torch.float64, device=dev)
        self.out = torch.zeros(3, dtype=torch.float64, device=dev)

    def __call__(self, stream=None):
        import ctypes

        import torch
        import torch.distributed as dist

        s = (stream or torch.cuda.current_stream()).cuda_stream
        lib = _abi.lib()
        d = self.cs.sdesc
        d.stream = s
        _abi.check(lib.eagle_backend_x_b200_compact_sum_count(ctypes.byref(d)))
        _abi.check(lib.eagle_backend_x_b200_compact_sum_head(ctypes.byref(d), self.values.data_ptr(),
                                                              self.block.data_ptr()))
        dist.all_gather_into_tensor(self.blocks, self.block, group=self.group)
        _abi.check(lib.eagle_backend_x_b200_compact_sum_leaves(
            ctypes.byref(d), self.values.data_ptr(), self.blocks.data_ptr(), self.rank, self.world,
            self.partials.data_ptr(), self.cap))
        _abi.check(lib.eagle_backend_x_b200_compact_sum_straddle(
            ctypes.byref(d), self.blocks.data_ptr(), self.rank, self.world, self.partials.data_ptr(), self.cap))
        dist.all_gather_into_tensor(self.all_partials, self.partials, group=self.group)
        _abi.check(lib.eagle_backend_x_b200_ragged_fold(
            self.all_partials.data_ptr(), self.world, self.cap, self.work.data_ptr(), self.out.data_ptr(), s))
        return self.out


class ShardedCompactor:
    """This rank's compaction, placed in the map over every rank's shard with no host
    round trip: each call compacts the shard (``begin`` is its first sample) and
    all-gathers the counts on the device; ``offset`` (this rank's first place in the
    concatenated map) and ``total`` are then device tensors. The rank's part of the
    map is ``index_map[:count] + begin`` (:meth:`indices` forms it, int64)."""

    def __init__(self, mask, begin: int, *, drop: bool = True, group=None):
        import torch
        import torch.distributed as dist

        from ._api import Compactor

        self.comp = Compactor(mask, drop=drop)
        self.begin = int(begin)
        self.group = group
        self.rank = dist.get_rank(group)
        self.counts = torch.zeros(dist.get_world_size(group), dtype=torch.int32, device=mask.device)
        self.offset = None
        self.total = None

    def __call__(self, stream=None):
        import torch
        import torch.distributed as dist

        self.comp(stream)
        dist.all_gather_into_tensor(self.counts, self.comp.count, group=self.group)
        c = self.counts.to(torch.int64)
        self.offset = c[:self.rank].sum()
        self.total = c.sum()
        return self.offset, self.total

    def indices(self):
        """This rank's survivors as global sample indices (int64), in map order."""
        import torch

        count = int(self.comp.count.item())
        return self.comp.index_map[:count].to(torch.int64) + self.begin
