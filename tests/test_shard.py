"""The multi-rank host logic, on CPU ranks (gloo, world size 2 and 4): contiguous
aligned shards cover the batch, the all-gather of per-rank partials arrives in
rank order, and folding the gathered partials with the canonical pairwise levels
(the oracle's restatement, eagle/reduce/canonical.h:358-381) gives the bits of the
one-rank reduction (eagle/exec/RankPartition.h:222-241's rank-order fold)."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from eagle_b200 import shard


def test_shard_ranges_cover_the_batch():
    for n in (1, 7, 4096, 100_003, 1 << 24):
        for world in (1, 2, 3, 4, 8):
            got = [shard.shard_range(n, r, world) for r in range(world)]
            assert got[0][0] == 0 and sum(c for _, c in got) == n
            assert all(b + c == nb for (b, c), (nb, _) in zip(got, got[1:]))
    assert shard.is_aligned_split(1 << 24, 8) and shard.is_aligned_split(1 << 22, 2)
    assert not shard.is_aligned_split(100_003, 2) and not shard.is_aligned_split(1 << 24, 3)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, n, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import oracle

        x = oracle.corpus(n, 99)
        begin, count = shard.shard_range(n, rank, world)
        local = torch.from_numpy(oracle.pairwise(oracle.leaf_partials(x[begin:begin + count])))
        gathered = [torch.zeros(2, dtype=torch.float64) for _ in range(world)]
        dist.all_gather(gathered, local)
        pairs = np.stack([g.numpy() for g in gathered])
        root = oracle.pairwise(pairs)
        out[rank] = (oracle.partial_value(root[0], root[1]), float(oracle.reduce(x)[0]),
                     [float(p[0]) for p in pairs], float(local[0]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", (2, 4))
def test_rank_order_fold_is_the_whole(orc, world):
    n = 1 << 20
    with mp.get_context("spawn").Manager() as mgr:  # no fork of this threaded process
        out = mgr.dict()
        mp.spawn(_rank, args=(world, _free_port(), n, out), nprocs=world, join=True)
        res = dict(out)
    for r in range(world):
        folded, whole, his, mine = res[r]
        assert np.float64(folded).tobytes() == np.float64(whole).tobytes()
        assert his[r] == mine  # the gather is in rank order


def _ragged_rank(rank, world, port, counts, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import oracle

        whole = oracle.corpus(sum(counts), 7)
        begin = sum(counts[:rank])
        kept = torch.zeros(counts[rank] + 3, dtype=torch.float64)  # capacity past the count, as a compaction leaves
        kept[:counts[rank]] = torch.from_numpy(whole[begin:begin + counts[rank]])

        def leaves(x):
            return torch.from_numpy(oracle.leaf_partials(x.numpy()))

        def combine(pairs):
            h, c = oracle.pairwise(pairs.numpy())
            return torch.tensor([h, c, oracle.partial_value(h, c)], dtype=torch.float64)

        r = shard.ragged_fold(kept, counts[rank], leaf_partials=leaves, combine=combine)
        want = oracle.reduce(whole, pair_out=True) if sum(counts) else np.zeros(2)
        out[rank] = (r.numpy().tobytes(), np.float64(oracle.reduce(whole)[0] if sum(counts) else 0.0).tobytes(),
                     np.asarray(want, dtype=np.float64)[:2].tobytes())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("counts", ([5000, 3000], [0, 9000, 1, 4095], [4096, 4096, 8192, 10], [1, 2, 3],
                                    [20000, 0, 0, 123]))
def test_ragged_survivors_fold_to_the_whole(orc, counts):
    """Ragged per-rank survivors (zeros, fragments smaller than a leaf, exact leaves):
    the exchange of heads and leaf partials gives the bits of the one-rank canonical
    sum over the concatenation."""
    world = len(counts)
    with mp.get_context("spawn").Manager() as mgr:  # no fork of this threaded process
        out = mgr.dict()
        mp.spawn(_ragged_rank, args=(world, _free_port(), counts, out), nprocs=world, join=True)
        res = dict(out)
    for r in range(world):
        got, want_value, want_pair = res[r]
        got = np.frombuffer(got, dtype=np.float64)
        assert got[2:3].tobytes() == want_value
        assert got[:2].tobytes() == want_pair


def _map_rank(rank, world, port, n, p, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import oracle

        keep = np.random.default_rng([17, n]).random(n) < p
        begin, count = shard.shard_range(n, rank, world)
        local, c = oracle.compact(keep[begin:begin + count], drop=False)
        assert c == local.size
        idx, offset, total = shard.global_map(torch.from_numpy(np.asarray(local, dtype=np.int32)), c, begin)
        out[rank] = (idx.numpy().tobytes(), offset, total, str(idx.dtype))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,n,p", ((2, 100_003, 0.5), (4, 4096 * 5 + 7, 0.01), (4, 1000, 0.0), (2, 3, 1.0)))
def test_sharded_maps_concatenate_to_the_whole(orc, world, n, p):
    """Each rank's survivors, shifted to global sample indices and placed at the
    survivors of the earlier ranks, make the one-rank ascending map of the batch."""
    with mp.get_context("spawn").Manager() as mgr:  # no fork of this threaded process
        out = mgr.dict()
        mp.spawn(_map_rank, args=(world, _free_port(), n, p, out), nprocs=world, join=True)
        res = dict(out)
    keep = np.random.default_rng([17, n]).random(n) < p
    want, total = orc.compact(keep, drop=False)
    got = np.zeros(total, dtype=np.int64)
    for r in range(world):
        idx, offset, tot, dtype = res[r]
        part = np.frombuffer(idx, dtype=np.int64)
        assert tot == total and dtype == "torch.int64"
        got[offset:offset + part.size] = part
        assert offset + part.size <= total
    assert sum(np.frombuffer(res[r][0], dtype=np.int64).size for r in range(world)) == total
    assert np.array_equal(got, np.asarray(want, dtype=np.int64))
