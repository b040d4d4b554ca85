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
    with mp.Manager() as mgr:
        out = mgr.dict()
        mp.spawn(_rank, args=(world, _free_port(), n, out), nprocs=world, join=True)
        res = dict(out)
    for r in range(world):
        folded, whole, his, mine = res[r]
        assert np.float64(folded).tobytes() == np.float64(whole).tobytes()
        assert his[r] == mine  # the gather is in rank order
