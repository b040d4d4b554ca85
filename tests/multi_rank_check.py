"""One rank of the multi-GPU check (launched by tests/test_gpu_multi.py under
torchrun): the engine on this rank's shard of a 2^22-sample batch, the canonical
partial of x, an NCCL all-gather and the device fold; then a compaction of this
rank's shard of an uneven batch and the ragged exchange of its survivors. Rank 0
compares both results' bits with the oracle's one-device runs of the whole batch."""

import datetime
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import eagle_b200 as eb  # noqa: E402
from eagle_b200 import shard  # noqa: E402


def main():
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", local))
    rank, world = dist.get_rank(), dist.get_world_size()
    n = 1 << 22
    rng = np.random.default_rng(42)
    om, x0, te = rng.uniform(1, 3, n), rng.normal(1, 0.1, n), 10.0 ** rng.uniform(-2, 1, n)
    begin, count = shard.shard_range(n, rank, world)
    sl = slice(begin, begin + count)
    dev = dict(omega=torch.from_numpy(om[sl].copy()).cuda(), t_end=torch.from_numpy(te[sl].copy()).cuda(),
               x=torch.from_numpy(x0[sl].copy()).cuda(), v=torch.zeros(count, dtype=torch.float64, device="cuda"),
               t=torch.zeros(count, dtype=torch.float64, device="cuda"))
    res = eb.simulate(eb.oscillator, max_steps=10_000, fma=True, mode="persist", dt=1e-3, **dev)
    pair = eb.reduce(res.x, pair_out=True)
    folded = shard.fold_partials(shard.gather_partials(pair))
    torch.cuda.synchronize()
    if rank == 0:
        import oracle

        st = [x0.copy(), np.zeros(n), np.zeros(n), np.zeros(n, np.uint8)]
        oracle.oscillator_run(om, *st, t_end=te, dt=1e-3, max_steps=10_000, fused=True)
        want = oracle.reduce(st[0])[0]
        got = folded[2].item()
        if np.float64(got).tobytes() != np.float64(want).tobytes():
            print(f"MISMATCH folded {got!r} whole {want!r}", flush=True)
            sys.exit(1)
        print("RANK-ORDER FOLD OK", world, got, flush=True)
    # compact-then-sum over ragged survivors: an uneven batch, so no shard is a subtree
    nv = (1 << 22) + 12_345
    g = np.random.default_rng(7)
    vals, keep = g.standard_normal(nv), g.random(nv) < 0.37
    b, c = shard.shard_range(nv, rank, world)
    got = shard.compact_sum_sharded(torch.from_numpy(keep[b:b + c].copy()).cuda(),
                                    torch.from_numpy(vals[b:b + c].copy()).cuda())
    torch.cuda.synchronize()
    if rank == 0:
        import oracle

        want = oracle.reduce(vals[keep])[0]
        if np.float64(got[2].item()).tobytes() != np.float64(want).tobytes():
            print(f"MISMATCH ragged {got[2].item()!r} whole {want!r}", flush=True)
            sys.exit(1)
        print("RAGGED COMPACT-SUM OK", world, want, flush=True)
    # the same survivors through the device-side exchange (no host round trip), and a
    # batch whose shards keep few survivors, so that one leaf spans several ranks' heads
    for frac, label in ((0.37, "dense"), (0.0003, "sparse")):
        keep2 = keep if label == "dense" else g.random(nv) < frac
        sc = shard.ShardedCompactSum(torch.from_numpy(keep2[b:b + c].copy()).cuda(),
                                     torch.from_numpy(vals[b:b + c].copy()).cuda())
        for _ in range(2):  # twice: the prepared buffers are reused
            out = sc()
        torch.cuda.synchronize()
        if rank == 0:
            import oracle

            want = oracle.reduce(vals[keep2])[0]
            if np.float64(out[2].item()).tobytes() != np.float64(want).tobytes():
                print(f"MISMATCH device ragged ({label}) {out[2].item()!r} whole {want!r}", flush=True)
                sys.exit(1)
    if rank == 0:
        print("DEVICE RAGGED COMPACT-SUM OK", world, flush=True)
    sm = shard.ShardedCompactor(torch.from_numpy(keep[b:b + c].copy()).cuda(), b, drop=False)
    offset_d, total_d = sm()
    whole = np.flatnonzero(keep)
    mine = sm.indices().cpu().numpy()
    off = int(offset_d.item())
    if int(total_d.item()) != whole.size or not np.array_equal(mine, whole[off:off + mine.size]):
        print(f"MISMATCH device map rank {rank} offset {off}", flush=True)
        sys.exit(1)
    # the compaction map over every shard: each rank's global indices at its offset
    idx, offset, total = shard.compact_map_sharded(torch.from_numpy(keep[b:b + c].copy()).cuda(), b, drop=False)
    whole = np.flatnonzero(keep)
    mine = idx.cpu().numpy()
    if total != whole.size or not np.array_equal(mine, whole[offset:offset + mine.size]):
        print(f"MISMATCH map rank {rank} offset {offset} total {total}", flush=True)
        sys.exit(1)
    dist.barrier()
    if rank == 0:
        print("SHARDED MAP OK", world, total, flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
