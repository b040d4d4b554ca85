"""Multi-GPU: every rank runs the until-done engine on its contiguous shard, the
per-rank canonical partials of x are all-gathered over NCCL and folded in rank
order on the device; the result's bits equal the one-device run over the whole
batch (checked against the oracle); and a compaction's ragged survivors, summed
across ranks by the head and leaf-partial exchange, give the bits of the one-device
compact-then-sum; and each rank's compaction map, placed by the all-gathered
counts, is its part of the one-device map of the whole batch. Runs under
torchrun when two or more GPUs are visible; skipped otherwise."""

import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SCRIPT = os.path.join(ROOT, "tests", "multi_rank_check.py")


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("world", (2, 4, 8))
def test_shards_fold_to_the_whole(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr=127.0.0.1", "--master-port=29511", SCRIPT]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, cwd=ROOT)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "RANK-ORDER FOLD OK" in r.stdout
    assert "RAGGED COMPACT-SUM OK" in r.stdout
    assert "SHARDED MAP OK" in r.stdout
    assert "DEVICE RAGGED COMPACT-SUM OK" in r.stdout
