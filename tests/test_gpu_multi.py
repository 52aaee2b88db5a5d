"""Head sharding on real GPUs (needs two): tests/multi_gpu_worker.py under torch.distributed.run, NCCL all-gather per layer
captured in the decode graph. Skipped on a single-GPU box."""
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.parametrize("serve", ["sparse", "fsb"])
def test_head_sharded_decode_matches_unsharded(serve):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2", "--master-addr", "127.0.0.1",
           "--master-port", "29531", os.path.join(HERE, "multi_gpu_worker.py"), serve]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "ranks agree True" in r.stdout
