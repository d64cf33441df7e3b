"""Multi-GPU builds (one process per GPU, NCCL): the all-gather builder and
the ring pass of base blocks both give a graph bit-identical to the
single-GPU graph. Needs two or more GPUs."""
import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
HERE = Path(__file__).resolve().parent


def test_two_gpu_sharded_build_equals_single_gpu(cuda_ok):
    import torch

    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs 2 GPUs")
    world = min(n, 4)
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--standalone", "--nproc-per-node", str(world),
                        str(HERE / "dist_worker.py")], capture_output=True, text=True, timeout=900, env=env)
    print(r.stdout[-4000:], r.stderr[-4000:])
    assert r.returncode == 0
    assert r.stdout.count("equal=True") == 5
