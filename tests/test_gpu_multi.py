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


def test_python_cli_two_gpus_equals_oracle(cuda_ok, tmp_path):
    """python -m knng_gpu_b200.cli --gpus 2 relaunches itself as two NCCL
    ranks and writes the same .knng as the oracle graph."""
    import numpy as np
    import torch

    from knng_gpu_b200 import io as kio
    from knng_gpu_b200 import synthetic as syn
    from refs import oracle_knn

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    x = syn.generate(syn.KIND_UNIFORM_INT, 31, 3000, 64)
    p = tmp_path / "d.fvecs"
    kio.write_vecs(p, x)
    out = tmp_path / "o.knng"
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run([sys.executable, "-m", "knng_gpu_b200.cli", "--dataset", str(p), "--k", "9", "--gpus", "2",
                        "--output", str(out)], capture_output=True, text=True, timeout=900, env=env,
                       cwd=HERE.parent)
    assert r.returncode == 0, r.stderr[-4000:]
    ids, dists, _, _ = kio.read_knng(out)
    oi, od = oracle_knn(x, 9, 0)
    assert np.array_equal(ids, oi) and np.array_equal(dists, od)
