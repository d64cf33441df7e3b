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
    assert r.stdout.count("equal=True") == 8


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


@pytest.mark.parametrize("ring", [False, True])
def test_single_process_multi_gpu_equals_oracle(cuda_ok, ring):
    """knng_gpu_brute_force_multi (one process, NCCL inside the library) on
    every GPU of the box: bit-identical to the oracle graph."""
    import numpy as np
    import torch

    import knng_gpu_b200 as kg
    from knng_gpu_b200 import synthetic as syn
    from refs import oracle_knn

    g = torch.cuda.device_count()
    if g < 2:
        pytest.skip("needs 2 GPUs")
    # Shard sizes whose packed blocks and key offsets end off a 16-byte
    # boundary (3001, 20011 on two ranks) as well as even ones.
    for kind, n, d, k, metric in [(syn.KIND_UNIFORM_INT, 6007, 128, 10, 0), (syn.KIND_UNIFORM_INT, 3001, 128, 10, 0),
                                  (syn.KIND_UNIFORM_INT, 20011, 128, 10, 0), (syn.KIND_SPARSE_INT, 3001, 784, 64, 1),
                                  (syn.KIND_UNIFORM_INT, 4001, 300, 16, 0)]:
        x = syn.generate(kind, 41, n, d, p_zero=0.6)
        out = kg.brute_force_knn_multi(x, k, metric, num_gpus=g, ring=ring)
        oi, od = oracle_knn(x, k, metric)
        assert np.array_equal(out.neighbors.reshape(n, k), oi)
        assert np.array_equal(out.distances.reshape(n, k).view(np.uint32), od.view(np.uint32))
    if not ring:
        y = syn.generate(syn.KIND_GAUSSIAN_MIXTURE, 42, 4000, 64, components=10, sigma=0.1)
        out = kg.brute_force_knn_multi(y, 7, 0, num_gpus=g)
        oi, od = oracle_knn(y, 7, 0)
        assert np.array_equal(out.neighbors.reshape(-1, 7), oi) and np.array_equal(out.distances.reshape(-1, 7), od)


@pytest.mark.parametrize("ring", [False, True])
def test_sharded_path_on_one_gpu_equals_oracle(cuda_ok, ring):
    """The multi-GPU code path (knng_gpu_brute_force_multi: NCCL communicator,
    pack, flag all-reduce, base all-gather or ring pass, gather to rank 0)
    with a single rank, so it runs on every GPU box; fp32 data goes through
    the fp32 exchange and path."""
    import numpy as np

    import knng_gpu_b200 as kg
    from knng_gpu_b200 import synthetic as syn
    from refs import oracle_knn

    x = syn.generate(syn.KIND_UNIFORM_INT, 43, 5000, 128)
    out = kg.brute_force_knn_multi(x, 10, 0, num_gpus=1, ring=ring)
    oi, od = oracle_knn(x, 10, 0)
    assert np.array_equal(out.neighbors.reshape(-1, 10), oi)
    assert np.array_equal(out.distances.reshape(-1, 10), od)
    if not ring:
        y = syn.generate(syn.KIND_GAUSSIAN_MIXTURE, 44, 3000, 48, components=8, sigma=0.1)
        out = kg.brute_force_knn_multi(y, 6, 0, num_gpus=1)
        oi, od = oracle_knn(y, 6, 0)
        assert np.array_equal(out.neighbors.reshape(-1, 6), oi) and np.array_equal(out.distances.reshape(-1, 6), od)
