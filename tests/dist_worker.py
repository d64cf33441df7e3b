"""torchrun worker for tests/test_gpu_multi.py: the C-ABI sharded build
(replicate and ring modes, NCCL inside the library), compared on rank 0 with
the single-GPU build of the same dataset."""
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.join(os.path.dirname(__file__), ".."))
import knng_gpu_b200 as kg  # noqa: E402
from knng_gpu_b200 import synthetic as syn  # noqa: E402
from knng_gpu_b200.distributed import MODE_RING, ShardedBuilder  # noqa: E402


def main():
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    ok = True
    for (kind, n, d, k, metric) in [(syn.KIND_UNIFORM_INT, 20011, 128, 10, 0), (syn.KIND_SPARSE_INT, 5003, 784, 64, 1),
                                     (syn.KIND_UNIFORM_PM1, 3001, 64, 8, 0)]:
        x = syn.generate(kind, 1234, n, d, p_zero=0.6)
        b = ShardedBuilder(n, d, k, metric)
        lo, hi = b.slice_bounds
        ids, dists = b.build(torch.from_numpy(x[lo:hi]).cuda())
        if dist.get_rank() == 0:
            g = kg.brute_force_knn(x, k, metric)
            same = np.array_equal(ids.cpu().numpy().view(np.uint32), g.neighbors.reshape(n, k)) and \
                np.array_equal(dists.cpu().numpy(), g.distances.reshape(n, k))
            print(f"n={n} d={d} k={k} metric={metric} world={dist.get_world_size()} equal={same}", flush=True)
            ok &= same
    # ring pass of base blocks (integer data)
    # Blocks on the CTA-pair kernel (d > 256) get the running k-th key of the
    # blocks before them as an outside bound: small blocks (no seeding pass),
    # L2 and inner product, and blocks above the seeding threshold (the
    # seeding pass runs under the outside bound too).
    for (kind, n, d, k, metric) in [(syn.KIND_SPARSE_INT, 5003, 784, 64, 1), (syn.KIND_UNIFORM_INT, 20011, 128, 10, 0),
                                     (syn.KIND_UNIFORM_INT, 6007, 300, 16, 0),
                                     (syn.KIND_SPARSE_INT, 300007, 320, 32, 1),
                                     (syn.KIND_UNIFORM_INT, 300007, 320, 16, 0)]:
        x = syn.generate(kind, 77, n, d, p_zero=0.6)
        rb = ShardedBuilder(n, d, k, metric, MODE_RING)
        lo, hi = rb.slice_bounds
        ids, dists = rb.build(torch.from_numpy(x[lo:hi]).cuda())
        if dist.get_rank() == 0:
            g = kg.brute_force_knn(x, k, metric)
            same = np.array_equal(ids.cpu().numpy().view(np.uint32), g.neighbors.reshape(n, k)) and \
                np.array_equal(dists.cpu().numpy(), g.distances.reshape(n, k))
            print(f"ring n={n} d={d} k={k} metric={metric} world={dist.get_world_size()} equal={same}", flush=True)
            ok &= same
    dist.barrier()
    dist.destroy_process_group()
    sys.exit(0 if ok else 1)


if __name__ == "__main__":
    main()
