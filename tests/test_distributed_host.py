"""Host logic of the sharded build on CPU: query sharding follows the
reference's compute_shard (include/knng/dist/sharded_dataset.hpp:145-155),
and the padded all-gather reassembles the graph rows in global order. Two
gloo ranks stand in for two GPUs; each computes its shard with the CPU
oracle (the GPU kernel's place) and the gathered graph must equal the
single-process oracle graph."""
from __future__ import annotations

import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from knng_gpu_b200.distributed import compute_shard, gather_shards, slice_rows


def test_compute_shard_matches_reference_rule():
    # base = n / P, the last rank takes the remainder
    assert compute_shard(10, 3, 0).start == 0 and compute_shard(10, 3, 0).count == 3
    assert compute_shard(10, 3, 1).start == 3 and compute_shard(10, 3, 1).count == 3
    assert compute_shard(10, 3, 2).start == 6 and compute_shard(10, 3, 2).count == 4
    for n in (1, 7, 1000, 1_000_003):
        for p in (1, 2, 4, 8):
            shards = [compute_shard(n, p, r) for r in range(p)]
            assert sum(s.count for s in shards) == n
            assert all(shards[r].start + shards[r].count == shards[r + 1].start for r in range(p - 1))
    assert slice_rows(10, 4) == 3


def _worker(rank, world, port, n, d, k, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import sys
        sys.path.insert(0, os.path.dirname(__file__))
        from refs import oracle_knn
        from knng_gpu_b200 import synthetic as syn

        x = syn.generate(syn.KIND_UNIFORM_INT, 77, n, d)
        sh = compute_shard(n, world, rank)
        ids, dists = oracle_knn(x, k, 0, queries=np.arange(sh.start, sh.start + sh.count, dtype=np.uint64))
        all_ids = gather_shards(torch.from_numpy(ids.astype(np.int32)), n, world)
        all_d = gather_shards(torch.from_numpy(dists), n, world)
        full_ids, full_d = oracle_knn(x, k, 0)
        q.put((rank, bool(np.array_equal(all_ids.numpy().view(np.uint32), full_ids)),
               bool(np.array_equal(all_d.numpy(), full_d))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n", [101, 256])
def test_two_rank_gather_reassembles_the_graph(n):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29650 + n % 100
    procs = [ctx.Process(target=_worker, args=(r, 2, port, n, 16, 5, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    assert all(r[1] and r[2] for r in res), res
