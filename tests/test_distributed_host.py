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
    assert slice_rows(10, 4) == 256 and slice_rows(1000, 2) == 512 and slice_rows(1_000_000, 8) == 125_184


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


def _ring_worker(rank, world, port, n, d, k, metric, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import sys
        sys.path.insert(0, os.path.dirname(__file__))
        from refs import oracle_knn
        from knng_gpu_b200 import synthetic as syn
        from ring_reference import RingSchedule

        x = syn.generate(syn.KIND_UNIFORM_INT, 91, n, d)

        def knn_block(q_packed, q_norms, q_id0, b_packed, b_norms, b_id0, b_count, kk, exclude_self):
            # exact integer distances, ordered by (distance, id) like knng::TopK
            qv = q_packed[:, :d].to(torch.int64)
            bv = b_packed[:b_count, :d].to(torch.int64)
            if metric == 0:
                dd = ((qv[:, None, :] - bv[None, :, :]) ** 2).sum(-1)
            else:
                dd = -(qv @ bv.T)
            gid = torch.arange(b_count, dtype=torch.int64) + b_id0
            if exclude_self:
                qid = torch.arange(qv.shape[0], dtype=torch.int64) + q_id0
                dd = torch.where(gid[None, :] == qid[:, None], torch.iinfo(torch.int64).max, dd)
            order = torch.from_numpy(np.lexsort((np.broadcast_to(gid.numpy(), dd.shape), dd.numpy()), axis=1))
            sel = order[:, :kk]
            return (gid[sel].to(torch.int32), torch.gather(dd, 1, sel).to(torch.float32))

        def merge(a_ids, a_d, b_ids, b_d):
            ids = torch.cat([a_ids, b_ids], 1).numpy().view(np.uint32).astype(np.int64)
            ds = torch.cat([a_d, b_d], 1).numpy()
            order = np.lexsort((ids, ds), axis=1)[:, :k]
            return (torch.from_numpy(np.take_along_axis(ids, order, 1).astype(np.uint32).view(np.int32)),
                    torch.from_numpy(np.take_along_axis(ds, order, 1)))

        rb = RingSchedule(n, d, k, metric, knn_block=knn_block, merge=merge, device=torch.device("cpu"))
        sh = rb.shard
        ids, dists = rb.build(torch.from_numpy(x[sh.start:sh.start + sh.count]))
        full_ids, full_d = oracle_knn(x, k, metric)
        q.put((rank, bool(np.array_equal(ids.numpy().view(np.uint32), full_ids)),
               bool(np.array_equal(dists.numpy(), full_d))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,n,k,metric", [(2, 101, 5, 0), (3, 64, 7, 1), (3, 20, 9, 0)])
def test_ring_schedule_reassembles_the_graph(world, n, k, metric):
    """The ring schedule (send right, receive left, merge per block) gives the
    single-process oracle graph, including blocks smaller than k."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29700 + n + world
    procs = [ctx.Process(target=_ring_worker, args=(r, world, port, n, 8, k, metric, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=180) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    assert all(r[1] and r[2] for r in res), res
