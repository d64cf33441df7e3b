"""Reference schedule of the ring build on CPU (test infrastructure).

The library's ring mode (knng_gpu_brute_force_sharded with mode 1,
knng_gpu_b200/csrc/sharded.cuh) follows the reference's ring
(src/dist/brute_force_mpi.cpp:71-124): in step s rank r searches base block
(r - s) mod P, sends it to rank r + 1 and receives the next from rank r - 1,
and merges the block's k best into its running k best by (distance, id).
This module restates that schedule over torch.distributed point-to-point
calls with injected block-search and merge functions, so that gloo ranks on
CPU can check the schedule itself (including blocks smaller than k) against
the oracle graph. The GPU product does not use it.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from knng_gpu_b200 import api
from knng_gpu_b200.distributed import compute_shard, gather_shards


class RingSchedule:
    """Sharded build that never replicates the base: the reference's ring
    (src/dist/brute_force_mpi.cpp:71-124, one ``MPI_Sendrecv`` right/left per
    step) over NCCL point-to-point.

    Rank r packs its own rows (``compute_shard``) -- they are both its query
    shard and its base block. In step s it holds block b = (r - s) mod P,
    scores its queries against that block (global ids, self excluded by id,
    src/dist/brute_force_mpi.cpp:80-82), merges the block's k best into its
    running k best by (distance, id), and meanwhile already sends the block to
    rank r+1 and receives the next one from rank r-1 (double-buffered, the
    transfer overlaps the kernel). Blocks smaller than k contribute what they
    have, padded with (UINT32_MAX, +inf) like the reference's sentinels
    (src/dist/brute_force_mpi.cpp:136-139). Integer-valued data only (the u8
    path); ``ShardedBuilder`` handles fp32 data.

    ``knn_block(q_packed, q_norms, q_id0, b_packed, b_norms, b_id0, b_count,
    k, exclude_self) -> (ids, dists)`` and ``merge(a_ids, a_d, b_ids, b_d) ->
    (ids, dists)`` default to the GPU kernels; tests inject CPU versions.
    """

    def __init__(self, n: int, d: int, k: int, metric: int, group=None, knn_block=None, merge=None,
                 device=None):
        self.n, self.d, self.k, self.metric = n, d, k, metric
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.shard = compute_shard(n, self.world, self.rank)
        self.max_shard = compute_shard(n, self.world, self.world - 1).count
        self.pitch = api.padded_dim(d) if device is None or device.type == "cuda" else d
        ms = self.max_shard
        self.bufs = [torch.zeros((ms, self.pitch), dtype=torch.uint8, device=self.dev) for _ in range(2)]
        self.nbufs = [torch.zeros(ms, dtype=torch.int32, device=self.dev) for _ in range(2)]
        self.flag = torch.zeros(1, dtype=torch.int32, device=self.dev)
        self.knn_block = knn_block or self._gpu_knn_block
        self.merge = merge or self._gpu_merge
        self._scratch = None

    # -- default GPU implementations
    def _gpu_knn_block(self, q_packed, q_norms, q_id0, b_packed, b_norms, b_id0, b_count, k, exclude_self):
        if self._scratch is None:
            self._scratch = torch.empty(api.knn_scratch_bytes(self.max_shard, self.k), dtype=torch.uint8, device=self.dev)
        ids = torch.empty((q_packed.shape[0], k), dtype=torch.int32, device=self.dev)
        dists = torch.empty((q_packed.shape[0], k), dtype=torch.float32, device=self.dev)
        api.knn_u8_sets(q_packed, q_norms, q_id0, b_packed[:b_count], b_norms[:b_count], b_id0, self.d, k,
                        self.metric, exclude_self, ids, dists, self._scratch)
        return ids, dists

    def _gpu_merge(self, a_ids, a_d, b_ids, b_d):
        o_ids, o_d = torch.empty_like(a_ids), torch.empty_like(a_d)
        api.merge_topk(a_ids, a_d, b_ids, b_d, o_ids, o_d)
        return o_ids, o_d

    def _pad(self, ids, dists):
        k = self.k
        if ids.shape[1] == k:
            return ids, dists
        pad = k - ids.shape[1]
        pi = torch.full((ids.shape[0], pad), -1, dtype=ids.dtype, device=ids.device)  # UINT32_MAX
        pd = torch.full((ids.shape[0], pad), float("inf"), dtype=dists.dtype, device=dists.device)
        return torch.cat([ids, pi], 1), torch.cat([dists, pd], 1)

    def build(self, x_shard: torch.Tensor, gather: bool = True):
        """``x_shard``: this rank's rows (``self.shard``) as float32 on the
        device. Returns (ids, dists) of all n rows (``gather``) or of the
        rank's own query rows."""
        sh = self.shard
        cur = 0
        self.flag.zero_()
        if self.dev.type == "cuda":
            api.pack_u8(x_shard, self.bufs[cur][: sh.count], self.nbufs[cur][: sh.count], self.flag)
        else:  # CPU ranks of the host-logic test: rows are already integers
            self.bufs[cur][: sh.count, : self.d] = x_shard.to(torch.uint8)
            self.nbufs[cur][: sh.count] = (x_shard.to(torch.int64) ** 2).sum(1).to(torch.int32)
        if self.world > 1:
            dist.all_reduce(self.flag, op=dist.ReduceOp.MAX, group=self.group)
        if int(self.flag.item()) != 0:
            raise NotImplementedError("RingBuilder: data is not integer-valued in [0, 255]; use ShardedBuilder")
        q_packed = self.bufs[cur][: sh.count].clone()
        q_norms = self.nbufs[cur][: sh.count].clone()
        best_ids = best_d = None
        right, left = (self.rank + 1) % self.world, (self.rank - 1) % self.world
        for step in range(self.world):
            blk = (self.rank - step) % self.world
            bsh = compute_shard(self.n, self.world, blk)
            reqs = []
            if step + 1 < self.world:
                ops = [dist.P2POp(dist.isend, self.bufs[cur], right, group=self.group),
                       dist.P2POp(dist.irecv, self.bufs[1 - cur], left, group=self.group),
                       dist.P2POp(dist.isend, self.nbufs[cur], right, group=self.group),
                       dist.P2POp(dist.irecv, self.nbufs[1 - cur], left, group=self.group)]
                reqs = dist.batch_isend_irecv(ops)
            own = blk == self.rank
            kb = min(self.k, bsh.count - (1 if own else 0))
            if kb > 0:
                ids, dists = self.knn_block(q_packed, q_norms, sh.start, self.bufs[cur], self.nbufs[cur], bsh.start,
                                            bsh.count, kb, own)
                ids, dists = self._pad(ids, dists)
                best_ids, best_d = (ids, dists) if best_ids is None else self.merge(best_ids, best_d, ids, dists)
            for r in reqs:
                r.wait()
            cur = 1 - cur
        if not gather or self.world == 1:
            return best_ids, best_d
        return gather_shards(best_ids, self.n, self.world, self.group), gather_shards(best_d, self.n, self.world,
                                                                                      self.group)
