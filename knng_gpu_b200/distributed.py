"""Sharded multi-GPU build: one process per GPU, torch.distributed (NCCL) for
the exchange steps, the C-ABI kernels for the compute.

Mirrors the reference's distributed brute force (src/dist/brute_force_mpi.cpp:36-142,
include/knng/dist/sharded_dataset.hpp:145-155) with the base replicated
instead of ring-passed:

1. every rank packs its slice of rows (u8 + norms + integer check) -- the
   ``MPI_Scatterv`` of src/dist/sharded_dataset.cpp:72 becomes a local H2D
   of the rank's slice;
2. ``all_reduce(MAX)`` of the "not integer" flag, then ``all_gather`` of the
   packed slices so every GPU holds the full packed base (128 MB for 1M x 128);
3. every rank runs the fused kernel on its query shard (``compute_shard``:
   contiguous blocks, the last rank takes the remainder) against the full base;
4. the Knng rows are gathered to rank 0 -- the two ``MPI_Gatherv`` of
   src/dist/brute_force_mpi.cpp:179-200 -- as one ``all_gather`` of padded
   equal shards (NCCL has no Gatherv).

Non-integer data takes the same steps with fp32 rows and the exact kernel.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

from . import api


@dataclass(frozen=True)
class ShardBounds:
    start: int
    count: int


def compute_shard(global_n: int, num_ranks: int, rank: int) -> ShardBounds:
    """Contiguous query shard of ``rank``: include/knng/dist/sharded_dataset.hpp:145-155."""
    base = global_n // num_ranks
    rem = global_n % num_ranks
    return ShardBounds(rank * base, base + (rem if rank == num_ranks - 1 else 0))


SLICE_ALIGN = 256


def slice_rows(global_n: int, num_ranks: int) -> int:
    """Rows per rank in the equal-size slices that are packed and all-gathered:
    ceil(n / ranks) rounded up to SLICE_ALIGN rows, so every slice starts on a
    base-tile boundary of the fused kernel (the pack derives each 128-row
    tile's augmentation offset from that tile alone; tiles that straddle two
    packs stay exact but filter less sharply). Trailing ranks may get an empty
    slice when n is small."""
    per = (global_n + num_ranks - 1) // num_ranks
    return (per + SLICE_ALIGN - 1) // SLICE_ALIGN * SLICE_ALIGN


def gather_shards(local: torch.Tensor, n: int, world: int, group=None) -> torch.Tensor:
    """All-gather each rank's ``compute_shard`` rows (padded to the largest
    shard so the collective has equal chunks) and return the (n, ...) rows
    in global order on every rank."""
    max_shard = compute_shard(n, world, world - 1).count
    if local.shape[0] != max_shard:
        pad = torch.zeros((max_shard - local.shape[0],) + tuple(local.shape[1:]), dtype=local.dtype,
                          device=local.device)
        local = torch.cat([local, pad], 0)
    out = torch.empty((world * max_shard,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(out, local.contiguous(), group=group)
    return unpad_shards(out, n, world)


def unpad_shards(t: torch.Tensor, n: int, world: int) -> torch.Tensor:
    """Drop the padding rows of a gathered (world * max_shard, ...) tensor."""
    max_shard = compute_shard(n, world, world - 1).count
    parts = [t[r * max_shard: r * max_shard + compute_shard(n, world, r).count] for r in range(world)]
    return torch.cat(parts, 0)


class ShardedBuilder:
    """Reusable buffers for repeated sharded builds of an (n, d) dataset with k
    neighbours on this rank's GPU. All collectives run on the current stream."""

    def __init__(self, n: int, d: int, k: int, metric: int, group=None):
        self.n, self.d, self.k, self.metric = n, d, k, metric
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        dev = torch.device("cuda", torch.cuda.current_device())
        self.dev = dev
        self.s = slice_rows(n, self.world)
        self.pitch = api.padded_dim(d)
        self.packed = torch.empty((self.world * self.s, self.pitch), dtype=torch.uint8, device=dev)
        self.norms = torch.empty((self.world * self.s,), dtype=torch.int32, device=dev)
        self.flag = torch.zeros((1,), dtype=torch.int32, device=dev)
        self.shard = compute_shard(n, self.world, self.rank)
        self.max_shard = compute_shard(n, self.world, self.world - 1).count
        self.ids = torch.empty((self.max_shard, k), dtype=torch.int32, device=dev)
        self.dists = torch.empty((self.max_shard, k), dtype=torch.float32, device=dev)
        self.scratch = torch.empty(api.knn_scratch_bytes(self.max_shard), dtype=torch.uint8, device=dev)
        self.all_ids = torch.empty((self.world * self.max_shard, k), dtype=torch.int32, device=dev)
        self.all_dists = torch.empty((self.world * self.max_shard, k), dtype=torch.float32, device=dev)
        self.f32_full = None
        self.f32_scratch = None
        # Optional per-phase device timing (set .timing = True): CUDA events on
        # the current stream; phase_ms() reads them after a build.
        self.timing = False
        self._marks: list = []
        self.last_stats: dict = {}

    @property
    def slice_bounds(self) -> tuple[int, int]:
        lo = min(self.rank * self.s, self.n)
        return lo, min(lo + self.s, self.n)

    def build(self, x_slice: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """``x_slice``: this rank's rows ``slice_bounds`` as CUDA float32.
        Returns (ids, dists) of shape (n, k) on every rank (valid on all)."""
        lo, hi = self.slice_bounds
        assert x_slice.shape == (hi - lo, self.d)
        self._marks = []
        self._mark("start")
        self.flag.zero_()
        api.pack_u8(x_slice, self.packed[lo:hi], self.norms[lo:hi], self.flag)
        self._mark("pack")
        if self.world > 1:
            dist.all_reduce(self.flag, op=dist.ReduceOp.MAX, group=self.group)
            dist.all_gather_into_tensor(self.packed, self.packed[self.rank * self.s:(self.rank + 1) * self.s],
                                        group=self.group)
            dist.all_gather_into_tensor(self.norms, self.norms[self.rank * self.s:(self.rank + 1) * self.s],
                                        group=self.group)
        self._mark("exchange_base")
        # The flag decides the kernel family: one host read per build.
        integer = int(self.flag.item()) == 0
        self._mark("flag_read")
        sh = self.shard
        ids = self.ids[: sh.count]
        dists = self.dists[: sh.count]
        if integer:
            self.last_stats = api.knn_u8(self.packed, self.norms, self.n, self.d, sh.start, sh.count, self.k,
                                         self.metric, ids, dists, self.scratch)
        else:
            if self.f32_full is None:
                self.f32_full = torch.empty((self.world * self.s, self.d), dtype=torch.float32, device=self.dev)
            self.f32_full[lo:hi].copy_(x_slice)
            if self.world > 1:
                dist.all_gather_into_tensor(self.f32_full,
                                            self.f32_full[self.rank * self.s:(self.rank + 1) * self.s],
                                            group=self.group)
            if self.f32_scratch is None:
                nb = api.knn_f32_scratch_bytes(self.n, self.d, self.max_shard, self.k)
                self.f32_scratch = torch.empty(nb, dtype=torch.uint8, device=self.dev)
            self.last_stats = api.knn_f32(self.f32_full, self.n, self.d, sh.start, sh.count, self.k, self.metric,
                                          ids, dists, self.f32_scratch)
        self._mark("knn")
        if self.world == 1:
            return ids, dists
        dist.all_gather_into_tensor(self.all_ids, self.ids, group=self.group)
        dist.all_gather_into_tensor(self.all_dists, self.dists, group=self.group)
        out = self._unpad(self.all_ids), self._unpad(self.all_dists)
        self._mark("gather_rows")
        return out

    def _mark(self, name: str) -> None:
        if self.timing:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            self._marks.append((name, ev))

    def phase_ms(self) -> dict:
        """Device time of each phase of the last build (needs .timing)."""
        torch.cuda.synchronize()
        return {b[0]: a[1].elapsed_time(b[1]) for a, b in zip(self._marks, self._marks[1:])}

    def _unpad(self, t: torch.Tensor) -> torch.Tensor:
        return unpad_shards(t, self.n, self.world)


class RingBuilder:
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
            self._scratch = torch.empty(api.knn_scratch_bytes(self.max_shard), dtype=torch.uint8, device=self.dev)
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
