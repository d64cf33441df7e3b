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


def slice_rows(global_n: int, num_ranks: int) -> int:
    """Rows per rank in the equal-size slices that are packed and all-gathered."""
    return (global_n + num_ranks - 1) // num_ranks


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
