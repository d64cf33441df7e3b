"""Sharded multi-GPU build, one process per GPU: a thin Python layer over the
C-ABI sharded build (knng_gpu_brute_force_sharded, include/knng_gpu.h).

The library owns the NCCL communicator of each rank and every exchange step
(all-reduce of the integer flag, all-gather of the packed base or the ring
pass of base blocks, gather of graph rows to rank 0). torch.distributed only
hands the NCCL unique id from rank 0 to the other ranks.

Mirrors the reference's distributed brute force (src/dist/brute_force_mpi.cpp:36-203,
include/knng/dist/sharded_dataset.hpp:145-155):

* query rows are sharded by ``compute_shard`` (contiguous blocks, the last
  rank takes the remainder);
* mode 0 replicates the packed base on every GPU (all-gather); mode 1 keeps
  it sharded and passes the blocks around a ring while the kernel searches the
  current block (the reference's ring of MPI_Sendrecv);
* rank 0 receives the whole graph.
"""
from __future__ import annotations

import ctypes
import time
from dataclasses import dataclass

import torch
import torch.distributed as dist

from . import api
from ._native import KnngGpuStats, gpu_lib


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
    """Rows per rank in the replicate mode's equal slices (packed and
    all-gathered): ceil(n / ranks) rounded up to SLICE_ALIGN rows, so every
    slice starts on a base tile of the fused kernel. Trailing ranks may get an
    empty slice when n is small. Same rule as the library's."""
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


class NcclComm:
    """This rank's communicator inside the library (knng_gpu_comm_create).
    The unique id travels from rank 0 over the default torch.distributed
    group; create it with the rank's GPU current."""

    def __init__(self, group=None):
        lib = gpu_lib()
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        nbytes = int(lib.knng_gpu_nccl_id_bytes())
        idbuf = (ctypes.c_uint8 * nbytes)()
        if self.rank == 0:
            api.check(lib.knng_gpu_nccl_unique_id(idbuf))
        dev = torch.device("cuda", torch.cuda.current_device())
        t = torch.tensor(list(bytes(idbuf)), dtype=torch.uint8, device=dev)
        dist.broadcast(t, src=dist.get_global_rank(group, 0) if group is not None else 0, group=group)
        idbytes = bytes(t.cpu().tolist())
        ctypes.memmove(idbuf, idbytes, nbytes)
        handle = ctypes.c_void_p()
        api.check(lib.knng_gpu_comm_create(idbuf, self.world, self.rank, ctypes.byref(handle)))
        self.handle = handle

    def close(self) -> None:
        if self.handle:
            gpu_lib().knng_gpu_comm_destroy(self.handle)
            self.handle = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


MODE_REPLICATE = 0
MODE_RING = 1


class ShardedBuilder:
    """Repeated sharded builds of an (n, d) dataset with k neighbours on this
    rank's GPU, through the C ABI. ``mode``: MODE_REPLICATE (base all-gathered)
    or MODE_RING (base blocks passed around the ring; integer data only).
    ``build`` takes this rank's rows ``slice_bounds`` as CUDA float32 and
    returns the (n, k) graph on rank 0, (None, None) on the other ranks."""

    def __init__(self, n: int, d: int, k: int, metric: int, mode: int = MODE_REPLICATE, group=None):
        self.n, self.d, self.k, self.metric, self.mode = n, d, k, metric, mode
        self.comm = NcclComm(group)
        self.world, self.rank = self.comm.world, self.comm.rank
        self.dev = torch.device("cuda", torch.cuda.current_device())
        lib = gpu_lib()
        b, c = ctypes.c_uint64(), ctypes.c_uint64()
        lib.knng_gpu_shard_rows(n, self.world, self.rank, mode, ctypes.byref(b), ctypes.byref(c))
        self._slice = (int(b.value), int(b.value) + int(c.value))
        self.shard = compute_shard(n, self.world, self.rank)
        self.ws = torch.empty(int(lib.knng_gpu_sharded_workspace_bytes(n, d, k, self.world, mode)),
                              dtype=torch.uint8, device=self.dev)
        if self.rank == 0:
            self.ids = torch.empty((n, k), dtype=torch.int32, device=self.dev)
            self.dists = torch.empty((n, k), dtype=torch.float32, device=self.dev)
        else:
            self.ids = self.dists = None
        self.last_stats: dict = {}

    @property
    def slice_bounds(self) -> tuple[int, int]:
        return self._slice

    def describe(self) -> str:
        how = "base all-gathered" if self.mode == MODE_REPLICATE else "base blocks ring-passed"
        return f"query-shard x{self.world}, {how}, graph rows gathered to rank 0 (NCCL inside the C ABI)"

    def build(self, x_rows: torch.Tensor, stream=None):
        lo, hi = self._slice
        if tuple(x_rows.shape) != (hi - lo, self.d) or x_rows.dtype != torch.float32 or not x_rows.is_contiguous():
            raise api.InvalidArgument("ShardedBuilder.build: expected this rank's contiguous float32 rows")
        stats = KnngGpuStats()
        api.check(gpu_lib().knng_gpu_brute_force_sharded(
            x_rows.data_ptr() if x_rows.numel() else None, self.n, self.d, self.k, self.metric, self.mode,
            self.comm.handle, None if self.ids is None else self.ids.data_ptr(),
            None if self.dists is None else self.dists.data_ptr(), self.ws.data_ptr(), self.ws.numel(),
            api._stream_handle(stream), ctypes.byref(stats)))
        self.last_stats = stats.as_dict()
        return self.ids, self.dists

    def last_phase_ms(self) -> dict:
        out = (ctypes.c_float * 6)()
        api.check(gpu_lib().knng_gpu_comm_phase_ms(self.comm.handle, out))
        names = ("pack", "exchange_base", "search", "fp32_exchange_search", "gather_rows", "total")
        return dict(zip(names, [float(v) for v in out]))

    def time_e2e(self, x_host: torch.Tensor, steps: int, warmup: int) -> dict:
        """Each step: pinned host rows of this rank -> device, the sharded
        build, and on rank 0 the graph -> pinned host memory. Max over ranks."""
        out_ids = out_d = None
        if self.rank == 0:
            out_ids = torch.empty((self.n, self.k), dtype=torch.int32).pin_memory()
            out_d = torch.empty((self.n, self.k), dtype=torch.float32).pin_memory()

        def step():
            xs = x_host.to(self.dev, non_blocking=True)
            ids, dd = self.build(xs)
            if self.rank == 0:
                out_ids.copy_(ids, non_blocking=True)
                out_d.copy_(dd, non_blocking=True)
            torch.cuda.synchronize()

        for _ in range(warmup):
            step()
        dist.barrier()
        t0 = time.perf_counter()
        for _ in range(steps):
            step()
        t = torch.tensor([(time.perf_counter() - t0) / steps], device=self.dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return {"seconds_per_build": float(t.item()), "h2d_bytes_per_step": self.n * self.d * 4,
                "d2h_bytes_per_step": self.n * self.k * 8,
                "api": "knng_gpu_brute_force_sharded (C ABI): pinned H2D of each rank's rows, build, "
                       "rank 0 graph D2H"}


class SingleBuilder:
    """One GPU, no collective: the device-resident C-ABI build
    (knng_gpu_brute_force_device) with a workspace kept between builds. Same
    interface as ShardedBuilder."""

    def __init__(self, n: int, d: int, k: int, metric: int):
        self.n, self.d, self.k, self.metric = n, d, k, metric
        self.world, self.rank = 1, 0
        self.dev = torch.device("cuda", torch.cuda.current_device())
        self.shard = ShardBounds(0, n)
        self.ids = torch.empty((n, k), dtype=torch.int32, device=self.dev)
        self.dists = torch.empty((n, k), dtype=torch.float32, device=self.dev)
        self.ws = torch.empty(api.workspace_bytes(n, d, k), dtype=torch.uint8, device=self.dev)
        self.last_stats: dict = {}

    @property
    def slice_bounds(self) -> tuple[int, int]:
        return 0, self.n

    def describe(self) -> str:
        return "one GPU (knng_gpu_brute_force_device)"

    def build(self, x: torch.Tensor, stream=None):
        _, _, self.last_stats = api.brute_force_knn_device(x, self.k, self.metric, self.ids, self.dists, self.ws,
                                                           stream)
        return self.ids, self.dists

    def last_phase_ms(self) -> dict:
        s = self.last_stats
        return {"pack": s.get("pack_ms"), "knn": s.get("knn_ms"), "tensor_kernel": s.get("tc_ms"),
                "total": s.get("total_ms")}

    def time_e2e(self, x_host: torch.Tensor, steps: int, warmup: int) -> dict:
        """Public host API (knng_gpu_brute_force): host rows in, host graph out."""
        xnp = x_host.numpy()
        for _ in range(warmup):
            api.brute_force_knn(xnp, self.k, self.metric)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(steps):
            api.brute_force_knn(xnp, self.k, self.metric)
        sec = (time.perf_counter() - t0) / steps
        return {"seconds_per_build": sec, "h2d_bytes_per_step": self.n * self.d * 4,
                "d2h_bytes_per_step": self.n * self.k * 8, "api": "knng_gpu_brute_force (C ABI, host buffers)"}


def make_builder(n: int, d: int, k: int, metric: int, ring: bool = False):
    """The builder for this process: one GPU without torch.distributed, else
    the sharded builder (base replicated, or ring-passed with ``ring``)."""
    world = dist.get_world_size() if dist.is_initialized() else 1
    if world == 1:
        return SingleBuilder(n, d, k, metric)
    return ShardedBuilder(n, d, k, metric, MODE_RING if ring else MODE_REPLICATE)
