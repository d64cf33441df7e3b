"""Host-side mirror of the reference's brute-force API, backed by the C ABI.

The reference's boundary (include/knng/cpu/brute_force.hpp:336-376) is::

    template <Distance D>
    Knng knng::cpu::brute_force_knn(const Dataset& ds, std::size_t k, D d = D{});

This module keeps the same names, argument meaning and error behaviour:
``Dataset`` (include/knng/core/dataset.hpp:76-152), ``Knng``
(include/knng/core/graph.hpp:35-84), the two metrics of
include/knng/core/distance.hpp:86-116, and ``brute_force_knn`` raising
:class:`InvalidArgument` (a ``ValueError``, the analogue of
``std::invalid_argument``) for n == 0, k == 0 and k > n - 1 with the
reference's messages. Everything runs on the GPU through ``libknng_gpu.so``;
there is no CPU path here.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field

import numpy as np

from ._native import KnngGpuStats, gpu_lib

STATUS_NAMES = {
    0: "OK",
    1: "INVALID_ARGUMENT",
    2: "CUDA_ERROR",
    3: "TIMEOUT",
    4: "NOT_SUPPORTED",
    5: "OUT_OF_MEMORY",
    6: "WORKSPACE_TOO_SMALL",
}


class KnngGpuError(RuntimeError):
    """A non-argument failure of the GPU library (CUDA error, timeout, ...)."""

    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


class InvalidArgument(ValueError):
    """Raised where the reference throws std::invalid_argument."""


class L2Squared:
    """knng::L2Squared (distance.hpp:86-95); metric id 0."""

    metric_id = 0


class NegativeInnerProduct:
    """knng::NegativeInnerProduct (distance.hpp:105-116); metric id 1."""

    metric_id = 1


@dataclass
class Dataset:
    """Row-major n x d fp32 feature matrix (knng::Dataset)."""

    n: int = 0
    d: int = 0
    data: np.ndarray = field(default_factory=lambda: np.zeros(0, np.float32))

    @staticmethod
    def from_array(x: np.ndarray) -> "Dataset":
        x = np.ascontiguousarray(x, dtype=np.float32)
        if x.ndim != 2:
            raise InvalidArgument("Dataset.from_array: expected a 2-D array")
        return Dataset(x.shape[0], x.shape[1], x.reshape(-1))

    def row(self, i: int) -> np.ndarray:
        return self.data[i * self.d:(i + 1) * self.d]

    def data_ptr(self) -> int:
        return self.data.ctypes.data

    def is_contiguous(self) -> bool:
        return self.data.size == self.n * self.d


@dataclass
class Knng:
    """Flat (n, k) adjacency: knng::Knng (graph.hpp:35-84)."""

    n: int
    k: int
    neighbors: np.ndarray  # uint32[n*k]
    distances: np.ndarray  # float32[n*k]
    stats: dict | None = None

    def neighbors_of(self, i: int) -> np.ndarray:
        return self.neighbors[i * self.k:(i + 1) * self.k]

    def distances_of(self, i: int) -> np.ndarray:
        return self.distances[i * self.k:(i + 1) * self.k]


def _metric_id(distance) -> int:
    if isinstance(distance, (int, np.integer)):
        return int(distance)
    if isinstance(distance, str):
        return {"l2": 0, "negip": 1}[distance]
    mid = getattr(distance, "metric_id", None)
    if mid is None:
        raise TypeError("brute_force_knn: distance must be L2Squared or NegativeInnerProduct")
    return mid


def _last_error() -> str:
    msg = gpu_lib().knng_gpu_last_error()
    return msg.decode() if msg else ""


def check(status: int) -> None:
    """Raise the Python analogue of the C status (no-op for OK)."""
    if status == 0:
        return
    msg = _last_error()
    if status == 1:
        raise InvalidArgument(msg)
    raise KnngGpuError(status, msg)


def brute_force_knn(ds: Dataset | np.ndarray, k: int, distance=L2Squared()) -> Knng:
    """Exact all-points KNN graph on the GPU; drop-in for knng::cpu::brute_force_knn.

    Rows are sorted ascending by (distance, id); self is excluded by index.
    """
    if isinstance(ds, np.ndarray):
        ds = Dataset.from_array(ds)
    if k < 0:
        raise InvalidArgument("knng::gpu::brute_force_knn: k must be > 0")
    data = np.ascontiguousarray(ds.data, dtype=np.float32)
    n, d = int(ds.n), int(ds.d)
    ids = np.empty(max(n * k, 1), dtype=np.uint32)
    dists = np.empty(max(n * k, 1), dtype=np.float32)
    stats = KnngGpuStats()
    st = gpu_lib().knng_gpu_brute_force(
        data.ctypes.data if data.size else None, n, d, k, _metric_id(distance),
        ids.ctypes.data, dists.ctypes.data, ctypes.byref(stats))
    check(st)
    return Knng(n, k, ids[: n * k], dists[: n * k], stats.as_dict())


def brute_force_knn_u8(rows: np.ndarray, k: int, distance=L2Squared(), d: int | None = None) -> Knng:
    """As :func:`brute_force_knn` for rows that are already bytes (u8 path
    without the fp32 round trip). ``rows``: a contiguous uint8 array of shape
    (n, d), or of shape (n, stride) with the values in the first ``d`` bytes
    of each row (e.g. a .bvecs payload viewed as (n, d + 4) after its first
    4-byte header). Same output as :func:`brute_force_knn` on the same values."""
    rows = np.ascontiguousarray(rows, dtype=np.uint8)
    if rows.ndim != 2:
        raise InvalidArgument("brute_force_knn_u8: rows must be 2-D")
    n, stride = int(rows.shape[0]), int(rows.shape[1])
    d = stride if d is None else int(d)
    if k < 0:
        raise InvalidArgument("knng::gpu::brute_force_knn: k must be > 0")
    ids = np.empty(max(n * k, 1), dtype=np.uint32)
    dists = np.empty(max(n * k, 1), dtype=np.float32)
    stats = KnngGpuStats()
    check(gpu_lib().knng_gpu_brute_force_u8(rows.ctypes.data if rows.size else None, n, d, stride, k,
                                            _metric_id(distance), ids.ctypes.data, dists.ctypes.data,
                                            ctypes.byref(stats)))
    return Knng(n, k, ids[: n * k], dists[: n * k], stats.as_dict())


def brute_force_knn_multi(ds: Dataset | np.ndarray, k: int, distance=L2Squared(), num_gpus: int = 1,
                          ring: bool = False) -> Knng:
    """:func:`brute_force_knn` on ``num_gpus`` GPUs of this process (devices
    0..num_gpus-1, NCCL between them): query rows sharded like the reference's
    distributed build, the base all-gathered (or ring-passed with ``ring``),
    the graph gathered on GPU 0. Same output as :func:`brute_force_knn`."""
    if isinstance(ds, np.ndarray):
        ds = Dataset.from_array(ds)
    if k < 0:
        raise InvalidArgument("knng::gpu::brute_force_knn: k must be > 0")
    data = np.ascontiguousarray(ds.data, dtype=np.float32)
    n, d = int(ds.n), int(ds.d)
    ids = np.empty(max(n * k, 1), dtype=np.uint32)
    dists = np.empty(max(n * k, 1), dtype=np.float32)
    stats = KnngGpuStats()
    check(gpu_lib().knng_gpu_brute_force_multi(
        data.ctypes.data if data.size else None, n, d, k, _metric_id(distance), num_gpus, 1 if ring else 0,
        ids.ctypes.data, dists.ctypes.data, ctypes.byref(stats)))
    return Knng(n, k, ids[: n * k], dists[: n * k], stats.as_dict())


# ---------------------------------------------------------------- device API
def _ptr(t) -> int | None:
    return None if t is None else int(t.data_ptr())


def _stream_handle(stream) -> int | None:
    if stream is None:
        import torch

        stream = torch.cuda.current_stream()
    return int(stream.cuda_stream)


def workspace_bytes(n: int, d: int, k: int) -> int:
    return int(gpu_lib().knng_gpu_workspace_bytes(n, d, k))


def brute_force_knn_device(x, k: int, distance=L2Squared(), out_ids=None, out_dists=None, workspace=None,
                           stream=None):
    """Device-resident build: ``x`` is a CUDA float32 (n, d) torch tensor.

    Returns ``(ids, dists, stats)`` as CUDA tensors of shape (n, k) and a
    dict of device timings. ``workspace`` (uint8 CUDA tensor of at least
    :func:`workspace_bytes` (n, d, k) bytes) is allocated here when not given.
    """
    import torch

    if x.dim() != 2 or x.dtype != torch.float32 or not x.is_cuda or not x.is_contiguous():
        raise InvalidArgument("brute_force_knn_device: x must be a contiguous CUDA float32 (n, d) tensor")
    n, d = x.shape
    dev = x.device
    if out_ids is None:
        out_ids = torch.empty((n, max(k, 0)), dtype=torch.int32, device=dev)
    if out_dists is None:
        out_dists = torch.empty((n, max(k, 0)), dtype=torch.float32, device=dev)
    wsb = workspace_bytes(n, d, k)
    if workspace is None:
        workspace = torch.empty(wsb, dtype=torch.uint8, device=dev)
    stats = KnngGpuStats()
    st = gpu_lib().knng_gpu_brute_force_device(
        _ptr(x), n, d, k, _metric_id(distance), _ptr(out_ids), _ptr(out_dists), _ptr(workspace),
        workspace.numel(), _stream_handle(stream), ctypes.byref(stats))
    check(st)
    return out_ids, out_dists, stats.as_dict()


def padded_dim(d: int) -> int:
    return int(gpu_lib().knng_gpu_padded_dim(d))


def pack_u8(x, packed, norms, nonint_flag, stream=None) -> None:
    """u8 pack + integer check + row norms of a CUDA float32 (rows, d) tensor."""
    rows, d = x.shape
    check(gpu_lib().knng_gpu_pack_u8(_ptr(x), rows, d, _ptr(packed), _ptr(norms), _ptr(nonint_flag),
                                     _stream_handle(stream)))


def pack_u8_bytes(rows, packed, norms, d: int | None = None, stream=None) -> None:
    """u8 pack + key offsets of a CUDA uint8 (rows, stride) tensor whose first
    ``d`` bytes per row are the values (no fp32 round trip)."""
    n, stride = rows.shape
    d = stride if d is None else d
    check(gpu_lib().knng_gpu_pack_u8_bytes(_ptr(rows), n, d, stride, _ptr(packed), _ptr(norms),
                                           _stream_handle(stream)))


def knn_scratch_bytes(q_count: int, k: int) -> int:
    return int(gpu_lib().knng_gpu_knn_scratch_bytes(q_count, k))


def knn_u8(packed, norms, n: int, d: int, q_begin: int, q_count: int, k: int, distance, out_ids, out_dists,
           scratch, stream=None) -> dict:
    """Fused tensor-core KNN of packed query rows [q_begin, q_begin+q_count) against all n rows."""
    stats = KnngGpuStats()
    check(gpu_lib().knng_gpu_knn_u8(_ptr(packed), _ptr(norms), n, d, q_begin, q_count, k, _metric_id(distance),
                                    _ptr(out_ids), _ptr(out_dists), _ptr(scratch), scratch.numel(),
                                    _stream_handle(stream), ctypes.byref(stats)))
    return stats.as_dict()


def knn_u8_sets(q_packed, q_norms, q_id0: int, b_packed, b_norms, b_id0: int, d: int, k: int, distance,
                exclude_self: bool, out_ids, out_dists, scratch, stream=None) -> dict:
    """Fused KNN of packed query rows against a separate packed base (global ids)."""
    stats = KnngGpuStats()
    check(gpu_lib().knng_gpu_knn_u8_sets(_ptr(q_packed), _ptr(q_norms), q_packed.shape[0], q_id0, _ptr(b_packed),
                                         _ptr(b_norms), b_packed.shape[0], b_id0, d, k, _metric_id(distance),
                                         int(exclude_self), _ptr(out_ids), _ptr(out_dists), _ptr(scratch),
                                         scratch.numel(), _stream_handle(stream), ctypes.byref(stats)))
    return stats.as_dict()


def merge_topk(a_ids, a_dists, b_ids, b_dists, out_ids, out_dists, stream=None) -> None:
    """Row-wise merge of two sorted (rows, k) lists into the k best by (distance, id)."""
    rows, k = a_ids.shape
    check(gpu_lib().knng_gpu_merge_topk(_ptr(a_ids), _ptr(a_dists), _ptr(b_ids), _ptr(b_dists), rows, k,
                                        _ptr(out_ids), _ptr(out_dists), _stream_handle(stream)))


def knn_f32_scratch_bytes(n: int, d: int, q_count: int, k: int) -> int:
    return int(gpu_lib().knng_gpu_knn_f32_scratch_bytes(n, d, q_count, k))


def knn_f32(x, n: int, d: int, q_begin: int, q_count: int, k: int, distance, out_ids, out_dists, scratch,
            stream=None) -> dict:
    """KNN of fp32 rows [q_begin, q_begin+q_count) of x against all n rows
    (tensor-core candidate filter, exact re-rank, exact fallback)."""
    stats = KnngGpuStats()
    check(gpu_lib().knng_gpu_knn_f32(_ptr(x), n, d, q_begin, q_count, k, _metric_id(distance), _ptr(out_ids),
                                     _ptr(out_dists), _ptr(scratch), scratch.numel(), _stream_handle(stream),
                                     ctypes.byref(stats)))
    return stats.as_dict()


def knn_f32_sets_scratch_bytes(n_q: int, n_b: int, d: int, k: int, exclude_self: bool = False) -> int:
    return int(gpu_lib().knng_gpu_knn_f32_sets_scratch_bytes(n_q, n_b, d, k, int(exclude_self)))


def knn_f32_sets(q, q_id0: int, b, b_id0: int, k: int, distance, exclude_self: bool, out_ids, out_dists,
                 scratch=None, stream=None) -> dict:
    """Exact KNN of fp32 query rows ``q`` (CUDA (n_q, d)) against separate fp32
    base rows ``b`` (CUDA (n_b, d)) with global ids; the fp32 path of
    :func:`knn_f32` for two sets."""
    import torch

    n_q, d = q.shape
    n_b = b.shape[0]
    if scratch is None:
        scratch = torch.empty(knn_f32_sets_scratch_bytes(n_q, n_b, d, k, exclude_self), dtype=torch.uint8,
                              device=q.device)
    stats = KnngGpuStats()
    check(gpu_lib().knng_gpu_knn_f32_sets(_ptr(q), n_q, q_id0, _ptr(b), n_b, b_id0, d, k, _metric_id(distance),
                                          int(exclude_self), _ptr(out_ids), _ptr(out_dists), _ptr(scratch),
                                          scratch.numel(), _stream_handle(stream), ctypes.byref(stats)))
    return stats.as_dict()


def recall_at_k(approx_ids, truth_ids, stream=None) -> float:
    """knng::bench::recall_at_k (src/bench/recall.cpp:79-96) on the GPU: both
    arguments are CUDA (n, k) id tensors; a repeated approximate id counts once."""
    import torch

    if approx_ids.shape != truth_ids.shape:
        raise InvalidArgument("knng::bench::recall: approx and truth shapes differ")
    n, k = approx_ids.shape
    counter = torch.empty(1, dtype=torch.int64, device=approx_ids.device)
    out = ctypes.c_double()
    check(gpu_lib().knng_gpu_recall_at_k(_ptr(approx_ids.contiguous()), _ptr(truth_ids.contiguous()), n, k,
                                         _ptr(counter), _stream_handle(stream), ctypes.byref(out)))
    return float(out.value)


def device_count() -> int:
    return int(gpu_lib().knng_gpu_device_count())
