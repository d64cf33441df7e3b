"""File formats around the brute-force path (numpy; no reference code).

* ``read_vecs`` / ``write_vecs``: .fvecs / .ivecs / .bvecs records
  (include/knng/io/fvecs.hpp:9-30): per record an int32 dim then the
  elements; n from the file size; every dim must match the first.
* ``write_knng`` / ``read_knng``: .knng v1 graph files
  (tools/build_knng.cpp:13-33).
* ``save_ground_truth`` / ``load_ground_truth``: the ground-truth cache
  (src/bench/ground_truth.cpp:36-40, 103-234), keyed by ``dataset_hash``
  (FNV-1a 64 over n, d and the fp32 payload, :45-56 and :90-101).
* ``load_or_compute_ground_truth``: cache hit or a GPU build
  (src/bench/ground_truth.cpp:236-256 with the GPU builder in place of
  compute_ground_truth, :74-86).
* ``recall_at_k``: mean per-row share of truth ids found, duplicates in the
  approximate row counted once (src/bench/recall.cpp:52-96).
"""
from __future__ import annotations

import ctypes
import os
import struct
from pathlib import Path

import numpy as np

from ._native import synth_lib

_DTYPES = {".fvecs": np.float32, ".ivecs": np.int32, ".bvecs": np.uint8}

KNNG_MAGIC = b"KNNGRAPH"
GT_MAGIC = b"KNNGRDTR"
ALGORITHM_BRUTE_FORCE = 0
ALGORITHM_BRUTE_FORCE_GPU = 1


def _dtype_for(path, dtype=None):
    if dtype is not None:
        return np.dtype(dtype)
    suffix = Path(path).suffix
    if suffix not in _DTYPES:
        raise ValueError(f"knng::io: unknown vecs suffix '{suffix}'")
    return np.dtype(_DTYPES[suffix])


def read_vecs(path, dtype=None) -> np.ndarray:
    """Rows of a *vecs file as an (n, d) array (errors like load_fvecs)."""
    dt = _dtype_for(path, dtype)
    raw = np.fromfile(path, dtype=np.uint8)
    if raw.size < 4:
        raise RuntimeError(f"knng::io: file too small to hold a single record: '{path}'")
    dim = int(raw[:4].view(np.int32)[0])
    if dim <= 0:
        raise RuntimeError(f"knng::io: invalid dim prefix {dim} in '{path}'")
    rec = 4 + dim * dt.itemsize
    if raw.size % rec:
        raise RuntimeError(f"knng::io: file size {raw.size} is not a multiple of record size {rec} for '{path}'")
    recs = raw.reshape(-1, rec)
    dims = recs[:, :4].copy().view(np.int32)[:, 0]
    bad = np.nonzero(dims != dim)[0]
    if bad.size:
        i = int(bad[0])
        raise RuntimeError(f"knng::io: record {i} has dim {int(dims[i])} but the first record has dim {dim} "
                           f"in '{path}'")
    return np.ascontiguousarray(recs[:, 4:]).view(dt).reshape(-1, dim)


def write_vecs(path, x: np.ndarray, dtype=None) -> None:
    dt = _dtype_for(path, dtype)
    x = np.ascontiguousarray(x, dtype=dt)
    n, d = x.shape
    rec = np.empty((n, 4 + d * dt.itemsize), np.uint8)
    rec[:, :4] = np.frombuffer(struct.pack("<i", d), np.uint8)
    rec[:, 4:] = x.view(np.uint8).reshape(n, -1)
    rec.tofile(path)


def write_knng(path, ids: np.ndarray, dists: np.ndarray, metric: int,
               algorithm: int = ALGORITHM_BRUTE_FORCE_GPU) -> None:
    ids = np.ascontiguousarray(ids, np.uint32)
    dists = np.ascontiguousarray(dists, np.float32)
    n, k = ids.shape
    hdr = KNNG_MAGIC + struct.pack("<IIIIIQQ", 1, 4, 4, metric, algorithm, n, k) + bytes(20)
    with open(path, "wb") as f:
        f.write(hdr)
        f.write(ids.tobytes())
        f.write(dists.tobytes())


def read_knng(path):
    """Returns (ids[n, k], dists[n, k], metric, algorithm)."""
    with open(path, "rb") as f:
        hdr = f.read(64)
        if len(hdr) != 64 or hdr[:8] != KNNG_MAGIC:
            raise RuntimeError(f"not a .knng v1 file: '{path}'")
        version, iw, dw, metric, algorithm, n, k = struct.unpack("<IIIIIQQ", hdr[8:44])
        if version != 1 or iw != 4 or dw != 4:
            raise RuntimeError(f"unsupported .knng header in '{path}'")
        ids = np.frombuffer(f.read(n * k * 4), np.uint32).reshape(n, k)
        dists = np.frombuffer(f.read(n * k * 4), np.float32).reshape(n, k)
    return ids, dists, metric, algorithm


def dataset_hash(x: np.ndarray) -> int:
    """FNV-1a 64 of (u64 n, u64 d, fp32 payload), in C."""
    x = np.ascontiguousarray(x, np.float32)
    n, d = x.shape
    lib = synth_lib()
    return int(lib.knng_dataset_hash(x.ctypes.data if x.size else None, n, d))


def save_ground_truth(path, ids: np.ndarray, dists: np.ndarray, data_hash: int, metric: int) -> None:
    ids = np.ascontiguousarray(ids, np.uint32)
    dists = np.ascontiguousarray(dists, np.float32)
    n, k = ids.shape
    hdr = GT_MAGIC + struct.pack("<IIIIQQQ", 1, 4, 4, metric, data_hash, n, k) + bytes(16)
    tmp = str(path) + ".tmp"
    with open(tmp, "wb") as f:
        f.write(hdr)
        f.write(ids.tobytes())
        f.write(dists.tobytes())
    os.replace(tmp, path)


def load_ground_truth(path, x: np.ndarray, k: int, metric: int):
    """(ids, dists) when the cache matches (magic, version, widths, metric,
    dataset hash, n, k, exact length), else None -- as load_ground_truth."""
    try:
        with open(path, "rb") as f:
            blob = f.read()
    except OSError:
        return None
    if len(blob) < 64 or blob[:8] != GT_MAGIC:
        return None
    version, iw, dw, m, h, n, kk = struct.unpack("<IIIIQQQ", blob[8:48])
    if (version, iw, dw, m, n, kk) != (1, 4, 4, metric, x.shape[0], k) or h != dataset_hash(x):
        return None
    if len(blob) != 64 + 8 * n * k:
        return None
    ids = np.frombuffer(blob, np.uint32, n * k, 64).reshape(n, k)
    dists = np.frombuffer(blob, np.float32, n * k, 64 + 4 * n * k).reshape(n, k)
    return ids, dists


def load_or_compute_ground_truth(x: np.ndarray, k: int, metric: int, cache_path):
    got = load_ground_truth(cache_path, x, k, metric)
    if got is not None:
        return got
    from .api import brute_force_knn

    g = brute_force_knn(x, k, metric)
    ids, dists = g.neighbors.reshape(-1, k), g.distances.reshape(-1, k)
    Path(cache_path).parent.mkdir(parents=True, exist_ok=True)
    save_ground_truth(cache_path, ids, dists, dataset_hash(x), metric)
    return ids, dists


def recall_at_k(approx: np.ndarray, truth: np.ndarray) -> float:
    approx = np.asarray(approx)
    truth = np.asarray(truth)
    if approx.shape != truth.shape:
        raise ValueError("recall_at_k: shape mismatch")
    n, k = approx.shape
    if n == 0:
        return 1.0
    srt = np.sort(approx, axis=1)
    first = np.ones_like(srt, dtype=bool)
    first[:, 1:] = srt[:, 1:] != srt[:, :-1]  # count each approximate id once
    hits = 0
    for q in range(n):
        hits += np.isin(srt[q][first[q]], truth[q]).sum()
    return hits / (n * k)
