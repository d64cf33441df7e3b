"""ctypes access to the CPU checkers (test infrastructure only).

* ``oracle()``  -- oracle/_build/libknng_oracle.so, the plain-C restatement
* ``reference()`` -- oracle/_ref/libknng_ref.so, the reference's own sources
  compiled by oracle/Makefile (None when it was never built)

Both are built on demand with ``make -C oracle`` when the sources are here.
"""
from __future__ import annotations

import ctypes
import subprocess
from ctypes import c_double, c_int, c_uint64, c_void_p, c_float
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent.parent
ORACLE_SO = ROOT / "oracle" / "_build" / "libknng_oracle.so"
REF_SO = ROOT / "oracle" / "_ref" / "libknng_ref.so"

_oracle = None
_ref = None


def _make() -> None:
    subprocess.run(["make", "-s", "-C", str(ROOT / "oracle")], check=False, capture_output=True)


def oracle() -> ctypes.CDLL:
    global _oracle
    if _oracle is None:
        if not ORACLE_SO.exists():
            _make()
        lib = ctypes.CDLL(str(ORACLE_SO))
        lib.oracle_brute_force_knn.restype = c_int
        lib.oracle_brute_force_knn.argtypes = [c_void_p, c_uint64, c_uint64, c_uint64, c_int, c_void_p, c_uint64,
                                               c_void_p, c_void_p]
        lib.oracle_knn_sets.restype = c_int
        lib.oracle_knn_sets.argtypes = [c_void_p, c_uint64, c_uint64, c_void_p, c_uint64, c_uint64, c_uint64,
                                        c_uint64, c_int, c_int, c_void_p, c_void_p]
        lib.oracle_xorshift64_stream.argtypes = [c_uint64, c_uint64, c_void_p]
        lib.oracle_next_float01.restype = c_float
        lib.oracle_next_float01.argtypes = [c_void_p]
        lib.oracle_next_below.restype = c_uint64
        lib.oracle_next_below.argtypes = [c_void_p, c_uint64]
        lib.oracle_squared_l2.restype = c_float
        lib.oracle_squared_l2.argtypes = [c_void_p, c_void_p, c_uint64]
        lib.oracle_negative_inner_product.restype = c_float
        lib.oracle_negative_inner_product.argtypes = [c_void_p, c_void_p, c_uint64]
        lib.oracle_norms_squared.argtypes = [c_void_p, c_uint64, c_uint64, c_void_p]
        lib.oracle_topk_run.restype = c_uint64
        lib.oracle_topk_run.argtypes = [c_uint64, c_uint64, c_void_p, c_void_p, c_void_p, c_void_p]
        lib.oracle_dataset_hash.restype = c_uint64
        lib.oracle_dataset_hash.argtypes = [c_void_p, c_uint64, c_uint64]
        lib.oracle_recall_at_k.restype = c_double
        lib.oracle_recall_at_k.argtypes = [c_void_p, c_void_p, c_uint64, c_uint64]
        _oracle = lib
    return _oracle


def reference() -> ctypes.CDLL | None:
    global _ref
    if _ref is None:
        if not REF_SO.exists():
            _make()
        if not REF_SO.exists():
            return None
        lib = ctypes.CDLL(str(REF_SO))
        lib.ref_brute_force_knn.restype = c_int
        lib.ref_brute_force_knn.argtypes = [c_void_p, c_uint64, c_uint64, c_uint64, c_int, c_void_p, c_void_p]
        lib.ref_brute_force_knn_omp.restype = c_int
        lib.ref_brute_force_knn_omp.argtypes = [c_void_p, c_uint64, c_uint64, c_uint64, c_int, c_void_p, c_void_p]
        lib.ref_subset_knn.restype = c_int
        lib.ref_subset_knn.argtypes = [c_void_p, c_uint64, c_uint64, c_uint64, c_int, c_void_p, c_uint64, c_int,
                                       c_void_p, c_void_p]
        lib.ref_last_error.restype = ctypes.c_char_p
        lib.ref_xorshift_u64.argtypes = [c_uint64, c_uint64, c_void_p]
        lib.ref_xorshift_float01.argtypes = [c_uint64, c_uint64, c_void_p]
        lib.ref_xorshift_below.argtypes = [c_uint64, c_uint64, c_uint64, c_void_p]
        lib.ref_dataset_hash.restype = c_uint64
        lib.ref_dataset_hash.argtypes = [c_void_p, c_uint64, c_uint64]
        lib.ref_recall_at_k.restype = c_double
        lib.ref_recall_at_k.argtypes = [c_void_p, c_void_p, c_uint64, c_uint64]
        lib.ref_topk_run.restype = c_uint64
        lib.ref_topk_run.argtypes = [c_uint64, c_uint64, c_void_p, c_void_p, c_void_p, c_void_p]
        _ref = lib
    return _ref


# ------------------------------------------------------------ convenience
def oracle_knn(x: np.ndarray, k: int, metric: int = 0, queries: np.ndarray | None = None):
    """Oracle brute force; returns (ids[nq, k], dists[nq, k]) or raises ValueError."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    n, d = x.shape
    nq = n if queries is None else len(queries)
    ids = np.zeros((max(nq, 1), max(k, 1)), np.uint32)
    dists = np.zeros((max(nq, 1), max(k, 1)), np.float32)
    q = None if queries is None else np.ascontiguousarray(queries, dtype=np.uint64)
    rc = oracle().oracle_brute_force_knn(x.ctypes.data if x.size else None, n, d, k, metric,
                                         None if q is None else q.ctypes.data, nq, ids.ctypes.data,
                                         dists.ctypes.data)
    if rc != 0:
        raise ValueError(f"oracle rc={rc}")
    return ids[:nq, :k], dists[:nq, :k]


def oracle_knn_sets(q: np.ndarray, q_id0: int, b: np.ndarray, b_id0: int, k: int, metric: int = 0,
                    exclude_self: bool = False):
    """Oracle cross-set KNN (global ids); returns (ids[n_q, k], dists[n_q, k])."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    ids = np.zeros((q.shape[0], k), np.uint32)
    dists = np.zeros((q.shape[0], k), np.float32)
    rc = oracle().oracle_knn_sets(q.ctypes.data, q.shape[0], q_id0, b.ctypes.data, b.shape[0], b_id0, b.shape[1], k,
                                  metric, int(exclude_self), ids.ctypes.data, dists.ctypes.data)
    if rc != 0:
        raise ValueError(f"oracle rc={rc}")
    return ids, dists


def ref_knn(x: np.ndarray, k: int, metric: int = 0):
    lib = reference()
    x = np.ascontiguousarray(x, dtype=np.float32)
    n, d = x.shape
    ids = np.zeros((max(n, 1), max(k, 1)), np.uint32)
    dists = np.zeros((max(n, 1), max(k, 1)), np.float32)
    rc = lib.ref_brute_force_knn(x.ctypes.data if x.size else None, n, d, k, metric, ids.ctypes.data,
                                 dists.ctypes.data)
    if rc != 0:
        raise ValueError(lib.ref_last_error().decode())
    return ids[:n, :k], dists[:n, :k]


def ref_subset_knn(x: np.ndarray, k: int, metric: int, queries: np.ndarray, threads: int = 0):
    lib = reference()
    n, d = x.shape
    q = np.ascontiguousarray(queries, dtype=np.uint64)
    ids = np.zeros((len(q), k), np.uint32)
    dists = np.zeros((len(q), k), np.float32)
    rc = lib.ref_subset_knn(x.ctypes.data, n, d, k, metric, q.ctypes.data, len(q), threads, ids.ctypes.data,
                            dists.ctypes.data)
    if rc != 0:
        raise ValueError(lib.ref_last_error().decode())
    return ids, dists


def eight_points() -> np.ndarray:
    """Two unit squares at (0,0) and (4,4): tests/brute_force_test.cpp:36-54."""
    return np.array([[0, 0], [1, 0], [0, 1], [1, 1], [4, 4], [5, 4], [4, 5], [5, 5]], dtype=np.float32)
