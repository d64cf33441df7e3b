"""Generate the golden fixtures in this folder from the reference itself.

Run here, where the reference checkout exists (oracle/Makefile compiles its
own unmodified sources into oracle/_ref/libknng_ref.so):

    python tests/golden/make_golden.py

Writes
  xorshift.npz      raw XorShift64 / next_float01 / next_below streams
  topk.npz          knng::TopK on a tie-heavy push sequence
  knn_<case>.npz    knng::cpu::brute_force_knn ids + dists for every case of
                    tests/cases.py, with the reference's dataset_hash of the
                    input (pins the generator that recreates it)
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))
sys.path.insert(0, str(HERE.parent.parent))

from cases import CASES  # noqa: E402
from refs import ref_knn, reference  # noqa: E402


def main() -> None:
    lib = reference()
    if lib is None:
        raise SystemExit("reference library not built (make -C oracle)")
    seeds = np.array([1, 42, 7, 1234, 99, 2024], np.uint64)
    u64 = np.zeros((len(seeds), 64), np.uint64)
    f01 = np.zeros((len(seeds), 64), np.float32)
    b256 = np.zeros((len(seeds), 64), np.uint64)
    b100 = np.zeros((len(seeds), 64), np.uint64)
    for i, s in enumerate(seeds):
        lib.ref_xorshift_u64(int(s), 64, u64[i].ctypes.data)
        lib.ref_xorshift_float01(int(s), 64, f01[i].ctypes.data)
        lib.ref_xorshift_below(int(s), 256, 64, b256[i].ctypes.data)
        lib.ref_xorshift_below(int(s), 100, 64, b100[i].ctypes.data)
    np.savez_compressed(HERE / "xorshift.npz", seeds=seeds, u64=u64, float01=f01, below256=b256, below100=b100)

    rng = np.random.default_rng(0)
    ids = rng.permutation(200).astype(np.uint32)
    dists = rng.integers(0, 12, 200).astype(np.float32) * 0.5
    out = {}
    for k in (0, 1, 2, 5, 17, 200, 250):
        oi = np.zeros(max(k, 1), np.uint32)
        od = np.zeros(max(k, 1), np.float32)
        m = lib.ref_topk_run(k, 200, ids.ctypes.data, dists.ctypes.data, oi.ctypes.data, od.ctypes.data)
        out[f"ids_{k}"] = oi[:m]
        out[f"dists_{k}"] = od[:m]
    np.savez_compressed(HERE / "topk.npz", push_ids=ids, push_dists=dists, **out)

    for c in CASES:
        x = np.ascontiguousarray(c.make(), dtype=np.float32)
        h = lib.ref_dataset_hash(x.ctypes.data, x.shape[0], x.shape[1])
        gi, gd = ref_knn(x, c.k, c.metric)
        np.savez_compressed(HERE / f"knn_{c.name}.npz", ids=gi, dists=gd, data_hash=np.uint64(h),
                            n=x.shape[0], d=x.shape[1], k=c.k, metric=c.metric)
        print(f"{c.name}: n={x.shape[0]} d={x.shape[1]} k={c.k} hash={h:#x}")


if __name__ == "__main__":
    main()
