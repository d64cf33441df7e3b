"""ctypes bindings of the native libraries that ship inside this package.

``libknng_gpu.so`` is the C ABI declared in ``include/knng_gpu.h``;
``libknng_synth.so`` holds the seeded dataset generators. Both are built
in-tree by :mod:`knng_gpu_b200.build`. A missing library is an error, never a
reason to fall back to another implementation.
"""
from __future__ import annotations

import ctypes
from ctypes import POINTER, c_char_p, c_float, c_int, c_int32, c_uint32, c_uint64, c_void_p
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
GPU_LIB_PATH = PKG_DIR / "libknng_gpu.so"
SYNTH_LIB_PATH = PKG_DIR / "libknng_synth.so"

# Every symbol include/knng_gpu.h declares (tests check the library exports them).
GPU_SYMBOLS = (
    "knng_gpu_last_error",
    "knng_gpu_device_count",
    "knng_gpu_brute_force",
    "knng_gpu_release_cached_buffers",
    "knng_gpu_workspace_bytes",
    "knng_gpu_brute_force_device",
    "knng_gpu_padded_dim",
    "knng_gpu_pack_u8",
    "knng_gpu_knn_scratch_bytes",
    "knng_gpu_knn_u8",
    "knng_gpu_knn_u8_sets",
    "knng_gpu_merge_topk",
    "knng_gpu_knn_f32_scratch_bytes",
    "knng_gpu_knn_f32",
    "knng_gpu_knn_u8_noalloc",
    "knng_gpu_brute_force_u8",
    "knng_gpu_pack_u8_bytes",
    "knng_gpu_selftest_bounded_wait",
    "knng_gpu_nccl_id_bytes",
    "knng_gpu_nccl_unique_id",
    "knng_gpu_comm_create",
    "knng_gpu_comm_destroy",
    "knng_gpu_shard_rows",
    "knng_gpu_sharded_workspace_bytes",
    "knng_gpu_brute_force_sharded",
    "knng_gpu_comm_phase_ms",
    "knng_gpu_brute_force_multi",
    "knng_gpu_release_multi",
    "knng_gpu_knn_f32_sets_scratch_bytes",
    "knng_gpu_knn_f32_sets",
    "knng_gpu_recall_at_k",
)


class KnngGpuStats(ctypes.Structure):
    """Mirror of ``knng_gpu_stats`` (include/knng_gpu.h)."""

    _fields_ = [
        ("path", c_int),
        ("fallback_rows", c_uint64),
        ("pack_ms", c_float),
        ("knn_ms", c_float),
        ("fallback_ms", c_float),
        ("total_ms", c_float),
        ("kernel_launches", c_uint32),
        ("f32_err_ratio", c_float),
        ("tc_ms", c_float),
    ]

    def as_dict(self) -> dict:
        return {name: getattr(self, name) for name, _ in self._fields_}


_gpu = None
_synth = None


def gpu_lib() -> ctypes.CDLL:
    """Load ``libknng_gpu.so`` (raises if it has not been built)."""
    global _gpu
    if _gpu is None:
        if not GPU_LIB_PATH.exists():
            raise RuntimeError(
                f"knng_gpu_b200: {GPU_LIB_PATH.name} is not built; run "
                "`python -c 'import __graft_entry__ as g; g.build()'` or "
                "`python -m knng_gpu_b200.build`"
            )
        lib = ctypes.CDLL(str(GPU_LIB_PATH))
        f32p, u32p, i32p = POINTER(c_float), POINTER(c_uint32), POINTER(c_int32)
        st = POINTER(KnngGpuStats)
        sig = {
            "knng_gpu_last_error": (c_char_p, []),
            "knng_gpu_device_count": (c_int, []),
            "knng_gpu_brute_force": (c_int, [c_void_p, c_uint64, c_uint64, c_uint64, c_int, c_void_p, c_void_p, st]),
            "knng_gpu_release_cached_buffers": (None, []),
            "knng_gpu_workspace_bytes": (c_uint64, [c_uint64, c_uint64, c_uint64]),
            "knng_gpu_knn_f32_scratch_bytes": (c_uint64, [c_uint64, c_uint64, c_uint64, c_uint64]),
            "knng_gpu_brute_force_device": (
                c_int,
                [c_void_p, c_uint64, c_uint64, c_uint64, c_int, c_void_p, c_void_p, c_void_p, c_uint64, c_void_p, st],
            ),
            "knng_gpu_padded_dim": (c_uint64, [c_uint64]),
            "knng_gpu_pack_u8": (c_int, [c_void_p, c_uint64, c_uint64, c_void_p, c_void_p, c_void_p, c_void_p]),
            "knng_gpu_knn_scratch_bytes": (c_uint64, [c_uint64, c_uint64]),
            "knng_gpu_selftest_bounded_wait": (c_int, [c_uint64]),
            "knng_gpu_nccl_id_bytes": (c_uint64, []),
            "knng_gpu_nccl_unique_id": (c_int, [c_void_p]),
            "knng_gpu_comm_create": (c_int, [c_void_p, c_int, c_int, POINTER(c_void_p)]),
            "knng_gpu_comm_destroy": (None, [c_void_p]),
            "knng_gpu_shard_rows": (None, [c_uint64, c_int, c_int, c_int, POINTER(c_uint64), POINTER(c_uint64)]),
            "knng_gpu_sharded_workspace_bytes": (c_uint64, [c_uint64, c_uint64, c_uint64, c_int, c_int]),
            "knng_gpu_brute_force_sharded": (
                c_int, [c_void_p, c_uint64, c_uint64, c_uint64, c_int, c_int, c_void_p, c_void_p, c_void_p,
                        c_void_p, c_uint64, c_void_p, st]),
            "knng_gpu_comm_phase_ms": (c_int, [c_void_p, POINTER(c_float)]),
            "knng_gpu_brute_force_multi": (
                c_int, [c_void_p, c_uint64, c_uint64, c_uint64, c_int, c_int, c_int, c_void_p, c_void_p, st]),
            "knng_gpu_release_multi": (None, []),
            "knng_gpu_knn_f32_sets_scratch_bytes": (c_uint64, [c_uint64, c_uint64, c_uint64, c_uint64, c_int]),
            "knng_gpu_knn_f32_sets": (
                c_int, [c_void_p, c_uint64, c_uint64, c_void_p, c_uint64, c_uint64, c_uint64, c_uint64, c_int, c_int,
                        c_void_p, c_void_p, c_void_p, c_uint64, c_void_p, st]),
            "knng_gpu_recall_at_k": (c_int, [c_void_p, c_void_p, c_uint64, c_uint64, c_void_p, c_void_p,
                                             POINTER(ctypes.c_double)]),
            "knng_gpu_brute_force_u8": (
                c_int, [c_void_p, c_uint64, c_uint64, c_uint64, c_uint64, c_int, c_void_p, c_void_p, st]),
            "knng_gpu_pack_u8_bytes": (c_int, [c_void_p, c_uint64, c_uint64, c_uint64, c_void_p, c_void_p, c_void_p]),
            "knng_gpu_knn_u8": (
                c_int,
                [c_void_p, c_void_p, c_uint64, c_uint64, c_uint64, c_uint64, c_uint64, c_int, c_void_p, c_void_p,
                 c_void_p, c_uint64, c_void_p, st],
            ),
            "knng_gpu_knn_u8_sets": (
                c_int,
                [c_void_p, c_void_p, c_uint64, c_uint64, c_void_p, c_void_p, c_uint64, c_uint64, c_uint64, c_uint64,
                 c_int, c_int, c_void_p, c_void_p, c_void_p, c_uint64, c_void_p, st],
            ),
            "knng_gpu_merge_topk": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_uint64, c_uint64, c_void_p,
                                            c_void_p, c_void_p]),
            "knng_gpu_knn_u8_noalloc": (
                c_int,
                [c_void_p, c_void_p, c_uint64, c_uint64, c_uint64, c_uint64, c_uint64, c_int, c_void_p, c_void_p,
                 c_void_p, st],
            ),
            "knng_gpu_knn_f32": (
                c_int,
                [c_void_p, c_uint64, c_uint64, c_uint64, c_uint64, c_uint64, c_int, c_void_p, c_void_p, c_void_p,
                 c_uint64, c_void_p, st],
            ),
        }
        del f32p, u32p, i32p
        for name, (res, args) in sig.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _gpu = lib
    return _gpu


def synth_lib() -> ctypes.CDLL:
    """Load ``libknng_synth.so`` (raises if it has not been built)."""
    global _synth
    if _synth is None:
        if not SYNTH_LIB_PATH.exists():
            raise RuntimeError(f"knng_gpu_b200: {SYNTH_LIB_PATH.name} is not built")
        lib = ctypes.CDLL(str(SYNTH_LIB_PATH))
        lib.knng_synth_generate.restype = c_int
        lib.knng_synth_generate.argtypes = [c_int, c_uint64, c_uint64, c_uint64, c_void_p, c_uint64, c_float,
                                            c_float, c_void_p]
        lib.knng_synth_generate_rows.restype = c_int
        lib.knng_synth_generate_rows.argtypes = [c_int, c_uint64, c_uint64, c_uint64, c_uint64, c_void_p, c_uint64,
                                                 c_float, c_float, c_void_p]
        lib.knng_dataset_hash.restype = c_uint64
        lib.knng_dataset_hash.argtypes = [c_void_p, c_uint64, c_uint64]
        lib.knng_synth_sample_ids.restype = c_int
        lib.knng_synth_sample_ids.argtypes = [c_uint64, c_uint64, c_uint64, c_void_p]
        _synth = lib
    return _synth
