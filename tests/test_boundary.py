"""The C-ABI library: it loads, exports every symbol its header declares,
and rejects bad arguments with the reference's errors (no GPU needed)."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import numpy as np
import pytest

from knng_gpu_b200 import InvalidArgument, L2Squared, brute_force_knn, padded_dim, workspace_bytes
from knng_gpu_b200 import _native

ROOT = Path(__file__).resolve().parent.parent


def declared_functions() -> set[str]:
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = h.read_text()
        names |= set(re.findall(r"\b(knng_gpu_[a-z0-9_]+)\s*\(", text))
    return names


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(_native.GPU_LIB_PATH))
    declared = declared_functions()
    assert declared, "no declarations found"
    for name in declared:
        assert hasattr(lib, name), name
    assert declared == set(_native.GPU_SYMBOLS)


def test_padded_dim_and_workspace():
    # data rounded up to 128 bytes, then 32 bytes of augmentation
    assert padded_dim(1) == 160 and padded_dim(128) == 160 and padded_dim(129) == 288
    assert padded_dim(960) == 1056 and padded_dim(784) == 928
    assert workspace_bytes(1000, 128, 10) >= 1000 * 128 + 1000 * 4
    assert workspace_bytes(1000, 960, 100) >= 2 * 1000 * 1024 * 2  # fp32 path: bf16 hi + lo planes


@pytest.mark.parametrize(
    "n,k,msg",
    [
        (8, 0, "k must be > 0"),
        (8, 8, r"k \(8\) must be <= ds.n - 1 \(7\)"),
        (0, 1, "dataset is empty"),
    ],
)
def test_invalid_arguments_match_reference(n, k, msg):
    # include/knng/cpu/brute_force.hpp:339-352
    x = np.zeros((n, 2), np.float32)
    with pytest.raises(InvalidArgument, match=msg):
        brute_force_knn(x, k, L2Squared())


def test_unknown_metric_rejected():
    with pytest.raises(InvalidArgument):
        brute_force_knn(np.zeros((4, 2), np.float32), 1, 7)
