"""Compile tests/cpp/brute_force_gpu_test.cpp into tests/cpp/_bin/ when the
reference's headers are available (they are not on the GPU box, where the
prebuilt binary is used). Usage: python tests/cpp/build.py [REF_INCLUDE]"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent


def reference_include() -> Path | None:
    """include/ of the reference checkout: KNNG_REFERENCE, else a `reference`
    directory beside this repository; None when neither exists."""
    ref = os.environ.get("KNNG_REFERENCE")
    if ref:
        return Path(ref) / "include"
    sibling = ROOT.parent / "reference" / "include"
    return sibling if sibling.exists() else None


def build(ref_include: str | None = None) -> Path | None:
    if ref_include is None:
        inc = reference_include()
        if inc is None:
            return None
        ref_include = str(inc)
    if not (Path(ref_include) / "knng" / "core" / "dataset.hpp").exists():
        return None
    out = HERE / "_bin" / "brute_force_gpu_test"
    out.parent.mkdir(exist_ok=True)
    lib = ROOT / "knng_gpu_b200"
    subprocess.run(["g++", "-std=c++20", "-O2", f"-I{ref_include}", f"-I{ROOT / 'include'}", "-o", str(out),
                    str(HERE / "brute_force_gpu_test.cpp"), f"-L{lib}", "-lknng_gpu",
                    "-Wl,-rpath,$ORIGIN/../../../knng_gpu_b200"], check=True)
    return out


if __name__ == "__main__":
    print(build(*sys.argv[1:]))
