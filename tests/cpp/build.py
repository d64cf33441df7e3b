"""Compile tests/cpp/brute_force_gpu_test.cpp into tests/cpp/_bin/ when the
reference's headers are available (they are not on the GPU box, where the
prebuilt binary is used). Usage: python tests/cpp/build.py [REF_INCLUDE]"""
from __future__ import annotations

import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent


def build(ref_include: str = "/root/reference/include") -> Path | None:
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
