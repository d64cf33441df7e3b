"""In-tree build of the native libraries (``python -m knng_gpu_b200.build``).

* ``libknng_gpu.so``   -- CUDA kernels + C ABI, nvcc for sm_100a only
* ``libknng_synth.so`` -- seeded dataset generators (gcc)

Outputs land next to this file so they travel with the source tree. A target
is rebuilt only when one of its sources is newer than it.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _stale(target: Path, sources: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(s.stat().st_mtime > t for s in sources)


def _run(cmd: list[str], verbose: bool) -> None:
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)


def build_gpu(verbose: bool = False, force: bool = False) -> Path:
    out = PKG / "libknng_gpu.so"
    srcs = sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + [ROOT / "include" / "knng_gpu.h"]
    if force or _stale(out, srcs):
        tmp = out.with_suffix(".so.tmp")
        _run([NVCC, *ARCH, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC,-O2", "-shared",
              f"-I{ROOT / 'include'}", "-o", str(tmp), str(CSRC / "knng_gpu.cu"), "-lnccl"], verbose)
        tmp.replace(out)
    return out


def build_synth(verbose: bool = False, force: bool = False) -> Path:
    out = PKG / "libknng_synth.so"
    src = CSRC / "synthetic.c"
    if force or _stale(out, [src]):
        _run(["gcc", "-std=c11", "-O2", "-ffp-contract=off", "-fPIC", "-shared", "-o", str(out), str(src), "-lm"],
             verbose)
    return out


def build_cli(verbose: bool = False, force: bool = False) -> Path:
    """build_knng_gpu: the reference's build_knng CLI over libknng_gpu.so."""
    out = PKG / "bin" / "build_knng_gpu"
    srcs = [PKG / "cli" / "build_knng_gpu.cpp", PKG / "cli" / "knng_files.hpp", ROOT / "include" / "knng_gpu.h",
            PKG / "libknng_gpu.so"]
    if force or _stale(out, srcs):
        out.parent.mkdir(exist_ok=True)
        _run(["g++", "-std=c++17", "-O2", f"-I{ROOT / 'include'}", "-I/usr/local/cuda/include", "-o", str(out),
              str(PKG / "cli" / "build_knng_gpu.cpp"), f"-L{PKG}", "-lknng_gpu", "-L/usr/local/cuda/lib64",
              "-lcudart", "-Wl,-rpath,$ORIGIN/..:/usr/local/cuda/lib64"], verbose)
    return out


def build_all(verbose: bool = False, force: bool = False) -> None:
    build_synth(verbose, force)
    build_gpu(verbose, force)
    build_cli(verbose, force)


if __name__ == "__main__":
    build_all(verbose=True, force="--force" in sys.argv)
