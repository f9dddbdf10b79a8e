"""Build the in-tree native libraries of bitnetrs_b200.

    python -m bitnetrs_b200.build [--force]

* ``libbitnet_cuda.so``  — the CUDA backend (every ``csrc/*.cu``), compiled for
  sm_100a only, C ABI declared in ``include/bitnet_cuda.h``.
* ``libbitnet_synth.so`` — the seeded synthetic-input generator (host C++).

Both land next to this file so they travel with the source tree.  Object
files go to ``_build/``.  nvcc cross-compiles without a GPU.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
INCLUDE = PKG.parent / "include"
CUDA_LIB = PKG / "libbitnet_cuda.so"
SYNTH_LIB = PKG / "libbitnet_synth.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
# -fmad=false: no implicit FMA contraction; kernels spell out every FMA the
# reference performs, which is what keeps them bit-identical to it.
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "-fmad=false",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-ffp-contract=off",
    "-I", str(INCLUDE),
]


def nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build bitnetrs_b200")


def _stale(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(Path(d).stat().st_mtime > t for d in deps)


def _run(cmd) -> None:
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError(f"build step failed: {' '.join(map(str, cmd))}")


def build_cuda(force: bool = False, verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    headers = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + [INCLUDE / "bitnet_cuda.h"]
    objs = []
    for src in sorted(CSRC.glob("*.cu")):
        obj = BUILD / (src.stem + ".o")
        if force or _stale(obj, [src] + headers):
            cmd = [nvcc()] + NVCC_FLAGS + ["-c", str(src), "-o", str(obj)]
            if verbose:
                print(" ".join(cmd))
            _run(cmd)
        objs.append(obj)
    if force or _stale(CUDA_LIB, objs):
        _run([nvcc()] + ARCH + ["-shared", "-cudart", "static", "-o", str(CUDA_LIB)] + [str(o) for o in objs])
    return CUDA_LIB


def build_synth(force: bool = False) -> Path:
    src = CSRC / "synth.cpp"
    if force or _stale(SYNTH_LIB, [src]):
        _run(["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-pthread", "-ffp-contract=off",
              str(src), "-o", str(SYNTH_LIB)])
    return SYNTH_LIB


def build(force: bool = False, verbose: bool = False) -> None:
    build_synth(force)
    build_cuda(force, verbose)


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    build(a.force, a.verbose)
    print(CUDA_LIB)
    print(SYNTH_LIB)
