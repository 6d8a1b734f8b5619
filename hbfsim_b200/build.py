"""Build the in-tree CUDA library hbfsim_b200/libhbfsim_b200.so for sm_100a.

nvcc compiles the kernels and the C ABI directly (no torch extension
machinery): the library exports only extern "C" symbols with plain pointers,
so it can be bound from ctypes, cgo, JNI or a C/C++ host alike.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
LIB = PKG / "libhbfsim_b200.so"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
SOURCES = ["timing.cu", "empirical.cu", "context.cu", "thermal.cu", "capacity.cu",
           "retention.cu", "prefetch.cu", "link.cu", "profile.cpp"]


def sources() -> list[Path]:
    return [CSRC / s for s in SOURCES]


def stale() -> bool:
    if not LIB.exists():
        return True
    built = LIB.stat().st_mtime
    deps = list(CSRC.glob("*")) + list((PKG.parent / "include" / "hbfsim").glob("*.h"))
    return any(p.stat().st_mtime > built for p in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not stale():
        return LIB
    cmd = [NVCC, *ARCH, "-O3", "-lineinfo", "-std=c++17", "-shared",
           "-Xcompiler", "-fPIC", "-cudart", "static",
           "-Xptxas", "-warn-spills",
           "-o", str(LIB), *map(str, sources())]
    # exported C ABI: visibility comes from the version script below
    script = CSRC / "exports.map"
    cmd += ["-Xlinker", f"--version-script={script}"]
    if verbose:
        print(" ".join(cmd))
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError("nvcc build of libhbfsim_b200.so failed")
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
