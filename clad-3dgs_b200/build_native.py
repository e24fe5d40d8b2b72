"""Builds libclad3dgs_b200.so, the C-ABI library of the hot path, for sm_100a.

nvcc cross-compiles without a GPU, so this runs on any machine with CUDA 12.9.
Objects are rebuilt when a source or header is newer than the library.

The per-Gaussian kernels are compiled with -fmad=false: every floating-point
operation is rounded on its own, in source order, which is what lets the CPU
oracle reproduce their results bit for bit.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
CSRC = HERE / "csrc"
INCLUDE = ROOT / "include"
LIBRARY = HERE / "libclad3dgs_b200.so"
BUILD = ROOT / "_build" / "native"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=default",
    "-I", str(INCLUDE), "-I", str(CSRC),
]
# Per-source extra flags.
FLAGS = {
    "gaussian_step.cu": ["-fmad=false"],
    "host_step.cu": [],
    "rasterizer.cu": [],
    "sh_backward.cu": ["-fmad=false"],
    "train_step.cu": ["-fmad=false"],
}


def nvcc() -> str:
    found = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(found).exists():
        raise RuntimeError("nvcc not found; the CUDA 12.9 toolkit is required")
    return found


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(verbose: bool = False, ptxas_info: bool = False) -> Path:
    """Compiles every csrc/*.cu and links the shared library; returns its path."""
    BUILD.mkdir(parents=True, exist_ok=True)
    headers = sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))
    objects = []
    for name, extra in FLAGS.items():
        source = CSRC / name
        obj = BUILD / (source.stem + ".o")
        objects.append(obj)
        if not _stale(obj, [source, *headers, Path(__file__)]) and not ptxas_info:
            continue
        cmd = [nvcc(), *COMMON, *extra, "-c", str(source), "-o", str(obj)]
        if ptxas_info:
            cmd.insert(1, "-Xptxas=-v")
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    if _stale(LIBRARY, objects):
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(LIBRARY), *map(str, objects)]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return LIBRARY


if __name__ == "__main__":
    print(build(verbose=True, ptxas_info="--ptxas" in sys.argv))
