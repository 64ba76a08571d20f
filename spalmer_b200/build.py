"""Build libspx in-tree for sm_100a.

``python -m spalmer_b200.build`` compiles every ``csrc/*.cu`` into
``spalmer_b200/libspx.so`` with nvcc (``-gencode arch=compute_100a,code=sm_100a``).
The .so is git-ignored and travels with the working tree; nothing is
compiled at import time.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
TARGET = HERE / "libspx.so"
SOURCES = ("abi.cu", "gemm.cu", "route.cu", "dispatch.cu", "pack.cu", "dispatch_static.cu", "launch.cu", "mxfp8.cu", "calibration.cu", "backward.cu", "block.cu", "paged.cu", "nvfp4.cu", "peer.cu", "gemv.cu", "quant_error.cu", "wgrad.cu")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
    "--expt-relaxed-constexpr",
]


def nvcc_path() -> str:
    found = shutil.which("nvcc")
    if found:
        return found
    cand = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda")) / "bin" / "nvcc"
    if cand.exists():
        return str(cand)
    raise RuntimeError("nvcc not found")


def _stale() -> bool:
    if not TARGET.exists():
        return True
    built = TARGET.stat().st_mtime
    deps = list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h"))
    deps.append(HERE.parent / "include" / "spx.h")
    return any(p.stat().st_mtime > built for p in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not _stale():
        return TARGET
    tmp = TARGET.with_suffix(f".{os.getpid()}.tmp.so")
    cmd = [nvcc_path(), *NVCC_FLAGS, *(str(CSRC / s) for s in SOURCES), "-o", str(tmp)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    subprocess.run(cmd, check=True)
    os.replace(tmp, TARGET)
    return TARGET


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
