"""Compile the oracle's C++ checker (test infrastructure only).

``python -m oracle.build`` (or ``__graft_entry__.build()``) compiles
``oracle/topk_std.cpp`` with g++ into ``oracle/liboracle_topk.so``.  The
shared object is git-ignored and travels to the GPU box with the working
tree.  The reference (mESmaC/spalmer) is pure Python, so there is no
reference C/C++ source to compile into ``oracle/_ref``.
"""

from __future__ import annotations

import os
import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
SOURCE = HERE / "topk_std.cpp"
TARGET = HERE / "liboracle_topk.so"


def build(force: bool = False) -> Path:
    if not force and TARGET.exists() and TARGET.stat().st_mtime >= SOURCE.stat().st_mtime:
        return TARGET
    tmp = TARGET.with_suffix(f".{os.getpid()}.tmp")
    cmd = [
        "g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-fopenmp",
        str(SOURCE), "-o", str(tmp),
    ]
    subprocess.run(cmd, check=True)
    os.replace(tmp, TARGET)
    return TARGET


if __name__ == "__main__":
    print(build(force=True))
