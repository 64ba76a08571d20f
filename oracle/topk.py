"""ctypes front end of ``oracle/topk_std.cpp`` (test infrastructure only)."""

from __future__ import annotations

import ctypes

import numpy as np

from oracle.build import TARGET, build

_lib = None


def _load():
    global _lib
    if _lib is None:
        build()
        lib = ctypes.CDLL(str(TARGET))
        lib.oracle_topk_least.restype = ctypes.c_int
        lib.oracle_topk_least.argtypes = [
            ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p,
        ]
        _lib = lib
    return _lib


def topk_least(scores: np.ndarray, k: int) -> np.ndarray:
    """Indices of the ``k`` smallest entries per row in PyTorch CPU tie order.

    ``scores`` is ``[rows, n]`` float32 (BF16 values widened exactly).  Mirrors
    ``scores.topk(k, dim=-1, largest=False).indices`` of
    ``experts/router.py:92``.
    """

    s = np.ascontiguousarray(scores, dtype=np.float32)
    if s.ndim != 2:
        raise ValueError("scores must be [rows, n]")
    rows, n = s.shape
    out = np.empty((rows, k), dtype=np.int64)
    rc = _load().oracle_topk_least(s.ctypes.data, rows, n, k, out.ctypes.data)
    if rc != 0:
        raise ValueError(f"invalid top-k arguments rows={rows} n={n} k={k}")
    return out
