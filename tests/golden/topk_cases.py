"""Seeded tie-heavy score matrices for the top-k tie-order fixtures.

Shared by ``make_golden.py`` (which records ``torch.topk`` indices for them in
the build container) and the tests (which regenerate the same matrices from
the seeds and check a SHA-256 of the bytes before comparing indices).
"""

from __future__ import annotations

import numpy as np

from oracle.bf16 import f32_to_bf16_bits
from oracle.mixer_ref import softplus_lut

TOPK_CASES = [
    # Router-like: softplus of BF16 N(0, 0.55) logits (x~N(0,1), W~N(0,0.02), d=768).
    dict(name="router_like", rows=2048, n=200, kind="softplus", std=0.55, seed=11,
         ks=(1, 2, 3, 4, 8, 16, 20)),
    # Very few distinct values: almost every row is all ties.
    dict(name="coarse4", rows=1024, n=200, kind="levels", levels=4, seed=12, ks=(2, 3, 4, 8, 17)),
    dict(name="coarse16", rows=1024, n=200, kind="levels", levels=16, seed=13, ks=(4, 8)),
    # Every entry equal.
    dict(name="all_equal", rows=8, n=200, kind="levels", levels=1, seed=14, ks=(1, 2, 4, 8, 20)),
    # Resident mask: 30 of 200 eligible, the rest +inf.
    dict(name="masked30", rows=1024, n=200, kind="softplus", std=0.55, seed=15, mask=30, ks=(4, 8)),
    # Small banks (the reference's unit tests use 4-8 experts) and a mid-size one.
    dict(name="n3", rows=512, n=3, kind="levels", levels=2, seed=16, ks=(1, 2, 3)),
    dict(name="n6", rows=1024, n=6, kind="levels", levels=3, seed=17, ks=(1, 2, 3, 6)),
    dict(name="n64", rows=1024, n=64, kind="levels", levels=8, seed=18, ks=(1, 2, 8, 20)),
    dict(name="n256", rows=512, n=256, kind="softplus", std=0.3, seed=19, ks=(4, 8)),
    # NaNs sprinkled in (ordered last by the CPU comparator).
    dict(name="with_nan", rows=512, n=200, kind="softplus", std=0.55, seed=20, nan=0.05, ks=(4, 8)),
]


def generate_scores(case: dict) -> tuple[np.ndarray, np.ndarray | None]:
    """Return ``(bf16 bits [rows, n], resident mask [n] or None)``."""

    rng = np.random.Generator(np.random.PCG64(case["seed"]))
    rows, n = case["rows"], case["n"]
    if case["kind"] == "softplus":
        logits = f32_to_bf16_bits(rng.normal(0.0, case["std"], size=(rows, n)).astype(np.float32))
        bits = softplus_lut()[logits]
    else:
        levels = case["levels"]
        values = (rng.integers(0, levels, size=(rows, n)).astype(np.float32) + 1.0) * 0.5
        bits = f32_to_bf16_bits(values)
    if case.get("nan"):
        hit = rng.random((rows, n)) < case["nan"]
        bits = bits.copy()
        bits[hit] = np.uint16(0x7FC0)
    mask = None
    if case.get("mask"):
        mask = np.zeros(n, dtype=bool)
        mask[rng.permutation(n)[: case["mask"]]] = True
    return np.ascontiguousarray(bits), mask
