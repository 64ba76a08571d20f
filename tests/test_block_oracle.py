"""The channel RMSNorm: the oracle restatement and the module's own torch
forward against the reference's RMSNorm (tests/golden/block_rmsnorm.npz,
written by make_block.py)."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import torch

from oracle.mixer_ref import rms_norm
from spalmer_b200 import RMSNorm
from tests.helpers import bf16_bits, from_bits

GOLDEN = Path(__file__).resolve().parent / "golden" / "block_rmsnorm.npz"


def test_rms_norm_oracle_matches_reference():
    d = np.load(GOLDEN)
    assert np.array_equal(rms_norm(d["h"], d["weight"], float(d["eps"])), d["out"])


def test_module_rms_norm_matches_reference():
    d = np.load(GOLDEN)
    norm = RMSNorm(768, eps=float(d["eps"]), dtype=torch.bfloat16)
    with torch.no_grad():
        norm.weight.copy_(from_bits(d["weight"]))
        out = norm(from_bits(d["h"]))
    assert np.array_equal(bf16_bits(out), d["out"])
