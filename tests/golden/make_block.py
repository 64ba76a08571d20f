"""Generate the RMSNorm golden vectors by running the reference's ``RMSNorm``
(mESmaC/spalmer ``nn/norm.py``) itself.

    python tests/golden/make_block.py /path/to/reference/src

Rows: ``torch.randn(512, 768, generator=manual_seed(21))`` scaled per row by
``exp(randn)`` (so the variance spans orders of magnitude), in BF16; weight
``1 + 0.1 * randn(768, generator=manual_seed(22))`` in BF16; eps 1e-6.
Stored: input, weight, eps and the reference's output (BF16 bits).
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def main() -> None:
    if len(sys.argv) > 1:
        sys.path.insert(0, sys.argv[1])
    from spalmer.nn.norm import RMSNorm

    g = torch.Generator().manual_seed(21)
    h = torch.randn(512, 768, generator=g) * torch.exp(torch.randn(512, 1, generator=g))
    h = h.to(torch.bfloat16)
    w = (1.0 + 0.1 * torch.randn(768, generator=torch.Generator().manual_seed(22))).to(torch.bfloat16)
    norm = RMSNorm(768, eps=1e-6, dtype=torch.bfloat16)
    with torch.no_grad():
        norm.weight.copy_(w)
        out = norm(h)
    np.savez_compressed(HERE / "block_rmsnorm.npz", h=_bits(h), weight=_bits(w), eps=np.float32(1e-6),
                        out=_bits(out))
    print("wrote block_rmsnorm")


if __name__ == "__main__":
    main()
