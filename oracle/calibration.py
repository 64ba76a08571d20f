"""Router calibration loss term and per-expert NLL attribution (test
infrastructure only; restates mESmaC/spalmer src/spalmer/modeling.py:1468-1534).

Per layer, over positions s < S-1 (the last position has no next-token NLL):
  predicted[b,s]  = bf16( sum_j bf16(score[b,s,id_j] * w[b,s,j]) )   (fp32 sum)
  calibration     = mean over valid positions of smooth_l1(predicted, nll),
                    beta 1, in float32 (modeling.py:1484-1491)
  counts[e]       = sum of w * valid over pairs of expert e      (float32)
  totals[e]       = sum of w * valid * nll over pairs of expert e
  attributed[e]   = totals / max(counts, 1e-8) where counts > 0, else 0
  utilization[e]  = counts / max(number of valid positions, 1)  (modeling.py:1513-1534)
"""

from __future__ import annotations

import numpy as np

from oracle.bf16 import bf16_bits_to_f32, f32_to_bf16_bits, round_bf16


def surprise_calibration(score_bits: np.ndarray, ids: np.ndarray, weight_bits: np.ndarray, token_nll: np.ndarray,
                         valid: np.ndarray) -> tuple[np.float32, np.ndarray, np.ndarray]:
    """``score_bits [B,S,E]``, ``ids [B,S,k]``, ``weight_bits [B,S,k]``,
    ``token_nll [B,S-1]`` float32, ``valid [B,S-1]`` bool."""

    B, S, E = score_bits.shape
    ids = ids[:, :-1].astype(np.int64)
    w = bf16_bits_to_f32(weight_bits[:, :-1])
    sel = bf16_bits_to_f32(np.take_along_axis(score_bits[:, :-1], ids, axis=-1))
    predicted = round_bf16(round_bf16(sel * w).sum(axis=-1, dtype=np.float32))
    d = np.abs(predicted.astype(np.float32) - token_nll.astype(np.float32))
    sl1 = np.where(d < 1.0, 0.5 * d * d, d - 0.5).astype(np.float32)
    calibration = np.float32(sl1[valid].mean(dtype=np.float64)) if valid.any() else np.float32(np.nan)
    wv = (w * valid[..., None]).astype(np.float32)
    counts = np.zeros(E, np.float64)
    totals = np.zeros(E, np.float64)
    np.add.at(counts, ids.reshape(-1), wv.reshape(-1))
    np.add.at(totals, ids.reshape(-1), (wv * token_nll[..., None].astype(np.float32)).reshape(-1))
    attributed = np.where(counts > 0, totals / np.maximum(counts, 1e-8), 0.0).astype(np.float32)
    utilization = (counts / max(float(valid.sum()), 1.0)).astype(np.float32)
    return calibration, attributed, utilization


__all__ = ["surprise_calibration"]
