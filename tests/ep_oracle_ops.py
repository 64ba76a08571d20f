"""CPU stand-in for `spalmer_b200.ep.CudaOps` built on the oracle (test-only).

It lets the expert-parallel exchange of `ExpertParallelMixer` run over gloo
ranks on the CPU: the stages compute with `oracle.mixer_ref` on BF16 bit
patterns, the exchange is the production code.  The same ops applied to all
tokens on one process give the reference result the exchange must reproduce.
"""

from __future__ import annotations

import numpy as np
import torch

from oracle import mixer_ref as R
from oracle.bf16 import bf16_bits_to_f32, f32_to_bf16_bits, round_bf16


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().view(torch.int16).numpy().view(np.uint16)


def _tensor(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16).copy()).view(torch.bfloat16)


class OracleOps:
    device = torch.device("cpu")

    def __init__(self, params: R.LayerParams, k: int, rank: int, world: int):
        self.p = params
        self.k = k
        self.E = params.router_w.shape[0]
        self.e_local = self.E // world
        self.e0 = rank * self.e_local
        self.d = params.router_w.shape[1]

    def route(self, x: torch.Tensor, logits=None) -> dict:
        xb = _bits(x)
        lg = R.router_logits(xb, self.p.router_w, self.p.router_b) if logits is None else _bits(logits)
        scores = R.router_scores(lg)
        ids, weights = R.select_least_surprised(scores, self.k)
        order = R.dispatch_order(ids).astype(np.int32)
        rank = np.empty_like(order)
        rank[order] = np.arange(order.size, dtype=np.int32)
        counts = np.bincount(ids.reshape(-1), minlength=self.E).astype(np.int32)
        return {
            "router_scores": _tensor(scores), "expert_ids": torch.from_numpy(ids.astype(np.int64)),
            "routing_weights": _tensor(weights), "expert_utilization": torch.from_numpy(R.expert_utilization(ids, self.E)),
            "auxiliary_loss": torch.zeros(1, dtype=torch.bfloat16),
            "order": torch.from_numpy(order), "counts": torch.from_numpy(counts), "rank": torch.from_numpy(rank),
        }

    def gather(self, x: torch.Tensor, order: torch.Tensor, div: int) -> torch.Tensor:
        return x[order.long() // div].contiguous()

    def experts(self, rows: torch.Tensor, row_expert: torch.Tensor, lanes) -> torch.Tensor:
        rb = _bits(rows)
        out = np.zeros_like(rb)
        ids = row_expert.numpy()
        for e in np.unique(ids):
            sel = np.nonzero(ids == e)[0]
            g = self.e0 + int(e)
            out[sel] = R._swiglu_rows(rb[sel], bf16_bits_to_f32(self.p.gate[g]), bf16_bits_to_f32(self.p.up[g]),
                                      bf16_bits_to_f32(self.p.down[g]))
        return _tensor(out)

    def shared(self, x: torch.Tensor):
        if self.p.shared_gate is None:
            return None
        return _tensor(R.shared_swiglu(_bits(x), self.p.shared_gate, self.p.shared_up, self.p.shared_down))

    def combine(self, rows: torch.Tensor, rank: torch.Tensor, weights, shared, tokens: int | None = None):
        y = bf16_bits_to_f32(_bits(rows))
        w = np.zeros(0, np.float32) if weights is None else bf16_bits_to_f32(_bits(weights)).reshape(-1)
        rk = rank.numpy().reshape(-1)
        T = weights.shape[0] if tokens is None else tokens
        acc = np.zeros((T, self.d), np.float32) if shared is None else bf16_bits_to_f32(_bits(shared)).copy()
        k = rk.size // T
        for j in range(k):
            p = np.arange(T) * k + j
            ok = rk[p] >= 0  # a negative rank is an empty slot
            add = round_bf16(y[np.where(ok, rk[p], 0)] * w[p][:, None]) if w.size else y[np.where(ok, rk[p], 0)]
            acc = acc + np.where(ok[:, None], add, np.float32(0))
        return _tensor(f32_to_bf16_bits(acc))


def single_process_update(ops: OracleOps, x: torch.Tensor) -> torch.Tensor:
    """The layer on all tokens without any exchange (world = 1 semantics)."""

    r = ops.route(x)
    rows = ops.gather(x, r["order"], ops.k)
    row_expert = torch.from_numpy(np.repeat(np.arange(ops.E), r["counts"].numpy()).astype(np.int64))
    saved = ops.e0
    ops.e0 = 0
    try:
        out_rows = ops.experts(rows, row_expert, None)
    finally:
        ops.e0 = saved
    return ops.combine(out_rows, r["rank"], r["routing_weights"], ops.shared(x))
