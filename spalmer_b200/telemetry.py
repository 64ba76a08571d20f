"""Router calibration loss term and per-expert NLL attribution on the GPU.

Drop-in for ``_attach_surprise_telemetry`` / ``_attribute_nll_to_experts``
(mESmaC/spalmer src/spalmer/modeling.py:1468-1534): the model shell hands over
every layer's metrics and the next-token NLL; each layer's smooth-L1
calibration term and its ``expert_attributed_nll`` /
``potentiation_utilization`` are computed by ``spx_surprise_calibration``.
"""

from __future__ import annotations

from collections.abc import Mapping, Sequence
from typing import Any

import torch
from torch import Tensor

from spalmer_b200 import _lib


def layer_calibration(router_scores: Tensor, expert_ids: Tensor, routing_weights: Tensor, token_nll: Tensor,
                      valid: Tensor) -> tuple[Tensor, Tensor, Tensor]:
    """(calibration loss scalar, attributed NLL [E], responsibility utilization [E]) of one layer."""

    if router_scores.ndim != 3 or not router_scores.is_cuda:
        raise ValueError("router_scores must be a [batch, seq, experts] CUDA tensor")
    B, S, E = router_scores.shape
    k = expert_ids.shape[-1]
    if expert_ids.shape != (B, S, k) or routing_weights.shape != (B, S, k):
        raise ValueError("expert_ids / routing_weights must be [batch, seq, k]")
    if token_nll.shape != (B, S - 1) or valid.shape != (B, S - 1):
        raise ValueError("token_nll and valid must be [batch, seq - 1]")
    dev = router_scores.device
    scores = router_scores.to(torch.bfloat16).contiguous()
    ids = expert_ids.to(torch.int64).contiguous()
    weights = routing_weights.to(torch.bfloat16).contiguous()
    nll = token_nll.detach().to(device=dev, dtype=torch.float32).contiguous()
    v = valid.to(device=dev, dtype=torch.uint8).contiguous()
    lib = _lib.load()
    nbytes = lib.spx_calibration_workspace(B, S, E)
    ws = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=dev)
    cal = torch.empty((), dtype=torch.float32, device=dev)
    attributed = torch.empty(E, dtype=torch.float32, device=dev)
    utilization = torch.empty(E, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    _lib.check(lib.spx_surprise_calibration(scores.data_ptr(), ids.data_ptr(), weights.data_ptr(), nll.data_ptr(),
                                            v.data_ptr(), B, S, E, k, cal.data_ptr(), attributed.data_ptr(),
                                            utilization.data_ptr(), ws.data_ptr(), nbytes, stream),
               "spx_surprise_calibration")
    return cal, attributed, utilization


def attach_surprise_telemetry(layer_metrics: Sequence[Mapping[str, Any]], token_nll: Tensor,
                              valid: Tensor) -> tuple[tuple[Mapping[str, Any], ...], Tensor | None]:
    """``_attach_surprise_telemetry`` (modeling.py:1468-1510): per layer the
    calibration loss and the metrics enriched with ``expert_attributed_nll``
    and ``potentiation_utilization``; returns (enriched, mean calibration)."""

    enriched: list[Mapping[str, Any]] = []
    losses: list[Tensor] = []
    for metrics in layer_metrics:
        scores = metrics.get("router_scores")
        ids = metrics.get("expert_ids")
        weights = metrics.get("routing_weights")
        if not all(isinstance(v, Tensor) for v in (scores, ids, weights)):
            enriched.append(metrics)
            continue
        cal, attributed, utilization = layer_calibration(scores, ids, weights, token_nll, valid)
        losses.append(cal)
        updated = dict(metrics)
        updated["expert_attributed_nll"] = attributed
        updated["potentiation_utilization"] = utilization
        enriched.append(updated)
    total = torch.stack(losses).mean() if losses else None
    return tuple(enriched), total


__all__ = ["attach_surprise_telemetry", "layer_calibration"]
