"""Helpers shared by the CPU and GPU tests."""

from __future__ import annotations

import hashlib

import numpy as np
import torch

from oracle.mixer_ref import LayerParams
from spalmer_b200.config import MicroExpertsConfig


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16).copy()


def from_bits(bits: np.ndarray, device=None) -> torch.Tensor:
    t = torch.from_numpy(np.ascontiguousarray(bits).view(np.int16).copy()).view(torch.bfloat16)
    return t if device is None else t.to(device)


def digest(t: torch.Tensor) -> str:
    t = t.detach().contiguous().cpu()
    raw = t.view(torch.int16).numpy() if t.dtype == torch.bfloat16 else t.numpy()
    return hashlib.sha256(raw.tobytes()).hexdigest()


def build_mixer(meta: dict, device=None):
    """The B200 mixer for a golden case, seeded exactly like the reference build."""

    from spalmer_b200 import B200MicroExpertChannelMixer
    from tests.golden.make_golden import zipf_bias

    config = MicroExpertsConfig(**meta["config"])
    torch.manual_seed(0)
    mixer = B200MicroExpertChannelMixer(config).to(torch.bfloat16).eval()
    if meta.get("bias_zipf") is not None:
        with torch.no_grad():
            mixer.router.proj.bias.copy_(zipf_bias(config.num_experts, meta["bias_zipf"]))
    if meta.get("resident"):
        mixer.residency.set(meta["resident"])
    if device is not None:
        mixer = mixer.to(device)
    return mixer


def oracle_params(mixer) -> LayerParams:
    sd = mixer.state_dict()
    get = lambda k: bf16_bits(sd[k]) if k in sd else None  # noqa: E731
    return LayerParams(
        router_w=get("router.proj.weight"),
        gate=get("experts.gate_proj"),
        up=get("experts.up_proj"),
        down=get("experts.down_proj"),
        router_b=get("router.proj.bias"),
        shared_gate=get("shared.gate_projection.weight"),
        shared_up=get("shared.up_projection.weight"),
        shared_down=get("shared.down_projection.weight"),
    )


def resident_mask(meta: dict) -> np.ndarray | None:
    if not meta.get("resident"):
        return None
    mask = np.zeros(meta["config"]["num_experts"], dtype=bool)
    mask[meta["resident"]] = True
    return mask


def mxfp8_experts(num_experts: int, fraction: float, seed: int = 2) -> np.ndarray:
    """Seeded MXFP8 expert set: the first ceil(fraction * E) of randperm(E, seed)."""

    import math

    gen = torch.Generator().manual_seed(seed)
    perm = torch.randperm(num_experts, generator=gen).numpy()
    lane = np.zeros(num_experts, dtype=bool)
    lane[perm[: math.ceil(fraction * num_experts)]] = True
    return lane


def mxfp8_config(**kw) -> MicroExpertsConfig:
    """MXFP8 expert weights whose promoted experts run BF16 (experts/bank.py:462-475)."""

    kw.setdefault("expert_weight_format", "mxfp8")
    kw.setdefault("expert_activation_format", "mxfp8")
    kw.setdefault("expert_promotion_format", "bfloat16")
    return MicroExpertsConfig(**kw)


def set_mxfp8_lanes(mixer, lane_mx: np.ndarray) -> None:
    """Run exactly the experts in `lane_mx` as MXFP8: promote (to BF16) all the others."""

    with torch.no_grad():
        mask = mixer.potentiation_controller.promoted_mask
        mask.copy_(torch.from_numpy(~lane_mx).to(mask.device))
