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


def torch_layer_update(mixer, x: torch.Tensor, expert_ids: torch.Tensor, weights: torch.Tensor,
                       lane_mx: np.ndarray | None = None) -> torch.Tensor:
    """The layer update for every token, restated in FP32 torch ops on the
    tensors' device with the reference's BF16 rounding points, given the
    layer's own routing: per routed pair bf16(bf16(SwiGLU_e(x)) * w) with
    h = bf16(bf16(silu(bf16(x@G))) * bf16(x@U)) (experts/bank.py:755-763,
    970-978), the token's k pairs summed in FP32 and rounded once (the grouped
    executor's index_add), plus the shared SwiGLU (nn/ffn.py:27-30), rounded.
    Experts with lane_mx[e] run the ("mxfp8", "mxfp8") pair: each projection's
    operands quantised row-wise along K by the oracle's quantiser
    (experts/native.py:113-140), dequantised and multiplied in FP32.  The
    full-size tests check every row against it (and a token sample against the
    oracle); sums run in torch's order, so it is compared within the BF16
    tolerance."""

    from oracle.mxfp8 import dequantize_rows, quantize_rows

    def mx(t: torch.Tensor) -> torch.Tensor:  # [rows, K] FP32 -> deq(mx(rows)) on the same device
        q, sb = quantize_rows(t.float().cpu().numpy())
        return torch.from_numpy(dequantize_rows(q, sb)).to(t.device)

    def mx_mm(a: torch.Tensor, w_io: torch.Tensor) -> torch.Tensor:  # a [n, K] @ w_io [K, N], both quantised along K
        return mx(a) @ mx(w_io.float().T.contiguous()).T

    def bf(t: torch.Tensor) -> torch.Tensor:
        return t.to(torch.bfloat16).float()

    prev_tf32 = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        sd = mixer.state_dict()
        dev = x.device
        T, d = x.shape
        k = expert_ids.shape[1]
        xf = x.float()
        flat = expert_ids.reshape(-1).to(dev)
        order = torch.argsort(flat, stable=True)
        counts = torch.bincount(flat, minlength=sd["experts.gate_proj"].shape[0]).tolist()
        wf = weights.reshape(-1).to(dev).float()
        weighted = torch.zeros(T * k, d, dtype=torch.float32, device=dev)
        start = 0
        for e, n in enumerate(counts):
            if n == 0:
                continue
            rows = order[start:start + n]
            start += n
            xe = xf[rows // k]
            gate_e, up_e, down_e = (sd[f"experts.{n}_proj"][e].to(dev).float() for n in ("gate", "up", "down"))
            mm = mx_mm if lane_mx is not None and lane_mx[e] else torch.matmul
            g = bf(mm(xe, gate_e))
            u = bf(mm(xe, up_e))
            h = bf(bf(torch.nn.functional.silu(g)) * u)
            y = bf(mm(h, down_e))
            weighted[rows] = bf(y * wf[rows, None])
        routed = bf(weighted.view(T, k, d).sum(dim=1))
        if "shared.gate_projection.weight" in sd:
            sg = bf(xf @ sd["shared.gate_projection.weight"].to(dev).float().T)
            su = bf(xf @ sd["shared.up_projection.weight"].to(dev).float().T)
            sh = bf(bf(torch.nn.functional.silu(sg)) * su)
            routed = bf(routed + bf(sh @ sd["shared.down_projection.weight"].to(dev).float().T))
        return routed.to(torch.bfloat16)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev_tf32
