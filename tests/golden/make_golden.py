"""Generate golden vectors by running the reference (mESmaC/spalmer) itself.

Run in the build container, where the reference source is importable::

    python tests/golden/make_golden.py /path/to/reference/src [--only name,name]

It writes small ``.npz`` fixtures next to this file.  The GPU box never runs
this script; tests there read only the committed fixtures.

Layer fixtures (``layer_<name>.npz``): the reference ``MicroExpertChannelMixer``
built under ``torch.manual_seed(0)`` and cast to BF16, input
``torch.randn(B, S, d, generator=torch.Generator().manual_seed(1))`` in BF16,
one forward under ``torch.no_grad()``.  Stored: input, router logits, every
metric the forward returns, the stable dispatch permutation, and SHA-256
digests of the state_dict tensors (the weights themselves are regenerated from
the seed by the module under test, and the digests prove it did so exactly).

Top-k fixtures (``topk_ties.npz``): tie-heavy BF16 score matrices generated
from seeded numpy PCG64 streams, with ``torch.topk(largest=False)`` indices
computed by the reference's arithmetic library (torch CPU).
"""

from __future__ import annotations

import hashlib
import json
import sys
from dataclasses import asdict
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from tests.golden.topk_cases import TOPK_CASES, generate_scores  # noqa: E402

LAYER_CASES = {
    # BASELINE config 0 (smoke): d=128, E=200, I=32, k=4, S=128, 2x256 tokens.
    "smoke": dict(cfg=dict(d_model=128, num_experts=200, expert_inter_dim=32,
                           shared_inter_dim=128, active_experts=4), shape=(2, 256)),
    # 10M-preset shape on a 2x128-token slice.
    "m10_slice": dict(cfg=dict(d_model=256, num_experts=200, expert_inter_dim=64,
                               shared_inter_dim=256, active_experts=8), shape=(2, 128)),
    # 100M-preset shape on a 1x128-token slice (all experts BF16).
    "m100_slice": dict(cfg=dict(d_model=768, num_experts=200, expert_inter_dim=128,
                                shared_inter_dim=768, active_experts=8), shape=(1, 128)),
    # k=2 takes torch's partial_sort branch (k*64 <= 200); no shared path.
    "k2_routed_only": dict(cfg=dict(d_model=64, num_experts=200, expert_inter_dim=32,
                                    shared_inter_dim=0, active_experts=2), shape=(2, 128)),
    # Router bias (Zipf-style) and a restricted resident set of 40 experts.
    "bias_resident": dict(cfg=dict(d_model=64, num_experts=200, expert_inter_dim=16,
                                   shared_inter_dim=64, active_experts=8, router_bias=True,
                                   max_resident_experts=64),
                          shape=(2, 128), bias_zipf=1.0, resident=40),
    # The loop executor (experts/bank.py:674-703): per-expert execution, index_add in
    # ascending expert order, loop telemetry (padded pairs = real pairs).
    "smoke_loop": dict(cfg=dict(d_model=128, num_experts=200, expert_inter_dim=32,
                                shared_inter_dim=128, active_experts=4, expert_execution="loop"),
                       shape=(2, 256)),
    "m10_loop": dict(cfg=dict(d_model=256, num_experts=200, expert_inter_dim=64,
                              shared_inter_dim=256, active_experts=8, expert_execution="loop"),
                     shape=(2, 128)),
    # Tiny bank like the reference's unit tests, legacy identity scores.
    "tiny_identity": dict(cfg=dict(d_model=16, num_experts=6, expert_inter_dim=8,
                                   active_experts=2, router_score_transform="identity"),
                          shape=(2, 5)),
}


def _bits(t: torch.Tensor) -> np.ndarray:
    t = t.detach().contiguous().cpu()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16).copy()
    return t.numpy().copy()


def _digest(t: torch.Tensor) -> str:
    t = t.detach().contiguous().cpu()
    raw = t.view(torch.int16).numpy() if t.dtype == torch.bfloat16 else t.numpy()
    return hashlib.sha256(raw.tobytes()).hexdigest()


def zipf_bias(num_experts: int, alpha: float, seed: int = 3) -> torch.Tensor:
    """``b_e = alpha * ln(rank_e)`` over a seeded permutation of expert ids."""

    perm = torch.randperm(num_experts, generator=torch.Generator().manual_seed(seed))
    rank = torch.empty(num_experts)
    rank[perm] = torch.arange(1, num_experts + 1, dtype=torch.float32)
    return alpha * torch.log(rank)


def make_layer(name: str, spec: dict) -> dict:
    from spalmer.experts import MicroExpertChannelMixer, MicroExpertsConfig

    config = MicroExpertsConfig(**spec["cfg"])
    torch.manual_seed(0)
    mixer = MicroExpertChannelMixer(config).to(torch.bfloat16).eval()
    if "bias_zipf" in spec:
        with torch.no_grad():
            mixer.router.proj.bias.copy_(zipf_bias(config.num_experts, spec["bias_zipf"]))
    resident = None
    if "resident" in spec:
        g = torch.Generator().manual_seed(4)
        resident = sorted(torch.randperm(config.num_experts, generator=g)[: spec["resident"]].tolist())
        mixer.residency.set(resident)
    batch, seq = spec["shape"]
    x = torch.randn(batch, seq, config.d_model, generator=torch.Generator().manual_seed(1))
    x = x.to(torch.bfloat16)
    with torch.no_grad():
        logits = mixer.router.proj(x)
        out = mixer(x)
    m = out.metrics
    ids = m["expert_ids"]
    order = torch.argsort(ids.reshape(-1), stable=True)
    counts = torch.bincount(ids.reshape(-1), minlength=config.num_experts)
    scalars = {
        key: float(m[key]) if m[key].is_floating_point() else int(m[key])
        for key in (
            "num_active_experts",
            "expert_group_count",
            "expert_group_max_load",
            "expert_group_real_pairs",
            "expert_group_padded_pairs",
            "expert_group_padding_amplification",
            "expert_group_global_max_counterfactual_padded_pairs",
            "expert_group_global_max_counterfactual_padding_amplification",
        )
    }
    digests = {key: _digest(value) for key, value in mixer.state_dict().items()}
    cfg_dict = {k: v for k, v in asdict(config).items()}
    meta = dict(
        name=name, config=cfg_dict, shape=list(spec["shape"]), resident=resident,
        bias_zipf=spec.get("bias_zipf"), scalars=scalars, digests=digests,
        aux_bf16=float(out.auxiliary_loss.float()), torch=torch.__version__,
    )
    arrays = dict(
        x=_bits(x.reshape(-1, config.d_model)),
        logits=_bits(logits.reshape(-1, config.num_experts)),
        router_scores=_bits(m["router_scores"].reshape(-1, config.num_experts)),
        expert_ids=_bits(ids.reshape(-1, ids.shape[-1])).astype(np.int16),
        routing_weights=_bits(m["routing_weights"].reshape(-1, ids.shape[-1])),
        update=_bits(out.update.reshape(-1, config.d_model)),
        expert_utilization=_bits(m["expert_utilization"]),
        order=_bits(order).astype(np.int32),
        counts=_bits(counts).astype(np.int32),
        router_bias=_bits(mixer.router.proj.bias) if mixer.router.proj.bias is not None
        else np.zeros(0, np.uint16),
        meta=np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8),
    )
    return arrays


def make_topk() -> dict:
    arrays: dict[str, np.ndarray] = {}
    for case in TOPK_CASES:
        scores_bits, mask = generate_scores(case)
        eligible = torch.from_numpy(scores_bits.view(np.int16)).view(torch.bfloat16)
        if mask is not None:
            eligible = eligible.masked_fill(~torch.from_numpy(mask), torch.inf)
        for k in case["ks"]:
            ids = eligible.topk(k, dim=-1, largest=False).indices
            arrays[f"{case['name']}__k{k}"] = ids.numpy().astype(np.int16)
        arrays[f"{case['name']}__sha256"] = np.frombuffer(
            hashlib.sha256(scores_bits.tobytes()).hexdigest().encode(), dtype=np.uint8
        )
    return arrays


def main() -> None:
    if len(sys.argv) > 1:
        sys.path.insert(0, sys.argv[1])
    torch.set_num_threads(max(1, torch.get_num_threads()))
    only = None
    if "--only" in sys.argv:
        only = set(sys.argv[sys.argv.index("--only") + 1].split(","))
    for name, spec in LAYER_CASES.items():
        if only is not None and name not in only:
            continue
        arrays = make_layer(name, spec)
        np.savez_compressed(HERE / f"layer_{name}.npz", **arrays)
        print("wrote", name)
    if only is None:
        np.savez_compressed(HERE / "topk_ties.npz", **make_topk())
        print("wrote topk_ties")


if __name__ == "__main__":
    main()
