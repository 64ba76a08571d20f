"""Generate backward golden vectors by running the reference (mESmaC/spalmer) itself.

Run in the build container, where the reference source is importable::

    python tests/golden/make_backward.py /path/to/reference/src

For each case the reference ``MicroExpertChannelMixer`` is built under
``torch.manual_seed(0)`` and cast to BF16 (the module under test regenerates
the same weights from the seed; SHA-256 digests of the state_dict prove it),
the input is ``torch.randn(B, S, d, generator=manual_seed(1))`` in BF16, and
the loss is ``sum(update * d_update) + d_aux * auxiliary_loss`` with
``d_update = 0.05 * randn(generator=manual_seed(5))`` in BF16.  Stored: the
input, ``d_update``, the forward's expert ids, and the gradients of the input
and of every parameter (BF16 bits), plus the digests and ``d_aux``.
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

BACKWARD_CASES = {
    # Decode-sized batch (the narrow-tile class): 128 tokens.
    "small": dict(cfg=dict(d_model=64, num_experts=16, expert_inter_dim=32,
                           shared_inter_dim=64, active_experts=4), shape=(2, 64)),
    # Large-batch class (512 tokens), k = 8, router bias.
    "large": dict(cfg=dict(d_model=128, num_experts=16, expert_inter_dim=64,
                           shared_inter_dim=128, active_experts=8, router_bias=True), shape=(2, 256)),
}
D_AUX = 0.25


def _bits(t: torch.Tensor) -> np.ndarray:
    t = t.detach().contiguous().cpu()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16).copy()
    return t.numpy().copy()


def _digest(t: torch.Tensor) -> str:
    t = t.detach().contiguous().cpu()
    raw = t.view(torch.int16).numpy() if t.dtype == torch.bfloat16 else t.numpy()
    return hashlib.sha256(raw.tobytes()).hexdigest()


def make_case(name: str, spec: dict) -> dict:
    from spalmer.experts import MicroExpertChannelMixer, MicroExpertsConfig

    config = MicroExpertsConfig(**spec["cfg"])
    torch.manual_seed(0)
    mixer = MicroExpertChannelMixer(config).to(torch.bfloat16).train()
    digests = {key: _digest(value) for key, value in mixer.state_dict().items()}
    batch, seq = spec["shape"]
    x = torch.randn(batch, seq, config.d_model, generator=torch.Generator().manual_seed(1)).to(torch.bfloat16)
    d_update = (0.05 * torch.randn(batch, seq, config.d_model, generator=torch.Generator().manual_seed(5)))
    d_update = d_update.to(torch.bfloat16)
    x.requires_grad_(True)
    out = mixer(x)
    torch.autograd.backward([out.update, out.auxiliary_loss],
                            [d_update, torch.tensor(D_AUX, dtype=out.auxiliary_loss.dtype)])
    arrays = dict(
        x=_bits(x.reshape(-1, config.d_model)),
        d_update=_bits(d_update.reshape(-1, config.d_model)),
        expert_ids=_bits(out.metrics["expert_ids"].reshape(-1, config.active_experts)).astype(np.int16),
        grad_x=_bits(x.grad.reshape(-1, config.d_model)),
    )
    grads = {}
    for pname, p in mixer.named_parameters():
        if p.grad is not None:
            arrays["grad__" + pname] = _bits(p.grad)
            grads[pname] = list(p.shape)
    meta = dict(name=name, config=asdict(config), shape=list(spec["shape"]), d_aux=D_AUX, grads=grads,
                digests=digests, aux_bf16=float(out.auxiliary_loss.detach().float()), torch=torch.__version__)
    arrays["meta"] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
    return arrays


def main() -> None:
    if len(sys.argv) > 1:
        sys.path.insert(0, sys.argv[1])
    for name, spec in BACKWARD_CASES.items():
        np.savez_compressed(HERE / f"backward_{name}.npz", **make_case(name, spec))
        print("wrote", name)


if __name__ == "__main__":
    main()
