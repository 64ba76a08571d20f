"""Golden vectors for the bank seam, made by running the reference itself.

    python tests/golden/make_bank.py /path/to/reference/src

Runs ``MicroExpertBank.execute_routing`` of the reference (mESmaC/spalmer
src/spalmer/experts/bank.py:593-646) on arbitrary (token, expert, weight)
pairs -- ragged pairs per token, tokens without pairs, a token with more
pairs than a layer's top-k, a restricted resident set -- with the bank of a
``MicroExpertChannelMixer`` built under ``torch.manual_seed(0)`` and cast to
BF16 (smoke widths).  Writes ``bank_pairs.npz`` next to this file: inputs,
pairs and the reference's output per case, plus the state_dict digests of the
bank.  The GPU box never runs this script.
"""

from __future__ import annotations

import hashlib
import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent

CFG = dict(d_model=128, num_experts=200, expert_inter_dim=32, shared_inter_dim=128, active_experts=4)
TOKENS = 64


def _bits(t: torch.Tensor) -> np.ndarray:
    t = t.detach().contiguous().cpu()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16).copy()
    return t.numpy().copy()


def _digest(t: torch.Tensor) -> str:
    t = t.detach().contiguous().cpu()
    raw = t.view(torch.int16).numpy() if t.dtype == torch.bfloat16 else t.numpy()
    return hashlib.sha256(raw.tobytes()).hexdigest()


def pairs(seed: int) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """Ragged pairs: tokens 48..63 get none, token 5 gets 30, the rest a few each."""

    rng = np.random.default_rng(seed)
    tok = [5] * 30
    for t in range(48):
        tok += [t] * int(rng.integers(1, 9))
    tok = np.array(tok, dtype=np.int64)
    rng.shuffle(tok)
    p = 1.0 / np.arange(1, CFG["num_experts"] + 1) ** 1.1
    p /= p.sum()
    ids = rng.choice(CFG["num_experts"], size=tok.size, p=p).astype(np.int64)
    w = torch.from_numpy(rng.uniform(0.05, 1.0, size=tok.size).astype(np.float32)).to(torch.bfloat16)
    return tok, ids, _bits(w)


def main() -> None:
    if len(sys.argv) > 1:
        sys.path.insert(0, sys.argv[1])
    from spalmer.experts import MicroExpertChannelMixer, MicroExpertsConfig

    x = torch.randn(TOKENS, CFG["d_model"], generator=torch.Generator().manual_seed(1)).to(torch.bfloat16)
    arrays: dict[str, np.ndarray] = {"x": _bits(x)}
    cases = {}
    for name, execution, seed, resident in (("grouped", "grouped", 21, None), ("loop", "loop", 21, None),
                                            ("resident", "grouped", 22, 60)):
        config = MicroExpertsConfig(**CFG, expert_execution=execution)
        torch.manual_seed(0)
        mixer = MicroExpertChannelMixer(config).to(torch.bfloat16).eval()
        bank = mixer.experts
        tok, ids, w_bits = pairs(seed)
        resident_ids = None
        if resident is not None:
            perm = torch.randperm(CFG["num_experts"], generator=torch.Generator().manual_seed(seed))
            resident_ids = perm[:resident].clone()
        with torch.no_grad():
            out = bank.execute_routing(
                x, torch.from_numpy(tok), torch.from_numpy(ids),
                torch.from_numpy(w_bits.view(np.int16)).view(torch.bfloat16),
                None, resident_ids,
            )
        arrays[f"{name}__token_index"] = tok.astype(np.int32)
        arrays[f"{name}__expert_index"] = ids.astype(np.int32)
        arrays[f"{name}__weights"] = w_bits
        arrays[f"{name}__update"] = _bits(out)
        if resident_ids is not None:
            arrays[f"{name}__resident_ids"] = resident_ids.numpy().astype(np.int32)
        cases[name] = {"execution": execution}
        digests = {key: _digest(value) for key, value in bank.state_dict().items()}
    meta = {"config": CFG, "tokens": TOKENS, "cases": cases, "digests": digests, "torch": torch.__version__}
    arrays["meta"] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
    np.savez_compressed(HERE / "bank_pairs.npz", **arrays)
    print("wrote bank_pairs.npz")


if __name__ == "__main__":
    main()
