"""The routed experts' weight gradients on tcgen05 (wgrad.cu, reached through
spx_layer_backward): the rows gathered inside the kernels (no sorted copies)
bit for bit as from the sorted copies the backward GEMMs write on the side,
and against the library grouped GEMM (torch._grouped_mm) on the same sorted
rows -- both accumulate in FP32 and round once, so they
differ only by summation order (relative L2 < 2e-3, every element within
1e-2 + 2e-2 |want|) -- with ragged per-expert row counts (partial last K
blocks), experts that receive no rows (zero gradients), both batch classes
and the 100M widths."""

from __future__ import annotations

import pytest
import torch

from spalmer_b200 import B200MicroExpertChannelMixer, MicroExpertsConfig

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _inputs(config, tokens, seed=0):
    torch.manual_seed(seed)
    mixer = B200MicroExpertChannelMixer(config).to(torch.bfloat16).to(DEV).train()
    g = torch.Generator().manual_seed(seed + 1)
    x = torch.randn(tokens, config.d_model, generator=g).to(torch.bfloat16).to(DEV)
    du = (torch.randn(tokens, config.d_model, generator=g) * 0.1).to(torch.bfloat16).to(DEV)
    with torch.no_grad():
        out = mixer(x.unsqueeze(0))
    k = config.active_experts
    return mixer, x, out.metrics["expert_ids"].reshape(tokens, k), out.metrics["routing_weights"].reshape(tokens, k), \
        out.metrics["router_scores"].reshape(tokens, -1), du


def _relnorm(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / b.norm().clamp_min(1e-30)).item()


@pytest.mark.parametrize("tokens", [8, 300, 2048], ids=["tiny", "decode_class", "prefill_class"])
@pytest.mark.parametrize("shape", [dict(d_model=256, num_experts=40, expert_inter_dim=64, shared_inter_dim=0,
                                        active_experts=4),
                                   dict(d_model=768, num_experts=200, expert_inter_dim=128, shared_inter_dim=0,
                                        active_experts=8)], ids=["m10ish", "m100"])
def test_native_expert_wgrad_matches_library(shape, tokens):
    config = MicroExpertsConfig(**shape)
    mixer, x, ids, w, scores, du = _inputs(config, tokens)
    counts = torch.bincount(ids.reshape(-1), minlength=config.num_experts)
    if tokens * config.active_experts < config.num_experts:
        assert (counts == 0).any()  # experts without rows get zero gradients
    assert ((counts % 64) != 0).any()  # partial last K blocks
    native = mixer._backward_native(x, ids, w, scores, du, None, None, expert_wgrad="native")
    gathered = mixer._backward_native(x, ids, w, scores, du, None, None, expert_wgrad="native_gathered")
    library = mixer._backward_native(x, ids, w, scores, du, None, None, expert_wgrad="library")
    torch.cuda.synchronize()
    # rows gathered inside the weight-gradient kernels: the same operands in the same order
    for key in ("experts.gate_proj", "experts.up_proj", "experts.down_proj", "x"):
        assert torch.equal(gathered[key], native[key]), key
    for key in ("experts.gate_proj", "experts.up_proj", "experts.down_proj"):
        got, want = native[key], library[key]
        assert got.shape == want.shape and got.dtype == torch.bfloat16, key
        assert _relnorm(got, want) < 2e-3, (key, _relnorm(got, want))
        bad = (got.float() - want.float()).abs() > 1e-2 + 2e-2 * want.float().abs()
        assert not bad.any(), (key, int(bad.sum()))
        empty = counts == 0
        if empty.any():
            assert (got[empty] == 0).all(), key
    # the rest of the backward is the same call: bit for bit
    assert torch.equal(native["x"], library["x"])


@pytest.mark.parametrize("shape", [dict(d_model=256, num_experts=40, expert_inter_dim=80, shared_inter_dim=64,
                                        active_experts=4),
                                   dict(d_model=768, num_experts=200, expert_inter_dim=128, shared_inter_dim=768,
                                        active_experts=8)], ids=["m10ish_odd_inter", "m100"])
def test_saved_forward_activations_match_recompute(shape):
    """The training forward writes the dispatch-order hidden rows and the gate | up
    pre-activations from its expert GEMM1 (spx_layer_outputs.saved_x / saved_gu)
    and keeps the router logits; the backward given them skips its router GEMM and
    GEMM1 and must produce the same gradients, bit for bit, as the backward that
    recomputes them."""
    config = MicroExpertsConfig(**shape)
    tokens = 2048
    mixer, x, _, _, _, du = _inputs(config, tokens)
    saved = mixer._training_saves(x.unsqueeze(0))
    assert saved is not None
    with torch.no_grad():
        out = mixer._forward_native(x.unsqueeze(0), None, saved=saved)
    k = config.active_experts
    ids = out.metrics["expert_ids"].reshape(tokens, k)
    w = out.metrics["routing_weights"].reshape(tokens, k)
    scores = out.metrics["router_scores"].reshape(tokens, -1)
    # the saved rows are the token rows in dispatch order (stable sort of the expert ids)
    order = torch.argsort(ids.reshape(-1), stable=True)
    assert torch.equal(saved[0], x[order // k])
    # the forward's dispatch read back from its workspace (no forward since): the same gradients
    forward_ws = (mixer._last_forward[1], out.metrics["expert_utilization"])
    from_ws = mixer._backward_native(x, ids, w, scores, du, None, None, saved=saved, forward_ws=forward_ws)
    recomputed = mixer._backward_native(x, ids, w, scores, du, None, None)
    from_saved = mixer._backward_native(x, ids, w, scores, du, None, None, saved=saved)
    torch.cuda.synchronize()
    assert set(recomputed) == set(from_saved) == set(from_ws)
    for key in from_ws:
        assert torch.equal(from_ws[key], from_saved[key]), key
    # The shared SwiGLU's pre-activations come from the forward's tcgen05 GEMM
    # instead of a library GEMM (another summation order): its weights' and
    # the input's gradients agree within BF16 GEMM tolerance; the rest is bit
    # for bit.
    shared_keys = {"x"} | {key for key in recomputed if key.startswith("shared.")}
    if saved[3] is None:
        shared_keys = set()
    for key in recomputed:
        if key in shared_keys:
            got, want = from_saved[key].float(), recomputed[key].float()
            assert ((got - want).norm() / want.norm()).item() < 1e-2, key
        else:
            assert torch.equal(from_saved[key], recomputed[key]), key
    if saved[3] is not None:
        # the saved shared values are the forward's bf16 gate | up (chunk layout) of x
        sh = mixer.shared
        w1 = torch.cat([sh.gate_projection.weight, sh.up_projection.weight], 0).detach()
        ref = torch.nn.functional.linear(x, w1).float()
        gu, chunk = saved[3]
        S = sh.gate_projection.weight.shape[0]
        cols = torch.cat([torch.arange(n * 2 * chunk + h * chunk, n * 2 * chunk + (h + 1) * chunk)
                          for h in (0, 1) for n in range(S // chunk)]).to(gu.device)
        got = gu[:, cols].float()
        assert ((got - ref).norm() / ref.norm()).item() < 1e-2
