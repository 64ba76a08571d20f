"""PyTorch restatement of the reference mixer forward, for gradients.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).  The backward of the
routed micro-expert layer is checked against PyTorch autograd run through this
restatement on CPU, in BF16 like the reference: every operation below is the
one the reference applies, in the same order and dtype, so autograd takes the
same backward steps (paths inside mESmaC/spalmer ``src/spalmer``):

* router: ``softplus(F.linear(x, W, b))`` (``experts/router.py:51-56``);
* selection: resident mask to +inf, ``topk(largest=False)``, gather, softmax of
  the negated selected scores (``experts/router.py:80-95``);
* experts: per routed pair ``silu(x @ G_e) * (x @ U_e) @ D_e`` (the grouped
  path ``experts/bank.py:705-779`` batches pairs by expert; a pair's values do
  not depend on the batching), weighted in BF16 (``bank.py:970-978``) and
  index-added into a BF16 zero buffer;
* shared SwiGLU ``down(silu(gate x) * up x)`` (``nn/ffn.py:27-30``);
* load-balance loss ``m * sum_i f_i * mean_t softmax(-s)_ti`` with detached
  fractions (``experts/losses.py:36-70``).

Pinned against gradients of the reference module itself
(``tests/golden/make_backward.py`` -> ``tests/golden/backward_*.npz``,
checked by ``tests/test_backward_oracle.py``): the weight gradients agree bit
for bit, the input gradient up to the accumulation order of the index_add.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

PARAM_NAMES = (
    "router.proj.weight",
    "router.proj.bias",
    "experts.gate_proj",
    "experts.up_proj",
    "experts.down_proj",
    "shared.gate_projection.weight",
    "shared.up_projection.weight",
    "shared.down_projection.weight",
)


def forward(params: dict[str, torch.Tensor], x: torch.Tensor, top_k: int, *,
            identity_scores: bool = False, resident: torch.Tensor | None = None,
            ids: torch.Tensor | None = None):
    """Return ``(update, aux_loss, scores, ids, weights)`` for ``x`` [T, d] (BF16).

    ``params`` maps reference state_dict names to BF16 tensors (leaves that may
    require grad); absent names (no bias, no shared path) are skipped.  ``ids``
    ([T, k], optional) replaces the top-k selection -- for comparing gradients
    with an implementation whose router GEMM rounded a logit differently and
    so routed a token elsewhere; everything downstream follows the given ids.
    """

    num_tokens, d_model = x.shape
    bias = params.get("router.proj.bias")
    logits = F.linear(x, params["router.proj.weight"], bias)
    scores = logits if identity_scores else F.softplus(logits)

    eligible = scores
    if resident is not None:
        eligible = scores.masked_fill(~resident, torch.inf)
    if ids is None:
        ids = eligible.topk(top_k, dim=-1, largest=False).indices
    weights = F.softmax(-scores.gather(-1, ids), dim=-1)

    token_index = torch.arange(num_tokens).repeat_interleave(top_k)
    expert_index = ids.reshape(-1)
    flat_weights = weights.reshape(-1)
    gate, up, down = params["experts.gate_proj"], params["experts.up_proj"], params["experts.down_proj"]
    order = torch.argsort(expert_index, stable=True)
    rows, outs = [], []
    for e in torch.unique(expert_index).tolist():
        pairs = order[expert_index[order] == e]
        inputs = x[token_index[pairs]]
        hidden = F.silu(inputs @ gate[e]) * (inputs @ up[e])
        outputs = hidden @ down[e]
        rows.append(pairs)
        outs.append(outputs.to(x.dtype) * flat_weights.index_select(0, pairs).to(x.dtype).unsqueeze(-1))
    pair_rows = torch.cat(rows)
    update = x.new_zeros(num_tokens, d_model).index_add(0, token_index.index_select(0, pair_rows), torch.cat(outs))

    if "shared.gate_projection.weight" in params:
        shared = F.linear(
            F.silu(F.linear(x, params["shared.gate_projection.weight"]))
            * F.linear(x, params["shared.up_projection.weight"]),
            params["shared.down_projection.weight"],
        )
        update = update + shared

    num_experts = scores.shape[-1]
    lb_logits = -scores
    if resident is not None:
        lb_logits = lb_logits.masked_fill(~resident, -torch.inf)
        eligible_count = resident.to(lb_logits.dtype).sum()
    else:
        eligible_count = torch.tensor(float(num_experts), dtype=lb_logits.dtype)
    probabilities = F.softmax(lb_logits, dim=-1)
    mean_probability = probabilities.mean(dim=0)
    counts = torch.zeros(num_experts, dtype=torch.long).scatter_add_(0, expert_index, torch.ones_like(expert_index))
    fractions = (counts.to(torch.float32) / expert_index.numel()).to(mean_probability.dtype)
    aux = eligible_count * (fractions * mean_probability).sum()
    return update, aux, scores, ids, weights


def gradients(params: dict[str, torch.Tensor], x: torch.Tensor, top_k: int, d_update: torch.Tensor,
              d_aux: float, d_scores: torch.Tensor | None = None, **kw) -> dict[str, torch.Tensor]:
    """Gradients of ``sum(update * d_update) + d_aux * aux [+ sum(scores * d_scores)]``
    w.r.t. x and params."""

    leaves = {k: v.detach().clone().requires_grad_(True) for k, v in params.items()}
    xg = x.detach().clone().requires_grad_(True)
    update, aux, scores, *_ = forward(leaves, xg, top_k, **kw)
    outs, grads = [update, aux], [d_update, torch.tensor(d_aux, dtype=aux.dtype)]
    if d_scores is not None:
        outs.append(scores)
        grads.append(d_scores)
    torch.autograd.backward(outs, grads)
    out = {"x": xg.grad}
    for k, v in leaves.items():
        out[k] = v.grad if v.grad is not None else torch.zeros_like(v)
    return out
