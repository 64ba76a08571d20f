"""numpy restatement of the reference micro-expert channel mixer forward.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).  Every function names
the reference lines it restates (paths inside mESmaC/spalmer ``src/spalmer``).
BF16 tensors are ``uint16`` bit patterns; each place where the reference's
PyTorch CPU kernels materialise a BF16 tensor is an explicit RNE rounding here.
GEMMs accumulate in float32 (numpy/OpenBLAS), as PyTorch's CPU BF16 GEMMs do,
so results can differ from the reference in accumulation order only.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

from oracle.bf16 import bf16_bits_to_f32, f32_to_bf16_bits, f64_to_bf16_bits, round_bf16
from oracle.topk import topk_least

_SOFTPLUS_LUT: np.ndarray | None = None


def softplus_lut() -> np.ndarray:
    """BF16 -> BF16 table of ``F.softplus`` (beta=1, threshold=20).

    Restates ``experts/router.py:56``.  PyTorch's CPU kernel evaluates
    ``x > 20 ? x : log1p(exp(x))`` in float and rounds to BF16; over all 65536
    BF16 inputs that equals the correctly rounded value, which is what this
    table holds (pinned against torch in ``tests/test_oracle_golden.py``).
    """

    global _SOFTPLUS_LUT
    if _SOFTPLUS_LUT is None:
        bits = np.arange(65536, dtype=np.uint32).astype(np.uint16)
        x = bf16_bits_to_f32(bits).astype(np.float64)
        with np.errstate(over="ignore", invalid="ignore"):
            y = np.where(x > 20.0, x, np.log1p(np.exp(x)))
        out = f64_to_bf16_bits(y)
        keep = x > 20.0
        out[keep] = bits[keep]
        out[np.isnan(x)] = np.uint16(0x7FC0)
        _SOFTPLUS_LUT = out
    return _SOFTPLUS_LUT


def bf16_matmul(a_bits: np.ndarray, b_f32: np.ndarray) -> np.ndarray:
    """``a @ b`` with BF16 operands, float32 accumulation, BF16 result (bits)."""

    return f32_to_bf16_bits(bf16_bits_to_f32(a_bits) @ b_f32)


def router_logits(x_bits: np.ndarray, w_bits: np.ndarray, bias_bits: np.ndarray | None = None):
    """``self.proj(hidden_states)`` of ``experts/router.py:51`` (nn.Linear, BF16)."""

    acc = bf16_bits_to_f32(x_bits) @ bf16_bits_to_f32(w_bits).T
    if bias_bits is not None:
        acc = acc + bf16_bits_to_f32(bias_bits)[None, :]
    return f32_to_bf16_bits(acc)


def router_scores(logit_bits: np.ndarray, transform: str = "softplus") -> np.ndarray:
    """``experts/router.py:52-56``: identity (legacy) or softplus, BF16 out."""

    if transform == "identity":
        return np.array(logit_bits, dtype=np.uint16, copy=True)
    return softplus_lut()[logit_bits]


def routing_softmax(selected_bits: np.ndarray) -> np.ndarray:
    """``F.softmax(-selected_scores, dim=-1)`` of ``experts/router.py:94`` (BF16 out)."""

    neg = -bf16_bits_to_f32(selected_bits).astype(np.float64)
    m = neg.max(axis=-1, keepdims=True)
    with np.errstate(invalid="ignore"):
        e = np.exp(neg - m)
        p = e / e.sum(axis=-1, keepdims=True)
    return f64_to_bf16_bits(p)


def select_least_surprised(score_bits: np.ndarray, k: int, resident_mask: np.ndarray | None = None):
    """``select_least_surprised_experts`` of ``experts/router.py:59-95``.

    Returns ``(expert_ids int64 [T,k], routing_weight_bits uint16 [T,k])``.
    """

    n = score_bits.shape[-1]
    if not 1 <= k <= n:
        raise ValueError(f"num_active must be in [1, {n}]; got {k}")
    eligible = bf16_bits_to_f32(score_bits).reshape(-1, n).copy()
    if resident_mask is not None:
        eligible[:, ~np.asarray(resident_mask, dtype=bool)] = np.inf
    ids = topk_least(eligible, k)
    flat = score_bits.reshape(-1, n)
    selected = np.take_along_axis(flat, ids, axis=1)
    return ids.reshape(*score_bits.shape[:-1], k), routing_softmax(selected).reshape(
        *score_bits.shape[:-1], k
    )


def expert_utilization(expert_ids: np.ndarray, num_experts: int) -> np.ndarray:
    """``experts/losses.py:17-33``: pair fraction per expert (float32)."""

    flat = expert_ids.reshape(-1)
    counts = np.bincount(flat, minlength=num_experts).astype(np.float32)
    return counts / np.float32(flat.size)


def load_balance_loss(score_bits: np.ndarray, expert_ids: np.ndarray,
                      resident_mask: np.ndarray | None = None) -> float:
    """``experts/losses.py:36-70`` with its BF16 rounding points; returns the BF16 value."""

    n = score_bits.shape[-1]
    logits = -bf16_bits_to_f32(score_bits.reshape(-1, n)).astype(np.float64)
    if resident_mask is not None:
        mask = np.asarray(resident_mask, dtype=bool)
        logits[:, ~mask] = -np.inf
        eligible = float(mask.sum())
    else:
        eligible = float(n)
    m = logits.max(axis=-1, keepdims=True)
    e = np.exp(logits - m)
    prob = bf16_bits_to_f32(f64_to_bf16_bits(e / e.sum(axis=-1, keepdims=True)))
    mean_p = round_bf16((prob.astype(np.float64).sum(axis=0) / prob.shape[0]).astype(np.float32))
    frac = round_bf16(expert_utilization(expert_ids, n))
    prod = round_bf16(frac * mean_p)
    total = round_bf16(np.array([prod.astype(np.float64).sum()], dtype=np.float32))[0]
    elig = round_bf16(np.array([eligible], dtype=np.float32))[0]
    return float(round_bf16(np.array([elig * total], dtype=np.float32))[0])


def pair_counts(expert_index: np.ndarray, num_experts: int) -> np.ndarray:
    """``_pair_counts`` of ``experts/bank.py:981-985``."""

    return np.bincount(expert_index.reshape(-1), minlength=num_experts).astype(np.int64)


def dispatch_order(expert_index: np.ndarray) -> np.ndarray:
    """``torch.argsort(expert_index, stable=True)`` of ``experts/bank.py:723``."""

    return np.argsort(expert_index.reshape(-1), kind="stable").astype(np.int64)


def _silu_bf16(g_bits: np.ndarray) -> np.ndarray:
    g = bf16_bits_to_f32(g_bits)
    with np.errstate(over="ignore"):
        return f32_to_bf16_bits(g / (np.float32(1.0) + np.exp(-g)))


def _swiglu_rows(x_bits, gate_f32, up_f32, down_f32):
    """``silu(x@G)*(x@U) @ D`` with the BF16 rounding of ``experts/bank.py:760-763``."""

    g = bf16_matmul(x_bits, gate_f32)
    u = bf16_matmul(x_bits, up_f32)
    h = f32_to_bf16_bits(bf16_bits_to_f32(_silu_bf16(g)) * bf16_bits_to_f32(u))
    return bf16_matmul(h, down_f32)


def _swiglu_rows_mxfp8(x_bits, gate_io_bits, up_io_bits, down_io_bits):
    """``MicroExpertBank.expert_forward`` for the ("mxfp8", "mxfp8") pair (experts/bank.py:408-461).

    Each projection is ``native_expert_matmul(v, W)`` = ``_mxfp8_mm_nt(v, W.T)``
    (experts/native.py:113-140, 305-350): both operands quantised row-wise along K.
    """

    from oracle.mxfp8 import mxfp8_matmul_bits

    g = mxfp8_matmul_bits(x_bits, np.ascontiguousarray(gate_io_bits.T))
    u = mxfp8_matmul_bits(x_bits, np.ascontiguousarray(up_io_bits.T))
    h = f32_to_bf16_bits(bf16_bits_to_f32(_silu_bf16(g)) * bf16_bits_to_f32(u))
    return mxfp8_matmul_bits(h, np.ascontiguousarray(down_io_bits.T))


def _swiglu_rows_nvfp4(x_bits, gate_io_bits, up_io_bits, down_io_bits):
    """``expert_forward`` for the ("nvfp4", "nvfp4") pair: each projection is one
    ``native_expert_matmul`` call (experts/native.py:324-326 -> 224-262) over all
    of the expert's rows, so each operand gets one per-tensor scale per call."""

    from oracle.nvfp4 import nvfp4_matmul_bits

    g = nvfp4_matmul_bits(x_bits, np.ascontiguousarray(gate_io_bits.T))
    u = nvfp4_matmul_bits(x_bits, np.ascontiguousarray(up_io_bits.T))
    h = f32_to_bf16_bits(bf16_bits_to_f32(_silu_bf16(g)) * bf16_bits_to_f32(u))
    return nvfp4_matmul_bits(h, np.ascontiguousarray(down_io_bits.T))


def _next_pow2(n: np.ndarray) -> np.ndarray:
    out = np.ones_like(n)
    pos = n > 1
    out[pos] = 1 << np.ceil(np.log2(n[pos])).astype(np.int64)
    return out


def grouped_experts(x_bits: np.ndarray, expert_ids: np.ndarray, weight_bits: np.ndarray,
                    gate_bits: np.ndarray, up_bits: np.ndarray, down_bits: np.ndarray,
                    lane_mx: np.ndarray | None = None, execution: str = "grouped",
                    lane_nv: np.ndarray | None = None):
    """``MicroExpertBank._execute_grouped`` (``experts/bank.py:705-779``).

    ``x_bits [T,d]``, ``expert_ids [T,k]``, ``weight_bits [T,k]``; expert stacks
    ``gate/up [E,d,I]``, ``down [E,I,d]`` (BF16 bits).  Returns the routed
    update ``[T,d]`` (BF16 bits), reduced as the reference's ``index_add``
    calls reduce: grouped (bank.py:779) is one call over every pair in bucket
    order (buckets by padded capacity, then expert id, then sorted pair order),
    which torch's CPU index_add on BF16 accumulates in FP32 and rounds once;
    loop (bank.py:674-701) is one call per expert in ascending id order, a BF16
    rounding after each.  ``lane_mx[e]`` selects the MXFP8 pair for
    expert e (``_execution_pair``, bank.py:462-475); ``lane_nv[e]`` the NVFP4 pair.
    """

    T, d = x_bits.shape
    k = expert_ids.shape[-1]
    E = gate_bits.shape[0]
    ids = expert_ids.reshape(-1)
    P = ids.size
    counts = pair_counts(ids, E)
    starts = np.cumsum(counts) - counts
    order = dispatch_order(ids)
    w_bf = bf16_bits_to_f32(weight_bits.reshape(-1))
    weighted = np.zeros((P, d), dtype=np.float32)
    for e in np.nonzero(counts)[0]:
        rows = order[starts[e]: starts[e] + counts[e]]
        tokens = rows // k
        if lane_nv is not None and lane_nv[e]:
            y = _swiglu_rows_nvfp4(x_bits[tokens], gate_bits[e], up_bits[e], down_bits[e])
        elif lane_mx is not None and lane_mx[e]:
            y = _swiglu_rows_mxfp8(x_bits[tokens], gate_bits[e], up_bits[e], down_bits[e])
        else:
            y = _swiglu_rows(
                x_bits[tokens],
                bf16_bits_to_f32(gate_bits[e]),
                bf16_bits_to_f32(up_bits[e]),
                bf16_bits_to_f32(down_bits[e]),
            )
        # _weighted_expert_updates (bank.py:970-978): bf16(out) * bf16(w)
        weighted[rows] = round_bf16(bf16_bits_to_f32(y) * w_bf[rows][:, None])
    # index_add order per token: key (capacity(e), e) over the token's k slots.
    cap = _next_pow2(counts) if execution == "grouped" else np.zeros_like(counts)
    slot_e = ids.reshape(T, k)
    key = cap[slot_e] * (E + 1) + slot_e
    seq = np.argsort(key, axis=1, kind="stable")
    contrib = weighted.reshape(T, k, d)
    acc = np.zeros((T, d), dtype=np.float32)
    for j in range(k):
        step = np.take_along_axis(contrib, seq[:, j][:, None, None], axis=1)[:, 0, :]
        acc = acc + step if execution == "grouped" else round_bf16(acc + step)
    return f32_to_bf16_bits(acc), order, counts


def execute_routing(x_bits: np.ndarray, token_index: np.ndarray, expert_index: np.ndarray,
                    weight_bits: np.ndarray, gate_bits: np.ndarray, up_bits: np.ndarray, down_bits: np.ndarray,
                    *, execution: str = "grouped", resident_ids: np.ndarray | None = None,
                    lane_mx: np.ndarray | None = None) -> np.ndarray:
    """``MicroExpertBank.execute_routing`` for arbitrary (token, expert, weight)
    pairs (``experts/bank.py:593-646``): ``_execute_grouped`` (``bank.py:705-779``)
    or ``_execute_loop`` (``bank.py:674-703``).

    ``x_bits [N,d]``; ``token_index``, ``expert_index`` int ``[P]``;
    ``weight_bits [P]`` BF16.  Returns ``[N,d]`` BF16 bits: each pair's
    ``bf16(bf16(out) * w)`` index_added into BF16 zeros as the reference does
    -- grouped: one index_add over the pairs in bucket order (ascending
    power-of-two capacity, within a bucket the candidate experts in order --
    ``resident_ids`` order or ascending id -- within an expert the stable
    sorted pair order), pairs whose expert is not a candidate not executed;
    loop: one index_add per selected expert in ascending id order, pairs in
    index order.  torch's CPU index_add on BF16 adds a call's sources in FP32
    onto the FP32 value of the row and rounds once per call.
    """

    N, d = x_bits.shape
    E = gate_bits.shape[0]
    tok = np.asarray(token_index, dtype=np.int64).reshape(-1)
    ids = np.asarray(expert_index, dtype=np.int64).reshape(-1)
    w = bf16_bits_to_f32(np.asarray(weight_bits).reshape(-1))
    P = ids.size
    acc = np.zeros((N, d), dtype=np.float32)
    if P == 0:
        return f32_to_bf16_bits(acc)
    counts = pair_counts(ids, E)
    starts = np.cumsum(counts) - counts
    order = dispatch_order(ids)

    def run(e: int, rows: np.ndarray) -> np.ndarray:
        xs = x_bits[tok[rows]]
        if lane_mx is not None and lane_mx[e]:
            y = _swiglu_rows_mxfp8(xs, gate_bits[e], up_bits[e], down_bits[e])
        else:
            y = _swiglu_rows(xs, bf16_bits_to_f32(gate_bits[e]), bf16_bits_to_f32(up_bits[e]),
                             bf16_bits_to_f32(down_bits[e]))
        return round_bf16(bf16_bits_to_f32(y) * w[rows][:, None])

    if execution == "loop":
        seq = []
        for e in np.unique(ids):
            rows = np.nonzero(ids == e)[0]
            seq.append((rows, run(int(e), rows)))
    elif execution == "grouped":
        candidates = np.arange(E) if resident_ids is None else np.asarray(resident_ids, dtype=np.int64)
        groups = [int(e) for e in candidates if counts[e] > 0]
        cap = {e: int(_next_pow2(np.array([counts[e]]))[0]) for e in groups}
        seq = []
        for c in sorted(set(cap.values())):
            for e in (g for g in groups if cap[g] == c):
                rows = order[starts[e]: starts[e] + counts[e]]
                seq.append((rows, run(e, rows)))
    else:
        raise ValueError(f"unsupported expert execution mode: {execution!r}")
    def index_add(calls) -> None:  # each call: FP32 sums onto the rows, one rounding
        for rows, weighted in calls:
            touched = np.unique(tok[rows])
            for i, p in enumerate(rows):
                acc[tok[p]] = acc[tok[p]] + weighted[i]
            acc[touched] = round_bf16(acc[touched])

    if execution == "loop":
        index_add(seq)
    else:
        index_add([(np.concatenate([r for r, _ in seq]), np.concatenate([w_ for _, w_ in seq]))])
    return f32_to_bf16_bits(acc)


def shared_swiglu(x_bits, gate_w_bits, up_w_bits, down_w_bits):
    """``SwiGLU.forward`` of ``nn/ffn.py:27-30`` (nn.Linear weights ``[out,in]``)."""

    return _swiglu_rows(
        x_bits,
        bf16_bits_to_f32(gate_w_bits).T,
        bf16_bits_to_f32(up_w_bits).T,
        bf16_bits_to_f32(down_w_bits).T,
    )


def execution_metrics(expert_ids: np.ndarray, num_experts: int, execution: str = "grouped") -> dict:
    """``_expert_execution_metrics`` of ``experts/mixer.py:244-297`` (host ints/floats)."""

    counts = np.bincount(expert_ids.reshape(-1), minlength=num_experts).astype(np.int64)
    active = counts > 0
    groups = int(active.sum())
    max_load = int(counts.max())
    real = int(counts.sum())
    if execution == "grouped":
        padded = int(_next_pow2(counts[active]).sum())
    elif execution == "loop":
        padded = real
    else:
        raise ValueError(f"unsupported expert execution mode: {execution!r}")
    cf = max_load * groups
    return {
        "expert_group_count": groups,
        "expert_group_max_load": max_load,
        "expert_group_real_pairs": real,
        "expert_group_padded_pairs": padded,
        "expert_group_padding_amplification": float(np.float32(padded) / np.float32(real)),
        "expert_group_global_max_counterfactual_padded_pairs": cf,
        "expert_group_global_max_counterfactual_padding_amplification": float(
            np.float32(cf) / np.float32(real)
        ),
    }


@dataclass
class LayerParams:
    """BF16 bit patterns of one mixer's state_dict (reference key names in comments)."""

    router_w: np.ndarray            # router.proj.weight [E,d]
    gate: np.ndarray                # experts.gate_proj [E,d,I]
    up: np.ndarray                  # experts.up_proj [E,d,I]
    down: np.ndarray                # experts.down_proj [E,I,d]
    router_b: np.ndarray | None = None   # router.proj.bias [E]
    shared_gate: np.ndarray | None = None  # shared.gate_projection.weight [S,d]
    shared_up: np.ndarray | None = None    # shared.up_projection.weight [S,d]
    shared_down: np.ndarray | None = None  # shared.down_projection.weight [d,S]


def mixer_forward(params: LayerParams, x_bits: np.ndarray, k: int, *,
                  resident_mask: np.ndarray | None = None, transform: str = "softplus",
                  logit_bits: np.ndarray | None = None, lane_mx: np.ndarray | None = None,
                  execution: str = "grouped", lane_nv: np.ndarray | None = None) -> dict:
    """``MicroExpertChannelMixer.forward`` of ``experts/mixer.py:145-241``.

    ``x_bits [T,d]``.  ``logit_bits`` injects router logits (the bit-exact
    routing contract is stated "given identical logits").  ``lane_mx [E]``
    marks experts executed in MXFP8.
    """

    T, d = x_bits.shape
    E = params.router_w.shape[0]
    if logit_bits is None:
        logit_bits = router_logits(x_bits, params.router_w, params.router_b)
    scores = router_scores(logit_bits, transform)
    ids, weights = select_least_surprised(scores, k, resident_mask)
    routed, order, counts = grouped_experts(x_bits, ids, weights, params.gate, params.up, params.down,
                                            lane_mx=lane_mx, execution=execution, lane_nv=lane_nv)
    if params.shared_gate is not None:
        shared = shared_swiglu(x_bits, params.shared_gate, params.shared_up, params.shared_down)
        update = f32_to_bf16_bits(bf16_bits_to_f32(routed) + bf16_bits_to_f32(shared))
    else:
        shared = None
        update = routed
    util = expert_utilization(ids, E)
    return {
        "logits": logit_bits,
        "router_scores": scores,
        "expert_ids": ids,
        "routing_weights": weights,
        "order": order,
        "counts": counts,
        "routed": routed,
        "shared": shared,
        "update": update,
        "auxiliary_loss": load_balance_loss(scores, ids, resident_mask),
        "expert_utilization": util,
        "num_active_experts": int((util > 0).sum()),
        **execution_metrics(ids, E, execution),
    }


def isclose_bf16(a_bits: np.ndarray, b_bits: np.ndarray, rtol: float = 2e-2, atol: float = 1e-2) -> bool:
    a = bf16_bits_to_f32(a_bits).astype(np.float64)
    b = bf16_bits_to_f32(b_bits).astype(np.float64)
    return bool(np.all(np.abs(a - b) <= atol + rtol * np.abs(b)))


__all__ = [name for name in dir() if not name.startswith("_") and name not in {"annotations", "math"}]


def rms_norm(h_bits: np.ndarray, w_bits: np.ndarray, eps: float) -> np.ndarray:
    """``RMSNorm.forward`` of ``nn/norm.py:28-31`` on BF16 rows (bits in, bits out):
    variance in float32, ``rsqrt(variance + eps)`` cast to BF16, then the two
    BF16 products ``h * r`` and ``* weight``.  The float32 sum runs in numpy's
    pairwise order (the reference's order differs: ``r`` can move by one BF16
    ulp when the variance lands within a float ulp of a rounding boundary)."""

    h = bf16_bits_to_f32(h_bits)
    var = np.square(h, dtype=np.float32).mean(axis=-1, keepdims=True, dtype=np.float32)
    r = bf16_bits_to_f32(f32_to_bf16_bits((np.float32(1.0) / np.sqrt(var + np.float32(eps))).astype(np.float32)))
    x = f32_to_bf16_bits((h * r).astype(np.float32))
    return f32_to_bf16_bits((bf16_bits_to_f32(x) * bf16_bits_to_f32(w_bits)).astype(np.float32))


def block_channel_forward(h_bits: np.ndarray, norm_w_bits: np.ndarray, eps: float, update_bits: np.ndarray):
    """``hidden_states + channel_update`` of ``modeling.py:302`` in BF16 (bits)."""

    return f32_to_bf16_bits((bf16_bits_to_f32(h_bits) + bf16_bits_to_f32(update_bits)).astype(np.float32))


def reconstruction_error(w_t_bits: np.ndarray, weight_format: str) -> np.float32:
    """``native_weight_reconstruction_error`` (experts/native.py:391-417) of one
    expert matrix given as ``W^T`` [rows, K] (BF16 bits): the matrix packed the
    way its GEMM reads it -- MXFP8 row-wise along K in 32-value blocks, or
    NVFP4 in 16-value blocks under the matrix's own per-tensor scale -- then
    dequantised to BF16, and ``sum((W - restored)^2) / max(sum(W^2), 1e-12)``
    in float32 (the sums taken exactly and rounded once).  Zero padding of K
    (and of the rows for NVFP4) adds nothing."""

    w = bf16_bits_to_f32(w_t_bits).astype(np.float32)
    rows, K = w.shape
    if weight_format == "mxfp8":
        from oracle.mxfp8 import dequantize_rows, quantize_rows

        kp = -(-K // 32) * 32
        padded = np.zeros((rows, kp), dtype=np.float32)
        padded[:, :K] = w
        q, sb = quantize_rows(padded)
        restored = dequantize_rows(q, sb)[:, :K]
    elif weight_format == "nvfp4":
        from oracle.mxfp8 import E4M3_VALUES
        from oracle.nvfp4 import BLOCK, TENSOR_DIV, e2m1_values, quantize_rows

        codes, sb, amax = quantize_rows(w)
        pts = np.float32(np.float32(amax) / TENSOR_DIV)
        if not pts > 0:
            restored = np.zeros_like(w)
        else:
            total = (pts * E4M3_VALUES[sb]).astype(np.float32)  # the per-block scale torchao applies
            vals = e2m1_values(codes).reshape(rows, -1, BLOCK)
            restored = (vals * total[..., None]).astype(np.float32).reshape(rows, -1)[:, :K]
    elif weight_format in ("bfloat16", "float32"):
        return np.float32(0.0)
    else:
        raise ValueError(f"no packed representation for {weight_format!r}")
    restored = round_bf16(restored.astype(np.float32))
    diff = w.astype(np.float64) - restored.astype(np.float64)
    num = np.float32(np.sum(diff * diff))
    den = np.float32(max(np.float32(np.sum(w.astype(np.float64) ** 2)), np.float32(1e-12)))
    return np.float32(num / den)


def expert_reconstruction_errors(gate_bits: np.ndarray, up_bits: np.ndarray, down_bits: np.ndarray,
                                 weight_format: str, experts=None) -> np.ndarray:
    """``MicroExpertBank._quantization_error_for_rows`` (experts/bank.py:568-592):
    per expert, the mean of its gate, up and down reconstruction errors
    (each projection's ``expert_matrix.t()``), in float32.  ``experts``
    limits the computation to those ids (others stay 0)."""

    E = gate_bits.shape[0]
    out = np.zeros(E, dtype=np.float32)
    ids = range(E) if experts is None else experts
    for e in ids:
        eg = reconstruction_error(np.ascontiguousarray(gate_bits[e].T), weight_format)
        eu = reconstruction_error(np.ascontiguousarray(up_bits[e].T), weight_format)
        ed = reconstruction_error(np.ascontiguousarray(down_bits[e].T), weight_format)
        out[e] = np.float32(np.float32(np.float32(eg + eu) + ed) / np.float32(3.0))
    return out


def quantization_error(expert_ids: np.ndarray, gate_bits: np.ndarray, up_bits: np.ndarray, down_bits: np.ndarray,
                       weight_format: str) -> np.ndarray:
    """``MicroExpertBank.quantization_error`` (experts/bank.py:526-566): the
    reconstruction error of every expert selected in ``expert_ids``, zero for
    the others and for bfloat16 / float32 expert weights."""

    if weight_format in ("bfloat16", "float32"):
        return np.zeros(gate_bits.shape[0], dtype=np.float32)
    selected = np.unique(np.asarray(expert_ids).reshape(-1))
    return expert_reconstruction_errors(gate_bits, up_bits, down_bits, weight_format, experts=selected)
