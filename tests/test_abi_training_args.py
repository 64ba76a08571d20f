"""Host-side argument rules of the training entry points, checked on the CPU:
the sizes of the saved activations, and the pairs of spx_layer_outputs /
spx_layer_grads fields that must come together.  Every call here is refused
(or answered) before any device work, so the pointers are stand-ins that are
never dereferenced."""

from __future__ import annotations

import ctypes

from spalmer_b200 import _lib

SPX_ERR_INVALID_ARG = -1
FAKE = 0x10000  # 16-byte aligned, never dereferenced: the calls return before any launch


def _dims(**kw):
    base = dict(tokens=65536, d_model=768, num_experts=200, inter_dim=128, shared_dim=768, top_k=8,
                score_transform=0, execution_loop=0)
    base.update(kw)
    return _lib.LayerDims(**base)


def _weights():
    return _lib.PackedWeights(router_weight=FAKE, softplus_table=FAKE, expert_w1=FAKE, expert_w2=FAKE,
                              shared_w1=FAKE, shared_w2=FAKE)


def test_saved_activation_sizes():
    lib = _lib.load()
    cols = ctypes.c_int64()
    chunk = ctypes.c_int32()
    # 100M shape: one 128-column chunk of gate then up for the experts; six for the shared SwiGLU
    assert lib.spx_layer_saved_gu_cols(_dims(), cols) == 0 and cols.value == 256
    assert lib.spx_layer_saved_shared_gu(_dims(), cols, chunk) == 0
    assert (cols.value, chunk.value) == (6 * 256, 128)
    # a hidden width past one chunk: whole chunks of 128
    assert lib.spx_layer_saved_gu_cols(_dims(inter_dim=320), cols) == 0 and cols.value == 3 * 256
    assert lib.spx_layer_saved_gu_cols(_dims(inter_dim=80), cols) == 0 and cols.value == 160


def test_forward_saved_rows_come_in_pairs():
    lib = _lib.load()
    outs = _lib.LayerOutputs(update=FAKE, router_scores=FAKE, expert_ids=FAKE, routing_weights=FAKE,
                             saved_x=FAKE, saved_gu=None)
    assert lib.spx_layer_forward(_dims(), _weights(), FAKE, outs, FAKE, None) == SPX_ERR_INVALID_ARG
    outs = _lib.LayerOutputs(update=FAKE, router_scores=FAKE, expert_ids=FAKE, routing_weights=FAKE,
                             saved_x=None, saved_gu=FAKE)
    assert lib.spx_layer_forward(_dims(), _weights(), FAKE, outs, FAKE, None) == SPX_ERR_INVALID_ARG


def _grads(**kw):
    base = dict(expert_ids=FAKE, routing_weights=FAKE, router_scores=FAKE, gate_proj=FAKE, up_proj=FAKE,
                down_proj=FAKE, d_update=FAKE, d_hidden_experts=FAKE, d_logits=FAKE, x_sorted=FAKE,
                h_sorted=FAKE, du_sorted=FAKE, dgu_sorted=FAKE, expert_counts=FAKE)
    base.update(kw)
    return _lib.LayerGrads(**base)


def test_backward_forward_workspace_needs_utilization():
    lib = _lib.load()
    for gr in (_grads(forward_workspace=FAKE, expert_utilization=None),
               _grads(forward_workspace=None, expert_utilization=FAKE)):
        assert lib.spx_layer_backward(_dims(), _weights(), FAKE, gr, FAKE, None) == SPX_ERR_INVALID_ARG


def test_backward_saved_gu_needs_sorted_rows():
    lib = _lib.load()
    wg = dict(d_gate_proj=FAKE, d_up_proj=FAKE, d_down_proj=FAKE)
    # without x_sorted (rows gathered in-kernel) the forward's saved rows have nowhere to come from
    gr = _grads(x_sorted=None, du_sorted=None, saved_gu=FAKE, **wg)
    assert lib.spx_layer_backward(_dims(), _weights(), FAKE, gr, FAKE, None) == SPX_ERR_INVALID_ARG
    # x_sorted and du_sorted come together
    gr = _grads(du_sorted=None, **wg)
    assert lib.spx_layer_backward(_dims(), _weights(), FAKE, gr, FAKE, None) == SPX_ERR_INVALID_ARG
