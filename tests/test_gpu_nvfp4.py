"""NVFP4 on the GPU: the quantiser (spx_nvfp4_quantize_rows) bit for bit
against the restatement (oracle/nvfp4.py), and the block-scaled tcgen05
kind::mxf4nvf4 matmul (spx_nvfp4_mm_nt, the forward of the reference's
native_nvfp4_linear, experts/native.py:224-302) against the restatement's
matmul: the same quantised operands, FP32 accumulation in another order."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import nvfp4 as NV
from oracle.bf16 import bf16_bits_to_f32
from spalmer_b200 import _lib
from tests.helpers import bf16_bits, from_bits

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def rand_bf16(shape, scale=1.0, seed=0):
    g = torch.Generator().manual_seed(seed)
    return (scale * torch.randn(*shape, generator=g)).to(torch.bfloat16)


@pytest.mark.parametrize("rows,cols", [(300, 200), (64, 768), (1, 16), (129, 1000)])
def test_quantize_rows_matches_restatement(rows, cols):
    lib = _lib.load()
    x = rand_bf16((rows, cols), seed=rows)
    x[0, :3] = torch.tensor([0.0, -0.0, 1e-3])
    kp = NV.padded_k(cols)
    xd = x.to(DEV)
    q = torch.empty(rows, kp // 2, dtype=torch.uint8, device=DEV)
    sf = torch.empty(rows, kp // 16, dtype=torch.uint8, device=DEV)
    amax = torch.empty(1, dtype=torch.float32, device=DEV)
    st = torch.cuda.current_stream(DEV).cuda_stream
    assert lib.spx_nvfp4_quantize_rows(xd.data_ptr(), rows, cols, q.data_ptr(), sf.data_ptr(), amax.data_ptr(), st) == 0
    codes, sb, am = NV.quantize_rows(bf16_bits_to_f32(bf16_bits(x)))
    assert amax.item() == am
    np.testing.assert_array_equal(sf.cpu().numpy(), sb)
    np.testing.assert_array_equal(q.cpu().numpy(), NV.pack_codes(codes))


@pytest.mark.parametrize("m,n,k", [(256, 256, 512), (200, 96, 300), (1, 16, 64), (1000, 384, 768), (130, 40, 1024)])
def test_mm_nt_matches_restatement(m, n, k):
    lib = _lib.load()
    a = rand_bf16((m, k), seed=1)
    b = rand_bf16((n, k), scale=0.02, seed=2)
    ws = torch.empty(lib.spx_nvfp4_mm_workspace(m, n, k), dtype=torch.uint8, device=DEV)
    out = torch.empty(m, n, dtype=torch.bfloat16, device=DEV)
    st = torch.cuda.current_stream(DEV).cuda_stream
    ad, bd = a.to(DEV), b.to(DEV)
    assert lib.spx_nvfp4_mm_nt(ad.data_ptr(), bd.data_ptr(), m, n, k, out.data_ptr(), ws.data_ptr(), ws.numel(), st) == 0
    got = out.float().cpu().numpy()
    want = bf16_bits_to_f32(NV.nvfp4_matmul_bits(bf16_bits(a), bf16_bits(b)))
    # identical products, FP32 sums in another order: BF16 results within an ulp or two
    np.testing.assert_allclose(got, want, rtol=2e-2, atol=1e-3 * np.abs(want).max())
    assert (got == want).mean() > 0.9
    exact = a.float().numpy() @ b.float().numpy().T
    assert np.linalg.norm(got - exact) / np.linalg.norm(exact) < 0.30  # the reference's bound


# ---- the layer with NVFP4 experts (the ("nvfp4", "nvfp4") pair, promoted experts BF16)
from oracle import mixer_ref as R  # noqa: E402
from spalmer_b200 import B200MicroExpertChannelMixer, MicroExpertsConfig  # noqa: E402
from tests.helpers import mxfp8_experts, oracle_params, set_mxfp8_lanes  # noqa: E402

NV_LAYERS = {
    # decode-sized batch, d below 256 (K padding), loop telemetry
    "small": (dict(d_model=128, num_experts=32, expert_inter_dim=64, shared_inter_dim=128, active_experts=4,
                   expert_execution="loop"), (1, 96)),
    # throughput tiles, fused combine, I = 128 (256-column GEMM1 tiles)
    "wide": (dict(d_model=256, num_experts=48, expert_inter_dim=128, shared_inter_dim=256, active_experts=8,
                  expert_execution="loop"), (2, 384)),
}


def nv_config(**kw):
    kw.setdefault("expert_weight_format", "nvfp4")
    kw.setdefault("expert_activation_format", "nvfp4")
    kw.setdefault("expert_promotion_format", "bfloat16")
    return MicroExpertsConfig(**kw)


def relnorm(a, b):
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.mark.parametrize("name", list(NV_LAYERS))
@pytest.mark.parametrize("fraction", [0.5, 1.0])
def test_nvfp4_layer_matches_oracle_given_logits(name, fraction):
    cfg_kw, (batch, seq) = NV_LAYERS[name]
    config = nv_config(**cfg_kw)
    torch.manual_seed(0)
    mixer = B200MicroExpertChannelMixer(config).to(torch.bfloat16).eval().to(DEV)
    lane = mxfp8_experts(config.num_experts, fraction)
    set_mxfp8_lanes(mixer, lane)  # the unpromoted experts run the layer's low-precision (NVFP4) lane
    gen = torch.Generator().manual_seed(1)
    x = torch.randn(batch, seq, config.d_model, generator=gen).to(torch.bfloat16)
    x_bits = bf16_bits(x).reshape(-1, config.d_model)
    params = oracle_params(mixer)
    k = config.active_experts
    logits = R.router_logits(x_bits, params.router_w, params.router_b)
    with torch.no_grad():
        out = mixer(x.to(DEV), router_logits=from_bits(logits, DEV).reshape(batch, seq, -1))
    torch.cuda.synchronize()
    assert mixer.device_status() == 0
    want = R.mixer_forward(params, x_bits, k, logit_bits=logits, lane_nv=lane, execution="loop")
    assert np.array_equal(out.metrics["expert_ids"].cpu().numpy().reshape(-1, k), want["expert_ids"])
    got = bf16_bits_to_f32(bf16_bits(out.update).reshape(want["update"].shape)).astype(np.float64)
    ref = bf16_bits_to_f32(want["update"]).astype(np.float64)
    # Same quantiser, same products; a hidden value that rounds one BF16 ulp
    # apart (accumulation order, the epilogue's SiLU) can land on another E2M1
    # code, so the bound is on the whole update plus a per-element majority.
    assert relnorm(got, ref) < 2e-2, relnorm(got, ref)
    close = np.abs(got - ref) <= 1e-2 + 2e-2 * np.abs(ref)
    assert close.mean() > 0.97, close.mean()
    # and the NVFP4 lane is genuinely quantised: the all-BF16 layer differs
    set_mxfp8_lanes(mixer, np.zeros_like(lane))
    with torch.no_grad():
        out_bf16 = mixer(x.to(DEV), router_logits=from_bits(logits, DEV).reshape(batch, seq, -1))
    assert not torch.equal(out_bf16.update, out.update)


def test_reference_native_nvfp4_bound_and_provider():
    """test_native_precision.py's ("nvfp4", "nvfp4", 0.30) forward bound through the
    module-level helpers, the expert layout, and the provider claim."""

    from spalmer_b200.native import (native_expert_matmul, native_nvfp4_linear, native_provider_capabilities,
                                     nvfp4_quantize_rows)

    gen = torch.Generator(device="cpu").manual_seed(1204)
    x = torch.randn((7, 37), generator=gen).to(device=DEV, dtype=torch.bfloat16)
    w = torch.randn((23, 37), generator=gen).to(device=DEV, dtype=torch.bfloat16)
    out = native_nvfp4_linear(x, w)
    ref = x.float() @ w.float().t()
    rel = float((out.float() - ref).norm() / ref.norm().clamp_min(1e-12))
    assert rel < 0.30, rel
    out2 = native_expert_matmul(x, w.t().contiguous(), weight_format="nvfp4", activation_format="nvfp4")
    assert torch.equal(out2, out)
    values, scales, amax = nvfp4_quantize_rows(x)
    assert values.shape == (7, 128) and scales.shape == (7, 16)
    assert float(amax) == float(x.float().abs().max())
    claims = {c["weight_format"]: c for c in native_provider_capabilities(DEV)}
    assert claims["nvfp4"]["forward_available"] and not claims["nvfp4"]["backward_available"]
    assert claims["bfloat16"]["backward_available"]
