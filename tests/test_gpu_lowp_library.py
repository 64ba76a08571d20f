"""Pin the block-scaled GEMMs of the low-precision lanes to a library.

The reference's MXFP8 and NVFP4 products come from torchao, which is not
installed; the quantisers are pinned to the restatement in ``oracle/`` (bit
for bit) and to torch's own ``float8_e4m3fn`` / ``float8_e8m0fnu`` casts.
Here the GEMM half is pinned as well: the E4M3/E8M0 (and E2M1/UE4M3) operands
this library's quantisers produce are handed to ``torch.nn.functional.
scaled_mm`` (cuBLASLt block-scaled GEMMs, 1x32 and 1x16 scale blocks in the
32x4x4 swizzled scale layout) and the result is compared with
``spx_mxfp8_mm_nt`` / ``spx_nvfp4_mm_nt`` on the same BF16 inputs.  Both
accumulate in FP32; they may differ in accumulation order only, so the BF16
outputs must agree within the contract's tolerance (rtol 2e-2, atol 1e-2) and
almost all of them bit for bit.  One GPU, local memory only.
"""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

from spalmer_b200.native import mx_quantize_rows, mxfp8_mm_nt, nvfp4_mm_nt, nvfp4_quantize_rows

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
RTOL, ATOL = 2e-2, 1e-2
SHAPES = ((256, 384, 768), (128, 256, 512), (512, 128, 256))


def swizzle_32_4_4(scales: torch.Tensor) -> torch.Tensor:
    """Scale bytes [rows, cols] -> the 32x4x4 block layout: 512-byte atoms of
    128 rows x 4 scale columns, row blocks outer, byte (r % 32) * 16 +
    (r // 32) * 4 + c inside an atom; rows and columns zero-padded."""

    rows, cols = scales.shape
    R, C = -(-rows // 128) * 128, -(-cols // 4) * 4
    pad = torch.zeros(R, C, dtype=torch.uint8, device=scales.device)
    pad[:rows, :cols] = scales
    atoms = pad.view(R // 128, 4, 32, C // 4, 4)      # [rb, r/32, r%32, cb, c]
    return atoms.permute(0, 3, 2, 1, 4).contiguous().view(-1)  # [rb, cb, r%32, r/32, c]


def _inputs(m, n, k, seed):
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(m, k, generator=g).to(torch.bfloat16).to(DEV)
    b = (0.02 * torch.randn(n, k, generator=g)).to(torch.bfloat16).to(DEV)
    return a, b


def _agree(got: torch.Tensor, want: torch.Tensor) -> None:
    g, w = got.float(), want.float()
    bad = (g - w).abs() > ATOL + RTOL * w.abs()
    assert not bool(bad.any()), f"{int(bad.sum())} outside tolerance; max diff {float((g - w).abs().max())}"
    assert float((got == want).float().mean()) >= 0.97


@pytest.mark.parametrize("m,n,k", SHAPES)
def test_mxfp8_gemm_matches_cublas_block_scaled(m, n, k):
    a, b = _inputs(m, n, k, 31)
    with torch.no_grad():
        ours = mxfp8_mm_nt(a, b)
        qa, sa = mx_quantize_rows(a)
        qb, sb = mx_quantize_rows(b)
        lib = F.scaled_mm(qa.view(torch.float8_e4m3fn), qb.view(torch.float8_e4m3fn).t(),
                          swizzle_32_4_4(sa).view(torch.float8_e8m0fnu), F.ScalingType.BlockWise1x32,
                          swizzle_32_4_4(sb).view(torch.float8_e8m0fnu), F.ScalingType.BlockWise1x32,
                          swizzle_a=F.SwizzleType.SWIZZLE_32_4_4, swizzle_b=F.SwizzleType.SWIZZLE_32_4_4,
                          output_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    assert lib.shape == ours.shape == (m, n)
    _agree(ours, lib)


@pytest.mark.parametrize("m,n,k", SHAPES)
def test_nvfp4_gemm_matches_cublas_block_scaled(m, n, k):
    """E2M1 pairs (even element in the low nibble) with UE4M3 scales per 16;
    the per-tensor factors amax/2688 of both operands multiply the FP32
    product once, as in spx_nvfp4_mm_nt."""

    a, b = _inputs(m, n, k, 32)
    with torch.no_grad():
        ours = nvfp4_mm_nt(a, b)
        qa, sa, amax_a = nvfp4_quantize_rows(a)
        qb, sb, amax_b = nvfp4_quantize_rows(b)
        kp = qa.shape[1] * 2
        assert kp == k  # k is a multiple of 256 here: no padding columns
        acc = F.scaled_mm(qa.view(torch.float4_e2m1fn_x2), qb.view(torch.float4_e2m1fn_x2).t(),
                          swizzle_32_4_4(sa).view(torch.float8_e4m3fn), F.ScalingType.BlockWise1x16,
                          swizzle_32_4_4(sb).view(torch.float8_e4m3fn), F.ScalingType.BlockWise1x16,
                          swizzle_a=F.SwizzleType.SWIZZLE_32_4_4, swizzle_b=F.SwizzleType.SWIZZLE_32_4_4,
                          output_dtype=torch.float32)
        pts = (amax_a / 2688.0) * (amax_b / 2688.0)
        lib = (acc * pts).to(torch.bfloat16)
    torch.cuda.synchronize()
    assert lib.shape == ours.shape == (m, n)
    _agree(ours, lib)
