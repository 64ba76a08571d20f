// NVFP4 block quantisation on the device: E2M1 elements (two per byte, the
// even element in the low nibble) with one UE4M3 scale per block of 16
// consecutive K elements, relative to a per-tensor FP32 scale.
//
// Reference: mESmaC/spalmer experts/native.py:205-262 packs both operands of
// every NVFP4 matmul with torchao's NVFP4Tensor.to_nvfp4(v, per_tensor_scale=
// per_tensor_amax_to_scale(amax(|v|))).  torchao is not part of this build;
// its published algorithm, restated:
//   per_tensor_scale = amax / (448 * 6)                        (FP32)
//   per block of 16:  s = e4m3_rn(clamp((blk_amax / 6) / per_tensor_scale, 2^-6, 448))
//   element:          e2m1_rn(clamp(v / (per_tensor_scale * s), -6, 6))
// and the matmul multiplies the block-scaled product by the two per-tensor
// scales.  A tensor whose amax is 0 quantises to zeros here (the restated
// formula would divide by zero).
#pragma once

#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <stdint.h>

namespace spx {

constexpr int kNvBlock = 16;             // elements per UE4M3 scale
constexpr float kNvTensorDiv = 2688.0f;  // 448 (E4M3 max) * 6 (E2M1 max)
constexpr float kNvScaleMin = 0.015625f; // 2^-6, the smallest normal E4M3

// E2M1 code (sign in bit 3) of v, round to nearest even on the grid
// {0, 0.5, 1, 1.5, 2, 3, 4, 6}; |v| <= 6 expected (clamped by the caller).
// The grid has spacing 0.5 below 2, 1 on [2, 4] and 2 above, and its codes
// count along it, so one round-to-nearest-even to the spacing of |v|'s range
// gives the code: below 2 the code is rint(2|v|) (0..4), on [2, 4) it is
// rint(|v|) + 2 (4..6), from 4 it is rint(|v| / 2) + 4 (6..7).  The ties of
// the grid (0.25, 0.75, ..., 5) are the ties of these roundings, and the
// range boundaries 2 and 4 are grid points.
// Round-to-nearest-even of 0 <= x < 2^22 to an unsigned integer.  On the
// device: adding 1.5 * 2^23 lands x in a binade whose ulp is 1, so the float
// add itself rounds x to an integer (to even on ties) and the integer sits in
// the low mantissa bits -- one add instead of a round and a conversion on the
// special-function pipe, which the quantisers otherwise saturate.
__host__ __device__ __forceinline__ uint32_t nv_rne_small(float x) {
#if defined(__CUDA_ARCH__)
  return __float_as_uint(x + 12582912.0f) - 0x4B400000u;
#else
  return static_cast<uint32_t>(rintf(x));
#endif
}

__host__ __device__ __forceinline__ uint32_t nv_e2m1(float v) {
  const float m = fminf(fabsf(v), 6.0f);
  uint32_t c;
  if (m < 2.0f)
    c = nv_rne_small(2.0f * m);
  else if (m < 4.0f)
    c = nv_rne_small(m) + 2u;
  else
    c = nv_rne_small(0.5f * m) + 4u;
  return c | (signbit(v) ? 8u : 0u);
}

// The per-tensor scale of a tensor whose largest magnitude is amax.
__host__ __device__ __forceinline__ float nv_tensor_scale(float amax) { return amax / kNvTensorDiv; }

#if defined(__CUDACC__)
// Quantise 16 values with per-tensor scale `pts` (> 0): two words of E2M1
// nibbles (element j in bits 4*(j%8) .. of word j/8) and the UE4M3 scale byte.
__device__ __forceinline__ uint32_t nv_quantize16(const float (&v)[16], float pts, uint32_t& w0, uint32_t& w1) {
  w0 = w1 = 0u;
  if (!(pts > 0.0f)) return 0u;
  float amax = 0.0f;
#pragma unroll
  for (int j = 0; j < 16; ++j) amax = fmaxf(amax, fabsf(v[j]));
  float s = (amax / 6.0f) / pts;
  s = fminf(fmaxf(s, kNvScaleMin), 448.0f);
  const __nv_fp8_storage_t sb = __nv_cvt_float_to_fp8(s, __NV_SATFINITE, __NV_E4M3);
  const float sf = __half2float(__half(__nv_cvt_fp8_to_halfraw(sb, __NV_E4M3)));
  const float total = pts * sf;
  if (amax == 0.0f) {  // zeros (K padding): only the signs remain
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const uint32_t c = signbit(v[j]) ? 8u : 0u;
      if (j < 8)
        w0 |= c << (4 * j);
      else
        w1 |= c << (4 * (j - 8));
    }
    return static_cast<uint32_t>(sb);
  }
  // The code of v is nv_e2m1(RN(v / total)): it steps up where RN(v / total)
  // passes a rounding threshold of the E2M1 grid, i.e. where |v| passes that
  // threshold widened by half an ulp, times total.  Those seven boundaries
  // are exact in double (a 25-bit widened threshold times a 24-bit float) and
  // rounded to float toward the side that keeps the comparison exact, once
  // per block; each element then costs seven float compares instead of a
  // division.  Steps: above 0.25 (ties down), from 0.75 (ties up), above 1.25,
  // from 1.75, above 2.5, from 3.5, above 5 -- ties go to the even code.
  const double t = total;
  const float b0 = __double2float_rd((0.25 + 0x1p-26) * t), b1 = __double2float_ru((0.75 - 0x1p-25) * t);
  const float b2 = __double2float_rd((1.25 + 0x1p-24) * t), b3 = __double2float_ru((1.75 - 0x1p-24) * t);
  const float b4 = __double2float_rd((2.5 + 0x1p-23) * t), b5 = __double2float_ru((3.5 - 0x1p-23) * t);
  const float b6 = __double2float_rd((5.0 + 0x1p-22) * t);
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const float a = fabsf(v[j]);
    uint32_t c = (a > b0 ? 1u : 0u) + (a >= b1 ? 1u : 0u) + (a > b2 ? 1u : 0u) + (a >= b3 ? 1u : 0u) +
                 (a > b4 ? 1u : 0u) + (a >= b5 ? 1u : 0u) + (a > b6 ? 1u : 0u);
    c |= signbit(v[j]) ? 8u : 0u;
    if (j < 8)
      w0 |= c << (4 * j);
    else
      w1 |= c << (4 * (j - 8));
  }
  return static_cast<uint32_t>(sb);
}
#endif

}  // namespace spx
