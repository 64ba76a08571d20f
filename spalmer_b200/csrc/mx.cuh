// MXFP8 block quantisation on the device: E4M3 elements with one E8M0 scale
// per block of 32 consecutive K elements, scale chosen by the RCEIL rule.
//
// Reference: mESmaC/spalmer experts/native.py:91-110 calls torchao's
// MXTensor.to_mx(v, float8_e4m3fn, 32, ScaleCalculationMode.RCEIL); the
// published rule (OCP Microscaling Formats v1.0 with the RCEIL scale) is
//   descale = amax / 448, e = clamp(ceil(log2(descale)), -127, 127),
//   scale byte = e + 127, element = e4m3_rn(clamp(v * 2^-e, +-448)),
// with a multiplier of 1 for blocks whose scale byte is 0.  ceil(log2(.)) is
// taken exactly from the float's bits here.
#pragma once

#include <cuda_fp8.h>
#include <stdint.h>

#include "kernels.h"
#include "sm100.cuh"

namespace spx {

// E8M0 scale byte of a block whose largest magnitude is `amax` (finite, >= 0).
__device__ __forceinline__ uint32_t mx_scale_byte(float amax) {
  const float descale = amax / 448.0f;  // IEEE division (the build does not use fast math)
  if (!(descale > 0.0f)) return 0u;
  const uint32_t b = __float_as_uint(descale);
  const int ex = static_cast<int>((b >> 23) & 0xFFu);
  const uint32_t man = b & 0x7FFFFFu;
  int e;
  if (ex == 0) {
    e = (32 - __clz(static_cast<int>(man - 1u))) - 149;  // subnormal: ceil(log2(man)) - 149
  } else {
    e = ex - 127 + (man != 0u ? 1 : 0);
  }
  e = max(-127, min(127, e));
  return static_cast<uint32_t>(e + 127);
}

// Multiplier 2^-(byte-127) applied before the E4M3 cast; 1 for byte 0.
__device__ __forceinline__ float mx_multiplier(uint32_t byte) {
  if (byte == 0u) return 1.0f;
  const int neg_e = 127 - static_cast<int>(byte);   // -e, in [-127, 126]
  if (neg_e >= -126) return __uint_as_float(static_cast<uint32_t>(neg_e + 127) << 23);
  return __uint_as_float(0x00400000u);              // 2^-127 (subnormal)
}

// Two floats (already scaled) -> two E4M3 bytes, round to nearest even, clamped to +-448.
__device__ __forceinline__ uint32_t mx_e4m3x2(float lo, float hi) {
  lo = fminf(fmaxf(lo, -448.0f), 448.0f);
  hi = fminf(fmaxf(hi, -448.0f), 448.0f);
  return static_cast<uint32_t>(__nv_cvt_float2_to_fp8x2(make_float2(lo, hi), __NV_SATFINITE, __NV_E4M3));
}

// Quantise 32 values held by one thread: 8 words of E4M3 bytes (element j in
// byte j % 4 of word j / 4) and the block's scale byte.
__device__ __forceinline__ uint32_t mx_quantize32(const float (&v)[32], uint32_t (&q)[8]) {
  float amax = 0.0f;
#pragma unroll
  for (int j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(v[j]));
  const uint32_t sb = mx_scale_byte(amax);
  const float m = mx_multiplier(sb);
#pragma unroll
  for (int w = 0; w < 8; ++w) {
    const uint32_t p0 = mx_e4m3x2(v[4 * w] * m, v[4 * w + 1] * m);
    const uint32_t p1 = mx_e4m3x2(v[4 * w + 2] * m, v[4 * w + 3] * m);
    q[w] = p0 | (p1 << 16);
  }
  return sb;
}

// Byte offset of scale (row r of a 128-row tile, sub-block j of a 128-element
// K block) inside its 512-byte atom.  tcgen05.cp (32x128b, warpx4) copies the
// atom's 32 rows of 16 bytes to TMEM lanes 0..31 (replicated to the four lane
// quadrants); the block-scaled MMA then reads row r's scale for K sub-block j
// from column r / 32, byte j.
__host__ __device__ __forceinline__ int mx_atom_offset(int r, int j) { return (r & 31) * 16 + (r >> 5) * 4 + j; }

// Source element (row `row` of group `g`, K index `k`) of a B operand.
struct MxBSource {
  int mode;               // kMxSrcW1 / kMxSrcW2 / kMxSrcRows
  const uint16_t* a;      // W1: gate [E,d,I]; W2: down [E,I,d]; rows: [rows, ld]
  const uint16_t* b;      // W1: up [E,d,I]
  int d, inter, chunk;    // W1 / W2 shapes
  int64_t ld;             // rows: row stride
  int k_real;
  int rows_real;          // rows of one group that exist (beyond: zero)
};

__device__ __forceinline__ float mx_b_elem(const MxBSource& s, int g, int row, int k) {
  if (k >= s.k_real || row >= s.rows_real) return 0.0f;
  if (s.mode == kMxSrcW1) {
    const int ch = row / (2 * s.chunk);
    const int within = row - ch * 2 * s.chunk;
    const int half = within / s.chunk;
    const int i = ch * s.chunk + (within - half * s.chunk);
    if (i >= s.inter) return 0.0f;
    const uint16_t* p = half == 0 ? s.a : s.b;
    return bf16_to_f32(p[(static_cast<int64_t>(g) * s.d + k) * s.inter + i]);
  }
  if (s.mode == kMxSrcW2) return bf16_to_f32(s.a[(static_cast<int64_t>(g) * s.inter + k) * s.d + row]);
  return bf16_to_f32(s.a[static_cast<int64_t>(row) * s.ld + k]);
}

}  // namespace spx
