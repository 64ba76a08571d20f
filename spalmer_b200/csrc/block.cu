// The channel half of a block around the layer (mESmaC/spalmer
// src/spalmer/modeling.py:283-302): normalized = channel_norm(h), then
// h + channel_mixer(normalized).update.  This file holds the RMSNorm
// (nn/norm.py:28-31); the residual add rides on the combine (gemm.cu
// kEpiCombine, pack.cu combine_kernel).
//
//   x = bf16(bf16(h * bf16(rsqrt(mean_d(float(h)^2) + eps))) * w)
//
// One warp per row; a lane keeps its 16-byte chunks of the row in registers
// between the sum of squares and the scaling.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "kernels.h"
#include "sm100.cuh"

namespace spx {

namespace {
constexpr int kNormMaxChunks = 8;  // 16-byte chunks per lane: d <= 2048 on the register path

__device__ __forceinline__ uint32_t mul_bf16x2_rn(uint32_t a, float s) {
  const float lo = __uint_as_float(a << 16) * s, hi = __uint_as_float(a & 0xFFFF0000u) * s;
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ uint32_t mul_bf16x2_rn(uint32_t a, uint32_t b) {
  const float lo = __uint_as_float(a << 16) * __uint_as_float(b << 16);
  const float hi = __uint_as_float(a & 0xFFFF0000u) * __uint_as_float(b & 0xFFFF0000u);
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ uint4 norm_chunk(const uint4& h, const uint4& w, float r) {
  return make_uint4(mul_bf16x2_rn(mul_bf16x2_rn(h.x, r), w.x), mul_bf16x2_rn(mul_bf16x2_rn(h.y, r), w.y),
                    mul_bf16x2_rn(mul_bf16x2_rn(h.z, r), w.z), mul_bf16x2_rn(mul_bf16x2_rn(h.w, r), w.w));
}

__device__ __forceinline__ float sumsq_chunk(const uint4& h) {
  const uint32_t u[4] = {h.x, h.y, h.z, h.w};
  float s = 0.0f;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float lo = __uint_as_float(u[q] << 16), hi = __uint_as_float(u[q] & 0xFFFF0000u);
    s += lo * lo + hi * hi;
  }
  return s;
}
}  // namespace

__global__ void rmsnorm_rows_kernel(const uint16_t* __restrict__ h, const uint16_t* __restrict__ w, float eps,
                                    int64_t rows, int d, uint16_t* __restrict__ out, int ld_out) {
  const int lane = threadIdx.x & 31;
  const int nchunks = d / 8;
  const int64_t nwarps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t row = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5); row < rows;
       row += nwarps) {
    const uint4* hr = reinterpret_cast<const uint4*>(h + row * d);
    uint4 hv[kNormMaxChunks];
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < kNormMaxChunks; ++i) {
      const int c = lane + 32 * i;
      if (c < nchunks) {
        hv[i] = __ldg(hr + c);
        s += sumsq_chunk(hv[i]);
      }
    }
    for (int c = lane + 32 * kNormMaxChunks; c < nchunks; c += 32) s += sumsq_chunk(__ldg(hr + c));
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) s += __shfl_xor_sync(0xFFFFFFFFu, s, off);
    // rsqrt(variance + eps) in float, then the reference's cast to BF16
    const float r = __bfloat162float(__float2bfloat16_rn(1.0f / sqrtf(s / static_cast<float>(d) + eps)));
    uint4* orow = reinterpret_cast<uint4*>(out + row * ld_out);
    const uint4* wr = reinterpret_cast<const uint4*>(w);
#pragma unroll
    for (int i = 0; i < kNormMaxChunks; ++i) {
      const int c = lane + 32 * i;
      if (c < nchunks) orow[c] = norm_chunk(hv[i], __ldg(wr + c), r);
    }
    for (int c = lane + 32 * kNormMaxChunks; c < nchunks; c += 32) orow[c] = norm_chunk(__ldg(hr + c), __ldg(wr + c), r);
    for (int c = nchunks + lane; c < ld_out / 8; c += 32) orow[c] = make_uint4(0u, 0u, 0u, 0u);  // K padding
  }
}

int launch_rmsnorm_rows(const uint16_t* h, const uint16_t* w, float eps, int64_t rows, int d, uint16_t* out,
                        int ld_out, cudaStream_t stream) {
  if (rows <= 0) return SPX_OK;
  if (d % 8 != 0 || ld_out % 8 != 0 || ld_out < d || !(eps > 0.0f)) return SPX_ERR_INVALID_ARG;
  if ((reinterpret_cast<uintptr_t>(h) & 15u) != 0 || (reinterpret_cast<uintptr_t>(w) & 15u) != 0 ||
      (reinterpret_cast<uintptr_t>(out) & 15u) != 0)
    return SPX_ERR_ALIGNMENT;
  int64_t blocks = (rows + 7) / 8;
  if (blocks > 148 * 16) blocks = 148 * 16;
  rmsnorm_rows_kernel<<<static_cast<int>(blocks), 256, 0, stream>>>(h, w, eps, rows, d, out, ld_out);
  return cudaGetLastError() == cudaSuccess ? SPX_OK : SPX_ERR_CUDA;
}

}  // namespace spx
