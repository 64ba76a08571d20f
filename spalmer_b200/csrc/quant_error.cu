// Reconstruction error of each expert's low-precision copies: the telemetry
// MicroExpertBank.quantization_error reports (mESmaC/spalmer
// src/spalmer/experts/bank.py:526-592) with native_weight_reconstruction_error
// (experts/native.py:391-417).  For each projection W of expert e (gate and
// up [d, I], down [I, d]) the matrix W^T is quantised row-wise along its K
// axis -- the packing the expert GEMMs read -- and
//
//   err(W) = sum((W - bf16(deq(q(W^T)))^T)^2) / max(sum(W^2), 1e-12)
//
// with both sums in FP32 (accumulated here in double and rounded once, so the
// result does not depend on an FP32 summation order); the expert's error is
// (err(gate) + err(up) + err(down)) / 3 in FP32.  MXFP8: 32-value blocks with
// E8M0 scales (mx_quantize32); NVFP4: 16-value blocks with UE4M3 scales under
// one per-tensor scale amax / 2688 of the matrix (nv_quantize16), restored as
// e2m1 * (pts * scale).  Zero K padding quantises to zero and adds nothing.
//
// The weights are static between updates, so the errors are computed once per
// pack (spx_expert_quant_error) and each forward's dispatch writes the
// selected experts' entries (zero for the others).
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "kernels.h"
#include "mx.cuh"
#include "nv.cuh"
#include "sm100.cuh"

namespace spx {

namespace {

constexpr int kErrThreads = 256;

// Block-wide sum of doubles (every thread receives it).
__device__ __forceinline__ double block_sum(double v, double* red) {
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, off);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  double t = 0.0;
  for (int w = 0; w < kErrThreads / 32; ++w) t += red[w];
  return t;
}

__device__ __forceinline__ float block_max_f(float v, float* red) {
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, off));
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.0f;
  for (int w = 0; w < kErrThreads / 32; ++w) t = fmaxf(t, red[w]);
  return t;
}

__device__ __forceinline__ float e4m3_byte_value(uint32_t b) {
  return __half2float(__half(__nv_cvt_fp8_to_halfraw(static_cast<__nv_fp8_storage_t>(b), __NV_E4M3)));
}

__device__ __forceinline__ float e2m1_code_value(uint32_t c) {
  const float mag[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};
  const float v = mag[c & 7u];
  return (c & 8u) ? -v : v;
}

// err(W) for one matrix given in the reference layout: element (r, k) of W^T
// is w[k * R + r] (R rows, K along the quantised axis).
template <int FMT>
__device__ float matrix_error(const uint16_t* __restrict__ w, int R, int K, double* red, float* redf) {
  constexpr int B = FMT == 1 ? kMxBlock : kNvBlock;
  const int nblk = (K + B - 1) / B;
  float pts = 0.0f;
  if (FMT == 2) {
    float m = 0.0f;
    for (int64_t i = threadIdx.x; i < static_cast<int64_t>(R) * K; i += blockDim.x) m = fmaxf(m, fabsf(bf16_to_f32(w[i])));
    pts = nv_tensor_scale(block_max_f(m, redf));
  }
  double d2 = 0.0, w2 = 0.0;
  // thread -> (row r, block b): consecutive threads read consecutive r
  for (int64_t item = threadIdx.x; item < static_cast<int64_t>(R) * nblk; item += blockDim.x) {
    const int r = static_cast<int>(item % R), b = static_cast<int>(item / R);
    float v[B];
#pragma unroll
    for (int j = 0; j < B; ++j) {
      const int k = b * B + j;
      v[j] = k < K ? bf16_to_f32(w[static_cast<int64_t>(k) * R + r]) : 0.0f;
    }
    float back[B];
    if constexpr (FMT == 1) {
      float vv[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) vv[j] = v[j];
      uint32_t q[8];
      const uint32_t sb = mx_quantize32(vv, q);
      const float s = sb == 0u ? __uint_as_float(0x00400000u) : __uint_as_float(sb << 23);  // 2^(sb - 127)
#pragma unroll
      for (int j = 0; j < 32; ++j) back[j] = round_bf16(e4m3_byte_value((q[j / 4] >> (8 * (j % 4))) & 0xFFu) * s);
    } else {
      float vv[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) vv[j] = v[j];
      uint32_t w0, w1;
      const uint32_t sb = nv_quantize16(vv, pts, w0, w1);
      const float total = pts * e4m3_byte_value(sb);
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const uint32_t c = ((j < 8 ? w0 : w1) >> (4 * (j % 8))) & 0xFu;
        back[j] = pts > 0.0f ? round_bf16(e2m1_code_value(c) * total) : 0.0f;
      }
    }
#pragma unroll
    for (int j = 0; j < B; ++j) {
      const double diff = static_cast<double>(v[j]) - static_cast<double>(back[j]);
      d2 += diff * diff;
      w2 += static_cast<double>(v[j]) * static_cast<double>(v[j]);
    }
  }
  const float num = static_cast<float>(block_sum(d2, red));
  const float den = fmaxf(static_cast<float>(block_sum(w2, red)), 1e-12f);
  return num / den;
}

// One CTA per expert.
template <int FMT>
__global__ void __launch_bounds__(kErrThreads) expert_quant_error_kernel(const uint16_t* __restrict__ gate,
                                                                         const uint16_t* __restrict__ up,
                                                                         const uint16_t* __restrict__ down, int d,
                                                                         int inter, float* __restrict__ out) {
  __shared__ double red[kErrThreads / 32];
  __shared__ float redf[kErrThreads / 32];
  const int64_t e = blockIdx.x;
  const int64_t n = static_cast<int64_t>(d) * inter;
  // gate / up [d, I]: W^T has I rows, K = d; down [I, d]: W^T has d rows, K = I
  const float eg = matrix_error<FMT>(gate + e * n, inter, d, red, redf);
  const float eu = matrix_error<FMT>(up + e * n, inter, d, red, redf);
  const float ed = matrix_error<FMT>(down + e * n, d, inter, red, redf);
  if (threadIdx.x == 0) out[e] = ((eg + eu) + ed) / 3.0f;
}

}  // namespace

int launch_expert_quant_error(const uint16_t* gate, const uint16_t* up, const uint16_t* down, int E, int d, int inter,
                              int format, float* out, cudaStream_t stream) {
  if (E <= 0 || d <= 0 || inter <= 0) return SPX_ERR_INVALID_ARG;
  if (format == 1)
    expert_quant_error_kernel<1><<<E, kErrThreads, 0, stream>>>(gate, up, down, d, inter, out);
  else if (format == 2)
    expert_quant_error_kernel<2><<<E, kErrThreads, 0, stream>>>(gate, up, down, d, inter, out);
  else
    return SPX_ERR_INVALID_ARG;
  return cudaGetLastError() == cudaSuccess ? SPX_OK : SPX_ERR_CUDA;
}

}  // namespace spx
