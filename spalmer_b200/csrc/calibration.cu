// Router calibration loss term and per-expert NLL attribution from one
// layer's routing outputs (mESmaC/spalmer src/spalmer/modeling.py:1468-1534).
//
// Over positions s < S-1 of every sequence (the last position has no
// next-token NLL), with w the routing weights and v the validity mask:
//   predicted = bf16(sum_j bf16(score[id_j] * w_j))        (FP32 sum, slot order)
//   calibration = mean over valid positions of smooth_l1(predicted - nll), beta 1
//   counts[e] = sum of w*v, totals[e] = sum of w*v*nll over pairs of expert e
//   attributed[e] = totals / counts (0 when counts == 0), utilization = counts / #valid
// Deterministic: every warp walks a fixed range of positions and adds its
// pairs into warp-private per-expert arrays (a position's k experts are
// distinct, so the lanes never collide); CTAs and then one final CTA reduce
// in a fixed order.
#include <cuda_runtime.h>
#include <stdint.h>

#include "kernels.h"
#include "sm100.cuh"

namespace spx {

namespace {
constexpr int kCalWarps = 8;
constexpr int kCalMaxBlocks = 296;

int cal_blocks(int64_t positions) {
  const int64_t want = (positions + kCalWarps * 64 - 1) / (kCalWarps * 64);
  return static_cast<int>(want < 1 ? 1 : (want > kCalMaxBlocks ? kCalMaxBlocks : want));
}
}  // namespace

// partial[b] = {counts[E], totals[E]}; stats[b] = {sum smooth_l1, valid positions}
__global__ void __launch_bounds__(kCalWarps * 32)
    calibration_partial_kernel(const uint16_t* __restrict__ scores, const int64_t* __restrict__ ids,
                               const uint16_t* __restrict__ weights, const float* __restrict__ nll,
                               const uint8_t* __restrict__ valid, int64_t B, int64_t S, int E, int k,
                               float* __restrict__ partial, double* __restrict__ stats) {
  extern __shared__ float cal_smem[];  // [warps][2][E]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* cnt = cal_smem + warp * 2 * E;
  float* tot = cnt + E;
  for (int e = lane; e < E; e += 32) cnt[e] = tot[e] = 0.0f;
  __syncwarp();
  const int64_t per_seq = S - 1;
  const int64_t positions = B * per_seq;
  const int64_t nwarps = static_cast<int64_t>(gridDim.x) * kCalWarps;
  const int64_t gw = static_cast<int64_t>(blockIdx.x) * kCalWarps + warp;
  const int64_t chunk = (positions + nwarps - 1) / nwarps;
  const int64_t q0 = gw * chunk;
  const int64_t q1 = q0 + chunk < positions ? q0 + chunk : positions;
  double sl1_sum = 0.0;
  double n_valid = 0.0;
  for (int64_t q = q0; q < q1; ++q) {
    const int64_t b = q / per_seq;
    const int64_t row = b * S + (q - b * per_seq);  // position (b, s) of the routing outputs
    const float t = nll[q];
    const bool v = valid[q] != 0;
    int id = 0;
    float w = 0.0f, prod = 0.0f;
    bool ok = false;
    if (lane < k) {
      const int64_t e = ids[row * k + lane];
      ok = e >= 0 && e < E;  // out-of-range ids are skipped
      id = ok ? static_cast<int>(e) : 0;
      w = bf16_to_f32(weights[row * k + lane]);
      prod = ok ? round_bf16(bf16_to_f32(scores[row * E + id]) * w) : 0.0f;
    }
    float sum = 0.0f;
    for (int j = 0; j < k; ++j) sum += __shfl_sync(0xFFFFFFFFu, prod, j);
    if (lane == 0 && v) {
      const float d = fabsf(round_bf16(sum) - t);
      sl1_sum += d < 1.0f ? 0.5f * d * d : d - 0.5f;
      n_valid += 1.0;
    }
    if (lane < k && v && ok) {
      cnt[id] += w;
      tot[id] += w * t;
    }
    __syncwarp();
  }
  __shared__ double warp_stats[kCalWarps][2];
  if (lane == 0) {
    warp_stats[warp][0] = sl1_sum;
    warp_stats[warp][1] = n_valid;
  }
  __syncthreads();
  float* out = partial + static_cast<int64_t>(blockIdx.x) * 2 * E;
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    float c = 0.0f, s = 0.0f;
    for (int w = 0; w < kCalWarps; ++w) {
      c += cal_smem[w * 2 * E + e];
      s += cal_smem[w * 2 * E + E + e];
    }
    out[e] = c;
    out[E + e] = s;
  }
  if (threadIdx.x == 0) {
    double a = 0.0, n = 0.0;
    for (int w = 0; w < kCalWarps; ++w) {
      a += warp_stats[w][0];
      n += warp_stats[w][1];
    }
    stats[2 * blockIdx.x] = a;
    stats[2 * blockIdx.x + 1] = n;
  }
}

__global__ void calibration_final_kernel(const float* __restrict__ partial, const double* __restrict__ stats,
                                         int blocks, int E, float* calibration, float* attributed,
                                         float* utilization) {
  __shared__ double s_valid;
  if (threadIdx.x == 0) {
    double a = 0.0, n = 0.0;
    for (int b = 0; b < blocks; ++b) {
      a += stats[2 * b];
      n += stats[2 * b + 1];
    }
    s_valid = n;
    if (calibration != nullptr) *calibration = n > 0.0 ? static_cast<float>(a / n) : __int_as_float(0x7FC00000);
  }
  __syncthreads();
  const double denom = s_valid > 1.0 ? s_valid : 1.0;
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    double c = 0.0, s = 0.0;
    for (int b = 0; b < blocks; ++b) {
      c += partial[static_cast<int64_t>(b) * 2 * E + e];
      s += partial[static_cast<int64_t>(b) * 2 * E + E + e];
    }
    if (attributed != nullptr) attributed[e] = c > 0.0 ? static_cast<float>(s / (c > 1e-8 ? c : 1e-8)) : 0.0f;
    if (utilization != nullptr) utilization[e] = static_cast<float>(c / denom);
  }
}

size_t calibration_workspace_bytes(int64_t B, int64_t S, int E) {
  const int blocks = cal_blocks(B * (S > 1 ? S - 1 : 0));
  return static_cast<size_t>(blocks) * (2 * E * sizeof(float) + 2 * sizeof(double)) + 256;
}

int launch_calibration(const uint16_t* scores, const int64_t* ids, const uint16_t* weights, const float* nll,
                       const uint8_t* valid, int64_t B, int64_t S, int E, int k, float* calibration,
                       float* attributed, float* utilization, void* workspace, cudaStream_t stream) {
  const int blocks = cal_blocks(B * (S - 1));
  float* partial = static_cast<float*>(workspace);
  double* stats = reinterpret_cast<double*>(
      (reinterpret_cast<uintptr_t>(partial + static_cast<size_t>(blocks) * 2 * E) + 15) & ~uintptr_t(15));
  const size_t smem = static_cast<size_t>(kCalWarps) * 2 * E * sizeof(float);
  if (ensure_max_dynamic_smem(reinterpret_cast<const void*>(calibration_partial_kernel)) != SPX_OK)
    return SPX_ERR_CUDA;
  calibration_partial_kernel<<<blocks, kCalWarps * 32, smem, stream>>>(scores, ids, weights, nll, valid, B, S, E, k,
                                                                      partial, stats);
  if (cudaGetLastError() != cudaSuccess) return SPX_ERR_CUDA;
  calibration_final_kernel<<<1, 256, 0, stream>>>(partial, stats, blocks, E, calibration, attributed, utilization);
  return cudaGetLastError() == cudaSuccess ? SPX_OK : SPX_ERR_CUDA;
}

}  // namespace spx
