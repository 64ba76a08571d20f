// Weight repacking (a derived cache of the reference state_dict) and the
// standalone combine used when the layer has no shared path (expert rows Y in
// sorted order, gathered per token through the pair -> position rank).
//
// The reference stores expert projections as [E, d, I] / [E, I, d] ("x @ W",
// experts/bank.py:52-54) and the shared SwiGLU as nn.Linear [out, in]
// (nn/ffn.py:16-18).  The tensor-core kernels want every B operand K-major
// ([N rows, K contiguous]) and GEMM1 wants gate and up side by side:
//   W1[e] rows: for chunk c: [gate cols c*C .. c*C+C) ++ [up cols c*C .. c*C+C)
//   W2[e] = down[e]^T  ([d rows, I contiguous], K zero-padded to a multiple of 64)
// Rows or columns beyond the real sizes are zero, so padding contributes 0.
#include <cuda_runtime.h>
#include <stdint.h>

#include "kernels.h"
#include "sm100.cuh"

namespace spx {

__global__ void pack_chunked_w1_kernel(const uint16_t* __restrict__ gate, const uint16_t* __restrict__ up,
                                       int experts, int d, int inter, int kd, int chunk, int chunks,
                                       int transposed_src, uint16_t* __restrict__ out) {
  const int64_t rows_per_e = static_cast<int64_t>(chunks) * 2 * chunk;
  const int64_t total = static_cast<int64_t>(experts) * rows_per_e * kd;
  for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int kk = static_cast<int>(idx % kd);
    const int64_t rowg = idx / kd;
    const int row = static_cast<int>(rowg % rows_per_e);
    const int e = static_cast<int>(rowg / rows_per_e);
    const int ch = row / (2 * chunk);
    const int within = row - ch * 2 * chunk;
    const int half = within / chunk;
    const int i = ch * chunk + (within - half * chunk);
    uint16_t v = 0;
    if (i < inter && kk < d) {
      const uint16_t* src = half == 0 ? gate : up;
      v = transposed_src ? src[static_cast<int64_t>(i) * d + kk]
                         : src[(static_cast<int64_t>(e) * d + kk) * inter + i];
    }
    out[idx] = v;
  }
}

__global__ void pack_w2_kernel(const uint16_t* __restrict__ down, int experts, int inter, int d, int kp,
                               int transposed_src, uint16_t* __restrict__ out) {
  const int64_t total = static_cast<int64_t>(experts) * d * kp;
  for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int i = static_cast<int>(idx % kp);
    const int64_t rest = idx / kp;
    const int n = static_cast<int>(rest % d);
    const int e = static_cast<int>(rest / d);
    uint16_t v = 0;
    if (i < inter) {
      v = transposed_src ? down[static_cast<int64_t>(n) * inter + i]
                         : down[(static_cast<int64_t>(e) * inter + i) * d + n];
    }
    out[idx] = v;
  }
}

__global__ void pad_rows_kernel(const uint16_t* __restrict__ src, int64_t rows, int cols, int ld_out,
                                uint16_t* __restrict__ out) {
  const int64_t total = rows * ld_out;
  for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(idx % ld_out);
    const int64_t r = idx / ld_out;
    out[idx] = c < cols ? src[r * cols + c] : static_cast<uint16_t>(0);
  }
}

// update[t] = bf16(base[t] + sum_j row_j) in FP32 (base first, then slots in
// order), row_j = Y[rank[t*k + j]] -- or bf16(Y[rank[t*k + j]] * w[t*k + j])
// when pair weights are given (expert rows computed elsewhere, unweighted).
// A negative rank marks an empty slot (no row).
// base is the shared SwiGLU output (BF16) or absent.  8 columns per thread;
// consecutive threads take consecutive 16-byte chunks of one token, so every
// slot's row is read in whole 128-byte lines, and a thread issues all k row
// loads before it adds any.
template <int KMAX, bool WEIGHTED>
__global__ void combine_kernel(const uint16_t* __restrict__ y, const int* __restrict__ rank,
                               const uint16_t* __restrict__ weights, const uint16_t* __restrict__ base,
                               int64_t tokens, int d, int k, uint16_t* __restrict__ out,
                               const uint16_t* __restrict__ residual, uint16_t* __restrict__ residual_out) {
  const int vec = d / 8;
  const int64_t total = tokens * vec;
  griddep_wait();
  griddep_launch_dependents();
  for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t t = idx / vec;
    const int c = static_cast<int>(idx - t * vec) * 8;
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (base != nullptr) add_row8<false>(acc, __ldg(reinterpret_cast<const uint4*>(base + t * d + c)), 1.0f);
    int r[KMAX];
#pragma unroll
    for (int j = 0; j < KMAX; ++j) r[j] = j < k ? __ldg(rank + t * k + j) : 0;
    uint4 v[KMAX];
#pragma unroll
    for (int j = 0; j < KMAX; ++j)
      if (j < k && r[j] >= 0) v[j] = __ldg(reinterpret_cast<const uint4*>(y + static_cast<int64_t>(r[j]) * d + c));
#pragma unroll
    for (int j = 0; j < KMAX; ++j) {
      if (j < k && r[j] >= 0) {
        const float w = WEIGHTED ? bf16_to_f32(__ldg(weights + t * k + j)) : 1.0f;
        add_row8<WEIGHTED>(acc, v[j], w);
      }
    }
    uint4 o;
    uint16_t* oh = reinterpret_cast<uint16_t*>(&o);
#pragma unroll
    for (int q8 = 0; q8 < 8; ++q8) oh[q8] = f32_to_bf16_rne(acc[q8]);
    if (out != nullptr) *reinterpret_cast<uint4*>(out + t * d + c) = o;
    if (residual != nullptr) {  // the block's residual add: bf16(h + update)
      float hs[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      add_row8<false>(hs, __ldg(reinterpret_cast<const uint4*>(residual + t * d + c)), 1.0f);
      add_row8<false>(hs, o, 1.0f);
#pragma unroll
      for (int q8 = 0; q8 < 8; ++q8) oh[q8] = f32_to_bf16_rne(hs[q8]);
      *reinterpret_cast<uint4*>(residual_out + t * d + c) = o;
    }
  }
}

__global__ void combine_scalar_kernel(const uint16_t* __restrict__ y, const int* __restrict__ rank,
                                      const uint16_t* __restrict__ weights, const uint16_t* __restrict__ base,
                                      int64_t tokens, int d, int k, uint16_t* __restrict__ out,
                                      const uint16_t* __restrict__ residual, uint16_t* __restrict__ residual_out) {
  const int64_t total = tokens * d;
  for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t t = idx / d;
    const int c = static_cast<int>(idx - t * d);
    float acc = base != nullptr ? bf16_to_f32(base[idx]) : 0.0f;
    for (int j = 0; j < k; ++j) {
      if (rank[t * k + j] < 0) continue;  // empty slot
      float v = bf16_to_f32(y[static_cast<int64_t>(rank[t * k + j]) * d + c]);
      if (weights != nullptr) v = round_bf16(v * bf16_to_f32(weights[t * k + j]));
      acc += v;
    }
    const uint16_t u = f32_to_bf16_rne(acc);
    if (out != nullptr) out[idx] = u;
    if (residual != nullptr) residual_out[idx] = f32_to_bf16_rne(bf16_to_f32(residual[idx]) + bf16_to_f32(u));
  }
}

// out[i] = src[index[i] / div], 16 bytes per thread when aligned.
__global__ void gather_rows_kernel(const uint16_t* __restrict__ src, int64_t ld_src, const int* __restrict__ index,
                                   int div, int64_t rows, int d, uint16_t* __restrict__ out, int64_t ld_out,
                                   bool vec) {
  const int per_row = vec ? d / 8 : d;
  const int64_t total = rows * per_row;
  for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t i = idx / per_row;
    const int c = static_cast<int>(idx - i * per_row);
    const int64_t r = __ldg(index + i) / div;
    if (vec)
      *reinterpret_cast<uint4*>(out + i * ld_out + 8 * c) = __ldg(reinterpret_cast<const uint4*>(src + r * ld_src + 8 * c));
    else
      out[i * ld_out + c] = src[r * ld_src + c];
  }
}

static int grid_for(int64_t total) {
  int64_t g = (total + 255) / 256;
  if (g > 148 * 32) g = 148 * 32;
  return static_cast<int>(g < 1 ? 1 : g);
}

int launch_pack_chunked_w1(const uint16_t* gate, const uint16_t* up, int experts, int d, int inter, int kd,
                           int chunk, int chunks, int transposed_src, uint16_t* out, cudaStream_t stream) {
  const int64_t total = static_cast<int64_t>(experts) * chunks * 2 * chunk * kd;
  pack_chunked_w1_kernel<<<grid_for(total), 256, 0, stream>>>(gate, up, experts, d, inter, kd, chunk, chunks,
                                                               transposed_src, out);
  return cudaGetLastError() == cudaSuccess ? SPX_OK : SPX_ERR_CUDA;
}

int launch_pack_w2(const uint16_t* down, int experts, int inter, int d, int kp, int transposed_src, uint16_t* out,
                   cudaStream_t stream) {
  const int64_t total = static_cast<int64_t>(experts) * d * kp;
  pack_w2_kernel<<<grid_for(total), 256, 0, stream>>>(down, experts, inter, d, kp, transposed_src, out);
  return cudaGetLastError() == cudaSuccess ? SPX_OK : SPX_ERR_CUDA;
}

int launch_pad_rows(const uint16_t* src, int64_t rows, int cols, int ld_out, uint16_t* out, cudaStream_t stream) {
  pad_rows_kernel<<<grid_for(rows * ld_out), 256, 0, stream>>>(src, rows, cols, ld_out, out);
  return cudaGetLastError() == cudaSuccess ? SPX_OK : SPX_ERR_CUDA;
}

int launch_combine_residual(const uint16_t* y, const int* rank, const uint16_t* weights, const uint16_t* base,
                            const uint16_t* residual, int64_t tokens, int d, int k, uint16_t* out,
                            uint16_t* residual_out, cudaStream_t stream) {
  if (out == nullptr && residual == nullptr) return SPX_ERR_INVALID_ARG;
  if (residual != nullptr && residual_out == nullptr) return SPX_ERR_INVALID_ARG;
  auto a16 = [](const void* p) { return p == nullptr || (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  const bool vec_ok = (d % 8) == 0 && a16(y) && a16(out) && a16(base) && a16(residual) && a16(residual_out);
  if (vec_ok) {
    const int64_t total = tokens * (d / 8);
    int64_t g = (total + 255) / 256;
    if (g > 148 * 64) g = 148 * 64;
    const int grid = static_cast<int>(g < 1 ? 1 : g);
    auto fn = weights == nullptr ? (k <= 8 ? combine_kernel<8, false> : combine_kernel<kMaxTopK, false>)
                                 : (k <= 8 ? combine_kernel<8, true> : combine_kernel<kMaxTopK, true>);
    return launch_pdl(fn, dim3(grid), dim3(256), 0, stream, y, rank, weights, base, tokens, d, k, out, residual,
                      residual_out);
  } else {
    combine_scalar_kernel<<<grid_for(tokens * d), 256, 0, stream>>>(y, rank, weights, base, tokens, d, k, out,
                                                                    residual, residual_out);
  }
  return cudaGetLastError() == cudaSuccess ? SPX_OK : SPX_ERR_CUDA;
}

int launch_combine(const uint16_t* y, const int* rank, const uint16_t* weights, const uint16_t* base, int64_t tokens,
                   int d, int k, uint16_t* out, cudaStream_t stream) {
  return launch_combine_residual(y, rank, weights, base, nullptr, tokens, d, k, out, nullptr, stream);
}

int launch_gather_rows(const uint16_t* src, int64_t ld_src, const int* index, int index_div, int64_t rows, int d,
                       uint16_t* out, int64_t ld_out, cudaStream_t stream) {
  const bool vec = (d % 8) == 0 && (ld_src % 8) == 0 && (ld_out % 8) == 0 &&
                   (reinterpret_cast<uintptr_t>(src) & 15u) == 0 && (reinterpret_cast<uintptr_t>(out) & 15u) == 0;
  const int64_t total = rows * (vec ? d / 8 : d);
  gather_rows_kernel<<<grid_for(total), 256, 0, stream>>>(src, ld_src, index, index_div, rows, d, out, ld_out, vec);
  return cudaGetLastError() == cudaSuccess ? SPX_OK : SPX_ERR_CUDA;
}

}  // namespace spx
