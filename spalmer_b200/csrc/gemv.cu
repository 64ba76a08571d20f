// Decode-sized expert projections: grouped GEMVs on the CUDA cores.
//
// With a few tokens per step every routed expert sees a handful of rows, and
// the expert projections are bound by reading the selected experts' weights
// once (589,824 bytes per expert in BF16 at the 100M shape).  A 128-row
// tcgen05 tile would hold those few rows and spend its time filling and
// draining; these kernels instead stream each weight row once per CTA with
// 16-byte coalesced loads and keep the expert's token rows in shared memory.
//
// Same rounding points as the tensor-core path (experts/bank.py:755-763 and
// 970-978): gate and up accumulate in FP32, h = bf16(bf16(silu(bf16(g))) *
// bf16(u)), y = bf16(bf16(h @ D) * w).  MXFP8-lane experts (experts/native.py
// :91-140) dot the E4M3 values with their E8M0 block scales applied: the
// activations' blocks are dequantised exactly into BF16 (an E4M3 value times
// a power of two is representable), the weights' into FP32, the products are
// summed in FP32, and GEMV1 writes the hidden rows quantised again for GEMV2.
//
// Layouts (the packed weights of spx_pack_weights / spx_pack_weights_mxfp8):
//   W1 BF16   [E][nc * 2c][kd]   per chunk of c hidden columns: gate rows, then up rows
//   W2 BF16   [E][d][kp]
//   W1 MXFP8  [E][ncm * 2cm][kx] E4M3, scale atoms per (2cm)-row tile
//   W2 MXFP8  [E][d][kh]         E4M3, scale atoms per bn2m-row tile
// Rows of one expert are its dispatch range [starts[e], starts[e] + counts[e]).
//
// Work split: a CTA owns one expert and a block of 32 hidden columns (GEMV1)
// or 64 output columns (GEMV2); each warp walks 4 weight rows at a time, one
// group of 8 lanes per row, so one warp instruction reads 4 x 128 contiguous
// bytes.  The token rows sit in shared memory (up to 16 per pass).
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

#include "kernels.h"
#include "mx.cuh"
#include "sm100.cuh"

namespace spx {

namespace {

constexpr int kGemvThreads = 256;
constexpr int kGemvWarps = kGemvThreads / 32;
constexpr int kGemvRows = 16;   // token rows per pass
constexpr int kGemv1Cols = 32;  // hidden columns per GEMV1 CTA (one MXFP8 block of the hidden row)
constexpr int kGemv2Cols = 64;  // output columns per GEMV2 CTA

__device__ __forceinline__ float silu_ref(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

// 2^(byte - 127): the value of an E8M0 scale byte.
__device__ __forceinline__ float e8m0_value(uint32_t byte) {
  if (byte == 0u) return __uint_as_float(0x00400000u);  // 2^-127
  return __uint_as_float(byte << 23);
}

// Eight BF16 values (one 16-byte word) to floats.
__device__ __forceinline__ void bf16x8(const uint4& v, float (&f)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    f[2 * q] = __uint_as_float(w[q] << 16);
    f[2 * q + 1] = __uint_as_float(w[q] & 0xFFFF0000u);
  }
}

// Four E4M3 bytes (one word) to floats, times `s`.
__device__ __forceinline__ void e4m3x4(uint32_t w, float s, float* f) {
  const __half2_raw lo = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(w & 0xFFFFu), __NV_E4M3);
  const __half2_raw hi = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(w >> 16), __NV_E4M3);
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&lo));
  const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&hi));
  f[0] = a.x * s;
  f[1] = a.y * s;
  f[2] = b.x * s;
  f[3] = b.y * s;
}

// Scale byte of (row, K block `blk` of 32) in the atoms of a packed MXFP8 weight:
// atoms [E][tiles][K/128][ceil(tile_rows/128)][512] (mxfp8.cu, mx_quantize_b_kernel).
__device__ __forceinline__ uint32_t w_scale(const uint8_t* atoms, int e, int row, int blk, int rows_per_group,
                                            int tile_rows, int kp) {
  const int tiles = (rows_per_group + tile_rows - 1) / tile_rows;
  const int per_tile = (tile_rows + 127) / 128;
  const int tile = row / tile_rows, r = row - tile * tile_rows;
  const int64_t atom = ((static_cast<int64_t>(e) * tiles + tile) * (kp / 128) + (blk >> 2)) * per_tile + (r >> 7);
  return atoms[atom * kMxAtomBytes + mx_atom_offset(r & 127, blk & 3)];
}

// Token rows [row0, row0 + R) of the expert's dispatch range into shared
// memory as BF16 [R][K]: plain copies, or E4M3 rows dequantised with their
// block scales (exact).  `gather`: rows are token rows through src_row.
__device__ void load_rows(const GemvArgs& a, bool mx, const int* src, bool gather, int64_t pos0, int R,
                          const uint16_t* rows_bf16, int64_t ld_bf16, const uint8_t* rows_q, const uint8_t* rows_sf,
                          int64_t ld_q, int K, uint16_t* xs) {
  if (!mx) {
    const int per_row = K / 8;
    for (int i = threadIdx.x; i < R * per_row; i += blockDim.x) {
      const int r = i / per_row, c = i - r * per_row;
      const int64_t src_row = gather ? src[pos0 + r] : pos0 + r;
      reinterpret_cast<uint4*>(xs + static_cast<int64_t>(r) * K)[c] =
          __ldg(reinterpret_cast<const uint4*>(rows_bf16 + src_row * ld_bf16) + c);
    }
    return;
  }
  // E4M3: 16 values per thread step, their block scale applied, stored as BF16
  const int per_row = K / 16;
  for (int i = threadIdx.x; i < R * per_row; i += blockDim.x) {
    const int r = i / per_row, c = i - r * per_row;
    const int64_t src_row = gather ? src[pos0 + r] : pos0 + r;
    const uint4 q = __ldg(reinterpret_cast<const uint4*>(rows_q + src_row * ld_q) + c);
    const float s = e8m0_value(__ldg(rows_sf + src_row * (ld_q / kMxBlock) + (c >> 1)));
    float f[16];
    e4m3x4(q.x, s, f);
    e4m3x4(q.y, s, f + 4);
    e4m3x4(q.z, s, f + 8);
    e4m3x4(q.w, s, f + 12);
    uint32_t h[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) h[j] = static_cast<uint32_t>(f32_to_bf16_rne(f[2 * j])) |
                                       (static_cast<uint32_t>(f32_to_bf16_rne(f[2 * j + 1])) << 16);
    uint4* dst = reinterpret_cast<uint4*>(xs + static_cast<int64_t>(r) * K + c * 16);
    dst[0] = make_uint4(h[0], h[1], h[2], h[3]);
    dst[1] = make_uint4(h[4], h[5], h[6], h[7]);
  }
}

// acc[i] += <weight row slice, xs row i slice> for the lane's K positions.
// BF16 weights: per step the 8 lanes of a group read 8 x 16 bytes (64 values);
// E4M3 weights: 8 x 16 bytes = 128 values with per-32 scales.  Each lane
// issues the loads of kBatch steps before it uses any of them, so a warp keeps
// 4 rows x 8 lanes x kBatch x 16 bytes in flight.
template <bool MX>
__device__ __forceinline__ void dot_rows(const void* wrow, const uint8_t* atoms, int e, int wr, int rows_per_group,
                                         int tile_rows, int K, int k_valid, const uint16_t* xs, int R, int seg,
                                         bool live, float (&acc)[kGemvRows]) {
  constexpr int kEl = MX ? 16 : 8;   // values per lane per step
  constexpr int kStep = 8 * kEl;     // values per group per step
  constexpr int kBatch = 4;
  for (int kb = 0; kb < k_valid; kb += kBatch * kStep) {
    uint4 raw[kBatch];
    float sc[kBatch];
#pragma unroll
    for (int b = 0; b < kBatch; ++b) {
      const int k = kb + b * kStep + seg * kEl;
      raw[b] = make_uint4(0u, 0u, 0u, 0u);
      sc[b] = 0.0f;
      if (live && k < k_valid) {
        if constexpr (MX) {
          raw[b] = __ldg(reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(wrow) + k));
          sc[b] = e8m0_value(w_scale(atoms, e, wr, k / kMxBlock, rows_per_group, tile_rows, K));
        } else {
          raw[b] = __ldg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(wrow) + k));
        }
      }
    }
#pragma unroll
    for (int b = 0; b < kBatch; ++b) {
      const int k = kb + b * kStep + seg * kEl;
      if (!(live && k < k_valid)) continue;
      float w[kEl];
      if constexpr (MX) {
        e4m3x4(raw[b].x, sc[b], w);
        e4m3x4(raw[b].y, sc[b], w + 4);
        e4m3x4(raw[b].z, sc[b], w + 8);
        e4m3x4(raw[b].w, sc[b], w + 12);
      } else {
        bf16x8(raw[b], *reinterpret_cast<float(*)[8]>(w));
      }
#pragma unroll
      for (int i = 0; i < kGemvRows; ++i) {
        if (i < R) {
          const uint4* xp = reinterpret_cast<const uint4*>(xs + static_cast<int64_t>(i) * K + k);
#pragma unroll
          for (int h = 0; h < kEl / 8; ++h) {
            float x[8];
            bf16x8(xp[h], x);
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[i] = fmaf(w[8 * h + j], x[j], acc[i]);
          }
        }
      }
    }
  }
}

__device__ __forceinline__ float group_sum8(float v) {
  v += __shfl_xor_sync(0xFFFFFFFFu, v, 1);
  v += __shfl_xor_sync(0xFFFFFFFFu, v, 2);
  v += __shfl_xor_sync(0xFFFFFFFFu, v, 4);
  return v;
}

// GEMV1: gate/up of 32 hidden columns of one expert for its routed rows, SwiGLU,
// hidden rows out (BF16 [P][kp], or E4M3 [P][kh] + scales for the MXFP8 lane).
__global__ void __launch_bounds__(kGemvThreads) gemv_swiglu_kernel(const GemvArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int e = blockIdx.x;
  const int j0 = blockIdx.y * kGemv1Cols;
  const int n = a.counts[e];
  if (n <= 0 || j0 >= a.inter) return;
  const bool mx = a.lane_mx != nullptr && a.lane_mx[e] != 0;
  const int K = mx ? a.kx : a.kd;
  uint16_t* xs = reinterpret_cast<uint16_t*>(smem);
  float* hs = reinterpret_cast<float*>(smem + static_cast<size_t>(kGemvRows) * K * 2);  // [kGemvRows][32]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int grp = lane >> 3, seg = lane & 7;
  const int64_t start = a.starts[e];
  const int c = mx ? a.cm : a.chunk;
  const int rows1 = (mx ? a.ncm : a.nc) * 2 * c;
  for (int r0 = 0; r0 < n; r0 += kGemvRows) {
    const int R = min(kGemvRows, n - r0);
    load_rows(a, mx, a.src_row, true, start + r0, R, a.x, a.ldx, a.xq, a.xsf, a.kx, K, xs);
    __syncthreads();
    // warp: hidden columns j0 + warp*4 + {0..3}, two passes of two columns;
    // lane groups: 0 gate(jj), 1 gate(jj+1), 2 up(jj), 3 up(jj+1)
    for (int p = 0; p < 2; ++p) {
      const int jj = j0 + warp * 4 + p * 2 + (grp & 1);
      const bool live = jj < a.inter;
      const int ch = jj / c;
      const int wr = ch * 2 * c + (grp >> 1) * c + (jj - ch * c);  // packed row of gate / up column jj
      float acc[kGemvRows];
#pragma unroll
      for (int i = 0; i < kGemvRows; ++i) acc[i] = 0.0f;
      if (mx) {
        const uint8_t* wrow = a.w1q + (static_cast<int64_t>(e) * rows1 + wr) * a.kx;
        dot_rows<true>(wrow, a.w1sf, e, wr, rows1, 2 * c, a.kx, a.kx, xs, R, seg, live, acc);
      } else {
        const uint16_t* wrow = a.w1 + (static_cast<int64_t>(e) * rows1 + wr) * a.kd;
        dot_rows<false>(wrow, nullptr, e, wr, rows1, 0, a.kd, a.kd, xs, R, seg, live, acc);
      }
#pragma unroll
      for (int i = 0; i < kGemvRows; ++i) {
        const float g = group_sum8(acc[i]);
        const float u = __shfl_down_sync(0xFFFFFFFFu, g, 16);  // group 2 -> 0, group 3 -> 1
        if (i < R && grp < 2 && seg == 0 && live) {
          const float gb = round_bf16(g), ub = round_bf16(u);
          const float h = round_bf16(round_bf16(silu_ref(gb)) * ub);
          if (mx) {
            hs[i * kGemv1Cols + (jj - j0)] = h;
          } else {
            a.hid[(start + r0 + i) * a.kp + jj] = f32_to_bf16_rne(h);
          }
        }
      }
    }
    __syncthreads();
    if (mx && static_cast<int>(threadIdx.x) < R) {
      // the 32-column block of this row: E4M3 + its scale (the tensor-core path's epilogue rule)
      const int i = threadIdx.x;
      float v[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = (j0 + j < a.inter) ? hs[i * kGemv1Cols + j] : 0.0f;
      uint32_t q[8];
      const uint32_t sb = mx_quantize32(v, q);
      uint4* dst = reinterpret_cast<uint4*>(a.hq + (start + r0 + i) * a.kh + j0);
      dst[0] = make_uint4(q[0], q[1], q[2], q[3]);
      dst[1] = make_uint4(q[4], q[5], q[6], q[7]);
      a.hsf[(start + r0 + i) * (a.kh / kMxBlock) + j0 / kMxBlock] = static_cast<uint8_t>(sb);
    }
    __syncthreads();
  }
}

// GEMV2: down projection of 64 output columns of one expert for its rows,
// weighted by the pair's routing weight (unit when sorted_w is null), rows
// written to Y [P][d] in dispatch order.
__global__ void __launch_bounds__(kGemvThreads) gemv_down_kernel(const GemvArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int e = blockIdx.x;
  const int n0 = blockIdx.y * kGemv2Cols;
  const int n = a.counts[e];
  if (n <= 0 || n0 >= a.d) return;
  const bool mx = a.lane_mx != nullptr && a.lane_mx[e] != 0;
  const int K = mx ? a.kh : a.kp;
  uint16_t* hsm = reinterpret_cast<uint16_t*>(smem);
  uint16_t* ys = reinterpret_cast<uint16_t*>(smem + static_cast<size_t>(kGemvRows) * K * 2);  // [rows][64]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int grp = lane >> 3, seg = lane & 7;
  const int64_t start = a.starts[e];
  const int cols = min(kGemv2Cols, a.d - n0);
  for (int r0 = 0; r0 < n; r0 += kGemvRows) {
    const int R = min(kGemvRows, n - r0);
    load_rows(a, mx, nullptr, false, start + r0, R, a.hid, a.kp, a.hq, a.hsf, a.kh, K, hsm);
    __syncthreads();
    for (int p = 0; p < kGemv2Cols / (kGemvWarps * 4); ++p) {
      const int nl = warp * (kGemv2Cols / kGemvWarps) + p * 4 + grp;  // local output column
      const int nn = n0 + nl;
      const bool live = nl < cols;
      float acc[kGemvRows];
#pragma unroll
      for (int i = 0; i < kGemvRows; ++i) acc[i] = 0.0f;
      if (mx) {
        const uint8_t* wrow = a.w2q + (static_cast<int64_t>(e) * a.d + nn) * a.kh;
        dot_rows<true>(wrow, a.w2sf, e, nn, a.d, a.bn2m, a.kh, a.inter, hsm, R, seg, live, acc);
      } else {
        const uint16_t* wrow = a.w2 + (static_cast<int64_t>(e) * a.d + nn) * a.kp;
        dot_rows<false>(wrow, nullptr, e, nn, a.d, 0, a.kp, a.inter, hsm, R, seg, live, acc);
      }
#pragma unroll
      for (int i = 0; i < kGemvRows; ++i) {
        const float y = group_sum8(acc[i]);
        if (i < R && seg == 0 && live) {
          const float w = a.sorted_w != nullptr ? bf16_to_f32(a.sorted_w[start + r0 + i]) : 1.0f;
          ys[i * kGemv2Cols + nl] = f32_to_bf16_rne(round_bf16(y) * w);
        }
      }
    }
    __syncthreads();
    // staged rows out: 8 lanes per row segment of up to 64 columns (16 bytes each)
    const bool vec = (cols % 8) == 0 && (a.d % 8) == 0;
    if (vec) {
      const int per_row = cols / 8;
      for (int t = threadIdx.x; t < R * per_row; t += blockDim.x) {
        const int i = t / per_row, q = t - i * per_row;
        reinterpret_cast<uint4*>(a.y + (start + r0 + i) * a.d + n0)[q] =
            reinterpret_cast<const uint4*>(ys + i * kGemv2Cols)[q];
      }
    } else {
      for (int t = threadIdx.x; t < R * cols; t += blockDim.x) {
        const int i = t / cols, q = t - i * cols;
        a.y[(start + r0 + i) * a.d + n0 + q] = ys[i * kGemv2Cols + q];
      }
    }
    __syncthreads();
  }
}

}  // namespace

bool gemv_supported(const GemvArgs& a) {
  // 16-byte row loads: BF16 rows of kd / kp values, E4M3 rows of kx / kh bytes.
  return a.d % 8 == 0 && a.inter % kMxBlock == 0 && a.kd % 64 == 0 && a.kp % 64 == 0 && a.kp >= a.inter &&
         (a.lane_mx == nullptr || (a.kx % 128 == 0 && a.kh % 128 == 0));
}

size_t gemv_smem_bytes(const GemvArgs& a, int which) {
  const int k = which == 1 ? std::max(a.kd, a.lane_mx ? a.kx : 0) : std::max(a.kp, a.lane_mx ? a.kh : 0);
  const size_t rows = static_cast<size_t>(kGemvRows) * k * 2;
  return rows + (which == 1 ? kGemvRows * kGemv1Cols * 4 : kGemvRows * kGemv2Cols * 2);
}

int launch_gemv_experts(const GemvArgs& a, cudaStream_t stream, int which) {
  if (!gemv_supported(a)) return SPX_ERR_UNSUPPORTED;
  const size_t smem = gemv_smem_bytes(a, which);
  if (which == 1) {
    if (smem > 48 * 1024) {
      if (int rc = ensure_max_dynamic_smem(reinterpret_cast<const void*>(gemv_swiglu_kernel)); rc != SPX_OK)
        return rc;
    }
    const dim3 grid(a.num_experts, (a.inter + kGemv1Cols - 1) / kGemv1Cols);
    gemv_swiglu_kernel<<<grid, kGemvThreads, smem, stream>>>(a);
  } else {
    if (smem > 48 * 1024) {
      if (int rc = ensure_max_dynamic_smem(reinterpret_cast<const void*>(gemv_down_kernel)); rc != SPX_OK)
        return rc;
    }
    const dim3 grid(a.num_experts, (a.d + kGemv2Cols - 1) / kGemv2Cols);
    gemv_down_kernel<<<grid, kGemvThreads, smem, stream>>>(a);
  }
  return cudaGetLastError() == cudaSuccess ? SPX_OK : SPX_ERR_CUDA;
}

}  // namespace spx
