// tcgen05 GEMM engine for the micro-expert layer (sm_100a).
//
// C[128-row tile, BN cols] = A[rows, K] * B[group][BN rows, K]^T, BF16 operands,
// FP32 accumulation in tensor memory.  One CTA computes one output tile:
//   warp 0      TMA producer: A either as a 128-row box or gathered 4 rows at a
//               time (tile::gather4, local memory only), B as a 3-D box of the
//               tile's expert; STAGES-deep shared-memory ring of 128B-swizzled
//               K-major tiles (64 BF16 of K per stage).
//   warp 1      allocates TMEM; one lane issues tcgen05.mma (M=128, N=BN,
//               K=16 per instruction) and commits stage releases.
//   warps 2..5  epilogue: tcgen05.ld of the accumulator (warp w reads TMEM lane
//               quadrant w%4, i.e. one output row per thread) and a fused
//               per-use-site epilogue:
//     kEpiStore    bf16(acc [+ bias])                   router logits
//     kEpiSwiglu   bf16(bf16(silu(bf16(g))) * bf16(u))  expert / shared GEMM1,
//                  B rows hold [gate chunk | up chunk]
//     kEpiScatter  bf16(bf16(acc) * w_pair) -> Y[pair]  expert GEMM2
//     kEpiCombine  bf16(bf16(acc) + sum_j Y[t*k+j])     shared GEMM2 + combine
// The BF16 rounding points follow the reference's tensor boundaries
// (mESmaC/spalmer experts/bank.py:760-763, bank.py:970-978, nn/ffn.py:27-30,
// experts/mixer.py:207); accumulation is FP32 throughout.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "kernels.h"
#include "sm100.cuh"

namespace spx {

namespace {

__device__ __forceinline__ uint8_t* align_1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + expf(-x)); }

__device__ __forceinline__ void store_bf16x16(uint16_t* dst, const uint16_t (&h)[16], int valid) {
  if (valid >= 16 && (reinterpret_cast<uintptr_t>(dst) & 15u) == 0) {
    const uint4* s = reinterpret_cast<const uint4*>(h);
    reinterpret_cast<uint4*>(dst)[0] = s[0];
    reinterpret_cast<uint4*>(dst)[1] = s[1];
  } else {
#pragma unroll
    for (int j = 0; j < 16; ++j)
      if (j < valid) dst[j] = h[j];
  }
}

__device__ __forceinline__ void load_bf16x16_f32(const uint16_t* src, float (&f)[16], int valid) {
  if (valid >= 16 && (reinterpret_cast<uintptr_t>(src) & 15u) == 0) {
    uint4 q[2];
    q[0] = reinterpret_cast<const uint4*>(src)[0];
    q[1] = reinterpret_cast<const uint4*>(src)[1];
    const uint16_t* h = reinterpret_cast<const uint16_t*>(q);
#pragma unroll
    for (int j = 0; j < 16; ++j) f[j] = bf16_to_f32(h[j]);
  } else {
#pragma unroll
    for (int j = 0; j < 16; ++j) f[j] = j < valid ? bf16_to_f32(src[j]) : 0.0f;
  }
}

template <int EPI>
__device__ __forceinline__ void run_epilogue(const GemmArgs& a, uint32_t taddr, int r, int row0, int rows,
                                             int n0, int nt) {
  const bool live = r < rows;
  const int bn = a.bn;
  if constexpr (EPI == kEpiStore) {
    uint16_t* out = static_cast<uint16_t*>(a.out);
    for (int c = 0; c < bn; c += 16) {
      uint32_t v[16];
      tmem_ld16(taddr + c, v);
      tmem_wait_ld();
      const int gcol = n0 + c;
      const int valid = a.n_valid - gcol;
      if (live && valid > 0) {
        uint16_t h[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          float f = __uint_as_float(v[j]);
          if (a.bias != nullptr && j < valid) f += bf16_to_f32(a.bias[gcol + j]);
          h[j] = f32_to_bf16_rne(f);
        }
        store_bf16x16(out + static_cast<int64_t>(row0 + r) * a.ldo + gcol, h, valid);
      }
    }
  } else if constexpr (EPI == kEpiSwiglu) {
    uint16_t* out = static_cast<uint16_t*>(a.out);
    const int c_half = a.chunk;
    const int col0 = nt * c_half;
    for (int c = 0; c < c_half; c += 16) {
      uint32_t g[16], u[16];
      tmem_ld16(taddr + c, g);
      tmem_ld16(taddr + c_half + c, u);
      tmem_wait_ld();
      if (live) {
        uint16_t h[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const float gb = round_bf16(__uint_as_float(g[j]));
          const float ub = round_bf16(__uint_as_float(u[j]));
          const float sb = round_bf16(silu_f(gb));
          h[j] = f32_to_bf16_rne(sb * ub);
        }
        store_bf16x16(out + static_cast<int64_t>(row0 + r) * a.ldo + col0 + c, h, 16);
      }
    }
    // Zero the K padding of the hidden matrix (columns [chunks*c, h_cols)).
    if (live && nt == a.n_tiles - 1) {
      uint16_t* dst = out + static_cast<int64_t>(row0 + r) * a.ldo;
      for (int col = a.n_tiles * c_half; col < a.h_cols; ++col) dst[col] = 0;
    }
  } else if constexpr (EPI == kEpiScatter) {
    uint16_t* out = static_cast<uint16_t*>(a.out);
    int64_t pair = 0;
    float w = 0.0f;
    if (live) {
      pair = a.pos_to_pair[row0 + r];
      w = bf16_to_f32(a.pair_weight[pair]);
    }
    for (int c = 0; c < bn; c += 16) {
      uint32_t v[16];
      tmem_ld16(taddr + c, v);
      tmem_wait_ld();
      const int gcol = n0 + c;
      const int valid = a.n_valid - gcol;
      if (live && valid > 0) {
        uint16_t h[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) h[j] = f32_to_bf16_rne(round_bf16(__uint_as_float(v[j])) * w);
        store_bf16x16(out + pair * a.ldo + gcol, h, valid);
      }
    }
  } else {  // kEpiCombine
    uint16_t* out = static_cast<uint16_t*>(a.out);
    const int64_t t = static_cast<int64_t>(row0) + r;
    for (int c = 0; c < bn; c += 16) {
      uint32_t v[16];
      tmem_ld16(taddr + c, v);
      tmem_wait_ld();
      const int gcol = n0 + c;
      const int valid = a.n_valid - gcol;
      if (live && valid > 0) {
        float acc[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) acc[j] = round_bf16(__uint_as_float(v[j]));
        for (int s = 0; s < a.top_k; ++s) {
          float y[16];
          load_bf16x16_f32(a.y_pairs + (t * a.top_k + s) * a.ld_y + gcol, y, valid);
#pragma unroll
          for (int j = 0; j < 16; ++j) acc[j] += y[j];
        }
        uint16_t h[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) h[j] = f32_to_bf16_rne(acc[j]);
        store_bf16x16(out + t * a.ldo + gcol, h, valid);
      }
    }
  }
}

}  // namespace

// Tile coordinates of linear tile `t` (N tiles fastest, so consecutive tiles
// of one CTA share A rows in L2).  Returns false for a malformed table entry.
__device__ __forceinline__ bool decode_tile(const GemmArgs& a, int t, int& group, int& row0, int& rows, int& nt) {
  const int mt = t / a.n_tiles;
  nt = t - mt * a.n_tiles;
  if (a.tiles != nullptr) {
    const int4 e = a.tiles[mt];
    group = e.x;
    row0 = e.y;
    rows = e.z;
    return rows > 0 && rows <= kTileRows && group >= 0 && group < a.groups;
  }
  group = 0;
  row0 = mt * kTileRows;
  rows = min(kTileRows, a.m_rows - row0);
  return rows > 0;
}

// Persistent GEMM: each CTA walks tiles blockIdx.x, blockIdx.x + gridDim.x, ...
// The TMA producer and the MMA issuer stream k-blocks through the stage ring
// without stopping at tile boundaries; the accumulator is double-buffered in
// TMEM so the epilogue of one tile overlaps the MMAs of the next.
template <int EPI>
__global__ void __launch_bounds__(kGemmThreads, 1) gemm_kernel(const __grid_constant__ GemmArgs a) {
  extern __shared__ uint8_t gemm_smem_raw[];
  uint8_t* smem = align_1024(gemm_smem_raw);
  const int bn = a.bn;
  const int S = a.stages;
  const uint32_t a_bytes = kTileRows * 128u;
  const uint32_t b_bytes = static_cast<uint32_t>(bn) * 128u;
  uint8_t* sa = smem;
  uint8_t* sb = smem + S * a_bytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(sb + S * b_bytes);
  uint64_t* empty = full + S;
  uint64_t* tfull = empty + S;   // [2] accumulator ready
  uint64_t* tempty = tfull + 2;  // [2] accumulator drained
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int m_tiles = a.tiles != nullptr ? *a.num_tiles : (a.m_rows + kTileRows - 1) / kTileRows;
  const int total = m_tiles * a.n_tiles;
  if (static_cast<int>(blockIdx.x) >= total) return;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], kGemmEpilogueWarps);
    }
    fence_mbar_init();
    prefetch_tensormap(&a.tma_a);
    prefetch_tensormap(&a.tma_b);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 2 * a.tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer
    uint32_t it = 0;
    bool ok = true;
    for (int t = blockIdx.x; ok && t < total; t += gridDim.x) {
      int group, row0, rows, nt;
      if (!decode_tile(a, t, group, row0, rows, nt)) {
        if (lane == 0) record_error(a.status, SPX_DEV_BAD_TILE);
        break;
      }
      int gi0 = 0, gi1 = 0, gi2 = 0, gi3 = 0;
      if (a.gather) {
        const int r = lane * 4;
        gi0 = a.gather_idx[row0 + (r + 0 < rows ? r + 0 : 0)];
        gi1 = a.gather_idx[row0 + (r + 1 < rows ? r + 1 : 0)];
        gi2 = a.gather_idx[row0 + (r + 2 < rows ? r + 2 : 0)];
        gi3 = a.gather_idx[row0 + (r + 3 < rows ? r + 3 : 0)];
      }
      const int n0 = nt * bn;
      for (int kb = 0; kb < a.k_blocks; ++kb, ++it) {
        const int s = static_cast<int>(it % S);
        const uint32_t ph = (it / S) & 1u;
        int go = 1;
        if (lane == 0) {
          go = mbar_wait(&empty[s], ph ^ 1u, a.status, SPX_DEV_TIMEOUT_PRODUCER) ? 1 : 0;
          if (go) mbar_arrive_expect_tx(&full[s], a_bytes + b_bytes);
        }
        go = __shfl_sync(0xFFFFFFFFu, go, 0);
        if (!go) {
          ok = false;
          break;
        }
        if (a.gather) {
          tma_gather4(sa + s * a_bytes + lane * 512, &a.tma_a, &full[s], kb * 64, gi0, gi1, gi2, gi3);
        } else if (lane == 0) {
          tma_load_2d(sa + s * a_bytes, &a.tma_a, &full[s], kb * 64, row0);
        }
        if (lane == 0) tma_load_3d(sb + s * b_bytes, &a.tma_b, &full[s], kb * 64, n0, group);
        __syncwarp();
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16_f32(kTileRows, bn);
      uint32_t it = 0, lt = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < total; t += gridDim.x, ++lt) {
        const uint32_t b = lt & 1u;
        const uint32_t tph = (lt >> 1) & 1u;
        if (!mbar_wait(&tempty[b], tph ^ 1u, a.status, SPX_DEV_TIMEOUT_MMA)) break;
        tc_fence_after();
        const uint32_t acc = tmem + b * a.tmem_cols;
        for (int kb = 0; kb < a.k_blocks; ++kb, ++it) {
          const int s = static_cast<int>(it % S);
          const uint32_t ph = (it / S) & 1u;
          if (!mbar_wait(&full[s], ph, a.status, SPX_DEV_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(sa + s * a_bytes);
          const uint32_t b_base = smem_u32(sb + s * b_bytes);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            mma_bf16_ss(acc, desc_kmajor_sw128(a_base + kk * 32), desc_kmajor_sw128(b_base + kk * 32), idesc,
                        (kb | kk) != 0 ? 1u : 0u);
          }
          mma_commit(&empty[s]);
        }
        mma_commit(&tfull[b]);
      }
    }
    __syncwarp();
  } else {
    // ---------------- epilogue (warps 2..5): warp w drains TMEM lanes 32*(w%4) .. +31
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    uint32_t lt = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x, ++lt) {
      int group, row0, rows, nt;
      if (!decode_tile(a, t, group, row0, rows, nt)) break;
      const uint32_t b = lt & 1u;
      const uint32_t tph = (lt >> 1) & 1u;
      int go = 1;
      if (lane == 0) go = mbar_wait(&tfull[b], tph, a.status, SPX_DEV_TIMEOUT_EPILOGUE) ? 1 : 0;
      go = __shfl_sync(0xFFFFFFFFu, go, 0);
      if (!go) break;
      tc_fence_after();
      run_epilogue<EPI>(a, tmem + b * a.tmem_cols + (static_cast<uint32_t>(quad * 32) << 16), r, row0, rows,
                        nt * bn, nt);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[b]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 2 * a.tmem_cols);
  }
}

// ------------------------------------------------------------------ host side

namespace {

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

int get_encoder() {
  if (g_encode != nullptr) return SPX_OK;
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess || fn == nullptr)
    return SPX_ERR_DRIVER;
  g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  return SPX_OK;
}

}  // namespace

// 2-D BF16 tensor [rows, cols] (row pitch `ld` elements), box {64, box_rows}, 128B swizzle.
int encode_2d(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
  if (int rc = get_encoder(); rc != SPX_OK) return rc;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0 || (ld * 2) % 16 != 0) return SPX_ERR_ALIGNMENT;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * 2)};
  cuuint32_t box[2] = {64u, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? SPX_OK : SPX_ERR_DRIVER;
}

// 3-D BF16 tensor [groups, rows, cols], box {64, box_rows, 1}, 128B swizzle.
int encode_3d(CUtensorMap* map, const void* base, int64_t groups, int64_t rows, int64_t cols, int box_rows) {
  if (int rc = get_encoder(); rc != SPX_OK) return rc;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0 || (cols * 2) % 16 != 0) return SPX_ERR_ALIGNMENT;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows),
                        static_cast<cuuint64_t>(groups)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(cols * 2), static_cast<cuuint64_t>(rows * cols * 2)};
  cuuint32_t box[3] = {64u, static_cast<cuuint32_t>(box_rows), 1u};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? SPX_OK : SPX_ERR_DRIVER;
}

size_t gemm_smem_bytes(int bn, int stages) {
  return 1024 + static_cast<size_t>(stages) * (kTileRows * 128 + static_cast<size_t>(bn) * 128) +
         (2 * stages + 4) * 8 + 16;
}

// As many stages as fit: the persistent producer keeps prefetching the next
// tile's k-blocks, so stages beyond one tile's K still hide load latency.
int gemm_pick_stages(int bn, int k_blocks) {
  (void)k_blocks;
  int stages = 2;
  for (int s = 3; s <= 8; ++s)
    if (gemm_smem_bytes(bn, s) <= kGemmSmemBudget) stages = s;
  return stages;
}

template <int EPI>
static int launch_gemm_t(const GemmArgs& a, int grid_m, int grid_n, cudaStream_t stream) {
  const size_t smem = gemm_smem_bytes(a.bn, a.stages);
  if (int rc = ensure_max_dynamic_smem(reinterpret_cast<const void*>(gemm_kernel<EPI>)); rc != SPX_OK) return rc;
  // Persistent grid: one CTA per SM, never more CTAs than (upper bound of) tiles.
  const int sms = device_sm_count();
  const int64_t tiles = static_cast<int64_t>(grid_m) * grid_n;
  const int grid = static_cast<int>(tiles < sms ? tiles : sms);
  GemmArgs b = a;
  b.n_tiles = grid_n;
  gemm_kernel<EPI><<<grid, kGemmThreads, smem, stream>>>(b);
  return cudaGetLastError() == cudaSuccess ? SPX_OK : SPX_ERR_CUDA;
}

int launch_gemm(int epi, const GemmArgs& a, int grid_m, int grid_n, cudaStream_t stream) {
  if (grid_m <= 0 || grid_n <= 0) return SPX_OK;
  if (a.bn < 16 || a.bn > 256 || (a.bn % 16) != 0) return SPX_ERR_UNSUPPORTED;
  switch (epi) {
    case kEpiStore:
      return launch_gemm_t<kEpiStore>(a, grid_m, grid_n, stream);
    case kEpiSwiglu:
      return launch_gemm_t<kEpiSwiglu>(a, grid_m, grid_n, stream);
    case kEpiScatter:
      return launch_gemm_t<kEpiScatter>(a, grid_m, grid_n, stream);
    case kEpiCombine:
      return launch_gemm_t<kEpiCombine>(a, grid_m, grid_n, stream);
    default:
      return SPX_ERR_INVALID_ARG;
  }
}

}  // namespace spx
