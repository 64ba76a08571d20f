// Routed experts' weight gradients on tcgen05: for every expert e,
//
//   out[e] = A_e^T . B_e      (FP32 accumulation, one BF16 rounding)
//
// where A_e, B_e are the expert's rows of two matrices kept in dispatch order
// (rows of one expert contiguous): d gate | d up = x_e^T . [dg | du]_e and
// d down = bf16(h w)_e^T . dU_e (the routing weight on the hidden rows) --
// the gradients autograd gives the reference's
// expert parameters (experts/bank.py:755-763 differentiated; its grouped
// executor's torch.bmm / grouped GEMMs).  The reduction runs over an
// expert's rows, so both operands enter the MMA MN-major: TMA copies
// 64-row x 64-column boxes (128-byte swizzle) straight from the row-major
// matrices, and the shared-memory descriptors describe them as the
// canonical MN-major layout (LBO = 8 KB between 64-column boxes, SBO = 1 KB
// between 8-row groups along K); nothing is transposed in memory.
//
// One operand may instead be gathered from unsorted rows (x rows by token for
// d gate | d up, dU rows by token for d down), so no sorted copies (two
// P x d matrices) are needed.  The producer loads
// a gathered operand with TMA gathers (four rows of 64 columns per
// instruction, the 128-byte swizzle of the box layout the MMA expects).
//
// A CTA (persistent, one per SM) walks tiles (expert, 128 output rows, bn
// output columns) expert-major, so the tiles of one expert run side by side
// and share its rows through L2.  Warp roles: 0 TMA producer, 1 MMA issuer
// (and TMEM owner), 2-3 fixers -- an expert's last K block holds rows of the
// next expert (or TMA zero fill past the end); the fixers zero the rows past
// the segment in shared memory and pass the
// stage on --, 4-7 epilogue (TMEM lane quadrants 0-3).  Two accumulators of
// bn columns let the epilogue of one tile overlap the MMAs of the next.
// Experts without rows get zero gradients.  Every wait is bounded (status
// word, then return).
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

#include "kernels.h"
#include "sm100.cuh"

namespace spx {

namespace {

constexpr int kWgThreads = 256;
constexpr int kWgBoxBytes = 64 * 128;  // one TMA box: 64 rows x 64 BF16 columns
constexpr int kWgMaxExperts = 1024;
constexpr int kWgFixers = 2;           // warps 2 and 3

// Shared-memory descriptor of an MN-major operand tile made of 64-column
// boxes (128-byte rows, 128B swizzle) laid out one after another.
__device__ __forceinline__ uint64_t desc_mnmajor_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>(kWgBoxBytes >> 4) << 16;  // LBO: next 64 MN elements (next box)
  d |= static_cast<uint64_t>(1024u >> 4) << 32;        // SBO: next 8 K rows
  d |= static_cast<uint64_t>(1u) << 46;                // version
  d |= static_cast<uint64_t>(2u) << 61;                // SWIZZLE_128B
  return d;
}

struct WgTile {
  int e, mt, nt;
};

__device__ __forceinline__ WgTile wg_tile(const WgradArgs& a, int t) {
  const int per = a.m_tiles * a.n_tiles;
  WgTile w;
  w.e = t / per;
  const int r = t - w.e * per;
  w.mt = r / a.n_tiles;
  w.nt = r - w.mt * a.n_tiles;
  return w;
}

}  // namespace

__global__ void __launch_bounds__(kWgThreads, 1) wgrad_kernel(const __grid_constant__ WgradArgs a) {
  extern __shared__ uint8_t wg_smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(wg_smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = a.stages;
  const int nbox_b = a.bn / 64;
  const uint32_t a_bytes = 2 * kWgBoxBytes;
  const uint32_t b_bytes = static_cast<uint32_t>(nbox_b) * kWgBoxBytes;
  const uint32_t stage_bytes = a_bytes + b_bytes;
  const bool gathered = a.g_src != nullptr;
  // TMA bytes per stage (the stored operands)
  const uint32_t tma_bytes = (gathered && a.g_is_a ? 0u : a_bytes) + (gathered && !a.g_is_a ? 0u : b_bytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * stage_bytes);
  uint64_t* ready = full + S;   // the fixer has passed the stage on
  uint64_t* empty = ready + S;
  uint64_t* tfull = empty + S;   // [2]
  uint64_t* tempty = tfull + 2;  // [2]
  uint64_t* drained = tempty + 2;  // every MMA issued by this CTA has completed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drained + 1);
  int* s_start = reinterpret_cast<int*>(tmem_slot + 4);  // [E]
  int* s_count = s_start + kWgMaxExperts;                // [E]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int total = a.E * a.m_tiles * a.n_tiles;

  // expert starts: exclusive scan of the counts (E <= 1024, 4 per thread)
  {
    __shared__ int part[kWgThreads / 32];
    int c[4], sum = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int e = threadIdx.x * 4 + j;
      c[j] = e < a.E ? a.counts[e] : 0;
      sum += c[j];
    }
    int incl = sum;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int v = __shfl_up_sync(0xFFFFFFFFu, incl, off);
      if (lane >= off) incl += v;
    }
    if (lane == 31) part[warp] = incl;
    if (threadIdx.x == 0) {
      for (int s = 0; s < S; ++s) {
        mbar_init(&full[s], 1);
        mbar_init(&ready[s], kWgFixers);
        mbar_init(&empty[s], 1);
      }
      for (int b = 0; b < 2; ++b) {
        mbar_init(&tfull[b], 1);
        mbar_init(&tempty[b], 4);
      }
      mbar_init(drained, 1);
      fence_mbar_init();
      prefetch_tensormap(&a.tma_a);
      prefetch_tensormap(&a.tma_b);
    }
    if (warp == 1) {
      tmem_alloc(tmem_slot, 2u * static_cast<uint32_t>(a.bn));
      tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    int base = 0;
    for (int w = 0; w < warp; ++w) base += part[w];
    int run = base + incl - sum;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int e = threadIdx.x * 4 + j;
      if (e < a.E) {
        s_start[e] = run;
        s_count[e] = c[j];
      }
      run += c[j];
    }
    __syncthreads();
  }
  const uint32_t tmem = *tmem_slot;
  auto kblocks = [&](int e) { return (s_count[e] + 63) / 64; };

  if (warp == 0) {
    // ---------------- producer (TMA): stored operands as 64 x 64 boxes, a
    // gathered one four rows at a time (tile::gather4; lane l of 0..15 takes
    // block rows 4l .. 4l + 3 of every box).  Rows past the expert's segment
    // are loaded from the block's first row and zeroed by the fixers.
    const int gboxes = gathered ? (a.g_is_a ? 2 : nbox_b) : 0;
    const uint32_t g_bytes = static_cast<uint32_t>(gboxes) * kWgBoxBytes;
    uint32_t it = 0;
    bool ok = true;
    for (int t = blockIdx.x; ok && t < total; t += gridDim.x) {
      const WgTile w = wg_tile(a, t);
      const int nkb = kblocks(w.e);
      const int start = s_start[w.e], cnt = s_count[w.e];
      for (int kb = 0; kb < nkb; ++kb, ++it) {
        const int s = static_cast<int>(it % S);
        const uint32_t ph = (it / S) & 1u;
        const int row = start + kb * 64;
        const int valid = cnt - kb * 64;  // rows of this block inside the segment (> 0)
        int src[4] = {0, 0, 0, 0};
        if (gathered && lane < 16) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int rr = 4 * lane + q;
            src[q] = __ldg(a.g_index + row + (rr < valid ? rr : 0));
          }
        }
        int go = 1;
        if (lane == 0) {
          go = mbar_wait(&empty[s], ph ^ 1u, a.status, SPX_DEV_TIMEOUT_PRODUCER) ? 1 : 0;
          if (go) {
            mbar_arrive_expect_tx(&full[s], tma_bytes + g_bytes);
            uint8_t* st = smem + s * stage_bytes;
            if (!gathered || !a.g_is_a) {
              tma_load_2d(st, &a.tma_a, &full[s], w.mt * 128, row);
              tma_load_2d(st + kWgBoxBytes, &a.tma_a, &full[s], w.mt * 128 + 64, row);
            }
            if (!gathered || a.g_is_a) {
              for (int j = 0; j < nbox_b; ++j)
                tma_load_2d(st + a_bytes + j * kWgBoxBytes, &a.tma_b, &full[s], w.nt * a.bn + 64 * j, row);
            }
          }
        }
        go = __shfl_sync(0xFFFFFFFFu, go, 0);
        if (!go) {
          ok = false;
          break;
        }
        if (gathered && lane < 16) {  // after lane 0's expect_tx (the shuffle above orders them)
          const uint32_t base = smem_u32(smem + s * stage_bytes) + (a.g_is_a ? 0u : a_bytes) + lane * 512u;
          const CUtensorMap* map = a.g_is_a ? &a.tma_a : &a.tma_b;
          const int col0 = a.g_is_a ? w.mt * 128 : w.nt * a.bn;
          for (int j = 0; j < gboxes; ++j)
            tma_gather4_2d(base + j * kWgBoxBytes, map, &full[s], col0 + 64 * j, src[0], src[1], src[2], src[3]);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16_f32(128, a.bn) | (1u << 15) | (1u << 16);  // A and B MN-major
      uint32_t it = 0, lt = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < total; t += gridDim.x) {
        const WgTile w = wg_tile(a, t);
        const int nkb = kblocks(w.e);
        if (nkb == 0) continue;  // the epilogue writes zeros without an accumulator
        const uint32_t b = lt & 1u;
        if (!mbar_wait(&tempty[b], ((lt >> 1) & 1u) ^ 1u, a.status, SPX_DEV_TIMEOUT_MMA)) break;
        tc_fence_after();
        const uint32_t acc = tmem + b * static_cast<uint32_t>(a.bn);
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = static_cast<int>(it % S);
          // the fixer passes every stage on, after zeroing the tail rows of the last block
          if (!mbar_wait(&ready[s], (it / S) & 1u, a.status, SPX_DEV_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + s * stage_bytes);
          const uint32_t sb = sa + a_bytes;
#pragma unroll
          for (uint32_t q = 0; q < 4; ++q)  // K = 16 rows per MMA: 2 KB of each box
            mma_bf16_ss(acc, desc_mnmajor_sw128(sa + q * 2048u), desc_mnmajor_sw128(sb + q * 2048u), idesc,
                        (kb != 0 || q != 0) ? 1u : 0u);
          mma_commit(&empty[s]);
        }
        if (!ok) break;
        mma_commit(&tfull[b]);
        ++lt;
      }
      mma_commit(drained);  // arrives once everything issued above has completed
    }
  } else if (warp == 2 || warp == 3) {
    // ---------------- fixers: a pipeline stage between the loads and the MMA.
    // They pass every stage on in order (so no barrier phase can be skipped or
    // overtaken); first they zero the rows past the expert's segment in the
    // segment's last block (split between the two fixers).
    const int f = warp - 2;
    uint32_t it = 0;
    bool ok = true;
    for (int t = blockIdx.x; ok && t < total; t += gridDim.x) {
      const WgTile w = wg_tile(a, t);
      const int cnt = s_count[w.e];
      const int nkb = kblocks(w.e);
      for (int kb = 0; kb < nkb; ++kb, ++it) {
        const int s = static_cast<int>(it % S);
        const int valid = cnt - kb * 64;
        int go = 1;
        if (lane == 0) go = mbar_wait(&full[s], (it / S) & 1u, a.status, SPX_DEV_TIMEOUT_PRODUCER) ? 1 : 0;
        go = __shfl_sync(0xFFFFFFFFu, go, 0);
        if (!go) {
          ok = false;
          break;
        }
        uint8_t* st = smem + s * stage_bytes;
        bool wrote = false;
        if (valid < 64) {
          // rows [valid, 64) of every box: whole 128-byte rows (the swizzle stays inside a row)
          const int nbox = 2 + nbox_b;
          const int chunks = (64 - valid) * 8;  // 16-byte chunks per box
          for (int i = f * 32 + lane; i < nbox * chunks; i += 32 * kWgFixers) {
            const int box = i / chunks, c = i - box * chunks;
            *reinterpret_cast<uint4*>(st + box * kWgBoxBytes + valid * 128 + c * 16) = make_uint4(0u, 0u, 0u, 0u);
          }
          wrote = true;
        }
        if (wrote) fence_proxy_async_smem();  // generic-proxy writes -> the MMA's operand reads
        __syncwarp();
        if (lane == 0) mbar_arrive(&ready[s]);
      }
    }
  } else if (warp >= 4) {
    // ---------------- epilogue: TMEM lanes 32*(warp%4) .. +32
    const int quad = warp & 3;
    uint32_t lt = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x) {
      const WgTile w = wg_tile(a, t);
      const int m = w.mt * 128 + quad * 32 + lane;
      const bool row_ok = m < a.m_total;
      const bool empty_tile = kblocks(w.e) == 0;
      const uint32_t b = lt & 1u;
      if (!empty_tile) {
        int go = 1;
        if (lane == 0) go = mbar_wait(&tfull[b], (lt >> 1) & 1u, a.status, SPX_DEV_TIMEOUT_EPILOGUE) ? 1 : 0;
        go = __shfl_sync(0xFFFFFFFFu, go, 0);
        if (!go) break;
        tc_fence_after();
      }
      for (int c0 = 0; c0 < a.bn; c0 += 32) {
        uint32_t r[32];
        if (!empty_tile) {
          tmem_ld32(tmem + b * static_cast<uint32_t>(a.bn) + static_cast<uint32_t>(c0) + ((quad * 32u) << 16), r);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) r[j] = 0u;
        }
        // output columns n .. n+31 of the tile: out0 [0, n_valid0), out1 [n_start1, n_start1 + n_valid1)
        const int n = w.nt * a.bn + c0;
        uint16_t* dst = nullptr;
        int col = 0, valid = 0;
        if (n < a.n_valid0) {
          dst = a.out0 + (static_cast<int64_t>(w.e) * a.m_total + m) * a.ld0;
          col = n;
          valid = a.n_valid0 - n;
        } else if (a.out1 != nullptr && n >= a.n_start1 && n < a.n_start1 + a.n_valid1) {
          dst = a.out1 + (static_cast<int64_t>(w.e) * a.m_total + m) * a.ld1;
          col = n - a.n_start1;
          valid = a.n_start1 + a.n_valid1 - n;
        }
        if (dst == nullptr || !row_ok) continue;
        uint32_t h[16];
#pragma unroll
        for (int j = 0; j < 16; ++j)
          h[j] = static_cast<uint32_t>(f32_to_bf16_rne(__uint_as_float(r[2 * j]))) |
                 (static_cast<uint32_t>(f32_to_bf16_rne(__uint_as_float(r[2 * j + 1]))) << 16);
        if (valid >= 32 && (col % 8) == 0) {
          uint4* d4 = reinterpret_cast<uint4*>(dst + col);
#pragma unroll
          for (int j = 0; j < 4; ++j) d4[j] = make_uint4(h[4 * j], h[4 * j + 1], h[4 * j + 2], h[4 * j + 3]);
        } else {
          for (int j = 0; j < 32 && j < valid; ++j)
            dst[col + j] = static_cast<uint16_t>(j & 1 ? h[j / 2] >> 16 : h[j / 2] & 0xFFFFu);
        }
      }
      if (!empty_tile) {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[b]);
        ++lt;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    // no MMA may still write the accumulators when they are freed
    if (lane == 0) mbar_wait(drained, 0u, a.status, SPX_DEV_TIMEOUT_MMA);
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 2u * static_cast<uint32_t>(a.bn));
  }
}

size_t wgrad_smem_bytes(int bn, int stages) {
  return 1024 + static_cast<size_t>(stages) * (2 + bn / 64) * kWgBoxBytes + (3 * stages + 5) * 8 + 16 +
         2 * kWgMaxExperts * sizeof(int);
}

// out0/out1 as WgradArgs; A has m_total columns (a.total), B n_total (b.total),
// each either stored [rows, total] (ld) or gathered (at most one of them).
int launch_wgrad(const WgradOperand& A, const WgradOperand& B, int64_t rows, const int* counts, int E,
                 uint16_t* out0, int ld0, int n_valid0, uint16_t* out1, int ld1, int n_start1, int n_valid1,
                 int* status, cudaStream_t stream) {
  const int m_total = A.total, n_total = B.total;
  if (E <= 0 || E > kWgMaxExperts || m_total <= 0 || n_total <= 0 || out0 == nullptr) return SPX_ERR_INVALID_ARG;
  if (m_total % 8 != 0 || n_total % 8 != 0 || ld0 % 8 != 0 || (out1 != nullptr && ld1 % 8 != 0) || A.ld % 8 != 0 ||
      B.ld % 8 != 0)
    return SPX_ERR_UNSUPPORTED;  // 16-byte rows for TMA, cp.async and the vector stores
  const bool ga = A.rows == nullptr, gb = B.rows == nullptr;
  if ((ga && gb) || (ga && (A.src == nullptr || A.index == nullptr)) ||
      (gb && (B.src == nullptr || B.index == nullptr)))
    return SPX_ERR_INVALID_ARG;
  WgradArgs w{};
  // empty batches still need the zero gradients: a 1-row view keeps the maps valid
  const int64_t map_rows = rows > 0 ? rows : 1;
  // stored operands: 64-row boxes; a gathered one: one-row boxes over its
  // source rows (tile::gather4)
  if (int rc = ga ? encode_2d(&w.tma_a, A.src, std::max<int64_t>(A.src_rows, 1), m_total, A.ld, 1)
                  : encode_2d(&w.tma_a, A.rows, map_rows, m_total, A.ld, 64);
      rc != SPX_OK)
    return rc;
  if (int rc = gb ? encode_2d(&w.tma_b, B.src, std::max<int64_t>(B.src_rows, 1), n_total, B.ld, 1)
                  : encode_2d(&w.tma_b, B.rows, map_rows, n_total, B.ld, 64);
      rc != SPX_OK)
    return rc;
  if (ga || gb) {
    const WgradOperand& g = ga ? A : B;
    w.g_src = g.src;
    w.g_index = g.index;
    w.g_ld = g.ld;
    w.g_is_a = ga ? 1 : 0;
  }
  w.n_total = n_total;
  w.counts = counts;
  w.E = E;
  w.m_total = m_total;
  w.bn = 64;  // accumulator columns: 64, 128 or 256 (two of them fill at most the 512 TMEM columns)
  while (w.bn < 256 && w.bn < n_total) w.bn *= 2;
  w.m_tiles = (m_total + 127) / 128;
  w.n_tiles = (n_total + w.bn - 1) / w.bn;
  w.out0 = out0;
  w.ld0 = ld0;
  w.n_valid0 = n_valid0;
  w.out1 = out1;
  w.ld1 = ld1;
  w.n_start1 = n_start1;
  w.n_valid1 = n_valid1;
  w.status = status;
  int stages = 2;
  for (int s = 3; s <= 6; ++s)
    if (wgrad_smem_bytes(w.bn, s) <= kGemmSmemBudget) stages = s;
  w.stages = stages;
  const size_t smem = wgrad_smem_bytes(w.bn, stages);
  if (smem > kGemmSmemBudget) return SPX_ERR_UNSUPPORTED;
  if (int rc = ensure_max_dynamic_smem(reinterpret_cast<const void*>(wgrad_kernel)); rc != SPX_OK) return rc;
  const int total = E * w.m_tiles * w.n_tiles;
  const int sms = device_sm_count();
  const int grid = std::min(total, sms > 0 ? sms : 148);
  wgrad_kernel<<<grid, kWgThreads, smem, stream>>>(w);
  return cudaGetLastError() == cudaSuccess ? SPX_OK : SPX_ERR_CUDA;
}

}  // namespace spx
