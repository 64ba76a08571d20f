// tcgen05 GEMM engine for the micro-expert layer (sm_100a).
//
// C[128-row tile, BN cols] = A[rows, K] * B[group][BN rows, K]^T, BF16 operands,
// FP32 accumulation in tensor memory.  Persistent: one CTA per SM walks the
// tiles; the accumulator is double-buffered in TMEM.  Warp roles:
//   warp 0      producer: B (and ungathered A) as TMA boxes; gathered A rows
//               (the dispatched tokens of an expert tile) with cp.async, 4 rows
//               x 128 B per instruction -- measured 1.7x faster on this
//               kernel than TMA tile::gather4; STAGES-deep shared-memory
//               ring of 128B-swizzled K-major tiles (64 BF16 of K per stage).
//               In the BF16 instantiations that gather, warp 10 gathers the
//               second half of each tile's rows (one warp could not keep the
//               tensor pipe fed: expert GEMM1 246 vs 269 us at the 100M shape).
//   warp 1      allocates TMEM; one lane issues tcgen05.mma (M=128, N=BN,
//               K=16 per instruction) and commits stage releases.
//   warps 2..9  epilogue: tcgen05.ld of the accumulator (warp w reads TMEM lane
//               quadrant w%4, i.e. one output row per thread, two warps per
//               quadrant splitting the columns) and a fused per-use-site epilogue:
//     kEpiStore    bf16(acc [+ bias])                   router logits
//     kEpiSwiglu   bf16(bf16(silu(bf16(g))) * bf16(u))  expert / shared GEMM1,
//                  B rows hold [gate chunk | up chunk]
//     kEpiStore    (also) shared down projection -> shared output
//     kEpiScatter  bf16(bf16(acc) * w_pos) -> Y[pos]    expert GEMM2: rows in sorted
//                  (dispatch) order, written by TMA tile stores
// The BF16 rounding points follow the reference's tensor boundaries
// (mESmaC/spalmer experts/bank.py:760-763, bank.py:970-978, nn/ffn.py:27-30,
// experts/mixer.py:207); accumulation is FP32 throughout.
//
// MXFP8 lane (template flag MX): E4M3 operands (128 elements = 128 B of K per
// stage) with E8M0 scales per 32 elements.  The producer also copies one
// 512-byte scale atom for A (gathered 4-byte words, one per row) and one for
// B (pre-packed) per stage; the MMA warp moves them to tensor memory with
// tcgen05.cp and issues kind::mxf8f6f4.block_scale MMAs (K = 32).  TMEM holds
// three 128-column accumulators and rotating scale slots from column 384.
// The SwiGLU epilogue of this lane writes the hidden rows already quantised
// (the reference quantises `silu(g) * u` row-wise before the down
// projection, experts/native.py:113-140 via bank.py:440-461).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "kernels.h"
#include "mx.cuh"
#include "nv.cuh"
#include "sm100.cuh"

namespace spx {

namespace {

__device__ __forceinline__ uint8_t* align_1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

// Epilogue arithmetic on BF16 pairs.  The hardware conversions round to
// nearest even like the reference's CPU tensors (NaN payloads aside).
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ float lo_f(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float hi_f(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
// Both values rounded to BF16 (nearest even) and widened back, with one
// packed conversion instead of two scalar ones.
__device__ __forceinline__ void bfr2(float& x, float& y) {
  const uint32_t p = pack_bf16x2(x, y);
  x = lo_f(p);
  y = hi_f(p);
}
// Product of two BF16 pairs, rounded to nearest even in one instruction.  The
// FP32 product of two BF16 values is exact (8 x 8 significant bits) above the
// FP32 normal range's floor, so this is pack_bf16x2(lo_f(a) * lo_f(b), ...)
// bit for bit -- the reference's BF16 tensor multiply -- for every operand
// pair whose product is at least 2^-126 in magnitude (or zero, inf, NaN).
__device__ __forceinline__ uint32_t bmul2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
// silu(x) = x / (1 + e^-x); approximate exp/divide, the result is rounded to BF16.
__device__ __forceinline__ float silu_fast(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

// Epilogue staging: each epilogue warp owns a 32-row x 64-column BF16 slice
// buffer (4 KB).  Threads write their own row (TMEM lane = row), then the warp
// writes 4 rows x 128 B per instruction, so global stores (and the combine's
// loads of Y) move whole row segments.  16-byte chunk c of row i sits at chunk
// position c ^ (i & 7): conflict-free for both access patterns.
__device__ __forceinline__ uint32_t stage_off(int i, int chunk) {
  return static_cast<uint32_t>(i * 128 + ((chunk ^ (i & 7)) << 4));
}

// 16 BF16 values (8 packed words) of row i starting at column col (multiple of 16).
__device__ __forceinline__ void stage_put16(uint8_t* buf, int i, int col, const uint32_t* w) {
  *reinterpret_cast<uint4*>(buf + stage_off(i, col >> 3)) = make_uint4(w[0], w[1], w[2], w[3]);
  *reinterpret_cast<uint4*>(buf + stage_off(i, (col >> 3) + 1)) = make_uint4(w[4], w[5], w[6], w[7]);
}

__device__ __forceinline__ void put8(uint16_t* dst, const uint4& v, int n) {
  if (n >= 8 && (reinterpret_cast<uintptr_t>(dst) & 15u) == 0) {
    *reinterpret_cast<uint4*>(dst) = v;
  } else {
    const uint16_t* h = reinterpret_cast<const uint16_t*>(&v);
    for (int j = 0; j < n; ++j) dst[j] = h[j];
  }
}

// One epilogue warp: TMEM lane quadrant `quad` (32 tile rows), output column
// slices half, half + 2, ... of the tile (two warps share a quadrant).
// `my_row` is the output row of this thread's tile row.
// SC (NVFP4 lane): the accumulator is first scaled by alpha0 (alpha1 for the
// up half of a SwiGLU tile), and a SwiGLU tile raises *amax_out to the
// largest |hidden| it writes.
template <int EPI, bool SC = false>
__device__ __forceinline__ void run_epilogue(const GemmArgs& a, uint32_t taddr, uint8_t* stage, int quad, int half,
                                             int lane, int row0, int rows, int n0, int nt, long long my_row,
                                             float alpha0 = 1.0f, float alpha1 = 1.0f, float* amax_out = nullptr) {
  float hmax = 0.0f;
  constexpr int W = (EPI == kEpiSwiglu) ? 32 : 64;  // output columns per slice
  const int r = quad * 32 + lane;                   // tile row owned by this thread (its TMEM lane)
  const bool live = r < rows;
  const int wrows = rows - quad * 32;               // valid rows of this quadrant (may be <= 0)
  uint16_t* out = static_cast<uint16_t*>(a.out);
  const int out_cols = (EPI == kEpiSwiglu) ? a.chunk : a.bn;
  const int col_base = (EPI == kEpiSwiglu) ? nt * a.chunk : n0;
  for (int s0 = half * W; s0 < out_cols; s0 += 2 * W) {
    const int w = min(W, out_cols - s0);
    // 1) accumulator -> registers (one TMEM wait per slice) -> staged BF16 row slice
    uint32_t hw[W / 2];
    if constexpr (EPI == kEpiSwiglu) {
      uint32_t g[32], u[32];
      tmem_ld32(taddr + s0, g);
      tmem_ld32(taddr + a.chunk + s0, u);
      tmem_wait_ld();
#pragma unroll
      for (int j = 0; j < 32; j += 2) {
        float g0 = __uint_as_float(g[j]), g1 = __uint_as_float(g[j + 1]);
        float u0 = __uint_as_float(u[j]), u1 = __uint_as_float(u[j + 1]);
        if constexpr (SC) {
          g0 *= alpha0;
          g1 *= alpha0;
          u0 *= alpha1;
          u1 *= alpha1;
        }
        bfr2(g0, g1);
        const uint32_t u2 = pack_bf16x2(u0, u1);
        hw[j / 2] = bmul2(pack_bf16x2(silu_fast(g0), silu_fast(g1)), u2);
        if constexpr (SC) {
          if (live && j < w) hmax = fmaxf(hmax, fabsf(lo_f(hw[j / 2])));
          if (live && j + 1 < w) hmax = fmaxf(hmax, fabsf(hi_f(hw[j / 2])));
        }
      }
    } else {
      uint32_t v[64];
      tmem_ld32(taddr + s0, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
      if (w > 32) tmem_ld32(taddr + s0 + 32, *reinterpret_cast<uint32_t(*)[32]>(&v[32]));
      tmem_wait_ld();
      if constexpr (EPI == kEpiStore) {
        const int gcol = col_base + s0;
#pragma unroll
        for (int j = 0; j < 64; j += 2) {
          float f0 = __uint_as_float(v[j]), f1 = __uint_as_float(v[j + 1]);
          if constexpr (SC) {
            f0 *= alpha0;
            f1 *= alpha0;
          }
          if (a.bias != nullptr) {
            if (j < w && gcol + j < a.n_valid) f0 += bf16_to_f32(a.bias[gcol + j]);
            if (j + 1 < w && gcol + j + 1 < a.n_valid) f1 += bf16_to_f32(a.bias[gcol + j + 1]);
          }
          hw[j / 2] = pack_bf16x2(f0, f1);
        }
      }
    }
#pragma unroll
    for (int c = 0; c < W; c += 16) stage_put16(stage, lane, c, &hw[c / 2]);
    __syncwarp();
    // 2) staged rows -> global: lane group (lane >> 3) takes one row, lane & 7 its 16-byte chunk
    const int gcol0 = col_base + s0;
    const int valid = (EPI == kEpiSwiglu) ? w : min(w, a.n_valid - gcol0);
    const int j = lane & 7;
#pragma unroll 2
    for (int step = 0; step < 8; ++step) {
      const int ri = step * 4 + (lane >> 3);
      const long long rowid = __shfl_sync(0xFFFFFFFFu, my_row, ri);
      const int n = min(8, valid - j * 8);
      if (ri < wrows && n > 0) {
        uint4 v = *reinterpret_cast<const uint4*>(stage + stage_off(ri, j));
        put8(out + rowid * a.ldo + gcol0 + j * 8, v, n);
      }
    }
    __syncwarp();
  }
  if constexpr (EPI == kEpiSwiglu) {
    // Zero the K padding of the hidden matrix (columns [chunks*c, h_cols)).
    if (half == 0 && live && nt == a.n_tiles - 1) {
      uint16_t* dst = out + static_cast<int64_t>(row0 + r) * a.ldo;
      for (int col = a.n_tiles * a.chunk; col < a.h_cols; ++col) dst[col] = 0;
    }
    if constexpr (SC) {
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) hmax = fmaxf(hmax, __shfl_xor_sync(0xFFFFFFFFu, hmax, off));
      if (lane == 0 && amax_out != nullptr && hmax > 0.0f)
        atomicMax(reinterpret_cast<int*>(amax_out), __float_as_int(hmax));
    }
  }
}

// Expert GEMM2 epilogue: bf16(bf16(acc) * w) rows written in sorted order.
// Each 32-row x 64-column slice is staged in one of the warp's two 4 KB
// buffers (the 128B-swizzled layout of the output tensor map's box) and sent
// with one TMA tile store, so the warp moves on while the copy drains.  A
// warp whose 32 rows are not all inside the tile (the last tile of an expert)
// stores its valid rows with plain stores instead: a box would spill into the
// next expert's rows.  `slices` counts this warp's slices across tiles (it
// picks the buffer); `committed` remembers whether the previous slice left a
// bulk group behind.
__device__ __forceinline__ void run_epilogue_rows(const GemmArgs& a, uint32_t taddr, uint8_t* stage, int quad,
                                                  int half, int lane, int row0, int rows, int n0, float my_w,
                                                  uint32_t& slices, bool& committed, float alpha = 1.0f) {
  const int wrows = rows - quad * 32;  // valid rows of this quadrant
  if (wrows <= 0) return;
  uint16_t* out = static_cast<uint16_t*>(a.out);
  const uint32_t w2 = pack_bf16x2(my_w, my_w);  // my_w is a BF16 routing weight (or 1)
  for (int s0 = half * 64; s0 < a.bn; s0 += 128) {
    uint8_t* buf = stage + (slices & 1u) * kStageBytesPerWarp;
    ++slices;
    // The bulk store that last read `buf` (two slices ago) must be done reading.
    if (lane == 0) {
      if (committed)
        bulk_wait_read<1>();
      else
        bulk_wait_read<0>();
    }
    __syncwarp();
    const int w = min(64, a.bn - s0);
    uint32_t v[64];
    tmem_ld32(taddr + s0, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
    if (w > 32) tmem_ld32(taddr + s0 + 32, *reinterpret_cast<uint32_t(*)[32]>(&v[32]));
    tmem_wait_ld();
    uint32_t hw[32];
#pragma unroll
    for (int j = 0; j < 64; j += 2)
      hw[j / 2] = bmul2(pack_bf16x2(__uint_as_float(v[j]) * alpha, __uint_as_float(v[j + 1]) * alpha), w2);
#pragma unroll
    for (int c = 0; c < 64; c += 16) stage_put16(buf, lane, c, &hw[c / 2]);
    const int gcol0 = n0 + s0;
    if (wrows >= 32 && a.tma_store && a.row_out == nullptr) {
      fence_proxy_async_smem();  // generic-proxy staging writes -> TMA reads
      __syncwarp();
      if (lane == 0) {
        tma_store_2d(&a.tma_out, buf, gcol0, row0 + quad * 32);
        bulk_commit();
      }
      committed = true;
    } else {
      __syncwarp();
      const int valid = min(w, a.n_valid - gcol0);
      const int j = lane & 7;
#pragma unroll 2
      for (int step = 0; step < 8; ++step) {
        const int ri = step * 4 + (lane >> 3);
        const int n = min(8, valid - j * 8);
        if (ri < wrows && n > 0) {
          const uint4 val = *reinterpret_cast<const uint4*>(buf + stage_off(ri, j));
          const int p = row0 + quad * 32 + ri;
          uint16_t* dst = a.row_out != nullptr ? a.row_out[a.row_out_idx[p]] : out + static_cast<int64_t>(p) * a.ldo;
          put8(dst + gcol0 + j * 8, val, n);
        }
      }
      committed = false;
    }
    __syncwarp();
  }
}

// Shared down projection fused with the combine (kEpiCombine):
//   update[t] = bf16(bf16(acc_t) + sum_j Y[rank[t*k + j]])
// in FP32, base first and then the slots in order -- the combine kernel's
// arithmetic, so the result is the same bit for bit.  The warp stages its
// accumulator slices (BF16, at most two of 64 columns) in its two 4 KB
// buffers and releases the accumulator.  It then walks its 32 tokens 4 at a
// time: each 8-lane group reads one token's k expert rows in whole 128-byte
// segments for both slices (2k loads in flight per lane) and stores the
// finished segments.  The expert rows are too few per SM to cover HBM
// latency with loads alone, so every token's rows are prefetched into L2
// (by the token's own thread, which holds its ranks) kPrefetchSteps steps
// before they are read.  Requires n_valid % 64 == 0 and bn % 64 == 0.
__device__ __forceinline__ void run_epilogue_combine(const GemmArgs& a, uint32_t taddr, uint8_t* stage, int quad,
                                                     int half, int lane, int rows, int n0, long long my_row,
                                                     uint64_t* release) {
  constexpr int kPrefetchSteps = 3;
  const int r = quad * 32 + lane;
  const int wrows = rows - quad * 32;
  const int k = a.comb_k;
  int rk[kCombineMaxK];
#pragma unroll
  for (int j = 0; j < kCombineMaxK; ++j)
    rk[j] = (j < k && r < rows) ? __ldg(a.comb_rank + my_row * k + j) : 0;
  const int cb = n0 + half * 64;  // first column of slice 0; slice 1 is 128 columns on
  const bool ok0 = cb < a.bn + n0 && cb < a.n_valid;
  const bool ok1 = cb + 128 < a.bn + n0 && cb + 128 < a.n_valid;
  // Rows of step s belong to lanes 4s .. 4s+3.
  auto prefetch_step = [&](int s) {
    if ((lane >> 2) == s && lane < wrows) {
#pragma unroll
      for (int j = 0; j < kCombineMaxK; ++j) {
        if (j < k) {
          const uint16_t* src = a.comb_y + static_cast<int64_t>(rk[j]) * a.ldy + cb;
          if (ok0) prefetch_l2(src);
          if (ok1) prefetch_l2(src + 128);
        }
      }
    }
  };
  if (wrows > 0) {
    for (int s = 0; s < kPrefetchSteps; ++s) prefetch_step(s);
  }
  // 1) accumulator -> BF16 staging
#pragma unroll
  for (int sl = 0; sl < 2; ++sl) {
    const int s0 = half * 64 + sl * 128;
    if (s0 < a.bn) {
      uint32_t v[64];
      tmem_ld32(taddr + s0, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
      tmem_ld32(taddr + s0 + 32, *reinterpret_cast<uint32_t(*)[32]>(&v[32]));
      tmem_wait_ld();
      uint32_t hw[32];
#pragma unroll
      for (int j = 0; j < 64; j += 2) hw[j / 2] = pack_bf16x2(__uint_as_float(v[j]), __uint_as_float(v[j + 1]));
      uint8_t* buf = stage + sl * kStageBytesPerWarp;
#pragma unroll
      for (int c = 0; c < 64; c += 16) stage_put16(buf, lane, c, &hw[c / 2]);
    }
  }
  tc_fence_before();
  __syncwarp();
  if (lane == 0) mbar_arrive(release);
  if (wrows <= 0) return;
  // 2) gather the expert rows, add, store
  const int g = lane >> 3, j8 = lane & 7;
  uint16_t* out = static_cast<uint16_t*>(a.out);
#pragma unroll 1
  for (int step = 0; step < 8; ++step) {
    if (step + kPrefetchSteps < 8) prefetch_step(step + kPrefetchSteps);
    const int ri = step * 4 + g;
    int pr[kCombineMaxK];
#pragma unroll
    for (int j = 0; j < kCombineMaxK; ++j) pr[j] = __shfl_sync(0xFFFFFFFFu, rk[j], ri);
    const long long t = __shfl_sync(0xFFFFFFFFu, my_row, ri);
    if (ri < wrows) {
      uint4 y0[kCombineMaxK], y1[kCombineMaxK], r0, r1;
#pragma unroll
      for (int j = 0; j < kCombineMaxK; ++j) {
        if (j < k) {
          const uint16_t* src = a.comb_y + static_cast<int64_t>(pr[j]) * a.ldy + cb + j8 * 8;
          if (ok0) y0[j] = __ldg(reinterpret_cast<const uint4*>(src));
          if (ok1) y1[j] = __ldg(reinterpret_cast<const uint4*>(src + 128));
        }
      }
      if (a.comb_res != nullptr) {
        const uint16_t* res = a.comb_res + t * a.ldo + cb + j8 * 8;
        if (ok0) r0 = __ldg(reinterpret_cast<const uint4*>(res));
        if (ok1) r1 = __ldg(reinterpret_cast<const uint4*>(res + 128));
      }
#pragma unroll
      for (int sl = 0; sl < 2; ++sl) {
        if (sl == 0 ? ok0 : ok1) {
          float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
          add_row8<false>(acc, *reinterpret_cast<const uint4*>(stage + sl * kStageBytesPerWarp + stage_off(ri, j8)),
                          1.0f);
#pragma unroll
          for (int j = 0; j < kCombineMaxK; ++j)
            if (j < k) add_row8<false>(acc, sl == 0 ? y0[j] : y1[j], 1.0f);
          uint4 o;
          o.x = pack_bf16x2(acc[0], acc[1]);
          o.y = pack_bf16x2(acc[2], acc[3]);
          o.z = pack_bf16x2(acc[4], acc[5]);
          o.w = pack_bf16x2(acc[6], acc[7]);
          const int64_t at = t * a.ldo + cb + sl * 128 + j8 * 8;
          if (out != nullptr) *reinterpret_cast<uint4*>(out + at) = o;
          if (a.comb_res != nullptr) {
            // the block's residual add: bf16(h + update), update already BF16
            float hs[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            add_row8<false>(hs, sl == 0 ? r0 : r1, 1.0f);
            add_row8<false>(hs, o, 1.0f);
            uint4 ro;
            ro.x = pack_bf16x2(hs[0], hs[1]);
            ro.y = pack_bf16x2(hs[2], hs[3]);
            ro.z = pack_bf16x2(hs[4], hs[5]);
            ro.w = pack_bf16x2(hs[6], hs[7]);
            *reinterpret_cast<uint4*>(a.comb_res_out + at) = ro;
          }
        }
      }
    }
  }
}

// MXFP8-lane SwiGLU epilogue: each thread holds 32 hidden values of its row
// per slice (one scale block) and writes them as E4M3 bytes plus the block's
// scale byte.  The accumulator is released as soon as the thread's slices are
// in registers (at most two slices of gate and up: 128 values), so a single
// 256-column TMEM accumulator still lets the next tile's MMAs overlap this
// tile's arithmetic and stores.
__device__ __forceinline__ void run_epilogue_swiglu_mx(const GemmArgs& a, uint32_t taddr, int quad, int half,
                                                       int lane, int row0, int rows, int nt, uint64_t* release) {
  const int r = quad * 32 + lane;
  const bool live = r < rows;
  uint8_t* hq = static_cast<uint8_t*>(a.out);
  const int64_t row = static_cast<int64_t>(row0) + r;
  if (rows - quad * 32 <= 0) {  // nothing of this quadrant is stored: release at once
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(release);
    return;
  }
  // gate and up rounded to BF16 right away (the reference's tensor boundary),
  // two values per register: 64 registers hold both slices.
  uint32_t gp[2][16], up[2][16];
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int s0 = half * 32 + 64 * j;
    if (s0 < a.chunk) {
      uint32_t g[32], u[32];
      tmem_ld32(taddr + s0, g);
      tmem_ld32(taddr + a.chunk + s0, u);
      tmem_wait_ld();
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        gp[j][c] = pack_bf16x2(__uint_as_float(g[2 * c]), __uint_as_float(g[2 * c + 1]));
        up[j][c] = pack_bf16x2(__uint_as_float(u[2 * c]), __uint_as_float(u[2 * c + 1]));
      }
    }
  }
  tc_fence_before();
  __syncwarp();
  if (lane == 0) mbar_arrive(release);
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int s0 = half * 32 + 64 * j;
    if (s0 >= a.chunk) break;
    float h[32];
#pragma unroll
    for (int c = 0; c < 16; ++c) {
      const uint32_t hp = bmul2(pack_bf16x2(silu_fast(lo_f(gp[j][c])), silu_fast(hi_f(gp[j][c]))), up[j][c]);
      h[2 * c] = lo_f(hp);
      h[2 * c + 1] = hi_f(hp);
    }
    uint32_t q[8];
    const uint32_t sb = mx_quantize32(h, q);
    if (live) {
      const int col = nt * a.chunk + s0;
      uint4* dst = reinterpret_cast<uint4*>(hq + row * a.ldo + col);
      dst[0] = make_uint4(q[0], q[1], q[2], q[3]);
      dst[1] = make_uint4(q[4], q[5], q[6], q[7]);
      a.out_sf[row * a.ld_out_sf + col / kMxBlock] = static_cast<uint8_t>(sb);
    }
  }
  // Zero the K padding of the quantised hidden row (values and scales).
  if (half == 0 && live && nt == a.n_tiles - 1) {
    const int c0 = a.n_tiles * a.chunk;
    for (int col = c0; col < a.h_cols; col += 16)
      *reinterpret_cast<uint4*>(hq + row * a.ldo + col) = make_uint4(0u, 0u, 0u, 0u);
    for (int b = c0 / kMxBlock; b < a.h_cols / kMxBlock; ++b) a.out_sf[row * a.ld_out_sf + b] = 0;
  }
}

// BF16 expert / shared GEMM1 epilogue (kEpiSwiglu, BF16 lane):
//   hidden = bf16(bf16(silu(bf16(gate))) * bf16(up))
// The warp reads both of its 32-column slices of gate and up from TMEM,
// rounding them to BF16 at once (the reference's tensor boundary, two values
// per register), and releases the accumulator before any arithmetic, so the
// next tile's MMAs need not wait for the SwiGLU.  Each slice of hidden rows
// (in tile order) then goes through the warp's 4 KB staging buffer: threads
// write their own row, and each store instruction moves 8 rows x 64 B.
// With gu_out (training) the BF16-rounded gate and up values of the slice
// go out the same way first, for the backward.  Needs chunk % 8 == 0 and
// ldo % 8 == 0, ld_gu % 8 == 0 (16-byte aligned row segments).
__device__ __forceinline__ void run_epilogue_swiglu_bf16(const GemmArgs& a, uint32_t taddr, uint8_t* stage,
                                                         int quad, int half, int lane, int row0, int rows, int nt,
                                                         uint64_t* release) {
  const int r = quad * 32 + lane;
  const bool live = r < rows;
  uint16_t* out = static_cast<uint16_t*>(a.out);
  const int64_t row = static_cast<int64_t>(row0) + r;
  if (rows - quad * 32 <= 0) {  // nothing of this quadrant is stored: release at once
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(release);
    return;
  }
  uint32_t gp[2][16], up[2][16];
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int s0 = half * 32 + 64 * j;
    if (s0 < a.chunk) {
      uint32_t g[32], u[32];
      tmem_ld32(taddr + s0, g);
      tmem_ld32(taddr + a.chunk + s0, u);
      tmem_wait_ld();
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        gp[j][c] = pack_bf16x2(__uint_as_float(g[2 * c]), __uint_as_float(g[2 * c + 1]));
        up[j][c] = pack_bf16x2(__uint_as_float(u[2 * c]), __uint_as_float(u[2 * c + 1]));
      }
    }
  }
  tc_fence_before();
  __syncwarp();
  if (lane == 0) mbar_arrive(release);
  const int wrows = rows - quad * 32;
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int s0 = half * 32 + 64 * j;
    if (s0 >= a.chunk) break;
    const int nchunk = min(32, a.chunk - s0) >> 3;  // 16-byte chunks per row (the width is a multiple of 8)
    if (a.gu_out != nullptr) {
      // the pre-activations (training): gate at columns [0, 32) and up at
      // [32, 64) of the staged rows, each stored to its own columns
      __syncwarp();
      stage_put16(stage, lane, 0, &gp[j][0]);
      stage_put16(stage, lane, 16, &gp[j][8]);
      stage_put16(stage, lane, 32, &up[j][0]);
      stage_put16(stage, lane, 48, &up[j][8]);
      __syncwarp();
      const int q = lane & 7;
      const int part = q >> 2, qc = q & 3;
      uint16_t* col = a.gu_out + nt * 2 * a.chunk + part * a.chunk + s0 + qc * 8;
#pragma unroll
      for (int step = 0; step < 8; ++step) {
        const int ri = step * 4 + (lane >> 3);
        if (ri < wrows && qc < nchunk)
          *reinterpret_cast<uint4*>(col + static_cast<int64_t>(row0 + quad * 32 + ri) * a.ld_gu) =
              *reinterpret_cast<const uint4*>(stage + stage_off(ri, q));
      }
    }
    uint32_t hw[16];
#pragma unroll
    for (int c = 0; c < 16; ++c)
      hw[c] = bmul2(pack_bf16x2(silu_fast(lo_f(gp[j][c])), silu_fast(hi_f(gp[j][c]))), up[j][c]);
    __syncwarp();  // the previous reads of the buffer are done
    stage_put16(stage, lane, 0, &hw[0]);
    stage_put16(stage, lane, 16, &hw[8]);
    __syncwarp();
    const int q = lane & 3;
    uint16_t* col = out + nt * a.chunk + s0 + q * 8;
#pragma unroll
    for (int step = 0; step < 4; ++step) {
      const int ri = step * 8 + (lane >> 2);
      if (ri < wrows && q < nchunk)
        *reinterpret_cast<uint4*>(col + static_cast<int64_t>(row0 + quad * 32 + ri) * a.ldo) =
            *reinterpret_cast<const uint4*>(stage + stage_off(ri, q));
    }
  }
  // Zero the K padding of the hidden matrix (columns [chunks*c, h_cols)).
  if (half == 0 && live && nt == a.n_tiles - 1) {
    uint16_t* dst = out + row * a.ldo;
    for (int col = a.n_tiles * a.chunk; col < a.h_cols; ++col) dst[col] = 0;
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

// Producer warp for the stages that need the load/store unit: A rows gathered
// through `gather_idx` (each cp.async instruction moves 4 rows x 128 B, fully
// coalesced) and, in the MXFP8 lane, the two scale atoms of every stage.  B
// (and an ungathered A) come by TMA.  full[s] expects 1 + 32 arrivals: lane
// 0's arrive.expect_tx for the TMA bytes, and one cp.async-tracked arrival per
// lane (cp.async.mbarrier.arrive.noinc), which fires when that lane's copies
// for the stage have landed.  The warp never waits for its own copies, so
// every stage of the ring can be in flight at once.
constexpr uint32_t kCpAsyncArrivals = 32;

// PART 0: one producer warp gathers all 128 rows of a tile; PART 1..N: N
// producer warps split them into equal row ranges (PART 1 also issues the B
// TMA and the expect_tx), each lane's copies arriving on full[s] as before.
template <bool MX, bool NV = false, int PART = 0>
__device__ __forceinline__ void produce_cp_async(const GemmArgs& a, uint8_t* sa, uint8_t* sb, uint8_t* ssf,
                                                 uint64_t* full, uint64_t* empty, int S, uint32_t a_bytes,
                                                 uint32_t b_bytes, int total, int lane) {
  constexpr int kPer = PART == 0 ? 32 : 32 / kGemmGatherProducers;
  constexpr int kI0 = PART == 0 ? 0 : (PART - 1) * kPer;
  constexpr int kI1 = kI0 + kPer;
  constexpr bool kLead = PART <= 1;
  const int bn = a.bn;
  const int chunk = lane & 7;
  const bool gather = a.gather != 0;
  const uint32_t tx_bytes = b_bytes + (gather ? 0u : a_bytes);
  uint32_t it = 0;
  bool ok = true;
  for (int t = blockIdx.x; ok && t < total; t += gridDim.x) {
    int group, row0, rows, nt;
    if (!decode_tile(a, t, group, row0, rows, nt)) {
      if (lane == 0) record_error(a.status, SPX_DEV_BAD_TILE);
      break;
    }
    int src[32];  // source row of tile row 4*i + (lane >> 3)
    if (gather) {
#pragma unroll
      for (int i = kI0; i < kI1; ++i) {
        const int rr = 4 * i + (lane >> 3);
        src[i] = a.gather_idx[row0 + (rr < rows ? rr : 0)];
      }
    }
    int sfr[4];  // MX: source row of tile row lane + 32*j (scale words)
    if constexpr (MX) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int rr = lane + 32 * j;
        const int rc = rr < rows ? rr : 0;
        sfr[j] = gather ? a.gather_idx[row0 + rc] : row0 + rc;
      }
    }
    const int n0 = nt * bn;
    for (int kb = 0; kb < a.k_blocks; ++kb, ++it) {
      const int s = static_cast<int>(it % S);
      const uint32_t ph = (it / S) & 1u;
      int go = 1;
      if (lane == 0) {
        go = mbar_wait(&empty[s], ph ^ 1u, a.status, SPX_DEV_TIMEOUT_PRODUCER) ? 1 : 0;
        if (go && kLead) {
          mbar_arrive_expect_tx(&full[s], tx_bytes);
          tma_load_3d(sb + s * b_bytes, &a.tma_b, &full[s], kb * 64 * (MX ? 2 : 1), n0, group);
          if (!gather) tma_load_2d(sa + s * a_bytes, &a.tma_a, &full[s], kb * 64 * (MX ? 2 : 1), row0);
        }
      }
      go = __shfl_sync(0xFFFFFFFFu, go, 0);
      if (!go) {
        ok = false;
        break;
      }
      if (gather) {
        const uint32_t dst0 = smem_u32(sa + s * a_bytes);
        if (a.a_rows != nullptr) {
          // rows anywhere (a peer GPU's memory included), one pointer per source row
          const int off = kb * 128 + chunk * 16;
#pragma unroll
          for (int i = kI0; i < kI1; ++i) {
            const int rr = 4 * i + (lane >> 3);
            const uint32_t dst = dst0 + (rr >> 3) * 1024 + (rr & 7) * 128 + ((chunk ^ (rr & 7)) << 4);
            cp_async16(dst, a.a_rows[src[i]] + off);
          }
        } else {
          const uint8_t* col = a.a_base + kb * 128 + chunk * 16;
#pragma unroll
          for (int i = kI0; i < kI1; ++i) {
            const int rr = 4 * i + (lane >> 3);
            const uint32_t dst = dst0 + (rr >> 3) * 1024 + (rr & 7) * 128 + ((chunk ^ (rr & 7)) << 4);
            cp_async16(dst, col + static_cast<int64_t>(src[i]) * a.lda);
          }
        }
      }
      if constexpr (MX && NV && kLead) {
        // Four K-64 MMAs per stage: A atom q holds bytes 4q..4q+3 of each
        // row's 16 scale bytes of the stage; the B atoms of the stage are
        // contiguous ([q][128-row block]).
        const uint32_t sf = smem_u32(ssf + s * kNvStageSfBytes);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
#pragma unroll
          for (int j = 0; j < 4; ++j)
            cp_async4(sf + q * kMxAtomBytes + lane * 16 + j * 4, a.sfa + sfr[j] * a.ld_sfa + kb * 16 + q * 4);
        }
        const int sfb_atoms = 4 * ((bn + 127) / 128);
        const int64_t atom = ((static_cast<int64_t>(group) * a.n_tiles + nt) * a.k_blocks + kb) * sfb_atoms;
        for (int q = 0; q < sfb_atoms; ++q)
          cp_async16(sf + (4 + q) * kMxAtomBytes + lane * 16, a.sfb + (atom + q) * kMxAtomBytes + lane * 16);
      } else if constexpr (MX && !NV && kLead) {
        const uint32_t sf = smem_u32(ssf + s * kMxStageSfBytes);
#pragma unroll
        for (int j = 0; j < 4; ++j) cp_async4(sf + lane * 16 + j * 4, a.sfa + sfr[j] * a.ld_sfa + kb * 4);
        const int sfb_atoms = (bn + 127) / 128;
        const int64_t atom = ((static_cast<int64_t>(group) * a.n_tiles + nt) * a.k_blocks + kb) * sfb_atoms;
        for (int q = 0; q < sfb_atoms; ++q)
          cp_async16(sf + (1 + q) * kMxAtomBytes + lane * 16, a.sfb + (atom + q) * kMxAtomBytes + lane * 16);
      }
      cp_async_mbar_arrive_noinc(&full[s]);
    }
  }
  cp_async_wait_all();  // no copy outlives the producer (error paths included)
}

// Persistent GEMM: each CTA walks tiles blockIdx.x, blockIdx.x + gridDim.x, ...
// The TMA producer and the MMA issuer stream k-blocks through the stage ring
// without stopping at tile boundaries; the accumulator is multi-buffered in
// TMEM so the epilogue of one tile overlaps the MMAs of the next.
// Instantiations that can gather A rows (BF16 kEpiStore / kEpiSwiglu, the
// MXFP8 kEpiSwiglu; the NVFP4 GEMM1 reads A by TMA) carry the extra producer
// warps; the others keep 10 warps (and their registers).  Only the lead
// producer copies scale factors.
// 4 KB epilogue staging buffers per epilogue warp (the MXFP8 SwiGLU epilogue
// stores from registers).
constexpr int gemm_stage_bufs(int epi, bool mx, bool nv) {
  return (epi == kEpiScatter || epi == kEpiCombine) ? 2 : (mx && !nv && epi == kEpiSwiglu) ? 0 : 1;
}

template <int EPI, bool MX, bool NV>
constexpr int gemm_threads() {
  return ((!MX && (EPI == kEpiStore || EPI == kEpiSwiglu)) || (MX && !NV && EPI == kEpiSwiglu)) ? kGemmKernelThreads
                                                                                                  : kGemmThreads;
}

template <int EPI, bool MX, bool NV = false>
__global__ void __launch_bounds__(gemm_threads<EPI, MX, NV>(), 1) gemm_kernel(const __grid_constant__ GemmArgs a) {
  constexpr uint32_t kSfStage = NV ? kNvStageSfBytes : kMxStageSfBytes;
  extern __shared__ uint8_t gemm_smem_raw[];
  uint8_t* smem = align_1024(gemm_smem_raw);
  const int bn = a.bn;
  const int S = a.stages;
  const uint32_t a_bytes = kTileRows * 128u;
  const uint32_t b_bytes = static_cast<uint32_t>(bn) * 128u;
  uint8_t* sa = smem;
  uint8_t* sb = smem + S * a_bytes;
  uint8_t* ssf = sb + S * b_bytes;                           // MX: [S][SFA atom | SFB atom]
  // Epilogue staging: one 4 KB buffer per epilogue warp, two for the TMA-store
  // epilogue, none for the MXFP8 SwiGLU epilogue.
  constexpr int kStageBufs = gemm_stage_bufs(EPI, MX, NV);
  // 1024-byte aligned: the TMA store reads the buffers with the 128B swizzle.
  uint8_t* stage_all = align_1024(ssf + (MX ? S * kSfStage : 0u));
  uint64_t* full = reinterpret_cast<uint64_t*>(stage_all + kGemmEpilogueWarps * kStageBufs * kStageBytesPerWarp);
  uint64_t* empty = full + S;
  uint64_t* tfull = empty + S;                 // [kMaxAccBufs] accumulator ready
  uint64_t* tempty = tfull + kMaxAccBufs;      // [kMaxAccBufs] accumulator drained
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + kMaxAccBufs);
  // As many accumulators as fit in the 512 TMEM columns (2 for 256-column
  // tiles); the MXFP8 lane keeps columns 384.. for scale factors.
  const uint32_t acc_limit = MX ? kMxSfColumn : 512u;
  const uint32_t nacc = min(static_cast<uint32_t>(kMaxAccBufs), acc_limit / a.tmem_cols);
  const uint32_t tmem_alloc_cols = MX ? 512u : nacc * a.tmem_cols;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int m_tiles = a.tiles != nullptr ? *a.num_tiles : (a.m_rows + kTileRows - 1) / kTileRows;
  const int total = m_tiles * a.n_tiles;
  if (static_cast<int>(blockIdx.x) >= total) return;
  const bool ldst_producer = MX || a.gather != 0;
  const bool gather_producers = gemm_threads<EPI, MX, NV>() == kGemmKernelThreads && a.gather != 0;
  const bool copier = !MX && gather_producers && a.copy_out != nullptr;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], ldst_producer ? 1 + kCpAsyncArrivals * (gather_producers ? kGemmGatherProducers : 1) : 1);
      mbar_init(&empty[s], copier ? 2 : 1);  // MMA commit (+ copier)
    }
    for (int b = 0; b < kMaxAccBufs; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], kGemmEpilogueWarps);
    }
    fence_mbar_init();
    if (!a.gather) prefetch_tensormap(&a.tma_a);  // gathered A has no tensor map
    prefetch_tensormap(&a.tma_b);
    if constexpr (EPI == kEpiScatter) {
      if (a.tma_store) prefetch_tensormap(&a.tma_out);
    }
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, tmem_alloc_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == kGemmCopierWarp) {
    // ---------------- copier: every gathered A stage (128 rows x 64 columns)
    // to copy_out in tile-row order -- whole 32-row groups by TMA stores
    // straight from the staged (swizzled) rows, the rows of a last partial
    // group by plain copies -- then it releases the stage together with the
    // MMA once the stores have read it.  Only N tile 0 copies.
    if (copier) {
      uint32_t it = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < total; t += gridDim.x) {
        int group, row0, rows, nt;
        if (!decode_tile(a, t, group, row0, rows, nt)) break;
        const int groups32 = rows >> 5;  // whole 32-row groups
        for (int kb = 0; kb < a.k_blocks; ++kb, ++it) {
          const int s = static_cast<int>(it % S);
          const uint32_t ph = (it / S) & 1u;
          int go = 1;
          if (lane == 0) go = mbar_wait(&full[s], ph, a.status, SPX_DEV_TIMEOUT_PRODUCER) ? 1 : 0;
          go = __shfl_sync(0xFFFFFFFFu, go, 0);
          if (!go) {
            ok = false;
            break;
          }
          if (nt == 0) {
            const uint8_t* st = sa + s * a_bytes;
            if (lane == 0 && groups32 > 0) {
              fence_proxy_async_smem();  // the staged rows (cp.async) -> the bulk stores' reads
              for (int q = 0; q < groups32; ++q) tma_store_2d(&a.tma_copy, st + q * 4096, kb * 64, row0 + 32 * q);
              bulk_commit();
            }
            const int r = 32 * groups32 + lane;
            if (r < rows) {
#pragma unroll
              for (int c = 0; c < 8; ++c)
                *reinterpret_cast<uint4*>(a.copy_out + static_cast<int64_t>(row0 + r) * a.ld_copy + kb * 64 + c * 8) =
                    *reinterpret_cast<const uint4*>(st + r * 128 + ((c ^ (r & 7)) << 4));
            }
            if (lane == 0 && groups32 > 0) bulk_wait_read<0>();  // the stores are done reading the stage
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&empty[s]);
        }
      }
      if (lane == 0) bulk_wait_all();  // stores complete before the CTA goes away
      __syncwarp();
    }
  } else if (warp >= kGemmExtraProducerWarp0) {
    if (gather_producers) {
      const int part = 2 + warp - kGemmExtraProducerWarp0;
      if (part == 2) produce_cp_async<MX, NV, 2>(a, sa, sb, ssf, full, empty, S, a_bytes, b_bytes, total, lane);
      if constexpr (kGemmGatherProducers > 2) {
        if (part == 3) produce_cp_async<MX, NV, 3>(a, sa, sb, ssf, full, empty, S, a_bytes, b_bytes, total, lane);
        if (part == 4) produce_cp_async<MX, NV, 4>(a, sa, sb, ssf, full, empty, S, a_bytes, b_bytes, total, lane);
      }
    }
  } else if (warp == 0 && gather_producers) {
    produce_cp_async<MX, NV, 1>(a, sa, sb, ssf, full, empty, S, a_bytes, b_bytes, total, lane);
  } else if (warp == 0 && ldst_producer) {
    produce_cp_async<MX, NV>(a, sa, sb, ssf, full, empty, S, a_bytes, b_bytes, total, lane);
  } else if (warp == 0) {
    // ---------------- TMA producer
    uint32_t it = 0;
    bool ok = true;
    for (int t = blockIdx.x; ok && t < total; t += gridDim.x) {
      int group, row0, rows, nt;
      if (!decode_tile(a, t, group, row0, rows, nt)) {
        if (lane == 0) record_error(a.status, SPX_DEV_BAD_TILE);
        break;
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
        if (lane == 0) tma_load_2d(sa + s * a_bytes, &a.tma_a, &full[s], kb * 64, row0);
        if (lane == 0) {
          if (a.b_split > 0 && kb >= a.b_split)  // K blocks past the split come from the second operand
            tma_load_3d(sb + s * b_bytes, &a.tma_b2, &full[s], (kb - a.b_split) * 64, n0, group);
          else
            tma_load_3d(sb + s * b_bytes, &a.tma_b, &full[s], kb * 64, n0, group);
        }
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
        const uint32_t b = lt % nacc;
        const uint32_t tph = (lt / nacc) & 1u;
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
          if constexpr (MX && NV) {
            // Per K-64 MMA: its SFA atom and SFB atom(s) -> a rotating
            // 12-column TMEM slot, then the MMA (scale ids 0).
            const uint32_t sf_smem = smem_u32(ssf + s * kNvStageSfBytes);
            const uint32_t nb = bn > 128 ? 2u : 1u;
            const uint32_t idesc_nv = idesc_nvf4(kTileRows, bn);
#pragma unroll
            for (uint32_t q = 0; q < 4; ++q) {
              const uint32_t slot = (it * 4u + q) % kNvSfSlots;
              const uint32_t sfa_t = tmem + kMxSfColumn + slot * kNvSfSlotCols;
              const uint32_t sfb_t = sfa_t + 4u;
              tmem_cp_32x128b_x4(sfa_t, desc_sf_atom(sf_smem + q * kMxAtomBytes));
              tmem_cp_32x128b_x4(sfb_t, desc_sf_atom(sf_smem + (4u + q * nb) * kMxAtomBytes));
              if (nb > 1u) tmem_cp_32x128b_x4(sfb_t + 4u, desc_sf_atom(sf_smem + (5u + q * nb) * kMxAtomBytes));
              mma_nvf4_ss(acc, desc_kmajor_sw128(a_base + q * 32), desc_kmajor_sw128(b_base + q * 32), idesc_nv,
                          sfa_t, sfb_t, (kb != 0 || q != 0) ? 1u : 0u);
            }
          } else if constexpr (MX) {
            // Scales of this stage -> a rotating TMEM slot (tcgen05.cp and the
            // MMAs that read it are issued in order by this thread).
            const uint32_t sfa_t = tmem + kMxSfColumn + (it % kMxSfSlots) * kMxSfSlotCols;
            const uint32_t sfb_t = sfa_t + 4u;
            const uint32_t sf_smem = smem_u32(ssf + s * kMxStageSfBytes);
            tmem_cp_32x128b_x4(sfa_t, desc_sf_atom(sf_smem));
            tmem_cp_32x128b_x4(sfb_t, desc_sf_atom(sf_smem + kMxAtomBytes));
            if (bn > 128) tmem_cp_32x128b_x4(sfb_t + 4u, desc_sf_atom(sf_smem + 2 * kMxAtomBytes));
#pragma unroll
            for (uint32_t kk = 0; kk < 4; ++kk) {
              mma_mxf8_ss(acc, desc_kmajor_sw128(a_base + kk * 32), desc_kmajor_sw128(b_base + kk * 32),
                          idesc_mxf8(kTileRows, bn, kk, kk), sfa_t | (kk << 30), sfb_t | (kk << 30),
                          (kb != 0 || kk != 0) ? 1u : 0u);
            }
          } else {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              mma_bf16_ss(acc, desc_kmajor_sw128(a_base + kk * 32), desc_kmajor_sw128(b_base + kk * 32), idesc,
                          (kb | kk) != 0 ? 1u : 0u);
            }
          }
          mma_commit(&empty[s]);
        }
        mma_commit(&tfull[b]);
      }
    }
    __syncwarp();
  } else {
    // ---------------- epilogue (warps 2..9): warp w drains TMEM lanes 32*(w%4) .. +31,
    // column slices (w-2)/4, +2, ...
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;
    uint8_t* my_stage = stage_all + (warp - 2) * kStageBufs * kStageBytesPerWarp;
    uint32_t slices = 0;
    bool committed = false;
    uint32_t lt = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x, ++lt) {
      int group, row0, rows, nt;
      if (!decode_tile(a, t, group, row0, rows, nt)) break;
      const uint32_t b = lt % nacc;
      const uint32_t tph = (lt / nacc) & 1u;
      const int r = quad * 32 + lane;
      long long my_row = static_cast<long long>(row0) + r;
      float my_w = 0.0f;
      if constexpr (EPI == kEpiScatter) {
        my_w = 1.0f;  // no weights: unweighted rows (the caller applies the routing weights)
        if (r < rows && a.pos_weight != nullptr) my_w = bf16_to_f32(a.pos_weight[row0 + r]);
      }
      int go = 1;
      if (lane == 0) go = mbar_wait(&tfull[b], tph, a.status, SPX_DEV_TIMEOUT_EPILOGUE) ? 1 : 0;
      go = __shfl_sync(0xFFFFFFFFu, go, 0);
      if (!go) break;
      tc_fence_after();
      const uint32_t taddr = tmem + b * a.tmem_cols + (static_cast<uint32_t>(quad * 32) << 16);
      if constexpr (MX && !NV && EPI == kEpiSwiglu) {
        run_epilogue_swiglu_mx(a, taddr, quad, half, lane, row0, rows, nt, &tempty[b]);  // releases early
      } else if constexpr (NV) {
        // NVFP4: scale by the per-tensor scales of A (this tile's group) and
        // of B (gate / up / down of the group) before the BF16 epilogue.
        const int expert = a.tiles != nullptr ? a.tiles[t / a.n_tiles].w : 0;
        const float pa = nv_tensor_scale(a.nv_amax_a[expert]);
        const float* bamax = a.nv_amax_b + static_cast<int64_t>(group) * a.nv_b_stride + a.nv_b_off;
        const float al0 = pa * nv_tensor_scale(bamax[0]);
        if constexpr (EPI == kEpiScatter) {
          run_epilogue_rows(a, taddr, my_stage, quad, half, lane, row0, rows, nt * bn, my_w, slices, committed, al0);
        } else if constexpr (EPI == kEpiSwiglu) {
          const float al1 = pa * nv_tensor_scale(bamax[1]);
          run_epilogue<EPI, true>(a, taddr, my_stage, quad, half, lane, row0, rows, nt * bn, nt, my_row, al0, al1,
                                  a.nv_amax_out != nullptr ? a.nv_amax_out + expert : nullptr);
        } else {
          run_epilogue<EPI, true>(a, taddr, my_stage, quad, half, lane, row0, rows, nt * bn, nt, my_row, al0);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[b]);
      } else if constexpr (EPI == kEpiCombine) {
        run_epilogue_combine(a, taddr, my_stage, quad, half, lane, rows, nt * bn, my_row, &tempty[b]);  // releases early
      } else if constexpr (EPI == kEpiSwiglu) {
        run_epilogue_swiglu_bf16(a, taddr, my_stage, quad, half, lane, row0, rows, nt, &tempty[b]);  // releases early
      } else {
        if constexpr (EPI == kEpiScatter)
          run_epilogue_rows(a, taddr, my_stage, quad, half, lane, row0, rows, nt * bn, my_w, slices, committed);
        else
          run_epilogue<EPI>(a, taddr, my_stage, quad, half, lane, row0, rows, nt * bn, nt, my_row);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[b]);
      }
    }
    if constexpr (EPI == kEpiScatter) {
      if (lane == 0) bulk_wait_all();  // stores complete before the CTA (and its smem) goes away
      __syncwarp();
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, tmem_alloc_cols);
  }
}

// CTA-pair GEMM (cluster of two CTAs, tcgen05 cta_group::2): one 256-row
// tile of A (TMA, uniform tiling) x bn columns per pair.  Each CTA loads its
// 128 rows of A and half of the B rows into its own shared memory; the TMA
// loads of both CTAs complete on the leader's full barrier, for which the
// leader alone expects the bytes of both.  The leader's lane 0 issues the
// M = 256 MMAs and commits stage releases and accumulator-ready signals to
// both CTAs at once; each CTA's epilogue drains its own 128 accumulator rows
// exactly as the single-CTA kernel does.  The peer's epilogue warps arrive on
// a local barrier and one peer thread forwards each completed release to the
// leader (a cluster-scope release from the epilogue warps themselves would
// wait for their global stores).  Per SM this halves the B bytes of every
// tile.  Every wait is bounded; both CTAs always reach the final cluster
// barrier, so a pipeline that gives up still tears down in step.
template <int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kGemmThreads, 1)
    gemm_pair_kernel(const __grid_constant__ GemmArgs a) {
  extern __shared__ uint8_t gemm_smem_raw[];
  uint8_t* smem = align_1024(gemm_smem_raw);
  const int bn = a.bn;  // the pair's N; each CTA holds bn / 2 rows of B
  const int S = a.stages;
  const uint32_t a_bytes = kTileRows * 128u;
  const uint32_t b_bytes = static_cast<uint32_t>(bn / 2) * 128u;
  uint8_t* sa = smem;
  uint8_t* sb = smem + S * a_bytes;
  uint8_t* stage_all = align_1024(sb + S * b_bytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(stage_all + kGemmEpilogueWarps * kStageBytesPerWarp);
  uint64_t* empty = full + S;
  uint64_t* tfull = empty + S;
  uint64_t* tempty = tfull + kMaxAccBufs;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + kMaxAccBufs);
  const uint32_t nacc = min(static_cast<uint32_t>(kMaxAccBufs), 512u / a.tmem_cols);
  const uint32_t tmem_alloc_cols = nacc * a.tmem_cols;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int pair = static_cast<int>(blockIdx.x >> 1);
  const int npairs = static_cast<int>(gridDim.x >> 1);
  const int m_tiles = (a.m_rows + 2 * kTileRows - 1) / (2 * kTileRows);
  const int total = m_tiles * a.n_tiles;
  if (pair >= total) return;  // both CTAs of a pair share `pair`: they leave together

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);   // the leader's expect_tx arrival (+ both CTAs' bytes)
      mbar_init(&empty[s], 1);  // one multicast commit
    }
    for (int b = 0; b < kMaxAccBufs; ++b) {
      mbar_init(&tfull[b], 1);  // one multicast commit
      // Local epilogue warps; on the leader also the peer's forwarded release.
      mbar_init(&tempty[b], kGemmEpilogueWarps + (rank == 0 ? 1 : 0));
    }
    fence_mbar_init();
    prefetch_tensormap(&a.tma_a);
    prefetch_tensormap(&a.tma_b);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, tmem_alloc_cols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised, TMEM allocated
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer (both CTAs)
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (int t = pair; ok && t < total; t += npairs) {
        const int mt = t / a.n_tiles;
        const int nt = t - mt * a.n_tiles;
        const int row0 = mt * 2 * kTileRows + static_cast<int>(rank) * kTileRows;
        const int n0 = nt * bn + static_cast<int>(rank) * (bn / 2);
        for (int kb = 0; kb < a.k_blocks; ++kb, ++it) {
          const int s = static_cast<int>(it % S);
          const uint32_t ph = (it / S) & 1u;
          if (!mbar_wait(&empty[s], ph ^ 1u, a.status, SPX_DEV_TIMEOUT_PRODUCER)) {
            ok = false;
            break;
          }
          const uint32_t full_leader = mapa_shared(smem_u32(&full[s]), 0);
          if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * (a_bytes + b_bytes));
          tma_load_2d_pair(sa + s * a_bytes, &a.tma_a, full_leader, kb * 64, row0);
          tma_load_3d_pair(sb + s * b_bytes, &a.tma_b, full_leader, kb * 64, n0, 0);
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (rank != 0 && lane == 0) {
      // ---------------- peer: forward the epilogue's releases to the leader
      uint32_t lt = 0;
      for (int t = pair; t < total; t += npairs, ++lt) {
        const uint32_t b = lt % nacc;
        if (!mbar_wait(&tempty[b], (lt / nacc) & 1u, a.status, SPX_DEV_TIMEOUT_MMA)) break;
        tc_fence_after();
        mbar_arrive_cluster(mapa_shared(smem_u32(&tempty[b]), 0));
      }
    } else if (rank == 0 && lane == 0) {
      // ---------------- leader: MMA issuer
      const uint32_t idesc = idesc_bf16_f32(2 * kTileRows, bn);
      uint32_t it = 0, lt = 0;
      bool ok = true;
      for (int t = pair; ok && t < total; t += npairs, ++lt) {
        const uint32_t b = lt % nacc;
        const uint32_t tph = (lt / nacc) & 1u;
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
          for (int kk = 0; kk < 4; ++kk)
            mma_bf16_pair(acc, desc_kmajor_sw128(a_base + kk * 32), desc_kmajor_sw128(b_base + kk * 32), idesc,
                          (kb | kk) != 0 ? 1u : 0u);
          mma_commit_pair(&empty[s], 0x3);
        }
        if (!ok) break;
        mma_commit_pair(&tfull[b], 0x3);
      }
    }
    __syncwarp();
  } else {
    // ---------------- epilogue (both CTAs): this CTA's 128 accumulator rows
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;
    uint8_t* my_stage = stage_all + (warp - 2) * kStageBytesPerWarp;
    uint32_t lt = 0;
    for (int t = pair; t < total; t += npairs, ++lt) {
      const int mt = t / a.n_tiles;
      const int nt = t - mt * a.n_tiles;
      const int row0 = mt * 2 * kTileRows + static_cast<int>(rank) * kTileRows;
      const int rows = max(0, min(kTileRows, a.m_rows - row0));
      const uint32_t b = lt % nacc;
      const uint32_t tph = (lt / nacc) & 1u;
      int go = 1;
      if (lane == 0) go = mbar_wait(&tfull[b], tph, a.status, SPX_DEV_TIMEOUT_EPILOGUE) ? 1 : 0;
      go = __shfl_sync(0xFFFFFFFFu, go, 0);
      if (!go) break;
      tc_fence_after();
      const uint32_t taddr = tmem + b * a.tmem_cols + (static_cast<uint32_t>(quad * 32) << 16);
      if constexpr (EPI == kEpiSwiglu) {
        run_epilogue_swiglu_bf16(a, taddr, my_stage, quad, half, lane, row0, rows, nt, &tempty[b]);  // releases early
      } else {
        const long long my_row = static_cast<long long>(row0) + quad * 32 + lane;
        run_epilogue<EPI>(a, taddr, my_stage, quad, half, lane, row0, rows, nt * bn, nt, my_row);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[b]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // no CTA leaves while its pair may still touch its shared or tensor memory
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, tmem_alloc_cols);
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

// 2-D tensor [rows, cols] (row pitch `ld` elements), box {128 bytes, box_rows}, 128B swizzle.
int encode_2d(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int64_t ld, int box_rows,
              int elem_bytes) {
  if (int rc = get_encoder(); rc != SPX_OK) return rc;
  if (elem_bytes != 1 && elem_bytes != 2) return SPX_ERR_INVALID_ARG;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0 || (ld * elem_bytes) % 16 != 0) return SPX_ERR_ALIGNMENT;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * elem_bytes)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(128 / elem_bytes), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1u, 1u};
  const CUtensorMapDataType dt = elem_bytes == 2 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8;
  CUresult r = g_encode(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? SPX_OK : SPX_ERR_DRIVER;
}

// 3-D tensor [groups, rows, cols], box {128 bytes, box_rows, 1}, 128B swizzle.
int encode_3d(CUtensorMap* map, const void* base, int64_t groups, int64_t rows, int64_t cols, int box_rows,
              int elem_bytes) {
  if (int rc = get_encoder(); rc != SPX_OK) return rc;
  if (elem_bytes != 1 && elem_bytes != 2) return SPX_ERR_INVALID_ARG;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0 || (cols * elem_bytes) % 16 != 0) return SPX_ERR_ALIGNMENT;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows),
                        static_cast<cuuint64_t>(groups)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(cols * elem_bytes),
                           static_cast<cuuint64_t>(rows * cols * elem_bytes)};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(128 / elem_bytes), static_cast<cuuint32_t>(box_rows), 1u};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  const CUtensorMapDataType dt = elem_bytes == 2 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8;
  CUresult r = g_encode(map, dt, 3, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? SPX_OK : SPX_ERR_DRIVER;
}

size_t gemm_smem_bytes(int bn, int stages, bool mx, int epi, bool nv) {
  const size_t per_stage =
      kTileRows * 128 + static_cast<size_t>(bn) * 128 + (mx ? (nv ? kNvStageSfBytes : kMxStageSfBytes) : 0);
  const size_t staging = static_cast<size_t>(kGemmEpilogueWarps) * kStageBytesPerWarp * gemm_stage_bufs(epi, mx, nv);
  return 2048 + static_cast<size_t>(stages) * per_stage + staging + (2 * stages + 2 * kMaxAccBufs) * 8 + 16;
}

size_t gemm_pair_smem_bytes(int bn, int stages) {
  const size_t per_stage = kTileRows * 128 + static_cast<size_t>(bn / 2) * 128;
  const size_t staging = static_cast<size_t>(kGemmEpilogueWarps) * kStageBytesPerWarp;
  return 2048 + static_cast<size_t>(stages) * per_stage + staging + (2 * stages + 2 * kMaxAccBufs) * 8 + 16;
}

int gemm_pair_pick_stages(int bn) {
  int stages = 2;
  for (int s = 3; s <= 8; ++s)
    if (gemm_pair_smem_bytes(bn, s) <= kGemmSmemBudget) stages = s;
  return stages;
}

// As many stages as fit: the persistent producer keeps prefetching the next
// tile's k-blocks, so stages beyond one tile's K still hide load latency.
int gemm_pick_stages(int bn, int k_blocks, bool mx, int epi, bool nv) {
  (void)k_blocks;
  int stages = 2;
  for (int s = 3; s <= 8; ++s)
    if (gemm_smem_bytes(bn, s, mx, epi, nv) <= kGemmSmemBudget) stages = s;
  return stages;
}

template <int EPI, bool MX, bool NV = false>
static int launch_gemm_t(const GemmArgs& a, int grid_m, int grid_n, cudaStream_t stream) {
  const size_t smem = gemm_smem_bytes(a.bn, a.stages, MX, EPI, NV);
  if (smem > kGemmSmemBudget) return SPX_ERR_INVALID_ARG;
  if (int rc = ensure_max_dynamic_smem(reinterpret_cast<const void*>(gemm_kernel<EPI, MX, NV>)); rc != SPX_OK)
    return rc;
  // Persistent grid: one CTA per SM, never more CTAs than (upper bound of) tiles.
  const int sms = a.max_ctas > 0 && a.max_ctas < device_sm_count() ? a.max_ctas : device_sm_count();
  const int64_t tiles = static_cast<int64_t>(grid_m) * grid_n;
  const int grid = static_cast<int>(tiles < sms ? tiles : sms);
  GemmArgs b = a;
  b.n_tiles = grid_n;
  gemm_kernel<EPI, MX, NV><<<grid, gemm_threads<EPI, MX, NV>(), smem, stream>>>(b);
  return cudaGetLastError() == cudaSuccess ? SPX_OK : SPX_ERR_CUDA;
}

template <int EPI>
static int launch_gemm_pair_t(const GemmArgs& a, int grid_m, int grid_n, cudaStream_t stream) {
  const size_t smem = gemm_pair_smem_bytes(a.bn, a.stages);
  if (smem > kGemmSmemBudget) return SPX_ERR_INVALID_ARG;
  const void* fn = reinterpret_cast<const void*>(gemm_pair_kernel<EPI>);
  if (int rc = ensure_max_dynamic_smem(fn); rc != SPX_OK) return rc;
  // Persistent grid of CTA pairs: no more pairs than tiles, nor than fit on
  // the device at once.
  const int pairs_max = device_max_pairs(fn, smem);
  const int64_t tiles = static_cast<int64_t>(grid_m) * grid_n;
  const int pairs = static_cast<int>(tiles < pairs_max ? tiles : pairs_max);
  GemmArgs b = a;
  b.n_tiles = grid_n;
  gemm_pair_kernel<EPI><<<2 * pairs, kGemmThreads, smem, stream>>>(b);
  return cudaGetLastError() == cudaSuccess ? SPX_OK : SPX_ERR_CUDA;
}

// CTA-pair GEMM over 256-row tiles of a TMA-loaded A (grid_m counts 256-row
// tiles).  bn: 32..256, a multiple of 32 (each CTA holds bn / 2 rows of B).
int launch_gemm_pair(int epi, const GemmArgs& a, int grid_m, int grid_n, cudaStream_t stream) {
  if (grid_m <= 0 || grid_n <= 0) return SPX_OK;
  if (a.bn < 32 || a.bn > 256 || (a.bn % 32) != 0 || a.gather != 0 || a.tiles != nullptr)
    return SPX_ERR_UNSUPPORTED;
  switch (epi) {
    case kEpiStore:
      return launch_gemm_pair_t<kEpiStore>(a, grid_m, grid_n, stream);
    case kEpiSwiglu:
      return launch_gemm_pair_t<kEpiSwiglu>(a, grid_m, grid_n, stream);
    default:
      return SPX_ERR_UNSUPPORTED;
  }
}

int launch_gemm(int epi, const GemmArgs& a, int grid_m, int grid_n, cudaStream_t stream, bool mx, bool nv) {
  if (grid_m <= 0 || grid_n <= 0) return SPX_OK;
  if (a.bn < 16 || a.bn > 256 || (a.bn % 16) != 0) return SPX_ERR_UNSUPPORTED;
  if (nv) {
    // NVFP4: E2M1 operands (128 B = 256 elements per stage), UE4M3 scales per 16.
    if (a.bn > kMxMaxBn || a.tmem_cols > kMxMaxBn || a.sfa == nullptr || a.sfb == nullptr ||
        (a.ld_sfa % 16) != 0 || a.nv_amax_a == nullptr || a.nv_amax_b == nullptr || a.gather != 0)
      return SPX_ERR_INVALID_ARG;
    switch (epi) {
      case kEpiStore:
        return launch_gemm_t<kEpiStore, true, true>(a, grid_m, grid_n, stream);
      case kEpiSwiglu:
        return launch_gemm_t<kEpiSwiglu, true, true>(a, grid_m, grid_n, stream);
      case kEpiScatter:
        return launch_gemm_t<kEpiScatter, true, true>(a, grid_m, grid_n, stream);
      default:
        return SPX_ERR_INVALID_ARG;
    }
  }
  if (mx) {
    // Block-scaled lane: one scale atom per 128 B rows of N, accumulators of 128 columns at most.
    if (a.bn > kMxMaxBn || a.tmem_cols > kMxMaxBn || a.sfa == nullptr || a.sfb == nullptr || (a.ld_sfa % 4) != 0)
      return SPX_ERR_INVALID_ARG;
    if (epi == kEpiSwiglu &&
        (a.out_sf == nullptr || (a.chunk % kMxBlock) != 0 || a.chunk > 128 || (a.ldo % 16) != 0))
      return SPX_ERR_INVALID_ARG;
    switch (epi) {
      case kEpiStore:
        return launch_gemm_t<kEpiStore, true>(a, grid_m, grid_n, stream);
      case kEpiSwiglu:
        return launch_gemm_t<kEpiSwiglu, true>(a, grid_m, grid_n, stream);
      case kEpiScatter:
        return launch_gemm_t<kEpiScatter, true>(a, grid_m, grid_n, stream);
      default:
        return SPX_ERR_INVALID_ARG;
    }
  }
  switch (epi) {
    case kEpiStore:
      return launch_gemm_t<kEpiStore, false>(a, grid_m, grid_n, stream);
    case kEpiSwiglu:
      return launch_gemm_t<kEpiSwiglu, false>(a, grid_m, grid_n, stream);
    case kEpiScatter:
      return launch_gemm_t<kEpiScatter, false>(a, grid_m, grid_n, stream);
    case kEpiCombine:
      if (a.comb_y == nullptr || a.comb_rank == nullptr || a.comb_k < 1 || a.comb_k > kCombineMaxK ||
          (a.n_valid % 64) != 0 || (a.bn % 64) != 0 || (a.ldy % 8) != 0 || (a.ldo % 8) != 0 ||
          (reinterpret_cast<uintptr_t>(a.comb_y) & 15u) != 0 || (reinterpret_cast<uintptr_t>(a.out) & 15u) != 0 ||
          (a.out == nullptr && a.comb_res == nullptr) ||
          (a.comb_res != nullptr && (a.comb_res_out == nullptr || (reinterpret_cast<uintptr_t>(a.comb_res) & 15u) != 0 ||
                                     (reinterpret_cast<uintptr_t>(a.comb_res_out) & 15u) != 0)))
        return SPX_ERR_INVALID_ARG;
      return launch_gemm_t<kEpiCombine, false>(a, grid_m, grid_n, stream);
    default:
      return SPX_ERR_INVALID_ARG;
  }
}

}  // namespace spx
