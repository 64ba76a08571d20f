// Decode-sized projections: grouped GEMVs on the CUDA cores.
//
// With a few tokens per step every routed expert sees a handful of rows, and
// the projections are bound by reading their weights once (589,824 bytes per
// expert in BF16 at the 100M shape).  A 128-row tcgen05 tile would hold those
// few rows and spend its time filling and draining; here each CTA instead
// pulls a slab of weight rows into shared memory with bulk asynchronous
// copies (one or two cp.async.bulk per CTA, all of a slab in flight at once)
// while its threads stage the token rows, then dots every token row with
// every weight row from shared memory.
//
// Same rounding points as the tensor-core path (experts/bank.py:755-763 and
// 970-978, nn/ffn.py:27-30, experts/router.py:51): FP32 accumulation;
// SwiGLU h = bf16(bf16(silu(bf16(g))) * bf16(u)); projections
// bf16(bf16(acc [+ bias]) * w).  MXFP8-lane experts (experts/native.py:91-140)
// dot the E4M3 values with their E8M0 block scales applied: the activations'
// blocks are dequantised exactly into BF16 (an E4M3 value times a power of two
// is representable), the weights' into FP32, the products are summed in FP32,
// and the SwiGLU GEMV writes the hidden rows quantised again (32-column
// blocks, the epilogue rule of the tensor-core path).
//
// Two kernels:
//   gemv_swiglu_kernel  a group's rows x [gate | up] slab of 16 hidden columns
//                       (32 for the MXFP8 lane, one scale block) -> hidden rows
//   gemv_rows_kernel    a group's rows x slab of N_blk output rows -> outputs
//                       (+ bias, x routing weight), rows staged and stored
//                       as whole row segments
// Expert passes run over the dispatch's tile tables (a tile = up to 128 rows
// of one expert's dispatch range, token rows gathered through src_row); the
// dense projections (router, shared SwiGLU) over the whole batch.  Each warp walks 4 weight rows at a time, one group of 8
// lanes per row (16 bytes per lane per step), accumulators in registers for
// up to 16 token rows per pass, reduced over the 8 lanes by shuffles.
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
constexpr int kGemvRows = 8;        // token rows per pass (one 8-column mma.sync tile)
constexpr int kSwigluCols = 16;     // hidden columns per swiglu CTA (BF16 lane)
constexpr int kSwigluColsMx = 32;   // ... MXFP8 lane (one scale block of the hidden row)
constexpr size_t kSlabBytes = 48 * 1024;  // weight slab budget per CTA

__device__ __forceinline__ float silu_ref(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

// 2^(byte - 127): the value of an E8M0 scale byte.
__device__ __forceinline__ float e8m0_value(uint32_t byte) {
  if (byte == 0u) return __uint_as_float(0x00400000u);  // 2^-127
  return __uint_as_float(byte << 23);
}

__device__ __forceinline__ void bf16x8(const uint4& v, float* f) {
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
// atoms [groups][tiles][K/128][ceil(tile_rows/128)][512] (mx_quantize_b_kernel).
__device__ __forceinline__ uint32_t w_scale(const uint8_t* atoms, int g, int row, int blk, int rows_per_group,
                                            int tile_rows, int kp) {
  const int tiles = (rows_per_group + tile_rows - 1) / tile_rows;
  const int per_tile = (tile_rows + 127) / 128;
  const int tile = row / tile_rows, r = row - tile * tile_rows;
  const int64_t atom = ((static_cast<int64_t>(g) * tiles + tile) * (kp / 128) + (blk >> 2)) * per_tile + (r >> 7);
  return __ldg(atoms + atom * kMxAtomBytes + mx_atom_offset(r & 127, blk & 3));
}

// Contiguous global -> shared bulk copy completing on `bar` (16-byte aligned, size % 16 == 0).
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// One thread waits (bounded) for phase `parity` of the CTA's barrier; the
// others wait at the CTA barrier that follows, so only one thread polls.  On
// a timeout the status word records it, the thread waits once more (bounded)
// for the copies still in flight, and every thread of the CTA returns.
__device__ __forceinline__ bool pass_ready(uint64_t* bar, uint32_t parity, int* status, int* abort_flag) {
  if (threadIdx.x == 0) {
    bool ok = mbar_wait(bar, parity, status, SPX_DEV_TIMEOUT_PRODUCER);
    if (!ok) mbar_wait(bar, parity, nullptr, 0);
    *abort_flag = ok ? 0 : 1;
  }
  __syncthreads();
  return *abort_flag == 0;
}

// Token rows into shared memory as BF16 [R][K] (row stride xstride values):
// 16-byte copies, or E4M3 rows dequantised with their block scales (exact).
// Row i of the pass is token row src[pos0 + i] (gather) or pos0 + i.
__device__ void stage_rows(bool mx, const int* src, int64_t pos0, int R, const uint16_t* rows_bf16, int64_t ld_bf16,
                           const uint8_t* rows_q, const uint8_t* rows_sf, int64_t ld_q, int K, int xstride,
                           uint16_t* xs) {
  if (!mx) {
    const int per_row = K / 8;
    for (int i = threadIdx.x; i < R * per_row; i += blockDim.x) {
      const int r = i / per_row, c = i - r * per_row;
      const int64_t row = src != nullptr ? src[pos0 + r] : pos0 + r;
      reinterpret_cast<uint4*>(xs + static_cast<int64_t>(r) * xstride)[c] =
          __ldg(reinterpret_cast<const uint4*>(rows_bf16 + row * ld_bf16) + c);
    }
    return;
  }
  const int per_row = K / 16;
  for (int i = threadIdx.x; i < R * per_row; i += blockDim.x) {
    const int r = i / per_row, c = i - r * per_row;
    const int64_t row = src != nullptr ? src[pos0 + r] : pos0 + r;
    const uint4 q = __ldg(reinterpret_cast<const uint4*>(rows_q + row * ld_q) + c);
    const float s = e8m0_value(__ldg(rows_sf + row * (ld_q / kMxBlock) + (c >> 1)));
    float f[16];
    e4m3x4(q.x, s, f);
    e4m3x4(q.y, s, f + 4);
    e4m3x4(q.z, s, f + 8);
    e4m3x4(q.w, s, f + 12);
    uint32_t h[8];
#pragma unroll
    for (int j = 0; j < 8; ++j)
      h[j] = static_cast<uint32_t>(f32_to_bf16_rne(f[2 * j])) |
             (static_cast<uint32_t>(f32_to_bf16_rne(f[2 * j + 1])) << 16);
    uint4* dst = reinterpret_cast<uint4*>(xs + static_cast<int64_t>(r) * xstride + c * 16);
    dst[0] = make_uint4(h[0], h[1], h[2], h[3]);
    dst[1] = make_uint4(h[4], h[5], h[6], h[7]);
  }
}

// acc[j] += <weight row, token row j> over k < k_valid for the lane's K slots,
// for NR token rows xs[0..NR) (all valid): lane `seg` of the row's 8-lane
// group takes 16 bytes per step.  `wrow` is the weight row in shared memory
// (BF16, or E4M3 with scales from global atoms).
template <bool MX, int NR>
__device__ __forceinline__ void dot_chunk(const uint8_t* wrow, const uint8_t* atoms, int g, int wr, int rows_per_group,
                                          int tile_rows, int Kw, int K, int k_valid, const uint16_t* xs, int seg,
                                          float (&acc)[NR]) {
  constexpr int kEl = MX ? 16 : 8;  // values per lane per step
  constexpr int kStep = 8 * kEl;
#pragma unroll 2
  for (int k = seg * kEl; k < k_valid; k += kStep) {
    float w[kEl];
    if constexpr (MX) {
      const uint4 q = *reinterpret_cast<const uint4*>(wrow + k);
      const float s = e8m0_value(w_scale(atoms, g, wr, k / kMxBlock, rows_per_group, tile_rows, Kw));
      e4m3x4(q.x, s, w);
      e4m3x4(q.y, s, w + 4);
      e4m3x4(q.z, s, w + 8);
      e4m3x4(q.w, s, w + 12);
    } else {
      bf16x8(*reinterpret_cast<const uint4*>(wrow + 2 * k), w);
    }
#pragma unroll
    for (int i = 0; i < NR; ++i) {
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

// All R token rows of a pass against one weight row, in chunks of 4, 2 and 1
// rows (no issue slots spent on absent rows); emit(i, partial) receives each
// row's lane partial sum (every lane of the warp calls it, in the same order).
template <bool MX, typename Emit>
__device__ __forceinline__ void dot_rows(const uint8_t* wrow, const uint8_t* atoms, int g, int wr, int rows_per_group,
                                         int tile_rows, int Kw, int K, int k_valid, const uint16_t* xs, int R,
                                         int seg, bool live, Emit emit) {
  int i0 = 0;
  for (; i0 + 4 <= R; i0 += 4) {
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    if (live)
      dot_chunk<MX, 4>(wrow, atoms, g, wr, rows_per_group, tile_rows, Kw, K, k_valid,
                       xs + static_cast<int64_t>(i0) * K, seg, acc);
#pragma unroll
    for (int j = 0; j < 4; ++j) emit(i0 + j, acc[j]);
  }
  if (i0 + 2 <= R) {
    float acc[2] = {0.0f, 0.0f};
    if (live)
      dot_chunk<MX, 2>(wrow, atoms, g, wr, rows_per_group, tile_rows, Kw, K, k_valid,
                       xs + static_cast<int64_t>(i0) * K, seg, acc);
    emit(i0, acc[0]);
    emit(i0 + 1, acc[1]);
    i0 += 2;
  }
  if (i0 < R) {
    float acc[1] = {0.0f};
    if (live)
      dot_chunk<MX, 1>(wrow, atoms, g, wr, rows_per_group, tile_rows, Kw, K, k_valid,
                       xs + static_cast<int64_t>(i0) * K, seg, acc);
    emit(i0, acc[0]);
  }
}

__device__ __forceinline__ float group_sum8(float v) {
  v += __shfl_xor_sync(0xFFFFFFFFu, v, 1);
  v += __shfl_xor_sync(0xFFFFFFFFu, v, 2);
  v += __shfl_xor_sync(0xFFFFFFFFu, v, 4);
  return v;
}

// The rows of this CTA's tile: weight group g, lane, rows [start, start + n)
// of the row space (n = 0: nothing to do).  Dense passes split their rows over
// gridDim.z CTAs (16-row chunks); a tile's rows (<= 128) loop in one CTA.
__device__ __forceinline__ void tile_rows(const GemvPass& a, int& g, bool& mx, int64_t& start, int& n) {
  g = 0;
  mx = false;
  start = 0;
  n = 0;
  if (a.tiles == nullptr) {
    n = a.dense_rows;
    return;
  }
  int t = blockIdx.x;
  int4 tile;
  if (t >= a.max_tiles) {
    t -= a.max_tiles;
    if (a.tiles_mx == nullptr || t >= *a.num_tiles_mx) return;
    tile = a.tiles_mx[t];
    mx = true;
  } else {
    if (t >= *a.num_tiles) return;
    tile = a.tiles[t];
  }
  g = tile.x;
  start = tile.y;
  n = tile.z;
}

// The row GEMV's BF16 tiles run on the tensor cores when the column block
// splits into 16-row m-tiles that divide the 8 warps and the K range splits
// evenly over the remaining warp factor in steps of 16.
__host__ __device__ __forceinline__ bool gemv_rows_tc(const GemvPass& a) {
  if (a.nblk % 16 != 0 || a.nblk > 16 * kGemvWarps) return false;
  const int mtiles = a.nblk / 16;
  if (kGemvWarps % mtiles != 0) return false;
  return a.k_valid2 % (16 * (kGemvWarps / mtiles)) == 0;
}

// ---- BF16 tiles on the tensor cores: mma.sync m16n8k16 (BF16 in, FP32
// accumulate) with the weight rows as the 16-row A operand and up to 8 token
// rows as the B operand, both read from shared memory by ldmatrix.  Rows in
// shared memory are padded by 16 bytes so that the 8 row addresses of an
// 8x8 ldmatrix fall in distinct banks.
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x2(uint32_t addr, uint32_t (&r)[2]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0, %1}, [%2];" : "=r"(r[0]), "=r"(r[1]) : "r"(addr));
}

__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// One warp: D[16 x 8 tokens] over k in [k0, k1).  a_row(m) gives the
// shared-memory byte offset of A row m (0..15) of the tile.
template <typename ARow>
__device__ __forceinline__ void mma_rows(uint32_t slab_u32, ARow a_row, uint32_t xs_u32, int xs_stride, int k0,
                                         int k1, int lane, float (&d)[4]) {
#pragma unroll
  for (int q = 0; q < 4; ++q) d[q] = 0.0f;
  // ldmatrix row addresses: A matrices 0..3 = (rows 0-7 | 8-15) x (k | k+8);
  // B matrices 0, 1 = tokens 0-7 x (k | k+8)
  const int mi = lane >> 3, ri = lane & 7;
  const uint32_t a_base = slab_u32 + a_row((mi & 1) * 8 + ri) + static_cast<uint32_t>((mi >> 1) * 16);
  const uint32_t b_base = xs_u32 + static_cast<uint32_t>(ri * xs_stride + (mi & 1) * 16);
#pragma unroll 4
  for (int k = k0; k < k1; k += 16) {
    uint32_t a[4];
    ldsm_x4(a_base + 2 * k, a);
    uint32_t b[2];
    ldsm_x2(b_base + 2 * k, b);
    mma_16816(d, a, b);
  }
}

// SwiGLU GEMV: gate/up of one block of hidden columns of group g for its rows.
__global__ void __launch_bounds__(kGemvThreads, 3) gemv_swiglu_kernel(const GemvPass a) {
  extern __shared__ __align__(128) uint8_t smem[];
  int g, n;
  bool mx;
  int64_t start;
  tile_rows(a, g, mx, start, n);
  if (n <= static_cast<int>(blockIdx.z) * kGemvRows) return;
  const int cols = mx ? kSwigluColsMx : kSwigluCols;
  const int j0 = blockIdx.y * kSwigluCols;
  if (mx && (j0 % kSwigluColsMx) != 0) return;  // MXFP8 CTAs take two column blocks
  if (j0 >= a.inter) return;
  const int c = mx ? a.cm : a.chunk;
  const int rows1 = (mx ? a.ncm : a.nc) * 2 * c;
  const int K = mx ? a.kx : a.kd;                    // token row width (BF16 values) in shared memory
  const int wbytes = mx ? a.kx : 2 * a.kd;           // weight row bytes
  const int ws = wbytes + 16;                        // padded row strides in shared memory
  const int xsb = 2 * K + 16;
  const int ncol = min(cols, a.inter - j0);
  // slab rows: gate rows [0, cols) then up rows [cols, 2 cols) of packed rows g0.. and g0 + c..
  const int ch = j0 / c;
  const int g0 = ch * 2 * c + (j0 - ch * c);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem);
  int* abort_flag = reinterpret_cast<int*>(smem + 64);
  uint8_t* slab = smem + 128;
  uint8_t* xsp = slab + 2 * static_cast<size_t>(cols) * ws;
  float* red = reinterpret_cast<float*>(xsp + static_cast<size_t>(kGemvRows) * xsb);  // [8 warps][32][4]
  uint16_t* hs = reinterpret_cast<uint16_t*>(red);  // MXFP8 lane: [kGemvRows][32] BF16 hidden values
  const uint8_t* wbase = mx ? a.w1q : reinterpret_cast<const uint8_t*>(a.w1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint32_t pass = 0;
  for (int r0 = blockIdx.z * kGemvRows; r0 < n; r0 += gridDim.z * kGemvRows, ++pass) {
    const int R = min(kGemvRows, n - r0);
    if (warp == 0) {
      const uint32_t bytes = (pass == 0 ? 2u * ncol * wbytes : 0u) + (mx ? 0u : static_cast<uint32_t>(R) * 2 * K);
      if (lane == 0) {
        if (pass == 0) {
          mbar_init(bar, 1);
          fence_mbar_init();
        } else {
          fence_proxy_async_smem();  // the previous pass's reads of the rows before the async writes below
        }
        if (bytes) mbar_arrive_expect_tx(bar, bytes); else mbar_arrive(bar);
      }
      __syncwarp();
      if (pass == 0) {
        for (int i = lane; i < 2 * ncol; i += 32) {
          const int half = i / ncol, jl = i - half * ncol;
          bulk_load(slab + static_cast<size_t>(half * cols + jl) * ws,
                    wbase + (static_cast<int64_t>(g) * rows1 + g0 + half * c + jl) * wbytes, wbytes, bar);
        }
      }
      if (!mx) {
        for (int i = lane; i < R; i += 32) {
          const int64_t row = a.src_row != nullptr ? a.src_row[start + r0 + i] : start + r0 + i;
          bulk_load(xsp + static_cast<size_t>(i) * xsb, a.x + row * a.ldx, 2u * K, bar);
        }
      }
    }
    if (mx) stage_rows(true, a.src_row, start + r0, R, a.x, a.ldx, a.xq, a.xsf, a.kx, a.kx, xsb / 2,
                       reinterpret_cast<uint16_t*>(xsp));
    // token rows R..15 of the tiles read by the tensor cores are zero
    for (int i = threadIdx.x; i < (kGemvRows - R) * (K / 8); i += blockDim.x) {
      const int r = R + i / (K / 8), q = i % (K / 8);
      reinterpret_cast<uint4*>(xsp + static_cast<size_t>(r) * xsb)[q] = make_uint4(0u, 0u, 0u, 0u);
    }
    if (!pass_ready(bar, pass & 1u, a.status, abort_flag)) return;
    if (!mx) {
      // warps: m-tile mt = warp & 1 (8 hidden columns: 8 gate rows + 8 up rows),
      // K quarter ks = warp >> 1; partial sums reduced in shared memory
      const int mt = warp & 1, ks = warp >> 1;
      const int kq = K / 4;
      float d[4];
      auto a_row = [&](int m) -> uint32_t {
        const int jl = mt * 8 + (m & 7);
        return static_cast<uint32_t>(((m >> 3) * cols + jl) * ws);  // m < 8: gate row jl, else up row jl
      };
      mma_rows(smem_u32(slab), a_row, smem_u32(xsp), xsb, ks * kq, (ks + 1) * kq, lane, d);
      *reinterpret_cast<float4*>(red + (warp * 32 + lane) * 4) = make_float4(d[0], d[1], d[2], d[3]);
      __syncthreads();
      if (ks == 0) {
        const int gq = lane >> 2, tq = lane & 3;
        const int jl = mt * 8 + gq;
        float4 sum = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
        for (int s2 = 0; s2 < 4; ++s2) {
          const float4 v = *reinterpret_cast<const float4*>(red + ((mt + 2 * s2) * 32 + lane) * 4);
          sum.x += v.x;
          sum.y += v.y;
          sum.z += v.z;
          sum.w += v.w;
        }
        // (x, y): gate of column jl for tokens 2tq, 2tq+1; (z, w): up of the same
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int i = 2 * tq + u;
          if (i < R && jl < ncol) {
            const float gv = u == 0 ? sum.x : sum.y, uv = u == 0 ? sum.z : sum.w;
            const float h = round_bf16(round_bf16(silu_ref(round_bf16(gv))) * round_bf16(uv));
            a.hid[(start + r0 + i) * a.ldh + j0 + jl] = f32_to_bf16_rne(h);
          }
        }
      }
      __syncthreads();
      continue;
    }
    // MXFP8 tiles on the CUDA cores: warp w: columns jl = w*2 + {0,1} (+16 on
    // the second pass); lane groups 0: gate(jl), 1: gate(jl+1), 2: up(jl), 3: up(jl+1)
    const int grp = lane >> 3, seg = lane & 7;
    for (int p = 0; p < cols / kSwigluCols; ++p) {
      const int jl = p * kSwigluCols + warp * 2 + (grp & 1);
      const bool live = jl < ncol;
      const int half = grp >> 1;
      const uint8_t* wrow = slab + static_cast<size_t>(half * cols + jl) * ws;
      const int wr = g0 + half * c + jl;  // packed row (for the MXFP8 scales)
      auto emit = [&](int i, float part) {
        const float gv = group_sum8(part);
        const float uv = __shfl_down_sync(0xFFFFFFFFu, gv, 16);  // up of the same column (groups 2, 3 -> 0, 1)
        if (grp < 2 && seg == 0 && live) {
          const float h = round_bf16(round_bf16(silu_ref(round_bf16(gv))) * round_bf16(uv));
          hs[i * kSwigluColsMx + jl] = f32_to_bf16_rne(h);
        }
      };
      dot_rows<true>(wrow, a.w1sf, g, wr, rows1, 2 * c, a.kx, xsb / 2, a.kx,
                     reinterpret_cast<const uint16_t*>(xsp), R, seg, live, emit);
    }
    __syncthreads();
    if (static_cast<int>(threadIdx.x) < R) {
      const int i = threadIdx.x;
      float v[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = j < ncol ? bf16_to_f32(hs[i * kSwigluColsMx + j]) : 0.0f;
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

// Row GEMV: out[pos, n] = bf16(bf16(<A[pos], W[g][n]> [+ bias[n]]) * w[pos])
// for a slab of nblk output columns of group g and the group's rows.
__global__ void __launch_bounds__(kGemvThreads, 3) gemv_rows_kernel(const GemvPass a) {
  extern __shared__ __align__(128) uint8_t smem[];
  int g, n;
  bool mx;
  int64_t start;
  tile_rows(a, g, mx, start, n);
  if (n <= static_cast<int>(blockIdx.z) * kGemvRows) return;
  const int n0 = blockIdx.y * a.nblk;
  if (n0 >= a.n_out) return;
  const int K = mx ? a.kh : a.k2;                    // A row width (BF16 values) in shared memory
  const int wbytes = mx ? a.kh : 2 * a.k2;
  const int ws = wbytes + 16;
  const int xsb = 2 * K + 16;
  const int ncol = min(a.nblk, a.n_out - n0);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem);
  int* abort_flag = reinterpret_cast<int*>(smem + 64);
  uint8_t* slab = smem + 128;
  uint8_t* xsp = slab + static_cast<size_t>(a.nblk) * ws;
  uint16_t* ys = reinterpret_cast<uint16_t*>(xsp + static_cast<size_t>(kGemvRows) * xsb);  // [kGemvRows][nblk]
  float* red = reinterpret_cast<float*>(ys + static_cast<size_t>(kGemvRows) * a.nblk);    // [8][32][4]
  const uint8_t* wbase = mx ? a.w2q : reinterpret_cast<const uint8_t*>(a.w2);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool tc = !mx && gemv_rows_tc(a);
  uint32_t pass = 0;
  for (int r0 = blockIdx.z * kGemvRows; r0 < n; r0 += gridDim.z * kGemvRows, ++pass) {
    const int R = min(kGemvRows, n - r0);
    if (warp == 0) {
      const uint32_t bytes = (pass == 0 ? static_cast<uint32_t>(ncol) * wbytes : 0u) +
                             (mx ? 0u : static_cast<uint32_t>(R) * 2 * K);
      if (lane == 0) {
        if (pass == 0) {
          mbar_init(bar, 1);
          fence_mbar_init();
        } else {
          fence_proxy_async_smem();
        }
        if (bytes) mbar_arrive_expect_tx(bar, bytes); else mbar_arrive(bar);
      }
      __syncwarp();
      if (pass == 0) {
        for (int i = lane; i < ncol; i += 32)
          bulk_load(slab + static_cast<size_t>(i) * ws, wbase + (static_cast<int64_t>(g) * a.n_out + n0 + i) * wbytes,
                    wbytes, bar);
      }
      if (!mx) {
        for (int i = lane; i < R; i += 32) {
          const int64_t row = a.src_row != nullptr ? a.src_row[start + r0 + i] : start + r0 + i;
          bulk_load(xsp + static_cast<size_t>(i) * xsb, a.a2 + row * a.lda2, 2u * K, bar);
        }
      }
    }
    if (mx) stage_rows(true, a.src_row, start + r0, R, a.a2, a.lda2, a.hq, a.hsf, a.kh, a.kh, xsb / 2,
                       reinterpret_cast<uint16_t*>(xsp));
    for (int i = threadIdx.x; i < (kGemvRows - R) * (K / 8); i += blockDim.x) {
      const int r = R + i / (K / 8), q = i % (K / 8);
      reinterpret_cast<uint4*>(xsp + static_cast<size_t>(r) * xsb)[q] = make_uint4(0u, 0u, 0u, 0u);
    }
    // slab rows ncol..nblk of a partial column block are not loaded: zero them once
    if (pass == 0 && tc) {
      for (int i = threadIdx.x; i < (a.nblk - ncol) * (wbytes / 16); i += blockDim.x) {
        const int r = ncol + i / (wbytes / 16), q = i % (wbytes / 16);
        reinterpret_cast<uint4*>(slab + static_cast<size_t>(r) * ws)[q] = make_uint4(0u, 0u, 0u, 0u);
      }
    }
    if (!pass_ready(bar, pass & 1u, a.status, abort_flag)) return;
    if (tc) {
      const int mtiles = a.nblk / 16, ksplit = kGemvWarps / mtiles;
      const int mt = warp % mtiles, ks = warp / mtiles;
      const int kq = a.k_valid2 / ksplit;
      float d[4];
      auto a_row = [&](int m) -> uint32_t { return static_cast<uint32_t>((mt * 16 + m) * ws); };
      mma_rows(smem_u32(slab), a_row, smem_u32(xsp), xsb, ks * kq, (ks + 1) * kq, lane, d);
      if (ksplit > 1) {
        *reinterpret_cast<float4*>(red + (warp * 32 + lane) * 4) = make_float4(d[0], d[1], d[2], d[3]);
        __syncthreads();
        if (ks == 0) {
          float4 sum = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
          for (int s2 = 0; s2 < ksplit; ++s2) {
            const float4 v = *reinterpret_cast<const float4*>(red + ((mt + mtiles * s2) * 32 + lane) * 4);
            sum.x += v.x;
            sum.y += v.y;
            sum.z += v.z;
            sum.w += v.w;
          }
          d[0] = sum.x;
          d[1] = sum.y;
          d[2] = sum.z;
          d[3] = sum.w;
        }
      }
      if (ks == 0) {
        // (d0, d1): output row mt*16 + gq for tokens 2tq, 2tq+1; (d2, d3): row + 8
        const int gq = lane >> 2, tq = lane & 3;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int nl = mt * 16 + gq + (q >> 1) * 8;
          const int i = 2 * tq + (q & 1);
          if (i < R && nl < ncol) {
            const float bias = a.bias != nullptr ? bf16_to_f32(a.bias[n0 + nl]) : 0.0f;
            const float w = a.row_w != nullptr ? bf16_to_f32(a.row_w[start + r0 + i]) : 1.0f;
            ys[i * a.nblk + nl] = f32_to_bf16_rne(round_bf16(d[q] + bias) * w);
          }
        }
      }
    } else {
      // CUDA cores (MXFP8 tiles, or K not splitting evenly): 4 rows per warp step
      const int grp = lane >> 3, seg = lane & 7;
      const int per_warp = a.nblk / kGemvWarps;  // output columns per warp (multiple of 4)
      for (int p = 0; p < per_warp; p += 4) {
        const int nl = warp * per_warp + p + grp;
        const bool live = nl < ncol;
        const uint8_t* wrow = slab + static_cast<size_t>(nl) * ws;
        const float bias = (live && a.bias != nullptr) ? bf16_to_f32(a.bias[n0 + nl]) : 0.0f;
        auto emit = [&](int i, float part) {
          const float y = group_sum8(part);
          if (seg == 0 && live) {
            const float w = a.row_w != nullptr ? bf16_to_f32(a.row_w[start + r0 + i]) : 1.0f;
            ys[i * a.nblk + nl] = f32_to_bf16_rne(round_bf16(y + bias) * w);
          }
        };
        if (mx)
          dot_rows<true>(wrow, a.w2sf, g, n0 + nl, a.n_out, a.bn2m, a.kh, xsb / 2, a.k_valid2,
                         reinterpret_cast<const uint16_t*>(xsp), R, seg, live, emit);
        else
          dot_rows<false>(wrow, nullptr, g, n0 + nl, a.n_out, 0, a.k2, xsb / 2, a.k_valid2,
                          reinterpret_cast<const uint16_t*>(xsp), R, seg, live, emit);
      }
    }
    __syncthreads();
    // staged rows out as row segments (16-byte stores when aligned)
    if ((ncol % 8) == 0 && (a.ldo % 8) == 0) {
      const int per_row = ncol / 8;
      for (int t = threadIdx.x; t < R * per_row; t += blockDim.x) {
        const int i = t / per_row, q = t - i * per_row;
        reinterpret_cast<uint4*>(a.out + (start + r0 + i) * a.ldo + n0)[q] =
            reinterpret_cast<const uint4*>(ys + i * a.nblk)[q];
      }
    } else {
      for (int t = threadIdx.x; t < R * ncol; t += blockDim.x) {
        const int i = t / ncol, q = t - i * ncol;
        a.out[(start + r0 + i) * a.ldo + n0 + q] = ys[i * a.nblk + q];
      }
    }
    __syncthreads();
  }
}

int pick_nblk(int row_bytes) {
  int nb = static_cast<int>(kSlabBytes / static_cast<size_t>(row_bytes));
  nb = std::max(32, std::min(128, nb));
  return nb / 32 * 32;
}

}  // namespace

bool gemv_swiglu_ok(const GemvPass& a) {
  return a.kd % 64 == 0 && a.chunk % kSwigluCols == 0 && a.ldh % 8 == 0 &&
         (a.tiles_mx == nullptr || (a.inter % kMxBlock == 0 && a.cm % kSwigluColsMx == 0 && a.kx % 128 == 0 &&
                                    a.kh % 128 == 0));
}

bool gemv_rows_ok(const GemvPass& a) {
  return a.k2 % 64 == 0 && a.k_valid2 <= a.k2 && a.k_valid2 % (a.tiles_mx != nullptr ? kMxBlock : 8) == 0 &&
         (a.tiles_mx == nullptr || (a.kh % 128 == 0 && a.k_valid2 <= a.kh));
}

// Grid: x = tiles (BF16 table, then the MXFP8 table) or 1 (dense), y = column
// blocks, z = 16-row chunks of a dense pass.
dim3 gemv_grid(const GemvPass& a, int col_blocks) {
  const unsigned x = a.tiles == nullptr ? 1u : static_cast<unsigned>(a.max_tiles * (a.tiles_mx != nullptr ? 2 : 1));
  const unsigned z = a.tiles == nullptr ? static_cast<unsigned>((a.dense_rows + kGemvRows - 1) / kGemvRows) : 1u;
  return dim3(x, static_cast<unsigned>(col_blocks), z);
}

int launch_gemv_swiglu(const GemvPass& a, cudaStream_t stream) {
  if (!gemv_swiglu_ok(a)) return SPX_ERR_UNSUPPORTED;
  const bool mx = a.tiles_mx != nullptr;
  const int K = std::max(a.kd, mx ? a.kx : 0);
  const size_t slab = std::max<size_t>(2 * kSwigluCols * (2 * static_cast<size_t>(a.kd) + 16),
                                       mx ? 2 * kSwigluColsMx * (static_cast<size_t>(a.kx) + 16) : 0);
  const size_t red = kGemvWarps * 32 * 4 * sizeof(float);
  const size_t smem = 128 + slab + static_cast<size_t>(kGemvRows) * (2 * static_cast<size_t>(K) + 16) + red;
  if (smem > kGemmSmemBudget) return SPX_ERR_UNSUPPORTED;
  if (int rc = ensure_max_dynamic_smem(reinterpret_cast<const void*>(gemv_swiglu_kernel)); rc != SPX_OK) return rc;
  gemv_swiglu_kernel<<<gemv_grid(a, (a.inter + kSwigluCols - 1) / kSwigluCols), kGemvThreads, smem, stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? SPX_OK : SPX_ERR_CUDA;
}

int launch_gemv_rows(GemvPass a, cudaStream_t stream) {
  if (!gemv_rows_ok(a)) return SPX_ERR_UNSUPPORTED;
  const bool mx = a.tiles_mx != nullptr;
  const int wbytes = std::max(2 * a.k2, mx ? a.kh : 0);
  a.nblk = pick_nblk(wbytes);
  const int K = std::max(a.k2, mx ? a.kh : 0);
  const size_t red = kGemvWarps * 32 * 4 * sizeof(float);
  const size_t smem = 128 + static_cast<size_t>(a.nblk) * (wbytes + 16) +
                      static_cast<size_t>(kGemvRows) * (2 * static_cast<size_t>(K) + 16) +
                      static_cast<size_t>(kGemvRows) * a.nblk * 2 + red;
  if (smem > kGemmSmemBudget) return SPX_ERR_UNSUPPORTED;
  if (int rc = ensure_max_dynamic_smem(reinterpret_cast<const void*>(gemv_rows_kernel)); rc != SPX_OK) return rc;
  gemv_rows_kernel<<<gemv_grid(a, (a.n_out + a.nblk - 1) / a.nblk), kGemvThreads, smem, stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? SPX_OK : SPX_ERR_CUDA;
}

}  // namespace spx
