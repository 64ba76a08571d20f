// Decode-sized projections: grouped GEMVs.
//
// With a few tokens per step every routed expert sees a handful of rows, and
// the projections are bound by reading their weights once (589,824 bytes per
// expert in BF16 at the 100M shape).  A 128-row tcgen05 tile would hold those
// few rows and spend its time filling and draining; here every warp streams
// its weight rows straight from HBM into registers (16-byte non-allocating
// loads, several K chunks in flight per thread, no shared-memory slab, no
// barrier inside the K loop) and multiplies them on mma.sync m16n8k16 (BF16
// in, FP32 accumulate) against up to 16 token rows staged once per pass in
// shared memory.  The weight rows are the 16-row A operand, the tokens the
// 8-column B operand: the tensor cores run at a fraction of their rate and
// still outrun the weight stream.
//
// Fragment layout.  The dot product is a sum over k, so A and B may read K in
// any order as long as both use the same one.  Thread (gq = lane / 4,
// tq = lane % 4) loads 16 contiguous bytes of its weight row at 8*tq of a
// 32-value chunk (E4M3: 16 values at 16*tq of a 64-value chunk) and feeds
// them as the a0/a2 registers of consecutive k16 steps; the B registers come
// from the same positions of the token rows.  A warp instruction reads 8
// rows x 64 contiguous bytes.
//
// Same rounding points as the tensor-core path (experts/bank.py:755-763 and
// 970-978, nn/ffn.py:27-30, experts/router.py:51): FP32 accumulation;
// SwiGLU h = bf16(bf16(silu(bf16(g))) * bf16(u)); projections
// bf16(bf16(acc [+ bias]) * w).  MXFP8-lane experts (experts/native.py:91-140)
// multiply the E4M3 values with their E8M0 block scales applied: both
// operands are dequantised exactly into BF16 (an E4M3 value times a power of
// two is representable), their products are exact in FP32 and summed there,
// and the SwiGLU GEMV writes the hidden rows quantised again (32-column
// blocks, the epilogue rule of the tensor-core path).
//
// Two kernels (128 threads, 4 warps; a warp owns one m-tile, or a K share of
// one when few tiles would leave SMs idle):
//   gemv_swiglu_kernel  m-tile = 8 gate + 8 up rows of 8 hidden columns, so a
//                       thread's accumulators hold the gate and up values of
//                       one column and the SwiGLU runs in registers
//   gemv_rows_kernel    m-tile = 16 output columns (+ bias, x routing weight)
// Expert passes run over the dispatch's tile tables (a tile = up to 128 rows
// of one expert's dispatch range, token rows gathered through src_row); the
// dense projections (router, shared SwiGLU) over the whole batch in 16-row
// chunks.
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

#include "kernels.h"
#include "mx.cuh"
#include "sm100.cuh"

namespace spx {

namespace {

constexpr int kGemvThreads = 128;
constexpr int kGemvWarps = kGemvThreads / 32;
constexpr int kPassRows = 16;   // token rows per pass: two 8-column mma tiles
constexpr int kRowPad = 32;     // token row padding in shared memory (values): rows 64 bytes apart mod 128
constexpr int kRedBytes = kGemvWarps * 32 * 8 * static_cast<int>(sizeof(float));

__device__ __forceinline__ float silu_ref(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

// 2^(byte - 127): the value of an E8M0 scale byte.
__device__ __forceinline__ float e8m0_value(uint32_t byte) {
  if (byte == 0u) return __uint_as_float(0x00400000u);  // 2^-127
  return __uint_as_float(byte << 23);
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

// Two floats that are BF16 values to a BF16 pair (lo in the low half).
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// 16 bytes of a weight row, read once: no L1 allocation, 256-byte L2 fetches.
__device__ __forceinline__ uint4 ld_stream(const void* p) {
  uint4 v;
  asm("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0, %1, %2, %3}, [%4];"
      : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
      : "l"(p));
  return v;
}

// 16 bytes of a staged token row.  Volatile, so that the loads stay between
// the MMAs that use them instead of being hoisted (and held in registers)
// ahead of a whole step.
__device__ __forceinline__ uint4 lds128(const uint16_t* p) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(smem_u32(p)));
  return v;
}

__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Token rows into shared memory as BF16 [R][K] (row stride xstride values):
// 16-byte cp.async copies (all in flight at once), or E4M3 rows dequantised
// with their block scales (exact), loads batched ahead of the conversions.
// Row i of the pass is token row src[pos0 + i] (gather) or pos0 + i.  The
// caller waits (cp_async_wait_all) and synchronises.
__device__ void stage_rows(bool mx, const int* src, int64_t pos0, int R, const uint16_t* rows_bf16, int64_t ld_bf16,
                           const uint8_t* rows_q, const uint8_t* rows_sf, int ld_q, int K, int xstride,
                           uint16_t* xs) {
  if (!mx) {
    const int per_row = K / 8;
    for (int i = threadIdx.x; i < R * per_row; i += blockDim.x) {
      const int r = i / per_row, c = i - r * per_row;
      const int64_t row = src != nullptr ? src[pos0 + r] : pos0 + r;
      cp_async16(smem_u32(xs + static_cast<int64_t>(r) * xstride + 8 * c), rows_bf16 + row * ld_bf16 + 8 * c);
    }
    return;
  }
  constexpr int kBatch = 2;
  const int per_row = K / 16;
  for (int i0 = threadIdx.x; i0 < R * per_row; i0 += kBatch * blockDim.x) {
    uint4 q[kBatch];
    uint32_t sb[kBatch];
#pragma unroll
    for (int j = 0; j < kBatch; ++j) {
      const int i = i0 + j * blockDim.x;
      if (i < R * per_row) {
        const int r = i / per_row, c = i - r * per_row;
        const int64_t row = src != nullptr ? src[pos0 + r] : pos0 + r;
        q[j] = __ldg(reinterpret_cast<const uint4*>(rows_q + row * ld_q) + c);
        sb[j] = __ldg(rows_sf + row * (ld_q / kMxBlock) + (c >> 1));
      }
    }
#pragma unroll
    for (int j = 0; j < kBatch; ++j) {
      const int i = i0 + j * blockDim.x;
      if (i < R * per_row) {
        const int r = i / per_row, c = i - r * per_row;
        const float s = e8m0_value(sb[j]);
        float f[16];
        e4m3x4(q[j].x, s, f);
        e4m3x4(q[j].y, s, f + 4);
        e4m3x4(q[j].z, s, f + 8);
        e4m3x4(q[j].w, s, f + 12);
        uint4* dst = reinterpret_cast<uint4*>(xs + static_cast<int64_t>(r) * xstride + c * 16);
        dst[0] = make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]), pack_bf16x2(f[4], f[5]),
                            pack_bf16x2(f[6], f[7]));
        dst[1] = make_uint4(pack_bf16x2(f[8], f[9]), pack_bf16x2(f[10], f[11]), pack_bf16x2(f[12], f[13]),
                            pack_bf16x2(f[14], f[15]));
      }
    }
  }
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
  const int per = a.tile_grid > 0 ? a.tile_grid : a.max_tiles;
  if (t >= per) {
    t -= per;
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

// ---- A warp's weight stream.  A step is U chunks of 32 values (BF16) or
// U / 2 chunks of 64 (E4M3) of the thread's two A rows, all its loads issued
// before the step multiplies.
template <bool MX, int U>
struct WBuf;
template <int U>
struct WBuf<false, U> {
  static constexpr int kStep = 32 * U;
  uint4 l[U], h[U];
};
template <int U>
struct WBuf<true, U> {
  static constexpr int kN = U / 2;
  static constexpr int kStep = 64 * kN;
  uint4 l[kN], h[kN];
  float sl[kN], sh[kN];
};

// The thread's A rows of one m-tile: rows gq (lo) and gq + 8 (hi).
struct ARows {
  const uint8_t* lo;  // row starts (bytes)
  const uint8_t* hi;
  const uint8_t* sc_lo;  // MXFP8: the rows' scale bytes of K block 0 (mx_scale_row)
  const uint8_t* sc_hi;
};

// Scale-atom layout of a packed MXFP8 weight: atoms [groups][tiles][K/128]
// [ceil(tile_rows/128)][512] (mx_quantize_b_kernel).  The scale byte of
// (row, K block blk) is row_ptr[(blk / 4) * stride + blk % 4] with
// row_ptr = mx_scale_row(row) and stride = 512 * ceil(tile_rows / 128).
struct MxAtoms {
  const uint8_t* atoms;
  int g, rows_per_group, tile_rows, kp;
  __device__ __forceinline__ int stride() const { return kMxAtomBytes * ((tile_rows + 127) / 128); }
  __device__ __forceinline__ const uint8_t* row(int r) const {
    const int tiles = (rows_per_group + tile_rows - 1) / tile_rows;
    const int per_tile = (tile_rows + 127) / 128;
    const int tile = r / tile_rows, rr = r - tile * tile_rows;
    const int64_t atom = ((static_cast<int64_t>(g) * tiles + tile) * (kp / 128)) * per_tile + (rr >> 7);
    return atoms + atom * kMxAtomBytes + mx_atom_offset(rr & 127, 0);
  }
};

template <int U>
__device__ __forceinline__ void load_step(const ARows& r, int k0, int ke, int tq, const MxAtoms&, WBuf<false, U>& b) {
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int k = k0 + 32 * u + 8 * tq;
    b.l[u] = k < ke ? ld_stream(r.lo + 2 * k) : make_uint4(0u, 0u, 0u, 0u);
    b.h[u] = k < ke ? ld_stream(r.hi + 2 * k) : make_uint4(0u, 0u, 0u, 0u);
  }
}

template <int U>
__device__ __forceinline__ void load_step(const ARows& r, int k0, int ke, int tq, const MxAtoms& m, WBuf<true, U>& b) {
  const int stride = m.stride();
#pragma unroll
  for (int u = 0; u < WBuf<true, U>::kN; ++u) {
    const int k = k0 + 64 * u + 16 * tq;
    const bool v = k < ke;
    const int blk = k / kMxBlock, so = (blk >> 2) * stride + (blk & 3);
    b.l[u] = v ? ld_stream(r.lo + k) : make_uint4(0u, 0u, 0u, 0u);
    b.h[u] = v ? ld_stream(r.hi + k) : make_uint4(0u, 0u, 0u, 0u);
    b.sl[u] = v ? e8m0_value(__ldg(r.sc_lo + so)) : 0.0f;
    b.sh[u] = v ? e8m0_value(__ldg(r.sc_hi + so)) : 0.0f;
  }
}

// acc[t] += A[16 rows] . X[8t .. 8t+8)^T for one step (whole thread slots
// past ke read as zero on both sides).
template <int U>
__device__ __forceinline__ void mma_step(const WBuf<false, U>& b, const uint16_t* xs, int xsl, int k0, int ke, int nt,
                                         int gq, int tq, float (&acc)[2][4]) {
#pragma unroll
  for (int u = 0; u < U; ++u) {
    if (k0 + 32 * u >= ke) break;  // warp-uniform
    const int k = k0 + 32 * u + 8 * tq;
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      if (t >= nt) break;
      const uint4 x = k < ke ? lds128(xs + (8 * t + gq) * xsl + k) : make_uint4(0u, 0u, 0u, 0u);
      mma_16816(acc[t], b.l[u].x, b.h[u].x, b.l[u].y, b.h[u].y, x.x, x.y);
      mma_16816(acc[t], b.l[u].z, b.h[u].z, b.l[u].w, b.h[u].w, x.z, x.w);
    }
  }
}

template <int U>
__device__ __forceinline__ void mma_step(const WBuf<true, U>& b, const uint16_t* xs, int xsl, int k0, int ke, int nt,
                                         int gq, int tq, float (&acc)[2][4]) {
#pragma unroll
  for (int u = 0; u < WBuf<true, U>::kN; ++u) {
    if (k0 + 64 * u >= ke) break;  // warp-uniform
    const int k = k0 + 64 * u + 16 * tq;
    uint32_t xw[2][8];
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      uint4 x0 = make_uint4(0u, 0u, 0u, 0u), x1 = x0;
      if (t < nt && k < ke) {
        x0 = lds128(xs + (8 * t + gq) * xsl + k);
        x1 = lds128(xs + (8 * t + gq) * xsl + k + 8);
      }
      xw[t][0] = x0.x, xw[t][1] = x0.y, xw[t][2] = x0.z, xw[t][3] = x0.w;
      xw[t][4] = x1.x, xw[t][5] = x1.y, xw[t][6] = x1.z, xw[t][7] = x1.w;
    }
    const uint32_t lw[4] = {b.l[u].x, b.l[u].y, b.l[u].z, b.l[u].w};
    const uint32_t hw[4] = {b.h[u].x, b.h[u].y, b.h[u].z, b.h[u].w};
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      float fl[4], fh[4];
      e4m3x4(lw[s], b.sl[u], fl);
      e4m3x4(hw[s], b.sh[u], fh);
      const uint32_t a0 = pack_bf16x2(fl[0], fl[1]), a2 = pack_bf16x2(fl[2], fl[3]);
      const uint32_t a1 = pack_bf16x2(fh[0], fh[1]), a3 = pack_bf16x2(fh[2], fh[3]);
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        if (t >= nt) break;
        mma_16816(acc[t], a0, a1, a2, a3, xw[t][2 * s], xw[t][2 * s + 1]);
      }
    }
  }
}

// `steps` steps over m-tiles m = s / G (K group s % G from kb); b holds step
// 0's loads on entry (issued before the token rows were staged).  end_tile(m)
// runs after m-tile m's last K group.  One register buffer: the warps of the
// SM (five CTAs of four) keep the weight stream busy between one warp's
// steps.
template <bool MX, int U, typename RowsOf, typename EndTile>
__device__ __forceinline__ void run_stream(int steps, int G, int kb, int ke, RowsOf rows_of, const MxAtoms& ma,
                                           const uint16_t* xs, int xsl, int nt, int gq, int tq, WBuf<MX, U>& b,
                                           float (&acc)[2][4], EndTile end_tile) {
  constexpr int kStep = WBuf<MX, U>::kStep;
#pragma unroll 1
  for (int s = 0; s < steps; ++s) {
    if (s > 0) load_step(rows_of(s / G), kb + (s % G) * kStep, ke, tq, ma, b);
    mma_step(b, xs, xsl, kb + (s % G) * kStep, ke, nt, gq, tq, acc);
    if (s % G == G - 1) end_tile(s / G);
  }
}

// Warps sharing an m-tile (ks > 0) add their partial sums into warp ks = 0's
// accumulators through shared memory.  Every thread of the CTA calls it.
__device__ __forceinline__ void reduce_ksplit(float* red, int ksplit, int mtiles, int mt, int ks, int lane,
                                              float (&acc)[2][4]) {
  if (ksplit == 1) return;
  if (ks > 0) {
    float4* dst = reinterpret_cast<float4*>(red + ((threadIdx.x >> 5) * 32 + lane) * 8);
    dst[0] = make_float4(acc[0][0], acc[0][1], acc[0][2], acc[0][3]);
    dst[1] = make_float4(acc[1][0], acc[1][1], acc[1][2], acc[1][3]);
  }
  __syncthreads();
  if (ks == 0) {
    for (int s = 1; s < ksplit; ++s) {
      const float4* src = reinterpret_cast<const float4*>(red + ((s * mtiles + mt) * 32 + lane) * 8);
      const float4 p0 = src[0], p1 = src[1];
      acc[0][0] += p0.x;
      acc[0][1] += p0.y;
      acc[0][2] += p0.z;
      acc[0][3] += p0.w;
      acc[1][0] += p1.x;
      acc[1][1] += p1.y;
      acc[1][2] += p1.z;
      acc[1][3] += p1.w;
    }
  }
}

__device__ __forceinline__ void zero_acc(float (&acc)[2][4]) {
#pragma unroll
  for (int t = 0; t < 2; ++t)
#pragma unroll
    for (int q = 0; q < 4; ++q) acc[t][q] = 0.0f;
}

// SwiGLU GEMV: hidden[pos, j] for 8 columns per m-tile.  A CTA covers
// 8 * (4 / ksplit) hidden columns of one tile (the MXFP8 lane: 32 columns,
// one scale block of the hidden row, ksplit 1) and loops over the tile's
// 16-row passes.
template <bool MX>
__device__ __forceinline__ void swiglu_cta(const GemvPass& a, int g, int64_t start, int n, uint8_t* smem,
                                           bool pending) {
  const int ksplit = MX ? 1 : a.ksplit;
  const int mtiles = kGemvWarps / ksplit;
  const int j_cta = static_cast<int>(blockIdx.y) * 8 * mtiles;
  if (j_cta >= a.inter) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gq = lane >> 2, tq = lane & 3;
  const int mt = warp % mtiles, ks = warp / mtiles;
  const int jw = j_cta + 8 * mt;
  const bool live = jw < a.inter;  // warp-uniform
  const int c = MX ? a.cm : a.chunk;
  const int rows1 = (MX ? a.ncm : a.nc) * 2 * c;
  const int K = MX ? a.kx : a.kd;  // weight row width = token row width (values)
  const int esz = MX ? 1 : 2;
  const int xsl = K + kRowPad;
  uint16_t* xs = reinterpret_cast<uint16_t*>(smem);
  float* red = reinterpret_cast<float*>(smem + static_cast<size_t>(kPassRows) * xsl * 2);
  uint16_t* hs = reinterpret_cast<uint16_t*>(red);  // MXFP8 lane: [kPassRows][32] hidden values
  // A rows of the thread: the gate row of column jw + gq (packed [gate | up]
  // chunks of c rows) and its up row c rows further
  const int ch = jw / c;
  const int grow = ch * 2 * c + (jw - ch * c) + gq;
  const uint8_t* wbase = MX ? a.w1q : reinterpret_cast<const uint8_t*>(a.w1);
  const MxAtoms ma{a.w1sf, g, rows1, 2 * c, K};
  const ARows rows{wbase + (static_cast<int64_t>(g) * rows1 + grow) * K * esz,
                   wbase + (static_cast<int64_t>(g) * rows1 + grow + c) * K * esz, MX ? ma.row(grow) : nullptr,
                   MX ? ma.row(grow + c) : nullptr};
  const int kq = K / ksplit;
  const int kb = ks * kq, ke = kb + kq;
  constexpr int U = 4;  // BF16 chunks per step
  const int G = (kq + WBuf<MX, U>::kStep - 1) / WBuf<MX, U>::kStep;
  for (int r0 = static_cast<int>(blockIdx.z) * kPassRows; r0 < n; r0 += static_cast<int>(gridDim.z) * kPassRows) {
    const int R = min(kPassRows, n - r0);
    const int nt = R > 8 ? 2 : 1;
    WBuf<MX, U> b0;
    if (live) load_step(rows, kb, ke, tq, ma, b0);  // under the staging below
    if (pending) {  // a dense pass: the weights above are static, the token rows are not
      griddep_wait();
      griddep_launch_dependents();
      pending = false;
    }
    __syncthreads();  // the previous pass no longer reads xs / hs
    stage_rows(MX, a.src_row, start + r0, R, a.x, a.ldx, a.xq, a.xsf, a.kx, K, xsl, xs);
    cp_async_wait_all();
    __syncthreads();
    float acc[2][4];
    zero_acc(acc);
    if (live) run_stream<MX, U>(G, G, kb, ke, [&](int) { return rows; }, ma, xs, xsl, nt, gq, tq, b0, acc, [](int) {});
    reduce_ksplit(red, ksplit, mtiles, mt, ks, lane, acc);
    // (d0, d1): gate of column jw + gq for tokens 2tq, 2tq + 1 of the n-tile; (d2, d3): up
    if (ks == 0 && live) {
#pragma unroll
      for (int t = 0; t < 2; ++t) {
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int i = 8 * t + 2 * tq + u;
          if (i < R) {
            const float h = round_bf16(round_bf16(silu_ref(round_bf16(acc[t][u]))) * round_bf16(acc[t][2 + u]));
            if (MX)
              hs[i * 32 + 8 * mt + gq] = f32_to_bf16_rne(h);
            else
              a.hid[(start + r0 + i) * a.ldh + jw + gq] = f32_to_bf16_rne(h);
          }
        }
      }
    }
    if (MX) {
      __syncthreads();
      if (static_cast<int>(threadIdx.x) < R) {
        const int i = threadIdx.x;
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = bf16_to_f32(hs[i * 32 + j]);
        uint32_t qw[8];
        const uint32_t sb = mx_quantize32(v, qw);
        uint4* dst = reinterpret_cast<uint4*>(a.hq + (start + r0 + i) * a.kh + j_cta);
        dst[0] = make_uint4(qw[0], qw[1], qw[2], qw[3]);
        dst[1] = make_uint4(qw[4], qw[5], qw[6], qw[7]);
        a.hsf[(start + r0 + i) * (a.kh / kMxBlock) + j_cta / kMxBlock] = static_cast<uint8_t>(sb);
      }
    }
  }
}

__global__ void __launch_bounds__(kGemvThreads, 5) gemv_swiglu_kernel(const GemvPass a) {
  extern __shared__ __align__(16) uint8_t smem[];
  // Expert passes read the dispatch's tile tables: wait first.  Dense passes
  // issue their first weight loads before waiting.
  const bool dense = a.tiles == nullptr;
  if (!dense) {
    griddep_wait();
    griddep_launch_dependents();
  }
  int g, n;
  bool mx;
  int64_t start;
  tile_rows(a, g, mx, start, n);
  if (n <= static_cast<int>(blockIdx.z) * kPassRows) return;
  if (mx)
    swiglu_cta<true>(a, g, start, n, smem, dense);
  else
    swiglu_cta<false>(a, g, start, n, smem, dense);
}

// Row GEMV: out[pos, n] = bf16(bf16(<A[pos], W[g][n]> [+ bias[n]]) * w[pos]).
// A warp walks a.mpw m-tiles of 16 output columns (a.mpw = 1 when warps
// split K); a CTA covers 16 * mpw * (4 / ksplit) columns of one tile (or of a
// dense pass's 16-row chunk) and loops over the tile's 16-row passes; K runs
// to k_valid2 (thread slots past it read as zero).
template <bool MX>
__device__ __forceinline__ void rows_cta(const GemvPass& a, int g, int64_t start, int n, uint8_t* smem,
                                         bool pending) {
  const int kv = a.k_valid2;
  const int ksplit = a.ksplit, mpw = a.mpw;
  const int mtiles = kGemvWarps / ksplit;
  const int n_cta = static_cast<int>(blockIdx.y) * 16 * mpw * mtiles;
  if (n_cta >= a.n_out) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gq = lane >> 2, tq = lane & 3;
  const int mt = warp % mtiles, ks = warp / mtiles;
  const int n_warp = n_cta + 16 * mpw * mt;  // the warp's first output column
  const int m_live = min(mpw, (a.n_out - n_warp + 15) / 16);  // m-tiles with columns (<= 0: none)
  const int K = MX ? a.kh : a.k2;  // weight row width = A row width (values)
  const int esz = MX ? 1 : 2;
  const int xsl = K + kRowPad;
  uint16_t* xs = reinterpret_cast<uint16_t*>(smem);
  float* red = reinterpret_cast<float*>(smem + static_cast<size_t>(kPassRows) * xsl * 2);
  const uint8_t* wbase = (MX ? a.w2q : reinterpret_cast<const uint8_t*>(a.w2)) +
                         static_cast<int64_t>(g) * a.n_out * K * esz;
  // A rows of m-tile m (clamped inside the weight; the extra rows' sums are not stored)
  const MxAtoms ma{a.w2sf, g, a.n_out, a.bn2m, K};
  auto rows_of = [&](int m) {
    const int nw = n_warp + 16 * m;
    const int lo = min(nw + gq, a.n_out - 1), hi = min(nw + gq + 8, a.n_out - 1);
    return ARows{wbase + static_cast<int64_t>(lo) * K * esz, wbase + static_cast<int64_t>(hi) * K * esz,
                 MX ? ma.row(lo) : nullptr, MX ? ma.row(hi) : nullptr};
  };
  constexpr int kSlot = MX ? 16 : 8;
  const int kq = (kv / kSlot + ksplit - 1) / ksplit * kSlot;  // K share per warp, whole thread slots
  const int kb = min(ks * kq, kv), ke = min(kb + kq, kv);
  constexpr int U = 4;  // BF16 chunks per step
  const int G = (ke - kb + WBuf<MX, U>::kStep - 1) / WBuf<MX, U>::kStep;
  const int steps = m_live > 0 ? m_live * G : 0;
  for (int r0 = static_cast<int>(blockIdx.z) * kPassRows; r0 < n; r0 += static_cast<int>(gridDim.z) * kPassRows) {
    const int R = min(kPassRows, n - r0);
    const int nt = R > 8 ? 2 : 1;
    WBuf<MX, U> b0;
    if (steps > 0) load_step(rows_of(0), kb, ke, tq, ma, b0);  // under the staging below
    if (pending) {  // a dense pass: the weights above are static, the A rows are not
      griddep_wait();
      griddep_launch_dependents();
      pending = false;
    }
    __syncthreads();  // the previous pass no longer reads xs / red
    stage_rows(MX, a.src_row, start + r0, R, a.a2, a.lda2, a.hq, a.hsf, a.kh, K, xsl, xs);
    // routing weights of the thread's output tokens
    float w[2][2];
#pragma unroll
    for (int t = 0; t < 2; ++t)
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int i = 8 * t + 2 * tq + u;
        w[t][u] = (a.row_w != nullptr && i < R) ? bf16_to_f32(a.row_w[start + r0 + i]) : 1.0f;
      }
    cp_async_wait_all();
    __syncthreads();
    float acc[2][4];
    zero_acc(acc);
    // (d0, d1): output column nw + gq for tokens 2tq, 2tq + 1 of the n-tile; (d2, d3): column + 8
    auto store = [&](int m) {
      const int nw = n_warp + 16 * m;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int col = nw + gq + (q >> 1) * 8;
        if (col >= a.n_out) continue;
        const float bias = a.bias != nullptr ? bf16_to_f32(a.bias[col]) : 0.0f;
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          const int i = 8 * t + 2 * tq + (q & 1);
          if (i < R)
            a.out[(start + r0 + i) * a.ldo + col] = f32_to_bf16_rne(round_bf16(acc[t][q] + bias) * w[t][q & 1]);
        }
      }
    };
    if (ksplit == 1) {
      run_stream<MX, U>(steps, G, kb, ke, rows_of, ma, xs, xsl, nt, gq, tq, b0, acc, [&](int m) {
        store(m);
        zero_acc(acc);
      });
    } else {
      // one m-tile per warp (mpw = 1)
      run_stream<MX, U>(steps, G, kb, ke, rows_of, ma, xs, xsl, nt, gq, tq, b0, acc, [](int) {});
      reduce_ksplit(red, ksplit, mtiles, mt, ks, lane, acc);
      if (ks == 0 && m_live > 0) store(0);
    }
  }
}

__global__ void __launch_bounds__(kGemvThreads, 5) gemv_rows_kernel(const GemvPass a) {
  extern __shared__ __align__(16) uint8_t smem[];
  const bool dense = a.tiles == nullptr;
  if (!dense) {
    griddep_wait();
    griddep_launch_dependents();
  }
  int g, n;
  bool mx;
  int64_t start;
  tile_rows(a, g, mx, start, n);
  if (n <= static_cast<int>(blockIdx.z) * kPassRows) return;
  if (mx)
    rows_cta<true>(a, g, start, n, smem, dense);
  else
    rows_cta<false>(a, g, start, n, smem, dense);
}

// K split that fills the SMs: the smallest of 1, 2, 4 (up to max_split) that
// gives at least two CTAs per SM over `units` x column groups.
int pick_ksplit(int64_t units, int cols, int cols_per_mtile, int max_split) {
  const int sms = device_sm_count();
  const int64_t target = 2 * static_cast<int64_t>(sms > 0 ? sms : 148);
  int ks = 1;
  while (ks < max_split) {
    const int per_cta = cols_per_mtile * (kGemvWarps / ks);
    if (units * ((cols + per_cta - 1) / per_cta) >= target) break;
    ks *= 2;
  }
  return ks;
}

int gemv_tile_grid(const GemvPass& a) { return a.tile_grid > 0 ? a.tile_grid : a.max_tiles; }

int64_t gemv_units(const GemvPass& a) {
  return a.tiles != nullptr ? gemv_tile_grid(a) : (a.dense_rows + kPassRows - 1) / kPassRows;
}

// Grid: x = tiles (BF16 table, then the MXFP8 table) or 1 (dense), y = column
// groups, z = 16-row chunks of a dense pass.
dim3 gemv_grid(const GemvPass& a, int col_groups) {
  const unsigned x = a.tiles == nullptr ? 1u : static_cast<unsigned>(gemv_tile_grid(a) * (a.tiles_mx != nullptr ? 2 : 1));
  const unsigned z = a.tiles == nullptr ? static_cast<unsigned>((a.dense_rows + kPassRows - 1) / kPassRows) : 1u;
  return dim3(x, static_cast<unsigned>(col_groups), z);
}

}  // namespace

bool gemv_swiglu_ok(const GemvPass& a) {
  return a.kd % 64 == 0 && a.chunk % 8 == 0 && a.inter > 0 &&
         (a.tiles_mx == nullptr || (a.inter % kMxBlock == 0 && a.cm % kMxBlock == 0 && a.kx % 128 == 0 &&
                                    a.kh % 128 == 0));
}

bool gemv_rows_ok(const GemvPass& a) {
  return a.k2 % 64 == 0 && a.k_valid2 > 0 && a.k_valid2 <= a.k2 && a.n_out > 0 &&
         a.k_valid2 % (a.tiles_mx != nullptr ? kMxBlock : 8) == 0 &&
         (a.tiles_mx == nullptr || (a.kh % 128 == 0 && a.k_valid2 <= a.kh));
}

int launch_gemv_swiglu(GemvPass a, cudaStream_t stream) {
  if (!gemv_swiglu_ok(a)) return SPX_ERR_UNSUPPORTED;
  const bool mx = a.tiles_mx != nullptr;
  const int K = std::max(a.kd, mx ? a.kx : 0);
  const size_t smem = static_cast<size_t>(kPassRows) * (K + kRowPad) * 2 + kRedBytes;
  if (smem > kGemmSmemBudget) return SPX_ERR_UNSUPPORTED;
  // the BF16 K share stays a multiple of one 32-value chunk
  a.ksplit = pick_ksplit(gemv_units(a), a.inter, 8, a.kd % 128 == 0 ? 4 : 2);
  if (smem > 48 * 1024)
    if (int rc = ensure_max_dynamic_smem(reinterpret_cast<const void*>(gemv_swiglu_kernel)); rc != SPX_OK) return rc;
  const int per_cta = 8 * (kGemvWarps / a.ksplit);
  const int groups = std::max((a.inter + per_cta - 1) / per_cta, mx ? (a.inter + 31) / 32 : 0);
  return launch_pdl(gemv_swiglu_kernel, gemv_grid(a, groups), dim3(kGemvThreads), smem, stream, a);
}

int launch_gemv_rows(GemvPass a, cudaStream_t stream) {
  if (!gemv_rows_ok(a)) return SPX_ERR_UNSUPPORTED;
  const bool mx = a.tiles_mx != nullptr;
  const int K = std::max(a.k2, mx ? a.kh : 0);
  const size_t smem = static_cast<size_t>(kPassRows) * (K + kRowPad) * 2 + kRedBytes;
  if (smem > kGemmSmemBudget) return SPX_ERR_UNSUPPORTED;
  const int64_t units = gemv_units(a);
  a.ksplit = pick_ksplit(units, a.n_out, 16, 4);
  // with whole m-tiles per warp, the most m-tiles per warp that still fill the SMs
  a.mpw = 1;
  if (a.ksplit == 1) {
    const int sms = device_sm_count();
    const int64_t target = 2 * static_cast<int64_t>(sms > 0 ? sms : 148);
    for (int m = 4; m > 1; m >>= 1) {
      const int per = 16 * kGemvWarps * m;
      if (units * ((a.n_out + per - 1) / per) >= target) {
        a.mpw = m;
        break;
      }
    }
  }
  if (smem > 48 * 1024)
    if (int rc = ensure_max_dynamic_smem(reinterpret_cast<const void*>(gemv_rows_kernel)); rc != SPX_OK) return rc;
  const int per_cta = 16 * a.mpw * (kGemvWarps / a.ksplit);
  return launch_pdl(gemv_rows_kernel, gemv_grid(a, (a.n_out + per_cta - 1) / per_cta), dim3(kGemvThreads), smem,
                    stream, a);
}

}  // namespace spx
