// NVFP4 quantisers (E2M1 values, UE4M3 scales per 1x16 block along K,
// per-tensor FP32 scale; the rule is restated in nv.cuh).
//
//  * tensor amax: the per-tensor scale of a matrix (dense matmul operands),
//    of each group's slice (expert weights, pack time), or of each expert's
//    rows (tile tables: a per-row amax, then the max over a tile's rows);
//  * rows: BF16 rows -> E2M1 [rows, kp/2] + scale bytes [rows, kp/16] (the
//    activations of NVFP4 experts in dispatch order, one per-tensor scale per
//    expert as experts/native.py:240-256 quantises each expert's input);
//  * B operands (pack time): E2M1 [groups, rows, kp/2] and the scale bytes in
//    the 512-byte atoms the GEMM copies into tensor memory, one atom per
//    K-64 MMA and 128-row block: [groups][row tiles][kp/256][4][blocks][512].
// K beyond the real width (kp is a multiple of 256) quantises to zero.
#include <cuda_runtime.h>
#include <stdint.h>

#include "kernels.h"
#include "mx.cuh"
#include "nv.cuh"
#include "sm100.cuh"

namespace spx {

namespace {

int nv_grid(int64_t total, int threads) {
  int64_t g = (total + threads - 1) / threads;
  if (g > 148 * 32) g = 148 * 32;
  return static_cast<int>(g < 1 ? 1 : g);
}

// amax values are non-negative floats: their bit patterns order like ints.
__device__ __forceinline__ void atomic_max_nonneg(float* addr, float v) {
  atomicMax(reinterpret_cast<int*>(addr), __float_as_int(v));
}

__device__ __forceinline__ float block_max(float v) {
  __shared__ float red[32];
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, off));
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  v = (threadIdx.x < (blockDim.x >> 5)) ? red[threadIdx.x] : 0.0f;
  if (warp == 0) {
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, off));
  }
  __syncthreads();
  return v;  // valid in thread 0
}

// 16 values of row `row` starting at column c0 (zero beyond `cols`).
__device__ __forceinline__ void load16(const uint16_t* row, int c0, int cols, bool vec, float (&v)[16]) {
  if (vec && c0 + 16 <= cols) {
#pragma unroll
    for (int w = 0; w < 2; ++w) {
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(row + c0) + w);
      const uint32_t words[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        v[8 * w + 2 * h] = __uint_as_float(words[h] << 16);
        v[8 * w + 2 * h + 1] = __uint_as_float(words[h] & 0xFFFF0000u);
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = (c0 + j < cols) ? bf16_to_f32(row[c0 + j]) : 0.0f;
  }
}

__device__ __forceinline__ void quantize_block(const uint16_t* src_row, int cols, bool vec, int blk, float pts,
                                               uint8_t* q_row, uint8_t* sf_row) {
  float v[16];
  load16(src_row, blk * kNvBlock, cols, vec, v);
  uint32_t w0, w1;
  const uint32_t sb = nv_quantize16(v, pts, w0, w1);
  *reinterpret_cast<uint2*>(q_row + blk * (kNvBlock / 2)) = make_uint2(w0, w1);
  sf_row[blk] = static_cast<uint8_t>(sb);
}

}  // namespace

__global__ void nv_amax_kernel(const uint16_t* __restrict__ src, int64_t rows, int cols, int64_t ld,
                               float* __restrict__ amax) {
  float m = 0.0f;
  const int64_t total = rows * cols;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / cols;
    m = fmaxf(m, fabsf(bf16_to_f32(src[r * ld + (i - r * cols)])));
  }
  m = block_max(m);
  if (threadIdx.x == 0) atomic_max_nonneg(amax, m);
}

// One warp per row.
__global__ void nv_row_amax_kernel(const uint16_t* __restrict__ src, int64_t rows, int cols, int64_t ld,
                                   float* __restrict__ row_amax) {
  const int lane = threadIdx.x & 31;
  const int64_t nwarps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  const bool vec = (cols % 8) == 0 && (ld % 8) == 0 && (reinterpret_cast<uintptr_t>(src) & 15u) == 0;
  for (int64_t row = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5); row < rows;
       row += nwarps) {
    const uint16_t* r = src + row * ld;
    float m = 0.0f;
    if (vec) {
      for (int c = lane * 8; c < cols; c += 256) {
        const uint4 u = __ldg(reinterpret_cast<const uint4*>(r + c));
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int h = 0; h < 4; ++h)
          m = fmaxf(m, fmaxf(fabsf(__uint_as_float(w[h] << 16)), fabsf(__uint_as_float(w[h] & 0xFFFF0000u))));
      }
    } else {
      for (int c = lane; c < cols; c += 32) m = fmaxf(m, fabsf(bf16_to_f32(r[c])));
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, off));
    if (lane == 0) row_amax[row] = m;
  }
}

// One CTA (128 threads) per tile.
__global__ void nv_tile_amax_kernel(const int4* __restrict__ tiles, const int* __restrict__ num_tiles,
                                    const int* __restrict__ gather, const float* __restrict__ row_amax,
                                    float* __restrict__ amax) {
  if (static_cast<int>(blockIdx.x) >= *num_tiles) return;
  const int4 t = tiles[blockIdx.x];
  float m = 0.0f;
  if (static_cast<int>(threadIdx.x) < t.z) {
    const int p = t.y + threadIdx.x;
    m = row_amax[gather != nullptr ? gather[p] : p];
  }
  m = block_max(m);
  if (threadIdx.x == 0 && t.w >= 0) atomic_max_nonneg(amax + t.w, m);
}

// One thread per (row, 16-element block).
__global__ void nv_quantize_rows_kernel(const uint16_t* __restrict__ src, int64_t rows, int cols, int64_t ld,
                                        const float* __restrict__ amax, int kp, uint8_t* __restrict__ q,
                                        uint8_t* __restrict__ sf) {
  const int nblk = kp / kNvBlock;
  const float pts = nv_tensor_scale(*amax);
  const bool vec = (cols % 8) == 0 && (ld % 8) == 0 && (reinterpret_cast<uintptr_t>(src) & 15u) == 0;
  const int64_t total = rows * nblk;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = i / nblk;
    const int blk = static_cast<int>(i - row * nblk);
    quantize_block(src + row * ld, cols, vec, blk, pts, q + row * (kp / 2), sf + row * nblk);
  }
}

// One CTA (256 threads) per tile: a warp per row, a lane per 16-element block.
__global__ void nv_quantize_tiles_kernel(const int4* __restrict__ tiles, const int* __restrict__ num_tiles,
                                         const uint16_t* __restrict__ src, int64_t ld, int cols,
                                         const int* __restrict__ gather, const float* __restrict__ amax, int kp,
                                         uint8_t* __restrict__ q, uint8_t* __restrict__ sf) {
  if (static_cast<int>(blockIdx.x) >= *num_tiles) return;
  const int4 t = tiles[blockIdx.x];
  if (t.w < 0) return;
  const int nblk = kp / kNvBlock;
  const float pts = nv_tensor_scale(amax[t.w]);
  const bool vec = (cols % 8) == 0 && (ld % 8) == 0 && (reinterpret_cast<uintptr_t>(src) & 15u) == 0;
  const int lane = threadIdx.x & 31;
  for (int r = threadIdx.x >> 5; r < t.z; r += blockDim.x >> 5) {
    const int64_t p = t.y + r;
    const int64_t srow = gather != nullptr ? gather[p] : p;
    const uint16_t* row = src + srow * ld;
    for (int blk = lane; blk < nblk; blk += 32)
      quantize_block(row, cols, vec, blk, pts, q + p * (kp / 2), sf + p * nblk);
  }
}

// Per group: amax over its `per_group` elements (grid.y = groups).
__global__ void nv_group_amax_kernel(const uint16_t* __restrict__ src, int64_t per_group, float* __restrict__ amax,
                                     int stride, int off) {
  const uint16_t* g = src + static_cast<int64_t>(blockIdx.y) * per_group;
  float m = 0.0f;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < per_group;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    m = fmaxf(m, fabsf(bf16_to_f32(g[i])));
  m = block_max(m);
  if (threadIdx.x == 0) atomic_max_nonneg(amax + static_cast<int64_t>(blockIdx.y) * stride + off, m);
}

// One thread per (group, row, 16-element block).  Pack time only.
__global__ void nv_quantize_b_kernel(MxBSource s, int groups, int rows_per_group, int kp, int tile_rows,
                                     const float* __restrict__ amax, uint8_t* __restrict__ q,
                                     uint8_t* __restrict__ atoms) {
  const int nblk = kp / kNvBlock;
  const int stages = kp / 256;
  const int tiles = (rows_per_group + tile_rows - 1) / tile_rows;
  const int per_tile = (tile_rows + 127) / 128;
  const int64_t total = static_cast<int64_t>(groups) * rows_per_group * nblk;
  for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int blk = static_cast<int>(idx % nblk);
    const int64_t rg = idx / nblk;
    const int row = static_cast<int>(rg % rows_per_group);
    const int g = static_cast<int>(rg / rows_per_group);
    int proj = 0;
    if (s.mode == kMxSrcW1) proj = (row % (2 * s.chunk)) / s.chunk;
    else if (s.mode == kMxSrcW2) proj = 2;
    const float pts = nv_tensor_scale(amax[static_cast<int64_t>(g) * 4 + proj]);
    float v[16];
#pragma unroll 4
    for (int j = 0; j < 16; ++j) v[j] = mx_b_elem(s, g, row, blk * kNvBlock + j);
    uint32_t w0, w1;
    const uint32_t sb = nv_quantize16(v, pts, w0, w1);
    *reinterpret_cast<uint2*>(q + (static_cast<int64_t>(g) * rows_per_group + row) * (kp / 2) + blk * 8) =
        make_uint2(w0, w1);
    const int tile = row / tile_rows, r = row - tile * tile_rows;
    const int stage = blk / 16, mma = (blk / 4) & 3;
    const int64_t atom =
        (((static_cast<int64_t>(g) * tiles + tile) * stages + stage) * 4 + mma) * per_tile + (r >> 7);
    atoms[atom * kMxAtomBytes + mx_atom_offset(r & 127, blk & 3)] = static_cast<uint8_t>(sb);
  }
}

size_t nv_atoms_bytes(int groups, int rows_per_group, int kp, int tile_rows) {
  const int tiles = (rows_per_group + tile_rows - 1) / tile_rows;
  const int per_tile = (tile_rows + 127) / 128;
  return static_cast<size_t>(groups) * tiles * (kp / 256) * 4 * per_tile * kMxAtomBytes;
}

int launch_nv_amax(const uint16_t* src, int64_t rows, int cols, int64_t ld, float* amax, cudaStream_t stream) {
  if (rows <= 0 || cols <= 0) return SPX_OK;
  nv_amax_kernel<<<nv_grid(rows * cols, 256), 256, 0, stream>>>(src, rows, cols, ld, amax);
  return cudaGetLastError() == cudaSuccess ? SPX_OK : SPX_ERR_CUDA;
}

int launch_nv_row_amax(const uint16_t* src, int64_t rows, int cols, int64_t ld, float* row_amax,
                       cudaStream_t stream) {
  if (rows <= 0) return SPX_OK;
  nv_row_amax_kernel<<<nv_grid(rows * 32, 256), 256, 0, stream>>>(src, rows, cols, ld, row_amax);
  return cudaGetLastError() == cudaSuccess ? SPX_OK : SPX_ERR_CUDA;
}

int launch_nv_tile_amax(const int4* tiles, const int* num_tiles, int max_tiles, const int* gather,
                        const float* row_amax, float* amax, cudaStream_t stream) {
  if (max_tiles <= 0) return SPX_OK;
  nv_tile_amax_kernel<<<max_tiles, kTileRows, 0, stream>>>(tiles, num_tiles, gather, row_amax, amax);
  return cudaGetLastError() == cudaSuccess ? SPX_OK : SPX_ERR_CUDA;
}

int launch_nv_quantize_rows(const uint16_t* src, int64_t rows, int cols, int64_t ld, const float* amax, int kp,
                            uint8_t* q, uint8_t* sf, cudaStream_t stream) {
  if (rows <= 0) return SPX_OK;
  if (kp % 256 != 0 || cols > kp) return SPX_ERR_INVALID_ARG;
  nv_quantize_rows_kernel<<<nv_grid(rows * (kp / kNvBlock), 256), 256, 0, stream>>>(src, rows, cols, ld, amax, kp,
                                                                                      q, sf);
  return cudaGetLastError() == cudaSuccess ? SPX_OK : SPX_ERR_CUDA;
}

int launch_nv_quantize_tiles(const int4* tiles, const int* num_tiles, int max_tiles, const uint16_t* src,
                             int64_t ld, int cols, const int* gather, const float* amax, int kp, uint8_t* q,
                             uint8_t* sf, cudaStream_t stream) {
  if (max_tiles <= 0) return SPX_OK;
  if (kp % 256 != 0 || cols > kp) return SPX_ERR_INVALID_ARG;
  nv_quantize_tiles_kernel<<<max_tiles, 256, 0, stream>>>(tiles, num_tiles, src, ld, cols, gather, amax, kp, q, sf);
  return cudaGetLastError() == cudaSuccess ? SPX_OK : SPX_ERR_CUDA;
}

int launch_nv_group_amax(const uint16_t* src, int groups, int64_t per_group, float* amax, int stride, int off,
                         cudaStream_t stream) {
  if (groups <= 0 || per_group <= 0) return SPX_OK;
  int64_t bx = (per_group + 255) / 256;
  if (bx > 64) bx = 64;
  nv_group_amax_kernel<<<dim3(static_cast<unsigned>(bx), static_cast<unsigned>(groups)), 256, 0, stream>>>(
      src, per_group, amax, stride, off);
  return cudaGetLastError() == cudaSuccess ? SPX_OK : SPX_ERR_CUDA;
}

int launch_nv_quantize_b(int mode, const uint16_t* a, const uint16_t* b, int groups, int rows_per_group,
                         int rows_real, int k_real, int kp, int tile_rows, int d, int inter, int chunk, int64_t ld,
                         const float* amax, uint8_t* q, uint8_t* atoms, cudaStream_t stream) {
  if (groups <= 0 || rows_per_group <= 0) return SPX_OK;
  if (kp % 256 != 0 || tile_rows < 16 || tile_rows > kMxMaxBn) return SPX_ERR_INVALID_ARG;
  if (cudaMemsetAsync(atoms, 0, nv_atoms_bytes(groups, rows_per_group, kp, tile_rows), stream) != cudaSuccess)
    return SPX_ERR_CUDA;
  MxBSource s{};
  s.mode = mode;
  s.a = a;
  s.b = b;
  s.d = d;
  s.inter = inter;
  s.chunk = chunk;
  s.ld = ld;
  s.k_real = k_real;
  s.rows_real = rows_real;
  const int64_t total = static_cast<int64_t>(groups) * rows_per_group * (kp / kNvBlock);
  nv_quantize_b_kernel<<<nv_grid(total, 256), 256, 0, stream>>>(s, groups, rows_per_group, kp, tile_rows, amax, q,
                                                                   atoms);
  return cudaGetLastError() == cudaSuccess ? SPX_OK : SPX_ERR_CUDA;
}

}  // namespace spx
