// MXFP8 quantisers (E4M3 values, E8M0 scales per 1x32 block along K).
//
//  * rows:  BF16 activations [rows, cols] -> E4M3 [rows, kp] (K zero-padded
//           to kp) + scale bytes [rows, kp/32] row-major.  Used online for the
//           hidden states of MXFP8 experts and for the left operand of the
//           dense MXFP8 matmul (experts/native.py:113-140 quantises both
//           operands of `left @ right_rows.T` row-wise along K).
//  * B operands (weights, pack time): E4M3 [groups, rows, kp] and the scales
//           rearranged into the 512-byte atoms the GEMM copies into tensor
//           memory, [groups][row tiles][kp/128][ceil(tile rows/128)][512].  Rows come from the
//           reference layouts directly: expert gate/up [E, d, I] (row = output
//           channel i, K = d, rows in the chunked [gate | up] order of the
//           GEMM1 tiles), expert down [E, I, d] (row = output column n, K = I),
//           or a plain row-major matrix.
// Padding (K beyond the real width, rows beyond the real count) quantises to
// zero with scale byte 0, the same as the reference's zero padding.
#include <cuda_runtime.h>
#include <stdint.h>

#include "kernels.h"
#include "mx.cuh"
#include "sm100.cuh"

namespace spx {

namespace {

int grid_for(int64_t total, int threads) {
  int64_t g = (total + threads - 1) / threads;
  if (g > 148 * 64) g = 148 * 64;
  return static_cast<int>(g < 1 ? 1 : g);
}

__device__ __forceinline__ void store32(uint8_t* dst, const uint32_t (&q)[8]) {
  if ((reinterpret_cast<uintptr_t>(dst) & 15u) == 0) {
    reinterpret_cast<uint4*>(dst)[0] = make_uint4(q[0], q[1], q[2], q[3]);
    reinterpret_cast<uint4*>(dst)[1] = make_uint4(q[4], q[5], q[6], q[7]);
  } else {
    for (int j = 0; j < 32; ++j) dst[j] = static_cast<uint8_t>(q[j >> 2] >> (8 * (j & 3)));
  }
}

}  // namespace

// One thread per (row, 32-element block); blocks of a row are consecutive
// threads, so a warp reads 2 KB of contiguous BF16.
__global__ void mx_quantize_rows_kernel(const uint16_t* __restrict__ src, int64_t rows, int cols, int64_t ld_src,
                                        int kp, uint8_t* __restrict__ q, int64_t ld_q, uint8_t* __restrict__ sf,
                                        int64_t ld_sf) {
  const int nblk = kp / kMxBlock;
  const int64_t total = rows * nblk;
  const bool vec = (cols % 8) == 0 && (ld_src % 8) == 0 && (reinterpret_cast<uintptr_t>(src) & 15u) == 0;
  griddep_wait();
  griddep_launch_dependents();
  for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = idx / nblk;
    const int blk = static_cast<int>(idx - row * nblk);
    const int c0 = blk * kMxBlock;
    const uint16_t* s = src + row * ld_src + c0;
    float v[32];
    if (vec && c0 + kMxBlock <= cols) {
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const uint4 u = __ldg(reinterpret_cast<const uint4*>(s) + w);
        const uint32_t words[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          v[8 * w + 2 * h] = __uint_as_float(words[h] << 16);
          v[8 * w + 2 * h + 1] = __uint_as_float(words[h] & 0xFFFF0000u);
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = (c0 + j < cols) ? bf16_to_f32(s[j]) : 0.0f;
    }
    uint32_t qw[8];
    const uint32_t sb = mx_quantize32(v, qw);
    store32(q + row * ld_q + c0, qw);
    sf[row * ld_sf + blk] = static_cast<uint8_t>(sb);
  }
}

// One thread per (group, row, 32-element block).  Pack time only.
__global__ void mx_quantize_b_kernel(MxBSource s, int groups, int rows_per_group, int kp, int tile_rows,
                                     uint8_t* __restrict__ q, uint8_t* __restrict__ atoms) {
  const int nblk = kp / kMxBlock;
  const int kblocks = kp / 128;
  const int tiles = (rows_per_group + tile_rows - 1) / tile_rows;
  const int64_t total = static_cast<int64_t>(groups) * rows_per_group * nblk;
  for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int blk = static_cast<int>(idx % nblk);
    const int64_t rg = idx / nblk;
    const int row = static_cast<int>(rg % rows_per_group);
    const int g = static_cast<int>(rg / rows_per_group);
    float v[32];
#pragma unroll 4
    for (int j = 0; j < 32; ++j) v[j] = mx_b_elem(s, g, row, blk * kMxBlock + j);
    uint32_t qw[8];
    const uint32_t sb = mx_quantize32(v, qw);
    store32(q + (static_cast<int64_t>(g) * rows_per_group + row) * kp + blk * kMxBlock, qw);
    const int tile = row / tile_rows, r = row - tile * tile_rows;
    const int per_tile = (tile_rows + 127) / 128;
    const int64_t atom = ((static_cast<int64_t>(g) * tiles + tile) * kblocks + (blk >> 2)) * per_tile + (r >> 7);
    atoms[atom * kMxAtomBytes + mx_atom_offset(r & 127, blk & 3)] = static_cast<uint8_t>(sb);
  }
}

int launch_mx_quantize_rows(const uint16_t* src, int64_t rows, int cols, int64_t ld_src, int kp, uint8_t* q,
                            int64_t ld_q, uint8_t* sf, int64_t ld_sf, cudaStream_t stream) {
  if (rows <= 0) return SPX_OK;
  if (kp % kMxBlock != 0 || cols > kp || ld_q < kp || ld_sf < kp / kMxBlock) return SPX_ERR_INVALID_ARG;
  const int64_t total = rows * (kp / kMxBlock);
  return launch_pdl(mx_quantize_rows_kernel, dim3(grid_for(total, 256)), dim3(256), 0, stream, src, rows, cols, ld_src,
                    kp, q, ld_q, sf, ld_sf);
}

size_t mx_atoms_bytes(int groups, int rows_per_group, int kp, int tile_rows) {
  const int tiles = (rows_per_group + tile_rows - 1) / tile_rows;
  const int per_tile = (tile_rows + 127) / 128;
  return static_cast<size_t>(groups) * tiles * (kp / 128) * per_tile * kMxAtomBytes;
}

int launch_mx_quantize_b(int mode, const uint16_t* a, const uint16_t* b, int groups, int rows_per_group,
                         int rows_real, int k_real, int kp, int tile_rows, int d, int inter, int chunk, int64_t ld,
                         uint8_t* q, uint8_t* atoms, cudaStream_t stream) {
  if (groups <= 0 || rows_per_group <= 0) return SPX_OK;
  if (kp % 128 != 0 || tile_rows < 16 || tile_rows > kMxMaxBn) return SPX_ERR_INVALID_ARG;
  if (cudaMemsetAsync(atoms, 0, mx_atoms_bytes(groups, rows_per_group, kp, tile_rows), stream) != cudaSuccess)
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
  const int64_t total = static_cast<int64_t>(groups) * rows_per_group * (kp / kMxBlock);
  mx_quantize_b_kernel<<<grid_for(total, 256), 256, 0, stream>>>(s, groups, rows_per_group, kp, tile_rows, q, atoms);
  return cudaGetLastError() == cudaSuccess ? SPX_OK : SPX_ERR_CUDA;
}

}  // namespace spx
