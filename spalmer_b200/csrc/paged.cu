// Paged expert execution: the tile tables of one page.
//
// mESmaC/spalmer experts/bank.py:821-899 (`_execute_paged_grouped`) runs the
// grouped executor page by page, staging each page's expert weights into a
// bounded device cache first (offload.py, bank.py:241-365).  Here the
// dispatch builds the full tile tables once per layer; a page keeps the
// tiles whose expert has a cache slot in this page (page_slot[e] >= 0) and
// renames their group to that slot, so the expert GEMMs read the cache.
// Rows stay at their dispatch positions, so the pages together write exactly
// the Y rows one unpaged pass writes and the combine is unchanged.
//
// One 1024-thread CTA per table (BF16 lane, MXFP8 lane): a stable stream
// compaction, 1024 entries per round (ballot + warp-sum scan).
#include <cuda_runtime.h>
#include <stdint.h>

#include "kernels.h"
#include "sm100.cuh"

namespace spx {

__global__ void __launch_bounds__(1024) page_tiles_kernel(const PageTilesArgs a) {
  const bool mx = blockIdx.x == 1;
  const int4* src = mx ? a.tiles_mx : a.tiles;
  int4* dst = mx ? a.out_mx : a.out;
  const int n = *(mx ? a.num_tiles_mx : a.num_tiles);
  __shared__ int warp_incl[32];
  __shared__ int base;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) base = 0;
  __syncthreads();
  for (int i0 = 0; i0 < n; i0 += 1024) {
    const int i = i0 + static_cast<int>(threadIdx.x);
    int4 t = make_int4(0, 0, 0, 0);
    int slot = -1;
    if (i < n) {
      t = src[i];
      if (t.x >= 0 && t.x < a.num_experts) slot = a.page_slot[t.x];
    }
    const bool keep = slot >= 0;
    const unsigned m = __ballot_sync(0xFFFFFFFFu, keep);
    if (lane == 0) warp_incl[warp] = __popc(m);
    __syncthreads();
    if (warp == 0) {
      int v = warp_incl[lane];
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int u = __shfl_up_sync(0xFFFFFFFFu, v, off);
        if (lane >= off) v += u;
      }
      warp_incl[lane] = v;
    }
    __syncthreads();
    const int pos = base + (warp > 0 ? warp_incl[warp - 1] : 0) + __popc(m & ((1u << lane) - 1u));
    if (keep) dst[pos] = make_int4(slot, t.y, t.z, t.w);
    __syncthreads();
    if (threadIdx.x == 0) base += warp_incl[31];
    __syncthreads();
  }
  if (threadIdx.x == 0) *(mx ? a.out_count_mx : a.out_count) = base;
}

int launch_page_tiles(const PageTilesArgs& a, cudaStream_t stream) {
  if (a.tiles == nullptr || a.num_tiles == nullptr || a.page_slot == nullptr || a.out == nullptr ||
      a.out_count == nullptr || a.num_experts < 1)
    return SPX_ERR_INVALID_ARG;
  const bool mx = a.tiles_mx != nullptr;
  if (mx && (a.num_tiles_mx == nullptr || a.out_mx == nullptr || a.out_count_mx == nullptr))
    return SPX_ERR_INVALID_ARG;
  page_tiles_kernel<<<mx ? 2 : 1, 1024, 0, stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? SPX_OK : SPX_ERR_CUDA;
}

// Staging of whole experts into cache slots: for every (expert, slot) pair
// and every packed array a, dst[a][slot] <- src[a][expert] (bytes[a] each).
// The sources are the host bank (page-locked, mapped into the device's
// address space), so the GPU pulls the rows over the host link itself: one
// launch per chunk of experts instead of one DMA copy per expert and array.
// A small persistent grid (a few SMs; the paged expert GEMMs leave those SMs
// free) walks 64 KB segments of the (pair, array) blocks with 512 threads x
// four 16-byte loads in flight each, enough to keep the host link busy.
constexpr int64_t kStageSegBytes = 64 * 1024;

__global__ void __launch_bounds__(512) stage_slots_kernel(const StageSlotsArgs a) {
  int64_t segs[kStageMaxArrays];
  int64_t per_pair = 0;
  for (int i = 0; i < a.arrays; ++i) {
    segs[i] = (a.bytes[i] + kStageSegBytes - 1) / kStageSegBytes;
    per_pair += segs[i];
  }
  const int64_t total = per_pair * a.num_pairs;
  constexpr int kUnroll = 4;
  for (int64_t sg = blockIdx.x; sg < total; sg += gridDim.x) {
    const int pair = static_cast<int>(sg / per_pair);
    int64_t r = sg - pair * per_pair;
    int arr = 0;
    while (arr + 1 < a.arrays && r >= segs[arr]) r -= segs[arr++];
    const int expert = a.pairs[2 * pair];
    const int slot = a.pairs[2 * pair + 1];
    if (expert < 0 || expert >= a.num_experts || slot < 0 || slot >= a.slots) {
      if (threadIdx.x == 0 && r == 0 && arr == 0 && a.status != nullptr) record_error(a.status, SPX_DEV_BAD_TILE);
      continue;
    }
    const int64_t b0 = r * kStageSegBytes;
    const int64_t b1 = b0 + kStageSegBytes < a.bytes[arr] ? b0 + kStageSegBytes : a.bytes[arr];
    const uint4* src = reinterpret_cast<const uint4*>(a.src[arr] + static_cast<int64_t>(expert) * a.bytes[arr] + b0);
    uint4* dst = reinterpret_cast<uint4*>(a.dst[arr] + static_cast<int64_t>(slot) * a.bytes[arr] + b0);
    const int64_t units = (b1 - b0) / 16;
    for (int64_t i0 = threadIdx.x; i0 < units; i0 += static_cast<int64_t>(blockDim.x) * kUnroll) {
      uint4 v[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int64_t i = i0 + static_cast<int64_t>(u) * blockDim.x;
        if (i < units) v[u] = src[i];
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int64_t i = i0 + static_cast<int64_t>(u) * blockDim.x;
        if (i < units) dst[i] = v[u];
      }
    }
  }
}

int launch_stage_slots(StageSlotsArgs a, cudaStream_t stream) {
  if (a.pairs == nullptr || a.num_pairs < 0 || a.arrays < 1 || a.arrays > kStageMaxArrays || a.num_experts < 1 ||
      a.slots < 1 || a.ctas < 0)
    return SPX_ERR_INVALID_ARG;
  if (a.num_pairs == 0) return SPX_OK;
  for (int i = 0; i < a.arrays; ++i) {
    if (a.src[i] == nullptr || a.dst[i] == nullptr || a.bytes[i] <= 0 || a.bytes[i] % 16 != 0)
      return SPX_ERR_INVALID_ARG;
    if ((reinterpret_cast<uintptr_t>(a.src[i]) & 15u) != 0 || (reinterpret_cast<uintptr_t>(a.dst[i]) & 15u) != 0)
      return SPX_ERR_ALIGNMENT;
    // The source must be page-locked host memory mapped for the device (or
    // device memory): translate it, and refuse anything else.
    cudaPointerAttributes attr{};
    if (cudaPointerGetAttributes(&attr, a.src[i]) != cudaSuccess) {
      cudaGetLastError();
      return SPX_ERR_INVALID_ARG;
    }
    if (attr.type == cudaMemoryTypeHost) {
      void* mapped = nullptr;
      if (cudaHostGetDevicePointer(&mapped, const_cast<uint8_t*>(a.src[i]), 0) != cudaSuccess) {
        cudaGetLastError();
        return SPX_ERR_INVALID_ARG;
      }
      a.src[i] = static_cast<const uint8_t*>(mapped);
    } else if (attr.type != cudaMemoryTypeDevice) {
      return SPX_ERR_INVALID_ARG;
    }
  }
  const int ctas = a.ctas > 0 ? a.ctas : 16;
  stage_slots_kernel<<<ctas, 512, 0, stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? SPX_OK : SPX_ERR_CUDA;
}

}  // namespace spx
