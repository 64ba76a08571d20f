// Expert-parallel row exchange over peer memory (NVLink / NVSwitch).
//
// Every rank allocates its exchange buffers with cudaMalloc and shares CUDA
// IPC handles; the others open them as peer pointers.  A row exchange is
// then one kernel on the sending GPU that stores each row straight into the
// destination GPU's buffer, replacing an all-to-all-v and its staging copy:
// the dispatch gather writes the hidden-state rows of every routed pair into
// the receive buffers of the experts' ranks, and the expert outputs go back
// into the senders' buffers in their dispatch order.  Ordering across GPUs
// is the caller's: a stream-ordered collective (the NCCL barrier of the
// exchange) after each kernel; the kernel fences its stores at system scope
// before it ends.
#include <cuda_runtime.h>
#include <stdint.h>

#include "kernels.h"
#include "sm100.cuh"

namespace spx {

// One warp per row: the row's segment (destination) by a scan of the G+1
// segment offsets, then 16-byte stores of the row into the destination.
__global__ void rows_to_peers_kernel(const uint16_t* __restrict__ src, int64_t ld_src, const int* __restrict__ index,
                                     int index_div, int64_t rows, int d, const int64_t* __restrict__ seg,
                                     uint16_t* const* __restrict__ dst, const int64_t* __restrict__ dst_row,
                                     int64_t ld_dst, int groups, bool vec) {
  const int lane = threadIdx.x & 31;
  const int64_t nwarps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5); i < rows; i += nwarps) {
    int g = 0;
    while (g + 1 < groups && i >= seg[g + 1]) ++g;
    const int64_t srow = index != nullptr ? index[i] / index_div : i;
    const uint16_t* s = src + srow * ld_src;
    uint16_t* t = dst[g] + (dst_row[g] + (i - seg[g])) * ld_dst;
    if (vec) {
      const uint4* s4 = reinterpret_cast<const uint4*>(s);
      uint4* t4 = reinterpret_cast<uint4*>(t);
      for (int c = lane; c < d / 8; c += 32) t4[c] = __ldg(s4 + c);
    } else {
      for (int c = lane; c < d; c += 32) t[c] = s[c];
    }
  }
  __threadfence_system();  // the stores reach the peers before the kernel completes
}

int launch_rows_to_peers(const uint16_t* src, int64_t ld_src, const int* index, int index_div, int64_t rows, int d,
                         const int64_t* seg, uint16_t* const* dst, const int64_t* dst_row, int64_t ld_dst,
                         int groups, cudaStream_t stream) {
  if (rows <= 0) return SPX_OK;
  bool vec = (d % 8) == 0 && (ld_src % 8) == 0 && (ld_dst % 8) == 0 && (reinterpret_cast<uintptr_t>(src) & 15u) == 0;
  int64_t blocks = (rows + 7) / 8;
  if (blocks > 148 * 8) blocks = 148 * 8;
  rows_to_peers_kernel<<<static_cast<int>(blocks), 256, 0, stream>>>(src, ld_src, index, index_div, rows, d, seg, dst,
                                                                     dst_row, ld_dst, groups, vec);
  return cudaGetLastError() == cudaSuccess ? SPX_OK : SPX_ERR_CUDA;
}

// Row pointers of the rows a rank receives, taken from its senders' own
// buffers: received row i from sender s (recv_seg[s] <= i < recv_seg[s+1])
// is s's pair at dispatch position send_at[s] + i - recv_seg[s], whose token
// is order_s[pos] / top_k and whose row is rows_s + token * ld.
__global__ void peer_row_pointers_kernel(const int* const* __restrict__ order, const int64_t* __restrict__ send_at,
                                         const int64_t* __restrict__ recv_seg, int groups, int top_k,
                                         const uint16_t* const* __restrict__ src_rows, int64_t ld, int64_t rows,
                                         const uint16_t** __restrict__ out) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < rows;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    int g = 0;
    while (g + 1 < groups && i >= recv_seg[g + 1]) ++g;
    const int64_t pos = send_at[g] + (i - recv_seg[g]);
    const int64_t token = order[g][pos] / top_k;
    out[i] = src_rows[g] + token * ld;
  }
}

int launch_peer_row_pointers(const int* const* order, const int64_t* send_at, const int64_t* recv_seg, int groups,
                             int top_k, const uint16_t* const* src_rows, int64_t ld, int64_t rows,
                             const uint16_t** out, cudaStream_t stream) {
  if (rows <= 0) return SPX_OK;
  int64_t blocks = (rows + 255) / 256;
  if (blocks > 148 * 8) blocks = 148 * 8;
  peer_row_pointers_kernel<<<static_cast<int>(blocks), 256, 0, stream>>>(order, send_at, recv_seg, groups, top_k,
                                                                        src_rows, ld, rows, out);
  return cudaGetLastError() == cudaSuccess ? SPX_OK : SPX_ERR_CUDA;
}

}  // namespace spx
