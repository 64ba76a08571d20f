// spx_dispatch_static: the dispatch counting sort with its scratch memory in a
// file-scope device array instead of a caller-provided workspace.
//
// Some callers cannot allocate device memory at all: a plain C / FFI client
// that holds only the buffers it was handed and has no device allocator of
// its own, or code running where a cudaMalloc is not allowed or would
// synchronise the device (CUDA stream capture in global mode, a serving loop
// with a fixed memory plan).  This entry point needs nothing from them but the
// input ids and the two output buffers; it calls no cudaMalloc/cudaFree and no
// allocating library routine.
//
// The scratch lives in `g_dispatch_scratch` below (kStaticScratchBytes, about
// 6.2 MiB).  Every GPU that loads libspx holds that array until the process
// exits.  Host code cannot use the array's name as a device address, so the
// first call on each device (with that device current) looks the address up
// with cudaGetSymbolAddress and caches it; make that first call before any
// stream capture.  The cached address is kept for the life of the process and
// is not refreshed after cudaDeviceReset.  The stream must belong to the
// current device (checked).  All calls share the one array and it keeps the
// previous call's contents: everything a call reads is rewritten by the same
// call, and the status word is cleared at the start of every call.  Calls
// whose kernels overlap on the GPU (different streams, no ordering) race on
// the array — serialise them.  spx_dispatch_static_status reads the status
// word the kernels leave (an expert id out of range, a malformed tile).
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "kernels.h"
#include "sm100.cuh"

namespace spx {
namespace {

constexpr int64_t kStaticMaxPairs = int64_t(1) << 20;  // T * k
constexpr int kStaticMaxExperts = 1024;
constexpr int kStaticMaxChunks = static_cast<int>(kStaticMaxPairs / kDispatchChunk);
constexpr int kStaticMaxTiles = static_cast<int>(kStaticMaxPairs / kTileRows) + kStaticMaxExperts;

constexpr size_t align256(size_t v) { return (v + 255) / 256 * 256; }

// Layout of the static scratch (byte offsets).
constexpr size_t kOffSmall = 0;  // [0] status, [2] num_tiles
constexpr size_t kOffHist = align256(kOffSmall + 64);
constexpr size_t kOffStarts = align256(kOffHist + sizeof(int) * size_t(kStaticMaxChunks) * kStaticMaxExperts);
constexpr size_t kOffTiles = align256(kOffStarts + sizeof(int) * size_t(kStaticMaxExperts));
constexpr size_t kOffSrcRow = align256(kOffTiles + sizeof(int4) * size_t(kStaticMaxTiles));
constexpr size_t kStaticScratchBytes = align256(kOffSrcRow + sizeof(int) * size_t(kStaticMaxPairs));

constexpr int kMaxDevices = 64;

}  // namespace
}  // namespace spx

// File-scope scratch of spx_dispatch_static (see the header comment).
static __device__ __align__(256) unsigned char g_dispatch_scratch[spx::kStaticScratchBytes];

namespace spx {
namespace {

std::mutex g_scratch_mutex;
void* g_scratch_addr[kMaxDevices] = {};

// Device address of g_dispatch_scratch on the current device (looked up once per device).
int static_scratch(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return SPX_ERR_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return SPX_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (g_scratch_addr[dev] == nullptr) {
    void* addr = nullptr;
    if (cudaGetSymbolAddress(&addr, g_dispatch_scratch) != cudaSuccess || addr == nullptr) return SPX_ERR_CUDA;
    g_scratch_addr[dev] = addr;
  }
  *out = g_scratch_addr[dev];
  return SPX_OK;
}

// The stream (NULL = the current device's legacy stream) must belong to the current device.
int check_stream_device(cudaStream_t st) {
  if (st == nullptr) return SPX_OK;
  int cur = 0, dev = 0;
  if (cudaGetDevice(&cur) != cudaSuccess) return SPX_ERR_CUDA;
  if (cudaStreamGetDevice(st, &dev) != cudaSuccess) return SPX_ERR_CUDA;
  return dev == cur ? SPX_OK : SPX_ERR_INVALID_ARG;
}

}  // namespace
}  // namespace spx

extern "C" int spx_dispatch_static_status(int* device_status, int clear, void* stream) {
  using namespace spx;
  if (device_status == nullptr) return SPX_ERR_INVALID_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (int rc = check_stream_device(st); rc != SPX_OK) return rc;
  void* base = nullptr;
  if (int rc = static_scratch(&base); rc != SPX_OK) return rc;
  int* word = reinterpret_cast<int*>(static_cast<uint8_t*>(base) + kOffSmall);
  int v = 0;
  if (cudaMemcpyAsync(&v, word, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess) return SPX_ERR_CUDA;
  if (cudaStreamSynchronize(st) != cudaSuccess) return SPX_ERR_CUDA;
  *device_status = v;
  if (clear && v != 0 && cudaMemsetAsync(word, 0, sizeof(int), st) != cudaSuccess) return SPX_ERR_CUDA;
  return SPX_OK;
}

extern "C" int spx_dispatch_static(const spx_layer_dims* dims, const int64_t* expert_ids, int32_t* order,
                                   int32_t* counts, void* stream) {
  using namespace spx;
  if (dims == nullptr || expert_ids == nullptr || order == nullptr || counts == nullptr) return SPX_ERR_INVALID_ARG;
  const int64_t tokens = dims->tokens;
  const int k = dims->top_k;
  const int experts = dims->num_experts;
  if (tokens < 1 || k < 1 || experts < 1 || k > experts) return SPX_ERR_INVALID_ARG;
  if (tokens * k > kStaticMaxPairs || experts > kStaticMaxExperts) return SPX_ERR_SCRATCH_LIMIT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (int rc = check_stream_device(st); rc != SPX_OK) return rc;
  void* base = nullptr;
  if (int rc = static_scratch(&base); rc != SPX_OK) return rc;
  uint8_t* s = static_cast<uint8_t*>(base);
  int* small = reinterpret_cast<int*>(s + kOffSmall);
  if (cudaMemsetAsync(small, 0, 64, st) != cudaSuccess) return SPX_ERR_CUDA;
  DispatchArgs a{};
  a.ids = expert_ids;
  a.pairs = tokens * k;
  a.tokens = tokens;
  a.num_experts = experts;
  a.top_k = k;
  a.chunk_hist = reinterpret_cast<int*>(s + kOffHist);
  a.counts = counts;
  a.starts = reinterpret_cast<int*>(s + kOffStarts);
  a.tiles = reinterpret_cast<int4*>(s + kOffTiles);
  a.num_tiles = small + 2;
  a.order = order;
  a.src_row = reinterpret_cast<int*>(s + kOffSrcRow);
  a.lb_blocks = 0;
  a.eligible_experts = experts;
  a.execution_loop = dims->execution_loop;
  a.status = small;
  return launch_dispatch(a, st);
}
