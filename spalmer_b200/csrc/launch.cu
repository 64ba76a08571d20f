// Host-side launch helpers shared by the kernels: cached per-device queries.
#include <cuda_runtime.h>

#include <map>
#include <mutex>
#include <utility>

#include "kernels.h"

namespace spx {
namespace {

constexpr int kMaxDevices = 64;
constexpr int kMaxFuncs = 64;

std::mutex g_mu;
int g_sm_count[kMaxDevices] = {};
const void* g_func[kMaxDevices][kMaxFuncs] = {};

int current_device() {
  int dev = 0;
  return cudaGetDevice(&dev) == cudaSuccess && dev >= 0 && dev < kMaxDevices ? dev : -1;
}

}  // namespace

int device_sm_count() {
  const int dev = current_device();
  if (dev < 0) return 148;
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_sm_count[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    g_sm_count[dev] = n;
  }
  return g_sm_count[dev];
}

// Side streams: a pool of kSidePool non-blocking streams (three events each)
// per device, created on the first call on the device that is not being
// captured and kept for the life of the process.  A caller stream takes the
// next pool entry the first time it forks, which needs no creation, so a
// stream first seen inside a capture (torch.cuda.graph captures on a stream
// of its own) still forks.  Work forked onto the side stream joins the caller's
// stream through the events, so the pair behaves as one stream to the caller,
// CUDA graph capture included.  Past kSidePool caller streams, entries are
// shared: their side work serialises on one stream (still correct, joined by
// events), and a stream that one thread captures must not also run another
// thread's eager side work.
namespace {
constexpr int kSidePool = 4;
struct SidePool {
  SideStream entry[kSidePool];
  int next = 0;
};
std::map<int, SidePool> g_pool;
std::map<std::pair<int, cudaStream_t>, int> g_side;

bool make_pool(int dev, SidePool* pool) {
  int lo = 0, hi = 0;
  if (cudaDeviceGetStreamPriorityRange(&lo, &hi) != cudaSuccess) lo = hi = 0;
  for (int i = 0; i < kSidePool; ++i) {
    SideStream& s = pool->entry[i];
    // the highest priority: side work is short and sits beside the critical path
    if (cudaStreamCreateWithPriority(&s.side, cudaStreamNonBlocking, hi) != cudaSuccess ||
        cudaEventCreateWithFlags(&s.fork, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&s.join, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&s.join2, cudaEventDisableTiming) != cudaSuccess) {
      cudaGetLastError();
      return false;
    }
  }
  (void)dev;
  return true;
}
}  // namespace

bool side_stream(cudaStream_t main, SideStream* out) {
  const int dev = current_device();
  if (dev < 0) return false;
  std::lock_guard<std::mutex> lock(g_mu);
  auto pool_it = g_pool.find(dev);
  if (pool_it == g_pool.end()) {
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(main, &cap) != cudaSuccess || cap != cudaStreamCaptureStatusNone) {
      cudaGetLastError();
      return false;  // create nothing inside a capture: the caller runs unforked
    }
    SidePool pool;
    if (!make_pool(dev, &pool)) return false;
    pool_it = g_pool.emplace(dev, pool).first;
  }
  const auto key = std::make_pair(dev, main);
  auto it = g_side.find(key);
  int index;
  if (it != g_side.end()) {
    index = it->second;
  } else {
    index = pool_it->second.next;
    pool_it->second.next = (index + 1) % kSidePool;
    g_side.emplace(key, index);
  }
  *out = pool_it->second.entry[index];
  return true;
}

int ensure_max_dynamic_smem(const void* func) {
  const int dev = current_device();
  if (dev < 0) return SPX_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_mu);
  for (int i = 0; i < kMaxFuncs; ++i) {
    if (g_func[dev][i] == func) return SPX_OK;
    if (g_func[dev][i] == nullptr) {
      int optin = 0;
      cudaFuncAttributes attr{};
      if (cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess ||
          cudaFuncGetAttributes(&attr, func) != cudaSuccess) {
        cudaGetLastError();  // clear, so later launch checks do not see it
        return SPX_ERR_CUDA;
      }
      // The opt-in limit covers static and dynamic shared memory together.
      const int dyn = optin - static_cast<int>(attr.sharedSizeBytes);
      if (cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, dyn) != cudaSuccess) {
        cudaGetLastError();
        return SPX_ERR_CUDA;
      }
      g_func[dev][i] = func;
      return SPX_OK;
    }
  }
  return SPX_ERR_UNSUPPORTED;
}

int device_max_pairs(const void* func, size_t smem) {
  const int fallback = device_sm_count() / 2;
  const int dev = current_device();
  if (dev < 0) return fallback;
  static const void* cached_func[kMaxDevices][kMaxFuncs] = {};
  static size_t cached_smem[kMaxDevices][kMaxFuncs] = {};
  static int cached_pairs[kMaxDevices][kMaxFuncs] = {};
  std::lock_guard<std::mutex> lock(g_mu);
  int slot = -1;
  for (int i = 0; i < kMaxFuncs; ++i) {
    if (cached_func[dev][i] == func && cached_smem[dev][i] == smem) return cached_pairs[dev][i];
    if (cached_func[dev][i] == nullptr) {
      slot = i;
      break;
    }
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(2 * static_cast<unsigned>(fallback > 0 ? fallback : 1), 1, 1);
  cfg.blockDim = dim3(kGemmThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr{};
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = 2;
  attr.val.clusterDim.y = 1;
  attr.val.clusterDim.z = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  int clusters = 0;
  if (cudaOccupancyMaxActiveClusters(&clusters, func, &cfg) != cudaSuccess || clusters <= 0) {
    cudaGetLastError();
    clusters = fallback;
  }
  if (slot >= 0) {
    cached_func[dev][slot] = func;
    cached_smem[dev][slot] = smem;
    cached_pairs[dev][slot] = clusters;
  }
  return clusters;
}

}  // namespace spx
