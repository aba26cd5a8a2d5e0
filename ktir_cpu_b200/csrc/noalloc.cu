// Allocation-free variant of the indirect gather -> f -> scatter entry point.
//
// ktir_gather_rmw() needs an int32 count per table row as scratch, which its
// caller allocates.  Some callers cannot allocate device memory at all: code
// running inside a CUDA graph that is being captured or replayed by a host
// framework that forbids allocation, or an embedding that only hands this
// library the tensors it must read and write.  For them the scratch lives in
// a file-scope __device__ array of fixed size, created when the library is
// loaded and held by every GPU that loads it until the process exits.
#include <cuda_runtime.h>
#include <mutex>

#include "../../include/ktir_b200.h"

int ktir_set_error(int code, const char* msg);

namespace {

constexpr int64_t kMaxRows = KTIR_STATIC_RMW_MAX_ROWS;
constexpr int kMaxDevices = 64;

// One count per table row; only host code needs its address.
static __device__ __align__(256) int32_t g_rmw_counts[kMaxRows];

int32_t* g_counts_addr[kMaxDevices] = {nullptr};
std::mutex g_lock;

}  // namespace

extern "C" int ktir_gather_rmw(const KtirGatherRmwDesc* desc, const KtirBuffers* bufs,
                               int32_t* counts, int64_t n_rows, int32_t* status, void* stream);

extern "C" int ktir_gather_rmw_static(const KtirGatherRmwDesc* desc, const KtirBuffers* bufs,
                                      int64_t n_rows, int32_t* status, void* stream) {
  if (!desc || !bufs || !status)
    return ktir_set_error(KTIR_ERR_ARG, "ktir_gather_rmw_static: null argument");
  if (n_rows < 0 || n_rows > kMaxRows)
    return ktir_set_error(KTIR_ERR_UNSUPPORTED,
                          "ktir_gather_rmw_static: n_rows outside [0, KTIR_STATIC_RMW_MAX_ROWS]");
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return ktir_set_error(KTIR_ERR_CUDA, "ktir_gather_rmw_static: no usable current device");
  int32_t* counts;
  {
    // set-up, once per device, with that device current
    std::lock_guard<std::mutex> guard(g_lock);
    if (!g_counts_addr[dev]) {
      void* p = nullptr;
      cudaError_t e = cudaGetSymbolAddress(&p, g_rmw_counts);
      if (e != cudaSuccess || p == nullptr)
        return ktir_set_error(KTIR_ERR_CUDA, "ktir_gather_rmw_static: cudaGetSymbolAddress failed");
      g_counts_addr[dev] = static_cast<int32_t*>(p);
    }
    counts = g_counts_addr[dev];
  }
  // The array keeps the previous call's contents.  The count pass needs them
  // at zero; an apply-only call (phases == 2) consumes the counts that its
  // count-only call (phases == 1) left, so it must not clear them.
  const bool do_count = desc->phases == 0 || (desc->phases & 1);
  if (do_count && n_rows > 0 &&
      cudaMemsetAsync(counts, 0, (size_t)n_rows * sizeof(int32_t), (cudaStream_t)stream) != cudaSuccess)
    return ktir_set_error(KTIR_ERR_CUDA, "ktir_gather_rmw_static: clearing the counts failed");
  return ktir_gather_rmw(desc, bufs, counts, n_rows, status, stream);
}
