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

namespace {

constexpr int64_t kMaxRows = KTIR_STATIC_RMW_MAX_ROWS;
constexpr int kMaxDevices = 64;

// One count per table row; only host code needs its address.
static __device__ __align__(256) int32_t g_rmw_counts[kMaxRows];

int32_t* g_counts_addr[kMaxDevices] = {nullptr};
std::mutex g_lock;
thread_local char g_msg[256];

}  // namespace

extern "C" int ktir_gather_rmw(const KtirGatherRmwDesc* desc, const KtirBuffers* bufs,
                               int32_t* counts, int64_t n_rows, int32_t* status, void* stream);

extern "C" int ktir_gather_rmw_static(const KtirGatherRmwDesc* desc, const KtirBuffers* bufs,
                                      int64_t n_rows, int32_t* status, void* stream) {
  if (!desc || !bufs || !status) return KTIR_ERR_ARG;
  if (n_rows < 0 || n_rows > kMaxRows) return KTIR_ERR_UNSUPPORTED;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return KTIR_ERR_CUDA;
  int32_t* counts;
  {
    // set-up, once per device, with that device current
    std::lock_guard<std::mutex> guard(g_lock);
    if (!g_counts_addr[dev]) {
      void* p = nullptr;
      cudaError_t e = cudaGetSymbolAddress(&p, g_rmw_counts);
      if (e != cudaSuccess || p == nullptr) return KTIR_ERR_CUDA;
      g_counts_addr[dev] = static_cast<int32_t*>(p);
    }
    counts = g_counts_addr[dev];
  }
  // the array keeps the previous call's contents: the counts must start at zero
  if (n_rows > 0 &&
      cudaMemsetAsync(counts, 0, (size_t)n_rows * sizeof(int32_t), (cudaStream_t)stream) != cudaSuccess)
    return KTIR_ERR_CUDA;
  return ktir_gather_rmw(desc, bufs, counts, n_rows, status, stream);
}
