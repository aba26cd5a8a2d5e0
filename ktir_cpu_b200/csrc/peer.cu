// Peer memory between the GPUs of one node, one process per GPU.
//
// A split attention call passes K/V shares between the GPUs of an exchange
// group.  Each GPU's staging buffer is allocated here and exported as a CUDA
// IPC handle; the other processes of the group map it (cudaIpcOpenMemHandle)
// and pull the shares they need with the copy engines (cudaMemcpyAsync over
// NVLink), so the SMs stay with the attention kernel.  The processes order
// their copies with 32-bit epoch flags that live in the owners' buffers:
// a one-thread kernel stores a flag with release semantics at system scope
// after the stream's earlier work, and another one-thread kernel polls flags
// with acquire loads, at most spin_limit times (a nanosleep between polls),
// before the stream's later work may start.  A wait that runs out sets
// KTIR_STATUS_TIMEOUT in the caller's status word and returns: the stream goes
// on, and the host raises the error after the call.  Nothing here has a
// counterpart in the reference, whose cores share one host memory.
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include "../../include/ktir_b200.h"

int ktir_set_error(int code, const char* msg);

namespace {

__global__ void k_flag_set(uint32_t* flag, uint32_t value) {
  if (threadIdx.x != 0) return;
  // the stream's earlier kernels and copies are complete before this kernel
  // starts; the release orders their writes before the flag for every GPU
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(flag), "r"(value) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// every flags[i * stride] reaches `value` (compared modulo 2^32, so the epoch
// may wrap), or the poll limit runs out
__global__ void k_flag_wait(const uint32_t* flags, int n, int stride, uint32_t value,
                            uint32_t spin_limit, int32_t* status) {
  if (threadIdx.x != 0) return;
  for (int i = 0; i < n; ++i) {
    const uint32_t* f = flags + (int64_t)i * stride;
    uint32_t spins = 0;
    while ((int32_t)(ld_acquire_sys(f) - value) < 0) {
      if (++spins >= spin_limit) {
        atomicOr(status, KTIR_STATUS_TIMEOUT);
        return;
      }
      __nanosleep(256);
    }
  }
}

}  // namespace

extern "C" int ktir_ipc_alloc(int64_t bytes, void** ptr, void* handle) {
  if (!ptr || !handle || bytes <= 0) return ktir_set_error(KTIR_ERR_ARG, "ktir_ipc_alloc: bad arguments");
  *ptr = nullptr;
  cudaError_t e = cudaMalloc(ptr, (size_t)bytes);
  if (e != cudaSuccess) return ktir_set_error(KTIR_ERR_CUDA, cudaGetErrorString(e));
  // flags and staging start cleared: epoch 0 is "nothing packed, nothing taken"
  e = cudaMemset(*ptr, 0, (size_t)bytes);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, *ptr);
  if (e != cudaSuccess) {
    cudaFree(*ptr);
    *ptr = nullptr;
    return ktir_set_error(KTIR_ERR_CUDA, cudaGetErrorString(e));
  }
  memcpy(handle, &h, sizeof(h));
  return KTIR_OK;
}

extern "C" int ktir_ipc_open(const void* handle, void** ptr) {
  if (!handle || !ptr) return ktir_set_error(KTIR_ERR_ARG, "ktir_ipc_open: bad arguments");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  *ptr = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return ktir_set_error(KTIR_ERR_CUDA, cudaGetErrorString(e));
  return KTIR_OK;
}

extern "C" int ktir_ipc_close(void* ptr) {
  if (!ptr) return KTIR_OK;
  cudaError_t e = cudaIpcCloseMemHandle(ptr);
  return e == cudaSuccess ? KTIR_OK : ktir_set_error(KTIR_ERR_CUDA, cudaGetErrorString(e));
}

extern "C" int ktir_ipc_free(void* ptr) {
  if (!ptr) return KTIR_OK;
  cudaError_t e = cudaFree(ptr);
  return e == cudaSuccess ? KTIR_OK : ktir_set_error(KTIR_ERR_CUDA, cudaGetErrorString(e));
}

extern "C" int ktir_flag_set(uint32_t* flag, uint32_t value, void* stream) {
  if (!flag || (reinterpret_cast<uintptr_t>(flag) & 3))
    return ktir_set_error(KTIR_ERR_ARG, "ktir_flag_set: null or unaligned flag");
  k_flag_set<<<1, 32, 0, (cudaStream_t)stream>>>(flag, value);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? KTIR_OK : ktir_set_error(KTIR_ERR_CUDA, cudaGetErrorString(e));
}

extern "C" int ktir_flag_wait(const uint32_t* flags, int32_t n, int32_t stride, uint32_t value,
                              uint32_t spin_limit, int32_t* status, void* stream) {
  if (!flags || !status || n < 0 || stride < 1 || (reinterpret_cast<uintptr_t>(flags) & 3) ||
      spin_limit == 0 || spin_limit > (1u << 26))
    return ktir_set_error(KTIR_ERR_ARG, "ktir_flag_wait: bad arguments");
  if (n == 0) return KTIR_OK;
  k_flag_wait<<<1, 32, 0, (cudaStream_t)stream>>>(flags, n, stride, value, spin_limit, status);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? KTIR_OK : ktir_set_error(KTIR_ERR_CUDA, cudaGetErrorString(e));
}

extern "C" int ktir_copy_async(void* dst, const void* src, int64_t bytes, void* stream) {
  if (!dst || !src || bytes < 0) return ktir_set_error(KTIR_ERR_ARG, "ktir_copy_async: bad arguments");
  if (bytes == 0) return KTIR_OK;
  cudaError_t e = cudaMemcpyAsync(dst, src, (size_t)bytes, cudaMemcpyDeviceToDevice,
                                  (cudaStream_t)stream);
  return e == cudaSuccess ? KTIR_OK : ktir_set_error(KTIR_ERR_CUDA, cudaGetErrorString(e));
}
