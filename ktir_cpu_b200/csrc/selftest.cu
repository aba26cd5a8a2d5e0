// Bounded-wait self test: one thread waits on an mbarrier that nothing ever
// arrives at, using the same bounded wait as the tensor-core kernels, and
// must come back with KTIR_STATUS_TIMEOUT instead of hanging.
#include <cuda_runtime.h>

#include "../../include/ktir_b200.h"
#include "tc_common.cuh"

using namespace ktir::tc;

__global__ void k_wait_selftest(int* status, unsigned spin_limit) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x != 0) return;
  const uint32_t b = smem_u32(&bar);
  mbar_init(b, 1);
  fence_barrier_init();
  bool done = false;
  for (unsigned i = 0; i < spin_limit && !done; ++i) done = mbar_try_wait(b, 0);
  if (!done) atomicOr(status, KTIR_STATUS_TIMEOUT);
  asm volatile("mbarrier.inval.shared::cta.b64 [%0];" ::"r"(b) : "memory");
}

extern "C" int ktir_wait_selftest(int32_t* status, uint32_t spin_limit, void* stream) {
  if (!status || spin_limit == 0 || spin_limit > (1u << 20)) return KTIR_ERR_ARG;
  k_wait_selftest<<<1, 32, 0, (cudaStream_t)stream>>>(status, spin_limit);
  return cudaGetLastError() == cudaSuccess ? KTIR_OK : KTIR_ERR_CUDA;
}
