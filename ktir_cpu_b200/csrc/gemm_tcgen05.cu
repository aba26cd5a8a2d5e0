// f16 GEMM on the 5th-generation tensor cores: C = A @ B, f32 accumulation in
// TMEM, f16 result.  Row-major A[M,K], B[K,N], C[M,N] exactly as KTIR views
// lay them out: A is consumed K-major, B is consumed MN-major (no transpose
// pass over B).
//
// Persistent: one CTA per SM walks 128x256 output tiles (tile t, t + grid,
// ...).  The accumulator is double-buffered in TMEM (2 x 256 columns), so the
// epilogue of one tile overlaps the main loop of the next:
//   warp 0      one thread issues TMA loads: A box 64(k) x 128(m), four B
//               boxes 64(n) x 64(k), 128-byte swizzle, into a 4-stage ring
//               that runs continuously across tiles
//   warp 1      allocates 512 TMEM columns; one thread issues tcgen05.mma
//               (M=128, N=256, K=16) four times per 64-wide k step into the
//               tile's accumulator buffer, commits each stage back to the
//               producer and the finished accumulator to the epilogue
//   warps 2..5  epilogue: tcgen05.ld 32 lanes x 32 columns at a time, convert
//               to f16, 128-bit stores; the accumulator buffer is handed back
//               to the MMA warp as soon as the last column is read
// Every wait is bounded (tc_common.cuh); a wait that runs out raises
// KTIR_STATUS_TIMEOUT in the caller's status word instead of hanging.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdio.h>

#include "../../include/ktir_b200.h"
#include "tc_common.cuh"

using namespace ktir::tc;

namespace {

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;            // 16 KiB
constexpr int B_BOX_BYTES = 64 * BK * 2;        // 8 KiB per 64-column box
constexpr int B_BYTES = BK * BN * 2;            // 32 KiB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;  // 48 KiB
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024;
constexpr uint32_t TMEM_COLS = 512;             // two 256-column accumulators

struct GemmParams {
  __half* c;
  long long ldc;
  int m, n, k;
  int add_zero;
  int* status;
};

__global__ void __launch_bounds__(192, 1)
    k_gemm_tcgen05(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb,
                   const __grid_constant__ GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[STAGES];
  __shared__ __align__(8) uint64_t empty_bar[STAGES];
  __shared__ __align__(8) uint64_t acc_full[2];
  __shared__ __align__(8) uint64_t acc_empty[2];
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;

  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t smem = (raw + 1023u) & ~1023u;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int MT = p.m / BM;
  const int n_tiles = MT * (p.n / BN);
  const int KT = p.k / BK;
  volatile int* abort = &abort_flag;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&full_bar[s]), 1);
      mbar_init(smem_u32(&empty_bar[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&acc_full[b]), 1);
      mbar_init(smem_u32(&acc_empty[b]), 128);
    }
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&tmem_base), TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&ta);
      tma_prefetch_desc(&tb);
      uint32_t g = 0;   // k steps issued so far, across tiles
      for (int t = blockIdx.x; t < n_tiles && !*abort; t += gridDim.x) {
        const int m0 = (t % MT) * BM;
        const int n0 = (t / MT) * BN;
        for (int kt = 0; kt < KT; ++kt, ++g) {
          const int s = g % STAGES;
          if (!mbar_wait(smem_u32(&empty_bar[s]), ((g / STAGES) & 1) ^ 1, abort)) break;
          const uint32_t fb = smem_u32(&full_bar[s]);
          mbar_arrive_expect_tx(fb, STAGE_BYTES);
          const uint32_t a_dst = smem + s * STAGE_BYTES;
          const uint32_t b_dst = a_dst + A_BYTES;
          tma_load_2d(a_dst, &ta, fb, kt * BK, m0);
#pragma unroll
          for (int j = 0; j < BN / 64; ++j)
            tma_load_2d(b_dst + j * B_BOX_BYTES, &tb, fb, n0 + 64 * j, kt * BK);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16(BM, BN, 0, 1);
      uint32_t g = 0;
      int i = 0;   // local tile count
      for (int t = blockIdx.x; t < n_tiles && !*abort; t += gridDim.x, ++i) {
        const int b = i & 1;
        // accumulator b was last drained by the epilogue of local tile i - 2
        if (i >= 2 && !mbar_wait(smem_u32(&acc_empty[b]), ((i - 2) >> 1) & 1, abort)) break;
        tc_fence_after();
        const uint32_t acc = tmem + (uint32_t)(b * BN);
        bool ok = true;
        for (int kt = 0; kt < KT; ++kt, ++g) {
          const int s = g % STAGES;
          if (!mbar_wait(smem_u32(&full_bar[s]), (g / STAGES) & 1, abort)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem + s * STAGE_BYTES;
          const uint32_t b_addr = a_addr + A_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            // A: K-major, 16 k = 32 bytes further along each 128-byte row
            const uint64_t ad = sdesc_sw128(a_addr + kk * 32, 16, 1024);
            // B: MN-major, 16 k = 16 rows of 128 bytes further; 64-column
            // groups 8 KiB apart (LBO), 8-row groups 1 KiB apart (SBO)
            const uint64_t bd = sdesc_sw128(b_addr + kk * 16 * 128, B_BOX_BYTES, 1024);
            mma_f16(acc, ad, bd, idesc, (kt | kk) != 0);
          }
          mma_commit(smem_u32(&empty_bar[s]));
        }
        if (!ok) break;
        mma_commit(smem_u32(&acc_full[b]));
      }
    }
  } else {
    // epilogue warps 2..5: warp w reads TMEM lanes 32*(w%4) .. +31
    const int q = warp & 3;
    const int row = 32 * q + lane;
    const float z = p.add_zero ? 0.0f : -0.0f;
    int i = 0;
    for (int t = blockIdx.x; t < n_tiles; t += gridDim.x, ++i) {
      const int b = i & 1;
      const bool ok = mbar_wait(smem_u32(&acc_full[b]), (i >> 1) & 1, abort);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
      const int m0 = (t % MT) * BM;
      const int n0 = (t / MT) * BN;
      __half* crow = p.c + (long long)(m0 + row) * p.ldc + n0;
      const uint32_t acc = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(b * BN);
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        uint32_t r[32];
        tmem_ld32_wait(acc + c, r);
        if (c + 32 == BN) {
          // every column of this accumulator is in registers: hand it back
          tc_fence_before();
          mbar_arrive(smem_u32(&acc_empty[b]));
        }
        __half2 h[16];
#pragma unroll
        for (int j = 0; j < 16; ++j)
          h[j] = __floats2half2_rn(__uint_as_float(r[2 * j]) + z, __uint_as_float(r[2 * j + 1]) + z);
        uint4* dst = reinterpret_cast<uint4*>(crow + c);
        const uint4* src = reinterpret_cast<const uint4*>(h);
#pragma unroll
        for (int j = 0; j < 4; ++j) dst[j] = src[j];
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
  if (threadIdx.x == 0 && abort_flag) atomicOr(p.status, KTIR_STATUS_TIMEOUT);
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

// 2-D f16 row-major tensor [rows, cols] with row stride `ld` elements
bool make_map(CUtensorMap* m, const void* base, long long rows, long long cols, long long ld,
              int box_cols, int box_rows) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box,
             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

thread_local char g_msg[256];

}  // namespace

extern "C" const char* ktir_gemm_error(void) { return g_msg; }

extern "C" int ktir_gemm_f16(const KtirGemmDesc* d, void* stream) {
  if (!d || !d->a || !d->b || !d->c || !d->status) return KTIR_ERR_ARG;
  if (d->m % BM || d->n % BN || d->k % BK || d->k < BK) return KTIR_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(d->a) | reinterpret_cast<uintptr_t>(d->b) |
       reinterpret_cast<uintptr_t>(d->c)) & 15)
    return KTIR_ERR_UNSUPPORTED;
  if ((d->lda | d->ldb | d->ldc) & 7) return KTIR_ERR_UNSUPPORTED;
  CUtensorMap ta, tb;
  if (!make_map(&ta, d->a, d->m, d->k, d->lda, 64, BM) ||
      !make_map(&tb, d->b, d->k, d->n, d->ldb, 64, BK))
    return KTIR_ERR_CUDA;
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(k_gemm_tcgen05, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             SMEM_BYTES) != cudaSuccess)
      return KTIR_ERR_CUDA;
    attr = true;
  }
  GemmParams p;
  p.c = static_cast<__half*>(d->c);
  p.ldc = d->ldc;
  p.m = (int)d->m;
  p.n = (int)d->n;
  p.k = (int)d->k;
  p.add_zero = d->add_zero;
  p.status = static_cast<int*>(d->status);
  static int n_sm = 0;
  if (!n_sm) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n_sm < 1)
      return KTIR_ERR_CUDA;
  }
  const long long tiles = (d->m / BM) * (d->n / BN);
  if (tiles > 0x7fffffffLL) return KTIR_ERR_UNSUPPORTED;
  const unsigned grid = (unsigned)(tiles < n_sm ? tiles : n_sm);
  k_gemm_tcgen05<<<grid, 192, SMEM_BYTES, static_cast<cudaStream_t>(stream)>>>(ta, tb, p);
  return cudaGetLastError() == cudaSuccess ? KTIR_OK : KTIR_ERR_CUDA;
}
