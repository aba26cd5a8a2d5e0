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

// Output tiles are BM x BN with BN = 256, or 128 when a problem has too few
// 256-wide tiles to give every SM one (a slice of a GEMM split across GPUs).
constexpr int BM = 128, BK = 64, STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;            // 16 KiB
constexpr int B_BOX_BYTES = 64 * BK * 2;        // 8 KiB per 64-column box
template <int BN> struct GemmShape {
  static constexpr int B_BYTES = BK * BN * 2;            // 32 / 16 KiB
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;  // 48 / 32 KiB
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024;
  static constexpr uint32_t TMEM_COLS = 2 * BN;          // two accumulators
};

struct GemmParams {
  __half* c;
  long long ldc;
  int m, n, k;
  int add_zero;
  int* status;
};

template <int BN>
__global__ void __launch_bounds__(192, 1)
    k_gemm_tcgen05(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb,
                   const __grid_constant__ GemmParams p) {
  constexpr int STAGE_BYTES = GemmShape<BN>::STAGE_BYTES;
  constexpr uint32_t TMEM_COLS = GemmShape<BN>::TMEM_COLS;
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

// ---------------------------------------------------------------------------
// GEMM of any shape with the reference's rounding of each K block: KTIR that
// multiplies f16 tiles without widening them first gets each block product
// as an f16 tile (NumPy's f16 matmul: the sum in f32, one f16 rounding) and
// adds it to an f16 or f32 running sum (ktir_cpu/dialects/linalg_ops.py:273-297
// with ops/arith_ops.py:403-419).  One CTA per 128x128 output tile: warp 0
// streams A (64 k x 128 m) and B (two 64 n x 64 k boxes) through a 4-stage TMA
// ring (rows, columns and k past the matrix read as zero), warp 1 issues the
// block's tcgen05.mma (M128 N128 K16) into one of two TMEM buffers and
// commits each finished block, warps 2..5 round each block product to f16
// and add it to their rows' running sums in registers while the next block
// accumulates in the other buffer, then store the rows and columns inside C.
// block_k = 0: one block of all of K (one f16 rounding at the end, the
// product of f16 tiles widened to f32).
constexpr int GB_BM = 128, GB_BN = 128, GB_BK = 64, GB_STAGES = 4;
constexpr int GB_A_BYTES = GB_BM * GB_BK * 2;          // 16 KiB
constexpr int GB_B_BYTES = GB_BK * GB_BN * 2;          // 16 KiB
constexpr int GB_STAGE_BYTES = GB_A_BYTES + GB_B_BYTES;
constexpr int GB_SMEM_BYTES = GB_STAGES * GB_STAGE_BYTES + 1024;
constexpr uint32_t GB_TMEM_COLS = 256;                 // two 128-column block products

struct GemmBlockedParams {
  __half* c;
  long long ldc;
  int m, n, k;
  int block_steps;   // 16-wide k steps per block
  int round_blocks;  // each block product rounded to f16 (else one block, widened operands)
  int acc_f16;       // running sum rounded to f16 after each block
  int* status;
};

__global__ void __launch_bounds__(192, 1)
    k_gemm_blocked(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb,
                   const __grid_constant__ GemmBlockedParams p) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[GB_STAGES];
  __shared__ __align__(8) uint64_t empty_bar[GB_STAGES];
  __shared__ __align__(8) uint64_t x_full[2];
  __shared__ __align__(8) uint64_t x_empty[2];
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;

  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t smem = (raw + 1023u) & ~1023u;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * GB_BM;
  const int n0 = blockIdx.y * GB_BN;
  const int KT = (p.k + GB_BK - 1) / GB_BK;
  const int n_steps = (p.k + 15) / 16;
  const int spb = p.block_steps;
  const int n_blocks = (n_steps + spb - 1) / spb;
  volatile int* abort = &abort_flag;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < GB_STAGES; ++s) {
      mbar_init(smem_u32(&full_bar[s]), 1);
      mbar_init(smem_u32(&empty_bar[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&x_full[b]), 1);
      mbar_init(smem_u32(&x_empty[b]), 128);
    }
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&tmem_base), GB_TMEM_COLS);
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
      for (int kt = 0; kt < KT && !*abort; ++kt) {
        const int s = kt % GB_STAGES;
        if (!mbar_wait(smem_u32(&empty_bar[s]), ((kt / GB_STAGES) & 1) ^ 1, abort)) break;
        const uint32_t fb = smem_u32(&full_bar[s]);
        mbar_arrive_expect_tx(fb, GB_STAGE_BYTES);
        const uint32_t a_dst = smem + s * GB_STAGE_BYTES;
        const uint32_t b_dst = a_dst + GB_A_BYTES;
        tma_load_2d(a_dst, &ta, fb, kt * GB_BK, m0);
        tma_load_2d(b_dst, &tb, fb, n0, kt * GB_BK);
        tma_load_2d(b_dst + B_BOX_BYTES, &tb, fb, n0 + 64, kt * GB_BK);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16(GB_BM, GB_BN, 0, 1);
      bool ok = true;
      for (int kt = 0; kt < KT && ok; ++kt) {
        const int s = kt % GB_STAGES;
        if (!mbar_wait(smem_u32(&full_bar[s]), (kt / GB_STAGES) & 1, abort)) break;
        tc_fence_after();
        const uint32_t a_addr = smem + s * GB_STAGE_BYTES;
        const uint32_t b_addr = a_addr + GB_A_BYTES;
        for (int kk = 0; kk < GB_BK / 16; ++kk) {
          const int step = kt * (GB_BK / 16) + kk;
          if (step >= n_steps) break;
          const int blk = step / spb;
          const int in_blk = step - blk * spb;
          const uint32_t xb = (uint32_t)(blk & 1);
          if (in_blk == 0 && blk >= 2) {
            // the epilogue has read block blk - 2 out of this buffer
            if (!mbar_wait(smem_u32(&x_empty[xb]), ((blk - 2) >> 1) & 1, abort)) {
              ok = false;
              break;
            }
            tc_fence_after();
          }
          const uint64_t ad = sdesc_sw128(a_addr + kk * 32, 16, 1024);
          const uint64_t bd = sdesc_sw128(b_addr + kk * 16 * 128, B_BOX_BYTES, 1024);
          mma_f16(tmem + xb * GB_BN, ad, bd, idesc, in_blk != 0);
          if (in_blk == spb - 1 || step == n_steps - 1) mma_commit(smem_u32(&x_full[xb]));
        }
        mma_commit(smem_u32(&empty_bar[s]));
      }
    }
  } else {
    // epilogue warps 2..5: warp w reads TMEM lanes 32*(w%4) .. +31 (rows)
    const int q = warp & 3;
    const int row = 32 * q + lane;
    float acc[GB_BN];
#pragma unroll
    for (int i = 0; i < GB_BN; ++i) acc[i] = 0.f;
    bool ok = true;
    for (int blk = 0; blk < n_blocks; ++blk) {
      const uint32_t xb = (uint32_t)(blk & 1);
      ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&x_full[xb]), (blk >> 1) & 1, abort));
      if (!ok) break;
      tc_fence_after();
      const uint32_t x = tmem + ((uint32_t)(32 * q) << 16) + xb * GB_BN;
#pragma unroll
      for (int c = 0; c < GB_BN; c += 32) {
        uint32_t r[32];
        tmem_ld32_wait(x + c, r);
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float v = __uint_as_float(r[i]);
          if (!p.round_blocks) {
            acc[c + i] = 0.f + v;            // one block of all of K, widened operands
          } else {
            const float b16 = __half2float(__float2half_rn(v));   // the block's f16 product
            const float s = acc[c + i] + b16;
            acc[c + i] = p.acc_f16 ? __half2float(__float2half_rn(s)) : s;
          }
        }
      }
      tc_fence_before();
      mbar_arrive(smem_u32(&x_empty[xb]));
    }
    if (ok && m0 + row < p.m) {
      __half* crow = p.c + (long long)(m0 + row) * p.ldc;
      const bool vec = (p.ldc & 7) == 0 && ((reinterpret_cast<uintptr_t>(p.c) & 15) == 0);
#pragma unroll
      for (int c = 0; c < GB_BN; c += 8) {
        const int col = n0 + c;
        if (vec && col + 8 <= p.n) {
          __half2 h[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) h[j] = __floats2half2_rn(acc[c + 2 * j], acc[c + 2 * j + 1]);
          *reinterpret_cast<uint4*>(crow + col) = *reinterpret_cast<const uint4*>(h);
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j)
            if (col + j < p.n) crow[col + j] = __float2half_rn(acc[c + j]);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, GB_TMEM_COLS);
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
  if (!d || !d->a || !d->b || !d->c || !d->status)
    return ktir_set_error(KTIR_ERR_ARG, "ktir_gemm_f16: null argument");
  if (d->m % BM || d->n % 128 || d->k % BK || d->k < BK)
    return ktir_set_error(KTIR_ERR_UNSUPPORTED,
                          "ktir_gemm_f16: M, N, K must be multiples of 128, 128, 64");
  if ((reinterpret_cast<uintptr_t>(d->a) | reinterpret_cast<uintptr_t>(d->b) |
       reinterpret_cast<uintptr_t>(d->c)) & 15)
    return ktir_set_error(KTIR_ERR_UNSUPPORTED, "ktir_gemm_f16: operands not 16-byte aligned");
  if ((d->lda | d->ldb | d->ldc) & 7)
    return ktir_set_error(KTIR_ERR_UNSUPPORTED,
                          "ktir_gemm_f16: row strides must be multiples of 8 elements");
  CUtensorMap ta, tb;
  if (!make_map(&ta, d->a, d->m, d->k, d->lda, 64, BM) ||
      !make_map(&tb, d->b, d->k, d->n, d->ldb, 64, BK))
    return ktir_set_error(KTIR_ERR_CUDA, "ktir_gemm_f16: tensor map encoding failed");
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(k_gemm_tcgen05<256>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             GemmShape<256>::SMEM_BYTES) != cudaSuccess ||
        cudaFuncSetAttribute(k_gemm_tcgen05<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             GemmShape<128>::SMEM_BYTES) != cudaSuccess)
      return ktir_set_error(KTIR_ERR_CUDA, "ktir_gemm_f16: shared-memory attribute refused");
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
      return ktir_set_error(KTIR_ERR_CUDA, "ktir_gemm_f16: no SM count for the current device");
  }
  // 256-wide tiles when N allows them and they fill more than half the SMs;
  // else 128-wide ones (twice the CTAs for the same work)
  const bool wide = d->n % 256 == 0 && (d->m / BM) * (d->n / 256) > n_sm / 2;
  const long long tiles = (d->m / BM) * (d->n / (wide ? 256 : 128));
  if (tiles > 0x7fffffffLL) return ktir_set_error(KTIR_ERR_UNSUPPORTED, "ktir_gemm_f16: too many tiles");
  const unsigned grid = (unsigned)(tiles < n_sm ? tiles : n_sm);
  if (wide)
    k_gemm_tcgen05<256><<<grid, 192, GemmShape<256>::SMEM_BYTES, static_cast<cudaStream_t>(stream)>>>(ta, tb, p);
  else
    k_gemm_tcgen05<128><<<grid, 192, GemmShape<128>::SMEM_BYTES, static_cast<cudaStream_t>(stream)>>>(ta, tb, p);
  return cudaGetLastError() == cudaSuccess
             ? KTIR_OK : ktir_set_error(KTIR_ERR_CUDA, "ktir_gemm_f16: launch failed");
}

extern "C" int ktir_gemm_f16_blocked(const KtirGemmBlockedDesc* d, void* stream) {
  if (!d || !d->a || !d->b || !d->c || !d->status)
    return ktir_set_error(KTIR_ERR_ARG, "ktir_gemm_f16_blocked: null argument");
  if (d->m < 1 || d->n < 1 || d->k < 1 || d->block_k < 0 || (d->block_k & 15))
    return ktir_set_error(KTIR_ERR_UNSUPPORTED,
                          "ktir_gemm_f16_blocked: empty matrix or block_k not a multiple of 16");
  if (d->m > 0x7fffffffLL || d->n > 0x7fffffffLL || d->k > 0x7fffffffLL)
    return ktir_set_error(KTIR_ERR_UNSUPPORTED, "ktir_gemm_f16_blocked: dimension above 2^31");
  if ((reinterpret_cast<uintptr_t>(d->a) | reinterpret_cast<uintptr_t>(d->b)) & 15)
    return ktir_set_error(KTIR_ERR_UNSUPPORTED, "ktir_gemm_f16_blocked: A or B not 16-byte aligned");
  if ((d->lda | d->ldb) & 7 || d->lda < d->k || d->ldb < d->n || d->ldc < d->n)
    return ktir_set_error(KTIR_ERR_UNSUPPORTED,
                          "ktir_gemm_f16_blocked: lda / ldb must be multiples of 8 elements, "
                          "and no row stride below its row length");
  const long long gy = (d->n + GB_BN - 1) / GB_BN, gx = (d->m + GB_BM - 1) / GB_BM;
  if (gy > 65535 || gx > 0x7fffffffLL)
    return ktir_set_error(KTIR_ERR_UNSUPPORTED, "ktir_gemm_f16_blocked: too many tiles");
  CUtensorMap ta, tb;
  if (!make_map(&ta, d->a, d->m, d->k, d->lda, 64, GB_BM) ||
      !make_map(&tb, d->b, d->k, d->n, d->ldb, 64, GB_BK))
    return ktir_set_error(KTIR_ERR_CUDA, "ktir_gemm_f16_blocked: tensor map encoding failed");
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(k_gemm_blocked, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             GB_SMEM_BYTES) != cudaSuccess)
      return ktir_set_error(KTIR_ERR_CUDA, "ktir_gemm_f16_blocked: shared-memory attribute refused");
    attr = true;
  }
  GemmBlockedParams p;
  p.c = static_cast<__half*>(d->c);
  p.ldc = d->ldc;
  p.m = (int)d->m;
  p.n = (int)d->n;
  p.k = (int)d->k;
  const int n_steps = (int)((d->k + 15) / 16);
  p.block_steps = d->block_k ? (int)(d->block_k / 16) : n_steps;
  p.round_blocks = d->block_k ? 1 : 0;
  p.acc_f16 = d->acc_f16 ? 1 : 0;
  p.status = static_cast<int*>(d->status);
  k_gemm_blocked<<<dim3((unsigned)gx, (unsigned)gy), 192, GB_SMEM_BYTES,
                   static_cast<cudaStream_t>(stream)>>>(ta, tb, p);
  return cudaGetLastError() == cudaSuccess
             ? KTIR_OK : ktir_set_error(KTIR_ERR_CUDA, "ktir_gemm_f16_blocked: launch failed");
}
