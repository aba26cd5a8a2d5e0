// Causal / full flash attention on the 5th-generation tensor cores.
//
// Q, K, V, O are f16 [bh*seq, 128] row-major (one head = seq consecutive
// rows).  One CTA owns 128 query rows of one head; thread t of the 4 warps
// owns query row t, which is also TMEM lane t.  Key blocks are 64 rows:
//   S_j  = Q K_j^T    tcgen05.mma M=128 N=64 K=128 into one of two TMEM
//                     S buffers, issued one block ahead so the tensor cores
//                     compute S_{j+1} while the threads run softmax on S_j
//   softmax           thread-local per row (tcgen05.ld of S_j), P_j = 2^(x - m)
//                     written to shared memory as f16, 128-byte swizzled
//   O   += P_j V_j    tcgen05.mma M=128 N=128 K=64, O accumulates in TMEM
// The running max m is only moved when a row's new max exceeds it by more
// than 2^8 (then O and l are rescaled through tcgen05.ld/st, warp-uniform);
// otherwise P stays below 2^8, which f16 holds exactly enough, and O / l is
// unchanged because O and l share the same m.  K/V stream through a 3-stage
// TMA ring.  Every wait is bounded; after a timed-out wait the CTA skips the
// remaining work but still runs every barrier and frees its TMEM.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>

#include "../../include/ktir_b200.h"
#include "tc_common.cuh"

using namespace ktir::tc;

namespace {

constexpr int D = 128;          // head dim
constexpr int BQ = 128;         // query rows per CTA
constexpr int BKV = 64;         // key rows per block
constexpr int STAGES = 3;
constexpr int Q_BYTES = BQ * D * 2;             // 32 KiB (two 64-column boxes)
constexpr int KV_BOX = BKV * 64 * 2;            // 8 KiB: 64 rows x 64 columns
constexpr int K_BYTES = BKV * D * 2;            // 16 KiB
constexpr int V_BYTES = BKV * D * 2;            // 16 KiB
constexpr int STAGE_BYTES = K_BYTES + V_BYTES;  // 32 KiB
constexpr int P_BYTES = BQ * BKV * 2;           // 16 KiB
constexpr int SMEM_BYTES = Q_BYTES + STAGES * STAGE_BYTES + P_BYTES + 1024;
constexpr uint32_t TMEM_COLS = 256;             // S0: 0..63, S1: 64..127, O: 128..255
constexpr uint32_t O_COL = 128;
constexpr float RESCALE_THRESHOLD = 8.0f;       // log2 units

struct FmhaParams {
  __half* o;
  long long seq;
  long long row_stride;
  float scale_log2;   // scale * log2(e)
  int causal;
  int n_qtiles;
  int* status;
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__global__ void __launch_bounds__(128, 1)
    k_fmha_tcgen05(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                   const __grid_constant__ CUtensorMap tv, const __grid_constant__ FmhaParams p) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t q_bar;
  __shared__ __align__(8) uint64_t kv_bar[STAGES];
  __shared__ __align__(8) uint64_t s_bar[2];
  __shared__ __align__(8) uint64_t pv_bar;
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;
  volatile int* abort = &abort_flag;

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int qt = p.n_qtiles - 1 - (int)blockIdx.x;   // heaviest query tiles first
  const long long head = blockIdx.y;
  const long long row0 = head * p.seq + (long long)qt * BQ;
  const int q0 = qt * BQ;
  const int n_kv = p.causal ? (q0 + BQ) / BKV : (int)(p.seq / BKV);

  const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  const uint32_t sQ = base;
  const uint32_t sKV = base + Q_BYTES;
  const uint32_t sP = sKV + STAGES * STAGE_BYTES;

  if (tid == 0) {
    abort_flag = 0;
    mbar_init(smem_u32(&q_bar), 1);
    for (int s = 0; s < STAGES; ++s) mbar_init(smem_u32(&kv_bar[s]), 1);
    mbar_init(smem_u32(&s_bar[0]), 1);
    mbar_init(smem_u32(&s_bar[1]), 1);
    mbar_init(smem_u32(&pv_bar), 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(&tmem_base), TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;
  const uint32_t lane_base = (uint32_t)(warp * 32) << 16;

  constexpr uint32_t idesc_s = idesc_f16(BQ, BKV, 0, 0);   // Q, K both K-major
  constexpr uint32_t idesc_pv = idesc_f16(BQ, D, 0, 1);    // P K-major, V MN-major

  auto load_kv = [&](int j) {
    const int s = j % STAGES;
    const uint32_t kb = sKV + s * STAGE_BYTES;
    const uint32_t vb = kb + K_BYTES;
    const uint32_t bar = smem_u32(&kv_bar[s]);
    const int kr = (int)(head * p.seq) + j * BKV;
    mbar_arrive_expect_tx(bar, STAGE_BYTES);
    tma_load_2d(kb, &tk, bar, 0, kr);
    tma_load_2d(kb + KV_BOX, &tk, bar, 64, kr);
    tma_load_2d(vb, &tv, bar, 0, kr);
    tma_load_2d(vb + KV_BOX, &tv, bar, 64, kr);
  };
  // S_j = Q K_j^T into S buffer j & 1 (thread 0 only)
  auto issue_s = [&](int j) {
    const int s = j % STAGES;
    if (!mbar_wait(smem_u32(&kv_bar[s]), (j / STAGES) & 1, abort)) return;
    tc_fence_after();
    const uint32_t kb = sKV + s * STAGE_BYTES;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      const uint32_t chunk = kk >> 2;
      const uint32_t koff = (kk & 3) * 32;
      const uint64_t ad = sdesc_sw128(sQ + chunk * (Q_BYTES / 2) + koff, 16, 1024);
      const uint64_t bd = sdesc_sw128(kb + chunk * KV_BOX + koff, 16, 1024);
      mma_f16(tmem + (uint32_t)((j & 1) * BKV), ad, bd, idesc_s, kk != 0);
    }
    mma_commit(smem_u32(&s_bar[j & 1]));
  };

  if (tid == 0) {
    tma_prefetch_desc(&tq);
    tma_prefetch_desc(&tk);
    tma_prefetch_desc(&tv);
    const uint32_t qb = smem_u32(&q_bar);
    mbar_arrive_expect_tx(qb, Q_BYTES);
    tma_load_2d(sQ, &tq, qb, 0, (int)row0);
    tma_load_2d(sQ + Q_BYTES / 2, &tq, qb, 64, (int)row0);
    for (int j = 0; j < STAGES && j < n_kv; ++j) load_kv(j);
    if (mbar_wait(qb, 0, abort)) issue_s(0);
  }

  float m_used = -INFINITY, l_run = 0.f;
  const int qpos = q0 + tid;
  for (int j = 0; j < n_kv; ++j) {
    __syncwarp();
    mbar_wait(smem_u32(&s_bar[j & 1]), (j >> 1) & 1, abort);
    tc_fence_after();
    float sv[BKV];
    {
      uint32_t r[32];
      tmem_ld32(tmem + lane_base + (uint32_t)((j & 1) * BKV), r);
      tmem_ld_wait();
#pragma unroll
      for (int i = 0; i < 32; ++i) sv[i] = __uint_as_float(r[i]);
      tmem_ld32(tmem + lane_base + (uint32_t)((j & 1) * BKV) + 32, r);
      tmem_ld_wait();
#pragma unroll
      for (int i = 0; i < 32; ++i) sv[32 + i] = __uint_as_float(r[i]);
    }
    // the next block's S goes to the other buffer, read last in iteration j-1
    if (tid == 0 && j + 1 < n_kv && !*abort) issue_s(j + 1);

    const int kpos0 = j * BKV;
    const bool diag = p.causal && kpos0 + BKV - 1 > q0;
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < BKV; ++i) {
      float x = sv[i] * p.scale_log2;
      if (diag && kpos0 + i > qpos) x = -INFINITY;
      sv[i] = x;
      mx = fmaxf(mx, x);
    }
    const float m_new = fmaxf(m_used, mx);
    float factor = 1.f;
    bool rescale = false;
    if (m_used == -INFINITY || m_new > m_used + RESCALE_THRESHOLD) {
      factor = (m_used == -INFINITY) ? 0.f : ex2(m_used - m_new);
      rescale = m_used != -INFINITY;
      l_run *= factor;
      m_used = m_new;
    }
    float psum = 0.f;
    __half2 ph[BKV / 2];
#pragma unroll
    for (int i = 0; i < BKV; i += 2) {
      const float a = (m_used == -INFINITY) ? 0.f : ex2(sv[i] - m_used);
      const float b = (m_used == -INFINITY) ? 0.f : ex2(sv[i + 1] - m_used);
      psum += a + b;
      ph[i / 2] = __floats2half2_rn(a, b);
    }
    l_run += psum;

    // PV_{j-1} done: O is complete up to block j-1, P and K/V stage (j-1)%3 are free
    if (j > 0) {
      __syncwarp();
      mbar_wait(smem_u32(&pv_bar), (j - 1) & 1, abort);
      tc_fence_after();
    }
    if (tid == 0 && j > 0 && j + 2 < n_kv && !*abort) load_kv(j + 2);
    if (j > 0 && __any_sync(0xffffffffu, rescale)) {
#pragma unroll 1
      for (int c = 0; c < D; c += 32) {
        uint32_t r[32];
        tmem_ld32(tmem + lane_base + O_COL + c, r);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * factor);
        tmem_st32(tmem + lane_base + O_COL + c, r);
      }
      tmem_st_wait();
    }
    {
      const uint32_t rowaddr = sP + tid * 128;
      const uint4* src = reinterpret_cast<const uint4*>(ph);
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const uint32_t dst = rowaddr + ((u ^ (tid & 7)) << 4);
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(dst), "r"(src[u].x),
                     "r"(src[u].y), "r"(src[u].z), "r"(src[u].w)
                     : "memory");
      }
    }
    fence_proxy_async();
    tc_fence_before();
    __syncthreads();
    if (tid == 0 && !*abort) {
      tc_fence_after();
      const uint32_t vb = sKV + (j % STAGES) * STAGE_BYTES + K_BYTES;
#pragma unroll
      for (int kk = 0; kk < BKV / 16; ++kk) {
        const uint64_t ad = sdesc_sw128(sP + kk * 32, 16, 1024);
        const uint64_t bd = sdesc_sw128(vb + kk * 16 * 128, KV_BOX, 1024);
        mma_f16(tmem + O_COL, ad, bd, idesc_pv, (j | kk) != 0);
      }
      mma_commit(smem_u32(&pv_bar));
    }
  }

  __syncwarp();
  mbar_wait(smem_u32(&pv_bar), (n_kv - 1) & 1, abort);
  tc_fence_after();
  if (!*abort) {
    const float inv = 1.f / l_run;
    __half* orow = p.o + (row0 + tid) * p.row_stride;
#pragma unroll 1
    for (int c = 0; c < D; c += 32) {
      uint32_t r[32];
      tmem_ld32(tmem + lane_base + O_COL + c, r);
      tmem_ld_wait();
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        __half2 h[4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
          h[i] = __floats2half2_rn(__uint_as_float(r[8 * q + 2 * i]) * inv,
                                   __uint_as_float(r[8 * q + 2 * i + 1]) * inv);
        *reinterpret_cast<uint4*>(orow + c + 8 * q) = *reinterpret_cast<const uint4*>(h);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
  if (tid == 0 && abort_flag) atomicOr(p.status, KTIR_STATUS_TIMEOUT);
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

bool make_map(CUtensorMap* m, const void* base, long long rows, long long ld, int box_rows) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {(cuuint64_t)D, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box,
             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

extern "C" int ktir_fmha_f16(const KtirFmhaDesc* d, void* stream) {
  if (!d || !d->q || !d->k || !d->v || !d->o || !d->status) return KTIR_ERR_ARG;
  if (d->d != D || d->seq % BQ || d->bh < 1 || d->row_stride < D || (d->row_stride & 7))
    return KTIR_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(d->q) | reinterpret_cast<uintptr_t>(d->k) |
       reinterpret_cast<uintptr_t>(d->v) | reinterpret_cast<uintptr_t>(d->o)) & 15)
    return KTIR_ERR_UNSUPPORTED;
  const long long rows = d->bh * d->seq;
  if (rows > 0x7fffffffLL) return KTIR_ERR_UNSUPPORTED;
  CUtensorMap tq, tk, tv;
  if (!make_map(&tq, d->q, rows, d->row_stride, BQ) || !make_map(&tk, d->k, rows, d->row_stride, BKV) ||
      !make_map(&tv, d->v, rows, d->row_stride, BKV))
    return KTIR_ERR_CUDA;
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(k_fmha_tcgen05, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             SMEM_BYTES) != cudaSuccess)
      return KTIR_ERR_CUDA;
    attr = true;
  }
  FmhaParams p;
  p.o = static_cast<__half*>(d->o);
  p.seq = d->seq;
  p.row_stride = d->row_stride;
  p.scale_log2 = d->scale * 1.4426950408889634f;
  p.causal = d->causal;
  p.n_qtiles = (int)(d->seq / BQ);
  p.status = d->status;
  dim3 grid((unsigned)p.n_qtiles, (unsigned)d->bh);
  k_fmha_tcgen05<<<grid, 128, SMEM_BYTES, static_cast<cudaStream_t>(stream)>>>(tq, tk, tv, p);
  return cudaGetLastError() == cudaSuccess ? KTIR_OK : KTIR_ERR_CUDA;
}
