// Causal / full flash attention on the 5th-generation tensor cores.
//
// Q, K, V, O are f16 [bh*seq, 128] row-major (one head = seq consecutive
// rows).  One CTA owns 128 query rows of one head (thread t of the 4 warps
// owns query row t, which is also TMEM lane t) and walks the key blocks
// of 64 rows:
//   S  = Q K^T        tcgen05.mma M=128 N=64  K=128 (Q and K both K-major)
//   softmax           thread-local per row from tcgen05.ld of S: running
//                     max / sum in f32, P = exp(S - m) written to shared
//                     memory as f16 in the 128-byte swizzled K-major layout
//   PV = P V          tcgen05.mma M=128 N=128 K=64  (V consumed MN-major)
//   O  = O*alpha + PV in registers (f32), O / l at the end
// K/V blocks stream through a 2-stage TMA ring.  Waits are bounded.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>

#include "../../include/ktir_b200.h"
#include "tc_common.cuh"

using namespace ktir::tc;

namespace {

constexpr int D = 128;         // head dim
constexpr int BQ = 128;        // query rows per CTA
constexpr int BKV = 64;        // key rows per block
constexpr int Q_BYTES = BQ * D * 2;            // 32 KiB (two 64-column boxes)
constexpr int KV_BOX = BKV * 64 * 2;           // 8 KiB: 64 rows x 64 columns
constexpr int K_BYTES = BKV * D * 2;           // 16 KiB
constexpr int V_BYTES = BKV * D * 2;           // 16 KiB
constexpr int STAGE_BYTES = K_BYTES + V_BYTES; // 32 KiB
constexpr int P_BYTES = BQ * BKV * 2;          // 16 KiB
constexpr int SMEM_BYTES = Q_BYTES + 2 * STAGE_BYTES + P_BYTES + 1024;
constexpr uint32_t TMEM_COLS = 256;            // S: 64 columns, PV: 128 columns
constexpr uint32_t S_COL = 0, PV_COL = 128;

struct FmhaParams {
  __half* o;
  long long seq;
  long long row_stride;
  float scale_log2;   // scale * log2(e)
  int causal;
  int n_qtiles;
  int* status;
};

__device__ __forceinline__ void tmem_ld32f(uint32_t taddr, float (&f)[32]) {
  uint32_t r[32];
  tmem_ld32(taddr, r);
  tmem_ld_wait();
#pragma unroll
  for (int i = 0; i < 32; ++i) f[i] = __uint_as_float(r[i]);
}

__global__ void __launch_bounds__(128, 1)
    k_fmha_tcgen05(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                   const __grid_constant__ CUtensorMap tv, const __grid_constant__ FmhaParams p) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t q_bar;
  __shared__ __align__(8) uint64_t kv_bar[2];
  __shared__ __align__(8) uint64_t s_bar;
  __shared__ __align__(8) uint64_t pv_bar;
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;
  volatile int* abort = &abort_flag;

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  // heaviest (last) query tiles first
  const int qt = p.n_qtiles - 1 - (int)blockIdx.x;
  const long long head = blockIdx.y;
  const long long row0 = head * p.seq + (long long)qt * BQ;
  const int q0 = qt * BQ;
  const int n_kv = p.causal ? (q0 + BQ) / BKV : (int)(p.seq / BKV);

  const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  const uint32_t sQ = base;
  const uint32_t sKV = base + Q_BYTES;           // stage s at sKV + s * STAGE_BYTES (K then V)
  const uint32_t sP = sKV + 2 * STAGE_BYTES;

  if (tid == 0) {
    abort_flag = 0;
    mbar_init(smem_u32(&q_bar), 1);
    mbar_init(smem_u32(&kv_bar[0]), 1);
    mbar_init(smem_u32(&kv_bar[1]), 1);
    mbar_init(smem_u32(&s_bar), 1);
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

  auto load_kv = [&](int j, int s) {
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

  if (tid == 0) {
    tma_prefetch_desc(&tq);
    tma_prefetch_desc(&tk);
    tma_prefetch_desc(&tv);
    const uint32_t qb = smem_u32(&q_bar);
    mbar_arrive_expect_tx(qb, Q_BYTES);
    tma_load_2d(sQ, &tq, qb, 0, (int)row0);
    tma_load_2d(sQ + Q_BYTES / 2, &tq, qb, 64, (int)row0);
    load_kv(0, 0);
    if (n_kv > 1) load_kv(1, 1);
  }

  // S: M=128 N=64, A = Q K-major, B = K K-major;  PV: M=128 N=128, A = P K-major, B = V MN-major
  constexpr uint32_t idesc_s = idesc_f16(BQ, BKV, 0, 0);
  constexpr uint32_t idesc_pv = idesc_f16(BQ, D, 0, 1);

  float o[D];
#pragma unroll
  for (int i = 0; i < D; ++i) o[i] = 0.f;
  float m_run = -INFINITY, l_run = 0.f;
  const int qpos = q0 + tid;
  const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
  // Every thread runs every iteration and every barrier; after a timed-out
  // wait (abort flag set) the remaining work is skipped, never the barriers.
  for (int j = 0; j < n_kv; ++j) {
    const int s = j & 1;
    const uint32_t kb = sKV + s * STAGE_BYTES;
    const uint32_t vb = kb + K_BYTES;
    if (tid == 0 && !*abort) {
      bool good = (j > 0 || mbar_wait(smem_u32(&q_bar), 0, abort)) &&
                  mbar_wait(smem_u32(&kv_bar[s]), (j >> 1) & 1, abort);
      if (good) {
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t chunk = kk >> 2;          // 64-column chunk of d
          const uint32_t koff = (kk & 3) * 32;     // 16 d = 32 bytes within a 128-byte row
          const uint64_t ad = sdesc_sw128(sQ + chunk * (Q_BYTES / 2) + koff, 16, 1024);
          const uint64_t bd = sdesc_sw128(kb + chunk * KV_BOX + koff, 16, 1024);
          mma_f16(tmem + S_COL, ad, bd, idesc_s, kk != 0);
        }
        mma_commit(smem_u32(&s_bar));
      }
    }
    __syncwarp();
    mbar_wait(smem_u32(&s_bar), j & 1, abort);
    tc_fence_after();

    // ---- softmax on this thread's row ------------------------------------
    float sv[BKV];
    {
      float t[32];
      tmem_ld32f(tmem + lane_base + S_COL, t);
#pragma unroll
      for (int i = 0; i < 32; ++i) sv[i] = t[i];
      tmem_ld32f(tmem + lane_base + S_COL + 32, t);
#pragma unroll
      for (int i = 0; i < 32; ++i) sv[32 + i] = t[i];
    }
    const int kpos0 = j * BKV;
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < BKV; ++i) {
      float x = sv[i] * p.scale_log2;
      if (p.causal && kpos0 + i > qpos) x = -INFINITY;
      sv[i] = x;
      mx = fmaxf(mx, x);
    }
    const float m_new = fmaxf(m_run, mx);
    const float alpha = (m_new == -INFINITY) ? 1.f : exp2f(m_run - m_new);
    float psum = 0.f;
    __half2 ph[BKV / 2];
#pragma unroll
    for (int i = 0; i < BKV; i += 2) {
      const float a = (m_new == -INFINITY) ? 0.f : exp2f(sv[i] - m_new);
      const float b = (m_new == -INFINITY) ? 0.f : exp2f(sv[i + 1] - m_new);
      psum += a + b;
      ph[i / 2] = __floats2half2_rn(a, b);
    }
    l_run = l_run * alpha + psum;
    m_run = m_new;
#pragma unroll
    for (int i = 0; i < D; ++i) o[i] *= alpha;
    // P row -> shared memory, 128-byte swizzle: 16-byte unit u of row r lands at u ^ (r & 7)
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
#pragma unroll
      for (int kk = 0; kk < BKV / 16; ++kk) {
        const uint64_t ad = sdesc_sw128(sP + kk * 32, 16, 1024);
        const uint64_t bd = sdesc_sw128(vb + kk * 16 * 128, KV_BOX, 1024);
        mma_f16(tmem + PV_COL, ad, bd, idesc_pv, kk != 0);
      }
      mma_commit(smem_u32(&pv_bar));
    }
    __syncwarp();
    mbar_wait(smem_u32(&pv_bar), j & 1, abort);
    tc_fence_after();
#pragma unroll
    for (int c = 0; c < D; c += 32) {
      float t[32];
      tmem_ld32f(tmem + lane_base + PV_COL + c, t);
#pragma unroll
      for (int i = 0; i < 32; ++i) o[c + i] += t[i];
    }
    tc_fence_before();
    __syncthreads();
    // stage s is free (its S and PV MMAs are complete): prefetch block j + 2
    if (tid == 0 && j + 2 < n_kv && !*abort) load_kv(j + 2, s);
  }

  if (!*abort) {
    const float inv = 1.f / l_run;
    __half* orow = p.o + (row0 + tid) * p.row_stride;
#pragma unroll
    for (int c = 0; c < D; c += 8) {
      __half2 h[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(o[c + 2 * i] * inv, o[c + 2 * i + 1] * inv);
      *reinterpret_cast<uint4*>(orow + c) = *reinterpret_cast<const uint4*>(h);
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
