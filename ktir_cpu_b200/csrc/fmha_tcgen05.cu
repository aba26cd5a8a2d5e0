// Causal / full flash attention on the 5th-generation tensor cores.
//
// Q, K, V, O are f16 [bh*seq, 128] row-major (one head = seq consecutive
// rows).  One CTA per SM owns two 128-row query tiles of one head (query rows
// q0 .. q0+255) and walks the key blocks of 128 rows; each K and V block is
// loaded once and used by both tiles.  Warp roles meet only at mbarriers:
//   warp 8 (TMA)      Q tiles once, K_j into a 2-stage ring
//   warp 9 (TMA)      V_j into a 2-stage ring; every slot is refilled as soon
//                     as the MMAs that read it complete
//   warp 10 (MMA)     S_t = Q_t K_j^T (M=128 N=128 K=128) into tile t's S
//                     buffer; once the softmax warps of tile t hand over P_t
//                     it issues O_t += P_t V_j (M=128 N=128 K=128) with P read
//                     straight from TMEM, and S_t for block j+1 into the same
//                     buffer once that PV product has completed (a later MMA
//                     may write TMEM while an earlier one still reads it).
//                     An event loop issues whichever tile's product is ready,
//                     so while tile 0's softmax works the tensor cores run
//                     tile 1's products and the other way round
//   warps 0-3, 4-7    softmax of tile 0 / tile 1: thread r owns query row r
//                     of its tile = TMEM lane r: tcgen05.ld of the 128 scores,
//                     masked max of x = s * scale * log2(e), P = 2^(x - m)
//                     (five pairs in eight by ex2.approx.f16x2 on MUFU, three
//                     by a cubic on the FMA pipe: MUFU alone cannot keep up
//                     with the tensor cores), tcgen05.st of P over the first 64 columns of
//                     the S buffer, row sum l from f16 pair partials
// TMEM (512 columns): S_0 / P_0 0..127, S_1 / P_1 128..255, O_0 256..383,
// O_1 384..511.  The running max m only moves when a row's max exceeds it by
// more than 2^8; then the softmax warp rescales its O rows in TMEM before
// handing over P (the S block it just read was committed after the previous
// PV product, so that product has landed), otherwise O and l keep sharing m.
// Every wait is bounded; a timed-out wait raises the CTA's abort flag, every
// role then leaves its loop, and the CTA still frees its TMEM.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>

#include "../../include/ktir_b200.h"
#include "tc_common.cuh"

using namespace ktir::tc;

namespace {

constexpr int D = 128;          // head dim
constexpr int BQ = 128;         // query rows per tile (two tiles per CTA)
constexpr int BKV = 128;        // key rows per block
constexpr int KST = 2;          // K ring stages
constexpr int VST = 2;          // V ring stages
constexpr int THREADS = 352;    // 8 softmax warps, 2 TMA warps, 1 MMA warp
constexpr int W_TMA_K = 8, W_TMA_V = 9, W_MMA = 10;
constexpr int Q_HALF = BQ * 64 * 2;             // 16 KiB: 128 rows x 64 columns
constexpr int Q_BYTES = 2 * Q_HALF;             // 32 KiB per tile
constexpr int KV_HALF = BKV * 64 * 2;           // 16 KiB: 128 rows x 64 columns
constexpr int KV_BYTES = 2 * KV_HALF;           // 32 KiB: 128 rows x 128 columns
constexpr int TILE_BYTES = 2 * Q_BYTES + (KST + VST) * KV_BYTES;

struct Bars {
  uint64_t q_full[2];
  uint64_t k_full[KST], k_empty[KST];
  uint64_t v_full[VST], v_empty[VST];
  uint64_t s_full[2], p_full[2], pv_done[2];
  uint64_t o_full;
  uint32_t tmem_base;
  int abort_flag;
};
constexpr int SMEM_BYTES = TILE_BYTES + (int)sizeof(Bars) + 1024;
static_assert(SMEM_BYTES <= 227 * 1024, "one CTA per SM");

constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t O_COL = 256;
constexpr float RESCALE_THRESHOLD = 8.0f;       // log2 units

struct FmhaParams {
  __half* o;
  long long seq;
  long long row_stride;
  float scale_log2;   // scale * log2(e)
  int causal;
  int n_qtiles;
  int n_pairs;
  int* status;
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^x for a pair: x rounded to f16, one MUFU op for both lanes of the pair
__device__ __forceinline__ uint32_t ex2_pair(float a, float b) {
  uint32_t h, y;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(h) : "f"(b), "f"(a));
  asm("ex2.approx.f16x2 %0, %1;" : "=r"(y) : "r"(h));
  return y;
}

// 2^x on the FMA and integer pipes, for the share of P the MUFU unit (16
// exponentials per clock per SM) does not take: x = n + t with n = round(x)
// by the 1.5 * 2^23 shift, 2^t on [-0.5, 0.5] by a cubic fitted to the
// relative error (max 7.5e-5, below the f16 rounding P gets), and n added to
// the exponent field.  x is clamped at -125 so the exponent cannot wrap;
// 2^-125 rounds to 0 in f16 like any P below the f16 range.
__device__ __forceinline__ float exp2_fma(float x) {
  x = fmaxf(x, -125.f);
  const float r = x + 12582912.f;
  const float t = x - (r - 12582912.f);
  const float q = fmaf(fmaf(fmaf(0.0551716536f, t, 0.242611125f), t, 0.693260968f), t, 0.999928057f);
  return __uint_as_float(__float_as_uint(q) + (__float_as_uint(r) << 23));
}

__device__ __forceinline__ uint32_t pack_f16x2(float a, float b) {
  uint32_t h;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(h) : "f"(b), "f"(a));
  return h;
}

// three-input max (NaN inputs ignored, like fmaxf)
__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// number of key blocks query tile qt reads (0 for a tile past the end)
__device__ __forceinline__ int blocks_of(const FmhaParams& p, int qt) {
  if (qt >= p.n_qtiles) return 0;
  return p.causal ? qt + 1 : (int)(p.seq / BKV);
}

__global__ void __launch_bounds__(THREADS, 1)
    k_fmha_tcgen05(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                   const __grid_constant__ CUtensorMap tv, const __grid_constant__ FmhaParams p) {
  extern __shared__ uint8_t smem_raw[];
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  const uint32_t sQ = base;                       // tile t at sQ + t * Q_BYTES
  const uint32_t sK = base + 2 * Q_BYTES;
  const uint32_t sV = sK + KST * KV_BYTES;
  Bars& B = *reinterpret_cast<Bars*>(smem_raw + (base - raw) + TILE_BYTES);
  volatile int* abort = &B.abort_flag;

  const int pair = p.n_pairs - 1 - (int)blockIdx.x;   // heaviest query tiles first
  const long long head = blockIdx.y;
  const int qt0 = 2 * pair;
  const int n_0 = blocks_of(p, qt0), n_1 = blocks_of(p, qt0 + 1);
  const int n_kv = n_0 > n_1 ? n_0 : n_1;

  if (tid == 0) {
    B.abort_flag = 0;
    for (int t = 0; t < 2; ++t) {
      mbar_init(smem_u32(&B.q_full[t]), 1);
      mbar_init(smem_u32(&B.s_full[t]), 1);
      mbar_init(smem_u32(&B.p_full[t]), BQ);
      mbar_init(smem_u32(&B.pv_done[t]), 1);
    }
    for (int s = 0; s < KST; ++s) {
      mbar_init(smem_u32(&B.k_full[s]), 1);
      mbar_init(smem_u32(&B.k_empty[s]), 1);
    }
    for (int s = 0; s < VST; ++s) {
      mbar_init(smem_u32(&B.v_full[s]), 1);
      mbar_init(smem_u32(&B.v_empty[s]), 1);
    }
    mbar_init(smem_u32(&B.o_full), 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(&B.tmem_base), TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = B.tmem_base;

  if (warp == W_TMA_K || warp == W_TMA_V) {
    // ---------------- TMA producers ----------------
    if (lane == 0) {
      const bool is_k = warp == W_TMA_K;
      const int kv_row0 = (int)(head * p.seq);
      if (is_k) {
        tma_prefetch_desc(&tq);
        tma_prefetch_desc(&tk);
        for (int t = 0; t < 2; ++t) {
          if ((t ? n_1 : n_0) == 0) continue;
          const uint32_t qb = smem_u32(&B.q_full[t]);
          const int qr = (int)(head * p.seq) + (qt0 + t) * BQ;
          mbar_arrive_expect_tx(qb, Q_BYTES);
          tma_load_2d(sQ + t * Q_BYTES, &tq, qb, 0, qr);
          tma_load_2d(sQ + t * Q_BYTES + Q_HALF, &tq, qb, 64, qr);
        }
      } else {
        tma_prefetch_desc(&tv);
      }
      const CUtensorMap* map = is_k ? &tk : &tv;
      uint64_t* full = is_k ? B.k_full : B.v_full;
      uint64_t* empty = is_k ? B.k_empty : B.v_empty;
      const int stages = is_k ? KST : VST;
      const uint32_t ring = is_k ? sK : sV;
      for (int j = 0; j < n_kv && !*abort; ++j) {
        const int kr = kv_row0 + j * BKV;
        const int st = j % stages;
        if (j >= stages && !mbar_wait(smem_u32(&empty[st]), ((j / stages) - 1) & 1, abort)) break;
        const uint32_t fb = smem_u32(&full[st]);
        const uint32_t dst = ring + st * KV_BYTES;
        mbar_arrive_expect_tx(fb, KV_BYTES);
        tma_load_2d(dst, map, fb, 0, kr);
        tma_load_2d(dst + KV_HALF, map, fb, 64, kr);
      }
    }
  } else if (warp == W_MMA) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_f16(BQ, BKV, 0, 0);   // Q, K both K-major
      constexpr uint32_t idesc_pv = idesc_f16(BQ, D, 0, 1);    // P (TMEM) K-major, V MN-major
      // S_t = Q_t K^T for the key block in ring slot ks
      auto issue_s = [&](int t, int ks) {
        const uint32_t qb = sQ + t * Q_BYTES;
        const uint32_t kb = sK + ks * KV_BYTES;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t chunk = kk >> 2;
          const uint32_t koff = (kk & 3) * 32;
          const uint64_t ad = sdesc_sw128(qb + chunk * Q_HALF + koff, 16, 1024);
          const uint64_t bd = sdesc_sw128(kb + chunk * KV_HALF + koff, 16, 1024);
          mma_f16(tmem + (uint32_t)(t * BKV), ad, bd, idesc_s, kk != 0);
        }
        mma_commit(smem_u32(&B.s_full[t]));
      };
      // O_t += P_t V for the value block in ring slot vs
      auto issue_pv = [&](int t, int vs, bool acc) {
        const uint32_t vb = sV + vs * KV_BYTES;
#pragma unroll
        for (int kk = 0; kk < BKV / 16; ++kk) {
          const uint64_t bd = sdesc_sw128(vb + kk * 16 * 128, KV_HALF, 1024);
          mma_f16_ts(tmem + O_COL + (uint32_t)(t * D), tmem + (uint32_t)(t * BKV + kk * 8), bd,
                     idesc_pv, (acc || kk != 0) ? 1u : 0u);
        }
      };
      // Event loop over the two tiles: for tile t the next step is either
      // PV(t, jp) (its softmax has handed over P, value block jp loaded) or
      // S(t, js) (key block js loaded and PV(t, js - 1), which reads P where
      // S lands, completed).  Whatever is ready is issued, so one tile's
      // wait never holds back the other tile's products.
      const int nt[2] = {n_0, n_1};
      int jp[2] = {0, 0}, js[2] = {0, 0};
      bool pv_pending[2] = {false, false};   // PV(t, jp - 1) issued, not yet seen complete
      int kf = 0, vf = 0;                    // key / value blocks seen loaded
      int k_users[KST], v_users[VST];
      for (int i = 0; i < KST; ++i) k_users[i] = 0;
      for (int i = 0; i < VST; ++i) v_users[i] = 0;
      bool q_ok[2] = {n_0 == 0, n_1 == 0};
      uint32_t idle = 0;
      bool ok = n_kv > 0;
      while (ok) {
        bool progress = false;
        while (kf < n_kv && mbar_test_wait(smem_u32(&B.k_full[kf % KST]), (kf / KST) & 1)) ++kf;
        while (vf < n_kv && mbar_test_wait(smem_u32(&B.v_full[vf % VST]), (vf / VST) & 1)) ++vf;
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          if (!q_ok[t] && mbar_test_wait(smem_u32(&B.q_full[t]), 0)) q_ok[t] = true;
          if (pv_pending[t] && mbar_test_wait(smem_u32(&B.pv_done[t]), (jp[t] - 1) & 1))
            pv_pending[t] = false;
          // S(t, js): block js of the keys (every block a tile reads comes
          // from both tiles' S products; the slot is released after the last)
          if (js[t] < nt[t] && js[t] == jp[t] && !pv_pending[t] && kf > js[t] && q_ok[t]) {
            tc_fence_after();
            const int ks = js[t] % KST;
            issue_s(t, ks);
            const int users = (js[t] < n_0) + (js[t] < n_1);
            if (++k_users[ks] == users) {
              mma_commit(smem_u32(&B.k_empty[ks]));
              k_users[ks] = 0;
            }
            ++js[t];
            progress = true;
          }
          // PV(t, jp): the softmax of tile t has read S and written P
          if (jp[t] < js[t] && vf > jp[t] && mbar_test_wait(smem_u32(&B.p_full[t]), jp[t] & 1)) {
            tc_fence_after();
            const int vs = jp[t] % VST;
            issue_pv(t, vs, jp[t] != 0);
            mma_commit(smem_u32(&B.pv_done[t]));
            const int users = (jp[t] < n_0) + (jp[t] < n_1);
            if (++v_users[vs] == users) {
              mma_commit(smem_u32(&B.v_empty[vs]));
              v_users[vs] = 0;
            }
            ++jp[t];
            pv_pending[t] = true;
            progress = true;
          }
        }
        if (jp[0] == n_0 && jp[1] == n_1) break;
        if (progress) {
          idle = 0;
        } else {
          if (*abort) ok = false;
          if (++idle > kSpinLimit) {
            *abort = 1;
            ok = false;
          }
          if (idle > 4096) __nanosleep(32);
        }
      }
      if (ok) mma_commit(smem_u32(&B.o_full));
    }
  } else {
    // ---------------- softmax warps: 0-3 tile 0, 4-7 tile 1 ----------------
    const int t = warp >> 2;
    const int r = tid & 127;
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t s_col = tmem + lane_base + (uint32_t)(t * BKV);
    const uint32_t o_col = tmem + lane_base + O_COL + (uint32_t)(t * D);
    const int qpos = (qt0 + t) * BQ + r;
    const int nb = t ? n_1 : n_0;
    float m_used = -INFINITY, l_run = 0.f;
    // waits are made warp-uniform: tcgen05.ld/st need the whole warp
    for (int j = 0; j < nb; ++j) {
      if (!__all_sync(0xffffffffu, mbar_wait(smem_u32(&B.s_full[t]), j & 1, abort))) break;
      tc_fence_after();
      float sv[BKV];
      {
        uint32_t r0[32], r1[32], r2[32], r3[32];
        tmem_ld32(s_col, r0);
        tmem_ld32(s_col + 32, r1);
        tmem_ld32(s_col + 64, r2);
        tmem_ld32(s_col + 96, r3);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          sv[i] = __uint_as_float(r0[i]);
          sv[32 + i] = __uint_as_float(r1[i]);
          sv[64 + i] = __uint_as_float(r2[i]);
          sv[96 + i] = __uint_as_float(r3[i]);
        }
      }
      const int kpos0 = j * BKV;
      if (p.causal && kpos0 + BKV - 1 > (qt0 + t) * BQ) {
#pragma unroll
        for (int i = 0; i < BKV; ++i)
          if (kpos0 + i > qpos) sv[i] = -INFINITY;
      }
      // sixteen independent partial maxima / sums keep the dependency chains short
      float m16[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) m16[i] = max3(sv[i], sv[16 + i], sv[32 + i]);
#pragma unroll
      for (int i = 48; i < BKV; i += 32) {
#pragma unroll
        for (int k = 0; k < 16; ++k) m16[k] = max3(m16[k], sv[i + k], sv[i + 16 + k]);
      }
#pragma unroll
      for (int k = 0; k < 16; ++k) m16[k] = fmaxf(m16[k], sv[112 + k]);
#pragma unroll
      for (int h = 8; h >= 1; h >>= 1)
#pragma unroll
        for (int i = 0; i < h; ++i) m16[i] = fmaxf(m16[i], m16[i + h]);
      const float mx = m16[0] * p.scale_log2;
      const float m_new = fmaxf(m_used, mx);
      float factor = 1.f;
      bool rescale = false;
      if (m_used == -INFINITY || m_new > m_used + RESCALE_THRESHOLD) {
        factor = (m_used == -INFINITY) ? 0.f : ex2(m_used - m_new);
        rescale = m_used != -INFINITY;
        l_run *= factor;
        m_used = m_new;
      }
      const float msub = (m_used == -INFINITY) ? 0.f : m_used;
      // P over the first 64 columns of the S buffer (already read above); the
      // row sum adds P in f16 pairs four at a time (each P <= 2^8, so a
      // partial stays below 2^11 and keeps 2^-11 relative precision), then
      // in f32
      __half2 h16[16];
#pragma unroll
      for (int qtr = 0; qtr < 4; ++qtr) {
        uint32_t ph[16];
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const int c = 32 * qtr + i;
          const float xa = fmaf(sv[c], p.scale_log2, -msub);
          const float xb = fmaf(sv[c + 1], p.scale_log2, -msub);
          // three pairs in eight on the FMA pipe, the rest on MUFU
          ph[i / 2] = ((i / 2) % 8 == 1 || (i / 2) % 8 == 4 || (i / 2) % 8 == 6)
                          ? pack_f16x2(exp2_fma(xa), exp2_fma(xb))
                          : ex2_pair(xa, xb);
          const __half2 v2 = *reinterpret_cast<const __half2*>(&ph[i / 2]);
          const int slot = (c / 2) & 15;
          h16[slot] = (c < 32) ? v2 : __hadd2(h16[slot], v2);
        }
        tmem_st16(s_col + (uint32_t)(16 * qtr), ph);
      }
      float s16[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float2 f = __half22float2(h16[i]);
        s16[i] = f.x + f.y;
      }
#pragma unroll
      for (int h = 8; h >= 1; h >>= 1)
#pragma unroll
        for (int i = 0; i < h; ++i) s16[i] += s16[i + h];
      l_run += s16[0];
      // O_t rows move only when a row's max moved: the PV product of block
      // j-1 was issued before S_t of block j, so it has landed
      if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll 1
        for (int c = 0; c < D; c += 32) {
          uint32_t o[32];
          tmem_ld32(o_col + c, o);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * factor);
          tmem_st32(o_col + c, o);
        }
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(smem_u32(&B.p_full[t]));
    }
    const bool done = nb > 0 && !*abort && mbar_wait(smem_u32(&B.o_full), 0, abort);
    if (__all_sync(0xffffffffu, done)) {
      tc_fence_after();
      const float inv = 1.f / l_run;
      __half* orow = p.o + (head * p.seq + qpos) * p.row_stride;
#pragma unroll 1
      for (int c = 0; c < D; c += 32) {
        uint32_t o[32];
        tmem_ld32(o_col + c, o);
        tmem_ld_wait();
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint4 v;
          v.x = pack_h2(__uint_as_float(o[8 * q + 0]) * inv, __uint_as_float(o[8 * q + 1]) * inv);
          v.y = pack_h2(__uint_as_float(o[8 * q + 2]) * inv, __uint_as_float(o[8 * q + 3]) * inv);
          v.z = pack_h2(__uint_as_float(o[8 * q + 4]) * inv, __uint_as_float(o[8 * q + 5]) * inv);
          v.w = pack_h2(__uint_as_float(o[8 * q + 6]) * inv, __uint_as_float(o[8 * q + 7]) * inv);
          *reinterpret_cast<uint4*>(orow + c + 8 * q) = v;
        }
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
  if (tid == 0 && B.abort_flag) atomicOr(p.status, KTIR_STATUS_TIMEOUT);
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
  // the row max is taken before scaling, which needs a positive scale
  if (d->d != D || d->seq % BQ || d->bh < 1 || d->row_stride < D || (d->row_stride & 7) ||
      !(d->scale > 0.f))
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
    // the tiles and rings take most of an SM's shared memory
    if (cudaFuncSetAttribute(k_fmha_tcgen05, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             SMEM_BYTES) != cudaSuccess ||
        cudaFuncSetAttribute(k_fmha_tcgen05, cudaFuncAttributePreferredSharedMemoryCarveout,
                             cudaSharedmemCarveoutMaxShared) != cudaSuccess)
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
  p.n_pairs = (p.n_qtiles + 1) / 2;
  p.status = d->status;
  dim3 grid((unsigned)p.n_pairs, (unsigned)d->bh);
  k_fmha_tcgen05<<<grid, THREADS, SMEM_BYTES, static_cast<cudaStream_t>(stream)>>>(tq, tk, tv, p);
  return cudaGetLastError() == cudaSuccess ? KTIR_OK : KTIR_ERR_CUDA;
}
