// Causal / full flash attention on the 5th-generation tensor cores.
//
// Q, K, V, O are f16 [bh*seq, 128] row-major (one head = seq consecutive
// rows).  One CTA owns 128 query rows of one head and walks the key blocks of
// 64 rows with three warp roles that meet only at mbarriers; two CTAs share
// an SM, so while one CTA's softmax warps work the other's keep the tensor
// cores busy:
//   warps 4, 6 (TMA)  warp 4 loads Q once and K_j, warp 6 loads V_j, each into
//                     its own 2-stage ring, every slot refilled as soon as the
//                     MMA that read it completes
//   warp 5 (MMA)      S_j = Q K_j^T (M=128 N=64 K=128) into TMEM S buffer
//                     j & 1; as soon as the softmax warps hand over P_j it
//                     issues O += Phi_j V_j + Plo_j V_j (M=128 N=128 K=2x64,
//                     P read from TMEM) and then S_{j+2} into the same TMEM
//                     buffer: the tensor pipe runs one thread's tcgen05.mma in
//                     issue order, so the PV product has read P_j before
//                     S_{j+2} is written over it; the next two S blocks are
//                     always computed ahead of the softmax
//   warps 0-3         thread t owns query row t = TMEM lane t: tcgen05.ld of
//                     S_j, masked max of x = s * scale * log2(e), P = 2^(x - m)
//                     in f32, split into Phi = f16(P) and Plo = f16(P - Phi),
//                     written with tcgen05.st over S_j's TMEM columns (S_j is
//                     in registers by then): Phi in columns 0..31, Plo in
//                     32..63, two f16 per column; row sum l in f32.  The two
//                     f16 halves
//                     carry P to about 22 bits, so the PV product keeps the
//                     f32 probabilities of the reference's online softmax
//                     (an f16 P alone moves outputs that cancel by more than
//                     1e-2 of their value)
// TMEM (256 columns): S0 0..63, S1 64..127, O 128..255.  The running max m
// only moves when a row's max exceeds it by more than 2^8; then the softmax
// warp waits for the previous PV and rescales its O rows in TMEM
// (warp-uniform), otherwise O and l keep sharing m.
// Shared memory (Q, K and V rings, mbarriers) fits two CTAs per SM with 896
// bytes for aligning the tiles to the 1024 bytes the 128-byte swizzle needs; a
// CTA whose window cannot be aligned within that reports KTIR_STATUS_TIMEOUT
// and does nothing.  With P in TMEM no shared memory carries P: the tensor
// pipe reads only Q, K and V there.
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
constexpr int BQ = 128;         // query rows per CTA
constexpr int BKV = 64;         // key rows per block
constexpr int KST = 2;          // K ring stages
constexpr int VST = 2;          // V ring stages
constexpr int THREADS = 224;
constexpr int HEAD_GROUP = 16;   // heads per group of the CTA order (16 MiB of K/V at S=2048)
constexpr int Q_HALF = BQ * 64 * 2;             // 16 KiB: 128 rows x 64 columns
constexpr int Q_BYTES = 2 * Q_HALF;             // 32 KiB
constexpr int KV_HALF = BKV * 64 * 2;           // 8 KiB: 64 rows x 64 columns
constexpr int KV_BYTES = 2 * KV_HALF;           // 16 KiB: 64 rows x 128 columns
constexpr int TILE_BYTES = Q_BYTES + (KST + VST) * KV_BYTES;
constexpr int ALIGN_SLACK = 896;
constexpr int MAX_TILES = 32;   // 128-row tiles of a sequence in a partial call (seq <= 4096)

struct Bars {
  uint64_t q_full;
  uint64_t k_full[KST], k_empty[KST];
  uint64_t v_full[VST], v_empty[VST];
  uint64_t s_full[2];
  // P_j handed over / PV_j complete, one barrier per parity of j: a waiter
  // names the phase it wants by (j >> 1) & 1, which stays unambiguous because
  // a barrier's next phase (j + 2) needs this warp's own later work
  uint64_t p_full[2], pv_done[2];
  uint32_t tmem_base;
  int abort_flag;
};
constexpr int SMEM_BYTES = TILE_BYTES + (int)sizeof(Bars) + ALIGN_SLACK;
static_assert(2 * (SMEM_BYTES + 1024) <= 228 * 1024, "two CTAs per SM");

constexpr uint32_t TMEM_COLS = 256;
constexpr uint32_t O_COL = 128;
constexpr float RESCALE_THRESHOLD = 8.0f;       // log2 units
// P is evaluated as 2^(x - m + P_OFFSET): the row's largest P lies in
// [2^7, 2^15] (below the f16 maximum), and P down to 2^-14 * 2^-7 of the row's
// largest stays a normal f16 in both halves; O and l carry the same factor
constexpr float P_OFFSET = 7.0f;

struct FmhaParams {
  __half* o;
  long long seq;
  long long row_stride;
  float scale_log2;   // scale * log2(e)
  int causal;
  int n_qtiles;       // query tiles per head this launch computes
  long long bh;
  int* status;
  // partial calls (part != 0): the query tiles are qtiles[0..n_qtiles), key
  // tile kt lives at row ((kv_owner[kt] * bh + head) * kv_tiles + kv_local[kt])
  // * 128 of K and V, only key tiles in key_mask are added, and the softmax
  // state of each (head, query tile) is carried between calls in o_acc / ml
  int part;
  int flags;          // bit 0: first call (no carried state); bit 1: last call (write O)
  int kv_tiles;
  unsigned key_mask;
  float* o_acc;       // per (head, query tile): O as [128 columns][128 rows] f32
  float2* ml;         // per (head, query tile): (running max, row sum) per row
  unsigned char qtiles[MAX_TILES];
  unsigned char kv_owner[MAX_TILES];
  unsigned char kv_local[MAX_TILES];
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
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

__global__ void __launch_bounds__(THREADS, 2)
    k_fmha_tcgen05(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                   const __grid_constant__ CUtensorMap tv, const __grid_constant__ FmhaParams p) {
  extern __shared__ uint8_t smem_raw[];
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  if (base - raw > (uint32_t)ALIGN_SLACK) {
    if (tid == 0) atomicOr(p.status, KTIR_STATUS_TIMEOUT);
    return;   // uniform: every thread sees the same window
  }
  const uint32_t sQ = base;
  const uint32_t sK = base + Q_BYTES;
  const uint32_t sV = sK + KST * KV_BYTES;
  Bars& B = *reinterpret_cast<Bars*>(smem_raw + (base - raw) + TILE_BYTES);
  volatile int* abort = &B.abort_flag;

  // CTA order (blocks are dispatched in index order): groups of HEAD_GROUP
  // heads, and within a group every head's heaviest query tile, then every
  // head's next one, ... so the grid ends on the lightest tiles while the
  // CTAs in flight share the K/V of a few heads in L2
  const long long lin = blockIdx.x;
  const long long gsize = (long long)HEAD_GROUP * p.n_qtiles;
  const long long grp = lin / gsize;
  const long long heads = p.bh - grp * HEAD_GROUP < HEAD_GROUP ? p.bh - grp * HEAD_GROUP : HEAD_GROUP;
  const long long w = lin - grp * gsize;
  const int qi = p.n_qtiles - 1 - (int)(w / heads);
  const int qt = p.part ? (int)p.qtiles[qi] : qi;
  const long long head = grp * HEAD_GROUP + w % heads;
  const long long row0 = head * p.seq + (long long)qt * BQ;
  const int q0 = qt * BQ;
  const bool first = !p.part || (p.flags & 1);
  const bool last = !p.part || (p.flags & 2);

  if (tid == 0) {
    B.abort_flag = 0;
    mbar_init(smem_u32(&B.q_full), 1);
    for (int s = 0; s < KST; ++s) {
      mbar_init(smem_u32(&B.k_full[s]), 1);
      mbar_init(smem_u32(&B.k_empty[s]), 1);
    }
    for (int s = 0; s < VST; ++s) {
      mbar_init(smem_u32(&B.v_full[s]), 1);
      mbar_init(smem_u32(&B.v_empty[s]), 1);
    }
    for (int b = 0; b < 2; ++b) mbar_init(smem_u32(&B.s_full[b]), 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&B.p_full[b]), BQ);
      mbar_init(smem_u32(&B.pv_done[b]), 1);
    }
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
  // partial calls: the key tiles this CTA adds are those of the mask up to
  // its own query tile when causal; each gives two key blocks, in order
  const unsigned n_seq_tiles = (unsigned)(p.seq / BQ);
  unsigned kmask = p.key_mask & (n_seq_tiles >= 32 ? ~0u : ((1u << n_seq_tiles) - 1u));
  if (p.causal && qt < 31) kmask &= (2u << qt) - 1u;
  const int n_kv = p.part ? 2 * __popc(kmask) : (p.causal ? (q0 + BQ) / BKV : (int)(p.seq / BKV));
  // key block j of this CTA: its index in the sequence and its row in K / V
  auto kv_block = [&](int j) -> int {
    return p.part ? 2 * (int)__fns(kmask, 0, (j >> 1) + 1) + (j & 1) : j;
  };
  auto kv_row = [&](int j) -> int {
    if (!p.part) return (int)(head * p.seq) + j * BKV;
    const int kt = (int)__fns(kmask, 0, (j >> 1) + 1);
    return (int)((((long long)p.kv_owner[kt] * p.bh + head) * p.kv_tiles + p.kv_local[kt]) * BQ) +
           (j & 1) * BKV;
  };

  if (warp == 4 || warp == 6) {
    // ---------------- TMA producers: warp 4 Q and K, warp 6 V ----------------
    if (lane == 0) {
      const bool is_k = warp == 4;
      if (is_k) {
        tma_prefetch_desc(&tq);
        tma_prefetch_desc(&tk);
        const uint32_t qb = smem_u32(&B.q_full);
        mbar_arrive_expect_tx(qb, Q_BYTES);
        tma_load_2d(sQ, &tq, qb, 0, (int)row0);
        tma_load_2d(sQ + Q_HALF, &tq, qb, 64, (int)row0);
      } else {
        tma_prefetch_desc(&tv);
      }
      const CUtensorMap* map = is_k ? &tk : &tv;
      uint64_t* full = is_k ? B.k_full : B.v_full;
      uint64_t* empty = is_k ? B.k_empty : B.v_empty;
      const int stages = is_k ? KST : VST;
      const uint32_t ring = is_k ? sK : sV;
      for (int j = 0; j < n_kv && !*abort; ++j) {
        const int kr = kv_row(j);
        const int st = j % stages;
        if (j >= stages && !mbar_wait(smem_u32(&empty[st]), ((j / stages) - 1) & 1, abort)) break;
        const uint32_t fb = smem_u32(&full[st]);
        const uint32_t dst = ring + st * KV_BYTES;
        mbar_arrive_expect_tx(fb, KV_BYTES);
        tma_load_2d(dst, map, fb, 0, kr);
        tma_load_2d(dst + KV_HALF, map, fb, 64, kr);
      }
    }
  } else if (warp == 5) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_f16(BQ, BKV, 0, 0);   // Q, K both K-major
      constexpr uint32_t idesc_pv = idesc_f16(BQ, D, 0, 1);    // P K-major, V MN-major
      auto issue_s = [&](int j) -> bool {
        const int ks = j % KST;
        if (!mbar_wait(smem_u32(&B.k_full[ks]), (j / KST) & 1, abort)) return false;
        tc_fence_after();
        const uint32_t kb = sK + ks * KV_BYTES;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t chunk = kk >> 2;
          const uint32_t koff = (kk & 3) * 32;
          const uint64_t ad = sdesc_sw128(sQ + chunk * Q_HALF + koff, 16, 1024);
          const uint64_t bd = sdesc_sw128(kb + chunk * KV_HALF + koff, 16, 1024);
          mma_f16(tmem + (uint32_t)((j & 1) * BKV), ad, bd, idesc_s, kk != 0);
        }
        mma_commit(smem_u32(&B.s_full[j & 1]));
        mma_commit(smem_u32(&B.k_empty[ks]));
        return true;
      };
      bool ok = mbar_wait(smem_u32(&B.q_full), 0, abort);
      for (int j = 0; ok && j < 2 && j < n_kv; ++j) ok = issue_s(j);
      for (int j = 0; ok && j < n_kv; ++j) {
        // softmax j has read S_j and written P_j
        if (!mbar_wait(smem_u32(&B.p_full[j & 1]), (j >> 1) & 1, abort)) break;
        const int vs = j % VST;
        if (!mbar_wait(smem_u32(&B.v_full[vs]), (j / VST) & 1, abort)) break;
        tc_fence_after();
        const uint32_t vb = sV + vs * KV_BYTES;
        // O += Phi V + Plo V: A from TMEM (S_j's columns: Phi 0..31, Plo
        // 32..63, 8 columns per 16 keys); the K steps of both halves read the
        // same V rows
        const uint32_t pbuf = tmem + (uint32_t)((j & 1) * BKV);
#pragma unroll
        for (int kk = 0; kk < 2 * (BKV / 16); ++kk) {
          const uint32_t at = pbuf + (uint32_t)((kk >> 2) * 32 + (kk & 3) * 8);
          const uint64_t bd = sdesc_sw128(vb + (kk & 3) * 16 * 128, KV_HALF, 1024);
          // a partial call after the first adds onto the carried O
          mma_f16_ts(tmem + O_COL, at, bd, idesc_pv, (j | kk) != 0 || !first);
        }
        mma_commit(smem_u32(&B.pv_done[j & 1]));
        mma_commit(smem_u32(&B.v_empty[vs]));
        if (j + 2 < n_kv) ok = issue_s(j + 2);
      }
    }
  } else {
    // ---------------- softmax warps 0-3 ----------------
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    const int qpos = q0 + tid;
    float m_used = -INFINITY, l_run = 0.f;
    // carried state of a partial call ([128 columns][128 rows] f32, so a warp's
    // 32 rows of one column are one 128-byte line)
    const long long slot = head * p.n_qtiles + qi;
    float* oacc = p.part ? p.o_acc + slot * (long long)(BQ * D) : nullptr;
    float2* ml = p.part ? p.ml + slot * BQ : nullptr;
    if (!first) {
      const float2 st = ml[tid];
      m_used = st.x;
      l_run = st.y;
      if (n_kv > 0) {
        // O into TMEM before P_0 is handed over (the first PV adds onto it)
#pragma unroll 1
        for (int c = 0; c < D; c += 32) {
          uint32_t r[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(oacc[(c + i) * BQ + tid]);
          tmem_st32_wait(tmem + lane_base + O_COL + c, r);
        }
      }
    }
    // waits are made warp-uniform: tcgen05.ld/st need the whole warp
    for (int j = 0; j < n_kv; ++j) {
      if (!__all_sync(0xffffffffu, mbar_wait(smem_u32(&B.s_full[j & 1]), (j >> 1) & 1, abort)))
        break;
      tc_fence_after();
      float sv[BKV];
      {
        uint32_t rs[BKV];
        tmem_ld64_wait(tmem + lane_base + (uint32_t)((j & 1) * BKV), rs);
#pragma unroll
        for (int i = 0; i < BKV; ++i) sv[i] = __uint_as_float(rs[i]);
      }
      const int kpos0 = kv_block(j) * BKV;
      const bool diag = p.causal && kpos0 + BKV - 1 > q0;
      if (diag) {
#pragma unroll
        for (int i = 0; i < BKV; ++i)
          if (kpos0 + i > qpos) sv[i] = -INFINITY;
      }
      // eight independent partial maxima / sums keep the dependency chains short
      float m8[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) m8[i] = fmaxf(sv[i], sv[8 + i]);
#pragma unroll
      for (int i = 16; i < BKV; i += 16) {
#pragma unroll
        for (int k = 0; k < 8; ++k) m8[k] = max3(m8[k], sv[i + k], sv[i + 8 + k]);
      }
#pragma unroll
      for (int h = 4; h >= 1; h >>= 1)
#pragma unroll
        for (int i = 0; i < h; ++i) m8[i] = fmaxf(m8[i], m8[i + h]);
      const float mx = m8[0] * p.scale_log2;
      const float m_new = fmaxf(m_used, mx);
      float factor = 1.f;
      bool rescale = false;
      if (m_used == -INFINITY || m_new > m_used + RESCALE_THRESHOLD) {
        factor = (m_used == -INFINITY) ? 0.f : ex2(m_used - m_new);
        rescale = m_used != -INFINITY;
        l_run *= factor;
        m_used = m_new;
      }
      const float msub = (m_used == -INFINITY) ? 0.f : m_used - P_OFFSET;
      uint32_t ph[BKV / 2], pl[BKV / 2];
      // P in f32, its f16 head and the f16 rounding of the remainder; the row
      // sum adds the f32 P in eight partial sums
      float s8[8];
#pragma unroll
      for (int i = 0; i < BKV; i += 2) {
        const float a = ex2(fmaf(sv[i], p.scale_log2, -msub));
        const float b = ex2(fmaf(sv[i + 1], p.scale_log2, -msub));
        ph[i / 2] = pack_h2(a, b);
        const float2 hf = __half22float2(*reinterpret_cast<const __half2*>(&ph[i / 2]));
        pl[i / 2] = pack_h2(a - hf.x, b - hf.y);
        s8[(i / 2) & 7] = (i < 16) ? a + b : s8[(i / 2) & 7] + (a + b);
      }
#pragma unroll
      for (int h = 4; h >= 1; h >>= 1)
#pragma unroll
        for (int i = 0; i < h; ++i) s8[i] += s8[i + h];
      l_run += s8[0];
      // a rescale of O waits for PV_{j-1} to finish adding into O (at j = 0
      // of a call that carries state, O holds the carried values and may need
      // the same rescale)
      if ((j >= 1 || !first) && __any_sync(0xffffffffu, rescale)) {
        if (j >= 1) {
          const bool ok = __all_sync(
              0xffffffffu, mbar_wait(smem_u32(&B.pv_done[(j - 1) & 1]), ((j - 1) >> 1) & 1, abort));
          tc_fence_after();
          if (!ok) break;
        }
        {
#pragma unroll 1
          for (int c = 0; c < D; c += 32) {
            uint32_t r[32];
            tmem_ld32_wait(tmem + lane_base + O_COL + c, r);
#pragma unroll
            for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * factor);
            tmem_st32_wait(tmem + lane_base + O_COL + c, r);
          }
        }
      }
      // Phi_j, Plo_j over S_j's columns of this warp's lanes (S_j is in
      // registers); the stores complete before the arrival (tcgen05.wait::st)
      const uint32_t pcol = tmem + lane_base + (uint32_t)((j & 1) * BKV);
      tmem_st32_wait(pcol, ph);
      tmem_st32_wait(pcol + 32, pl);
      tc_fence_before();
      mbar_arrive(smem_u32(&B.p_full[j & 1]));
      // no wait for PV_{j-1} here: S_{j+1}, which this warp waits for next, is
      // issued after PV_{j-1} by the same thread, so its completion implies
      // PV_{j-1}'s (and P_{j+1} may then overwrite P_{j-1})
    }
    const bool done =
        !*abort && (n_kv == 0 || mbar_wait(smem_u32(&B.pv_done[(n_kv - 1) & 1]),
                                           ((n_kv - 1) >> 1) & 1, abort));
    // O of this CTA: from TMEM, or, with no key block in this call, the
    // carried state (zero on a first call)
    auto o_cols = [&](int c, uint32_t (&r)[32]) {
      if (n_kv > 0) {
        tmem_ld32_wait(tmem + lane_base + O_COL + c, r);
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) r[i] = first ? 0u : __float_as_uint(oacc[(c + i) * BQ + tid]);
      }
    };
    if (__all_sync(0xffffffffu, done) && !last && (n_kv > 0 || first)) {
      // carry the state to the next call
      tc_fence_after();
#pragma unroll 1
      for (int c = 0; c < D; c += 32) {
        uint32_t r[32];
        o_cols(c, r);
#pragma unroll
        for (int i = 0; i < 32; ++i) oacc[(c + i) * BQ + tid] = __uint_as_float(r[i]);
      }
      ml[tid] = make_float2(m_used, l_run);
    } else if (__all_sync(0xffffffffu, done) && last) {
      tc_fence_after();
      const float inv = 1.f / l_run;
      __half* orow = p.o + (row0 + tid) * p.row_stride;
#pragma unroll 1
      for (int c = 0; c < D; c += 32) {
        uint32_t r[32];
        o_cols(c, r);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint4 v;
          v.x = pack_h2(__uint_as_float(r[8 * q + 0]) * inv, __uint_as_float(r[8 * q + 1]) * inv);
          v.y = pack_h2(__uint_as_float(r[8 * q + 2]) * inv, __uint_as_float(r[8 * q + 3]) * inv);
          v.z = pack_h2(__uint_as_float(r[8 * q + 4]) * inv, __uint_as_float(r[8 * q + 5]) * inv);
          v.w = pack_h2(__uint_as_float(r[8 * q + 6]) * inv, __uint_as_float(r[8 * q + 7]) * inv);
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

namespace {

int launch_fmha(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                const FmhaParams& p, cudaStream_t stream) {
  static bool attr = false;
  if (!attr) {
    // two CTAs per SM need the whole shared-memory carve-out
    if (cudaFuncSetAttribute(k_fmha_tcgen05, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             SMEM_BYTES) != cudaSuccess ||
        cudaFuncSetAttribute(k_fmha_tcgen05, cudaFuncAttributePreferredSharedMemoryCarveout,
                             cudaSharedmemCarveoutMaxShared) != cudaSuccess)
      return ktir_set_error(KTIR_ERR_CUDA, "attention: shared-memory attributes refused");
    attr = true;
  }
  dim3 grid((unsigned)((long long)p.n_qtiles * p.bh));   // rows / 128 < 2^31
  k_fmha_tcgen05<<<grid, THREADS, SMEM_BYTES, stream>>>(tq, tk, tv, p);
  return cudaGetLastError() == cudaSuccess
             ? KTIR_OK : ktir_set_error(KTIR_ERR_CUDA, "attention: launch failed");
}

bool aligned16(const void* a) { return (reinterpret_cast<uintptr_t>(a) & 15) == 0; }

}  // namespace

extern "C" int ktir_fmha_f16(const KtirFmhaDesc* d, void* stream) {
  if (!d || !d->q || !d->k || !d->v || !d->o || !d->status)
    return ktir_set_error(KTIR_ERR_ARG, "ktir_fmha_f16: null argument");
  // the row max is taken before scaling, which needs a positive scale
  if (d->d != D || d->seq % BQ || d->bh < 1 || d->row_stride < D || (d->row_stride & 7) ||
      !(d->scale > 0.f))
    return ktir_set_error(KTIR_ERR_UNSUPPORTED,
                          "ktir_fmha_f16: needs d = 128, seq a multiple of 128, a row stride "
                          "of at least 128 in multiples of 8, and a positive scale");
  if (!aligned16(d->q) || !aligned16(d->k) || !aligned16(d->v) || !aligned16(d->o))
    return ktir_set_error(KTIR_ERR_UNSUPPORTED, "ktir_fmha_f16: operands not 16-byte aligned");
  const long long rows = d->bh * d->seq;
  if (rows > 0x7fffffffLL) return ktir_set_error(KTIR_ERR_UNSUPPORTED, "ktir_fmha_f16: too many rows");
  CUtensorMap tq, tk, tv;
  if (!make_map(&tq, d->q, rows, d->row_stride, BQ) || !make_map(&tk, d->k, rows, d->row_stride, BKV) ||
      !make_map(&tv, d->v, rows, d->row_stride, BKV))
    return ktir_set_error(KTIR_ERR_CUDA, "ktir_fmha_f16: tensor map encoding failed");
  FmhaParams p = {};
  p.o = static_cast<__half*>(d->o);
  p.seq = d->seq;
  p.row_stride = d->row_stride;
  p.scale_log2 = d->scale * 1.4426950408889634f;
  p.causal = d->causal;
  p.n_qtiles = (int)(d->seq / BQ);
  p.bh = d->bh;
  p.status = d->status;
  return launch_fmha(tq, tk, tv, p, static_cast<cudaStream_t>(stream));
}

extern "C" int ktir_fmha_f16_part(const KtirFmhaPartDesc* d, void* stream) {
  if (!d || !d->q || !d->k || !d->v || !d->o || !d->status)
    return ktir_set_error(KTIR_ERR_ARG, "ktir_fmha_f16_part: null argument");
  const bool first = d->flags & 1, last = d->flags & 2;
  if ((!first || !last) && (!d->o_acc || !d->ml))
    return ktir_set_error(KTIR_ERR_ARG, "ktir_fmha_f16_part: a partial step needs o_acc and ml");
  if (d->d != D || d->seq % BQ || d->seq > MAX_TILES * BQ || d->bh < 1 || !(d->scale > 0.f))
    return ktir_set_error(KTIR_ERR_UNSUPPORTED,
                          "ktir_fmha_f16_part: needs d = 128, seq a multiple of 128 up to "
                          "4096, and a positive scale");
  const int n_tiles = (int)(d->seq / BQ);
  if (d->n_qtiles < 1 || d->n_qtiles > n_tiles || d->kv_tiles < 1 || d->kv_tiles > n_tiles)
    return ktir_set_error(KTIR_ERR_UNSUPPORTED, "ktir_fmha_f16_part: n_qtiles or kv_tiles out of range");
  if (!aligned16(d->q) || !aligned16(d->k) || !aligned16(d->v) || !aligned16(d->o) ||
      !aligned16(d->o_acc) || !aligned16(d->ml))
    return ktir_set_error(KTIR_ERR_UNSUPPORTED, "ktir_fmha_f16_part: buffers not 16-byte aligned");
  const long long rows = d->bh * d->seq;
  if (rows > 0x7fffffffLL || d->kv_rows < 1 || d->kv_rows > 0x7fffffffLL)
    return ktir_set_error(KTIR_ERR_UNSUPPORTED, "ktir_fmha_f16_part: row count out of range");
  for (int i = 0; i < d->n_qtiles; ++i)
    if (d->qtiles[i] < 0 || d->qtiles[i] >= n_tiles)
      return ktir_set_error(KTIR_ERR_UNSUPPORTED, "ktir_fmha_f16_part: query tile out of range");
  // every key tile the mask names must lie inside K / V
  for (int kt = 0; kt < n_tiles; ++kt) {
    if (!((d->key_mask >> kt) & 1u)) continue;
    if (d->kv_owner[kt] < 0 || d->kv_local[kt] < 0 || d->kv_local[kt] >= d->kv_tiles)
      return ktir_set_error(KTIR_ERR_UNSUPPORTED, "ktir_fmha_f16_part: key tile place out of range");
    const long long end =
        (((long long)d->kv_owner[kt] * d->bh + d->bh - 1) * d->kv_tiles + d->kv_local[kt] + 1) * BQ;
    if (end > d->kv_rows)
      return ktir_set_error(KTIR_ERR_UNSUPPORTED, "ktir_fmha_f16_part: key tile beyond kv_rows");
  }
  CUtensorMap tq, tk, tv;
  if (!make_map(&tq, d->q, rows, D, BQ) || !make_map(&tk, d->k, d->kv_rows, D, BKV) ||
      !make_map(&tv, d->v, d->kv_rows, D, BKV))
    return ktir_set_error(KTIR_ERR_CUDA, "ktir_fmha_f16_part: tensor map encoding failed");
  FmhaParams p = {};
  p.o = static_cast<__half*>(d->o);
  p.seq = d->seq;
  p.row_stride = D;
  p.scale_log2 = d->scale * 1.4426950408889634f;
  p.causal = d->causal;
  p.n_qtiles = d->n_qtiles;
  p.bh = d->bh;
  p.status = d->status;
  p.part = 1;
  p.flags = d->flags & 3;
  p.kv_tiles = d->kv_tiles;
  p.key_mask = d->key_mask;
  p.o_acc = d->o_acc;
  p.ml = reinterpret_cast<float2*>(d->ml);
  for (int i = 0; i < MAX_TILES; ++i) {
    p.qtiles[i] = d->qtiles[i];
    p.kv_owner[i] = d->kv_owner[i];
    p.kv_local[i] = d->kv_local[i];
  }
  return launch_fmha(tq, tk, tv, p, static_cast<cudaStream_t>(stream));
}
