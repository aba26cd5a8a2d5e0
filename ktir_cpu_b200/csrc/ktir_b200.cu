// B200 execution backend for KTIR: C ABI + CUDA-core kernels.
//
//  k_ew            fused elementwise bytecode over an N-d iteration space,
//                  batched over units (cores x loop iterations)
//  k_softmax_rows  fused row softmax, one warp per row, f16 rows moved with
//                  128-bit loads; max and sum fold in the reference's
//                  pairwise-halving order (ktir_cpu/dialects/linalg_ops.py:86-133)
//  k_rmw_count / k_rmw_apply
//                  indirect row gather -> f -> scatter over many units with the
//                  reference's sequential-unit semantics: a row named by m
//                  units ends as f applied m times (f16 rounding every time)
//  k_reduce, k_matmul, k_offsets, k_indirect_*
//                  generic-path kernels for programs no fused kernel covers
#include <cuda_runtime.h>
#include <utility>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include "ew_ops.cuh"

using namespace ktir;

// ---------------------------------------------------------------------------
// error plumbing
// ---------------------------------------------------------------------------
static thread_local char g_err[512] = "";

static int set_err(int code, const char* msg) {
  snprintf(g_err, sizeof(g_err), "%s", msg);
  return code;
}

static int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    snprintf(g_err, sizeof(g_err), "%s: %s", what, cudaGetErrorString(e));
    return KTIR_ERR_CUDA;
  }
  return KTIR_OK;
}

// shared with the other translation units of the library
int ktir_set_error(int code, const char* msg) { return set_err(code, msg); }

extern "C" int ktir_version(void) { return 100; }
extern "C" const char* ktir_last_error(void) { return g_err; }

extern "C" int ktir_copy_blocks(void* dst, int64_t dst_pitch, const void* src, int64_t src_pitch,
                                int64_t width, int64_t rows, void* stream) {
  if (!dst || !src || width < 0 || rows < 0 || dst_pitch < width || src_pitch < width)
    return set_err(KTIR_ERR_ARG, "ktir_copy_blocks: bad arguments");
  if (width == 0 || rows == 0) return KTIR_OK;
  cudaError_t e = cudaMemcpy2DAsync(dst, (size_t)dst_pitch, src, (size_t)src_pitch, (size_t)width,
                                    (size_t)rows, cudaMemcpyDeviceToDevice, (cudaStream_t)stream);
  if (e != cudaSuccess) return set_err(KTIR_ERR_CUDA, cudaGetErrorString(e));
  return KTIR_OK;
}
extern "C" int ktir_device_count(int* count) {
  cudaError_t e = cudaGetDeviceCount(count);
  if (e != cudaSuccess) return set_err(KTIR_ERR_CUDA, cudaGetErrorString(e));
  return KTIR_OK;
}

// Programmatic dependent launch: the kernel may be scheduled while the
// previous kernel on the stream drains; it runs pdl_prologue() before touching
// global memory, which waits for that kernel to complete and its writes to be
// visible, then lets the next kernel be scheduled the same way.
__device__ __forceinline__ void pdl_prologue() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename... KArgs, typename... Args>
static cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t s, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

static inline int grid_x(int64_t work, int threads, int cap) {
  int64_t g = (work + threads - 1) / threads;
  if (g < 1) g = 1;
  if (g > cap) g = cap;
  return (int)g;
}

// dst = a - b (sub != 0) or a + b, byte by byte modulo 256, four bytes per
// SIMD op and sixteen per thread where all three pointers allow it
__global__ void __launch_bounds__(256) k_bytes(uint8_t* __restrict__ dst, const uint8_t* __restrict__ a,
                                               const uint8_t* __restrict__ b, int64_t n, int sub) {
  const int64_t i0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 16;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x * 16;
  const bool vec = ((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(a) |
                     reinterpret_cast<uintptr_t>(b)) & 15) == 0;
  for (int64_t i = i0; i < n; i += stride) {
    if (vec && i + 16 <= n) {
      const uint4 x = *reinterpret_cast<const uint4*>(a + i);
      const uint4 y = *reinterpret_cast<const uint4*>(b + i);
      uint4 z;
      z.x = sub ? __vsub4(x.x, y.x) : __vadd4(x.x, y.x);
      z.y = sub ? __vsub4(x.y, y.y) : __vadd4(x.y, y.y);
      z.z = sub ? __vsub4(x.z, y.z) : __vadd4(x.z, y.z);
      z.w = sub ? __vsub4(x.w, y.w) : __vadd4(x.w, y.w);
      *reinterpret_cast<uint4*>(dst + i) = z;
    } else {
      for (int64_t k = i; k < n && k < i + 16; ++k)
        dst[k] = (uint8_t)(sub ? a[k] - b[k] : a[k] + b[k]);
    }
  }
}

extern "C" int ktir_bytes_delta(void* dst, const void* a, const void* b, int64_t n, int32_t subtract,
                                void* stream) {
  if (!dst || !a || !b || n < 0) return set_err(KTIR_ERR_ARG, "ktir_bytes_delta: bad arguments");
  if (n == 0) return KTIR_OK;
  k_bytes<<<grid_x((n + 15) / 16, 256, 148 * 16), 256, 0, (cudaStream_t)stream>>>(
      (uint8_t*)dst, (const uint8_t*)a, (const uint8_t*)b, n, subtract ? 1 : 0);
  return check_launch("ktir_bytes_delta");
}

// The K/V rows of the 128-row tiles in tile_mask, every head, packed as
// [K | V][head][i-th tile of the mask][128 rows][d] f16 (one CTA per 128-row
// block, 16-byte copies)
__global__ void __launch_bounds__(256) k_pack_kv(uint4* __restrict__ dst, const uint4* __restrict__ k,
                                                 const uint4* __restrict__ v, int64_t bh, int64_t seq,
                                                 unsigned tile_mask, int n_tiles, int64_t row_vecs) {
  const int64_t blk = blockIdx.x;                  // (which, head, i)
  const int i = (int)(blk % n_tiles);
  const int64_t head = (blk / n_tiles) % bh;
  const int which = (int)(blk / (n_tiles * bh));
  const int tile = (int)__fns(tile_mask, 0, i + 1);
  const int64_t n = 128 * row_vecs;                // 16-byte vectors per block
  const uint4* src = (which ? v : k) + (head * seq + (int64_t)tile * 128) * row_vecs;
  uint4* out = dst + blk * n;
  for (int64_t e = threadIdx.x; e < n; e += blockDim.x) out[e] = src[e];
}

extern "C" int ktir_pack_kv(void* dst, const void* k, const void* v, int64_t bh, int64_t seq,
                            int64_t d, uint32_t tile_mask, void* stream) {
  const int n = __builtin_popcount(tile_mask);
  if (!dst || !k || !v || bh < 1 || seq < 128 || seq % 128 || d < 8 || d % 8 || n == 0 ||
      (seq / 128 < 32 && (tile_mask >> (seq / 128)) != 0))
    return set_err(KTIR_ERR_ARG, "ktir_pack_kv: bad arguments");
  if (((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(k) |
        reinterpret_cast<uintptr_t>(v)) & 15) != 0)
    return set_err(KTIR_ERR_UNSUPPORTED, "ktir_pack_kv: pointers must be 16-byte aligned");
  const int64_t blocks = 2 * bh * n;
  if (blocks > 0x7fffffffLL) return set_err(KTIR_ERR_UNSUPPORTED, "ktir_pack_kv: too many blocks");
  k_pack_kv<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(
      (uint4*)dst, (const uint4*)k, (const uint4*)v, bh, seq, tile_mask, n, d * 2 / 16);
  return check_launch("ktir_pack_kv");
}

// ---------------------------------------------------------------------------
// fused elementwise
// ---------------------------------------------------------------------------
template <bool CONTIG>
__global__ void __launch_bounds__(256) k_ew(const __grid_constant__ KtirEwProgram p,
                                            const __grid_constant__ KtirBuffers b,
                                            const int64_t* __restrict__ ut) {
  __shared__ int64_t base[KTIR_MAX_VIEWS];
  pdl_prologue();
  for (int unit = blockIdx.y; unit < p.n_units; unit += gridDim.y) {
    __syncthreads();
    if (threadIdx.x < p.n_views) {
      const KtirView& v = p.view[threadIdx.x];
      base[threadIdx.x] =
          v.off + (v.unit_col >= 0 ? ut[(int64_t)unit * p.unit_cols + v.unit_col] : 0);
    }
    __syncthreads();
    Reg r[KTIR_NREG];
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < p.numel;
         e += (int64_t)gridDim.x * blockDim.x) {
      int64_t idx[KTIR_MAX_RANK];
      if (!CONTIG) {
        int64_t rem = e;
        for (int d = p.rank - 1; d >= 0; --d) {
          idx[d] = rem % p.shape[d];
          rem /= p.shape[d];
        }
      }
      for (int pc = 0; pc < p.n_instr; ++pc) {
        const KtirInstr in = p.code[pc];
        if (in.op == OP_LD || in.op == OP_ST) {
          const KtirView& v = p.view[in.aux];
          int64_t off = base[in.aux];
          if (CONTIG) {
            off += e;
          } else {
            for (int d = 0; d < p.rank; ++d) off += idx[d] * v.stride[d];
          }
          if (in.op == OP_LD)
            r[in.dst] = load_elem(b, v.slot, v.dtype, off);
          else
            store_elem(b, v.slot, v.dtype, off, r[in.a], in.dt);
        } else if (in.op == OP_IOTA) {
          r[in.dst].i = CONTIG ? 0 : idx[in.aux];
        } else {
          exec_arith(in, r);
        }
      }
    }
  }
}

// y = a op b over f16 views that are dense, 16-byte aligned and inside their
// buffers in every unit (the lowering marks such programs contiguous == 2):
// eight elements per thread in 16-byte loads and stores.  + - * on f16 pairs
// round the exact result once, which is what NumPy's f16 loops give (they
// compute in f32, whose 24 bits hold the exact sum or product of two f16s);
// the quotient goes through f32 (24 >= 2 * 11 + 2 bits: rounding to f32 and
// then to f16 equals rounding once).
template <int OP>
__global__ void __launch_bounds__(256) k_ew_bin_f16(const __grid_constant__ KtirEwProgram p,
                                                    const __grid_constant__ KtirBuffers b,
                                                    const int64_t* __restrict__ ut, int va, int vb,
                                                    int vo) {
  pdl_prologue();
  const int64_t chunks = p.numel >> 3;
  const int64_t items = chunks * p.n_units;
  const KtirView& A = p.view[va];
  const KtirView& Bv = p.view[vb];
  const KtirView& O = p.view[vo];
  const __half* pa = (const __half*)b.base[A.slot];
  const __half* pb = (const __half*)b.base[Bv.slot];
  __half* po = (__half*)b.base[O.slot];
  for (int64_t it = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; it < items;
       it += (int64_t)gridDim.x * blockDim.x) {
    const int64_t unit = it / chunks;
    const int64_t c = (it - unit * chunks) << 3;
    const int64_t* row = ut + unit * p.unit_cols;
    const int64_t oa = A.off + (A.unit_col >= 0 ? row[A.unit_col] : 0) + c;
    const int64_t ob = Bv.off + (Bv.unit_col >= 0 ? row[Bv.unit_col] : 0) + c;
    const int64_t oo = O.off + (O.unit_col >= 0 ? row[O.unit_col] : 0) + c;
    uint4 x = *reinterpret_cast<const uint4*>(pa + oa);
    const uint4 y = *reinterpret_cast<const uint4*>(pb + ob);
    __half2* hx = reinterpret_cast<__half2*>(&x);
    const __half2* hy = reinterpret_cast<const __half2*>(&y);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      if (OP == OP_FADD) hx[q] = __hadd2(hx[q], hy[q]);
      else if (OP == OP_FSUB) hx[q] = __hsub2(hx[q], hy[q]);
      else if (OP == OP_FMUL) hx[q] = __hmul2(hx[q], hy[q]);
      else {
        const float2 fx = __half22float2(hx[q]), fy = __half22float2(hy[q]);
        hx[q] = __floats2half2_rn(fx.x / fy.x, fx.y / fy.y);
      }
    }
    *reinterpret_cast<uint4*>(po + oo) = x;
  }
}

// the two-load binary f16 program the vector kernel covers: returns the op,
// with the views of the operands and of the result
static int match_bin_f16(const KtirEwProgram& p, int* va, int* vb, int* vo) {
  if (p.contiguous != 2 || p.n_instr != 4 || (p.numel & 7)) return 0;
  const KtirInstr* c = p.code;
  if (c[0].op != OP_LD || c[1].op != OP_LD || c[3].op != OP_ST) return 0;
  const int op = c[2].op;
  if (op != OP_FADD && op != OP_FSUB && op != OP_FMUL && op != OP_FDIV) return 0;
  if (c[2].dt != KTIR_F16 || c[3].a != c[2].dst || c[0].dst == c[1].dst) return 0;
  if (c[2].a == c[0].dst && c[2].b == c[1].dst) {
    *va = c[0].aux;
    *vb = c[1].aux;
  } else if (c[2].a == c[1].dst && c[2].b == c[0].dst) {
    *va = c[1].aux;
    *vb = c[0].aux;
  } else {
    return 0;
  }
  *vo = c[3].aux;
  if (*va >= p.n_views || *vb >= p.n_views || *vo >= p.n_views) return 0;
  if (p.view[*va].dtype != KTIR_F16 || p.view[*vb].dtype != KTIR_F16 ||
      p.view[*vo].dtype != KTIR_F16 || c[3].dt != KTIR_F16)
    return 0;
  return op;
}

extern "C" int ktir_ew(const KtirEwProgram* prog, const KtirBuffers* bufs,
                       const int64_t* unit_table, void* stream) {
  if (!prog || !bufs) return set_err(KTIR_ERR_ARG, "ktir_ew: null descriptor");
  if (prog->n_instr > KTIR_MAX_INSTR || prog->n_views > KTIR_MAX_VIEWS ||
      prog->rank > KTIR_MAX_RANK || prog->n_units < 1)
    return set_err(KTIR_ERR_ARG, "ktir_ew: descriptor out of range");
  if (prog->numel == 0) return KTIR_OK;
  cudaStream_t s = (cudaStream_t)stream;
  int va, vb, vo;
  if (const int op = match_bin_f16(*prog, &va, &vb, &vo)) {
    const int g = grid_x((prog->numel >> 3) * prog->n_units, 256, 148 * 8);
    switch (op) {
      case OP_FADD: launch_pdl(k_ew_bin_f16<OP_FADD>, dim3(g), dim3(256), 0, s, *prog, *bufs, unit_table, va, vb, vo); break;
      case OP_FSUB: launch_pdl(k_ew_bin_f16<OP_FSUB>, dim3(g), dim3(256), 0, s, *prog, *bufs, unit_table, va, vb, vo); break;
      case OP_FMUL: launch_pdl(k_ew_bin_f16<OP_FMUL>, dim3(g), dim3(256), 0, s, *prog, *bufs, unit_table, va, vb, vo); break;
      default: launch_pdl(k_ew_bin_f16<OP_FDIV>, dim3(g), dim3(256), 0, s, *prog, *bufs, unit_table, va, vb, vo); break;
    }
    return check_launch("ktir_ew");
  }
  dim3 grid(grid_x(prog->numel, 256, 148 * 16), prog->n_units < 65535 ? prog->n_units : 65535);
  if (prog->contiguous)
    launch_pdl(k_ew<true>, grid, dim3(256), 0, s, *prog, *bufs, unit_table);
  else
    launch_pdl(k_ew<false>, grid, dim3(256), 0, s, *prog, *bufs, unit_table);
  return check_launch("ktir_ew");
}

// ---------------------------------------------------------------------------
// fused row softmax
// ---------------------------------------------------------------------------
// Layout: lane l holds elements 64*m + 2*l + k (k < 2, m < M = cols/64) of its
// row, i.e. one f16 pair per m, so each warp load or store moves 128
// contiguous bytes.  With this layout the halving tree of the reference
// (combine [0,h) with [h,2h), h = n/2, n/4, ..., 1) maps to:
//   h >= 64      : pair m with pair m + h/64 in the same lane
//   2 <= h <= 32 : lane l with lane l + h/2 (m = 0, same k)
//   h == 1       : k = 0 with k = 1 inside lane 0
// so the sum below is the reference's fold, pair for pair, with only two
// values per lane crossing lanes in each of the five shuffle rounds.  The max
// does not depend on the order (fmax ignores NaN like arith.maxnumf, and a
// zero's sign cannot change exp(x - max)), so it is an in-lane max and one
// redux.sync.
template <int M, bool F16>
__device__ __forceinline__ float sum_fold(float (&v)[M][2]) {
  const unsigned full = 0xffffffffu;
#pragma unroll
  for (int hm = M / 2; hm >= 1; hm >>= 1) {
#pragma unroll
    for (int m = 0; m < hm; ++m) {
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const float r = v[m][k] + v[m + hm][k];
        v[m][k] = F16 ? __half2float(__float2half_rn(r)) : r;
      }
    }
  }
#pragma unroll
  for (int dl = 16; dl >= 1; dl >>= 1) {
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const float c = __shfl_down_sync(full, v[0][k], dl);
      const float r = v[0][k] + c;
      v[0][k] = F16 ? __half2float(__float2half_rn(r)) : r;
    }
  }
  float r = v[0][0] + v[0][1];
  r = F16 ? __half2float(__float2half_rn(r)) : r;
  return __shfl_sync(full, r, 0);
}

__device__ __forceinline__ float warp_max(float x) {
  float y;
  asm volatile("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <int M>
__device__ __forceinline__ void load_row(const __half* in, int64_t numel, int64_t ib, int lane,
                                         uint32_t (&raw)[M]) {
#pragma unroll
  for (int m = 0; m < M; ++m) {
    const int64_t e = ib + 64 * m + 2 * lane;
    if (e >= 0 && e + 2 <= numel) {
      raw[m] = __ldg(reinterpret_cast<const unsigned int*>(in + e));
    } else {
      __half2 h;
      h.x = (e >= 0 && e < numel) ? in[e] : __float2half(0.f);
      h.y = (e + 1 >= 0 && e + 1 < numel) ? in[e + 1] : __float2half(0.f);
      raw[m] = *reinterpret_cast<const uint32_t*>(&h);
    }
  }
}

// One warp per row; a warp walks rows `nwarps` apart and prefetches the next
// row's pairs before reducing the current one, so loads overlap the math.
template <int M, bool F16>
__global__ void __launch_bounds__(128) k_softmax_rows(const __grid_constant__ KtirSoftmaxDesc d,
                                                      const __grid_constant__ KtirBuffers b,
                                                      const int64_t* __restrict__ ut) {
  pdl_prologue();
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t total_rows = (int64_t)d.n_units * d.rows;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  constexpr bool f16c = F16;
  const __half* in = (const __half*)b.base[d.in.slot];
  __half* out = (__half*)b.base[d.out.slot];
  const int64_t in_numel = b.numel[d.in.slot];
  const int64_t out_numel = b.numel[d.out.slot];
  // units that are consecutive row blocks arrive as one unit (no table)
  auto in_base = [&](int64_t row) -> int64_t {
    if (d.in.unit_col < 0) return d.in.off + row * d.in.stride[0];
    const int unit = (int)row / d.rows;
    const int r = (int)row - unit * d.rows;
    return d.in.off + ut[(int64_t)unit * d.unit_cols + d.in.unit_col] + (int64_t)r * d.in.stride[0];
  };
  auto out_base = [&](int64_t row) -> int64_t {
    if (d.out.unit_col < 0) return d.out.off + row * d.out.stride[0];
    const int unit = (int)row / d.rows;
    const int r = (int)row - unit * d.rows;
    return d.out.off + ut[(int64_t)unit * d.unit_cols + d.out.unit_col] + (int64_t)r * d.out.stride[0];
  };
  uint32_t cur[M];
  if (warp < total_rows) load_row<M>(in, in_numel, in_base(warp), lane, cur);
  for (int64_t row = warp; row < total_rows; row += nwarps) {
    uint32_t nxt[M];
    const int64_t nrow = row + nwarps;
    if (nrow < total_rows) load_row<M>(in, in_numel, in_base(nrow), lane, nxt);
    const int64_t ob = out_base(row);
    float v[M][2];
    float pm[M];
#pragma unroll
    for (int m = 0; m < M; ++m) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&cur[m]));
      v[m][0] = f.x;
      v[m][1] = f.y;
      pm[m] = fmaxf(f.x, f.y);
    }
#pragma unroll
    for (int h = M / 2; h >= 1; h >>= 1)
#pragma unroll
      for (int m = 0; m < h; ++m) pm[m] = fmaxf(pm[m], pm[m + h]);
    const float mx = warp_max(pm[0]);
    // exp(x - max): the f32 program folds log2(e) into one FMA feeding ex2;
    // the f16 program rounds like NumPy's float16 loops (sub, round, exp, round)
    const float l2e = 1.4426950408889634f;
    const float mx2 = mx * l2e;
    float t[M][2];
#pragma unroll
    for (int m = 0; m < M; ++m)
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        float x;
        if (f16c) {
          x = __half2float(__float2half_rn(v[m][k] - mx));
          x = __half2float(__float2half_rn(expf(x)));
        } else {
          x = fast_exp2(fmaf(v[m][k], l2e, -mx2));
        }
        v[m][k] = x;
        t[m][k] = x;
      }
    const float sum = sum_fold<M, F16>(t);
    const float rs = 1.0f / sum;
#pragma unroll
    for (int m = 0; m < M; ++m) {
      const int64_t e = ob + 64 * m + 2 * lane;
      __half2 o2;
      if (f16c)
        o2 = __floats2half2_rn(v[m][0] / sum, v[m][1] / sum);
      else
        o2 = __floats2half2_rn(v[m][0] * rs, v[m][1] * rs);
      if (e >= 0 && e + 2 <= out_numel) {
        *reinterpret_cast<__half2*>(out + e) = o2;
      } else {
        if (e >= 0 && e < out_numel) out[e] = o2.x;
        if (e + 1 >= 0 && e + 1 < out_numel) out[e + 1] = o2.y;
      }
    }
#pragma unroll
    for (int m = 0; m < M; ++m) cur[m] = nxt[m];
  }
}

// The same row softmax for rows of 256 or more elements with 16-byte moves:
// lane l owns elements 256m + 8l + k (k < 8) of the row, so a warp load or
// store covers 512 contiguous bytes.  The sum is still the reference's
// pairwise-halving fold pair for pair: in-lane rounds over m (distances
// n/2 .. 256), five shuffle rounds (128 .. 8), then in-lane rounds over k
// (4, 2, 1).
template <int M, bool F16>
__device__ __forceinline__ float sum_fold8(float (&v)[M][8]) {
  const unsigned full = 0xffffffffu;
#pragma unroll
  for (int hm = M / 2; hm >= 1; hm >>= 1)
#pragma unroll
    for (int m = 0; m < hm; ++m)
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float r = v[m][k] + v[m + hm][k];
        v[m][k] = F16 ? __half2float(__float2half_rn(r)) : r;
      }
#pragma unroll
  for (int dl = 16; dl >= 1; dl >>= 1)
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float c = __shfl_down_sync(full, v[0][k], dl);
      const float r = v[0][k] + c;
      v[0][k] = F16 ? __half2float(__float2half_rn(r)) : r;
    }
#pragma unroll
  for (int hk = 4; hk >= 1; hk >>= 1)
#pragma unroll
    for (int k = 0; k < hk; ++k) {
      const float r = v[0][k] + v[0][k + hk];
      v[0][k] = F16 ? __half2float(__float2half_rn(r)) : r;
    }
  return __shfl_sync(full, v[0][0], 0);
}

template <int M>
__device__ __forceinline__ void load_row8(const __half* in, int64_t numel, int64_t ib, int lane,
                                          uint4 (&raw)[M]) {
  if (ib >= 0 && ib + 256 * M <= numel) {
    // the whole row lies inside the buffer: no per-chunk bounds
#pragma unroll
    for (int m = 0; m < M; ++m)
      raw[m] = __ldg(reinterpret_cast<const uint4*>(in + ib + 256 * m + 8 * lane));
    return;
  }
#pragma unroll
  for (int m = 0; m < M; ++m) {
    const int64_t e = ib + 256 * m + 8 * lane;
    if (e >= 0 && e + 8 <= numel) {
      raw[m] = __ldg(reinterpret_cast<const uint4*>(in + e));
    } else {
      __align__(16) __half h[8];
#pragma unroll
      for (int k = 0; k < 8; ++k)
        h[k] = (e + k >= 0 && e + k < numel) ? in[e + k] : __float2half(0.f);
      raw[m] = *reinterpret_cast<const uint4*>(h);
    }
  }
}

template <int M, bool F16>
__global__ void __launch_bounds__(128) k_softmax_rows8(const __grid_constant__ KtirSoftmaxDesc d,
                                                       const __grid_constant__ KtirBuffers b,
                                                       const int64_t* __restrict__ ut) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t total_rows = (int64_t)d.n_units * d.rows;
  // Before waiting for the previous kernel on the stream, ask L2 for this
  // warp's first input row (from the parameters alone, so only for affine
  // rows).  A prefetch changes no value that a later load returns, even if
  // the previous kernel writes that row, and it lets this kernel's HBM reads
  // overlap the previous kernel's last CTAs.
  if (d.in.unit_col < 0 && lane == 0 && warp < total_rows) {
    const int64_t ib = d.in.off + warp * d.in.stride[0];
    if (ib >= 0 && ib + 256 * M <= b.numel[d.in.slot])
      asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(
                       (const __half*)b.base[d.in.slot] + ib),
                   "r"(512 * M)
                   : "memory");
  }
  pdl_prologue();
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const __half* in = (const __half*)b.base[d.in.slot];
  __half* out = (__half*)b.base[d.out.slot];
  const int64_t in_numel = b.numel[d.in.slot];
  const int64_t out_numel = b.numel[d.out.slot];
  auto base_of = [&](const KtirView& vw, int64_t row) -> int64_t {
    if (vw.unit_col < 0) return vw.off + row * vw.stride[0];
    const int unit = (int)row / d.rows;
    const int r = (int)row - unit * d.rows;
    return vw.off + ut[(int64_t)unit * d.unit_cols + vw.unit_col] + (int64_t)r * vw.stride[0];
  };
  uint4 cur[M];
  if (warp < total_rows) load_row8<M>(in, in_numel, base_of(d.in, warp), lane, cur);
  for (int64_t row = warp; row < total_rows; row += nwarps) {
    uint4 nxt[M];
    const int64_t nrow = row + nwarps;
    if (nrow < total_rows) load_row8<M>(in, in_numel, base_of(d.in, nrow), lane, nxt);
    const int64_t ob = base_of(d.out, row);
    float v[M][8];
    float pm[M];
#pragma unroll
    for (int m = 0; m < M; ++m) {
      const __half2* h2 = reinterpret_cast<const __half2*>(&cur[m]);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = __half22float2(h2[q]);
        v[m][2 * q] = f.x;
        v[m][2 * q + 1] = f.y;
      }
      pm[m] = fmaxf(fmaxf(fmaxf(v[m][0], v[m][1]), fmaxf(v[m][2], v[m][3])),
                    fmaxf(fmaxf(v[m][4], v[m][5]), fmaxf(v[m][6], v[m][7])));
    }
#pragma unroll
    for (int h = M / 2; h >= 1; h >>= 1)
#pragma unroll
      for (int m = 0; m < h; ++m) pm[m] = fmaxf(pm[m], pm[m + h]);
    const float mx = warp_max(pm[0]);
    // exp(x - max) as in k_softmax_rows
    const float l2e = 1.4426950408889634f;
    const float mx2 = mx * l2e;
    float t[M][8];
#pragma unroll
    for (int m = 0; m < M; ++m)
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        float x;
        if (F16) {
          x = __half2float(__float2half_rn(v[m][k] - mx));
          x = __half2float(__float2half_rn(expf(x)));
        } else {
          x = fast_exp2(fmaf(v[m][k], l2e, -mx2));
        }
        v[m][k] = x;
        t[m][k] = x;
      }
    const float sum = sum_fold8<M, F16>(t);
    const float rs = 1.0f / sum;
    const bool whole = ob >= 0 && ob + 256 * M <= out_numel;
#pragma unroll
    for (int m = 0; m < M; ++m) {
      const int64_t e = ob + 256 * m + 8 * lane;
      __align__(16) __half2 o2[4];
#pragma unroll
      for (int q = 0; q < 4; ++q)
        o2[q] = F16 ? __floats2half2_rn(v[m][2 * q] / sum, v[m][2 * q + 1] / sum)
                    : __floats2half2_rn(v[m][2 * q] * rs, v[m][2 * q + 1] * rs);
      if (whole || (e >= 0 && e + 8 <= out_numel)) {
        *reinterpret_cast<uint4*>(out + e) = *reinterpret_cast<const uint4*>(o2);
      } else {
        const __half* oh = reinterpret_cast<const __half*>(o2);
#pragma unroll
        for (int k = 0; k < 8; ++k)
          if (e + k >= 0 && e + k < out_numel) out[e + k] = oh[k];
      }
    }
#pragma unroll
    for (int m = 0; m < M; ++m) cur[m] = nxt[m];
  }
}

extern "C" int ktir_softmax_rows(const KtirSoftmaxDesc* d, const KtirBuffers* bufs,
                                 const int64_t* unit_table, void* stream) {
  if (!d || !bufs) return set_err(KTIR_ERR_ARG, "ktir_softmax_rows: null descriptor");
  const int n = d->cols;
  if (n < 64 || (n & (n - 1)) || n > 4096 || d->in.stride[1] != 1 || d->out.stride[1] != 1 ||
      d->in.dtype != KTIR_F16 || d->out.dtype != KTIR_F16)
    return set_err(KTIR_ERR_UNSUPPORTED, "ktir_softmax_rows: needs f16 rows of 2^k in [64, 4096] elements");
  if (((d->in.off | d->out.off | d->in.stride[0] | d->out.stride[0]) & 7) != 0)
    return set_err(KTIR_ERR_UNSUPPORTED, "ktir_softmax_rows: rows must be 16-byte aligned");
  if ((int64_t)d->n_units * d->rows >= (1ll << 31))
    return set_err(KTIR_ERR_UNSUPPORTED, "ktir_softmax_rows: more than 2^31 rows");
  const int64_t rows = (int64_t)d->n_units * d->rows;
  const int threads = 128;
  // rows per warp (descriptor's spare field, 0 = default 1)
  const int rpw = d->pad > 0 ? d->pad : 1;
  const int blocks = grid_x((rows + rpw - 1) / rpw * 32, threads, 1 << 30);
  cudaStream_t s = (cudaStream_t)stream;
#define KTIR_SOFTMAX_CASE(V)                                                         \
  case V:                                                                            \
    if (d->compute_f16)                                                              \
      launch_pdl(k_softmax_rows<V, true>, dim3(blocks), dim3(threads), 0, s, *d, *bufs, \
                 unit_table);                                                        \
    else                                                                             \
      launch_pdl(k_softmax_rows<V, false>, dim3(blocks), dim3(threads), 0, s, *d, *bufs, \
                 unit_table);                                                        \
    break;
#define KTIR_SOFTMAX8_CASE(V)                                                         \
  case V:                                                                             \
    if (d->compute_f16)                                                               \
      launch_pdl(k_softmax_rows8<V, true>, dim3(blocks), dim3(threads), 0, s, *d, *bufs, \
                 unit_table);                                                         \
    else                                                                              \
      launch_pdl(k_softmax_rows8<V, false>, dim3(blocks), dim3(threads), 0, s, *d, *bufs, \
                 unit_table);                                                         \
    break;
  if (n >= 256) {
    // 16-byte moves (rows are 16-byte aligned, checked above)
    switch (n / 256) {
      KTIR_SOFTMAX8_CASE(1)
      KTIR_SOFTMAX8_CASE(2)
      KTIR_SOFTMAX8_CASE(4)
      KTIR_SOFTMAX8_CASE(8)
      KTIR_SOFTMAX8_CASE(16)
      default: return set_err(KTIR_ERR_UNSUPPORTED, "ktir_softmax_rows: row length");
    }
  } else {
    switch (n / 64) {
      KTIR_SOFTMAX_CASE(1)
      KTIR_SOFTMAX_CASE(2)
      default: return set_err(KTIR_ERR_UNSUPPORTED, "ktir_softmax_rows: row length");
    }
  }
#undef KTIR_SOFTMAX8_CASE
#undef KTIR_SOFTMAX_CASE
  return check_launch("ktir_softmax_rows");
}

// ---------------------------------------------------------------------------
// indirect gather -> f -> scatter, sequential-unit semantics
// ---------------------------------------------------------------------------
__device__ __forceinline__ int64_t read_index(const KtirBuffers& b, int slot, int dt, int64_t pos) {
  if (pos < 0 || pos >= b.numel[slot]) return 0;  // zero fill past the index tensor
  if (dt == KTIR_I64) return ((const long long*)b.base[slot])[pos];
  return ((const int*)b.base[slot])[pos];
}

// Phase 1: each CTA owns one unit, de-duplicates that unit's rows in a shared
// hash set and counts, per row, how many units name it.  RANGED (a row range,
// row_hi > 0): only rows in [row_lo, row_hi) are counted, the rows this call
// applies; the others keep a zero count.  (The range test is compiled only
// into the ranged form: in the loop of the whole-table form it cost 3 us per
// 262,144 indices.)
template <bool RANGED>
__global__ void __launch_bounds__(512) k_rmw_count(const __grid_constant__ KtirGatherRmwDesc d,
                                                   const __grid_constant__ KtirBuffers b,
                                                   int* __restrict__ counts, int64_t n_rows,
                                                   int* __restrict__ status) {
  extern __shared__ long long set[];
  pdl_prologue();
  int cap = 1;
  while (cap < 2 * d.unit_len) cap <<= 1;
  for (int unit = blockIdx.x; unit < d.n_units; unit += gridDim.x) {
    for (int i = threadIdx.x; i < cap; i += blockDim.x) set[i] = -1;
    __syncthreads();
    const int64_t base = d.idx_off + (int64_t)unit * d.idx_unit_stride;
    for (int i = threadIdx.x; i < d.unit_len; i += blockDim.x) {
      const int64_t row = read_index(b, d.idx_slot, d.idx_dtype, base + i);
      if (row < 0) {
        atomicOr(status, KTIR_STATUS_NEGATIVE_INDEX);
        continue;
      }
      if (row >= n_rows) continue;  // row wholly past the table end: no effect
      // a row outside the range is another call's to apply
      if (RANGED && (row < d.row_lo || row >= d.row_hi)) continue;
      unsigned h = (unsigned)((unsigned long long)row * 0x9E3779B97F4A7C15ull >> 40) & (cap - 1);
      for (int probe = 0; probe < cap; ++probe) {
        long long prev = atomicCAS((unsigned long long*)&set[h], (unsigned long long)-1ll,
                                   (unsigned long long)row);
        if (prev == -1) {
          atomicAdd(&counts[row], 1);
          break;
        }
        if (prev == row) break;
        h = (h + 1) & (cap - 1);
      }
    }
    __syncthreads();
  }
}

// Apply f once to one element: SOP != 0 is the common y = x op imm with an f16
// result (op fixed at compile time); SOP == 0 runs the bytecode.
template <int SOP>
__device__ __forceinline__ float apply_f(const KtirEwProgram& f, float x, float imm, int out_dt) {
  if (SOP != 0) return __half2float(__float2half_rn(binf(SOP, x, imm)));
  Reg r[KTIR_NREG];
  Reg res;
  res.f = x;
  for (int pc = 0; pc < f.n_instr; ++pc) {
    const KtirInstr in = f.code[pc];
    if (in.op == OP_LD) {
      r[in.dst].f = x;
    } else if (in.op == OP_ST) {
      res = convert(r[in.a], in.dt, out_dt);
    } else {
      exec_arith(in, r);
    }
  }
  return res.f;
}

// Phase 2: the first position to claim a row's count applies f count times.
// A 16-lane group owns one index position; rows move in 16-byte vectors.
template <int SOP>
__global__ void __launch_bounds__(256) k_rmw_apply(const __grid_constant__ KtirGatherRmwDesc d,
                                                   const __grid_constant__ KtirBuffers b,
                                                   int* __restrict__ counts, int64_t n_rows,
                                                   float simple_imm) {
  pdl_prologue();
  const int sub = threadIdx.x & 15;
  const int group = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 4);
  const int ngroups = (int)((gridDim.x * blockDim.x) >> 4);
  const int total = d.n_units * d.unit_len;
  const bool dense_units = d.idx_unit_stride == d.unit_len;
  const int64_t row_lo = d.row_hi > 0 ? d.row_lo : 0;
  const int64_t row_hi = d.row_hi > 0 ? d.row_hi : n_rows;
  __half* table = (__half*)b.base[d.table_slot];
  const int64_t tnumel = b.numel[d.table_slot];
  const int out_dt = d.f.view[1].dtype;
  for (int g = group; g < total; g += ngroups) {
    int64_t pos;
    if (dense_units) {
      pos = d.idx_off + g;
    } else {
      const int unit = g / d.unit_len;
      pos = d.idx_off + (int64_t)unit * d.idx_unit_stride + (g - unit * d.unit_len);
    }
    const int64_t row = read_index(b, d.idx_slot, d.idx_dtype, pos);
    int m = 0;
    if (sub == 0 && row >= 0 && row < n_rows) m = atomicExch(&counts[row], 0);
    // the 16 lanes of this position's group (the other half-warp may be on
    // a different trip of the loop)
    m = __shfl_sync(0xffffu << (threadIdx.x & 16), m, 0, 16);
    // rows owned by another shard are consumed (counts stay zero) but not applied
    if (m <= 0 || row < row_lo || row >= row_hi) continue;
    const int64_t rb = d.table_off + row * d.row_stride;
    for (int c = sub * 8; c < d.row_len; c += 128) {
      const int64_t e = rb + c;
      const bool vec = (c + 8 <= d.row_len) && ((e & 7) == 0) && (e + 8 <= tnumel) && e >= 0;
      if (SOP != 0 && vec) {
        // y = x op imm on f16 pairs: one f16 rounding of the exact result is
        // what the f32 operation rounded to f16 gives (f32 carries more than
        // 2 x 11 + 2 bits, so the double rounding cannot differ)
        uint4 raw = *reinterpret_cast<const uint4*>(table + e);
        __half2* h2 = reinterpret_cast<__half2*>(&raw);
        const __half2 imm2 = __float2half2_rn(simple_imm);
        for (int rep = 0; rep < m; ++rep) {
#pragma unroll
          for (int q = 0; q < 4; ++q)
            h2[q] = SOP == OP_FADD ? __hadd2(h2[q], imm2)
                                   : (SOP == OP_FSUB ? __hsub2(h2[q], imm2) : __hmul2(h2[q], imm2));
        }
        *reinterpret_cast<uint4*>(table + e) = raw;
        continue;
      }
      float x[8];
      if (vec) {
        uint4 raw = *reinterpret_cast<const uint4*>(table + e);
        const __half* h = reinterpret_cast<const __half*>(&raw);
#pragma unroll
        for (int k = 0; k < 8; ++k) x[k] = __half2float(h[k]);
      } else {
#pragma unroll
        for (int k = 0; k < 8; ++k)
          x[k] = (c + k < d.row_len && e + k >= 0 && e + k < tnumel) ? __half2float(table[e + k])
                                                                     : 0.f;
      }
      for (int rep = 0; rep < m; ++rep) {
#pragma unroll
        for (int k = 0; k < 8; ++k) x[k] = apply_f<SOP>(d.f, x[k], simple_imm, out_dt);
      }
      if (vec) {
        __half h[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) h[k] = __float2half_rn(x[k]);
        *reinterpret_cast<uint4*>(table + e) = *reinterpret_cast<uint4*>(h);
      } else {
#pragma unroll
        for (int k = 0; k < 8; ++k)
          if (c + k < d.row_len && e + k >= 0 && e + k < tnumel) table[e + k] = __float2half_rn(x[k]);
      }
    }
  }
}

// Phase 2 for the common y = x op imm on f16 rows: an 8-lane group owns one
// index position and each lane moves two 16-byte vectors of the row (loads of
// both issued before either store), so twice as many row bytes are in flight
// per thread as with one vector per lane; f16 pairs as in k_rmw_apply.
template <int SOP>
__global__ void __launch_bounds__(256) k_rmw_apply_pairs(const __grid_constant__ KtirGatherRmwDesc d,
                                                         const __grid_constant__ KtirBuffers b,
                                                         int* __restrict__ counts, int64_t n_rows,
                                                         float simple_imm) {
  pdl_prologue();
  const int sub = threadIdx.x & 7;
  const int group = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 3);
  const int ngroups = (int)((gridDim.x * blockDim.x) >> 3);
  const int total = d.n_units * d.unit_len;
  const bool dense_units = d.idx_unit_stride == d.unit_len;
  const int64_t row_lo = d.row_hi > 0 ? d.row_lo : 0;
  const int64_t row_hi = d.row_hi > 0 ? d.row_hi : n_rows;
  __half* table = (__half*)b.base[d.table_slot];
  const int64_t tnumel = b.numel[d.table_slot];
  const __half2 imm2 = __float2half2_rn(simple_imm);
  const unsigned gmask = 0xffu << (threadIdx.x & 24);
  for (int g = group; g < total; g += ngroups) {
    int64_t pos;
    if (dense_units) {
      pos = d.idx_off + g;
    } else {
      const int unit = g / d.unit_len;
      pos = d.idx_off + (int64_t)unit * d.idx_unit_stride + (g - unit * d.unit_len);
    }
    const int64_t row = read_index(b, d.idx_slot, d.idx_dtype, pos);
    int m = 0;
    if (sub == 0 && row >= 0 && row < n_rows) m = atomicExch(&counts[row], 0);
    m = __shfl_sync(gmask, m, 0, 8);
    if (m <= 0 || row < row_lo || row >= row_hi) continue;
    const int64_t rb = d.table_off + row * d.row_stride;
    for (int c0 = sub * 16; c0 < d.row_len; c0 += 128) {
      uint4 raw[2];
      bool vec[2];
#pragma unroll
      for (int v = 0; v < 2; ++v) {
        const int c = c0 + 8 * v;
        const int64_t e = rb + c;
        vec[v] = (c + 8 <= d.row_len) && ((e & 7) == 0) && (e + 8 <= tnumel) && e >= 0;
        if (vec[v]) raw[v] = *reinterpret_cast<const uint4*>(table + e);
      }
#pragma unroll
      for (int v = 0; v < 2; ++v) {
        const int c = c0 + 8 * v;
        const int64_t e = rb + c;
        if (vec[v]) {
          __half2* h2 = reinterpret_cast<__half2*>(&raw[v]);
          for (int rep = 0; rep < m; ++rep) {
#pragma unroll
            for (int q = 0; q < 4; ++q)
              h2[q] = SOP == OP_FADD ? __hadd2(h2[q], imm2)
                                     : (SOP == OP_FSUB ? __hsub2(h2[q], imm2) : __hmul2(h2[q], imm2));
          }
          *reinterpret_cast<uint4*>(table + e) = raw[v];
        } else {
          // a ragged or unaligned stretch: element by element, f32 op rounded to f16
          for (int k = 0; k < 8; ++k) {
            if (c + k >= d.row_len || e + k < 0 || e + k >= tnumel) continue;
            float x = __half2float(table[e + k]);
            for (int rep = 0; rep < m; ++rep) x = __half2float(__float2half_rn(binf(SOP, x, simple_imm)));
            table[e + k] = __float2half_rn(x);
          }
        }
      }
    }
  }
}

// Phase 2 for the common shape: 128-element rows whose every 16-byte vector
// is aligned (table_off and row_stride multiples of 8 elements), y = x op imm.
// A warp takes 32 consecutive index positions: each lane reads one index and
// claims that row's count, so the warp has 32 claims in flight at once; then
// the claimed rows go through the warp eight at a time, each 8-lane quarter
// moving two rows (two 16-byte vectors per lane and row), all eight rows'
// loads issued before any of their stores.
template <int SOP>
__device__ __forceinline__ void rmw_row_op(uint4& raw, int m, __half2 imm2) {
  __half2* h2 = reinterpret_cast<__half2*>(&raw);
  for (int rep = 0; rep < m; ++rep) {
#pragma unroll
    for (int q = 0; q < 4; ++q)
      h2[q] = SOP == OP_FADD ? __hadd2(h2[q], imm2)
                             : (SOP == OP_FSUB ? __hsub2(h2[q], imm2) : __hmul2(h2[q], imm2));
  }
}

template <int SOP>
__global__ void __launch_bounds__(256) k_rmw_apply_warp(const __grid_constant__ KtirGatherRmwDesc d,
                                                        const __grid_constant__ KtirBuffers b,
                                                        int* __restrict__ counts, int64_t n_rows,
                                                        float simple_imm) {
  pdl_prologue();
  const int lane = threadIdx.x & 31;
  const int quarter = lane >> 3, sub = lane & 7;
  const int64_t warp0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int64_t total = (int64_t)d.n_units * d.unit_len;
  const bool dense_units = d.idx_unit_stride == d.unit_len;
  const int64_t row_lo = d.row_hi > 0 ? d.row_lo : 0;
  const int64_t row_hi = d.row_hi > 0 ? d.row_hi : n_rows;
  __half* table = (__half*)b.base[d.table_slot];
  const int64_t tnumel = b.numel[d.table_slot];
  const __half2 imm2 = __float2half2_rn(simple_imm);
  for (int64_t base = warp0 * 32; base < total; base += nwarps * 32) {
    const int64_t g = base + lane;
    int64_t row = -1;
    if (g < total) {
      int64_t pos;
      if (dense_units) {
        pos = d.idx_off + g;
      } else {
        const int64_t unit = g / d.unit_len;
        pos = d.idx_off + unit * d.idx_unit_stride + (g - unit * d.unit_len);
      }
      row = read_index(b, d.idx_slot, d.idx_dtype, pos);
    }
    int m = 0;
    if (row >= 0 && row < n_rows) m = atomicExch(&counts[row], 0);
    // rows owned by another shard are consumed (counts stay zero) but not applied
    unsigned live = __ballot_sync(0xffffffffu, m > 0 && row >= row_lo && row < row_hi);
    while (live) {
      // this quarter's two rows of the next eight: lanes src[0], src[1]
      int src[2];
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        int pick = -1;
#pragma unroll
        for (int qq = 0; qq < 4; ++qq) {
          const int f = live ? __ffs(live) - 1 : -1;
          if (f >= 0) live &= live - 1;
          if (qq == quarter) pick = f;
        }
        src[t] = pick;
      }
      int64_t rr[2];
      int mm[2];
      uint4 raw[2][2];
      bool whole[2];
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        rr[t] = __shfl_sync(0xffffffffu, row, src[t] < 0 ? 0 : src[t]);
        mm[t] = __shfl_sync(0xffffffffu, m, src[t] < 0 ? 0 : src[t]);
        const int64_t e = d.table_off + rr[t] * d.row_stride + sub * 16;
        whole[t] = src[t] >= 0 && e >= 0 && e + 16 <= tnumel;
        if (whole[t]) {
          raw[t][0] = *reinterpret_cast<const uint4*>(table + e);
          raw[t][1] = *reinterpret_cast<const uint4*>(table + e + 8);
        }
      }
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        if (src[t] < 0) continue;
        const int64_t e = d.table_off + rr[t] * d.row_stride + sub * 16;
        if (whole[t]) {
          rmw_row_op<SOP>(raw[t][0], mm[t], imm2);
          rmw_row_op<SOP>(raw[t][1], mm[t], imm2);
          *reinterpret_cast<uint4*>(table + e) = raw[t][0];
          *reinterpret_cast<uint4*>(table + e + 8) = raw[t][1];
        } else {
          // the row runs past the table's end: element by element up to it
          for (int i = 0; i < 16; ++i) {
            if (e + i < 0 || e + i >= tnumel) continue;
            float x = __half2float(table[e + i]);
            for (int rep = 0; rep < mm[t]; ++rep)
              x = __half2float(__float2half_rn(binf(SOP, x, simple_imm)));
            table[e + i] = __float2half_rn(x);
          }
        }
      }
    }
  }
}

extern "C" int ktir_gather_rmw(const KtirGatherRmwDesc* d, const KtirBuffers* bufs, int32_t* counts,
                               int64_t n_rows, int32_t* status, void* stream) {
  if (!d || !bufs || !counts || !status) return set_err(KTIR_ERR_ARG, "ktir_gather_rmw: null argument");
  if (d->unit_len <= 0 || d->unit_len > 8192)
    return set_err(KTIR_ERR_UNSUPPORTED, "ktir_gather_rmw: unit length must be in [1, 8192]");
  if ((int64_t)d->n_units * d->unit_len >= (1ll << 31))
    return set_err(KTIR_ERR_UNSUPPORTED, "ktir_gather_rmw: more than 2^31 index positions");
  int cap = 1;
  while (cap < 2 * d->unit_len) cap <<= 1;
  const size_t smem = (size_t)cap * sizeof(long long);
  cudaStream_t s = (cudaStream_t)stream;
  const bool ranged = d->row_hi > 0;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(ranged ? k_rmw_count<true> : k_rmw_count<false>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return set_err(KTIR_ERR_CUDA, cudaGetErrorString(e));
  }
  const bool do_count = d->phases == 0 || (d->phases & 1);
  const bool do_apply = d->phases == 0 || (d->phases & 2);
  if (do_count) {
    if (ranged)
      launch_pdl(k_rmw_count<true>, dim3(d->n_units), dim3(512), smem, s, *d, *bufs, counts, n_rows,
                 status);
    else
      launch_pdl(k_rmw_count<false>, dim3(d->n_units), dim3(512), smem, s, *d, *bufs, counts, n_rows,
                 status);
    int rc = check_launch("ktir_gather_rmw(count)");
    if (rc) return rc;
  }
  if (!do_apply) return KTIR_OK;
  // recognise y = x op imm (one arithmetic instruction between load and store)
  int simple_op = 0;
  float simple_imm = 0.f;
  const KtirEwProgram& f = d->f;
  if (f.n_instr == 4 && f.code[0].op == OP_LD && f.code[1].op == OP_IMM &&
      (f.code[2].op == OP_FADD || f.code[2].op == OP_FSUB || f.code[2].op == OP_FMUL) &&
      f.code[3].op == OP_ST && f.view[1].dtype == KTIR_F16 &&
      f.code[2].a == f.code[0].dst && f.code[2].b == f.code[1].dst && f.code[3].a == f.code[2].dst &&
      f.code[2].dt == f.view[1].dtype && f.code[1].dt == f.code[2].dt) {
    double dv;
    memcpy(&dv, &f.code[1].imm, sizeof(dv));
    simple_op = f.code[2].op;
    simple_imm = f.code[1].dt == KTIR_F16 ? __half2float(__double2half(dv)) : (float)dv;
  }
  const int64_t groups = (int64_t)d->n_units * d->unit_len;
  const int blocks = grid_x(groups * 16, 256, 148 * 64);
  const int blocks8 = grid_x(groups * 8, 256, 148 * 64);
  if (simple_op && d->row_len == 128 && (d->table_off & 7) == 0 && (d->row_stride & 7) == 0) {
    // one wave of warps, each walking 32 positions at a time
    static int resident = 0;
    if (!resident) {
      int dev = 0, n_sm = 0, per_sm = 0;
      if (cudaGetDevice(&dev) != cudaSuccess ||
          cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
          cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_rmw_apply_warp<OP_FADD>, 256, 0) !=
              cudaSuccess)
        return set_err(KTIR_ERR_CUDA, "ktir_gather_rmw: occupancy query failed");
      resident = n_sm * (per_sm > 0 ? per_sm : 1);
    }
    // as many sweeps as one wave needs, spread evenly over the blocks
    const int64_t sweeps = (groups + (int64_t)resident * 256 - 1) / ((int64_t)resident * 256);
    const int bb = grid_x((groups + sweeps - 1) / sweeps, 256, resident);
    switch (simple_op) {
      case OP_FADD:
        launch_pdl(k_rmw_apply_warp<OP_FADD>, dim3(bb), dim3(256), 0, s, *d, *bufs, counts, n_rows, simple_imm);
        break;
      case OP_FSUB:
        launch_pdl(k_rmw_apply_warp<OP_FSUB>, dim3(bb), dim3(256), 0, s, *d, *bufs, counts, n_rows, simple_imm);
        break;
      default:
        launch_pdl(k_rmw_apply_warp<OP_FMUL>, dim3(bb), dim3(256), 0, s, *d, *bufs, counts, n_rows, simple_imm);
        break;
    }
    return check_launch("ktir_gather_rmw(apply)");
  }
  switch (simple_op) {
    case OP_FADD:
      launch_pdl(k_rmw_apply_pairs<OP_FADD>, dim3(blocks8), dim3(256), 0, s, *d, *bufs, counts, n_rows, simple_imm);
      break;
    case OP_FSUB:
      launch_pdl(k_rmw_apply_pairs<OP_FSUB>, dim3(blocks8), dim3(256), 0, s, *d, *bufs, counts, n_rows, simple_imm);
      break;
    case OP_FMUL:
      launch_pdl(k_rmw_apply_pairs<OP_FMUL>, dim3(blocks8), dim3(256), 0, s, *d, *bufs, counts, n_rows, simple_imm);
      break;
    default:
      launch_pdl(k_rmw_apply<0>, dim3(blocks), dim3(256), 0, s, *d, *bufs, counts, n_rows, 0.f);
      break;
  }
  return check_launch("ktir_gather_rmw(apply)");
}

// ---------------------------------------------------------------------------
// generic-path kernels
// ---------------------------------------------------------------------------
__device__ __forceinline__ Reg combine(int op, Reg a, Reg c, int dt) {
  Reg r;
  if (op >= OP_FADD && op <= OP_FPOW) {
    r.f = round_to(binf(op, a.f, c.f), dt);
  } else {
    r.i = wrap_to(bini(op, a.i, c.i), dt);
  }
  return r;
}

__global__ void k_reduce(const __grid_constant__ KtirReduceDesc d,
                         const __grid_constant__ KtirBuffers b) {
  const int64_t cols = d.outer * d.inner;
  const int dt = d.dt;
  for (int unit = blockIdx.y; unit < d.n_units; unit += gridDim.y) {
    const int64_t ustep = (int64_t)unit * d.unit_stride;
    for (int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c < cols;
         c += (int64_t)gridDim.x * blockDim.x) {
      const int64_t o = c / d.inner, i = c - o * d.inner;
      const int64_t base = o * d.n * d.inner + i;
      for (int64_t t = 0; t < d.n; ++t) {
        Reg v = load_elem(b, d.in_slot, dt, d.in_off + ustep + base + t * d.inner);
        store_elem(b, d.in_slot, dt, d.tmp_off + ustep + base + t * d.inner, v, dt);
      }
      int64_t m = d.n;
      while (m > 1) {
        const int64_t h = m / 2;
        for (int64_t t = 0; t < h; ++t) {
          Reg a = load_elem(b, d.in_slot, dt, d.tmp_off + ustep + base + t * d.inner);
          Reg q = load_elem(b, d.in_slot, dt, d.tmp_off + ustep + base + (t + h) * d.inner);
          store_elem(b, d.in_slot, dt, d.tmp_off + ustep + base + t * d.inner,
                     combine(d.combiner, a, q, dt), dt);
        }
        if (m & 1) {
          Reg tail = load_elem(b, d.in_slot, dt, d.tmp_off + ustep + base + 2 * h * d.inner);
          store_elem(b, d.in_slot, dt, d.tmp_off + ustep + base + h * d.inner, tail, dt);
        }
        m = h + (m & 1);
      }
      Reg res = load_elem(b, d.in_slot, dt, d.tmp_off + ustep + base);
      store_elem(b, d.out_slot, dt, d.out_off + ustep + c, res, dt);
    }
  }
}

extern "C" int ktir_reduce(const KtirReduceDesc* d, const KtirBuffers* bufs, void* stream) {
  if (!d || !bufs) return set_err(KTIR_ERR_ARG, "ktir_reduce: null descriptor");
  const int64_t cols = d->outer * d->inner;
  dim3 grid(grid_x(cols, 128, 4096), d->n_units < 65535 ? d->n_units : 65535);
  k_reduce<<<grid, 128, 0, (cudaStream_t)stream>>>(*d, *bufs);
  return check_launch("ktir_reduce");
}

__global__ void k_matmul(const __grid_constant__ KtirMatmulDesc d,
                         const __grid_constant__ KtirBuffers b, const int64_t* __restrict__ ut) {
  const int64_t total = d.batch * d.m * d.n;
  for (int unit = blockIdx.y; unit < d.n_units; unit += gridDim.y) {
    const int64_t ao = d.a.off + (d.a.unit_col >= 0 ? ut[(int64_t)unit * d.unit_cols + d.a.unit_col] : 0);
    const int64_t bo = d.b.off + (d.b.unit_col >= 0 ? ut[(int64_t)unit * d.unit_cols + d.b.unit_col] : 0);
    const int64_t oo = d.out.off + (d.out.unit_col >= 0 ? ut[(int64_t)unit * d.unit_cols + d.out.unit_col] : 0);
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
         e += (int64_t)gridDim.x * blockDim.x) {
      const int64_t bi = e / (d.m * d.n);
      const int64_t r = (e / d.n) % d.m;
      const int64_t c = e % d.n;
      const bool fl = is_float(d.a.dtype);
      float acc = 0.f;
      long long iacc = 0;
      for (int64_t k = 0; k < d.k; ++k) {
        Reg x = load_elem(b, d.a.slot, d.a.dtype, ao + bi * d.a.stride[0] + r * d.a.stride[1] + k * d.a.stride[2]);
        Reg y = load_elem(b, d.b.slot, d.b.dtype, bo + bi * d.b.stride[0] + k * d.b.stride[1] + c * d.b.stride[2]);
        if (fl) acc = fmaf(x.f, y.f, acc);
        else iacc += x.i * y.i;
      }
      Reg out;
      if (fl) out.f = round_to(acc, d.out.dtype);
      else out.i = wrap_to(iacc, d.out.dtype);
      store_elem(b, d.out.slot, d.out.dtype,
                 oo + bi * d.out.stride[0] + r * d.out.stride[1] + c * d.out.stride[2], out,
                 fl ? d.out.dtype : KTIR_I64);
    }
  }
}

extern "C" int ktir_matmul(const KtirMatmulDesc* d, const KtirBuffers* bufs,
                           const int64_t* unit_table, void* stream) {
  if (!d || !bufs) return set_err(KTIR_ERR_ARG, "ktir_matmul: null descriptor");
  dim3 grid(grid_x(d->batch * d->m * d->n, 128, 8192), d->n_units < 65535 ? d->n_units : 65535);
  k_matmul<<<grid, 128, 0, (cudaStream_t)stream>>>(*d, *bufs, unit_table);
  return check_launch("ktir_matmul");
}

__global__ void k_offsets(const __grid_constant__ KtirOffsetsDesc d,
                          const __grid_constant__ KtirBuffers b, const int64_t* __restrict__ ut,
                          int unit_cols, const int64_t* __restrict__ offs) {
  for (int unit = blockIdx.y; unit < d.n_units; unit += gridDim.y) {
    const int64_t bo = d.buf.off + (d.buf.unit_col >= 0 ? ut[(int64_t)unit * unit_cols + d.buf.unit_col] : 0);
    const int64_t dn = d.dense.off + (d.dense.unit_col >= 0 ? ut[(int64_t)unit * unit_cols + d.dense.unit_col] : 0);
    if (d.scatter) {
      // offsets were de-duplicated on the host keeping the last writer
      for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < d.count;
           i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t o = offs[(int64_t)unit * d.count + i];
        if (o < 0) continue;
        Reg v = load_elem(b, d.dense.slot, d.dense.dtype, dn + i);
        store_elem(b, d.buf.slot, d.buf.dtype, bo + o, v, d.dense.dtype);
      }
    } else {
      for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < d.count;
           i += (int64_t)gridDim.x * blockDim.x) {
        Reg v = load_elem(b, d.buf.slot, d.buf.dtype, bo + offs[(int64_t)unit * d.count + i]);
        store_elem(b, d.dense.slot, d.dense.dtype, dn + i, v, d.buf.dtype);
      }
    }
  }
}

extern "C" int ktir_offsets(const KtirOffsetsDesc* d, const KtirBuffers* bufs,
                            const int64_t* unit_table, const int64_t* offsets, void* stream) {
  if (!d || !bufs || !offsets) return set_err(KTIR_ERR_ARG, "ktir_offsets: null argument");
  if (d->count == 0) return KTIR_OK;
  dim3 grid(grid_x(d->count, 256, 4096), d->n_units < 65535 ? d->n_units : 65535);
  // the unit table width travels in dense.pad
  k_offsets<<<grid, 256, 0, (cudaStream_t)stream>>>(*d, *bufs, unit_table, d->dense.pad, offsets);
  return check_launch("ktir_offsets");
}

__device__ __forceinline__ int64_t indirect_offset(const KtirIndirectDesc& d, const KtirBuffers& b,
                                                   const int64_t* direct, const int64_t* idx_offs,
                                                   int64_t unit, int64_t i, int* status, bool* ok) {
  const int64_t p = unit * d.count + i;
  int64_t off = direct[p];
  *ok = true;
  for (int k = 0; k < d.n_ind; ++k) {
    const int64_t v = read_index(b, d.idx_slot[k], d.idx_dtype[k],
                                 idx_offs[(int64_t)k * d.n_units * d.count + p]);
    if (v < 0) {
      atomicOr(status, KTIR_STATUS_NEGATIVE_INDEX);
      *ok = false;
    }
    off += v * d.stride[k];
  }
  return off;
}

__global__ void k_indirect_gather(const __grid_constant__ KtirIndirectDesc d,
                                  const __grid_constant__ KtirBuffers b,
                                  const int64_t* __restrict__ ut, int unit_cols,
                                  const int64_t* __restrict__ direct,
                                  const int64_t* __restrict__ idx_offs, int* status) {
  for (int unit = blockIdx.y; unit < d.n_units; unit += gridDim.y) {
    const int64_t bo = d.buf.off + (d.buf.unit_col >= 0 ? ut[(int64_t)unit * unit_cols + d.buf.unit_col] : 0);
    const int64_t dn = d.dense.off + (d.dense.unit_col >= 0 ? ut[(int64_t)unit * unit_cols + d.dense.unit_col] : 0);
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < d.count;
         i += (int64_t)gridDim.x * blockDim.x) {
      bool ok;
      const int64_t o = indirect_offset(d, b, direct, idx_offs, unit, i, status, &ok);
      Reg v = load_elem(b, d.buf.slot, d.buf.dtype, ok ? bo + o : -1);
      store_elem(b, d.dense.slot, d.dense.dtype, dn + i, v, d.buf.dtype);
    }
  }
}

// Scatter in enumeration order (one thread per unit, units in order) so the
// last writer wins exactly as in the reference's fancy-index assignment.
__global__ void k_indirect_scatter(const __grid_constant__ KtirIndirectDesc d,
                                   const __grid_constant__ KtirBuffers b,
                                   const int64_t* __restrict__ ut, int unit_cols,
                                   const int64_t* __restrict__ direct,
                                   const int64_t* __restrict__ idx_offs, int* status) {
  if (blockIdx.x != 0 || threadIdx.x != 0) return;
  for (int unit = 0; unit < d.n_units; ++unit) {
    const int64_t bo = d.buf.off + (d.buf.unit_col >= 0 ? ut[(int64_t)unit * unit_cols + d.buf.unit_col] : 0);
    const int64_t dn = d.dense.off + (d.dense.unit_col >= 0 ? ut[(int64_t)unit * unit_cols + d.dense.unit_col] : 0);
    for (int64_t i = 0; i < d.count; ++i) {
      bool ok;
      const int64_t o = indirect_offset(d, b, direct, idx_offs, unit, i, status, &ok);
      if (!ok) continue;
      Reg v = load_elem(b, d.dense.slot, d.dense.dtype, dn + i);
      store_elem(b, d.buf.slot, d.buf.dtype, bo + o, v, d.dense.dtype);
    }
  }
}

extern "C" int ktir_indirect(const KtirIndirectDesc* d, const KtirBuffers* bufs,
                             const int64_t* unit_table, const int64_t* direct,
                             const int64_t* idx_offs, int32_t* status, void* stream) {
  if (!d || !bufs || !direct || !status) return set_err(KTIR_ERR_ARG, "ktir_indirect: null argument");
  if (d->n_ind > 4) return set_err(KTIR_ERR_UNSUPPORTED, "ktir_indirect: more than 4 indirect dims");
  if (d->count == 0) return KTIR_OK;
  cudaStream_t s = (cudaStream_t)stream;
  const int ucols = d->dense.pad;
  if (d->scatter) {
    k_indirect_scatter<<<1, 1, 0, s>>>(*d, *bufs, unit_table, ucols, direct, idx_offs, status);
  } else {
    dim3 grid(grid_x(d->count, 256, 4096), d->n_units < 65535 ? d->n_units : 65535);
    k_indirect_gather<<<grid, 256, 0, s>>>(*d, *bufs, unit_table, ucols, direct, idx_offs, status);
  }
  return check_launch("ktir_indirect");
}
