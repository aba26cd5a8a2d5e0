/*
 * ktir_b200.h — C ABI of the B200 execution backend for KTIR kernels.
 *
 * The reference interpreter (ktir-cpu) executes a KTIR function by running
 * every core's op list through NumPy handlers.  This library is what those
 * handlers are replaced by on a B200: the host lowers a traced KTIR function
 * into a short list of device programs, and each entry point below launches
 * one program over all the work units (cores x loop iterations) it covers.
 *
 * Conventions
 *  - Every entry point returns 0 on success or a negative code; the message
 *    of the last failure on the calling thread is ktir_last_error().
 *  - No C++ exception crosses this boundary.
 *  - Descriptors are plain structs passed by host pointer; they are copied
 *    into kernel parameters, so the caller may free them after the call.
 *  - Device pointers are passed as void*; `stream` is a cudaStream_t (NULL =
 *    the legacy default stream).  Calls are asynchronous on that stream.
 *  - A device-side status word (int32, device memory owned by the caller)
 *    collects data-dependent failures such as negative indirect indices;
 *    the caller reads it after synchronising and raises accordingly.
 *
 * Element bounds: every access names a slot of KtirBuffers; elements at or
 * past numel[slot] read as zero and are not written.  This is the
 * reference's memory rule — reads that run past the allocation holding
 * their start address are zero-filled and writes are truncated
 * (ktir_cpu/memory.py:131-198).
 */
#ifndef KTIR_B200_H
#define KTIR_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define KTIR_MAX_BUFFERS 16   /* call tensors + arena + scratch slots            */
#define KTIR_MAX_RANK 6
#define KTIR_MAX_VIEWS 12
#define KTIR_MAX_INSTR 64
#define KTIR_NREG 12

/* error codes */
#define KTIR_OK 0
#define KTIR_ERR_ARG (-1)
#define KTIR_ERR_CUDA (-2)
#define KTIR_ERR_UNSUPPORTED (-3)

/* status word bits set by kernels */
#define KTIR_STATUS_NEGATIVE_INDEX 1
#define KTIR_STATUS_TIMEOUT 2

enum KtirDtype { KTIR_F16 = 0, KTIR_F32 = 1, KTIR_I32 = 2, KTIR_I64 = 3, KTIR_BOOL = 4,
                 KTIR_U32 = 5 /* arith.fptoui results (NumPy uint32 tiles) */ };

typedef struct {
  void* base[KTIR_MAX_BUFFERS];
  int64_t numel[KTIR_MAX_BUFFERS];
} KtirBuffers;

/* A strided view over one buffer slot, aligned with an iteration space. */
typedef struct {
  int32_t slot;
  int32_t dtype;       /* KtirDtype of the stored elements */
  int32_t unit_col;    /* column of the per-unit offset table added to off, or -1 */
  int32_t pad;
  int64_t off;
  int64_t stride[KTIR_MAX_RANK];
} KtirView;

/* Elementwise bytecode (see csrc/ew_ops.cuh for the opcode list). */
typedef struct {
  uint8_t op, dst, a, b, c, dt, aux, flags;
  int64_t imm;         /* IMM: int64 value, or the bits of a double */
} KtirInstr;

typedef struct {
  int32_t rank;
  int32_t n_views;
  int32_t n_instr;
  int32_t n_units;
  int32_t unit_cols;   /* columns of the per-unit offset table */
  int32_t contiguous;  /* all views dense row-major over the iteration space; 2: also
                          every view's start a multiple of 8 elements and every access
                          inside its buffer in every unit (16-byte vector access) */
  int64_t numel;       /* elements of the iteration space per unit */
  int64_t shape[KTIR_MAX_RANK];
  KtirView view[KTIR_MAX_VIEWS];
  KtirInstr code[KTIR_MAX_INSTR];
} KtirEwProgram;

/* Row softmax: out = exp(x - max) / sum(exp(x - max)) over the last dim,
 * max/sum folded in the reference's pairwise-halving order. */
typedef struct {
  int32_t rows;        /* rows per unit */
  int32_t cols;
  int32_t n_units;
  int32_t unit_cols;
  int32_t compute_f16; /* 1: every intermediate rounded to f16 (f16 program) */
  int32_t pad;
  KtirView in;         /* stride[0] = row stride, stride[1] = 1 */
  KtirView out;
} KtirSoftmaxDesc;

/* Indirect row gather -> f -> scatter to the same rows, repeated over units
 * whose index ranges may overlap (each row gets f applied once per unit that
 * names it, in any order, as the reference's sequential units do). */
typedef struct {
  int32_t table_slot;
  int32_t idx_slot;
  int32_t idx_dtype;
  int32_t n_units;
  int32_t unit_len;    /* indices per unit */
  int32_t row_len;     /* elements per gathered row */
  int64_t table_off;   /* element offset of row 0 */
  int64_t row_stride;
  int64_t idx_off;     /* element offset of the first index of unit 0 */
  int64_t idx_unit_stride; /* index offset step between consecutive units */
  /* count and apply only table rows in [row_lo, row_hi); row_hi 0 = all.  The
   * apply pass still consumes (zeroes) every count it finds, so a count-only
   * call over all rows may be followed by an apply-only call over a range. */
  int64_t row_lo, row_hi;
  int32_t phases;      /* bit 0: count pass, bit 1: apply pass; 0 = both */
  int32_t pad2;
  KtirEwProgram f;     /* view 0 = the gathered element (load), view 1 = result (store) */
} KtirGatherRmwDesc;

/* Tree reduction along one axis of a dense [outer, n, inner] arena tile. */
typedef struct {
  int32_t combiner;    /* opcode of the binary combiner */
  int32_t dt;          /* compute/round dtype */
  int32_t n_units;
  int32_t pad;
  int64_t outer, n, inner;
  int64_t in_off, out_off, tmp_off;  /* arena element offsets (unit 0) */
  int64_t unit_stride;               /* arena elements between units */
  int32_t in_slot, out_slot;
} KtirReduceDesc;

/* Plain CUDA-core matmul for generic tiles: out[b,m,n] = sum_k a[b,m,k]*b[b,k,n],
 * accumulated in f32 in increasing k, rounded once to the output dtype. */
typedef struct {
  int64_t batch, m, n, k;
  KtirView a, b, out;  /* strides: [batch, row, col] */
  int32_t n_units, unit_cols;
} KtirMatmulDesc;

/* Gather / scatter through a per-unit element offset list. */
typedef struct {
  KtirView buf;        /* base view (slot, off, unit_col) */
  KtirView dense;      /* arena side, contiguous */
  int64_t count;       /* offsets per unit */
  int32_t n_units;
  int32_t scatter;     /* 0 gather buf->dense, 1 scatter dense->buf */
} KtirOffsetsDesc;

/* Indirect access: per point, element offset = direct[i] + sum_k idx_k * stride_k
 * where idx_k is read from buffer idx_slot[k] at idx_off_k[i]. */
typedef struct {
  KtirView buf;        /* parent tensor */
  KtirView dense;      /* arena side */
  int64_t count;       /* points per unit */
  int32_t n_units;
  int32_t n_ind;
  int32_t scatter;
  int32_t pad;
  int32_t idx_slot[4];
  int32_t idx_dtype[4];
  int64_t stride[4];
} KtirIndirectDesc;

/* Tiled f16 GEMM on the 5th-generation tensor cores (tcgen05 + TMEM, TMA fed).
 * C[m0:m0+TM, n0:n0+TN] = epilogue(A[m0:, k0:k0+K] @ B[k0:k0+K, n0:]) for every
 * listed output tile; f32 accumulation, f16 store. */
typedef struct {
  void* a; void* b; void* c;
  int64_t lda, ldb, ldc;       /* row strides in elements (row-major A[M,K], B[K,N], C[M,N]) */
  int64_t m, n, k;             /* full problem */
  int32_t add_zero;            /* epilogue adds +0.0 (normalises -0) as outs-init does */
  int32_t pad;
  int32_t* status;             /* device status word (KTIR_STATUS_TIMEOUT) */
} KtirGemmDesc;

/* GEMM of any shape with the reference's rounding of each K block: C (f16) =
 * the running sum over K blocks of block_k of f16(A_blk @ B_blk) (each block
 * product summed in f32 and rounded to f16, as NumPy multiplies f16 tiles),
 * the running sum rounded to f16 after each block when acc_f16, else kept in
 * f32 and rounded once at the end.  block_k = 0: one block of all of K.  Rows,
 * columns and k past the matrix read as zero; only C[0:m, 0:n] is written.
 * lda, ldb multiples of 8 elements; a, b 16-byte aligned. */
typedef struct {
  void* a; void* b; void* c;
  int64_t lda, ldb, ldc;
  int64_t m, n, k;
  int32_t block_k;             /* multiple of 16, or 0 */
  int32_t acc_f16;
  int32_t* status;
} KtirGemmBlockedDesc;

/* Causal flash attention over [bh, seq, d] f16 tensors laid out as
 * [bh*seq, d] rows; scale applied to S in f32; online softmax in f32. */
typedef struct {
  void* q; void* k; void* v; void* o;
  int64_t bh, seq, d;
  float scale;
  int32_t causal;
  int64_t row_stride;          /* elements between consecutive rows (= d for dense) */
  int32_t* status;             /* device status word (KTIR_STATUS_TIMEOUT) */
} KtirFmhaDesc;

/* One step of an attention call split over the sequence (query tiles on this
 * GPU, key tiles arriving from others).  Q and O are [bh*seq, 128] f16
 * row-major; the call computes query tiles qtiles[0..n_qtiles) (128 rows
 * each) of every head.  Key tile kt (128 rows) of head h is row
 * ((kv_owner[kt] * bh + h) * kv_tiles + kv_local[kt]) * 128 of K and V
 * (kv_rows rows of 128 f16 each): the blocks of each GPU's share of the
 * sequence are stored together, one share after the other.  Only key tiles
 * in key_mask (bit kt) are added, up to the query tile when causal.  The
 * online-softmax state of each (head, query tile) is carried between steps in
 * o_acc (bh * n_qtiles blocks of [128 columns][128 rows] f32) and ml (bh *
 * n_qtiles * 128 (max, sum) f32 pairs); flags bit 0 = first step (no state
 * read), bit 1 = last step (O written as f16, no state written).  seq <= 4096. */
typedef struct {
  const void* q;
  const void* k;
  const void* v;
  void* o;
  int64_t bh, seq, d;
  int64_t kv_rows;
  float scale;
  int32_t causal;
  int32_t n_qtiles;
  int32_t kv_tiles;
  uint32_t key_mask;
  int32_t flags;
  float* o_acc;
  float* ml;
  int32_t* status;
  uint8_t qtiles[32];
  uint8_t kv_owner[32];
  uint8_t kv_local[32];
} KtirFmhaPartDesc;

/* ----------------------------------------------------------------------- */

/* Library version (major*100 + minor). */
int ktir_version(void);
/* Message of the last failure on this thread ("" if none). */
const char* ktir_last_error(void);
/* Number of visible CUDA devices. */
int ktir_device_count(int* count);

/* Elementwise program over n_units units (replaces the arith/math handlers,
 * ktir_cpu/dialects/arith_ops.py:40-448, math_ops.py:24-110, and the
 * rectangular ktdp.load/store copies, ops/memory_ops.py:438-587). */
int ktir_ew(const KtirEwProgram* prog, const KtirBuffers* bufs, const int64_t* unit_table,
            void* stream);

/* Fused row softmax (replaces the linalg.reduce max/sum tree folds,
 * ktir_cpu/dialects/linalg_ops.py:86-219, and the elementwise chain between them). */
int ktir_softmax_rows(const KtirSoftmaxDesc* desc, const KtirBuffers* bufs,
                      const int64_t* unit_table, void* stream);

/* Indirect gather -> elementwise -> indirect scatter with the reference's
 * sequential-unit read-modify-write semantics (replaces MemoryOps.indirect_load /
 * indirect_store, ktir_cpu/ops/memory_ops.py:589-630, 914-966).  `counts` is
 * an int32 scratch array of one entry per table row, zero on entry and left
 * zero on exit; `status` receives KTIR_STATUS_NEGATIVE_INDEX. */
int ktir_gather_rmw(const KtirGatherRmwDesc* desc, const KtirBuffers* bufs, int32_t* counts,
                    int64_t n_rows, int32_t* status, void* stream);

/* Generic-path kernels (linalg.reduce tree fold, linalg.matmul on CUDA cores,
 * coordinate-set gathers/scatters, indirect access tiles). */
int ktir_reduce(const KtirReduceDesc* desc, const KtirBuffers* bufs, void* stream);
int ktir_matmul(const KtirMatmulDesc* desc, const KtirBuffers* bufs, const int64_t* unit_table,
                void* stream);
int ktir_offsets(const KtirOffsetsDesc* desc, const KtirBuffers* bufs, const int64_t* unit_table,
                 const int64_t* offsets, void* stream);
int ktir_indirect(const KtirIndirectDesc* desc, const KtirBuffers* bufs,
                  const int64_t* unit_table, const int64_t* direct, const int64_t* idx_offs,
                  int32_t* status, void* stream);

/* Allocation-free ktir_gather_rmw for callers that cannot allocate device
 * memory (no counterpart in the reference, which has no device memory).
 * The per-row count scratch is a file-scope __device__ array of
 * KTIR_STATIC_RMW_MAX_ROWS int32 (4 MiB) that every GPU loading this library
 * holds until the process exits; tables with more rows are rejected with
 * KTIR_ERR_UNSUPPORTED.  The first call on a device looks up the array's
 * device address (make that first call before any stream capture).  A call
 * that runs the count pass (phases 0 or 1) first clears the first n_rows
 * counts on `stream`; an apply-only call (phases 2) uses the counts its
 * count-only call left, so the two must go on one stream with no other call
 * of this entry point between them.  All calls share the one array, so calls
 * that overlap on the GPU (other streams, other threads) race and give wrong
 * results.  Allocates nothing: no cudaMalloc/cudaFree. */
#define KTIR_STATIC_RMW_MAX_ROWS (1 << 20)
int ktir_gather_rmw_static(const KtirGatherRmwDesc* desc, const KtirBuffers* bufs,
                           int64_t n_rows, int32_t* status, void* stream);

/* Failure-detection self test: a single thread waits, with at most
 * `spin_limit` polls (1 .. 2^20), on a barrier nothing arrives at, then sets
 * KTIR_STATUS_TIMEOUT in *status and returns — the bounded wait every
 * tensor-core kernel uses, exercised without faulting or hanging a GPU.
 * (No counterpart in the reference, whose cores are host generators.) */
int ktir_wait_selftest(int32_t* status, uint32_t spin_limit, void* stream);

/* tcgen05 GEMM (replaces the linalg.matmul K loop, ktir_cpu/dialects/linalg_ops.py:273-297
 * with ops/arith_ops.py:403-419, for whole-matrix tilings).  M, N, K multiples
 * of 128, 128, 64; persistent over 128 x 256 output tiles, or 128 x 128 ones
 * when N is not a multiple of 256 or the 256-wide tiles would not fill half
 * the SMs. */
int ktir_gemm_f16(const KtirGemmDesc* desc, void* stream);

/* tcgen05 GEMM of any shape with per-block f16 rounding (see
 * KtirGemmBlockedDesc): linalg.matmul of f16 tiles inside a K loop, and
 * whole-matrix tilings the aligned kernel does not take
 * (ktir_cpu/dialects/linalg_ops.py:273-297, ops/arith_ops.py:403-419). */
int ktir_gemm_f16_blocked(const KtirGemmBlockedDesc* desc, void* stream);

/* Causal attention (replaces the online-softmax scf.for of matmul / reduce /
 * exp ops the attention rewrite recognises). */
int ktir_fmha_f16(const KtirFmhaDesc* desc, void* stream);

/* `rows` device-to-device copies of `width` bytes, row i from src + i *
 * src_pitch to dst + i * dst_pitch, on `stream` (packs the K/V rows of one
 * GPU's query tiles into its share of the ring's staging buffer; no
 * counterpart in the reference, whose memory is one NumPy array). */
int ktir_copy_blocks(void* dst, int64_t dst_pitch, const void* src, int64_t src_pitch,
                     int64_t width, int64_t rows, void* stream);

/* Packs the K and V rows of the 128-row tiles in tile_mask (bit t = tile t
 * of every head's seq rows) from [bh*seq, d] f16 K and V into dst as
 * [K | V][head][i-th tile of the mask][128][d]: one GPU's share of the K/V
 * blocks that the sequence-split attention passes between GPUs (no
 * counterpart in the reference, which runs on one host). */
int ktir_pack_kv(void* dst, const void* k, const void* v, int64_t bh, int64_t seq, int64_t d,
                 uint32_t tile_mask, void* stream);

/* dst = a - b (subtract != 0) or a + b, byte by byte modulo 256, over n
 * bytes on `stream`.  A call split across GPUs returns whole tensors by
 * summing, over the GPUs, each one's byte differences from the tensor as it
 * was uploaded (every byte changes on at most one GPU); the sum is an NCCL
 * all-reduce between the two calls.  (No counterpart in the reference, which
 * runs on one host.) */
int ktir_bytes_delta(void* dst, const void* a, const void* b, int64_t n, int32_t subtract,
                     void* stream);

/* Peer memory between the GPUs of one node, one process per GPU (no
 * counterpart in the reference, whose cores share one host memory).  A split
 * attention call's staging buffer is allocated, zeroed and exported as a
 * 64-byte CUDA IPC handle (ktir_ipc_alloc); the other processes of its
 * exchange group map it (ktir_ipc_open, unmapped with ktir_ipc_close) and
 * pull K/V shares from it with the copy engines (ktir_copy_async).  32-bit
 * epoch flags in the owners' buffers order the copies across processes:
 * ktir_flag_set stores `value` at `flag` (local or a peer's) after the
 * stream's earlier work, with release semantics at system scope;
 * ktir_flag_wait holds the stream's later work until each of the n flags at
 * flags[i * stride] has reached `value` (modulo 2^32), polling with acquire
 * loads at most spin_limit times (1 .. 2^26, a short sleep between polls),
 * and on running out sets KTIR_STATUS_TIMEOUT in *status and lets the stream
 * go on. */
int ktir_ipc_alloc(int64_t bytes, void** ptr, void* handle);
int ktir_ipc_open(const void* handle, void** ptr);
int ktir_ipc_close(void* ptr);
int ktir_ipc_free(void* ptr);
int ktir_flag_set(uint32_t* flag, uint32_t value, void* stream);
int ktir_flag_wait(const uint32_t* flags, int32_t n, int32_t stride, uint32_t value,
                   uint32_t spin_limit, int32_t* status, void* stream);
int ktir_copy_async(void* dst, const void* src, int64_t bytes, void* stream);

/* One step of a sequence-split attention call (see KtirFmhaPartDesc): the
 * online-softmax K/V loop of the attention rewrite restricted to the key
 * tiles one GPU holds at that step of the ring that passes K/V blocks
 * between GPUs (the reference passes no data between cores: every core reads
 * HBM, ktir_cpu/ops/memory_ops.py:438-587). */
int ktir_fmha_f16_part(const KtirFmhaPartDesc* desc, void* stream);

/* Host staging for calls made with host buffers (the reference keeps a
 * call's arrays in host memory, ktir_cpu/interpreter.py:137-177 and
 * ktir_cpu/memory.py:201-288; here they travel to the device and back).
 * `pinned` is page-locked host memory of at least `bytes`, `device` device
 * memory of at least `bytes`. */
typedef struct {
  const void* host;            /* upload: source; download: destination (void* cast) */
  void* pinned;
  void* device;
  int64_t bytes;
} KtirHostXfer;

typedef struct {
  void* dst;
  const void* src;
  int64_t bytes;
} KtirHostCopy;

/* Number of host worker threads the staging copies run on
 * (KTIR_HOST_THREADS, default min(16, hardware threads / LOCAL_WORLD_SIZE)). */
int ktir_host_threads(void);

/* host -> pinned copies in chunks on the worker threads, at most
 * KTIR_UPLOAD_INFLIGHT (default 8, 0 = all) queued at a time; each chunk's
 * host-to-device copy is enqueued on `stream` as soon as it is staged.
 * Returns once every copy is enqueued (the pinned buffers must then stay
 * untouched until the stream has passed them). */
int ktir_host_upload(const KtirHostXfer* x, int n, int device, void* stream);

/* Enqueues the device-to-pinned copies of `x` on `stream` (after whatever the
 * stream already holds), copies each chunk on to its host destination as soon
 * as it lands (no copy where `host` is the pinned buffer itself), runs the
 * `extra` host-to-host copies meanwhile, and returns after all of them and
 * the stream have completed. */
int ktir_host_download(const KtirHostXfer* x, int n, const KtirHostCopy* extra, int m,
                       int device, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* KTIR_B200_H */
