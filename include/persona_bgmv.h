/*
 * persona_bgmv.h -- C ABI of the B200 (sm_100a) multi-LoRA BGMV / SGMV ops.
 *
 * Plain pointers, sizes and a cudaStream_t; no torch types.  Every function
 * returns PERSONA_OK (0) or a PERSONA_ERR_* status synchronously after
 * validating its arguments on the host and enqueuing its kernels on
 * `stream`.  Conditions only the device can see (a slot outside [-1, S), a
 * bounded wait that gave up) are ORed into the caller's device error word
 * `dev_err` (a device or host-mapped int32; may be NULL to ignore them).
 *
 * Layouts (element strides, 16-bit elements unless noted):
 *   x      [T, K]  row stride ldx          fp16 or bf16
 *   a_pool [S, R, K] slot stride a_slot_stride, row stride a_row_stride
 *   b_pool [S, N, R] slot stride b_slot_stride, rows of R contiguous values
 *   v      [T, R]  fp32, contiguous
 *   y      [T, N]  row stride ldy, same 16-bit type as x
 *   slots  [T]     int32; -1 = no adapter for this row
 * The LoRA scale alpha/r is folded into b_pool by the pool loader; no op
 * takes a scale.  All base pointers must be 16-byte aligned and K, N, ldx,
 * ldy and the strides multiples of 8 (the reference's own preconditions,
 * csrc/bgmv_shrink.cu:100-104, csrc/bgmv_expand.cu:107-111).
 */
#ifndef PERSONA_BGMV_H
#define PERSONA_BGMV_H

#include <stddef.h>
#include <stdint.h>

#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PERSONA_ABI_VERSION 1

/* 16-bit storage types of x / pools / y. */
#define PERSONA_DTYPE_F16 0
#define PERSONA_DTYPE_BF16 1

/* Host-side status codes. */
#define PERSONA_OK 0
#define PERSONA_ERR_INVALID_ARG 1 /* null pointer, negative size, bad flag   */
#define PERSONA_ERR_SHAPE 2       /* inconsistent or unsupported dimensions  */
#define PERSONA_ERR_DTYPE 3       /* dtype code not F16/BF16                 */
#define PERSONA_ERR_ALIGNMENT 4   /* pointer or stride not 16-byte aligned   */
#define PERSONA_ERR_RANK 5        /* LoRA rank this op does not support      */
#define PERSONA_ERR_WORKSPACE 6   /* workspace missing or too small          */
#define PERSONA_ERR_CUDA 7        /* CUDA runtime / launch failure           */
#define PERSONA_ERR_NOALLOC_ROWS 8 /* T above PERSONA_NOALLOC_MAX_ROWS          */

/* Device error-word bits (ORed into *dev_err by the kernels). */
#define PERSONA_DEV_ERR_SLOT 1    /* a slot < -1 or >= S: that row was left alone */
#define PERSONA_DEV_ERR_TIMEOUT 2 /* a bounded wait gave up                       */
#define PERSONA_DEV_ERR_SEGMENT 4 /* SGMV segment table out of order or range     */
#define PERSONA_DEV_ERR_PLAN 8    /* PERSONA_REUSE_PLAN: the workspace holds no plan
                                     for this T and S (nothing was computed), or a
                                     plan entry was out of range (that item skipped) */

/* Flags of the BGMV ops. */
#define PERSONA_REUSE_PLAN 1 /* workspace already holds the plan of these slots */
#define PERSONA_SPLIT_ONLY 2 /* fused ops: always the split kernels, also at decode sizes */
/* Fused ops on at most PERSONA_SMALL_MAX_ROWS rows (K <= 32768) run a kernel
 * without cross-CTA steps: each CTA recomputes its row's v and writes one
 * column slice.  Larger batches, or PERSONA_SPLIT_ONLY, use the split
 * kernels.  Both leave the plan in the workspace when REUSE_PLAN is unset.  */
#define PERSONA_SMALL_MAX_ROWS 64

const char* persona_status_string(int status);
int persona_abi_version(void);

/* ---- row grouping plan --------------------------------------------------
 * The BGMV kernels stream each used adapter's A and B once for all rows that
 * share it.  The plan (built on the device, no host sync) groups the rows of
 * `slots` by slot into items of at most 16 rows.  One plan serves every
 * projection of a decode step that shares the slot vector.
 * No reference counterpart: the reference validates and visits slots row by
 * row with a host sync per row (csrc/bgmv_shrink.cu:106-109).               */
size_t persona_bgmv_workspace_size(int64_t T);
int persona_bgmv_plan(const int32_t* slots, int64_t T, int64_t S, void* workspace,
                      size_t workspace_bytes, int32_t* dev_err, cudaStream_t stream);

/* ---- BGMV shrink --------------------------------------------------------
 * v[t, :] = A[slots[t]] @ x[t, :] in fp32; rows with slot -1 get zeros.
 * Replaces bgmv_shrink_cuda (csrc/bgmv_shrink.cu:81-122) behind
 * torch.ops.persona.bgmv_shrink (csrc/bindings.cpp:20).  R in {8,16,32,64}
 * runs the split kernel over a plan; any other R runs a row-by-row kernel.  */
int persona_bgmv_shrink(const void* x, int64_t ldx, const void* a_pool, int64_t a_slot_stride,
                        int64_t a_row_stride, const int32_t* slots, float* v, int64_t T,
                        int64_t K, int64_t R, int64_t S, int dtype, void* workspace,
                        size_t workspace_bytes, int flags, int32_t* dev_err,
                        cudaStream_t stream);

/* ---- BGMV expand --------------------------------------------------------
 * y[t, :] = round(y[t, :] + B[slots[t]] @ v[t, :]) (fp32 sum, one rounding);
 * rows with slot -1 are left bit-identical.  R in {8,16,32,64}, as in
 * the reference.  Replaces bgmv_expand_cuda (csrc/bgmv_expand.cu:88-129)
 * behind torch.ops.persona.bgmv_expand (csrc/bindings.cpp:21).             */
int persona_bgmv_expand(const float* v, const void* b_pool, int64_t b_slot_stride,
                        const int32_t* slots, void* y, int64_t ldy, int64_t T, int64_t N,
                        int64_t R, int64_t S, int dtype, void* workspace,
                        size_t workspace_bytes, int flags, int32_t* dev_err,
                        cudaStream_t stream);

/* ---- fused BGMV shrink -> expand -----------------------------------------
 * y[t, :] = round(y[t, :] + B[s] @ (A[s] @ x[t, :])) in one launch; the
 * rank-R intermediate never goes through HBM as a tensor (its K-slice
 * partials meet in L2-resident workspace).  The reference's fused kernel is a
 * stub (docs/BENCHMARKS.md:238);
 * its result equals bgmv_shrink followed by bgmv_expand
 * (persona/ops.py:59-68).  R in {8,16,32,64}.                              */
int persona_bgmv_fused(const void* x, int64_t ldx, const void* a_pool, int64_t a_slot_stride,
                       int64_t a_row_stride, const void* b_pool, int64_t b_slot_stride,
                       const int32_t* slots, void* y, int64_t ldy, int64_t T, int64_t K,
                       int64_t N, int64_t R, int64_t S, int dtype, void* workspace,
                       size_t workspace_bytes, int flags, int32_t* dev_err,
                       cudaStream_t stream);

/* ---- fused BGMV over several projections in one launch ------------------
 * No reference counterpart (the reference launches shrink and expand per
 * projection; persona/lora_layer.py:55-57).  Up to PERSONA_MAX_PROBLEMS
 * projections of one decoder layer (q/k/v/o/gate/up/down) that share the
 * batch's slots, the rank R, the pool size S and the dtype run as one
 * launch: each problem has its own x, pools (strides as for
 * persona_bgmv_fused) and y, and the result of each equals
 * persona_bgmv_fused on it.  The plan depends only on the slots, so
 * PERSONA_REUSE_PLAN works with a plan built by persona_bgmv_plan on this
 * workspace.  Workspace: persona_bgmv_multi_workspace_size(T, num_problems). */
#define PERSONA_MAX_PROBLEMS 8
typedef struct persona_bgmv_problem {
  const void* x;
  int64_t ldx;
  const void* a_pool;
  int64_t a_slot_stride;
  int64_t a_row_stride;
  const void* b_pool;
  int64_t b_slot_stride;
  void* y;
  int64_t ldy;
  int64_t K;
  int64_t N;
} persona_bgmv_problem;
/* LoRA term alone at decode sizes (T <= PERSONA_SMALL_MAX_ROWS):
 * deltas[i][t, n] = (B_i[s] (A_i[s] x_i[t]))[n] in fp32, 0 for rows without an
 * adapter; the problems' y / ldy are ignored.  Same math as the fused op
 * (reference persona/ops.py:12-56) without the add into y, for callers that
 * fold the term into the base projection's output (persona_nf4_linear_add). */
int persona_bgmv_lora_delta_multi(const persona_bgmv_problem* problems, int num_problems, float* const* deltas,
                                  const int64_t* ld_deltas, const int32_t* slots, int64_t T, int64_t R, int64_t S,
                                  int dtype, int32_t* dev_err, cudaStream_t stream);
size_t persona_bgmv_multi_workspace_size(int64_t T, int num_problems);
int persona_bgmv_fused_multi(const persona_bgmv_problem* problems, int num_problems, const int32_t* slots,
                             int64_t T, int64_t R, int64_t S, int dtype, void* workspace, size_t workspace_bytes,
                             int flags, int32_t* dev_err, cudaStream_t stream);

/* ---- segmented (SGMV) ------------------------------------------------------
 * A prefill batch whose rows are grouped contiguously by adapter: segment i
 * covers rows [seg_indptr[i], seg_indptr[i+1]) and uses slot seg_slots[i]
 * (-1 = no adapter).  Rows outside every segment behave like slot -1.  The
 * results equal the BGMV ops on the per-row slots the segments imply, which
 * is how the reference's callers express a prefill (LoRAContext.set_batch_slots,
 * persona/lora_layer.py:21-28); the reference itself has no segmented op.
 * seg_indptr [num_segments + 1] and seg_slots [num_segments] are int32 device
 * arrays.  A segment is used only if 0 <= lo <= hi <= T and no earlier
 * seg_indptr entry exceeds lo (used segments never overlap); any other
 * segment sets PERSONA_DEV_ERR_SEGMENT and is skipped.
 * Ranks 16 and 32 with K % 64 == 0 (shrink) and N % 64 == 0 (expand) run on
 * the tensor cores (tcgen05, accumulators in TMEM, 128-row tiles); other
 * shapes run the split BGMV kernels over the segments' rows.
 * Workspace: persona_sgmv_workspace_size(T). */
size_t persona_sgmv_workspace_size(int64_t T);
int persona_sgmv_shrink(const void* x, int64_t ldx, const void* a_pool, int64_t a_slot_stride,
                        int64_t a_row_stride, const int32_t* seg_indptr, const int32_t* seg_slots,
                        int64_t num_segments, float* v, int64_t T, int64_t K, int64_t R, int64_t S,
                        int dtype, void* workspace, size_t workspace_bytes, int32_t* dev_err,
                        cudaStream_t stream);
int persona_sgmv_expand(const float* v, const void* b_pool, int64_t b_slot_stride,
                        const int32_t* seg_indptr, const int32_t* seg_slots, int64_t num_segments,
                        void* y, int64_t ldy, int64_t T, int64_t N, int64_t R, int64_t S, int dtype,
                        void* workspace, size_t workspace_bytes, int32_t* dev_err, cudaStream_t stream);
int persona_sgmv_fused(const void* x, int64_t ldx, const void* a_pool, int64_t a_slot_stride,
                       int64_t a_row_stride, const void* b_pool, int64_t b_slot_stride,
                       const int32_t* seg_indptr, const int32_t* seg_slots, int64_t num_segments,
                       void* y, int64_t ldy, int64_t T, int64_t K, int64_t N, int64_t R, int64_t S,
                       int dtype, void* workspace, size_t workspace_bytes, int32_t* dev_err,
                       cudaStream_t stream);

/* ---- fused BGMV without any allocation -----------------------------------
 * No reference counterpart.  Same operation, arguments and results as
 * persona_bgmv_fused, minus the workspace: the workspace (row-grouping plan,
 * the split kernel's partial sums and counters) lives in a fixed device
 * array inside this library, one per device, about 6.7 MB, held by every
 * GPU that loads the library until the process exits.  The call needs no
 * buffer from the caller and allocates nothing itself.  It serves callers
 * that cannot hand out device memory per call: an engine that has already
 * carved all of HBM into its own pools (KV cache, adapter pool), or a host
 * binding with no device allocator of its own.
 * Limits and rules:
 *  - T <= PERSONA_NOALLOC_MAX_ROWS; a larger T returns
 *    PERSONA_ERR_NOALLOC_ROWS and enqueues nothing.
 *  - The first call on a device does a one-time set-up: it looks the
 *    array's device address up (cudaGetSymbolAddress, with that device
 *    current) and keeps it.  Make that first call on each device before any
 *    stream capture begins.
 *  - Nothing in the array has to start at zero: each call rewrites the plan
 *    and resets the counters before the kernel reads them.  Calls of at most
 *    PERSONA_SMALL_MAX_ROWS rows run the decode-sized kernel and do not
 *    touch the array.
 *  - All calls on one device share the array: calls whose device work can
 *    overlap (different streams, unsynchronised threads) race and must be
 *    serialised, e.g. on one stream.                                        */
#define PERSONA_NOALLOC_MAX_ROWS 8192
int persona_bgmv_fused_noalloc(const void* x, int64_t ldx, const void* a_pool, int64_t a_slot_stride,
                               int64_t a_row_stride, const void* b_pool, int64_t b_slot_stride,
                               const int32_t* slots, void* y, int64_t ldy, int64_t T, int64_t K,
                               int64_t N, int64_t R, int64_t S, int dtype, int32_t* dev_err,
                               cudaStream_t stream);

/* ---- tensor-parallel segmented fused, one kernel with its exchange -------
 * No reference counterpart (the reference is single-GPU).  Rank r of a group
 * computes columns [n0, n1) of y += B[s] @ (A[s] @ x) for a segmented batch
 * (same arguments as persona_sgmv_fused; b_pool and y cover all N columns)
 * and writes every finished tile both to its own y and, over NVLink, to the
 * y of every other rank: peer_ys[0..num_peers) are those ranks' y buffers
 * mapped into this process (persona_ipc_import), same shape and ldy.  After
 * the launch and a cross-rank barrier (any collective on this stream) every
 * rank holds the full updated y.  Tensor-core shapes only: R in {16, 32, 64},
 * K % 64 == 0, N % 64 == 0, n0 and n1 multiples of 64; at most
 * PERSONA_MAX_TP_PEERS peers.  The ranks' y must hold the same values before
 * the call (rows outside every segment are not written).                   */
#define PERSONA_MAX_TP_PEERS 7
int persona_sgmv_fused_tp(const void* x, int64_t ldx, const void* a_pool, int64_t a_slot_stride,
                          int64_t a_row_stride, const void* b_pool, int64_t b_slot_stride, const int32_t* seg_indptr,
                          const int32_t* seg_slots, int64_t num_segments, void* y, int64_t ldy, void* const* peer_ys,
                          int num_peers, int64_t n0, int64_t n1, int64_t T, int64_t K, int64_t N, int64_t R,
                          int64_t S, int dtype, void* workspace, size_t workspace_bytes, int32_t* dev_err,
                          cudaStream_t stream);

/* Cross-process mapping of a device buffer (CUDA IPC) for the peer_ys above:
 * export a 64-byte handle plus the buffer's offset in its allocation on the
 * owning rank, import it on the others (returns the buffer pointer and the
 * mapping base to close later).                                            */
int persona_ipc_export(const void* ptr, void* handle, size_t* offset);
int persona_ipc_import(const void* handle, size_t offset, void** ptr, void** base);
int persona_ipc_close(void* base);

/* ---- NF4 base linears ------------------------------------------------------
 * The base weights under the LoRA layers of the end-to-end decode.  The
 * reference runs them through bitsandbytes' Linear4bit (reference
 * bench/e2e.py:70-90: nf4, blocksize 64, double-quantised scales, fp16
 * compute) as MultiLoRALinear.base (persona/lora_layer.py:30-45); these entry
 * points replace that layer.  fp16 only; N and K multiples of 128.
 *
 * Storage, per 128 x 128 tile of W[N, K], tiles of a row of tiles adjacent:
 * PERSONA_NF4_CHUNK_BYTES bytes = 8192 bytes of 4-bit codes in the A-fragment
 * order of mma.m16n8k16, 256 int8 scale codes (one per 64 weights of a row),
 * an fp32 scale step s127 and 12 zero bytes.  A block's scale is
 * f32(code) * s127 + offset, offset one fp32 per matrix in device memory.  */
#define PERSONA_NF4_CHUNK_BYTES 8464
#define PERSONA_NF4_MAX_PROBLEMS 4
size_t persona_nf4_packed_bytes(int64_t N, int64_t K);
size_t persona_nf4_quantize_workspace_size(int64_t N, int64_t K);
/* w: fp16 [N, K], row stride ldw (a multiple of 8), 16-byte aligned;
 * packed: persona_nf4_packed_bytes(N, K); offset: one device float.         */
int persona_nf4_quantize(const void* w, int64_t ldw, int64_t N, int64_t K, void* packed, float* offset,
                         void* workspace, size_t workspace_bytes, cudaStream_t stream);
/* W[n, k] = fp16(fp32(NF4 value) * scale) into w (row stride ldw).          */
int persona_nf4_dequantize(const void* packed, const float* offset, int64_t N, int64_t K, void* w, int64_t ldw,
                           cudaStream_t stream);
/* One base linear of a launch: y[M, N] = x[M, K] W^T, fp32 accumulate, one
 * rounding to fp16.  x rows 16-byte aligned (ldx a multiple of 8).          */
typedef struct persona_nf4_problem {
  const void* packed;
  const float* offset;
  const void* x;
  int64_t ldx;
  void* y;
  int64_t ldy;
  int64_t N;
  int64_t K;
} persona_nf4_problem;
/* Workspace of persona_nf4_linear: zero-filled before its first use (calls
 * leave its counters at zero again); one launch at a time per workspace.
 * Its size depends on the current device's SM count (two fp32 tile pieces
 * per CTA); a call that finds it too small returns PERSONA_ERR_WORKSPACE.   */
size_t persona_nf4_linear_workspace_size(const persona_nf4_problem* problems, int num_problems);
/* Up to PERSONA_NF4_MAX_PROBLEMS linears in one launch (e.g. q / k / v on the
 * same x); any M (launches of at most 64 rows each).                        */
int persona_nf4_linear(const persona_nf4_problem* problems, int num_problems, int64_t M, void* workspace,
                       size_t workspace_bytes, int32_t* dev_err, cudaStream_t stream);
/* The same with an fp32 addend per problem (addends[i] may be NULL):
 * y = fp16(x W^T + addend), one rounding.  With the LoRA delta below as the
 * addend this is the patched projection base(x) + B[s] A[s] x of the
 * reference's MultiLoRALinear (persona/lora_layer.py:30-57) with one rounding
 * instead of two.  Launched as a programmatic dependent of the kernel before
 * it on the stream: its weight streaming starts while that kernel (which
 * writes x or the addend) finishes.                                         */
int persona_nf4_linear_add(const persona_nf4_problem* problems, int num_problems, const float* const* addends,
                           const int64_t* ld_addends, int64_t M, void* workspace, size_t workspace_bytes,
                           int32_t* dev_err, cudaStream_t stream);

/* ---- end-to-end decode helpers -------------------------------------------
 * Fused elementwise steps of the Mistral-7B decoder around the LoRA layers,
 * where the reference runs Hugging Face's modules (reference
 * persona/engine.py:101-107 calls model.generate).  fp16, head dim 128.
 * add_rmsnorm: h += delta (delta may be NULL), out = w * fp16(h / rms(h)),
 *   rows of D (a multiple of 8) elements.
 * rope_cache: rows r = b * per_seq + i of q [rows, Hq, 128], k, v [rows, Hkv,
 *   128] are at position *start + i of sequence b: rotate q and k in place
 *   (rotate-half, base theta) and store k, v into the caches [B, Hkv, L, 128].
 * silu_mul: out = fp16(silu(g)) * u over n elements (a multiple of 8).
 * decode_attention: one new token per sequence, softmax(q K^T scale) V over
 *   the first *len cache positions; q, out [B, Hq, 128], Hq / Hkv <= 8.      */
int persona_add_rmsnorm(void* h, const void* delta, const void* w, void* out, int64_t rows, int64_t D, float eps,
                        cudaStream_t stream);
int persona_rope_cache(void* q, void* k, const void* v, void* k_cache, void* v_cache, const int32_t* start,
                       int64_t rows, int64_t per_seq, int64_t Hq, int64_t Hkv, int64_t L, float theta,
                       cudaStream_t stream);
int persona_silu_mul(const void* g, const void* u, void* out, int64_t n, cudaStream_t stream);
int persona_decode_attention(const void* q, const void* k_cache, const void* v_cache, const int32_t* len, void* out,
                             int64_t B, int64_t Hq, int64_t Hkv, int64_t L, float scale, cudaStream_t stream);
/* rope_cache (per_seq 1, start = pos) and decode_attention in one launch,
 * with the same results: each (sequence, kv head) rotates its query heads
 * and its k head in place, writes k and v to the caches at *pos, then
 * attends over the first *len positions.  The two steps of the reference's
 * attention module at decode (rotary embedding, then SDPA over the cache).  */
int persona_rope_decode_attention(void* q, void* k, const void* v, void* k_cache, void* v_cache, const int32_t* pos,
                                  const int32_t* len, void* out, int64_t B, int64_t Hq, int64_t Hkv, int64_t L,
                                  float theta, float scale, cudaStream_t stream);

/* ---- warm-up GEMV ---------------------------------------------------------
 * y[n] = W[n, :] @ x (fp16, fp32 accumulate).  Replaces
 * persona::gemv_fp16_cuda (csrc/gemv_fp16.cu:33-50), kept so that
 * torch.ops.persona.gemv_fp16 (csrc/bindings.cpp:22) stays registered.     */
int persona_gemv_fp16(const void* x, const void* W, void* y, int64_t K, int64_t N,
                      cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* PERSONA_BGMV_H */
