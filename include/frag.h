/*
 * frag.h — C ABI of libfrag.so, the B200 (sm_100a) kernels for the memory-bound
 * Llama training-graph fragments collected in SherlockNoMad/KernelProblems.
 *
 * The reference exposes each fragment as a Python `kernel_function(*inputs)`
 * (a drop-in for the fragment's torch `Model.forward`).  These entry points are
 * what such a function binds to: plain device pointers, element counts and
 * strides, a CUDA stream, and an integer status.  No torch types cross this
 * boundary.
 *
 * Conventions shared by every entry point
 *   - bf16 tensors are passed as `const void*` / `void*` holding IEEE bfloat16
 *     bit patterns; fp32 tensors as `float*`; indices as int64 unless stated.
 *   - Row-major, innermost dimension contiguous.  Fast paths need 16-byte
 *     aligned base pointers and a row size that is a multiple of 8 bf16
 *     elements; other shapes run a slower generic kernel, never a CPU path.
 *   - Every call is asynchronous on `stream` (the caller's current stream) and
 *     never synchronises.  Inputs are read-only; outputs are caller-owned.
 *   - Return value: FRAG_OK (0) or one of the frag_status codes below.  Shape
 *     and pointer checks happen on the host before any launch; a failed launch
 *     returns FRAG_ERR_CUDA and frag_last_cuda_error() gives the cudaError_t.
 *   - Device-detected input errors (an index outside the table) are written to
 *     the optional `status` word (device memory, int32) with atomicOr of the
 *     FRAG_DEVFLAG_* bits; the call itself still returns FRAG_OK because the
 *     host cannot see device data without synchronising.
 *   - Entry points that need scratch memory take a caller-provided workspace
 *     and expose a *_workspace_bytes() size query; nothing here allocates
 *     except frag_peer_alloc (the one-time buffers a multi-GPU peer exchange
 *     shares between processes).
 */
#ifndef FRAG_H_
#define FRAG_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define FRAG_API __attribute__((visibility("default")))
#else
#define FRAG_API
#endif

typedef struct CUstream_st* frag_stream_t; /* == cudaStream_t */

enum frag_status {
  FRAG_OK = 0,
  FRAG_ERR_INVALID_ARG = 1, /* null pointer where one is required, negative size */
  FRAG_ERR_SHAPE = 2,       /* shape not supported by any kernel variant        */
  FRAG_ERR_ALIGN = 3,       /* misaligned pointer or stride                      */
  FRAG_ERR_WORKSPACE = 4,   /* workspace missing or smaller than the query says  */
  FRAG_ERR_CUDA = 5,        /* a CUDA runtime call or launch failed              */
  FRAG_ERR_NO_DEVICE = 6,   /* no CUDA device is visible                         */
  FRAG_ERR_SCRATCH_LIMIT = 7 /* needs more than the static scratch of a no-alloc entry point */
};

/* Bits written into a caller's device status word by kernels. */
enum frag_devflag {
  FRAG_DEVFLAG_INDEX_OOB = 1,   /* an embedding id was outside [0, vocab_total)  */
  FRAG_DEVFLAG_WAIT_TIMEOUT = 2 /* a kernel gave up waiting for its own copies  */
};

/* RoPE layouts.  NEOX pairs element i with i + D/2 (rotate-half);
 * INTERLEAVED pairs 2i with 2i+1 (complex view, the reference's layout). */
enum frag_rope_layout { FRAG_ROPE_NEOX = 0, FRAG_ROPE_INTERLEAVED = 1 };

/* RoPE output element types (frag_rope_tensor.out_dtype). */
enum frag_rope_out { FRAG_ROPE_OUT_BF16 = 0, FRAG_ROPE_OUT_F32 = 1 };

/* RoPE input element types (frag_rope_tensor.in_dtype). */
enum frag_rope_in { FRAG_ROPE_IN_BF16 = 0, FRAG_ROPE_IN_F32 = 1 };

/* Element types of frag_convert_rows. */
enum frag_dtype { FRAG_DT_BF16 = 0, FRAG_DT_F32 = 1 };

/* Position tensor dtypes for RoPE. NONE means position = token index s. */
enum frag_pos_dtype { FRAG_POS_NONE = 0, FRAG_POS_I32 = 1, FRAG_POS_I64 = 2 };

FRAG_API const char* frag_version(void);
FRAG_API const char* frag_status_string(int status);
/* cudaError_t of the most recent FRAG_ERR_CUDA on this host thread. */
FRAG_API int frag_last_cuda_error(void);

/* ------------------------------------------------------------------------- *
 * RMSNorm forward with saved rstd.
 *   rstd[m] = 1 / sqrt(mean_n(x[m,n]^2) + eps)            (fp32 accumulation)
 *   y[m,n]  = bf16((x[m,n] * rstd[m]) * w[n])
 * Replaces aten._fused_rms_norm as called by
 *   v8/f4e9e58fef73/problem.py:28 (y + rstd) and its Triton drop-in
 *   v8/f4e9e58fef73/optimized_kernel.py:43 `kernel_function(add_recomputed, weight)`,
 *   v8/4b90e2d83144/optimized_kernel.py:30 `kernel_function(embedding, weight, eps)`.
 * x, y: bf16 [M,N]; w: bf16 [N]; rstd: fp32 [M] or NULL.
 * ------------------------------------------------------------------------- */
FRAG_API int frag_rmsnorm_fwd(const void* x, const void* w, void* y, float* rstd,
                     int64_t M, int64_t N, float eps, frag_stream_t stream);

/* ------------------------------------------------------------------------- *
 * Residual add + RMSNorm forward.
 *   h = bf16(res + x);  rstd, y as frag_rmsnorm_fwd applied to h.
 * Replaces aten.add -> aten._fused_rms_norm of
 *   v8/7884328a5557/problem.py:20,23 and its drop-in
 *   v8/7884328a5557/optimized_kernel.py:37 `kernel_function(mm_220, add_61, w)`.
 * res, x, h, y: bf16 [M,N]; h and rstd may be NULL (not written).
 * ------------------------------------------------------------------------- */
FRAG_API int frag_add_rmsnorm_fwd(const void* res, const void* x, const void* w, void* h,
                         void* y, float* rstd, int64_t M, int64_t N, float eps,
                         frag_stream_t stream);

/* ------------------------------------------------------------------------- *
 * RMSNorm backward (dx and a deterministic column-reduced dweight), with the
 * optional residual-stream adds of the fused backward fragments.
 *   dy      = dy2 ? bf16(dy + dy2) : dy
 *   rstd    = rstd ? rstd : 1/sqrt(mean(x^2) + eps)          (recompute)
 *   xhat    = x * rstd;  gw = dy * w
 *   dx      = (gw - xhat * mean_n(xhat * gw)) * rstd
 *   dx_out  = dres ? bf16(dres + bf16(dx)) : bf16(dx)
 *   dw[n]   = sum_m dy[m,n] * xhat[m,n]      fp32, fixed summation order
 * Replaces aten._fused_rms_norm_backward as called by
 *   v7/45990c83cfd6/problem.py:23 (recompute + bwd; drop-in
 *     v7/45990c83cfd6/optimized_kernel.py:96 `kernel_function(x, weight, grad_out, eps)`),
 *   v7/7f544ceb2120/problem.py:23-38 (add -> bwd -> add -> fp32; drop-in
 *     v7/7f544ceb2120/optimized_kernel.py:71),
 *   v8/d8f596b3df34/problem.py:23-40 (drop-in v8/d8f596b3df34/optimized_kernel.py:64).
 * dx_out: bf16 [M,N]; dw: fp32 [N] or NULL; dw_bf16: bf16 [N] or NULL.
 * workspace: frag_rmsnorm_bwd_workspace_bytes(M, N) bytes of device memory.
 * The sum over rows is split into fixed row blocks whose fp32 partials are
 * added in block order, so dw is bitwise reproducible for a given M, N and GPU.
 * ------------------------------------------------------------------------- */
FRAG_API size_t frag_rmsnorm_bwd_workspace_bytes(int64_t M, int64_t N);
FRAG_API int frag_rmsnorm_bwd(const void* dy, const void* dy2, const void* x,
                     const float* rstd, const void* w, const void* dres,
                     void* dx_out, float* dw, void* dw_bf16, int64_t M,
                     int64_t N, float eps, void* workspace,
                     size_t workspace_bytes, frag_stream_t stream);

/* As frag_rmsnorm_bwd with a third gradient term: dy = bf16(bf16(dy + dy2) +
 * dy3) (dy3 requires dy2; NULL gives frag_rmsnorm_bwd).  Same workspace.
 * Replaces add -> add -> _fused_rms_norm_backward -> add -> _to_copy of
 *   v7/ed20955ec34b/problem.py:19-44 (drop-in v7/ed20955ec34b/optimized_kernel.py:118). */
FRAG_API int frag_rmsnorm_bwd3(const void* dy, const void* dy2, const void* dy3, const void* x,
                               const float* rstd, const void* w, const void* dres,
                               void* dx_out, float* dw, void* dw_bf16, int64_t M, int64_t N,
                               float eps, void* workspace, size_t workspace_bytes,
                               frag_stream_t stream);

/* ------------------------------------------------------------------------- *
 * RMSNorm forward recomputed inside its backward (activation checkpointing),
 * one pass over the rows:
 *   h    = bf16(bf16(x + x2) + x3)          x2, x3 optional (x3 requires x2)
 *   rstd = 1/sqrt(mean(h^2) + eps)          stored to rstd_out [M] if non-NULL
 *   y    = bf16((h * rstd) * w)             stored to y_out [M, N] if non-NULL
 *   g    = bf16(bf16(dy + dy2) + dy3)       dy2, dy3 optional (dy3 requires dy2)
 *   dx_out = bf16(dres + bf16(dh))          dh the RMSNorm backward of g at (h, rstd)
 *   dw / dw_bf16 = sum_rows(g * h * rstd)   as frag_rmsnorm_bwd
 * h is never written.  Same workspace (frag_rmsnorm_bwd_workspace_bytes) and
 * dweight order as frag_rmsnorm_bwd.  Replaces the _fused_rms_norm ->
 * [add ->] _fused_rms_norm_backward -> [add ->] _to_copy regions:
 *   v6/822931829090/problem.py:19-66 (x; dy + dy2 + dy3; dres; y returned),
 *   v6/e9198b707240/problem.py:18-56 (dy + dy2; dres; y returned),
 *   v6/408ac0979ac5/problem.py:19-63 (h = x + x2; dy + dy2; dres; y returned),
 *   v6/28b45679fca1/problem.py:17-41 (h = x + x2; dy),
 *   v8/3c6c589cdf81/problem.py:18-53 (h = (x + x2) + x3; dy),
 * and their other snapshots (v1-v5).
 * ------------------------------------------------------------------------- */
FRAG_API int frag_rmsnorm_fwd_bwd(const void* x, const void* x2, const void* x3, const void* w,
                                  const void* dy, const void* dy2, const void* dy3,
                                  const void* dres, void* y_out, float* rstd_out, void* dx_out,
                                  float* dw, void* dw_bf16, int64_t M, int64_t N, float eps,
                                  void* workspace, size_t workspace_bytes, frag_stream_t stream);

/* Row-block count G of frag_rmsnorm_bwd for 16-byte aligned operands.  After
 * a frag_rmsnorm_bwd call the first G*N floats of its workspace hold the
 * per-block dweight partials [G, N] (whether or not dw was requested), which
 * multi-GPU callers may reduce across ranks themselves. */
FRAG_API int64_t frag_rmsnorm_bwd_num_blocks(int64_t M, int64_t N);
/* G for a given alignment: a call whose row pointers (dy, dy2, dy3, x, w,
 * dres, dx_out, and for frag_rmsnorm_fwd_bwd x2, x3, y_out) are not all
 * 16-byte aligned takes the generic kernels, whose row blocks differ.  Pass
 * aligned = 0 for such a call to learn the G its partials were written with.
 * No reference counterpart (a query of this library's own plan). */
FRAG_API int64_t frag_rmsnorm_bwd_plan_blocks(int64_t M, int64_t N, int aligned);
/* Sum partials[G, N] over G in order into dw (fp32) and/or dw_bf16. */
FRAG_API int frag_dw_reduce(const float* partials, int64_t G, int64_t N, float* dw,
                   void* dw_bf16, frag_stream_t stream);

/* ------------------------------------------------------------------------- *
 * RMSNorm backward that allocates nothing and takes no workspace.  This entry
 * point has no counterpart in the reference (its Triton drop-ins allocate
 * their scratch with torch.empty on every call).  It serves callers that
 * cannot obtain device memory at call time: an executor that sizes all device
 * memory before a training step and must not call cudaMalloc in the middle of
 * it (cudaMalloc can synchronise the device and stall the queued work), or a
 * plugin host whose ABI hands over tensors but neither an allocator nor a
 * workspace argument.
 * Arguments and results are those of frag_rmsnorm_bwd without the workspace.
 * The scratch lives in one static device array of FRAG_NOALLOC_SCRATCH_BYTES
 * (16 MiB) that every GPU loading this library holds until the process exits.
 * It holds the per-block dweight partials (at most 296 x N floats, 9.7 MB at
 * N = 8192, for 16-byte aligned rows with N % 8 == 0 and N <= 8192) and, only
 * when the generic kernels run (other widths or unaligned rows), also a copy
 * of rstd (M floats).  A problem whose scratch would not fit returns
 * FRAG_ERR_SCRATCH_LIMIT before anything is launched; with the generic
 * kernels that limits M to about 4 million rows (the C1 and C4
 * configurations need about 4.9 MB).
 *   - The first call on each device looks up the array's device address
 *     (cudaGetSymbolAddress, with that device current).  Make that first call
 *     before any stream capture.
 *   - Every call uses the same array, which keeps the last call's contents.
 *     Each call writes every scratch byte before reading it, so nothing has to
 *     be cleared, but calls that overlap on the GPU (e.g. on two streams at
 *     once) race on the array: keep such calls ordered on one stream.
 *   - It calls no cudaMalloc, cudaFree or other allocating routine.
 * ------------------------------------------------------------------------- */
#define FRAG_NOALLOC_SCRATCH_BYTES (16u * 1024u * 1024u)
FRAG_API int frag_rmsnorm_bwd_noalloc(const void* dy, const void* dy2, const void* x,
                                      const float* rstd, const void* w, const void* dres,
                                      void* dx_out, float* dw, void* dw_bf16, int64_t M,
                                      int64_t N, float eps, frag_stream_t stream);

/* ------------------------------------------------------------------------- *
 * Token-embedding gather (optionally one vocab shard of a vocab-parallel table).
 *   v = ids[t] - vocab_lo
 *   out[t,:] = (0 <= v < shard_rows) ? table[v,:] : 0
 * ids outside [0, vocab_total) also produce a zero row and set
 * FRAG_DEVFLAG_INDEX_OOB in *status (if status is not NULL).
 * Replaces aten.embedding of v7/1e49beb8a123/problem.py:20-23 (drop-in
 * v7/1e49beb8a123/optimized_kernel.py:34 `kernel_function(wait_tensor_871, ids)`).
 * ids: int64 [T]; table: bf16 [shard_rows, D]; out: bf16 [T, D].  Bit exact.
 * ------------------------------------------------------------------------- */
FRAG_API int frag_embedding_fwd(const int64_t* ids, const void* table, void* out,
                       int64_t T, int64_t shard_rows, int64_t D,
                       int64_t vocab_lo, int64_t vocab_total, int32_t* status,
                       frag_stream_t stream);

/* ------------------------------------------------------------------------- *
 * Vocab-parallel embedding forward fused with its exchange over NVLink peer
 * memory (one process per GPU, up to FRAG_PEER_MAX_RANKS ranks on one node).
 * Replaces the masked gather + all-reduce of the [T, D] output for the
 * 8-way vocab split of the reference's FSDP table layout
 * (v7/1e49beb8a123/problem.py:16-23 gathered across ranks); no reference
 * counterpart for the exchange itself (the reference is single-GPU).
 *   rank r owns table rows [vocab_lo, vocab_lo + shard_rows); for each token
 *   t whose id it owns it loads table_shard[id - vocab_lo] once and stores it
 *   to out_ptrs[p] + t*D for every rank p (its own output included); ids
 *   outside [0, vocab_total) give zero rows (written by rank 0) and set
 *   FRAG_DEVFLAG_INDEX_OOB in *status.  On return (stream order) this rank's
 *   output holds every token's row, bit exact.
 * out_ptrs[p]: rank p's bf16 [T, D] output, mapped into this process
 *   (frag_peer_open), out_ptrs[rank] this rank's own; flag_ptrs[p]: rank
 *   p's block of 2 * world int32 flags, zero at creation; state: this rank's
 *   own int32[2] (CTA counter, call count), zero at creation.  All three come
 *   from frag_peer_alloc buffers, exchanged once between the ranks as IPC
 *   handles.  Every rank calls with the same T, equally often; calls on one
 *   rank must be ordered on one stream.  The call count advances on the
 *   device, so the two launches take no per-call arguments and can be
 *   captured in a CUDA graph.  Every flag wait is bounded (~2 s): on expiry
 *   the wait sets FRAG_DEVFLAG_WAIT_TIMEOUT in frag_device_errors() and
 *   returns.
 * ------------------------------------------------------------------------- */
#define FRAG_PEER_MAX_RANKS 8
#define FRAG_IPC_HANDLE_BYTES 64
/* cudaMalloc + zero fill of `bytes` of device memory whose IPC handle
 * (FRAG_IPC_HANDLE_BYTES) another process opens with frag_peer_open. */
FRAG_API int frag_peer_alloc(size_t bytes, void** dev_ptr, void* ipc_handle);
FRAG_API int frag_peer_open(const void* ipc_handle, void** dev_ptr);
FRAG_API int frag_peer_close(void* dev_ptr);
FRAG_API int frag_peer_free(void* dev_ptr);
/* The dweight exchange of a data-parallel RMSNorm backward over NVLink peer
 * memory (no reference counterpart: the reference is single-GPU; it replaces
 * the all-gather + fixed-order sum of the [W, N] per-rank vectors).
 *   dw_out[n] = sum over r = 0..world-1 of dw_local_r[n], added in rank order
 *   (bitwise the same on every rank and equal to frag_dw_reduce of the
 *   gathered [world, N] block).
 * slot_ptrs[p]: rank p's fp32 [world, N] buffer, flag_ptrs[p]: rank p's
 *   2 * world int32 flags, both from frag_peer_alloc (zero at creation) and
 *   mapped with frag_peer_open; state: this rank's own int32 call counter
 *   (zero at creation, advanced by every call on the device).
 *   One CTA per call, no per-call arguments (the launch can be captured in a
 *   CUDA graph); every wait bounded (~2 s, FRAG_DEVFLAG_WAIT_TIMEOUT, dw_out
 *   not written).  N % 4 == 0, dw_local 16-byte aligned. */
FRAG_API int frag_dw_exchange_peer(const float* dw_local, int64_t N, float* const* slot_ptrs,
                                   int32_t* const* flag_ptrs, int32_t* state, int rank, int world,
                                   float* dw_out, frag_stream_t stream);
FRAG_API int frag_embedding_fwd_vp_peer(const int64_t* ids, const void* table_shard, int64_t T,
                                        int64_t shard_rows, int64_t D, int64_t vocab_lo,
                                        int64_t vocab_total, void* const* out_ptrs,
                                        int32_t* const* flag_ptrs, int32_t* state, int rank,
                                        int world, int32_t* status, frag_stream_t stream);

/* ------------------------------------------------------------------------- *
 * Token-embedding gather fused with RMSNorm.
 *   e = table[ids[t]];  rstd[t] = 1/sqrt(mean(e^2) + eps);  y[t] = bf16((e*rstd)*w)
 * The gathered row is normalised in registers; it is also written to emb_out
 * (bit exact) when emb_out is not NULL.  Ids outside [0, V) give zero rows
 * and set FRAG_DEVFLAG_INDEX_OOB in *status.
 * Replaces aten.embedding -> aten._fused_rms_norm of v8/12545c1e9b06/problem.py:16-51
 * (drop-in v8/12545c1e9b06/optimized_kernel.py:66, whose Triton kernel
 * `_embedding_rmsnorm_kernel` is at :7).
 * ids: int64 [T]; table: bf16 [V, D]; w: bf16 [D]; y, emb_out: bf16 [T, D];
 * rstd: fp32 [T] or NULL.
 * ------------------------------------------------------------------------- */
FRAG_API int frag_embedding_rmsnorm_fwd(const int64_t* ids, const void* table, const void* w,
                                        void* y, float* rstd, void* emb_out, int64_t T,
                                        int64_t V, int64_t D, float eps, int32_t* status,
                                        frag_stream_t stream);

/* ------------------------------------------------------------------------- *
 * Token-embedding backward into an fp32 table gradient (deterministic).
 *   G[v,:] = sum over t in increasing order with ids[t]-vocab_lo == v and
 *            ids[t] != padding_idx of grad[t,:]      (fp32 accumulation)
 * Every row of G in [0, shard_rows) is written exactly once (zero rows
 * included), so G needs no prior memset.
 * Replaces aten.embedding_dense_backward -> _to_copy(fp32) of
 *   v7/a12a160cb11b/problem.py:16,19 (drop-in
 *   v7/a12a160cb11b/optimized_kernel.py:37 `kernel_function(add_223, ids)`),
 * whose Triton version accumulates with fp32 atomics (not reproducible).
 * ids: int64 [T]; grad: bf16 [T, D]; G: fp32 [shard_rows, D].
 * padding_idx < 0 disables padding.  workspace: *_workspace_bytes(T, shard_rows).
 * ------------------------------------------------------------------------- */
FRAG_API size_t frag_embedding_bwd_workspace_bytes(int64_t T, int64_t shard_rows);
FRAG_API int frag_embedding_bwd(const int64_t* ids, const void* grad, float* G,
                       int64_t T, int64_t shard_rows, int64_t D,
                       int64_t vocab_lo, int64_t vocab_total,
                       int64_t padding_idx, void* workspace,
                       size_t workspace_bytes, int32_t* status,
                       frag_stream_t stream);

/* ------------------------------------------------------------------------- *
 * RMSNorm backward fused into the token-embedding backward (deterministic).
 * For every token t (x = the embedding output that entered the norm):
 *   dy     = bf16(bf16(dy_a + dy_b) + dy_c)     (dy_b, dy_c optional, in order)
 *   rstd   = the saved rstd[t], or rsqrt(mean(x^2) + eps) when rstd is NULL
 *   y      = bf16((x * rstd) * w)               (written when y is not NULL)
 *   dx     = bf16(rstd * (dy*w - xhat * mean(dy*w*xhat))),  xhat = x * rstd
 *   d_emb  = bf16(dres + dx), or dx without dres (written when d_emb is not NULL)
 *   G[v,:] = sum of d_emb over the tokens of row v (as frag_embedding_bwd:
 *            shard-local rows, padding skipped, every row written once, fixed
 *            order), dw = sum over t of dy * xhat (fp32, fixed order).
 * d_emb never has to exist in memory.
 * Replaces _fused_rms_norm -> add -> add -> _fused_rms_norm_backward -> add ->
 * _to_copy -> embedding_dense_backward -> _to_copy of
 *   v6/0b493aad68f0/problem.py:21-70 (drop-in v6/0b493aad68f0/optimized_kernel.py:100),
 *   v5/118d525f44e0/problem.py (drop-in v5/118d525f44e0/optimized_kernel.py:72),
 *   v4/680e4c57cdc8/problem.py (drop-in v4/680e4c57cdc8/optimized_kernel.py:69),
 *   and, with the saved rstd, v8/f6251e84e3fa/problem.py:22-57.
 * x, dy_*, dres, y, d_emb: bf16 [T, D]; w: bf16 [D]; rstd: fp32 [T] or NULL;
 * ids: int64 [T]; G: fp32 [shard_rows, D]; dw: fp32 [D] and/or dw_bf16: bf16 [D].
 * workspace: frag_rmsnorm_embedding_bwd_workspace_bytes(T, D, shard_rows).
 * ------------------------------------------------------------------------- */
FRAG_API size_t frag_rmsnorm_embedding_bwd_workspace_bytes(int64_t T, int64_t D,
                                                           int64_t shard_rows);
FRAG_API int frag_rmsnorm_embedding_bwd(const void* x, const void* w, const float* rstd,
                                        void* y, const void* dy_a, const void* dy_b,
                                        const void* dy_c, const void* dres, void* d_emb,
                                        const int64_t* ids, float* G, float* dw,
                                        void* dw_bf16, int64_t T, int64_t D,
                                        int64_t shard_rows, int64_t vocab_lo,
                                        int64_t vocab_total, int64_t padding_idx, float eps,
                                        void* workspace, size_t workspace_bytes,
                                        int32_t* status, frag_stream_t stream);

/* ------------------------------------------------------------------------- *
 * Row-strided copy: dst + r*dst_stride <- src + r*src_stride, row_bytes bytes
 * per row, for r in [0, rows) (strides in bytes; rows must not overlap).
 * The FSDP unshard of a parameter out of the flat all-gather buffer:
 * replaces the clone of the [8, 65667072] split of wait_tensor_969 (row
 * stride 65667584) into the contiguous [128256, 4096] table in
 *   v8/8e33a91b7364/problem.py:44-51 (drop-in v8/8e33a91b7364/optimized_kernel.py:99),
 * and the [8, 512] weight-shard gathers (clone -> _unsafe_view [4096]) of
 *   v8/8e33a91b7364/problem.py:23-32 and v7/215dd2e6a519/problem.py:16-22.
 * 16-byte aligned pointers, strides and row_bytes take the vector kernel.
 * ------------------------------------------------------------------------- */
FRAG_API int frag_copy_rows(const void* src, int64_t src_stride, void* dst, int64_t dst_stride,
                            int64_t rows, int64_t row_bytes, frag_stream_t stream);

/* ------------------------------------------------------------------------- *
 * Grouped row-strided copy: up to FRAG_COPY_MAX_SEGMENTS frag_copy_rows
 * copies in ONE launch, CTAs shared out in proportion to each segment's
 * bytes.  The unshard of a whole FSDP parameter group out of one all-gather
 * buffer: replaces the nine split_with_sizes -> clone chains of
 *   v8/7815074de963/problem.py:23-103 and v8/94985bdb7630/problem.py:23-106
 * (splits [512, 2097152, 524288, 524288, 2097152, 512, 7340032 x3] of the
 * [8, 27264000] view), and the weight + table pair of
 *   v5/013a3088b488/problem.py:23-55 and v8/8e33a91b7364/problem.py:23-51.
 * Segments with rows == 0 or row_bytes == 0 are skipped; no destination may
 * overlap a source or another destination.  When every segment is 16-byte
 * aligned (pointers, strides, row_bytes) the group is one launch; otherwise
 * each segment is copied by frag_copy_rows in turn.
 * ------------------------------------------------------------------------- */
#define FRAG_COPY_MAX_SEGMENTS 16

typedef struct frag_copy_segment {
  const void* src;
  void* dst;
  int64_t src_stride; /* bytes between source rows */
  int64_t dst_stride; /* bytes between destination rows */
  int64_t rows;
  int64_t row_bytes;
} frag_copy_segment;

FRAG_API int frag_copy_rows_grouped(const frag_copy_segment* segs, int32_t n, frag_stream_t stream);

/* ------------------------------------------------------------------------- *
 * Element type conversion of row-strided rows: dst row r (and dst2 row r when
 * dst2 is non-NULL) <- src row r converted from src_dtype to dst_dtype
 * (FRAG_DT_BF16 / FRAG_DT_F32), `cols` elements per row, rows src_stride /
 * dst_stride elements (of each side's type) apart; fp32 -> bf16 rounds to
 * nearest even, bf16 -> fp32 is exact.  No destination may overlap the
 * source or the other destination.  Replaces the aten._to_copy casts around
 * the complex RoPE multiply of the v1-v3 snapshots:
 *   v2/dcf660c50ef3/problem.py:14-37 and v2/5d51b24b8d83/problem.py:14-37
 *     (q / k projections widened to fp32, twice: dst and dst2),
 *   v2/b3f1b1135abc/problem.py:16-43 (the SDPA-layout q / k gradients),
 *   v2/d800447a68f6/problem.py:14-26, v2/3e3eb10963d7/problem.py:14-26,
 *   v2/db48e1361360/problem.py:14-22, v2/b508c9141fed/problem.py:14-22
 *     (view_as_real results rounded back to bf16),
 * and their v1 / v3 snapshots.
 * ------------------------------------------------------------------------- */
FRAG_API int frag_convert_rows(const void* src, int32_t src_dtype, int64_t src_stride, void* dst,
                               void* dst2, int32_t dst_dtype, int64_t dst_stride, int64_t rows,
                               int64_t cols, frag_stream_t stream);

/* ------------------------------------------------------------------------- *
 * Rotary position embedding on up to two tensors (q and k) in one launch.
 * Tensor i (i = 0, 1) is bf16 [B, S, H_i, D] addressed by element strides
 * (stride_b, stride_s, stride_h; the last dimension is contiguous), and is
 * written to out_i with its own strides (bf16, or fp32 when out_dtype says
 * so).  A bf16 in and out may alias exactly.
 * Angle for pair j (0 <= j < D/2) at position p:
 *   freqs == NULL : theta_j = p * inv_freq[j], inv_freq[j] = theta^(-2j/D)
 *                   (fp32, cos/sin evaluated in registers; nothing is read
 *                   from HBM besides x and the positions)
 *   freqs != NULL : (cos, sin) := (re, im) of freqs[p, j], a complex64 table
 *                   of freqs_rows rows of stride freqs_stride (in complex
 *                   elements) — the reference's freqs_cis input (not
 *                   necessarily unit modulus).  A position outside
 *                   [0, freqs_rows) is not read: it sets
 *                   FRAG_DEVFLAG_INDEX_OOB in the library's error word
 *                   (frag_device_errors) and its token is copied unrotated.
 * layout NEOX rotates (x_j, x_{j+D/2}); INTERLEAVED rotates (x_2j, x_2j+1).
 * inverse != 0 rotates by the conjugate (the backward of RoPE).
 * Positions p = pos[b*pos_stride_b + s*pos_stride_s] (int32 or int64), or s.
 * Replaces the complex-mul RoPE of v8/c8c60d8f7015/problem.py:18-70 (drop-in
 * v8/c8c60d8f7015/optimized_kernel.py:48), v8/97032595d968 (:44),
 * v8/e29b92927600 (:54), v8/493cad38cac9 (:48), v7/0f38bc55457c (fp32 q,
 * drop-in v7/0f38bc55457c/optimized_kernel.py:84), and the backward fragments
 * v7/bfe872e373e4 (:54), v7/5c65f62b0422 (:45), v6/03d64c25b654 (:51).
 * ------------------------------------------------------------------------- */
typedef struct frag_rope_tensor {
  const void* x;
  void* out;
  int64_t H;
  int64_t x_stride_b, x_stride_s, x_stride_h;
  int64_t out_stride_b, out_stride_s, out_stride_h;
  /* FRAG_ROPE_OUT_BF16 (0): out is bf16 (rounded once); FRAG_ROPE_OUT_F32
   * (1): out is fp32, not rounded (v7/0f38bc55457c/problem.py:10-40 returns
   * q that way); out strides are in elements of out's type. */
  int32_t out_dtype;
  /* FRAG_ROPE_IN_BF16 (0): x is bf16; FRAG_ROPE_IN_F32 (1): x is fp32, a
   * complex64 tensor viewed as (re, im) pairs -- the v1/v2 snapshots' complex
   * multiply (v2/075cb40f3d5d/problem.py:15-27, v2/9cd8f72e74ce/problem.py:13-16)
   * -- which needs FRAG_ROPE_INTERLEAVED, out_dtype FRAG_ROPE_OUT_F32 and the
   * same in_dtype for every tensor of the call; x strides in elements of x. */
  int32_t in_dtype;
} frag_rope_tensor;

FRAG_API int frag_rope(const frag_rope_tensor* tensors, int num_tensors, int64_t B,
              int64_t S, int64_t D, const void* pos, int pos_dtype,
              int64_t pos_stride_b, int64_t pos_stride_s, const float* freqs,
              int64_t freqs_stride, int64_t freqs_rows, float theta, int layout,
              int inverse, frag_stream_t stream);

/* Self-test of the bounded waits: one thread waits limit_cycles
 * (0 < limit_cycles <= 4e9) on an mbarrier that nothing arrives on, with the
 * same wait every TMA kernel here uses.  The wait gives up and sets
 * FRAG_DEVFLAG_WAIT_TIMEOUT in the error word (frag_device_errors); the
 * context stays usable.  No counterpart in the reference, which has no
 * device-side waits. */
FRAG_API int frag_selftest_bounded_wait(int64_t limit_cycles, frag_stream_t stream);

/* Device properties the host layer uses to size launches and workspaces. */
FRAG_API int frag_device_sm_count(void);

/* Error bits (FRAG_DEVFLAG_*) that kernels on the current device recorded in
 * the library's own error word (a static device variable), e.g. a bounded
 * wait that expired.  Synchronises the device to read it; clears it if
 * `clear` is non-zero.  Returns the bits (>= 0) or -FRAG_ERR_CUDA. */
FRAG_API int frag_device_errors(int clear);

#ifdef __cplusplus
}
#endif

#endif /* FRAG_H_ */
