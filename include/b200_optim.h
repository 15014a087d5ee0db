/*
 * b200_optim.h -- C ABI of the B200 fused mixed-precision optimizer step.
 *
 * The reference (TuraLucrs/minigpt-train-infra) runs this step through PyTorch
 * (train.py:485-491):
 *
 *     scaler.unscale_(optimizer)          -> torch._amp_foreach_non_finite_check_and_unscale_
 *     clip_grad_norm_(params, max_norm)   -> torch._foreach_norm, vector_norm, _foreach_mul_
 *     scaler.step(optimizer)              -> torch._fused_adamw_ (CUDA) / _single_tensor_adam
 *     scaler.update()                     -> torch._amp_update_scale_
 *
 * Each entry point below replaces one of those ATen operator calls; the comment of each names the
 * torch Python line that issues the call it replaces (paths relative to the installed torch
 * package).  The Python layer of this package (optim.py, amp.py, clip.py, zero1.py) binds them
 * through ctypes; a C, C++ or other FFI host binds the same symbols directly.
 *
 * Conventions
 *  - Every pointer is a device pointer unless its comment says "host".
 *  - Every launching entry point is asynchronous on `stream` (a cudaStream_t passed as void*),
 *    performs no host synchronisation and allocates no memory.  Buffers are owned by the caller.
 *  - Return value: B2O_OK (0) or a negative b2o_status.  Nothing aborts or traps.
 *  - Calls that share a workspace must be ordered on one stream (not re-entrant per workspace).
 */
#ifndef B200_OPTIM_H_
#define B200_OPTIM_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define B2O_ABI_VERSION 1
#define B2O_MAX_GROUPS 16
#define B2O_VEC 8 /* elements per vector step: one 16-byte bf16 load, two 16-byte fp32 loads */

typedef enum {
  B2O_OK = 0,
  B2O_ERR_ARG = -1,       /* null pointer, negative size, unknown dtype, too many groups   */
  B2O_ERR_CAPACITY = -2,  /* an output array is too small for the plan                      */
  B2O_ERR_LAUNCH = -3,    /* the kernel launch failed (cudaGetLastError)                    */
  B2O_ERR_CUDA = -4,      /* another CUDA runtime call failed                               */
  B2O_ERR_TABLE = -5,     /* a tensor table entry is inconsistent (overlap, bad slot/group) */
  B2O_ERR_TOO_LARGE = -6  /* the plan exceeds the fixed scratch of b2o_grad_stats_noalloc    */
} b2o_status;

typedef enum { B2O_BF16 = 0, B2O_F32 = 1 } b2o_dtype;

/* One tensor (or, under ZeRO-1, the part of one tensor inside this rank's shard). */
typedef struct b2o_tensor {
  const void* grad;     /* gradient, dtype = grad_dtype of the call                          */
  void* param;          /* bf16 model parameter to refresh from the master; NULL when the
                           parameters are fp32 (then `master` is the parameter itself)      */
  float* master;        /* fp32 master weights                                               */
  float* exp_avg;       /* fp32 first moment                                                 */
  float* exp_avg_sq;    /* fp32 second moment                                                */
  int64_t numel;        /* elements in this slice (0 allowed)                                */
  int32_t group;        /* index into the b2o_group array of the call                        */
  int32_t slot;         /* per-parameter index: step counter and norm accumulator            */
  int32_t chunk_begin;  /* written by b2o_plan_chunks                                        */
  int32_t chunk_count;  /* written by b2o_plan_chunks                                        */
  int32_t flags;        /* written by b2o_plan_chunks: B2O_FLAG_VECTOR when every pointer is
                           16-byte aligned so the 128-bit path may be used                  */
  int32_t reserved;
} b2o_tensor;

#define B2O_FLAG_VECTOR 1

/* A contiguous element range [begin, end) of one tensor, processed by one CTA iteration. */
typedef struct b2o_chunk {
  int32_t tensor;
  int32_t reserved;
  int64_t begin;
  int64_t end;
} b2o_chunk;

/* Hyper-parameters of one param_group, as the Python floats torch's AdamW holds. */
typedef struct b2o_group {
  double lr;
  double beta1;
  double beta2;
  double eps;
  double weight_decay;
} b2o_group;

/* ---------------------------------------------------------------------------------------- */
/* Library identity                                                                          */
/* ---------------------------------------------------------------------------------------- */

/* ABI version this library was built with (B2O_ABI_VERSION). */
int b2o_abi_version(void);

/* Human-readable text of a b2o_status value (static storage). */
const char* b2o_status_string(int status);

/* ---------------------------------------------------------------------------------------- */
/* Multi-tensor-apply planning (host only)                                                   */
/* Replaces the tensor-list chunking of ATen's multi_tensor_apply that                        */
/* torch._amp_foreach_non_finite_check_and_unscale_ / torch._fused_adamw_ perform per call    */
/* (issued from torch/amp/grad_scaler.py:294 and torch/optim/adam.py:880).                    */
/* ---------------------------------------------------------------------------------------- */

/* Split every tensor of `tensors` (host array, n_tensors entries) into chunks of `chunk_elems`
 * elements (a positive multiple of B2O_VEC), write them to `chunks` (host array, capacity
 * `chunk_cap`) and the count to *n_chunks (host).  Fills chunk_begin, chunk_count and flags of
 * each tensor entry.  Validates the table: non-null pointers for non-empty tensors, group in
 * [0, n_groups), slot in [0, n_slots), no slot used twice.  Pass chunks == NULL to only count. */
int b2o_plan_chunks(b2o_tensor* tensors, int32_t n_tensors, int32_t n_groups, int32_t n_slots,
                    int64_t chunk_elems, int32_t grad_dtype, b2o_chunk* chunks,
                    int64_t chunk_cap, int64_t* n_chunks);

/* Bytes of device workspace a plan needs (the statistics and update passes of one plan share
 * it): completion and chunk-claim counters, one partial sum per chunk and the per-slot exchange
 * vector. */
size_t b2o_workspace_bytes(int64_t n_chunks, int32_t n_slots);

/* Zero a freshly allocated workspace of `bytes` bytes (cudaMemsetAsync on `stream`).  The
 * passes return every counter to zero when they finish, so this is needed once. */
int b2o_workspace_init(void* workspace, size_t bytes, void* stream);

/* ---------------------------------------------------------------------------------------- */
/* Pass 1: unscale + non-finite check + L2 partial sums                                      */
/* Replaces torch._amp_foreach_non_finite_check_and_unscale_ (torch/amp/grad_scaler.py:294)   */
/* and torch._foreach_norm + linalg.vector_norm (torch/nn/utils/clip_grad.py:96,106).         */
/* Gradients are read, never written: the unscale and clip factors are applied by pass 2.     */
/* ---------------------------------------------------------------------------------------- */

/* Reads every gradient once.  x = float(g) * inv_scale (fp32) with inv_scale =
 * fp32(1 / double(*loss_scale)) -- GradScaler's `_scale.double().reciprocal().float()`
 * (grad_scaler.py:351) -- or 1 when loss_scale is NULL; accumulates x*x per chunk and
 * flags any non-finite g (tested before scaling, as torch does).  The last CTA to finish folds
 * the chunk partials, in chunk order, into the per-slot exchange vector: exch[slot] (double) for
 * every slot of the table and exch[n_slots] += 1.0 if a non-finite value was seen.
 * `flags`:
 *   B2O_STATS_CLEAR     zero exch[0..n_slots] first (the first table of a step);
 *   B2O_STATS_FINALIZE  also write *found_inf_out (1.0f or 0.0f) and *norm_out (total norm,
 *                       fp32) from exch, exactly as b2o_finalize_norm would for one rank.
 * `exch` (n_slots+1 doubles) may be NULL to use the
 * exchange area inside `workspace`. */
#define B2O_STATS_FINALIZE 1
#define B2O_STATS_CLEAR 2
int b2o_grad_stats(const b2o_tensor* tensors, int32_t n_tensors, const b2o_chunk* chunks,
                   int64_t n_chunks, int32_t n_slots, int32_t grad_dtype,
                   const float* loss_scale, void* workspace, double* exch, int32_t flags,
                   float* found_inf_out, float* norm_out, void* stream);

/* Allocation-free variant of b2o_grad_stats, for callers that cannot allocate device memory:
 * an FFI host that only holds pointers handed to it by another runtime and has no allocator to
 * give this library, or a training process already at its memory ceiling where one more
 * allocation would fail.  No counterpart in the reference (torch allocates its own scratch).
 *
 * Same pass and same results as b2o_grad_stats called with
 * B2O_STATS_CLEAR | B2O_STATS_FINALIZE, but the scratch (completion counters, one double per
 * chunk, n_slots + 1 per-slot sums) lives in one fixed array inside this library instead of a
 * caller workspace.  That array holds B2O_NOALLOC_MAX_CHUNKS chunks and B2O_NOALLOC_MAX_SLOTS
 * slots (about 288 KiB); every GPU that loads the library keeps it until the process exits.
 * Larger plans are rejected with B2O_ERR_TOO_LARGE -- use a larger chunk_elems or
 * b2o_grad_stats.  The call allocates and frees nothing.
 *
 * The array exists once per CUDA context that runs this library's code: for callers of the
 * runtime API that is the device's primary context; a host that made a driver context of its own
 * current gets that context's copy.  The call uses the array of the context current on the
 * calling thread, whose address it looks up (cudaGetSymbolAddress) on the first call in that
 * context and caches under the context's id; make that first call before any stream capture,
 * and pass a `stream` of the same context.  Each call
 * clears the counters on `stream` before its kernel.  All calls share the one array and it keeps
 * the last call's contents, so calls whose kernels overlap on the GPU (different streams without
 * ordering, or different threads) race and give wrong results: order them on one stream. */
#define B2O_NOALLOC_MAX_CHUNKS 32768
#define B2O_NOALLOC_MAX_SLOTS 4096
int b2o_grad_stats_noalloc(const b2o_tensor* tensors, int32_t n_tensors, const b2o_chunk* chunks,
                           int64_t n_chunks, int32_t n_slots, int32_t grad_dtype,
                           const float* loss_scale, float* found_inf_out, float* norm_out,
                           void* stream);

/* Fold `n_ranks` exchange vectors (laid out rank-major, n_slots+1 doubles each) in rank order:
 * per-slot norm = fp32(sqrt(sum)), total = fp32(sqrt(sum of squared per-slot norms)), and
 * found_inf = 1.0f if any rank saw a non-finite gradient.  One CTA; deterministic. */
int b2o_finalize_norm(const double* exch_all, int32_t n_ranks, int32_t n_slots,
                      float* found_inf_out, float* norm_out, void* stream);

/* ---------------------------------------------------------------------------------------- */
/* Pass 2: fused AdamW + bf16 parameter refresh                                              */
/* Replaces torch._fused_adamw_ (torch/optim/adam.py:880) and, on the CPU path the reference  */
/* runs, _single_tensor_adam (torch/optim/adam.py:347-552) plus clip_grad.py:174's            */
/* torch._foreach_mul_ of the clip coefficient.                                               */
/* ---------------------------------------------------------------------------------------- */

/* For every element: g = (float(grad) * inv_scale) * clip_coef (inv_scale formed from
 * *loss_scale exactly as in b2o_grad_stats), then the decoupled-weight-decay
 * AdamW update of master/exp_avg/exp_avg_sq in the rounding order of torch's single-tensor
 * AdamW, then param = bf16(master) when `param_dtype` is B2O_BF16.
 *   steps[slot]     fp32 step counters (torch state["step"]); the update uses steps+1 and the
 *                   last CTA stores steps+1 for every slot of the table.
 *   found_inf       NULL or a device flag; non-zero skips the whole update, counters included.
 *   loss_scale      NULL (factor 1) or the loss scale the gradients carry; the same pointer
 *                   pass 1 read, unchanged in between.
 *   norm, max_norm  when norm != NULL: clip_coef = min(max_norm / (norm + 1e-6), 1) rounded as
 *                   torch/nn/utils/clip_grad.py:165-169 does; NULL means no clipping.
 *   clip_coef_out   NULL or where to store the coefficient used (for reporting).
 * `groups` is a host array of n_groups (<= B2O_MAX_GROUPS) entries, passed by value. */
int b2o_adamw_step(const b2o_tensor* tensors, int32_t n_tensors, const b2o_chunk* chunks,
                   int64_t n_chunks, const b2o_group* groups, int32_t n_groups,
                   int32_t grad_dtype, int32_t param_dtype, float* steps,
                   const float* found_inf, const float* loss_scale, const float* norm,
                   float max_norm, float* clip_coef_out, void* workspace, void* stream);

/* b2o_adamw_step with the group hyper-parameters read from device memory (`dev_groups`,
 * n_groups entries) when the kernel runs, instead of passed by value at launch: a launch
 * recorded in a CUDA graph then follows learning-rate schedules by rewriting `dev_groups`
 * between replays.  No counterpart in the reference (torch's AdamW(capturable=True) holds lr in
 * a device tensor for the same reason). */
int b2o_adamw_step_dev(const b2o_tensor* tensors, int32_t n_tensors, const b2o_chunk* chunks,
                       int64_t n_chunks, const b2o_group* dev_groups, int32_t n_groups,
                       int32_t grad_dtype, int32_t param_dtype, float* steps,
                       const float* found_inf, const float* loss_scale, const float* norm,
                       float max_norm, void* workspace, void* stream);

/* ---------------------------------------------------------------------------------------- */
/* Peer memory and fused collectives (ZeRO-1 over the GPUs of one node)                        */
/* No counterpart in the reference, which has no data-parallel training path; they replace the */
/* NCCL reduce-scatter and all-gather a ZeRO-1 trainer would issue around the step.            */
/* Peer buffers use legacy CUDA IPC (cudaMalloc + cudaIpcGetMemHandle / OpenMemHandle): plain  */
/* loads and stores over NVLink, no multicast objects.                                        */
/* ---------------------------------------------------------------------------------------- */

#define B2O_IPC_HANDLE_BYTES 64
#define B2O_MAX_PEERS 8

/* Allocate `bytes` of device memory on the current device that other processes may map. */
int b2o_peer_alloc(size_t bytes, void** ptr_out);
/* Free memory from b2o_peer_alloc (after every peer closed its mapping). */
int b2o_peer_free(void* ptr);
/* Write the 64-byte IPC handle of a b2o_peer_alloc allocation to `handle_out` (host). */
int b2o_peer_export(void* ptr, void* handle_out);
/* Map another process's allocation from its 64-byte handle (host); *ptr_out is its base. */
int b2o_peer_import(const void* handle, void** ptr_out);
/* Unmap an imported allocation. */
int b2o_peer_close(void* ptr);

/* Reduce-scatter of bf16 gradients fused with the statistics pass.  `peer_grads` (host array
 * of n_ranks device pointers, index = rank) holds the base address of every rank's flat
 * gradient buffer as mapped in this process; `my_grad_base` is this rank's own base.  For every
 * element of the table (this rank's shard): g = bf16(scale_factor * sum over ranks in rank
 * order of float(grad_r)), accumulated in fp32 and written in place into this rank's buffer;
 * then the same per-chunk sums of squares and non-finite flag as b2o_grad_stats (flags
 * B2O_STATS_CLEAR only; finalize with b2o_finalize_norm after exchanging `exch`).  Every rank
 * must have finished writing its gradients before any rank starts, and no rank may overwrite its
 * gradients before every rank has finished (order both with a collective on `stream`). */
int b2o_reduce_scatter_stats(const void* const* peer_grads, int32_t n_ranks,
                             const void* my_grad_base, float scale_factor,
                             const b2o_tensor* tensors, int32_t n_tensors,
                             const b2o_chunk* chunks, int64_t n_chunks, int32_t n_slots,
                             const float* loss_scale, void* workspace, double* exch,
                             void* stream);

/* b2o_adamw_step for bf16 parameters that also stores every updated bf16 value into the
 * parameter buffer of each other rank (`peer_params`, host array of n_ranks bases as mapped in
 * this process, index = rank; `my_param_base` is this rank's own base): the ZeRO-1 all-gather of
 * the updated shards fused into the update.  Order it after every rank stopped reading its
 * parameters and before any rank reads them again (a collective on `stream` on both sides). */
int b2o_adamw_step_bcast(const b2o_tensor* tensors, int32_t n_tensors, const b2o_chunk* chunks,
                         int64_t n_chunks, const b2o_group* groups, int32_t n_groups,
                         int32_t grad_dtype, float* steps, const float* found_inf,
                         const float* loss_scale, const float* norm, float max_norm,
                         void* const* peer_params, int32_t n_ranks, int32_t my_rank,
                         const void* my_param_base, void* workspace, void* stream);

/* ---------------------------------------------------------------------------------------- */
/* Loss-scale update                                                                         */
/* Replaces torch._amp_update_scale_ (torch/amp/grad_scaler.py:549).                          */
/* ---------------------------------------------------------------------------------------- */

/* If *found_inf != 0: scale *= backoff, tracker = 0.  Else tracker += 1 and, when it reaches
 * growth_interval, scale *= growth (kept only if finite) and tracker = 0.  One thread. */
int b2o_scaler_update(float* scale, int32_t* growth_tracker, const float* found_inf,
                      double growth_factor, double backoff_factor, int32_t growth_interval,
                      void* stream);

#ifdef __cplusplus
}
#endif

#endif /* B200_OPTIM_H_ */
