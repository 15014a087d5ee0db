// Pass 1 of the optimizer step: unscale + non-finite flag + L2 partial sums (sm_100a).
//
// Replaces, for the reference's train.py:485-486, the two gradient passes torch makes:
//   torch._amp_foreach_non_finite_check_and_unscale_   (torch/amp/grad_scaler.py:294)
//   torch._foreach_norm + linalg.vector_norm           (torch/nn/utils/clip_grad.py:96,106)
// Gradients are read once (2 bytes per bf16 element) and never written; the unscale factor and
// the clip coefficient are folded into pass 2 (b2o_adamw.cu).
//
// Reduction order (deterministic for a given plan and grid):
//   element -> fp32 sum of squares over one 8-element vector (fma chain)
//   vector  -> fp64 per-thread sum -> fixed-order CTA sum = one fp64 partial per chunk
//   chunk   -> the last CTA to finish folds each tensor's chunk partials in chunk order,
//              staged in shared memory 4096 at a time: a tensor's piece of at most 128
//              partials by one thread (four interleaved accumulators, then (a0+a1)+(a2+a3)),
//              a longer piece by one warp (fixed lane-strided walk + xor-shuffle tree), the
//              pieces of a tensor that spans windows added in window order; the result goes to
//              exch[slot]
//   slot    -> per-tensor norm fp32(sqrt(sum)), total fp32(sqrt(sum of squared norms)); the
//              same two-level structure as clip_grad.py:_get_total_norm.
#include <cuda.h>
#include <cuda_runtime.h>

#include <climits>
#include <mutex>

#include "b2o_device.cuh"
#include "b2o_host.h"

namespace b2o {

// Folds n_ranks exchange vectors into found_inf / norm.  Executed by one whole CTA.
__device__ void finalize_norm_cta(const double* exch_all, int n_ranks, int n_slots,
                                  float* found_inf_out, float* norm_out, double* scratch) {
  const int stride = n_slots + 1;
  // Thread 0 reads the non-finite counts first, so their latency overlaps the slot loop.
  double bad = 0.0;
  if (threadIdx.x == 0)
    for (int r = 0; r < n_ranks; ++r) bad += __ldcg(exch_all + (int64_t)r * stride + n_slots);
  double local = 0.0;
  for (int s = threadIdx.x; s < n_slots; s += blockDim.x) {
    double sum = 0.0;
    for (int r = 0; r < n_ranks; ++r) sum += __ldcg(exch_all + (int64_t)r * stride + s);
    const float tn = (float)sqrt(sum);  // per-tensor norm rounded to fp32, as torch returns it
    const double t = (double)tn;
    local += t * t;
  }
  const double total_sq = block_sum(local, scratch);
  if (threadIdx.x == 0) {
    if (found_inf_out) *found_inf_out = bad != 0.0 ? 1.0f : 0.0f;
    if (norm_out) *norm_out = (float)sqrt(total_sq);
  }
}

// The final fold stages the chunk partials in shared memory, kFoldWin at a time: each thread
// keeps kFoldLoads loads in flight, and the loads of the next window are issued before the
// current window is folded, so the fold costs about one L2 round trip per window instead of
// one per tensor.  Within a window the tensors are folded in parallel: a piece of at most
// kThreadFoldMax partials by the thread holding its tensor, a longer one by a warp.
constexpr int kFoldWin = 4096;
constexpr int kFoldLoads = kFoldWin / kThreads;
constexpr int kThreadFoldMax = 128;
static_assert(kFoldWin % kThreads == 0, "whole loads per thread");
static_assert(kWarps == 8, "a long piece's warp is picked with a mask of every 8th bit");

// End of a statistics pass, executed by every thread of every CTA after its chunk loop: record
// the CTA's non-finite flag, take a completion ticket, and let the CTA holding the last ticket
// fold the chunk partials (per tensor, in chunk order) into exch, then optionally finish the norm.
__device__ __forceinline__ void stats_epilogue(bool bad, const b2o_tensor* __restrict__ tensors,
                                               int n_tensors, int64_t n_chunks, int n_slots,
                                               Workspace ws, double* exch, int flags,
                                               float* found_inf_out, float* norm_out,
                                               double* scratch, int* is_last_p) {
  int& is_last = *is_last_p;
  if (__syncthreads_or(bad) && threadIdx.x == 0) atomicOr(ws.stats_nonfinite, 1u);

  // Completion ticket: the CTA that takes the last ticket sees every partial.
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) is_last = atomicAdd(ws.stats_done, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!is_last) return;
  __threadfence();

  __shared__ double s_part[kFoldWin];     // the window's chunk partials
  __shared__ double s_acc[kThreads];      // running sum of a tensor whose chunks span windows
  __shared__ int s_begin[kThreads], s_end[kThreads], s_slot[kThreads];  // one block of the table
  __shared__ unsigned int s_mask[kWarps];  // tensors of the block with a long piece in the window
  __shared__ int s_lo, s_hi;

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // Every CTA has set its non-finite bit and taken its ticket: the flag and both counters are
  // final, so they are taken and reset now and the exchange's latency overlaps the fold.
  unsigned int nonfinite = 0;
  if (threadIdx.x == 0) {
    nonfinite = atomicExch(ws.stats_nonfinite, 0u);
    *ws.stats_tile = 0u;
    *ws.stats_done = 0u;
  }
  if (flags & B2O_STATS_CLEAR)
    for (int s = threadIdx.x; s <= n_slots; s += kThreads) exch[s] = 0.0;
  const int n_part = int(n_chunks);  // the planner keeps chunk counts below 2**31

  // The table is taken in blocks of kThreads tensors, thread t holding tensor base + t.  The
  // partials of a block's tensors are staged window by window over [lo, hi), the span of their
  // chunk ranges.  A tensor's piece of a window is summed in chunk order, by one of two fixed
  // rules chosen by the piece's length alone:
  //   at most kThreadFoldMax partials: by the tensor's thread, partial i of the piece into
  //     accumulator i % 4, then (a0 + a1) + (a2 + a3);
  //   longer: by warp t % kWarps, lane l summing partials l, l + 32, ... in that order, then the
  //     warp's xor tree.  A warp takes its long pieces as soon as its own short ones are done.
  // A tensor whose chunks span windows adds its windows' sums in window order.  The result
  // depends only on the plan, so it is deterministic.
  double a[kFoldLoads];
  // The first window of the first block is almost always [0, ...): its loads are issued before
  // the table is read, and issued again below only if the table says otherwise.
  int staged_from = 0;
#pragma unroll
  for (int u = 0; u < kFoldLoads; ++u) {
    const int i = threadIdx.x + u * kThreads;
    a[u] = i < n_part ? __ldcg(ws.chunk_sums + i) : 0.0;
  }
  for (int base = 0; base < n_tensors; base += kThreads) {
    const int nt = min(kThreads, n_tensors - base);
    if (threadIdx.x == 0) {
      s_lo = INT_MAX;
      s_hi = 0;
    }
    __syncthreads();  // also orders the CLEAR stores and the previous block before this one
    int tb = 0, te = 0, slot = 0;
    if (threadIdx.x < nt) {
      const b2o_tensor& t = tensors[base + threadIdx.x];
      tb = max(t.chunk_begin, 0);
      te = min(t.chunk_begin + t.chunk_count, n_part);
      slot = t.slot;
      s_begin[threadIdx.x] = tb;
      s_end[threadIdx.x] = te;
      s_slot[threadIdx.x] = slot;
      if (te <= tb) {
        exch[slot] = 0.0;  // a tensor with no chunks
      } else {
        atomicMin(&s_lo, tb);
        atomicMax(&s_hi, te);
      }
    }
    __syncthreads();
    const int lo = s_lo, hi = s_hi;  // lo > hi when no tensor of the block has a chunk
    if (lo < hi && lo != staged_from) {
#pragma unroll
      for (int u = 0; u < kFoldLoads; ++u) {
        const int64_t i = int64_t(lo) + threadIdx.x + u * kThreads;
        a[u] = i < hi ? __ldcg(ws.chunk_sums + i) : 0.0;
      }
    }
    staged_from = -1;  // later blocks always load their first window here
    for (int w0 = lo; w0 < hi; w0 += kFoldWin) {
      const int w1 = min(w0 + kFoldWin, hi);
      const int pb = max(tb, w0), pe = min(te, w1);  // this thread's tensor's piece
      const bool has = tb < te && pb < pe;
      const bool is_long = has && pe - pb > kThreadFoldMax;
      const unsigned int m = __ballot_sync(0xffffffffu, is_long);
      if (lane == 0) s_mask[warp] = m;
#pragma unroll
      for (int u = 0; u < kFoldLoads; ++u) {
        const int i = threadIdx.x + u * kThreads;
        if (w0 + i < w1) s_part[i] = a[u];
      }
      __syncthreads();
      if (w1 < hi) {
#pragma unroll
        for (int u = 0; u < kFoldLoads; ++u) {
          const int64_t i = int64_t(w1) + threadIdx.x + u * kThreads;
          a[u] = i < hi ? __ldcg(ws.chunk_sums + i) : 0.0;
        }
      }
      if (has && !is_long) {
        double a0 = 0.0, a1 = 0.0, a2 = 0.0, a3 = 0.0;
        int j = pb - w0;
        const int je = pe - w0;
#pragma unroll 2
        for (; j + 3 < je; j += 4) {
          a0 += s_part[j];
          a1 += s_part[j + 1];
          a2 += s_part[j + 2];
          a3 += s_part[j + 3];
        }
        if (j < je) a0 += s_part[j];
        if (j + 1 < je) a1 += s_part[j + 1];
        if (j + 2 < je) a2 += s_part[j + 2];
        const double sum = (a0 + a1) + (a2 + a3);
        const double acc = pb > tb ? s_acc[threadIdx.x] + sum : sum;
        if (pe < te)
          s_acc[threadIdx.x] = acc;
        else
          exch[slot] = acc;
      }
      for (int q = 0; q < kWarps; ++q) {
        unsigned int mm = s_mask[q] & (0x01010101u << warp);  // tensors q*32 + warp + 8k
        while (mm) {
          const int p = q * 32 + __ffs(mm) - 1;
          mm &= mm - 1;
          const int b = max(s_begin[p], w0), e = min(s_end[p], w1);
          // four loads in flight before the additions, which stay in partial order
          double sum = 0.0;
          int j = b - w0 + lane;
          const int je = e - w0;
          for (; j + 3 * 32 < je; j += 4 * 32) {
            const double x0 = s_part[j], x1 = s_part[j + 32];
            const double x2 = s_part[j + 64], x3 = s_part[j + 96];
            sum += x0;
            sum += x1;
            sum += x2;
            sum += x3;
          }
          for (; j < je; j += 32) sum += s_part[j];
          sum = warp_sum(sum);
          if (lane == 0) {
            const double acc = b > s_begin[p] ? s_acc[p] + sum : sum;
            if (e < s_end[p])
              s_acc[p] = acc;
            else
              exch[s_slot[p]] = acc;
          }
        }
      }
      __syncthreads();  // s_part, s_mask and s_acc are written again in the next window
    }
  }
  __syncthreads();  // after the CLEAR stores even when the table is empty
  if (threadIdx.x == 0 && nonfinite) exch[n_slots] += 1.0;
  __syncthreads();  // the CTA's exch stores are visible to the CTA's finalize loads
  if (flags & B2O_STATS_FINALIZE)
    finalize_norm_cta(exch, 1, n_slots, found_inf_out, norm_out, scratch);
}

// Vectors (8 elements) each thread keeps in flight per loop iteration: 8 for bf16 gradients
// (128 bytes), 4 for fp32 (also 128 bytes, each vector being two 16-byte loads).  Measured on
// B200 with the claim-after-read schedule: 8 bf16 vectors beat 4 by 0-12% from MiniGPT to
// Qwen3-8B (2364 -> 2324 us for the 8B pass).
template <class G> struct StatsUnroll { static constexpr int value = 8; };
template <> struct StatsUnroll<GradF32> { static constexpr int value = 4; };
// Chunk scheduling: 0 static round-robin over CTAs, 1 dynamic in-order from a counter.
#ifndef B2O_STATS_SCHED
#define B2O_STATS_SCHED 1
#endif

template <class G, int U = StatsUnroll<G>::value>
__global__ void __launch_bounds__(kThreads, 4)
grad_stats_kernel(const b2o_tensor* __restrict__ tensors, int n_tensors,
                  const b2o_chunk* __restrict__ chunks, int64_t n_chunks, int n_slots,
                  const float* __restrict__ loss_scale, Workspace ws, double* exch,
                  int flags, float* found_inf_out, float* norm_out) {
  __shared__ double scratch[kWarps];
  __shared__ int is_last;
  const float inv = inv_scale_of(loss_scale);
  bool bad = false;

#if B2O_STATS_SCHED == 1
  // dynamic: thread 0 takes the next chunk from a global counter, so the chunks being read stay
  // a compact window of the gradient buffer
  __shared__ unsigned int s_tile[2];
  if (threadIdx.x == 0) s_tile[0] = atomicAdd(ws.stats_tile, 1u);
  __syncthreads();
  int buf = 0;
  for (int64_t c = s_tile[0]; c < n_chunks;) {
#else
  for (int64_t c = blockIdx.x; c < n_chunks; c += gridDim.x) {
#endif
    const b2o_chunk ch = chunks[c];
    const b2o_tensor& t = tensors[ch.tensor];
    const void* g = t.grad;
    double acc = 0.0;
    const int64_t n = ch.end - ch.begin;
    int64_t done = 0;
    if (t.flags & B2O_FLAG_VECTOR) {
      const int64_t nv = n & ~int64_t(B2O_VEC - 1);
      done = nv;
      constexpr int64_t kStride = int64_t(kThreads) * B2O_VEC;
      for (int64_t i0 = int64_t(threadIdx.x) * B2O_VEC; i0 < nv; i0 += kStride * U) {
        typename G::vec_t v[U];
        // Issue all U loads before reducing any of them.
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int64_t i = i0 + u * kStride;
          if (i < nv) v[u] = G::load(g, ch.begin + i);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int64_t i = i0 + u * kStride;
          if (i < nv) {
            bad |= G::nonfinite(v[u]);
            float x[B2O_VEC];
            G::unpack(v[u], x);
            float s = 0.0f;
#pragma unroll
            for (int k = 0; k < B2O_VEC; ++k) {
              const float e = __fmul_rn(x[k], inv);
              s = __fmaf_rn(e, e, s);
            }
            acc += (double)s;
          }
        }
      }
    }
    for (int64_t i = done + threadIdx.x; i < n; i += kThreads) {
      const double u = (double)__fmul_rn(G::load1(g, ch.begin + i, bad), inv);
      acc += u * u;  // exact: a squared fp32 value fits in fp64
    }
#if B2O_STATS_SCHED == 1
    // The next chunk is claimed only once this one is read (the claim's latency overlaps the
    // block sum), so a CTA that started early cannot hold a second chunk while another CTA has
    // none; a chunk is many loop iterations long here.
    if (threadIdx.x == 0) s_tile[buf ^ 1] = atomicAdd(ws.stats_tile, 1u);
#endif
    const double total = block_sum(acc, scratch);
    if (threadIdx.x == 0) ws.chunk_sums[c] = total;
#if B2O_STATS_SCHED == 1
    __syncthreads();  // s_tile[buf ^ 1] is written; every thread moves on together
    buf ^= 1;
    c = s_tile[buf];
#endif
  }

  stats_epilogue(bad, tensors, n_tensors, n_chunks, n_slots, ws, exch, flags, found_inf_out,
                 norm_out, scratch, &is_last);
}

// Reduce-scatter of bf16 gradients fused with the statistics pass.  Each element of this rank's
// shard is summed over every rank's buffer (peer loads over NVLink, fp32, rank order), scaled,
// rounded to bf16 and written in place; the statistics are taken on the rounded values, i.e. on
// exactly what the update pass will read.
template <int U>
__global__ void __launch_bounds__(kThreads, 4)
rs_stats_kernel(PeerPtrs peers, int n_ranks, const char* my_base, float scale_factor,
                const b2o_tensor* __restrict__ tensors, int n_tensors,
                const b2o_chunk* __restrict__ chunks, int64_t n_chunks, int n_slots,
                const float* __restrict__ loss_scale, Workspace ws, double* exch) {
  __shared__ double scratch[kWarps];
  __shared__ int is_last;
  __shared__ unsigned int s_tile[2];
  const float inv = inv_scale_of(loss_scale);
  bool bad = false;
  if (threadIdx.x == 0) s_tile[0] = atomicAdd(ws.stats_tile, 1u);
  __syncthreads();
  int buf = 0;
  for (int64_t c = s_tile[0]; c < n_chunks;) {
    if (threadIdx.x == 0) s_tile[buf ^ 1] = atomicAdd(ws.stats_tile, 1u);
    const b2o_chunk ch = chunks[c];
    const b2o_tensor& t = tensors[ch.tensor];
    uint16_t* g = static_cast<uint16_t*>(const_cast<void*>(t.grad));
    const int64_t off = reinterpret_cast<const char*>(t.grad) - my_base;  // bytes into the buffer
    double acc = 0.0;
    const int64_t n = ch.end - ch.begin;
    int64_t done = 0;
    if (t.flags & B2O_FLAG_VECTOR) {
      const int64_t nv = n & ~int64_t(B2O_VEC - 1);
      done = nv;
      constexpr int64_t kStride = int64_t(kThreads) * B2O_VEC;
      for (int64_t i0 = int64_t(threadIdx.x) * B2O_VEC; i0 < nv; i0 += kStride * U) {
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int64_t i = i0 + u * kStride;
          if (i < nv) {
            const int64_t byte = off + 2 * (ch.begin + i);
            uint4 v[B2O_MAX_PEERS];
#pragma unroll
            for (int r = 0; r < B2O_MAX_PEERS; ++r)
              if (r < n_ranks) v[r] = ld_stream(reinterpret_cast<const uint4*>(peers.p[r] + byte));
            float sum[B2O_VEC];
            {
              const GradBF16::vec_t v0{v[0]};
              GradBF16::unpack(v0, sum);
            }
#pragma unroll
            for (int r = 1; r < B2O_MAX_PEERS; ++r) {
              if (r < n_ranks) {
                float x[B2O_VEC];
                const GradBF16::vec_t vr{v[r]};
                GradBF16::unpack(vr, x);
#pragma unroll
                for (int k = 0; k < B2O_VEC; ++k) sum[k] = __fadd_rn(sum[k], x[k]);
              }
            }
            uint4 q;
            q.x = pack_bf16x2(__fmul_rn(sum[0], scale_factor), __fmul_rn(sum[1], scale_factor));
            q.y = pack_bf16x2(__fmul_rn(sum[2], scale_factor), __fmul_rn(sum[3], scale_factor));
            q.z = pack_bf16x2(__fmul_rn(sum[4], scale_factor), __fmul_rn(sum[5], scale_factor));
            q.w = pack_bf16x2(__fmul_rn(sum[6], scale_factor), __fmul_rn(sum[7], scale_factor));
            st_stream(reinterpret_cast<uint4*>(g + ch.begin + i), q);
            const GradBF16::vec_t red{q};
            bad |= GradBF16::nonfinite(red);
            float x[B2O_VEC];
            GradBF16::unpack(red, x);
            float s2 = 0.0f;
#pragma unroll
            for (int k = 0; k < B2O_VEC; ++k) {
              const float e = __fmul_rn(x[k], inv);
              s2 = __fmaf_rn(e, e, s2);
            }
            acc += (double)s2;
          }
        }
      }
    }
    for (int64_t i = done + threadIdx.x; i < n; i += kThreads) {
      const int64_t byte = off + 2 * (ch.begin + i);
      float sum = 0.0f;
      for (int r = 0; r < n_ranks; ++r) {
        const uint16_t b = *reinterpret_cast<const uint16_t*>(peers.p[r] + byte);
        const float x = __uint_as_float(static_cast<uint32_t>(b) << 16);
        sum = r == 0 ? x : __fadd_rn(sum, x);
      }
      const uint16_t red = to_bf16_bits(__fmul_rn(sum, scale_factor));
      g[ch.begin + i] = red;
      bad |= (red & 0x7f80u) == 0x7f80u;
      const double u = (double)__fmul_rn(__uint_as_float(static_cast<uint32_t>(red) << 16), inv);
      acc += u * u;
    }
    const double total = block_sum(acc, scratch);
    if (threadIdx.x == 0) ws.chunk_sums[c] = total;
    __syncthreads();  // s_tile[buf ^ 1] is written; every thread moves on together
    buf ^= 1;
    c = s_tile[buf];
  }
  stats_epilogue(bad, tensors, n_tensors, n_chunks, n_slots, ws, exch, B2O_STATS_CLEAR, nullptr,
                 nullptr, scratch, &is_last);
}

__global__ void __launch_bounds__(kThreads, 4)
finalize_norm_kernel(const double* exch_all, int n_ranks, int n_slots, float* found_inf_out,
                     float* norm_out) {
  __shared__ double scratch[kWarps];
  finalize_norm_cta(exch_all, n_ranks, n_slots, found_inf_out, norm_out, scratch);
}

}  // namespace b2o

using namespace b2o;

extern "C" int b2o_grad_stats(const b2o_tensor* tensors, int32_t n_tensors,
                              const b2o_chunk* chunks, int64_t n_chunks, int32_t n_slots,
                              int32_t grad_dtype, const float* loss_scale, void* workspace,
                              double* exch, int32_t flags, float* found_inf_out,
                              float* norm_out, void* stream) {
  if (!tensors || !workspace || n_tensors < 0 || n_chunks < 0 || n_slots < 0) return B2O_ERR_ARG;
  if (n_chunks > 0 && !chunks) return B2O_ERR_ARG;
  if ((flags & B2O_STATS_FINALIZE) && (!found_inf_out || !norm_out)) return B2O_ERR_ARG;
  Workspace ws = carve_workspace(workspace, n_chunks);
  if (!exch) exch = ws.exch;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (grad_dtype == B2O_BF16) {
    const int grid = stream_grid((const void*)grad_stats_kernel<GradBF16>, kThreads, n_chunks);
    if (grid <= 0) return B2O_ERR_CUDA;
    grad_stats_kernel<GradBF16><<<grid, kThreads, 0, s>>>(tensors, n_tensors, chunks, n_chunks,
                                                          n_slots, loss_scale, ws, exch, flags,
                                                          found_inf_out, norm_out);
  } else if (grad_dtype == B2O_F32) {
    const int grid = stream_grid((const void*)grad_stats_kernel<GradF32>, kThreads, n_chunks);
    if (grid <= 0) return B2O_ERR_CUDA;
    grad_stats_kernel<GradF32><<<grid, kThreads, 0, s>>>(tensors, n_tensors, chunks, n_chunks,
                                                         n_slots, loss_scale, ws, exch, flags,
                                                         found_inf_out, norm_out);
  } else {
    return B2O_ERR_ARG;
  }
  return cudaGetLastError() == cudaSuccess ? B2O_OK : B2O_ERR_LAUNCH;
}

extern "C" int b2o_reduce_scatter_stats(const void* const* peer_grads, int32_t n_ranks,
                                        const void* my_grad_base, float scale_factor,
                                        const b2o_tensor* tensors, int32_t n_tensors,
                                        const b2o_chunk* chunks, int64_t n_chunks,
                                        int32_t n_slots, const float* loss_scale,
                                        void* workspace, double* exch, void* stream) {
  if (!peer_grads || n_ranks < 1 || n_ranks > B2O_MAX_PEERS || !my_grad_base || !tensors ||
      !workspace || n_tensors < 0 || n_chunks < 0 || n_slots < 0)
    return B2O_ERR_ARG;
  if (n_chunks > 0 && !chunks) return B2O_ERR_ARG;
  PeerPtrs peers{};
  for (int r = 0; r < n_ranks; ++r) {
    if (!peer_grads[r]) return B2O_ERR_ARG;
    peers.p[r] = static_cast<char*>(const_cast<void*>(peer_grads[r]));
  }
  Workspace ws = carve_workspace(workspace, n_chunks);
  if (!exch) exch = ws.exch;
  const int grid = stream_grid((const void*)rs_stats_kernel<2>, kThreads, n_chunks);
  if (grid <= 0) return B2O_ERR_CUDA;
  rs_stats_kernel<2><<<grid, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      peers, n_ranks, static_cast<const char*>(my_grad_base), scale_factor, tensors, n_tensors,
      chunks, n_chunks, n_slots, loss_scale, ws, exch);
  return cudaGetLastError() == cudaSuccess ? B2O_OK : B2O_ERR_LAUNCH;
}

extern "C" int b2o_finalize_norm(const double* exch_all, int32_t n_ranks, int32_t n_slots,
                                 float* found_inf_out, float* norm_out, void* stream) {
  if (!exch_all || n_ranks <= 0 || n_slots < 0 || !found_inf_out || !norm_out) return B2O_ERR_ARG;
  finalize_norm_kernel<<<1, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      exch_all, n_ranks, n_slots, found_inf_out, norm_out);
  return cudaGetLastError() == cudaSuccess ? B2O_OK : B2O_ERR_LAUNCH;
}

// ---------------------------------------------------------------------------------------------
// Allocation-free variant (b2o_grad_stats_noalloc).  Some hosts cannot allocate device memory
// for the statistics scratch -- an FFI caller that only holds pointers another runtime handed it,
// or a process at its memory ceiling -- so this entry point keeps its scratch in one fixed array
// of this library and launches the same kernel as b2o_grad_stats over it.
// ---------------------------------------------------------------------------------------------

namespace b2o {

constexpr size_t kNoallocScratchBytes =
    (64 + sizeof(double) * (size_t(B2O_NOALLOC_MAX_CHUNKS) + B2O_NOALLOC_MAX_SLOTS + 1) + 255) /
    256 * 256;

// The fixed scratch: completion counters, per-chunk partials and per-slot sums, laid out as
// carve_workspace() expects.  Host code must not take its address directly; the device address
// comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoallocScratchBytes];

// A module global exists once per CUDA context, so its device address belongs to the context
// that is current when it is looked up.  Runtime-API callers always run in the device's primary
// context, but an FFI host may have made a context of its own current (cuCtxCreate /
// cuCtxSetCurrent), and the array's address there is a different one.  The cache is therefore
// keyed by the process-unique id of the current context (cuCtxGetId; ids are never reused, so a
// destroyed context's entry cannot be mistaken for a new one).  The two driver calls are taken
// through the runtime's entry-point query, so the library does not link libcuda itself.
using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);

static bool current_context_id(unsigned long long* id) {
  static CtxGetCurrentFn get_current = nullptr;
  static CtxGetIdFn get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &f, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<CtxGetCurrentFn>(f);
    f = nullptr;
    q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetId", &f, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<CtxGetIdFn>(f);
  });
  if (get_current == nullptr || get_id == nullptr) return false;
  CUcontext ctx = nullptr;
  if (get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return false;
  return get_id(ctx, id) == CUDA_SUCCESS;
}

// Device address of g_noalloc_scratch in the context current on the calling thread, looked up
// once per context (for runtime-API callers: once per device, on that device's first call).
static void* noalloc_scratch_ptr() {
  struct Slot { unsigned long long ctx_id; void* ptr; };
  static std::mutex mu;
  static Slot cache[64];
  static int n_cache = 0;
  unsigned long long id = 0;
  void* fresh = nullptr;
  if (!current_context_id(&id)) {
    // No context is current on this thread yet: the lookup makes the current device's primary
    // context current, after which it can be identified.
    if (cudaGetSymbolAddress(&fresh, g_noalloc_scratch) != cudaSuccess) return nullptr;
    if (!current_context_id(&id)) return fresh;  // unidentifiable context: use it uncached
  }
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < n_cache; ++i)
    if (cache[i].ctx_id == id) return cache[i].ptr;
  if (fresh == nullptr && cudaGetSymbolAddress(&fresh, g_noalloc_scratch) != cudaSuccess)
    return nullptr;
  if (n_cache < 64) cache[n_cache++] = Slot{id, fresh};
  return fresh;
}

}  // namespace b2o

extern "C" int b2o_grad_stats_noalloc(const b2o_tensor* tensors, int32_t n_tensors,
                                      const b2o_chunk* chunks, int64_t n_chunks,
                                      int32_t n_slots, int32_t grad_dtype,
                                      const float* loss_scale, float* found_inf_out,
                                      float* norm_out, void* stream) {
  if (!tensors || n_tensors < 0 || n_chunks < 0 || n_slots < 0 || !found_inf_out || !norm_out)
    return B2O_ERR_ARG;
  if (n_chunks > 0 && !chunks) return B2O_ERR_ARG;
  if (grad_dtype != B2O_BF16 && grad_dtype != B2O_F32) return B2O_ERR_ARG;
  if (n_chunks > B2O_NOALLOC_MAX_CHUNKS || n_slots > B2O_NOALLOC_MAX_SLOTS)
    return B2O_ERR_TOO_LARGE;
  void* scratch = noalloc_scratch_ptr();
  if (scratch == nullptr) return B2O_ERR_CUDA;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // The counters must start at zero; the partial sums are written before they are read.
  if (cudaMemsetAsync(scratch, 0, ws_counter_bytes(), s) != cudaSuccess) return B2O_ERR_CUDA;
  Workspace ws = carve_workspace(scratch, n_chunks);
  const int flags = B2O_STATS_CLEAR | B2O_STATS_FINALIZE;
  if (grad_dtype == B2O_BF16) {
    const int grid = stream_grid((const void*)grad_stats_kernel<GradBF16>, kThreads, n_chunks);
    if (grid <= 0) return B2O_ERR_CUDA;
    grad_stats_kernel<GradBF16><<<grid, kThreads, 0, s>>>(tensors, n_tensors, chunks, n_chunks,
                                                          n_slots, loss_scale, ws, ws.exch, flags,
                                                          found_inf_out, norm_out);
  } else {
    const int grid = stream_grid((const void*)grad_stats_kernel<GradF32>, kThreads, n_chunks);
    if (grid <= 0) return B2O_ERR_CUDA;
    grad_stats_kernel<GradF32><<<grid, kThreads, 0, s>>>(tensors, n_tensors, chunks, n_chunks,
                                                         n_slots, loss_scale, ws, ws.exch, flags,
                                                         found_inf_out, norm_out);
  }
  return cudaGetLastError() == cudaSuccess ? B2O_OK : B2O_ERR_LAUNCH;
}
