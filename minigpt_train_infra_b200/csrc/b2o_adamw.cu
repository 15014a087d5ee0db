// Pass 2 of the optimizer step: fused AdamW + bf16 parameter refresh (sm_100a).
//
// One read of grad (2 B bf16), master, exp_avg, exp_avg_sq (12 B) and one write of master,
// exp_avg, exp_avg_sq (12 B) and the bf16 parameter (2 B) per element: 28 bytes, the HBM
// roofline of this pass.  No tensor cores: the step is ~15 flops per 28 bytes.
//
// Per element, in the order and rounding of torch's single-tensor AdamW on the reference's
// CPU path (torch/optim/adam.py:414-547, decoupled weight decay from torch/optim/adamw.py):
//   g  = (float(grad) * inv_scale) * clip_coef          grad_scaler.py:294, clip_grad.py:174
//   w  = w * fp32(1 - lr*wd)                            adam.py:419
//   m  = fma(fp32(1-b1), g - m, m)                      adam.py:457 (lerp, weight < 0.5)
//   v  = fma(fp32(1-b2) * g, g, v * fp32(b2))           adam.py:476 (mul_ then addcmul_)
//   d  = sqrt(v) / fp32(sqrt(1 - b2^step)) + fp32(eps)  adam.py:536,545
//   w  = w + (fp32(-lr/(1 - b1^step)) * m) / d          adam.py:534,547 (addcdiv_)
//   p  = bf16_rne(w)                                    the mixed-precision parameter copy
// The bias-correction scalars are formed in fp64 from the device step counter, as the
// reference forms them in Python doubles from state["step"].
//
// Skipping: when *found_inf != 0 every CTA returns before touching memory, so a skipped step
// moves ~0 bytes and leaves the step counters alone (GradScaler.step's skip, grad_scaler.py:
// 363-374).  Otherwise the last CTA to finish stores step+1 for every slot of the table.
#include <cuda_runtime.h>

#include "b2o_device.cuh"
#include "b2o_host.h"

namespace b2o {

struct GroupArgs {
  b2o_group g[B2O_MAX_GROUPS];
};

struct ChunkScalars {
  float decay, w1, w1m1, beta2, omb2, bc2_sqrt, neg_step_size, eps;
  int small_w1;
};

// The per-tensor scalars of one step, formed by a whole warp: lane 0 evaluates beta1^step and
// lane 1 beta2^step (one pow per lane, no divergence) and the results are shuffled to every lane.
// Python evaluates these in double with one rounding per operator; the explicit _rn forms keep
// nvcc from contracting `1 - lr*wd` into an fma.
__device__ __forceinline__ void warp_scalars(const b2o_group& hp, float step_old, int lane,
                                             ChunkScalars& s) {
  const double step = (double)__fadd_rn(step_old, 1.0f);  // torch: step_t += 1 (fp32), .item()
  const double pw = pow(lane == 0 ? hp.beta1 : hp.beta2, step);
  const double p1 = __shfl_sync(0xffffffffu, pw, 0);
  const double p2 = __shfl_sync(0xffffffffu, pw, 1);
  const double bc1 = __dsub_rn(1.0, p1);
  const double bc2 = __dsub_rn(1.0, p2);
  s.decay = (float)__dsub_rn(1.0, __dmul_rn(hp.lr, hp.weight_decay));
  s.w1 = (float)__dsub_rn(1.0, hp.beta1);
  s.w1m1 = __fsub_rn(s.w1, 1.0f);
  s.small_w1 = fabsf(s.w1) < 0.5f;
  s.beta2 = (float)hp.beta2;
  s.omb2 = (float)__dsub_rn(1.0, hp.beta2);
  s.bc2_sqrt = (float)__dsqrt_rn(bc2);  // bias_correction2 ** 0.5
  s.neg_step_size = (float)(-__ddiv_rn(hp.lr, bc1));
  s.eps = (float)hp.eps;
}

__device__ __forceinline__ void adamw_elem(const ChunkScalars& s, float g, float& w, float& m,
                                           float& v) {
  w = __fmul_rn(w, s.decay);
  const float diff = __fsub_rn(g, m);
  m = s.small_w1 ? __fmaf_rn(s.w1, diff, m) : __fmaf_rn(s.w1m1, diff, g);
  v = __fmaf_rn(__fmul_rn(s.omb2, g), g, __fmul_rn(v, s.beta2));
  const float d = __fadd_rn(__fdiv_rn(__fsqrt_rn(v), s.bc2_sqrt), s.eps);
  w = __fadd_rn(w, __fdiv_rn(__fmul_rn(s.neg_step_size, m), d));
}

__device__ __forceinline__ float clip_coefficient(float norm, float max_norm) {
  // clip_grad.py:165-169: clamp(max_norm / (norm + 1e-6), max=1); python_float / tensor is
  // tensor.reciprocal() * python_float; clamp keeps NaN.
  const float t = __fadd_rn(norm, 1e-6f);
  const float c = __fmul_rn(__frcp_rn(t), max_norm);
  return c > 1.0f ? 1.0f : c;
}

// TMA bulk stores (the plain shared -> global form of cp.async.bulk, one destination each) of a
// staged chunk of updated bf16 values to the other ranks' buffers: one instruction per peer
// moves the whole chunk, so the NVLink writes go out as large contiguous transfers instead of
// one 16-byte store per lane.
__device__ __forceinline__ void bulk_store_global(char* dst, const void* smem_src,
                                                  uint32_t bytes) {
  uint64_t g;
  asm volatile("cvta.to.global.u64 %0, %1;" : "=l"(g) : "l"(dst));
  const uint32_t src = static_cast<uint32_t>(__cvta_generic_to_shared(smem_src));
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;"
               :: "l"(g), "r"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Waits until at most N bulk groups of this thread still read their shared-memory source.
template <int N> __device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" :: "n"(N) : "memory");
}
// Waits until every bulk group of this thread has completed (its writes performed).
__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}
// Orders this CTA's ordinary shared-memory writes before the bulk copies that read them.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Largest update chunk the broadcast variant stages in shared memory (elements); the plan's
// update chunks are 2 Ki elements.  Longer or ragged chunks take the per-lane stores.
constexpr int kStageElems = 2048;

// Quads (4 consecutive elements) each thread keeps in flight per loop iteration, and the CTAs per
// SM the register budget is sized for.  Both are build-time knobs; the defaults were measured.
#ifndef B2O_ADAMW_QUADS
#define B2O_ADAMW_QUADS 2
#endif
#ifndef B2O_ADAMW_MIN_CTAS
#define B2O_ADAMW_MIN_CTAS 4
#endif
// Chunk scheduling of the update pass: 0 static round-robin over CTAs, 1 dynamic per CTA,
// 2 dynamic per warp (both dynamic modes take chunks in order from a counter in the workspace,
// so the chunks in flight stay a compact window of each array).
#ifndef B2O_ADAMW_SCHED
#define B2O_ADAMW_SCHED 1
#endif

// Where the updated bf16 parameters also go when the ZeRO-1 all-gather is fused into the
// update: every other rank's copy of the flat parameter buffer (index = rank).
struct Broadcast {
  PeerPtrs peers;
  const char* my_base;
  int n_ranks;
  int my_rank;
};

// Stores one updated quad (4 bf16 = 8 bytes; quad q of a chunk's nq quads, at `dst` in this
// rank's buffer) at the same offset of every other rank's buffer.  The quads of lanes 2k and 2k+1
// are adjacent (q even and q + 1), so together they are 16 bytes on a 16-byte boundary: when both
// exist the pair swaps them with a shuffle and each lane stores the 16 bytes to half of the peers
// (even lane: peers 0, 2, 4, ... of the CTA's rotated list; odd lane: 1, 3, 5, ...).  A quad
// whose partner is past the end of the chunk goes to every peer as 8 bytes.  Both lanes of a
// pair evaluate the same condition (q_odd < nq), so the pair shuffle always has both lanes.
__device__ __forceinline__ void broadcast_quad(const Broadcast& bc, char* const* s_peer,
                                               const uint16_t* dst, uint2 pq, int64_t q,
                                               int64_t nq, int lane) {
  const int64_t byte = reinterpret_cast<const char*>(dst) - bc.my_base;
  const int n_peers = bc.n_ranks - 1;
  if ((q ^ 1) < nq) {
    const unsigned pair = 3u << (lane & ~1);
    const unsigned ox = __shfl_xor_sync(pair, pq.x, 1);
    const unsigned oy = __shfl_xor_sync(pair, pq.y, 1);
    const int odd = lane & 1;
    const uint4 v = odd ? make_uint4(ox, oy, pq.x, pq.y) : make_uint4(pq.x, pq.y, ox, oy);
    const int64_t base = odd ? byte - 8 : byte;
#pragma unroll
    for (int j = 0; j < B2O_MAX_PEERS - 1; j += 2) {
      const int k = j + odd;
      if (k < n_peers) __stcs(reinterpret_cast<uint4*>(s_peer[k] + base), v);
    }
  } else {
    for (int k = 0; k < n_peers; ++k) __stcs(reinterpret_cast<uint2*>(s_peer[k] + byte), pq);
  }
}

template <class G, bool BF16_PARAM, int Q, bool BCAST = false, bool DEV_HP = false>
__global__ void __launch_bounds__(kThreads, B2O_ADAMW_MIN_CTAS)
adamw_kernel(const b2o_tensor* __restrict__ tensors, int n_tensors,
             const b2o_chunk* __restrict__ chunks, int64_t n_chunks, GroupArgs groups,
             float* __restrict__ steps, const float* __restrict__ found_inf,
             const float* __restrict__ loss_scale, const float* __restrict__ norm_p,
             float max_norm, float* clip_coef_out, Workspace ws, Broadcast bc = Broadcast{},
             const b2o_group* __restrict__ dev_groups = nullptr) {
  if (found_inf != nullptr && *found_inf != 0.0f) return;  // skipped step: no traffic at all
  __shared__ int is_last;
  // The other ranks' buffers in the order this CTA stores to them: starting after this rank and
  // rotated by the CTA index, so the stores in flight spread over all peers at any moment.
  __shared__ char* s_peer[B2O_MAX_PEERS];
  if (BCAST) {
    const int n_peers = bc.n_ranks - 1;
    if (threadIdx.x < n_peers) {
      const int j = int((threadIdx.x + blockIdx.x) % unsigned(n_peers));
      s_peer[threadIdx.x] = bc.peers.p[(bc.my_rank + 1 + j) % bc.n_ranks];
    }
    __syncthreads();
  }
  // Two shared-memory stages of one chunk's updated bf16 values, for the bulk stores to the
  // peers (only the broadcast variant with CTA-wide chunk scheduling uses them).
  constexpr bool kStaged = BCAST && B2O_ADAMW_SCHED != 2;
  __shared__ __align__(128) uint2 s_stage[kStaged ? 2 : 1][kStaged ? kStageElems / 4 : 1];
  int sb = 0;
  const float inv = inv_scale_of(loss_scale);
  const float coef = norm_p ? clip_coefficient(*norm_p, max_norm) : 1.0f;
  if (clip_coef_out && blockIdx.x == 0 && threadIdx.x == 0) *clip_coef_out = coef;
  const int lane = threadIdx.x & 31;

  // Per-tensor state, refreshed only when the chunk sequence enters another tensor.  Every
  // thread of a scheduling unit (the CTA, or the warp when B2O_ADAMW_SCHED == 2) walks the same
  // chunks, so the refresh branch is uniform within it.
  int cur = -1;
  ChunkScalars s{};
  const void* gp = nullptr;
  float* wp = nullptr;
  float* mp = nullptr;
  float* vp = nullptr;
  uint16_t* pp = nullptr;
  int flags = 0;
#if B2O_ADAMW_SCHED == 0
  // static: CTA b takes chunks b, b + grid, b + 2*grid, ...
  constexpr int kUnit = kThreads;
  const int utid = threadIdx.x;
  b2o_chunk next{};
  if (blockIdx.x < n_chunks) next = chunks[blockIdx.x];
  for (int64_t c = blockIdx.x; c < n_chunks; c += gridDim.x) {
    const b2o_chunk ch = next;
    if (c + gridDim.x < n_chunks) next = chunks[c + gridDim.x];  // prefetch the next record
#elif B2O_ADAMW_SCHED == 1
  // dynamic per CTA: thread 0 takes the next chunk from a global counter one chunk ahead
  constexpr int kUnit = kThreads;
  const int utid = threadIdx.x;
  __shared__ unsigned int s_tile[2];
  if (threadIdx.x == 0) s_tile[0] = atomicAdd(ws.adamw_tile, 1u);
  __syncthreads();
  int buf = 0;
  for (int64_t c = s_tile[0]; c < n_chunks; ) {
    if (threadIdx.x == 0) s_tile[buf ^ 1] = atomicAdd(ws.adamw_tile, 1u);
    const b2o_chunk ch = chunks[c];
#else
  // dynamic per warp: lane 0 takes the next chunk one chunk ahead, shuffled to the warp
  constexpr int kUnit = 32;
  const int utid = lane;
  unsigned int tile = 0;
  if (lane == 0) tile = atomicAdd(ws.adamw_tile, 1u);
  tile = __shfl_sync(0xffffffffu, tile, 0);
  for (int64_t c = tile; c < n_chunks; ) {
    unsigned int nt = 0;
    if (lane == 0) nt = atomicAdd(ws.adamw_tile, 1u);
    const b2o_chunk ch = chunks[c];
#endif
    if (ch.tensor != cur) {
      cur = ch.tensor;
      const b2o_tensor& t = tensors[cur];
      gp = t.grad;
      wp = t.master;
      mp = t.exp_avg;
      vp = t.exp_avg_sq;
      pp = static_cast<uint16_t*>(t.param);
      flags = t.flags;
      warp_scalars(DEV_HP ? dev_groups[t.group] : groups.g[t.group], steps[t.slot], lane, s);
    }
    const int64_t n = ch.end - ch.begin;
    int64_t done = 0;
    // The whole chunk goes to the peers as bulk stores when it fits a stage and is a multiple
    // of 8 elements (16 bytes); the condition is the same for every thread of the CTA.
    const bool staged = kStaged && (flags & B2O_FLAG_VECTOR) && n <= kStageElems &&
                        (n & 7) == 0 && bc.n_ranks > 1;
    if (flags & B2O_FLAG_VECTOR) {
      const int64_t nq = n >> 2;
      done = nq << 2;
      for (int64_t q0 = utid; q0 < nq; q0 += int64_t(kUnit) * Q) {
        typename G::quad_t gq[Q];
        float4 w[Q], m[Q], v[Q];
        // Issue every load of the Q quads before any arithmetic.
#pragma unroll
        for (int u = 0; u < Q; ++u) {
          const int64_t q = q0 + int64_t(u) * kUnit;
          if (q < nq) {
            const int64_t e = ch.begin + 4 * q;
            gq[u] = G::load4(gp, e);
            w[u] = ld_stream(reinterpret_cast<const float4*>(wp + e));
            m[u] = ld_stream(reinterpret_cast<const float4*>(mp + e));
            v[u] = ld_stream(reinterpret_cast<const float4*>(vp + e));
          }
        }
#pragma unroll
        for (int u = 0; u < Q; ++u) {
          const int64_t q = q0 + int64_t(u) * kUnit;
          if (q < nq) {
            const int64_t e = ch.begin + 4 * q;
            float x[4];
            G::unpack4(gq[u], x);
            float* wf = reinterpret_cast<float*>(&w[u]);
            float* mf = reinterpret_cast<float*>(&m[u]);
            float* vf = reinterpret_cast<float*>(&v[u]);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const float g = __fmul_rn(__fmul_rn(x[k], inv), coef);
              adamw_elem(s, g, wf[k], mf[k], vf[k]);
            }
            st_stream(reinterpret_cast<float4*>(wp + e), w[u]);
            st_stream(reinterpret_cast<float4*>(mp + e), m[u]);
            st_stream(reinterpret_cast<float4*>(vp + e), v[u]);
            if (BF16_PARAM) {
              uint2 pq;
              pq.x = pack_bf16x2(wf[0], wf[1]);
              pq.y = pack_bf16x2(wf[2], wf[3]);
              __stcs(reinterpret_cast<uint2*>(pp + e), pq);
              if (BCAST) {
                if (staged)
                  s_stage[kStaged ? sb : 0][q] = pq;
                else
                  broadcast_quad(bc, s_peer, pp + e, pq, q, nq, lane);
              }
            }
          }
        }
      }
    }
    for (int64_t i = done + utid; i < n; i += kUnit) {
      const int64_t e = ch.begin + i;
      bool unused = false;
      const float g = __fmul_rn(__fmul_rn(G::load1(gp, e, unused), inv), coef);
      float w = wp[e], m = mp[e], v = vp[e];
      adamw_elem(s, g, w, m, v);
      wp[e] = w;
      mp[e] = m;
      vp[e] = v;
      if (BF16_PARAM) {
        const uint16_t b = to_bf16_bits(w);
        pp[e] = b;
        if (BCAST) {
          const int64_t byte = reinterpret_cast<const char*>(pp + e) - bc.my_base;
          for (int j = 0; j < bc.n_ranks - 1; ++j)
            *reinterpret_cast<uint16_t*>(s_peer[j] + byte) = b;
        }
      }
    }
    if (kStaged && staged) {
      __syncthreads();  // the whole chunk is in s_stage[sb]
      if (threadIdx.x == 0) {
        fence_proxy_async_smem();
        const int64_t byte = reinterpret_cast<const char*>(pp + ch.begin) - bc.my_base;
        const uint32_t bytes = uint32_t(n) * 2u;
        for (int j = 0; j < bc.n_ranks - 1; ++j)
          bulk_store_global(s_peer[j] + byte, &s_stage[sb][0], bytes);
        bulk_commit();
        bulk_wait_read<1>();  // the group of the chunk before this one has read s_stage[sb ^ 1]
      }
      __syncthreads();  // s_stage[sb ^ 1] may be written again
      sb ^= 1;
    }
#if B2O_ADAMW_SCHED == 1
    __syncthreads();  // s_tile[buf ^ 1] is written; every thread moves on together
    buf ^= 1;
    c = s_tile[buf];
#elif B2O_ADAMW_SCHED == 2
    c = __shfl_sync(0xffffffffu, nt, 0);
#endif
  }

  // Completion ticket; the last CTA advances the step counters after every CTA has read them.
  if (kStaged && threadIdx.x == 0) bulk_wait_all();  // the bulk stores to the peers are done
  if (BCAST) __threadfence_system();  // peer stores performed before the kernel completes
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) is_last = atomicAdd(ws.adamw_done, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  for (int ti = threadIdx.x; ti < n_tensors; ti += kThreads) {
    const int slot = tensors[ti].slot;
    steps[slot] = __fadd_rn(__ldcg(steps + slot), 1.0f);
  }
  if (threadIdx.x == 0) {
    *ws.adamw_tile = 0u;
    *ws.adamw_done = 0u;
  }
}

template <class G, bool P>
int launch_adamw(cudaStream_t s, const b2o_tensor* tensors, int n_tensors,
                 const b2o_chunk* chunks, int64_t n_chunks, const GroupArgs& ga, float* steps,
                 const float* found_inf, const float* loss_scale, const float* norm, float max_norm,
                 float* coef_out, Workspace ws, const b2o_group* dev_groups = nullptr) {
  constexpr int Q = B2O_ADAMW_QUADS;
  if (dev_groups) {
    const int grid =
        stream_grid((const void*)adamw_kernel<G, P, Q, false, true>, kThreads, n_chunks);
    if (grid <= 0) return B2O_ERR_CUDA;
    adamw_kernel<G, P, Q, false, true><<<grid, kThreads, 0, s>>>(
        tensors, n_tensors, chunks, n_chunks, ga, steps, found_inf, loss_scale, norm, max_norm,
        coef_out, ws, Broadcast{}, dev_groups);
  } else {
    const int grid = stream_grid((const void*)adamw_kernel<G, P, Q>, kThreads, n_chunks);
    if (grid <= 0) return B2O_ERR_CUDA;
    adamw_kernel<G, P, Q><<<grid, kThreads, 0, s>>>(tensors, n_tensors, chunks, n_chunks, ga,
                                                    steps, found_inf, loss_scale, norm, max_norm,
                                                    coef_out, ws);
  }
  return cudaGetLastError() == cudaSuccess ? B2O_OK : B2O_ERR_LAUNCH;
}

int launch_adamw_bcast(cudaStream_t s, const b2o_tensor* tensors, int n_tensors,
                       const b2o_chunk* chunks, int64_t n_chunks, const GroupArgs& ga,
                       float* steps, const float* found_inf, const float* loss_scale,
                       const float* norm, float max_norm, Workspace ws, int grad_dtype,
                       const Broadcast& bc) {
  constexpr int Q = B2O_ADAMW_QUADS;
  if (grad_dtype == B2O_BF16) {
    const int grid =
        stream_grid((const void*)adamw_kernel<GradBF16, true, Q, true>, kThreads, n_chunks);
    if (grid <= 0) return B2O_ERR_CUDA;
    adamw_kernel<GradBF16, true, Q, true><<<grid, kThreads, 0, s>>>(
        tensors, n_tensors, chunks, n_chunks, ga, steps, found_inf, loss_scale, norm, max_norm,
        nullptr, ws, bc);
  } else {
    const int grid =
        stream_grid((const void*)adamw_kernel<GradF32, true, Q, true>, kThreads, n_chunks);
    if (grid <= 0) return B2O_ERR_CUDA;
    adamw_kernel<GradF32, true, Q, true><<<grid, kThreads, 0, s>>>(
        tensors, n_tensors, chunks, n_chunks, ga, steps, found_inf, loss_scale, norm, max_norm,
        nullptr, ws, bc);
  }
  return cudaGetLastError() == cudaSuccess ? B2O_OK : B2O_ERR_LAUNCH;
}

}  // namespace b2o

using namespace b2o;

extern "C" int b2o_adamw_step_bcast(const b2o_tensor* tensors, int32_t n_tensors,
                                    const b2o_chunk* chunks, int64_t n_chunks,
                                    const b2o_group* groups, int32_t n_groups,
                                    int32_t grad_dtype, float* steps, const float* found_inf,
                                    const float* loss_scale, const float* norm, float max_norm,
                                    void* const* peer_params, int32_t n_ranks, int32_t my_rank,
                                    const void* my_param_base, void* workspace, void* stream) {
  if (!tensors || !groups || !steps || !workspace || !peer_params || !my_param_base ||
      n_tensors < 0 || n_chunks < 0)
    return B2O_ERR_ARG;
  if (n_chunks > 0 && !chunks) return B2O_ERR_ARG;
  if (n_groups <= 0 || n_groups > B2O_MAX_GROUPS) return B2O_ERR_ARG;
  if (n_ranks < 1 || n_ranks > B2O_MAX_PEERS || my_rank < 0 || my_rank >= n_ranks)
    return B2O_ERR_ARG;
  if (grad_dtype != B2O_BF16 && grad_dtype != B2O_F32) return B2O_ERR_ARG;
  Broadcast bc{};
  for (int r = 0; r < n_ranks; ++r) {
    if (!peer_params[r]) return B2O_ERR_ARG;
    bc.peers.p[r] = static_cast<char*>(peer_params[r]);
  }
  bc.my_base = static_cast<const char*>(my_param_base);
  bc.n_ranks = n_ranks;
  bc.my_rank = my_rank;
  GroupArgs ga{};
  for (int i = 0; i < n_groups; ++i) ga.g[i] = groups[i];
  return launch_adamw_bcast(static_cast<cudaStream_t>(stream), tensors, n_tensors, chunks,
                            n_chunks, ga, steps, found_inf, loss_scale, norm, max_norm,
                            carve_workspace(workspace, 0), grad_dtype, bc);
}

extern "C" int b2o_adamw_step(const b2o_tensor* tensors, int32_t n_tensors,
                              const b2o_chunk* chunks, int64_t n_chunks, const b2o_group* groups,
                              int32_t n_groups, int32_t grad_dtype, int32_t param_dtype,
                              float* steps, const float* found_inf, const float* loss_scale,
                              const float* norm, float max_norm, float* clip_coef_out,
                              void* workspace, void* stream) {
  if (!tensors || !groups || !steps || !workspace || n_tensors < 0 || n_chunks < 0)
    return B2O_ERR_ARG;
  if (n_chunks > 0 && !chunks) return B2O_ERR_ARG;
  if (n_groups <= 0 || n_groups > B2O_MAX_GROUPS) return B2O_ERR_ARG;
  GroupArgs ga{};
  for (int i = 0; i < n_groups; ++i) ga.g[i] = groups[i];
  Workspace ws = carve_workspace(workspace, n_chunks);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool bf16p = param_dtype == B2O_BF16;
  if (param_dtype != B2O_BF16 && param_dtype != B2O_F32) return B2O_ERR_ARG;
  if (grad_dtype == B2O_BF16) {
    return bf16p ? launch_adamw<GradBF16, true>(s, tensors, n_tensors, chunks, n_chunks, ga,
                                                steps, found_inf, loss_scale, norm, max_norm,
                                                clip_coef_out, ws)
                 : launch_adamw<GradBF16, false>(s, tensors, n_tensors, chunks, n_chunks,
                                                 ga, steps, found_inf, loss_scale, norm, max_norm,
                                                 clip_coef_out, ws);
  }
  if (grad_dtype == B2O_F32) {
    return bf16p ? launch_adamw<GradF32, true>(s, tensors, n_tensors, chunks, n_chunks, ga,
                                               steps, found_inf, loss_scale, norm, max_norm,
                                               clip_coef_out, ws)
                 : launch_adamw<GradF32, false>(s, tensors, n_tensors, chunks, n_chunks, ga,
                                                steps, found_inf, loss_scale, norm, max_norm,
                                                clip_coef_out, ws);
  }
  return B2O_ERR_ARG;
}

extern "C" int b2o_adamw_step_dev(const b2o_tensor* tensors, int32_t n_tensors,
                                  const b2o_chunk* chunks, int64_t n_chunks,
                                  const b2o_group* dev_groups, int32_t n_groups,
                                  int32_t grad_dtype, int32_t param_dtype, float* steps,
                                  const float* found_inf, const float* loss_scale,
                                  const float* norm, float max_norm, void* workspace,
                                  void* stream) {
  if (!tensors || !dev_groups || !steps || !workspace || n_tensors < 0 || n_chunks < 0)
    return B2O_ERR_ARG;
  if (n_chunks > 0 && !chunks) return B2O_ERR_ARG;
  if (n_groups <= 0 || n_groups > B2O_MAX_GROUPS) return B2O_ERR_ARG;
  if (param_dtype != B2O_BF16 && param_dtype != B2O_F32) return B2O_ERR_ARG;
  const GroupArgs ga{};
  Workspace ws = carve_workspace(workspace, n_chunks);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool bf16p = param_dtype == B2O_BF16;
  if (grad_dtype == B2O_BF16)
    return bf16p ? launch_adamw<GradBF16, true>(s, tensors, n_tensors, chunks, n_chunks, ga,
                                                steps, found_inf, loss_scale, norm, max_norm,
                                                nullptr, ws, dev_groups)
                 : launch_adamw<GradBF16, false>(s, tensors, n_tensors, chunks, n_chunks, ga,
                                                 steps, found_inf, loss_scale, norm, max_norm,
                                                 nullptr, ws, dev_groups);
  if (grad_dtype == B2O_F32)
    return bf16p ? launch_adamw<GradF32, true>(s, tensors, n_tensors, chunks, n_chunks, ga,
                                               steps, found_inf, loss_scale, norm, max_norm,
                                               nullptr, ws, dev_groups)
                 : launch_adamw<GradF32, false>(s, tensors, n_tensors, chunks, n_chunks, ga,
                                                steps, found_inf, loss_scale, norm, max_norm,
                                                nullptr, ws, dev_groups);
  return B2O_ERR_ARG;
}
