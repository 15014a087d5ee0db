// Device helpers shared by the optimizer-step kernels (sm_100a).
//
// All arithmetic that must reproduce the reference's fp32 results is written with explicit
// IEEE round-to-nearest intrinsics (__fmul_rn, __fadd_rn, __fdiv_rn, __fsqrt_rn, __fmaf_rn)
// so that nvcc never contracts or reassociates it; the library is built without
// --use_fast_math and with -ftz=false so denormals are kept as the CPU keeps them.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "b200_optim.h"

namespace b2o {

constexpr int kThreads = 256;                  // threads per CTA of the streaming passes
constexpr int kWarps = kThreads / 32;

// ---------------------------------------------------------------------------------------------
// bf16 <-> fp32
// ---------------------------------------------------------------------------------------------

// Exact widening of a bf16 bit pattern.
__device__ __forceinline__ float bf16_lo(uint32_t pair) { return __uint_as_float(pair << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t pair) { return __uint_as_float(pair & 0xffff0000u); }

// Round-to-nearest-even narrowing of two floats into one packed bf16 pair (lo, hi).
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 p = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&p);
}

__device__ __forceinline__ uint16_t to_bf16_bits(float x) {
  __nv_bfloat16 b = __float2bfloat16_rn(x);
  return *reinterpret_cast<uint16_t*>(&b);
}

// ---------------------------------------------------------------------------------------------
// Streaming 128-bit global memory access.  Optimizer state is touched exactly once per step, so
// loads and stores carry the evict-first ("cache streaming") policy.
// ---------------------------------------------------------------------------------------------

__device__ __forceinline__ uint4 ld_stream(const uint4* p) { return __ldcs(p); }
__device__ __forceinline__ float4 ld_stream(const float4* p) { return __ldcs(p); }
__device__ __forceinline__ void st_stream(uint4* p, uint4 v) { __stcs(p, v); }
__device__ __forceinline__ void st_stream(float4* p, float4 v) { __stcs(p, v); }

// ---------------------------------------------------------------------------------------------
// Gradient element access for the two supported gradient dtypes.  A "vector" is B2O_VEC (8)
// consecutive elements: one 16-byte load for bf16, two for fp32.
// ---------------------------------------------------------------------------------------------

struct GradBF16 {
  struct vec_t { uint4 q; };
  static __device__ __forceinline__ vec_t load(const void* base, int64_t i) {
    return vec_t{ld_stream(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(base) + i))};
  }
  static __device__ __forceinline__ void unpack(const vec_t& v, float (&x)[B2O_VEC]) {
    x[0] = bf16_lo(v.q.x); x[1] = bf16_hi(v.q.x);
    x[2] = bf16_lo(v.q.y); x[3] = bf16_hi(v.q.y);
    x[4] = bf16_lo(v.q.z); x[5] = bf16_hi(v.q.z);
    x[6] = bf16_lo(v.q.w); x[7] = bf16_hi(v.q.w);
  }
  // Any element with an all-ones exponent (inf or NaN).
  static __device__ __forceinline__ bool nonfinite(const vec_t& v) {
    auto bad = [](uint32_t w) {
      return ((w & 0x7f80u) == 0x7f80u) | ((w & 0x7f800000u) == 0x7f800000u);
    };
    return bad(v.q.x) | bad(v.q.y) | bad(v.q.z) | bad(v.q.w);
  }
  static __device__ __forceinline__ float load1(const void* base, int64_t i, bool& bad) {
    uint16_t b = static_cast<const uint16_t*>(base)[i];
    bad |= (b & 0x7f80u) == 0x7f80u;
    return __uint_as_float(static_cast<uint32_t>(b) << 16);
  }
  // Four consecutive elements (8 bytes); a warp's 32 quads cover 256 contiguous bytes.
  using quad_t = uint2;
  static __device__ __forceinline__ quad_t load4(const void* base, int64_t i) {
    return __ldcs(reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(base) + i));
  }
  static __device__ __forceinline__ void unpack4(const quad_t& q, float (&x)[4]) {
    x[0] = bf16_lo(q.x); x[1] = bf16_hi(q.x); x[2] = bf16_lo(q.y); x[3] = bf16_hi(q.y);
  }
};

struct GradF32 {
  struct vec_t { float4 a, b; };
  static __device__ __forceinline__ vec_t load(const void* base, int64_t i) {
    const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(base) + i);
    return vec_t{ld_stream(p), ld_stream(p + 1)};
  }
  static __device__ __forceinline__ void unpack(const vec_t& v, float (&x)[B2O_VEC]) {
    x[0] = v.a.x; x[1] = v.a.y; x[2] = v.a.z; x[3] = v.a.w;
    x[4] = v.b.x; x[5] = v.b.y; x[6] = v.b.z; x[7] = v.b.w;
  }
  static __device__ __forceinline__ bool nonfinite(const vec_t& v) {
    auto bad = [](float f) { return (__float_as_uint(f) & 0x7f800000u) == 0x7f800000u; };
    return bad(v.a.x) | bad(v.a.y) | bad(v.a.z) | bad(v.a.w) | bad(v.b.x) | bad(v.b.y) |
           bad(v.b.z) | bad(v.b.w);
  }
  static __device__ __forceinline__ float load1(const void* base, int64_t i, bool& bad) {
    float f = static_cast<const float*>(base)[i];
    bad |= (__float_as_uint(f) & 0x7f800000u) == 0x7f800000u;
    return f;
  }
  using quad_t = float4;
  static __device__ __forceinline__ quad_t load4(const void* base, int64_t i) {
    return __ldcs(reinterpret_cast<const float4*>(static_cast<const float*>(base) + i));
  }
  static __device__ __forceinline__ void unpack4(const quad_t& q, float (&x)[4]) {
    x[0] = q.x; x[1] = q.y; x[2] = q.z; x[3] = q.w;
  }
};

// GradScaler's unscale factor: `self._scale.double().reciprocal().float()` (grad_scaler.py:351).
__device__ __forceinline__ float inv_scale_of(const float* loss_scale) {
  return loss_scale ? (float)__drcp_rn((double)*loss_scale) : 1.0f;
}

// ---------------------------------------------------------------------------------------------
// Deterministic reductions (fixed shuffle pattern, fixed shared-memory order)
// ---------------------------------------------------------------------------------------------

__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Sum over the CTA; the result is valid in every thread.  `scratch` holds kWarps doubles.
__device__ __forceinline__ double block_sum(double v, double* scratch) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  double t = 0.0;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) t += scratch[w];
  return t;
}

// Base addresses of every rank's copy of one flat buffer, as mapped in this process (index =
// rank); passed to kernels by value.
struct PeerPtrs {
  char* p[B2O_MAX_PEERS];
};

// ---------------------------------------------------------------------------------------------
// Workspace layout (b2o_workspace_bytes): [counters: 8 x uint32][chunk partials: n_chunks x
// double][exchange: (n_slots + 1) x double].  The counters are the completion tickets of the
// two passes and the non-finite flag; each pass's last CTA returns its counter to zero.
// ---------------------------------------------------------------------------------------------

struct Workspace {
  unsigned int* stats_done;
  unsigned int* stats_nonfinite;
  unsigned int* adamw_done;
  unsigned int* adamw_tile;  // next chunk to hand out when the update pass schedules dynamically
  unsigned int* stats_tile;  // the same for the statistics pass
  double* chunk_sums;
  double* exch;
};

__host__ __device__ inline size_t ws_counter_bytes() { return 64; }

__host__ __device__ inline Workspace carve_workspace(void* ws, int64_t n_chunks) {
  Workspace w;
  unsigned int* c = static_cast<unsigned int*>(ws);
  w.stats_done = c + 0;
  w.stats_nonfinite = c + 1;
  w.adamw_done = c + 2;
  w.adamw_tile = c + 3;
  w.stats_tile = c + 4;
  w.chunk_sums = reinterpret_cast<double*>(static_cast<char*>(ws) + ws_counter_bytes());
  w.exch = w.chunk_sums + n_chunks;
  return w;
}

}  // namespace b2o
