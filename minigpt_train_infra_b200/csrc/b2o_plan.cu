// Host side of the multi-tensor-apply launcher: chunk planning, table validation, workspace
// sizing and the library-identity entry points.
//
// The reference's step hands torch lists of tensors (torch/amp/grad_scaler.py:294,
// torch/optim/adam.py:880) and ATen re-chunks them on every call.  Here the plan is built once
// per parameter set by b2o_plan_chunks and uploaded by the caller; every step then launches
// against the same device tables with no per-step host work beyond the launch itself.
#include <cuda_runtime.h>

#include <mutex>
#include <unordered_set>

#include "b200_optim.h"
#include "b2o_device.cuh"
#include "b2o_host.h"

namespace b2o {

int resident_ctas(const void* kernel, int threads) {
  struct Entry { const void* kernel; int device; int threads; int ctas; };
  static std::mutex mu;
  static Entry cache[64];
  static int n_cache = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  {
    std::lock_guard<std::mutex> lock(mu);
    for (int i = 0; i < n_cache; ++i)
      if (cache[i].kernel == kernel && cache[i].device == dev && cache[i].threads == threads)
        return cache[i].ctas;
  }
  int sms = 0, per_sm = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return -1;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, 0) != cudaSuccess)
    return -1;
  const int ctas = sms * (per_sm > 0 ? per_sm : 1);
  std::lock_guard<std::mutex> lock(mu);
  if (n_cache < 64) cache[n_cache++] = Entry{kernel, dev, threads, ctas};
  return ctas;
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace b2o

using namespace b2o;

extern "C" int b2o_abi_version(void) { return B2O_ABI_VERSION; }

extern "C" const char* b2o_status_string(int status) {
  switch (status) {
    case B2O_OK: return "ok";
    case B2O_ERR_ARG: return "invalid argument";
    case B2O_ERR_CAPACITY: return "output capacity too small";
    case B2O_ERR_LAUNCH: return "kernel launch failed";
    case B2O_ERR_CUDA: return "CUDA runtime call failed";
    case B2O_ERR_TABLE: return "inconsistent tensor table";
    case B2O_ERR_TOO_LARGE:
      return "plan exceeds the fixed scratch of b2o_grad_stats_noalloc (too many chunks or slots)";
    default: return "unknown status";
  }
}

// Validates the table, fills chunk_begin / chunk_count / flags of every entry and, when `chunks`
// is not NULL, writes the chunks of `chunk_elems` elements (the last of a tensor shorter).
static int plan_walk(b2o_tensor* tensors, int32_t n_tensors, int32_t n_groups, int32_t n_slots,
                     int64_t chunk_elems, int32_t grad_dtype, b2o_chunk* chunks,
                     int64_t chunk_cap, int64_t* n_chunks) {
  if (!n_chunks || n_tensors < 0 || (n_tensors > 0 && !tensors)) return B2O_ERR_ARG;
  if (n_groups <= 0 || n_groups > B2O_MAX_GROUPS || n_slots < n_tensors) return B2O_ERR_ARG;
  if (grad_dtype != B2O_BF16 && grad_dtype != B2O_F32) return B2O_ERR_ARG;
  std::unordered_set<int32_t> seen;
  seen.reserve(size_t(n_tensors) * 2);
  int64_t total = 0;
  for (int32_t i = 0; i < n_tensors; ++i) {
    b2o_tensor& t = tensors[i];
    if (t.numel < 0) return B2O_ERR_TABLE;
    if (t.group < 0 || t.group >= n_groups) return B2O_ERR_TABLE;
    if (t.slot < 0 || t.slot >= n_slots) return B2O_ERR_TABLE;
    if (!seen.insert(t.slot).second) return B2O_ERR_TABLE;
    if (t.numel > 0 && (!t.grad || !t.master || !t.exp_avg || !t.exp_avg_sq)) return B2O_ERR_TABLE;
    const int64_t count = (t.numel + chunk_elems - 1) / chunk_elems;
    if (total + count > INT32_MAX) return B2O_ERR_CAPACITY;
    t.chunk_begin = int32_t(total);
    t.chunk_count = int32_t(count);
    const bool vec = aligned16(t.grad) && aligned16(t.master) && aligned16(t.exp_avg) &&
                     aligned16(t.exp_avg_sq) && (t.param == nullptr || aligned16(t.param));
    t.flags = vec ? B2O_FLAG_VECTOR : 0;
    t.reserved = 0;
    if (chunks) {
      if (total + count > chunk_cap) return B2O_ERR_CAPACITY;
      for (int64_t k = 0; k < count; ++k) {
        b2o_chunk& c = chunks[total + k];
        c.tensor = i;
        c.reserved = 0;
        c.begin = k * chunk_elems;
        const int64_t e = c.begin + chunk_elems;
        c.end = e < t.numel ? e : t.numel;
      }
    }
    total += count;
  }
  *n_chunks = total;
  return B2O_OK;
}

extern "C" int b2o_plan_chunks(b2o_tensor* tensors, int32_t n_tensors, int32_t n_groups,
                               int32_t n_slots, int64_t chunk_elems, int32_t grad_dtype,
                               b2o_chunk* chunks, int64_t chunk_cap, int64_t* n_chunks) {
  if (chunk_elems <= 0 || chunk_elems % B2O_VEC != 0 || chunk_elems > (int64_t(1) << 30))
    return B2O_ERR_ARG;
  return plan_walk(tensors, n_tensors, n_groups, n_slots, chunk_elems, grad_dtype, chunks,
                   chunk_cap, n_chunks);
}

extern "C" size_t b2o_workspace_bytes(int64_t n_chunks, int32_t n_slots) {
  if (n_chunks < 0 || n_slots < 0) return 0;
  return ws_counter_bytes() + size_t(n_chunks) * sizeof(double) +
         size_t(n_slots + 1) * sizeof(double);
}

extern "C" int b2o_workspace_init(void* workspace, size_t bytes, void* stream) {
  if (!workspace || bytes < ws_counter_bytes()) return B2O_ERR_ARG;
  return cudaMemsetAsync(workspace, 0, bytes, static_cast<cudaStream_t>(stream)) == cudaSuccess
             ? B2O_OK
             : B2O_ERR_CUDA;
}
