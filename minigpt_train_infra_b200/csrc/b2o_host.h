// Host-side helpers shared by the launch wrappers.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace b2o {

// Number of CTAs of `kernel` (launched with `threads` threads, no dynamic shared memory) that
// are resident at once on the current device: SM count x occupancy, cached per kernel/device.
// Returns <= 0 if the device cannot be queried.
int resident_ctas(const void* kernel, int threads);

// Grid for a pass over `n_chunks` chunks: one wave of resident CTAs, fewer when there are fewer
// chunks, and at least one CTA so the completion ticket always runs.
inline int stream_grid(const void* kernel, int threads, int64_t n_chunks) {
  const int wave = resident_ctas(kernel, threads);
  if (wave <= 0) return wave;
  const int64_t g = n_chunks < wave ? n_chunks : wave;
  return g < 1 ? 1 : int(g);
}

}  // namespace b2o
