// Loss-scale update of the mixed-precision step (one thread, no host synchronisation).
//
// Replaces torch._amp_update_scale_, issued by GradScaler.update (torch/amp/grad_scaler.py:549):
// back off on a step whose gradients held an inf/NaN, otherwise count clean steps and grow the
// scale every `growth_interval` of them.  The product scale*factor is formed in double and
// stored as fp32, and a grown scale is kept only when it is finite.
#include <cuda_runtime.h>

#include "b200_optim.h"

namespace b2o {

__global__ void scaler_update_kernel(float* scale, int32_t* tracker, const float* found_inf,
                                     double growth, double backoff, int32_t interval) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  if (*found_inf != 0.0f) {
    *scale = (float)__dmul_rn((double)*scale, backoff);
    *tracker = 0;
    return;
  }
  const int32_t successful = *tracker + 1;
  if (successful == interval) {
    const float grown = (float)__dmul_rn((double)*scale, growth);
    if (isfinite(grown)) *scale = grown;
    *tracker = 0;
  } else {
    *tracker = successful;
  }
}

}  // namespace b2o

extern "C" int b2o_scaler_update(float* scale, int32_t* growth_tracker, const float* found_inf,
                                 double growth_factor, double backoff_factor,
                                 int32_t growth_interval, void* stream) {
  if (!scale || !growth_tracker || !found_inf || growth_interval <= 0) return B2O_ERR_ARG;
  b2o::scaler_update_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      scale, growth_tracker, found_inf, growth_factor, backoff_factor, growth_interval);
  return cudaGetLastError() == cudaSuccess ? B2O_OK : B2O_ERR_LAUNCH;
}
