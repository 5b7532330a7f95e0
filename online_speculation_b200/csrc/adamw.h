// Host API of the fused AdamW step (see adamw.cu).
#pragma once
#include <algorithm>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace osb {

struct AdamWArgs {
  float* params;
  const float* grads;
  float* exp_avg;
  float* exp_avg_sq;
  __nv_bfloat16* publish;   // bf16 execution copy or null
  long long n;
  const float* sq_norm;     // squared global grad norm (device) or null: no clipping
  float clip;
  float lr, beta1, beta2, eps, weight_decay;
  float bias_correction1, bias_correction2;
  int* nonfinite;           // set to 1 when the norm is not finite (step skipped)
  const int* step_ptr;      // device step counter (>= 1) for the bias corrections, or null
};

cudaError_t grad_sq_norm_launch(const float* g, long long n, float* out, cudaStream_t stream);
cudaError_t adamw_launch(const AdamWArgs& a, cudaStream_t stream);

}  // namespace osb
