// Fused AdamW over flat fp32 master buffers with on-device gradient clipping.
//
// Reference: the online suffix learner's fused torch AdamW with clip_grad_norm_
// (online-speculation/src/blockspec/parallel/online.py:65-66,141-157) and the
// trainers' `adamw_torch_fused`.  All trainable tensors of a learner live in
// one flat fp32 master buffer (with flat grads and moments), so one launch
// computes the global L2 norm, a second applies clip + AdamW and publishes the
// bf16 execution copy, with no host synchronisation in between.
#include "adamw.h"
#include "common.cuh"

namespace osb {
namespace {

__global__ void sq_norm_kernel(const float* __restrict__ g, long long n, float* __restrict__ out) {
  float s = 0.0f;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const float v = g[i];
    s += v * v;
  }
  s = warp_sum(s);
  __shared__ float red[32];
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (lane == 0) red[warp] = s;
  __syncthreads();
  if (warp == 0) {
    s = lane < blockDim.x / 32 ? red[lane] : 0.0f;
    s = warp_sum(s);
    if (lane == 0) atomicAdd(out, s);
  }
}

__global__ void adamw_kernel(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
                             float* __restrict__ v, __nv_bfloat16* __restrict__ publish, long long n,
                             const float* __restrict__ sq_norm, float clip, float lr, float beta1, float beta2,
                             float eps, float weight_decay, float bc1, float bc2, int* __restrict__ nonfinite,
                             const int* __restrict__ step_ptr) {
  if (step_ptr) {
    // bias corrections from the device-side step counter (graph-replayable)
    const float t = static_cast<float>(*step_ptr);
    bc1 = 1.0f - powf(beta1, t);
    bc2 = 1.0f - powf(beta2, t);
  }
  float scale = 1.0f;
  if (sq_norm) {
    const float norm = sqrtf(*sq_norm);
    if (!isfinite(norm)) {
      if (blockIdx.x == 0 && threadIdx.x == 0 && nonfinite) *nonfinite = 1;
      return;
    }
    if (clip > 0.0f) scale = fminf(1.0f, clip / (norm + 1e-6f));
  }
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const float gi = g[i] * scale;
    float pi = p[i];
    pi *= 1.0f - lr * weight_decay;
    const float mi = beta1 * m[i] + (1.0f - beta1) * gi;
    const float vi = beta2 * v[i] + (1.0f - beta2) * gi * gi;
    m[i] = mi;
    v[i] = vi;
    const float denom = sqrtf(vi / bc2) + eps;
    pi -= lr * (mi / bc1) / denom;
    p[i] = pi;
    if (publish) publish[i] = f2bf(pi);
  }
}

}  // namespace

cudaError_t grad_sq_norm_launch(const float* g, long long n, float* out, cudaStream_t stream) {
  cudaError_t e = cudaMemsetAsync(out, 0, sizeof(float), stream);
  if (e != cudaSuccess) return e;
  if (n <= 0) return cudaSuccess;
  const int blocks = static_cast<int>(std::min<long long>(1184, (n + 255) / 256));
  sq_norm_kernel<<<blocks, 256, 0, stream>>>(g, n, out);
  return cudaGetLastError();
}

cudaError_t adamw_launch(const AdamWArgs& a, cudaStream_t stream) {
  if (a.n <= 0) return cudaSuccess;
  const int blocks = static_cast<int>(std::min<long long>(1184, (a.n + 255) / 256));
  adamw_kernel<<<blocks, 256, 0, stream>>>(a.params, a.grads, a.exp_avg, a.exp_avg_sq, a.publish, a.n, a.sq_norm,
                                           a.clip, a.lr, a.beta1, a.beta2, a.eps, a.weight_decay, a.bias_correction1,
                                           a.bias_correction2, a.nonfinite, a.step_ptr);
  return cudaGetLastError();
}

}  // namespace osb
