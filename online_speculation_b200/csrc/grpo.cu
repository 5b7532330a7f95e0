// Fused GRPO loss: clipped-ratio objective, k3 KL penalty, masked means, metrics and the
// gradient with respect to the policy log-probabilities, in one launch.
//
// Reference objective: the TRL GRPO loss used by experiments/arllm/train_gsm8k_grpo.py
// (per token min(r A, clip(r, 1 - eps, 1 + eps) A) - beta (exp(ref - lp) - (ref - lp) - 1),
// r = exp(lp - old); token mean per sequence, then the mean over sequences, negated).
//
// One block per sequence.  The block first counts the sequence's completion tokens, then
// visits every token once: it accumulates the objective, the KL term and the clipped flag,
// and writes dLoss/dlp = -(1 / B) m / n (dobj - beta (1 - exp(ref - lp))) directly, where
// dobj = r A when the unclipped term is the minimum (the two terms tie inside the clip
// range) and 0 when the clipped term is strictly smaller (the clamp is flat there).  Each
// block stores its row statistics; the last block to arrive (arrival counter) folds the
// rows in sequence order -- a deterministic reduction -- into the loss and the metrics,
// and resets the counter for the next launch.
#include "common.cuh"
#include "grpo.h"

namespace osb {
namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  __syncthreads();                       // red may still be read by a previous reduction
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float s = lane < kThreads / 32 ? red[lane] : 0.0f;
  return warp_sum(s);
}

__global__ void __launch_bounds__(kThreads) grpo_loss_kernel(GrpoLossArgs a) {
  __shared__ float red[kThreads / 32];
  __shared__ bool last;
  const int b = blockIdx.x;
  const long long row = static_cast<long long>(b) * a.C;
  float n = 0.0f;
  for (int t = threadIdx.x; t < a.C; t += kThreads) n += a.mask[row + t] ? 1.0f : 0.0f;
  n = block_sum(n, red);
  const float adv = a.adv[b];
  const float scale = -1.0f / (static_cast<float>(a.B) * fmaxf(n, 1.0f));
  float obj_sum = 0.0f, kl_sum = 0.0f, clip_sum = 0.0f;
  for (int t = threadIdx.x; t < a.C; t += kThreads) {
    const long long i = row + t;
    if (!a.mask[i]) {
      a.grad[i] = 0.0f;
      continue;
    }
    const float lp = a.logp[i];
    const float r = expf(lp - a.old_logp[i]);
    const float plain = r * adv;
    const float clipped = fminf(fmaxf(r, 1.0f - a.eps), 1.0f + a.eps) * adv;
    const float obj = fminf(plain, clipped);
    const float dobj = plain <= clipped ? plain : 0.0f;
    const float d = a.ref_logp[i] - lp;
    const float e = expf(d);
    const float kl = e - d - 1.0f;
    obj_sum += obj - a.beta * kl;
    kl_sum += kl;
    clip_sum += fabsf(r - 1.0f) > a.eps ? 1.0f : 0.0f;
    a.grad[i] = scale * (dobj - a.beta * (1.0f - e));
  }
  obj_sum = block_sum(obj_sum, red);
  kl_sum = block_sum(kl_sum, red);
  clip_sum = block_sum(clip_sum, red);
  if (threadIdx.x == 0) {
    float4* rs = reinterpret_cast<float4*>(a.row_stats) + b;
    *rs = make_float4(obj_sum / fmaxf(n, 1.0f), n, kl_sum, clip_sum);
    __threadfence();
    last = atomicAdd(a.counter, 1u) == static_cast<unsigned>(a.B - 1);
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  if (threadIdx.x == 0) {
    // sequence order: the same sums on every launch
    double per_seq = 0.0, tokens = 0.0, kl = 0.0, clip = 0.0;
    const volatile float4* rs = reinterpret_cast<const volatile float4*>(a.row_stats);
    for (int s = 0; s < a.B; ++s) {
      const float x = rs[s].x, y = rs[s].y, z = rs[s].z, w = rs[s].w;
      per_seq += x;
      tokens += y;
      kl += z;
      clip += w;
    }
    const double denom = tokens > 0.0 ? tokens : 1.0;
    a.out[0] = static_cast<float>(-per_seq / a.B);
    a.out[1] = static_cast<float>(kl / denom);
    a.out[2] = static_cast<float>(clip / denom);
    *a.counter = 0u;
  }
}

}  // namespace

cudaError_t grpo_loss_launch(const GrpoLossArgs& a, cudaStream_t stream) {
  if (a.B <= 0 || a.C <= 0) return cudaErrorInvalidValue;
  grpo_loss_kernel<<<a.B, kThreads, 0, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace osb
