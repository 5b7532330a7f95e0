// Host API of the fused GRPO loss (see grpo.cu).
#pragma once
#include <cuda_runtime.h>

namespace osb {

struct GrpoLossArgs {
  const float* logp;          // [B, C] policy log-probabilities of the completion tokens
  const float* old_logp;      // [B, C] behaviour (rollout-time) log-probabilities
  const float* ref_logp;      // [B, C] frozen reference log-probabilities
  const float* adv;           // [B] group advantages
  const unsigned char* mask;  // [B, C] 1 for completion tokens, 0 for padding
  int B, C;
  float beta, eps;
  float* grad;                // [B, C] dLoss / dlogp
  float* row_stats;           // [B, 4] per sequence: masked token-mean objective, tokens, KL sum, clipped tokens
  float* out;                 // [3]: loss, token-mean KL, clipped-token fraction
  unsigned int* counter;      // arrival counter, zero between launches (the last block resets it)
};

cudaError_t grpo_loss_launch(const GrpoLossArgs& a, cudaStream_t stream);

}  // namespace osb
