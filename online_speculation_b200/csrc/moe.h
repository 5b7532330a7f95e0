// Mixture-of-experts routing, dispatch and combine for the sm_100a MoE layer.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace osb {

// Softmax over E router logits per token, top-k selection (ties -> lower
// expert id), optional renormalisation of the k weights; counts[e] += tokens.
cudaError_t moe_route_launch(const float* logits, long long ld, int T, int E, int k, int renorm, int* topk_idx,
                             float* topk_w, int* counts, cudaStream_t stream);

// offsets[e] = sum of counts[< e] (offsets[E] = total), cursor[e] = offsets[e];
// counts are reset to zero for the next routing.
cudaError_t moe_offsets_launch(int* counts, int E, int* offsets, int* cursor, cudaStream_t stream);

// Copies token rows into expert-sorted order: slot = cursor[e]++ for each
// (token, choice); xp[slot] = x[token]; slot_of[token * k + j] = slot.
cudaError_t moe_dispatch_launch(const __nv_bfloat16* x, long long ldx, int T, int k, int H, const int* topk_idx,
                                int* cursor, __nv_bfloat16* xp, int* slot_of, cudaStream_t stream);

// h[t] (+)= sum_j w[t, j] * y[slot_of[t, j]]  (fp32 accumulation in choice order).
cudaError_t moe_combine_launch(const __nv_bfloat16* y, long long ldy, const int* slot_of, const float* topk_w, int T,
                               int k, int H, __nv_bfloat16* h, long long ldh, int accumulate, cudaStream_t stream);

}  // namespace osb
