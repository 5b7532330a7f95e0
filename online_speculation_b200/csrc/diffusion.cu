// Block-diffusion remasking (one warp per sequence).
//
// A denoising step of block diffusion draws a token for every position of the
// current block, then keeps only the `tc` most confident still-masked positions
// (low-confidence remasking), a uniformly random subset (random remasking: the
// priorities are uniforms), or the earliest ones.  The unfused form is a chain of
// small tensor ops per step (mask test, masked fill, top-k, sort, gather, scatter,
// sum); here one warp owns a sequence: every lane holds up to eight positions,
// ranks them against the whole block through warp shuffles (rank = number of
// positions with a higher priority, or an equal one at a lower position), and the
// positions of rank < tc are committed, compacted in position order with a ballot
// prefix count, and their log-probabilities summed in double.
// Reference: src/inference_scaling/dllm/backends/llada.py:562-590 (per-row top-k
// selection of the transfer positions).
#include "common.cuh"
#include "diffusion.h"

namespace osb {
namespace {

constexpr int kPerLane = kRemaskMaxBlock / 32;

__global__ void __launch_bounds__(128) remask_select_kernel(RemaskArgs a) {
  pdl_wait();
  pdl_trigger();
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  if (row >= a.rows) return;
  long long* seq = a.tokens + static_cast<long long>(row) * a.ld_tokens + a.a0;
  const int chunks = (a.bl + 31) / 32;
  float pr[kPerLane];
  bool masked[kPerLane];
  int avail = 0;
#pragma unroll
  for (int k = 0; k < kPerLane; ++k) {
    const int i = lane + 32 * k;
    masked[k] = k < chunks && i < a.bl && seq[i] == a.mask_id;
    const float p = a.prio != nullptr ? (i < a.bl && k < chunks ? a.prio[row * a.bl + i] : 0.0f)
                                      : -static_cast<float>(i);
    pr[k] = masked[k] ? p : -INFINITY;
    avail += __popc(__ballot_sync(0xffffffffu, masked[k]));
  }
  int rank[kPerLane];
#pragma unroll
  for (int k = 0; k < kPerLane; ++k) rank[k] = 0;
  for (int kk = 0; kk < chunks; ++kk) {
    for (int src = 0; src < 32; ++src) {
      float other = 0.0f;
#pragma unroll
      for (int q = 0; q < kPerLane; ++q)
        if (q == kk) other = __shfl_sync(0xffffffffu, pr[q], src);
      const int j = src + 32 * kk;
      if (j >= a.bl) continue;
#pragma unroll
      for (int k = 0; k < kPerLane; ++k) {
        const int i = lane + 32 * k;
        if (other > pr[k] || (other == pr[k] && j < i)) ++rank[k];
      }
    }
  }
  double lp = 0.0;
  int before = 0;                                  // chosen positions in earlier chunks
#pragma unroll
  for (int k = 0; k < kPerLane; ++k) {
    if (k >= chunks) break;
    const int i = lane + 32 * k;
    const bool chosen = masked[k] && rank[k] < a.tc;
    const unsigned bits = __ballot_sync(0xffffffffu, chosen);
    if (chosen) {
      const int slot = before + __popc(bits & ((1u << lane) - 1u));
      const int tok = a.drawn[row * a.bl + i];
      seq[i] = tok;
      a.out_pos[static_cast<long long>(row) * a.out_ld + slot] = i + a.pos_offset;
      a.out_tok[static_cast<long long>(row) * a.out_ld + slot] = tok;
      if (a.logq != nullptr) lp += static_cast<double>(a.logq[row * a.bl + i]);
    }
    before += __popc(bits);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) lp += __shfl_xor_sync(0xffffffffu, lp, o);
  if (lane == 0 && a.logq != nullptr) {
    if (a.subset) {
      const double n = avail, t = a.tc;
      lp -= lgamma(n + 1.0) - lgamma(t + 1.0) - lgamma(n - t + 1.0);
    }
    if (a.step_lp) a.step_lp[row] = lp;
    if (a.traj) a.traj[row] += lp;
  }
}

}  // namespace

cudaError_t remask_select_launch(const RemaskArgs& a, cudaStream_t stream) {
  if (a.rows <= 0) return cudaSuccess;
  if (a.bl <= 0 || a.bl > kRemaskMaxBlock || a.tc < 0 || a.tc > a.bl || a.tokens == nullptr ||
      a.drawn == nullptr || a.out_pos == nullptr || a.out_tok == nullptr || a.out_ld < a.tc)
    return cudaErrorInvalidValue;
  const int blocks = (a.rows * 32 + 127) / 128;
  return launch_pdl(remask_select_kernel, dim3(blocks), dim3(128), 0, stream, a);
}

}  // namespace osb
