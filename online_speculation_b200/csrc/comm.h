// Host API of the fused tensor-parallel all-reduce + residual add + RMSNorm.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace osb {

constexpr int kMaxRanks = 8;

struct ArArgs {
  const __nv_bfloat16* parts[kMaxRanks];  // every rank's partial sums [T, H] (symmetric, peer-mapped)
  __nv_bfloat16* rows[kMaxRanks];         // every rank's reduced-rows buffer [T, H] (symmetric)
  uint32_t* pads[kMaxRanks];              // every rank's signal pad (uint32 flags, symmetric)
  uint32_t* epoch;                        // local [4]: completed-call counter, two block arrival counters
  __nv_bfloat16* h;                       // local residual stream [T, H] (row stride ldh)
  long long ldh;
  const __nv_bfloat16* w;                 // RMSNorm weight [H]
  __nv_bfloat16* x;                       // normalised output [T, H] (row stride ldx)
  long long ldx;
  int T, H, rank, world;
  float eps;
  int* status;
};

cudaError_t allreduce_add_rmsnorm_launch(const ArArgs& a, int blocks, cudaStream_t stream);

}  // namespace osb
