// Host API of the fused tensor-parallel all-reduce + residual add + RMSNorm.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace osb {

constexpr int kMaxRanks = 8;
// Flag slot (in units of kMaxRanks words of every signal pad) that the pushing
// row-parallel GEMMs release into; slots 0..3 belong to the pull collectives.
constexpr int kPushSlot = 4;

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
  int algorithm;                          // 0: one-shot up to four ranks, two-shot above; 1: one-shot; 2: two-shot
  unsigned long long wait_ns;             // limit of every cross-rank wait (0: two seconds)
  unsigned long long* trace;              // one-shot timeline of block 0 (tuning) or null
};

// Timeline capture for tuning the one-shot reduction: when non-null, block 0 of every
// later one-shot call writes 8 globaltimer stamps (entry, predecessor done, barrier
// published, barrier passed, partial rows loaded, norm reduced, output stored, call
// retired) over the previous call's, into this device buffer of at least 8 values.
unsigned long long*& allreduce_trace_buffer();

cudaError_t allreduce_add_rmsnorm_launch(const ArArgs& a, int blocks, cudaStream_t stream);

// Reduction of partials that the ranks' GEMMs pushed into this rank's memory
// (parts[q] = local receive slot of rank q): waits for every rank's completion
// flag in slot kPushSlot of this rank's pad, then h += sum_q parts[q] (rank
// order) and x = rmsnorm(h) * w in one pass over local memory.
cudaError_t allreduce_pushed_add_rmsnorm_launch(const ArArgs& a, int blocks, cudaStream_t stream);

}  // namespace osb
