// Host API of the data-parallel gradient reduce-scatter and parameter all-gather over
// symmetric peer memory (see dp.cu).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "comm.h"   // kMaxRanks

namespace osb {

// Signal-pad slots (units of kMaxRanks words of the gradient allocation's pads).
constexpr int kDpScatterSlot = 0;
constexpr int kDpGatherStartSlot = 1;
constexpr int kDpGatherDoneSlot = 2;

struct DpArgs {
  const float* grads[kMaxRanks];      // every rank's flat fp32 gradient buffer (symmetric, peer-mapped)
  __nv_bfloat16* params[kMaxRanks];   // every rank's flat bf16 parameter buffer (symmetric, peer-mapped)
  uint32_t* pads[kMaxRanks];          // every rank's signal pad (uint32 flags, symmetric)
  uint32_t* counters;                 // local [4]: scatter calls, scatter arrivals, gather calls, gather arrivals
  int rank, world;
  int* status;
  unsigned long long wait_ns;         // limit of every cross-rank wait (0: two seconds)
};

// shard[i] = scale * sum_q grads[q][lo + rank * n + i] for i < n, summed in rank order after a
// barrier that every rank enters once its own gradients of [lo, lo + world * n) are complete.
cudaError_t dp_reduce_scatter_launch(const DpArgs& a, long long lo, long long n, float* shard, float scale,
                                     cudaStream_t stream);

// params[q][lo + rank * n + i] = src[i] for every rank q and i < n (peer stores), after a barrier
// that every rank enters once it no longer reads its parameters, and before a closing barrier
// that holds the kernel until every rank's stores into this rank have landed.
cudaError_t dp_all_gather_launch(const DpArgs& a, const __nv_bfloat16* src, long long lo, long long n,
                                 cudaStream_t stream);

}  // namespace osb
