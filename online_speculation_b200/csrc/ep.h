// Host API of the expert-parallel MoE exchange over NVLink peer memory.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace osb {

constexpr int kEpMaxRanks = 8;
constexpr int kEpMaxExperts = 256;

struct EpArgs {
  int world, rank, E, E_local, k, T, H;
  int* tables[kEpMaxRanks];               // every rank's routing-count table [world][E] int32 (symmetric)
  __nv_bfloat16* recv_x[kEpMaxRanks];     // every rank's receive buffer [R_max, H] (symmetric)
  __nv_bfloat16* recv_y[kEpMaxRanks];     // every rank's expert-output buffer [R_max, H] (symmetric)
  uint32_t* pads[kEpMaxRanks];            // every rank's signal pad (symmetric)
  uint32_t* epoch;                        // local [2]: completed-call counter, block arrival counter
  long long r_max;                        // rows of every receive buffer
  const int* counts;                      // local [E]: this rank's (token, choice) count per expert
  const int* topk_idx;                    // local [T * k]
  const float* topk_w;                    // local [T * k]
  const __nv_bfloat16* x;                 // local tokens [T, H] (row stride ldx)
  long long ldx;
  int* cursor;                            // local scratch [E], zero on entry (left zero on exit)
  int* slot_of;                           // local [T * k]: row of every (token, choice) in its owner's buffer
  int* local_offsets;                     // local [E_local + 1]: received rows per local expert (prefix sums)
  __nv_bfloat16* h;                       // local residual [T, H] (row stride ldh), combine adds into it
  long long ldh;
  int* status;
  unsigned long long wait_ns;             // limit of every cross-rank wait (0: two seconds)
};

// Exchange routing counts, then copy every (token, choice) row into the receive
// buffer of the expert's owner (peer stores); returns once every rank's rows for
// this rank have landed.  Writes slot_of and local_offsets.
cudaError_t ep_dispatch_launch(const EpArgs& a, int blocks, cudaStream_t stream);

// After every owner ran its experts into recv_y: h[t] += sum_j w[t, j] * y_owner[slot_of[t, j]]
// (peer loads, fp32 accumulation in choice order).
cudaError_t ep_combine_launch(const EpArgs& a, int blocks, cudaStream_t stream);

}  // namespace osb
