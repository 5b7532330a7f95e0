// Host API of the tcgen05 dense GEMM (see gemm.cu).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace osb {

struct GemmProblem {
  const __nv_bfloat16* w;  // [M, K] row-major weights (row stride ldw)
  long long ldw;
  const __nv_bfloat16* x;  // [N, K] row-major activations (row stride ldx)
  long long ldx;
  int M, N, K;
  void* out;               // [N, M] (or [N, M/2] for swiglu), row stride ldo
  long long ldo;
  int out_f32;
  const __nv_bfloat16* bias;      // [M] or null
  const __nv_bfloat16* residual;  // same layout as out (bf16) or null; may alias out
  long long ldr;
  int epilogue;                   // 0 linear, 1 swiglu on [64 gate | 64 up] row tiles, 2 row statistics
  // Row statistics (epilogue 2, the vocabulary head without stored logits): for every
  // token t and weight-row tile tm the kernel writes stat_part[t * tiles_m + tm] =
  // {max, sum exp(l - max), sum exp((l - max) * inv_temp[t]), 0} over the tile's rows,
  // and the tile that holds row targets[t] writes that logit to target_logit[t].
  // `out` is not written.  head_stats_merge_launch (sampling.h) folds the partials.
  const float* stat_inv_temp;     // [N] or null (T = 1)
  const int* stat_targets;        // [N] or null
  float* stat_part;               // [N, ceil(M / 128), 4]
  float* stat_target_logit;       // [N] or null
  int allow_split;
  int split_mode;                 // 0: split-K over a cluster (DSMEM reduction); 1: global workspace
  float* workspace;               // split-K partials
  long long workspace_floats;
  int* counters;                  // per-tile arrival counters, zero at rest
  int counter_slots;
  int* status;                    // bounded-wait error word
  int prefetch_weights;           // stream weight tiles before the predecessor kernel completes
                                  // (only where no kernel earlier in the stream writes w)
  // Grouped GEMM (e.g. MoE experts): w holds `groups` stacked [M, K] weights; the
  // tile list {group, tm, row0, row_end} (int4) and its length live in device memory,
  // so the row segments of each group may be data dependent.  group_bn fixes the token
  // tile (32/64/128/256) used to build the list.
  const int* group_tiles;
  const int* group_total;
  int groups;
  int group_tile_cap;
  int group_bn;
  // Tensor-parallel push (push_world > 0; bf16 output, no residual / SwiGLU): the output
  // tile goes to push_dst[q] (rank q's receive slot for this rank, row stride ldo) for
  // every rank q instead of `out`; when the whole grid is done, *push_epoch + 1 is
  // released (system scope) into push_flags[q] on every rank.  push_count is a device
  // arrival counter, zero at rest.
  int push_world;
  __nv_bfloat16* push_dst[8];
  uint32_t* push_flags[8];
  const uint32_t* push_epoch;
  unsigned int* push_count;
};

cudaError_t gemm_launch(const GemmProblem& p, cudaStream_t stream);
bool& pdl_enabled();   // programmatic dependent launch for the forward-path kernels

// Tile list of a grouped GEMM from group row offsets [groups + 1] (device): every
// group contributes ceil(rows / bn) x tiles_m tiles; *total receives the count.
cudaError_t grouped_tiles_launch(const int* offsets, int groups, int tiles_m, int bn, int* tiles, int cap, int* total,
                                 cudaStream_t stream);
int gemm_pick_bn(int tokens);

// The launcher's plan for a plain (non-grouped) problem: the token tile it uses and,
// when split-K partials go to a global workspace (split_mode 1), the split factor and
// the scratch that needs.  gemm_launch and every caller that sizes a workspace for it
// use this one function, so the sizes agree.
struct GemmPlan {
  int bn;                      // token tile (32 / 64 / 128 / 256)
  int tiles;                   // output tiles (128 weight rows x bn tokens)
  int splits;                  // split-K factor over the workspace (1: no split)
  int kb_per_split;            // 64-wide K blocks per split
  long long workspace_floats;  // fp32 partial tiles the split needs (0 without split)
};
int gemm_token_tile(int M, int N, int K);
GemmPlan gemm_workspace_plan(int M, int N, int K, int sms);
// Timeline capture for tuning: when non-null, every later launch writes 32 globaltimer
// slots per CTA (entry, setup, first TMA, first stage, last MMA, first accumulator,
// epilogue done, exit, then per-chunk and cluster-epilogue stamps) into this device
// buffer, which must hold grid x 32 values.
unsigned long long*& gemm_trace_buffer();

}  // namespace osb
