// Host API of the masked-diffusion denoising kernels.
#pragma once
#include <cuda_runtime.h>

namespace osb {

// One remasking step of block diffusion for every sequence of a batch: among the
// still-masked positions of the current block, choose the `tc` with the highest
// priority (ties: lower position first), commit their drawn tokens, and record the
// chosen positions in increasing order with their tokens and the step's log density.
struct RemaskArgs {
  long long* tokens;          // [rows, ld_tokens] int64 sequences (updated in place)
  long long ld_tokens;
  int a0;                     // first position of the block
  int bl;                     // block length (<= kRemaskMaxBlock)
  long long mask_id;
  const int* drawn;           // [rows * bl] drawn token per block position
  const float* prio;          // [rows * bl] priorities, or null: earliest position first
  const float* logq;          // [rows * bl] log-probability of each drawn token, or null (no density)
  int tc;                     // positions committed this step
  int rows;
  int subset;                 // add log 1 / C(masked, tc) (uniformly random subsets)
  double* traj;               // [rows] running log density (accumulated) or null
  double* step_lp;            // [rows] this step's log density or null
  long long* out_pos;         // [rows, out_ld] chosen positions + pos_offset, increasing
  long long* out_tok;         // [rows, out_ld] chosen tokens
  long long out_ld;
  long long pos_offset;
};

constexpr int kRemaskMaxBlock = 256;

cudaError_t remask_select_launch(const RemaskArgs& a, cudaStream_t stream);

}  // namespace osb
