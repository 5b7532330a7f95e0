// Host API of the sampling / scoring / speculative-correction kernels.
#pragma once
#include <cuda_runtime.h>

namespace osb {

struct SampleArgs {
  const float* logits;  // [rows, V] row stride ld
  long long ld;
  int V;
  const float* inv_temp;      // [rows] or null (T = 1)
  const double* uniforms;     // uniforms[r * uniform_stride]
  long long uniform_stride;
  int* tokens;                // [rows]
  float* logq;                // [rows] policy log-prob or null
  float* logp;                // [rows] T=1 log-prob or null
  // Arithmetic-coding rows (arith[r] != 0): the uniform u of the row is a code
  // point; after drawing token t with cumulative mass [c, c + q_t) it writes
  // the rescaled point (u - c) / q_t to next_uniforms[r * uniform_stride].
  const int* arith;           // [rows] or null
  double* next_uniforms;      // or null
  // Truncated policies (either may be null): top_k[r] > 0 keeps the k largest
  // tempered logits (ties at the k-th kept), top_p[r] < 1 then keeps the
  // smallest descending prefix of that set whose mass exceeds top_p[r].
  const int* top_k;
  const float* top_p;
};

struct RowStatsArgs {
  const float* logits;
  long long ld;
  int V;
  const float* inv_temp;
  const int* targets;         // [rows] or null
  float* lse1;
  float* lseT;
  float* logp;
  float* logq;
  // Truncated policies as in SampleArgs: logq and lseT are taken over the kept
  // columns (a target outside them gets -inf); rows are not split.
  const int* top_k;
  const float* top_p;
  // Split rows (set by the launcher): `split` CTAs per row over `chunk` columns each;
  // partial (max, sum exp, sum exp at 1/T) go to part[row][chunk][3] and the last CTA
  // of a row to arrive (count[row]) merges them and resets its counter (zero at rest).
  int split;
  int chunk;
  float* part;
  int* count;
};

// Rows up to this count may be split across at most kRowStatsMaxSplit CTAs each.
constexpr int kRowStatsSplitRows = 4096;
constexpr int kRowStatsMaxSplit = 16;

// Rows up to this count may be split across CTAs (the scratch holds one word per row).
constexpr int kGumbelSplitRows = 4096;

struct GumbelArgs {
  const float* logits;
  long long ld;
  int V;
  const float* inv_temp;
  const unsigned long long* seeds;  // per sequence
  const int* seed_index;            // [rows] -> sequence, or null (row = sequence)
  const int* streams;               // [rows] per-draw counters (e.g. round index), or null
  const int* row_in_seq;            // [rows] or null
  int salt;
  int* tokens;
  // Vocabulary-parallel mode: the rows hold columns [v_lo, v_lo + V) of the
  // full vocabulary.  Noise is keyed by the global column, and with `keys` set
  // the kernel writes the packed (score, global column) key of its local best
  // instead of a token; the maximum key over ranks is the global draw.
  int v_lo;
  unsigned long long* keys;
  // Split rows (set by the launcher): `split` CTAs per row, `chunk` columns each (a
  // multiple of 4).  With split > 1 every CTA folds its key into row_best[r]
  // (unsigned maximum) and the last to arrive (row_count[r]) writes the result and
  // resets both words; the buffers are zero at rest.
  int split;
  int chunk;
  unsigned long long* row_best;
  int* row_count;
};

struct SpecArgs {
  const float* target;        // [B * (n + 1), V]
  long long ld_target;
  const float* draft;         // [B * n, V]
  long long ld_draft;
  const int* candidates;      // [B, n]
  int n, V;
  const float* inv_temp;      // [B] or null
  const unsigned long long* seeds;  // [B]
  const int* streams;         // [B] round counters or null
  int salt;
  int* count;                 // [B]
  int* tail;                  // [B]
  int* valid;                 // [B]
  int* emitted;               // [B, n + 1]
  float* logq;                // [B, n + 1]
  float* logp;                // [B, n + 1]
  // optional precomputed row statistics (row_stats_kernel); null = computed in-kernel
  const float* lseT_target;   // [B * (n + 1)]
  const float* lse1_target;   // [B * (n + 1)]
  const float* lseT_draft;    // [B * n]
  // Vocabulary-parallel mode (see GumbelArgs): the rows hold columns
  // [v_lo, v_lo + V) of V_total; cand_logits [B, n, 2] carries the global
  // (target, draft) logits of every candidate; the kernel writes count / valid
  // and the packed key of its local tail draw to `keys`; the caller reduces the
  // keys across ranks and finishes the outputs.
  int v_lo, V_total;
  const float* cand_logits;
  unsigned long long* keys;
};

// Fold the per-tile partials of a row-statistics head GEMM (GemmProblem epilogue 2)
// into lse at T = 1 and at T and the target log-probabilities (one warp per row).
struct HeadStatsArgs {
  const float* part;          // [rows, tiles, 4] {max, sum exp, sum exp at 1/T, -}
  int tiles;
  int rows;
  int V;
  const float* inv_temp;      // [rows] or null
  const int* targets;         // [rows] or null
  const float* target_logit;  // [rows] (written by the GEMM for in-range targets)
  float* lse1;                // each output may be null
  float* lseT;
  float* logp;
  float* logq;
};
cudaError_t head_stats_merge_launch(const HeadStatsArgs& a, cudaStream_t stream);

cudaError_t sample_launch(const SampleArgs& a, int rows, cudaStream_t stream);
cudaError_t row_stats_launch(const RowStatsArgs& a, int rows, cudaStream_t stream);
cudaError_t gumbel_sample_launch(const GumbelArgs& a, int rows, cudaStream_t stream);
cudaError_t spec_verify_launch(const SpecArgs& a, int batch, cudaStream_t stream);

}  // namespace osb

#include <cuda_bf16.h>
namespace osb {
cudaError_t divergence_stats_launch(const float* s, const float* t, long long ld_s, long long ld_t, int rows, int V,
                                    float* out, cudaStream_t stream);
cudaError_t divergence_loss_launch(const float* s, const float* t, long long ld_s, long long ld_t, int rows, int V,
                                   const float* lse, int kind, float* out, cudaStream_t stream);
cudaError_t divergence_grad_launch(const float* s, const float* t, long long ld_s, long long ld_t, int rows, int V,
                                   const float* lse, const float* pieces, const float* w, int kind,
                                   __nv_bfloat16* grad, long long ld_g, cudaStream_t stream);
}  // namespace osb
namespace osb {
cudaError_t logprob_grad_launch(const float* logits, long long ld, int rows, int V, const float* lse,
                                const int* targets, const float* w, void* grad, bool grad_bf16, long long ldg,
                                cudaStream_t stream);
// Per row: [target log p at T, sum p log p, mean_v log p, -(mean of the top-K log p)]  (out: [rows, 4]).
cudaError_t score_stats_launch(const float* logits, long long ld, int rows, int V, const float* inv_temp,
                               const int* targets, int topk, float* out, cudaStream_t stream);

}  // namespace osb
