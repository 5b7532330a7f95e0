// Host API of the paged attention kernel (see attention.cu).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace osb {

struct AttentionProblem {
  const __nv_bfloat16* q;        // [T, Hq, D]
  const __nv_bfloat16* k_cache;  // [pages, Hkv, P, D]
  const __nv_bfloat16* v_cache;
  const int* table;              // [B, table_stride]
  int table_stride;
  const int* q_start;            // [B]
  const int* q_len;              // [B]
  const int* kv_len;             // [B]
  const int* mode;               // [B] 0 causal, 1 bidirectional
  const int* tile_seq;           // [num_tiles]
  const int* tile_row0;          // [num_tiles]
  int num_tiles;
  int tile_rows;                 // 128: tcgen05 kernel; 64 / 16 / 32: mma.sync kernels (rows / keys split across warps)
  int kv_splits;                 // tcgen05 kernel: key ranges per tile, merged within a cluster (1, 2, 4, 8)
  __nv_bfloat16* out;            // [T, Hq, D]
  int Hq, Hkv, head_dim, page_size;
  int cache_pages;               // pages in k_cache / v_cache
  float scale;
  int* status;
  // Two-pass attention over a shared key prefix (tile_rows 16 / 32 only; each may be null):
  // keys [k_lo[b], kv_len[b]) only; fp32 output and/or the log2-domain log-sum-exp of the
  // range; and an earlier range's normalised output and log-sum-exp merged into the result.
  const int* k_lo;
  float* o_f32;
  float* lse_out;
  const float* prior_o;
  const float* prior_lse;
};

cudaError_t attention_launch(const AttentionProblem& p, cudaStream_t stream);

// Timeline capture for tuning the tcgen05 kernel: when non-null, its first 8 CTAs
// write 128 globaltimer stamps each (entry, set-up, and per key chunk the producer's
// issue, the S product's issue, P's arrival at the MMA issuer, S and P as seen by the
// first softmax warp) into this device buffer of at least 1024 values.
unsigned long long*& attention_trace_buffer();

}  // namespace osb
