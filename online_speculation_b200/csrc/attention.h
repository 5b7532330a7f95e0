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
  int tile_rows;                 // 64 (rows split across warps) or 16 / 32 (keys split across warps)
  __nv_bfloat16* out;            // [T, Hq, D]
  int Hq, Hkv, head_dim, page_size;
  int cache_pages;               // pages in k_cache / v_cache
  float scale;
  int* status;
};

cudaError_t attention_launch(const AttentionProblem& p, cudaStream_t stream);

}  // namespace osb
