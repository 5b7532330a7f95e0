// Dense linear layers on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// Computes out[t, f] = sum_k X[t, k] * W[f, k]  (+ bias[f]) (+ residual[t, f])
// for every linear layer of the decoders: QKV / O / gate-up / down / lm_head.
// Replaces the cuBLAS `nn.Linear` calls of the reference
// (online-speculation/src/blockspec/parallel/backbone.py:93-96,157-159,201 and the
// HF Qwen2 model driven by src/inference_scaling/arllm/backends/transformers_backend.py).
//
// Design (B200-first):
//  * The weight matrix is the MMA "A" operand (M = 128 output features per tile)
//    and the token activations are the "B" operand (N = BN tokens per tile).
//    Decode batches (16..256 tokens) then map to a single N tile while the
//    128-row weight tiles stream through a deep TMA pipeline: the kernel runs
//    at HBM speed for skinny decode GEMMs and at tensor-core speed for prefill.
//  * Persistent grid (one CTA per SM), warp-specialised: warp 0 issues TMA,
//    warp 1 owns TMEM and issues tcgen05.mma from one elected lane, warps 2-5
//    drain the double-buffered fp32 accumulators with tcgen05.ld, so the
//    epilogue of one tile overlaps the main loop of the next.
//  * Split-K over the reduction dimension when there are too few tiles to fill
//    148 SMs (every decode GEMM).  Partial tiles go to an fp32 workspace; the
//    last split to finish (per-tile arrival counter, reset by that split) sums
//    them and runs the epilogue.  No CTA ever waits on another one.
//  * Epilogues: bias, residual add (in-place hidden += ...), SwiGLU of an
//    interleaved gate/up weight ([64 gate rows | 64 up rows] per tile), fp32 or
//    bf16 output; or row statistics (per-tile max / sum exp at T = 1 and at 1/T
//    plus the target logit) for vocabulary-head scoring without storing logits.
//  * TMA loads are plain tiled loads (no cluster multicast).
#include "common.cuh"
#include "gemm.h"

#include <algorithm>
#include <cstdio>
#include <mutex>

namespace osb {

namespace {

constexpr int kBM = 128;   // weight rows per tile (MMA M)
constexpr int kBK = 64;    // reduction elements per stage: one 128-byte swizzle row
constexpr int kUmmaK = 16; // K per tcgen05.mma for 16-bit inputs
constexpr int kEpiGroups = 2;                      // epilogue warpgroups, alternating 32-token chunks
constexpr int kThreads = 64 + 128 * kEpiGroups;
constexpr int kPushMaxRanks = 8;
constexpr int kMaxClusterSplit = 8;                // portable thread-block cluster size

struct Args {
  int M, N, K;          // M = weight rows (features), N = tokens
  int k_blocks;
  int tiles_m, tiles_n, splits, kb_per_split;
  void* out;
  long long ldo;
  const __nv_bfloat16* residual;
  long long ldr;
  const __nv_bfloat16* bias;
  int epilogue;         // 0 linear, 1 swiglu, 2 row statistics (no output tile)
  const float* stat_inv_temp;
  const int* stat_targets;
  float4* stat_part;
  float* stat_target_logit;
  int out_f32;
  int vec_ok;           // output / residual rows are 16-byte aligned
  int cluster;          // >1: split-K over a thread-block cluster, reduced through DSMEM
  float* workspace;
  int* counters;
  int* status;
  int prefetch_a;       // issue the first stages' weight tiles before griddepcontrol.wait
  // Grouped mode (gtiles != null): tile w is gtiles[w] = {group, tm, row0, row_end}; the
  // weight rows of group g start at g * M; the tile count is *gtotal (device memory).
  const int4* gtiles;
  const int* gtotal;
  // Optional timeline (null in normal runs): per CTA kTraceSlots globaltimer stamps.
  unsigned long long* trace;
  // Tensor-parallel push (push_world > 0): the bf16 output tile is stored to every
  // rank's receive slot for this rank (peer memory, row stride ldo) instead of `out`,
  // and the last CTA to finish publishes *push_epoch + 1 to every rank's flag word.
  int push_world;
  __nv_bfloat16* push_dst[kPushMaxRanks];
  uint32_t* push_flags[kPushMaxRanks];
  const uint32_t* push_epoch;
  unsigned int* push_count;
};

__device__ __forceinline__ void put_bf16x8(const Args& a, long long off, const uint4& pk) {
  if (a.push_world == 0) {
    *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(a.out) + off) = pk;
    return;
  }
  for (int q = 0; q < a.push_world; ++q) *reinterpret_cast<uint4*>(a.push_dst[q] + off) = pk;
}

__device__ __forceinline__ void put_bf16(const Args& a, long long off, float v) {
  const __nv_bfloat16 b = f2bf(v);
  if (a.push_world == 0) {
    static_cast<__nv_bfloat16*>(a.out)[off] = b;
    return;
  }
  for (int q = 0; q < a.push_world; ++q) a.push_dst[q][off] = b;
}

// Timeline slots: 0 entry, 1 setup done, 2 first TMA issued, 3 first stage landed,
// 4 last MMA committed, 5 first accumulator ready, 7 exit; 8..23 the loaded /
// finished stamps of the 32-token chunks of the CTA's last tile; 24 cluster
// partial staged, 25 cluster synchronised, 26 cluster reduction stored.
constexpr int kTraceSlots = 32;
__device__ __forceinline__ void trace_stamp(const Args& a, int slot) {
  if (a.trace != nullptr) a.trace[blockIdx.x * kTraceSlots + slot] = global_ns();
}

struct TileCoord {
  int split, tile, tm, arow, row0, row_end;
};

template <int BN>
__device__ __forceinline__ TileCoord tile_coord(const Args& a, int w) {
  TileCoord c;
  if (a.gtiles != nullptr) {
    const int4 t = a.gtiles[w];
    c.split = 0;
    c.tile = w;
    c.tm = t.y;
    c.arow = t.x * a.M + t.y * kBM;
    c.row0 = t.z;
    c.row_end = t.w;
  } else {
    c.split = w % a.splits;
    c.tile = w / a.splits;
    c.tm = c.tile % a.tiles_m;
    c.arow = c.tm * kBM;
    c.row0 = (c.tile / a.tiles_m) * BN;
    c.row_end = a.N;
  }
  return c;
}

template <int BN>
struct Smem {
  static constexpr int kStages = BN <= 32 ? 9 : BN <= 64 ? 8 : BN <= 128 ? 6 : 4;
  static constexpr int kABytes = kBM * kBK * 2;
  static constexpr int kBBytes = BN * kBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kTmemCols = 2 * BN < 32 ? 32 : 2 * BN;
  static constexpr int kXchgBytes = kEpiGroups * 32 * (kBM + 4) * 4;   // one transpose buffer per group
  static constexpr int kBarBytes = 256;
  static constexpr int kTotal = 1024 + kStages * kStageBytes + kBarBytes + kXchgBytes;
};

// Epilogue of one 32-token chunk.  Every epilogue thread owns one accumulator
// row r (an output feature) and holds its 32 token values in v.  The chunk is
// transposed through shared memory (stage[j][r], fp32) so that the global
// writes -- and the residual reads -- are 16-byte vectors along the feature
// dimension, issued in batches (the residual may alias the output, so loads
// are grouped ahead of the stores instead of alternating with them).
template <int BN>
__device__ __forceinline__ void finish_chunk(const Args& a, const float (&v)[32], int tm, int row0, int row_end,
                                             int chunk, int r, float* stage, int ep_tid, int bar) {
  const int t0 = row0 + chunk * 32;
  const bool swiglu = a.epilogue == 1;
  const int f0 = swiglu ? tm * 64 : tm * kBM;       // first output feature of this tile
  const int out_cols = swiglu ? a.M / 2 : a.M;      // output row width (valid features)
  const int width = swiglu ? 64 : kBM;              // features produced by this tile
  const float b = (!swiglu && a.bias && tm * kBM + r < a.M) ? bf2f(a.bias[tm * kBM + r]) : 0.0f;
#pragma unroll
  for (int j = 0; j < 32; ++j) stage[j * (kBM + 4) + r] = v[j] + b;
  named_barrier(bar, 128);
  const int valid_t = min(32, row_end - t0);
  if (a.vec_ok) {
    // vectors of 8 features; width/8 vectors per token row
    constexpr int kMaxIter = (32 * kBM / 8 + 127) / 128;  // 4
    const int vec_per_row = width / 8;
    const int total = 32 * vec_per_row;
    float res[kMaxIter][8];
    int tv[kMaxIter], fv[kMaxIter];
#pragma unroll
    for (int it = 0; it < kMaxIter; ++it) {
      const int idx = ep_tid + it * 128;
      tv[it] = idx / vec_per_row;
      fv[it] = (idx % vec_per_row) * 8;
      const bool ok = idx < total && tv[it] < valid_t && f0 + fv[it] + 8 <= out_cols;
#pragma unroll
      for (int e = 0; e < 8; ++e) res[it][e] = 0.0f;
      if (ok && a.residual) {
        const uint4 raw = *reinterpret_cast<const uint4*>(a.residual + (t0 + tv[it]) * a.ldr + f0 + fv[it]);
        const __nv_bfloat16* rb = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
        for (int e = 0; e < 8; ++e) res[it][e] = bf2f(rb[e]);
      }
    }
#pragma unroll
    for (int it = 0; it < kMaxIter; ++it) {
      const int idx = ep_tid + it * 128;
      const int t = tv[it], fl = fv[it];
      if (idx >= total || t >= valid_t) continue;
      float o[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float* row = stage + t * (kBM + 4);
        float val;
        if (swiglu) {
          const float g = row[fl + e], u = row[fl + e + 64];
          val = g / (1.0f + __expf(-g)) * u;
        } else {
          val = row[fl + e];
        }
        o[e] = val + res[it][e];
      }
      const long long base = static_cast<long long>(t0 + t) * a.ldo + f0 + fl;
      if (f0 + fl + 8 <= out_cols) {
        if (a.out_f32) {
          float4* dst = reinterpret_cast<float4*>(static_cast<float*>(a.out) + base);
          dst[0] = make_float4(o[0], o[1], o[2], o[3]);
          dst[1] = make_float4(o[4], o[5], o[6], o[7]);
        } else {
          uint4 pk;
          __nv_bfloat162* pb = reinterpret_cast<__nv_bfloat162*>(&pk);
#pragma unroll
          for (int e = 0; e < 4; ++e) pb[e] = __floats2bfloat162_rn(o[2 * e], o[2 * e + 1]);
          put_bf16x8(a, base, pk);
        }
      } else {
        for (int e = 0; e < 8 && f0 + fl + e < out_cols; ++e) {
          float val = o[e];
          if (a.residual) val = o[e] - res[it][e] + bf2f(a.residual[(t0 + t) * a.ldr + f0 + fl + e]);
          if (a.out_f32)
            static_cast<float*>(a.out)[base + e] = val;
          else
            put_bf16(a, base + e, val);
        }
      }
    }
  } else {
    // scalar fallback for unaligned output / residual rows
    for (int idx = ep_tid; idx < 32 * width; idx += 128) {
      const int t = idx / width, fl = idx % width;
      if (t >= valid_t || f0 + fl >= out_cols) continue;
      const float* row = stage + t * (kBM + 4);
      float val;
      if (swiglu) {
        const float g = row[fl], u = row[fl + 64];
        val = g / (1.0f + __expf(-g)) * u;
      } else {
        val = row[fl];
      }
      const long long off = static_cast<long long>(t0 + t) * a.ldo + f0 + fl;
      if (a.residual) val += bf2f(a.residual[(t0 + t) * a.ldr + f0 + fl]);
      if (a.out_f32)
        static_cast<float*>(a.out)[off] = val;
      else
        put_bf16(a, off, val);
    }
  }
  named_barrier(bar, 128);
}


// Row-statistics epilogue of one 32-token chunk (vocabulary head scoring): the
// logits never leave the SM.  After the transpose, four threads share a token and
// take 32 weight rows each; they reduce (max, sum exp, sum exp at 1/T) and merge
// through two lane shuffles (lanes 4j..4j+3 hold token j), and the partial of the
// tile goes out as one 16-byte store.  The thread whose rows hold the token's
// target writes its logit.
__device__ __forceinline__ void merge_stats(float& m, float& s1, float& sT, float m2, float s12, float sT2,
                                            float invT) {
  const float hi = fmaxf(m, m2);
  if (hi == -INFINITY) return;
  const float a = m == -INFINITY ? 0.0f : expf(m - hi), b = m2 == -INFINITY ? 0.0f : expf(m2 - hi);
  const float aT = m == -INFINITY ? 0.0f : expf((m - hi) * invT), bT = m2 == -INFINITY ? 0.0f : expf((m2 - hi) * invT);
  s1 = s1 * a + s12 * b;
  sT = sT * aT + sT2 * bT;
  m = hi;
}

template <int BN>
__device__ __forceinline__ void stats_chunk(const Args& a, const float (&v)[32], int tm, int row0, int row_end,
                                            int chunk, int r, float* stage, int ep_tid, int bar) {
#pragma unroll
  for (int j = 0; j < 32; ++j) stage[j * (kBM + 4) + r] = v[j];
  named_barrier(bar, 128);
  const int j = ep_tid >> 2, q = ep_tid & 3;
  const int t = row0 + chunk * 32 + j;
  const int f = tm * kBM + q * 32;                 // first weight row of this thread's quarter
  const int nf = min(32, a.M - f);
  const float* row = stage + j * (kBM + 4) + q * 32;
  const bool live = t < row_end;
  const float invT = (live && a.stat_inv_temp != nullptr) ? a.stat_inv_temp[t] : 1.0f;
  float m = -INFINITY;
#pragma unroll
  for (int e = 0; e < 32; ++e)
    if (e < nf) m = fmaxf(m, row[e]);
  float s1 = 0.0f, sT = 0.0f;
  if (m != -INFINITY) {
#pragma unroll
    for (int e = 0; e < 32; ++e) {
      if (e < nf) {
        const float d = row[e] - m;
        s1 += expf(d);
        sT += expf(d * invT);
      }
    }
  }
#pragma unroll
  for (int o = 1; o <= 2; o <<= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    const float s12 = __shfl_xor_sync(0xffffffffu, s1, o);
    const float sT2 = __shfl_xor_sync(0xffffffffu, sT, o);
    merge_stats(m, s1, sT, m2, s12, sT2, invT);
  }
  if (live && q == 0) a.stat_part[static_cast<long long>(t) * a.tiles_m + tm] = make_float4(m, s1, sT, 0.0f);
  if (live && a.stat_targets != nullptr && a.stat_target_logit != nullptr) {
    const int tg = a.stat_targets[t] - f;
    if (tg >= 0 && tg < nf) a.stat_target_logit[t] = row[tg];
  }
  named_barrier(bar, 128);
}

// Cluster split-K reduction.  Every CTA of the cluster holds one split's fp32
// tile in its own shared memory, token-major: stage[c][r] (row stride kBM + 4).
// CTA `rank` reduces tokens [rank * BN / S, (rank + 1) * BN / S) across all S
// CTAs through distributed shared memory and writes them with the fused
// epilogue (bias, SwiGLU, residual) as 16-byte vectors.
template <int BN>
__device__ __forceinline__ void cluster_reduce_store(const Args& a, const float* stage, int tm, int tn) {
  const int S = a.cluster;
  const uint32_t rank = cluster_ctarank();
  const int cs = (BN + S - 1) / S;          // tokens reduced by each cluster rank (the last may get fewer)
  const bool swiglu = a.epilogue == 1;
  const int width = swiglu ? 64 : kBM;
  const int f0 = swiglu ? tm * 64 : tm * kBM;
  const int out_cols = swiglu ? a.M / 2 : a.M;
  const int vpr = width / 8;
  const int c_end = min(BN, static_cast<int>(rank + 1) * cs);
  const int items = max(0, c_end - static_cast<int>(rank) * cs) * vpr;
  const uint32_t base = smem_u32(stage);
  for (int it = threadIdx.x; it < items; it += blockDim.x) {
    const int cl = it / vpr;
    const int fl = (it % vpr) * 8;
    const int c = rank * cs + cl;           // token within the tile
    const int t = tn * BN + c;
    if (t >= a.N) continue;
    float g[8], u[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) g[e] = u[e] = 0.0f;
    const uint32_t row = base + static_cast<uint32_t>(c * (kBM + 4) + fl) * 4;
    // Issue the loads of four ranks before their adds: DSMEM loads are independent, and
    // summing in rank order afterwards keeps the result identical to a sequential reduction.
    constexpr int kBatch = 4;
    for (int q0 = 0; q0 < S; q0 += kBatch) {
      float4 xs[kBatch][2], ys[kBatch][2];
#pragma unroll
      for (int i = 0; i < kBatch; ++i) {
        if (q0 + i < S) {
          const uint32_t ra = map_shared_rank(row, q0 + i);
          xs[i][0] = ld_dsmem_f4(ra);
          xs[i][1] = ld_dsmem_f4(ra + 16);
          if (swiglu) {
            ys[i][0] = ld_dsmem_f4(ra + 64 * 4);
            ys[i][1] = ld_dsmem_f4(ra + 64 * 4 + 16);
          }
        }
      }
#pragma unroll
      for (int i = 0; i < kBatch; ++i) {
        if (q0 + i < S) {
          g[0] += xs[i][0].x; g[1] += xs[i][0].y; g[2] += xs[i][0].z; g[3] += xs[i][0].w;
          g[4] += xs[i][1].x; g[5] += xs[i][1].y; g[6] += xs[i][1].z; g[7] += xs[i][1].w;
          if (swiglu) {
            u[0] += ys[i][0].x; u[1] += ys[i][0].y; u[2] += ys[i][0].z; u[3] += ys[i][0].w;
            u[4] += ys[i][1].x; u[5] += ys[i][1].y; u[6] += ys[i][1].z; u[7] += ys[i][1].w;
          }
        }
      }
    }
    const int f = f0 + fl;
    float o[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      if (swiglu) {
        o[e] = g[e] / (1.0f + __expf(-g[e])) * u[e];
      } else {
        o[e] = g[e] + ((a.bias && f + e < out_cols) ? bf2f(a.bias[f + e]) : 0.0f);
      }
    }
    const long long off = static_cast<long long>(t) * a.ldo + f;
    if (a.vec_ok && f + 8 <= out_cols) {
      if (a.residual) {
        const uint4 raw = *reinterpret_cast<const uint4*>(a.residual + static_cast<long long>(t) * a.ldr + f);
        const __nv_bfloat16* rb = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] += bf2f(rb[e]);
      }
      if (a.out_f32) {
        float4* dst = reinterpret_cast<float4*>(static_cast<float*>(a.out) + off);
        dst[0] = make_float4(o[0], o[1], o[2], o[3]);
        dst[1] = make_float4(o[4], o[5], o[6], o[7]);
      } else {
        uint4 pk;
        __nv_bfloat162* pb = reinterpret_cast<__nv_bfloat162*>(&pk);
#pragma unroll
        for (int e = 0; e < 4; ++e) pb[e] = __floats2bfloat162_rn(o[2 * e], o[2 * e + 1]);
        put_bf16x8(a, off, pk);
      }
    } else {
      for (int e = 0; e < 8 && f + e < out_cols; ++e) {
        float val = o[e];
        if (a.residual) val += bf2f(a.residual[static_cast<long long>(t) * a.ldr + f + e]);
        if (a.out_f32)
          static_cast<float*>(a.out)[off + e] = val;
        else
          put_bf16(a, off + e, val);
      }
    }
  }
}

template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tn_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, const Args a) {
  using S = Smem<BN>;
  constexpr int STAGES = S::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * S::kABytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * S::kStageBytes);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* tfull = bars + 2 * STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  int* last_flag = reinterpret_cast<int*>(tmem_slot + 1);
  int* abort_flag = last_flag + 1;
  float* xchg = reinterpret_cast<float*>(smem + STAGES * S::kStageBytes + S::kBarBytes);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (threadIdx.x == 0) trace_stamp(a, 0);
  pdl_trigger();

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 4 * kEpiGroups);
    }
    *abort_flag = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, S::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  if (threadIdx.x == 0) trace_stamp(a, 1);

  const int total = a.gtiles != nullptr ? *a.gtotal : a.tiles_m * a.tiles_n * a.splits;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      // Weight tiles do not depend on the predecessor kernel: with prefetch_a
      // the first stages of this CTA's first work item are armed and their A
      // tiles requested before griddepcontrol.wait; their B tiles follow it.
      int armed = 0;
      if (a.prefetch_a && a.gtiles == nullptr && blockIdx.x < total) {
        const TileCoord c = tile_coord<BN>(a, blockIdx.x);
        const int kb0 = c.split * a.kb_per_split;
        const int kb1 = min(a.k_blocks, kb0 + a.kb_per_split);
        armed = min(STAGES, kb1 - kb0);
        for (int s = 0; s < armed; ++s) {
          mbar_arrive_expect_tx(&full[s], S::kStageBytes);
          tma_load_2d(sA + s * S::kABytes, &tmA, (kb0 + s) * kBK, c.arow, &full[s]);
        }
      }
      pdl_wait();
      for (int w = blockIdx.x; w < total && ok; w += gridDim.x) {
        const TileCoord c = tile_coord<BN>(a, w);
        const int kb0 = c.split * a.kb_per_split;
        const int kb1 = min(a.k_blocks, kb0 + a.kb_per_split);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (issued < armed) {
            tma_load_2d(sB + stage * S::kBBytes, &tmB, kb * kBK, c.row0, &full[stage]);
          } else {
            if (!mbar_wait(&empty[stage], phase ^ 1, a.status, kErrTmaWait)) {
              ok = false;
              *abort_flag = 1;
              break;
            }
            mbar_arrive_expect_tx(&full[stage], S::kStageBytes);
            tma_load_2d(sA + stage * S::kABytes, &tmA, kb * kBK, c.arow, &full[stage]);
            tma_load_2d(sB + stage * S::kBBytes, &tmB, kb * kBK, c.row0, &full[stage]);
          }
          if (issued == 0) trace_stamp(a, 2);
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {
        // Drain: wait (bounded) for the latest fill of every stage that was
        // issued, so no copy is still writing shared memory at exit.
        for (int s = 0; s < STAGES && s < issued; ++s) {
          const int fills = (issued - s + STAGES - 1) / STAGES;
          mbar_wait(&full[s], static_cast<uint32_t>((fills - 1) & 1), nullptr, 0);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(kBM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      const uint32_t a_base = smem_u32(sA);
      const uint32_t b_base = smem_u32(sB);
      bool ok = true;
      for (int w = blockIdx.x; w < total && ok; w += gridDim.x) {
        const int split = w % a.splits;
        const int kb0 = split * a.kb_per_split;
        const int kb1 = min(a.k_blocks, kb0 + a.kb_per_split);
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, a.status, kErrAccumWait)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, a.status, kErrMmaWait)) {
            ok = false;
            break;
          }
          if (w == static_cast<int>(blockIdx.x) && kb == kb0) trace_stamp(a, 3);
          tc_fence_after();
#pragma unroll
          for (int k = 0; k < kBK / kUmmaK; ++k) {
            const uint64_t ad = sdesc_k_sw128(a_base + stage * S::kABytes + k * kUmmaK * 2);
            const uint64_t bd = sdesc_k_sw128(b_base + stage * S::kBBytes + k * kUmmaK * 2);
            tc_mma_bf16(d_tmem, ad, bd, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
          }
          tc_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        tc_commit(&tfull[acc]);
        trace_stamp(a, 4);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
      if (!ok) *abort_flag = 1;
    }
  } else {
    // Epilogue warps 2..5 -> TMEM lane quarter (warp % 4).
    pdl_wait();   // residual / bias / output belong to the stream's data flow
    // Warps 2..(1 + 4 * kEpiGroups): group g = (warp - 2) / 4 finishes the 32-token
    // chunks c with c % kEpiGroups == g; every group covers the four TMEM lane quarters.
    const int quarter = warp % 4;
    const int grp = (warp - 2) / 4;
    const int gbar = 1 + grp;                         // named barrier of this group (128 threads)
    constexpr int kAllEpi = 128 * kEpiGroups;
    constexpr int kAllBar = 1 + kEpiGroups;           // named barrier of all epilogue threads
    const int r = quarter * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    int acc = 0;
    uint32_t acc_phase = 0;
    const int ep_tid = (threadIdx.x - 64) % 128;    // thread index within the group
    const bool ep_lead = threadIdx.x == 64;           // first epilogue thread of the CTA
    float* gstage = xchg + grp * 32 * (kBM + 4);
    for (int w = blockIdx.x; w < total; w += gridDim.x) {
      const TileCoord tc = tile_coord<BN>(a, w);
      const int split = tc.split;
      const int tile = tc.tile;
      const int tm = tc.tm;
      bool ok = mbar_wait(&tfull[acc], acc_phase, a.status, kErrEpilogueWait);
      if (ep_lead && w == static_cast<int>(blockIdx.x)) trace_stamp(a, 5);
      // All epilogue threads must agree before touching shared state.
      if (!ok) *abort_flag = 1;
      named_barrier(kAllBar, kAllEpi);
      if (*abort_flag) break;
      tc_fence_after();
      const uint32_t t_acc = tmem_base + lane_base + acc * BN;
      if (a.cluster > 1) {
        // Stage this split's tile token-major into the (now idle) pipeline smem.
        float* st = reinterpret_cast<float*>(smem);
        for (int c = grp; c < BN / 32; c += kEpiGroups) {
          float v[32];
          tmem_ld32(t_acc + c * 32, v);
#pragma unroll
          for (int j = 0; j < 32; ++j) st[(c * 32 + j) * (kBM + 4) + r] = v[j];
        }
        if (ep_lead) trace_stamp(a, 24);
        tc_fence_before();
      } else if (a.splits == 1) {
        for (int c = grp; c < BN / 32; c += kEpiGroups) {
          float v[32];
          tmem_ld32(t_acc + c * 32, v);
          if (ep_tid == 0 && c < 8) trace_stamp(a, 8 + 2 * c);
          if (a.epilogue == 2)
            stats_chunk<BN>(a, v, tm, tc.row0, tc.row_end, c, r, gstage, ep_tid, gbar);
          else
            finish_chunk<BN>(a, v, tm, tc.row0, tc.row_end, c, r, gstage, ep_tid, gbar);
          if (ep_tid == 0 && c < 8) trace_stamp(a, 9 + 2 * c);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[acc]);
      } else {
        float* part = a.workspace + (static_cast<long long>(split) * a.tiles_m * a.tiles_n + tile) * (kBM * BN);
        for (int c = grp; c < BN / 32; c += kEpiGroups) {
          float v[32];
          tmem_ld32(t_acc + c * 32, v);
#pragma unroll
          for (int j = 0; j < 32; ++j) __stcg(&part[(c * 32 + j) * kBM + r], v[j]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[acc]);
        __threadfence();
        named_barrier(kAllBar, kAllEpi);
        if (ep_lead) {
          const int prev = atomicAdd(&a.counters[tile], 1);
          const int last = prev == a.splits - 1;
          if (last) a.counters[tile] = 0;
          *last_flag = last;
        }
        named_barrier(kAllBar, kAllEpi);
        const int is_last = *last_flag;
        named_barrier(kAllBar, kAllEpi);
        if (is_last) {
          __threadfence();
          const long long tile_stride = static_cast<long long>(a.tiles_m) * a.tiles_n * (kBM * BN);
          const float* base = a.workspace + static_cast<long long>(tile) * (kBM * BN);
          for (int c = grp; c < BN / 32; c += kEpiGroups) {
            float v[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = 0.0f;
            for (int s = 0; s < a.splits; ++s) {
              const float* p = base + s * tile_stride;
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] += __ldcg(&p[(c * 32 + j) * kBM + r]);
            }
            finish_chunk<BN>(a, v, tm, tc.row0, tc.row_end, c, r, gstage, ep_tid, gbar);
          }
        }
      }
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (a.cluster > 1) {
    // Every CTA holds exactly one split of one tile (grid = tiles x cluster).
    const int tile = blockIdx.x / a.cluster;
    cluster_sync();                       // all splits staged
    if (threadIdx.x == 0) trace_stamp(a, 25);
    if (!*abort_flag) cluster_reduce_store<BN>(a, reinterpret_cast<const float*>(smem), tile % a.tiles_m,
                                               tile / a.tiles_m);
    if (threadIdx.x == 0) trace_stamp(a, 26);
    cluster_sync();                       // peers finished reading this CTA's tile
  }
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, S::kTmemCols);
    if (lane == 0) trace_stamp(a, 7);
  }
  if (a.push_world > 0) {
    // Every thread's peer stores are made visible system-wide before its CTA
    // arrives; the last CTA to arrive releases the completion flag on every rank.
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
      const unsigned int prev = atomicAdd(a.push_count, 1u);
      if (prev == gridDim.x - 1) {
        atomicExch(a.push_count, 0u);
        const uint32_t flag = *reinterpret_cast<const volatile uint32_t*>(a.push_epoch) + 1u;
        __threadfence_system();
        for (int q = 0; q < a.push_world; ++q)
          asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(a.push_flags[q]), "r"(flag) : "memory");
      }
    }
  }
}

// ------------------------------------------------------------------ host ----
EncodeTiledFn encode_fn() { return tensor_map_encoder(); }

bool make_map(CUtensorMap* map, const void* ptr, int rows, int cols, long long ld, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(kBK), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

int sm_count(int device) {
  static int cached[64] = {0};
  if (device < 0 || device >= 64) return 148;
  if (!cached[device]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device);
    cached[device] = n > 0 ? n : 148;
  }
  return cached[device];
}

// Largest number of co-resident clusters of `cluster` CTAs for this kernel (cached per device).
template <int BN>
int max_active_clusters(int dev, int cluster) {
  static int cache[64][kMaxClusterSplit + 1] = {};
  if (dev < 0 || dev >= 64 || cluster < 2 || cluster > kMaxClusterSplit) return 0;
  const int slot = cluster;
  if (cache[dev][slot] == 0) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(cluster * 64);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = Smem<BN>::kTotal;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = cluster;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, gemm_tn_kernel<BN>, &cfg) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = -1;
    }
    cache[dev][slot] = n;
  }
  return cache[dev][slot];
}

template <int BN>
cudaError_t launch_bn(const GemmProblem& p, const Args& a0, cudaStream_t stream) {
  using S = Smem<BN>;
  CUtensorMap ma, mb;
  const int a_rows = p.group_tiles != nullptr ? p.groups * p.M : p.M;
  if (!make_map(&ma, p.w, a_rows, p.K, p.ldw, kBM)) return cudaErrorInvalidValue;
  if (!make_map(&mb, p.x, p.N, p.K, p.ldx, BN)) return cudaErrorInvalidValue;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(gemm_tn_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kTotal);
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  Args a = a0;
  const int tiles = a.tiles_m * a.tiles_n;
  const int sms = sm_count(dev);
  if (p.group_tiles != nullptr) {
    a.splits = 1;
    a.kb_per_split = a.k_blocks;
    a.cluster = 1;
    a.gtiles = reinterpret_cast<const int4*>(p.group_tiles);
    a.gtotal = p.group_total;
    const int grid = std::max(1, std::min(p.group_tile_cap, sms));
    return launch_pdl(gemm_tn_kernel<BN>, dim3(grid), dim3(kThreads), S::kTotal, stream, ma, mb, a);
  }
  a.splits = 1;
  a.kb_per_split = a.k_blocks;
  a.cluster = 1;
  const bool may_split = p.allow_split && p.epilogue != 2;   // statistics need whole accumulators
  if (may_split && p.split_mode == 0 && tiles < sms) {
    // Split-K across a thread-block cluster of 2..8 CTAs, reduced through DSMEM.
    // Only cluster sizes whose clusters all fit on the GPU at once are used, so
    // the launch is a single wave; the largest such size streams the weights with
    // the most SMs (36 weight tiles: 3-CTA clusters, 108 SMs, where 4-CTA clusters
    // do not all fit and 2-CTA clusters leave half the GPU idle).
    const int want = sms / tiles;
    for (int c = kMaxClusterSplit; c >= 2; --c) {
      const int per = (a.k_blocks + c - 1) / c;
      if (c <= want && a.k_blocks >= 2 * c && (c - 1) * per < a.k_blocks &&
          tiles <= max_active_clusters<BN>(dev, c)) {
        a.cluster = c;
        a.splits = c;
        a.kb_per_split = per;
        break;
      }
    }
    if (a.cluster > 1) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(tiles * a.cluster);
      cfg.blockDim = dim3(kThreads);
      cfg.dynamicSmemBytes = S::kTotal;
      cfg.stream = stream;
      cudaLaunchAttribute attr[2];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = a.cluster;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      attr[1].val.programmaticStreamSerializationAllowed = 1;
      cfg.attrs = attr;
      cfg.numAttrs = pdl_enabled() ? 2 : 1;
      return cudaLaunchKernelEx(&cfg, gemm_tn_kernel<BN>, ma, mb, a);
    }
  }
  if (may_split && p.split_mode == 1 && tiles < sms && p.workspace != nullptr) {
    const GemmPlan plan = gemm_workspace_plan(p.M, p.N, p.K, sms);
    if (plan.bn == BN && plan.splits > 1 && plan.workspace_floats <= p.workspace_floats &&
        tiles <= p.counter_slots) {
      a.splits = plan.splits;
      a.kb_per_split = plan.kb_per_split;
    }
  }
  const int total = tiles * a.splits;
  const int grid = std::min(total, sms);
  return launch_pdl(gemm_tn_kernel<BN>, dim3(grid), dim3(kThreads), S::kTotal, stream, ma, mb, a);
}

}  // namespace

EncodeTiledFn tensor_map_encoder() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// On by default: the 7B suffix-MH round (bench.py, one B200) ran 6904 tok/s with
// programmatic dependent launch against 6788 without it, once the GEMM epilogue
// used two warpgroups (an earlier build, with a single-warpgroup epilogue, ran
// decode steps about 6% slower with it).  Every kernel launched this way waits
// (griddepcontrol.wait) before it reads its predecessor's output; only static
// weights are prefetched ahead of that wait.  The extension's set_pdl(False) disables it
// (for A/B timing).
bool& pdl_enabled() {
  static bool on = true;
  return on;
}

namespace {
// One CTA: exclusive scan of the per-group tile counts, then every thread
// writes the tiles of its groups (tm outer, token tile inner, so that CTAs
// running at the same time share weight tiles in L2).
__global__ void __launch_bounds__(1024) grouped_tiles_kernel(const int* __restrict__ offsets, int groups, int tiles_m,
                                                             int bn, int4* __restrict__ tiles, int cap,
                                                             int* __restrict__ total) {
  __shared__ int warp_sums[32];
  __shared__ int carry;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  for (int base = 0; base < groups; base += blockDim.x) {
    const int g = base + threadIdx.x;
    int n = 0, rows = 0, lo = 0;
    if (g < groups) {
      lo = offsets[g];
      rows = offsets[g + 1] - lo;
      n = rows > 0 ? ((rows + bn - 1) / bn) * tiles_m : 0;
    }
    // block-wide inclusive scan of n
    int x = n;
    const int lane = threadIdx.x % 32, warp = threadIdx.x / 32;
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) warp_sums[warp] = x;
    __syncthreads();
    if (warp == 0) {
      int s = lane < (blockDim.x + 31) / 32 ? warp_sums[lane] : 0;
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, s, o);
        if (lane >= o) s += y;
      }
      warp_sums[lane] = s;
    }
    __syncthreads();
    const int start = carry + (warp > 0 ? warp_sums[warp - 1] : 0) + x - n;
    if (g < groups) {
      const int nt = rows > 0 ? (rows + bn - 1) / bn : 0;
      int k = start;
      for (int tm = 0; tm < tiles_m; ++tm)
        for (int t = 0; t < nt; ++t, ++k)
          if (k < cap) tiles[k] = make_int4(g, tm, lo + t * bn, lo + rows);
    }
    __syncthreads();
    if (threadIdx.x == blockDim.x - 1) carry = start + n;
    __syncthreads();
  }
  if (threadIdx.x == 0) *total = min(carry, cap);
}
}  // namespace

cudaError_t grouped_tiles_launch(const int* offsets, int groups, int tiles_m, int bn, int* tiles, int cap, int* total,
                                 cudaStream_t stream) {
  if (groups <= 0 || tiles_m <= 0 || bn <= 0 || cap <= 0) return cudaErrorInvalidValue;
  grouped_tiles_kernel<<<1, 1024, 0, stream>>>(offsets, groups, tiles_m, bn, reinterpret_cast<int4*>(tiles), cap,
                                               total);
  return cudaGetLastError();
}

unsigned long long*& gemm_trace_buffer() {
  static unsigned long long* buf = nullptr;
  return buf;
}

int gemm_pick_bn(int tokens) {
  if (tokens <= 32) return 32;
  if (tokens <= 64) return 64;
  if (tokens <= 128) return 128;
  return 256;
}

int gemm_token_tile(int M, int N, int K) {
  int bn = gemm_pick_bn(N);
  // Few weight-row tiles and a short reduction: 128-token tiles double the CTAs
  // that stream weights and still split K over a cluster pair (measured on B200
  // at 256 tokens: 7B qkv 22.9 -> 18.5 us, 1.5B qkv 14.7 -> 11.5 us, 1.5B down
  // 23.1 -> 20.1 us; the 7B down projection, K = 18944, is faster with 256).
  if (bn == 256 && K <= 10240 && (M + kBM - 1) / kBM < 64) bn = 128;
  return bn;
}

GemmPlan gemm_workspace_plan(int M, int N, int K, int sms) {
  GemmPlan plan{};
  plan.bn = gemm_token_tile(M, N, K);
  plan.tiles = ((M + kBM - 1) / kBM) * ((N + plan.bn - 1) / plan.bn);
  const int kb = (K + kBK - 1) / kBK;
  plan.splits = 1;
  plan.kb_per_split = kb;
  plan.workspace_floats = 0;
  if (plan.tiles < sms) {
    const int want = std::min(std::max(1, sms / plan.tiles), std::max(1, kb / 2));
    const int per = (kb + want - 1) / want;
    const int splits = (kb + per - 1) / per;
    if (splits > 1) {
      plan.splits = splits;
      plan.kb_per_split = per;
      plan.workspace_floats = static_cast<long long>(splits) * plan.tiles * kBM * plan.bn;
    }
  }
  return plan;
}

cudaError_t gemm_launch(const GemmProblem& p, cudaStream_t stream) {
  if (p.M <= 0 || p.N <= 0 || p.K <= 0) return cudaErrorInvalidValue;
  if ((p.ldw % 8) || (p.ldx % 8) || (reinterpret_cast<uintptr_t>(p.w) % 16) ||
      (reinterpret_cast<uintptr_t>(p.x) % 16))
    return cudaErrorInvalidValue;  // TMA needs 16-byte aligned rows
  if (p.epilogue == 1 && (p.M % kBM)) return cudaErrorInvalidValue;
  if (p.epilogue == 2 && (p.stat_part == nullptr || p.group_tiles != nullptr || p.push_world > 0 ||
                          (reinterpret_cast<uintptr_t>(p.stat_part) % 16)))
    return cudaErrorInvalidValue;
  Args a{};
  a.M = p.M;
  a.N = p.N;
  a.K = p.K;
  a.k_blocks = (p.K + kBK - 1) / kBK;
  if (p.group_tiles != nullptr) {
    if (p.M % kBM || p.groups <= 0 || p.group_total == nullptr || p.group_tile_cap <= 0 ||
        (p.group_bn != 32 && p.group_bn != 64 && p.group_bn != 128 && p.group_bn != 256))
      return cudaErrorInvalidValue;
  }
  const int bn = p.group_tiles != nullptr ? p.group_bn : gemm_token_tile(p.M, p.N, p.K);
  const GemmProblem& q = p;
  a.tiles_m = (p.M + kBM - 1) / kBM;
  a.tiles_n = (p.N + bn - 1) / bn;
  a.out = p.out;
  a.ldo = p.ldo;
  a.residual = p.residual;
  a.ldr = p.ldr;
  a.bias = p.bias;
  a.epilogue = p.epilogue;
  a.stat_inv_temp = p.stat_inv_temp;
  a.stat_targets = p.stat_targets;
  a.stat_part = reinterpret_cast<float4*>(p.stat_part);
  a.stat_target_logit = p.stat_target_logit;
  a.out_f32 = p.out_f32;
  a.workspace = p.workspace;
  a.counters = p.counters;
  a.status = p.status;
  a.prefetch_a = p.prefetch_weights;
  a.trace = gemm_trace_buffer();
  a.push_world = 0;
  if (p.push_world > 0) {
    if (p.push_world > kPushMaxRanks || p.out_f32 || p.residual != nullptr || p.epilogue != 0 ||
        p.group_tiles != nullptr || p.push_epoch == nullptr || p.push_count == nullptr)
      return cudaErrorInvalidValue;
    a.push_world = p.push_world;
    for (int q = 0; q < p.push_world; ++q) {
      a.push_dst[q] = p.push_dst[q];
      a.push_flags[q] = p.push_flags[q];
    }
    a.push_epoch = p.push_epoch;
    a.push_count = p.push_count;
  }
  a.gtiles = nullptr;
  a.gtotal = nullptr;
  {
    const int esz = p.out_f32 ? 4 : 2;
    const bool out_ok = (reinterpret_cast<uintptr_t>(p.out) % 16 == 0) && ((p.ldo * esz) % 16 == 0);
    const bool res_ok = p.residual == nullptr ||
                        ((reinterpret_cast<uintptr_t>(p.residual) % 16 == 0) && ((p.ldr * 2) % 16 == 0));
    a.vec_ok = out_ok && res_ok;
  }
  switch (bn) {
    case 32: return launch_bn<32>(q, a, stream);
    case 64: return launch_bn<64>(q, a, stream);
    case 128: return launch_bn<128>(q, a, stream);
    default: return launch_bn<256>(q, a, stream);
  }
}

}  // namespace osb
