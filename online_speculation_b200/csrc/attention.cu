// Paged attention with per-sequence causal or bidirectional masks.
//
// One kernel serves every attention shape of the package:
//   * causal prefill of prompts (queries = keys = the prompt),
//   * single-token decode against a paged, prefix-shared KV history,
//   * speculative verification (a block of query tokens appended causally),
//   * block-bidirectional drafting (a block of query tokens that see the
//     read-only history plus each other in both directions),
//   * full bidirectional masked-diffusion steps (no history).
// Reference call sites: online-speculation/src/blockspec/parallel/backbone.py:113-148
// (AR / draft views), src/inference_scaling/arllm/backends/transformers_backend.py
// decode loop (HF SDPA with DynamicCache), src/inference_scaling/dllm/backends/llada.py:417-448.
//
// Layouts
//   q     [T, Hq, D]  bf16, rows of sequence b start at q_start[b]
//   cache [pages, Hkv, P, D] bf16 for K and for V (P = kPage tokens per page)
//   table [B, max_pages] int32 physical page ids
//   out   [T, Hq, D]  bf16
// Query rows of one (sequence, kv head) are flattened token-major:
// row = token * G + head_in_group with G = Hq / Hkv.  Query token i of a block of
// length L sits at absolute position kv_len - L + i.
//
// Tensor cores: bf16 mma.sync m16n8k16 with ldmatrix operand loads, online
// softmax in fp32 with exp2.  Two warp layouts:
//   kRowsSplit  : 4 warps x 16 rows share each 32-key page (prefill / diffusion),
//   TMA key split: up to 32 rows (two m16 tiles) of one sequence; four key
//                 groups stream 16-key chunks with TMA and merge their partial
//                 softmax states in shared memory (decode / verify / draft).
#include "attention.h"
#include "common.cuh"

namespace osb {
namespace {

constexpr int kD = 128;
constexpr int kPage = 32;
constexpr int kStride = kD + 8;  // padded smem row (elements) to avoid ldmatrix bank conflicts

struct AttnArgs {
  const __nv_bfloat16* q;
  const __nv_bfloat16* k_cache;
  const __nv_bfloat16* v_cache;
  const int* table;
  int table_stride;
  const int* q_start;
  const int* q_len;
  const int* kv_len;
  const int* mode;  // per sequence: 0 causal, 1 bidirectional
  const int* tile_seq;
  const int* tile_row0;
  __nv_bfloat16* out;
  int Hq, Hkv, G;
  float scale_log2;  // softmax scale * log2(e)
  int* status;
  unsigned long long* trace;  // tcgen05 kernel timeline (tuning): kTraceSlots globaltimer stamps per CTA, or null
  // Two-pass (shared-prefix) attention, TMA kernel only; every field may be null:
  const int* k_lo;            // [B] first key of each sequence's range (a multiple of the page size)
  float* o_f32;               // [T, Hq, D] fp32 normalised output instead of `out`
  float* lse_out;             // [T, Hq] log2-domain log-sum-exp of the scaled scores of the range
  const float* prior_o;       // [T, Hq, D] normalised output of an earlier key range, merged in
  const float* prior_lse;     // [T, Hq] its log2-domain log-sum-exp
};

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem)), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Copy one 32-key page of K and V for kv head g into padded smem rows.
// Keys at or beyond `valid` are zero-filled so masked products stay finite.
__device__ __forceinline__ void load_page(const AttnArgs& a, int page, int g, int valid, __nv_bfloat16* sK,
                                          __nv_bfloat16* sV, int tid, int nthreads) {
  const long long base = (static_cast<long long>(page) * a.Hkv + g) * (kPage * kD);
  const __nv_bfloat16* gk = a.k_cache + base;
  const __nv_bfloat16* gv = a.v_cache + base;
  // 32 rows x 16 chunks of 16 bytes
  for (int c = tid; c < kPage * (kD / 8); c += nthreads) {
    const int row = c / (kD / 8);
    const int col = (c % (kD / 8)) * 8;
    if (row < valid) {
      cp_async16(sK + row * kStride + col, gk + row * kD + col);
      cp_async16(sV + row * kStride + col, gv + row * kD + col);
    } else {
      *reinterpret_cast<uint4*>(sK + row * kStride + col) = make_uint4(0, 0, 0, 0);
      *reinterpret_cast<uint4*>(sV + row * kStride + col) = make_uint4(0, 0, 0, 0);
    }
  }
}

// Copy keys [k0, k0 + CH) of one page (CH = 16) of K and V for kv head g.
template <int CH>
__device__ __forceinline__ void load_chunk(const AttnArgs& a, int page, int g, int k0, int valid, __nv_bfloat16* sK,
                                           __nv_bfloat16* sV, int lane) {
  const long long base = ((static_cast<long long>(page) * a.Hkv + g) * kPage + k0) * kD;
  const __nv_bfloat16* gk = a.k_cache + base;
  const __nv_bfloat16* gv = a.v_cache + base;
  for (int c = lane; c < CH * (kD / 8); c += 32) {
    const int row = c / (kD / 8);
    const int col = (c % (kD / 8)) * 8;
    if (row < valid) {
      cp_async16(sK + row * kStride + col, gk + row * kD + col);
      cp_async16(sV + row * kStride + col, gv + row * kD + col);
    } else {
      *reinterpret_cast<uint4*>(sK + row * kStride + col) = make_uint4(0, 0, 0, 0);
      *reinterpret_cast<uint4*>(sV + row * kStride + col) = make_uint4(0, 0, 0, 0);
    }
  }
}

// Per-warp flash-attention state for 16 query rows.
struct WarpState {
  uint32_t qf[kD / 16][4];
  float o[kD / 8][4];
  float m[2], l[2];
  int qpos[2];   // absolute query position of this thread's two rows (-1 = padding row)
  int frontier;  // keys below this index are visible to every row of the warp (no masking needed)
};

__device__ __forceinline__ void load_q(const AttnArgs& a, WarpState& st, int q0, int rows, int row_base, int g,
                                       int qlen, int kvlen, int lane, int bidir) {
  const int r_lo = lane / 4, c2 = (lane % 4) * 2;
  // the warp's first row has the earliest causal horizon; padding rows (zero queries) need no mask
  st.frontier = (bidir || row_base >= rows) ? kvlen : min(kvlen, kvlen - qlen + row_base / a.G + 1);
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int row = row_base + r_lo + h * 8;
    st.qpos[h] = row < rows ? kvlen - qlen + row / a.G : -1;
  }
#pragma unroll
  for (int kk = 0; kk < kD / 16; ++kk) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int row = row_base + r_lo + h * 8;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t v = 0;
        if (row < rows) {
          const int tok = row / a.G, head = g * a.G + row % a.G;
          const __nv_bfloat16* p = a.q + (static_cast<long long>(q0 + tok) * a.Hq + head) * kD + kk * 16 + c2 + half * 8;
          v = *reinterpret_cast<const uint32_t*>(p);
        }
        st.qf[kk][h + half * 2] = v;
      }
    }
  }
#pragma unroll
  for (int n = 0; n < kD / 8; ++n)
#pragma unroll
    for (int i = 0; i < 4; ++i) st.o[n][i] = 0.0f;
  st.m[0] = st.m[1] = -INFINITY;
  st.l[0] = st.l[1] = 0.0f;
}

// Process one chunk of CH (16 or 32) keys already resident in shared memory.
// kaddr(key, d) / vaddr(key, d): shared-memory byte address of the 8-element
// (16-byte) row segment starting at column d of key row `key` of K / V.
template <int CH, class KAddr, class VAddr>
__device__ __forceinline__ void process_keys(const AttnArgs& a, WarpState& st, KAddr kaddr, VAddr vaddr, int key0,
                                             int kvlen, int bidir, int lane) {
  constexpr int NB = CH / 8;  // key blocks of 8
  float s[NB][4];
#pragma unroll
  for (int n = 0; n < NB; ++n)
#pragma unroll
    for (int i = 0; i < 4; ++i) s[n][i] = 0.0f;
  // S = Q K^T over NB key blocks of 8
#pragma unroll
  for (int n = 0; n < NB; ++n) {
#pragma unroll
    for (int kk = 0; kk < kD / 16; kk += 2) {
      // matrices: (keys n*8.., d kk*16+0..7), (.., +8), (.., (kk+1)*16), (.., +8)
      const int mi = lane / 8, ri = lane % 8;
      const uint32_t addr = kaddr(n * 8 + ri, kk * 16 + mi * 8);
      uint32_t b0, b1, b2, b3;
      ldsm_x4(addr, b0, b1, b2, b3);
      mma16816(s[n], st.qf[kk], b0, b1);
      mma16816(s[n], st.qf[kk + 1], b2, b3);
    }
  }
  // mask + online softmax (chunks below the warp's causal frontier need no mask)
  const int c2 = (lane % 4) * 2;
  float mx[2] = {-INFINITY, -INFINITY};
  if (key0 + CH <= st.frontier) {
#pragma unroll
    for (int n = 0; n < NB; ++n)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        s[n][i] *= a.scale_log2;
        mx[i / 2] = fmaxf(mx[i / 2], s[n][i]);
      }
  } else {
#pragma unroll
    for (int n = 0; n < NB; ++n) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int h = i / 2;
        const int key = key0 + n * 8 + c2 + (i & 1);
        const int qp = st.qpos[h];
        const bool ok = qp >= 0 && key < kvlen && (bidir || key <= qp);
        s[n][i] = ok ? s[n][i] * a.scale_log2 : -INFINITY;
        mx[h] = fmaxf(mx[h], s[n][i]);
      }
    }
  }
  float corr[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 1));
    mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 2));
    const float mnew = fmaxf(st.m[h], mx[h]);
    corr[h] = (mnew == -INFINITY) ? 1.0f : exp2f(st.m[h] - mnew);
    st.m[h] = mnew;
  }
  float rs[2] = {0.0f, 0.0f};
#pragma unroll
  for (int n = 0; n < NB; ++n) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int h = i / 2;
      const float p = (st.m[h] == -INFINITY) ? 0.0f : exp2f(s[n][i] - st.m[h]);
      s[n][i] = p;
      rs[h] += p;
    }
  }
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    rs[h] += __shfl_xor_sync(0xffffffffu, rs[h], 1);
    rs[h] += __shfl_xor_sync(0xffffffffu, rs[h], 2);
    st.l[h] = st.l[h] * corr[h] + rs[h];
  }
  // the running maximum rarely moves after the first chunks: skip the rescale when no row needs it
  if (__any_sync(0xffffffffu, corr[0] != 1.0f || corr[1] != 1.0f)) {
#pragma unroll
    for (int n = 0; n < kD / 8; ++n) {
      st.o[n][0] *= corr[0];
      st.o[n][1] *= corr[0];
      st.o[n][2] *= corr[1];
      st.o[n][3] *= corr[1];
    }
  }
  // O += P V  (CH / 16 k-steps of 16 keys)
#pragma unroll
  for (int kk = 0; kk < CH / 16; ++kk) {
    uint32_t pa[4];
    pa[0] = pack_bf16(s[2 * kk][0], s[2 * kk][1]);
    pa[1] = pack_bf16(s[2 * kk][2], s[2 * kk][3]);
    pa[2] = pack_bf16(s[2 * kk + 1][0], s[2 * kk + 1][1]);
    pa[3] = pack_bf16(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
    for (int n = 0; n < kD / 8; n += 2) {
      // matrices: (keys kk*16+0..7, d n*8), (keys +8, d n*8), (keys 0..7, d (n+1)*8), (keys +8, d (n+1)*8)
      const int mi = lane / 8, ri = lane % 8;
      const int key = kk * 16 + (mi & 1) * 8 + ri;
      const int d = n * 8 + (mi >> 1) * 8;
      uint32_t b0, b1, b2, b3;
      ldsm_x4_t(vaddr(key, d), b0, b1, b2, b3);
      mma16816(st.o[n], pa, b0, b1);
      mma16816(st.o[n + 1], pa, b2, b3);
    }
  }
}

// Chunk of CH keys stored as padded rows (kStride elements per key row).
template <int CH = 32>
__device__ __forceinline__ void process_page(const AttnArgs& a, WarpState& st, const __nv_bfloat16* sK,
                                             const __nv_bfloat16* sV, int key0, int kvlen, int bidir, int lane) {
  const uint32_t kb = smem_u32(sK), vb = smem_u32(sV);
  process_keys<CH>(
      a, st, [kb](int key, int d) { return kb + (key * kStride + d) * 2; },
      [vb](int key, int d) { return vb + (key * kStride + d) * 2; }, key0, kvlen, bidir, lane);
}

__device__ __forceinline__ void store_rows(const AttnArgs& a, const WarpState& st, int q0, int rows, int row_base,
                                           int g, int lane) {
  const int r_lo = lane / 4, c2 = (lane % 4) * 2;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int row = row_base + r_lo + h * 8;
    if (row >= rows) continue;
    const float inv = st.l[h] > 0.0f ? 1.0f / st.l[h] : 0.0f;
    const int tok = row / a.G, head = g * a.G + row % a.G;
    __nv_bfloat16* p = a.out + (static_cast<long long>(q0 + tok) * a.Hq + head) * kD;
#pragma unroll
    for (int n = 0; n < kD / 8; ++n) {
      *reinterpret_cast<uint32_t*>(p + n * 8 + c2) = pack_bf16(st.o[n][2 * h] * inv, st.o[n][2 * h + 1] * inv);
    }
  }
}

// 4 warps x 16 rows share each page.
__global__ void __launch_bounds__(128) attn_rows_kernel(const AttnArgs a) {
  __shared__ __align__(16) __nv_bfloat16 sK[2][kPage * kStride];
  __shared__ __align__(16) __nv_bfloat16 sV[2][kPage * kStride];
  pdl_wait();
  pdl_trigger();
  const int tile = blockIdx.x, g = blockIdx.y;
  const int b = a.tile_seq[tile];
  const int row0 = a.tile_row0[tile];
  const int qlen = a.q_len[b], kvlen = a.kv_len[b], q0 = a.q_start[b];
  const int bidir = a.mode[b];
  const int rows = qlen * a.G;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  WarpState st;
  load_q(a, st, q0, rows, row0 + warp * 16, g, qlen, kvlen, lane, bidir);
  // last key any row of this tile can see
  const int last_row = min(rows - 1, row0 + 63);
  const int max_key = bidir ? kvlen : min(kvlen, kvlen - qlen + last_row / a.G + 1);
  const int npages = (max_key + kPage - 1) / kPage;
  const int* tbl = a.table + static_cast<long long>(b) * a.table_stride;
  if (npages > 0) {
    load_page(a, tbl[0], g, min(kPage, kvlen), sK[0], sV[0], threadIdx.x, 128);
    cp_async_commit();
  }
  for (int p = 0; p < npages; ++p) {
    if (p + 1 < npages) {
      load_page(a, tbl[p + 1], g, min(kPage, kvlen - (p + 1) * kPage), sK[(p + 1) & 1], sV[(p + 1) & 1],
                threadIdx.x, 128);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    process_page<32>(a, st, sK[p & 1], sV[p & 1], p * kPage, kvlen, bidir, lane);
    __syncthreads();
  }
  store_rows(a, st, q0, rows, row0 + warp * 16, g, lane);
}

// Decode / verify / draft tiles (at most 32 query rows of one sequence and kv
// head).  MT m-tiles of 16 rows x 4 key groups = 4 * MT warps.  Key group kg
// owns the 16-key chunks j = kg, kg + 4, ...; one lane of its first warp
// streams them with TMA (two 64-column boxes of K and of V, 128-byte swizzle)
// into a kTStages ring guarded by full / empty mbarriers, and the MT warps of
// the group share every chunk, so the KV of a (sequence, kv head) crosses into
// shared memory once per tile.  The key groups' softmax states merge in shared
// memory at the end.
constexpr int kCh = 16;
constexpr int kKG = 4;
constexpr int kTStages = 3;
constexpr int kBoxBytes = kCh * 64 * 2;          // 16 key rows x 64 bf16 columns
constexpr int kChunkBytes = 4 * kBoxBytes;       // K lo | K hi | V lo | V hi
constexpr int kGroupBytes = kTStages * kChunkBytes;
constexpr int kMergeStride = kD + 8;            // fp32 merge row (floats)

template <int MT>
struct TmaSmem {
  static constexpr int kPipe = kKG * kGroupBytes;
  static constexpr int kMerge = MT * kKG * (16 * kMergeStride + 32) * 4;
  static constexpr int kBody = kPipe > kMerge ? kPipe : kMerge;
  static constexpr int kBarOffset = kBody;
  static constexpr int kTotal = 1024 + kBody + 2 * kKG * kTStages * 8;
};

// Address of the 16-byte segment (key, d..d+7) inside a 128B-swizzled chunk
// whose two 64-column boxes start at box0 and box0 + kBoxBytes.
__device__ __forceinline__ uint32_t sw128_addr(uint32_t box0, int key, int d) {
  return box0 + (d >> 6) * kBoxBytes + key * 128 + ((((d & 63) >> 3) ^ (key & 7)) << 4);
}

template <int MT>
__global__ void __launch_bounds__(128 * MT, 2)
    attn_tma_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                    const AttnArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(base + TmaSmem<MT>::kBarOffset);
  uint64_t* empty = full + kKG * kTStages;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int mt = warp / kKG, kg = warp % kKG;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kKG * kTStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], MT);
    }
    fence_barrier_init();
    prefetch_tmap(&kmap);
    prefetch_tmap(&vmap);
  }
  __syncthreads();
  pdl_wait();
  pdl_trigger();
  const int tile = blockIdx.x, g = blockIdx.y;
  const int b = a.tile_seq[tile];
  const int row0 = a.tile_row0[tile];
  const int qlen = a.q_len[b], kvlen = a.kv_len[b], q0 = a.q_start[b];
  const int bidir = a.mode[b];
  const int rows = qlen * a.G;
  WarpState st;
  load_q(a, st, q0, rows, row0 + mt * 16, g, qlen, kvlen, lane, bidir);
  const int last_row = min(rows - 1, row0 + 16 * MT - 1);
  const int max_key = bidir ? kvlen : min(kvlen, kvlen - qlen + last_row / a.G + 1);
  const int klo = a.k_lo != nullptr ? a.k_lo[b] : 0;      // keys [klo, max_key)
  const int nchunks = (max(max_key - klo, 0) + kCh - 1) / kCh;
  const int mine = nchunks > kg ? (nchunks - kg + kKG - 1) / kKG : 0;
  const int* tbl = a.table + static_cast<long long>(b) * a.table_stride;
  uint8_t* gbase = base + kg * kGroupBytes;
  uint64_t* gfull = full + kg * kTStages;
  uint64_t* gempty = empty + kg * kTStages;
  const bool producer = mt == 0 && lane == 0;
  auto issue = [&](int i) {
    const int key0 = klo + (kg + kKG * i) * kCh;
    const int y = (tbl[key0 / kPage] * a.Hkv + g) * kPage + key0 % kPage;
    const int s = i % kTStages;
    uint8_t* dst = gbase + s * kChunkBytes;
    mbar_arrive_expect_tx(&gfull[s], kChunkBytes);
    tma_load_2d(dst, &kmap, 0, y, &gfull[s]);
    tma_load_2d(dst + kBoxBytes, &kmap, 64, y, &gfull[s]);
    tma_load_2d(dst + 2 * kBoxBytes, &vmap, 0, y, &gfull[s]);
    tma_load_2d(dst + 3 * kBoxBytes, &vmap, 64, y, &gfull[s]);
  };
  int issued = 0;
  if (producer)
    for (; issued < min(mine, kTStages); ++issued) issue(issued);
  bool ok = true;
  int consumed = 0;
  for (int i = 0; i < mine; ++i) {
    const int s = i % kTStages;
    const uint32_t ph = (i / kTStages) & 1;
    if (!mbar_wait(&gfull[s], ph, a.status, kErrMmaWait)) {
      ok = false;
      break;
    }
    consumed = i + 1;
    const int key0 = klo + (kg + kKG * i) * kCh;
    const uint32_t kb = smem_u32(gbase + s * kChunkBytes);
    const uint32_t vb = kb + 2 * kBoxBytes;
    if (kvlen - key0 < kCh) {
      // Rows past the sequence end hold whatever the page held before; their
      // probabilities are exactly zero, but 0 * (non-finite V) is not, so zero them.
      if (mt == 0) {
        const int valid = kvlen - key0;
        uint8_t* v = gbase + s * kChunkBytes + 2 * kBoxBytes;
        for (int c = lane; c < 2 * kCh * 8; c += 32) {
          const int box = c / (kCh * 8), row = (c / 8) % kCh, seg = c % 8;
          if (row >= valid) *reinterpret_cast<uint4*>(v + box * kBoxBytes + row * 128 + seg * 16) = make_uint4(0, 0, 0, 0);
        }
      }
      if (MT > 1) named_barrier(1 + kg, 32 * MT);
      else __syncwarp();
    }
    process_keys<kCh>(
        a, st, [kb](int key, int d) { return sw128_addr(kb, key, d); },
        [vb](int key, int d) { return sw128_addr(vb, key, d); }, key0, kvlen, bidir, lane);
    __syncwarp();
    if (lane == 0) mbar_arrive(&gempty[s]);
    if (producer && issued < mine) {
      if (!mbar_wait(&gempty[s], ph, a.status, kErrTmaWait)) {
        ok = false;
        break;
      }
      issue(issued);
      ++issued;
    }
  }
  if (!ok && producer) {
    // Drain this group's copies still in flight before the CTA can exit.
    for (int i = consumed; i < issued; ++i) mbar_wait(&gfull[i % kTStages], (i / kTStages) & 1, a.status, kErrMmaWait);
  }
  __syncthreads();
  // Merge the key groups of each m-tile: per warp 16 x 128 fp32 partial outputs plus (m, l).
  // Rows are padded to kMergeStride floats: the fragment stores (8 rows x 4 column pairs per
  // half-warp phase) and the float4 reads (8 lanes per row) then hit 32 distinct banks.
  float* so = reinterpret_cast<float*>(base);            // [4 * MT][16][kMergeStride]
  float* sm = so + 4 * MT * 16 * kMergeStride;           // [4 * MT][16]
  float* sl = sm + 4 * MT * 16;                           // [4 * MT][16]
  {
    const int r_lo = lane / 4, c2 = (lane % 4) * 2;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int row = r_lo + h * 8;
      float* dst = so + (warp * 16 + row) * kMergeStride + c2;
#pragma unroll
      for (int n = 0; n < kD / 8; ++n)
        *reinterpret_cast<float2*>(dst + n * 8) = make_float2(st.o[n][2 * h], st.o[n][2 * h + 1]);
      if ((lane % 4) == 0) {
        sm[warp * 16 + row] = st.m[h];
        sl[warp * 16 + row] = st.l[h];
      }
    }
  }
  __syncthreads();
  const int r = threadIdx.x / 8;             // 16 * MT rows, 8 threads per row
  const int c4 = (threadIdx.x % 8) * 4;      // columns c4 + 32 j, j < 4
  const int tm = r / 16, rr = r % 16;
  const int row = row0 + r;
  if (row < rows) {
    const int tok = row / a.G, head = g * a.G + row % a.G;
    const long long slot = static_cast<long long>(q0 + tok) * a.Hq + head;    // (token, head)
    // an earlier key range enters as one more partial: (max = its lse, sum = 1, normalised output)
    const float prior_m = a.prior_lse != nullptr ? a.prior_lse[slot] : -INFINITY;
    float M = prior_m;
#pragma unroll
    for (int k = 0; k < kKG; ++k) M = fmaxf(M, sm[(tm * kKG + k) * 16 + rr]);
    float wgt[kKG], L = 0.0f;
#pragma unroll
    for (int k = 0; k < kKG; ++k) {
      const float mk = sm[(tm * kKG + k) * 16 + rr];
      wgt[k] = (M == -INFINITY || mk == -INFINITY) ? 0.0f : exp2f(mk - M);
      L += wgt[k] * sl[(tm * kKG + k) * 16 + rr];
    }
    const float wprior = (M == -INFINITY || prior_m == -INFINITY) ? 0.0f : exp2f(prior_m - M);
    L += wprior;
    const float inv = L > 0.0f ? 1.0f / L : 0.0f;
    if (a.lse_out != nullptr && (threadIdx.x % 8) == 0) a.lse_out[slot] = L > 0.0f ? M + log2f(L) : -INFINITY;
    __nv_bfloat16* p = a.out + slot * kD;
#pragma unroll
    for (int j = 0; j < kD / 32; ++j) {
      float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
      for (int k = 0; k < kKG; ++k) {
        const float4 x = *reinterpret_cast<const float4*>(so + ((tm * kKG + k) * 16 + rr) * kMergeStride + c4 + 32 * j);
        v.x += wgt[k] * x.x;
        v.y += wgt[k] * x.y;
        v.z += wgt[k] * x.z;
        v.w += wgt[k] * x.w;
      }
      if (wprior != 0.0f) {
        const float4 x = *reinterpret_cast<const float4*>(a.prior_o + slot * kD + c4 + 32 * j);
        v.x += wprior * x.x;
        v.y += wprior * x.y;
        v.z += wprior * x.z;
        v.w += wprior * x.w;
      }
      if (a.o_f32 != nullptr) {
        *reinterpret_cast<float4*>(a.o_f32 + slot * kD + c4 + 32 * j) =
            make_float4(v.x * inv, v.y * inv, v.z * inv, v.w * inv);
      } else {
        uint2 packed;
        packed.x = pack_bf16(v.x * inv, v.y * inv);
        packed.y = pack_bf16(v.z * inv, v.w * inv);
        *reinterpret_cast<uint2*>(p + c4 + 32 * j) = packed;
      }
    }
  }
}


// ------------------------------------------------------------------------------
// tcgen05 attention (every shape: prefill, decode, verify / draft blocks, diffusion).
//
// One CTA computes a 128-row query tile of one (sequence, kv head) over a range of
// key chunks; with key splitting, the S CTAs of a thread-block cluster take
// consecutive chunk ranges of the same tile and merge their partial softmax states
// through distributed shared memory.
//
//   warp 0      TMA producer: per 64-key chunk (two pages) the K and V rows of this
//               kv head, two 64-column boxes each with 128-byte swizzle, into a
//               3-stage ring (full / empty mbarriers).
//   warp 1      TMEM owner and MMA issuer (one thread):
//                 S_j = Q K_j^T     M=128, N=64, K=128  (Q, K both K-major)
//                 O  += P_j V_j     M=128, N=128, K=64  (P K-major, V MN-major)
//               S is double-buffered in TMEM (columns 0-63 / 64-127), O lives in
//               columns 128-255.  S_{j+1} is issued before O += P_j V_j, so the
//               softmax of chunk j+1 overlaps the P V product of chunk j.
//   warps 2-5   one thread per query row (TMEM lane): load the row of S, mask,
//               online softmax in the log2 domain, write P (bf16, K-major SW128)
//               to shared memory, arrive.  The running maximum is only raised when
//               a chunk's maximum exceeds it by more than 8 (a factor of 256), so
//               the O rescale (TMEM load, scale, store) is rare; it waits for the
//               previous P V product first.  Rows past the sequence end in the last
//               chunk are zeroed in the V stage before P V (their probabilities are
//               exactly zero, but 0 x a non-finite stale value is not).
// Query rows of one (sequence, kv head) are flattened token-major (row = token * G
// + head_in_group), as in the kernels above.  Every wait is bounded.
namespace tca {
constexpr int kRows = 128;
constexpr int kNC = 64;                         // keys per chunk (two 32-key pages)
constexpr int kStages = 4;
constexpr int kBox = kRows * 128;               // 128 rows x 64 bf16 columns, SW128: 16 KB
constexpr int kQBytes = 2 * kBox;               // Q tile: two column boxes
constexpr int kKVBox = kNC * 128;               // 64 keys x 64 columns: 8 KB
constexpr int kPageBox = kPage * 128;           // 32 keys x 64 columns: 4 KB (one TMA box)
constexpr int kStageBytes = 4 * kKVBox;         // K lo | K hi | V lo | V hi
constexpr int kPBytes = kRows * 128;            // P tile: 128 rows x 64 keys bf16
constexpr int kOffKV = kQBytes;
constexpr int kOffP = kOffKV + kStages * kStageBytes;
constexpr int kOffBar = kOffP + 2 * kPBytes;
constexpr int kNumBars = 14;
constexpr int kOffMisc = kOffBar + 16 * 8;
constexpr int kOffML = kOffMisc + 16;
constexpr int kSmem = 1024 + kOffML + 2 * kRows * 4;
constexpr int kThreads = 192;
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t kColO = 128;
constexpr int kMergeRow = 132;                  // fp32 row of the cluster merge buffer
constexpr float kRescaleLog2 = 8.0f;
constexpr int kMaxSplits = 8;
constexpr uint32_t kIdescS = idesc_bf16_f32(kRows, kNC);
constexpr uint32_t kIdescPV = idesc_bf16_f32(kRows, kD) | (1u << 16);   // B (V) MN-major
static_assert(kRows * kMergeRow * 4 <= kStages * kStageBytes, "merge buffer reuses the KV ring");

// Timeline slots per traced CTA (the first kTraceCtas CTAs of the grid): 0 entry,
// 1 after set-up, then per chunk j < 24: 2+j producer issued, 26+j S issued,
// 50+j P arrived at the MMA issuer, 74+j S seen by softmax warp 2, 98+j P written
// by softmax warp 2; 122 softmax done, 123 exit.
constexpr int kTraceSlots = 128;
constexpr int kTraceCtas = 8;
constexpr int kTraceChunks = 24;

__device__ __forceinline__ uint32_t sw128_row_chunk(int row, int chunk) {
  return (row >> 3) * 1024 + (row & 7) * 128 + (((chunk ^ row) & 7) << 4);
}

// Non-blocking test of one mbarrier phase (the MMA issuer polls two barriers).
__device__ __forceinline__ bool mbar_ready(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// 2^x with the hardware approximation (flush-to-zero); probabilities are rounded to
// bf16 right after, so its error (a few ulp of fp32) is far below what is kept.
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 32 lanes x 64 consecutive fp32 TMEM columns in one load, one wait.
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float (&v)[64]) {
  uint32_t r[64];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x64.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,"
      "%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,"
      "%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%64];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]),
        "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]),
        "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]),
        "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]),
        "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 64; ++i) v[i] = __uint_as_float(r[i]);
}
}  // namespace tca

template <bool kSplit>
__global__ void __launch_bounds__(tca::kThreads, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                   const AttnArgs a, int splits) {
  using namespace tca;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = base;
  uint8_t* sKV = base + kOffKV;
  uint8_t* sP = base + kOffP;
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + kOffBar);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;
  uint64_t* kv_empty = bars + 1 + kStages;
  uint64_t* s_full = bars + 1 + 2 * kStages;
  uint64_t* p_full = s_full + 2;
  // o_done[j & 1] completes when O += P_j V_j is done.  Two barriers alternate by
  // chunk so that every wait targets a phase at most one completion away: when the
  // softmax waits for product j, product j - 2 is known complete and product j + 2
  // cannot have been issued.
  uint64_t* o_done = p_full + 2;
  uint64_t* drain = o_done + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(base + kOffMisc);
  float* sm_m = reinterpret_cast<float*>(base + kOffML);
  float* sm_l = sm_m + kRows;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (threadIdx.x == 0 && a.trace != nullptr && blockIdx.y * gridDim.x + blockIdx.x < tca::kTraceCtas)
    a.trace[(blockIdx.y * gridDim.x + blockIdx.x) * tca::kTraceSlots] = global_ns();
  if (threadIdx.x == 0) {
    mbar_init(q_full, 4);
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4);
    }
    mbar_init(&o_done[0], 1);
    mbar_init(&o_done[1], 1);
    mbar_init(drain, 1);
    fence_barrier_init();
    prefetch_tmap(&kmap);
    prefetch_tmap(&vmap);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();
  pdl_trigger();
  const int cta = blockIdx.y * gridDim.x + blockIdx.x;
  unsigned long long* trace = (a.trace != nullptr && cta < kTraceCtas) ? a.trace + cta * kTraceSlots : nullptr;
  auto stamp = [&](int slot) {
    if (trace != nullptr) trace[slot] = global_ns();
  };
  if (threadIdx.x == 0) stamp(1);

  const int S = kSplit ? splits : 1;
  const int split = kSplit ? static_cast<int>(cluster_ctarank()) : 0;
  const int tile = blockIdx.x / S, g = blockIdx.y;
  const int b = a.tile_seq[tile];
  const int row0 = a.tile_row0[tile];
  const int qlen = a.q_len[b], kvlen = a.kv_len[b], q0 = a.q_start[b];
  const int bidir = a.mode[b];
  const int rows = qlen * a.G;
  const int last_row = min(rows - 1, row0 + kRows - 1);
  const int max_key = bidir ? kvlen : min(kvlen, kvlen - qlen + last_row / a.G + 1);
  const int nch_all = (max(max_key, 0) + kNC - 1) / kNC;
  const int per = (nch_all + S - 1) / S;
  const int c0 = min(nch_all, split * per);
  const int n = min(nch_all, c0 + per) - c0;
  const int* tbl = a.table + static_cast<long long>(b) * a.table_stride;

  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    if (lane == 0) {
      int issued = 0;
      for (int j = 0; j < n; ++j) {
        const int s = j % kStages;
        if (!mbar_wait(&kv_empty[s], ((j / kStages) & 1) ^ 1, a.status, kErrTmaWait)) break;
        const int key0 = (c0 + j) * kNC;
        const int pages = min(2, (kvlen - key0 + kPage - 1) / kPage);
        uint8_t* dst = sKV + s * kStageBytes;
        mbar_arrive_expect_tx(&kv_full[s], pages * 4 * kPageBox);
        for (int pi = 0; pi < pages; ++pi) {
          const int y = (tbl[key0 / kPage + pi] * a.Hkv + g) * kPage;
          tma_load_2d(dst + pi * kPageBox, &kmap, 0, y, &kv_full[s]);
          tma_load_2d(dst + kKVBox + pi * kPageBox, &kmap, 64, y, &kv_full[s]);
          tma_load_2d(dst + 2 * kKVBox + pi * kPageBox, &vmap, 0, y, &kv_full[s]);
          tma_load_2d(dst + 3 * kKVBox + pi * kPageBox, &vmap, 64, y, &kv_full[s]);
        }
        issued = j + 1;
        if (j < kTraceChunks) stamp(2 + j);
      }
      // Copies still in flight must land before the CTA exits: wait for the last
      // stages' phases (their stage was not reused, so the parity is unambiguous).
      for (int j = max(0, issued - kStages); j < issued; ++j)
        mbar_wait(&kv_full[j % kStages], (j / kStages) & 1, a.status, kErrTmaWait);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0 && n > 0) {
      const uint32_t qa = smem_u32(sQ);
      auto issue_s = [&](int j) {
        const uint32_t kb = smem_u32(sKV + (j % kStages) * kStageBytes);
        const uint32_t d = tmem + (j & 1) * kNC;
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk) {
          const uint64_t ad = sdesc_k_sw128(qa + (kk >> 2) * kBox + (kk & 3) * 32);
          const uint64_t bd = sdesc_k_sw128(kb + (kk >> 2) * kKVBox + (kk & 3) * 32);
          tc_mma_bf16(d, ad, bd, kIdescS, kk > 0 ? 1u : 0u);
        }
        tc_commit(&s_full[j & 1]);
        if (j < kTraceChunks) stamp(26 + j);
      };
      auto issue_pv = [&](int j) {
        const int s = j % kStages;
        const uint32_t vb = smem_u32(sKV + s * kStageBytes + 2 * kKVBox);
        const uint32_t pb = smem_u32(sP + (j & 1) * kPBytes);
#pragma unroll
        for (int kk = 0; kk < kNC / 16; ++kk) {
          const uint64_t ad = sdesc_k_sw128(pb + kk * 32);
          const uint64_t bd = sdesc_mn_sw128(vb + kk * 16 * 128, kKVBox, 1024);
          tc_mma_bf16(tmem + kColO, ad, bd, kIdescPV, (j > 0 || kk > 0) ? 1u : 0u);
        }
        tc_commit(&kv_empty[s]);
        tc_commit(&o_done[j & 1]);
      };
      // Issue whichever product is ready, never holding a P V product (which frees a
      // KV stage) behind a K tile that is still in flight.  S_ns may be issued once the
      // softmax has read S_{ns-2} (same TMEM buffer), i.e. once P_{ns-2} arrived, which
      // holds when ns - np < 2; P_np needs S_np, so np < ns.
      bool ok = mbar_wait(q_full, 0, a.status, kErrMmaWait);
      tc_fence_after();
      int ns = 0, np = 0;
      unsigned long long idle_since = 0;
      while (ok && np < n) {
        if (ns < n && ns - np < 2 && mbar_ready(&kv_full[ns % kStages], (ns / kStages) & 1)) {
          tc_fence_after();
          issue_s(ns);
          ++ns;
          idle_since = 0;
        } else if (np < ns && mbar_ready(&p_full[np & 1], (np >> 1) & 1)) {
          tc_fence_after();
          if (np < kTraceChunks) stamp(50 + np);
          issue_pv(np);
          ++np;
          idle_since = 0;
        } else if (idle_since == 0) {
          idle_since = global_ns();
        } else if (global_ns() - idle_since > kWaitLimitNs) {
          record_error(a.status, kErrMmaWait);
          ok = false;
        }
      }
      // every issued MMA completes before TMEM can be released
      tc_commit(drain);
      mbar_wait(drain, 0, a.status, kErrMmaWait);
    }
  } else {
    // ---------------------------------------------------------------- softmax
    const int quarter = warp & 3;
    const int t = quarter * 32 + lane;
    const int row = row0 + t;
    const bool valid_row = row < rows;
    const int qpos = valid_row ? kvlen - qlen + row / a.G : -1;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    {
      const uint4* src = nullptr;
      if (valid_row) {
        const int tok = row / a.G, head = g * a.G + row % a.G;
        src = reinterpret_cast<const uint4*>(a.q + (static_cast<long long>(q0 + tok) * a.Hq + head) * kD);
      }
#pragma unroll
      for (int c = 0; c < kD / 8; ++c) {
        const uint4 v = valid_row ? src[c] : make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4*>(sQ + (c >> 3) * kBox + sw128_row_chunk(t, c & 7)) = v;
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(q_full);
    }
    float m = -INFINITY, l = 0.0f;
    bool ok = true;
    for (int j = 0; j < n; ++j) {
      ok = __all_sync(0xffffffffu, mbar_wait(&s_full[j & 1], (j >> 1) & 1, a.status, kErrEpilogueWait));
      if (!ok) break;
      tc_fence_after();
      if (warp == 2 && lane == 0 && j < kTraceChunks) stamp(74 + j);
      float sc[kNC];
      tmem_ld64(tmem + lane_base + (j & 1) * kNC, sc);
      const int key0 = (c0 + j) * kNC;
      // eight independent max chains, then a short tree
      float mp[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) mp[k] = -INFINITY;
      if (valid_row && key0 + kNC <= kvlen && (bidir || key0 + kNC - 1 <= qpos)) {
#pragma unroll
        for (int i = 0; i < kNC; ++i) {
          sc[i] *= a.scale_log2;
          mp[i & 7] = fmaxf(mp[i & 7], sc[i]);
        }
      } else {
#pragma unroll
        for (int i = 0; i < kNC; ++i) {
          const int key = key0 + i;
          const bool vis = valid_row && key < kvlen && (bidir || key <= qpos);
          sc[i] = vis ? sc[i] * a.scale_log2 : -INFINITY;
          mp[i & 7] = fmaxf(mp[i & 7], sc[i]);
        }
      }
      const float mx = fmaxf(fmaxf(fmaxf(mp[0], mp[1]), fmaxf(mp[2], mp[3])),
                             fmaxf(fmaxf(mp[4], mp[5]), fmaxf(mp[6], mp[7])));
      if (j == 0) {
        m = mx;
      } else {
        const bool need = mx > m + kRescaleLog2;
        if (__any_sync(0xffffffffu, need)) {
          const float mnew = need ? mx : m;
          const float corr = (m == -INFINITY) ? 0.0f : exp2f(m - mnew);
          // O holds the products of chunks < j once the previous P V product is done
          ok = __all_sync(0xffffffffu,
                          mbar_wait(&o_done[(j - 1) & 1], ((j - 1) >> 1) & 1, a.status, kErrEpilogueWait));
          if (!ok) break;
          tc_fence_after();
#pragma unroll
          for (int c = 0; c < kD / 32; ++c) {
            float o[32];
            tmem_ld32(tmem + lane_base + kColO + c * 32, o);
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] *= corr;
            tmem_st32(tmem + lane_base + kColO + c * 32, o);
          }
          l *= corr;
          m = mnew;
        }
      }
      if (key0 + kNC > kvlen) {
        // last chunk: zero the V rows past the sequence end (acquire the stage first;
        // its phase is complete and not yet reused, so this returns at once)
        const int s = j % kStages;
        mbar_wait(&kv_full[s], (j / kStages) & 1, a.status, kErrEpilogueWait);
        const int valid = max(0, kvlen - key0);
        uint8_t* v = sKV + s * kStageBytes + 2 * kKVBox;
        for (int c = t; c < 2 * kNC * 8; c += kRows) {
          const int box = c / (kNC * 8), r = (c / 8) % kNC, seg = c % 8;
          if (r >= valid) *reinterpret_cast<uint4*>(v + box * kKVBox + r * 128 + seg * 16) = make_uint4(0, 0, 0, 0);
        }
      }
      uint8_t* prow = sP + (j & 1) * kPBytes;
      // rows that see no key yet keep m = -inf: shift by 0 instead (every score is -inf, 2^-inf = 0)
      const float shift = (m == -INFINITY) ? 0.0f : m;
      float sp[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) sp[k] = 0.0f;
#pragma unroll
      for (int c = 0; c < kNC / 8; ++c) {
        uint32_t w4[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float p0 = fast_exp2(sc[c * 8 + 2 * e] - shift);
          const float p1 = fast_exp2(sc[c * 8 + 2 * e + 1] - shift);
          sp[2 * e] += p0;
          sp[2 * e + 1] += p1;
          w4[e] = pack_bf16(p0, p1);
        }
        *reinterpret_cast<uint4*>(prow + sw128_row_chunk(t, c)) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
      }
      l += ((sp[0] + sp[1]) + (sp[2] + sp[3])) + ((sp[4] + sp[5]) + (sp[6] + sp[7]));
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[j & 1]);
      if (warp == 2 && lane == 0 && j < kTraceChunks) stamp(98 + j);
    }
    if (warp == 2 && lane == 0) stamp(122);
    const bool have = n > 0 && ok &&
                      __all_sync(0xffffffffu, mbar_wait(&o_done[(n - 1) & 1], ((n - 1) >> 1) & 1, a.status,
                                                        kErrEpilogueWait));
    if (have) tc_fence_after();
    if (!kSplit) {
      if (have) {
        const float inv = l > 0.0f ? 1.0f / l : 0.0f;
        __nv_bfloat16* dst = nullptr;
        if (valid_row) {
          const int tok = row / a.G, head = g * a.G + row % a.G;
          dst = a.out + (static_cast<long long>(q0 + tok) * a.Hq + head) * kD;
        }
#pragma unroll
        for (int c = 0; c < kD / 32; ++c) {
          float o[32];
          tmem_ld32(tmem + lane_base + kColO + c * 32, o);
          if (valid_row) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              uint4 w;
              w.x = pack_bf16(o[8 * e] * inv, o[8 * e + 1] * inv);
              w.y = pack_bf16(o[8 * e + 2] * inv, o[8 * e + 3] * inv);
              w.z = pack_bf16(o[8 * e + 4] * inv, o[8 * e + 5] * inv);
              w.w = pack_bf16(o[8 * e + 6] * inv, o[8 * e + 7] * inv);
              *reinterpret_cast<uint4*>(dst + c * 32 + 8 * e) = w;
            }
          }
        }
      } else if (valid_row && n == 0) {
        // no visible key (empty sequence): the output row is zero
        const int tok = row / a.G, head = g * a.G + row % a.G;
        uint4* dst = reinterpret_cast<uint4*>(a.out + (static_cast<long long>(q0 + tok) * a.Hq + head) * kD);
        for (int c = 0; c < kD / 8; ++c) dst[c] = make_uint4(0, 0, 0, 0);
      }
    } else {
      // this CTA's partial state for the cluster merge (the KV ring is idle now)
      float* mo = reinterpret_cast<float*>(sKV) + t * kMergeRow;
      if (have) {
#pragma unroll
        for (int c = 0; c < kD / 32; ++c) {
          float o[32];
          tmem_ld32(tmem + lane_base + kColO + c * 32, o);
#pragma unroll
          for (int e = 0; e < 8; ++e)
            *reinterpret_cast<float4*>(mo + c * 32 + 4 * e) = make_float4(o[4 * e], o[4 * e + 1], o[4 * e + 2], o[4 * e + 3]);
        }
      }
      sm_m[t] = have ? m : -INFINITY;
      sm_l[t] = have ? l : 0.0f;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
  if (kSplit) {
    cluster_sync();
    if (warp >= 2) {
      const float* mo0 = reinterpret_cast<const float*>(sKV);
      for (int r = split + S * (warp - 2); r < kRows; r += 4 * S) {
        const int row = row0 + r;
        if (row >= rows) break;
        float mk[kMaxSplits], wk[kMaxSplits];
        float M = -INFINITY, L = 0.0f;
#pragma unroll
        for (int k = 0; k < kMaxSplits; ++k) {
          mk[k] = k < S ? ld_dsmem_f32(map_shared_rank(smem_u32(sm_m + r), k)) : -INFINITY;
          M = fmaxf(M, mk[k]);
        }
#pragma unroll
        for (int k = 0; k < kMaxSplits; ++k) {
          wk[k] = (k >= S || mk[k] == -INFINITY) ? 0.0f : exp2f(mk[k] - M);
          if (wk[k] != 0.0f) L += wk[k] * ld_dsmem_f32(map_shared_rank(smem_u32(sm_l + r), k));
        }
        float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
        for (int k = 0; k < kMaxSplits; ++k) {
          if (wk[k] == 0.0f) continue;
          const float4 x = ld_dsmem_f4(map_shared_rank(smem_u32(mo0 + r * kMergeRow + lane * 4), k));
          acc.x += wk[k] * x.x;
          acc.y += wk[k] * x.y;
          acc.z += wk[k] * x.z;
          acc.w += wk[k] * x.w;
        }
        const float inv = L > 0.0f ? 1.0f / L : 0.0f;
        const int tok = row / a.G, head = g * a.G + row % a.G;
        __nv_bfloat16* dst = a.out + (static_cast<long long>(q0 + tok) * a.Hq + head) * kD + lane * 4;
        uint2 w;
        w.x = pack_bf16(acc.x * inv, acc.y * inv);
        w.y = pack_bf16(acc.z * inv, acc.w * inv);
        *reinterpret_cast<uint2*>(dst) = w;
      }
    }
    cluster_sync();   // peers read this CTA's shared memory until here
  }
  if (threadIdx.x == 0) stamp(123);
}

// 2-D view [pages * Hkv * P rows, D columns] of one cache, box_rows-key x 64-column boxes.
bool make_cache_map(CUtensorMap* map, const void* ptr, long long rows, int box_rows = kCh) {
  EncodeTiledFn fn = tensor_map_encoder();
  if (!fn || rows <= 0 || (reinterpret_cast<uintptr_t>(ptr) % 16)) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(kD), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(kD) * 2};
  cuuint32_t box[2] = {64, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int MT>
cudaError_t launch_tma(const AttentionProblem& p, const AttnArgs& a, dim3 grid, cudaStream_t stream) {
  CUtensorMap km, vm;
  const long long rows = static_cast<long long>(p.cache_pages) * p.Hkv * kPage;
  if (!make_cache_map(&km, p.k_cache, rows) || !make_cache_map(&vm, p.v_cache, rows)) return cudaErrorInvalidValue;
  static bool attr[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr[dev]) {
    cudaError_t e = cudaFuncSetAttribute(attn_tma_kernel<MT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         TmaSmem<MT>::kTotal);
    if (e != cudaSuccess) return e;
    cudaFuncSetAttribute(attn_tma_kernel<MT>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    attr[dev] = true;
  }
  return launch_pdl(attn_tma_kernel<MT>, grid, dim3(128 * MT), TmaSmem<MT>::kTotal, stream, km, vm, a);
}


cudaError_t launch_tc(const AttentionProblem& p, const AttnArgs& a, cudaStream_t stream) {
  const int S = p.kv_splits;
  if (S != 1 && S != 2 && S != 4 && S != 8) return cudaErrorInvalidValue;
  CUtensorMap km, vm;
  const long long rows = static_cast<long long>(p.cache_pages) * p.Hkv * kPage;
  if (!make_cache_map(&km, p.k_cache, rows, kPage) || !make_cache_map(&vm, p.v_cache, rows, kPage))
    return cudaErrorInvalidValue;
  static bool attr[2][64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  const int which = S > 1 ? 1 : 0;
  if (dev < 64 && !attr[which][dev]) {
    cudaError_t e = cudaFuncSetAttribute(S > 1 ? attn_tc_kernel<true> : attn_tc_kernel<false>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, tca::kSmem);
    if (e != cudaSuccess) return e;
    attr[which][dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.num_tiles * S, p.Hkv);
  cfg.blockDim = dim3(tca::kThreads);
  cfg.dynamicSmemBytes = tca::kSmem;
  cfg.stream = stream;
  cudaLaunchAttribute at[2];
  int na = 0;
  if (S > 1) {
    at[na].id = cudaLaunchAttributeClusterDimension;
    at[na].val.clusterDim.x = S;
    at[na].val.clusterDim.y = 1;
    at[na].val.clusterDim.z = 1;
    ++na;
  }
  if (pdl_enabled()) {
    at[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = at;
  cfg.numAttrs = na;
  return S > 1 ? cudaLaunchKernelEx(&cfg, attn_tc_kernel<true>, km, vm, a, S)
               : cudaLaunchKernelEx(&cfg, attn_tc_kernel<false>, km, vm, a, 1);
}
}  // namespace

unsigned long long*& attention_trace_buffer() {
  static unsigned long long* buf = nullptr;
  return buf;
}

cudaError_t attention_launch(const AttentionProblem& p, cudaStream_t stream) {
  if (p.head_dim != kD || p.page_size != kPage || p.Hkv <= 0 || p.Hq % p.Hkv) return cudaErrorInvalidValue;
  AttnArgs a{};
  a.q = p.q;
  a.k_cache = p.k_cache;
  a.v_cache = p.v_cache;
  a.table = p.table;
  a.table_stride = p.table_stride;
  a.q_start = p.q_start;
  a.q_len = p.q_len;
  a.kv_len = p.kv_len;
  a.mode = p.mode;
  a.tile_seq = p.tile_seq;
  a.tile_row0 = p.tile_row0;
  a.out = p.out;
  a.Hq = p.Hq;
  a.Hkv = p.Hkv;
  a.G = p.Hq / p.Hkv;
  a.scale_log2 = p.scale * 1.4426950408889634f;
  a.status = p.status;
  a.trace = attention_trace_buffer();
  a.k_lo = p.k_lo;
  a.o_f32 = p.o_f32;
  a.lse_out = p.lse_out;
  a.prior_o = p.prior_o;
  a.prior_lse = p.prior_lse;
  const bool two_pass = p.k_lo || p.o_f32 || p.lse_out || p.prior_o || p.prior_lse;
  if (two_pass && ((p.tile_rows != 16 && p.tile_rows != 32) || (p.prior_o == nullptr) != (p.prior_lse == nullptr)))
    return cudaErrorInvalidValue;    // the key-range options are implemented by the TMA kernel
  if (p.num_tiles <= 0) return cudaSuccess;
  dim3 grid(p.num_tiles, p.Hkv);
  if (p.tile_rows == 128) {
    return launch_tc(p, a, stream);
  } else if (p.tile_rows == 64) {
    return launch_pdl(attn_rows_kernel, grid, dim3(128), 0, stream, a);
  } else if (p.tile_rows == 16) {
    return launch_tma<1>(p, a, grid, stream);
  } else if (p.tile_rows == 32) {
    return launch_tma<2>(p, a, grid, stream);
  } else {
    return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace osb
