// Vocabulary-wide sampling, scoring and speculative correction kernels.
//
//  * sample_kernel: one CTA per row.  A single pass computes the row max and
//    the two log-normalisers log sum exp(l) and log sum exp(l / T) with online
//    rescaling; a second pass draws the token by inverse CDF with a float64
//    prefix sum (segment sums per thread + block scan), so a request-local
//    uniform selects the same token whatever the batch shape.  It returns the
//    token, its log-probability under the sampling policy (temperature T) and
//    under the reference policy (T = 1) from the same logits.
//    Reference: src/inference_scaling/arllm/backends/transformers_backend.py:323-348
//    (policy log-softmax) and :895-906 (float64 inverse CDF).
//  * row_stats_kernel: the same statistics for every row without sampling, plus
//    the gathered log-probabilities of given target tokens (sequence scoring,
//    transformers_backend.py:1330-1411).
//  * gumbel_sample_kernel: exponential-race / Gumbel-max draft sampling
//    (online-speculation/src/blockspec/sampling_execution.py:15-17).
//  * spec_verify_kernel: exact p/q block correction with the positive residual
//    (sampling_execution.py:20-41, sampling.py:112-146): accept-prefix count,
//    residual or bonus draw, validity flag and both log-probabilities of every
//    emitted token, in one launch per batch.
// Random numbers come from a counter-based Philox-4x32-10 generator (Salmon et
// al., "Parallel random numbers: as easy as 1, 2, 3", SC 2011) keyed by a
// per-request seed, so draws do not depend on scheduling.
#include "common.cuh"
#include "sampling.h"

namespace osb {
namespace {

constexpr int kThreads = 1024;

// ---------------------------------------------------------------- Philox ----
__device__ __forceinline__ uint4 philox4x32(uint4 ctr, uint2 key) {
  const uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u, W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;
#pragma unroll
  for (int i = 0; i < 10; ++i) {
    const uint32_t hi0 = __umulhi(M0, ctr.x), lo0 = M0 * ctr.x;
    const uint32_t hi1 = __umulhi(M1, ctr.z), lo1 = M1 * ctr.z;
    ctr = make_uint4(hi1 ^ ctr.y ^ key.x, lo1, hi0 ^ ctr.w ^ key.y, lo0);
    key.x += W0;
    key.y += W1;
  }
  return ctr;
}

// Uniform in the open interval (0, 1) from 24 random bits.
__device__ __forceinline__ float u01(uint32_t x) { return (static_cast<float>(x >> 8) + 0.5f) * (1.0f / 16777216.0f); }

// Four uniforms for (seed, stream, index): stream separates uses, index counts.
__device__ __forceinline__ float4 uniform4(unsigned long long seed, uint32_t stream, uint32_t hi, uint32_t index) {
  const uint4 r = philox4x32(make_uint4(index, hi, stream, 0x5eedu),
                             make_uint2(static_cast<uint32_t>(seed), static_cast<uint32_t>(seed >> 32)));
  return make_float4(u01(r.x), u01(r.y), u01(r.z), u01(r.w));
}

// (score, column) -> 64-bit key whose signed order is (score, then lower column):
// monotone bit pattern of the float in the high word, complemented column in
// the low word, top bit flipped so that a signed 64-bit maximum (NCCL MAX on
// int64) picks the same winner as the unsharded argmax.
__device__ __forceinline__ uint32_t order_key(float x) {
  const uint32_t b = __float_as_uint(x);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__device__ __forceinline__ unsigned long long pack_argmax_key(float score, int column) {
  const uint32_t ord = order_key(score);
  const unsigned long long k =
      (static_cast<unsigned long long>(ord) << 32) | (0xFFFFFFFFu - static_cast<uint32_t>(column));
  return k ^ 0x8000000000000000ull;
}

// ------------------------------------------------------- block reductions ----
template <typename T>
__device__ __forceinline__ T warp_reduce_sum(T v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

struct MaxSum2 {
  float m;   // running max of raw logits
  float s1;  // sum exp(l - m)
  float sT;  // sum exp((l - m) * invT)
};

__device__ __forceinline__ void ms_add(MaxSum2& a, float l, float invT) {
  if (l > a.m) {
    const float d = a.m - l;  // <= 0 (or -inf)
    a.s1 = a.s1 * expf(d) + 1.0f;
    a.sT = a.sT * expf(d * invT) + 1.0f;
    a.m = l;
  } else {
    const float d = l - a.m;
    a.s1 += expf(d);
    a.sT += expf(d * invT);
  }
}

__device__ __forceinline__ MaxSum2 ms_merge(MaxSum2 a, MaxSum2 b, float invT) {
  if (b.m > a.m) {
    MaxSum2 t = a;
    a = b;
    b = t;
  }
  if (b.m == -INFINITY) return a;
  const float d = b.m - a.m;
  a.s1 += b.s1 * expf(d);
  a.sT += b.sT * expf(d * invT);
  return a;
}

// Block-reduced (max, sum exp, sum exp at 1/T) of columns [c0, c1) of a row.
// c0 must be a multiple of 4.  All threads get the result.
__device__ MaxSum2 row_partial(const float* __restrict__ row, int c0, int c1, float invT) {
  __shared__ MaxSum2 red[32];
  MaxSum2 a{-INFINITY, 0.0f, 0.0f};
  const bool vec = (reinterpret_cast<uintptr_t>(row) % 16 == 0) && (c1 % 4 == 0);
  if (vec) {
    const float4* r4 = reinterpret_cast<const float4*>(row);
    for (int i = c0 / 4 + threadIdx.x; i < c1 / 4; i += blockDim.x) {
      const float4 v = r4[i];
      ms_add(a, v.x, invT);
      ms_add(a, v.y, invT);
      ms_add(a, v.z, invT);
      ms_add(a, v.w, invT);
    }
  } else {
    for (int i = c0 + threadIdx.x; i < c1; i += blockDim.x) ms_add(a, row[i], invT);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    MaxSum2 b{__shfl_xor_sync(0xffffffffu, a.m, o), __shfl_xor_sync(0xffffffffu, a.s1, o),
              __shfl_xor_sync(0xffffffffu, a.sT, o)};
    a = ms_merge(a, b, invT);
  }
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (lane == 0) red[warp] = a;
  __syncthreads();
  if (warp == 0) {
    MaxSum2 b = lane < blockDim.x / 32 ? red[lane] : MaxSum2{-INFINITY, 0.0f, 0.0f};
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      MaxSum2 c{__shfl_xor_sync(0xffffffffu, b.m, o), __shfl_xor_sync(0xffffffffu, b.s1, o),
                __shfl_xor_sync(0xffffffffu, b.sT, o)};
      b = ms_merge(b, c, invT);
    }
    if (lane == 0) red[0] = b;
  }
  __syncthreads();
  const MaxSum2 r = red[0];
  __syncthreads();
  return r;
}

// Row statistics: max, lse at T=1, lse at temperature T.  All threads get the result.
__device__ void row_stats(const float* __restrict__ row, int V, float invT, float& mx, float& lse1, float& lseT) {
  const MaxSum2 r = row_partial(row, 0, V, invT);
  mx = r.m;
  lse1 = r.m + logf(r.s1);
  lseT = r.m * invT + logf(r.sT);
}

// Block-wide exclusive scan of one double per thread; `total` gets the sum.
__device__ double block_exclusive_scan(double v, double& total) {
  __shared__ double wsum[33];
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int nwarps = blockDim.x / 32;
  double inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double n = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += n;
  }
  if (lane == 31) wsum[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    const double w = lane < nwarps ? wsum[lane] : 0.0;
    double winc = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const double n = __shfl_up_sync(0xffffffffu, winc, o);
      if (lane >= o) winc += n;
    }
    if (lane < nwarps) wsum[lane] = winc - w;
    if (lane == 31) wsum[32] = winc;
  }
  __syncthreads();
  const double res = wsum[warp] + inc - v;
  total = wsum[32];
  __syncthreads();
  return res;
}


// ------------------------------------------------------ truncated policies ----
// A truncated policy keeps the columns whose tempered logit z = l / T is at least
// a per-row threshold key: the k-th largest z (top-k), then, inside that set, the
// smallest z at which the descending cumulative mass first exceeds top_p of the
// set's mass (top-p).  Columns tied with the threshold all stay.  The threshold is
// found by a radix select from the most significant byte of the order-preserving
// key of z: per byte one pass histograms the columns that share the bytes fixed so
// far (counts for top-k, masses exp(z - zmax) for top-p) and one warp scans the 256
// bins from the top for the bin where the running total reaches the target.
// Histogram bins are fp32 (counts are exact below 2^24 columns).

template <bool kMass>
__device__ uint32_t radix_select_desc(const float* __restrict__ row, int V, float invT, float zmax, uint32_t keep_from,
                                      float target) {
  __shared__ float hist[256];
  __shared__ uint32_t s_prefix;
  __shared__ float s_target;
  uint32_t prefix = 0, fixed = 0;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0.0f;
    __syncthreads();
    for (int v = threadIdx.x; v < V; v += blockDim.x) {
      const float z = row[v] * invT;
      const uint32_t key = order_key(z);
      if (key < keep_from || (key & fixed) != prefix) continue;
      atomicAdd(&hist[(key >> shift) & 0xFFu], kMass ? expf(z - zmax) : 1.0f);
    }
    __syncthreads();
    if (threadIdx.x < 32) {
      const int lane = threadIdx.x;
      float mine[8];
      float local = 0.0f;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        mine[j] = hist[255 - 8 * lane - j];   // lane 0 holds the top bins
        local += mine[j];
      }
      float inc = local;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float n = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += n;
      }
      const bool reached = kMass ? inc > target : inc >= target;
      const unsigned crossing = __ballot_sync(0xffffffffu, reached);
      const unsigned nonempty = __ballot_sync(0xffffffffu, local > 0.0f);
      // no bin reaches the target (rounding): keep every column of this prefix
      const bool keep_all = crossing == 0u;
      const int owner = keep_all ? (nonempty ? 31 - __clz(nonempty) : 31) : __ffs(crossing) - 1;
      if (lane == owner) {
        float before = inc - local;
        int pick = 7;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const bool hit = keep_all ? false : (kMass ? before + mine[j] > target : before + mine[j] >= target);
          if (hit) {
            pick = j;
            break;
          }
          if (keep_all && mine[j] > 0.0f) pick = j;
          before += keep_all ? 0.0f : mine[j];
        }
        s_prefix = prefix | (static_cast<uint32_t>(255 - 8 * lane - pick) << shift);
        s_target = target - before;
      }
    }
    __syncthreads();
    prefix = s_prefix;
    target = s_target;
    fixed |= 0xFFu << shift;
    __syncthreads();
  }
  return prefix;
}

// Block sum of exp(z - zmax) over columns with key >= keep_from (all threads get it).
__device__ float kept_mass(const float* __restrict__ row, int V, float invT, float zmax, uint32_t keep_from) {
  __shared__ float red[32];
  float s = 0.0f;
  for (int v = threadIdx.x; v < V; v += blockDim.x) {
    const float z = row[v] * invT;
    if (order_key(z) >= keep_from) s += expf(z - zmax);
  }
  s = warp_reduce_sum(s);
  if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : 0.0f;
    t = warp_reduce_sum(t);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const float total = red[0];
  __syncthreads();
  return total;
}

// Threshold key and log-normaliser of the kept set of a truncated policy.
// zmax = max_v l_v * invT.  Returns keep_from 0 (everything kept) when neither filter binds.
__device__ void truncation(const float* __restrict__ row, int V, float invT, float zmax, int top_k, float top_p,
                           uint32_t& keep_from, float& lse_kept) {
  keep_from = 0u;
  if (top_k > 0 && top_k < V) keep_from = radix_select_desc<false>(row, V, invT, zmax, 0u, static_cast<float>(top_k));
  float mass = kept_mass(row, V, invT, zmax, keep_from);
  if (top_p < 1.0f) {
    keep_from = radix_select_desc<true>(row, V, invT, zmax, keep_from, top_p * mass);
    mass = kept_mass(row, V, invT, zmax, keep_from);
  }
  lse_kept = zmax + logf(mass);
}

__global__ void __launch_bounds__(kThreads) sample_kernel(SampleArgs a) {
  pdl_wait();
  pdl_trigger();
  const int r = blockIdx.x;
  const float* row = a.logits + r * a.ld;
  const float invT = a.inv_temp ? a.inv_temp[r] : 1.0f;
  float mx, lse1, lseT;
  row_stats(row, a.V, invT, mx, lse1, lseT);
  const int top_k = a.top_k ? a.top_k[r] : 0;
  const float top_p = a.top_p ? a.top_p[r] : 1.0f;
  uint32_t keep_from = 0u;
  if ((top_k > 0 && top_k < a.V) || top_p < 1.0f) truncation(row, a.V, invT, mx * invT, top_k, top_p, keep_from, lseT);
  // policy mass of column v: exp(z - lseT) on the kept columns, zero elsewhere
  auto mass = [&](int v) -> double {
    const float z = row[v] * invT;
    return order_key(z) >= keep_from ? static_cast<double>(expf(z - lseT)) : 0.0;
  };
  const double u = a.uniforms[r * a.uniform_stride];
  // contiguous segment per thread
  const int seg = (a.V + blockDim.x - 1) / blockDim.x;
  const int b0 = min(a.V, static_cast<int>(threadIdx.x) * seg);
  const int b1 = min(a.V, b0 + seg);
  double s = 0.0;
  for (int v = b0; v < b1; ++v) s += mass(v);
  double total;
  const double excl = block_exclusive_scan(s, total);
  __shared__ int chosen;
  if (threadIdx.x == 0) chosen = a.V - 1;
  __syncthreads();
  const bool last_thread = (b1 == a.V && b0 < b1);
  if (b0 < b1 && (excl < u || b0 == 0) && (u <= excl + s || last_thread)) {
    double c = excl;
    int tok = b1 - 1;
    for (int v = b0; v < b1; ++v) {
      c += mass(v);
      if (c >= u) {
        tok = v;
        break;
      }
    }
    atomicMin(&chosen, tok);
  }
  __syncthreads();
  __shared__ double code_lo, code_mass;
  if (a.arith != nullptr && a.next_uniforms != nullptr && a.arith[r]) {
    // the owner of the chosen token recomputes its cumulative interval
    const int tok = chosen;
    if (b0 <= tok && tok < b1) {
      double c = excl;
      for (int v = b0; v < tok; ++v) c += mass(v);
      code_lo = c;
      code_mass = mass(tok);
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    const int tok = chosen;
    a.tokens[r] = tok;
    const float l = row[tok];
    // a column outside the kept set is only reached when u exceeds the fp64 total (it has no mass)
    if (a.logq) a.logq[r] = order_key(l * invT) >= keep_from ? l * invT - lseT : -INFINITY;
    if (a.logp) a.logp[r] = l - lse1;
    if (a.arith != nullptr && a.next_uniforms != nullptr && a.arith[r]) {
      double nu = code_mass > 0.0 ? (u - code_lo) / code_mass : 0.5;
      nu = fmin(fmax(nu, 0.0), 0.99999999999999989);   // largest double below one
      a.next_uniforms[r * a.uniform_stride] = nu;
    }
  }
}

__global__ void __launch_bounds__(kThreads) row_stats_kernel(RowStatsArgs a) {
  pdl_wait();
  pdl_trigger();
  const int r = blockIdx.x;
  const float* row = a.logits + r * a.ld;
  const float invT = a.inv_temp ? a.inv_temp[r] : 1.0f;
  float lse1, lseT;
  uint32_t keep_from = 0u;
  if (a.split > 1) {
    // This CTA's column chunk; the last CTA of the row to arrive merges the chunks
    // in chunk order (independent of arrival order) and finishes the row.
    const int c0 = blockIdx.y * a.chunk;
    const MaxSum2 part = row_partial(row, c0, min(a.V, c0 + a.chunk), invT);
    __shared__ int last;
    if (threadIdx.x == 0) {
      float* slot = a.part + (static_cast<long long>(r) * kRowStatsMaxSplit + blockIdx.y) * 3;
      slot[0] = part.m;
      slot[1] = part.s1;
      slot[2] = part.sT;
      __threadfence();
      last = atomicAdd(a.count + r, 1) == a.split - 1;
    }
    __syncthreads();
    if (!last) return;
    if (threadIdx.x != 0) return;
    __threadfence();
    const float* slots = a.part + static_cast<long long>(r) * kRowStatsMaxSplit * 3;
    MaxSum2 tot{-INFINITY, 0.0f, 0.0f};
    for (int k = 0; k < a.split; ++k)
      tot = ms_merge(tot, MaxSum2{__ldcg(slots + 3 * k), __ldcg(slots + 3 * k + 1), __ldcg(slots + 3 * k + 2)}, invT);
    a.count[r] = 0;
    lse1 = tot.m + logf(tot.s1);
    lseT = tot.m * invT + logf(tot.sT);
  } else {
    float mx;
    row_stats(row, a.V, invT, mx, lse1, lseT);
    const int top_k = a.top_k ? a.top_k[r] : 0;
    const float top_p = a.top_p ? a.top_p[r] : 1.0f;
    if ((top_k > 0 && top_k < a.V) || top_p < 1.0f) truncation(row, a.V, invT, mx * invT, top_k, top_p, keep_from, lseT);
  }
  if (threadIdx.x == 0) {
    if (a.lse1) a.lse1[r] = lse1;
    if (a.lseT) a.lseT[r] = lseT;
    if (a.targets) {
      const int t = a.targets[r];
      const float l = (t >= 0 && t < a.V) ? row[t] : -INFINITY;
      if (a.logp) a.logp[r] = l - lse1;
      if (a.logq) a.logq[r] = (t >= 0 && t < a.V && order_key(l * invT) >= keep_from) ? l * invT - lseT : -INFINITY;
    }
  }
}

// Gumbel-max sampling at temperature T: argmax_v (l_v / T + G_v).
__global__ void __launch_bounds__(kThreads) gumbel_sample_kernel(GumbelArgs a) {
  pdl_wait();
  pdl_trigger();
  const int r = blockIdx.x;
  const int c_begin = blockIdx.y * a.chunk;                  // this CTA's columns of the row
  const int c_end = min(a.V, c_begin + a.chunk);
  const float* row = a.logits + r * a.ld;
  const float invT = a.inv_temp ? a.inv_temp[r] : 1.0f;
  const unsigned long long seed = a.seeds[a.seed_index ? a.seed_index[r] : r];
  const uint32_t stream = a.streams ? static_cast<uint32_t>(a.streams[r]) : 0u;
  const uint32_t hi = static_cast<uint32_t>(a.salt) ^ (static_cast<uint32_t>(a.row_in_seq ? a.row_in_seq[r] : 0) << 24);
  float best = -INFINITY;
  int besti = 0x7fffffff;
  const int g0 = a.v_lo >> 2;   // v_lo is a multiple of 4: groups of four columns keep their noise
  for (int i = c_begin / 4 + threadIdx.x; i * 4 < c_end; i += blockDim.x) {
    const float4 u = uniform4(seed, stream, hi, static_cast<uint32_t>(g0 + i));
    const float uu[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int v = i * 4 + j;
      if (v < c_end) {
        const float g = -__logf(-__logf(uu[j]));
        const float sc = row[v] * invT + g;
        if (sc > best || (sc == best && v < besti)) {
          best = sc;
          besti = v;
        }
      }
    }
  }
  __shared__ float sb[32];
  __shared__ int si[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, besti, o);
    if (ob > best || (ob == best && oi < besti)) {
      best = ob;
      besti = oi;
    }
  }
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (lane == 0) {
    sb[warp] = best;
    si[warp] = besti;
  }
  __syncthreads();
  if (warp == 0) {
    best = lane < blockDim.x / 32 ? sb[lane] : -INFINITY;
    besti = lane < blockDim.x / 32 ? si[lane] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, besti, o);
      if (ob > best || (ob == best && oi < besti)) {
        best = ob;
        besti = oi;
      }
    }
    if (lane == 0) {
      if (a.split <= 1) {
        if (a.keys != nullptr) a.keys[r] = pack_argmax_key(best, a.v_lo + besti);
        else a.tokens[r] = a.v_lo + besti;
      } else {
        // unsigned order of the unflipped key = (score, then lower column)
        const unsigned long long k = pack_argmax_key(best, a.v_lo + besti) ^ 0x8000000000000000ull;
        atomicMax(a.row_best + r, k);
        __threadfence();
        if (atomicAdd(a.row_count + r, 1) == a.split - 1) {
          __threadfence();
          const unsigned long long win = atomicExch(a.row_best + r, 0ull);   // read the winner, reset
          a.row_count[r] = 0;
          if (a.keys != nullptr) a.keys[r] = win ^ 0x8000000000000000ull;
          else a.tokens[r] = static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(win & 0xFFFFFFFFull));
        }
      }
    }
  }
}

// One CTA per sequence: n candidates, n draft rows, n + 1 target rows.
__global__ void __launch_bounds__(kThreads) spec_verify_kernel(SpecArgs a) {
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.x;
  const int n = a.n;
  const float invT = a.inv_temp ? a.inv_temp[b] : 1.0f;
  const unsigned long long seed = a.seeds[b];
  const uint32_t stream = a.streams ? static_cast<uint32_t>(a.streams[b]) : 0u;
  __shared__ int s_count, s_valid;
  __shared__ float s_lseT[16], s_lse1[16], s_lseQ[16];
  // statistics of the target rows and the draft rows
  if (a.lseT_target != nullptr) {
    if (threadIdx.x <= n) {
      s_lseT[threadIdx.x] = a.lseT_target[b * (n + 1) + threadIdx.x];
      s_lse1[threadIdx.x] = a.lse1_target[b * (n + 1) + threadIdx.x];
    }
    if (threadIdx.x < n) s_lseQ[threadIdx.x] = a.lseT_draft[b * n + threadIdx.x];
  } else for (int i = 0; i <= n; ++i) {
    float mx, l1, lT;
    row_stats(a.target + (static_cast<long long>(b) * (n + 1) + i) * a.ld_target, a.V, invT, mx, l1, lT);
    if (threadIdx.x == 0) {
      s_lseT[i] = lT;
      s_lse1[i] = l1;
    }
  }
  if (a.lseT_target == nullptr) for (int i = 0; i < n; ++i) {
    float mx, l1, lT;
    row_stats(a.draft + (static_cast<long long>(b) * n + i) * a.ld_draft, a.V, invT, mx, l1, lT);
    if (threadIdx.x == 0) s_lseQ[i] = lT;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int count = n, valid = 1;
    const float4 ua = uniform4(seed, stream, static_cast<uint32_t>(a.salt), 0x7fffffffu);
    const float us[4] = {ua.x, ua.y, ua.z, ua.w};
    for (int i = 0; i < n; ++i) {
      const int x = a.candidates[b * n + i];
      if (x < 0 || x >= (a.V_total > 0 ? a.V_total : a.V)) {
        valid = 0;
        count = i;
        break;
      }
      const float tl = a.cand_logits ? a.cand_logits[(b * n + i) * 2]
                                     : a.target[(static_cast<long long>(b) * (n + 1) + i) * a.ld_target + x];
      const float dl = a.cand_logits ? a.cand_logits[(b * n + i) * 2 + 1]
                                     : a.draft[(static_cast<long long>(b) * n + i) * a.ld_draft + x];
      const float lp = tl * invT - s_lseT[i];
      const float lq = dl * invT - s_lseQ[i];
      const float ratio = __expf(fminf(lp - lq, 0.0f));
      const float u = i < 4 ? us[i] : u01(philox4x32(make_uint4(i, 0x51u, stream, a.salt),
                                                     make_uint2(static_cast<uint32_t>(seed), 0)).x);
      if (!(u < ratio)) {
        count = i;
        break;
      }
    }
    s_count = count;
    s_valid = valid;
  }
  __syncthreads();
  const int count = s_count;
  // tail draw: residual (p - q)+ at row `count`, or the bonus row p_n
  const float* prow = a.target + (static_cast<long long>(b) * (n + 1) + count) * a.ld_target;
  const float* qrow = count < n ? a.draft + (static_cast<long long>(b) * n + count) * a.ld_draft : nullptr;
  const float lseP = s_lseT[count];
  const float lseQ = count < n ? s_lseQ[count] : 0.0f;
  float best = -INFINITY;
  int besti = 0x7fffffff;
  const uint32_t hi = static_cast<uint32_t>(a.salt) ^ 0xA5000000u;
  const int g0 = a.v_lo >> 2;
  for (int i = threadIdx.x; i * 4 < a.V; i += blockDim.x) {
    const float4 u = uniform4(seed, stream, hi, static_cast<uint32_t>(g0 + i));
    const float uu[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int v = i * 4 + j;
      if (v >= a.V) continue;
      float w;
      const float lp = prow[v] * invT - lseP;
      if (qrow) {
        const float d = __expf(lp) - __expf(qrow[v] * invT - lseQ);
        w = d > 0.0f ? __logf(d) : -INFINITY;
      } else {
        w = lp;
      }
      const float sc = w - __logf(-__logf(uu[j]));
      if (sc > best || (sc == best && v < besti)) {
        best = sc;
        besti = v;
      }
    }
  }
  __shared__ float sb[32];
  __shared__ int si[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, besti, o);
    if (ob > best || (ob == best && oi < besti)) {
      best = ob;
      besti = oi;
    }
  }
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (lane == 0) {
    sb[warp] = best;
    si[warp] = besti;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float bb = -INFINITY;
    int bi = 0x7fffffff;
    for (int w = 0; w < blockDim.x / 32; ++w) {
      if (sb[w] > bb || (sb[w] == bb && si[w] < bi)) {
        bb = sb[w];
        bi = si[w];
      }
    }
    if (a.keys != nullptr) {
      // vocabulary-parallel: the caller reduces the keys over ranks and finishes
      a.count[b] = count;
      a.valid[b] = s_valid;
      a.keys[b] = pack_argmax_key(bb, a.v_lo + (bi < a.V ? bi : 0));
      return;
    }
    int valid = s_valid && bb > -INFINITY && bi < a.V;
    const int tail = valid ? bi : 0;
    a.count[b] = count;
    a.tail[b] = tail;
    a.valid[b] = valid;
    // log-probabilities of every emitted token under the target policy and T = 1
    for (int i = 0; i <= count; ++i) {
      const int x = i < count ? a.candidates[b * n + i] : tail;
      const float l = a.target[(static_cast<long long>(b) * (n + 1) + i) * a.ld_target + x];
      a.logq[b * (n + 1) + i] = l * invT - s_lseT[i];
      a.logp[b * (n + 1) + i] = l - s_lse1[i];
      a.emitted[b * (n + 1) + i] = x;
    }
  }
}


// One warp folds one row's head-GEMM partials: lanes stride over the tiles in a
// fixed order, then a butterfly merges the lanes, so the result does not depend
// on scheduling.
__global__ void __launch_bounds__(256) head_stats_merge_kernel(HeadStatsArgs a) {
  pdl_wait();
  pdl_trigger();
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  if (row >= a.rows) return;
  const float invT = a.inv_temp ? a.inv_temp[row] : 1.0f;
  const float4* p = reinterpret_cast<const float4*>(a.part) + static_cast<long long>(row) * a.tiles;
  MaxSum2 acc{-INFINITY, 0.0f, 0.0f};
  for (int i = lane; i < a.tiles; i += 32) {
    const float4 v = p[i];
    acc = ms_merge(acc, MaxSum2{v.x, v.y, v.z}, invT);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const MaxSum2 other{__shfl_xor_sync(0xffffffffu, acc.m, o), __shfl_xor_sync(0xffffffffu, acc.s1, o),
                        __shfl_xor_sync(0xffffffffu, acc.sT, o)};
    acc = ms_merge(acc, other, invT);
  }
  if (lane != 0) return;
  const float lse1 = acc.m + logf(acc.s1);
  const float lseT = acc.m * invT + logf(acc.sT);
  if (a.lse1) a.lse1[row] = lse1;
  if (a.lseT) a.lseT[row] = lseT;
  if (a.targets != nullptr) {
    const int t = a.targets[row];
    const float l = (t >= 0 && t < a.V) ? a.target_logit[row] : -INFINITY;
    if (a.logp) a.logp[row] = l - lse1;
    if (a.logq) a.logq[row] = l * invT - lseT;
  }
}
}  // namespace

cudaError_t head_stats_merge_launch(const HeadStatsArgs& a, cudaStream_t stream) {
  if (a.rows <= 0) return cudaSuccess;
  if (a.part == nullptr || a.tiles <= 0 || (a.targets != nullptr && a.target_logit == nullptr))
    return cudaErrorInvalidValue;
  const int blocks = (a.rows * 32 + 255) / 256;
  return launch_pdl(head_stats_merge_kernel, dim3(blocks), dim3(256), 0, stream, a);
}

cudaError_t sample_launch(const SampleArgs& a, int rows, cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  return launch_pdl(sample_kernel, dim3(rows), dim3(kThreads), 0, stream, a);
}

cudaError_t row_stats_launch(const RowStatsArgs& a0, int rows, cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  RowStatsArgs a = a0;
  a.split = 1;
  a.chunk = a.V;
  const bool truncated = a.top_k != nullptr || a.top_p != nullptr;
  if (!truncated && a.part != nullptr && a.count != nullptr && rows <= kRowStatsSplitRows) {
    // Few rows: about two CTAs per SM in total, at least 8192 columns per CTA.
    static int sms = 0;
    if (sms == 0) {
      int dev = 0;
      cudaGetDevice(&dev);
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
      if (sms <= 0) sms = 148;
    }
    int split = (2 * sms + rows - 1) / rows;
    split = split < a.V / 8192 ? split : a.V / 8192;
    split = split < kRowStatsMaxSplit ? split : kRowStatsMaxSplit;
    if (split > 1) {
      a.chunk = ((a.V + split - 1) / split + 3) / 4 * 4;
      a.split = (a.V + a.chunk - 1) / a.chunk;     // every chunk non-empty
    }
  }
  return launch_pdl(row_stats_kernel, dim3(rows, a.split), dim3(kThreads), 0, stream, a);
}

cudaError_t gumbel_sample_launch(const GumbelArgs& a0, int rows, cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  GumbelArgs a = a0;
  a.split = 1;
  a.chunk = (a.V + 3) / 4 * 4;
  if (a.row_best != nullptr && a.row_count != nullptr && rows <= kGumbelSplitRows) {
    // Few rows: about two CTAs per SM in total, at least 8192 columns per CTA.
    static int sms = 0;
    if (sms == 0) {
      int dev = 0;
      cudaGetDevice(&dev);
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
      if (sms <= 0) sms = 148;
    }
    int split = (2 * sms + rows - 1) / rows;
    split = split < a.V / 8192 ? split : a.V / 8192;
    if (split > 1) {
      a.chunk = ((a.V + split - 1) / split + 3) / 4 * 4;
      a.split = (a.V + a.chunk - 1) / a.chunk;     // every chunk non-empty
    }
  }
  return launch_pdl(gumbel_sample_kernel, dim3(rows, a.split), dim3(kThreads), 0, stream, a);
}

cudaError_t spec_verify_launch(const SpecArgs& a, int batch, cudaStream_t stream) {
  if (batch <= 0) return cudaSuccess;
  if (a.n < 1 || a.n > 15) return cudaErrorInvalidValue;
  return launch_pdl(spec_verify_kernel, dim3(batch), dim3(kThreads), 0, stream, a);
}

}  // namespace osb

// ------------------------------------------------------------ divergence --
// Full-vocabulary distillation loss between student and teacher logits, per
// row, at temperature one (online-speculation/src/blockspec/losses.py:6-18):
//   kind 0: total variation 0.5 * sum_v |q_v - p_v|
//   kind 1: forward KL(p || q) = sum_v p_v (log p_v - log q_v)
// with q = softmax(student), p = softmax(teacher).  Three kernels so a
// vocabulary-sharded caller can all-reduce between phases:
//   stats  : per-row max and sum exp of both rows (local shard),
//   loss   : per-row loss pieces given the global log-normalisers
//            (TV: sum |q - p| and A = sum sign(q - p) q; KL: sum p (log p - log q)),
//   grad   : d loss / d student = w * 0.5 q (sign(q - p) - A)   (TV)
//                               = w * (q - p)                    (KL)
namespace osb {
namespace {

__global__ void __launch_bounds__(1024) div_stats_kernel(const float* __restrict__ s, const float* __restrict__ t,
                                                        long long ld_s, long long ld_t, int V, float* __restrict__ out) {
  // out[r] = {max_s, sum_s, max_t, sum_t}
  const int r = blockIdx.x;
  float ms, ss, mt, st, l1, lT;
  row_stats(s + r * ld_s, V, 1.0f, ms, l1, lT);
  ss = expf(l1 - ms);
  row_stats(t + r * ld_t, V, 1.0f, mt, l1, lT);
  st = expf(l1 - mt);
  if (threadIdx.x == 0) {
    out[4 * r + 0] = ms;
    out[4 * r + 1] = ss;
    out[4 * r + 2] = mt;
    out[4 * r + 3] = st;
  }
}

__global__ void __launch_bounds__(1024) div_loss_kernel(const float* __restrict__ s, const float* __restrict__ t,
                                                       long long ld_s, long long ld_t, int V,
                                                       const float* __restrict__ lse, int kind,
                                                       float* __restrict__ out) {
  // lse[2r] = global lse of student row r, lse[2r+1] of teacher row r.  out[2r] = loss piece, out[2r+1] = A.
  const int r = blockIdx.x;
  const float ls = lse[2 * r], lt = lse[2 * r + 1];
  const float* sr = s + r * ld_s;
  const float* tr = t + r * ld_t;
  float x = 0.0f, y = 0.0f;
  for (int v = threadIdx.x; v < V; v += blockDim.x) {
    const float lq = sr[v] - ls, lp = tr[v] - lt;
    const float q = __expf(lq), p = __expf(lp);
    if (kind == 0) {
      const float d = q - p;
      x += fabsf(d);
      y += d > 0.0f ? q : (d < 0.0f ? -q : 0.0f);
    } else {
      x += p > 0.0f ? p * (lp - lq) : 0.0f;
    }
  }
  __shared__ float rx[32], ry[32];
  x = warp_sum(x);
  y = warp_sum(y);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (lane == 0) {
    rx[warp] = x;
    ry[warp] = y;
  }
  __syncthreads();
  if (warp == 0) {
    x = lane < blockDim.x / 32 ? rx[lane] : 0.0f;
    y = lane < blockDim.x / 32 ? ry[lane] : 0.0f;
    x = warp_sum(x);
    y = warp_sum(y);
    if (lane == 0) {
      out[2 * r] = kind == 0 ? 0.5f * x : x;
      out[2 * r + 1] = y;
    }
  }
}

__global__ void div_grad_kernel(const float* __restrict__ s, const float* __restrict__ t, long long ld_s,
                                long long ld_t, int V, const float* __restrict__ lse, const float* __restrict__ pieces,
                                const float* __restrict__ w, int kind, __nv_bfloat16* __restrict__ grad,
                                long long ld_g) {
  const int r = blockIdx.y;
  const float ls = lse[2 * r], lt = lse[2 * r + 1];
  const float A = pieces[2 * r + 1];
  const float wr = w[r];
  const float* sr = s + r * ld_s;
  const float* tr = t + r * ld_t;
  for (int v = blockIdx.x * blockDim.x + threadIdx.x; v < V; v += gridDim.x * blockDim.x) {
    const float q = __expf(sr[v] - ls), p = __expf(tr[v] - lt);
    float g;
    if (kind == 0) {
      const float d = q - p;
      const float sg = d > 0.0f ? 1.0f : (d < 0.0f ? -1.0f : 0.0f);
      g = 0.5f * q * (sg - A);
    } else {
      g = q - p;
    }
    grad[r * ld_g + v] = f2bf(wr * g);
  }
}

}  // namespace

cudaError_t divergence_stats_launch(const float* s, const float* t, long long ld_s, long long ld_t, int rows, int V,
                                    float* out, cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  div_stats_kernel<<<rows, 1024, 0, stream>>>(s, t, ld_s, ld_t, V, out);
  return cudaGetLastError();
}

cudaError_t divergence_loss_launch(const float* s, const float* t, long long ld_s, long long ld_t, int rows, int V,
                                   const float* lse, int kind, float* out, cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  div_loss_kernel<<<rows, 1024, 0, stream>>>(s, t, ld_s, ld_t, V, lse, kind, out);
  return cudaGetLastError();
}

cudaError_t divergence_grad_launch(const float* s, const float* t, long long ld_s, long long ld_t, int rows, int V,
                                   const float* lse, const float* pieces, const float* w, int kind,
                                   __nv_bfloat16* grad, long long ld_g, cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  dim3 grid((V + 1023) / 1024 < 32 ? (V + 1023) / 1024 : 32, rows);
  div_grad_kernel<<<grid, 1024, 0, stream>>>(s, t, ld_s, ld_t, V, lse, pieces, w, kind, grad, ld_g);
  return cudaGetLastError();
}

}  // namespace osb

// --------------------------------------------------------- target logprob --
// Backward of log p(target) = l_t - lse(l) per row:  d/dl_v = w_r (1[v = t] - p_v)
// written as bf16 (or fp32) gradient rows; lse from row_stats.
namespace osb {
namespace {
// d log softmax(l)[t] / d l_v = [v == t] - p_v, scaled by the row's upstream gradient.
// Rows are processed in float4 chunks when the row stride allows it.
template <typename T>
__global__ void logprob_grad_kernel(const float* __restrict__ logits, long long ld, int V,
                                    const float* __restrict__ lse, const int* __restrict__ targets,
                                    const float* __restrict__ w, T* __restrict__ grad, long long ldg) {
  const int r = blockIdx.y;
  const float l = lse[r], wr = w[r];
  const int t = targets[r];
  const float* row = logits + r * ld;
  T* out = grad + r * ldg;
  const bool vec = (V % 4 == 0) && (ld % 4 == 0) && (ldg % 4 == 0);
  if (vec) {
    const int n4 = V / 4;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += gridDim.x * blockDim.x) {
      const float4 x = reinterpret_cast<const float4*>(row)[i];
      float g[4] = {-wr * __expf(x.x - l), -wr * __expf(x.y - l), -wr * __expf(x.z - l), -wr * __expf(x.w - l)};
      const int v0 = 4 * i;
      if (t >= v0 && t < v0 + 4) g[t - v0] += wr;
      if constexpr (sizeof(T) == 4) {
        reinterpret_cast<float4*>(out)[i] = make_float4(g[0], g[1], g[2], g[3]);
      } else {
        __nv_bfloat162 a = __floats2bfloat162_rn(g[0], g[1]);
        __nv_bfloat162 b = __floats2bfloat162_rn(g[2], g[3]);
        uint2 u;
        u.x = *reinterpret_cast<unsigned*>(&a);
        u.y = *reinterpret_cast<unsigned*>(&b);
        reinterpret_cast<uint2*>(out)[i] = u;
      }
    }
    return;
  }
  for (int v = blockIdx.x * blockDim.x + threadIdx.x; v < V; v += gridDim.x * blockDim.x) {
    const float g = wr * ((v == t ? 1.0f : 0.0f) - __expf(row[v] - l));
    if constexpr (sizeof(T) == 4) out[v] = g;
    else out[v] = __float2bfloat16(g);
  }
}
}  // namespace

cudaError_t logprob_grad_launch(const float* logits, long long ld, int rows, int V, const float* lse,
                                const int* targets, const float* w, void* grad, bool grad_bf16, long long ldg,
                                cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  const int per = (V + 4095) / 4096;
  dim3 grid(per < 32 ? per : 32, rows);
  if (grad_bf16)
    logprob_grad_kernel<__nv_bfloat16><<<grid, 1024, 0, stream>>>(logits, ld, V, lse, targets, w,
                                                                   static_cast<__nv_bfloat16*>(grad), ldg);
  else
    logprob_grad_kernel<float><<<grid, 1024, 0, stream>>>(logits, ld, V, lse, targets, w,
                                                          static_cast<float*>(grad), ldg);
  return cudaGetLastError();
}
}  // namespace osb

// --------------------------------------------------------------------------
// Scoring statistics of one logits row at temperature T, one pass:
//   target log-probability, sum_v p_v log p_v (negative entropy),
//   mean_v log p_v (for self-certainty), mean of the top-K log-probabilities.
// Every thread keeps an online (max, sum e, sum e*(x-max)) state and a sorted
// top-K list of its strided elements; the block merges states and lists.
namespace osb {
namespace {
constexpr int kStatThreads = 512;
constexpr int kMaxTopK = 16;

struct OnlineSums {
  float m, s1, s2;  // max, sum e^(x-m), sum e^(x-m) (x-m)
};

__device__ __forceinline__ OnlineSums merge_sums(OnlineSums a, OnlineSums b) {
  if (a.m == -INFINITY) return b;
  if (b.m == -INFINITY) return a;
  const float m = fmaxf(a.m, b.m);
  const float ea = __expf(a.m - m), eb = __expf(b.m - m);
  // rescale: s2' = e^(m_old - m) (s2 + (m_old - m) s1)
  return {m, a.s1 * ea + b.s1 * eb, ea * (a.s2 + (a.m - m) * a.s1) + eb * (b.s2 + (b.m - m) * b.s1)};
}

__global__ void __launch_bounds__(kStatThreads) score_stats_kernel(const float* __restrict__ logits, long long ld,
                                                                   int V, const float* __restrict__ inv_temp,
                                                                   const int* __restrict__ targets, int topk,
                                                                   float* __restrict__ out) {
  const int r = blockIdx.x;
  const float* row = logits + r * ld;
  const float it = inv_temp ? inv_temp[r] : 1.0f;
  OnlineSums st{-INFINITY, 0.0f, 0.0f};
  float sum_x = 0.0f;
  float top[kMaxTopK];
#pragma unroll
  for (int i = 0; i < kMaxTopK; ++i) top[i] = -INFINITY;
  for (int v = threadIdx.x; v < V; v += blockDim.x) {
    const float x = row[v] * it;
    sum_x += x;
    if (x == -INFINITY) continue;                  // excluded token: no mass
    if (x > st.m) {
      if (st.m == -INFINITY) {
        st = {x, 1.0f, 0.0f};
      } else {
        const float e = __expf(st.m - x);
        st.s2 = e * (st.s2 + (st.m - x) * st.s1);
        st.s1 = st.s1 * e + 1.0f;
        st.m = x;
      }
    } else {
      const float e = __expf(x - st.m);
      st.s1 += e;
      st.s2 += e * (x - st.m);
    }
    if (topk > 0 && x > top[topk - 1]) {          // insertion into the sorted list
      int j = topk - 1;
      while (j > 0 && top[j - 1] < x) {
        top[j] = top[j - 1];
        --j;
      }
      top[j] = x;
    }
  }
  __shared__ OnlineSums s_st[kStatThreads / 32];
  __shared__ float s_x[kStatThreads / 32];
  __shared__ float s_top[kStatThreads / 32];
  __shared__ int s_arg[kStatThreads / 32];
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32;
  for (int o = 16; o > 0; o >>= 1) {
    OnlineSums other{__shfl_xor_sync(0xffffffffu, st.m, o), __shfl_xor_sync(0xffffffffu, st.s1, o),
                     __shfl_xor_sync(0xffffffffu, st.s2, o)};
    st = merge_sums(st, other);
    sum_x += __shfl_xor_sync(0xffffffffu, sum_x, o);
  }
  if (lane == 0) {
    s_st[warp] = st;
    s_x[warp] = sum_x;
  }
  __syncthreads();
  __shared__ float s_lse;
  if (threadIdx.x == 0) {
    OnlineSums a = s_st[0];
    float sx = s_x[0];
    for (int w = 1; w < kStatThreads / 32; ++w) {
      a = merge_sums(a, s_st[w]);
      sx += s_x[w];
    }
    const float lse = a.m + logf(a.s1);
    s_lse = lse;
    out[r * 4 + 0] = targets ? row[targets[r]] * it - lse : 0.0f;
    out[r * 4 + 1] = a.s2 / a.s1 - logf(a.s1);          // sum p log p
    out[r * 4 + 2] = sx / static_cast<float>(V) - lse;  // mean log p over the vocabulary
  }
  __syncthreads();
  // top-K: K rounds of block argmax over the heads of the per-thread lists
  float acc = 0.0f;
  int head = 0;
  for (int k = 0; k < topk; ++k) {
    float best = head < topk ? top[head] : -INFINITY;
    int who = threadIdx.x;
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int ow = __shfl_xor_sync(0xffffffffu, who, o);
      if (ob > best || (ob == best && ow < who)) {
        best = ob;
        who = ow;
      }
    }
    if (lane == 0) {
      s_top[warp] = best;
      s_arg[warp] = who;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      float b = s_top[0];
      int w0 = s_arg[0];
      for (int w = 1; w < kStatThreads / 32; ++w)
        if (s_top[w] > b || (s_top[w] == b && s_arg[w] < w0)) {
          b = s_top[w];
          w0 = s_arg[w];
        }
      s_top[0] = b;
      s_arg[0] = w0;
    }
    __syncthreads();
    if (threadIdx.x == s_arg[0]) ++head;
    acc += s_top[0];
    __syncthreads();
  }
  if (threadIdx.x == 0) out[r * 4 + 3] = topk > 0 ? -(acc / topk - s_lse) : 0.0f;
}
}  // namespace

cudaError_t score_stats_launch(const float* logits, long long ld, int rows, int V, const float* inv_temp,
                               const int* targets, int topk, float* out, cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  if (topk < 0 || topk > kMaxTopK) return cudaErrorInvalidValue;
  score_stats_kernel<<<rows, kStatThreads, 0, stream>>>(logits, ld, V, inv_temp, targets, topk, out);
  return cudaGetLastError();
}
}  // namespace osb
