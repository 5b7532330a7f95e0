// Mixture-of-experts routing / dispatch / combine kernels.
//
// The expert FFNs themselves run on the tcgen05 GEMM in grouped mode (one
// launch per projection for all experts, tile list built on the device from
// the routing counts), so no host synchronisation sits between routing and
// the expert GEMMs.
#include <cfloat>

#include "common.cuh"
#include "moe.h"

namespace osb {
namespace {

constexpr int kMaxExpertsPerLane = 8;   // E <= 256

__global__ void __launch_bounds__(256) moe_route_kernel(const float* __restrict__ logits, long long ld, int T, int E,
                                                        int k, int renorm, int* __restrict__ topk_idx,
                                                        float* __restrict__ topk_w, int* __restrict__ counts) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  if (warp >= T) return;
  const float* row = logits + static_cast<long long>(warp) * ld;
  float v[kMaxExpertsPerLane];
  float mx = -FLT_MAX;
#pragma unroll
  for (int i = 0; i < kMaxExpertsPerLane; ++i) {
    const int e = lane + 32 * i;
    v[i] = e < E ? row[e] : -FLT_MAX;
    mx = fmaxf(mx, v[i]);
  }
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float sum = 0.0f;
#pragma unroll
  for (int i = 0; i < kMaxExpertsPerLane; ++i) {
    const int e = lane + 32 * i;
    v[i] = e < E ? expf(v[i] - mx) : -1.0f;   // probabilities are >= 0; -1 marks "absent"
    if (e < E) sum += v[i];
  }
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  const float inv = 1.0f / sum;
  float chosen_sum = 0.0f;
  float my_w = 0.0f;
  int my_e = -1;
  for (int j = 0; j < k; ++j) {
    // warp argmax over (prob, -expert)
    float best = -2.0f;
    int best_e = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < kMaxExpertsPerLane; ++i) {
      const int e = lane + 32 * i;
      if (v[i] > best || (v[i] == best && e < best_e)) {
        best = v[i];
        best_e = e;
      }
    }
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oe = __shfl_xor_sync(0xffffffffu, best_e, o);
      if (ob > best || (ob == best && oe < best_e)) {
        best = ob;
        best_e = oe;
      }
    }
    if (best_e % 32 == lane) v[best_e / 32] = -2.0f;   // remove from later rounds
    const float p = best * inv;
    chosen_sum += p;
    if (lane == j) {
      my_w = p;
      my_e = best_e;
    }
  }
  if (lane < k) {
    topk_idx[warp * k + lane] = my_e;
    topk_w[warp * k + lane] = renorm ? my_w / chosen_sum : my_w;
    atomicAdd(&counts[my_e], 1);
  }
}

__global__ void __launch_bounds__(1024) moe_offsets_kernel(int* __restrict__ counts, int E, int* __restrict__ offsets,
                                                           int* __restrict__ cursor) {
  __shared__ int s[1025];
  for (int e = threadIdx.x; e < E; e += blockDim.x) s[e] = counts[e];
  __syncthreads();
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int e = 0; e < E; ++e) {
      const int c = s[e];
      s[e] = acc;
      acc += c;
    }
    s[E] = acc;
  }
  __syncthreads();
  for (int e = threadIdx.x; e <= E; e += blockDim.x) {
    offsets[e] = s[e];
    if (e < E) {
      cursor[e] = s[e];
      counts[e] = 0;
    }
  }
}

__global__ void __launch_bounds__(128) moe_dispatch_kernel(const __nv_bfloat16* __restrict__ x, long long ldx, int k,
                                                           int H, const int* __restrict__ topk_idx,
                                                           int* __restrict__ cursor, __nv_bfloat16* __restrict__ xp,
                                                           int* __restrict__ slot_of) {
  __shared__ int slots[32];
  const int t = blockIdx.x;
  if (threadIdx.x < k) {
    const int e = topk_idx[t * k + threadIdx.x];
    const int slot = atomicAdd(&cursor[e], 1);
    slots[threadIdx.x] = slot;
    slot_of[t * k + threadIdx.x] = slot;
  }
  __syncthreads();
  const uint4* src = reinterpret_cast<const uint4*>(x + static_cast<long long>(t) * ldx);
  const int nv = H / 8;
  for (int i = threadIdx.x; i < nv; i += blockDim.x) {
    const uint4 val = src[i];
    for (int j = 0; j < k; ++j) reinterpret_cast<uint4*>(xp + static_cast<long long>(slots[j]) * H)[i] = val;
  }
}

__global__ void __launch_bounds__(256) moe_combine_kernel(const __nv_bfloat16* __restrict__ y, long long ldy,
                                                          const int* __restrict__ slot_of,
                                                          const float* __restrict__ topk_w, int k, int H,
                                                          __nv_bfloat16* h, long long ldh, int accumulate) {
  __shared__ int slots[32];
  __shared__ float ws[32];
  const int t = blockIdx.x;
  if (threadIdx.x < k) {
    slots[threadIdx.x] = slot_of[t * k + threadIdx.x];
    ws[threadIdx.x] = topk_w[t * k + threadIdx.x];
  }
  __syncthreads();
  __nv_bfloat16* dst = h + static_cast<long long>(t) * ldh;
  const int nv = H / 8;
  for (int i = threadIdx.x; i < nv; i += blockDim.x) {
    float acc[8];
    if (accumulate) {
      const uint4 raw = reinterpret_cast<const uint4*>(dst)[i];
      const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = __bfloat162float(b[e]);
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = 0.0f;
    }
    float part[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) part[e] = 0.0f;
    for (int j = 0; j < k; ++j) {
      const uint4 raw = reinterpret_cast<const uint4*>(y + static_cast<long long>(slots[j]) * ldy)[i];
      const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
      for (int e = 0; e < 8; ++e) part[e] += ws[j] * __bfloat162float(b[e]);
    }
    uint4 out;
    __nv_bfloat162* o = reinterpret_cast<__nv_bfloat162*>(&out);
#pragma unroll
    for (int e = 0; e < 4; ++e) o[e] = __floats2bfloat162_rn(acc[2 * e] + part[2 * e], acc[2 * e + 1] + part[2 * e + 1]);
    reinterpret_cast<uint4*>(dst)[i] = out;
  }
}

}  // namespace

cudaError_t moe_route_launch(const float* logits, long long ld, int T, int E, int k, int renorm, int* topk_idx,
                             float* topk_w, int* counts, cudaStream_t stream) {
  if (T <= 0) return cudaSuccess;
  if (E <= 0 || E > 32 * kMaxExpertsPerLane || k <= 0 || k > 32 || k > E) return cudaErrorInvalidValue;
  const int blocks = (T * 32 + 255) / 256;
  moe_route_kernel<<<blocks, 256, 0, stream>>>(logits, ld, T, E, k, renorm, topk_idx, topk_w, counts);
  return cudaGetLastError();
}

cudaError_t moe_offsets_launch(int* counts, int E, int* offsets, int* cursor, cudaStream_t stream) {
  if (E <= 0 || E > 1024) return cudaErrorInvalidValue;
  moe_offsets_kernel<<<1, 1024, 0, stream>>>(counts, E, offsets, cursor);
  return cudaGetLastError();
}

cudaError_t moe_dispatch_launch(const __nv_bfloat16* x, long long ldx, int T, int k, int H, const int* topk_idx,
                                int* cursor, __nv_bfloat16* xp, int* slot_of, cudaStream_t stream) {
  if (T <= 0) return cudaSuccess;
  if (H % 8 || ldx % 8 || k > 32) return cudaErrorInvalidValue;
  moe_dispatch_kernel<<<T, 128, 0, stream>>>(x, ldx, k, H, topk_idx, cursor, xp, slot_of);
  return cudaGetLastError();
}

cudaError_t moe_combine_launch(const __nv_bfloat16* y, long long ldy, const int* slot_of, const float* topk_w, int T,
                               int k, int H, __nv_bfloat16* h, long long ldh, int accumulate, cudaStream_t stream) {
  if (T <= 0) return cudaSuccess;
  if (H % 8 || ldy % 8 || ldh % 8 || k > 32) return cudaErrorInvalidValue;
  moe_combine_kernel<<<T, 256, 0, stream>>>(y, ldy, slot_of, topk_w, k, H, h, ldh, accumulate);
  return cudaGetLastError();
}

}  // namespace osb
