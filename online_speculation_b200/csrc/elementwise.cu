// Memory-bound per-token kernels of the decoder layers.
//
//  * rmsnorm: y = w * bf16(x * rsqrt(mean(x^2) + eps)), the Qwen2/Qwen3 RMSNorm
//    (reference: online-speculation/src/blockspec/parallel/backbone.py:74-83),
//    optionally fused with a residual add (h += delta; y = norm(h)).
//  * rope_cache: splits a fused QKV row, applies the optional per-head Q/K
//    RMSNorm of Qwen3 (backbone.py:117-118), rotate-half RoPE with fp32 angles
//    (backbone.py:101-103, 277-279), writes Q to a packed buffer and K/V into
//    their paged-cache slots (replaces DynamicCache / torch.cat growth,
//    src/inference_scaling/arllm/backends/growing_cache.py:45-64).
//  * embedding gather and paged-cache page copy (copy-on-write fork of a
//    partially filled page at a suffix-MH cut).
#include "common.cuh"
#include "elementwise.h"

namespace osb {
namespace {

__global__ void rmsnorm_kernel(const __nv_bfloat16* __restrict__ x, long long ldx, __nv_bfloat16* h, long long ldh,
                               const __nv_bfloat16* __restrict__ delta, long long ldd,
                               const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ y, long long ldy, int H,
                               float eps) {
  // If delta != null: h[row] = x[row] + delta[row] (written back), then normalise h.
  pdl_wait();
  pdl_trigger();
  const int row = blockIdx.x;
  const __nv_bfloat16* xr = x + row * ldx;
  extern __shared__ float red[];
  float ss = 0.0f;
  const int nvec = H / 8;
  for (int i = threadIdx.x; i < nvec; i += blockDim.x) {
    uint4 raw = *reinterpret_cast<const uint4*>(xr + i * 8);
    __nv_bfloat16* e = reinterpret_cast<__nv_bfloat16*>(&raw);
    if (delta) {
      uint4 draw = *reinterpret_cast<const uint4*>(delta + row * ldd + i * 8);
      const __nv_bfloat16* de = reinterpret_cast<const __nv_bfloat16*>(&draw);
#pragma unroll
      for (int j = 0; j < 8; ++j) e[j] = f2bf(bf2f(e[j]) + bf2f(de[j]));
      *reinterpret_cast<uint4*>(h + row * ldh + i * 8) = raw;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float v = bf2f(e[j]);
      ss += v * v;
    }
  }
  ss = warp_sum(ss);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  if (warp == 0) {
    float t = lane < (blockDim.x + 31) / 32 ? red[lane] : 0.0f;
    t = warp_sum(t);
    if (lane == 0) red[32] = rsqrtf(t / H + eps);
  }
  __syncthreads();
  const float r = red[32];
  const __nv_bfloat16* src = delta ? h + row * ldh : xr;
  for (int i = threadIdx.x; i < nvec; i += blockDim.x) {
    uint4 raw = *reinterpret_cast<const uint4*>(src + i * 8);
    uint4 wr = *reinterpret_cast<const uint4*>(w + i * 8);
    const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&raw);
    const __nv_bfloat16* we = reinterpret_cast<const __nv_bfloat16*>(&wr);
    uint4 out;
    __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(&out);
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = f2bf(bf2f(we[j]) * bf2f(f2bf(bf2f(e[j]) * r)));
    *reinterpret_cast<uint4*>(y + row * ldy + i * 8) = out;
  }
}

// One warp per (token, head).  Heads [0, Hq) are queries, [Hq, Hq+Hkv) keys,
// [Hq+Hkv, Hq+2Hkv) values.  D = 128: lane l owns elements 2l, 2l+1 and
// their rotation partners 2l+64, 2l+65.
__global__ void rope_cache_kernel(const __nv_bfloat16* __restrict__ qkv, long long ldqkv,
                                  const int* __restrict__ positions, const int* __restrict__ slots,
                                  const float* __restrict__ inv_freq, const __nv_bfloat16* __restrict__ qn_w,
                                  const __nv_bfloat16* __restrict__ kn_w, float eps, __nv_bfloat16* __restrict__ q_out,
                                  __nv_bfloat16* __restrict__ k_cache, __nv_bfloat16* __restrict__ v_cache, int T,
                                  int Hq, int Hkv, int page, long long slot_capacity, int* status) {
  pdl_wait();
  pdl_trigger();
  const int warps = blockDim.x / 32;
  const int gw = blockIdx.x * warps + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int heads = Hq + 2 * Hkv;
  if (gw >= T * heads) return;
  const int t = gw / heads, hh = gw % heads;
  const __nv_bfloat16* src = qkv + t * ldqkv + hh * 128;
  const int d0 = 2 * lane;
  float a0 = bf2f(src[d0]), a1 = bf2f(src[d0 + 1]);
  float b0 = bf2f(src[d0 + 64]), b1 = bf2f(src[d0 + 65]);
  int slot = slots ? slots[t] : -1;
#if OSB_DEVICE_CHECKS
  if (slot >= slot_capacity) {      // beyond the cache: store nothing, report once per token
    if (lane == 0 && hh == Hq) record_error(status, kErrBadIndex);
    slot = -1;
  }
#endif
  if (hh >= Hq + Hkv) {
    if (slot >= 0) {
      const int g = hh - Hq - Hkv;
      const long long off = ((static_cast<long long>(slot / page) * Hkv + g) * page + slot % page) * 128;
      __nv_bfloat16* dst = v_cache + off;
      *reinterpret_cast<__nv_bfloat162*>(dst + d0) = __floats2bfloat162_rn(a0, a1);
      *reinterpret_cast<__nv_bfloat162*>(dst + d0 + 64) = __floats2bfloat162_rn(b0, b1);
    }
    return;
  }
  const __nv_bfloat16* nw = hh < Hq ? qn_w : kn_w;
  if (nw) {
    float ss = warp_sum(a0 * a0 + a1 * a1 + b0 * b0 + b1 * b1);
    const float r = rsqrtf(ss / 128.0f + eps);
    a0 = bf2f(nw[d0]) * bf2f(f2bf(a0 * r));
    a1 = bf2f(nw[d0 + 1]) * bf2f(f2bf(a1 * r));
    b0 = bf2f(nw[d0 + 64]) * bf2f(f2bf(b0 * r));
    b1 = bf2f(nw[d0 + 65]) * bf2f(f2bf(b1 * r));
    // the reference keeps normalised projections in the model dtype
    a0 = bf2f(f2bf(a0));
    a1 = bf2f(f2bf(a1));
    b0 = bf2f(f2bf(b0));
    b1 = bf2f(f2bf(b1));
  }
  const float pos = static_cast<float>(positions[t]);
  float s0, c0, s1, c1;
  sincosf(pos * inv_freq[d0], &s0, &c0);
  sincosf(pos * inv_freq[d0 + 1], &s1, &c1);
  const float ra0 = a0 * c0 - b0 * s0, rb0 = b0 * c0 + a0 * s0;
  const float ra1 = a1 * c1 - b1 * s1, rb1 = b1 * c1 + a1 * s1;
  __nv_bfloat16* dst;
  if (hh < Hq) {
    dst = q_out + (static_cast<long long>(t) * Hq + hh) * 128;
  } else {
    if (slot < 0) return;
    const int g = hh - Hq;
    dst = k_cache + ((static_cast<long long>(slot / page) * Hkv + g) * page + slot % page) * 128;
  }
  *reinterpret_cast<__nv_bfloat162*>(dst + d0) = __floats2bfloat162_rn(ra0, ra1);
  *reinterpret_cast<__nv_bfloat162*>(dst + d0 + 64) = __floats2bfloat162_rn(rb0, rb1);
}

__global__ void embed_kernel(const int* __restrict__ ids, const __nv_bfloat16* __restrict__ table, int V, int H,
                             __nv_bfloat16* __restrict__ out, long long ldo, int* status) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x;
  const int id = ids[t];
  uint4* dst = reinterpret_cast<uint4*>(out + t * ldo);
#if OSB_DEVICE_CHECKS
  if (id < 0 || id >= V) {          // outside the table: zero row, report
    if (threadIdx.x == 0) record_error(status, kErrBadIndex);
    for (int i = threadIdx.x; i < H / 8; i += blockDim.x) dst[i] = make_uint4(0, 0, 0, 0);
    return;
  }
#endif
  const uint4* src = reinterpret_cast<const uint4*>(table + static_cast<long long>(id) * H);
  for (int i = threadIdx.x; i < H / 8; i += blockDim.x) dst[i] = src[i];
}

// Copy the first `count` token slots of page src -> page dst for every layer
// and every kv head of one cache tensor [layers, pages, Hkv, P, D].
__global__ void page_copy_kernel(__nv_bfloat16* cache, long long layer_stride, const int* __restrict__ pairs,
                                 int npairs, int Hkv, int page) {
  const int pair = blockIdx.x;
  const int layer = blockIdx.y;
  const int src = pairs[3 * pair], dst = pairs[3 * pair + 1], count = pairs[3 * pair + 2];
  __nv_bfloat16* base = cache + layer * layer_stride;
  const long long per_page = static_cast<long long>(Hkv) * page * 128;
  for (int g = 0; g < Hkv; ++g) {
    const uint4* s = reinterpret_cast<const uint4*>(base + src * per_page + static_cast<long long>(g) * page * 128);
    uint4* d = reinterpret_cast<uint4*>(base + dst * per_page + static_cast<long long>(g) * page * 128);
    for (int i = threadIdx.x; i < count * 16; i += blockDim.x) d[i] = s[i];
  }
}

}  // namespace

cudaError_t rmsnorm_launch(const __nv_bfloat16* x, long long ldx, __nv_bfloat16* h, long long ldh,
                           const __nv_bfloat16* delta, long long ldd, const __nv_bfloat16* w, __nv_bfloat16* y,
                           long long ldy, int T, int H, float eps, cudaStream_t stream) {
  if (H % 8 || T <= 0) return T == 0 ? cudaSuccess : cudaErrorInvalidValue;
  const int threads = H >= 2048 ? 256 : 128;
  return launch_pdl(rmsnorm_kernel, dim3(T), dim3(threads), 33 * sizeof(float), stream, x, ldx, h, ldh, delta, ldd,
                    w, y, ldy, H, eps);
}

cudaError_t rope_cache_launch(const __nv_bfloat16* qkv, long long ldqkv, const int* positions, const int* slots,
                              const float* inv_freq, const __nv_bfloat16* qn_w, const __nv_bfloat16* kn_w, float eps,
                              __nv_bfloat16* q_out, __nv_bfloat16* k_cache, __nv_bfloat16* v_cache, int T, int Hq,
                              int Hkv, int page, long long slot_capacity, int* status, cudaStream_t stream) {
  if (T <= 0) return cudaSuccess;
  const int heads = Hq + 2 * Hkv;
  const long long warps = static_cast<long long>(T) * heads;
  const int per_block = 8;
  return launch_pdl(rope_cache_kernel, dim3(static_cast<int>((warps + per_block - 1) / per_block)),
                    dim3(per_block * 32), 0, stream, qkv, ldqkv, positions, slots, inv_freq, qn_w, kn_w, eps, q_out,
                    k_cache, v_cache, T, Hq, Hkv, page, slot_capacity, status);
}

cudaError_t embed_launch(const int* ids, const __nv_bfloat16* table, int V, int T, int H, __nv_bfloat16* out,
                         long long ldo, int* status, cudaStream_t stream) {
  if (T <= 0) return cudaSuccess;
  if (H % 8) return cudaErrorInvalidValue;
  return launch_pdl(embed_kernel, dim3(T), dim3(256), 0, stream, ids, table, V, H, out, ldo, status);
}

cudaError_t page_copy_launch(__nv_bfloat16* cache, long long layer_stride, int layers, const int* pairs, int npairs,
                             int Hkv, int page, cudaStream_t stream) {
  if (npairs <= 0) return cudaSuccess;
  dim3 grid(npairs, layers);
  page_copy_kernel<<<grid, 256, 0, stream>>>(cache, layer_stride, pairs, npairs, Hkv, page);
  return cudaGetLastError();
}

}  // namespace osb
