// Expert-parallel MoE exchange over NVLink / NVSwitch peer memory.
//
// Rank r owns experts [r * E_local, (r + 1) * E_local).  Every buffer named
// below is a symmetric allocation mapped into every rank's address space.
//
// ep_dispatch_kernel
//   1. block 0 stores this rank's routing counts into row `rank` of every
//      peer's count table, then publishes the call's epoch into every peer's
//      signal pad (slot 0); all blocks wait until every peer has published.
//   2. from the now complete table every block derives, for each expert e, the
//      first row of this rank's share in the owner's receive buffer (owner
//      rows are grouped by local expert, then by source rank), and block 0
//      writes the per-local-expert row offsets of its own receive buffer.
//   3. one warp per (token, choice): slot = base[e] + atomicAdd(cursor[e]),
//      and the token row is stored straight into the owner's buffer.
//   4. the last block to finish resets the cursors, publishes slot 1 and waits
//      until every peer has finished writing into this rank's buffer.
// The grouped expert GEMMs then run on the local receive buffer and write the
// expert outputs into the local (symmetric) output buffer.
// ep_combine_kernel
//   publishes slot 2 (this rank's expert outputs are complete), waits for every
//   peer, then one block per token pulls its k expert rows from their owners
//   (peer loads) and adds the weighted sum to the residual in choice order --
//   the same arithmetic as the single-GPU combine, so results do not depend on
//   the expert placement.
// Every wait is bounded: on timeout the kernel records kErrPeerWait and skips
// its remaining work.  The epoch advances at the end of the combine.
//
// There is no counterpart in the reference (its MoE layers run inside one
// process on one GPU); this is the expert-parallel path of the MoE layer.
#include "common.cuh"
#include "ep.h"

namespace osb {
namespace {

constexpr int kEpThreads = 256;

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void publish(const EpArgs& a, int slot, uint32_t epoch) {
  // caller: one block, after its writes; threads < world each signal one peer
  if (threadIdx.x < a.world) {
    __threadfence_system();
    st_release_sys(a.pads[threadIdx.x] + slot * kEpMaxRanks + a.rank, epoch);
  }
}

// Thread 0 waits until every rank has published `epoch` in `slot` of this rank's pad.
__device__ __forceinline__ bool await_all(const EpArgs& a, int slot, uint32_t epoch) {
  bool ok = true;
  const uint32_t* mine = a.pads[a.rank] + slot * kEpMaxRanks;
  const unsigned long long start = global_ns();
  for (int q = 0; q < a.world && ok; ++q) {
    while (static_cast<int>(ld_acquire_sys(mine + q) - epoch) < 0) {
      if (global_ns() - start > wait_limit(a.wait_ns)) {
        record_error(a.status, kErrPeerWait);
        ok = false;
        break;
      }
    }
  }
  return ok;
}

__global__ void __launch_bounds__(kEpThreads) ep_dispatch_kernel(const EpArgs a) {
  const uint32_t epoch = *a.epoch + 1;
  __shared__ int base[kEpMaxExperts];
  __shared__ int ok;
  const int E = a.E, El = a.E_local, W = a.world;
  if (blockIdx.x == 0) {
    for (int i = threadIdx.x; i < W * E; i += blockDim.x) {
      const int q = i / E, e = i % E;
      a.tables[q][a.rank * E + e] = a.counts[e];
    }
    __threadfence_system();   // every writer orders its peer stores before the signal
    __syncthreads();
    publish(a, 0, epoch);
  }
  if (threadIdx.x == 0) ok = await_all(a, 0, epoch) ? 1 : 0;
  __syncthreads();
  if (ok) {
    const volatile int* tab = a.tables[a.rank];   // [source][expert]
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
      const int o = e / El, j = e % El;
      int b = 0;
      for (int jj = 0; jj < j; ++jj)
        for (int s = 0; s < W; ++s) b += tab[s * E + o * El + jj];
      for (int s = 0; s < a.rank; ++s) b += tab[s * E + e];
      base[e] = b;
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) {
      int off = 0;
      a.local_offsets[0] = 0;
      for (int j = 0; j < El; ++j) {
        for (int s = 0; s < W; ++s) off += tab[s * E + a.rank * El + j];
        a.local_offsets[j + 1] = off;
      }
    }
    __syncthreads();
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int warps = blockDim.x / 32;
    const int rows = a.T * a.k;
    const int nv = a.H / 8;
    for (int tk = blockIdx.x * warps + warp; tk < rows; tk += gridDim.x * warps) {
      int slot = 0, e = 0;
      if (lane == 0) {
        e = a.topk_idx[tk];
        slot = base[e] + atomicAdd(&a.cursor[e], 1);
        a.slot_of[tk] = slot;
      }
      slot = __shfl_sync(0xffffffffu, slot, 0);
      e = __shfl_sync(0xffffffffu, e, 0);
      if (slot < 0 || slot >= a.r_max) {
        if (lane == 0) record_error(a.status, kErrBadArgument);
        continue;
      }
      const uint4* src = reinterpret_cast<const uint4*>(a.x + static_cast<long long>(tk / a.k) * a.ldx);
      uint4* dst = reinterpret_cast<uint4*>(a.recv_x[e / El] + static_cast<long long>(slot) * a.H);
      for (int i = lane; i < nv; i += 32) dst[i] = src[i];
    }
  }
  // order this block's peer stores before the arrival count
  __threadfence_system();
  __syncthreads();
  __shared__ int last;
  if (threadIdx.x == 0) {
    const uint32_t done = atomicAdd(a.epoch + 1, 1u);
    last = done == gridDim.x - 1;
  }
  __syncthreads();
  if (!last) return;
  for (int e = threadIdx.x; e < E; e += blockDim.x) a.cursor[e] = 0;
  if (threadIdx.x == 0) a.epoch[1] = 0;
  __syncthreads();
  publish(a, 1, epoch);
  if (threadIdx.x == 0 && ok) await_all(a, 1, epoch);
}

__global__ void __launch_bounds__(kEpThreads) ep_combine_kernel(const EpArgs a) {
  const uint32_t epoch = *a.epoch + 1;
  if (blockIdx.x == 0) publish(a, 2, epoch);
  __shared__ int ok;
  if (threadIdx.x == 0) ok = await_all(a, 2, epoch) ? 1 : 0;
  __syncthreads();
  if (ok) {
    __shared__ int slots[32], owners[32];
    __shared__ float ws[32];
    const int nv = a.H / 8;
    for (int t = blockIdx.x; t < a.T; t += gridDim.x) {
      if (threadIdx.x < a.k) {
        slots[threadIdx.x] = a.slot_of[t * a.k + threadIdx.x];
        owners[threadIdx.x] = a.topk_idx[t * a.k + threadIdx.x] / a.E_local;
        ws[threadIdx.x] = a.topk_w[t * a.k + threadIdx.x];
      }
      __syncthreads();
      __nv_bfloat16* dst = a.h + static_cast<long long>(t) * a.ldh;
      for (int i = threadIdx.x; i < nv; i += blockDim.x) {
        float acc[8], part[8];
        const uint4 raw = reinterpret_cast<const uint4*>(dst)[i];
        const __nv_bfloat16* hb = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          acc[e] = bf2f(hb[e]);
          part[e] = 0.0f;
        }
        for (int j = 0; j < a.k; ++j) {
          const uint4 y = __ldcg(reinterpret_cast<const uint4*>(a.recv_y[owners[j]] +
                                                               static_cast<long long>(slots[j]) * a.H) + i);
          const __nv_bfloat16* yb = reinterpret_cast<const __nv_bfloat16*>(&y);
#pragma unroll
          for (int e = 0; e < 8; ++e) part[e] += ws[j] * bf2f(yb[e]);
        }
        uint4 out;
        __nv_bfloat162* o = reinterpret_cast<__nv_bfloat162*>(&out);
#pragma unroll
        for (int e = 0; e < 4; ++e) o[e] = __floats2bfloat162_rn(acc[2 * e] + part[2 * e], acc[2 * e + 1] + part[2 * e + 1]);
        reinterpret_cast<uint4*>(dst)[i] = out;
      }
      __syncthreads();
    }
  }
  __shared__ int last;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const uint32_t done = atomicAdd(a.epoch + 1, 1u);
    last = done == gridDim.x - 1;
    if (last) {
      a.epoch[1] = 0;
      __threadfence();
      a.epoch[0] = epoch;
    }
  }
}

bool valid(const EpArgs& a) {
  return a.world >= 1 && a.world <= kEpMaxRanks && a.E > 0 && a.E <= kEpMaxExperts && a.E % a.world == 0 &&
         a.E_local == a.E / a.world && a.k >= 1 && a.k <= 32 && a.H % 8 == 0 && a.ldx % 8 == 0 && a.ldh % 8 == 0 &&
         a.rank >= 0 && a.rank < a.world;
}

}  // namespace

cudaError_t ep_dispatch_launch(const EpArgs& a, int blocks, cudaStream_t stream) {
  if (!valid(a)) return cudaErrorInvalidValue;
  ep_dispatch_kernel<<<blocks > 0 ? blocks : 1, kEpThreads, 0, stream>>>(a);
  return cudaGetLastError();
}

cudaError_t ep_combine_launch(const EpArgs& a, int blocks, cudaStream_t stream) {
  if (!valid(a)) return cudaErrorInvalidValue;
  const int grid = a.T < blocks ? (a.T > 0 ? a.T : 1) : blocks;
  ep_combine_kernel<<<grid, kEpThreads, 0, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace osb
