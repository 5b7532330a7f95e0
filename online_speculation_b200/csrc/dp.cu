// Data-parallel gradient reduce-scatter and parameter all-gather for the sharded trainers,
// over NVLink / NVSwitch peer memory.
//
// The flat fp32 gradient buffer and the flat bf16 parameter buffer of every rank are
// symmetric allocations, so a rank can load its peers' gradients and store into its peers'
// parameters directly.
//
//   reduce-scatter (one launch per gradient bucket, on the trainer's side stream as soon as
//   the bucket's gradients are complete, overlapping the rest of the backward pass): block 0
//   releases the call's epoch into every rank's pad; every block waits (bounded) until all
//   ranks have done so, then sums its part of this rank's shard over all ranks' buffers in
//   rank order (float4 peer loads) and writes scale * sum into the local shard.  No closing
//   barrier: a rank rewrites its gradients only in its next backward pass, which starts after
//   the all-gather, and no rank's all-gather can finish before every rank's reduce-scatters.
//
//   all-gather (one launch per optimizer step, after the sharded AdamW): an opening barrier
//   (no rank stores into a peer that still reads its parameters), then every block stores its
//   part of this rank's bf16 shard into every rank's parameter buffer (uint4 peer stores);
//   the last block to finish releases a completion flag on every rank and waits (bounded)
//   for all ranks' flags, so the kernel ends once this rank's parameters are complete.
//
// A wait that runs out records kErrPeerWait in the status word and the kernel skips its
// data movement instead of hanging.  Purpose of the reference GRPO trainer's DeepSpeed /
// DDP gradient reduction (experiments/arllm/train_gsm8k_grpo.py); the sharded layout is
// this package's ZeRO-1 trainer.
#include "common.cuh"
#include "dp.h"

namespace osb {
namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Every rank's entry of `slot` in this rank's pad: thread 0 waits (bounded) for `epoch`.
__device__ bool await_ranks(const DpArgs& a, int slot, uint32_t epoch) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    ok = 1;
    const uint32_t* mine = a.pads[a.rank] + slot * kMaxRanks;
    const unsigned long long start = global_ns();
    for (int q = 0; q < a.world && ok; ++q) {
      while (static_cast<int>(ld_acquire_sys(mine + q) - epoch) < 0) {
        if (global_ns() - start > wait_limit(a.wait_ns)) {
          record_error(a.status, kErrPeerWait);
          ok = 0;
          break;
        }
      }
    }
  }
  __syncthreads();
  return ok != 0;
}

__device__ __forceinline__ void release_to_ranks(const DpArgs& a, int slot, uint32_t epoch) {
  if (threadIdx.x < a.world) st_release_sys(a.pads[threadIdx.x] + slot * kMaxRanks + a.rank, epoch);
}

// Counts the block's arrival; true in the last block of the grid (which resets the counter).
__device__ __forceinline__ bool last_block(uint32_t* arrivals) {
  __shared__ int last;
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t done = atomicAdd(arrivals, 1u);
    last = done == gridDim.x - 1;
    if (last) *arrivals = 0;
  }
  __syncthreads();
  return last != 0;
}

__global__ void __launch_bounds__(kThreads) reduce_scatter_kernel(const DpArgs a, long long lo, long long n,
                                                                  float* __restrict__ shard, float scale) {
  const uint32_t epoch = a.counters[0] + 1;
  if (blockIdx.x == 0) release_to_ranks(a, kDpScatterSlot, epoch);
  if (await_ranks(a, kDpScatterSlot, epoch)) {
    const long long base = lo + static_cast<long long>(a.rank) * n;
    const long long nv = n / 4;
    const long long stride = static_cast<long long>(gridDim.x) * kThreads;
    for (long long v = blockIdx.x * static_cast<long long>(kThreads) + threadIdx.x; v < nv; v += stride) {
      float4 g[kMaxRanks];
#pragma unroll
      for (int q = 0; q < kMaxRanks; ++q)     // every load in flight before the first add
        if (q < a.world) g[q] = __ldcg(reinterpret_cast<const float4*>(a.grads[q] + base) + v);
      float4 s = g[0];
#pragma unroll
      for (int q = 1; q < kMaxRanks; ++q) {
        if (q < a.world) {
          s.x += g[q].x;
          s.y += g[q].y;
          s.z += g[q].z;
          s.w += g[q].w;
        }
      }
      reinterpret_cast<float4*>(shard)[v] = make_float4(s.x * scale, s.y * scale, s.z * scale, s.w * scale);
    }
  }
  if (last_block(a.counters + 1) && threadIdx.x == 0) a.counters[0] = epoch;
}

__global__ void __launch_bounds__(kThreads) all_gather_kernel(const DpArgs a, const __nv_bfloat16* __restrict__ src,
                                                              long long lo, long long n) {
  const uint32_t epoch = a.counters[2] + 1;
  if (blockIdx.x == 0) release_to_ranks(a, kDpGatherStartSlot, epoch);
  const bool ok = await_ranks(a, kDpGatherStartSlot, epoch);
  if (ok) {
    const long long base = lo + static_cast<long long>(a.rank) * n;
    const long long nv = n / 8;
    const long long stride = static_cast<long long>(gridDim.x) * kThreads;
    for (long long v = blockIdx.x * static_cast<long long>(kThreads) + threadIdx.x; v < nv; v += stride) {
      const uint4 x = reinterpret_cast<const uint4*>(src)[v];
#pragma unroll
      for (int q = 0; q < kMaxRanks; ++q)
        if (q < a.world) reinterpret_cast<uint4*>(a.params[q] + base)[v] = x;
    }
  }
  // this block's peer stores are visible system-wide before the completion flag
  __threadfence_system();
  if (!last_block(a.counters + 3)) return;
  release_to_ranks(a, kDpGatherDoneSlot, epoch);
  await_ranks(a, kDpGatherDoneSlot, epoch);      // a timeout is recorded; the call count stays in step
  if (threadIdx.x == 0) a.counters[2] = epoch;
}

int grid_for(long long vectors) {
  static int cap = 0;
  if (cap == 0) {
    int dev = 0, sms = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    // one 256-thread block per SM: resident beside the backward pass's GEMM CTAs, so a rank that
    // waits for a slower peer at the opening barrier does not hold its own backward pass back
    cap = sms > 0 ? sms : 148;
  }
  const long long want = (vectors + kThreads - 1) / kThreads;
  return static_cast<int>(want < 1 ? 1 : (want < cap ? want : cap));
}

bool valid(const DpArgs& a) {
  if (a.world < 2 || a.world > kMaxRanks || a.rank < 0 || a.rank >= a.world || a.counters == nullptr) return false;
  for (int q = 0; q < a.world; ++q)
    if (a.pads[q] == nullptr) return false;
  return true;
}

}  // namespace

cudaError_t dp_reduce_scatter_launch(const DpArgs& a, long long lo, long long n, float* shard, float scale,
                                     cudaStream_t stream) {
  if (!valid(a) || n <= 0 || n % 4 || lo % 4 || shard == nullptr) return cudaErrorInvalidValue;
  for (int q = 0; q < a.world; ++q)
    if (a.grads[q] == nullptr || reinterpret_cast<uintptr_t>(a.grads[q]) % 16) return cudaErrorInvalidValue;
  if (reinterpret_cast<uintptr_t>(shard) % 16) return cudaErrorInvalidValue;
  reduce_scatter_kernel<<<grid_for(n / 4), kThreads, 0, stream>>>(a, lo, n, shard, scale);
  return cudaGetLastError();
}

cudaError_t dp_all_gather_launch(const DpArgs& a, const __nv_bfloat16* src, long long lo, long long n,
                                 cudaStream_t stream) {
  if (!valid(a) || n <= 0 || n % 8 || lo % 8 || src == nullptr) return cudaErrorInvalidValue;
  for (int q = 0; q < a.world; ++q)
    if (a.params[q] == nullptr || reinterpret_cast<uintptr_t>(a.params[q]) % 16) return cudaErrorInvalidValue;
  if (reinterpret_cast<uintptr_t>(src) % 16) return cudaErrorInvalidValue;
  all_gather_kernel<<<grid_for(n / 8), kThreads, 0, stream>>>(a, src, lo, n);
  return cudaGetLastError();
}

}  // namespace osb
