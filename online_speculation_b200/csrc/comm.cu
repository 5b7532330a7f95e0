// Tensor-parallel all-reduce of row-parallel GEMM partials over NVLink peer
// memory, fused with the residual add and the following RMSNorm.
//
//   h <- h + sum_r P_r ;  x <- rmsnorm(h) * w
//
// Up to four ranks (and above that for small batches): one-shot.  After a cross-rank barrier every rank loads the
// rows of every rank's partial (peer loads), sums them in rank order (so the
// residual stream stays bitwise identical on all ranks), adds the residual,
// and applies RMSNorm in the same pass: one kernel, one barrier, and each rank
// reads (world - 1) x T x H x 2 bytes over NVLink.
//
// More ranks: two-shot in one kernel over symmetric buffers (every rank can
// load every other rank's buffers through NVLink / NVSwitch peer mappings):
//   phase A  each rank owns a slice of rows; it loads those rows of every
//            rank's partial P_r (peer loads), adds the residual, and stores the
//            reduced rows into its own symmetric row buffer and its local
//            residual stream;
//   phase B  after a cross-rank barrier (the grid is co-resident, the last
//            block of phase A signals), every rank gathers the other ranks'
//            reduced rows (peer loads) and applies RMSNorm to all rows.
// Barriers: block 0 (or the last block) publishes the call's epoch into every
// rank's signal pad (release, system scope) and every block polls its own pad
// (acquire) with a bounded wait.  On timeout the kernel records an error and
// skips its work instead of hanging.  Partials are double-buffered by the
// caller, so a rank can only overwrite a partial buffer after every peer has
// passed the next reduction's first barrier.
//
// There is no counterpart in the reference (it has no distributed code); this
// is the fused collective behind the tensor-parallel decoder layers.
#include "comm.h"
#include "common.cuh"

namespace osb {
namespace {

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Cross-rank barrier at the start of a kernel (slot distinguishes kernels).
// The data a peer reads after this barrier was written by the predecessor kernel, which
// has completed (and its writes are visible) once griddepcontrol.wait returns, so the
// signal needs no fence of its own beyond its release.
__device__ __forceinline__ bool rank_barrier(const ArArgs& a, int slot, uint32_t epoch) {
  if (blockIdx.x == 0 && threadIdx.x < a.world) {
    st_release_sys(a.pads[threadIdx.x] + slot * kMaxRanks + a.rank, epoch);
    if (threadIdx.x == 0 && a.trace != nullptr) a.trace[2] = global_ns();
  }
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

// Waits (bounded) until every rank has released at least `epoch` into this rank's
// flag words of `slot` (the pushing GEMMs publish there; nothing is signalled here).
__device__ __forceinline__ bool wait_flags(const ArArgs& a, int slot, uint32_t epoch) {
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

__device__ __forceinline__ int slice_begin(int T, int world, int r) { return (T * r) / world; }

// Marks this call complete once every block has finished (the next call's epoch).
__device__ __forceinline__ void finish_call(const ArArgs& a, uint32_t epoch) {
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

constexpr int kOneShotThreads = 256;
// "auto" above four ranks: one-shot up to this peer read per rank (eight B200s, 3584-wide rows,
// graph-replayed: 16.0 vs 28.4 us at 64 rows = 3.2 MB, 34.7 vs 37.1 us at 256 rows = 12.8 MB)
constexpr long long kOneShotPeerBytes = 16ll << 20;
constexpr int kOneShotRegVecs = 4;   // rows up to 256 * 4 * 8 = 8192 wide stay in registers (even count)

// kPushed: the partials were stored into this rank's memory by the ranks' GEMMs
// (parts[q] are local slots) and each GEMM released the call's epoch into flag
// slot kPushSlot; the kernel waits for those flags and reads only local memory.
__device__ __forceinline__ void ar_stamp(const ArArgs& a, int slot) {
  if (a.trace != nullptr && blockIdx.x == 0 && threadIdx.x == 0) a.trace[slot] = global_ns();
}

template <bool kPushed, int kRanks>
__global__ void __launch_bounds__(kOneShotThreads) oneshot_norm_kernel(const ArArgs a) {
  ar_stamp(a, 0);
  // The partials (and the previous call's epoch) belong to the predecessor; every block is
  // resident once it gets here, so the successor may launch (its own wait covers this grid).
  pdl_wait();
  pdl_trigger();
  ar_stamp(a, 1);
  const uint32_t epoch = *a.epoch + 1;
  const bool ok = kPushed ? wait_flags(a, kPushSlot, epoch) : rank_barrier(a, 2, epoch);
  ar_stamp(a, 3);
  const int nvec = a.H / 8;
  __shared__ float red[33];
  if (ok) {
    for (int row = blockIdx.x; row < a.T; row += gridDim.x) {
      __nv_bfloat16* hr = a.h + static_cast<long long>(row) * a.ldh;
      uint4 keep[kOneShotRegVecs];
      float ss = 0.0f;
      // Two vectors at a time: both vectors' peer loads are issued before either is summed
      // (the stores to h could alias them for the compiler), so a row costs one round trip
      // to the peers per pair instead of one per vector.
#pragma unroll
      for (int i0 = 0; i0 < kOneShotRegVecs; i0 += 2) {
        uint4 parts[2][kRanks], hv[2];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int v = threadIdx.x + (i0 + j) * kOneShotThreads;
          if (v < nvec) {
#pragma unroll
            for (int q = 0; q < kRanks; ++q)
              if (q < a.world)
                parts[j][q] =
                    __ldcg(reinterpret_cast<const uint4*>(a.parts[q] + static_cast<long long>(row) * a.H + v * 8));
            hv[j] = *reinterpret_cast<const uint4*>(hr + v * 8);
          }
        }
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int v = threadIdx.x + (i0 + j) * kOneShotThreads;
          if (v >= nvec) continue;
          const __nv_bfloat16* he = reinterpret_cast<const __nv_bfloat16*>(&hv[j]);
          float acc[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[e] = bf2f(he[e]);
#pragma unroll
          for (int q = 0; q < kRanks; ++q) {
            if (q < a.world) {
              const __nv_bfloat16* pe = reinterpret_cast<const __nv_bfloat16*>(&parts[j][q]);
#pragma unroll
              for (int e = 0; e < 8; ++e) acc[e] += bf2f(pe[e]);
            }
          }
          uint4 out;
          __nv_bfloat162* ob = reinterpret_cast<__nv_bfloat162*>(&out);
#pragma unroll
          for (int e = 0; e < 4; ++e) ob[e] = __floats2bfloat162_rn(acc[2 * e], acc[2 * e + 1]);
          *reinterpret_cast<uint4*>(hr + v * 8) = out;
          keep[i0 + j] = out;
          const __nv_bfloat16* oe = reinterpret_cast<const __nv_bfloat16*>(&out);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const float f = bf2f(oe[e]);
            ss += f * f;
          }
        }
      }
      // rows wider than the register window: finish them from global memory
      for (int v = threadIdx.x + kOneShotRegVecs * kOneShotThreads; v < nvec; v += kOneShotThreads) {
        float acc[8];
        const uint4 hv = *reinterpret_cast<const uint4*>(hr + v * 8);
        const __nv_bfloat16* he = reinterpret_cast<const __nv_bfloat16*>(&hv);
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] = bf2f(he[e]);
        for (int q = 0; q < a.world; ++q) {
          const uint4 pv = __ldcg(reinterpret_cast<const uint4*>(a.parts[q] + static_cast<long long>(row) * a.H + v * 8));
          const __nv_bfloat16* pe = reinterpret_cast<const __nv_bfloat16*>(&pv);
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[e] += bf2f(pe[e]);
        }
        uint4 out;
        __nv_bfloat162* ob = reinterpret_cast<__nv_bfloat162*>(&out);
#pragma unroll
        for (int e = 0; e < 4; ++e) ob[e] = __floats2bfloat162_rn(acc[2 * e], acc[2 * e + 1]);
        *reinterpret_cast<uint4*>(hr + v * 8) = out;
        const __nv_bfloat16* oe = reinterpret_cast<const __nv_bfloat16*>(&out);
#pragma unroll
        for (int e = 0; e < 8; ++e) ss += bf2f(oe[e]) * bf2f(oe[e]);
      }
      if (row == static_cast<int>(blockIdx.x)) ar_stamp(a, 4);
      ss = warp_sum(ss);
      const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
      if (lane == 0) red[warp] = ss;
      __syncthreads();
      if (warp == 0) {
        float t = lane < kOneShotThreads / 32 ? red[lane] : 0.0f;
        t = warp_sum(t);
        if (lane == 0) red[32] = rsqrtf(t / a.H + a.eps);
      }
      __syncthreads();
      if (row == static_cast<int>(blockIdx.x)) ar_stamp(a, 5);
      const float rs = red[32];
      auto emit = [&](int v, const uint4& hv) {
        const uint4 wv = *reinterpret_cast<const uint4*>(a.w + v * 8);
        const __nv_bfloat16* he = reinterpret_cast<const __nv_bfloat16*>(&hv);
        const __nv_bfloat16* we = reinterpret_cast<const __nv_bfloat16*>(&wv);
        uint4 out;
        __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(&out);
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = f2bf(bf2f(we[e]) * bf2f(f2bf(bf2f(he[e]) * rs)));
        *reinterpret_cast<uint4*>(a.x + static_cast<long long>(row) * a.ldx + v * 8) = out;
      };
#pragma unroll
      for (int i = 0; i < kOneShotRegVecs; ++i) {
        const int v = threadIdx.x + i * kOneShotThreads;
        if (v < nvec) emit(v, keep[i]);
      }
      for (int v = threadIdx.x + kOneShotRegVecs * kOneShotThreads; v < nvec; v += kOneShotThreads)
        emit(v, *reinterpret_cast<const uint4*>(hr + v * 8));
      __syncthreads();
      if (row == static_cast<int>(blockIdx.x)) ar_stamp(a, 6);
    }
  }
  finish_call(a, epoch);
  ar_stamp(a, 7);
}

// Two-shot in one kernel (more than four ranks): phase A reduces this rank's row
// slice (peer loads of every rank's partial, rank order) into h and the
// symmetric row buffer; the last block to finish publishes slot 3 and every
// block waits for all peers (the grid is sized to be co-resident); phase B
// copies the other ranks' reduced rows and applies RMSNorm to every row.
__global__ void __launch_bounds__(kOneShotThreads) twoshot_norm_kernel(const ArArgs a) {
  pdl_wait();
  const uint32_t epoch = *a.epoch + 1;
  bool ok = rank_barrier(a, 2, epoch);
  const int r0 = slice_begin(a.T, a.world, a.rank), r1 = slice_begin(a.T, a.world, a.rank + 1);
  const int nvec = a.H / 8;
  if (ok) {
    for (int row = r0 + blockIdx.x; row < r1; row += gridDim.x) {
      __nv_bfloat16* hr = a.h + static_cast<long long>(row) * a.ldh;
      for (int v = threadIdx.x; v < nvec; v += blockDim.x) {
        uint4 parts[kMaxRanks];
#pragma unroll
        for (int q = 0; q < kMaxRanks; ++q)
          if (q < a.world)
            parts[q] = __ldcg(reinterpret_cast<const uint4*>(a.parts[q] + static_cast<long long>(row) * a.H + v * 8));
        const uint4 hv = *reinterpret_cast<const uint4*>(hr + v * 8);
        const __nv_bfloat16* he = reinterpret_cast<const __nv_bfloat16*>(&hv);
        float acc[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] = bf2f(he[e]);
#pragma unroll
        for (int q = 0; q < kMaxRanks; ++q) {
          if (q < a.world) {
            const __nv_bfloat16* pe = reinterpret_cast<const __nv_bfloat16*>(&parts[q]);
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[e] += bf2f(pe[e]);
          }
        }
        uint4 out;
        __nv_bfloat162* ob = reinterpret_cast<__nv_bfloat162*>(&out);
#pragma unroll
        for (int e = 0; e < 4; ++e) ob[e] = __floats2bfloat162_rn(acc[2 * e], acc[2 * e + 1]);
        *reinterpret_cast<uint4*>(hr + v * 8) = out;
        *reinterpret_cast<uint4*>(a.rows[a.rank] + static_cast<long long>(row) * a.H + v * 8) = out;
      }
    }
  }
  // every block's reduced rows must be visible to the peers before the slot-3 signal
  __threadfence_system();
  __syncthreads();
  __shared__ int last, ok2;
  if (threadIdx.x == 0) {
    const uint32_t done = atomicAdd(a.epoch + 2, 1u);   // phase-A arrivals (epoch[1] counts the call's end)
    last = done == gridDim.x - 1;
    if (last) a.epoch[2] = 0;
  }
  __syncthreads();
  if (last && threadIdx.x < a.world) st_release_sys(a.pads[threadIdx.x] + 3 * kMaxRanks + a.rank, epoch);
  if (threadIdx.x == 0) {
    ok2 = 1;
    const uint32_t* mine = a.pads[a.rank] + 3 * kMaxRanks;
    const unsigned long long start = global_ns();
    for (int q = 0; q < a.world && ok2; ++q) {
      while (static_cast<int>(ld_acquire_sys(mine + q) - epoch) < 0) {
        if (global_ns() - start > wait_limit(a.wait_ns)) {
          record_error(a.status, kErrPeerWait);
          ok2 = 0;
          break;
        }
      }
    }
  }
  __syncthreads();
  pdl_trigger();     // every block has passed the phase barrier: the grid no longer needs co-residency
  __shared__ float red[33];
  if (ok && ok2) {
    for (int row = blockIdx.x; row < a.T; row += gridDim.x) {
      int owner = 0;
      while (owner + 1 < a.world && slice_begin(a.T, a.world, owner + 1) <= row) ++owner;
      __nv_bfloat16* hr = a.h + static_cast<long long>(row) * a.ldh;
      float ss = 0.0f;
      for (int v = threadIdx.x; v < nvec; v += blockDim.x) {
        uint4 val;
        if (owner == a.rank) {
          val = *reinterpret_cast<const uint4*>(hr + v * 8);
        } else {
          val = __ldcg(reinterpret_cast<const uint4*>(a.rows[owner] + static_cast<long long>(row) * a.H + v * 8));
          *reinterpret_cast<uint4*>(hr + v * 8) = val;
        }
        const __nv_bfloat16* e8 = reinterpret_cast<const __nv_bfloat16*>(&val);
#pragma unroll
        for (int e = 0; e < 8; ++e) ss += bf2f(e8[e]) * bf2f(e8[e]);
      }
      ss = warp_sum(ss);
      const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
      if (lane == 0) red[warp] = ss;
      __syncthreads();
      if (warp == 0) {
        float t = lane < kOneShotThreads / 32 ? red[lane] : 0.0f;
        t = warp_sum(t);
        if (lane == 0) red[32] = rsqrtf(t / a.H + a.eps);
      }
      __syncthreads();
      const float rs = red[32];
      for (int v = threadIdx.x; v < nvec; v += blockDim.x) {
        const uint4 hv = *reinterpret_cast<const uint4*>(hr + v * 8);
        const uint4 wv = *reinterpret_cast<const uint4*>(a.w + v * 8);
        const __nv_bfloat16* he = reinterpret_cast<const __nv_bfloat16*>(&hv);
        const __nv_bfloat16* we = reinterpret_cast<const __nv_bfloat16*>(&wv);
        uint4 out;
        __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(&out);
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = f2bf(bf2f(we[e]) * bf2f(f2bf(bf2f(he[e]) * rs)));
        *reinterpret_cast<uint4*>(a.x + static_cast<long long>(row) * a.ldx + v * 8) = out;
      }
      __syncthreads();
    }
  }
  finish_call(a, epoch);
}

}  // namespace

unsigned long long*& allreduce_trace_buffer() {
  static unsigned long long* buf = nullptr;
  return buf;
}

cudaError_t allreduce_add_rmsnorm_launch(const ArArgs& a0, int blocks, cudaStream_t stream) {
  ArArgs a = a0;
  a.trace = allreduce_trace_buffer();
  if (a.world < 1 || a.world > kMaxRanks || a.H % 8 || a.T <= 0) return cudaErrorInvalidValue;
  if (a.algorithm < 0 || a.algorithm > 2) return cudaErrorInvalidValue;
  // "auto": one-shot up to four ranks, and above that while each rank's peer reads stay small.
  // Measured on two B200s with graph-replayed calls (T = 64 / 256 rows of 3584): one-shot 12.0 /
  // 13.6 us, two-shot 24.6 / 26.4 us -- a call is bound by its barriers, not its bytes, so the
  // second barrier of two-shot costs more than reading 7 partials of a decode batch would.
  const long long peer_bytes = static_cast<long long>(a.world - 1) * a.T * a.H * 2;
  const bool oneshot = a.algorithm == 1 || (a.algorithm == 0 && (a.world <= 4 || peer_bytes <= kOneShotPeerBytes));
  if (oneshot) {
    // one row per block (the blocks of a row wait on remote loads; more rows in flight hide that latency)
    const int cap = 4 * blocks;
    const int grid = a.T < cap ? a.T : cap;
    const dim3 g(grid > 0 ? grid : 1), blk(kOneShotThreads);
    if (a.world <= 2) return launch_pdl(oneshot_norm_kernel<false, 2>, g, blk, 0, stream, a);
    if (a.world <= 4) return launch_pdl(oneshot_norm_kernel<false, 4>, g, blk, 0, stream, a);
    return launch_pdl(oneshot_norm_kernel<false, kMaxRanks>, g, blk, 0, stream, a);
  }
  // every block of the two-shot kernel waits for the others between its phases: keep the grid co-resident
  static int resident = 0;
  if (resident == 0) {
    int per_sm = 0, dev = 0, sms = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, twoshot_norm_kernel, kOneShotThreads, 0) !=
            cudaSuccess || per_sm < 1)
      per_sm = 1;
    resident = per_sm * (sms > 0 ? sms : 148);
  }
  int grid = blocks < a.T ? blocks : a.T;
  if (grid > resident) grid = resident;
  return launch_pdl(twoshot_norm_kernel, dim3(grid > 0 ? grid : 1), dim3(kOneShotThreads), 0, stream, a);
}

cudaError_t allreduce_pushed_add_rmsnorm_launch(const ArArgs& a0, int blocks, cudaStream_t stream) {
  ArArgs a = a0;
  a.trace = allreduce_trace_buffer();
  if (a.world < 1 || a.world > kMaxRanks || a.H % 8 || a.T <= 0) return cudaErrorInvalidValue;
  const int cap = 4 * blocks;
  const int grid = a.T < cap ? a.T : cap;
  const dim3 g(grid > 0 ? grid : 1), blk(kOneShotThreads);
  if (a.world <= 2) return launch_pdl(oneshot_norm_kernel<true, 2>, g, blk, 0, stream, a);
  if (a.world <= 4) return launch_pdl(oneshot_norm_kernel<true, 4>, g, blk, 0, stream, a);
  return launch_pdl(oneshot_norm_kernel<true, kMaxRanks>, g, blk, 0, stream, a);
}

}  // namespace osb
