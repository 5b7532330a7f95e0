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
//    bf16 output.
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
constexpr int kThreads = 192;

struct Args {
  int M, N, K;          // M = weight rows (features), N = tokens
  int k_blocks;
  int tiles_m, tiles_n, splits, kb_per_split;
  void* out;
  long long ldo;
  const __nv_bfloat16* residual;
  long long ldr;
  const __nv_bfloat16* bias;
  int epilogue;         // 0 linear, 1 swiglu
  int out_f32;
  float* workspace;
  int* counters;
  int* status;
};

template <int BN>
struct Smem {
  static constexpr int kStages = BN <= 32 ? 10 : BN <= 64 ? 8 : BN <= 128 ? 6 : 4;
  static constexpr int kABytes = kBM * kBK * 2;
  static constexpr int kBBytes = BN * kBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kTmemCols = 2 * BN < 32 ? 32 : 2 * BN;
  static constexpr int kXchgBytes = 32 * 64 * 4;
  static constexpr int kBarBytes = 256;
  static constexpr int kTotal = 1024 + kStages * kStageBytes + kBarBytes + kXchgBytes;
};

template <int BN>
__device__ __forceinline__ void finish_chunk(const Args& a, const float (&v)[32], int tm, int tn, int chunk, int r,
                                             float* xchg) {
  const int t0 = tn * BN + chunk * 32;
  if (a.epilogue == 1) {
    // rows [0,64) hold gate, rows [64,128) hold up for the same 64 features.
    if (r >= 64) {
#pragma unroll
      for (int j = 0; j < 32; ++j) xchg[j * 64 + (r - 64)] = v[j];
    }
    named_barrier(1, 128);
    const int f = tm * 64 + r;
    if (r < 64 && f < a.M / 2) {
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int t = t0 + j;
        if (t < a.N) {
          const float g = v[j];
          const float u = xchg[j * 64 + r];
          const float s = g / (1.0f + __expf(-g));
          float val = s * u;
          if (a.residual) val += bf2f(a.residual[t * a.ldr + f]);
          if (a.out_f32)
            static_cast<float*>(a.out)[t * a.ldo + f] = val;
          else
            static_cast<__nv_bfloat16*>(a.out)[t * a.ldo + f] = f2bf(val);
        }
      }
    }
    named_barrier(1, 128);
    return;
  }
  const int f = tm * kBM + r;
  if (f >= a.M) return;
  const float b = a.bias ? bf2f(a.bias[f]) : 0.0f;
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const int t = t0 + j;
    if (t < a.N) {
      float val = v[j] + b;
      if (a.residual) val += bf2f(a.residual[t * a.ldr + f]);
      if (a.out_f32)
        static_cast<float*>(a.out)[t * a.ldo + f] = val;
      else
        static_cast<__nv_bfloat16*>(a.out)[t * a.ldo + f] = f2bf(val);
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

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 4);
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

  const int total = a.tiles_m * a.tiles_n * a.splits;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      for (int w = blockIdx.x; w < total && ok; w += gridDim.x) {
        const int split = w % a.splits;
        const int tile = w / a.splits;
        const int tm = tile % a.tiles_m;
        const int tn = tile / a.tiles_m;
        const int kb0 = split * a.kb_per_split;
        const int kb1 = min(a.k_blocks, kb0 + a.kb_per_split);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, a.status, kErrTmaWait)) {
            ok = false;
            *abort_flag = 1;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], S::kStageBytes);
          tma_load_2d(sA + stage * S::kABytes, &tmA, kb * kBK, tm * kBM, &full[stage]);
          tma_load_2d(sB + stage * S::kBBytes, &tmB, kb * kBK, tn * BN, &full[stage]);
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
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
      if (!ok) *abort_flag = 1;
    }
  } else {
    // Epilogue warps 2..5 -> TMEM lane quarter (warp % 4).
    const int quarter = warp % 4;
    const int r = quarter * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    int acc = 0;
    uint32_t acc_phase = 0;
    const int ep_tid = threadIdx.x - 64;
    for (int w = blockIdx.x; w < total; w += gridDim.x) {
      const int split = w % a.splits;
      const int tile = w / a.splits;
      const int tm = tile % a.tiles_m;
      const int tn = tile / a.tiles_m;
      bool ok = mbar_wait(&tfull[acc], acc_phase, a.status, kErrEpilogueWait);
      // All epilogue threads must agree before touching shared state.
      if (!ok) *abort_flag = 1;
      named_barrier(1, 128);
      if (*abort_flag) break;
      tc_fence_after();
      const uint32_t t_acc = tmem_base + lane_base + acc * BN;
      if (a.splits == 1) {
        for (int c = 0; c < BN / 32; ++c) {
          float v[32];
          tmem_ld32(t_acc + c * 32, v);
          finish_chunk<BN>(a, v, tm, tn, c, r, xchg);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[acc]);
      } else {
        float* part = a.workspace + (static_cast<long long>(split) * a.tiles_m * a.tiles_n + tile) * (kBM * BN);
        for (int c = 0; c < BN / 32; ++c) {
          float v[32];
          tmem_ld32(t_acc + c * 32, v);
#pragma unroll
          for (int j = 0; j < 32; ++j) __stcg(&part[(c * 32 + j) * kBM + r], v[j]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[acc]);
        __threadfence();
        named_barrier(1, 128);
        if (ep_tid == 0) {
          const int prev = atomicAdd(&a.counters[tile], 1);
          const int last = prev == a.splits - 1;
          if (last) a.counters[tile] = 0;
          *last_flag = last;
        }
        named_barrier(1, 128);
        const int is_last = *last_flag;
        named_barrier(1, 128);
        if (is_last) {
          __threadfence();
          const long long tile_stride = static_cast<long long>(a.tiles_m) * a.tiles_n * (kBM * BN);
          const float* base = a.workspace + static_cast<long long>(tile) * (kBM * BN);
          for (int c = 0; c < BN / 32; ++c) {
            float v[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = 0.0f;
            for (int s = 0; s < a.splits; ++s) {
              const float* p = base + s * tile_stride;
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] += __ldcg(&p[(c * 32 + j) * kBM + r]);
            }
            finish_chunk<BN>(a, v, tm, tn, c, r, xchg);
          }
        }
      }
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, S::kTmemCols);
  }
}

// ------------------------------------------------------------------ host ----
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
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

template <int BN>
cudaError_t launch_bn(const GemmProblem& p, const Args& a0, cudaStream_t stream) {
  using S = Smem<BN>;
  CUtensorMap ma, mb;
  if (!make_map(&ma, p.w, p.M, p.K, p.ldw, kBM)) return cudaErrorInvalidValue;
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
  a.splits = 1;
  a.kb_per_split = a.k_blocks;
  if (p.allow_split && tiles < sms && p.workspace != nullptr) {
    int want = std::max(1, sms / tiles);
    want = std::min(want, std::max(1, a.k_blocks / 2));
    int per = (a.k_blocks + want - 1) / want;
    int splits = (a.k_blocks + per - 1) / per;
    const long long need = static_cast<long long>(splits) * tiles * kBM * BN;
    if (splits > 1 && need <= p.workspace_floats && tiles <= p.counter_slots) {
      a.splits = splits;
      a.kb_per_split = per;
    }
  }
  const int total = tiles * a.splits;
  const int grid = std::min(total, sms);
  gemm_tn_kernel<BN><<<grid, kThreads, S::kTotal, stream>>>(ma, mb, a);
  return cudaGetLastError();
}

}  // namespace

int gemm_pick_bn(int tokens) {
  if (tokens <= 32) return 32;
  if (tokens <= 64) return 64;
  if (tokens <= 128) return 128;
  return 256;
}

long long gemm_workspace_floats(int M, int N, int K, int sms) {
  const int bn = gemm_pick_bn(N);
  const long long tiles = static_cast<long long>((M + kBM - 1) / kBM) * ((N + bn - 1) / bn);
  const int kb = (K + kBK - 1) / kBK;
  long long splits = std::min<long long>(std::max<long long>(1, sms / std::max<long long>(1, tiles)),
                                         std::max(1, kb / 2));
  return splits * tiles * kBM * bn;
}

cudaError_t gemm_launch(const GemmProblem& p, cudaStream_t stream) {
  if (p.M <= 0 || p.N <= 0 || p.K <= 0) return cudaErrorInvalidValue;
  if ((p.ldw % 8) || (p.ldx % 8) || (reinterpret_cast<uintptr_t>(p.w) % 16) ||
      (reinterpret_cast<uintptr_t>(p.x) % 16))
    return cudaErrorInvalidValue;  // TMA needs 16-byte aligned rows
  if (p.epilogue == 1 && (p.M % kBM)) return cudaErrorInvalidValue;
  Args a{};
  a.M = p.M;
  a.N = p.N;
  a.K = p.K;
  a.k_blocks = (p.K + kBK - 1) / kBK;
  const int bn = gemm_pick_bn(p.N);
  a.tiles_m = (p.M + kBM - 1) / kBM;
  a.tiles_n = (p.N + bn - 1) / bn;
  a.out = p.out;
  a.ldo = p.ldo;
  a.residual = p.residual;
  a.ldr = p.ldr;
  a.bias = p.bias;
  a.epilogue = p.epilogue;
  a.out_f32 = p.out_f32;
  a.workspace = p.workspace;
  a.counters = p.counters;
  a.status = p.status;
  switch (bn) {
    case 32: return launch_bn<32>(p, a, stream);
    case 64: return launch_bn<64>(p, a, stream);
    case 128: return launch_bn<128>(p, a, stream);
    default: return launch_bn<256>(p, a, stream);
  }
}

}  // namespace osb
