// No-allocation entry point of the tcgen05 GEMM (see gemm_noalloc.h).
//
// The split-K scratch of the regular GEMM lives here in one file-scope device
// array.  In host code the array's name is only a host-side stand-in, never a
// device address, so the entry point resolves the real device address once per
// device with cudaGetSymbolAddress (with that device current) and passes that
// pointer to the existing GEMM launcher.
#include <cstdio>
#include <mutex>

#include "gemm.h"
#include "gemm_noalloc.h"

namespace {

constexpr long long kPartialFloats = 2621440;  // 10 MiB of fp32 partial tiles
constexpr int kCounterSlots = 1024;
constexpr int kMaxDevices = 64;
constexpr size_t kScratchBytes = kPartialFloats * 4 + kCounterSlots * 4 + 256;

// [partials: kPartialFloats fp32][counters: kCounterSlots int32][status: int32, padded to 256 B]
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

std::once_flag g_once[kMaxDevices];
cudaError_t g_setup_error[kMaxDevices];
unsigned char* g_scratch_ptr[kMaxDevices];
int g_sm_count[kMaxDevices];

thread_local char g_message[256] = "no error";

int fail(int code, const char* fmt, long long a = 0, long long b = 0) {
  std::snprintf(g_message, sizeof(g_message), fmt, a, b);
  return code;
}

}  // namespace

extern "C" __attribute__((visibility("default"))) long long osb_gemm_noalloc_scratch_floats(void) {
  return kPartialFloats;
}

extern "C" __attribute__((visibility("default"))) const char* osb_gemm_noalloc_last_error(void) { return g_message; }

extern "C" __attribute__((visibility("default"))) int osb_gemm_bf16_noalloc(
    const void* w, long long ldw, const void* x, long long ldx, int M, int N, int K, void* out, long long ldo,
    int out_f32, const void* bias, const void* residual, long long ldr, int swiglu, void* stream) {
  if (!w || !x || !out || M <= 0 || N <= 0 || K <= 0 || ldw < K || ldx < K)
    return fail(OSB_NOALLOC_ERR_ARGUMENT, "invalid GEMM arguments (M=%lld, N=%lld)", M, N);
  if (swiglu && (M % 128)) return fail(OSB_NOALLOC_ERR_ARGUMENT, "swiglu needs M %% 128 == 0 (M=%lld)", M);

  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return fail(OSB_NOALLOC_ERR_SETUP, "no usable current CUDA device (%lld)", dev);
  // Once per device, with that device current: resolve the scratch address.
  std::call_once(g_once[dev], [dev] {
    void* p = nullptr;
    g_setup_error[dev] = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    g_scratch_ptr[dev] = static_cast<unsigned char*>(p);
    int sms = 0;
    if (g_setup_error[dev] == cudaSuccess)
      g_setup_error[dev] = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    g_sm_count[dev] = sms > 0 ? sms : 148;
  });
  if (g_setup_error[dev] != cudaSuccess || g_scratch_ptr[dev] == nullptr)
    return fail(OSB_NOALLOC_ERR_SETUP, "cudaGetSymbolAddress of the GEMM scratch failed (error %lld)",
                static_cast<long long>(g_setup_error[dev]));

  // The split-K plan of the regular launcher, to size the scratch it will use.
  const int bn = osb::gemm_pick_bn(N);
  const long long tiles = static_cast<long long>((M + 127) / 128) * ((N + bn - 1) / bn);
  const int kb = (K + 63) / 64;
  const int sms = g_sm_count[dev];
  long long splits = 1;
  if (tiles < sms) {
    long long want = sms / tiles;
    if (want < 1) want = 1;
    const long long cap = kb / 2 > 1 ? kb / 2 : 1;
    if (want > cap) want = cap;
    const long long per = (kb + want - 1) / want;
    splits = (kb + per - 1) / per;
  }
  const long long need = splits > 1 ? splits * tiles * 128 * bn : 0;
  if (need > kPartialFloats || (splits > 1 && tiles > kCounterSlots))
    return fail(OSB_NOALLOC_ERR_SCRATCH_TOO_SMALL,
                "problem needs %lld fp32 of split-K scratch; the no-allocation GEMM holds at most %lld", need,
                kPartialFloats);

  unsigned char* base = g_scratch_ptr[dev];
  float* partials = reinterpret_cast<float*>(base);
  int* counters = reinterpret_cast<int*>(base + kPartialFloats * 4);
  int* status = counters + kCounterSlots;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // Counters and the status word must start at zero; the array keeps the last call's contents.
  if (cudaMemsetAsync(counters, 0, (kCounterSlots + 1) * sizeof(int), s) != cudaSuccess)
    return fail(OSB_NOALLOC_ERR_LAUNCH, "clearing the scratch counters failed (%lld)", 0);

  osb::GemmProblem p{};
  p.w = static_cast<const __nv_bfloat16*>(w);
  p.ldw = ldw;
  p.x = static_cast<const __nv_bfloat16*>(x);
  p.ldx = ldx;
  p.M = M;
  p.N = N;
  p.K = K;
  p.out = out;
  p.ldo = ldo;
  p.out_f32 = out_f32 ? 1 : 0;
  p.bias = static_cast<const __nv_bfloat16*>(bias);
  p.residual = static_cast<const __nv_bfloat16*>(residual);
  p.ldr = ldr;
  p.epilogue = swiglu ? 1 : 0;
  p.allow_split = 1;
  p.split_mode = 1;  // split-K partials in the static scratch
  p.workspace = partials;
  p.workspace_floats = kPartialFloats;
  p.counters = counters;
  p.counter_slots = kCounterSlots;
  p.status = status;
  const cudaError_t e = osb::gemm_launch(p, s);
  if (e != cudaSuccess)
    return fail(OSB_NOALLOC_ERR_LAUNCH, "GEMM launch failed (cuda error %lld)", static_cast<long long>(e));
  std::snprintf(g_message, sizeof(g_message), "no error");
  return OSB_NOALLOC_OK;
}
