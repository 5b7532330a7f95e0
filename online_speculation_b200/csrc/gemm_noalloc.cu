// No-allocation entry point of the tcgen05 GEMM (see gemm_noalloc.h).
//
// The split-K scratch of the regular GEMM lives here in one file-scope device
// array.  In host code the array's name is only a host-side stand-in, never a
// device address, so the entry point resolves the real device address once per
// device with cudaGetSymbolAddress (with that device current) and passes that
// pointer to the existing GEMM launcher.
#include <cstdint>
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

struct DeviceSetup {
  std::mutex lock;
  bool ready = false;              // set only once the address and the SM count are known
  unsigned char* scratch = nullptr;
  int sms = 0;
};
DeviceSetup g_setup[kMaxDevices];

thread_local char g_message[256] = "no error";

int fail(int code, const char* fmt, long long a = 0, long long b = 0) {
  std::snprintf(g_message, sizeof(g_message), fmt, a, b);
  return code;
}

// Resolves the scratch address for the current device `dev`; a failure leaves the
// device un-initialised, so a later call retries.
cudaError_t setup_device(int dev, unsigned char** scratch, int* sms) {
  DeviceSetup& d = g_setup[dev];
  std::lock_guard<std::mutex> guard(d.lock);
  if (!d.ready) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return e;
    int n = 0;
    e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    d.scratch = static_cast<unsigned char*>(p);
    d.sms = n > 0 ? n : 148;
    d.ready = true;
  }
  *scratch = d.scratch;
  *sms = d.sms;
  return cudaSuccess;
}

int current_device_scratch(unsigned char** scratch, int* sms) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return fail(OSB_NOALLOC_ERR_SETUP, "no usable current CUDA device (%lld)", dev);
  const cudaError_t e = setup_device(dev, scratch, sms);
  if (e != cudaSuccess)
    return fail(OSB_NOALLOC_ERR_SETUP, "resolving the GEMM scratch address failed (cuda error %lld)",
                static_cast<long long>(e));
  return OSB_NOALLOC_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" __attribute__((visibility("default"))) long long osb_gemm_noalloc_scratch_floats(void) {
  return kPartialFloats;
}

extern "C" __attribute__((visibility("default"))) const char* osb_gemm_noalloc_last_error(void) { return g_message; }

extern "C" __attribute__((visibility("default"))) int osb_gemm_noalloc_status(void* stream, int* code) {
  if (code == nullptr) return fail(OSB_NOALLOC_ERR_ARGUMENT, "status destination is null (%lld)", 0);
  unsigned char* base = nullptr;
  int sms = 0;
  const int rc = current_device_scratch(&base, &sms);
  if (rc != OSB_NOALLOC_OK) return rc;
  int* status = reinterpret_cast<int*>(base + kPartialFloats * 4 + kCounterSlots * 4);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // Wait for the stream's GEMMs, then read and clear the word (synchronous copies).
  if (cudaStreamSynchronize(s) != cudaSuccess || cudaMemcpy(code, status, sizeof(int), cudaMemcpyDeviceToHost) !=
                                                     cudaSuccess ||
      cudaMemsetAsync(status, 0, sizeof(int), s) != cudaSuccess || cudaStreamSynchronize(s) != cudaSuccess)
    return fail(OSB_NOALLOC_ERR_LAUNCH, "reading the GEMM status word failed (%lld)", 0);
  return OSB_NOALLOC_OK;
}

extern "C" __attribute__((visibility("default"))) int osb_gemm_bf16_noalloc(
    const void* w, long long ldw, const void* x, long long ldx, int M, int N, int K, void* out, long long ldo,
    int out_f32, const void* bias, const void* residual, long long ldr, int swiglu, void* stream) {
  if (!w || !x || !out || M <= 0 || N <= 0 || K <= 0 || ldw < K || ldx < K)
    return fail(OSB_NOALLOC_ERR_ARGUMENT, "invalid GEMM arguments (M=%lld, N=%lld)", M, N);
  if (swiglu && (M % 128)) return fail(OSB_NOALLOC_ERR_ARGUMENT, "swiglu needs M %% 128 == 0 (M=%lld)", M);
  if (!aligned16(w) || !aligned16(x) || (ldw % 8) || (ldx % 8))
    return fail(OSB_NOALLOC_ERR_ARGUMENT,
                "w and x must start on 16-byte boundaries with row strides that are multiples of 8 (ldw=%lld, "
                "ldx=%lld)",
                ldw, ldx);
  const long long width = swiglu ? M / 2 : M;
  if (ldo < width)
    return fail(OSB_NOALLOC_ERR_ARGUMENT, "output row stride %lld is below the output width %lld", ldo, width);
  if (residual != nullptr && ldr < width)
    return fail(OSB_NOALLOC_ERR_ARGUMENT, "residual row stride %lld is below the output width %lld", ldr, width);

  unsigned char* base = nullptr;
  int sms = 0;
  const int rc = current_device_scratch(&base, &sms);
  if (rc != OSB_NOALLOC_OK) return rc;

  // The regular launcher's own split-K plan decides how much scratch the call needs.
  const osb::GemmPlan plan = osb::gemm_workspace_plan(M, N, K, sms);
  if (plan.workspace_floats > kPartialFloats || (plan.splits > 1 && plan.tiles > kCounterSlots))
    return fail(OSB_NOALLOC_ERR_SCRATCH_TOO_SMALL,
                "problem needs %lld fp32 of split-K scratch; the no-allocation GEMM holds at most %lld",
                plan.workspace_floats, kPartialFloats);

  float* partials = reinterpret_cast<float*>(base);
  int* counters = reinterpret_cast<int*>(base + kPartialFloats * 4);
  int* status = counters + kCounterSlots;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // The tile counters must start at zero; the array keeps the last call's contents
  // (a GEMM whose wait gave up can leave a counter raised).  The status word is
  // left alone: it holds the first error until osb_gemm_noalloc_status reads it.
  if (cudaMemsetAsync(counters, 0, kCounterSlots * sizeof(int), s) != cudaSuccess)
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
