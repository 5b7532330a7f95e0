// No-allocation entry point of the tcgen05 GEMM.
//
// This entry point has no counterpart in the reference project; it exists
// for callers that cannot allocate GPU memory themselves -- for example code
// running inside a custom allocator or memory-pool callback, a plugin host
// that forbids cudaMalloc after start-up, or a real-time loop where an
// allocation could block or fail.  The regular GEMM (osb::gemm_launch) needs a
// caller-provided split-K workspace and counter array; this variant keeps that
// scratch in a fixed, file-scope device array instead, so the caller passes
// only inputs and outputs.
//
// Limits and behaviour:
//  * Scratch: a static device array of 10 MiB of fp32 split-K partial tiles
//    (2,621,440 floats) plus 1024 tile counters and one status word.  Every GPU
//    that loads this library holds that memory until the process exits.
//  * Problems whose split-K plan needs more partial-tile scratch than that are
//    rejected with OSB_NOALLOC_ERR_SCRATCH_TOO_SMALL (the GEMM is not run).  The
//    plan is the regular launcher's own (osb::gemm_workspace_plan), so exactly
//    the problems that it would serve from this scratch are accepted.
//  * The first call on a device resolves the scratch address for that device
//    (cudaGetSymbolAddress, which may load the module); make that first call
//    before any stream capture on the device.  If that set-up fails, the call
//    returns OSB_NOALLOC_ERR_SETUP and the next call on the device tries again.
//  * Device-side waits inside the GEMM are bounded; one that gives up writes an
//    error code into the scratch's status word, and the output is then not
//    valid.  The word keeps its first error until osb_gemm_noalloc_status reads
//    and clears it, so check it after the calls whose result you rely on.
//  * All calls share the one scratch array, which keeps the last call's
//    contents.  Calls whose executions overlap on the GPU (different streams,
//    or different host threads without ordering) race on it; serialise them.
//  * The call allocates nothing: no cudaMalloc, no cudaFree, no allocating
//    library routine.  It clears the counters and the status word it uses with
//    cudaMemsetAsync on the given stream before launching.
#pragma once

#ifdef __cplusplus
extern "C" {
#endif

enum {
  OSB_NOALLOC_OK = 0,
  OSB_NOALLOC_ERR_ARGUMENT = 1,            // bad sizes, strides or alignment
  OSB_NOALLOC_ERR_SCRATCH_TOO_SMALL = 2,   // split-K plan exceeds the static scratch
  OSB_NOALLOC_ERR_SETUP = 3,               // resolving the scratch address failed
  OSB_NOALLOC_ERR_LAUNCH = 4,              // memset, copy or kernel launch failed
};

// out[N, M] (or [N, M/2] with swiglu) = x[N, K] @ w[M, K]^T (+ bias[M]) (+ residual)
// All matrices bf16 row-major (out fp32 when out_f32 != 0); strides in elements.
// w and x must start on 16-byte boundaries with ldw and ldx multiples of 8;
// ldo (and ldr when a residual is given) must cover the output width.
// `stream` is a cudaStream_t (may be null for the legacy default stream).
int osb_gemm_bf16_noalloc(const void* w, long long ldw, const void* x, long long ldx, int M, int N, int K, void* out,
                          long long ldo, int out_f32, const void* bias, const void* residual, long long ldr,
                          int swiglu, void* stream);

// Waits for `stream`, then stores the status word of the current device's scratch
// into *code (0: every GEMM since the last read finished its waits) and clears
// it.  Returns OSB_NOALLOC_OK or an error code of the copy itself.
int osb_gemm_noalloc_status(void* stream, int* code);

// Capacity of the static split-K scratch, in fp32 elements.
long long osb_gemm_noalloc_scratch_floats(void);

// Human-readable text of the last error returned on this host thread.
const char* osb_gemm_noalloc_last_error(void);

#ifdef __cplusplus
}
#endif
