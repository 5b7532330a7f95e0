// Host API of the per-token kernels (see elementwise.cu).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace osb {

cudaError_t rmsnorm_launch(const __nv_bfloat16* x, long long ldx, __nv_bfloat16* h, long long ldh,
                           const __nv_bfloat16* delta, long long ldd, const __nv_bfloat16* w, __nv_bfloat16* y,
                           long long ldy, int T, int H, float eps, cudaStream_t stream);
cudaError_t rope_cache_launch(const __nv_bfloat16* qkv, long long ldqkv, const int* positions, const int* slots,
                              const float* inv_freq, const __nv_bfloat16* qn_w, const __nv_bfloat16* kn_w, float eps,
                              __nv_bfloat16* q_out, __nv_bfloat16* k_cache, __nv_bfloat16* v_cache, int T, int Hq,
                              int Hkv, int page, long long slot_capacity, int* status, cudaStream_t stream);
// Indices are checked on the device (OSB_DEVICE_CHECKS): token ids outside [0, V) give a zero
// row and slots at or beyond slot_capacity store nothing; both record kErrBadIndex in *status.
cudaError_t embed_launch(const int* ids, const __nv_bfloat16* table, int V, int T, int H, __nv_bfloat16* out,
                         long long ldo, int* status, cudaStream_t stream);
cudaError_t page_copy_launch(__nv_bfloat16* cache, long long layer_stride, int layers, const int* pairs, int npairs,
                             int Hkv, int page, cudaStream_t stream);

}  // namespace osb
