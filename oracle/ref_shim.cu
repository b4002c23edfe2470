// ref_shim.cu — extern "C" entry points over fluxrt-cpp's own CUDA kernels (compiled from the
// reference sources by oracle/build_ref.sh). TEST INFRASTRUCTURE ONLY: used by the GPU tests to
// cross-check the bit-exact steps against the reference itself, and as a timing baseline.
// Wrapped interfaces: gather_scatter_kernels.h:21-36,46-49, flux2_kernels.h:15-24,
// attention_kernels.h:20-24, spatial_kv_cache.h:12-55.
#include <cstdint>
#include <cuda_runtime.h>

#include "attention_kernels.h"
#include "flux2_kernels.h"
#include "gather_scatter_kernels.h"
#include "spatial_kv_cache.h"

extern "C" {

void ref_gather_tokens(const float* src, float* dst, const int32_t* idx, int32_t n, int32_t dim,
                       void* stream) {
    fluxrt::plugins::gather_tokens(src, dst, idx, n, dim, static_cast<cudaStream_t>(stream));
}

void ref_scatter_tokens(const float* src, float* dst, const int32_t* idx, int32_t n, int32_t dim,
                        void* stream) {
    fluxrt::plugins::scatter_tokens(src, dst, idx, n, dim, static_cast<cudaStream_t>(stream));
}

void ref_rms_norm(const float* x, float* y, const float* w, float eps, int32_t rows, int32_t dim,
                  void* stream) {
    fluxrt::plugins::launch_rms_norm(x, y, w, eps, rows, dim, static_cast<cudaStream_t>(stream));
}

void ref_gelu(float* data, int32_t n, void* stream) {
    fluxrt::plugins::launch_gelu(data, n, static_cast<cudaStream_t>(stream));
}

void ref_bias_add(float* data, const float* bias, int32_t rows, int32_t dim, void* stream) {
    fluxrt::plugins::launch_bias_add(data, bias, rows, dim, static_cast<cudaStream_t>(stream));
}

void ref_apply_modulation(const float* x, const float* scale, const float* shift, float* out,
                          int32_t rows, int32_t dim, void* stream) {
    fluxrt::plugins::apply_modulation(x, scale, shift, out, rows, dim, static_cast<cudaStream_t>(stream));
}

void ref_attention_fwd(const float* q, const float* k, const float* v, float* out, int32_t b,
                       int32_t h, int32_t q_len, int32_t kv_len, int32_t d, void* stream) {
    fluxrt::plugins::attention_fwd(q, k, v, out, b, h, q_len, kv_len, d,
                                   static_cast<cudaStream_t>(stream));
}

// SpatialCache through an opaque handle; returns nullptr / nonzero on a thrown RuntimeError.
void* ref_cache_create(int img, int txt, int out_ch, int heads, int head_dim, int n_double,
                       int n_single) {
    try {
        return new fluxrt::kernels::SpatialCache(img, txt, out_ch, heads, head_dim, n_double, n_single);
    } catch (...) {
        return nullptr;
    }
}
void ref_cache_destroy(void* c) { delete static_cast<fluxrt::kernels::SpatialCache*>(c); }
int ref_cache_reset(void* c, void* s) {
    try { static_cast<fluxrt::kernels::SpatialCache*>(c)->reset(static_cast<cudaStream_t>(s)); } catch (...) { return 1; }
    return 0;
}
int ref_cache_preprocess_mask(void* c, int32_t* mask, void* s) {
    try { static_cast<fluxrt::kernels::SpatialCache*>(c)->preprocess_mask(mask, static_cast<cudaStream_t>(s)); } catch (...) { return 1; }
    return 0;
}
int ref_cache_sync_output(void* c, float* pred, const int32_t* mask, void* s) {
    try { static_cast<fluxrt::kernels::SpatialCache*>(c)->sync_output_cache(pred, mask, static_cast<cudaStream_t>(s)); } catch (...) { return 1; }
    return 0;
}
int ref_cache_sync_kv(void* c, float* keys, float* values, const int32_t* mask, int block_id,
                      int is_double, void* s) {
    try {
        static_cast<fluxrt::kernels::SpatialCache*>(c)->sync_kv_cache(keys, values, mask, block_id, is_double != 0,
                                                                      static_cast<cudaStream_t>(s));
    } catch (...) { return 1; }
    return 0;
}

}  // extern "C"
