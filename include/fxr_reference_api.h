// fxr_reference_api.h — the fluxrt-cpp kernel-layer interfaces of the sparse attention path,
// re-implemented on the sm_100a library so that existing C++ callers of those functions link
// unchanged. Names, argument order and meaning, fp32 data, asynchronous void-returning launches on
// the caller's stream and the throwing SpatialCache follow the reference declarations cited below;
// the implementations are this library's kernels (include/fxr.h).
//
// Replaced declarations (fluxrt-cpp paths):
//   fluxrt::plugins::gather_tokens / scatter_tokens   src/inference/plugins/gather_scatter_kernels.h:21-36
//   fluxrt::plugins::apply_modulation                 src/inference/plugins/gather_scatter_kernels.h:38-49
//   fluxrt::plugins::layer_norm_modulated             src/inference/plugins/gather_scatter_kernels.h:51-63
//   fluxrt::plugins::launch_gelu / launch_bias_add /  src/inference/plugins/flux2_kernels.h:15-33
//     launch_rms_norm / launch_elem_add / launch_scale_add
//   fluxrt::plugins::attention_fwd                    src/inference/plugins/attention_kernels.h:20-24
//   fluxrt::kernels::SpatialCache                     src/inference/kernels/spatial_kv_cache.h:12-55
// With these, libfxr.so takes the place of the reference's fluxrt_kernels library and of the kernel
// sources its plugins compile (src/CMakeLists.txt:25-27; gather_scatter_kernels.cu, flux2_kernels.cu,
// attention_kernels.cu). The forwarding headers under include/fluxrt_dropin/ carry the reference's
// header paths, for callers that include them by those names.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <stdexcept>
#include <string>
#include <vector>

// fluxrt::RuntimeError, the exception type SpatialCache throws. A caller built inside the
// reference's source tree (include root src/, src/CMakeLists.txt:10-13) already has it from
// src/utils/error.h:18-21, which is then included here so that the class is defined once; elsewhere
// (this library's own build) the same class is declared here.
#if __has_include("utils/error.h")
#include "utils/error.h"
#else
namespace fluxrt {
class RuntimeError : public std::runtime_error {
public:
    explicit RuntimeError(const std::string& msg) : std::runtime_error(msg) {}
};
}  // namespace fluxrt
#endif

namespace fluxrt {
namespace plugins {

// dst[m, :] = src[indices[m], :] for m < active_count; fp32 rows of `dim` values.
void gather_tokens(const float* src, float* dst, const int32_t* indices, int32_t active_count,
                   int32_t dim, cudaStream_t stream);

// dst[indices[m], :] = src[m, :]; rows not listed keep their values.
void scatter_tokens(const float* src, float* dst, const int32_t* indices, int32_t active_count,
                    int32_t dim, cudaStream_t stream);

// out = (1 + scale) * x + shift; x, out (seq_len, dim), scale, shift (dim).
void apply_modulation(const float* x, const float* scale, const float* shift, float* out,
                      int32_t seq_len, int32_t dim, cudaStream_t stream);

// y = (x - mean) / sqrt(var + eps) [* gamma] [+ beta] per row of `dim` values; gamma, beta (dim)
// or nullptr.
void layer_norm_modulated(const float* x, float* y, const float* gamma, const float* beta, float eps,
                          int32_t seq_len, int32_t dim, cudaStream_t stream);

// In place: data = data * 0.5 * (1 + tanh(0.7978845608 * (data + 0.044715 data^3))).
void launch_gelu(float* data, int32_t n, cudaStream_t stream);

// data[r, :] += bias over (seq_len, dim); a null bias does nothing.
void launch_bias_add(float* data, const float* bias, int32_t seq_len, int32_t dim, cudaStream_t stream);

// y = x * rsqrt(mean(x^2) + eps) * weight over rows of `dim` values (seq_len rows).
void launch_rms_norm(const float* x, float* y, const float* weight, float eps, int32_t seq_len,
                     int32_t dim, cudaStream_t stream);

// z = x + y over n values.
void launch_elem_add(const float* x, const float* y, float* z, int32_t n, cudaStream_t stream);

// out = x + gate * y over n values.
void launch_scale_add(const float* x, const float* y, float* out, float gate, int32_t n,
                      cudaStream_t stream);

// out = softmax(Q K^T / sqrt(head_dim)) V per (batch, head), layout (batch, heads, len, head_dim),
// fp32. Computes the intended joint softmax over all kv_len keys (the reference kernel's
// warp-local reduction is not reproduced).
void attention_fwd(const float* Q, const float* K, const float* V, float* out, int32_t batch,
                   int32_t num_heads, int32_t q_len, int32_t kv_len, int32_t head_dim,
                   cudaStream_t stream);

}  // namespace plugins

namespace kernels {

// Owns the per-token validity flags, the image output cache [image, output_channels] and per-layer
// K/V caches [text + image, heads * head_dim] (fp32), like the reference class; every method
// launches on `stream` and throws RuntimeError on a CUDA error.
class SpatialCache {
public:
    SpatialCache(int image_seq_len, int text_seq_len, int output_channels, int num_attention_heads,
                 int attention_head_dim, int num_double_layers, int num_single_layers);
    ~SpatialCache();
    SpatialCache(const SpatialCache&) = delete;
    SpatialCache& operator=(const SpatialCache&) = delete;

    // All validity flags to false; cached values are kept.
    void reset(cudaStream_t stream = nullptr);
    // mask[i] = 2 wherever the cache row i is invalid.
    void preprocess_mask(int32_t* d_mask, cudaStream_t stream = nullptr);
    // Image rows: prediction = execute ? prediction : cache; on update cache = prediction, valid.
    void sync_output_cache(float* d_prediction, const int32_t* d_mask, cudaStream_t stream = nullptr);
    // K/V = execute ? fresh : cached; on update cached = fresh (layer block_id of the double or
    // single stack).
    void sync_kv_cache(float* d_keys, float* d_values, const int32_t* d_mask, int block_id,
                       bool is_double_block, cudaStream_t stream = nullptr);

    // Device buffers (additions for callers that drive the sparse path directly).
    uint8_t* valid() const { return d_valid_; }
    float* output_cache() const { return d_output_cache_; }
    float* keys(int block_id, bool is_double_block) const;
    float* values(int block_id, bool is_double_block) const;

private:
    int image_seq_len_, text_seq_len_, full_seq_len_, output_channels_, num_heads_, head_dim_;
    int num_double_layers_, num_single_layers_;
    uint8_t* d_valid_ = nullptr;
    float* d_output_cache_ = nullptr;
    std::vector<float*> d_double_keys_, d_double_values_, d_single_keys_, d_single_values_;
    void free_buffers() noexcept;
};

}  // namespace kernels
}  // namespace fluxrt
