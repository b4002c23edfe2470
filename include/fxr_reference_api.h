// fxr_reference_api.h — the fluxrt-cpp kernel-layer interfaces of the sparse attention path,
// re-implemented on the sm_100a library so that existing C++ callers of those functions link
// unchanged. Names, argument order and meaning, fp32 data, asynchronous void-returning launches on
// the caller's stream and the throwing SpatialCache follow the reference declarations cited below;
// the implementations are this library's kernels (include/fxr.h).
//
// Replaced declarations (fluxrt-cpp paths):
//   fluxrt::plugins::gather_tokens / scatter_tokens   src/inference/plugins/gather_scatter_kernels.h:21-36
//   fluxrt::plugins::launch_rms_norm                  src/inference/plugins/flux2_kernels.h:22-24
//   fluxrt::plugins::attention_fwd                    src/inference/plugins/attention_kernels.h:20-24
//   fluxrt::kernels::SpatialCache                     src/inference/kernels/spatial_kv_cache.h:12-55
// Off-path declarations of those headers (AdaLN modulation, LayerNorm, GELU, bias/residual adds)
// are not part of this library.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <stdexcept>
#include <string>
#include <vector>

namespace fluxrt {

// Error type thrown by SpatialCache, as the reference's RuntimeError (src/utils/error.h:18-21).
class RuntimeError : public std::runtime_error {
public:
    explicit RuntimeError(const std::string& msg) : std::runtime_error(msg) {}
};

namespace plugins {

// dst[m, :] = src[indices[m], :] for m < active_count; fp32 rows of `dim` values.
void gather_tokens(const float* src, float* dst, const int32_t* indices, int32_t active_count,
                   int32_t dim, cudaStream_t stream);

// dst[indices[m], :] = src[m, :]; rows not listed keep their values.
void scatter_tokens(const float* src, float* dst, const int32_t* indices, int32_t active_count,
                    int32_t dim, cudaStream_t stream);

// y = x * rsqrt(mean(x^2) + eps) * weight over rows of `dim` values (seq_len rows).
void launch_rms_norm(const float* x, float* y, const float* weight, float eps, int32_t seq_len,
                     int32_t dim, cudaStream_t stream);

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
