// fxr_reference_api.cpp — the reference's kernel-layer C++ interfaces (include/fxr_reference_api.h)
// implemented on the C ABI of this library.
//
// The free functions keep the reference contract: void, asynchronous on `stream`, no exception.
// A rejected argument or failed launch is recorded and readable through fxr_last_error_string()
// (the reference did not check launches at all). SpatialCache throws fluxrt::RuntimeError on a
// CUDA error, as the reference class does (spatial_kv_cache.cu:157,168,186).
#include "fxr_reference_api.h"

#include <cstdio>

#include "fxr.h"

namespace fluxrt {
namespace plugins {

void gather_tokens(const float* src, float* dst, const int32_t* indices, int32_t active_count,
                   int32_t dim, cudaStream_t stream) {
    if (active_count <= 0 || dim <= 0) return;
    const int64_t row = (int64_t)dim * (int64_t)sizeof(float);
    fxr_gather_rows(src, row, indices, nullptr, active_count, dst, row, row, 0, stream);
}

void scatter_tokens(const float* src, float* dst, const int32_t* indices, int32_t active_count,
                    int32_t dim, cudaStream_t stream) {
    if (active_count <= 0 || dim <= 0) return;
    const int64_t row = (int64_t)dim * (int64_t)sizeof(float);
    fxr_scatter_rows(src, row, indices, nullptr, active_count, dst, row, row, 0, stream);
}

void apply_modulation(const float* x, const float* scale, const float* shift, float* out,
                      int32_t seq_len, int32_t dim, cudaStream_t stream) {
    if (seq_len <= 0 || dim <= 0) return;
    fxr_modulate_f32(x, scale, shift, out, seq_len, dim, stream);
}

void layer_norm_modulated(const float* x, float* y, const float* gamma, const float* beta, float eps,
                          int32_t seq_len, int32_t dim, cudaStream_t stream) {
    if (seq_len <= 0 || dim <= 0) return;
    fxr_layer_norm_f32(x, y, gamma, beta, eps, seq_len, dim, stream);
}

void launch_gelu(float* data, int32_t n, cudaStream_t stream) {
    if (n <= 0) return;
    fxr_gelu_tanh_f32(data, n, stream);
}

void launch_bias_add(float* data, const float* bias, int32_t seq_len, int32_t dim, cudaStream_t stream) {
    if (!bias || seq_len <= 0 || dim <= 0) return;
    fxr_bias_add_f32(data, bias, seq_len, dim, stream);
}

void launch_rms_norm(const float* x, float* y, const float* weight, float eps, int32_t seq_len,
                     int32_t dim, cudaStream_t stream) {
    if (seq_len <= 0 || dim <= 0) return;
    fxr_rms_norm(x, y, weight, eps, seq_len, dim, FXR_F32, stream);
}

void launch_elem_add(const float* x, const float* y, float* z, int32_t n, cudaStream_t stream) {
    if (n <= 0) return;
    fxr_add_f32(x, y, z, n, stream);
}

void launch_scale_add(const float* x, const float* y, float* out, float gate, int32_t n,
                      cudaStream_t stream) {
    if (n <= 0) return;
    fxr_scale_add_f32(x, y, out, gate, n, stream);
}

void attention_fwd(const float* Q, const float* K, const float* V, float* out, int32_t batch,
                   int32_t num_heads, int32_t q_len, int32_t kv_len, int32_t head_dim,
                   cudaStream_t stream) {
    fxr_attention_f32_bhsd(Q, K, V, out, batch, num_heads, q_len, kv_len, head_dim, stream);
}

}  // namespace plugins

namespace kernels {

namespace {
void check(cudaError_t e, const char* what) {
    if (e != cudaSuccess) {
        char buf[512];
        std::snprintf(buf, sizeof(buf), "[CUDA] %s failed: %s (%d): %s", what, cudaGetErrorName(e),
                      (int)e, cudaGetErrorString(e));
        throw RuntimeError(buf);
    }
}
void check_fxr(int32_t st, const char* what) {
    if (st != FXR_OK) {
        char buf[512];
        std::snprintf(buf, sizeof(buf), "[fxr] %s failed (%d): %s", what, (int)st, fxr_last_error_string());
        throw RuntimeError(buf);
    }
}
float* alloc_zero(size_t bytes) {
    void* p = nullptr;
    check(cudaMalloc(&p, bytes), "cudaMalloc");
    check(cudaMemset(p, 0, bytes), "cudaMemset");
    return static_cast<float*>(p);
}
}  // namespace

SpatialCache::SpatialCache(int image_seq_len, int text_seq_len, int output_channels,
                           int num_attention_heads, int attention_head_dim, int num_double_layers,
                           int num_single_layers)
    : image_seq_len_(image_seq_len), text_seq_len_(text_seq_len),
      full_seq_len_(image_seq_len + text_seq_len), output_channels_(output_channels),
      num_heads_(num_attention_heads), head_dim_(attention_head_dim),
      num_double_layers_(num_double_layers), num_single_layers_(num_single_layers) {
    try {
        void* v = nullptr;
        check(cudaMalloc(&v, (size_t)full_seq_len_), "cudaMalloc(valid)");
        d_valid_ = static_cast<uint8_t*>(v);
        check(cudaMemset(d_valid_, 0, (size_t)full_seq_len_), "cudaMemset(valid)");
        d_output_cache_ = alloc_zero((size_t)image_seq_len_ * output_channels_ * sizeof(float));
        const size_t kv = (size_t)full_seq_len_ * num_heads_ * head_dim_ * sizeof(float);
        for (int i = 0; i < num_double_layers_; ++i) {
            d_double_keys_.push_back(alloc_zero(kv));
            d_double_values_.push_back(alloc_zero(kv));
        }
        for (int i = 0; i < num_single_layers_; ++i) {
            d_single_keys_.push_back(alloc_zero(kv));
            d_single_values_.push_back(alloc_zero(kv));
        }
    } catch (...) {
        free_buffers();
        throw;
    }
}

SpatialCache::~SpatialCache() { free_buffers(); }

void SpatialCache::free_buffers() noexcept {
    auto f = [](void* p) {
        if (p) cudaFree(p);
    };
    f(d_valid_);
    f(d_output_cache_);
    for (auto* p : d_double_keys_) f(p);
    for (auto* p : d_double_values_) f(p);
    for (auto* p : d_single_keys_) f(p);
    for (auto* p : d_single_values_) f(p);
    d_valid_ = nullptr;
    d_output_cache_ = nullptr;
    d_double_keys_.clear();
    d_double_values_.clear();
    d_single_keys_.clear();
    d_single_values_.clear();
}

void SpatialCache::reset(cudaStream_t stream) {
    check(cudaMemsetAsync(d_valid_, 0, (size_t)full_seq_len_, stream), "cudaMemsetAsync(valid)");
}

void SpatialCache::preprocess_mask(int32_t* d_mask, cudaStream_t stream) {
    check_fxr(fxr_preprocess_mask(d_mask, d_valid_, full_seq_len_, stream), "preprocess_mask");
}

void SpatialCache::sync_output_cache(float* d_prediction, const int32_t* d_mask, cudaStream_t stream) {
    check_fxr(fxr_output_cache_sync(d_prediction, d_output_cache_, d_mask, d_valid_, text_seq_len_,
                                    image_seq_len_, output_channels_, FXR_F32, stream),
              "sync_output_cache");
}

float* SpatialCache::keys(int block_id, bool is_double_block) const {
    const auto& v = is_double_block ? d_double_keys_ : d_single_keys_;
    if (block_id < 0 || block_id >= (int)v.size()) throw RuntimeError("SpatialCache: block_id out of range");
    return v[block_id];
}

float* SpatialCache::values(int block_id, bool is_double_block) const {
    const auto& v = is_double_block ? d_double_values_ : d_single_values_;
    if (block_id < 0 || block_id >= (int)v.size()) throw RuntimeError("SpatialCache: block_id out of range");
    return v[block_id];
}

void SpatialCache::sync_kv_cache(float* d_keys, float* d_values, const int32_t* d_mask, int block_id,
                                 bool is_double_block, cudaStream_t stream) {
    check_fxr(fxr_kv_sync(d_keys, d_values, keys(block_id, is_double_block),
                          values(block_id, is_double_block), d_mask, full_seq_len_,
                          (int64_t)num_heads_ * head_dim_, FXR_F32, stream),
              "sync_kv_cache");
}

}  // namespace kernels
}  // namespace fluxrt
