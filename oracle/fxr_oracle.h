/*
 * fxr_oracle.h — CPU fp32 restatement of fluxrt-cpp's sparse stream-editing attention path.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker for the CUDA path: only the tests,
 * the smoke check and the CPU-baseline leg of the benchmark load it. The product path never
 * calls it and has no CPU fallback.
 *
 * Every function states the reference code it restates (paths are inside the fluxrt-cpp
 * project). Where the reference kernel is defective (see the notes per function), the
 * oracle restates the intended math and says so.
 *
 * Pinning status:
 *   - mask protocol, compaction, gather, scatter, K/V merge/update, output-cache sync:
 *     pinned bit-exactly against the reference's known-answer tests
 *     (src/spike/test_gather_scatter.cpp:39-103, src/spike/test_spatial_cache.cu:32-87,
 *      src/spike/test_spatial_cache_trt.cpp:243-296) and, on a GPU, against the reference's
 *     own kernels compiled from source.
 *   - RMSNorm: pinned against an independent torch fp32 evaluation of the formula in
 *     src/inference/plugins/flux2_kernels.cu:58-82.
 *   - attention: pinned against torch.nn.functional.scaled_dot_product_attention (fp32, CPU).
 *   - LayerNorm: pinned against the known answer of src/spike/test_gather_scatter.cpp:106-133;
 *     modulation, tanh GELU and bias add: pinned on a GPU against the reference's own
 *     apply_modulation / gelu / bias_add kernels compiled from source; linear projection and
 *     gated residual: checked against numpy fp64 (the reference calls cublasSgemm there).
 *   - RoPE: parity unpinned. The reference has no RoPE code; the formula follows the
 *     published FLUX rotary embedding (interleaved pairs, per-axis frequencies
 *     theta^(-2j/d_a)) and is checked only through its algebraic properties.
 */
#ifndef FXR_ORACLE_H
#define FXR_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Number of OpenMP threads the oracle will use (0 = library default). Returns the count in use. */
int fxo_set_threads(int n);

/* Mask protocol + compaction.
 * preprocess (spatial_kv_cache.cu:12-19): mask[i] = 2 where valid[i] == 0 (valid may be NULL = all valid).
 * compaction (absent in the reference, whose indices are host-given, test_gather_scatter.cpp:47):
 *   idx = ascending list of i with mask[i] != 0; returns the count M. */
int32_t fxo_mask_compact(int32_t* mask, const uint8_t* valid, int32_t n_tokens, int32_t* idx);

/* Row gather (gather_scatter_kernels.cu:15-41): dst[m, :] = src[idx[m], :], rows of row_bytes bytes. */
void fxo_gather_rows(const void* src, int64_t ld_src_bytes, const int32_t* idx, int32_t count,
                     void* dst, int64_t ld_dst_bytes, int64_t row_bytes);

/* Row scatter (gather_scatter_kernels.cu:46-72): dst[idx[m], :] = src[m, :]; other rows untouched. */
void fxo_scatter_rows(const void* src, int64_t ld_src_bytes, const int32_t* idx, int32_t count,
                      void* dst, int64_t ld_dst_bytes, int64_t row_bytes);

/* Row RMSNorm (flux2_kernels.cu:58-82, intended semantics): y = x * rsqrt(mean(x^2) + eps) * w.
 * The reference kernel accumulates into an uninitialised shared scalar (flux2_kernels.cu:73-76);
 * this restates the formula. x, y: [rows, dim] fp32; w: [dim]. */
void fxo_rms_norm(const float* x, float* y, const float* w, float eps, int64_t rows, int32_t dim);

/* Multi-axis rotary embedding on one head row of D values, in place (fp32).
 * Pair j = (x[2j], x[2j+1]) belongs to axis a (axes laid out in order, axes_dim[a] values each);
 * angle = pos[a] * theta^(-2*jj/axes_dim[a]) with jj the pair index inside the axis, evaluated in
 * double precision and rounded to fp32 cos/sin;
 * out[2j] = x[2j]*cos - x[2j+1]*sin, out[2j+1] = x[2j+1]*cos + x[2j]*sin. */
void fxo_rope_row(float* x, int32_t head_dim, const int32_t* pos, int32_t n_axes,
                  const int32_t* axes_dim, float theta);

/* RMSNorm + RoPE of rows idx[0..count) of x, every head (the per-row step of fxo_frame_forward):
 * y[r, h*D:(h+1)*D] = rope(rms_norm(x[idx[r], h*D:(h+1)*D], w), pos[idx[r]]). fp32. */
void fxo_norm_rope_rows(const float* x, int64_t ld_x, const int32_t* idx, int32_t count,
                        const int32_t* pos, int32_t n_axes, const int32_t* axes_dim, float theta,
                        const float* w, float eps, int32_t n_heads, int32_t head_dim,
                        float* y, int64_t ld_y);

/* Joint non-causal attention of compact queries against all keys (attention_kernels.cu:85-155,
 * intended semantics: one softmax over every key, scale 1/sqrt(D) unless scale > 0).
 * q: [M, ld_q] (heads at column h*D), k, v: [N, ld_kv], o: [M, ld_o]; fp32. */
void fxo_attention(const float* q, int64_t ld_q, int32_t M,
                   const float* k, const float* v, int64_t ld_kv, int32_t N,
                   int32_t n_heads, int32_t head_dim, float scale,
                   float* o, int64_t ld_o);

/* K/V merge + update (spatial_kv_cache.cu:55-87), the reference's full-frame pass:
 * keys[i] = execute ? keys[i] : cached_keys[i]; if update: cached_keys[i] = fresh keys[i]
 * (same for values), with execute = mask != 0, update = mask == 2. fp32 rows of row_elems. */
void fxo_kv_sync(float* keys, float* values, float* cached_keys, float* cached_values,
                 const int32_t* mask, int32_t n_tokens, int64_t row_elems);

/* Output-cache merge + update (spatial_kv_cache.cu:21-53): over image tokens i in [0, n_image),
 * mask index T+i: pred = execute ? pred : cache; if update: cache = old pred, valid[T+i] = 1. */
void fxo_output_cache_sync(float* pred, float* cache, const int32_t* mask, uint8_t* valid,
                           int32_t n_text, int32_t n_image, int32_t channels);

/* Block-row math around the attention slice (the dense steps of one double- or single-stream
 * block, restated row by row so that a caller can apply them to the executed rows only).
 *
 * LayerNorm without affine weights + modulation (gather_scatter_kernels.cu:106-169 then
 * apply_modulation, gather_scatter_kernels.cu:77-99; called at flux2_double_block_plugin.cpp:373-383):
 *   y = (1 + scale) * (x - mean) * rsqrt(var + eps) + shift, biased variance over dim.
 * scale/shift may be NULL (plain LayerNorm, the reference's gamma = beta = NULL call). The reference
 * kernel accumulates into uninitialised shared scalars (gather_scatter_kernels.cu:127-147); this
 * restates the formula. Pinned against the known answer of test_gather_scatter.cpp:106-133.
 * x: [rows, ld_x], y: [rows, dim]; mean and variance in double. */
void fxo_layer_norm_modulate(const float* x, int64_t ld_x, float* y, const float* scale,
                             const float* shift, float eps, int64_t rows, int32_t dim);

/* tanh GELU in place (flux2_kernels.cu:14-29): x * 0.5 * (1 + tanh(0.7978845608 * (x + 0.044715 x^3))). */
void fxo_gelu_tanh(float* x, int64_t n);

/* Linear projection y = x W^T + b (the plugin's row-major cublasSgemm, flux2_double_block_plugin.cpp:28-45,
 * followed by bias_add, flux2_kernels.cu:34-53). x: [rows, k] (row stride ld_x), W: [n, k], b: [n] or
 * NULL, y: [rows, n]. Products accumulate in double and round once to fp32. */
void fxo_linear(const float* x, int64_t ld_x, int64_t rows, int32_t k, const float* w, const float* b,
                float* y, int32_t n);

/* Gated residual out = x + gate * proj (scale_add, flux2_kernels.cu:116-135, with the per-channel gate
 * of the modulation vector that flux2_double_block_plugin.cpp:449-458 leaves at 1.0). x: [rows, ld_x],
 * proj/out: [rows, dim]; gate: [dim] or NULL (= 1.0, the reference as written). */
void fxo_gated_residual(const float* x, int64_t ld_x, const float* gate, const float* proj, float* out,
                        int64_t rows, int32_t dim);

/* One frame of the sparse attention slice, fp32 end to end (storage rounding is the caller's).
 *   q, k, v      [N, C] fresh projections (C = H*D), fp32
 *   mask         [N] in/out (preprocessed in place with valid)
 *   pos          [N, n_axes] position ids
 *   norm_q/_k    [D] RMSNorm weights
 *   cache_k/_v   [N, C] in/out: attention-ready K' (normed + roped) and V per token
 *   out          [N, C] in/out: rows of executed tokens receive the attention output
 *   qc           [N, C] scratch/out: compact normed + roped queries (first M rows written)
 *   idx          [N] out: compaction indices
 * Steps: preprocess + compaction; per executed token and head, RMSNorm + RoPE of q and k;
 * attention K/V = execute ? fresh : cached (spatial_kv_cache.cu:64-67); joint attention of the
 * M executed queries over all N keys; scatter into out; cache rows := fresh where mask == 2.
 * Returns M. */
int32_t fxo_frame_forward(const float* q, const float* k, const float* v,
                          int32_t* mask, const uint8_t* valid, const int32_t* pos,
                          const float* norm_q, const float* norm_k,
                          float* cache_k, float* cache_v, float* out, float* qc, int32_t* idx,
                          int32_t n_tokens, int32_t n_heads, int32_t head_dim,
                          int32_t n_axes, const int32_t* axes_dim, float theta, float eps,
                          float scale);

#ifdef __cplusplus
}
#endif
#endif
