/*
 * fxr_oracle.c — CPU fp32 restatement of fluxrt-cpp's sparse stream-editing attention path.
 *
 * TEST INFRASTRUCTURE ONLY: the checker for the CUDA path and the timed CPU baseline.
 * Nothing in the product library links or calls this file. See fxr_oracle.h for the
 * reference citations and the pinning status of each function (RoPE: parity unpinned).
 *
 * Build: gcc -O3 -fopenmp -fPIC -shared (oracle/build_oracle.sh).
 */
#include "fxr_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

int fxo_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
    return omp_get_max_threads();
#else
    (void)n;
    return 1;
#endif
}

/* spatial_kv_cache.cu:12-19 (preprocess) + compaction of the executed tokens in ascending order. */
int32_t fxo_mask_compact(int32_t* mask, const uint8_t* valid, int32_t n_tokens, int32_t* idx) {
    int32_t m = 0;
    for (int32_t i = 0; i < n_tokens; ++i) {
        if (valid && !valid[i]) mask[i] = 2;
        if (mask[i] != 0) idx[m++] = i;
    }
    return m;
}

/* gather_scatter_kernels.cu:15-29: dst row m <- src row idx[m] (a plain copy of bytes). */
void fxo_gather_rows(const void* src, int64_t ld_src_bytes, const int32_t* idx, int32_t count,
                     void* dst, int64_t ld_dst_bytes, int64_t row_bytes) {
    const char* s = (const char*)src;
    char* d = (char*)dst;
    for (int32_t m = 0; m < count; ++m)
        memcpy(d + (int64_t)m * ld_dst_bytes, s + (int64_t)idx[m] * ld_src_bytes, (size_t)row_bytes);
}

/* gather_scatter_kernels.cu:46-60: dst row idx[m] <- src row m; rows not listed keep their bytes. */
void fxo_scatter_rows(const void* src, int64_t ld_src_bytes, const int32_t* idx, int32_t count,
                      void* dst, int64_t ld_dst_bytes, int64_t row_bytes) {
    const char* s = (const char*)src;
    char* d = (char*)dst;
    for (int32_t m = 0; m < count; ++m)
        memcpy(d + (int64_t)idx[m] * ld_dst_bytes, s + (int64_t)m * ld_src_bytes, (size_t)row_bytes);
}

/* flux2_kernels.cu:58-82 (formula y = x * rsqrt(mean(x^2) + eps) * w), sum of squares in double. */
static void rms_norm_row(const float* x, float* y, const float* w, float eps, int32_t dim) {
    double ss = 0.0;
    for (int32_t i = 0; i < dim; ++i) ss += (double)x[i] * (double)x[i];
    const float r = (float)(1.0 / sqrt(ss / (double)dim + (double)eps));
    for (int32_t i = 0; i < dim; ++i) y[i] = x[i] * r * w[i];
}

void fxo_rms_norm(const float* x, float* y, const float* w, float eps, int64_t rows, int32_t dim) {
    #pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r) rms_norm_row(x + r * dim, y + r * dim, w, eps, dim);
}

/* FLUX multi-axis rotary embedding (published formulation; no reference code exists). */
static void rope_tables(const int32_t* pos, int32_t n_axes, const int32_t* axes_dim, float theta,
                        int32_t head_dim, float* cs, float* sn) {
    int32_t j = 0;
    for (int32_t a = 0; a < n_axes; ++a) {
        const int32_t half = axes_dim[a] / 2;
        for (int32_t jj = 0; jj < half; ++jj, ++j) {
            const double omega = pow((double)theta, -2.0 * (double)jj / (double)axes_dim[a]);
            const double ang = (double)pos[a] * omega;
            cs[j] = (float)cos(ang);
            sn[j] = (float)sin(ang);
        }
    }
    for (; j < head_dim / 2; ++j) { cs[j] = 1.0f; sn[j] = 0.0f; }
}

static void rope_apply(float* x, int32_t head_dim, const float* cs, const float* sn) {
    for (int32_t j = 0; j < head_dim / 2; ++j) {
        const float a = x[2 * j], b = x[2 * j + 1];
        x[2 * j] = a * cs[j] - b * sn[j];
        x[2 * j + 1] = b * cs[j] + a * sn[j];
    }
}

void fxo_rope_row(float* x, int32_t head_dim, const int32_t* pos, int32_t n_axes,
                  const int32_t* axes_dim, float theta) {
    float cs[512], sn[512];
    rope_tables(pos, n_axes, axes_dim, theta, head_dim, cs, sn);
    rope_apply(x, head_dim, cs, sn);
}

/* RMSNorm + RoPE of the listed rows, every head: y[r] = rope(rms_norm(x[idx[r]])) per head
 * (flux2_kernels.cu:58-82 formula, then the published FLUX rotary embedding). The per-row step of
 * fxo_frame_forward on its own, so that a caller can round the results to a storage type. */
void fxo_norm_rope_rows(const float* x, int64_t ld_x, const int32_t* idx, int32_t count,
                        const int32_t* pos, int32_t n_axes, const int32_t* axes_dim, float theta,
                        const float* w, float eps, int32_t n_heads, int32_t head_dim,
                        float* y, int64_t ld_y) {
    #pragma omp parallel for schedule(static)
    for (int32_t r = 0; r < count; ++r) {
        const int32_t i = idx[r];
        float cs[512], sn[512];
        rope_tables(pos + (int64_t)i * n_axes, n_axes, axes_dim, theta, head_dim, cs, sn);
        for (int32_t h = 0; h < n_heads; ++h) {
            float* yo = y + (int64_t)r * ld_y + (int64_t)h * head_dim;
            rms_norm_row(x + (int64_t)i * ld_x + (int64_t)h * head_dim, yo, w, eps, head_dim);
            rope_apply(yo, head_dim, cs, sn);
        }
    }
}

/* attention_kernels.cu:85-155, intended semantics: softmax over every key of one head, scale
 * 1/sqrt(D), then the weighted sum of V. Work is split over (head, 64-query block). Dot products
 * accumulate in 16 independent fp32 lanes; the softmax denominator in double. */
#define FXO_QB 64
#define FXO_LANES 16

static float dot_lanes(const float* a, const float* b, int32_t n) {
    float acc[FXO_LANES];
    for (int l = 0; l < FXO_LANES; ++l) acc[l] = 0.0f;
    int32_t d = 0;
    for (; d + FXO_LANES <= n; d += FXO_LANES)
        for (int l = 0; l < FXO_LANES; ++l) acc[l] += a[d + l] * b[d + l];
    float s = 0.0f;
    for (; d < n; ++d) s += a[d] * b[d];
    for (int l = 0; l < FXO_LANES; ++l) s += acc[l];
    return s;
}

void fxo_attention(const float* q, int64_t ld_q, int32_t M,
                   const float* k, const float* v, int64_t ld_kv, int32_t N,
                   int32_t n_heads, int32_t head_dim, float scale,
                   float* o, int64_t ld_o) {
    if (M <= 0) return;
    if (!(scale > 0.0f)) scale = 1.0f / sqrtf((float)head_dim);
    const int32_t nqb = (M + FXO_QB - 1) / FXO_QB;
    const int64_t n_units = (int64_t)n_heads * nqb;
    #pragma omp parallel
    {
        float* s = (float*)malloc(sizeof(float) * (size_t)N);
        double* acc = (double*)malloc(sizeof(double) * (size_t)head_dim);
        #pragma omp for schedule(dynamic, 1)
        for (int64_t u = 0; u < n_units; ++u) {
            const int32_t h = (int32_t)(u / nqb), qb = (int32_t)(u % nqb);
            const int32_t m_end = (qb + 1) * FXO_QB < M ? (qb + 1) * FXO_QB : M;
            for (int32_t m = qb * FXO_QB; m < m_end; ++m) {
                const float* qr = q + (int64_t)m * ld_q + (int64_t)h * head_dim;
                float mx = -INFINITY;
                for (int32_t n = 0; n < N; ++n) {
                    s[n] = dot_lanes(qr, k + (int64_t)n * ld_kv + (int64_t)h * head_dim, head_dim) * scale;
                    if (s[n] > mx) mx = s[n];
                }
                double sum = 0.0;
                for (int32_t n = 0; n < N; ++n) {
                    s[n] = expf(s[n] - mx);
                    sum += (double)s[n];
                }
                for (int32_t d = 0; d < head_dim; ++d) acc[d] = 0.0;
                for (int32_t n = 0; n < N; ++n) {
                    const float p = s[n];
                    const float* vr = v + (int64_t)n * ld_kv + (int64_t)h * head_dim;
                    for (int32_t d = 0; d < head_dim; ++d) acc[d] += (double)(p * vr[d]);
                }
                float* orow = o + (int64_t)m * ld_o + (int64_t)h * head_dim;
                const double inv = 1.0 / sum;
                for (int32_t d = 0; d < head_dim; ++d) orow[d] = (float)(acc[d] * inv);
            }
        }
        free(s);
        free(acc);
    }
}

/* spatial_kv_cache.cu:55-87. */
void fxo_kv_sync(float* keys, float* values, float* cached_keys, float* cached_values,
                 const int32_t* mask, int32_t n_tokens, int64_t row_elems) {
    for (int32_t i = 0; i < n_tokens; ++i) {
        const int execute = mask[i] != 0, update = mask[i] == 2;
        float* kr = keys + (int64_t)i * row_elems;
        float* vr = values + (int64_t)i * row_elems;
        float* ck = cached_keys + (int64_t)i * row_elems;
        float* cv = cached_values + (int64_t)i * row_elems;
        for (int64_t e = 0; e < row_elems; ++e) {
            const float kv = kr[e], vv = vr[e], ckv = ck[e], cvv = cv[e];
            kr[e] = execute ? kv : ckv;
            vr[e] = execute ? vv : cvv;
            if (update) { ck[e] = kv; cv[e] = vv; }
        }
    }
}

/* spatial_kv_cache.cu:21-53. */
void fxo_output_cache_sync(float* pred, float* cache, const int32_t* mask, uint8_t* valid,
                           int32_t n_text, int32_t n_image, int32_t channels) {
    for (int32_t i = 0; i < n_image; ++i) {
        const int32_t mi = n_text + i;
        const int execute = mask[mi] != 0, update = mask[mi] == 2;
        float* pr = pred + (int64_t)i * channels;
        float* cr = cache + (int64_t)i * channels;
        for (int32_t c = 0; c < channels; ++c) {
            const float p = pr[c], cv = cr[c];
            pr[c] = execute ? p : cv;
            if (update) cr[c] = p;
        }
        if (update) valid[mi] = 1;
    }
}

int32_t fxo_frame_forward(const float* q, const float* k, const float* v,
                          int32_t* mask, const uint8_t* valid, const int32_t* pos,
                          const float* norm_q, const float* norm_k,
                          float* cache_k, float* cache_v, float* out, float* qc, int32_t* idx,
                          int32_t n_tokens, int32_t n_heads, int32_t head_dim,
                          int32_t n_axes, const int32_t* axes_dim, float theta, float eps,
                          float scale) {
    const int64_t C = (int64_t)n_heads * head_dim;
    const int32_t M = fxo_mask_compact(mask, valid, n_tokens, idx);
    if (M == 0) return 0;

    /* Attention K/V: cached rows for skipped tokens, fresh normed/roped rows for executed ones
     * (spatial_kv_cache.cu:64-67). */
    float* ak = (float*)malloc(sizeof(float) * (size_t)(n_tokens * C));
    float* av = (float*)malloc(sizeof(float) * (size_t)(n_tokens * C));
    memcpy(ak, cache_k, sizeof(float) * (size_t)(n_tokens * C));
    memcpy(av, cache_v, sizeof(float) * (size_t)(n_tokens * C));

    #pragma omp parallel for schedule(static)
    for (int32_t m = 0; m < M; ++m) {
        const int32_t i = idx[m];
        float cs[512], sn[512];
        rope_tables(pos + (int64_t)i * n_axes, n_axes, axes_dim, theta, head_dim, cs, sn);
        for (int32_t h = 0; h < n_heads; ++h) {
            const int64_t off = (int64_t)i * C + (int64_t)h * head_dim;
            float* qo = qc + (int64_t)m * C + (int64_t)h * head_dim;
            rms_norm_row(q + off, qo, norm_q, eps, head_dim);
            rope_apply(qo, head_dim, cs, sn);
            rms_norm_row(k + off, ak + off, norm_k, eps, head_dim);
            rope_apply(ak + off, head_dim, cs, sn);
            memcpy(av + off, v + off, sizeof(float) * (size_t)head_dim);
        }
    }

    float* oc = (float*)malloc(sizeof(float) * (size_t)((int64_t)M * C));
    fxo_attention(qc, C, M, ak, av, C, n_tokens, n_heads, head_dim, scale, oc, C);
    fxo_scatter_rows(oc, C * 4, idx, M, out, C * 4, C * 4);

    /* Cache update only where mask == 2 (spatial_kv_cache.cu:68-71). */
    for (int32_t m = 0; m < M; ++m) {
        const int32_t i = idx[m];
        if (mask[i] != 2) continue;
        memcpy(cache_k + (int64_t)i * C, ak + (int64_t)i * C, sizeof(float) * (size_t)C);
        memcpy(cache_v + (int64_t)i * C, av + (int64_t)i * C, sizeof(float) * (size_t)C);
    }
    free(oc);
    free(ak);
    free(av);
    return M;
}

/* gather_scatter_kernels.cu:106-169 (formula, without the uninitialised shared accumulators)
 * followed by apply_modulation (gather_scatter_kernels.cu:77-99). */
void fxo_layer_norm_modulate(const float* x, int64_t ld_x, float* y, const float* scale,
                             const float* shift, float eps, int64_t rows, int32_t dim) {
    #pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
        const float* xr = x + r * ld_x;
        float* yr = y + r * (int64_t)dim;
        double s = 0.0;
        for (int32_t i = 0; i < dim; ++i) s += (double)xr[i];
        const double mean = s / (double)dim;
        double ss = 0.0;
        for (int32_t i = 0; i < dim; ++i) {
            const double d = (double)xr[i] - mean;
            ss += d * d;
        }
        const double rstd = 1.0 / sqrt(ss / (double)dim + (double)eps);
        for (int32_t i = 0; i < dim; ++i) {
            double v = ((double)xr[i] - mean) * rstd;
            if (scale) v *= 1.0 + (double)scale[i];
            if (shift) v += (double)shift[i];
            yr[i] = (float)v;
        }
    }
}

/* flux2_kernels.cu:14-29. */
void fxo_gelu_tanh(float* x, int64_t n) {
    #pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
        const double v = (double)x[i];
        x[i] = (float)(0.5 * v * (1.0 + tanh(0.7978845608 * (v + 0.044715 * v * v * v))));
    }
}

/* flux2_double_block_plugin.cpp:28-45 (Y = X W^T) + bias_add (flux2_kernels.cu:34-53). */
void fxo_linear(const float* x, int64_t ld_x, int64_t rows, int32_t k, const float* w, const float* b,
                float* y, int32_t n) {
    #pragma omp parallel for schedule(dynamic, 4)
    for (int64_t r = 0; r < rows; ++r) {
        const float* xr = x + r * ld_x;
        float* yr = y + r * (int64_t)n;
        for (int32_t j = 0; j < n; ++j) {
            const float* wj = w + (int64_t)j * k;
            double a0 = 0.0, a1 = 0.0, a2 = 0.0, a3 = 0.0;
            int32_t i = 0;
            for (; i + 4 <= k; i += 4) {
                a0 += (double)xr[i] * (double)wj[i];
                a1 += (double)xr[i + 1] * (double)wj[i + 1];
                a2 += (double)xr[i + 2] * (double)wj[i + 2];
                a3 += (double)xr[i + 3] * (double)wj[i + 3];
            }
            for (; i < k; ++i) a0 += (double)xr[i] * (double)wj[i];
            yr[j] = (float)((a0 + a1) + (a2 + a3) + (b ? (double)b[j] : 0.0));
        }
    }
}

/* flux2_kernels.cu:116-135 with a per-channel gate (flux2_double_block_plugin.cpp:449-458). */
void fxo_gated_residual(const float* x, int64_t ld_x, const float* gate, const float* proj, float* out,
                        int64_t rows, int32_t dim) {
    #pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r)
        for (int32_t i = 0; i < dim; ++i) {
            const int64_t o = r * (int64_t)dim + i;
            out[o] = x[r * ld_x + i] + (gate ? gate[i] : 1.0f) * proj[o];
        }
}
