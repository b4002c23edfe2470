// fxr_mem_kernels.cuh — HBM-bound kernels of the sparse attention path (sm_100a):
//   compact_kernel           mask preprocess + ascending index compaction (warp ballot + block scan)
//   gather_norm_rope_kernel  executed-row gather, per-head RMSNorm + multi-axis RoPE, cache-row write
//   restore_rows_kernel      puts back the cache rows of mask==1 tokens after the attention
//   rows_copy_kernel         byte-exact indexed row gather / scatter
//   kv_sync_kernel           reference full-frame K/V merge + update
//   out_cache_sync_kernel    reference output-cache merge + valid update
//   rms_norm_kernel          standalone row RMSNorm
// Rows move as 16-byte vectors; grids are multiples of the SM count and loop over rows, reading the
// executed-row count M from device memory (no host synchronisation between the steps).
#pragma once

#include "fxr_device.cuh"

namespace fxr {

// ---------------------------------------------------------------------------------------------
// Compaction. One CTA of 8 warps walks the mask in chunks of up to 8 x 32 groups of 32 tokens;
// each warp owns a contiguous run of groups (18 groups per warp for 4608 tokens), takes one ballot
// per group, and a scan of the 8 warp totals gives every warp its output offset. Output order is
// ascending token index. Restates preprocess_mask_kernel (spatial_kv_cache.cu:12-19) and adds the
// compaction the reference leaves to the host.
// ---------------------------------------------------------------------------------------------
constexpr int kCompactThreads = 256;
constexpr int kCompactWarps = kCompactThreads / 32;
constexpr int kCompactGroups = 32;                              // per warp and chunk, at most
constexpr int kCompactChunk = kCompactWarps * kCompactGroups * 32;

__global__ void __launch_bounds__(kCompactThreads, 1)
compact_kernel(int32_t* __restrict__ mask, const uint8_t* __restrict__ valid, int32_t n,
               int32_t* __restrict__ idx, int32_t* __restrict__ count) {
    __shared__ int32_t warp_tot[kCompactWarps];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t lt = (1u << lane) - 1u;
    pdl_launch_dependents();
    pdl_wait();  // the previous frame's kernels may still read mask / idx / count
    int32_t base = 0;
    for (int32_t c0 = 0; c0 < n; c0 += kCompactChunk) {
        const int32_t n_chunk = min(n - c0, kCompactChunk);
        const int32_t groups = (n_chunk + 31) >> 5;
        const int32_t gpw = (groups + kCompactWarps - 1) / kCompactWarps;   // groups per warp
        const int32_t e0 = c0 + warp * gpw * 32 + lane;
        uint32_t ballot[kCompactGroups];
        int32_t mval[kCompactGroups];
#pragma unroll
        for (int g = 0; g < kCompactGroups; ++g) {
            const int32_t e = e0 + g * 32;
            mval[g] = (g < gpw && e < c0 + n_chunk) ? mask[e] : 0;
        }
        int32_t tot = 0;
#pragma unroll
        for (int g = 0; g < kCompactGroups; ++g) {
            const int32_t e = e0 + g * 32;
            if (valid != nullptr && g < gpw && e < c0 + n_chunk && valid[e] == 0) {
                if (mval[g] != 2) mask[e] = 2;
                mval[g] = 2;
            }
            ballot[g] = __ballot_sync(0xffffffffu, mval[g] != 0);
            tot += __popc(ballot[g]);
        }
        if (lane == 0) warp_tot[warp] = tot;
        __syncthreads();
        int32_t off = base, chunk_tot = 0;
#pragma unroll
        for (int w = 0; w < kCompactWarps; ++w) {
            const int32_t t = warp_tot[w];
            off += (w < warp) ? t : 0;
            chunk_tot += t;
        }
#pragma unroll
        for (int g = 0; g < kCompactGroups; ++g) {
            if ((ballot[g] >> lane) & 1u) idx[off + __popc(ballot[g] & lt)] = e0 + g * 32;
            off += __popc(ballot[g]);
        }
        base += chunk_tot;
        __syncthreads();
    }
    if (threadIdx.x == 0) *count = base;
}

__global__ void preprocess_mask_kernel(int32_t* __restrict__ mask, const uint8_t* __restrict__ valid,
                                       int32_t n) {
    const int32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n && valid[i] == 0) mask[i] = 2;
}

// valid[i] = 1 for image tokens (i >= n_text) whose cache row was updated (mask 2): the validity
// update of sync_output_cache_kernel (spatial_kv_cache.cu:49-51); text tokens stay invalid, so the
// preprocess executes them every frame.
__global__ void mark_updated_kernel(const int32_t* __restrict__ mask, uint8_t* __restrict__ valid,
                                    int32_t n_text, int32_t n) {
    const int32_t i = n_text + blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n && mask[i] == 2) valid[i] = 1;
}

// ---------------------------------------------------------------------------------------------
// Fused gather + QK-RMSNorm + RoPE + cache-row write.
// One warp per executed token; the two half-warps take two heads at a time; lane `sub` of a half
// owns elements [8*sub, 8*sub+8) of a 128-wide head row (one 16-byte vector), so each rotary pair
// is lane-local and the RMS reduction is a 4-step half-warp shuffle. cos/sin of a token's 4 pairs
// per lane are computed once and reused for every head of Q and K.
// ---------------------------------------------------------------------------------------------
constexpr int kHeadDim = 128;
constexpr int kPairs = kHeadDim / 2;

struct RopeTable {
    float omega[kPairs];     // theta^(-2*jj/d_a) for pair j (rounded from double on the host)
    int8_t axis[kPairs];     // axis of pair j, -1 for none (identity)
};

struct GatherArgs {
    const void* q;
    const void* k;
    const void* v;
    const int32_t* mask;
    const int32_t* idx;
    const int32_t* count;
    const int32_t* pos;
    const float* norm_q;
    const float* norm_k;
    void* qc;
    void* cache_k;
    void* cache_v;
    void* save;
    int64_t ld_qkv, ld_qc, ld_cache;
    int32_t n_tokens, n_heads, n_axes;
    float eps;
    RopeTable rope;
};

constexpr int kGatherThreads = 256;

// sin/cos of a rotary angle (|angle| up to a few thousand radians): Cody-Waite reduction by 2*pi
// with the constant split into an exactly representable head (6.28125) and a tail, then the
// hardware sine/cosine on [-pi, pi] (absolute error ~4e-7 there).
__device__ __forceinline__ void rope_sincos(float ang, float* s, float* c) {
    const float k = rintf(ang * 0.15915494309189535f);
    float r = fmaf(-k, 6.28125f, ang);
    r = fmaf(-k, 1.9353071795864769e-3f, r);
    __sincosf(r, s, c);
}

template <typename T>
__device__ __forceinline__ void norm_rope_store(const uint4& x, const float* w, float eps,
                                                const float* cs, const float* sn, T* dst,
                                                bool active) {
    const uint32_t u[4] = {x.x, x.y, x.z, x.w};
    float f[8];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
        const float2 p = StoreT<T>::unpack2(u[t]);
        f[2 * t] = p.x;
        f[2 * t + 1] = p.y;
    }
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) ss = fmaf(f[e], f[e], ss);
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float r = rsqrtf(ss * (1.0f / kHeadDim) + eps);
    uint32_t outw[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
        const float a = f[2 * t] * r * w[2 * t];
        const float b = f[2 * t + 1] * r * w[2 * t + 1];
        outw[t] = StoreT<T>::pack2(a * cs[t] - b * sn[t], b * cs[t] + a * sn[t]);
    }
    if (active) *reinterpret_cast<uint4*>(dst) = make_uint4(outw[0], outw[1], outw[2], outw[3]);
}

// Work item = (executed row m, group of up to 8 heads); one warp per item. All 12 of a lane's
// 16-byte loads (Q, K, V of 4 head pairs) are issued before any arithmetic so that every warp keeps
// 6 KB in flight; 2 CTAs of 8 warps per SM (measured faster than 4-head items at 3 CTAs per SM).
constexpr int kGatherHeadsPerItem = 8;
constexpr int kGatherMinBlocks = 2;

template <typename T>
__global__ void __launch_bounds__(kGatherThreads, kGatherMinBlocks)
gather_norm_rope_kernel(const __grid_constant__ GatherArgs a) {
    const int lane = threadIdx.x & 31, half = lane >> 4, sub = lane & 15;
    const int warps_per_cta = kGatherThreads / 32;
    pdl_launch_dependents();
    pdl_wait();  // count / idx come from the compaction
    const int32_t M = *a.count;
    const int64_t C = (int64_t)a.n_heads * kHeadDim;
    const int groups = (a.n_heads + kGatherHeadsPerItem - 1) / kGatherHeadsPerItem;
    const int64_t items = (int64_t)M * groups;
    const T* __restrict__ Q = static_cast<const T*>(a.q);
    const T* __restrict__ K = static_cast<const T*>(a.k);
    const T* __restrict__ V = static_cast<const T*>(a.v);
    T* __restrict__ QC = static_cast<T*>(a.qc);
    T* __restrict__ CK = static_cast<T*>(a.cache_k);
    T* __restrict__ CV = static_cast<T*>(a.cache_v);
    T* __restrict__ SV = static_cast<T*>(a.save);

    for (int64_t it = (int64_t)blockIdx.x * warps_per_cta + (threadIdx.x >> 5); it < items;
         it += (int64_t)gridDim.x * warps_per_cta) {
        const int32_t m = (int32_t)(it / groups);
        const int h0 = (int)(it - (int64_t)m * groups) * kGatherHeadsPerItem;
        const int32_t i = __ldg(a.idx + m);
        if (i < 0 || i >= a.n_tokens) {
            if (lane == 0) atomicOr(&g_error_word, kErrBounds);
            continue;
        }
        const T* qrow = Q + (int64_t)i * a.ld_qkv + 8 * sub;
        const T* krow = K + (int64_t)i * a.ld_qkv + 8 * sub;
        const T* vrow = V + (int64_t)i * a.ld_qkv + 8 * sub;
        constexpr int kU = kGatherHeadsPerItem / 2;  // head pairs per item
        uint4 qv[kU], kv[kU], vv[kU];
        bool act[kU];
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            const int h = h0 + 2 * u + half;
            act[u] = h < a.n_heads;
            if (act[u]) {
                qv[u] = __ldg(reinterpret_cast<const uint4*>(qrow + h * kHeadDim));
                kv[u] = __ldg(reinterpret_cast<const uint4*>(krow + h * kHeadDim));
                vv[u] = __ldg(reinterpret_cast<const uint4*>(vrow + h * kHeadDim));
            } else {
                qv[u] = kv[u] = vv[u] = make_uint4(0, 0, 0, 0);
            }
        }
        const int32_t mode = __ldg(a.mask + i);
        float cs[4], sn[4];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const int j = 4 * sub + t;
            const int ax = a.rope.axis[j];
            if (ax < 0) {
                cs[t] = 1.f;
                sn[t] = 0.f;
            } else {
                const float ang = (float)__ldg(a.pos + (int64_t)i * a.n_axes + ax) * a.rope.omega[j];
                rope_sincos(ang, &sn[t], &cs[t]);
            }
        }
        T* qcrow = QC + (int64_t)m * a.ld_qc + 8 * sub;
        T* ckrow = CK + (int64_t)i * a.ld_cache + 8 * sub;
        T* cvrow = CV + (int64_t)i * a.ld_cache + 8 * sub;
        if (mode == 1 && SV != nullptr) {
            T* srow = SV + (int64_t)m * 2 * C + 8 * sub;
#pragma unroll
            for (int u = 0; u < kU; ++u) {
                const int h = h0 + 2 * u + half;
                if (act[u]) {
                    *reinterpret_cast<uint4*>(srow + h * kHeadDim) =
                        *reinterpret_cast<const uint4*>(ckrow + h * kHeadDim);
                    *reinterpret_cast<uint4*>(srow + C + h * kHeadDim) =
                        *reinterpret_cast<const uint4*>(cvrow + h * kHeadDim);
                }
            }
        }
        float w[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) w[e] = __ldg(a.norm_q + 8 * sub + e);
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            // every lane joins the shuffles; inactive heads compute on zeros and skip the store
            const int h = h0 + 2 * u + half;
            norm_rope_store<T>(qv[u], w, a.eps, cs, sn, qcrow + h * kHeadDim, act[u]);
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) w[e] = __ldg(a.norm_k + 8 * sub + e);
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            const int h = h0 + 2 * u + half;
            norm_rope_store<T>(kv[u], w, a.eps, cs, sn, ckrow + h * kHeadDim, act[u]);
            if (act[u]) *reinterpret_cast<uint4*>(cvrow + h * kHeadDim) = vv[u];
        }
    }
}

// ---------------------------------------------------------------------------------------------
// Restore of mask==1 cache rows (execute without cache update) from the save buffer.
// ---------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256)
restore_rows_kernel(const int32_t* __restrict__ mask, const int32_t* __restrict__ idx,
                    const int32_t* __restrict__ count, const uint4* __restrict__ save,
                    char* __restrict__ cache_k, char* __restrict__ cache_v, int64_t ld_cache_bytes,
                    int32_t row_vec, int32_t n_tokens) {
    const int lane = threadIdx.x & 31;
    pdl_launch_dependents();
    pdl_wait();  // the attention must have finished reading the cache rows
    const int32_t M = *count;
    for (int32_t m = blockIdx.x * 8 + (threadIdx.x >> 5); m < M; m += gridDim.x * 8) {
        const int32_t i = idx[m];
        if (i < 0 || i >= n_tokens) continue;
        if (mask[i] != 1) continue;
        const uint4* s = save + (int64_t)m * 2 * row_vec;
        uint4* dk = reinterpret_cast<uint4*>(cache_k + (int64_t)i * ld_cache_bytes);
        uint4* dv = reinterpret_cast<uint4*>(cache_v + (int64_t)i * ld_cache_bytes);
        for (int32_t e = lane; e < row_vec; e += 32) {
            dk[e] = s[e];
            dv[e] = s[row_vec + e];
        }
    }
}

// ---------------------------------------------------------------------------------------------
// Arrival wait of a head-sharded frame. slots[0..8): arrivals from each source GPU (one per
// attention CTA of that GPU per frame); slots[8]: frames this GPU has waited for, kept on the
// device so that a CUDA graph of the frame can be replayed. Thread s waits (bounded) until slot s
// reaches (frames + 1) * ctas[s]; the acquire at system scope makes the O rows that GPU s stored
// here before its increments visible to the kernels after this one.
// ---------------------------------------------------------------------------------------------
struct ArrivalCounts {
    uint32_t ctas[8];
};

__global__ void __launch_bounds__(32)
arrival_wait_kernel(uint32_t* __restrict__ slots, ArrivalCounts c, int32_t n) {
    const int s = threadIdx.x;
    uint32_t per_frame = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k)
        if (k == s) per_frame = c.ctas[k];
    const uint32_t frame = *reinterpret_cast<volatile uint32_t*>(slots + 8) + 1u;
    __syncwarp();
    if (s < n) {
        const uint32_t target = frame * per_frame;
        const uint64_t t0 = global_timer_ns();
        while ((int32_t)(ld_acquire_sys(slots + s) - target) < 0) {
            if (global_timer_ns() - t0 > kWaitLimitNs) {
                atomicOr(&g_error_word, kErrTimeout);
                break;
            }
            __nanosleep(256);
        }
    }
    __syncwarp();
    if (s == 0) slots[8] = frame;
}

// ---------------------------------------------------------------------------------------------
// Byte-exact indexed row copy: gather (dst[m] = src[idx[m]]) or scatter (dst[idx[m]] = src[m]).
// ---------------------------------------------------------------------------------------------
template <typename V, bool kScatter>
__global__ void __launch_bounds__(256)
rows_copy_kernel(const char* __restrict__ src, int64_t ld_src, const int32_t* __restrict__ idx,
                 const int32_t* __restrict__ count, int32_t host_count, char* __restrict__ dst,
                 int64_t ld_dst, int64_t row_vec) {
    const int lane = threadIdx.x & 31;
    const int32_t M = count ? *count : host_count;
    for (int32_t m = blockIdx.x * 8 + (threadIdx.x >> 5); m < M; m += gridDim.x * 8) {
        const int32_t i = idx[m];
        const V* s = reinterpret_cast<const V*>(src + (kScatter ? (int64_t)m * ld_src : (int64_t)i * ld_src));
        V* d = reinterpret_cast<V*>(dst + (kScatter ? (int64_t)i * ld_dst : (int64_t)m * ld_dst));
        for (int64_t e = lane; e < row_vec; e += 32) d[e] = s[e];
    }
}

// ---------------------------------------------------------------------------------------------
// Reference K/V merge + update over every row (spatial_kv_cache.cu:55-87), element type E with
// W-byte words: each thread handles one word.
// ---------------------------------------------------------------------------------------------
template <typename W>
__global__ void __launch_bounds__(256)
kv_sync_kernel(W* __restrict__ keys, W* __restrict__ values, W* __restrict__ ck,
               W* __restrict__ cv, const int32_t* __restrict__ mask, int32_t n_tokens,
               int64_t row_words) {
    const int64_t total = (int64_t)n_tokens * row_words;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
         t += (int64_t)gridDim.x * blockDim.x) {
        const int32_t i = (int32_t)(t / row_words);
        const int32_t mv = mask[i];
        const W kv = keys[t], vv = values[t], ckv = ck[t], cvv = cv[t];
        if (mv == 0) {
            keys[t] = ckv;
            values[t] = cvv;
        }
        if (mv == 2) {
            ck[t] = kv;
            cv[t] = vv;
        }
    }
}

// Output-cache merge + valid update (spatial_kv_cache.cu:21-53).
template <typename W>
__global__ void __launch_bounds__(256)
out_cache_sync_kernel(W* __restrict__ pred, W* __restrict__ cache, const int32_t* __restrict__ mask,
                      uint8_t* __restrict__ valid, int32_t n_text, int32_t n_image,
                      int64_t row_words) {
    const int64_t total = (int64_t)n_image * row_words;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
         t += (int64_t)gridDim.x * blockDim.x) {
        const int32_t i = (int32_t)(t / row_words);
        const int32_t mv = mask[n_text + i];
        const W p = pred[t], c = cache[t];
        if (mv == 0) pred[t] = c;
        if (mv == 2) {
            cache[t] = p;
            if (t - (int64_t)i * row_words == 0) valid[n_text + i] = 1;
        }
    }
}

// ---------------------------------------------------------------------------------------------
// Standalone row RMSNorm, one warp per row (flux2_kernels.cu:58-90 semantics).
// ---------------------------------------------------------------------------------------------
template <typename T> __device__ __forceinline__ float load_f(const T* p);
template <> __device__ __forceinline__ float load_f<float>(const float* p) { return *p; }
template <> __device__ __forceinline__ float load_f<__half>(const __half* p) { return __half2float(*p); }
template <> __device__ __forceinline__ float load_f<__nv_bfloat16>(const __nv_bfloat16* p) {
    return __bfloat162float(*p);
}
template <typename T> __device__ __forceinline__ void store_f(T* p, float v);
template <> __device__ __forceinline__ void store_f<float>(float* p, float v) { *p = v; }
template <> __device__ __forceinline__ void store_f<__half>(__half* p, float v) { *p = __float2half_rn(v); }
template <> __device__ __forceinline__ void store_f<__nv_bfloat16>(__nv_bfloat16* p, float v) {
    *p = __float2bfloat16_rn(v);
}

template <typename T>
__global__ void __launch_bounds__(256)
rms_norm_kernel(const T* __restrict__ x, T* __restrict__ y, const float* __restrict__ w, float eps,
                int64_t rows, int32_t dim) {
    const int lane = threadIdx.x & 31;
    for (int64_t r = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5); r < rows;
         r += (int64_t)gridDim.x * 8) {
        const T* xr = x + r * dim;
        T* yr = y + r * dim;
        float ss = 0.f;
        for (int32_t e = lane; e < dim; e += 32) {
            const float v = load_f(xr + e);
            ss = fmaf(v, v, ss);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float rs = rsqrtf(ss / (float)dim + eps);
        for (int32_t e = lane; e < dim; e += 32) store_f(yr + e, load_f(xr + e) * rs * w[e]);
    }
}

}  // namespace fxr
