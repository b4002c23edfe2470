// fxr_compat_kernels.cuh — fp32 kernels behind the reference-signature C++ shims
// (include/fxr_reference_api.h). Not on the tensor-core hot path: they exist so that callers of the
// reference's fp32 attention_fwd keep working, with the intended math.
#pragma once

#include "fxr_device.cuh"

namespace fxr {

// out = softmax(Q K^T * scale) V for layout (batch, heads, len, head_dim), fp32, head_dim <= 256.
// A CTA of 4 warps takes 4 consecutive queries of one (batch, head) and streams the keys in tiles
// of 32 through shared memory: lane j scores key j of the tile against the warp's query, the warp
// keeps an online softmax, and lane l accumulates output dims l, l+32, ...
constexpr int kF32AttnWarps = 4;
constexpr int kF32AttnMaxD = 256;

inline size_t f32_attention_smem(int D) {
    return sizeof(float) * (size_t)(32 * (D + 1) + 32 * D + kF32AttnWarps * D);
}

__global__ void __launch_bounds__(kF32AttnWarps * 32)
attention_f32_bhsd_kernel(const float* __restrict__ Q, const float* __restrict__ K,
                          const float* __restrict__ V, float* __restrict__ O, int32_t Sq,
                          int32_t Skv, int32_t D, float scale) {
    extern __shared__ float sm[];
    float* sK = sm;                      // [32][D+1] (padded: lanes read different banks)
    float* sV = sK + 32 * (D + 1);       // [32][D]
    float* sQ = sV + 32 * D;             // [4][D], pre-scaled
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t bh = blockIdx.y;
    const int32_t q0 = blockIdx.x * kF32AttnWarps;
    const float* Qb = Q + bh * Sq * D;
    const float* Kb = K + bh * Skv * D;
    const float* Vb = V + bh * Skv * D;
    for (int e = threadIdx.x; e < kF32AttnWarps * D; e += blockDim.x) {
        const int w = e / D, d = e % D;
        sQ[e] = (q0 + w < Sq) ? Qb[(int64_t)(q0 + w) * D + d] * scale : 0.f;
    }
    float m = -INFINITY, l = 0.f;
    float acc[kF32AttnMaxD / 32];
#pragma unroll
    for (int t = 0; t < kF32AttnMaxD / 32; ++t) acc[t] = 0.f;
    for (int32_t k0 = 0; k0 < Skv; k0 += 32) {
        __syncthreads();
        for (int e = threadIdx.x; e < 32 * D; e += blockDim.x) {
            const int j = e / D, d = e % D;
            const bool ok = k0 + j < Skv;
            sK[j * (D + 1) + d] = ok ? Kb[(int64_t)(k0 + j) * D + d] : 0.f;
            sV[e] = ok ? Vb[(int64_t)(k0 + j) * D + d] : 0.f;
        }
        __syncthreads();
        float s = 0.f;
        const float* qr = sQ + warp * D;
        const float* kr = sK + lane * (D + 1);
        for (int d = 0; d < D; ++d) s = fmaf(qr[d], kr[d], s);
        if (k0 + lane >= Skv) s = -INFINITY;
        float tmax = s;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, o));
        const float m_new = fmaxf(m, tmax);
        const float alpha = expf(m - m_new);
        const float p = expf(s - m_new);
        float psum = p;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) psum += __shfl_xor_sync(0xffffffffu, psum, o);
        l = l * alpha + psum;
        m = m_new;
#pragma unroll
        for (int t = 0; t < kF32AttnMaxD / 32; ++t) acc[t] *= alpha;
        for (int j = 0; j < 32; ++j) {
            const float pj = __shfl_sync(0xffffffffu, p, j);
#pragma unroll
            for (int t = 0; t < kF32AttnMaxD / 32; ++t) {
                const int d = lane + 32 * t;
                if (d < D) acc[t] = fmaf(pj, sV[j * D + d], acc[t]);
            }
        }
    }
    const int32_t qi = q0 + warp;
    if (qi < Sq) {
        const float inv = 1.0f / l;
#pragma unroll
        for (int t = 0; t < kF32AttnMaxD / 32; ++t) {
            const int d = lane + 32 * t;
            if (d < D) O[bh * Sq * D + (int64_t)qi * D + d] = acc[t] * inv;
        }
    }
}

}  // namespace fxr
