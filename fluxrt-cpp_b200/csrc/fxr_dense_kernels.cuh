// fxr_dense_kernels.cuh — the reference's dense fp32 block helpers over whole sequences:
//   layer_norm_f32_kernel   LayerNorm without affine weights, then * gamma + beta
//                           (layer_norm_modulated, gather_scatter_kernels.cu:103-169)
//   modulate_f32_kernel     out = (1 + scale) * x + shift (apply_modulation, :74-99)
//   ew_f32_kernel           tanh GELU in place, bias add, x + y, x + gate * y
//                           (launch_gelu / launch_bias_add / launch_elem_add / launch_scale_add,
//                            flux2_kernels.cu:14-53,92-135)
// They back the C++ mirror of those declarations, so that a caller of the reference's kernel layer
// links against this library alone. They are off the sparse path (the block entry points of this
// library fuse the same math into their executed-row kernels) and are plain HBM-bound streams:
// 16-byte accesses where the pointers allow, grid-stride loops sized from the SM count.
#pragma once

#include "fxr_device.cuh"

namespace fxr {

// One warp per row; the row is read three times (sum, centred sum of squares, output), the later
// passes from L1/L2. Both reductions in fp32 over the warp, like the reference kernel's block
// reduction but without its uninitialised shared accumulators (gather_scatter_kernels.cu:127-147).
__global__ void __launch_bounds__(256)
layer_norm_f32_kernel(const float* x, float* y, const float* gamma,
                      const float* beta, float eps, int64_t rows, int32_t dim) {
    const int lane = threadIdx.x & 31;
    const float inv_dim = 1.0f / (float)dim;
    for (int64_t r = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5); r < rows; r += (int64_t)gridDim.x * 8) {
        const float* xr = x + r * dim;
        float* yr = y + r * dim;
        float s = 0.f;
        for (int32_t e = lane; e < dim; e += 32) s += xr[e];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        const float mean = s * inv_dim;
        float ss = 0.f;
        for (int32_t e = lane; e < dim; e += 32) {
            const float d = xr[e] - mean;
            ss = fmaf(d, d, ss);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float rs = rsqrtf(ss * inv_dim + eps);
        for (int32_t e = lane; e < dim; e += 32) {
            float v = (xr[e] - mean) * rs;
            if (gamma) v *= gamma[e];
            if (beta) v += beta[e];
            yr[e] = v;
        }
    }
}

__global__ void __launch_bounds__(256)
modulate_f32_kernel(const float* x, const float* scale,
                    const float* shift, float* out, int64_t rows, int32_t dim) {
    const int64_t total = rows * dim;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
         t += (int64_t)gridDim.x * blockDim.x) {
        const int32_t f = (int32_t)(t % dim);
        out[t] = (1.0f + scale[f]) * x[t] + shift[f];
    }
}

enum EwOp : int { kEwGelu = 0, kEwBias = 1, kEwAdd = 2, kEwScaleAdd = 3 };

struct EwArgs {
    const float* x;      // input (kEwGelu, kEwBias: also the output)
    const float* y;      // second input (kEwAdd, kEwScaleAdd) or the bias [dim]
    float* out;
    int64_t n;           // elements
    int32_t dim;         // bias period (kEwBias)
    float gate;          // kEwScaleAdd
};

template <int kOp>
__device__ __forceinline__ float ew_apply(float x, float y, float gate) {
    if constexpr (kOp == kEwGelu) {
        return x * (0.5f * (1.0f + tanhf(0.7978845608f * (x + 0.044715f * x * x * x))));
    } else if constexpr (kOp == kEwBias || kOp == kEwAdd) {
        return x + y;
    } else {
        return x + gate * y;
    }
}

// kVec: 4 elements per thread-iteration through float4 (every pointer 16-byte aligned and, for the
// bias, dim a multiple of 4), else one element.
template <int kOp, bool kVec>
__global__ void __launch_bounds__(256) ew_f32_kernel(const __grid_constant__ EwArgs a) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t t0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if constexpr (kVec) {
        const int64_t n4 = a.n / 4;
        const float4* x4 = reinterpret_cast<const float4*>(a.x);
        const float4* y4 = reinterpret_cast<const float4*>(a.y);
        float4* o4 = reinterpret_cast<float4*>(a.out);
        for (int64_t t = t0; t < n4; t += stride) {
            const float4 x = x4[t];
            float4 y = make_float4(0.f, 0.f, 0.f, 0.f);
            if constexpr (kOp == kEwBias) y = y4[(t * 4 % a.dim) / 4];
            else if constexpr (kOp != kEwGelu) y = y4[t];
            o4[t] = make_float4(ew_apply<kOp>(x.x, y.x, a.gate), ew_apply<kOp>(x.y, y.y, a.gate),
                                ew_apply<kOp>(x.z, y.z, a.gate), ew_apply<kOp>(x.w, y.w, a.gate));
        }
    } else {
        for (int64_t t = t0; t < a.n; t += stride) {
            float y = 0.f;
            if constexpr (kOp == kEwBias) y = a.y[t % a.dim];
            else if constexpr (kOp != kEwGelu) y = a.y[t];
            a.out[t] = ew_apply<kOp>(a.x[t], y, a.gate);
        }
    }
}

}  // namespace fxr
