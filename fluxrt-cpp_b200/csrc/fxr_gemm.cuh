// fxr_gemm.cuh — QKV projection of the executed tokens only (sm_100a, tcgen05 + TMEM).
//
// The reference projects every token's hidden state with six fp32 cublasSgemm calls
// (fluxrt-cpp src/inference/plugins/flux2_double_block_plugin.cpp:392-398) before any sparsity is
// applied. Here the projection runs on the executed rows only:
//   Y[idx[m], :] = X[idx[m], :] . W^T (+ bias)   for m < *count,  Y = [Q | K | V] split by columns
// A persistent CTA per SM walks 256 x 256 output tiles (m fastest, so the CTAs working at one time
// share a 256-column slice of W through L2):
//   * 8 warps gather the tile's 256 rows of X with cp.async (16 bytes per copy, each warp
//     instruction reading four whole 128-byte row segments, written in the 128-byte swizzle the
//     tensor core reads; rows past the count are zero-filled) — the row gather is the A load;
//   * 1 warp streams W's 256 x 64 slices with TMA (128-byte swizzle);
//   * 1 warp issues tcgen05.mma (M 128, N 256, K 16; bf16/fp16 in, fp32 in tensor memory) for both
//     128-row halves of the tile, which share each W slice, into two 256-column accumulators;
//   * 8 warps drain them: tensor memory -> registers, + bias, -> bf16/fp16, and store each row's
//     256 outputs (512 contiguous bytes) to its token row.
// Every wait is bounded (2 s); after a timeout the kernel sets the device error word and returns.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "fxr_device.cuh"

namespace fxr {
namespace gemm {

// A tile is 256 rows (two 128-row MMA halves sharing each W slice, which halves the W traffic per
// FLOP against 128-row tiles) x 256 columns; the two halves' accumulators fill tensor memory.
constexpr int kBM = 256, kHalf = 128, kBN = 256, kBK = 64;
constexpr int kStages = 3;
constexpr uint32_t kABytes = kBM * kBK * 2;          // 32 KB
constexpr uint32_t kBBytes = kBN * kBK * 2;          // 32 KB
constexpr uint32_t kStageBytes = kABytes + kBBytes;
constexpr int kAWarps = 8, kBWarp = 8, kMmaWarp = 9, kEpiWarp0 = 10, kEpiWarps = 8;
constexpr int kThreads = (kEpiWarp0 + kEpiWarps) * 32;   // 576
constexpr uint32_t kTmemCols = 2 * kBN;                  // the two halves' accumulators
constexpr uint32_t kSmemBar = kStages * kStageBytes;
enum : uint32_t { kFull = 0, kEmpty = kStages, kAccFull = 2 * kStages, kAccEmpty = 2 * kStages + 1,
                  kDrain = 2 * kStages + 2, kNumBars = 2 * kStages + 3 };
constexpr uint32_t kSlotTmem = kNumBars * 8, kSlotAbort = kSlotTmem + 4;
constexpr uint32_t kSmemBytes = kSmemBar + 256 + 1024;     // + alignment slack

struct Args {
    const void* x;            // [n_tokens, ld_x] hidden states
    const int32_t* idx;       // executed rows
    const int32_t* count;
    const float* bias;        // [n_out] or null
    void* y[3];               // Q, K, V [n_tokens, ld_y]; output column c goes to y[c / c_part]
    int64_t ld_x, ld_y;
    int32_t k_dim, n_out, c_part, n_tokens;
};

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
// all but the newest N committed groups of this thread have landed
template <int N>
__device__ __forceinline__ void cp_async_wait_group() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
// the rows this thread wrote (generic proxy) become visible to the tensor core (async proxy)
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
qkv_gather_gemm_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ Args a) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t* gbase = smem_raw + (base - raw);
    const uint32_t bar0 = base + kSmemBar;
    auto bar = [&](uint32_t i) { return bar0 + 8u * i; };
    volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(gbase + kSmemBar + kSlotTmem);
    volatile int* abort = reinterpret_cast<volatile int*>(gbase + kSmemBar + kSlotAbort);
    const int warp = threadIdx.x >> 5;
    const uint32_t lane = lane_id();

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(bar(kFull + s), kAWarps * 32 + 1);   // 256 gather threads + the W load
            mbar_init(bar(kEmpty + s), 1);
        }
        mbar_init(bar(kAccFull), 1);
        mbar_init(bar(kAccEmpty), kEpiWarps * 32);
        mbar_init(bar(kDrain), 1);
        *abort = 0;
        fence_mbar_init();
    }
    if (warp == kBWarp && lane == 0) prefetch_tmap(&tmW);
    if (warp == kMmaWarp) {
        tmem_alloc(smem_u32((const void*)tmem_slot), kTmemCols);
        tmem_relinquish();
    }
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    pdl_launch_dependents();
    pdl_wait();   // idx / count come from the compaction
    const int32_t M = *a.count;
    const int32_t n_mt = (M + kBM - 1) / kBM, n_nt = a.n_out / kBN;
    const int32_t n_tiles = n_mt * n_nt, n_kb = a.k_dim / kBK;

    if (warp < kAWarps) {
        // ---------------- row gather of X (A operand) ----------------
        // Stage `it` is signalled once its copies have landed and this thread has fenced them for
        // the tensor core, right after the copies of stage it + 1 are issued. Issuing a stage first
        // waits for the tensor core to free its buffer, so signalling any later than one stage
        // behind would leave the tensor core idle while this thread waits on that buffer.
        // Lane l of warp w moves 16-byte chunk (l % 8) of rows w*32 + 4j + l/8, j = 0..7: each copy
        // instruction of a warp reads four whole 128-byte row segments.
        constexpr int kLag = 1;
        const int c = (int)(lane & 7), sub = (int)(lane >> 3);
        uint32_t it = 0, signalled = 0;
        bool ok = true;
        auto signal_landed = [&](uint32_t upto) {          // stages [signalled, upto) have landed
            fence_proxy_async_smem();
            for (; signalled < upto; ++signalled) mbar_arrive(bar(kFull + signalled % kStages));
        };
        for (int32_t u = blockIdx.x; ok && u < n_tiles; u += gridDim.x) {
            const char* src[8];
            uint32_t nbytes[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int32_t m = (u % n_mt) * kBM + warp * 32 + 4 * j + sub;
                int32_t i = m < M ? __ldg(a.idx + m) : -1;
                if (i >= a.n_tokens) {
                    atomicOr(&g_error_word, kErrBounds);
                    i = -1;
                }
                src[j] = static_cast<const char*>(a.x) + (int64_t)(i < 0 ? 0 : i) * a.ld_x * (int64_t)sizeof(T) + c * 16;
                nbytes[j] = i < 0 ? 0u : 16u;               // rows past the count: zeros
            }
            for (int32_t kb = 0; kb < n_kb; ++kb, ++it) {
                const uint32_t st = it % kStages, use = it / kStages;
                if (use > 0 && !mbar_wait(bar(kEmpty + st), (use - 1) & 1, abort)) { ok = false; break; }
                const uint32_t stage = base + st * kStageBytes;
                const int64_t koff = (int64_t)kb * kBK * (int64_t)sizeof(T);
#pragma unroll
                for (int j = 0; j < 8; ++j) {   // 128-byte swizzle: chunk c of row r at (c ^ r % 8)
                    const int r = warp * 32 + 4 * j + sub;
                    cp_async16(stage + (uint32_t)(r * 128 + ((c ^ (r & 7)) * 16)), src[j] + koff, nbytes[j]);
                }
                cp_async_commit();
                if (it + 1 > (uint32_t)kLag) {
                    cp_async_wait_group<kLag>();
                    signal_landed(it + 1 - kLag);
                }
            }
        }
        cp_async_wait_all();   // nothing lands in shared memory after the CTA exits
        if (ok) signal_landed(it);
    } else if (warp == kBWarp) {
        if (lane == 0) {
            // ---------------- W slices (B operand) ----------------
            uint32_t it = 0;
            bool ok = true;
            for (int32_t u = blockIdx.x; ok && u < n_tiles; u += gridDim.x) {
                const int32_t n0 = (u / n_mt) * kBN;
                for (int32_t kb = 0; kb < n_kb; ++kb, ++it) {
                    const uint32_t st = it % kStages, use = it / kStages;
                    if (use > 0 && !mbar_wait(bar(kEmpty + st), (use - 1) & 1, abort)) { ok = false; break; }
                    mbar_arrive_expect_tx(bar(kFull + st), kBBytes);
                    tma_load_2d(base + st * kStageBytes + kABytes, &tmW, bar(kFull + st), kb * kBK, n0);
                }
            }
            if (*abort) {
                for (uint32_t t = (it > (uint32_t)kStages ? it - kStages : 0); t < it; ++t)
                    mbar_wait_drain_bounded(bar(kFull + t % kStages), (t / kStages) & 1);
            }
        }
    } else if (warp == kMmaWarp) {
        if (lane == 0) {
            // ---------------- MMA issuer ----------------
            constexpr uint32_t idesc = make_idesc_f16(StoreT<T>::kUmmaFormat, 0, kHalf, kBN);
            uint32_t it = 0, t_it = 0;
            bool ok = true, issued = false;
            for (int32_t u = blockIdx.x; ok && u < n_tiles; u += gridDim.x, ++t_it) {
                // the accumulators are free once the epilogue has drained the previous tile
                if (t_it > 0 && !mbar_wait(bar(kAccEmpty), (t_it - 1) & 1, abort)) { ok = false; break; }
                tc_fence_after();
                for (int32_t kb = 0; kb < n_kb; ++kb, ++it) {
                    const uint32_t st = it % kStages;
                    if (!mbar_wait(bar(kFull + st), (it / kStages) & 1, abort)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t sa = base + st * kStageBytes, sb = sa + kABytes;
#pragma unroll
                    for (int h = 0; h < 2; ++h)          // the two 128-row halves share the W slice
#pragma unroll
                        for (int k = 0; k < kBK / 16; ++k)
                            umma_ss(tmem + h * kBN, smem_desc_sw128(sa + h * (kHalf * 128u) + k * 32u, 16, 1024),
                                    smem_desc_sw128(sb + k * 32u, 16, 1024), idesc, (kb > 0 || k > 0) ? 1u : 0u);
                    issued = true;
                    umma_commit(bar(kEmpty + st));
                }
                if (!ok) break;
                umma_commit(bar(kAccFull));
            }
            if (*abort && issued) {   // the issued MMAs still read shared memory: wait for them
                umma_commit(bar(kDrain));
                mbar_wait_drain_bounded(bar(kDrain), 0);
            }
        }
    } else {
        // ---------- epilogue: 8 warps; warp (sub-partition s, half h) drains TMEM lanes of rows
        // h*128 + 32s .. +32 from accumulator h, one tile row per thread ----------
        auto wwait = [&](uint32_t b_, uint32_t par_) -> bool {
            return __all_sync(0xffffffffu, mbar_wait(b_, par_, abort));
        };
        const int sub = warp & 3;                          // TMEM sub-partition of this warp
        const int half = (warp - kEpiWarp0) / 4;
        const int r = half * kHalf + sub * 32 + (int)lane; // tile row
        const uint32_t lane_off = (uint32_t)(sub * 32) << 16;
        const uint32_t acc = (uint32_t)half;
        uint32_t t_it = 0;
        for (int32_t u = blockIdx.x; u < n_tiles; u += gridDim.x, ++t_it) {
            const int32_t m = (u % n_mt) * kBM + r, n0 = (u / n_mt) * kBN;
            const int32_t i = m < M ? __ldg(a.idx + m) : -1;
            if (!wwait(bar(kAccFull), t_it & 1)) break;
            tc_fence_after();
            const int32_t part = n0 / a.c_part, col0 = n0 - part * a.c_part;
            T* yrow = (i >= 0 && i < a.n_tokens)
                          ? static_cast<T*>(part == 0 ? a.y[0] : part == 1 ? a.y[1] : a.y[2]) + (int64_t)i * a.ld_y + col0
                          : nullptr;
#pragma unroll 1
            for (int c0 = 0; c0 < kBN; c0 += 32) {
                uint32_t v[32];
                FXR_TMEM_LD32(tmem + lane_off + acc * kBN + c0, v);
                if (yrow != nullptr) {
                    uint4 pk[4];
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        float f[8];
#pragma unroll
                        for (int e = 0; e < 8; ++e)
                            f[e] = __uint_as_float(v[8 * q + e]) + (a.bias ? __ldg(a.bias + n0 + c0 + 8 * q + e) : 0.f);
                        pk[q] = make_uint4(StoreT<T>::pack2(f[0], f[1]), StoreT<T>::pack2(f[2], f[3]),
                                           StoreT<T>::pack2(f[4], f[5]), StoreT<T>::pack2(f[6], f[7]));
                    }
                    uint4* dst = reinterpret_cast<uint4*>(yrow + c0);
#pragma unroll
                    for (int q = 0; q < 4; ++q) dst[q] = pk[q];
                }
            }
            tc_fence_before();
            mbar_arrive(bar(kAccEmpty));
        }
    }

    __syncwarp();
    tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

}  // namespace gemm
}  // namespace fxr
