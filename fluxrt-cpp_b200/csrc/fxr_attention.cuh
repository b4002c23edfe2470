// fxr_attention.cuh — active-query flash attention on the 5th-generation tensor cores (sm_100a).
//
// Work unit: 256 compact query rows (two 128-row tiles Q0, Q1) of one head against all N keys of
// that head in 128-key tiles. Persistent CTAs (one per SM) walk the work units round-robin; the
// executed-row count M is read from device memory, so the grid never depends on it.
//
// Warp roles (384 threads):
//   warp 0      TMA producer: Q0+Q1, a 3-deep K ring and a 2-deep V ring (128-byte swizzle)
//   warp 1      TMEM allocator and the single MMA-issuing thread
//   warps 4-7   softmax / O correction / epilogue of Q0 (one thread per row = TMEM lane)
//   warps 8-11  the same for Q1
// Tensor memory (512 columns): S0 [0,128), S1 [128,256), O0 [256,384), O1 [384,512).
// P_t (16-bit pairs) overwrites the first 64 columns of S_t and is the A operand of O_t += P_t V.
//
// MMA order per key tile j (ping-pong): PV0(j), QK0(j+1), PV1(j), QK1(j+1). While softmax 0 works
// on S0(j) the tensor core runs PV1(j-1) and QK1(j); while softmax 1 works on S1(j) it runs PV0(j)
// and QK0(j+1). tcgen05 operations of one thread execute in issue order, and a commit tracks all
// earlier operations of the thread, so the barrier that signals S_t(j) also guarantees that
// PV_t(j-1) finished: the softmax may rescale O_t right away.
// Softmax in the exp2 domain with lazy rescaling: O and the running sum are rescaled only when a
// row maximum grows by more than 2^8, so p <= 256 between rescales and O / l is exact. The
// special-function unit computes 16 exp2 per clock per SM, exactly the rate at which one SM's
// tensor core consumes them (4*128 FLOP per score), so a quarter of the exponentials run as a
// polynomial on the FMA pipe (ex2_poly).
// The reference's scatter is fused: the epilogue stores row m straight to out[idx[m], h*128 ...].
// Every mbarrier wait is bounded (2 s); on timeout the kernel sets the device error word, drains
// its outstanding copies and MMAs, frees its tensor memory and returns.
// Replaces attention_fwd (attention_kernels.cu:85-173) and scatter_tokens
// (gather_scatter_kernels.cu:46-72) on this path.
#pragma once

#include <cuda.h>

#include "fxr_device.cuh"

namespace fxr {
namespace attn {

constexpr int kBM = 128;                        // query rows per tile (two tiles per work unit)
constexpr int kUnitRows = 2 * kBM;
constexpr int kBN = 128;                        // keys per tile
constexpr int kD = 128;                         // head dim
constexpr int kKStages = 3;
constexpr int kVStages = 2;
constexpr int kThreads = 384;
constexpr uint32_t kHalfBytes = 128 * 128;      // 128 rows x 64 16-bit values (one swizzle span)
constexpr uint32_t kTileBytes = 2 * kHalfBytes; // 128 x 128 16-bit tile
constexpr uint32_t kSmemQ = 0;                  // Q0, Q1
constexpr uint32_t kSmemK = 2 * kTileBytes;
constexpr uint32_t kSmemV = kSmemK + kKStages * kTileBytes;
constexpr uint32_t kSmemBar = kSmemV + kVStages * kTileBytes;
constexpr uint32_t kSmemBytes = kSmemBar + 256 + 1024;  // barriers + alignment slack
constexpr uint32_t kTmemCols = 512;
constexpr float kRescaleThreshold = 8.0f;       // log2 units
constexpr int kPolyPeriod = 4;                  // of every 4 score pairs ...
constexpr int kPolyCount = 1;                   // ... this many use ex2_poly

enum Bar : uint32_t {
    kQFull = 0,
    kQEmpty,
    kKFull,                          // + stage
    kKEmpty = kKFull + kKStages,     // + stage
    kVFull = kKEmpty + kKStages,     // + stage
    kVEmpty = kVFull + kVStages,     // + stage
    kSFull = kVEmpty + kVStages,     // + q tile
    kPFull = kSFull + 2,             // + q tile
    kODone = kPFull + 2,             // + q tile
    kOFree = kODone + 2,             // + q tile
    kDrain = kOFree + 2,
    kNumBars,
};
constexpr uint32_t kSlotTmem = kNumBars * 8;
constexpr uint32_t kSlotAbort = kSlotTmem + 4;
static_assert(kSlotAbort + 4 <= 256, "barrier area overflow");
static_assert(kSmemBytes <= 232448, "shared memory budget");

struct Params {
    const int32_t* count;
    const int32_t* idx;
    void* out;
    int64_t ld_out;
    int32_t n_tokens;
    int32_t n_heads;
    float scale_log2;   // softmax scale * log2(e)
};

__device__ __forceinline__ void mbar_wait_drain(uint32_t bar, uint32_t parity) {
    // After an abort only: waits (bounded, ignoring the abort flag) for an asynchronous operation
    // this thread issued, so that nothing lands in this CTA's shared memory after it exits.
    const uint64_t t0 = global_timer_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (global_timer_ns() - t0 > kWaitLimitNs) break;
    }
}

__device__ __forceinline__ float max3f(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}
// (a.x*b.x + c.x, a.y*b.y + c.y) in one packed instruction
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;"
        : "=l"(d)
        : "l"(*reinterpret_cast<uint64_t*>(&a)), "l"(*reinterpret_cast<uint64_t*>(&b)),
          "l"(*reinterpret_cast<uint64_t*>(&c)));
    return *reinterpret_cast<float2*>(&d);
}
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;"
        : "=l"(d)
        : "l"(*reinterpret_cast<uint64_t*>(&a)), "l"(*reinterpret_cast<uint64_t*>(&b)));
    return *reinterpret_cast<float2*>(&d);
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
attention_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                 const __grid_constant__ CUtensorMap tmV, const Params p) {
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
        mbar_init(bar(kQFull), 1);
        mbar_init(bar(kQEmpty), 1);
        for (int s = 0; s < kKStages; ++s) {
            mbar_init(bar(kKFull + s), 1);
            mbar_init(bar(kKEmpty + s), 1);
        }
        for (int s = 0; s < kVStages; ++s) {
            mbar_init(bar(kVFull + s), 1);
            mbar_init(bar(kVEmpty + s), 1);
        }
        for (int t = 0; t < 2; ++t) {
            mbar_init(bar(kSFull + t), 1);
            mbar_init(bar(kPFull + t), 128);
            mbar_init(bar(kODone + t), 1);
            mbar_init(bar(kOFree + t), 128);
        }
        mbar_init(bar(kDrain), 1);
        *abort = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&tmQ);
        prefetch_tmap(&tmK);
        prefetch_tmap(&tmV);
    }
    if (warp == 1) {
        tmem_alloc(smem_u32((const void*)tmem_slot), kTmemCols);
        tmem_relinquish();
    }
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    const int32_t M = *p.count;
    const int32_t n_units_q = (M + kUnitRows - 1) / kUnitRows;
    const int32_t n_units = n_units_q * p.n_heads;
    const int32_t n_kv = (p.n_tokens + kBN - 1) / kBN;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer ----------------
            uint32_t k_it = 0, v_it = 0, q_it = 0;
            bool ok = true;
            for (int32_t u = blockIdx.x; ok && u < n_units; u += gridDim.x) {
                const int32_t head = u / n_units_q, row0 = (u % n_units_q) * kUnitRows;
                if (q_it > 0 && !mbar_wait(bar(kQEmpty), (q_it - 1) & 1, abort)) { ok = false; break; }
                mbar_arrive_expect_tx(bar(kQFull), 2 * kTileBytes);
#pragma unroll
                for (int t = 0; t < 2; ++t) {
                    const uint32_t sQ = base + kSmemQ + t * kTileBytes;
                    tma_load_2d(sQ, &tmQ, bar(kQFull), head * kD, row0 + t * kBM);
                    tma_load_2d(sQ + kHalfBytes, &tmQ, bar(kQFull), head * kD + 64, row0 + t * kBM);
                }
                ++q_it;
                for (int32_t j = 0; ok && j < n_kv; ++j) {
                    {
                        const uint32_t st = k_it % kKStages, use = k_it / kKStages;
                        if (use > 0 && !mbar_wait(bar(kKEmpty + st), (use - 1) & 1, abort)) { ok = false; break; }
                        const uint32_t sK = base + kSmemK + st * kTileBytes;
                        mbar_arrive_expect_tx(bar(kKFull + st), kTileBytes);
                        tma_load_2d(sK, &tmK, bar(kKFull + st), head * kD, j * kBN);
                        tma_load_2d(sK + kHalfBytes, &tmK, bar(kKFull + st), head * kD + 64, j * kBN);
                        ++k_it;
                    }
                    {
                        const uint32_t st = v_it % kVStages, use = v_it / kVStages;
                        if (use > 0 && !mbar_wait(bar(kVEmpty + st), (use - 1) & 1, abort)) { ok = false; break; }
                        const uint32_t sV = base + kSmemV + st * kTileBytes;
                        mbar_arrive_expect_tx(bar(kVFull + st), kTileBytes);
                        tma_load_2d(sV, &tmV, bar(kVFull + st), head * kD, j * kBN);
                        tma_load_2d(sV + kHalfBytes, &tmV, bar(kVFull + st), head * kD + 64, j * kBN);
                        ++v_it;
                    }
                }
            }
            if (*abort) {
                if (q_it > 0) mbar_wait_drain(bar(kQFull), (q_it - 1) & 1);
                for (uint32_t t = (k_it > kKStages ? k_it - kKStages : 0); t < k_it; ++t)
                    mbar_wait_drain(bar(kKFull + t % kKStages), (t / kKStages) & 1);
                for (uint32_t t = (v_it > kVStages ? v_it - kVStages : 0); t < v_it; ++t)
                    mbar_wait_drain(bar(kVFull + t % kVStages), (t / kVStages) & 1);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer ----------------
            constexpr uint32_t fmt = StoreT<T>::kUmmaFormat;
            constexpr uint32_t idesc_qk = make_idesc_f16(fmt, 0, kBM, kBN);
            constexpr uint32_t idesc_pv = make_idesc_f16(fmt, 1, kBM, kD);
            uint32_t k_it = 0, v_it = 0, q_it = 0, p_it = 0, units_done = 0;
            bool ok = true, issued = false;
            // S_t = Q_t K^T (A, B from shared memory, both K-major)
            auto qk = [&](int t, uint32_t st) {
                const uint32_t sQ = base + kSmemQ + t * kTileBytes;
                const uint32_t sK = base + kSmemK + st * kTileBytes;
#pragma unroll
                for (int k = 0; k < kD / 16; ++k) {
                    const uint32_t off = (k >> 2) * kHalfBytes + (k & 3) * 32u;
                    umma_ss(tmem + t * 128u, smem_desc_sw128(sQ + off, 16, 1024),
                            smem_desc_sw128(sK + off, 16, 1024), idesc_qk, k > 0 ? 1u : 0u);
                }
                umma_commit(bar(kSFull + t));
            };
            // O_t (+)= P_t V (A = P from tensor memory, B = V from shared memory, MN-major)
            auto pv = [&](int t, int32_t jj, uint32_t st) {
                const uint32_t sV = base + kSmemV + st * kTileBytes;
#pragma unroll
                for (int k = 0; k < kBN / 16; ++k) {
                    const uint64_t bdesc = smem_desc_sw128(sV + k * 2048u, kHalfBytes, 1024);
                    umma_ts(tmem + 256u + t * 128u, tmem + t * 128u + k * 8u, bdesc, idesc_pv,
                            (jj > 0 || k > 0) ? 1u : 0u);
                }
            };
            for (int32_t u = blockIdx.x; ok && u < n_units; u += gridDim.x) {
                if (!mbar_wait(bar(kQFull), q_it & 1, abort)) { ok = false; break; }
                ++q_it;
                {   // prologue: S0(0), S1(0)
                    const uint32_t st = k_it % kKStages;
                    if (!mbar_wait(bar(kKFull + st), (k_it / kKStages) & 1, abort)) { ok = false; break; }
                    tc_fence_after();
                    issued = true;
                    qk(0, st);
                    qk(1, st);
                    umma_commit(bar(kKEmpty + st));
                    if (n_kv == 1) umma_commit(bar(kQEmpty));
                    ++k_it;
                }
                for (int32_t j = 0; j < n_kv; ++j) {
                    const uint32_t vs = v_it % kVStages;
                    // O0 += P0(j) V(j)
                    if (!mbar_wait(bar(kPFull + 0), p_it & 1, abort)) { ok = false; break; }
                    if (!mbar_wait(bar(kVFull + vs), (v_it / kVStages) & 1, abort)) { ok = false; break; }
                    if (j == 0 && units_done > 0 &&
                        !mbar_wait(bar(kOFree + 0), (units_done - 1) & 1, abort)) { ok = false; break; }
                    tc_fence_after();
                    pv(0, j, vs);
                    if (j == n_kv - 1) umma_commit(bar(kODone + 0));
                    // S0(j+1)
                    uint32_t ks = 0;
                    if (j + 1 < n_kv) {
                        ks = k_it % kKStages;
                        if (!mbar_wait(bar(kKFull + ks), (k_it / kKStages) & 1, abort)) { ok = false; break; }
                        tc_fence_after();
                        qk(0, ks);
                    }
                    // O1 += P1(j) V(j)
                    if (!mbar_wait(bar(kPFull + 1), p_it & 1, abort)) { ok = false; break; }
                    if (j == 0 && units_done > 0 &&
                        !mbar_wait(bar(kOFree + 1), (units_done - 1) & 1, abort)) { ok = false; break; }
                    tc_fence_after();
                    pv(1, j, vs);
                    umma_commit(bar(kVEmpty + vs));
                    ++v_it;
                    if (j == n_kv - 1) umma_commit(bar(kODone + 1));
                    ++p_it;
                    // S1(j+1)
                    if (j + 1 < n_kv) {
                        qk(1, ks);
                        umma_commit(bar(kKEmpty + ks));
                        if (j + 1 == n_kv - 1) umma_commit(bar(kQEmpty));
                        ++k_it;
                    }
                }
                ++units_done;
            }
            if (*abort && issued) {
                umma_commit(bar(kDrain));
                mbar_wait_drain(bar(kDrain), 0);
            }
        }
    } else if (warp >= 4) {
        // ---------------- softmax / correction / epilogue (one warpgroup per Q tile) ----------------
        // Waits are warp-uniform (every lane polls, then __all_sync) so that the .sync.aligned
        // tensor-memory accesses below always run on a converged warp, also when a wait gives up.
        auto wwait = [&](uint32_t b_, uint32_t par_) -> bool {
            return __all_sync(0xffffffffu, mbar_wait(b_, par_, abort));
        };
        const int t = (warp - 4) >> 2;                            // Q tile of this warpgroup
        const int r = (threadIdx.x - 128) & 127;                  // row in the tile = TMEM lane
        const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
        const uint32_t tS = tmem + lane_off + t * 128u;
        const uint32_t tO = tmem + lane_off + 256u + t * 128u;
        const float c = p.scale_log2;
        const float2 c2 = make_float2(c, c);
        T* __restrict__ out = static_cast<T*>(p.out);
        uint32_t s_it = 0, units_done = 0;
        for (int32_t u = blockIdx.x; u < n_units; u += gridDim.x) {
            const int32_t head = u / n_units_q, row0 = (u % n_units_q) * kUnitRows + t * kBM;
            float m_run = -INFINITY, l_run = 0.f;
            bool ok = true;
            for (int32_t j = 0; j < n_kv; ++j, ++s_it) {
                if (!wwait(bar(kSFull + t), s_it & 1)) { ok = false; break; }
                tc_fence_after();
                uint32_t s[128];
                FXR_TMEM_LD128(tS, s);
                const int32_t kv_left = p.n_tokens - j * kBN;
                if (kv_left < kBN) {
#pragma unroll
                    for (int cc = 0; cc < 128; ++cc)
                        if (cc >= kv_left) s[cc] = __float_as_uint(-INFINITY);
                }
                // row maximum: 8 independent chains of 3-input max
                float mp[8];
#pragma unroll
                for (int k = 0; k < 8; ++k) mp[k] = fmaxf(__uint_as_float(s[2 * k]), __uint_as_float(s[2 * k + 1]));
#pragma unroll
                for (int i = 1; i < 8; ++i)
#pragma unroll
                    for (int k = 0; k < 8; ++k)
                        mp[k] = max3f(mp[k], __uint_as_float(s[16 * i + 2 * k]), __uint_as_float(s[16 * i + 2 * k + 1]));
                const float mx = max3f(max3f(mp[0], mp[1], mp[2]), max3f(mp[3], mp[4], mp[5]), fmaxf(mp[6], mp[7])) * c;
                if (j == 0) {
                    m_run = mx;
                } else if (__any_sync(0xffffffffu, mx > m_run + kRescaleThreshold)) {
                    // S_t(j) is complete, hence so is PV_t(j-1): O_t may be rewritten now.
                    const float m_new = fmaxf(m_run, mx);
                    const float alpha = ex2_approx(m_run - m_new);
                    l_run *= alpha;
                    m_run = m_new;
#pragma unroll
                    for (int h2 = 0; h2 < 4; ++h2) {
                        uint32_t o[32];
                        FXR_TMEM_LD32(tO + h2 * 32u, o);
#pragma unroll
                        for (int k = 0; k < 32; ++k) o[k] = __float_as_uint(__uint_as_float(o[k]) * alpha);
                        FXR_TMEM_ST32(tO + h2 * 32u, o);
                    }
                }
                const float2 nm2 = make_float2(-m_run, -m_run);
                float2 acc[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                                 make_float2(0.f, 0.f)};
                // P overwrites the score registers pairwise (pk[k] from s[2k], s[2k+1]); one
                // 64-column store and one store wait per tile.
                uint32_t* pk = s;
#pragma unroll
                for (int k = 0; k < 64; ++k) {
                    const float2 x = ffma2(make_float2(__uint_as_float(s[2 * k]), __uint_as_float(s[2 * k + 1])),
                                           c2, nm2);
                    float2 e;
                    if ((k % kPolyPeriod) < kPolyCount) {
                        e = make_float2(ex2_poly(x.x), ex2_poly(x.y));
                    } else {
                        e = make_float2(ex2_approx(x.x), ex2_approx(x.y));
                    }
                    acc[k & 3] = fadd2(acc[k & 3], e);
                    pk[k] = StoreT<T>::pack2(e.x, e.y);
                }
                FXR_TMEM_ST64(tS, pk);
                const float2 a01 = fadd2(fadd2(acc[0], acc[1]), fadd2(acc[2], acc[3]));
                l_run += a01.x + a01.y;
                tc_fence_before();
                mbar_arrive(bar(kPFull + t));
            }
            if (!ok) break;
            // epilogue: O_t is final once its last PV completed
            if (!wwait(bar(kODone + t), units_done & 1)) break;
            tc_fence_after();
            uint32_t o[128];
            FXR_TMEM_LD128(tO, o);
            tc_fence_before();
            mbar_arrive(bar(kOFree + t));
            ++units_done;
            const int32_t m = row0 + r;
            if (m < M) {
                const int32_t i = p.idx[m];
                if (i >= 0 && i < p.n_tokens) {
                    const float inv = 1.0f / l_run;
                    uint4* dst = reinterpret_cast<uint4*>(out + (int64_t)i * p.ld_out + (int64_t)head * kD);
#pragma unroll
                    for (int k = 0; k < 16; ++k) {
                        uint4 v;
                        v.x = StoreT<T>::pack2(__uint_as_float(o[8 * k + 0]) * inv, __uint_as_float(o[8 * k + 1]) * inv);
                        v.y = StoreT<T>::pack2(__uint_as_float(o[8 * k + 2]) * inv, __uint_as_float(o[8 * k + 3]) * inv);
                        v.z = StoreT<T>::pack2(__uint_as_float(o[8 * k + 4]) * inv, __uint_as_float(o[8 * k + 5]) * inv);
                        v.w = StoreT<T>::pack2(__uint_as_float(o[8 * k + 6]) * inv, __uint_as_float(o[8 * k + 7]) * inv);
                        dst[k] = v;
                    }
                } else {
                    atomicOr(&g_error_word, kErrBounds);
                }
            }
        }
    }

    __syncwarp();  // role warps ran their loops on one lane; reconverge before the CTA barrier
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

}  // namespace attn
}  // namespace fxr
