// fxr_attention.cuh — active-query flash attention on the 5th-generation tensor cores (sm_100a).
//
// Work unit: one 128-row tile of compact queries (qc) for one head, against all N keys of that
// head in 128-key tiles. Persistent CTAs (one per SM) walk the tiles round-robin; the executed-row
// count M is read from device memory, so the grid never depends on it.
//
// Warp roles (256 threads):
//   warp 0     TMA producer: Q tile, then K/V tiles into a STAGES-deep ring (128-byte swizzle)
//   warp 1     TMEM allocator and the single MMA-issuing thread:
//                S_b  = Q K_j^T   (tcgen05.mma kind::f16, A and B from shared memory, K-major)
//                O   += P_b V_j   (A = P read from tensor memory, B = V from shared memory, MN-major)
//   warps 4-7  softmax, O correction and epilogue, one thread per query row (= TMEM lane)
// Tensor memory (512 columns): S0 [0,128), S1 [128,256) double-buffered scores, O [256,384).
// P_b (bf16/fp16 pairs) overwrites the first 64 columns of S_b.
// Online softmax in the exp2 domain with lazy rescaling: O and the running sum are rescaled only
// when a row maximum grows by more than 2^8, so p <= 256 between rescales and the final O / l is
// exact. The scatter of the reference is fused: the epilogue stores row m of the tile straight to
// out[idx[m], h*128 ...].
// Every mbarrier wait is bounded (2 s); on timeout the kernel sets the device error word, drains
// its outstanding asynchronous copies and MMAs, frees its tensor memory and returns.
// Replaces attention_fwd (attention_kernels.cu:85-173) and scatter_tokens
// (gather_scatter_kernels.cu:46-72) on this path.
#pragma once

#include <cuda.h>

#include "fxr_device.cuh"

namespace fxr {
namespace attn {

constexpr int kBM = 128;                       // query rows per tile
constexpr int kBN = 128;                       // keys per tile
constexpr int kD = 128;                        // head dim
constexpr int kStages = 3;                     // K/V ring depth
constexpr int kThreads = 256;
constexpr uint32_t kHalfBytes = 128 * 128;     // 128 rows x 64 16-bit values (one 128-B swizzle span)
constexpr uint32_t kTileBytes = 2 * kHalfBytes;  // 128 x 128 16-bit tile
constexpr uint32_t kSmemQ = 0;
constexpr uint32_t kSmemKV = kTileBytes;       // stage s: K at kSmemKV + 2*s*kTileBytes, V right after
constexpr uint32_t kSmemBar = kSmemKV + kStages * 2 * kTileBytes;
constexpr uint32_t kSmemBytes = kSmemBar + 256 + 1024;  // barriers + 1024 B of alignment slack
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS0 = 0, kColO = 256;
constexpr float kRescaleThreshold = 8.0f;      // log2 units

// barrier slots (8 bytes each) after kSmemBar
enum Bar : uint32_t {
    kQFull = 0,
    kQEmpty = 1,
    kKFull = 2,                 // + stage
    kVFull = kKFull + kStages,  // + stage
    kKVEmpty = kVFull + kStages,
    kSFull = kKVEmpty + kStages,  // + buffer (2)
    kPFull = kSFull + 2,          // + buffer (2)
    kODone = kPFull + 2,          // + (PV index & 1)
    kOFree = kODone + 2,
    kDrain = kOFree + 1,
    kNumBars = kDrain + 1,
};
constexpr uint32_t kSlotTmem = kNumBars * 8;      // uint32 TMEM base address
constexpr uint32_t kSlotAbort = kSlotTmem + 4;    // int abort flag
static_assert(kSlotAbort + 4 <= 256, "barrier area overflow");

struct Params {
    const int32_t* count;
    const int32_t* idx;
    void* out;
    int64_t ld_out;
    int32_t n_tokens;
    int32_t n_heads;
    float scale_log2;   // softmax scale * log2(e)
    float* dbg;         // diagnostics (null in normal use): CTA 0's first tile dumps raw S of key
                        // tile 0 [128x128], unnormalised O [128x128], row sums and row maxima
};

__device__ __forceinline__ void mbar_wait_drain(uint32_t bar, uint32_t parity) {
    // Used only after an abort: waits (bounded, ignoring the abort flag) for an async operation
    // this thread issued, so that nothing writes this CTA's shared memory after it exits.
    const uint64_t t0 = global_timer_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (global_timer_ns() - t0 > kWaitLimitNs) break;
    }
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
attention_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                 const __grid_constant__ CUtensorMap tmV, const Params p) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t* gbase = smem_raw + (base - raw);
    const uint32_t sQ = base + kSmemQ;
    const uint32_t bar0 = base + kSmemBar;
    auto bar = [&](uint32_t i) { return bar0 + 8u * i; };
    volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(gbase + kSmemBar + kSlotTmem);
    volatile int* abort = reinterpret_cast<volatile int*>(gbase + kSmemBar + kSlotAbort);

    const int warp = threadIdx.x >> 5;
    const uint32_t lane = lane_id();

    if (threadIdx.x == 0) {
        mbar_init(bar(kQFull), 1);
        mbar_init(bar(kQEmpty), 1);
        for (int s = 0; s < kStages; ++s) {
            mbar_init(bar(kKFull + s), 1);
            mbar_init(bar(kVFull + s), 1);
            mbar_init(bar(kKVEmpty + s), 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(bar(kSFull + b), 1);
            mbar_init(bar(kPFull + b), 128);
            mbar_init(bar(kODone + b), 1);
        }
        mbar_init(bar(kOFree), 128);
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
    const int32_t n_qt = (M + kBM - 1) / kBM;
    const int32_t n_tiles = n_qt * p.n_heads;
    const int32_t n_kv = (p.n_tokens + kBN - 1) / kBN;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer ----------------
            uint32_t kv_it = 0, q_it = 0;
            bool ok = true;
            for (int32_t tile = blockIdx.x; ok && tile < n_tiles; tile += gridDim.x) {
                const int32_t head = tile / n_qt, qt = tile % n_qt;
                if (q_it > 0 && !mbar_wait(bar(kQEmpty), (q_it - 1) & 1, abort)) { ok = false; break; }
                mbar_arrive_expect_tx(bar(kQFull), kTileBytes);
                tma_load_2d(sQ, &tmQ, bar(kQFull), head * kD, qt * kBM);
                tma_load_2d(sQ + kHalfBytes, &tmQ, bar(kQFull), head * kD + 64, qt * kBM);
                ++q_it;
                for (int32_t j = 0; j < n_kv; ++j, ++kv_it) {
                    const uint32_t st = kv_it % kStages, use = kv_it / kStages;
                    if (use > 0 && !mbar_wait(bar(kKVEmpty + st), (use - 1) & 1, abort)) { ok = false; break; }
                    const uint32_t sK = base + kSmemKV + st * 2 * kTileBytes;
                    const uint32_t sV = sK + kTileBytes;
                    mbar_arrive_expect_tx(bar(kKFull + st), kTileBytes);
                    tma_load_2d(sK, &tmK, bar(kKFull + st), head * kD, j * kBN);
                    tma_load_2d(sK + kHalfBytes, &tmK, bar(kKFull + st), head * kD + 64, j * kBN);
                    mbar_arrive_expect_tx(bar(kVFull + st), kTileBytes);
                    tma_load_2d(sV, &tmV, bar(kVFull + st), head * kD, j * kBN);
                    tma_load_2d(sV + kHalfBytes, &tmV, bar(kVFull + st), head * kD + 64, j * kBN);
                }
            }
            if (*abort) {
                // drain: every load issued so far lands before the CTA exits
                if (q_it > 0) mbar_wait_drain(bar(kQFull), (q_it - 1) & 1);
                for (uint32_t t = (kv_it > kStages ? kv_it - kStages : 0); t < kv_it; ++t) {
                    mbar_wait_drain(bar(kKFull + t % kStages), (t / kStages) & 1);
                    mbar_wait_drain(bar(kVFull + t % kStages), (t / kStages) & 1);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer ----------------
            constexpr uint32_t fmt = StoreT<T>::kUmmaFormat;
            constexpr uint32_t idesc_qk = make_idesc_f16(fmt, 0, kBM, kBN);
            constexpr uint32_t idesc_pv = make_idesc_f16(fmt, 1, kBM, kD);
            uint32_t kv_it = 0, g = 0, tiles_done = 0, q_it = 0;
            bool ok = true;
            bool issued = false;
            auto issue_pv = [&](int32_t jj) -> bool {
                const uint32_t gg = g + jj, b = gg & 1;
                const uint32_t t = kv_it + jj, st = t % kStages, use = t / kStages;
                if (!mbar_wait(bar(kPFull + b), (gg >> 1) & 1, abort)) return false;
                if (!mbar_wait(bar(kVFull + st), use & 1, abort)) return false;
                if (jj == 0 && tiles_done > 0 && !mbar_wait(bar(kOFree), (tiles_done - 1) & 1, abort))
                    return false;
                tc_fence_after();
                const uint32_t sV = base + kSmemKV + st * 2 * kTileBytes + kTileBytes;
#pragma unroll
                for (int k = 0; k < kBN / 16; ++k) {
                    const uint64_t bdesc = smem_desc_sw128(sV + k * 2048u, kHalfBytes, 1024);
                    umma_ts(tmem + kColO, tmem + kColS0 + b * 128u + k * 8u, bdesc, idesc_pv,
                            (jj > 0 || k > 0) ? 1u : 0u);
                }
                umma_commit(bar(kKVEmpty + st));
                umma_commit(bar(kODone + (gg & 1)));
                return true;
            };
            for (int32_t tile = blockIdx.x; ok && tile < n_tiles; tile += gridDim.x) {
                if (!mbar_wait(bar(kQFull), q_it & 1, abort)) { ok = false; break; }
                ++q_it;
                tc_fence_after();
                for (int32_t j = 0; j < n_kv; ++j) {
                    const uint32_t t = kv_it + j, st = t % kStages, use = t / kStages;
                    if (!mbar_wait(bar(kKFull + st), use & 1, abort)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t b = (g + j) & 1;
                    const uint32_t sK = base + kSmemKV + st * 2 * kTileBytes;
#pragma unroll
                    for (int k = 0; k < kD / 16; ++k) {
                        const uint32_t off = (k >> 2) * kHalfBytes + (k & 3) * 32u;
                        umma_ss(tmem + kColS0 + b * 128u, smem_desc_sw128(sQ + off, 16, 1024),
                                smem_desc_sw128(sK + off, 16, 1024), idesc_qk, k > 0 ? 1u : 0u);
                    }
                    issued = true;
                    umma_commit(bar(kSFull + b));
                    if (j == n_kv - 1) umma_commit(bar(kQEmpty));
                    if (j > 0 && !issue_pv(j - 1)) { ok = false; break; }
                }
                if (!ok || !issue_pv(n_kv - 1)) { ok = false; break; }
                kv_it += n_kv;
                g += n_kv;
                ++tiles_done;
            }
            if (*abort && issued) {
                umma_commit(bar(kDrain));
                mbar_wait_drain(bar(kDrain), 0);
            }
        }
    } else if (warp >= 4) {
        // ---------------- softmax / correction / epilogue ----------------
        // Waits are made warp-uniform (every lane polls, then __all_sync) so that the
        // .sync.aligned tensor-memory loads/stores below are always executed by a converged warp,
        // also when a wait gives up.
        auto wwait = [&](uint32_t b_, uint32_t par_) -> bool {
            return __all_sync(0xffffffffu, mbar_wait(b_, par_, abort));
        };
        const int r = threadIdx.x - 128;                        // tile row = TMEM lane
        const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
        const uint32_t tS = tmem + lane_off + kColS0;
        const uint32_t tO = tmem + lane_off + kColO;
        const float c = p.scale_log2;
        T* __restrict__ out = static_cast<T*>(p.out);
        uint32_t g = 0;
        for (int32_t tile = blockIdx.x; tile < n_tiles; tile += gridDim.x) {
            const int32_t head = tile / n_qt, qt = tile % n_qt;
            float m_run = -INFINITY, l_run = 0.f;
            bool ok = true;
            for (int32_t j = 0; j < n_kv; ++j, ++g) {
                const uint32_t b = g & 1;
                if (!wwait(bar(kSFull + b), (g >> 1) & 1)) { ok = false; break; }
                tc_fence_after();
                uint32_t s[128];
                FXR_TMEM_LD64(tS + b * 128u, s);
                FXR_TMEM_LD64(tS + b * 128u + 64u, (s + 64));
                const int32_t kv_left = p.n_tokens - j * kBN;
                if (kv_left < kBN) {
#pragma unroll
                    for (int cc = 0; cc < 128; ++cc)
                        if (cc >= kv_left) s[cc] = __float_as_uint(-INFINITY);
                }
                if (p.dbg != nullptr && tile == (int32_t)blockIdx.x && blockIdx.x == 0 && j == 0) {
#pragma unroll
                    for (int cc = 0; cc < 128; ++cc) p.dbg[r * 128 + cc] = __uint_as_float(s[cc]);
                }
                float mx = __uint_as_float(s[0]);
#pragma unroll
                for (int cc = 1; cc < 128; ++cc) mx = fmaxf(mx, __uint_as_float(s[cc]));
                mx *= c;
                // keep this thread's view of the PV completions in step (PV(g-2) is done by now)
                if (j >= 2 && !wwait(bar(kODone + (g & 1)), ((g - 2) >> 1) & 1)) { ok = false; break; }
                if (j == 0) {
                    m_run = mx;
                } else {
                    const bool need = mx > m_run + kRescaleThreshold;
                    if (__any_sync(0xffffffffu, need)) {
                        if (!wwait(bar(kODone + ((g - 1) & 1)), ((g - 1) >> 1) & 1)) { ok = false; break; }
                        tc_fence_after();
                        const float m_new = fmaxf(m_run, mx);
                        const float alpha = ex2_approx(m_run - m_new);
                        l_run *= alpha;
                        m_run = m_new;
#pragma unroll
                        for (int h2 = 0; h2 < 2; ++h2) {
                            uint32_t o[64];
                            FXR_TMEM_LD64(tO + h2 * 64u, o);
#pragma unroll
                            for (int k = 0; k < 64; ++k) o[k] = __float_as_uint(__uint_as_float(o[k]) * alpha);
                            FXR_TMEM_ST32(tO + h2 * 64u, o);
                            FXR_TMEM_ST32(tO + h2 * 64u + 32u, (o + 32));
                        }
                    }
                }
                float sum = 0.f;
#pragma unroll
                for (int h2 = 0; h2 < 2; ++h2) {
                    uint32_t pk[32];
#pragma unroll
                    for (int k = 0; k < 32; ++k) {
                        const float p0 = ex2_approx(fmaf(__uint_as_float(s[h2 * 64 + 2 * k]), c, -m_run));
                        const float p1 = ex2_approx(fmaf(__uint_as_float(s[h2 * 64 + 2 * k + 1]), c, -m_run));
                        sum += p0 + p1;
                        pk[k] = StoreT<T>::pack2(p0, p1);
                    }
                    FXR_TMEM_ST32(tS + b * 128u + h2 * 32u, pk);
                }
                l_run += sum;
                tc_fence_before();
                mbar_arrive(bar(kPFull + b));
            }
            if (!ok) break;
            // epilogue: O is final once PV(g-1) completes
            if (!wwait(bar(kODone + ((g - 1) & 1)), ((g - 1) >> 1) & 1)) break;
            tc_fence_after();
            uint32_t o[128];
            FXR_TMEM_LD64(tO, o);
            FXR_TMEM_LD64(tO + 64u, (o + 64));
            tc_fence_before();
            mbar_arrive(bar(kOFree));
            if (p.dbg != nullptr && tile == (int32_t)blockIdx.x && blockIdx.x == 0) {
#pragma unroll
                for (int cc = 0; cc < 128; ++cc) p.dbg[16384 + r * 128 + cc] = __uint_as_float(o[cc]);
                p.dbg[32768 + r] = l_run;
                p.dbg[32768 + 128 + r] = m_run;
            }
            const int32_t m = qt * kBM + r;
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
