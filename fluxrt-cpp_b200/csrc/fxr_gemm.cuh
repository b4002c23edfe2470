// fxr_gemm.cuh — GEMMs over the executed rows of a frame (sm_100a, tcgen05 + TMEM).
//
// The reference runs every projection of a double-stream block on every token with fp32
// cublasSgemm (fluxrt-cpp src/inference/plugins/flux2_double_block_plugin.cpp:386-441: Q/K/V,
// out-projection, MLP up and down) and adds bias, GELU and the residual in separate passes
// (:400-458, flux2_kernels.cu:14-56,95-135). Here one kernel runs each of those products on the
// executed rows only, with the epilogue fused:
//
//   Y[r(m), :] = act( [A0 | A1][m, :] . [W0 | W1]^T + bias0 + bias1 )       or, with a residual,
//   Y[r(m), :] = R[r(m), :] + gate (.) ( [A0 | A1][m, :] . [W0 | W1]^T + bias0 + bias1 )
//
// for the compact rows m in [row0, row_end) (row_end < 0: the device count). Each A operand is
// gathered — row idx[m] of a token-major buffer — or compact — row m; A0 covers the first K0
// columns, A1 (if present) the rest, each with its own weight W_i [n_out, K_i] (row-major, the
// nn.Linear layout). The output columns are cut into up to four parts (Q | K | V, or
// Q | K | V | MLP for a fused single-stream projection), each written to its own buffer,
// scattered (row idx[m]) or compact (row m), with or without the tanh GELU.
//
// A persistent CTA per SM walks 128 x 256 output tiles (m fastest, so the CTAs working at one time
// share a 256-column slice of W through L2):
//   * 8 warps gather the tile's 128 rows of A with cp.async (16 bytes per copy, each warp
//     instruction reading four whole 128-byte row segments, written in the 128-byte swizzle the
//     tensor core reads; rows past the count are zero-filled);
//   * 1 warp streams W's 256 x 64 slices with TMA (128-byte swizzle);
//   * 1 warp issues tcgen05.mma (M 128, N 256, K 16; bf16/fp16 in, fp32 in tensor memory) into one
//     of two 256-column accumulators, alternating per tile, so the epilogue of a tile runs while the
//     next tile's products accumulate;
//   * 8 warps drain the other accumulator: tensor memory -> registers, epilogue, -> bf16/fp16,
//     staged in shared memory and stored as whole 128-byte row segments.
// Stream-K schedule (when a scratch area is given): the K slices of all tiles are cut into one
// contiguous range per CTA, so every SM gets the same work whatever the tile count. A tile whose
// slices span several CTAs is finished by the CTA holding its first slice (which reaches it last,
// at the end of its range); each of the others leaves its fp32 partial tile in scratch and raises
// one flag per epilogue warp. The finisher adds the partials in CTA order, so results do not
// depend on timing. Every wait is bounded (2 s); after a timeout the kernel sets the device error
// word and returns.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "fxr_device.cuh"

namespace fxr {
namespace gemm {

// A tile is 128 rows x 256 columns: one tcgen05.mma shape (M 128, N 256). Two accumulators of 256
// columns fill tensor memory, so consecutive tiles alternate between them.
constexpr int kBM = 128, kBN = 256, kBK = 64;
constexpr int kStages = 4;
constexpr uint32_t kABytes = kBM * kBK * 2;          // 16 KB
constexpr uint32_t kBBytes = kBN * kBK * 2;          // 32 KB
constexpr uint32_t kStageBytes = kABytes + kBBytes;
constexpr int kAWarps = 8, kBWarp = 8, kMmaWarp = 9, kEpiWarp0 = 10, kEpiWarps = 8;
constexpr int kThreads = (kEpiWarp0 + kEpiWarps) * 32;   // 576
constexpr int kRowsPerAWarp = kBM / kAWarps;             // 16: four copy instructions per stage
constexpr uint32_t kTmemCols = 2 * kBN;                  // two accumulators
// Output staging: per epilogue warp 32 rows x 64 columns (bf16/fp16), written back as whole
// 128-byte row segments.
constexpr int kOutCols = 64;
constexpr uint32_t kOutWarpBytes = 32 * kOutCols * 2;                // 4 KB
constexpr uint32_t kSmemOut = kStages * kStageBytes;                 // 192 KB
constexpr uint32_t kSmemBar = kSmemOut + kEpiWarps * kOutWarpBytes;  // 224 KB
enum : uint32_t { kFull = 0, kEmpty = kStages, kAccFull = 2 * kStages, kAccEmpty = 2 * kStages + 2,
                  kDrain = 2 * kStages + 4, kNumBars = 2 * kStages + 5 };
constexpr uint32_t kSlotTmem = kNumBars * 8, kSlotAbort = kSlotTmem + 4;
constexpr uint32_t kSmemBytes = kSmemBar + 256 + 1024;     // + alignment slack (225.25 KB)
static_assert(kSmemBytes <= 232448, "dynamic shared memory above the 227 KB per-block limit");
static_assert(kNumBars * 8 + 8 <= 256, "barrier area");
constexpr int kEpiCols = 16;                             // accumulator columns per epilogue step
constexpr int kEpiColsPerWarp = kBN / 2;                 // two warps per TMEM sub-partition

// Stream-K scratch: a sync area (word 0: launch generation, word 1: CTAs done; then a 128-byte line
// per CTA holding one flag per epilogue warp) followed by one fp32 partial tile per CTA. The flags
// of a launch are raised to generation + 1; the last CTA to finish advances the generation, so the
// area must be zero before its first use and needs no reset afterwards.
constexpr size_t kSyncBytes = 32768;
constexpr uint32_t kFlagWords = 32;
constexpr int kMaxCtas = (int)(kSyncBytes / (kFlagWords * 4)) - 1;   // 255
constexpr size_t kPartialBytes = (size_t)kBM * kBN * 4;              // 128 KB
constexpr int kMinItersPerCta = 8;   // below this a partial exchange costs more than it spreads

struct Operand {
    const void* rows;     // [*, ld] token-major (gathered) or compact rows
    int64_t ld;           // elements
    int32_t kb_end;       // the operand covers K slices [previous kb_end, kb_end)
    int32_t gathered;     // 1: row idx[m]; 0: row m
};
struct Part {
    void* rows;           // [*, ld]
    int64_t ld;
    int32_t col_end;      // the part holds output columns [previous col_end, col_end)
    int32_t scattered;    // 1: row idx[m]; 0: row m
    int32_t gelu;         // 1: tanh GELU after the bias
    int32_t pad;
};
struct Args {
    Operand op0, op1;                 // op1 is read for K slices >= op0.kb_end
    const int32_t* idx;
    const int32_t* count;
    int32_t row0, row_end;            // compact rows [row0, row_end); row_end < 0: *count
    int32_t n_tokens;                 // bound of idx values and compact rows
    int32_t n_kb, n_out, pad0;
    Part p0, p1, p2, p3;
    const float* bias0;               // [n_out] or null
    const float* bias1;
    const void* res;                  // [*, ld_res], rows like the output part's; null: no residual
    int64_t ld_res;
    const float* gate;                // [n_out] or null (gate 1)
    uint32_t* sync;                   // stream-K scratch; null: whole tiles per CTA
    float* partials;
};

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes)
                 : "memory");
}
// arrive on the barrier once every cp.async this thread issued so far has landed (the arrival is
// part of the barrier's expected count, hence .noinc)
__device__ __forceinline__ void cp_async_arrive_noinc(uint32_t bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
// rows written through the generic proxy become visible to the tensor core (async proxy)
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_gpu(uint32_t* p, uint32_t v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t x, uint32_t y, uint32_t z, uint32_t w) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(x), "r"(y), "r"(z), "r"(w)
                 : "memory");
}
__device__ __forceinline__ uint4 ld_shared_v4(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr)
                 : "memory");
    return v;
}
__device__ __forceinline__ void prefetch_l1(const void* p) {
    asm volatile("prefetch.global.L1 [%0];" ::"l"(p));
}
// tanh-form GELU, the formula of the reference's gelu_kernel (flux2_kernels.cu:14-21)
__device__ __forceinline__ float gelu_tanh(float x) {
    return 0.5f * x * (1.0f + tanhf(0.7978845608f * (x + 0.044715f * x * x * x)));
}

// ---- work schedule: every role walks the same segments ----
struct Sched {
    int64_t it, it_end;               // stream-K: this CTA's K slices
    int32_t n_kb, n_tiles, u, ctas;   // u: next tile (whole-tile schedule); ctas: CTAs with work
    bool sk;
};
struct Seg {
    int32_t tile, kb0, kb1;
    bool started, ended;              // holds the tile's first / last K slice
};
__device__ __forceinline__ int64_t sk_begin(int64_t total, int32_t c, int32_t ctas) {
    return total * c / ctas;
}
__device__ __forceinline__ Sched make_sched(int32_t n_tiles, int32_t n_kb, bool sk) {
    Sched s;
    s.n_kb = n_kb;
    s.n_tiles = n_tiles;
    s.u = blockIdx.x;
    s.ctas = (int32_t)gridDim.x;
    s.it = s.it_end = 0;
    // Whole tiles unless their last wave leaves SMs idle: with whole-tile waves at least 70 % busy
    // the partial exchanges of stream-K cost more than they save (measured on B200 over
    // 36..1296 tiles of 48 and 192 K slices).
    if (sk) {
        const int64_t waves = ((int64_t)n_tiles + gridDim.x - 1) / gridDim.x;
        if ((int64_t)n_tiles * 10 >= waves * gridDim.x * 7) sk = false;
    }
    s.sk = sk;
    if (sk) {
        const int64_t total = (int64_t)n_tiles * n_kb;
        const int64_t want = (total + kMinItersPerCta - 1) / kMinItersPerCta;
        s.ctas = (int32_t)min((int64_t)gridDim.x, max((int64_t)n_tiles, want));
        if ((int32_t)blockIdx.x < s.ctas) {
            s.it = sk_begin(total, blockIdx.x, s.ctas);
            s.it_end = sk_begin(total, blockIdx.x + 1, s.ctas);
        }
    }
    return s;
}
__device__ __forceinline__ bool next_seg(Sched& s, Seg& g) {
    if (!s.sk) {
        if (s.u >= s.n_tiles) return false;
        g.tile = s.u;
        g.kb0 = 0;
        g.kb1 = s.n_kb;
        g.started = g.ended = true;
        s.u += gridDim.x;
        return true;
    }
    if (s.it >= s.it_end) return false;
    const int32_t t = (int32_t)(s.it / s.n_kb);
    const int64_t t0 = (int64_t)t * s.n_kb;
    const int64_t e = min(s.it_end, t0 + s.n_kb);
    g.tile = t;
    g.kb0 = (int32_t)(s.it - t0);
    g.kb1 = (int32_t)(e - t0);
    g.started = g.kb0 == 0;
    g.ended = g.kb1 == s.n_kb;
    s.it = e;
    return true;
}

template <typename T, bool kRes>
__global__ void __launch_bounds__(kThreads, 1)
rows_gemm_kernel(const __grid_constant__ CUtensorMap tmW0, const __grid_constant__ CUtensorMap tmW1,
                 const __grid_constant__ Args a) {
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
        for (int b = 0; b < 2; ++b) {
            mbar_init(bar(kAccFull + b), 1);
            mbar_init(bar(kAccEmpty + b), kEpiWarps * 32);
        }
        mbar_init(bar(kDrain), 1);
        *abort = 0;
        fence_mbar_init();
    }
    if (warp == kBWarp && lane == 0) {
        prefetch_tmap(&tmW0);
        if (a.op1.rows) prefetch_tmap(&tmW1);
    }
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
    pdl_wait();   // idx / count and the A rows come from earlier kernels
    const int32_t row_end = a.row_end >= 0 ? a.row_end : *a.count;
    const int32_t rows = max(0, row_end - a.row0);
    const int32_t n_mt = (rows + kBM - 1) / kBM, n_nt = a.n_out / kBN;
    const int32_t n_tiles = n_mt * n_nt;
    const bool sk = a.sync != nullptr;

    if (warp < kAWarps) {
        // ---------------- row gather of A ----------------
        // Each thread's copies of a stage arrive on the stage's barrier by themselves once they have
        // landed (cp.async.mbarrier.arrive), so every stage can be in flight at once; the MMA thread
        // fences the landed rows for the tensor core after its wait.
        // Lane l of warp w moves 16-byte chunk (l % 8) of rows w*16 + 4j + l/8, j = 0..3: each copy
        // instruction of a warp reads four whole 128-byte row segments.
        constexpr int kJ = kRowsPerAWarp / 4;
        const int c = (int)(lane & 7), sub = (int)(lane >> 3);
        uint32_t it = 0;
        bool ok = true;
        Sched sc = make_sched(n_tiles, a.n_kb, sk);
        Seg g;
        while (ok && next_seg(sc, g)) {
            int32_t tok[kJ];   // token row of each of this thread's tile rows, -1 past the count
            int32_t crow[kJ];  // compact row, -1 past the count
#pragma unroll
            for (int j = 0; j < kJ; ++j) {
                const int32_t ml = (g.tile % n_mt) * kBM + warp * kRowsPerAWarp + 4 * j + sub;
                const int32_t m = a.row0 + ml;
                int32_t i = -1;
                if (ml < rows) {
                    i = m < a.n_tokens ? __ldg(a.idx + m) : -1;
                    if (i < 0 || i >= a.n_tokens) {
                        atomicOr(&g_error_word, kErrBounds);
                        i = -1;
                    }
                }
                tok[j] = i;
                crow[j] = i < 0 ? -1 : m;
            }
            const char* src[kJ];
            int cur_op = -1;
            for (int32_t kb = g.kb0; kb < g.kb1; ++kb, ++it) {
                const int op = kb < a.op0.kb_end ? 0 : 1;
                if (op != cur_op) {   // first slice of an operand in this segment: row addresses
                    cur_op = op;
                    const char* rb = static_cast<const char*>(op == 0 ? a.op0.rows : a.op1.rows);
                    const int64_t ldb = (op == 0 ? a.op0.ld : a.op1.ld) * (int64_t)sizeof(T);
                    const bool gath = (op == 0 ? a.op0.gathered : a.op1.gathered) != 0;
                    const int64_t k_base = (int64_t)(op == 0 ? 0 : a.op0.kb_end) * kBK * (int64_t)sizeof(T);
#pragma unroll
                    for (int j = 0; j < kJ; ++j) {
                        const int32_t r = gath ? tok[j] : crow[j];
                        src[j] = rb + (int64_t)(r < 0 ? 0 : r) * ldb + c * 16 - k_base;
                    }
                }
                const uint32_t st = it % kStages, use = it / kStages;
                if (use > 0 && !mbar_wait(bar(kEmpty + st), (use - 1) & 1, abort)) { ok = false; break; }
                const uint32_t stage = base + st * kStageBytes;
                const int64_t koff = (int64_t)kb * kBK * (int64_t)sizeof(T);
#pragma unroll
                for (int j = 0; j < kJ; ++j) {   // 128-byte swizzle: chunk c of row r at (c ^ r % 8)
                    const int r = warp * kRowsPerAWarp + 4 * j + sub;
                    cp_async16(stage + (uint32_t)(r * 128 + ((c ^ (r & 7)) * 16)), src[j] + koff,
                               tok[j] < 0 ? 0u : 16u);   // rows past the count: zeros
                }
                cp_async_arrive_noinc(bar(kFull + st));
            }
        }
        cp_async_wait_all();   // nothing lands in shared memory after the CTA exits
    } else if (warp == kBWarp) {
        if (lane == 0) {
            // ---------------- W slices (B operand) ----------------
            uint32_t it = 0;
            bool ok = true;
            Sched sc = make_sched(n_tiles, a.n_kb, sk);
            Seg g;
            while (ok && next_seg(sc, g)) {
                const int32_t n0 = (g.tile / n_mt) * kBN;
                for (int32_t kb = g.kb0; kb < g.kb1; ++kb, ++it) {
                    const uint32_t st = it % kStages, use = it / kStages;
                    if (use > 0 && !mbar_wait(bar(kEmpty + st), (use - 1) & 1, abort)) { ok = false; break; }
                    mbar_arrive_expect_tx(bar(kFull + st), kBBytes);
                    const uint32_t dst = base + st * kStageBytes + kABytes;
                    if (kb < a.op0.kb_end) tma_load_2d(dst, &tmW0, bar(kFull + st), kb * kBK, n0);
                    else tma_load_2d(dst, &tmW1, bar(kFull + st), (kb - a.op0.kb_end) * kBK, n0);
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
            constexpr uint32_t idesc = make_idesc_f16(StoreT<T>::kUmmaFormat, 0, kBM, kBN);
            uint32_t it = 0, t_it = 0;
            bool ok = true, issued = false;
            Sched sc = make_sched(n_tiles, a.n_kb, sk);
            Seg g;
            while (ok && next_seg(sc, g)) {
                const uint32_t buf = t_it & 1, use = t_it >> 1;
                // accumulator `buf` is free once the epilogue has drained the segment before last
                if (use > 0 && !mbar_wait(bar(kAccEmpty + buf), (use - 1) & 1, abort)) { ok = false; break; }
                tc_fence_after();
                const uint32_t d_tmem = tmem + buf * kBN;
                for (int32_t kb = g.kb0; kb < g.kb1; ++kb, ++it) {
                    const uint32_t st = it % kStages;
                    if (!mbar_wait(bar(kFull + st), (it / kStages) & 1, abort)) { ok = false; break; }
                    fence_proxy_async_smem();   // the gathered rows (generic proxy) for the tensor core
                    tc_fence_after();
                    const uint32_t sa = base + st * kStageBytes, sb = sa + kABytes;
#pragma unroll
                    for (int k = 0; k < kBK / 16; ++k)
                        umma_ss(d_tmem, smem_desc_sw128(sa + k * 32u, 16, 1024), smem_desc_sw128(sb + k * 32u, 16, 1024),
                                idesc, (kb > g.kb0 || k > 0) ? 1u : 0u);
                    issued = true;
                    umma_commit(bar(kEmpty + st));
                }
                if (!ok) break;
                umma_commit(bar(kAccFull + buf));
                ++t_it;
            }
            if (*abort && issued) {   // the issued MMAs still read shared memory: wait for them
                umma_commit(bar(kDrain));
                mbar_wait_drain_bounded(bar(kDrain), 0);
            }
        }
    } else {
        // ---------- epilogue: 8 warps; warp (sub-partition s, column half h) drains TMEM lanes of
        // rows 32s .. 32s + 32, columns [128h, 128h + 128), one tile row per thread ----------
        auto wwait = [&](uint32_t b_, uint32_t par_) -> bool {
            return __all_sync(0xffffffffu, mbar_wait(b_, par_, abort));
        };
        const int ew = warp - kEpiWarp0;                   // epilogue warp 0..7
        const int sub = warp & 3;                          // TMEM sub-partition of this warp
        const int colh = ew / 4;                           // which 128 columns
        const int r = sub * 32 + (int)lane;                // tile row
        const uint32_t lane_off = (uint32_t)(sub * 32) << 16;
        const uint32_t gen = sk ? ld_acquire_gpu(a.sync) : 0u;
        const uint32_t stg = base + kSmemOut + (uint32_t)ew * kOutWarpBytes;
        uint32_t t_it = 0;
        Sched sc = make_sched(n_tiles, a.n_kb, sk);
        Seg g;
        while (next_seg(sc, g)) {
            const uint32_t buf = t_it & 1;
            const int32_t mt = g.tile % n_mt, n0 = (g.tile / n_mt) * kBN;
            const int32_t ml = mt * kBM + r, m = a.row0 + ml;
            // the output part holding columns [n0, n0 + 256)
            Part P = a.p0;
            int32_t pc0 = 0;
            if (n0 >= a.p0.col_end) {
                pc0 = a.p0.col_end;
                P = a.p1;
                if (n0 >= a.p1.col_end) {
                    pc0 = a.p1.col_end;
                    P = a.p2;
                    if (n0 >= a.p2.col_end) {
                        pc0 = a.p2.col_end;
                        P = a.p3;
                    }
                }
            }
            int32_t orow = -1;
            if (g.started && ml < rows && m < a.n_tokens) {
                orow = P.scattered ? __ldg(a.idx + m) : m;
                if (orow < 0 || orow >= a.n_tokens) orow = -1;   // reported by the A gather
            }
            // epilogue operands fetched while the products accumulate: lane l holds the summed bias
            // (and the gate) of columns 4l .. 4l + 3 of this warp's 128; the residual row segment
            // is prefetched into L1
            const int32_t nw = n0 + colh * kEpiColsPerWarp;
            float4 bias_r = make_float4(0.f, 0.f, 0.f, 0.f), gate_r = make_float4(1.f, 1.f, 1.f, 1.f);
            if (g.started) {
                if (a.bias0) bias_r = __ldg(reinterpret_cast<const float4*>(a.bias0 + nw) + lane);
                if (a.bias1) {
                    const float4 b1 = __ldg(reinterpret_cast<const float4*>(a.bias1 + nw) + lane);
                    bias_r.x += b1.x;
                    bias_r.y += b1.y;
                    bias_r.z += b1.z;
                    bias_r.w += b1.w;
                }
                if (kRes && a.gate) gate_r = __ldg(reinterpret_cast<const float4*>(a.gate + nw) + lane);
                if (kRes && a.res && orow >= 0) {
                    const char* rp = reinterpret_cast<const char*>(static_cast<const T*>(a.res) + (int64_t)orow * a.ld_res + nw);
                    prefetch_l1(rp);
                    prefetch_l1(rp + 128);
                    prefetch_l1(rp + kEpiColsPerWarp * sizeof(T) - 1);
                }
            }
            if (!wwait(bar(kAccFull + buf), (t_it >> 1) & 1)) break;
            tc_fence_after();
            ++t_it;
            // contributors: the CTAs after this one whose ranges cover the rest of the tile; each
            // epilogue warp waits for the flag of the same warp of each contributor (which wrote the
            // same tile rows and columns)
            int32_t c_last = (int32_t)blockIdx.x;
            bool have_parts = true;
            if (g.started && !g.ended) {
                const int64_t total = (int64_t)n_tiles * a.n_kb, t_end = (int64_t)(g.tile + 1) * a.n_kb;
                while (c_last + 1 < sc.ctas && sk_begin(total, c_last + 1, sc.ctas) < t_end) ++c_last;
                for (int32_t cc = (int32_t)blockIdx.x + 1; have_parts && cc <= c_last; ++cc) {
                    const uint32_t* flag = a.sync + (size_t)(cc + 1) * kFlagWords + ew;
                    const uint64_t t0 = global_timer_ns();
                    uint32_t polls = 0;
                    while (ld_acquire_gpu(flag) != gen + 1u) {
                        if ((++polls & 63u) == 0 && (global_timer_ns() - t0 > kWaitLimitNs || *abort)) {
                            atomicOr(&g_error_word, kErrTimeout);
                            *abort = 1;
                            have_parts = false;
                            break;
                        }
                    }
                }
            }
            have_parts = __all_sync(0xffffffffu, have_parts);
            // output row of each tile row (-1: no store); the stores below read it by shuffle
            const int32_t orow_ok = (orow >= 0 && have_parts) ? orow : -1;
            const T* rrow = (kRes && orow_ok >= 0 && a.res)
                                ? static_cast<const T*>(a.res) + (int64_t)orow_ok * a.ld_res + n0
                                : nullptr;
#pragma unroll 1
            for (int cb = colh * kEpiColsPerWarp; cb < (colh + 1) * kEpiColsPerWarp; cb += kOutCols) {
                // 64 columns: 4 steps of 16 from tensor memory, each thread's row into the staging
                // block (128 bytes per row, 16-byte chunk c of row r at c ^ (r % 8))
#pragma unroll 1
                for (int c0 = cb; c0 < cb + kOutCols; c0 += kEpiCols) {
                    __syncwarp();
                    uint32_t v[kEpiCols];
                    FXR_TMEM_LD16(tmem + lane_off + buf * kBN + c0, v);
                    if (!g.started) {   // leave the partial for the finisher (512 B per instruction)
                        float4* my_part = reinterpret_cast<float4*>(a.partials + (size_t)blockIdx.x * (kPartialBytes / 4));
#pragma unroll
                        for (int q = 0; q < kEpiCols / 4; ++q)
                            __stcg(my_part + (size_t)(c0 / 4 + q) * kBM + r,
                                   make_float4(__uint_as_float(v[4 * q]), __uint_as_float(v[4 * q + 1]),
                                               __uint_as_float(v[4 * q + 2]), __uint_as_float(v[4 * q + 3])));
                        continue;
                    }
                    float f[kEpiCols];
#pragma unroll
                    for (int e = 0; e < kEpiCols; ++e) f[e] = __uint_as_float(v[e]);
                    if (orow_ok >= 0) {
                        for (int32_t cc = (int32_t)blockIdx.x + 1; cc <= c_last; ++cc) {
                            const float4* pp = reinterpret_cast<const float4*>(a.partials + (size_t)cc * (kPartialBytes / 4));
#pragma unroll
                            for (int q = 0; q < kEpiCols / 4; ++q) {
                                const float4 x = __ldcg(pp + (size_t)(c0 / 4 + q) * kBM + r);
                                f[4 * q] += x.x;
                                f[4 * q + 1] += x.y;
                                f[4 * q + 2] += x.z;
                                f[4 * q + 3] += x.w;
                            }
                        }
                    }
                    const int src0 = (c0 - colh * kEpiColsPerWarp) / 4;   // lane holding column c0
                    if (a.bias0 || a.bias1) {
#pragma unroll
                        for (int q = 0; q < kEpiCols / 4; ++q) {
                            f[4 * q] += __shfl_sync(0xffffffffu, bias_r.x, src0 + q);
                            f[4 * q + 1] += __shfl_sync(0xffffffffu, bias_r.y, src0 + q);
                            f[4 * q + 2] += __shfl_sync(0xffffffffu, bias_r.z, src0 + q);
                            f[4 * q + 3] += __shfl_sync(0xffffffffu, bias_r.w, src0 + q);
                        }
                    }
                    if (P.gelu) {
#pragma unroll
                        for (int e = 0; e < kEpiCols; ++e) f[e] = gelu_tanh(f[e]);
                    }
                    if (kRes && a.res) {   // f = residual + gate * f; the gate shuffles are warp-wide
                        const uint2* rs = rrow != nullptr ? reinterpret_cast<const uint2*>(rrow + c0) : nullptr;
#pragma unroll
                        for (int q = 0; q < kEpiCols / 4; ++q) {
                            const float g0 = __shfl_sync(0xffffffffu, gate_r.x, src0 + q);
                            const float g1 = __shfl_sync(0xffffffffu, gate_r.y, src0 + q);
                            const float g2 = __shfl_sync(0xffffffffu, gate_r.z, src0 + q);
                            const float g3 = __shfl_sync(0xffffffffu, gate_r.w, src0 + q);
                            const uint2 x = rs != nullptr ? rs[q] : make_uint2(0u, 0u);
                            const float2 r0 = StoreT<T>::unpack2(x.x), r1 = StoreT<T>::unpack2(x.y);
                            f[4 * q] = fmaf(g0, f[4 * q], r0.x);
                            f[4 * q + 1] = fmaf(g1, f[4 * q + 1], r0.y);
                            f[4 * q + 2] = fmaf(g2, f[4 * q + 2], r1.x);
                            f[4 * q + 3] = fmaf(g3, f[4 * q + 3], r1.y);
                        }
                    }
#pragma unroll
                    for (int q = 0; q < kEpiCols / 8; ++q) {
                        const int ch = (c0 - cb) / 8 + q;
                        st_shared_v4(stg + (uint32_t)(lane * 128 + ((ch ^ (lane & 7)) * 16)),
                                     StoreT<T>::pack2(f[8 * q], f[8 * q + 1]), StoreT<T>::pack2(f[8 * q + 2], f[8 * q + 3]),
                                     StoreT<T>::pack2(f[8 * q + 4], f[8 * q + 5]), StoreT<T>::pack2(f[8 * q + 6], f[8 * q + 7]));
                    }
                }
                if (!g.started) continue;
                __syncwarp();
                // the warp's 32 rows x 64 columns back out: each instruction stores four whole
                // 128-byte row segments (lane l: row 4i + l / 8, chunk l % 8)
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const int row = 4 * i + (int)(lane >> 3), ch = (int)(lane & 7);
                    const uint4 val = ld_shared_v4(stg + (uint32_t)(row * 128 + ((ch ^ (row & 7)) * 16)));
                    const int32_t orr = __shfl_sync(0xffffffffu, orow_ok, row);
                    if (orr >= 0)
                        *reinterpret_cast<uint4*>(static_cast<T*>(P.rows) + (int64_t)orr * P.ld + (n0 - pc0) + cb + ch * 8) = val;
                }
            }
            __syncwarp();
            tc_fence_before();
            mbar_arrive(bar(kAccEmpty + buf));
            if (!g.started) {   // publish this warp's part of the partial: its stores, then one flag
                __threadfence();
                __syncwarp();
                if (lane == 0) st_release_gpu(a.sync + (size_t)(blockIdx.x + 1) * kFlagWords + ew, gen + 1u);
            }
        }
    }

    __syncwarp();
    tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
    if (sk && threadIdx.x == 0) {
        // the last CTA of the launch advances the generation the next launch's flags compare to
        __threadfence();
        const uint32_t gen = ld_acquire_gpu(a.sync);
        const uint32_t done = atomicAdd(a.sync + 1, 1u);
        if (done == gridDim.x - 1) {
            a.sync[1] = 0u;
            __threadfence();
            st_release_gpu(a.sync, gen + 1u);
        }
    }
}

}  // namespace gemm
}  // namespace fxr
