// fxr_attention.cuh — active-query flash attention on the 5th-generation tensor cores (sm_100a).
//
// Work unit: one 128-row tile of compact queries of one head against all N keys of that head,
// in steps of 256 keys (two 128-key sub-tiles). Persistent CTAs (one per SM) walk the work units
// round-robin; the executed-row count M is read from device memory, so the grid never depends on it.
//
// Warp roles (576 threads):
//   warps 0-15  softmax: warpgroup g = warp/4 owns score columns [64g, 64g+64) of each step for
//               all 128 rows (one thread per row = TMEM lane), and O columns [32g, 32g+32) for the
//               correction and the epilogue
//   warp 16     TMA producer: Q tile and a 5-slot ring of 128-key K and V sub-tiles filled in
//               the tensor core's consumption order (128-byte swizzle)
//   warp 17     TMEM allocator and the single MMA-issuing thread
// Tensor memory (512 columns): S [0,256) fp32 scores of one step, P [256,384) the 16-bit
// probabilities of the step (pairs packed per column), O [384,512) fp32 output accumulator.
//
// Pipeline. S and P live in separate tensor memory, so the scores of step j+1 can be computed as
// soon as the softmax has loaded S(j) into registers (barrier S_FREE), while it still works on
// step j; the softmax only waits for PV(j-1) to finish (barrier P_FREE) right before it stores
// P(j). Tensor-core order: QK(j+1), PV(j), QK(j+2), ... A tcgen05.mma costs ~64-72 cycles for any
// N <= 128 (measured), so QK uses N = 128 per sub-tile and PV N = 128 (head dim) with A = P read
// from tensor memory.
// Softmax in the exp2 domain with lazy rescaling: O and the running sum are rescaled only when a
// row maximum grows by more than 2^8, so p <= 256 between rescales and O / l is exact. The four
// warps that hold the same 32 rows (one per warpgroup, same SM sub-partition) combine their
// partial row maxima through shared memory behind an mbarrier each step (bounded waits, no named
// barrier that could outlive an aborted partner), and their partial row sums once in the epilogue.
// The special-function unit computes 16 exp2 per clock per SM, the rate at which the tensor core
// consumes them (4*128 FLOP per score), so a quarter of the exponentials run as a polynomial on
// the FMA pipe (ex2_poly2).
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

constexpr int kBM = 128;                        // query rows per work unit
constexpr int kSubN = 128;                      // keys per K/V sub-tile
constexpr int kStepN = 2 * kSubN;               // keys per softmax step
constexpr int kD = 128;                         // head dim
constexpr int kSlots = 5;                       // K/V sub-tile ring, filled in consumption order
constexpr int kSoftmaxWarps = 16;
constexpr int kProducerWarp = 16;
constexpr int kMmaWarp = 17;
constexpr int kThreads = 32 * (kSoftmaxWarps + 2);
constexpr uint32_t kSoftmaxThreads = 32 * kSoftmaxWarps;
constexpr uint32_t kHalfBytes = 128 * 128;      // 128 rows x 64 16-bit values (one swizzle span)
constexpr uint32_t kTileBytes = 2 * kHalfBytes; // 128 x 128 16-bit tile
constexpr uint32_t kSmemQ = 0;
constexpr uint32_t kSmemRing = kTileBytes;
constexpr uint32_t kSmemX = kSmemRing + kSlots * kTileBytes;  // exchange [2 buf][4 wg][128 rows]
constexpr uint32_t kSmemRowIdx = kSmemX + 2 * 4 * 128 * 4;   // output row, stream of a softmax thread's item
constexpr uint32_t kSmemBar = kSmemRowIdx + 2 * kSoftmaxThreads * 4;   // [2][softmax thread]
constexpr uint32_t kSmemBytes = kSmemBar + 256 + 1024;       // barriers + alignment slack
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0, kColP = 256, kColO = 384;
constexpr float kRescaleThreshold = 8.0f;       // log2 units
constexpr int kPolyPeriod = 8;                  // of every 8 score pairs ...
constexpr int kPolyCount = 2;                   // ... this many use ex2_poly2

enum Bar : uint32_t {
    kQFull = 0,
    kQEmpty,
    kFull,                           // + ring slot: sub-tile landed
    kEmpty = kFull + kSlots,         // + ring slot: sub-tile consumed
    kSFull = kEmpty + kSlots,        // scores of a step computed
    kSFree,                          // scores loaded by every softmax thread
    kPFull,                          // probabilities of a step stored
    kPFree,                          // PV of a step finished (P and O may be touched)
    kOFree,                          // epilogue read O
    kXchg,                           // + (warp % 4): the four warps sharing 32 rows exchanged data
    kDrain = kXchg + 4,
    kNumBars,
};
constexpr uint32_t kSlotTmem = kNumBars * 8;
constexpr uint32_t kSlotAbort = kSlotTmem + 4;
constexpr uint32_t kSlotSched = kSlotAbort + 4;   // [parts per unit, work items] of the launch
static_assert(kSlotSched + 8 <= 256, "barrier area overflow");
static_assert(kSmemBytes <= 232448, "shared memory budget");

// Key-range split of a work unit across CTAs (when there are too few units to fill the GPU): each
// part writes its partial O (unnormalised, fp32) with its row maxima and sums to a scratch slot; per
// (unit, warp) portion an arrival counter elects the last-arriving part's warp, which combines all
// parts of its 32 rows x 32 columns and stores them. No CTA waits for another.
constexpr int kMaxSplits = 4;
// Costs in 256-key steps (measured: ~2.4 us per step at c2): the fixed cost of a work item (first
// Q tile, pipeline ramp, epilogue) and the extra cost of a split item (partial write, arrival
// counter, combine through L2).
constexpr float kItemOverheadSteps = 2.0f;
constexpr float kSplitOverheadSteps = 4.0f;
constexpr int kSplitSlotFloats = 128 * 128 + 2 * 4 * 128;   // O [128][128], m [4][128], l [4][128]
constexpr int kSplitPortions = 16;                   // softmax warps: counters per unit

struct Stream {                  // one edit stream of the launch
    const int32_t* count;        // executed rows (compaction output, device)
    const int32_t* idx;          // their token indices
    void* out;                   // O row base
    // Restore of the cache rows of mask==1 tokens at the end of the attention (two-tile kernel;
    // restore_rows == nullptr: the caller restores them with a separate launch). Lists written by
    // the compaction: compact rows, their number, and per head kRestoreSlots arrival counters that
    // start at zero.
    const int32_t* restore_rows;
    const int32_t* restore_count;
    const int32_t* restore_idx;  // compact row -> token (the attention's own idx may be a row numbering)
    int32_t* head_done;
    const uint4* save;           // [M][2 * row_vec] the saved K and V rows of each compact row
    char* cache_k;
    char* cache_v;
};

// Tensor maps of every stream: compact Q' and the K / V caches.
struct Maps {
    CUtensorMap q[kMaxBatch];
    CUtensorMap k[kMaxBatch];
    CUtensorMap v[kMaxBatch];
};

struct Params {
    Stream s[kMaxBatch];
    int32_t n_streams;
    int64_t ld_out;
    int32_t n_tokens;
    int32_t n_heads;
    float scale_log2;   // softmax scale * log2(e)
    float* split_scratch;        // [split_slots][kSplitSlotFloats]
    int32_t* split_cnt;          // [split_slots][kSplitPortions], zero at launch
    int32_t split_slots;         // 0: never split
    int64_t ld_cache_bytes;      // fused restore: cache row pitch
    int32_t row_vec;             // fused restore: 16-byte vectors per K (or V) row of the launch's heads
};

// Parts per unit: the shortest estimated kernel time (CTA rounds x steps per item + overheads);
// the same on every role of every CTA (a function of M, the grid and the scratch only). It splits
// only when the units leave SMs idle for long: a 2048^2 frame's 72 units of 66 steps per GPU of an
// 8-way head split, not the 1024^2 frame's 288 units of 18 steps.
__device__ __forceinline__ int32_t choose_splits(int32_t n_units, int32_t grid, int32_t n_steps,
                                                 int32_t slots) {
    int32_t best = 1;
    float best_cost = (float)((n_units + grid - 1) / grid) * ((float)n_steps + kItemOverheadSteps);
    for (int32_t sp = 2; sp <= kMaxSplits; ++sp) {
        if (sp > n_steps || n_units * sp > slots) break;
        const float cost = (float)((n_units * sp + grid - 1) / grid) *
                           ((float)n_steps / (float)sp + kItemOverheadSteps + kSplitOverheadSteps);
        if (cost < best_cost) {
            best = sp;
            best_cost = cost;
        }
    }
    return best;
}

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

// Two exp2 on the FMA pipe (ex2_poly in packed f32x2 form): magic-number rounding, degree-3
// polynomial on [-0.5, 0.5], exponent-field add.
__device__ __forceinline__ float2 ex2_poly2(float2 x) {
    constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
    x = make_float2(fmaxf(x.x, -125.0f), fmaxf(x.y, -125.0f));
    const float2 t = fadd2(x, make_float2(kMagic, kMagic));
    const float2 n = fadd2(t, make_float2(-kMagic, -kMagic));
    const float2 f = ffma2(n, make_float2(-1.0f, -1.0f), x);
    float2 q = ffma2(make_float2(0.055171654f, 0.055171654f), f, make_float2(0.24261114f, 0.24261114f));
    q = ffma2(q, f, make_float2(0.69326097f, 0.69326097f));
    q = ffma2(q, f, make_float2(0.99992806f, 0.99992806f));
    return make_float2(__int_as_float(__float_as_int(q.x) + (__float_as_int(t.x) << 23)),
                       __int_as_float(__float_as_int(q.y) + (__float_as_int(t.y) << 23)));
}

// End of a split unit for the part that arrived last at a (unit, warp) portion: every part (this one
// included) is read back from its slot and combined in part order — the result does not depend on
// which CTA arrived last — then normalised and stored like the unsplit epilogue.
// Work unit u of the launch -> stream b, head and first compact row; units are numbered stream
// after stream, (query tile, head) within a stream as tile + head * tiles. m_b: the stream's rows.
// (Loops over the streams use static indices only: a runtime index into the kernel parameters
// makes the compiler copy them to local memory, which costs the softmax warps ~130 bytes of spills.)
__device__ __forceinline__ void decode_unit(const Params& p, int32_t u, int32_t& b, int32_t& head,
                                            int32_t& row0, int32_t& m_b) {
    b = -1;
#pragma unroll
    for (int k = 0; k < kMaxBatch; ++k) {
        if (b < 0 && k < p.n_streams) {
            const int32_t mk = *p.s[k].count;
            const int32_t units = (mk + kBM - 1) / kBM * p.n_heads;
            if (u < units || k + 1 == p.n_streams) {
                b = k;
                m_b = mk;
            } else {
                u -= units;
            }
        }
    }
    const int32_t n_qt = (m_b + kBM - 1) / kBM;
    head = n_qt > 0 ? u / n_qt : 0;
    row0 = (u - head * n_qt) * kBM;
}

// Output row base of stream b (static-index selection, see above).
__device__ __forceinline__ void* stream_out(const Params& p, int32_t b) {
    void* o = p.s[0].out;
#pragma unroll
    for (int k = 1; k < kMaxBatch; ++k)
        if (k == b) o = p.s[k].out;
    return o;
}

// The fused-restore fields of stream b (static-index selection, see above).
struct RestoreRef {
    const int32_t* rows;
    const int32_t* count;
    int32_t* head_done;
    const uint4* save;
    char* cache_k;
    char* cache_v;
    const int32_t* idx;
    const int32_t* m;
};
__device__ __forceinline__ RestoreRef stream_restore(const Params& p, int32_t b) {
    RestoreRef r{p.s[0].restore_rows, p.s[0].restore_count, p.s[0].head_done, p.s[0].save,
                 p.s[0].cache_k, p.s[0].cache_v, p.s[0].restore_idx, p.s[0].count};
#pragma unroll
    for (int k = 1; k < kMaxBatch; ++k)
        if (k == b)
            r = RestoreRef{p.s[k].restore_rows, p.s[k].restore_count, p.s[k].head_done, p.s[k].save,
                           p.s[k].cache_k, p.s[k].cache_v, p.s[k].restore_idx, p.s[k].count};
    return r;
}

template <typename T>
__device__ __forceinline__ void split_combine_store(const Params& p, T* out, const float* slots, int32_t n_split,
                                                 int r, int wg, int32_t orow, int32_t head) {
    float m_all = -INFINITY;
    for (int32_t q = 0; q < n_split; ++q)
        m_all = fmaxf(m_all, slots[q * kSplitSlotFloats + kBM * kD + wg * kBM + r]);
    float acc[32];
#pragma unroll
    for (int k = 0; k < 32; ++k) acc[k] = 0.f;
    float l_tot = 0.f;
    for (int32_t q = 0; q < n_split; ++q) {
        const float* sq = slots + q * kSplitSlotFloats;
        const float a = ex2_approx(sq[kBM * kD + wg * kBM + r] - m_all);
        l_tot += a * sq[kBM * kD + 4 * kBM + wg * kBM + r];
        const float4* oq = reinterpret_cast<const float4*>(sq + r * kD + wg * 32);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const float4 x = oq[k];
            acc[4 * k] += a * x.x;
            acc[4 * k + 1] += a * x.y;
            acc[4 * k + 2] += a * x.z;
            acc[4 * k + 3] += a * x.w;
        }
    }
    if (orow < 0) return;                       // a padding row of the last tile
    if (orow >= p.n_tokens) {
        atomicOr(&g_error_word, kErrBounds);
        return;
    }
    const float inv = 1.0f / l_tot;
    const int64_t off = (int64_t)orow * p.ld_out + (int64_t)head * kD + wg * 32;
    uint4 v[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        v[k].x = StoreT<T>::pack2(acc[8 * k + 0] * inv, acc[8 * k + 1] * inv);
        v[k].y = StoreT<T>::pack2(acc[8 * k + 2] * inv, acc[8 * k + 3] * inv);
        v[k].z = StoreT<T>::pack2(acc[8 * k + 4] * inv, acc[8 * k + 5] * inv);
        v[k].w = StoreT<T>::pack2(acc[8 * k + 6] * inv, acc[8 * k + 7] * inv);
    }
    uint4* dst = reinterpret_cast<uint4*>(out + off);
#pragma unroll
    for (int k = 0; k < 4; ++k) dst[k] = v[k];
}

// kSplit: the instantiation that may split key ranges (launched for few heads per launch, where
// the units cannot fill the GPU); without it the split code is compiled out, since its mere presence
// costs the softmax loop ~10 % (register allocation).
template <typename T, bool kSplit>
__global__ void __launch_bounds__(kThreads, 1)
attention_kernel(const __grid_constant__ Maps maps, const __grid_constant__ Params p) {
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
        for (int s = 0; s < kSlots; ++s) {
            mbar_init(bar(kFull + s), 1);
            mbar_init(bar(kEmpty + s), 1);
        }
        mbar_init(bar(kSFull), 1);
        mbar_init(bar(kSFree), kSoftmaxThreads);
        mbar_init(bar(kPFull), kSoftmaxThreads);
        mbar_init(bar(kPFree), 1);
        mbar_init(bar(kOFree), kSoftmaxThreads);
        for (int q = 0; q < 4; ++q) mbar_init(bar(kXchg + q), kSoftmaxThreads / 4);
        mbar_init(bar(kDrain), 1);
        *abort = 0;
        fence_mbar_init();
    }
    if (warp == kProducerWarp && lane == 0) {
        // the first stream's descriptors (prefetching every stream's in a loop costs the softmax
        // warps ~130 bytes of register spills; the others are fetched on first use)
        prefetch_tmap(&maps.q[0]);
        prefetch_tmap(&maps.k[0]);
        prefetch_tmap(&maps.v[0]);
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

    // Everything above overlapped the previous kernel (programmatic dependent launch); the compact
    // queries, indices and count it wrote are read below.
    pdl_launch_dependents();
    pdl_wait();
    int32_t n_units = 0;
#pragma unroll
    for (int b = 0; b < kMaxBatch; ++b)
        if (b < p.n_streams) n_units += (*p.s[b].count + kBM - 1) / kBM * p.n_heads;
    const int32_t n_steps = (p.n_tokens + kStepN - 1) / kStepN;
    const int32_t n_split = kSplit ? choose_splits(n_units, (int32_t)gridDim.x, n_steps, p.split_slots) : 1;
    const int32_t n_items = n_units * n_split;   // item w: unit w / n_split, key part w % n_split
    // the softmax warps re-read the schedule from shared memory per item: in the split-capable
    // build, keeping it in registers across the step loop tips the allocation into spills
    volatile int32_t* sched = reinterpret_cast<volatile int32_t*>(gbase + kSmemBar + kSlotSched);
    if (kSplit) {
        if (threadIdx.x == 0) {
            sched[0] = n_split;
            sched[1] = n_items;
        }
        __syncthreads();
    }

    if (warp == kProducerWarp) {
        if (lane == 0) {
            // ---------------- TMA producer ----------------
            // Ring order = tensor-core consumption order of one unit:
            //   K(0) K(1) | K(2j) K(2j+1) V(2j-2) V(2j-1) for j = 1..n-1 | V(2n-2) V(2n-1)
            uint32_t it = 0, q_it = 0;
            bool ok = true;
            auto load = [&](const CUtensorMap* tm, int32_t head, int32_t key0) -> bool {
                const uint32_t st = it % kSlots, use = it / kSlots;
                if (use > 0 && !mbar_wait(bar(kEmpty + st), (use - 1) & 1, abort)) return false;
                const uint32_t dst = base + kSmemRing + st * kTileBytes;
                mbar_arrive_expect_tx(bar(kFull + st), kTileBytes);
                tma_load_2d(dst, tm, bar(kFull + st), head * kD, key0);
                tma_load_2d(dst + kHalfBytes, tm, bar(kFull + st), head * kD + 64, key0);
                ++it;
                return true;
            };
            for (int32_t w = blockIdx.x; ok && w < n_items; w += gridDim.x) {
                const int32_t u = w / n_split, part = w - u * n_split;
                int32_t b, head, row0, m_b;
                decode_unit(p, u, b, head, row0, m_b);
                const CUtensorMap* tmQ = &maps.q[0];
                const CUtensorMap* tmK = &maps.k[0];
                const CUtensorMap* tmV = &maps.v[0];
#pragma unroll
                for (int k = 1; k < kMaxBatch; ++k)
                    if (k == b) {
                        tmQ = &maps.q[k];
                        tmK = &maps.k[k];
                        tmV = &maps.v[k];
                    }
                const int32_t s0 = part * n_steps / n_split, s1 = (part + 1) * n_steps / n_split;
                if (q_it > 0 && !mbar_wait(bar(kQEmpty), (q_it - 1) & 1, abort)) { ok = false; break; }
                mbar_arrive_expect_tx(bar(kQFull), kTileBytes);
                tma_load_2d(base + kSmemQ, tmQ, bar(kQFull), head * kD, row0);
                tma_load_2d(base + kSmemQ + kHalfBytes, tmQ, bar(kQFull), head * kD + 64, row0);
                ++q_it;
                ok = load(tmK, head, s0 * kStepN) && load(tmK, head, s0 * kStepN + kSubN);
                for (int32_t j = s0 + 1; ok && j < s1; ++j)
                    ok = load(tmK, head, j * kStepN) && load(tmK, head, j * kStepN + kSubN) &&
                         load(tmV, head, (j - 1) * kStepN) && load(tmV, head, (j - 1) * kStepN + kSubN);
                ok = ok && load(tmV, head, (s1 - 1) * kStepN) &&
                     load(tmV, head, (s1 - 1) * kStepN + kSubN);
            }
            if (*abort) {
                if (q_it > 0) mbar_wait_drain(bar(kQFull), (q_it - 1) & 1);
                for (uint32_t t = (it > kSlots ? it - kSlots : 0); t < it; ++t)
                    mbar_wait_drain(bar(kFull + t % kSlots), (t / kSlots) & 1);
            }
        }
    } else if (warp == kMmaWarp) {
        if (lane == 0) {
            // ---------------- MMA issuer ----------------
            constexpr uint32_t fmt = StoreT<T>::kUmmaFormat;
            constexpr uint32_t idesc_qk = make_idesc_f16(fmt, 0, kBM, kSubN);
            constexpr uint32_t idesc_pv = make_idesc_f16(fmt, 1, kBM, kD);
            uint32_t it = 0, q_it = 0, g = 0, units_done = 0;
            bool ok = true, issued = false;
            // next ring sub-tile (in the producer's order); returns its shared-memory address or 0
            auto next_tile = [&]() -> uint32_t {
                const uint32_t st = it % kSlots;
                if (!mbar_wait(bar(kFull + st), (it / kSlots) & 1, abort)) return 0;
                tc_fence_after();
                return base + kSmemRing + st * kTileBytes;
            };
            auto release_tile = [&]() {
                umma_commit(bar(kEmpty + it % kSlots));
                ++it;
            };
            // O (+)= P V for one step (A = P from tensor memory, B = V sub-tiles, MN-major)
            auto pv = [&](int32_t jj, uint32_t gg, int32_t first) -> bool {
                if (!mbar_wait(bar(kPFull), gg & 1, abort)) return false;
                if (jj == first && units_done > 0 && !mbar_wait(bar(kOFree), (units_done - 1) & 1, abort))
                    return false;
                tc_fence_after();
                for (int h = 0; h < 2; ++h) {
                    const uint32_t sV = next_tile();
                    if (!sV) return false;
#pragma unroll
                    for (int k = 0; k < kSubN / 16; ++k) {
                        const uint64_t bdesc = smem_desc_sw128(sV + k * 2048u, kHalfBytes, 1024);
                        umma_ts(tmem + kColO, tmem + kColP + (h * 8 + k) * 8u, bdesc, idesc_pv,
                                (jj > first || h > 0 || k > 0) ? 1u : 0u);
                    }
                    release_tile();
                }
                umma_commit(bar(kPFree));
                return true;
            };
            for (int32_t w = blockIdx.x; ok && w < n_items; w += gridDim.x) {
                const int32_t part = w % n_split;
                const int32_t s0 = part * n_steps / n_split, s1 = (part + 1) * n_steps / n_split;
                if (!mbar_wait(bar(kQFull), q_it & 1, abort)) { ok = false; break; }
                ++q_it;
                for (int32_t j = s0; j < s1; ++j, ++g) {
                    // S(j) = Q K(2j..2j+1)^T once every softmax thread has loaded S(j-1)
                    if (g > 0 && !mbar_wait(bar(kSFree), (g - 1) & 1, abort)) { ok = false; break; }
                    for (int h = 0; h < 2; ++h) {
                        const uint32_t sK = next_tile();
                        if (!sK) { ok = false; break; }
                        issued = true;
#pragma unroll
                        for (int k = 0; k < kD / 16; ++k) {
                            const uint32_t off = (k >> 2) * kHalfBytes + (k & 3) * 32u;
                            umma_ss(tmem + kColS + h * kSubN, smem_desc_sw128(base + kSmemQ + off, 16, 1024),
                                    smem_desc_sw128(sK + off, 16, 1024), idesc_qk, k > 0 ? 1u : 0u);
                        }
                        release_tile();
                    }
                    if (!ok) break;
                    umma_commit(bar(kSFull));
                    if (j == s1 - 1) umma_commit(bar(kQEmpty));
                    if (j > s0 && !pv(j - 1, g - 1, s0)) { ok = false; break; }
                }
                if (!ok || !pv(s1 - 1, g - 1, s0)) { ok = false; break; }
                ++units_done;
            }
            if (*abort && issued) {
                umma_commit(bar(kDrain));
                mbar_wait_drain(bar(kDrain), 0);
            }
        }
    } else {
        // ---------------- softmax / correction / epilogue: 4 warpgroups ----------------
        // Waits are warp-uniform (every lane polls, then __all_sync) so that the .sync.aligned
        // tensor-memory accesses below always run on a converged warp, also when a wait gives up.
        auto wwait = [&](uint32_t b_, uint32_t par_) -> bool {
            return __all_sync(0xffffffffu, mbar_wait(b_, par_, abort));
        };
        const int wg = warp >> 2;                                 // 0..3
        const int r = ((warp & 3) << 5) | (int)lane;              // row in the tile = TMEM lane
        const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
        const uint32_t tS = tmem + lane_off + kColS + wg * 64u;
        const uint32_t tP = tmem + lane_off + kColP + wg * 32u;
        const uint32_t tO = tmem + lane_off + kColO + wg * 32u;
        float* xch = reinterpret_cast<float*>(gbase + kSmemX);    // [buf][wg][row]
        const float c = p.scale_log2;
        const float2 c2 = make_float2(c, c);
        uint32_t s_it = 0, x_it = 0, units_done = 0;
        bool ok = true;
        // row data exchange among the four warps (one per warpgroup, same sub-partition) that hold
        // the same 32 rows; returns the four values of this row
        const uint32_t xbar = bar(kXchg + (warp & 3));
        auto exchange = [&](float v, float* o4) -> bool {
            float* xb = xch + (x_it & 1) * 512;
            xb[wg * 128 + r] = v;
            mbar_arrive(xbar);
            if (!wwait(xbar, x_it & 1)) return false;
            ++x_it;
#pragma unroll
            for (int k = 0; k < 4; ++k) o4[k] = xb[k * 128 + r];
            return true;
        };
        for (int32_t w = blockIdx.x; ok && w < (kSplit ? sched[1] : n_items); w += gridDim.x) {
            const int32_t ns = kSplit ? sched[0] : 1;
            int32_t b, head, row0, m_b;
            decode_unit(p, w / ns, b, head, row0, m_b);
            const int32_t s0 = (w % ns) * n_steps / ns, s1 = (w % ns + 1) * n_steps / ns;
            const bool live = row0 + r < m_b;
            // the output row and stream of this thread, loaded now (kept in shared memory: the step
            // loop has no register to spare) so that the epilogue does not wait on a global load
            int32_t* orow_slot = reinterpret_cast<int32_t*>(gbase + kSmemRowIdx) + threadIdx.x;
            orow_slot[0] = live ? __ldg(p.s[b].idx + row0 + r) : -1;
            orow_slot[kSoftmaxThreads] = b;
            float m_run = -INFINITY, l_run = 0.f;
            for (int32_t j = s0; j < s1; ++j, ++s_it) {
                if (!wwait(bar(kSFull), s_it & 1)) { ok = false; break; }
                tc_fence_after();
                uint32_t s[64];
                FXR_TMEM_LD64(tS, s);
                tc_fence_before();
                mbar_arrive(bar(kSFree));                         // the next QK may overwrite S
                const int32_t kv_left = p.n_tokens - j * kStepN - wg * 64;
                if (kv_left < 64) {
#pragma unroll
                    for (int cc = 0; cc < 64; ++cc)
                        if (cc >= kv_left) s[cc] = __float_as_uint(-INFINITY);
                }
                float mp[8];
#pragma unroll
                for (int k = 0; k < 8; ++k) mp[k] = fmaxf(__uint_as_float(s[2 * k]), __uint_as_float(s[2 * k + 1]));
#pragma unroll
                for (int i = 1; i < 4; ++i)
#pragma unroll
                    for (int k = 0; k < 8; ++k)
                        mp[k] = max3f(mp[k], __uint_as_float(s[16 * i + 2 * k]), __uint_as_float(s[16 * i + 2 * k + 1]));
                float pm4[4];
                if (!exchange(max3f(max3f(mp[0], mp[1], mp[2]), max3f(mp[3], mp[4], mp[5]), fmaxf(mp[6], mp[7])), pm4)) {
                    ok = false;
                    break;
                }
                const float mx = fmaxf(fmaxf(pm4[0], pm4[1]), fmaxf(pm4[2], pm4[3])) * c;
                float alpha = 1.f;
                bool rescale = false;
                if (j == s0) {
                    m_run = mx;
                } else if (__any_sync(0xffffffffu, live && mx > m_run + kRescaleThreshold)) {
                    // warp-uniform decision over the rows that will be stored: the padding rows of
                    // the last tile (stale compact-Q rows) must not change how live rows round
                    const float m_new = fmaxf(m_run, mx);
                    alpha = ex2_approx(m_run - m_new);
                    l_run *= alpha;
                    m_run = m_new;
                    rescale = true;
                }
                const float2 nm2 = make_float2(-m_run, -m_run);
                float2 acc[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                                 make_float2(0.f, 0.f)};
                // P overwrites the score registers pairwise (pk[k] from s[2k], s[2k+1]).
                uint32_t* pk = s;
#pragma unroll
                for (int k = 0; k < 32; ++k) {
                    const float2 x = ffma2(make_float2(__uint_as_float(s[2 * k]), __uint_as_float(s[2 * k + 1])),
                                           c2, nm2);
                    float2 e;
                    if ((k % kPolyPeriod) < kPolyCount) {
                        e = ex2_poly2(x);
                    } else {
                        e = make_float2(ex2_approx(x.x), ex2_approx(x.y));
                    }
                    acc[k & 3] = fadd2(acc[k & 3], e);
                    pk[k] = StoreT<T>::pack2(e.x, e.y);
                }
                const float2 a01 = fadd2(fadd2(acc[0], acc[1]), fadd2(acc[2], acc[3]));
                l_run += a01.x + a01.y;
                // P and O may be touched once the previous step's PV has finished
                if (s_it > 0 && !wwait(bar(kPFree), (s_it - 1) & 1)) { ok = false; break; }
                tc_fence_after();
                if (rescale) {
#pragma unroll 1
                    for (int h2 = 0; h2 < 2; ++h2) {
                        uint32_t o[16];
                        FXR_TMEM_LD16(tO + h2 * 16u, o);
#pragma unroll
                        for (int k = 0; k < 16; ++k) o[k] = __float_as_uint(__uint_as_float(o[k]) * alpha);
                        FXR_TMEM_ST16(tO + h2 * 16u, o);
                    }
                }
                FXR_TMEM_ST32(tP, pk);
                tc_fence_before();
                mbar_arrive(bar(kPFull));
            }
            if (!ok) break;
            // epilogue: the row sums are exchanged while the last PV runs; O is final once it is done
            float l4[4];
            if (!exchange(l_run, l4)) { ok = false; break; }
            float l_tot = (l4[0] + l4[1]) + (l4[2] + l4[3]);
            if (!wwait(bar(kPFree), (s_it - 1) & 1)) { ok = false; break; }
            tc_fence_after();
            uint32_t o[32];
            FXR_TMEM_LD32(tO, o);
            tc_fence_before();
            mbar_arrive(bar(kOFree));
            ++units_done;
            const int32_t n_split = kSplit ? sched[0] : 1;
            if (n_split > 1) {
                // partial of this part: O (32 columns of row r), row maximum and sum (unit and part
                // recomputed from the item, not kept live across the step loop)
                const int32_t u = w / n_split;
                float* slot = p.split_scratch + (size_t)w * kSplitSlotFloats;
                float4* od = reinterpret_cast<float4*>(slot + r * kD + wg * 32);
#pragma unroll
                for (int k = 0; k < 8; ++k)
                    od[k] = make_float4(__uint_as_float(o[4 * k]), __uint_as_float(o[4 * k + 1]),
                                        __uint_as_float(o[4 * k + 2]), __uint_as_float(o[4 * k + 3]));
                slot[kBM * kD + wg * kBM + r] = m_run;
                slot[kBM * kD + 4 * kBM + wg * kBM + r] = l_tot;
                __threadfence();
                __syncwarp();
                int32_t prev = 0;
                if (lane == 0) prev = atomicAdd(p.split_cnt + u * kSplitPortions + warp, 1);
                prev = __shfl_sync(0xffffffffu, prev, 0);
                if (prev == n_split - 1) {   // the last part to arrive combines this portion
                    if (lane == 0) p.split_cnt[u * kSplitPortions + warp] = 0;   // for the next launch
                    __threadfence();
                    // a live row with a negative index is out of bounds (flagged there), not padding
                    const int32_t orow = live ? (*orow_slot < 0 ? INT32_MAX : *orow_slot) : -1;
                    split_combine_store<T>(p, static_cast<T*>(stream_out(p, orow_slot[kSoftmaxThreads])),
                                           p.split_scratch + (size_t)u * n_split * kSplitSlotFloats,
                                           n_split, r, wg, orow, head);
                }
                continue;
            }
            if (live) {
                const int32_t i = *orow_slot;
                if (i >= 0 && i < p.n_tokens) {
                    const float inv = 1.0f / l_tot;
                    const int64_t off = (int64_t)i * p.ld_out + (int64_t)head * kD + wg * 32;
                    uint4 v[4];
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        v[k].x = StoreT<T>::pack2(__uint_as_float(o[8 * k + 0]) * inv, __uint_as_float(o[8 * k + 1]) * inv);
                        v[k].y = StoreT<T>::pack2(__uint_as_float(o[8 * k + 2]) * inv, __uint_as_float(o[8 * k + 3]) * inv);
                        v[k].z = StoreT<T>::pack2(__uint_as_float(o[8 * k + 4]) * inv, __uint_as_float(o[8 * k + 5]) * inv);
                        v[k].w = StoreT<T>::pack2(__uint_as_float(o[8 * k + 6]) * inv, __uint_as_float(o[8 * k + 7]) * inv);
                    }
                    uint4* dst = reinterpret_cast<uint4*>(static_cast<T*>(stream_out(p, orow_slot[kSoftmaxThreads])) + off);
#pragma unroll
                    for (int k = 0; k < 4; ++k) dst[k] = v[k];
                } else {
                    atomicOr(&g_error_word, kErrBounds);
                }
            }
        }
    }

    __syncwarp();  // role warps ran their loops on one lane; reconverge before the CTA barrier
    tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

}  // namespace attn
}  // namespace fxr
