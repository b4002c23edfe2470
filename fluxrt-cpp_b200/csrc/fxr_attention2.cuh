// fxr_attention2.cuh — active-query flash attention with two query tiles per CTA (sm_100a).
//
// Work unit: two 128-row tiles of compact queries of one head (256 rows) against all N keys of
// that head, in steps of 128 keys. Persistent CTAs walk the units round-robin; M is read on the
// device. When whole units would leave SMs idle (fewer units than SMs, or a last wave that is
// mostly empty), the kSplit instantiation runs a stream-K schedule instead: the (unit, key step)
// iterations are cut into one contiguous range per CTA, and units cut between CTAs are combined
// through L2 (choose_schedule below). The two tiles run as two dependency chains that the tensor
// core interleaves, so that the softmax of one tile overlaps the products of the other:
//   tile i, step j:  S_i = Q_i K_j^T  ->  softmax_i(j): P_i  ->  O_i += P_i V_j  ->  S_i(j+1) ...
// Warp roles (384 threads, three warpgroups):
//   warps 0-3   softmax of tile 0: one thread per query row (TMEM lane), all 128 scores of a step
//   warps 4-7   softmax of tile 1
//   warp 8      TMA producer: Q_0, Q_1 and a 5-slot ring of 128-key K and V tiles in the tensor
//               core's consumption order K_0 V_0 K_1 V_1 ... (128-byte swizzle)
//   warp 9      TMEM allocator and the single MMA-issuing thread
//   warp 10     after the CTA's last item: restore of the cache rows of mask==1 tokens, head by
//               head, once no CTA reads that head any more
//   warp 11     idle (it completes the third warpgroup)
// Tensor memory (512 columns): S_0 [0,128), S_1 [128,256) fp32 scores; O_0 [256,384), O_1 [384,512)
// fp32 outputs. The 16-bit probabilities P_i of a step are written over the first 64 columns of
// S_i (key pairs packed per column) and read from there by the PV product (A operand in tensor
// memory). Products with different accumulators are not ordered by the hardware, so the MMA thread
// issues S_i(j+1) only once O_i += P_i(j) V_j has completed (its own commit barrier); meanwhile the
// tensor core works on the other tile's products.
// Each softmax thread owns a whole row: the row maximum needs no exchange between warps. Softmax in
// the exp2 domain with lazy rescaling (threshold 2^8; the decision is warp-uniform over live rows so
// that padding rows of the last tile, stale compact-Q rows, cannot change a stored bit); a share of
// the exponentials runs as a polynomial on the FMA pipe (ex2_poly2). When a row maximum grows, the
// softmax thread rescales its own O row (the previous PV of its tile has completed by then: the
// scores it just read were issued after it). Epilogue: O / l stored straight to out[idx[m]]
// (the reference's scatter, fused).
// Every mbarrier wait is bounded (2 s); on timeout the kernel sets the device error word, drains its
// outstanding copies and products, frees its tensor memory and returns.
// Replaces attention_fwd (attention_kernels.cu:85-173) and scatter_tokens
// (gather_scatter_kernels.cu:46-72) on this path.
#pragma once

#include "fxr_attention.cuh"

namespace fxr {
namespace attn2 {

using attn::Maps;
using attn::Params;

constexpr int kBM = 128;                        // query rows per tile
constexpr int kRows = 2 * kBM;                  // query rows per work unit
constexpr int kBN = 128;                        // keys per step
constexpr int kD = 128;                         // head dim
constexpr int kSlots = 5;                       // K/V tile ring
constexpr int kSoftmaxWarps = 8;
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;
constexpr int kRestoreWarp = 10;
constexpr int kThreads = 32 * 12;
constexpr uint32_t kSoftmaxThreads = 32 * kSoftmaxWarps;
constexpr uint32_t kHalfBytes = 128 * 128;      // 128 rows x 64 16-bit values (one swizzle span)
constexpr uint32_t kTileBytes = 2 * kHalfBytes; // 128 x 128 16-bit tile
constexpr uint32_t kSmemQ = 0;                  // Q_0, Q_1
constexpr uint32_t kSmemRing = 2 * kTileBytes;
constexpr uint32_t kSmemRowIdx = kSmemRing + kSlots * kTileBytes;   // [softmax thread]
constexpr uint32_t kSmemBar = kSmemRowIdx + kSoftmaxThreads * 4;
constexpr uint32_t kSmemBytes = kSmemBar + 256 + 1024;               // barriers + alignment slack
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0, kColO = 256;      // + tile * 128
// Registers: the softmax warpgroups take more than the launch share, the producer / MMA warpgroup
// less (setmaxnreg). The launch gives the CTA kThreads x (registers per thread) registers; the two
// shares must fit in it, which the host checks against the compiled register count before launch.
constexpr uint32_t kRegsSoftmax = 200;
constexpr uint32_t kRegsOther = 104;            // the producer / MMA loops compile without spills
constexpr uint32_t kRegPool = 2 * 128 * kRegsSoftmax + 128 * kRegsOther;   // 64512 = 384 x 168
constexpr float kRescaleThreshold = 8.0f;       // log2 units
constexpr int kPolyPeriod = 4;                  // the last of every 4 score pairs uses ex2_poly2
                                                // (spread evenly: measured 3 % shorter steps than
                                                // two adjacent pairs of every 8)

enum Bar : uint32_t {
    kQFull = 0,
    kQEmpty,
    kFull,                           // + ring slot: tile landed
    kEmpty = kFull + kSlots,         // + ring slot: tile consumed
    kSFull = kEmpty + kSlots,        // + tile: scores of a step computed
    kPHalf0 = kSFull + 2,            // + tile: probabilities of keys 0-63 stored (and O rescaled)
    kPHalf1 = kPHalf0 + 2,           // + tile: probabilities of keys 64-127 stored
    kPVDone = kPHalf1 + 2,           // + tile: O += P V of a step completed
    kOFree = kPVDone + 2,            // + tile: epilogue read O
    kDrain = kOFree + 2,
    kNumBars,
};
constexpr uint32_t kSlotTmem = kNumBars * 8;
constexpr uint32_t kSlotAbort = kSlotTmem + 4;
constexpr uint32_t kSlotCursor = kSlotAbort + 4;   // [softmax warp] {next, end} of its item walk
static_assert(kSlotCursor % 8 == 0 && kSlotCursor + 8 * kSoftmaxWarps <= 256, "barrier area overflow");
static_assert(kSmemBytes <= 232448, "shared memory budget");

// Stream-K schedule (the kSplit instantiation): CTA c takes the iterations [c * per, (c+1) * per)
// of the (unit, key step) space, unit-major. Its first and last items may cover part of a unit
// only; such a part writes its tiles' unnormalised O rows with their running maxima and sums to
// scratch slots (per CTA two items x two tiles, column chunk-major so that a warp's stores are
// contiguous). Per (unit, softmax warp) an arrival counter elects the part that arrives last; its
// warp combines every part of its 32 rows in key order (the result does not depend on which CTA
// came last) and stores them. A unit cut between CTAs has its last part in the CTA c_last that
// holds its final step; no other cut unit ends there, so c_last indexes its counters.
// Costs in 128-key steps of both tiles (~1.7-2 us each): the fixed cost of an item (Q tiles,
// pipeline ramp, epilogue) and the extra cost of each cut end of a CTA's range (partial write,
// counter, combine through L2). Fitted to measured frames: a 2048^2 frame's 288 units of 132 steps
// run faster as two rounds of whole units (585.6 us) than as stream-K (627.8 us), a 1024^2 frame's
// 96 units of 36 steps faster as stream-K (84.7 -> 79.9 us per frame).
constexpr float kItemOverheadSteps = 2.0f;
constexpr float kCutOverheadSteps = 4.5f;
constexpr int kSlotsPerCta = 4;    // scratch slots (one tile's partial each) a stream-K CTA may use

struct Sched {
    int32_t n_units;
    int32_t n_steps;
    int32_t per;                   // stream-K iterations per CTA; 0: whole units round-robin
};

// The schedule of a launch, the same on every thread of every CTA (a function of M, the grid and
// the scratch only): stream-K when its estimated time (iterations per CTA + item overheads) beats
// whole units (CTA rounds x steps per unit).
__device__ __forceinline__ Sched choose_schedule(int32_t n_units, int32_t n_steps, int32_t grid,
                                                 int32_t slots, bool allow) {
    Sched sc{n_units, n_steps, 0};
    if (!allow || slots < kSlotsPerCta * grid || n_units <= 0) return sc;
    const float whole = (float)((n_units + grid - 1) / grid) * ((float)n_steps + kItemOverheadSteps);
    const int32_t per = (int32_t)(((int64_t)n_units * n_steps + grid - 1) / grid);
    const int32_t items = (per + n_steps - 1) / n_steps + 1;      // at most, counting both cut ends
    const float sk = (float)per + kItemOverheadSteps * (float)items + 2.0f * kCutOverheadSteps;
    if (sk < whole) sc.per = per;
    return sc;
}

// A CTA's walk over its items. Whole units: cur is the unit (stride: the grid). Stream-K: cur is
// the next iteration, end the CTA's last + 1.
struct Cursor {
    int32_t cur, end;
};

__device__ __forceinline__ Cursor first_cursor(const Sched& sc) {
    if (sc.per == 0) return Cursor{(int32_t)blockIdx.x, sc.n_units};
    const int32_t a = (int32_t)blockIdx.x * sc.per;
    return Cursor{a, min(sc.n_units * sc.n_steps, a + sc.per)};
}

// The next item of the walk: unit u and its key steps [s0, s1). False when the CTA is done.
__device__ __forceinline__ bool next_item(const Sched& sc, Cursor& c, int32_t& u, int32_t& s0, int32_t& s1) {
    if (c.cur >= c.end) return false;
    if (sc.per == 0) {
        u = c.cur;
        s0 = 0;
        s1 = sc.n_steps;
        c.cur += gridDim.x;
        return true;
    }
    u = c.cur / sc.n_steps;
    s0 = c.cur - u * sc.n_steps;
    s1 = min(sc.n_steps, s0 + (c.end - c.cur));
    c.cur += s1 - s0;
    return true;
}

// Scratch slot of the part of unit u that CTA c runs, tile t: its first item (slot pair 0) unless
// the unit starts inside the CTA's range after other items (pair 1).
__device__ __forceinline__ size_t part_slot(const Sched& sc, int32_t u, int32_t c, int t) {
    const int32_t c_first = (int32_t)((int64_t)u * sc.n_steps / sc.per);
    const int k = (c == c_first && u * sc.n_steps > c * sc.per) ? 1 : 0;
    return ((size_t)c * 2 + k) * 2 + t;
}

// The last part of unit u combines row r of tile t over every part (CTAs c_first..c_last, in key
// order) and stores it to out_row (nullptr: padding row, or a bad index already flagged).
template <typename T>
__device__ __forceinline__ void combine_store(const float* scratch, const Sched& sc, int32_t u, int t, int r,
                                              T* out_row) {
    const int32_t c0 = (int32_t)((int64_t)u * sc.n_steps / sc.per);
    const int32_t c1 = (int32_t)(((int64_t)(u + 1) * sc.n_steps - 1) / sc.per);
    float m_all = -INFINITY;
    for (int32_t c = c0; c <= c1; ++c)
        m_all = fmaxf(m_all, __ldcg(scratch + part_slot(sc, u, c, t) * attn::kSplitSlotFloats + kBM * kD + r));
    float acc[kD];
#pragma unroll
    for (int k = 0; k < kD; ++k) acc[k] = 0.f;
    float l_tot = 0.f;
    for (int32_t c = c0; c <= c1; ++c) {
        const float* sq = scratch + part_slot(sc, u, c, t) * attn::kSplitSlotFloats;
        const float a = ex2_approx(__ldcg(sq + kBM * kD + r) - m_all);
        l_tot += a * __ldcg(sq + kBM * kD + kBM + r);
        const float4* oq = reinterpret_cast<const float4*>(sq);
#pragma unroll
        for (int q = 0; q < kD / 4; ++q) {
            const float4 x = __ldcg(oq + q * kBM + r);
            acc[4 * q] += a * x.x;
            acc[4 * q + 1] += a * x.y;
            acc[4 * q + 2] += a * x.z;
            acc[4 * q + 3] += a * x.w;
        }
    }
    if (out_row == nullptr) return;
    const float inv = 1.0f / l_tot;
    uint4* dst = reinterpret_cast<uint4*>(out_row);
#pragma unroll
    for (int k = 0; k < kD / 8; ++k) {
        uint4 v;
        v.x = StoreT<T>::pack2(acc[8 * k + 0] * inv, acc[8 * k + 1] * inv);
        v.y = StoreT<T>::pack2(acc[8 * k + 2] * inv, acc[8 * k + 3] * inv);
        v.z = StoreT<T>::pack2(acc[8 * k + 4] * inv, acc[8 * k + 5] * inv);
        v.w = StoreT<T>::pack2(acc[8 * k + 6] * inv, acc[8 * k + 7] * inv);
        dst[k] = v;
    }
}

// End of an item that covers part of a cut unit (stream-K schedule): the part's O rows, maxima and
// sums go to its scratch slot, then O is released to the MMA thread (kOFree); the warp whose arrival
// completes the unit combines every part of its 32 rows and stores them. Kept out of line: inlined,
// this rarely run code changed the code of the step loop around it enough to slow whole-unit
// schedules of the same kernel by up to 20 % (measured), which a call does not.
template <typename T>
__device__ __noinline__ void cut_unit_epilogue(float* scratch, int32_t* split_cnt, int32_t n_tokens,
                                               int64_t ld_out, T* out, const Sched sc, int32_t u,
                                               int32_t head, int t, int r, int warp, uint32_t tO,
                                               float m_run, float l_run, uint32_t ofree_bar, bool live,
                                               int32_t orow) {
    const uint32_t lane = lane_id();
    float* slot = scratch + part_slot(sc, u, (int32_t)blockIdx.x, t) * attn::kSplitSlotFloats;
    float4* od = reinterpret_cast<float4*>(slot);
#pragma unroll 1
    for (int h = 0; h < 4; ++h) {
        uint32_t o[32];
        FXR_TMEM_LD32(tO + h * 32u, o);
#pragma unroll
        for (int k = 0; k < 8; ++k)
            od[(h * 8 + k) * kBM + r] = make_float4(__uint_as_float(o[4 * k]), __uint_as_float(o[4 * k + 1]),
                                                    __uint_as_float(o[4 * k + 2]), __uint_as_float(o[4 * k + 3]));
    }
    slot[kBM * kD + r] = m_run;
    slot[kBM * kD + kBM + r] = l_run;
    tc_fence_before();
    mbar_arrive(ofree_bar);
    __threadfence();
    __syncwarp();
    const int32_t c_first = (int32_t)((int64_t)u * sc.n_steps / sc.per);
    const int32_t c_last = (int32_t)(((int64_t)(u + 1) * sc.n_steps - 1) / sc.per);
    int32_t* cnt = split_cnt + c_last * attn::kSplitPortions + warp;
    int32_t prev = 0;
    if (lane == 0) prev = atomicAdd(cnt, 1);
    prev = __shfl_sync(0xffffffffu, prev, 0);
    if (prev != c_last - c_first) return;
    // the last part to arrive combines these 32 rows
    if (lane == 0) *cnt = 0;      // for the next launch
    __threadfence();
    const bool store = live && orow >= 0 && orow < n_tokens;
    if (live && !store) atomicOr(&g_error_word, kErrBounds);
    combine_store<T>(scratch, sc, u, t, r, store ? out + (int64_t)orow * ld_out + (int64_t)head * kD : nullptr);
}

// Work unit u of the launch -> stream b, head and first compact row of tile 0. Units are numbered
// stream after stream, (row pair, head) within a stream as pair + head * pairs, so that the CTAs
// running at the same time share each head's keys in L2.
__device__ __forceinline__ void decode_pair_unit(const Params& p, int32_t u, int32_t& b, int32_t& head,
                                            int32_t& row0, int32_t& m_b) {
    b = -1;
#pragma unroll
    for (int k = 0; k < kMaxBatch; ++k) {
        if (b < 0 && k < p.n_streams) {
            const int32_t mk = *p.s[k].count;
            const int32_t units = (mk + kRows - 1) / kRows * p.n_heads;
            if (u < units || k + 1 == p.n_streams) {
                b = k;
                m_b = mk;
            } else {
                u -= units;
            }
        }
    }
    const int32_t pairs = (m_b + kRows - 1) / kRows;
    head = pairs > 0 ? u / pairs : 0;
    row0 = (u - head * pairs) * kRows;
}

// Fused restore of the cache rows of mask==1 tokens, head by head: the saved K and V slices of head
// `head` of every listed row are copied back into the cache by one warp (lanes 0-15 the K slice,
// 16-31 the V slice of a row), 32 rows' indices fetched at a time.
__device__ __forceinline__ void restore_head_rows(const attn::RestoreRef rr, int64_t ld_cache_bytes, int32_t row_vec,
                                                  int32_t n_tokens, int32_t head) {
    const uint32_t lane = lane_id();
    const int32_t n1 = __ldcg(rr.count);
    const int32_t half = (int32_t)(lane >> 4), l = (int32_t)(lane & 15);
    for (int32_t e0 = 0; e0 < n1; e0 += 32) {
        const int32_t e = e0 + (int32_t)lane;
        int32_t m = -1, i = -1;
        if (e < n1) {
            m = __ldcg(rr.rows + e);
            i = __ldcg(rr.idx + m);
        }
        for (int q = 0; q < 32; ++q) {
            const int32_t mq = __shfl_sync(0xffffffffu, m, q), iq = __shfl_sync(0xffffffffu, i, q);
            if (mq < 0) break;
            if (iq < 0 || iq >= n_tokens) continue;   // flagged by the gather, which skipped the row
            const uint4 v = rr.save[(int64_t)mq * 2 * row_vec + half * row_vec + head * (kD / 8) + l];
            char* dst = (half ? rr.cache_v : rr.cache_k) + (int64_t)iq * ld_cache_bytes + (int64_t)head * kD * 2 + l * 16;
            *reinterpret_cast<uint4*>(dst) = v;
        }
    }
}

// Whether any stream of the launch lists mask==1 rows to restore (read once the compaction is over).
__device__ __forceinline__ bool restore_pending(const attn::Params& p) {
    if (p.s[0].restore_rows == nullptr) return false;
    bool any = false;
#pragma unroll
    for (int k = 0; k < kMaxBatch; ++k)
        if (k < p.n_streams) any = any || __ldcg(attn::stream_restore(p, k).count) > 0;
    return any;
}

// Restore of mask==1 cache rows by warp 10 after its CTA has finished all its items: it adds the key
// steps of each of the CTA's items to that head's counter; the arrival that completes a head (every
// item of the head done in every CTA, so no CTA reads its K / V any more) restores that head's rows.
// Runs only for launches that list such rows. Out of line: the other roles' code is the same with
// and without it.
__device__ __noinline__ void restore_tail(const attn::Params& p, const Sched sc, int32_t n_steps) {
    const uint32_t lane = lane_id();
    Cursor cur = first_cursor(sc);
    int32_t u, s0, s1;
    while (next_item(sc, cur, u, s0, s1)) {
        int32_t b, head, row0, m_b;
        decode_pair_unit(p, u, b, head, row0, m_b);
        const attn::RestoreRef rr = attn::stream_restore(p, b);
        int32_t prev = 0;
        if (lane == 0) prev = atom_add_acq_rel_gpu(rr.head_done + head, s1 - s0);
        prev = __shfl_sync(0xffffffffu, prev, 0);
        if (prev + (s1 - s0) == (m_b + kRows - 1) / kRows * n_steps)
            restore_head_rows(rr, p.ld_cache_bytes, p.row_vec, p.n_tokens, head);
    }
}

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
        for (int t = 0; t < 2; ++t) {
            mbar_init(bar(kSFull + t), 1);
            mbar_init(bar(kPHalf0 + t), kBM);
            mbar_init(bar(kPHalf1 + t), kBM);
            mbar_init(bar(kPVDone + t), 1);
            mbar_init(bar(kOFree + t), kBM);
        }
        mbar_init(bar(kDrain), 1);
        *abort = 0;
        fence_mbar_init();
    }
    if (warp == kProducerWarp && lane == 0) {
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
        if (b < p.n_streams) n_units += (*p.s[b].count + kRows - 1) / kRows * p.n_heads;
    const int32_t n_steps = (p.n_tokens + kBN - 1) / kBN;
    const Sched sc = choose_schedule(n_units, n_steps, (int32_t)gridDim.x, p.split_slots, kSplit);
    bool restore = false;   // warp 10: this launch restores mask==1 rows at the end

    if (warp >= kSoftmaxWarps) {
      // warpgroup 2: producer, MMA issuer and two idle warps
      asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsOther));
      if (warp == kProducerWarp) {
        if (lane == 0) {
            // ---------------- TMA producer ----------------
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
            Cursor cur = first_cursor(sc);
            int32_t u, s0, s1;
            while (ok && next_item(sc, cur, u, s0, s1)) {
                int32_t b, head, row0, m_b;
                decode_pair_unit(p, u, b, head, row0, m_b);
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
                if (q_it > 0 && !mbar_wait(bar(kQEmpty), (q_it - 1) & 1, abort)) { ok = false; break; }
                mbar_arrive_expect_tx(bar(kQFull), 2 * kTileBytes);
                for (int t = 0; t < 2; ++t) {
                    const uint32_t dq = base + kSmemQ + t * kTileBytes;
                    tma_load_2d(dq, tmQ, bar(kQFull), head * kD, row0 + t * kBM);
                    tma_load_2d(dq + kHalfBytes, tmQ, bar(kQFull), head * kD + 64, row0 + t * kBM);
                }
                ++q_it;
                ok = load(tmK, head, s0 * kBN);
                for (int32_t j = s0; ok && j < s1; ++j) {
                    ok = load(tmV, head, j * kBN);
                    if (ok && j + 1 < s1) ok = load(tmK, head, (j + 1) * kBN);
                }
            }
            if (*abort) {
                if (q_it > 0) attn::mbar_wait_drain(bar(kQFull), (q_it - 1) & 1);
                for (uint32_t t = (it > kSlots ? it - kSlots : 0); t < it; ++t)
                    attn::mbar_wait_drain(bar(kFull + t % kSlots), (t / kSlots) & 1);
            }
        }
      } else if (warp == kMmaWarp) {
        if (lane == 0) {
            // ---------------- MMA issuer ----------------
            constexpr uint32_t fmt = StoreT<T>::kUmmaFormat;
            constexpr uint32_t idesc_qk = make_idesc_f16(fmt, 0, kBM, kBN);
            constexpr uint32_t idesc_pv = make_idesc_f16(fmt, 1, kBM, kD);
            uint32_t acq = 0, rel = 0, q_it = 0, g = 0, units_done = 0;
            bool ok = true, issued = false;
            // the issuer reacts to every phase by spinning (try_wait may keep it suspended for
            // hundreds of cycles after a phase completes, which the tensor core would sit out)
            auto wait = [&](uint32_t b_, uint32_t par_) { return mbar_wait_spin(b_, par_, abort); };
            // ring tiles are acquired and released in the producer's order (two counters: a V tile
            // and the next K tile are held at the same time)
            auto acquire = [&]() -> uint32_t {
                const uint32_t st = acq % kSlots;
                if (!wait(bar(kFull + st), (acq / kSlots) & 1)) return 0;
                ++acq;
                return base + kSmemRing + st * kTileBytes;
            };
            auto release = [&]() {
                umma_commit(bar(kEmpty + rel % kSlots));
                ++rel;
            };
            // Shared-memory descriptors: the start-address field is the low part of the descriptor,
            // so the K slices of a tile are the base descriptor plus (byte offset >> 4).
            const uint64_t dq[2] = {smem_desc_sw128(base + kSmemQ, 16, 1024),
                                    smem_desc_sw128(base + kSmemQ + kTileBytes, 16, 1024)};
            // S_t = Q_t K^T (K-major A and B in shared memory)
            auto qk = [&](int t, uint32_t sK) {
                const uint64_t dk = smem_desc_sw128(sK, 16, 1024);
                const uint32_t d = tmem + kColS + t * 128u;
#pragma unroll
                for (int k = 0; k < kD / 16; ++k) {
                    const uint64_t off = ((k >> 2) * kHalfBytes + (k & 3) * 32u) >> 4;
                    umma_ss(d, dq[t] + off, dk + off, idesc_qk, k > 0 ? 1u : 0u);
                }
                umma_commit(bar(kSFull + t));
            };
            // O_t (+)= P_t V over keys [64h, 64h+64) (P in tensor memory over the first 64 columns of
            // S_t, V MN-major)
            auto pv = [&](int t, uint32_t sV, int h, bool acc) {
                const uint64_t dv = smem_desc_sw128(sV, kHalfBytes, 1024);
                const uint32_t d = tmem + kColO + t * 128u, a = tmem + kColS + t * 128u;
#pragma unroll
                for (int k = 4 * h; k < 4 * h + 4; ++k)
                    umma_ts(d, a + k * 8u, dv + (uint64_t)((k * 2048u) >> 4), idesc_pv, (acc || k > 0) ? 1u : 0u);
            };
            // Per step the tensor core alternates between the tiles: O_0 += P_0 V_j (in two halves of
            // keys, the first as soon as its probabilities are stored), S_0(j+1), O_1 += P_1 V_j,
            // S_1(j+1); the softmax of one tile runs while the other tile's products execute.
            Cursor cur = first_cursor(sc);
            int32_t u, s0, s1;
            while (ok && next_item(sc, cur, u, s0, s1)) {
                const int32_t nst = s1 - s0;
                if (!wait(bar(kQFull), q_it & 1)) { ok = false; break; }
                ++q_it;
                // the previous unit's last products read P_t from S_t: S_t may be rewritten once
                // they have completed
                if (g > 0 && (!wait(bar(kPVDone + 0), (g - 1) & 1) || !wait(bar(kPVDone + 1), (g - 1) & 1))) {
                    ok = false;
                    break;
                }
                uint32_t sK = acquire();
                if (!sK) { ok = false; break; }
                tc_fence_after();
                issued = true;
                qk(0, sK);
                qk(1, sK);
                release();
                if (nst == 1) umma_commit(bar(kQEmpty));
                for (int32_t j = 0; j < nst; ++j, ++g) {
                    const uint32_t sV = acquire();
                    if (!sV) { ok = false; break; }
                    const bool more = j + 1 < nst;
                    for (int t = 0; t < 2; ++t) {
                        if (!wait(bar(kPHalf0 + t), g & 1)) { ok = false; break; }
                        if (j == 0 && units_done > 0 && !wait(bar(kOFree + t), (units_done - 1) & 1)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        pv(t, sV, 0, j > 0);
                        if (!wait(bar(kPHalf1 + t), g & 1)) { ok = false; break; }
                        tc_fence_after();
                        pv(t, sV, 1, true);
                        umma_commit(bar(kPVDone + t));
                        if (t == 1) release();                        // V_j
                        if (more) {
                            if (t == 0) {
                                sK = acquire();
                                if (!sK) { ok = false; break; }
                            }
                            // S_t(j+1) overwrites P_t(j): wait until O_t += P_t(j) V_j has completed
                            if (!wait(bar(kPVDone + t), g & 1)) { ok = false; break; }
                            tc_fence_after();
                            qk(t, sK);
                            if (t == 1) {
                                release();                            // K_{j+1}
                                if (j + 2 == nst) umma_commit(bar(kQEmpty));
                            }
                        }
                    }
                    if (!ok) break;
                }
                if (!ok) break;
                ++units_done;
            }
            if (*abort && issued) {
                umma_commit(bar(kDrain));
                attn::mbar_wait_drain(bar(kDrain), 0);
            }
        }
      } else if (warp == kRestoreWarp) {
        restore = restore_pending(p);   // after the compaction (pdl_wait above); used at the end
      }
    } else {
        asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsSoftmax));
        // ---------------- softmax / epilogue: one thread per query row ----------------
        // Waits are warp-uniform (every lane polls, then __all_sync) so that the .sync.aligned
        // tensor-memory accesses below always run on a converged warp, also when a wait gives up.
        auto wwait = [&](uint32_t b_, uint32_t par_) -> bool {
            return __all_sync(0xffffffffu, mbar_wait(b_, par_, abort));
        };
        const int t = warp >> 2;                                  // query tile 0 / 1
        const int r = ((warp & 3) << 5) | (int)lane;              // row in the tile = TMEM lane
        const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
        const uint32_t tS = tmem + lane_off + kColS + t * 128u;   // scores; P over its first 64 cols
        const uint32_t tO = tmem + lane_off + kColO + t * 128u;
        const float c = p.scale_log2;
        const float2 c2 = make_float2(c, c);
        uint32_t s_it = 0, units_done = 0;
        bool ok = true;
        int32_t* orow_slot = reinterpret_cast<int32_t*>(gbase + kSmemRowIdx) + threadIdx.x;
        // The walk's cursor is kept in shared memory (a slot per warp, written by every lane with
        // the same value): across the step loop only its countdown stays in registers.
        volatile int32_t* wcur = reinterpret_cast<volatile int32_t*>(gbase + kSmemBar + kSlotCursor) + 2 * warp;
        {
            const Cursor c0 = first_cursor(sc);
            wcur[0] = c0.cur;
            wcur[1] = c0.end;
        }
        while (ok) {
            int32_t u, s0, s1;
            {
                Cursor cc{wcur[0], wcur[1]};
                if (!next_item(sc, cc, u, s0, s1)) break;
                wcur[0] = cc.cur;
            }
            int32_t b, head, row0, m_b;
            decode_pair_unit(p, u, b, head, row0, m_b);
            const int32_t row = row0 + t * kBM + r;
            const bool live = row < m_b;
            // the output row and stream of this thread, loaded now (kept in shared memory: the step
            // loop has no register to spare) so that the epilogue does not wait on a global load
            orow_slot[0] = live ? __ldg(p.s[b].idx + row) : -1;
            float m_run = -INFINITY, l_run = 0.f;
            for (int32_t j = s0; j < s1; ++j, ++s_it) {
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
                float mp[8];
#pragma unroll
                for (int k = 0; k < 8; ++k) mp[k] = fmaxf(__uint_as_float(s[2 * k]), __uint_as_float(s[2 * k + 1]));
#pragma unroll
                for (int i = 1; i < 8; ++i)
#pragma unroll
                    for (int k = 0; k < 8; ++k)
                        mp[k] = attn::max3f(mp[k], __uint_as_float(s[16 * i + 2 * k]),
                                            __uint_as_float(s[16 * i + 2 * k + 1]));
                const float mx = attn::max3f(attn::max3f(mp[0], mp[1], mp[2]), attn::max3f(mp[3], mp[4], mp[5]),
                                             fmaxf(mp[6], mp[7])) * c;
                float alpha = 1.f;
                bool rescale = false;
                if (j == s0) {
                    m_run = mx;
                } else if (__any_sync(0xffffffffu, live && mx > m_run + kRescaleThreshold)) {
                    const float m_new = fmaxf(m_run, mx);
                    alpha = ex2_approx(m_run - m_new);
                    l_run *= alpha;
                    m_run = m_new;
                    rescale = true;
                }
                if (rescale) {
                    // O_t has no product in flight: S_t(j) was issued after O_t += P_t(j-1) V completed
#pragma unroll 1
                    for (int h = 0; h < 4; ++h) {
                        uint32_t o[32];
                        FXR_TMEM_LD32(tO + h * 32u, o);
#pragma unroll
                        for (int k = 0; k < 32; ++k) o[k] = __float_as_uint(__uint_as_float(o[k]) * alpha);
                        FXR_TMEM_ST32(tO + h * 32u, o);
                    }
                }
                const float2 nm2 = make_float2(-m_run, -m_run);
                float2 acc[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                                 make_float2(0.f, 0.f)};
                // P overwrites the score registers pairwise (pk[k] from s[2k], s[2k+1]), in two
                // halves of 64 keys: the product of the first half starts while the second is computed
                uint32_t* pk = s;
#pragma unroll
                for (int hh = 0; hh < 2; ++hh) {
#pragma unroll
                    for (int k = 32 * hh; k < 32 * hh + 32; ++k) {
                        const float2 x = attn::ffma2(make_float2(__uint_as_float(s[2 * k]), __uint_as_float(s[2 * k + 1])),
                                                     c2, nm2);
                        float2 e;
                        if ((k % kPolyPeriod) == kPolyPeriod - 1) {
                            e = attn::ex2_poly2(x);
                        } else {
                            e = make_float2(ex2_approx(x.x), ex2_approx(x.y));
                        }
                        acc[k & 3] = attn::fadd2(acc[k & 3], e);
                        pk[k] = StoreT<T>::pack2(e.x, e.y);
                    }
                    FXR_TMEM_ST32(tS + 32u * hh, (pk + 32 * hh));
                    tc_fence_before();
                    mbar_arrive(bar((hh == 0 ? kPHalf0 : kPHalf1) + t));
                }
                const float2 a01 = attn::fadd2(attn::fadd2(acc[0], acc[1]), attn::fadd2(acc[2], acc[3]));
                l_run += a01.x + a01.y;
            }
            if (!ok) break;
            // epilogue: O is final once the last product of the tile has completed
            if (!wwait(bar(kPVDone + t), (s_it - 1) & 1)) { ok = false; break; }
            tc_fence_after();
            int32_t steps_done = n_steps;
            if (kSplit && sc.per > 0) {
                // the item again, from the cursor (its end iteration), not kept across the loop
                const int32_t it_end = wcur[0];
                u = (it_end - 1) / n_steps;
                s1 = it_end - u * n_steps;
                s0 = max(0, (int32_t)blockIdx.x * sc.per - u * n_steps);
                steps_done = s1 - s0;
            }
            if (kSplit && sc.per > 0 && (s0 > 0 || s1 < n_steps)) {
                cut_unit_epilogue<T>(p.split_scratch, p.split_cnt, p.n_tokens, p.ld_out,
                                     static_cast<T*>(attn::stream_out(p, b)), sc, u, head, t, r, warp, tO,
                                     m_run, l_run, bar(kOFree + t), live, *orow_slot);
                ++units_done;
                (void)steps_done;
                continue;
            }
            const int32_t i = *orow_slot;
            const bool store = live && i >= 0 && i < p.n_tokens;
            if (live && !store) atomicOr(&g_error_word, kErrBounds);
            const float inv = 1.0f / l_run;
            T* out = static_cast<T*>(attn::stream_out(p, b));
            const int64_t off = (int64_t)(store ? i : 0) * p.ld_out + (int64_t)head * kD;
#pragma unroll 1
            for (int h = 0; h < 4; ++h) {
                uint32_t o[32];
                FXR_TMEM_LD32(tO + h * 32u, o);
                uint4 v[4];
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    v[k].x = StoreT<T>::pack2(__uint_as_float(o[8 * k + 0]) * inv, __uint_as_float(o[8 * k + 1]) * inv);
                    v[k].y = StoreT<T>::pack2(__uint_as_float(o[8 * k + 2]) * inv, __uint_as_float(o[8 * k + 3]) * inv);
                    v[k].z = StoreT<T>::pack2(__uint_as_float(o[8 * k + 4]) * inv, __uint_as_float(o[8 * k + 5]) * inv);
                    v[k].w = StoreT<T>::pack2(__uint_as_float(o[8 * k + 6]) * inv, __uint_as_float(o[8 * k + 7]) * inv);
                }
                if (store) {
                    uint4* dst = reinterpret_cast<uint4*>(out + off + h * 32);
#pragma unroll
                    for (int k = 0; k < 4; ++k) dst[k] = v[k];
                }
            }
            tc_fence_before();
            mbar_arrive(bar(kOFree + t));
            ++units_done;
            (void)steps_done;
        }
    }

    __syncwarp();  // role warps ran their loops on one lane; reconverge before the CTA barrier
    tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
    // ---------------- restore of mask==1 cache rows (whole warp, after every item of the CTA) ----
    if (warp == kRestoreWarp && restore && !*abort) restore_tail(p, sc, n_steps);
}

}  // namespace attn2
}  // namespace fxr
