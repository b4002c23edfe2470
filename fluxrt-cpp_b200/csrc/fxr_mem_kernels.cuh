// fxr_mem_kernels.cuh — HBM-bound kernels of the sparse attention path (sm_100a):
//   compact_kernel           mask preprocess + ascending index compaction (warp ballot + block scan)
//   gather_bulk_kernel       executed-row gather (bulk copies through shared memory), per-head
//                            RMSNorm + multi-axis RoPE, cache-row write
//   arrival_wait_kernel      end of a head-split frame: waits for every GPU's O rows
//   restore_rows_kernel      puts back the cache rows of mask==1 tokens after the attention
//   host_rows_kernel         executed rows between page-locked host memory and the device (PCIe)
//   rows_copy_kernel         byte-exact indexed row gather / scatter
//   kv_sync_kernel           reference full-frame K/V merge + update
//   out_cache_sync_kernel    reference output-cache merge + valid update
//   rms_norm_kernel          standalone row RMSNorm
//   ln_modulate_rows_kernel  executed-row gather + LayerNorm (no affine) + (1 + scale) x + shift
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

// Rows whose cache rows must be put back after the attention (mask 1, execute without updating the
// cache), listed by the compaction for the attention's fused restore (two-tile kernel) or for
// restore_rows_kernel. rows == nullptr: no list.
struct RestoreList {
    int32_t* rows;        // [N] compact rows of mask==1 tokens, in no particular order
    int32_t* count;       // how many
    int32_t* head_done;   // [n_heads * kRestoreSlots] the attention's arrival counters, zeroed here
};

struct CompactStream {
    int32_t* mask;
    const uint8_t* valid;
    int32_t* idx;
    int32_t* count;
    RestoreList rl;
};

struct CompactArgs {
    CompactStream s[kMaxBatch];   // CTA b compacts stream b
    int32_t n;
    uint4* zero;                  // the attention's key-split arrival counters, zeroed by CTA 0
    int32_t zero_vec;
    uint4* zero2;                 // a second area CTA 0 zeroes (the block's GEMM sync words)
    int32_t zero2_vec;
    int32_t n_force;              // tokens below this one execute whatever their mask (0 -> 2)
    int32_t n_heads;              // restore lists: counters per stream = n_heads * kRestoreSlots
};

__global__ void __launch_bounds__(kCompactThreads, 1) compact_kernel(const __grid_constant__ CompactArgs a) {
    int32_t* __restrict__ mask = a.s[blockIdx.x].mask;
    const uint8_t* __restrict__ valid = a.s[blockIdx.x].valid;
    int32_t* __restrict__ idx = a.s[blockIdx.x].idx;
    int32_t* __restrict__ count = a.s[blockIdx.x].count;
    const int32_t n = a.n;
    const RestoreList rl = a.s[blockIdx.x].rl;
    __shared__ int32_t warp_tot[kCompactWarps];
    __shared__ int32_t n_restore;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t lt = (1u << lane) - 1u;
    pdl_launch_dependents();
    pdl_wait();  // the previous frame's kernels may still read mask / idx / count
    if (threadIdx.x == 0) n_restore = 0;
    if (rl.head_done)
        for (int32_t e = threadIdx.x; e < a.n_heads * kRestoreSlots; e += kCompactThreads) rl.head_done[e] = 0;
    // the attention's key-split arrival counters of this frame (zero_vec 16-byte words)
    if (blockIdx.x == 0) {
        for (int32_t e = threadIdx.x; e < a.zero_vec; e += kCompactThreads) a.zero[e] = make_uint4(0, 0, 0, 0);
        for (int32_t e = threadIdx.x; e < a.zero2_vec; e += kCompactThreads) a.zero2[e] = make_uint4(0, 0, 0, 0);
    }
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
            if (g < gpw && e < c0 + n_chunk && e < a.n_force && mval[g] == 0) {
                mask[e] = 2;
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
            if ((ballot[g] >> lane) & 1u) {
                const int32_t R = off + __popc(ballot[g] & lt);
                idx[R] = e0 + g * 32;
                if (rl.rows != nullptr && mval[g] == 1) rl.rows[atomicAdd(&n_restore, 1)] = R;
            }
            off += __popc(ballot[g]);
        }
        base += chunk_tot;
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        *count = base;
        if (rl.count) *rl.count = n_restore;
    }
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
// Fused gather + QK-RMSNorm + RoPE + cache-row write: shared definitions.
// Lane `sub` of a half-warp owns elements [8*sub, 8*sub+8) of a 128-wide head row (one 16-byte
// vector), so each rotary pair is lane-local and the RMS reduction is a 4-step half-warp shuffle;
// cos/sin of a token's 4 pairs per lane are computed once and reused for every head of Q and K.
// ---------------------------------------------------------------------------------------------
constexpr int kHeadDim = 128;
constexpr int kPairs = kHeadDim / 2;

struct RopeTable {
    float omega[kPairs];     // theta^(-2*jj/d_a) for pair j (rounded from double on the host)
    int8_t axis[kPairs];     // axis of pair j, -1 for none (identity)
};

struct GatherStream {           // one stream's buffers
    const void* q;
    const void* k;
    const void* v;
    const int32_t* mask;
    const int32_t* idx;
    const int32_t* count;
    void* qc;
    void* cache_k;
    void* cache_v;
    void* save;
    const uint8_t* valid;       // compacting launches: cache-row validity (NULL: every row valid)
    RestoreList rl;             // compacting launches: the mask==1 list for the restore
};

struct GatherArgs {
    GatherStream s[kMaxBatch];
    int32_t n_streams;
    // compact != 0: the launch also does the mask protocol and compaction of every stream (the
    // work of compact_kernel): each CTA scans the masks itself and keeps the list of its own rows
    // in shared memory; CTA 0 writes the preprocessed masks, idx and count for the later kernels
    // and zeroes the attention's key-split arrival counters (zero, zero_vec 16-byte words).
    int32_t compact;
    uint32_t grid_magic;         // ceil(2^32 / grid) for grids above 1 (the compaction's row split)
    uint4* zero;
    int32_t zero_vec;
    // iota != null: the launch also writes iota[m] = m for m < iota_cap and -1 up to iota_n (the
    // output rows of an attention into a compact buffer, as a head-split frame's share uses)
    int32_t* iota;
    int32_t iota_n, iota_cap;
    const int32_t* pos;
    const float* norm_q;
    const float* norm_k;
    const float* norm_q_txt;     // tokens below n_text_norm use these (a double-stream block's
    const float* norm_k_txt;     // text stream); null: norm_q / norm_k for every token
    int32_t n_text_norm;
    int64_t ld_qkv, ld_qc, ld_cache;
    int32_t n_tokens, n_heads, n_axes;
    float eps;
    RopeTable rope;
};

// sin/cos of a rotary angle (|angle| up to a few thousand radians): Cody-Waite reduction by 2*pi
// with the constant split into an exactly representable head (6.28125) and a tail, then the
// hardware sine/cosine on [-pi, pi] (absolute error ~4e-7 there).
__device__ __forceinline__ void rope_sincos(float ang, float* s, float* c) {
    const float k = rintf(ang * 0.15915494309189535f);
    float r = fmaf(-k, 6.28125f, ang);
    r = fmaf(-k, 1.9353071795864769e-3f, r);
    __sincosf(r, s, c);
}

// RMSNorm + RoPE of one lane's 8 elements of a 128-wide head vector (16 lanes per head; the sum of
// squares is reduced over the half-warp), stored as 16 bytes. The element products run in packed
// f32x2 form (two values of a 64-bit register pair per instruction); the rotation stays scalar.
__device__ __forceinline__ float2 f2mul(float2 a, float2 b) {
    uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d)
        : "l"(*reinterpret_cast<uint64_t*>(&a)), "l"(*reinterpret_cast<uint64_t*>(&b)));
    return *reinterpret_cast<float2*>(&d);
}
__device__ __forceinline__ float2 f2fma(float2 a, float2 b, float2 c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d)
        : "l"(*reinterpret_cast<uint64_t*>(&a)), "l"(*reinterpret_cast<uint64_t*>(&b)),
          "l"(*reinterpret_cast<uint64_t*>(&c)));
    return *reinterpret_cast<float2*>(&d);
}

template <typename T>
__device__ __forceinline__ void norm_rope_store_x2(const uint4& x, const float2* w2, float eps,
                                                   const float* cs, const float* sn, T* dst,
                                                   bool active) {
    const uint32_t u[4] = {x.x, x.y, x.z, x.w};
    float2 p[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) p[t] = StoreT<T>::unpack2(u[t]);
    float2 s2 = f2mul(p[0], p[0]);
#pragma unroll
    for (int t = 1; t < 4; ++t) s2 = f2fma(p[t], p[t], s2);
    float ss = s2.x + s2.y;
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float r = rsqrtf(ss * (1.0f / kHeadDim) + eps);
    const float2 r2 = make_float2(r, r);
    uint32_t outw[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
        const float2 ab = f2mul(p[t], f2mul(w2[t], r2));
        outw[t] = StoreT<T>::pack2(ab.x * cs[t] - ab.y * sn[t], ab.y * cs[t] + ab.x * sn[t]);
    }
    if (active) *reinterpret_cast<uint4*>(dst) = make_uint4(outw[0], outw[1], outw[2], outw[3]);
}

// ---------------------------------------------------------------------------------------------
// The gather step as a bulk-copy pipeline. One persistent CTA per SM walks its
// executed rows r = blockIdx.x, +gridDim.x, ...; a producer warp reads the indices of 32 rows at a
// time and streams each row's Q, K and V (C contiguous elements each) into a ring of shared-memory
// stages with cp.async.bulk, then posts the row's token, mode and position ids (second arrival on
// the stage's full barrier, so that those loads overlap the row copies). Four groups of four
// consumer warps take every fourth row: in a group, warps 0-1 normalise and rotate the row's Q
// heads and warps 2-3 its K heads out of shared memory (a half-warp per 128-wide head vector,
// 16-byte lanes, its heads h, h+4, h+8, ... in one unrolled batch), store Q' compact and K' into
// the cache row, and one lane writes the V row back to the cache with a bulk store. Rows with
// mode 1 first copy their old cache rows to the save buffer.
// ---------------------------------------------------------------------------------------------
constexpr int kBulkGroupWarps = 4;
constexpr int kBulkGroups = 6;
constexpr int kBulkProducerWarp = kBulkGroupWarps * kBulkGroups;
constexpr int kBulkThreads = (kBulkProducerWarp + 1) * 32;
constexpr int kBulkMaxStages = 32;
constexpr int kBulkInfoWords = 8;   // per stage: token, mode, position ids[4], stream, compact row
constexpr int kBulkListCap = 1024;  // rows per CTA of a compacting launch (token|mode, stream|row)
constexpr int kScanPer = 8;         // tokens per thread and pass of the in-kernel compaction
constexpr int kScanWarps = kBulkThreads / 32;

struct BulkLayout {
    uint32_t stage_bytes;   // 3 rows (Q, K, V) of C elements, 128-byte aligned
    uint32_t stages;
};

// In-kernel mask protocol + compaction of every stream of a gather launch (compact_kernel's work,
// done redundantly by every CTA so that no CTA waits for another). Tokens are scanned in passes of
// kScanPer x kBulkThreads: thread t holds tokens pass0 + k*kBulkThreads + t (coalesced loads), a
// ballot per (k, warp) and an exclusive scan of the kScanPer x kScanWarps counts give each executed
// token its rank R in ascending token order. Launch row g = (earlier streams' rows) + R belongs to
// CTA g % grid, slot g / grid of its list: (token | mode << 28, stream << 24 | R), mode 1 for mask 1
// (execute, keep the cache row) and 2 for any other executed value. CTA 0 also writes the
// preprocessed mask (valid == 0 -> 2), idx[R] and count, and zeroes the key-split counters.
// Returns the executed rows of all streams.
__device__ __forceinline__ int32_t compact_into_list(const GatherArgs& a, uint2* list) {
    __shared__ int32_t cnt[kScanPer * kScanWarps];
    __shared__ int32_t off[kScanPer * kScanWarps + 1];
    __shared__ int32_t n_restore;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t lt = (1u << lane) - 1u;
    const bool writer = blockIdx.x == 0;
    if (writer)
        for (int32_t e = threadIdx.x; e < a.zero_vec; e += kBulkThreads) a.zero[e] = make_uint4(0, 0, 0, 0);
    const int32_t n = a.n_tokens;
    int32_t pre = 0;
    for (int b = 0; b < a.n_streams; ++b) {
        int32_t* mask = const_cast<int32_t*>(a.s[b].mask);
        const uint8_t* valid = a.s[b].valid;
        int32_t* idx = const_cast<int32_t*>(a.s[b].idx);
        const RestoreList rl = a.s[b].rl;
        if (writer) {
            if (threadIdx.x == 0) n_restore = 0;
            if (rl.head_done)
                for (int32_t e = threadIdx.x; e < a.n_heads * kRestoreSlots; e += kBulkThreads) rl.head_done[e] = 0;
        }
        int32_t base = 0;
        for (int32_t c0 = 0; c0 < n; c0 += kScanPer * kBulkThreads) {
            int32_t mv[kScanPer];
            uint32_t bal[kScanPer];
#pragma unroll
            for (int k = 0; k < kScanPer; ++k) {
                const int32_t tok = c0 + k * kBulkThreads + (int32_t)threadIdx.x;
                mv[k] = tok < n ? mask[tok] : 0;
                if (valid != nullptr && tok < n && valid[tok] == 0) {
                    if (writer && mv[k] != 2) mask[tok] = 2;
                    mv[k] = 2;
                }
            }
#pragma unroll
            for (int k = 0; k < kScanPer; ++k) {
                bal[k] = __ballot_sync(0xffffffffu, mv[k] != 0);
                if (lane == 0) cnt[k * kScanWarps + warp] = __popc(bal[k]);
            }
            __syncthreads();
            if (warp == 0) {
                // exclusive scan of the counts in (k, warp) order: lane l sums a run of entries
                constexpr int kRun = (kScanPer * kScanWarps + 31) / 32;
                int32_t v[kRun], sum = 0;
#pragma unroll
                for (int q = 0; q < kRun; ++q) {
                    const int e = lane * kRun + q;
                    v[q] = e < kScanPer * kScanWarps ? cnt[e] : 0;
                    sum += v[q];
                }
                int32_t incl = sum;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const int32_t y = __shfl_up_sync(0xffffffffu, incl, o);
                    if (lane >= o) incl += y;
                }
                int32_t run = incl - sum;
#pragma unroll
                for (int q = 0; q < kRun; ++q) {
                    const int e = lane * kRun + q;
                    if (e < kScanPer * kScanWarps) off[e] = run;
                    run += v[q];
                }
                if (lane == 31) off[kScanPer * kScanWarps] = incl;
            }
            __syncthreads();
#pragma unroll
            for (int k = 0; k < kScanPer; ++k) {
                if ((bal[k] >> lane) & 1u) {
                    const int32_t tok = c0 + k * kBulkThreads + (int32_t)threadIdx.x;
                    const int32_t R = base + off[k * kScanWarps + warp] + __popc(bal[k] & lt);
                    if (writer) {
                        idx[R] = tok;
                        if (rl.rows != nullptr && mv[k] == 1) rl.rows[atomicAdd(&n_restore, 1)] = R;
                    }
                    // g / grid by a multiply with ceil(2^32 / grid): exact while g x grid < 2^32,
                    // and a compacting launch has g < 1024 x grid (gather_can_compact)
                    const uint32_t g = (uint32_t)(pre + R);
                    const uint32_t q = gridDim.x > 1 ? __umulhi(g, a.grid_magic) : g;
                    if (g - q * gridDim.x == blockIdx.x)
                        list[q] = make_uint2((uint32_t)tok | ((mv[k] == 1 ? 1u : 2u) << 28),
                                             ((uint32_t)b << 24) | (uint32_t)R);
                }
            }
            base += off[kScanPer * kScanWarps];
            __syncthreads();   // cnt / off are rewritten by the next pass
        }
        if (writer && threadIdx.x == 0) {
            *const_cast<int32_t*>(a.s[b].count) = base;
            if (rl.count) *rl.count = n_restore;
        }
        pre += base;
    }
    __syncthreads();       // the list is complete
    return pre;
}

template <typename T>
__global__ void __launch_bounds__(kBulkThreads, 1)
gather_bulk_kernel(const __grid_constant__ GatherArgs a, const BulkLayout lay) {
    extern __shared__ __align__(128) uint8_t bsm[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t S = lay.stages;
    uint8_t* ring = bsm;
    int32_t* info = reinterpret_cast<int32_t*>(bsm + S * lay.stage_bytes);
    const uint32_t bars = smem_u32(info + S * kBulkInfoWords);     // full[S], empty[S]
    __shared__ int abort_flag;
    auto full = [&](uint32_t st) { return bars + st * 8u; };
    auto empty = [&](uint32_t st) { return bars + (S + st) * 8u; };
    if (threadIdx.x == 0) {
        abort_flag = 0;
        for (uint32_t st = 0; st < S; ++st) {
            mbar_init(full(st), 2);                  // copies (expect_tx) + bookkeeping
            mbar_init(empty(st), kBulkGroupWarps);
        }
        fence_mbar_init();
    }
    __syncthreads();
    volatile int* abort = &abort_flag;
    pdl_launch_dependents();
    // Warm L2 with the bookkeeping inputs while the preceding kernel finishes: the masks (compacting
    // launches) or index lists, and the position ids. A prefetch brings nothing into the CTA, so it
    // is safe before the dependency wait even for data the preceding kernel writes.
    {
        const int64_t t = (int64_t)blockIdx.x * kBulkThreads + threadIdx.x, stride = (int64_t)gridDim.x * kBulkThreads;
        const int64_t mask_lines = ((int64_t)a.n_tokens * 4 + 127) / 128;
        for (int b = 0; b < a.n_streams; ++b) {
            const char* src = reinterpret_cast<const char*>(a.compact ? a.s[b].mask : a.s[b].idx);
            for (int64_t l = t; l < mask_lines; l += stride) prefetch_l2(src + l * 128);
        }
        const int64_t pos_lines = ((int64_t)a.n_tokens * a.n_axes * 4 + 127) / 128;
        for (int64_t l = t; l < pos_lines; l += stride) prefetch_l2(reinterpret_cast<const char*>(a.pos) + l * 128);
    }
    pdl_wait();  // count / idx / mask come from the compaction
    if (a.iota != nullptr)
        for (int32_t m = blockIdx.x * kBulkThreads + threadIdx.x; m < a.iota_n; m += gridDim.x * kBulkThreads)
            a.iota[m] = m < a.iota_cap ? m : -1;

    // executed rows of all streams, stream after stream: row r of the launch is row r - pre[b] of
    // stream b (pre = exclusive prefix of the streams' counts)
    uint2* list = reinterpret_cast<uint2*>(bsm + S * lay.stage_bytes + S * (kBulkInfoWords * 4 + 16));
    int32_t M = 0;
    if (a.compact) {
        M = compact_into_list(a, list);
    } else {
        for (int b = 0; b < a.n_streams; ++b) M += *a.s[b].count;
    }
    const int64_t C = (int64_t)a.n_heads * kHeadDim;
    const uint32_t row_bytes = (uint32_t)(C * (int64_t)sizeof(T));
    const int32_t rows_here =
        M > (int32_t)blockIdx.x ? (M - 1 - (int32_t)blockIdx.x) / (int32_t)gridDim.x + 1 : 0;

    if (warp == kBulkProducerWarp) {
        // ---------------- producer warp ----------------
        bool ok = true;
        int32_t issued = 0;
        for (int32_t kb = 0; ok && kb < rows_here; kb += 32) {
            const int32_t kl = kb + lane;
            int32_t i = -1, sb = 0, m = 0, mode = 0;
            if (kl < rows_here) {
                if (a.compact) {
                    const uint2 e = list[kl];
                    i = (int32_t)(e.x & 0x0FFFFFFFu);
                    mode = (int32_t)(e.x >> 28);
                    sb = (int32_t)(e.y >> 24);
                    m = (int32_t)(e.y & 0x00FFFFFFu);
                } else {
                    m = (int32_t)blockIdx.x + kl * (int32_t)gridDim.x;
                    while (sb + 1 < a.n_streams && m >= *a.s[sb].count) m -= *a.s[sb++].count;
                    i = __ldg(a.s[sb].idx + m);
                }
                if (i < 0 || i >= a.n_tokens) i = -1;
            }
            // bookkeeping loads of the 32 rows, in flight while the row copies are issued
            int32_t p[4] = {0, 0, 0, 0};
            if (i >= 0) {
                if (!a.compact) mode = __ldg(a.s[sb].mask + i);
#pragma unroll
                for (int ax = 0; ax < 4; ++ax)
                    if (ax < a.n_axes) p[ax] = __ldg(a.pos + (int64_t)i * a.n_axes + ax);
            }
            const int32_t nb = min(32, rows_here - kb);
            for (int32_t j = 0; j < nb; ++j) {
                const int32_t k = kb + j;
                const uint32_t st = (uint32_t)k % S, use = (uint32_t)k / S;
                if (use > 0 && !__all_sync(0xffffffffu, mbar_wait_suspend(empty(st), (use - 1) & 1, abort))) {
                    ok = false;
                    break;
                }
                const int32_t ti = __shfl_sync(0xffffffffu, i, j);
                const int32_t tb = __shfl_sync(0xffffffffu, sb, j);
                const int32_t tmr = __shfl_sync(0xffffffffu, m, j);
                if (lane == 0) {
                    if (ti >= 0) {
                        const uint32_t dst = smem_u32(ring + st * lay.stage_bytes);
                        const int64_t off = (int64_t)ti * a.ld_qkv;
                        const GatherStream& gs = a.s[tb];
                        mbar_arrive_expect_tx(full(st), 3u * row_bytes);
                        bulk_load(dst, static_cast<const T*>(gs.q) + off, row_bytes, full(st));
                        bulk_load(dst + row_bytes, static_cast<const T*>(gs.k) + off, row_bytes, full(st));
                        bulk_load(dst + 2 * row_bytes, static_cast<const T*>(gs.v) + off, row_bytes, full(st));
                    } else {
                        atomicOr(&g_error_word, kErrBounds);
                        mbar_arrive(full(st));
                    }
                }
                const int32_t tm = __shfl_sync(0xffffffffu, mode, j);
                int32_t tp[4];
#pragma unroll
                for (int ax = 0; ax < 4; ++ax) tp[ax] = __shfl_sync(0xffffffffu, p[ax], j);
                if (lane == 0) {
                    int32_t* inf = info + st * kBulkInfoWords;
                    inf[0] = ti;
                    inf[1] = tm;
#pragma unroll
                    for (int ax = 0; ax < 4; ++ax) inf[2 + ax] = tp[ax];
                    inf[6] = tb;
                    inf[7] = tmr;
                    mbar_arrive(full(st));
                }
                __syncwarp();
                ++issued;
            }
        }
        if (lane == 0 && *abort) {
            // after an abort: the copies of the last stages may still be in flight
            for (int32_t k = max(0, issued - (int32_t)S); k < issued; ++k)
                mbar_wait_drain_bounded(full((uint32_t)k % S), ((uint32_t)k / S) & 1);
        }
    } else {
        // ---------------- consumer groups ----------------
        const int grp = warp / kBulkGroupWarps, gw = warp % kBulkGroupWarps;
        const int half = lane >> 4, sub = lane & 15;
        const bool isq = gw < kBulkGroupWarps / 2;           // warp-uniform: Q or K heads
        constexpr int kHeadStride = kBulkGroupWarps;         // half-warps per tensor
        const int hw0 = (gw % (kBulkGroupWarps / 2)) * 2;     // first head of this warp
        // norm weights: the image stream's (every token's without a text stream) and the text
        // stream's (rows < n_text_norm); this lane's 8 are read per row (L1 hits)
        const float* wimg = (isq ? a.norm_q : a.norm_k) + 8 * sub;
        const float* wtxt = isq ? a.norm_q_txt : a.norm_k_txt;
        if (wtxt != nullptr) wtxt += 8 * sub;
        const bool bulk_lane = gw == 0 && lane == 0;
        const int gtid = gw * 32 + lane;
        // this lane's four rotary pairs (the same in every row): frequency and axis
        float om[4];
        int axv[4];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            om[t] = a.rope.omega[4 * sub + t];
            axv[t] = a.rope.axis[4 * sub + t];
        }
        for (int32_t k = grp; k < rows_here; k += kBulkGroups) {
            const uint32_t st = (uint32_t)k % S, use = (uint32_t)k / S;
            if (!__all_sync(0xffffffffu, mbar_wait_suspend(full(st), use & 1, abort))) break;
            const int32_t* inf = info + st * kBulkInfoWords;
            const int32_t i = inf[0], mode = inf[1];
            const GatherStream& gs = a.s[inf[6]];
            const int32_t r = inf[7];                       // compact row within its stream
            T* __restrict__ QC = static_cast<T*>(gs.qc);
            T* __restrict__ CK = static_cast<T*>(gs.cache_k);
            T* __restrict__ CV = static_cast<T*>(gs.cache_v);
            T* __restrict__ SV = static_cast<T*>(gs.save);
            const uint8_t* stage = ring + st * lay.stage_bytes;
            if (i >= 0) {
                if (mode == 1 && SV != nullptr) {
                    // keep the old cache rows: the attention reads the fresh ones, the restore
                    // puts these back afterwards
                    const int64_t nvec = C * (int64_t)sizeof(T) / 16;
                    const uint4* okr = reinterpret_cast<const uint4*>(CK + (int64_t)i * a.ld_cache);
                    const uint4* ovr = reinterpret_cast<const uint4*>(CV + (int64_t)i * a.ld_cache);
                    uint4* sk = reinterpret_cast<uint4*>(SV + (int64_t)r * 2 * C);
                    uint4* svv = reinterpret_cast<uint4*>(SV + (int64_t)r * 2 * C + C);
                    for (int64_t e = gtid; e < nvec; e += kBulkGroupWarps * 32) {
                        sk[e] = okr[e];
                        svv[e] = ovr[e];
                    }
                    named_barrier_sync(1 + grp, kBulkGroupWarps * 32);
                }
                if (bulk_lane) {
                    if (mode == 1) fence_proxy_async();   // old V row read before it is overwritten
                    bulk_store(CV + (int64_t)i * a.ld_cache, smem_u32(stage + 2 * row_bytes), row_bytes);
                    bulk_commit();
                }
                float2 w2[4];
                {
                    const float* ws = (wtxt != nullptr && i < a.n_text_norm) ? wtxt : wimg;
#pragma unroll
                    for (int t = 0; t < 4; ++t) w2[t] = make_float2(__ldg(ws + 2 * t), __ldg(ws + 2 * t + 1));
                }
                float cs[4], sn[4];
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                    if (axv[t] < 0) {
                        cs[t] = 1.f;
                        sn[t] = 0.f;
                    } else {
                        rope_sincos((float)inf[2 + axv[t]] * om[t], &sn[t], &cs[t]);
                    }
                }
                // kUnitBatch independent head vectors per half-warp at a time (their loads,
                // shuffles and stores interleave); 24 heads = 2 batches of 3 x 4 half-warps
                constexpr int kUnitBatch = 3;
                const uint8_t* src = stage + (isq ? 0 : row_bytes) + (size_t)(8 * sub) * sizeof(T);
                T* dst = (isq ? QC + (int64_t)r * a.ld_qc : CK + (int64_t)i * a.ld_cache) + 8 * sub;
                // warp-uniform loop bound: both half-warps join every shuffle
                for (int hw = hw0; hw < a.n_heads; hw += kUnitBatch * kHeadStride) {
                    const int h0 = hw + half;
                    uint4 x[kUnitBatch];
                    bool act[kUnitBatch];
#pragma unroll
                    for (int b = 0; b < kUnitBatch; ++b) {
                        const int h = h0 + b * kHeadStride;
                        act[b] = h < a.n_heads;
                        x[b] = act[b] ? *reinterpret_cast<const uint4*>(src + (size_t)h * kHeadDim * sizeof(T))
                                      : make_uint4(0, 0, 0, 0);
                    }
#pragma unroll
                    for (int b = 0; b < kUnitBatch; ++b)
                        norm_rope_store_x2<T>(x[b], w2, a.eps, cs, sn,
                                              dst + (int64_t)(h0 + b * kHeadStride) * kHeadDim, act[b]);
                }
            }
            if (bulk_lane) bulk_wait_read_all();   // the V stage has been read by its bulk store
            __syncwarp();
            if (lane == 0) mbar_arrive(empty(st));
        }
        if (bulk_lane) bulk_wait_all();
    }
}

// ---------------------------------------------------------------------------------------------
// Restore of mask==1 cache rows (execute without cache update) from the save buffer.
// ---------------------------------------------------------------------------------------------
struct RestoreStream {
    const int32_t* mask;
    const int32_t* idx;
    const int32_t* count;
    const uint4* save;
    char* cache_k;
    char* cache_v;
};

struct RestoreArgs {
    RestoreStream s[kMaxBatch];   // grid row blockIdx.y restores stream blockIdx.y
    int64_t ld_cache_bytes;
    int32_t row_vec, n_tokens;
};

__global__ void __launch_bounds__(256) restore_rows_kernel(const __grid_constant__ RestoreArgs a) {
    const RestoreStream& rs = a.s[blockIdx.y];
    const int32_t* __restrict__ mask = rs.mask;
    const int32_t* __restrict__ idx = rs.idx;
    const int32_t* __restrict__ count = rs.count;
    const uint4* __restrict__ save = rs.save;
    char* __restrict__ cache_k = rs.cache_k;
    char* __restrict__ cache_v = rs.cache_v;
    const int64_t ld_cache_bytes = a.ld_cache_bytes;
    const int32_t row_vec = a.row_vec, n_tokens = a.n_tokens;
    const int lane = threadIdx.x & 31;
    // The last kernel of a frame: it lets its successor start only once the attention is over, since
    // that successor may be code outside this library (a collective, a copy) that reads the frame's
    // output without a programmatic-dependency wait of its own.
    pdl_wait();  // the attention must have finished reading the cache rows
    pdl_launch_dependents();
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
// Executed rows across PCIe for a frame whose tensors live in page-locked host memory: the rows
// idx[0..M) of up to three tensors move between the host and the device at the same row position
// (dst row i = src row i), so only executed rows cross the bus. One side is mapped host memory read
// or written by the SMs directly (zero-copy); a warp moves one row of one tensor, each lane eight
// 16-byte vectors at a time with the loads issued before the stores. 64 CTAs of 64 threads keep
// 512 KB of reads in flight, enough to fill PCIe (one CTA per SM reaches the same rate as two), and
// each CTA is small enough (under 3.6K registers) to sit beside a persistent gather or attention
// CTA on its SM: the next frame's upload then runs under this frame's kernels instead of keeping
// them off the SMs it holds.
// ---------------------------------------------------------------------------------------------
constexpr int kHostRowsThreads = 64;
constexpr int kHostRowsUnroll = 8;
constexpr int kHostRowsCtas = 64;

struct HostRowsArgs {
    const uint4* src[3];
    uint4* dst[3];
    const int32_t* idx;
    const int32_t* count;
    int64_t ld_vec;        // row stride of every tensor, 16-byte units
    int32_t row_vec;       // 16-byte units per row
    int32_t n_tensors, n_tokens;
};

__global__ void __launch_bounds__(kHostRowsThreads) host_rows_kernel(const __grid_constant__ HostRowsArgs a) {
    pdl_wait();   // idx / count of the compaction; for the download, the frame's output rows
    const int32_t M = min(*a.count, a.n_tokens);
    const int lane = threadIdx.x & 31;
    const int32_t warps = kHostRowsThreads / 32;
    const int64_t items = (int64_t)M * a.n_tensors;
    for (int64_t it = (int64_t)blockIdx.x * warps + (threadIdx.x >> 5); it < items;
         it += (int64_t)gridDim.x * warps) {
        const int32_t m = (int32_t)(it / a.n_tensors);
        const int32_t t = (int32_t)(it - (int64_t)m * a.n_tensors);
        const int32_t i = a.idx[m];
        if (i < 0 || i >= a.n_tokens) continue;
        const uint4* s = a.src[t] + (int64_t)i * a.ld_vec;
        uint4* d = a.dst[t] + (int64_t)i * a.ld_vec;
        for (int32_t j0 = lane; j0 < a.row_vec; j0 += 32 * kHostRowsUnroll) {
            uint4 v[kHostRowsUnroll];
#pragma unroll
            for (int u = 0; u < kHostRowsUnroll; ++u)
                if (j0 + 32 * u < a.row_vec) v[u] = s[j0 + 32 * u];
#pragma unroll
            for (int u = 0; u < kHostRowsUnroll; ++u)
                if (j0 + 32 * u < a.row_vec) d[j0 + 32 * u] = v[u];
        }
    }
}

// ---------------------------------------------------------------------------------------------
// Exchange of a head-split frame: every executed row's slice of this GPU's heads (compact O, written
// by the attention) goes to the full-frame output of every GPU of the group — the all-gather and the
// scatter in one pass, over NVLink through peer mappings. A warp per row; each lane moves 16-byte
// pieces of the slice (hn x 256 contiguous bytes at the destination), the slice loaded once and
// stored to every destination. Each CTA then adds one arrival (release, system scope) to its slot
// at every destination.
// ---------------------------------------------------------------------------------------------
constexpr int kPushThreads = 256;
constexpr int kPushMaxVecs = 8;    // 16-byte pieces per lane of a row slice: up to 8 heads x 256 B / 32

struct PushArgs {
    const uint4* o;            // compact O [rows][row_vecs], this GPU's heads
    const int32_t* idx;
    const int32_t* count;
    int64_t ld_out_vecs;       // destination row stride in 16-byte units
    int32_t row_vecs;          // 16-byte pieces per row slice (hn * head_dim * size / 16)
    int32_t n_tokens, world, src_rank;
    uint4* out[8];             // destinations, offset to this GPU's first head column
    uint32_t* arrive[8];
};

__global__ void __launch_bounds__(kPushThreads) heads_push_kernel(const __grid_constant__ PushArgs a) {
    const int lane = threadIdx.x & 31;
    pdl_wait();                // the attention's compact O
    const int32_t M = *a.count;
    for (int32_t m = blockIdx.x * (kPushThreads / 32) + (threadIdx.x >> 5); m < M;
         m += gridDim.x * (kPushThreads / 32)) {
        const int32_t i = a.idx[m];
        if (i < 0 || i >= a.n_tokens) {
            if (lane == 0) atomicOr(&g_error_word, kErrBounds);
            continue;
        }
        for (int32_t c0 = 0; c0 < a.row_vecs; c0 += 32 * kPushMaxVecs) {
            uint4 v[kPushMaxVecs];
            const uint4* src = a.o + (int64_t)m * a.row_vecs + c0;
            const int32_t nv = min(a.row_vecs - c0, 32 * kPushMaxVecs);
#pragma unroll
            for (int k = 0; k < kPushMaxVecs; ++k)
                if (lane + 32 * k < nv) v[k] = src[lane + 32 * k];
#pragma unroll
            for (int t = 0; t < 8; ++t) {
                if (t >= a.world) break;
                uint4* dst = a.out[t] + (int64_t)i * a.ld_out_vecs + c0;
#pragma unroll
                for (int k = 0; k < kPushMaxVecs; ++k)
                    if (lane + 32 * k < nv) dst[lane + 32 * k] = v[k];
            }
        }
    }
    __threadfence_system();    // this thread's stores, visible to every GPU before the arrival
    __syncthreads();
    if (threadIdx.x < a.world) red_release_sys_add(a.arrive[threadIdx.x] + a.src_rank, 1u);
}

// ---------------------------------------------------------------------------------------------
// Arrival wait of a head-sharded frame. slots[0..8): arrivals from each source GPU (one per
// exchange CTA of that GPU per frame); slots[8]: frames this GPU has waited for, kept on the
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
// NCCL variant of the head-split frame: compact-row index list for the attention's compact O
// output (m < m_cap: m; beyond: -1, which the attention skips and reports), and the scatter of the
// all-gathered compact rows of every rank into the full-frame output.
// ---------------------------------------------------------------------------------------------
struct HeadsScatterArgs {
    const char* gathered;      // [world][m_cap][row_bytes]
    const int32_t* idx;
    const int32_t* count;
    char* out;
    int64_t row_bytes;         // hmax * head_dim * element size
    int64_t ld_out_bytes;
    int32_t m_cap, world, n_tokens;
    int32_t col_bytes[8];      // each rank's first column in bytes (head0 * head_dim * element size)
    int32_t vecs[8];           // each rank's 16-byte vectors per row (n_heads * head_dim * size / 16)
};

__global__ void __launch_bounds__(256) heads_scatter_kernel(const __grid_constant__ HeadsScatterArgs a) {
    const int lane = threadIdx.x & 31;
    const int32_t M = min(*a.count, a.m_cap);
    if (blockIdx.x == 0 && threadIdx.x == 0 && *a.count > a.m_cap) atomicOr(&g_error_word, kErrBounds);
    const int64_t units = (int64_t)M * a.world;
    for (int64_t u = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5); u < units; u += (int64_t)gridDim.x * 8) {
        const int32_t m = (int32_t)(u / a.world), r = (int32_t)(u % a.world);
        const int32_t i = a.idx[m];
        if (i < 0 || i >= a.n_tokens) {
            if (lane == 0) atomicOr(&g_error_word, kErrBounds);
            continue;
        }
        int32_t col = 0, nv = 0;
#pragma unroll
        for (int k = 0; k < 8; ++k)
            if (k == r) {
                col = a.col_bytes[k];
                nv = a.vecs[k];
            }
        const uint4* src = reinterpret_cast<const uint4*>(a.gathered + ((int64_t)r * a.m_cap + m) * a.row_bytes);
        uint4* dst = reinterpret_cast<uint4*>(a.out + (int64_t)i * a.ld_out_bytes + col);
        for (int32_t e = lane; e < nv; e += 32) dst[e] = src[e];
    }
}

// ---------------------------------------------------------------------------------------------
// Byte-exact indexed row copy: gather (dst[m] = src[idx[m]]) or scatter (dst[idx[m]] = src[m]).
// ---------------------------------------------------------------------------------------------
template <typename V, bool kScatter>
__global__ void __launch_bounds__(256)
rows_copy_kernel(const char* __restrict__ src, int64_t ld_src, const int32_t* __restrict__ idx,
                 const int32_t* __restrict__ count, int32_t host_count, char* __restrict__ dst,
                 int64_t ld_dst, int64_t row_vec, int32_t n_index_rows) {
    const int lane = threadIdx.x & 31;
    const int32_t M = count ? *count : host_count;
    for (int32_t m = blockIdx.x * 8 + (threadIdx.x >> 5); m < M; m += gridDim.x * 8) {
        const int32_t i = idx[m];
        if (i < 0 || i >= n_index_rows) {          // skipped: neither the indexed nor the compact row moves
            if (lane == 0) atomicOr(&g_error_word, kErrBounds);
            continue;
        }
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

// ---------------------------------------------------------------------------------------------
// Executed-row LayerNorm + modulation, the input of the block's projections: for compact rows m in
// [row0, row_end) (row_end < 0: *count),
//   y[m, :] = (1 + scale) * (x[idx[m], :] - mean) * rsqrt(var + eps) + shift
// with mean and the biased variance over the row's dim values (fp32). Restates
// layer_norm_modulated_kernel without gamma/beta and apply_modulation_kernel
// (gather_scatter_kernels.cu:77-99,106-169; called at flux2_double_block_plugin.cpp:373-383) on the
// executed rows only, in one pass over HBM. A warp per row, the row held in registers: lane l reads
// 16-byte chunks l, l + 32, ... so each warp instruction covers 512 contiguous bytes; dim is a
// multiple of 256 up to 4096.
// ---------------------------------------------------------------------------------------------
constexpr int kLnMaxChunks = 16;   // 16-byte chunks per lane: dim <= 16 * 32 * 8

template <typename T>
__global__ void __launch_bounds__(256)
ln_modulate_rows_kernel(const T* __restrict__ x, int64_t ld_x, const int32_t* __restrict__ idx,
                        const int32_t* __restrict__ count, int32_t row0, int32_t row_end_arg,
                        int32_t n_tokens, int32_t dim, const float* __restrict__ scale,
                        const float* __restrict__ shift, float eps, T* __restrict__ y, int64_t ld_y) {
    pdl_launch_dependents();
    pdl_wait();   // idx / count come from the compaction
    const int lane = threadIdx.x & 31;
    const int32_t row_end = min(row_end_arg >= 0 ? row_end_arg : *count, n_tokens);
    const int nch = dim / 256;
    const float inv_dim = 1.0f / (float)dim;
    for (int32_t m = row0 + (int32_t)blockIdx.x * 8 + (int32_t)(threadIdx.x >> 5); m < row_end;
         m += (int32_t)gridDim.x * 8) {
        const int32_t i = __ldg(idx + m);
        if (i < 0 || i >= n_tokens) {
            if (lane == 0) atomicOr(&g_error_word, kErrBounds);
            continue;
        }
        const uint4* xr = reinterpret_cast<const uint4*>(x + (int64_t)i * ld_x);
        uint4 v[kLnMaxChunks];
        float s = 0.f;
#pragma unroll
        for (int j = 0; j < kLnMaxChunks; ++j) {
            if (j < nch) {
                v[j] = __ldg(xr + j * 32 + lane);
                const uint32_t w4[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float2 f = StoreT<T>::unpack2(w4[e]);
                    s += f.x + f.y;
                }
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        const float mean = s * inv_dim;
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < kLnMaxChunks; ++j) {
            if (j < nch) {
                const uint32_t w4[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float2 f = StoreT<T>::unpack2(w4[e]);
                    const float d0 = f.x - mean, d1 = f.y - mean;
                    ss = fmaf(d0, d0, fmaf(d1, d1, ss));
                }
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float rstd = rsqrtf(ss * inv_dim + eps);
        uint4* yr = reinterpret_cast<uint4*>(y + (int64_t)m * ld_y);
#pragma unroll
        for (int j = 0; j < kLnMaxChunks; ++j) {
            if (j < nch) {
                const int col = (j * 32 + lane) * 8;
                float sc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f}, sh[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
                if (scale) {
                    const float4 s0 = __ldg(reinterpret_cast<const float4*>(scale + col));
                    const float4 s1 = __ldg(reinterpret_cast<const float4*>(scale + col) + 1);
                    sc[0] = s0.x; sc[1] = s0.y; sc[2] = s0.z; sc[3] = s0.w;
                    sc[4] = s1.x; sc[5] = s1.y; sc[6] = s1.z; sc[7] = s1.w;
                }
                if (shift) {
                    const float4 s0 = __ldg(reinterpret_cast<const float4*>(shift + col));
                    const float4 s1 = __ldg(reinterpret_cast<const float4*>(shift + col) + 1);
                    sh[0] = s0.x; sh[1] = s0.y; sh[2] = s0.z; sh[3] = s0.w;
                    sh[4] = s1.x; sh[5] = s1.y; sh[6] = s1.z; sh[7] = s1.w;
                }
                const uint32_t w4[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
                uint32_t o4[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float2 f = StoreT<T>::unpack2(w4[e]);
                    const float a0 = (f.x - mean) * rstd, a1 = (f.y - mean) * rstd;
                    o4[e] = StoreT<T>::pack2(fmaf(1.0f + sc[2 * e], a0, sh[2 * e]),
                                             fmaf(1.0f + sc[2 * e + 1], a1, sh[2 * e + 1]));
                }
                yr[j * 32 + lane] = make_uint4(o4[0], o4[1], o4[2], o4[3]);
            }
        }
    }
}

}  // namespace fxr
