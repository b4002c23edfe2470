// fxr_capi.cu — extern "C" entry points declared in include/fxr.h: argument validation, workspace
// carve-up, TMA tensor-map encoding and kernel launches. All kernels of the library are compiled in
// this one translation unit so they share one device error word.
#include <cuda.h>
#include <cuda_runtime.h>

#include <array>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <type_traits>
#include <string>

#include "fxr.h"
#include "fxr_attention.cuh"
#include "fxr_attention2.cuh"
#include "fxr_compat_kernels.cuh"
#include "fxr_dense_kernels.cuh"
#include "fxr_device.cuh"
#include "fxr_gemm.cuh"
#include "fxr_mem_kernels.cuh"

#include <nvtx3/nvToolsExt.h>

// Built-in frame scratch of fxr_frame_forward_noalloc (see that function). 128 MiB holds the
// workspace of a 1024x1024 frame (4608 tokens, 24 heads, 16-bit storage: ~85 MB) with the scratch
// slots of the attention's stream-K schedule (~39 MB on 148 SMs). Every GPU that loads this
// library keeps this array for the life of the process.
constexpr size_t kNoAllocScratchBytes = size_t(128) << 20;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

namespace {

// NVTX range over a host-side scope (an entry point, one step's launch), named "fxr:<step>":
// profilers that record NVTX (ncu --nvtx, Nsight Systems) attribute the kernels launched inside it.
// Without a tool attached a push / pop is a check of a function pointer.
struct NvtxRange {
    explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
    ~NvtxRange() { nvtxRangePop(); }
    NvtxRange(const NvtxRange&) = delete;
    NvtxRange& operator=(const NvtxRange&) = delete;
};

thread_local std::string t_last_error;

int32_t fail(int32_t status, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    std::vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    t_last_error = buf;
    return status;
}

int32_t cuda_status(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return FXR_OK;
    return fail(FXR_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

#define FXR_CHECK_LAUNCH(what)                                                                     \
    do {                                                                                           \
        cudaError_t e_ = cudaGetLastError();                                                       \
        if (e_ != cudaSuccess) return cuda_status(e_, what);                                       \
    } while (0)

constexpr int kMaxDevices = 64;

// Launch with programmatic stream serialisation: the kernel may begin (prologue only, until its
// griddepcontrol.wait) while the previous kernel on the stream finishes. Used for the four frame
// kernels, each of which waits before touching data shared with its predecessor.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t stream, Args&&... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

int sm_count() {
    static int counts[kMaxDevices] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
    if (counts[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
            n = 148;
        counts[dev] = n;
    }
    return counts[dev];
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

size_t dtype_bytes(int32_t dt) {
    switch (dt) {
        case FXR_F32: return 4;
        case FXR_F16: return 2;
        case FXR_BF16: return 2;
        default: return 0;
    }
}

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// ---- tensor maps ----------------------------------------------------------------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

// 2-D map over a row-major [rows, cols] 16-bit matrix with row stride ld (elements); box 64 x 128
// (one 128-byte swizzle span wide), 128-byte swizzle, zero fill out of bounds.
int32_t make_tmap(CUtensorMap* map, const void* ptr, int32_t dtype, int64_t cols, int64_t rows,
                  int64_t ld, uint32_t box_rows = 128) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return fail(FXR_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
    const cuuint32_t box[2] = {64, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const CUtensorMapDataType t =
        dtype == FXR_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    CUresult r = fn(map, t, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(FXR_ERR_INVALID, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return FXR_OK;
}

// ---- descriptor checks ------------------------------------------------------------------------
int32_t check_desc(const fxr_frame_desc* d, bool need_tc) {
    if (!d) return fail(FXR_ERR_INVALID, "null descriptor");
    if (d->n_tokens < 0 || d->n_heads <= 0 || d->head_dim <= 0)
        return fail(FXR_ERR_INVALID, "bad geometry: n_tokens=%d n_heads=%d head_dim=%d",
                    d->n_tokens, d->n_heads, d->head_dim);
    if (d->head_dim != fxr::kHeadDim)
        return fail(FXR_ERR_UNSUPPORTED, "head_dim %d unsupported (this path is built for 128)",
                    d->head_dim);
    if (d->dtype != FXR_BF16 && d->dtype != FXR_F16)
        return fail(FXR_ERR_UNSUPPORTED, "dtype %d unsupported on the tensor-core path", d->dtype);
    if (d->rope_n_axes < 0 || d->rope_n_axes > 4)
        return fail(FXR_ERR_INVALID, "rope_n_axes %d outside [0,4]", d->rope_n_axes);
    int sum = 0;
    for (int a = 0; a < d->rope_n_axes; ++a) {
        if (d->rope_axes_dim[a] <= 0 || (d->rope_axes_dim[a] & 1))
            return fail(FXR_ERR_INVALID, "rope_axes_dim[%d]=%d must be positive and even", a,
                        d->rope_axes_dim[a]);
        sum += d->rope_axes_dim[a];
    }
    if (sum > d->head_dim) return fail(FXR_ERR_INVALID, "rope axes sum %d > head_dim", sum);
    if (d->rope_n_axes > 0 && !(d->rope_theta > 0.f))
        return fail(FXR_ERR_INVALID, "rope_theta must be > 0");
    const int64_t C = (int64_t)d->n_heads * d->head_dim;
    if (d->ld_qkv < C || d->ld_cache < C || d->ld_out < C)
        return fail(FXR_ERR_INVALID, "row strides must be >= n_heads*head_dim (%lld)", (long long)C);
    if ((d->ld_qkv % 8) || (d->ld_cache % 8) || (d->ld_out % 8))
        return fail(FXR_ERR_INVALID, "row strides must be multiples of 8 elements (16 bytes)");
    (void)need_tc;
    return FXR_OK;
}

void fill_rope(const fxr_frame_desc* d, fxr::RopeTable* t) {
    for (int j = 0; j < fxr::kPairs; ++j) {
        t->omega[j] = 0.f;
        t->axis[j] = -1;
    }
    int j = 0;
    for (int a = 0; a < d->rope_n_axes; ++a) {
        const int half = d->rope_axes_dim[a] / 2;
        for (int jj = 0; jj < half && j < fxr::kPairs; ++jj, ++j) {
            t->omega[j] = (float)std::pow((double)d->rope_theta,
                                          -2.0 * (double)jj / (double)d->rope_axes_dim[a]);
            t->axis[j] = (int8_t)a;
        }
    }
}

struct Views {
    int32_t* count;
    int32_t* idx;
    void* qc;
    int64_t ld_qc;
    void* save;
    fxr::RestoreList restore;   // mask==1 rows for the restore (written by the compaction)
    size_t total;
};

Views carve(const fxr_frame_desc* d, void* ws) {
    Views v{};
    const size_t N = (size_t)(d->n_tokens > 0 ? d->n_tokens : 1);
    const size_t C = (size_t)d->n_heads * d->head_dim;
    const size_t eb = dtype_bytes(d->dtype);
    size_t off = 0;
    char* b = static_cast<char*>(ws);
    v.count = reinterpret_cast<int32_t*>(b ? b + off : nullptr);
    off = align_up(off + sizeof(int32_t), 256);
    v.idx = reinterpret_cast<int32_t*>(b ? b + off : nullptr);
    off = align_up(off + N * sizeof(int32_t), 256);
    v.qc = b ? b + off : nullptr;
    v.ld_qc = (int64_t)C;
    off = align_up(off + N * C * eb, 256);
    v.save = b ? b + off : nullptr;
    off = align_up(off + N * 2 * C * eb, 256);
    v.restore.count = reinterpret_cast<int32_t*>(b ? b + off : nullptr);
    v.restore.head_done = reinterpret_cast<int32_t*>(b ? b + off + 16 : nullptr);
    off = align_up(off + 16 + (size_t)d->n_heads * fxr::kRestoreSlots * sizeof(int32_t), 256);
    v.restore.rows = reinterpret_cast<int32_t*>(b ? b + off : nullptr);
    off = align_up(off + N * sizeof(int32_t), 256);
    v.total = off;
    return v;
}

// Optional key-range split scratch after a frame's workspace: per slot 16 arrival counters and one
// partial-result slot of the attention. A workspace of at least the base size works without it;
// fxr_workspace_size includes room for kSplitSlotsPerSm slots per SM.
constexpr int kSplitSlotsPerSm = 4;
constexpr int kSplitMaxHeads = 8;   // one-tile kernel: launches with at most this many heads may split key ranges
constexpr size_t kSplitSlotBytes = (size_t)fxr::attn::kSplitSlotFloats * sizeof(float);
constexpr size_t kSplitCntBytes = (size_t)fxr::attn::kSplitPortions * sizeof(int32_t);

struct SplitArea {
    int32_t* cnt = nullptr;
    float* scratch = nullptr;
    int32_t slots = 0;
};

size_t split_bytes(int32_t slots) {
    return align_up((size_t)slots * kSplitCntBytes, 256) + (size_t)slots * kSplitSlotBytes;
}

// The scratch slots and arrival counters that a workspace leaves after its base part (none when it
// ends there): key-range split of the one-tile kernel, stream-K schedule of the two-tile kernel.
SplitArea split_area(size_t base, void* ws, size_t ws_bytes, int32_t n_heads) {
    SplitArea a;
    (void)n_heads;
    if (!ws || ws_bytes <= base) return a;
    const int32_t max_slots = kSplitSlotsPerSm * sm_count();
    int32_t slots = (int32_t)std::min<size_t>(max_slots, (ws_bytes - base) / (kSplitSlotBytes + kSplitCntBytes));
    while (slots > 0 && split_bytes(slots) > ws_bytes - base) --slots;
    if (slots <= 0) return a;
    char* b = static_cast<char*>(ws) + base;
    a.cnt = reinterpret_cast<int32_t*>(b);
    a.scratch = reinterpret_cast<float*>(b + align_up((size_t)slots * kSplitCntBytes, 256));
    a.slots = slots;
    return a;
}

int grid_rows(int64_t rows, int rows_per_cta) {
    const int64_t need = (rows + rows_per_cta - 1) / rows_per_cta;
    const int64_t cap = (int64_t)sm_count() * 8;
    return (int)std::max<int64_t>(1, std::min(need, cap));
}

// Where the attention epilogue stores O: one buffer (a single-GPU frame), or every rank's buffer
// of a head group plus the arrival slots it increments there.
struct OutSet {
    void* out = nullptr;
    SplitArea split;   // key-range split scratch (none: never split)
    // SMs the attention leaves free, for the zero-copy row transfers of host-resident frames that
    // run beside it: the two-tile kernel holds a whole SM's registers, so nothing else fits next to
    // one of its CTAs
    int32_t reserve_sms = 0;
};

// Attention kernel for launches that need no key-range split: two query tiles per CTA unless
// FXR_ATTENTION_TILES=1 selects the one-tile kernel (read once per process).
static bool attention_pairs() {
    static const bool pairs = [] {
        const char* v = std::getenv("FXR_ATTENTION_TILES");
        return !(v && v[0] == '1');
    }();
    return pairs;
}

int64_t attention_ctas(int64_t n_tokens, int64_t n_heads) {
    if (n_tokens <= 0 || n_heads <= 0) return 0;
    const int64_t max_tiles = (n_tokens + fxr::attn::kBM - 1) / fxr::attn::kBM * n_heads;
    return std::max<int64_t>(1, std::min<int64_t>(max_tiles, sm_count()));
}

// One edit stream's operands of an attention launch.
struct AttnStreamArgs {
    const void* qc;
    int64_t ld_qc;
    const int32_t* count;
    const void* ck;
    const void* cv;
    const int32_t* idx;
    void* out;
    // the frame whose mask==1 cache rows the attention may restore itself (nullptr: it does not)
    const Views* frame = nullptr;
};

// Whether the two-tile kernel serves attention launches of this dtype on the current device (it
// then also restores the frame's mask==1 cache rows, so the frame needs no restore launch).
static bool g_pairs_ready[2][kMaxDevices] = {{false}};
static bool attention_restores(int32_t dtype) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return false;
    return attention_pairs() && g_pairs_ready[dtype == FXR_BF16 ? 1 : 0][dev];
}

template <typename T>
int32_t launch_attention_streams(const fxr_frame_desc* d, int32_t n_streams, const AttnStreamArgs* st,
                                 const SplitArea& split, cudaStream_t stream, bool* restored = nullptr,
                                 int32_t reserve_sms = 0) {
    if (restored) *restored = false;
    NvtxRange nvtx_("fxr:attention");
    if (n_streams < 1 || n_streams > fxr::kMaxBatch) return fail(FXR_ERR_INVALID, "1..%d streams per launch", fxr::kMaxBatch);
    static bool configured[kMaxDevices] = {false};
    static bool pairs_ok[kMaxDevices] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < kMaxDevices && !configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(fxr::attn::attention_kernel<T, false>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)fxr::attn::kSmemBytes);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(fxr::attn::attention_kernel<T, true>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)fxr::attn::kSmemBytes);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(fxr::attn2::attention_kernel<T, false>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)fxr::attn2::kSmemBytes);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(fxr::attn2::attention_kernel<T, true>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)fxr::attn2::kSmemBytes);
        // the two-tile kernel redistributes its launch registers between warpgroups (setmaxnreg):
        // it only runs when the compiled register count gives the CTA enough of them
        cudaFuncAttributes fa{}, fs{};
        if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, fxr::attn2::attention_kernel<T, false>);
        if (e == cudaSuccess) e = cudaFuncGetAttributes(&fs, fxr::attn2::attention_kernel<T, true>);
        if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(attention)");
        pairs_ok[dev] = (uint32_t)fa.numRegs * (uint32_t)fxr::attn2::kThreads >= fxr::attn2::kRegPool &&
                        (uint32_t)fs.numRegs * (uint32_t)fxr::attn2::kThreads >= fxr::attn2::kRegPool;
        g_pairs_ready[std::is_same<T, __nv_bfloat16>::value ? 1 : 0][dev] = pairs_ok[dev];
        configured[dev] = true;
    }
    const int64_t C = (int64_t)d->n_heads * d->head_dim;
    const int64_t N = d->n_tokens;
    fxr::attn::Maps maps;
    std::memset(&maps, 0, sizeof(maps));
    fxr::attn::Params p{};
    int32_t rc;
    for (int32_t b = 0; b < n_streams; ++b) {
        if ((rc = make_tmap(&maps.q[b], st[b].qc, d->dtype, C, N, st[b].ld_qc)) != FXR_OK) return rc;
        if ((rc = make_tmap(&maps.k[b], st[b].ck, d->dtype, C, N, d->ld_cache)) != FXR_OK) return rc;
        if ((rc = make_tmap(&maps.v[b], st[b].cv, d->dtype, C, N, d->ld_cache)) != FXR_OK) return rc;
        p.s[b].count = st[b].count;
        p.s[b].idx = st[b].idx;
        p.s[b].out = st[b].out;
    }
    p.n_streams = n_streams;
    p.split_scratch = split.scratch;
    p.split_cnt = split.cnt;
    p.split_slots = split.slots;
    p.ld_out = d->ld_out;
    p.n_tokens = d->n_tokens;
    p.n_heads = d->n_heads;
    const float scale = d->softmax_scale > 0.f ? d->softmax_scale : 1.0f / std::sqrt((float)d->head_dim);
    p.scale_log2 = scale * 1.4426950408889634f;
    cudaError_t e;
    if (attention_pairs() && dev >= 0 && dev < kMaxDevices && pairs_ok[dev]) {
        // two query tiles per CTA (fxr_attention2.cuh). With scratch slots for a stream-K schedule,
        // the instantiation that can run it, on every SM (the kernel chooses on the device, from M;
        // CTAs without an item exit)
        const bool sk = split.slots >= fxr::attn2::kSlotsPerCta * sm_count();
        // the mask==1 rows of every stream's frame are restored by the kernel's tail
        bool fuse = restored != nullptr;
        for (int32_t b = 0; b < n_streams; ++b) fuse = fuse && st[b].frame != nullptr;
        if (fuse) {
            const size_t eb = dtype_bytes(d->dtype);
            for (int32_t b = 0; b < n_streams; ++b) {
                const Views& w = *st[b].frame;
                p.s[b].restore_rows = w.restore.rows;
                p.s[b].restore_count = w.restore.count;
                p.s[b].head_done = w.restore.head_done;
                p.s[b].restore_idx = w.idx;
                p.s[b].save = static_cast<const uint4*>(w.save);
                p.s[b].cache_k = static_cast<char*>(const_cast<void*>(st[b].ck));
                p.s[b].cache_v = static_cast<char*>(const_cast<void*>(st[b].cv));
            }
            p.ld_cache_bytes = d->ld_cache * (int64_t)eb;
            p.row_vec = (int32_t)((int64_t)d->n_heads * d->head_dim * (int64_t)eb / 16);
            *restored = true;
        }
        const int64_t units = (N + fxr::attn2::kRows - 1) / fxr::attn2::kRows * d->n_heads * n_streams;
        const int ctas = std::max(1, sm_count() - std::max(0, reserve_sms));
        const int grid = sk ? ctas : (int)std::max<int64_t>(1, std::min<int64_t>(units, ctas));
        e = sk ? launch_pdl(fxr::attn2::attention_kernel<T, true>, dim3(grid), dim3(fxr::attn2::kThreads),
                            fxr::attn2::kSmemBytes, stream, maps, p)
               : launch_pdl(fxr::attn2::attention_kernel<T, false>, dim3(grid), dim3(fxr::attn2::kThreads),
                            fxr::attn2::kSmemBytes, stream, maps, p);
    } else {
        // few heads per launch (a GPU's share of a head-split frame, small models): the query tiles
        // x heads may leave SMs idle, so launch the instantiation that can split key ranges
        const bool split_ok = split.slots > 0 && d->n_heads <= kSplitMaxHeads;
        const int grid = split_ok ? sm_count()
                                  : (int)std::min<int64_t>(attention_ctas(N, d->n_heads) * n_streams, sm_count());
        e = split_ok ? launch_pdl(fxr::attn::attention_kernel<T, true>, dim3(grid), dim3(fxr::attn::kThreads),
                                  fxr::attn::kSmemBytes, stream, maps, p)
                     : launch_pdl(fxr::attn::attention_kernel<T, false>, dim3(grid), dim3(fxr::attn::kThreads),
                                  fxr::attn::kSmemBytes, stream, maps, p);
    }
    if (e != cudaSuccess) return cuda_status(e, "attention_kernel launch");
    return FXR_OK;
}

// frame / restored: as for launch_attention_streams (the frame's views, whose mask==1 rows the
// kernel restores when it can; *restored tells whether it will)
template <typename T>
int32_t launch_attention(const fxr_frame_desc* d, const void* qc, int64_t ld_qc, const int32_t* count,
                         const void* ck, const void* cv, const int32_t* idx, const OutSet& os,
                         cudaStream_t stream, const Views* frame = nullptr, bool* restored = nullptr) {
    const AttnStreamArgs st{qc, ld_qc, count, ck, cv, idx, os.out, frame};
    return launch_attention_streams<T>(d, 1, &st, os.split, stream, restored, os.reserve_sms);
}

// Gather of n_streams frames of the same geometry (one launch; rows stream after stream).
// Whether a gather launch over n_streams frames of n_tokens can do the compaction itself (every
// CTA's share of the rows fits its shared-memory list; token and row indices fit the list entries).
static bool gather_can_compact(int32_t n_streams, int32_t n_tokens) {
    const int64_t rows = (int64_t)n_streams * n_tokens;
    const int64_t grid = std::max<int64_t>(1, std::min<int64_t>(sm_count(), n_tokens));
    return n_tokens < (1 << 24) && (rows + grid - 1) / grid <= fxr::kBulkListCap;
}

// Identity output rows that a gather launch writes besides its own work (GatherArgs::iota).
struct RowIota {
    int32_t* idx = nullptr;
    int32_t n = 0, cap = 0;
};

template <typename T>
int32_t launch_gather_streams(const fxr_frame_desc* d, int32_t n_streams, const fxr::GatherStream* gs,
                              const int32_t* pos, const float* nq, const float* nk, int64_t ld_qc,
                              cudaStream_t stream, const float* nq_txt = nullptr,
                              const float* nk_txt = nullptr, int32_t n_text_norm = 0,
                              const SplitArea* compact_split = nullptr, RowIota iota = RowIota{}) {
    NvtxRange nvtx_("fxr:gather");
    if (n_streams < 1 || n_streams > fxr::kMaxBatch) return fail(FXR_ERR_INVALID, "1..%d streams per launch", fxr::kMaxBatch);
    fxr::GatherArgs a{};
    // compact_split != nullptr: the gather compacts the masks itself (gs[b].valid) and zeroes these
    // key-split counters; the caller launched no compaction kernel
    if (compact_split) {
        a.compact = 1;
        a.zero = reinterpret_cast<uint4*>(compact_split->cnt);
        a.zero_vec = (int32_t)((size_t)compact_split->slots * kSplitCntBytes / 16);
    }
    for (int32_t b = 0; b < n_streams; ++b) a.s[b] = gs[b];
    a.n_streams = n_streams;
    a.iota = iota.idx;
    a.iota_n = iota.n;
    a.iota_cap = iota.cap;
    a.pos = pos;
    a.norm_q = nq;
    a.norm_k = nk;
    a.norm_q_txt = nq_txt;
    a.norm_k_txt = nk_txt;
    a.n_text_norm = n_text_norm;
    a.ld_qkv = d->ld_qkv;
    a.ld_qc = ld_qc;
    a.ld_cache = d->ld_cache;
    a.n_tokens = d->n_tokens;
    a.n_heads = d->n_heads;
    a.n_axes = d->rope_n_axes;
    a.eps = d->eps;
    fill_rope(d, &a.rope);
    // bulk-copy pipeline: stages of 3 rows, up to ~190 KB of rows in flight per SM
    const size_t row_bytes = (size_t)d->n_heads * d->head_dim * sizeof(T);
    fxr::BulkLayout lay{};
    lay.stage_bytes = (uint32_t)align_up(3 * row_bytes, 128);
    const size_t budget = 190 * 1024;
    lay.stages = (uint32_t)std::max<size_t>(2, std::min<size_t>(fxr::kBulkMaxStages, budget / lay.stage_bytes));
    const size_t smem = (size_t)lay.stages * lay.stage_bytes + (size_t)lay.stages * fxr::kBulkInfoWords * 4 +
                        (size_t)lay.stages * 16 + (compact_split ? fxr::kBulkListCap * sizeof(uint2) : 0);
    if (smem > 220 * 1024)
        return fail(FXR_ERR_UNSUPPORTED, "gather rows of %zu bytes do not fit the bulk pipeline", row_bytes);
    static bool configured[kMaxDevices] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < kMaxDevices && !configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(fxr::gather_bulk_kernel<T>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024);
        if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(gather)");
        configured[dev] = true;
    }
    const int grid = std::max(1, std::min<int>(sm_count(), d->n_tokens));
    a.grid_magic = grid > 1 ? (uint32_t)(((1ull << 32) + (uint64_t)grid - 1) / (uint64_t)grid) : 0u;
    cudaError_t e = launch_pdl(fxr::gather_bulk_kernel<T>, dim3(grid), dim3(fxr::kBulkThreads), smem,
                               stream, a, lay);
    if (e != cudaSuccess) return cuda_status(e, "gather_bulk_kernel launch");
    return FXR_OK;
}

template <typename T>
int32_t launch_gather(const fxr_frame_desc* d, const void* q, const void* k, const void* v,
                      const int32_t* mask, const int32_t* idx, const int32_t* count,
                      const int32_t* pos, const float* nq, const float* nk, void* qc, int64_t ld_qc,
                      void* ck, void* cv, void* save, cudaStream_t stream) {
    const fxr::GatherStream gs{q, k, v, mask, idx, count, qc, ck, cv, save};
    return launch_gather_streams<T>(d, 1, &gs, pos, nq, nk, ld_qc, stream);
}

}  // namespace

static int32_t check_gather_args(const fxr_frame_desc* desc, const void* q, const void* k, const void* v,
                                 const int32_t* mask, const int32_t* idx, const int32_t* count,
                                 const int32_t* pos, const float* norm_q, const float* norm_k, void* qc,
                                 int64_t ld_qc, void* cache_k, void* cache_v, void* save) {
    if (!q || !k || !v || !mask || !idx || !count || !norm_q || !norm_k || !qc || !cache_k ||
        !cache_v || (desc->rope_n_axes > 0 && !pos))
        return fail(FXR_ERR_INVALID, "null pointer argument");
    if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(qc) || !aligned16(cache_k) ||
        !aligned16(cache_v) || (save && !aligned16(save)) || (ld_qc % 8))
        return fail(FXR_ERR_INVALID, "Q/K/V/qc/cache/save must be 16-byte aligned");
    return FXR_OK;
}

// =============================================================================================
extern "C" {

int32_t fxr_abi_version(void) { return FXR_ABI_VERSION; }

const char* fxr_build_info(void) {
    return "fxr sm_100a: tcgen05/TMEM flash attention + fused gather/RMSNorm/RoPE; nvcc "
#ifdef __CUDACC_VER_MAJOR__
           "12.x"
#endif
        ;
}

const char* fxr_last_error_string(void) { return t_last_error.c_str(); }

int32_t fxr_check_device_error(void* stream, uint32_t* word_out) {
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cuda_status(e, "cudaStreamSynchronize");
    uint32_t w = 0;
    e = cudaMemcpyFromSymbol(&w, fxr::g_error_word, sizeof(w));
    if (e != cudaSuccess) return cuda_status(e, "read error word");
    const uint32_t zero = 0;
    e = cudaMemcpyToSymbol(fxr::g_error_word, &zero, sizeof(zero));
    if (e != cudaSuccess) return cuda_status(e, "clear error word");
    if (word_out) *word_out = w;
    if (w & fxr::kErrTimeout) return fail(FXR_ERR_TIMEOUT, "device wait timed out (word 0x%x)", w);
    if (w) return fail(FXR_ERR_BOUNDS, "a kernel skipped a row index outside its buffer (word 0x%x)", w);
    return FXR_OK;
}

size_t fxr_workspace_size(const fxr_frame_desc* desc) {
    if (!desc || dtype_bytes(desc->dtype) == 0 || desc->n_heads <= 0 || desc->head_dim <= 0) return 0;
    return carve(desc, nullptr).total + split_bytes(kSplitSlotsPerSm * sm_count());
}

size_t fxr_workspace_min_size(const fxr_frame_desc* desc) {
    if (!desc || dtype_bytes(desc->dtype) == 0 || desc->n_heads <= 0 || desc->head_dim <= 0) return 0;
    return carve(desc, nullptr).total;
}

// Device address of g_noalloc_scratch on the current device. The first call on a device resolves
// it with cudaGetSymbolAddress (with that device current); later calls reuse the stored address.
// The host-side name g_noalloc_scratch is only a stand-in and must never be handed to a kernel.
static int32_t noalloc_scratch(void** out) {
    static std::mutex mu;
    static void* addr[kMaxDevices] = {nullptr};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_status(e, "cudaGetDevice");
    if (dev < 0 || dev >= kMaxDevices) return fail(FXR_ERR_UNSUPPORTED, "device ordinal %d too large", dev);
    std::lock_guard<std::mutex> lock(mu);
    if (!addr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return cuda_status(e, "cudaGetSymbolAddress(frame scratch)");
        if (!p) return fail(FXR_ERR_CUDA, "cudaGetSymbolAddress returned a null frame scratch");
        addr[dev] = p;
    }
    *out = addr[dev];
    return FXR_OK;
}

int32_t fxr_frame_forward_noalloc(const fxr_frame_desc* desc, const void* q, const void* k,
                                  const void* v, int32_t* mask, const uint8_t* valid,
                                  const int32_t* pos, const float* norm_q, const float* norm_k,
                                  void* cache_k, void* cache_v, void* out, void* stream) {
    int32_t st = check_desc(desc, true);
    if (st != FXR_OK) return st;
    if (desc->n_tokens == 0) return FXR_OK;
    const size_t need = carve(desc, nullptr).total;
    if (need > kNoAllocScratchBytes)
        return fail(FXR_ERR_WORKSPACE,
                    "frame needs %zu bytes of scratch but the built-in scratch of "
                    "fxr_frame_forward_noalloc holds %zu; use fxr_frame_forward with a caller workspace",
                    need, kNoAllocScratchBytes);
    void* scratch = nullptr;
    if ((st = noalloc_scratch(&scratch)) != FXR_OK) return st;
    return fxr_frame_forward(desc, q, k, v, mask, valid, pos, norm_q, norm_k, cache_k, cache_v, out,
                             scratch, kNoAllocScratchBytes, stream);
}

int32_t fxr_workspace_views(const fxr_frame_desc* desc, void* workspace, int32_t** idx,
                            int32_t** count, void** qc, int64_t* ld_qc, void** save) {
    if (!desc || !workspace) return fail(FXR_ERR_INVALID, "null descriptor or workspace");
    Views v = carve(desc, workspace);
    if (idx) *idx = v.idx;
    if (count) *count = v.count;
    if (qc) *qc = v.qc;
    if (ld_qc) *ld_qc = v.ld_qc;
    if (save) *save = v.save;
    return FXR_OK;
}

// Compaction of n_streams frames (CTA b: stream b); the attention's split counters of the launch
// start at zero.
static int32_t launch_compact_streams(fxr::CompactArgs a, int32_t n_streams, int32_t n_tokens,
                                      const SplitArea& split, void* stream, void* zero2 = nullptr,
                                      size_t zero2_bytes = 0, int32_t n_force = 0, int32_t n_heads = 0) {
    NvtxRange nvtx_("fxr:compact");
    a.n = n_tokens;
    a.n_heads = n_heads;
    a.zero2 = reinterpret_cast<uint4*>(zero2);
    a.zero2_vec = (int32_t)(zero2_bytes / 16);
    a.n_force = n_force;
    a.zero = reinterpret_cast<uint4*>(split.cnt);
    a.zero_vec = (int32_t)((size_t)split.slots * kSplitCntBytes / 16);
    cudaError_t e = launch_pdl(fxr::compact_kernel, dim3(n_streams), dim3(fxr::kCompactThreads), 0,
                               static_cast<cudaStream_t>(stream), a);
    if (e != cudaSuccess) return cuda_status(e, "compact_kernel launch");
    return FXR_OK;
}

// restore: the mask==1 list of a frame's workspace (and its heads' counters), or nullptr
static int32_t launch_compact(int32_t* mask, const uint8_t* valid, int32_t n_tokens, int32_t* idx,
                              int32_t* count, const SplitArea& split, void* stream,
                              const fxr::RestoreList* restore = nullptr, int32_t n_heads = 0) {
    if (n_tokens < 0) return fail(FXR_ERR_INVALID, "n_tokens < 0");
    if (!count || (n_tokens > 0 && (!mask || !idx))) return fail(FXR_ERR_INVALID, "null pointer");
    fxr::CompactArgs a{};
    a.s[0] = fxr::CompactStream{mask, valid, idx, count, restore ? *restore : fxr::RestoreList{}};
    return launch_compact_streams(a, 1, n_tokens, split, stream, nullptr, 0, 0, n_heads);
}

int32_t fxr_mask_compact(int32_t* mask, const uint8_t* valid, int32_t n_tokens, int32_t* idx,
                         int32_t* count, void* stream) {
    return launch_compact(mask, valid, n_tokens, idx, count, SplitArea{}, stream);
}

int32_t fxr_preprocess_mask(int32_t* mask, const uint8_t* valid, int32_t n_tokens, void* stream) {
    if (n_tokens < 0) return fail(FXR_ERR_INVALID, "n_tokens < 0");
    if (n_tokens == 0) return FXR_OK;
    if (!mask || !valid) return fail(FXR_ERR_INVALID, "null pointer");
    fxr::preprocess_mask_kernel<<<(n_tokens + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        mask, valid, n_tokens);
    FXR_CHECK_LAUNCH("preprocess_mask_kernel launch");
    return FXR_OK;
}

int32_t fxr_mark_updated(const int32_t* mask, uint8_t* valid, int32_t n_text, int32_t n_tokens,
                         void* stream) {
    if (n_tokens < 0 || n_text < 0) return fail(FXR_ERR_INVALID, "negative size");
    if (n_tokens <= n_text) return FXR_OK;
    if (!mask || !valid) return fail(FXR_ERR_INVALID, "null pointer");
    const int32_t n_img = n_tokens - n_text;
    fxr::mark_updated_kernel<<<(n_img + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        mask, valid, n_text, n_tokens);
    FXR_CHECK_LAUNCH("mark_updated_kernel launch");
    return FXR_OK;
}

void fxr_internal_set_error(const char* msg) { t_last_error = msg ? msg : ""; }

int32_t fxr_gather_norm_rope(const fxr_frame_desc* desc, const void* q, const void* k,
                             const void* v, const int32_t* mask, const int32_t* idx,
                             const int32_t* count, const int32_t* pos, const float* norm_q,
                             const float* norm_k, void* qc, int64_t ld_qc, void* cache_k,
                             void* cache_v, void* save, void* stream) {
    int32_t st = check_desc(desc, false);
    if (st != FXR_OK) return st;
    if (desc->n_tokens == 0) return FXR_OK;
    if ((st = check_gather_args(desc, q, k, v, mask, idx, count, pos, norm_q, norm_k, qc, ld_qc, cache_k,
                                cache_v, save)) != FXR_OK)
        return st;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (desc->dtype == FXR_BF16)
        return launch_gather<__nv_bfloat16>(desc, q, k, v, mask, idx, count, pos, norm_q, norm_k, qc,
                                            ld_qc, cache_k, cache_v, save, s);
    return launch_gather<__half>(desc, q, k, v, mask, idx, count, pos, norm_q, norm_k, qc, ld_qc,
                                 cache_k, cache_v, save, s);
}

int32_t fxr_attention_active(const fxr_frame_desc* desc, const void* qc, int64_t ld_qc,
                             const int32_t* count, const void* cache_k, const void* cache_v,
                             const int32_t* idx, void* out, void* stream) {
    int32_t st = check_desc(desc, true);
    if (st != FXR_OK) return st;
    if (desc->n_tokens == 0) return FXR_OK;
    if (!qc || !count || !cache_k || !cache_v || !idx || !out)
        return fail(FXR_ERR_INVALID, "null pointer argument");
    if (!aligned16(qc) || !aligned16(cache_k) || !aligned16(cache_v) || !aligned16(out) ||
        (ld_qc % 8) || ld_qc < (int64_t)desc->n_heads * desc->head_dim)
        return fail(FXR_ERR_INVALID, "qc/cache/out must be 16-byte aligned with ld_qc >= C, %% 8");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    OutSet os;
    os.out = out;
    if (desc->dtype == FXR_BF16)
        return launch_attention<__nv_bfloat16>(desc, qc, ld_qc, count, cache_k, cache_v, idx, os, s);
    return launch_attention<__half>(desc, qc, ld_qc, count, cache_k, cache_v, idx, os, s);
}

static int32_t launch_restore_streams(const fxr_frame_desc* desc, fxr::RestoreArgs a, int32_t n_streams,
                                     void* stream) {
    const int64_t row_bytes = (int64_t)desc->n_heads * desc->head_dim * (int64_t)dtype_bytes(desc->dtype);
    a.ld_cache_bytes = desc->ld_cache * (int64_t)dtype_bytes(desc->dtype);
    a.row_vec = (int32_t)(row_bytes / 16);
    a.n_tokens = desc->n_tokens;
    // one CTA per SM at most: usually no row has mask 1 and the kernel only scans M mask values
    const int grid = std::max(1, std::min(grid_rows(desc->n_tokens, 8), sm_count() / n_streams));
    cudaError_t e = launch_pdl(fxr::restore_rows_kernel, dim3(grid, n_streams), dim3(256), 0,
                               static_cast<cudaStream_t>(stream), a);
    if (e != cudaSuccess) return cuda_status(e, "restore_rows_kernel launch");
    return FXR_OK;
}

int32_t fxr_restore_rows(const fxr_frame_desc* desc, const int32_t* mask, const int32_t* idx,
                         const int32_t* count, const void* save, void* cache_k, void* cache_v,
                         void* stream) {
    NvtxRange nvtx_("fxr:restore");
    int32_t st = check_desc(desc, false);
    if (st != FXR_OK) return st;
    if (desc->n_tokens == 0) return FXR_OK;
    if (!mask || !idx || !count || !save || !cache_k || !cache_v)
        return fail(FXR_ERR_INVALID, "null pointer argument");
    if (!aligned16(save) || !aligned16(cache_k) || !aligned16(cache_v))
        return fail(FXR_ERR_INVALID, "save/cache must be 16-byte aligned");
    fxr::RestoreArgs a{};
    a.s[0] = fxr::RestoreStream{mask, idx, count, static_cast<const uint4*>(save), static_cast<char*>(cache_k),
                                static_cast<char*>(cache_v)};
    return launch_restore_streams(desc, a, 1, stream);
}

static int32_t rows_copy(bool scatter, const void* src, int64_t ld_src, const int32_t* idx,
                         const int32_t* count, int32_t host_count, void* dst, int64_t ld_dst,
                         int64_t row_bytes, int32_t n_index_rows, void* stream) {
    const int32_t n_rows = n_index_rows > 0 ? n_index_rows : INT32_MAX;
    if (!count && host_count < 0) return fail(FXR_ERR_INVALID, "need a device count or host_count >= 0");
    if (!count && host_count == 0) return FXR_OK;
    if (!src || !dst || !idx || row_bytes <= 0) return fail(FXR_ERR_INVALID, "null pointer or row_bytes <= 0");
    const int64_t rows_hint = count ? (int64_t)1 << 16 : host_count;
    const int grid = grid_rows(rows_hint, 8);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const char* sp = static_cast<const char*>(src);
    char* dp = static_cast<char*>(dst);
    const bool v16 = aligned16(src) && aligned16(dst) && row_bytes % 16 == 0 && ld_src % 16 == 0 &&
                     ld_dst % 16 == 0;
    const bool v4 = ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 3) == 0 &&
                    row_bytes % 4 == 0 && ld_src % 4 == 0 && ld_dst % 4 == 0;
    if (v16) {
        if (scatter)
            fxr::rows_copy_kernel<uint4, true><<<grid, 256, 0, s>>>(sp, ld_src, idx, count, host_count, dp, ld_dst, row_bytes / 16, n_rows);
        else
            fxr::rows_copy_kernel<uint4, false><<<grid, 256, 0, s>>>(sp, ld_src, idx, count, host_count, dp, ld_dst, row_bytes / 16, n_rows);
    } else if (v4) {
        if (scatter)
            fxr::rows_copy_kernel<uint32_t, true><<<grid, 256, 0, s>>>(sp, ld_src, idx, count, host_count, dp, ld_dst, row_bytes / 4, n_rows);
        else
            fxr::rows_copy_kernel<uint32_t, false><<<grid, 256, 0, s>>>(sp, ld_src, idx, count, host_count, dp, ld_dst, row_bytes / 4, n_rows);
    } else {
        if (scatter)
            fxr::rows_copy_kernel<uint8_t, true><<<grid, 256, 0, s>>>(sp, ld_src, idx, count, host_count, dp, ld_dst, row_bytes, n_rows);
        else
            fxr::rows_copy_kernel<uint8_t, false><<<grid, 256, 0, s>>>(sp, ld_src, idx, count, host_count, dp, ld_dst, row_bytes, n_rows);
    }
    FXR_CHECK_LAUNCH("rows_copy_kernel launch");
    return FXR_OK;
}

int32_t fxr_gather_rows(const void* src, int64_t ld_src_bytes, const int32_t* idx,
                        const int32_t* count, int32_t host_count, void* dst, int64_t ld_dst_bytes,
                        int64_t row_bytes, int32_t n_index_rows, void* stream) {
    return rows_copy(false, src, ld_src_bytes, idx, count, host_count, dst, ld_dst_bytes, row_bytes,
                     n_index_rows, stream);
}

int32_t fxr_scatter_rows(const void* src, int64_t ld_src_bytes, const int32_t* idx,
                         const int32_t* count, int32_t host_count, void* dst, int64_t ld_dst_bytes,
                         int64_t row_bytes, int32_t n_index_rows, void* stream) {
    return rows_copy(true, src, ld_src_bytes, idx, count, host_count, dst, ld_dst_bytes, row_bytes,
                     n_index_rows, stream);
}

int32_t fxr_kv_sync(void* keys, void* values, void* cached_keys, void* cached_values,
                    const int32_t* mask, int32_t n_tokens, int64_t row_elems, int32_t dtype,
                    void* stream) {
    const size_t eb = dtype_bytes(dtype);
    if (eb == 0) return fail(FXR_ERR_INVALID, "bad dtype %d", dtype);
    if (n_tokens < 0 || row_elems < 0) return fail(FXR_ERR_INVALID, "negative size");
    if (n_tokens == 0 || row_elems == 0) return FXR_OK;
    if (!keys || !values || !cached_keys || !cached_values || !mask)
        return fail(FXR_ERR_INVALID, "null pointer argument");
    const int64_t row_bytes = row_elems * (int64_t)eb;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int64_t cap = (int64_t)sm_count() * 16;
    const bool v16 = aligned16(keys) && aligned16(values) && aligned16(cached_keys) &&
                     aligned16(cached_values) && row_bytes % 16 == 0;
    if (v16) {
        const int64_t words = row_bytes / 16, total = words * n_tokens;
        const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((total + 255) / 256, cap));
        fxr::kv_sync_kernel<uint4><<<grid, 256, 0, s>>>(static_cast<uint4*>(keys), static_cast<uint4*>(values),
                                                        static_cast<uint4*>(cached_keys), static_cast<uint4*>(cached_values),
                                                        mask, n_tokens, words);
    } else {
        const int64_t words = row_bytes / (int64_t)eb, total = words * n_tokens;
        const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((total + 255) / 256, cap));
        if (eb == 4)
            fxr::kv_sync_kernel<uint32_t><<<grid, 256, 0, s>>>(static_cast<uint32_t*>(keys), static_cast<uint32_t*>(values),
                                                               static_cast<uint32_t*>(cached_keys), static_cast<uint32_t*>(cached_values),
                                                               mask, n_tokens, words);
        else
            fxr::kv_sync_kernel<uint16_t><<<grid, 256, 0, s>>>(static_cast<uint16_t*>(keys), static_cast<uint16_t*>(values),
                                                               static_cast<uint16_t*>(cached_keys), static_cast<uint16_t*>(cached_values),
                                                               mask, n_tokens, words);
    }
    FXR_CHECK_LAUNCH("kv_sync_kernel launch");
    return FXR_OK;
}

int32_t fxr_output_cache_sync(void* pred, void* cache, const int32_t* mask, uint8_t* valid,
                              int32_t n_text, int32_t n_image, int32_t channels, int32_t dtype,
                              void* stream) {
    const size_t eb = dtype_bytes(dtype);
    if (eb == 0) return fail(FXR_ERR_INVALID, "bad dtype %d", dtype);
    if (n_text < 0 || n_image < 0 || channels < 0) return fail(FXR_ERR_INVALID, "negative size");
    if (n_image == 0 || channels == 0) return FXR_OK;
    if (!pred || !cache || !mask || !valid) return fail(FXR_ERR_INVALID, "null pointer argument");
    const int64_t row_bytes = (int64_t)channels * (int64_t)eb;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int64_t cap = (int64_t)sm_count() * 16;
    if (aligned16(pred) && aligned16(cache) && row_bytes % 16 == 0) {
        const int64_t words = row_bytes / 16, total = words * n_image;
        const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((total + 255) / 256, cap));
        fxr::out_cache_sync_kernel<uint4><<<grid, 256, 0, s>>>(static_cast<uint4*>(pred), static_cast<uint4*>(cache),
                                                               mask, valid, n_text, n_image, words);
    } else {
        const int64_t words = channels, total = words * n_image;
        const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((total + 255) / 256, cap));
        if (eb == 4)
            fxr::out_cache_sync_kernel<uint32_t><<<grid, 256, 0, s>>>(static_cast<uint32_t*>(pred), static_cast<uint32_t*>(cache),
                                                                      mask, valid, n_text, n_image, words);
        else
            fxr::out_cache_sync_kernel<uint16_t><<<grid, 256, 0, s>>>(static_cast<uint16_t*>(pred), static_cast<uint16_t*>(cache),
                                                                      mask, valid, n_text, n_image, words);
    }
    FXR_CHECK_LAUNCH("out_cache_sync_kernel launch");
    return FXR_OK;
}

int32_t fxr_rms_norm(const void* x, void* y, const float* w, float eps, int64_t rows, int32_t dim,
                     int32_t dtype, void* stream) {
    if (rows < 0 || dim < 0) return fail(FXR_ERR_INVALID, "negative size");
    if (rows == 0 || dim == 0) return FXR_OK;
    if (!x || !y || !w) return fail(FXR_ERR_INVALID, "null pointer argument");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int grid = grid_rows(rows, 8);
    switch (dtype) {
        case FXR_F32:
            fxr::rms_norm_kernel<float><<<grid, 256, 0, s>>>(static_cast<const float*>(x), static_cast<float*>(y), w, eps, rows, dim);
            break;
        case FXR_F16:
            fxr::rms_norm_kernel<__half><<<grid, 256, 0, s>>>(static_cast<const __half*>(x), static_cast<__half*>(y), w, eps, rows, dim);
            break;
        case FXR_BF16:
            fxr::rms_norm_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x), static_cast<__nv_bfloat16*>(y), w, eps, rows, dim);
            break;
        default:
            return fail(FXR_ERR_INVALID, "bad dtype %d", dtype);
    }
    FXR_CHECK_LAUNCH("rms_norm_kernel launch");
    return FXR_OK;
}

int32_t fxr_layer_norm_f32(const float* x, float* y, const float* gamma, const float* beta, float eps,
                           int64_t rows, int32_t dim, void* stream) {
    if (rows < 0 || dim < 0) return fail(FXR_ERR_INVALID, "negative size");
    if (rows == 0 || dim == 0) return FXR_OK;
    if (!x || !y) return fail(FXR_ERR_INVALID, "null pointer argument");
    fxr::layer_norm_f32_kernel<<<grid_rows(rows, 8), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        x, y, gamma, beta, eps, rows, dim);
    FXR_CHECK_LAUNCH("layer_norm_f32_kernel launch");
    return FXR_OK;
}

int32_t fxr_modulate_f32(const float* x, const float* scale, const float* shift, float* out, int64_t rows,
                         int32_t dim, void* stream) {
    if (rows < 0 || dim < 0) return fail(FXR_ERR_INVALID, "negative size");
    if (rows == 0 || dim == 0) return FXR_OK;
    if (!x || !scale || !shift || !out) return fail(FXR_ERR_INVALID, "null pointer argument");
    const int64_t total = rows * dim;
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((total + 255) / 256, (int64_t)sm_count() * 16));
    fxr::modulate_f32_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(x, scale, shift, out, rows, dim);
    FXR_CHECK_LAUNCH("modulate_f32_kernel launch");
    return FXR_OK;
}

}  // extern "C"

template <int kOp>
static int32_t launch_ew(const fxr::EwArgs& a, bool vec_ok, cudaStream_t s) {
    const bool vec = vec_ok && a.n % 4 == 0 && aligned16(a.x) && aligned16(a.out) && (!a.y || aligned16(a.y));
    const int64_t work = vec ? a.n / 4 : a.n;
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((work + 255) / 256, (int64_t)sm_count() * 16));
    if (vec)
        fxr::ew_f32_kernel<kOp, true><<<grid, 256, 0, s>>>(a);
    else
        fxr::ew_f32_kernel<kOp, false><<<grid, 256, 0, s>>>(a);
    FXR_CHECK_LAUNCH("ew_f32_kernel launch");
    return FXR_OK;
}

extern "C" {

int32_t fxr_gelu_tanh_f32(float* data, int64_t n, void* stream) {
    if (n < 0) return fail(FXR_ERR_INVALID, "negative size");
    if (n == 0) return FXR_OK;
    if (!data) return fail(FXR_ERR_INVALID, "null pointer argument");
    fxr::EwArgs a{data, nullptr, data, n, 1, 0.f};
    return launch_ew<fxr::kEwGelu>(a, true, static_cast<cudaStream_t>(stream));
}

int32_t fxr_bias_add_f32(float* data, const float* bias, int64_t rows, int32_t dim, void* stream) {
    if (rows < 0 || dim < 0) return fail(FXR_ERR_INVALID, "negative size");
    if (rows == 0 || dim == 0) return FXR_OK;
    if (!data || !bias) return fail(FXR_ERR_INVALID, "null pointer argument");
    fxr::EwArgs a{data, bias, data, rows * dim, dim, 0.f};
    return launch_ew<fxr::kEwBias>(a, dim % 4 == 0, static_cast<cudaStream_t>(stream));
}

int32_t fxr_add_f32(const float* x, const float* y, float* z, int64_t n, void* stream) {
    if (n < 0) return fail(FXR_ERR_INVALID, "negative size");
    if (n == 0) return FXR_OK;
    if (!x || !y || !z) return fail(FXR_ERR_INVALID, "null pointer argument");
    fxr::EwArgs a{x, y, z, n, 1, 0.f};
    return launch_ew<fxr::kEwAdd>(a, true, static_cast<cudaStream_t>(stream));
}

int32_t fxr_scale_add_f32(const float* x, const float* y, float* out, float gate, int64_t n, void* stream) {
    if (n < 0) return fail(FXR_ERR_INVALID, "negative size");
    if (n == 0) return FXR_OK;
    if (!x || !y || !out) return fail(FXR_ERR_INVALID, "null pointer argument");
    fxr::EwArgs a{x, y, out, n, 1, gate};
    return launch_ew<fxr::kEwScaleAdd>(a, true, static_cast<cudaStream_t>(stream));
}

int32_t fxr_attention_f32_bhsd(const float* q, const float* k, const float* v, float* out,
                               int32_t batch, int32_t num_heads, int32_t q_len, int32_t kv_len,
                               int32_t head_dim, void* stream) {
    if (batch < 0 || num_heads < 0 || q_len < 0 || kv_len < 0 || head_dim < 0)
        return fail(FXR_ERR_INVALID, "negative size");
    if (batch == 0 || num_heads == 0 || q_len == 0 || kv_len == 0 || head_dim == 0) return FXR_OK;
    if (head_dim > fxr::kF32AttnMaxD)
        return fail(FXR_ERR_UNSUPPORTED, "head_dim %d > %d", head_dim, fxr::kF32AttnMaxD);
    if (!q || !k || !v || !out) return fail(FXR_ERR_INVALID, "null pointer argument");
    const size_t smem = fxr::f32_attention_smem(head_dim);
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(fxr::attention_f32_bhsd_kernel,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(attention_f32)");
    }
    const dim3 grid((q_len + fxr::kF32AttnWarps - 1) / fxr::kF32AttnWarps, batch * num_heads);
    const float scale = 1.0f / std::sqrt((float)head_dim);
    fxr::attention_f32_bhsd_kernel<<<grid, fxr::kF32AttnWarps * 32, smem, static_cast<cudaStream_t>(stream)>>>(
        q, k, v, out, q_len, kv_len, head_dim, scale);
    FXR_CHECK_LAUNCH("attention_f32_bhsd_kernel launch");
    return FXR_OK;
}

// Device-side addresses of a host-buffer frame's page-locked rows (fxr_frame_forward_host).
struct HostIo {
    const void* q;
    const void* k;
    const void* v;
    void* out;
};

// Executed rows idx[0..M) of n tensors from src to dst at the same row positions (one side mapped
// host memory), chained to the previous launch on the stream.
// SMs the attention of a host-resident frame leaves to the zero-copy row transfers (which reach the
// PCIe rate from 32 CTAs of 64 threads: four per SM fit there)
constexpr int kHostReserveSms = 8;

static int32_t launch_host_rows(const void* const* src, void* const* dst, int n, int64_t ld_elems,
                                int64_t row_bytes, size_t elem_bytes, const int32_t* idx,
                                const int32_t* count, int32_t n_tokens, cudaStream_t s) {
    fxr::HostRowsArgs a{};
    for (int t = 0; t < n; ++t) {
        a.src[t] = static_cast<const uint4*>(src[t]);
        a.dst[t] = static_cast<uint4*>(dst[t]);
    }
    a.idx = idx;
    a.count = count;
    a.ld_vec = ld_elems * (int64_t)elem_bytes / 16;
    a.row_vec = (int32_t)(row_bytes / 16);
    a.n_tensors = n;
    a.n_tokens = n_tokens;
    const int grid = std::min(fxr::kHostRowsCtas, sm_count());
    // the same L1 / shared-memory split as the persistent GEMM, gather and attention kernels: an SM
    // runs CTAs of two kernels side by side only when their carveouts agree
    cudaError_t e = cudaFuncSetAttribute(fxr::host_rows_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                         (int)cudaSharedmemCarveoutMaxShared);
    if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(host_rows_kernel)");
    e = launch_pdl(fxr::host_rows_kernel, dim3(grid), dim3(fxr::kHostRowsThreads), 0, s, a);
    if (e != cudaSuccess) return cuda_status(e, "host_rows_kernel launch");
    return FXR_OK;
}

static int32_t frame_forward_impl(const fxr_frame_desc* desc, const void* q, const void* k, const void* v,
                                  int32_t* mask, const uint8_t* valid, const int32_t* pos,
                                  const float* norm_q, const float* norm_k, void* cache_k, void* cache_v,
                                  void* out, void* workspace, size_t workspace_bytes, void* stream,
                                  const HostIo* host) {
    NvtxRange nvtx_("fxr:frame");
    int32_t st = check_desc(desc, true);
    if (st != FXR_OK) return st;
    if (desc->n_tokens == 0) return FXR_OK;
    if (!workspace) return fail(FXR_ERR_INVALID, "null workspace");
    const Views w = carve(desc, workspace);
    if (workspace_bytes < w.total)
        return fail(FXR_ERR_WORKSPACE, "workspace %zu < required %zu", workspace_bytes, w.total);
    if (!aligned16(workspace)) return fail(FXR_ERR_INVALID, "workspace must be 16-byte aligned");
    const SplitArea split = split_area(w.total, workspace, workspace_bytes, desc->n_heads);
    // device-resident frames: the gather compacts the mask itself (one launch fewer); host-resident
    // ones need the index list before the gather, for the row upload
    const bool fused = !host && gather_can_compact(1, desc->n_tokens);
    if (!fused && (st = launch_compact(mask, valid, desc->n_tokens, w.idx, w.count, split, stream, &w.restore,
                                       desc->n_heads)) != FXR_OK)
        return st;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const size_t eb = dtype_bytes(desc->dtype);
    const int64_t row_bytes = (int64_t)desc->n_heads * desc->head_dim * (int64_t)eb;
    if (host) {
        const void* src[3] = {host->q, host->k, host->v};
        void* dst[3] = {const_cast<void*>(q), const_cast<void*>(k), const_cast<void*>(v)};
        if ((st = launch_host_rows(src, dst, 3, desc->ld_qkv, row_bytes, eb, w.idx, w.count, desc->n_tokens,
                                   s)) != FXR_OK)
            return st;
    }
    if (!cache_k || !cache_v || !out || !aligned16(cache_k) || !aligned16(cache_v) || !aligned16(out))
        return fail(FXR_ERR_INVALID, "cache/out must be non-null and 16-byte aligned");
    if (fused) {
        if ((st = check_gather_args(desc, q, k, v, mask, w.idx, w.count, pos, norm_q, norm_k, w.qc, w.ld_qc,
                                    cache_k, cache_v, w.save)) != FXR_OK)
            return st;
        fxr::GatherStream gs{q, k, v, mask, w.idx, w.count, w.qc, cache_k, cache_v, w.save, valid, w.restore};
        st = desc->dtype == FXR_BF16
                 ? launch_gather_streams<__nv_bfloat16>(desc, 1, &gs, pos, norm_q, norm_k, w.ld_qc, s, nullptr,
                                                        nullptr, 0, &split)
                 : launch_gather_streams<__half>(desc, 1, &gs, pos, norm_q, norm_k, w.ld_qc, s, nullptr, nullptr, 0,
                                                 &split);
    } else {
        st = fxr_gather_norm_rope(desc, q, k, v, mask, w.idx, w.count, pos, norm_q, norm_k, w.qc, w.ld_qc,
                                  cache_k, cache_v, w.save, stream);
    }
    if (st != FXR_OK) return st;
    OutSet os;
    os.out = out;
    os.split = split;
    // host-resident frames: leave SMs to the row transfers of the frames before and after this one
    os.reserve_sms = host ? kHostReserveSms : 0;
    bool restored = false;
    st = desc->dtype == FXR_BF16
             ? launch_attention<__nv_bfloat16>(desc, w.qc, w.ld_qc, w.count, cache_k, cache_v, w.idx, os, s, &w,
                                               &restored)
             : launch_attention<__half>(desc, w.qc, w.ld_qc, w.count, cache_k, cache_v, w.idx, os, s, &w, &restored);
    if (st != FXR_OK) return st;
    if (!restored && (st = fxr_restore_rows(desc, mask, w.idx, w.count, w.save, cache_k, cache_v, stream)) != FXR_OK)
        return st;
    if (host) {
        const void* src[1] = {out};
        void* dst[1] = {host->out};
        return launch_host_rows(src, dst, 1, desc->ld_out, row_bytes, eb, w.idx, w.count, desc->n_tokens, s);
    }
    return FXR_OK;
}

int32_t fxr_frame_forward(const fxr_frame_desc* desc, const void* q, const void* k, const void* v,
                          int32_t* mask, const uint8_t* valid, const int32_t* pos,
                          const float* norm_q, const float* norm_k, void* cache_k, void* cache_v,
                          void* out, void* workspace, size_t workspace_bytes, void* stream) {
    return frame_forward_impl(desc, q, k, v, mask, valid, pos, norm_q, norm_k, cache_k, cache_v, out,
                              workspace, workspace_bytes, stream, nullptr);
}

// One step of fxr_frame_forward on its workspace layout (same index list, compact queries, save rows
// and split scratch), so that a step run on its own launches what the frame launches.
int32_t fxr_frame_step(int32_t step, const fxr_frame_desc* desc, const void* q, const void* k, const void* v,
                       int32_t* mask, const uint8_t* valid, const int32_t* pos, const float* norm_q,
                       const float* norm_k, void* cache_k, void* cache_v, void* out, void* workspace,
                       size_t workspace_bytes, void* stream) {
    NvtxRange nvtx_("fxr:frame_step");
    int32_t st = check_desc(desc, true);
    if (st != FXR_OK) return st;
    if (step < FXR_STEP_COMPACT || step > FXR_STEP_RESTORE) return fail(FXR_ERR_INVALID, "unknown frame step %d", step);
    if (desc->n_tokens == 0) return FXR_OK;
    if (!workspace) return fail(FXR_ERR_INVALID, "null workspace");
    const Views w = carve(desc, workspace);
    if (workspace_bytes < w.total)
        return fail(FXR_ERR_WORKSPACE, "workspace %zu < required %zu", workspace_bytes, w.total);
    if (!aligned16(workspace)) return fail(FXR_ERR_INVALID, "workspace must be 16-byte aligned");
    const SplitArea split = split_area(w.total, workspace, workspace_bytes, desc->n_heads);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    switch (step) {
    case FXR_STEP_COMPACT:
        return launch_compact(mask, valid, desc->n_tokens, w.idx, w.count, split, stream, &w.restore, desc->n_heads);
    case FXR_STEP_GATHER:
    case FXR_STEP_GATHER_COMPACT: {
        if (!cache_k || !cache_v || !aligned16(cache_k) || !aligned16(cache_v))
            return fail(FXR_ERR_INVALID, "cache must be non-null and 16-byte aligned");
        if (step == FXR_STEP_GATHER)
            return fxr_gather_norm_rope(desc, q, k, v, mask, w.idx, w.count, pos, norm_q, norm_k, w.qc, w.ld_qc,
                                        cache_k, cache_v, w.save, stream);
        if (!gather_can_compact(1, desc->n_tokens))
            return fail(FXR_ERR_UNSUPPORTED, "frame too large for the compacting gather");
        if ((st = check_gather_args(desc, q, k, v, mask, w.idx, w.count, pos, norm_q, norm_k, w.qc, w.ld_qc,
                                    cache_k, cache_v, w.save)) != FXR_OK)
            return st;
        fxr::GatherStream gs{q, k, v, mask, w.idx, w.count, w.qc, cache_k, cache_v, w.save, valid, w.restore};
        return desc->dtype == FXR_BF16
                   ? launch_gather_streams<__nv_bfloat16>(desc, 1, &gs, pos, norm_q, norm_k, w.ld_qc, s, nullptr,
                                                          nullptr, 0, &split)
                   : launch_gather_streams<__half>(desc, 1, &gs, pos, norm_q, norm_k, w.ld_qc, s, nullptr, nullptr, 0,
                                                   &split);
    }
    case FXR_STEP_ATTENTION: {
        if (!cache_k || !cache_v || !out || !aligned16(cache_k) || !aligned16(cache_v) || !aligned16(out))
            return fail(FXR_ERR_INVALID, "cache/out must be non-null and 16-byte aligned");
        OutSet os;
        os.out = out;
        os.split = split;
        bool restored = false;
        return desc->dtype == FXR_BF16
                   ? launch_attention<__nv_bfloat16>(desc, w.qc, w.ld_qc, w.count, cache_k, cache_v, w.idx, os, s,
                                                     &w, &restored)
                   : launch_attention<__half>(desc, w.qc, w.ld_qc, w.count, cache_k, cache_v, w.idx, os, s, &w,
                                              &restored);
    }
    default:
        // nothing left to do when the two-tile attention restored the rows in its tail
        if (attention_restores(desc->dtype)) return FXR_OK;
        return fxr_restore_rows(desc, mask, w.idx, w.count, w.save, cache_k, cache_v, stream);
    }
}

// Staging rows of a host-buffer frame at the start of its workspace: the mask copy, then Q, K, V
// (row stride ld_qkv) and the output (ld_out); the frame's own workspace follows.
struct HostStage {
    int32_t* mask;
    void* q;
    void* k;
    void* v;
    void* out;
    size_t total;
};

static HostStage carve_host(const fxr_frame_desc* d, void* ws) {
    HostStage h{};
    const size_t N = (size_t)(d->n_tokens > 0 ? d->n_tokens : 1);
    const size_t eb = dtype_bytes(d->dtype);
    char* b = static_cast<char*>(ws);
    size_t off = 0;
    auto take = [&](size_t bytes) {
        void* p = b ? b + off : nullptr;
        off += align_up(bytes, 256);
        return p;
    };
    h.mask = static_cast<int32_t*>(take(N * sizeof(int32_t)));
    h.q = take(N * (size_t)d->ld_qkv * eb);
    h.k = take(N * (size_t)d->ld_qkv * eb);
    h.v = take(N * (size_t)d->ld_qkv * eb);
    h.out = take(N * (size_t)d->ld_out * eb);
    h.total = off;
    return h;
}

size_t fxr_frame_host_workspace_size(const fxr_frame_desc* desc) {
    if (check_desc(desc, true) != FXR_OK) return 0;
    return carve_host(desc, nullptr).total + fxr_workspace_size(desc);
}

// Device-side address of page-locked, mapped host memory covering [p, p + bytes); null otherwise
// (pageable memory, device memory, or a range whose two ends do not map contiguously).
static const void* mapped_host_range(const void* p, size_t bytes) {
    if (!p || bytes == 0) return nullptr;
    cudaPointerAttributes a0{}, a1{};
    const char* last = static_cast<const char*>(p) + bytes - 1;
    if (cudaPointerGetAttributes(&a0, p) != cudaSuccess || cudaPointerGetAttributes(&a1, last) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    if (a0.type != cudaMemoryTypeHost || a1.type != cudaMemoryTypeHost || !a0.devicePointer ||
        static_cast<const char*>(a1.devicePointer) != static_cast<const char*>(a0.devicePointer) + bytes - 1)
        return nullptr;
    return a0.devicePointer;
}

int32_t fxr_frame_forward_host(const fxr_frame_desc* desc, const void* host_q, const void* host_k,
                               const void* host_v, const int32_t* host_mask, const uint8_t* valid,
                               const int32_t* pos, const float* norm_q, const float* norm_k, void* cache_k,
                               void* cache_v, void* host_out, void* workspace, size_t workspace_bytes,
                               void* stream) {
    NvtxRange nvtx_("fxr:frame_host");
    int32_t st = check_desc(desc, true);
    if (st != FXR_OK) return st;
    if (desc->n_tokens == 0) return FXR_OK;
    if (!workspace) return fail(FXR_ERR_INVALID, "null workspace");
    if (!aligned16(workspace)) return fail(FXR_ERR_INVALID, "workspace must be 16-byte aligned");
    const HostStage h = carve_host(desc, workspace);
    const size_t need = h.total + carve(desc, nullptr).total;
    if (workspace_bytes < need)
        return fail(FXR_ERR_WORKSPACE, "workspace %zu < required %zu", workspace_bytes, need);
    if (!host_q || !host_k || !host_v || !host_mask || !host_out)
        return fail(FXR_ERR_INVALID, "null host buffer");
    const size_t N = (size_t)desc->n_tokens, eb = dtype_bytes(desc->dtype);
    const size_t C = (size_t)desc->n_heads * desc->head_dim;
    const size_t qkv_bytes = ((N - 1) * (size_t)desc->ld_qkv + C) * eb;
    const size_t out_bytes = ((N - 1) * (size_t)desc->ld_out + C) * eb;
    HostIo io;
    io.q = mapped_host_range(host_q, qkv_bytes);
    io.k = mapped_host_range(host_k, qkv_bytes);
    io.v = mapped_host_range(host_v, qkv_bytes);
    io.out = const_cast<void*>(mapped_host_range(host_out, out_bytes));
    if (!io.q || !io.k || !io.v || !io.out)
        return fail(FXR_ERR_INVALID, "host_q / host_k / host_v / host_out must be page-locked host memory mapped "
                                     "into the device address space");
    if (!aligned16(io.q) || !aligned16(io.k) || !aligned16(io.v) || !aligned16(io.out))
        return fail(FXR_ERR_INVALID, "host buffers must be 16-byte aligned");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaMemcpyAsync(h.mask, host_mask, N * sizeof(int32_t), cudaMemcpyHostToDevice, s);
    if (e != cudaSuccess) return cuda_status(e, "mask copy");
    char* frame_ws = static_cast<char*>(workspace) + h.total;
    return frame_forward_impl(desc, h.q, h.k, h.v, h.mask, valid, pos, norm_q, norm_k, cache_k, cache_v, h.out,
                              frame_ws, workspace_bytes - h.total, stream, &io);
}

size_t fxr_rows_gemm_scratch_size(void) {
    return fxr::gemm::kSyncBytes + (size_t)std::min(sm_count(), fxr::gemm::kMaxCtas) * fxr::gemm::kPartialBytes;
}

int32_t fxr_ln_modulate_rows(int32_t dtype, const void* x, int64_t ld_x, int32_t dim, const int32_t* idx,
                             const int32_t* count, int32_t row0, int32_t row_end, int32_t n_tokens,
                             const float* scale, const float* shift, float eps, void* y, int64_t ld_y,
                             void* stream) {
    if (dtype != FXR_BF16 && dtype != FXR_F16) return fail(FXR_ERR_UNSUPPORTED, "dtype must be bf16 or fp16");
    if (dim <= 0 || dim % 256 != 0 || dim > fxr::kLnMaxChunks * 256)
        return fail(FXR_ERR_UNSUPPORTED, "dim %d must be a multiple of 256 up to %d", dim, fxr::kLnMaxChunks * 256);
    if (n_tokens < 0 || row0 < 0 || row_end > n_tokens) return fail(FXR_ERR_INVALID, "bad row range");
    if (ld_x < dim || ld_y < dim || ld_x % 8 || ld_y % 8)
        return fail(FXR_ERR_INVALID, "ld_x / ld_y must be >= dim and multiples of 8");
    if (!(eps >= 0.f)) return fail(FXR_ERR_INVALID, "eps must be >= 0");
    if (n_tokens == 0 || (row_end >= 0 && row_end <= row0)) return FXR_OK;
    if (!x || !idx || !y || (row_end < 0 && !count)) return fail(FXR_ERR_INVALID, "null pointer argument");
    if (!aligned16(x) || !aligned16(y) || !aligned16(scale) || !aligned16(shift))
        return fail(FXR_ERR_INVALID, "x / y / scale / shift must be 16-byte aligned");
    const int32_t max_rows = (row_end >= 0 ? row_end : n_tokens) - row0;
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((max_rows + 7) / 8, (int64_t)sm_count() * 8));
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e =
        dtype == FXR_BF16
            ? launch_pdl(fxr::ln_modulate_rows_kernel<__nv_bfloat16>, dim3(grid), dim3(256), 0, s,
                         static_cast<const __nv_bfloat16*>(x), ld_x, idx, count, row0, row_end, n_tokens, dim,
                         scale, shift, eps, static_cast<__nv_bfloat16*>(y), ld_y)
            : launch_pdl(fxr::ln_modulate_rows_kernel<__half>, dim3(grid), dim3(256), 0, s,
                         static_cast<const __half*>(x), ld_x, idx, count, row0, row_end, n_tokens, dim, scale,
                         shift, eps, static_cast<__half*>(y), ld_y);
    if (e != cudaSuccess) return cuda_status(e, "ln_modulate_rows_kernel launch");
    return FXR_OK;
}

int32_t fxr_rows_gemm(const fxr_rows_gemm_desc* d, const int32_t* idx, const int32_t* count, void* scratch,
                      size_t scratch_bytes, void* stream) {
    NvtxRange nvtx_("fxr:rows_gemm");
    namespace G = fxr::gemm;
    if (!d) return fail(FXR_ERR_INVALID, "null desc");
    if (d->dtype != FXR_BF16 && d->dtype != FXR_F16) return fail(FXR_ERR_UNSUPPORTED, "dtype must be bf16 or fp16");
    if (d->n_operands < 1 || d->n_operands > 2) return fail(FXR_ERR_INVALID, "n_operands must be 1 or 2");
    if (d->n_outputs < 1 || d->n_outputs > 4) return fail(FXR_ERR_INVALID, "n_outputs must be 1 to 4");
    if (d->n_tokens < 0 || d->row0 < 0 || d->row_end > d->n_tokens) return fail(FXR_ERR_INVALID, "bad row range");
    int64_t n_out = 0;
    for (int p = 0; p < d->n_outputs; ++p) {
        const fxr_rows_output& o = d->y[p];
        if (o.cols <= 0 || o.cols % G::kBN) return fail(FXR_ERR_UNSUPPORTED, "output %d: cols must be a positive multiple of %d", p, G::kBN);
        if (o.ld < o.cols || o.ld % 8) return fail(FXR_ERR_INVALID, "output %d: ld must be >= cols and a multiple of 8", p);
        if (o.act != FXR_ACT_NONE && o.act != FXR_ACT_GELU_TANH) return fail(FXR_ERR_INVALID, "output %d: unknown act", p);
        if (!o.rows || !aligned16(o.rows)) return fail(FXR_ERR_INVALID, "output %d: null or unaligned rows", p);
        n_out += o.cols;
    }
    for (int q = 0; q < d->n_operands; ++q) {
        const fxr_rows_operand& o = d->a[q];
        if (o.k <= 0 || o.k % G::kBK) return fail(FXR_ERR_UNSUPPORTED, "operand %d: k must be a positive multiple of %d", q, G::kBK);
        if (o.ld < o.k || o.ld % 8) return fail(FXR_ERR_INVALID, "operand %d: ld must be >= k and a multiple of 8", q);
        if (!o.rows || !o.w || !aligned16(o.rows) || !aligned16(o.w))
            return fail(FXR_ERR_INVALID, "operand %d: null or unaligned rows / w", q);
        if (o.ld_w != 0 && (o.ld_w < o.k || o.ld_w % 8))
            return fail(FXR_ERR_INVALID, "operand %d: ld_w must be 0 or >= k and a multiple of 8", q);
    }
    if (!aligned16(d->bias0) || !aligned16(d->bias1) || !aligned16(d->gate))
        return fail(FXR_ERR_INVALID, "bias0 / bias1 / gate must be 16-byte aligned");
    if (d->residual) {
        if (d->n_outputs != 1) return fail(FXR_ERR_INVALID, "a residual needs a single output part");
        if (d->ld_residual < n_out || d->ld_residual % 8 || !aligned16(d->residual))
            return fail(FXR_ERR_INVALID, "residual: ld must be >= n_out and a multiple of 8, 16-byte aligned");
    }
    if (!idx || (d->row_end < 0 && !count)) return fail(FXR_ERR_INVALID, "null idx / count");
    if (scratch && (scratch_bytes < fxr_rows_gemm_scratch_size() || !aligned16(scratch)))
        return fail(FXR_ERR_WORKSPACE, "scratch %zu < required %zu (or unaligned)", scratch_bytes,
                    fxr_rows_gemm_scratch_size());
    if (d->n_tokens == 0 || (d->row_end >= 0 && d->row_end <= d->row0)) return FXR_OK;

    // instantiations: dtype x (residual or not); the residual path costs registers the others keep
    const int ti = (d->dtype == FXR_BF16 ? 0 : 2) + (d->residual ? 1 : 0);
    using KernelFn = void (*)(const CUtensorMap, const CUtensorMap, const G::Args);
    const KernelFn kernels[4] = {G::rows_gemm_kernel<__nv_bfloat16, false>, G::rows_gemm_kernel<__nv_bfloat16, true>,
                                 G::rows_gemm_kernel<__half, false>, G::rows_gemm_kernel<__half, true>};
    static bool configured[kMaxDevices][4] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < kMaxDevices && !configured[dev][ti]) {
        cudaError_t e = cudaFuncSetAttribute(kernels[ti], cudaFuncAttributeMaxDynamicSharedMemorySize, (int)G::kSmemBytes);
        if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(rows gemm)");
        configured[dev][ti] = true;
    }
    int32_t st;
    CUtensorMap tw0, tw1;
    auto ldw = [](const fxr_rows_operand& o) { return o.ld_w ? o.ld_w : (int64_t)o.k; };
    if ((st = make_tmap(&tw0, d->a[0].w, d->dtype, d->a[0].k, n_out, ldw(d->a[0]), G::kBN)) != FXR_OK) return st;
    if (d->n_operands == 2) {
        if ((st = make_tmap(&tw1, d->a[1].w, d->dtype, d->a[1].k, n_out, ldw(d->a[1]), G::kBN)) != FXR_OK) return st;
    } else {
        tw1 = tw0;
    }
    G::Args a{};
    a.op0.rows = d->a[0].rows;
    a.op0.ld = d->a[0].ld;
    a.op0.kb_end = d->a[0].k / G::kBK;
    a.op0.gathered = d->a[0].gathered ? 1 : 0;
    int32_t k_total = d->a[0].k;
    if (d->n_operands == 2) {
        a.op1.rows = d->a[1].rows;
        a.op1.ld = d->a[1].ld;
        a.op1.kb_end = a.op0.kb_end + d->a[1].k / G::kBK;
        a.op1.gathered = d->a[1].gathered ? 1 : 0;
        k_total += d->a[1].k;
    } else {
        a.op1 = a.op0;
        a.op1.rows = nullptr;
    }
    a.idx = idx;
    a.count = count;
    a.row0 = d->row0;
    a.row_end = d->row_end;
    a.n_tokens = d->n_tokens;
    a.n_kb = k_total / G::kBK;
    a.n_out = (int32_t)n_out;
    G::Part* parts[4] = {&a.p0, &a.p1, &a.p2, &a.p3};
    int32_t col_end = 0;
    for (int p = 0; p < 4; ++p) {
        G::Part& P = *parts[p];
        if (p < d->n_outputs) {
            const fxr_rows_output& o = d->y[p];
            col_end += o.cols;
            P.rows = o.rows;
            P.ld = o.ld;
            P.scattered = o.scattered ? 1 : 0;
            P.gelu = o.act == FXR_ACT_GELU_TANH ? 1 : 0;
        } else {
            P = *parts[d->n_outputs - 1];
        }
        P.col_end = col_end;
    }
    a.bias0 = d->bias0;
    a.bias1 = d->bias1;
    a.res = d->residual;
    a.ld_res = d->ld_residual;
    a.gate = d->gate;
    a.sync = static_cast<uint32_t*>(scratch);
    a.partials = scratch ? reinterpret_cast<float*>(static_cast<char*>(scratch) + G::kSyncBytes) : nullptr;
    int grid;
    if (scratch) {
        grid = std::min(sm_count(), G::kMaxCtas);
    } else {
        const int64_t max_rows = (d->row_end >= 0 ? d->row_end : d->n_tokens) - d->row0;
        const int64_t max_tiles = (max_rows + G::kBM - 1) / G::kBM * (n_out / G::kBN);
        grid = (int)std::max<int64_t>(1, std::min<int64_t>(max_tiles, sm_count()));
    }
    cudaError_t e = launch_pdl(kernels[ti], dim3(grid), dim3(G::kThreads), G::kSmemBytes,
                               static_cast<cudaStream_t>(stream), tw0, tw1, a);
    if (e != cudaSuccess) return cuda_status(e, "rows_gemm_kernel launch");
    return FXR_OK;
}

int32_t fxr_qkv_project(const fxr_frame_desc* desc, const void* hidden, int64_t ld_hidden, int32_t k_dim,
                        const void* w_qkv, const float* bias, const int32_t* idx, const int32_t* count,
                        void* q, void* k, void* v, void* scratch, size_t scratch_bytes, void* stream) {
    int32_t st = check_desc(desc, true);
    if (st != FXR_OK) return st;
    const int64_t C = (int64_t)desc->n_heads * desc->head_dim;
    if (k_dim <= 0 || k_dim % fxr::gemm::kBK != 0)
        return fail(FXR_ERR_UNSUPPORTED, "k_dim %d must be a positive multiple of %d", k_dim, fxr::gemm::kBK);
    if (C % fxr::gemm::kBN != 0)
        return fail(FXR_ERR_UNSUPPORTED, "n_heads * head_dim = %lld must be a multiple of %d", (long long)C,
                    fxr::gemm::kBN);
    if (ld_hidden < k_dim || ld_hidden % 8) return fail(FXR_ERR_INVALID, "ld_hidden must be >= k_dim and a multiple of 8");
    if (desc->n_tokens == 0) return FXR_OK;
    if (!hidden || !w_qkv || !idx || !count || !q || !k || !v) return fail(FXR_ERR_INVALID, "null pointer argument");
    fxr_rows_gemm_desc g{};
    g.dtype = desc->dtype;
    g.n_tokens = desc->n_tokens;
    g.row0 = 0;
    g.row_end = -1;
    g.n_operands = 1;
    g.a[0] = fxr_rows_operand{hidden, ld_hidden, k_dim, 1, w_qkv, 0};
    g.n_outputs = 3;
    void* parts[3] = {q, k, v};
    for (int p = 0; p < 3; ++p) g.y[p] = fxr_rows_output{parts[p], desc->ld_qkv, (int32_t)C, 1, FXR_ACT_NONE, 0};
    g.bias0 = bias;
    return fxr_rows_gemm(&g, idx, count, scratch, scratch_bytes, stream);
}

// ---- the double-stream block on the executed rows ---------------------------------------------
// Workspace: the frame's views and split area, then Q/K/V, the LayerNorm rows, the attention rows
// (all [N, C]), the MLP rows [N, H] and the GEMM scratch.
struct BlockViews {
    Views frame;
    SplitArea split;
    char* q;
    char* k;
    char* v;
    char* xn;
    char* attn;
    char* h;
    char* gemm;
    size_t total;
};

static BlockViews carve_block(const fxr_frame_desc* d, int32_t hidden, void* ws) {
    BlockViews b{};
    char* base = static_cast<char*>(ws);
    b.frame = carve(d, ws);
    const size_t split_sz = split_bytes(kSplitSlotsPerSm * sm_count());
    size_t off = align_up(b.frame.total + split_sz, 256);
    if (base) b.split = split_area(b.frame.total, ws, b.frame.total + split_sz, d->n_heads);
    const size_t N = (size_t)(d->n_tokens > 0 ? d->n_tokens : 1);
    const size_t row = (size_t)d->n_heads * d->head_dim * dtype_bytes(d->dtype);
    char** parts[5] = {&b.q, &b.k, &b.v, &b.xn, &b.attn};
    for (char** p : parts) {
        *p = base ? base + off : nullptr;
        off = align_up(off + N * row, 256);
    }
    b.h = base ? base + off : nullptr;
    off = align_up(off + N * (size_t)hidden * dtype_bytes(d->dtype), 256);
    b.gemm = base ? base + off : nullptr;
    off += fxr_rows_gemm_scratch_size();
    b.total = off;
    return b;
}

size_t fxr_double_block_workspace_size(const fxr_frame_desc* desc, int32_t mlp_hidden) {
    if (!desc || dtype_bytes(desc->dtype) == 0 || desc->n_heads <= 0 || desc->head_dim <= 0 || mlp_hidden <= 0)
        return 0;
    return carve_block(desc, mlp_hidden, nullptr).total;
}

static int32_t check_block_stream(const fxr_block_stream& s, const char* which) {
    if (!s.w_qkv || !s.w_out || !s.w_mlp0 || !s.w_mlp2 || !s.norm_q || !s.norm_k)
        return fail(FXR_ERR_INVALID, "%s stream: null weight", which);
    const void* p16[] = {s.w_qkv, s.w_out, s.w_mlp0, s.w_mlp2, s.shift, s.scale, s.gate,
                         s.b_qkv, s.b_out, s.b_mlp0, s.b_mlp2};
    for (const void* p : p16)
        if (!aligned16(p)) return fail(FXR_ERR_INVALID, "%s stream: weights must be 16-byte aligned", which);
    return FXR_OK;
}

// Device-side addresses of a host-buffer block's page-locked hidden states.
struct BlockHostIo {
    const void* x_in;
    void* x_out;
};

static int32_t block_upload(const BlockHostIo* host, const void* x_in, int32_t C, size_t eb, const int32_t* idx,
                            const int32_t* count, int32_t N, cudaStream_t s) {
    if (!host) return FXR_OK;
    const void* src[1] = {host->x_in};
    void* dst[1] = {const_cast<void*>(x_in)};
    return launch_host_rows(src, dst, 1, C, (int64_t)C * (int64_t)eb, eb, idx, count, N, s);
}

static int32_t block_download(const BlockHostIo* host, const void* x_out, int32_t C, size_t eb, const int32_t* idx,
                              const int32_t* count, int32_t N, cudaStream_t s) {
    if (!host) return FXR_OK;
    const void* src[1] = {x_out};
    void* dst[1] = {host->x_out};
    return launch_host_rows(src, dst, 1, C, (int64_t)C * (int64_t)eb, eb, idx, count, N, s);
}

static int32_t double_block_impl(const fxr_frame_desc* desc, const fxr_double_block* blk, const void* x_in,
                                 void* x_out, int32_t* mask, uint8_t* valid, const int32_t* pos,
                                 void* cache_k, void* cache_v, void* workspace, size_t workspace_bytes,
                                 void* stream, const BlockHostIo* host) {
    int32_t st = check_desc(desc, true);
    if (st != FXR_OK) return st;
    if (!blk) return fail(FXR_ERR_INVALID, "null block");
    const int32_t N = desc->n_tokens, T = desc->n_text, H = blk->mlp_hidden;
    const int32_t C = desc->n_heads * desc->head_dim;
    if (C % fxr::gemm::kBN || H <= 0 || H % fxr::gemm::kBN)
        return fail(FXR_ERR_UNSUPPORTED, "n_heads * head_dim (%d) and mlp_hidden (%d) must be multiples of %d", C, H,
                    fxr::gemm::kBN);
    if (C > fxr::kLnMaxChunks * 256) return fail(FXR_ERR_UNSUPPORTED, "hidden size %d above %d", C, fxr::kLnMaxChunks * 256);
    if (!(blk->ln_eps >= 0.f)) return fail(FXR_ERR_INVALID, "ln_eps must be >= 0");
    if ((st = check_block_stream(blk->img, "image")) != FXR_OK) return st;
    if (T > 0 && (st = check_block_stream(blk->txt, "text")) != FXR_OK) return st;
    if (N == 0) return FXR_OK;
    if (!x_in || !x_out || !mask || !cache_k || !cache_v || !workspace || (desc->rope_n_axes > 0 && !pos))
        return fail(FXR_ERR_INVALID, "null pointer argument");
    if (!aligned16(x_in) || !aligned16(x_out) || !aligned16(cache_k) || !aligned16(cache_v) || !aligned16(workspace))
        return fail(FXR_ERR_INVALID, "x_in / x_out / caches / workspace must be 16-byte aligned");
    const BlockViews b = carve_block(desc, H, workspace);
    if (workspace_bytes < b.total)
        return fail(FXR_ERR_WORKSPACE, "workspace %zu < required %zu", workspace_bytes, b.total);
    // the frame steps see Q/K/V and the attention rows as contiguous [N, C] workspace buffers
    fxr_frame_desc fd = *desc;
    fd.ld_qkv = C;
    fd.ld_out = C;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int32_t dt = desc->dtype;
    int32_t* idx = b.frame.idx;
    int32_t* count = b.frame.count;
    char* gemm = b.gemm;
    const size_t gemm_bytes = fxr_rows_gemm_scratch_size();
    // 1. compaction; text tokens always execute; the GEMM sync words start from zero
    {
        fxr::CompactArgs ca{};
        ca.s[0] = fxr::CompactStream{mask, valid, idx, count, b.frame.restore};
        if ((st = launch_compact_streams(ca, 1, N, b.split, stream, gemm, fxr::gemm::kSyncBytes, T,
                                         desc->n_heads)) != FXR_OK)
            return st;
    }
    if ((st = block_upload(host, x_in, C, dtype_bytes(dt), idx, count, N, s)) != FXR_OK) return st;
    const fxr_block_stream* ss[2] = {&blk->txt, &blk->img};
    const int32_t r0[2] = {0, T}, r1[2] = {T, -1};
    const int first = T > 0 ? 0 : 1;
    // 2. LayerNorm + modulation of the executed rows (compact), 3. Q/K/V (scattered)
    for (int k = first; k < 2; ++k) {
        const fxr_block_stream& w = *ss[k];
        if ((st = fxr_ln_modulate_rows(dt, x_in, C, C, idx, count, r0[k], r1[k], N, w.scale, w.shift, blk->ln_eps,
                                       b.xn, C, stream)) != FXR_OK)
            return st;
    }
    for (int k = first; k < 2; ++k) {
        const fxr_block_stream& w = *ss[k];
        fxr_rows_gemm_desc g{};
        g.dtype = dt;
        g.n_tokens = N;
        g.row0 = r0[k];
        g.row_end = r1[k];
        g.n_operands = 1;
        g.a[0] = fxr_rows_operand{b.xn, C, C, 0, w.w_qkv, 0};
        g.n_outputs = 3;
        g.y[0] = fxr_rows_output{b.q, C, C, 1, FXR_ACT_NONE, 0};
        g.y[1] = fxr_rows_output{b.k, C, C, 1, FXR_ACT_NONE, 0};
        g.y[2] = fxr_rows_output{b.v, C, C, 1, FXR_ACT_NONE, 0};
        g.bias0 = w.b_qkv;
        if ((st = fxr_rows_gemm(&g, idx, count, gemm, gemm_bytes, stream)) != FXR_OK) return st;
    }
    // 4. gather + per-head QK-RMSNorm (each stream's weights) + RoPE, cache rows; 5. attention;
    // 6. restore of the mask-1 cache rows
    st = dt == FXR_BF16
             ? launch_gather_streams<__nv_bfloat16>(&fd, 1, std::array<fxr::GatherStream, 1>{fxr::GatherStream{
                                                                b.q, b.k, b.v, mask, idx, count, b.frame.qc,
                                                                cache_k, cache_v, b.frame.save}}.data(),
                                                    pos, blk->img.norm_q, blk->img.norm_k, b.frame.ld_qc, s,
                                                    T > 0 ? blk->txt.norm_q : nullptr,
                                                    T > 0 ? blk->txt.norm_k : nullptr, T)
             : launch_gather_streams<__half>(&fd, 1, std::array<fxr::GatherStream, 1>{fxr::GatherStream{
                                                         b.q, b.k, b.v, mask, idx, count, b.frame.qc, cache_k,
                                                         cache_v, b.frame.save}}.data(),
                                             pos, blk->img.norm_q, blk->img.norm_k, b.frame.ld_qc, s,
                                             T > 0 ? blk->txt.norm_q : nullptr, T > 0 ? blk->txt.norm_k : nullptr,
                                             T);
    if (st != FXR_OK) return st;
    OutSet os;
    os.out = b.attn;
    os.split = b.split;
    os.reserve_sms = host ? kHostReserveSms : 0;   // host-resident x: SMs for the row transfers
    bool restored = false;
    st = dt == FXR_BF16 ? launch_attention<__nv_bfloat16>(&fd, b.frame.qc, b.frame.ld_qc, count, cache_k, cache_v,
                                                          idx, os, s, &b.frame, &restored)
                        : launch_attention<__half>(&fd, b.frame.qc, b.frame.ld_qc, count, cache_k, cache_v, idx,
                                                   os, s, &b.frame, &restored);
    if (st != FXR_OK) return st;
    if (!restored && (st = fxr_restore_rows(&fd, mask, idx, count, b.frame.save, cache_k, cache_v, stream)) != FXR_OK)
        return st;
    // 7. MLP up with GELU (compact), 8. out-projection + MLP down + gated residual (scattered)
    for (int k = first; k < 2; ++k) {
        const fxr_block_stream& w = *ss[k];
        fxr_rows_gemm_desc g{};
        g.dtype = dt;
        g.n_tokens = N;
        g.row0 = r0[k];
        g.row_end = r1[k];
        g.n_operands = 1;
        g.a[0] = fxr_rows_operand{b.xn, C, C, 0, w.w_mlp0, 0};
        g.n_outputs = 1;
        g.y[0] = fxr_rows_output{b.h, H, H, 0, FXR_ACT_GELU_TANH, 0};
        g.bias0 = w.b_mlp0;
        if ((st = fxr_rows_gemm(&g, idx, count, gemm, gemm_bytes, stream)) != FXR_OK) return st;
    }
    for (int k = first; k < 2; ++k) {
        const fxr_block_stream& w = *ss[k];
        fxr_rows_gemm_desc g{};
        g.dtype = dt;
        g.n_tokens = N;
        g.row0 = r0[k];
        g.row_end = r1[k];
        g.n_operands = 2;
        g.a[0] = fxr_rows_operand{b.attn, C, C, 1, w.w_out, 0};
        g.a[1] = fxr_rows_operand{b.h, H, H, 0, w.w_mlp2, 0};
        g.n_outputs = 1;
        g.y[0] = fxr_rows_output{x_out, C, C, 1, FXR_ACT_NONE, 0};
        g.bias0 = w.b_out;
        g.bias1 = w.b_mlp2;
        g.residual = x_in;
        g.ld_residual = C;
        g.gate = w.gate;
        if ((st = fxr_rows_gemm(&g, idx, count, gemm, gemm_bytes, stream)) != FXR_OK) return st;
    }
    if ((st = block_download(host, x_out, C, dtype_bytes(dt), idx, count, N, s)) != FXR_OK) return st;
    // 9. validity of the cache rows this frame updated
    if (valid) return fxr_mark_updated(mask, valid, T, N, stream);
    return FXR_OK;
}

int32_t fxr_double_block_forward(const fxr_frame_desc* desc, const fxr_double_block* blk, const void* x_in,
                                 void* x_out, int32_t* mask, uint8_t* valid, const int32_t* pos,
                                 void* cache_k, void* cache_v, void* workspace, size_t workspace_bytes,
                                 void* stream) {
    NvtxRange nvtx_("fxr:double_block");
    return double_block_impl(desc, blk, x_in, x_out, mask, valid, pos, cache_k, cache_v, workspace,
                             workspace_bytes, stream, nullptr);
}

// ---- the single-stream block on the executed rows ----------------------------------------------
size_t fxr_single_block_workspace_size(const fxr_frame_desc* desc, int32_t mlp_hidden) {
    return fxr_double_block_workspace_size(desc, mlp_hidden);   // the same buffers
}

static int32_t single_block_impl(const fxr_frame_desc* desc, const fxr_single_block* blk, const void* x_in,
                                 void* x_out, int32_t* mask, uint8_t* valid, const int32_t* pos,
                                 void* cache_k, void* cache_v, void* workspace, size_t workspace_bytes,
                                 void* stream, const BlockHostIo* host) {
    int32_t st = check_desc(desc, true);
    if (st != FXR_OK) return st;
    if (!blk) return fail(FXR_ERR_INVALID, "null block");
    const int32_t N = desc->n_tokens, T = desc->n_text, H = blk->mlp_hidden;
    const int32_t C = desc->n_heads * desc->head_dim;
    if (C % fxr::gemm::kBN || H <= 0 || H % fxr::gemm::kBN)
        return fail(FXR_ERR_UNSUPPORTED, "n_heads * head_dim (%d) and mlp_hidden (%d) must be multiples of %d", C, H,
                    fxr::gemm::kBN);
    if (C > fxr::kLnMaxChunks * 256) return fail(FXR_ERR_UNSUPPORTED, "hidden size %d above %d", C, fxr::kLnMaxChunks * 256);
    if (!(blk->ln_eps >= 0.f)) return fail(FXR_ERR_INVALID, "ln_eps must be >= 0");
    if (!blk->w_qkv_mlp || !blk->w_out || !blk->norm_q || !blk->norm_k) return fail(FXR_ERR_INVALID, "null weight");
    const void* p16[] = {blk->w_qkv_mlp, blk->w_out, blk->shift, blk->scale, blk->gate, blk->b_qkv_mlp, blk->b_out};
    for (const void* p : p16)
        if (!aligned16(p)) return fail(FXR_ERR_INVALID, "weights must be 16-byte aligned");
    if (N == 0) return FXR_OK;
    if (!x_in || !x_out || !mask || !cache_k || !cache_v || !workspace || (desc->rope_n_axes > 0 && !pos))
        return fail(FXR_ERR_INVALID, "null pointer argument");
    if (!aligned16(x_in) || !aligned16(x_out) || !aligned16(cache_k) || !aligned16(cache_v) || !aligned16(workspace))
        return fail(FXR_ERR_INVALID, "x_in / x_out / caches / workspace must be 16-byte aligned");
    const BlockViews b = carve_block(desc, H, workspace);
    if (workspace_bytes < b.total)
        return fail(FXR_ERR_WORKSPACE, "workspace %zu < required %zu", workspace_bytes, b.total);
    fxr_frame_desc fd = *desc;
    fd.ld_qkv = C;
    fd.ld_out = C;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int32_t dt = desc->dtype;
    int32_t* idx = b.frame.idx;
    int32_t* count = b.frame.count;
    const size_t gemm_bytes = fxr_rows_gemm_scratch_size();
    {
        fxr::CompactArgs ca{};
        ca.s[0] = fxr::CompactStream{mask, valid, idx, count, b.frame.restore};
        if ((st = launch_compact_streams(ca, 1, N, b.split, stream, b.gemm, fxr::gemm::kSyncBytes, T,
                                         desc->n_heads)) != FXR_OK)
            return st;
    }
    if ((st = block_upload(host, x_in, C, dtype_bytes(dt), idx, count, N, s)) != FXR_OK) return st;
    if ((st = fxr_ln_modulate_rows(dt, x_in, C, C, idx, count, 0, -1, N, blk->scale, blk->shift, blk->ln_eps,
                                   b.xn, C, stream)) != FXR_OK)
        return st;
    {   // the fused projection: Q, K, V scattered to their token rows, the MLP rows compact + GELU
        fxr_rows_gemm_desc g{};
        g.dtype = dt;
        g.n_tokens = N;
        g.row0 = 0;
        g.row_end = -1;
        g.n_operands = 1;
        g.a[0] = fxr_rows_operand{b.xn, C, C, 0, blk->w_qkv_mlp, 0};
        g.n_outputs = 4;
        g.y[0] = fxr_rows_output{b.q, C, C, 1, FXR_ACT_NONE, 0};
        g.y[1] = fxr_rows_output{b.k, C, C, 1, FXR_ACT_NONE, 0};
        g.y[2] = fxr_rows_output{b.v, C, C, 1, FXR_ACT_NONE, 0};
        g.y[3] = fxr_rows_output{b.h, H, H, 0, FXR_ACT_GELU_TANH, 0};
        g.bias0 = blk->b_qkv_mlp;
        if ((st = fxr_rows_gemm(&g, idx, count, b.gemm, gemm_bytes, stream)) != FXR_OK) return st;
    }
    const fxr::GatherStream gs{b.q, b.k, b.v, mask, idx, count, b.frame.qc, cache_k, cache_v, b.frame.save};
    st = dt == FXR_BF16 ? launch_gather_streams<__nv_bfloat16>(&fd, 1, &gs, pos, blk->norm_q, blk->norm_k, b.frame.ld_qc, s)
                        : launch_gather_streams<__half>(&fd, 1, &gs, pos, blk->norm_q, blk->norm_k, b.frame.ld_qc, s);
    if (st != FXR_OK) return st;
    OutSet os;
    os.out = b.attn;
    os.split = b.split;
    os.reserve_sms = host ? kHostReserveSms : 0;   // host-resident x: SMs for the row transfers
    bool restored = false;
    st = dt == FXR_BF16 ? launch_attention<__nv_bfloat16>(&fd, b.frame.qc, b.frame.ld_qc, count, cache_k, cache_v,
                                                          idx, os, s, &b.frame, &restored)
                        : launch_attention<__half>(&fd, b.frame.qc, b.frame.ld_qc, count, cache_k, cache_v, idx,
                                                   os, s, &b.frame, &restored);
    if (st != FXR_OK) return st;
    if (!restored && (st = fxr_restore_rows(&fd, mask, idx, count, b.frame.save, cache_k, cache_v, stream)) != FXR_OK)
        return st;
    {   // x_out = x_in + gate * ([attention | MLP] . W_out^T + b_out): W_out's two column blocks
        fxr_rows_gemm_desc g{};
        g.dtype = dt;
        g.n_tokens = N;
        g.row0 = 0;
        g.row_end = -1;
        g.n_operands = 2;
        g.a[0] = fxr_rows_operand{b.attn, C, C, 1, blk->w_out, (int64_t)C + H};
        g.a[1] = fxr_rows_operand{b.h, H, H, 0, static_cast<const char*>(blk->w_out) + (size_t)C * dtype_bytes(dt),
                                  (int64_t)C + H};
        g.n_outputs = 1;
        g.y[0] = fxr_rows_output{x_out, C, C, 1, FXR_ACT_NONE, 0};
        g.bias0 = blk->b_out;
        g.residual = x_in;
        g.ld_residual = C;
        g.gate = blk->gate;
        if ((st = fxr_rows_gemm(&g, idx, count, b.gemm, gemm_bytes, stream)) != FXR_OK) return st;
    }
    if ((st = block_download(host, x_out, C, dtype_bytes(dt), idx, count, N, s)) != FXR_OK) return st;
    if (valid) return fxr_mark_updated(mask, valid, T, N, stream);
    return FXR_OK;
}

int32_t fxr_single_block_forward(const fxr_frame_desc* desc, const fxr_single_block* blk, const void* x_in,
                                 void* x_out, int32_t* mask, uint8_t* valid, const int32_t* pos,
                                 void* cache_k, void* cache_v, void* workspace, size_t workspace_bytes,
                                 void* stream) {
    NvtxRange nvtx_("fxr:single_block");
    return single_block_impl(desc, blk, x_in, x_out, mask, valid, pos, cache_k, cache_v, workspace,
                             workspace_bytes, stream, nullptr);
}

// ---- blocks with host-resident hidden states ----------------------------------------------------
// Staging at the start of the workspace: the mask copy, x_in and x_out rows [N, C]; the block's own
// workspace follows.
struct BlockHostStage {
    int32_t* mask;
    void* x_in;
    void* x_out;
    size_t total;
};

static BlockHostStage carve_block_host(const fxr_frame_desc* d, void* ws) {
    BlockHostStage h{};
    const size_t N = (size_t)(d->n_tokens > 0 ? d->n_tokens : 1);
    const size_t row = (size_t)d->n_heads * d->head_dim * dtype_bytes(d->dtype);
    char* b = static_cast<char*>(ws);
    size_t off = 0;
    h.mask = reinterpret_cast<int32_t*>(b ? b + off : nullptr);
    off = align_up(off + N * sizeof(int32_t), 256);
    h.x_in = b ? b + off : nullptr;
    off = align_up(off + N * row, 256);
    h.x_out = b ? b + off : nullptr;
    off = align_up(off + N * row, 256);
    h.total = off;
    return h;
}

size_t fxr_block_host_workspace_size(const fxr_frame_desc* desc, int32_t mlp_hidden) {
    const size_t inner = fxr_double_block_workspace_size(desc, mlp_hidden);
    if (inner == 0) return 0;
    return carve_block_host(desc, nullptr).total + inner;
}

// Validates the host side of a block call and stages it: the mask is copied, the host rows'
// device-side addresses returned in io; *inner / *inner_bytes receive the block's workspace.
static int32_t block_host_stage(const fxr_frame_desc* desc, int32_t mlp_hidden, const void* host_x_in,
                                void* host_x_out, const int32_t* host_mask, void* workspace, size_t workspace_bytes,
                                void* stream, BlockHostStage* h, BlockHostIo* io, void** inner, size_t* inner_bytes) {
    int32_t st = check_desc(desc, true);
    if (st != FXR_OK) return st;
    if (!workspace) return fail(FXR_ERR_INVALID, "null workspace");
    if (!aligned16(workspace)) return fail(FXR_ERR_INVALID, "workspace must be 16-byte aligned");
    *h = carve_block_host(desc, workspace);
    if (mlp_hidden <= 0) return fail(FXR_ERR_UNSUPPORTED, "mlp_hidden %d", mlp_hidden);
    const size_t need = h->total + carve_block(desc, mlp_hidden, nullptr).total;
    if (workspace_bytes < need) return fail(FXR_ERR_WORKSPACE, "workspace %zu < required %zu", workspace_bytes, need);
    if (!host_x_in || !host_x_out || !host_mask) return fail(FXR_ERR_INVALID, "null host buffer");
    const size_t bytes = (size_t)desc->n_tokens * desc->n_heads * desc->head_dim * dtype_bytes(desc->dtype);
    io->x_in = mapped_host_range(host_x_in, bytes);
    io->x_out = const_cast<void*>(mapped_host_range(host_x_out, bytes));
    if (!io->x_in || !io->x_out)
        return fail(FXR_ERR_INVALID, "host_x_in / host_x_out must be page-locked host memory mapped into the device "
                                     "address space");
    if (!aligned16(io->x_in) || !aligned16(io->x_out)) return fail(FXR_ERR_INVALID, "host buffers must be 16-byte aligned");
    cudaError_t e = cudaMemcpyAsync(h->mask, host_mask, (size_t)desc->n_tokens * sizeof(int32_t),
                                    cudaMemcpyHostToDevice, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_status(e, "mask copy");
    *inner = static_cast<char*>(workspace) + h->total;
    *inner_bytes = workspace_bytes - h->total;
    return FXR_OK;
}

int32_t fxr_double_block_forward_host(const fxr_frame_desc* desc, const fxr_double_block* blk,
                                      const void* host_x_in, void* host_x_out, const int32_t* host_mask,
                                      uint8_t* valid, const int32_t* pos, void* cache_k, void* cache_v,
                                      void* workspace, size_t workspace_bytes, void* stream) {
    if (!blk) return fail(FXR_ERR_INVALID, "null block");
    if (desc && desc->n_tokens == 0) return check_desc(desc, true);
    BlockHostStage h{};
    BlockHostIo io{};
    void* inner = nullptr;
    size_t inner_bytes = 0;
    int32_t st = block_host_stage(desc, blk->mlp_hidden, host_x_in, host_x_out, host_mask, workspace, workspace_bytes,
                                  stream, &h, &io, &inner, &inner_bytes);
    if (st != FXR_OK) return st;
    return double_block_impl(desc, blk, h.x_in, h.x_out, h.mask, valid, pos, cache_k, cache_v, inner, inner_bytes,
                             stream, &io);
}

int32_t fxr_single_block_forward_host(const fxr_frame_desc* desc, const fxr_single_block* blk,
                                      const void* host_x_in, void* host_x_out, const int32_t* host_mask,
                                      uint8_t* valid, const int32_t* pos, void* cache_k, void* cache_v,
                                      void* workspace, size_t workspace_bytes, void* stream) {
    if (!blk) return fail(FXR_ERR_INVALID, "null block");
    if (desc && desc->n_tokens == 0) return check_desc(desc, true);
    BlockHostStage h{};
    BlockHostIo io{};
    void* inner = nullptr;
    size_t inner_bytes = 0;
    int32_t st = block_host_stage(desc, blk->mlp_hidden, host_x_in, host_x_out, host_mask, workspace, workspace_bytes,
                                  stream, &h, &io, &inner, &inner_bytes);
    if (st != FXR_OK) return st;
    return single_block_impl(desc, blk, h.x_in, h.x_out, h.mask, valid, pos, cache_k, cache_v, inner, inner_bytes,
                             stream, &io);
}

size_t fxr_batch_workspace_size(const fxr_frame_desc* desc, int32_t n_streams) {
    if (!desc || dtype_bytes(desc->dtype) == 0 || desc->n_heads <= 0 || desc->head_dim <= 0 || n_streams < 0)
        return 0;
    return (size_t)std::min(n_streams, (int32_t)FXR_MAX_BATCH) * carve(desc, nullptr).total;
}

}  // extern "C"

template <typename T>
static int32_t batch_group(const fxr_frame_desc* desc, int32_t nb, const fxr_stream_frame* f,
                           const int32_t* pos, const float* nq, const float* nk, char* ws, size_t base,
                           cudaStream_t s) {
    fxr::CompactArgs ca{};
    fxr::GatherStream gs[fxr::kMaxBatch];
    AttnStreamArgs as[fxr::kMaxBatch];
    fxr::RestoreArgs ra{};
    Views wv[fxr::kMaxBatch];
    int64_t ld_qc = 0;
    for (int32_t b = 0; b < nb; ++b) {
        wv[b] = carve(desc, ws + (size_t)b * base);
        const Views& w = wv[b];
        const fxr_stream_frame& x = f[b];
        if (!x.q || !x.k || !x.v || !x.mask || !x.cache_k || !x.cache_v || !x.out)
            return fail(FXR_ERR_INVALID, "stream %d: null pointer", b);
        if (!aligned16(x.q) || !aligned16(x.k) || !aligned16(x.v) || !aligned16(x.cache_k) ||
            !aligned16(x.cache_v) || !aligned16(x.out))
            return fail(FXR_ERR_INVALID, "stream %d: buffers must be 16-byte aligned", b);
        ca.s[b] = fxr::CompactStream{x.mask, x.valid, w.idx, w.count, w.restore};
        gs[b] = fxr::GatherStream{x.q, x.k, x.v, x.mask, w.idx, w.count, w.qc, x.cache_k, x.cache_v, w.save,
                                  x.valid, w.restore};
        as[b] = AttnStreamArgs{w.qc, w.ld_qc, w.count, x.cache_k, x.cache_v, w.idx, x.out, &wv[b]};
        ra.s[b] = fxr::RestoreStream{x.mask, w.idx, w.count, static_cast<const uint4*>(w.save),
                                     static_cast<char*>(x.cache_k), static_cast<char*>(x.cache_v)};
        ld_qc = w.ld_qc;
    }
    int32_t st;
    // the gather compacts every stream's mask itself when its rows fit (one launch fewer)
    const SplitArea none{};
    const bool fused = gather_can_compact(nb, desc->n_tokens);
    if (!fused && (st = launch_compact_streams(ca, nb, desc->n_tokens, SplitArea{}, s, nullptr, 0, 0,
                                               desc->n_heads)) != FXR_OK)
        return st;
    if ((st = launch_gather_streams<T>(desc, nb, gs, pos, nq, nk, ld_qc, s, nullptr, nullptr, 0,
                                       fused ? &none : nullptr)) != FXR_OK)
        return st;
    bool restored = false;
    if ((st = launch_attention_streams<T>(desc, nb, as, SplitArea{}, s, &restored)) != FXR_OK) return st;
    return restored ? FXR_OK : launch_restore_streams(desc, ra, nb, s);
}

extern "C" {

int32_t fxr_frame_forward_batch(const fxr_frame_desc* desc, int32_t n_streams, const fxr_stream_frame* frames,
                                const int32_t* pos, const float* norm_q, const float* norm_k, void* workspace,
                                size_t workspace_bytes, void* stream) {
    NvtxRange nvtx_("fxr:frame_batch");
    int32_t st = check_desc(desc, true);
    if (st != FXR_OK) return st;
    if (n_streams < 0) return fail(FXR_ERR_INVALID, "n_streams < 0");
    if (n_streams == 0 || desc->n_tokens == 0) return FXR_OK;
    if (!frames || !workspace || !norm_q || !norm_k || (desc->rope_n_axes > 0 && !pos))
        return fail(FXR_ERR_INVALID, "null pointer argument");
    const size_t base = carve(desc, nullptr).total;
    const size_t need = fxr_batch_workspace_size(desc, n_streams);
    if (workspace_bytes < need) return fail(FXR_ERR_WORKSPACE, "workspace %zu < required %zu", workspace_bytes, need);
    if (!aligned16(workspace)) return fail(FXR_ERR_INVALID, "workspace must be 16-byte aligned");
    static_assert(FXR_MAX_BATCH == fxr::kMaxBatch, "batch limits");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    for (int32_t c0 = 0; c0 < n_streams; c0 += FXR_MAX_BATCH) {
        const int32_t nb = std::min(n_streams - c0, (int32_t)FXR_MAX_BATCH);
        st = desc->dtype == FXR_BF16
                 ? batch_group<__nv_bfloat16>(desc, nb, frames + c0, pos, norm_q, norm_k, static_cast<char*>(workspace), base, s)
                 : batch_group<__half>(desc, nb, frames + c0, pos, norm_q, norm_k, static_cast<char*>(workspace), base, s);
        if (st != FXR_OK) return st;
    }
    return FXR_OK;
}

// Exchange CTAs of a head-split frame (arrivals each GPU with heads sends per frame); every GPU of
// the group is assumed to have this GPU's SM count.
static int32_t push_ctas() { return sm_count(); }

int32_t fxr_head_group_init(fxr_head_group* g, int32_t world, int32_t rank, int32_t n_heads,
                            int32_t n_tokens) {
    if (!g) return fail(FXR_ERR_INVALID, "null head group");
    if (world < 1 || world > FXR_MAX_RANKS || rank < 0 || rank >= world || n_heads <= 0 || n_tokens < 0)
        return fail(FXR_ERR_INVALID, "bad head group: world=%d rank=%d n_heads=%d n_tokens=%d", world,
                    rank, n_heads, n_tokens);
    std::memset(g, 0, sizeof(*g));
    g->world = world;
    g->rank = rank;
    const int32_t base = n_heads / world, extra = n_heads % world;
    int32_t h = 0;
    for (int32_t r = 0; r < world; ++r) {
        const int32_t hn = base + (r < extra ? 1 : 0);
        if (r == rank) {
            g->head0 = h;
            g->n_heads = hn;
        }
        // a single GPU stores its rows directly; with peers every GPU that has heads runs the
        // exchange kernel, whose CTAs each send one arrival
        g->ctas[r] = (world > 1 && hn > 0 && n_tokens > 0) ? push_ctas() : 0;
        h += hn;
    }
    return FXR_OK;
}

// Gather of one GPU's share of a head-split frame (its heads of every executed token, read from
// the full-width rows at q/k/v + the share's first column). The gather compacts the mask itself
// when its lists fit (one launch), else a compaction kernel runs first; `iota` also receives the
// identity row list of a compact attention output.
static int32_t gather_share(const fxr_frame_desc* sd, const char* q, const char* k, const char* v, int32_t* mask,
                            const uint8_t* valid, const Views& fw, const int32_t* pos, const float* norm_q,
                            const float* norm_k, void* cache_k, void* cache_v, const SplitArea& split,
                            RowIota iota, cudaStream_t s) {
    int32_t st = check_desc(sd, false);
    if (st != FXR_OK) return st;
    const bool fused = gather_can_compact(1, sd->n_tokens);
    if (!fused && (st = launch_compact(mask, valid, sd->n_tokens, fw.idx, fw.count, split, s, &fw.restore,
                                       sd->n_heads)) != FXR_OK)
        return st;
    if ((st = check_gather_args(sd, q, k, v, mask, fw.idx, fw.count, pos, norm_q, norm_k, fw.qc, fw.ld_qc, cache_k,
                                cache_v, fw.save)) != FXR_OK)
        return st;
    fxr::GatherStream gs{q, k, v, mask, fw.idx, fw.count, fw.qc, cache_k, cache_v, fw.save,
                         fused ? valid : nullptr, fw.restore};
    const SplitArea* cs = fused ? &split : nullptr;
    return sd->dtype == FXR_BF16
               ? launch_gather_streams<__nv_bfloat16>(sd, 1, &gs, pos, norm_q, norm_k, fw.ld_qc, s, nullptr, nullptr,
                                                      0, cs, iota)
               : launch_gather_streams<__half>(sd, 1, &gs, pos, norm_q, norm_k, fw.ld_qc, s, nullptr, nullptr, 0, cs,
                                               iota);
}

// Workspace of one GPU's share of a head-split frame with peers: the share's frame workspace, then
// an identity row list (the attention's compact output) and the compact O rows of its heads.
struct HeadsViews {
    Views frame;
    int32_t* iota;
    void* o_local;
    size_t total;
};

static HeadsViews carve_heads(const fxr_frame_desc* sd, void* ws) {
    HeadsViews v{};
    v.frame = carve(sd, ws);
    char* b = static_cast<char*>(ws);
    size_t off = v.frame.total;
    v.iota = reinterpret_cast<int32_t*>(b ? b + off : nullptr);
    off = align_up(off + (size_t)std::max(sd->n_tokens, 1) * sizeof(int32_t), 256);
    v.o_local = b ? b + off : nullptr;
    off = align_up(off + (size_t)std::max(sd->n_tokens, 1) * sd->n_heads * sd->head_dim * dtype_bytes(sd->dtype), 256);
    v.total = off;
    return v;
}

int32_t fxr_frame_forward_heads(const fxr_frame_desc* desc, fxr_head_group* g, const void* q,
                                const void* k, const void* v, int32_t* mask, const uint8_t* valid,
                                const int32_t* pos, const float* norm_q, const float* norm_k,
                                void* cache_k, void* cache_v, void* workspace,
                                size_t workspace_bytes, void* stream) {
    NvtxRange nvtx_("fxr:frame_heads");
    int32_t st = check_desc(desc, true);
    if (st != FXR_OK) return st;
    if (!g || g->world < 1 || g->world > FXR_MAX_RANKS || g->rank < 0 || g->rank >= g->world)
        return fail(FXR_ERR_INVALID, "head group not initialised");
    if (g->n_heads < 0 || g->head0 < 0 || g->head0 + g->n_heads > desc->n_heads)
        return fail(FXR_ERR_INVALID, "head group heads [%d, %d) outside the frame's %d heads", g->head0,
                    g->head0 + g->n_heads, desc->n_heads);
    if (desc->n_tokens == 0 || g->n_heads == 0) return FXR_OK;
    const bool peers = g->world > 1;
    if (g->ctas[g->rank] != (peers ? push_ctas() : 0))
        return fail(FXR_ERR_INVALID, "head group was initialised for another frame or device");
    for (int32_t r = 0; r < g->world; ++r) {
        if (!g->out[r]) return fail(FXR_ERR_INVALID, "head group out[%d] is null", r);
        if (peers && !g->arrive[r]) return fail(FXR_ERR_INVALID, "head group arrive[%d] is null", r);
        if (!aligned16(g->out[r])) return fail(FXR_ERR_INVALID, "head group out[%d] not 16-byte aligned", r);
    }
    if (!workspace) return fail(FXR_ERR_INVALID, "null workspace");
    if (!q || !k || !v) return fail(FXR_ERR_INVALID, "null q/k/v");
    if (!cache_k || !cache_v || !aligned16(cache_k) || !aligned16(cache_v))
        return fail(FXR_ERR_INVALID, "cache must be non-null and 16-byte aligned");
    // this GPU's share of the frame: its heads, read from the full-width rows
    fxr_frame_desc sd = *desc;
    sd.n_heads = g->n_heads;
    sd.ld_cache = (int64_t)g->n_heads * desc->head_dim;
    const HeadsViews w = carve_heads(&sd, workspace);
    const size_t need = peers ? w.total : w.frame.total;
    if (workspace_bytes < need)
        return fail(FXR_ERR_WORKSPACE, "workspace %zu < required %zu", workspace_bytes, need);
    if (!aligned16(workspace)) return fail(FXR_ERR_INVALID, "workspace must be 16-byte aligned");
    const int32_t eb = (int32_t)dtype_bytes(desc->dtype);
    const size_t col = (size_t)g->head0 * desc->head_dim * eb;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    OutSet os;
    os.split = split_area(need, workspace, workspace_bytes, sd.n_heads);
    // with peers the attention writes a compact output, row m of this GPU's heads at o_local[m]
    // (identity row list written by the gather), which the exchange scatters
    const RowIota iota = peers ? RowIota{w.iota, desc->n_tokens, desc->n_tokens} : RowIota{};
    if ((st = gather_share(&sd, static_cast<const char*>(q) + col, static_cast<const char*>(k) + col,
                           static_cast<const char*>(v) + col, mask, valid, w.frame, pos, norm_q, norm_k, cache_k,
                           cache_v, os.split, iota, s)) != FXR_OK)
        return st;
    fxr_frame_desc od = sd;
    const int32_t* att_idx = w.frame.idx;
    if (peers) {
        od.ld_out = sd.ld_cache;
        os.out = w.o_local;
        att_idx = w.iota;
    } else {
        os.out = static_cast<char*>(g->out[0]) + col;
    }
    bool restored = false;
    st = sd.dtype == FXR_BF16
             ? launch_attention<__nv_bfloat16>(&od, w.frame.qc, w.frame.ld_qc, w.frame.count, cache_k, cache_v, att_idx,
                                               os, s, &w.frame, &restored)
             : launch_attention<__half>(&od, w.frame.qc, w.frame.ld_qc, w.frame.count, cache_k, cache_v, att_idx, os,
                                        s, &w.frame, &restored);
    if (st != FXR_OK) return st;
    if (!restored &&
        (st = fxr_restore_rows(&sd, mask, w.frame.idx, w.frame.count, w.frame.save, cache_k, cache_v, stream)) != FXR_OK)
        return st;
    if (!peers) return FXR_OK;
    fxr::PushArgs a{};
    a.o = static_cast<const uint4*>(w.o_local);
    a.idx = w.frame.idx;
    a.count = w.frame.count;
    a.ld_out_vecs = desc->ld_out * eb / 16;
    a.row_vecs = (int32_t)(sd.ld_cache * eb / 16);
    a.n_tokens = desc->n_tokens;
    a.world = g->world;
    a.src_rank = g->rank;
    for (int32_t r = 0; r < g->world; ++r) {
        a.out[r] = reinterpret_cast<uint4*>(static_cast<char*>(g->out[r]) + col);
        a.arrive[r] = g->arrive[r];
    }
    NvtxRange nvtx_push("fxr:exchange");
    cudaError_t e = launch_pdl(fxr::heads_push_kernel, dim3(push_ctas()), dim3(fxr::kPushThreads), 0, s, a);
    if (e != cudaSuccess) return cuda_status(e, "heads_push_kernel launch");
    g->epoch += 1;
    return FXR_OK;
}

int32_t fxr_head_group_wait(const fxr_head_group* g, void* stream) {
    NvtxRange nvtx_("fxr:head_group_wait");
    if (!g || g->world < 1 || g->world > FXR_MAX_RANKS || g->rank < 0 || g->rank >= g->world)
        return fail(FXR_ERR_INVALID, "head group not initialised");
    if (g->world == 1) return FXR_OK;   // a single GPU stored its rows itself
    uint32_t* slots = g->arrive[g->rank];
    if (!slots) return fail(FXR_ERR_INVALID, "head group arrive[rank] is null");
    fxr::ArrivalCounts c{};
    for (int32_t r = 0; r < g->world; ++r) c.ctas[r] = (uint32_t)g->ctas[r];
    fxr::arrival_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(slots, c, g->world);
    FXR_CHECK_LAUNCH("arrival_wait_kernel launch");
    return FXR_OK;
}

int32_t fxr_internal_nccl_allgather(const void* send, void* recv, size_t bytes, void* comm, void* stream);

struct NcclViews {
    Views frame;
    int32_t* iota;
    void* o_local;
    void* gathered;
    size_t row_bytes;
    size_t total;
};

static bool group_ok(const fxr_head_group* g) {
    return g && g->world >= 1 && g->world <= FXR_MAX_RANKS && g->rank >= 0 && g->rank < g->world;
}

// Heads of every rank (the balanced split of fxr_head_group_init, recomputed from the group's
// world and the frame's heads).
static void split_heads(int32_t n_heads, int32_t world, int32_t* head0, int32_t* nh) {
    const int32_t base = n_heads / world, extra = n_heads % world;
    int32_t h = 0;
    for (int32_t r = 0; r < world; ++r) {
        nh[r] = base + (r < extra ? 1 : 0);
        head0[r] = h;
        h += nh[r];
    }
}

static NcclViews carve_nccl(const fxr_frame_desc* d, const fxr_head_group* g, int32_t m_cap, void* ws) {
    NcclViews v{};
    fxr_frame_desc sd = *d;
    sd.n_heads = g->n_heads;
    v.frame = carve(&sd, ws);
    const int32_t hmax = (d->n_heads + g->world - 1) / g->world;
    v.row_bytes = (size_t)hmax * d->head_dim * dtype_bytes(d->dtype);
    char* b = static_cast<char*>(ws);
    size_t off = v.frame.total;
    v.iota = reinterpret_cast<int32_t*>(b ? b + off : nullptr);
    off = align_up(off + (size_t)std::max(d->n_tokens, 1) * sizeof(int32_t), 256);
    v.o_local = b ? b + off : nullptr;
    off = align_up(off + (size_t)std::max(m_cap, 1) * v.row_bytes, 256);
    v.gathered = b ? b + off : nullptr;
    off = align_up(off + (size_t)g->world * std::max(m_cap, 1) * v.row_bytes, 256);
    v.total = off;
    return v;
}

size_t fxr_heads_nccl_workspace_size(const fxr_frame_desc* desc, const fxr_head_group* g, int32_t m_cap) {
    if (check_desc(desc, false) != FXR_OK || !group_ok(g) || m_cap < 0) return 0;
    return carve_nccl(desc, g, m_cap, nullptr).total + split_bytes(kSplitSlotsPerSm * sm_count());
}

int32_t fxr_allgather_heads(const fxr_frame_desc* desc, const fxr_head_group* g, void* nccl_comm,
                            const void* o_local, int32_t m_cap, void* gathered, const int32_t* idx,
                            const int32_t* count, void* out, void* stream) {
    NvtxRange nvtx_("fxr:allgather_heads");
    int32_t st = check_desc(desc, false);
    if (st != FXR_OK) return st;
    if (!group_ok(g)) return fail(FXR_ERR_INVALID, "head group not initialised");
    if (m_cap < 0 || m_cap > desc->n_tokens) return fail(FXR_ERR_INVALID, "m_cap %d outside [0, n_tokens]", m_cap);
    if (desc->n_tokens == 0 || m_cap == 0) return FXR_OK;
    if (!nccl_comm || !o_local || !gathered || !idx || !count || !out)
        return fail(FXR_ERR_INVALID, "null pointer argument");
    if (!aligned16(o_local) || !aligned16(gathered) || !aligned16(out))
        return fail(FXR_ERR_INVALID, "buffers must be 16-byte aligned");
    const int32_t eb = (int32_t)dtype_bytes(desc->dtype);
    const int32_t hmax = (desc->n_heads + g->world - 1) / g->world;
    const int64_t row_bytes = (int64_t)hmax * desc->head_dim * eb;
    if ((st = fxr_internal_nccl_allgather(o_local, gathered, (size_t)m_cap * row_bytes, nccl_comm, stream)) != FXR_OK)
        return st;
    fxr::HeadsScatterArgs a{};
    a.gathered = static_cast<const char*>(gathered);
    a.idx = idx;
    a.count = count;
    a.out = static_cast<char*>(out);
    a.row_bytes = row_bytes;
    a.ld_out_bytes = desc->ld_out * eb;
    a.m_cap = m_cap;
    a.world = g->world;
    a.n_tokens = desc->n_tokens;
    int32_t head0[FXR_MAX_RANKS], nh[FXR_MAX_RANKS];
    split_heads(desc->n_heads, g->world, head0, nh);
    for (int32_t r = 0; r < g->world; ++r) {
        a.col_bytes[r] = head0[r] * desc->head_dim * eb;
        a.vecs[r] = nh[r] * desc->head_dim * eb / 16;
    }
    // a plain launch: the all-gather before it may be a copy rather than a kernel, and programmatic
    // dependent launch only orders kernel after kernel
    const int grid = grid_rows((int64_t)m_cap * g->world, 8);
    fxr::heads_scatter_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(a);
    FXR_CHECK_LAUNCH("heads_scatter_kernel launch");
    return FXR_OK;
}

int32_t fxr_frame_forward_heads_nccl(const fxr_frame_desc* desc, const fxr_head_group* g,
                                     void* nccl_comm, int32_t m_cap, const void* q, const void* k,
                                     const void* v, int32_t* mask, const uint8_t* valid,
                                     const int32_t* pos, const float* norm_q, const float* norm_k,
                                     void* cache_k, void* cache_v, void* out, void* workspace,
                                     size_t workspace_bytes, void* stream) {
    NvtxRange nvtx_("fxr:frame_heads_nccl");
    int32_t st = check_desc(desc, true);
    if (st != FXR_OK) return st;
    if (!group_ok(g)) return fail(FXR_ERR_INVALID, "head group not initialised");
    int32_t head0[FXR_MAX_RANKS], nh[FXR_MAX_RANKS];
    split_heads(desc->n_heads, g->world, head0, nh);
    if (g->head0 != head0[g->rank] || g->n_heads != nh[g->rank])
        return fail(FXR_ERR_INVALID, "head group was initialised for another head count");
    if (m_cap < 0 || m_cap > desc->n_tokens) return fail(FXR_ERR_INVALID, "m_cap %d outside [0, n_tokens]", m_cap);
    if (desc->n_tokens == 0) return FXR_OK;
    if (!q || !k || !v || !out || !workspace) return fail(FXR_ERR_INVALID, "null pointer argument");
    const NcclViews w = carve_nccl(desc, g, m_cap, workspace);
    if (workspace_bytes < w.total)
        return fail(FXR_ERR_WORKSPACE, "workspace %zu < required %zu", workspace_bytes, w.total);
    if (!aligned16(workspace) || !aligned16(out)) return fail(FXR_ERR_INVALID, "workspace/out must be 16-byte aligned");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    fxr_frame_desc sd = *desc;
    sd.n_heads = g->n_heads;
    sd.ld_cache = (int64_t)g->n_heads * desc->head_dim;
    const size_t col = (size_t)g->head0 * desc->head_dim * dtype_bytes(desc->dtype);
    const SplitArea split = split_area(w.total, workspace, workspace_bytes, sd.n_heads);
    if (g->n_heads == 0 &&
        (st = launch_compact(mask, valid, sd.n_tokens, w.frame.idx, w.frame.count, split, stream,
                             &w.frame.restore, sd.n_heads)) != FXR_OK)
        return st;
    if (g->n_heads > 0) {
        // compact output rows m < m_cap (identity list written by the gather; rows past m_cap are
        // flagged by the attention as out of range)
        if ((st = gather_share(&sd, static_cast<const char*>(q) + col, static_cast<const char*>(k) + col,
                               static_cast<const char*>(v) + col, mask, valid, w.frame, pos, norm_q, norm_k,
                               cache_k, cache_v, split, RowIota{w.iota, desc->n_tokens, m_cap}, s)) != FXR_OK)
            return st;
        fxr_frame_desc od = sd;                          // compact O output: row m, local heads
        od.ld_out = (int64_t)((desc->n_heads + g->world - 1) / g->world) * desc->head_dim;
        if (!cache_k || !cache_v || !aligned16(cache_k) || !aligned16(cache_v))
            return fail(FXR_ERR_INVALID, "cache must be non-null and 16-byte aligned");
        OutSet os;
        os.out = w.o_local;
        os.split = split;
        bool restored = false;
        st = od.dtype == FXR_BF16
                 ? launch_attention<__nv_bfloat16>(&od, w.frame.qc, w.frame.ld_qc, w.frame.count, cache_k, cache_v,
                                                   w.iota, os, s, &w.frame, &restored)
                 : launch_attention<__half>(&od, w.frame.qc, w.frame.ld_qc, w.frame.count, cache_k, cache_v, w.iota,
                                            os, s, &w.frame, &restored);
        if (st != FXR_OK) return st;
        if (!restored &&
            (st = fxr_restore_rows(&sd, mask, w.frame.idx, w.frame.count, w.frame.save, cache_k, cache_v, stream)) != FXR_OK)
            return st;
    }
    return fxr_allgather_heads(desc, g, nccl_comm, w.o_local, m_cap, w.gathered, w.frame.idx, w.frame.count,
                               out, stream);
}

int32_t fxr_ipc_alloc(size_t bytes, void** ptr, fxr_ipc_handle* handle) {
    static_assert(sizeof(cudaIpcMemHandle_t) == sizeof(fxr_ipc_handle), "IPC handle size");
    if (!ptr || !handle || bytes == 0) return fail(FXR_ERR_INVALID, "bad fxr_ipc_alloc arguments");
    *ptr = nullptr;
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) return cuda_status(e, "cudaMalloc (IPC buffer)");
    e = cudaMemset(p, 0, bytes);
    cudaIpcMemHandle_t h;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
    if (e != cudaSuccess) {
        cudaFree(p);
        return cuda_status(e, "cudaIpcGetMemHandle");
    }
    std::memcpy(handle->bytes, &h, sizeof(h));
    *ptr = p;
    return FXR_OK;
}

int32_t fxr_ipc_open(const fxr_ipc_handle* handle, void** ptr) {
    if (!handle || !ptr) return fail(FXR_ERR_INVALID, "bad fxr_ipc_open arguments");
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle->bytes, sizeof(h));
    cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return cuda_status(e, "cudaIpcOpenMemHandle");
    return FXR_OK;
}

int32_t fxr_ipc_close(void* ptr) {
    if (!ptr) return FXR_OK;
    cudaError_t e = cudaIpcCloseMemHandle(ptr);
    return e == cudaSuccess ? FXR_OK : cuda_status(e, "cudaIpcCloseMemHandle");
}

int32_t fxr_ipc_free(void* ptr) {
    if (!ptr) return FXR_OK;
    cudaError_t e = cudaFree(ptr);
    return e == cudaSuccess ? FXR_OK : cuda_status(e, "cudaFree (IPC buffer)");
}

}  // extern "C"
