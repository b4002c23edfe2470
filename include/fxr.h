/*
 * fxr.h — C ABI of the B200 (sm_100a) sparse stream-editing attention path.
 *
 * One frame of a FLUX.2 double-stream attention slice under a spatial KV cache:
 *   change mask -> ascending index list of executed tokens -> gather of their Q/K/V rows with
 *   per-head QK-RMSNorm and multi-axis RoPE in the gather's epilogue -> attention of the executed
 *   queries against every key (fresh K/V for executed tokens, cached K/V for skipped ones) ->
 *   scatter of the outputs into the full-frame buffer and update of the K/V cache rows.
 *
 * Conventions (all entry points):
 *   - plain C: pointers, sizes, an opaque stream handle (a cudaStream_t passed as void*);
 *   - every pointer argument except the descriptor is DEVICE memory owned by the caller;
 *     nothing allocates device memory except fxr_ipc_alloc (set-up of multi-GPU buffers);
 *   - asynchronous on `stream`; nothing synchronises the host, so a sequence of calls can be
 *     captured into a CUDA graph;
 *   - the number of executed tokens M is produced on the device by fxr_mask_compact and read on
 *     the device by the later steps (`count` argument), so no device->host copy is needed;
 *   - return FXR_OK (0) or an error status; fxr_last_error_string() describes the last error of
 *     the calling thread; no C++ exception crosses this boundary.
 *
 * Layouts: token-major rows, text tokens first ([0, T)) then image tokens ([T, N)).
 *   Q, K, V, out, cache_k, cache_v: [N rows, row stride ld (elements)], head h of a row at
 *   columns [h*D, (h+1)*D). For head sharding, pass base pointers offset by head_begin*D.
 *   mask: int32 [N], 0 = skip, 1 = execute, 2 = execute + update cache
 *   (fluxrt-cpp tools/export_onnx.py:126-129, src/inference/kernels/spatial_kv_cache.cu:12-87).
 *   valid: uint8 [N] cache-row validity (spatial_kv_cache.h:45), NULL = every row valid.
 *   pos: int32 [N, rope_n_axes] position ids.
 */
#ifndef FXR_H
#define FXR_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FXR_ABI_VERSION 2

/* Status codes. The reference's plugin enqueue returns 0 / -1
 * (src/inference/plugins/flux2_double_block_plugin.cpp:208,230); these refine the -1. */
typedef enum fxr_status {
    FXR_OK = 0,
    FXR_ERR_INVALID = 1,      /* bad argument: null pointer, unsupported size, misaligned buffer */
    FXR_ERR_CUDA = 2,         /* a CUDA runtime call or kernel launch failed */
    FXR_ERR_TIMEOUT = 3,      /* a bounded device-side wait gave up (device error word set) */
    FXR_ERR_UNSUPPORTED = 4,  /* valid request this build does not implement (e.g. head_dim != 128 on the tensor-core path) */
    FXR_ERR_WORKSPACE = 5,    /* workspace smaller than fxr_workspace_min_size() */
    FXR_ERR_NCCL = 6,         /* NCCL call failed */
    FXR_ERR_BOUNDS = 7        /* a kernel met a row index outside its buffer and skipped that row
                                 (reported by fxr_check_device_error) */
} fxr_status;

/* Storage element types (compute is fp32 throughout). */
typedef enum fxr_dtype { FXR_F32 = 0, FXR_F16 = 1, FXR_BF16 = 2 } fxr_dtype;

/* Frame geometry and RoPE / norm parameters. Plain old data; zero-initialise, then fill. */
typedef struct fxr_frame_desc {
    int32_t n_tokens;        /* N = T + I */
    int32_t n_text;          /* T (informational: text rows are [0, T)) */
    int32_t n_heads;         /* heads processed by this call (24 for FLUX.2-Klein) */
    int32_t head_dim;        /* D; the tensor-core attention supports 128 */
    int32_t dtype;           /* fxr_dtype of Q/K/V/out/cache: FXR_BF16 or FXR_F16 */
    int32_t rope_n_axes;     /* 1..4 */
    int32_t rope_axes_dim[4];/* even, sum == head_dim (e.g. 16/56/56 or 32/32/32/32) */
    float rope_theta;        /* 10000 (FLUX.1 layout) or 2000 (Klein config.json:22) */
    float eps;               /* RMSNorm epsilon, 1e-6 (flux2_double_block_plugin.cpp:413) */
    float softmax_scale;     /* <= 0 selects 1/sqrt(head_dim) (attention_kernels.cu:101) */
    int32_t reserved0;
    int64_t ld_qkv;          /* row stride (elements) of Q, K, V */
    int64_t ld_cache;        /* row stride of cache_k, cache_v */
    int64_t ld_out;          /* row stride of out */
} fxr_frame_desc;

/* Library ABI version (FXR_ABI_VERSION) and build information. */
int32_t fxr_abi_version(void);
const char* fxr_build_info(void);

/* Last error message of the calling thread ("" if none). */
const char* fxr_last_error_string(void);

/* Reads and clears the device error word of the current device. Kernels set it instead of faulting:
 * bit 0 when a bounded device wait gave up (2 s), bit 1 when an index outside [0, rows) of the
 * indexed buffer was met (the row was skipped: nothing was read from or written to it). The checks
 * are always compiled in. Synchronises `stream`, then returns FXR_OK, FXR_ERR_TIMEOUT (bit 0 set,
 * whatever else is) or FXR_ERR_BOUNDS; *word_out (may be NULL) receives the raw word.
 * There is one word per device, shared by every stream and thread that uses this library on it: a
 * check after one stream's work can report an error raised by another stream's work that ran in
 * the meantime. Pass stream NULL after cudaDeviceSynchronize for a check that covers all work. */
int32_t fxr_check_device_error(void* stream, uint32_t* word_out);

/* ---- workspace ------------------------------------------------------------------------------ */
/* Bytes of caller-provided workspace fxr_frame_forward needs (idx, count, compact Q, saved rows
 * of mask==1 tokens). Replaces the reference's workspace carve-up
 * (flux2_double_block_plugin.cpp:167-185, 347-366). */
size_t fxr_workspace_size(const fxr_frame_desc* desc);

/* The smallest workspace fxr_frame_forward accepts: idx, count, compact Q and saved rows, without
 * the optional area of scratch slots that lets the attention cut work units between CTAs (the
 * two-tile kernel's stream-K schedule, which needs 4 slots per SM; the one-tile kernel's key-range
 * split, calls of at most 8 heads). A workspace between this size and fxr_workspace_size gets as
 * many slots as fit in the rest; at this size the attention never cuts a unit. The outputs of a
 * frame can differ in the last bits between workspaces that allow different schedules. */
size_t fxr_workspace_min_size(const fxr_frame_desc* desc);

/* ---- individual steps ----------------------------------------------------------------------- */

/* Mask preprocess + compaction. Replaces preprocess_mask_kernel (spatial_kv_cache.cu:12-19,
 * SpatialCache::preprocess_mask spatial_kv_cache.cu:153-158) and the host-supplied index lists of
 * the reference (test_gather_scatter.cpp:47,77). mask[i] = 2 where valid[i] == 0; idx[0..M) =
 * ascending i with mask[i] != 0; *count = M (device int32). Warp-ballot + block scan. */
int32_t fxr_mask_compact(int32_t* mask, const uint8_t* valid, int32_t n_tokens,
                         int32_t* idx, int32_t* count, void* stream);

/* Reference preprocess alone (spatial_kv_cache.cu:12-19): mask[i] = 2 where !valid[i]. */
int32_t fxr_preprocess_mask(int32_t* mask, const uint8_t* valid, int32_t n_tokens, void* stream);

/* Validity update after a frame (sync_output_cache_kernel's valid write, spatial_kv_cache.cu:49-51):
 * valid[i] = 1 for image tokens i in [n_text, n_tokens) with mask[i] == 2. */
int32_t fxr_mark_updated(const int32_t* mask, uint8_t* valid, int32_t n_text, int32_t n_tokens,
                         void* stream);

/* Fused gather + per-head QK-RMSNorm + multi-axis RoPE + cache-row write.
 * Replaces gather_tokens (gather_scatter_kernels.cu:15-41) + rms_norm (flux2_kernels.cu:58-90,
 * per head) + the K/V merge/update of sync_kv_cache_kernel (spatial_kv_cache.cu:55-87) restricted
 * to the executed rows. For m < *count, token i = idx[m], mode = mask[i]:
 *   qc[m]      = rope(rmsnorm(Q[i], norm_q))          (compact, row stride ld_qc)
 *   if mode == 1: save[m] = (cache_k[i], cache_v[i])  (restored by fxr_restore_rows)
 *   cache_k[i] = rope(rmsnorm(K[i], norm_k)),  cache_v[i] = V[i]  (bit-exact copy)
 * save: [N, 2*n_heads*head_dim] elements, may be NULL when no mask value is 1. */
int32_t fxr_gather_norm_rope(const fxr_frame_desc* desc,
                             const void* q, const void* k, const void* v,
                             const int32_t* mask, const int32_t* idx, const int32_t* count,
                             const int32_t* pos, const float* norm_q, const float* norm_k,
                             void* qc, int64_t ld_qc, void* cache_k, void* cache_v, void* save,
                             void* stream);

/* Attention of the compact queries against all N cache rows, with the scatter fused into the
 * epilogue: out[idx[m], h*D..] = softmax(qc[m,h] K_h^T * scale) V_h for m < *count.
 * Replaces attention_fwd (attention_kernels.cu:85-173) + scatter_tokens
 * (gather_scatter_kernels.cu:46-72). tcgen05/TMEM flash attention, TMA-staged K/V tiles.
 * qc rows must be allocated for N rows (rows >= count are read but never stored). */
int32_t fxr_attention_active(const fxr_frame_desc* desc,
                             const void* qc, int64_t ld_qc, const int32_t* count,
                             const void* cache_k, const void* cache_v,
                             const int32_t* idx, void* out, void* stream);

/* Restores the cache rows of mask==1 tokens from `save` (written by fxr_gather_norm_rope). */
int32_t fxr_restore_rows(const fxr_frame_desc* desc, const int32_t* mask, const int32_t* idx,
                         const int32_t* count, const void* save, void* cache_k, void* cache_v,
                         void* stream);

/* Byte-exact row gather / scatter over the first *count indices (count may be a device
 * pointer, or NULL with host_count >= 0). 16-byte vectorised when row_bytes and strides allow.
 * Replace gather_tokens / scatter_tokens (gather_scatter_kernels.cu:15-72).
 * n_index_rows: rows of the indexed buffer (src of the gather, dst of the scatter); an index
 * outside [0, n_index_rows) is skipped and sets the device error word (FXR_ERR_BOUNDS from
 * fxr_check_device_error); the compact row m of a skipped index is left untouched.
 * n_index_rows <= 0: the size is unknown (the reference signature) and only negative indices are
 * caught. */
int32_t fxr_gather_rows(const void* src, int64_t ld_src_bytes, const int32_t* idx,
                        const int32_t* count, int32_t host_count,
                        void* dst, int64_t ld_dst_bytes, int64_t row_bytes, int32_t n_index_rows,
                        void* stream);
int32_t fxr_scatter_rows(const void* src, int64_t ld_src_bytes, const int32_t* idx,
                         const int32_t* count, int32_t host_count,
                         void* dst, int64_t ld_dst_bytes, int64_t row_bytes, int32_t n_index_rows,
                         void* stream);

/* Full-frame K/V merge + update with the reference's exact semantics
 * (sync_kv_cache_kernel, spatial_kv_cache.cu:55-87): keys[i] = execute ? keys[i] : cached[i];
 * if update: cached[i] = fresh keys[i]; same for values. row_elems elements of `dtype` per row. */
int32_t fxr_kv_sync(void* keys, void* values, void* cached_keys, void* cached_values,
                    const int32_t* mask, int32_t n_tokens, int64_t row_elems, int32_t dtype,
                    void* stream);

/* Output-cache merge + valid-flag update (sync_output_cache_kernel, spatial_kv_cache.cu:21-53):
 * image rows i in [0, n_image): pred = execute ? pred : cache; if update: cache = pred and
 * valid[n_text + i] = 1. */
int32_t fxr_output_cache_sync(void* pred, void* cache, const int32_t* mask, uint8_t* valid,
                              int32_t n_text, int32_t n_image, int32_t channels, int32_t dtype,
                              void* stream);

/* Standalone row RMSNorm with the reference signature semantics (launch_rms_norm,
 * flux2_kernels.h:22-24): y = x * rsqrt(mean(x^2) + eps) * w over rows of `dim` elements. */
int32_t fxr_rms_norm(const void* x, void* y, const float* w, float eps, int64_t rows,
                     int32_t dim, int32_t dtype, void* stream);

/* The reference's dense fp32 block helpers over whole sequences (rows of `dim` floats), for the
 * C++ mirror of its kernel layer (include/fxr_reference_api.h); off the sparse path.
 *   fxr_layer_norm_f32   y = (x - mean) * rsqrt(var + eps) [* gamma] [+ beta], biased variance per
 *                        row; gamma / beta may be NULL (layer_norm_modulated,
 *                        gather_scatter_kernels.h:46-61, gather_scatter_kernels.cu:103-169)
 *   fxr_modulate_f32     out = (1 + scale) * x + shift, scale / shift [dim] (apply_modulation,
 *                        gather_scatter_kernels.h:38-44, gather_scatter_kernels.cu:74-99)
 *   fxr_gelu_tanh_f32    data = data * 0.5 * (1 + tanh(0.7978845608 (data + 0.044715 data^3)))
 *                        (launch_gelu, flux2_kernels.h:15, flux2_kernels.cu:14-29)
 *   fxr_bias_add_f32     data[r, :] += bias (launch_bias_add, flux2_kernels.h:18-19, flux2_kernels.cu:34-53)
 *   fxr_add_f32          z = x + y (launch_elem_add, flux2_kernels.h:27-28, flux2_kernels.cu:92-108)
 *   fxr_scale_add_f32    out = x + gate * y (launch_scale_add, flux2_kernels.h:31-32, flux2_kernels.cu:113-135)
 * Outputs may alias inputs element for element. */
int32_t fxr_layer_norm_f32(const float* x, float* y, const float* gamma, const float* beta, float eps,
                           int64_t rows, int32_t dim, void* stream);
int32_t fxr_modulate_f32(const float* x, const float* scale, const float* shift, float* out, int64_t rows,
                         int32_t dim, void* stream);
int32_t fxr_gelu_tanh_f32(float* data, int64_t n, void* stream);
int32_t fxr_bias_add_f32(float* data, const float* bias, int64_t rows, int32_t dim, void* stream);
int32_t fxr_add_f32(const float* x, const float* y, float* z, int64_t n, void* stream);
int32_t fxr_scale_add_f32(const float* x, const float* y, float* out, float gate, int64_t n, void* stream);

/* fp32 attention in the reference's (batch, heads, len, head_dim) layout, head_dim <= 256:
 * out = softmax(Q K^T / sqrt(head_dim)) V with one softmax over all kv_len keys. Backs the
 * reference-signature attention_fwd (attention_kernels.h:20-24); SIMT fp32, not the tensor-core
 * path (fxr_attention_active). */
int32_t fxr_attention_f32_bhsd(const float* q, const float* k, const float* v, float* out,
                               int32_t batch, int32_t num_heads, int32_t q_len, int32_t kv_len,
                               int32_t head_dim, void* stream);

/* ---- composite ------------------------------------------------------------------------------ */
/* One frame: compact -> gather/norm/RoPE/cache write -> attention + scatter -> restore of
 * mask==1 rows. The body of the sparse attention plugin's enqueue. Workspace: see
 * fxr_workspace_size. Two kernel launches, no host synchronisation: the gather compacts the mask
 * itself, and the attention puts back the cache rows of mask==1 tokens in its tail, head by head
 * once no CTA reads that head any more (with FXR_ATTENTION_TILES=1, the one-tile kernel, a third
 * launch does that; frames of more than 1024 tokens per SM, over ~150 000 tokens on 148 SMs, exceed
 * the gather's row list and add a compaction launch). The kernels are chained with programmatic dependent launch: the last one lets
 * a successor launched the same way start early, and such a successor must wait for its
 * dependency (cudaGridDependencySynchronize) before it reads the frame's outputs, as every
 * kernel of this library does. */
int32_t fxr_frame_forward(const fxr_frame_desc* desc,
                          const void* q, const void* k, const void* v,
                          int32_t* mask, const uint8_t* valid, const int32_t* pos,
                          const float* norm_q, const float* norm_k,
                          void* cache_k, void* cache_v, void* out,
                          void* workspace, size_t workspace_bytes, void* stream);

/* One step of fxr_frame_forward, on the same arguments and workspace layout, for callers that run
 * their own work between the steps or time them one by one:
 *   FXR_STEP_COMPACT          mask preprocessing + index list of executed tokens (also zeroes the
 *                             workspace's split counters)
 *   FXR_STEP_GATHER           gather + QK-RMSNorm + RoPE + cache write of the listed rows
 *   FXR_STEP_GATHER_COMPACT   the two above in one launch, as fxr_frame_forward runs them
 *   FXR_STEP_ATTENTION        attention + scatter, with the workspace's split / stream-K scratch,
 *                             so that its schedule is the frame's
 *   FXR_STEP_RESTORE          restore of the cache rows of mask==1 tokens (launches nothing when
 *                             the attention step restored them itself, the two-tile kernel)
 * COMPACT, GATHER, ATTENTION, RESTORE in order (or GATHER_COMPACT, ATTENTION, RESTORE) give the
 * result of fxr_frame_forward bit for bit. Unused pointer arguments of a step may be null. */
enum {
    FXR_STEP_COMPACT = 0,
    FXR_STEP_GATHER = 1,
    FXR_STEP_GATHER_COMPACT = 2,
    FXR_STEP_ATTENTION = 3,
    FXR_STEP_RESTORE = 4
};
int32_t fxr_frame_step(int32_t step, const fxr_frame_desc* desc,
                       const void* q, const void* k, const void* v,
                       int32_t* mask, const uint8_t* valid, const int32_t* pos,
                       const float* norm_q, const float* norm_k,
                       void* cache_k, void* cache_v, void* out,
                       void* workspace, size_t workspace_bytes, void* stream);

/* One frame whose per-frame tensors live in page-locked host memory, for a streaming host that
 * produces each frame's projections on the CPU side and wants the output back. The reference moves
 * such tensors whole with Tensor::upload / Tensor::download (src/utils/tensor.cpp:50-56); here only
 * the executed rows cross PCIe:
 *   1. the mask is copied to the workspace and compacted on the device;
 *   2. a zero-copy kernel reads the executed tokens' Q, K, V rows from host memory into device
 *      staging rows (other rows are never read: the attention takes their K/V from the cache);
 *   3. the frame runs as fxr_frame_forward on the staging buffers, its attention on 8 fewer SMs
 *      so that the row transfers of the frames around it (another stream) keep running beside it
 *      (results equal fxr_frame_forward's bit for bit when both schedules run whole units, and
 *      within rounding when the smaller grid changes the attention's schedule);
 *   4. a zero-copy kernel writes the executed tokens' output rows into host_out.
 * Arguments:
 *   host_q, host_k, host_v  [n_tokens, n_heads * head_dim] dtype, page-locked host memory mapped
 *                           into the device's address space (cudaHostAlloc / cudaMallocHost memory
 *                           always is under unified addressing; cudaHostRegister with the mapped
 *                           flag); other memory is rejected with FXR_ERR_INVALID
 *   host_mask               [n_tokens] int32 mask in host memory (read only; its preprocessed copy
 *                           stays in the workspace)
 *   host_out                [n_tokens, n_heads * head_dim] dtype, page-locked and mapped like
 *                           host_q: the rows of executed tokens receive the attention output and
 *                           every other row keeps what it held (the output cache of the previous frame)
 *   valid, pos, norm_q, norm_k, cache_k, cache_v   device memory, as for fxr_frame_forward
 *   workspace               at least fxr_frame_host_workspace_size(desc) bytes of device memory
 * Asynchronous on `stream`; host_out is complete once the stream has passed this call, and the
 * host buffers must stay untouched until then. Six kernel launches and one 4 * n_tokens byte copy. */
size_t fxr_frame_host_workspace_size(const fxr_frame_desc* desc);
int32_t fxr_frame_forward_host(const fxr_frame_desc* desc,
                               const void* host_q, const void* host_k, const void* host_v,
                               const int32_t* host_mask, const uint8_t* valid, const int32_t* pos,
                               const float* norm_q, const float* norm_k,
                               void* cache_k, void* cache_v, void* host_out,
                               void* workspace, size_t workspace_bytes, void* stream);

/* fxr_frame_forward without a workspace argument, for callers that cannot allocate device memory
 * when they run a frame: for example a plugin enqueue inside an inference engine that owns every
 * device allocation, or a latency-critical loop that must not risk the device-wide
 * synchronisation an allocation can cause. This entry point has no counterpart in the reference.
 *   - Scratch: a fixed 128 MiB array inside this library (every GPU that loads the library holds
 *     it until the process exits). Frames whose fxr_workspace_min_size() exceeds 128 MiB are
 *     rejected with FXR_ERR_WORKSPACE; a 1024x1024 frame (4608 tokens, 24 heads, bf16/fp16) needs
 *     about 85 MB. The rest of the 128 MiB serves as the attention's optional split slots (its
 *     stream-K schedule and key-range split), exactly as a 128 MiB workspace does for
 *     fxr_frame_forward; for a 1024x1024 frame that is the full fxr_workspace_size().
 *   - No cudaMalloc, cudaFree or other allocating call is made. The first call on a device looks up
 *     the scratch address for that device (once, with that device current) and keeps it for the
 *     life of the process; make that first call before any stream capture, and do not call
 *     cudaDeviceReset on that device afterwards (the array would move and the kept address
 *     would be stale).
 *   - Every call on a device shares the same scratch, and each frame overwrites it completely
 *     before reading it (nothing has to start at zero). Calls whose work overlaps on the GPU (two
 *     streams, or two host threads) race on it: serialise them on one stream.
 * Arguments, layouts, results and errors are those of fxr_frame_forward. */
int32_t fxr_frame_forward_noalloc(const fxr_frame_desc* desc,
                                  const void* q, const void* k, const void* v,
                                  int32_t* mask, const uint8_t* valid, const int32_t* pos,
                                  const float* norm_q, const float* norm_k,
                                  void* cache_k, void* cache_v, void* out, void* stream);

/* ---- the block's projections on the executed rows -----------------------------------------------
 * The reference runs the double-stream block's dense math on every token in fp32: LayerNorm +
 * modulation (gather_scatter_kernels.cu:77-169, called at flux2_double_block_plugin.cpp:373-383),
 * the Q/K/V projections (:386-408), the out-projection (:429-432), the MLP with tanh GELU
 * (:434-448, flux2_kernels.cu:14-29) and the residual (:450-458). These functions run each step
 * on the executed rows only (compact rows m < *count of fxr_mask_compact's idx list), so the gather
 * happens before the projections and skipped tokens cost nothing.
 *
 * Executed-row LayerNorm + modulation, compact output:
 *   y[m, :] = (1 + scale) * (x[idx[m], :] - mean) / sqrt(var + eps) + shift,  m in [row0, row_end)
 * row_end < 0: *count. dim: multiple of 256, at most 4096; scale / shift: [dim] fp32 or NULL. */
int32_t fxr_ln_modulate_rows(int32_t dtype, const void* x, int64_t ld_x, int32_t dim,
                             const int32_t* idx, const int32_t* count, int32_t row0,
                             int32_t row_end, int32_t n_tokens, const float* scale,
                             const float* shift, float eps, void* y, int64_t ld_y, void* stream);

/* Executed-row GEMM with a fused epilogue (tcgen05, fp32 accumulation in tensor memory):
 *   Y[r(m), :] = act([A0 | A1][m, :] . [W0 | W1]^T + bias0 + bias1)                 or
 *   Y[r(m), :] = residual[r(m), :] + gate * ([A0 | A1][m, :] . [W0 | W1]^T + bias0 + bias1)
 * for compact rows m in [row0, row_end). Each A operand is gathered (row idx[m] of a token-major
 * buffer) or compact (row m); the output columns are cut into up to four parts, each written to
 * its own buffer, scattered (row idx[m]) or compact (row m), with or without the tanh GELU. The
 * residual (single output part only) is read at the output row. Recipes for the block:
 *   Q/K/V:          a[0] = {LN rows, compact, W_qkv};   y = {Q, K, V scattered}, bias0 = b_qkv
 *   MLP up:         a[0] = {LN rows, compact, W_mlp0};  y = {H compact, GELU},   bias0 = b_mlp0
 *   out + MLP down: a[0] = {attention output, gathered, W_out}, a[1] = {H, compact, W_mlp2};
 *                   y = {block output, scattered}, bias0 = b_out, bias1 = b_mlp2,
 *                   residual = block input, gate = the gate row (NULL: 1, as the reference)
 * K of each operand: multiple of 64; output part widths: multiples of 256; element type dtype
 * (bf16/fp16) everywhere except the fp32 bias and gate. scratch: fxr_rows_gemm_scratch_size()
 * bytes, ZERO before its first use and then reused as is (one scratch per stream; it balances the
 * work of every SM by splitting tiles over CTAs — stream-K); NULL runs whole tiles per CTA. */
#define FXR_ACT_NONE 0
#define FXR_ACT_GELU_TANH 1

typedef struct fxr_rows_operand {
    const void* rows;        /* [*, ld] */
    int64_t ld;              /* elements */
    int32_t k;               /* columns of this operand (multiple of 64) */
    int32_t gathered;        /* 1: row idx[m]; 0: row m */
    const void* w;           /* [n_out, k] with row stride ld_w (a column block of a wider W) */
    int64_t ld_w;            /* elements between W rows; 0: k */
} fxr_rows_operand;

typedef struct fxr_rows_output {
    void* rows;              /* [*, ld] */
    int64_t ld;
    int32_t cols;            /* multiple of 256 */
    int32_t scattered;       /* 1: row idx[m]; 0: row m */
    int32_t act;             /* FXR_ACT_NONE / FXR_ACT_GELU_TANH */
    int32_t reserved;
} fxr_rows_output;

typedef struct fxr_rows_gemm_desc {
    int32_t dtype;           /* FXR_BF16 or FXR_F16 */
    int32_t n_tokens;        /* bound of idx values and compact rows */
    int32_t row0;            /* compact rows [row0, row_end) */
    int32_t row_end;         /* < 0: *count */
    int32_t n_operands;      /* 1 or 2 */
    int32_t n_outputs;       /* 1 to 4 */
    fxr_rows_operand a[2];
    fxr_rows_output y[4];
    const float* bias0;      /* [n_out] fp32 or NULL */
    const float* bias1;
    const void* residual;    /* [*, ld_residual] or NULL */
    int64_t ld_residual;
    const float* gate;       /* [n_out] fp32 or NULL */
} fxr_rows_gemm_desc;

size_t fxr_rows_gemm_scratch_size(void);
int32_t fxr_rows_gemm(const fxr_rows_gemm_desc* d, const int32_t* idx, const int32_t* count,
                      void* scratch, size_t scratch_bytes, void* stream);

/* ---- the double-stream block on the executed rows -------------------------------------------------
 * One FLUX.2 double-stream block over a frame whose tokens are text [0, n_text) then image
 * [n_text, n_tokens), computing only the executed rows. The reference's Flux2DoubleBlockPlugin
 * enqueue (flux2_double_block_plugin.cpp:330-460) runs every step on every token in fp32:
 *   x_out = x_in + gate * (out_proj(attn(q, k, v)) + mlp(LN_mod(x_in))),  q/k/v = proj(LN_mod(x_in))
 * with separate text / image weights. Here, per frame (13 launches, no host synchronisation):
 *   compaction (text tokens always execute) -> LayerNorm + modulation of the executed rows ->
 *   Q/K/V (text rows with the text weights, image rows with the image weights) -> gather with each
 *   stream's QK-RMSNorm + RoPE, K/V cache rows -> joint attention of the executed queries over all
 *   cache rows -> restore of mask-1 cache rows -> MLP up (tanh GELU) -> out-projection + MLP down +
 *   gated residual into the executed rows of x_out -> validity of the updated cache rows.
 * Rows of skipped image tokens of x_out are left untouched (the caller's previous output: the
 * output cache). x_in / x_out: [n_tokens, C] contiguous, C = n_heads * head_dim (multiple of 256,
 * at most 4096); cache_k / cache_v: [n_tokens, ld_cache]; desc->ld_qkv / ld_out are not used. */
typedef struct fxr_block_stream {   /* one stream (text or image) of a double-stream block */
    const float* shift;      /* [C] modulation shift (temb[0:C] in the reference) or NULL */
    const float* scale;      /* [C] modulation scale (temb[C:2C]) or NULL */
    const float* gate;       /* [C] residual gate or NULL (1, as the reference) */
    const void* w_qkv;       /* [3C, C]: the rows of to_q, to_k, to_v stacked */
    const float* b_qkv;      /* [3C] or NULL */
    const float* norm_q;     /* [head_dim] QK-RMSNorm weights */
    const float* norm_k;
    const void* w_out;       /* [C, C] */
    const float* b_out;      /* [C] or NULL */
    const void* w_mlp0;      /* [H, C] */
    const float* b_mlp0;     /* [H] or NULL */
    const void* w_mlp2;      /* [C, H] */
    const float* b_mlp2;     /* [C] or NULL */
} fxr_block_stream;

typedef struct fxr_double_block {
    fxr_block_stream txt;    /* tokens [0, n_text) */
    fxr_block_stream img;    /* tokens [n_text, n_tokens) */
    int32_t mlp_hidden;      /* H: multiple of 256 (3C for FLUX.2) */
    float ln_eps;            /* LayerNorm eps (1e-6 in the reference) */
} fxr_double_block;

size_t fxr_double_block_workspace_size(const fxr_frame_desc* desc, int32_t mlp_hidden);
int32_t fxr_double_block_forward(const fxr_frame_desc* desc, const fxr_double_block* blk,
                                 const void* x_in, void* x_out, int32_t* mask, uint8_t* valid,
                                 const int32_t* pos, void* cache_k, void* cache_v,
                                 void* workspace, size_t workspace_bytes, void* stream);

/* ---- the single-stream block on the executed rows ------------------------------------------------
 * A FLUX.2 single-stream block: one set of weights over the joint text + image sequence, the
 * attention and the MLP fed by one fused projection and merged by one output projection
 * (to_qkv_mlp_proj and to_out, exported by tools/export_block_weights.py:79-113; the reference plans
 * the plugin, results.md:95, and has no kernel code for it):
 *   xn = LN_mod(x_in);  [q | k | v | h] = xn . W_qkv_mlp^T + b;  h = GELU(h)
 *   x_out = x_in + gate * ([attn(q, k, v) | h] . W_out^T + b_out)
 * on the executed rows only (8 launches: compaction, LayerNorm + modulation, the fused projection
 * with Q/K/V scattered and the MLP rows compact, gather + QK-RMSNorm + RoPE, attention, restore, the
 * two-operand output projection with the gated residual, cache validity). The MLP activation is
 * the tanh GELU of the reference's double block (flux2_kernels.cu:14-21). Shapes and the output
 * cache as for fxr_double_block_forward. */
typedef struct fxr_single_block {
    const float* shift;      /* [C] modulation or NULL */
    const float* scale;      /* [C] or NULL */
    const float* gate;       /* [C] or NULL (1) */
    const void* w_qkv_mlp;   /* [3C + H, C]: to_q, to_k, to_v rows, then the MLP-in rows */
    const float* b_qkv_mlp;  /* [3C + H] or NULL */
    const float* norm_q;     /* [head_dim] */
    const float* norm_k;
    const void* w_out;       /* [C, C + H]: columns [0, C) take the attention rows, [C, C + H) the MLP */
    const float* b_out;      /* [C] or NULL */
    int32_t mlp_hidden;      /* H: multiple of 256 */
    float ln_eps;
} fxr_single_block;

size_t fxr_single_block_workspace_size(const fxr_frame_desc* desc, int32_t mlp_hidden);
int32_t fxr_single_block_forward(const fxr_frame_desc* desc, const fxr_single_block* blk,
                                 const void* x_in, void* x_out, int32_t* mask, uint8_t* valid,
                                 const int32_t* pos, void* cache_k, void* cache_v,
                                 void* workspace, size_t workspace_bytes, void* stream);

/* The two blocks with the hidden states in page-locked host memory (as fxr_frame_forward_host for
 * the attention slice; the reference moves whole tensors, src/utils/tensor.cpp:50-56): host_mask
 * (int32, read only) is copied to the workspace; after the compaction a zero-copy kernel reads the
 * executed rows of host_x_in into device staging rows; the block runs on them; a zero-copy kernel
 * writes the executed rows of x_out into host_x_out, whose other rows keep the previous frame's
 * output. host_x_in / host_x_out: [n_tokens, C] page-locked and mapped (as for
 * fxr_frame_forward_host, else FXR_ERR_INVALID); valid, pos and the caches are device memory.
 * Workspace: fxr_block_host_workspace_size(desc, mlp_hidden) bytes, for either block. */
size_t fxr_block_host_workspace_size(const fxr_frame_desc* desc, int32_t mlp_hidden);
int32_t fxr_double_block_forward_host(const fxr_frame_desc* desc, const fxr_double_block* blk,
                                      const void* host_x_in, void* host_x_out, const int32_t* host_mask,
                                      uint8_t* valid, const int32_t* pos, void* cache_k, void* cache_v,
                                      void* workspace, size_t workspace_bytes, void* stream);
int32_t fxr_single_block_forward_host(const fxr_frame_desc* desc, const fxr_single_block* blk,
                                      const void* host_x_in, void* host_x_out, const int32_t* host_mask,
                                      uint8_t* valid, const int32_t* pos, void* cache_k, void* cache_v,
                                      void* workspace, size_t workspace_bytes, void* stream);

/* QKV projection of the executed tokens from token-major hidden states:
 *   [q | k | v][idx[m], :] = hidden[idx[m], :] . w_qkv^T (+ bias)   for m < *count
 * hidden: [n_tokens, ld_hidden] (k_dim columns, multiple of 64); w_qkv: [3C, k_dim] row-major
 * (C = n_heads * head_dim, multiple of 256), same element type as desc->dtype; bias: [3C] fp32 or
 * NULL; q/k/v: [n_tokens, ld_qkv] — rows of skipped tokens are left untouched. scratch as for
 * fxr_rows_gemm (NULL allowed). */
int32_t fxr_qkv_project(const fxr_frame_desc* desc, const void* hidden, int64_t ld_hidden,
                        int32_t k_dim, const void* w_qkv, const float* bias,
                        const int32_t* idx, const int32_t* count,
                        void* q, void* k, void* v, void* scratch, size_t scratch_bytes,
                        void* stream);

/* ---- independent edit streams in one set of launches -------------------------------------------
 * n_streams frames of the same geometry (the plugin's batch dimension; config 4 runs 8 streams of
 * 768x768): one gather launch over every stream's executed rows, which also compacts every
 * stream's mask, and one attention launch over every stream's (query tile, head) units — which
 * fills the GPU where one small frame leaves SMs idle — and also restores every stream's mask==1
 * cache rows (a compaction launch is added when the streams' rows exceed the gather's row list, a
 * restore launch with FXR_ATTENTION_TILES=1); more than FXR_MAX_BATCH streams run as consecutive
 * groups. Streams share the geometry, pos and the norm weights; each
 * has its own inputs, mask, validity, K/V cache and output. Results equal per-stream
 * fxr_frame_forward calls bit for bit. */
#define FXR_MAX_BATCH 8

typedef struct fxr_stream_frame {
    const void* q;
    const void* k;
    const void* v;
    int32_t* mask;            /* preprocessed in place */
    const uint8_t* valid;     /* NULL = every row valid */
    void* cache_k;
    void* cache_v;
    void* out;
} fxr_stream_frame;

/* Workspace of fxr_frame_forward_batch: min(n_streams, FXR_MAX_BATCH) frame workspaces. */
size_t fxr_batch_workspace_size(const fxr_frame_desc* desc, int32_t n_streams);

int32_t fxr_frame_forward_batch(const fxr_frame_desc* desc, int32_t n_streams,
                                const fxr_stream_frame* frames, const int32_t* pos,
                                const float* norm_q, const float* norm_k,
                                void* workspace, size_t workspace_bytes, void* stream);

/* Device pointers into the workspace (for callers that want idx / count / compact Q). */
int32_t fxr_workspace_views(const fxr_frame_desc* desc, void* workspace, int32_t** idx,
                            int32_t** count, void** qc, int64_t* ld_qc, void** save);

/* ---- one frame split by attention heads over the GPUs of one node ------------------------------
 * The reference runs a frame on one GPU. Here a high-resolution frame can be split by heads: rank r
 * (one process per GPU) owns heads [head0, head0 + n_heads), gathers, normalises and rotates its
 * heads of every executed token and keeps its heads' K/V cache locally (no cache traffic). Its
 * attention writes the executed rows of its heads compactly; an exchange kernel then stores each
 * row's slice (n_heads x head_dim contiguous elements) into the full-frame output of EVERY rank
 * through peer mappings — the all-gather and the scatter in one pass over NVLink, with coalesced
 * 16-byte stores — and each of its CTAs adds one arrival to slot `rank` of every rank's arrival
 * counters. fxr_head_group_wait makes a rank's stream wait (bounded) until all ranks' arrivals of
 * the frame are in, after which its output holds every head. */
#define FXR_MAX_RANKS 8

typedef struct fxr_head_group {
    int32_t world;                      /* ranks sharing the frame, 1..FXR_MAX_RANKS */
    int32_t rank;                       /* this rank */
    int32_t head0, n_heads;             /* this rank's heads (set by fxr_head_group_init) */
    int32_t ctas[FXR_MAX_RANKS];        /* exchange CTAs (arrivals sent) per frame, per rank */
    uint32_t epoch;                     /* frames issued by this rank (host count, informational) */
    int32_t reserved0;
    void* out[FXR_MAX_RANKS];           /* each rank's full-frame O [n_tokens, ld_out], mapped here */
    uint32_t* arrive[FXR_MAX_RANKS];    /* each rank's FXR_HEAD_GROUP_SLOTS arrival words,
                                           zero-initialised, mapped here */
} fxr_head_group;

/* uint32 words of a rank's arrival area: [0, FXR_MAX_RANKS) arrivals from each rank, then the
 * number of frames the rank has waited for (kept on the device, so a CUDA graph holding the frame
 * and its wait can be replayed). 64 bytes. */
#define FXR_HEAD_GROUP_SLOTS 16

/* Fills world, rank, the contiguous balanced head split (ranks < n_heads % world get one more
 * head), the per-rank arrival counts (all GPUs are assumed to have this GPU's SM count; none for a
 * single GPU, which stores its rows itself), epoch = 0, and clears out[] / arrive[] (the caller sets
 * them). */
int32_t fxr_head_group_init(fxr_head_group* g, int32_t world, int32_t rank, int32_t n_heads,
                            int32_t n_tokens);

/* One frame of this rank's heads. desc describes the FULL frame (n_heads = all heads, ld_qkv and
 * ld_out over all heads); q/k/v are the full-frame inputs; cache_k/cache_v hold this rank's heads
 * only, [n_tokens, g->n_heads * head_dim] packed. Workspace: fxr_workspace_size(desc) suffices.
 * Issues the gather/norm/RoPE (which also compacts the mask, and with peers writes the identity row
 * list of the compact output), the attention (which also restores the mask==1 cache rows) and, with
 * peers, the exchange with its arrivals: three launches, two on a single GPU (plus the compaction or
 * the restore launch in the cases fxr_frame_forward names). It does
 * not wait for the other ranks (fxr_head_group_wait does), so
 * a single GPU may emulate several ranks by issuing every rank's frame before any rank's wait.
 * Callers must not let a rank start frame f+1 while another rank still reads frame f's output. */
int32_t fxr_frame_forward_heads(const fxr_frame_desc* desc, fxr_head_group* g,
                                const void* q, const void* k, const void* v,
                                int32_t* mask, const uint8_t* valid, const int32_t* pos,
                                const float* norm_q, const float* norm_k,
                                void* cache_k, void* cache_v,
                                void* workspace, size_t workspace_bytes, void* stream);

/* Stream-ordered, bounded (2 s) wait until every rank's arrivals for this rank's next frame are
 * in (one wait per frame, after the frame); a timeout is reported by fxr_check_device_error
 * (bit 1). */
int32_t fxr_head_group_wait(const fxr_head_group* g, void* stream);

/* The same split with the O exchange as one NCCL all-gather instead of peer stores (the
 * collective-library baseline of the fused path). Each rank's attention writes compact O rows of
 * its heads, [m_cap, hmax * head_dim] (hmax = ceil(heads / world)); fxr_allgather_heads gathers
 * them from every rank over `nccl_comm` (an ncclComm_t of the group's ranks, rank order = g->rank)
 * and scatters them into the full-frame output rows out[idx[m]]. m_cap is a host-side upper bound
 * of the executed-token count (n_tokens is always safe; a tighter bound moves fewer bytes); a frame
 * with more executed tokens sets the device error word (bit 2) and leaves the excess rows out.
 * NCCL is resolved at run time (the libnccl.so.2 already in the process, else the loader's). */
int32_t fxr_nccl_unique_id(unsigned char id_out[128]);
int32_t fxr_nccl_comm_init(int32_t world, int32_t rank, const unsigned char id[128], void** comm);
int32_t fxr_nccl_comm_destroy(void* comm);

/* Workspace of fxr_frame_forward_heads_nccl (frame workspace + compact O + gather buffer). */
size_t fxr_heads_nccl_workspace_size(const fxr_frame_desc* desc, const fxr_head_group* g,
                                     int32_t m_cap);

/* All-gather of compact O rows + scatter into out. o_local: [m_cap, hmax*head_dim] of this rank;
 * gathered: [world, m_cap, hmax*head_dim]; idx/count: the frame's compaction; out: full frame. */
int32_t fxr_allgather_heads(const fxr_frame_desc* desc, const fxr_head_group* g, void* nccl_comm,
                            const void* o_local, int32_t m_cap, void* gathered,
                            const int32_t* idx, const int32_t* count, void* out, void* stream);

/* fxr_frame_forward_heads with the NCCL exchange: out is this rank's full-frame output; g->out and
 * g->arrive are not used. Returns when the all-gather and scatter are enqueued on `stream`. */
int32_t fxr_frame_forward_heads_nccl(const fxr_frame_desc* desc, const fxr_head_group* g,
                                     void* nccl_comm, int32_t m_cap,
                                     const void* q, const void* k, const void* v,
                                     int32_t* mask, const uint8_t* valid, const int32_t* pos,
                                     const float* norm_q, const float* norm_k,
                                     void* cache_k, void* cache_v, void* out,
                                     void* workspace, size_t workspace_bytes, void* stream);

/* Device memory shareable between the processes of one node (CUDA IPC), for the output buffers and
 * arrival counters of a head group. fxr_ipc_alloc zero-fills `bytes` on the current device and
 * returns a 64-byte handle; fxr_ipc_open maps another process's handle (peer access enabled on
 * first use); fxr_ipc_close unmaps it; fxr_ipc_free releases an allocation of this process. */
typedef struct fxr_ipc_handle {
    unsigned char bytes[64];
} fxr_ipc_handle;

int32_t fxr_ipc_alloc(size_t bytes, void** ptr, fxr_ipc_handle* handle);
int32_t fxr_ipc_open(const fxr_ipc_handle* handle, void** ptr);
int32_t fxr_ipc_close(void* ptr);
int32_t fxr_ipc_free(void* ptr);

#ifdef __cplusplus
}
#endif
#endif /* FXR_H */
