/*
 * fxr_plugin.h — C ABI of the sparse attention plugin core (Flux2SparseAttnPlugin).
 *
 * The reference's engine runs its custom layers as TensorRT IPluginV3 plugins derived from
 * Flux2PluginBase (fluxrt-cpp src/inference/plugins/flux2_plugin_base.h:30-121), created by an
 * IPluginCreatorV3One from a PluginFieldCollection (flux2_plugin_base.h:126-141,
 * flux2_double_block_plugin.cpp:476-496) and executed through enqueue(), which returns 0 / -1
 * (flux2_double_block_plugin.cpp:202-231). This header exposes the same lifecycle without
 * TensorRT types, so the plugin body is usable and testable where the TensorRT SDK is absent; the
 * IPluginV3 class in csrc/fxr_sparse_attn_plugin.cpp forwards to these functions when
 * NvInferRuntime.h is available.
 *
 * Plugin name "Flux2SparseAttnPlugin", version "1", namespace "fluxrt" (the reference's
 * name/version/namespace scheme, flux2_double_block_plugin.cpp:54).
 *
 * Tensors (batch B of independent edit streams, N = n_txt + image tokens, C = num_heads * 128):
 *   inputs  0 Q      [B, N, C]  bf16 or fp16 (kLINEAR)
 *           1 K      [B, N, C]  same type as Q
 *           2 V      [B, N, C]  same type as Q
 *           3 mask   [B, N]     int32 (0 skip, 1 execute, 2 execute + update)
 *           4 pos    [N, n_axes] int32 RoPE position ids
 *           5 norm_q [128]      fp32
 *           6 norm_k [128]      fp32
 *   output  0 O      [B, N, C]  same type as Q; rows of skipped tokens are left untouched
 * State owned by the plugin (per batch element, allocated by configure): the attention K/V cache
 * [N, C] x 2 and the per-token validity flags (a token is executed while its cache row is invalid;
 * image tokens become valid once updated, text tokens are always executed).
 */
#ifndef FXR_PLUGIN_H
#define FXR_PLUGIN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Field types, numbered as nvinfer1::PluginFieldType (kFLOAT32 = 1, kINT32 = 3, kCHAR = 6). */
enum { FXR_FIELD_FLOAT32 = 1, FXR_FIELD_INT32 = 3, FXR_FIELD_CHAR = 6 };

/* Mirrors nvinfer1::PluginField: name, data, type, number of elements. */
typedef struct fxr_plugin_field {
    const char* name;
    const void* data;
    int32_t type;
    int32_t length;
} fxr_plugin_field;

/* Mirrors the parts of nvinfer1::PluginTensorDesc the plugin reads: dims and element type. */
typedef struct fxr_tensor_desc {
    int32_t nb_dims;
    int32_t dtype;          /* fxr_dtype, or 3 for int32 */
    int64_t dims[8];
} fxr_tensor_desc;

#define FXR_DTYPE_INT32 3

typedef struct fxr_plugin fxr_plugin;

/* Creator: fields "num_heads" (int32, 24), "head_dim" (int32, 128), "n_txt" (int32),
 * "rope_axes" (int32[1..4], 16/56/56), "rope_theta" (float32, 10000), "eps" (float32, 1e-6),
 * "layer_idx" (int32, 0). Unknown fields are an error. Returns NULL on error
 * (fxr_last_error_string() says why). */
fxr_plugin* fxr_plugin_create(const fxr_plugin_field* fields, int32_t nb_fields);
/* IPluginV3::clone / attachToContext: same fields, no state (configure again). */
fxr_plugin* fxr_plugin_clone(const fxr_plugin* p);
void fxr_plugin_destroy(fxr_plugin* p);

const char* fxr_plugin_name(void);
const char* fxr_plugin_version(void);
const char* fxr_plugin_namespace(void);

/* IPluginV3OneCore::getFieldsToSerialize: writes up to `cap` fields, returns the number of fields.
 * The field data pointers stay valid for the plugin's lifetime. */
int32_t fxr_plugin_fields(const fxr_plugin* p, fxr_plugin_field* out, int32_t cap);

/* IPluginV3OneBuild::getOutputShapes / getOutputDataTypes: output 0 has Q's shape and type. */
int32_t fxr_plugin_output_desc(const fxr_plugin* p, const fxr_tensor_desc* in, int32_t nb_in,
                               fxr_tensor_desc* out, int32_t nb_out);
/* IPluginV3OneBuild::supportsFormatCombination for linear tensors: 1 supported, 0 not. */
int32_t fxr_plugin_supports(const fxr_plugin* p, int32_t pos, const fxr_tensor_desc* in_out,
                            int32_t nb_in, int32_t nb_out);
/* IPluginV3OneBuild::configurePlugin / IPluginV3OneRuntime::onShapeChange: validates the shapes
 * and (re)allocates the per-stream K/V caches and validity flags (all rows invalid). */
int32_t fxr_plugin_configure(fxr_plugin* p, const fxr_tensor_desc* in, int32_t nb_in,
                             const fxr_tensor_desc* out, int32_t nb_out);
/* Workspace bytes enqueue needs for these shapes. */
size_t fxr_plugin_workspace_size(const fxr_plugin* p, const fxr_tensor_desc* in, int32_t nb_in);
/* IPluginV3OneRuntime::enqueue: 0 on success, -1 on failure. */
int32_t fxr_plugin_enqueue(fxr_plugin* p, const fxr_tensor_desc* in, const fxr_tensor_desc* out,
                           const void* const* inputs, void* const* outputs, void* workspace,
                           size_t workspace_bytes, void* stream);
/* Cache access for callers that inspect or seed the state (device pointers of stream b). */
int32_t fxr_plugin_cache(fxr_plugin* p, int32_t b, void** cache_k, void** cache_v, uint8_t** valid);

#ifdef __cplusplus
}
#endif
#endif /* FXR_PLUGIN_H */
