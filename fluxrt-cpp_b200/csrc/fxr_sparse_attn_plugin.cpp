// fxr_sparse_attn_plugin.cpp — Flux2SparseAttnPlugin: the sparse attention frame as an inference
// engine plugin. The TensorRT-independent core (fields, shape/type/format rules, configure,
// workspace, enqueue, owned cache state) is exported through the C ABI of include/fxr_plugin.h;
// when TensorRT headers are present the IPluginV3 class at the end of this file forwards to it
// through the reference's plugin base (flux2_plugin_base.h:30-121).
#include "fxr_plugin.h"

#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "fxr.h"

extern "C" void fxr_internal_set_error(const char* msg);

namespace {

int32_t plugin_fail(const std::string& msg) {
    fxr_internal_set_error(msg.c_str());
    return -1;
}

size_t align256(size_t x) { return (x + 255) / 256 * 256; }

}  // namespace

namespace fluxrt {
namespace plugins {

// Plugin state. Fields follow the reference creator's parsing style
// (flux2_double_block_plugin.cpp:481-493): named scalars with defaults.
class SparseAttnCore {
public:
    int32_t num_heads = 24;
    int32_t head_dim = 128;
    int32_t n_txt = 0;
    int32_t layer_idx = 0;
    int32_t rope_n_axes = 3;
    int32_t rope_axes[4] = {16, 56, 56, 0};
    float rope_theta = 10000.f;
    float eps = 1e-6f;

    SparseAttnCore() = default;
    SparseAttnCore(const SparseAttnCore& o)
        : num_heads(o.num_heads), head_dim(o.head_dim), n_txt(o.n_txt), layer_idx(o.layer_idx),
          rope_n_axes(o.rope_n_axes), rope_theta(o.rope_theta), eps(o.eps) {
        std::memcpy(rope_axes, o.rope_axes, sizeof(rope_axes));
    }
    SparseAttnCore& operator=(const SparseAttnCore&) = delete;
    ~SparseAttnCore() { release(); }

    bool set_field(const fxr_plugin_field& f, std::string* err) {
        auto int_field = [&](int32_t* dst) {
            if (f.type != FXR_FIELD_INT32 || f.length != 1 || !f.data) {
                *err = std::string("field ") + f.name + " must be one int32";
                return false;
            }
            *dst = *static_cast<const int32_t*>(f.data);
            return true;
        };
        auto float_field = [&](float* dst) {
            if (f.type != FXR_FIELD_FLOAT32 || f.length != 1 || !f.data) {
                *err = std::string("field ") + f.name + " must be one float32";
                return false;
            }
            *dst = *static_cast<const float*>(f.data);
            return true;
        };
        if (!f.name) {
            *err = "field without a name";
            return false;
        }
        if (!std::strcmp(f.name, "num_heads")) return int_field(&num_heads);
        if (!std::strcmp(f.name, "head_dim")) return int_field(&head_dim);
        if (!std::strcmp(f.name, "n_txt")) return int_field(&n_txt);
        if (!std::strcmp(f.name, "layer_idx")) return int_field(&layer_idx);
        if (!std::strcmp(f.name, "rope_theta")) return float_field(&rope_theta);
        if (!std::strcmp(f.name, "eps")) return float_field(&eps);
        if (!std::strcmp(f.name, "rope_axes")) {
            if (f.type != FXR_FIELD_INT32 || f.length < 1 || f.length > 4 || !f.data) {
                *err = "field rope_axes must be 1 to 4 int32";
                return false;
            }
            rope_n_axes = f.length;
            for (int a = 0; a < 4; ++a)
                rope_axes[a] = a < f.length ? static_cast<const int32_t*>(f.data)[a] : 0;
            return true;
        }
        *err = std::string("unknown field ") + f.name;
        return false;
    }

    bool validate(std::string* err) const {
        if (num_heads <= 0 || head_dim != 128 || n_txt < 0) {
            *err = "num_heads > 0, head_dim == 128 and n_txt >= 0 are required";
            return false;
        }
        int sum = 0;
        for (int a = 0; a < rope_n_axes; ++a) {
            if (rope_axes[a] <= 0 || (rope_axes[a] & 1)) {
                *err = "rope_axes entries must be positive and even";
                return false;
            }
            sum += rope_axes[a];
        }
        if (sum > head_dim || !(rope_theta > 0.f) || !(eps >= 0.f)) {
            *err = "rope axes exceed head_dim, or rope_theta / eps out of range";
            return false;
        }
        return true;
    }

    std::vector<fxr_plugin_field> fields() const {
        return {{"num_heads", &num_heads, FXR_FIELD_INT32, 1},
                {"head_dim", &head_dim, FXR_FIELD_INT32, 1},
                {"n_txt", &n_txt, FXR_FIELD_INT32, 1},
                {"layer_idx", &layer_idx, FXR_FIELD_INT32, 1},
                {"rope_axes", rope_axes, FXR_FIELD_INT32, rope_n_axes},
                {"rope_theta", &rope_theta, FXR_FIELD_FLOAT32, 1},
                {"eps", &eps, FXR_FIELD_FLOAT32, 1}};
    }

    fxr_frame_desc desc(int32_t n_tokens, int32_t dtype) const {
        fxr_frame_desc d{};
        d.n_tokens = n_tokens;
        d.n_text = n_txt;
        d.n_heads = num_heads;
        d.head_dim = head_dim;
        d.dtype = dtype;
        d.rope_n_axes = rope_n_axes;
        for (int a = 0; a < 4; ++a) d.rope_axes_dim[a] = rope_axes[a];
        d.rope_theta = rope_theta;
        d.eps = eps;
        d.softmax_scale = 0.f;
        d.ld_qkv = d.ld_cache = d.ld_out = (int64_t)num_heads * head_dim;
        return d;
    }

    // Shapes: see include/fxr_plugin.h. Returns false with a message when they do not fit.
    bool check_shapes(const fxr_tensor_desc* in, int32_t nb_in, int32_t* B, int32_t* N,
                      int32_t* dtype, std::string* err) const {
        if (nb_in != 7 || !in) {
            *err = "the plugin takes 7 inputs";
            return false;
        }
        const fxr_tensor_desc& q = in[0];
        const int64_t C = (int64_t)num_heads * head_dim;
        if (q.nb_dims != 3 || q.dims[2] != C || q.dims[0] <= 0 || q.dims[1] <= 0 ||
            (q.dtype != FXR_BF16 && q.dtype != FXR_F16)) {
            *err = "input 0 (Q) must be [B, N, num_heads*head_dim] bf16 or fp16";
            return false;
        }
        for (int t = 1; t <= 2; ++t) {
            if (in[t].nb_dims != 3 || in[t].dtype != q.dtype || in[t].dims[0] != q.dims[0] ||
                in[t].dims[1] != q.dims[1] || in[t].dims[2] != C) {
                *err = "inputs 1, 2 (K, V) must match Q";
                return false;
            }
        }
        if (in[3].nb_dims != 2 || in[3].dtype != FXR_DTYPE_INT32 || in[3].dims[0] != q.dims[0] ||
            in[3].dims[1] != q.dims[1]) {
            *err = "input 3 (mask) must be [B, N] int32";
            return false;
        }
        if (in[4].nb_dims != 2 || in[4].dtype != FXR_DTYPE_INT32 || in[4].dims[0] != q.dims[1] ||
            in[4].dims[1] != rope_n_axes) {
            *err = "input 4 (pos) must be [N, n_axes] int32";
            return false;
        }
        for (int t = 5; t <= 6; ++t) {
            if (in[t].nb_dims != 1 || in[t].dtype != FXR_F32 || in[t].dims[0] != head_dim) {
                *err = "inputs 5, 6 (norm weights) must be [head_dim] fp32";
                return false;
            }
        }
        if (q.dims[1] <= n_txt || q.dims[1] > (int64_t)1 << 30) {
            *err = "N must exceed n_txt";
            return false;
        }
        *B = (int32_t)q.dims[0];
        *N = (int32_t)q.dims[1];
        *dtype = q.dtype;
        return true;
    }

    // The frames of all B streams run as one batched set of launches (fxr_frame_forward_batch);
    // the engine's read-only masks are copied behind that workspace.
    size_t workspace_bytes_for(int32_t B, int32_t N, int32_t dtype) const {
        fxr_frame_desc d = desc(N, dtype);
        return fxr_batch_workspace_size(&d, B) + (size_t)B * align256((size_t)N * sizeof(int32_t));
    }

    void release() {
        for (void* p : ck_) cudaFree(p);
        for (void* p : cv_) cudaFree(p);
        for (void* p : valid_) cudaFree(p);
        ck_.clear();
        cv_.clear();
        valid_.clear();
        B_ = N_ = 0;
        dtype_ = -1;
    }

    int32_t configure(int32_t B, int32_t N, int32_t dtype) {
        if (B == B_ && N == N_ && dtype == dtype_) return 0;
        release();
        const size_t row = (size_t)num_heads * head_dim * 2;
        for (int32_t b = 0; b < B; ++b) {
            void *k = nullptr, *v = nullptr, *f = nullptr;
            if (cudaMalloc(&k, row * N) != cudaSuccess || cudaMalloc(&v, row * N) != cudaSuccess ||
                cudaMalloc(&f, N) != cudaSuccess) {
                if (k) cudaFree(k);
                if (v) cudaFree(v);
                if (f) cudaFree(f);
                release();
                return plugin_fail("cudaMalloc of the plugin K/V cache failed");
            }
            ck_.push_back(k);
            cv_.push_back(v);
            valid_.push_back(f);
            if (cudaMemset(k, 0, row * N) != cudaSuccess || cudaMemset(v, 0, row * N) != cudaSuccess ||
                cudaMemset(f, 0, N) != cudaSuccess) {
                release();
                return plugin_fail("cudaMemset of the plugin state failed");
            }
        }
        B_ = B;
        N_ = N;
        dtype_ = dtype;
        return 0;
    }

    int32_t enqueue(const fxr_tensor_desc* in, const void* const* inputs, void* const* outputs,
                    void* workspace, size_t workspace_bytes, cudaStream_t stream) {
        std::string err;
        int32_t B = 0, N = 0, dtype = 0;
        if (!check_shapes(in, 7, &B, &N, &dtype, &err)) return plugin_fail(err);
        if (B != B_ || N != N_ || dtype != dtype_) return plugin_fail("enqueue shapes differ from configure");
        if (!inputs || !outputs || !workspace) return plugin_fail("null tensor or workspace pointer");
        const fxr_frame_desc d = desc(N, dtype);
        const size_t frames_ws = fxr_batch_workspace_size(&d, B);
        if (workspace_bytes < workspace_bytes_for(B, N, dtype)) return plugin_fail("workspace too small");
        // The engine's input tensors are read-only; the preprocess rewrites the mask in place, so
        // every stream's mask is first copied into the workspace (one copy for all streams).
        char* mask_area = static_cast<char*>(workspace) + frames_ws;
        const size_t mask_stride = align256((size_t)N * sizeof(int32_t));
        for (int32_t b = 0; b < B; ++b)
            if (cudaMemcpyAsync(mask_area + b * mask_stride, static_cast<const int32_t*>(inputs[3]) + (size_t)b * N,
                                (size_t)N * sizeof(int32_t), cudaMemcpyDeviceToDevice, stream) != cudaSuccess)
                return plugin_fail("mask copy failed");
        const size_t elem = 2, C = (size_t)num_heads * head_dim;
        std::vector<fxr_stream_frame> fr((size_t)B);
        for (int32_t b = 0; b < B; ++b) {
            const size_t off = (size_t)b * N * C * elem;
            fr[b].q = static_cast<const char*>(inputs[0]) + off;
            fr[b].k = static_cast<const char*>(inputs[1]) + off;
            fr[b].v = static_cast<const char*>(inputs[2]) + off;
            fr[b].mask = reinterpret_cast<int32_t*>(mask_area + b * mask_stride);
            fr[b].valid = static_cast<const uint8_t*>(valid_[b]);
            fr[b].cache_k = ck_[b];
            fr[b].cache_v = cv_[b];
            fr[b].out = static_cast<char*>(outputs[0]) + off;
        }
        int32_t st = fxr_frame_forward_batch(&d, B, fr.data(), static_cast<const int32_t*>(inputs[4]),
                                             static_cast<const float*>(inputs[5]),
                                             static_cast<const float*>(inputs[6]), workspace, frames_ws, stream);
        for (int32_t b = 0; st == FXR_OK && b < B; ++b)
            st = fxr_mark_updated(fr[b].mask, static_cast<uint8_t*>(valid_[b]), n_txt, N, stream);
        return st == FXR_OK ? 0 : -1;  // fxr_last_error_string() describes a failure
    }

    int32_t cache(int32_t b, void** k, void** v, uint8_t** valid) {
        if (b < 0 || b >= B_) return plugin_fail("stream index out of range (configure first)");
        if (k) *k = ck_[b];
        if (v) *v = cv_[b];
        if (valid) *valid = static_cast<uint8_t*>(valid_[b]);
        return 0;
    }

private:
    int32_t B_ = 0, N_ = 0, dtype_ = -1;
    std::vector<void*> ck_, cv_, valid_;
};

}  // namespace plugins
}  // namespace fluxrt

struct fxr_plugin {
    fluxrt::plugins::SparseAttnCore core;
    std::vector<fxr_plugin_field> serialized;
};

extern "C" {

const char* fxr_plugin_name(void) { return "Flux2SparseAttnPlugin"; }
const char* fxr_plugin_version(void) { return "1"; }
const char* fxr_plugin_namespace(void) { return "fluxrt"; }

fxr_plugin* fxr_plugin_create(const fxr_plugin_field* fields, int32_t nb_fields) {
    if (nb_fields < 0 || (nb_fields > 0 && !fields)) {
        plugin_fail("bad field collection");
        return nullptr;
    }
    fxr_plugin* p = new (std::nothrow) fxr_plugin();
    if (!p) {
        plugin_fail("out of host memory");
        return nullptr;
    }
    std::string err;
    for (int32_t i = 0; i < nb_fields; ++i) {
        if (!p->core.set_field(fields[i], &err)) {
            delete p;
            plugin_fail(err);
            return nullptr;
        }
    }
    if (!p->core.validate(&err)) {
        delete p;
        plugin_fail(err);
        return nullptr;
    }
    p->serialized = p->core.fields();
    return p;
}

fxr_plugin* fxr_plugin_clone(const fxr_plugin* src) {
    if (!src) return nullptr;
    fxr_plugin* p = new (std::nothrow) fxr_plugin{src->core, {}};
    if (p) p->serialized = p->core.fields();
    return p;
}

void fxr_plugin_destroy(fxr_plugin* p) { delete p; }

int32_t fxr_plugin_fields(const fxr_plugin* p, fxr_plugin_field* out, int32_t cap) {
    if (!p) return plugin_fail("null plugin");
    const int32_t n = (int32_t)p->serialized.size();
    for (int32_t i = 0; i < n && i < cap && out; ++i) out[i] = p->serialized[i];
    return n;
}

int32_t fxr_plugin_output_desc(const fxr_plugin* p, const fxr_tensor_desc* in, int32_t nb_in,
                               fxr_tensor_desc* out, int32_t nb_out) {
    if (!p || !out || nb_out != 1) return plugin_fail("the plugin has one output");
    std::string err;
    int32_t B, N, dt;
    if (!p->core.check_shapes(in, nb_in, &B, &N, &dt, &err)) return plugin_fail(err);
    out[0] = in[0];
    return 0;
}

int32_t fxr_plugin_supports(const fxr_plugin* p, int32_t pos, const fxr_tensor_desc* io,
                            int32_t nb_in, int32_t nb_out) {
    if (!p || !io || nb_in != 7 || nb_out != 1 || pos < 0 || pos >= 8) return 0;
    const int32_t t = io[pos].dtype;
    switch (pos) {
        case 0: return t == FXR_BF16 || t == FXR_F16;
        case 1: case 2: case 7: return t == io[0].dtype;
        case 3: case 4: return t == FXR_DTYPE_INT32;
        default: return t == FXR_F32;
    }
}

int32_t fxr_plugin_configure(fxr_plugin* p, const fxr_tensor_desc* in, int32_t nb_in,
                             const fxr_tensor_desc* out, int32_t nb_out) {
    if (!p) return plugin_fail("null plugin");
    std::string err;
    int32_t B, N, dt;
    if (!p->core.check_shapes(in, nb_in, &B, &N, &dt, &err)) return plugin_fail(err);
    if (out && nb_out == 1 && (out[0].nb_dims != 3 || out[0].dtype != dt || out[0].dims[0] != B ||
                              out[0].dims[1] != N || out[0].dims[2] != in[0].dims[2]))
        return plugin_fail("output 0 must match Q");
    return p->core.configure(B, N, dt);
}

size_t fxr_plugin_workspace_size(const fxr_plugin* p, const fxr_tensor_desc* in, int32_t nb_in) {
    if (!p) return 0;
    std::string err;
    int32_t B, N, dt;
    if (!p->core.check_shapes(in, nb_in, &B, &N, &dt, &err)) return 0;
    return p->core.workspace_bytes_for(B, N, dt);
}

int32_t fxr_plugin_enqueue(fxr_plugin* p, const fxr_tensor_desc* in, const fxr_tensor_desc* out,
                           const void* const* inputs, void* const* outputs, void* workspace,
                           size_t workspace_bytes, void* stream) {
    (void)out;
    if (!p) return plugin_fail("null plugin");
    return p->core.enqueue(in, inputs, outputs, workspace, workspace_bytes,
                           static_cast<cudaStream_t>(stream));
}

int32_t fxr_plugin_cache(fxr_plugin* p, int32_t b, void** cache_k, void** cache_v, uint8_t** valid) {
    if (!p) return plugin_fail("null plugin");
    return p->core.cache(b, cache_k, cache_v, valid);
}

}  // extern "C"

// ------------------------------------------------------------------------------------------------
// TensorRT IPluginV3 binding, compiled inside the fluxrt-cpp tree (next to flux2_plugin_base.h)
// with -DFXR_WITH_TENSORRT when the TensorRT SDK is installed.
// ------------------------------------------------------------------------------------------------
#if defined(FXR_WITH_TENSORRT) && __has_include(<NvInferRuntime.h>) && __has_include("flux2_plugin_base.h")
#include <NvInferRuntime.h>

#include "flux2_plugin_base.h"

namespace fluxrt {
namespace plugins {

static int32_t to_fxr_type(DataType t) {
    switch (t) {
        case DataType::kBF16: return FXR_BF16;
        case DataType::kHALF: return FXR_F16;
        case DataType::kFLOAT: return FXR_F32;
        case DataType::kINT32: return FXR_DTYPE_INT32;
        default: return -1;
    }
}

static fxr_tensor_desc to_fxr(PluginTensorDesc const& d) {
    fxr_tensor_desc t{};
    t.nb_dims = d.dims.nbDims;
    t.dtype = to_fxr_type(d.type);
    for (int i = 0; i < d.dims.nbDims && i < 8; ++i) t.dims[i] = d.dims.d[i];
    return t;
}

class Flux2SparseAttnPlugin : public Flux2PluginBase {
public:
    explicit Flux2SparseAttnPlugin(fxr_plugin* core)
        : Flux2PluginBase(fxr_plugin_name(), fxr_plugin_version(), fxr_plugin_namespace()), core_(core) {}
    ~Flux2SparseAttnPlugin() override { fxr_plugin_destroy(core_); }
    IPluginV3* clone() noexcept override { return new Flux2SparseAttnPlugin(fxr_plugin_clone(core_)); }
    int32_t getNbOutputs() const noexcept override { return 1; }
    size_t getWorkspaceSize(DynamicPluginTensorDesc const* in, int32_t nb_in,
                            DynamicPluginTensorDesc const*, int32_t) const noexcept override {
        std::vector<fxr_tensor_desc> d(nb_in);
        for (int i = 0; i < nb_in; ++i) {
            d[i] = fxr_tensor_desc{in[i].max.nbDims, to_fxr_type(in[i].desc.type), {}};
            for (int k = 0; k < in[i].max.nbDims && k < 8; ++k) d[i].dims[k] = in[i].max.d[k];
        }
        return fxr_plugin_workspace_size(core_, d.data(), nb_in);
    }

protected:
    int32_t configurePluginImpl(DynamicPluginTensorDesc const*, int32_t, DynamicPluginTensorDesc const*,
                                int32_t) noexcept override { return 0; }
    int32_t getOutputDataTypesImpl(DataType* out, int32_t nb_out, DataType const* in,
                                   int32_t nb_in) const noexcept override {
        if (nb_out != 1 || nb_in != 7) return -1;
        out[0] = in[0];
        return 0;
    }
    int32_t getOutputShapesImpl(DimsExprs const* in, int32_t nb_in, DimsExprs const*, int32_t,
                                DimsExprs* out, int32_t nb_out, IExprBuilder&) noexcept override {
        if (nb_in != 7 || nb_out != 1) return -1;
        out[0] = in[0];
        return 0;
    }
    bool supportsFormatCombinationImpl(int32_t pos, DynamicPluginTensorDesc const* io, int32_t nb_in,
                                       int32_t nb_out) noexcept override {
        if (io[pos].desc.format != TensorFormat::kLINEAR) return false;
        std::vector<fxr_tensor_desc> d(nb_in + nb_out);
        for (int i = 0; i < nb_in + nb_out; ++i) d[i].dtype = to_fxr_type(io[i].desc.type);
        return fxr_plugin_supports(core_, pos, d.data(), nb_in, nb_out) == 1;
    }
    int32_t onShapeChangeImpl(PluginTensorDesc const* in, int32_t nb_in, PluginTensorDesc const* out,
                              int32_t nb_out) noexcept override {
        std::vector<fxr_tensor_desc> di(nb_in), dout(nb_out);
        for (int i = 0; i < nb_in; ++i) di[i] = to_fxr(in[i]);
        for (int i = 0; i < nb_out; ++i) dout[i] = to_fxr(out[i]);
        return fxr_plugin_configure(core_, di.data(), nb_in, dout.data(), nb_out);
    }
    int32_t enqueueImpl(PluginTensorDesc const* in, PluginTensorDesc const* out, void const* const* inputs,
                        void* const* outputs, void* workspace, cudaStream_t stream) noexcept override {
        std::vector<fxr_tensor_desc> di(7);
        for (int i = 0; i < 7; ++i) di[i] = to_fxr(in[i]);
        fxr_tensor_desc dout = to_fxr(out[0]);
        return fxr_plugin_enqueue(core_, di.data(), &dout, inputs, outputs, workspace,
                                  fxr_plugin_workspace_size(core_, di.data(), 7), stream);
    }
    PluginFieldCollection const* getFieldsToSerializeImpl() noexcept override {
        fxr_plugin_field f[8];
        const int32_t n = fxr_plugin_fields(core_, f, 8);
        fields_.clear();
        for (int32_t i = 0; i < n; ++i)
            fields_.emplace_back(f[i].name, f[i].data, static_cast<PluginFieldType>(f[i].type), f[i].length);
        fc_.nbFields = (int32_t)fields_.size();
        fc_.fields = fields_.data();
        return &fc_;
    }

private:
    fxr_plugin* core_;
    std::vector<PluginField> fields_;
    PluginFieldCollection fc_{};
};

class Flux2SparseAttnPluginCreator : public Flux2PluginCreatorBase {
public:
    Flux2SparseAttnPluginCreator()
        : Flux2PluginCreatorBase(fxr_plugin_name(), fxr_plugin_version(), fxr_plugin_namespace()) {
        fieldVec_ = {PluginField("num_heads", nullptr, PluginFieldType::kINT32, 1),
                     PluginField("head_dim", nullptr, PluginFieldType::kINT32, 1),
                     PluginField("n_txt", nullptr, PluginFieldType::kINT32, 1),
                     PluginField("layer_idx", nullptr, PluginFieldType::kINT32, 1),
                     PluginField("rope_axes", nullptr, PluginFieldType::kINT32, 4),
                     PluginField("rope_theta", nullptr, PluginFieldType::kFLOAT32, 1),
                     PluginField("eps", nullptr, PluginFieldType::kFLOAT32, 1)};
    }
    IPluginV3* createPlugin(AsciiChar const*, PluginFieldCollection const* fc, TensorRTPhase) noexcept override {
        std::vector<fxr_plugin_field> f(fc ? fc->nbFields : 0);
        for (size_t i = 0; i < f.size(); ++i)
            f[i] = fxr_plugin_field{fc->fields[i].name, fc->fields[i].data,
                                    static_cast<int32_t>(fc->fields[i].type), fc->fields[i].length};
        fxr_plugin* core = fxr_plugin_create(f.data(), (int32_t)f.size());
        return core ? new Flux2SparseAttnPlugin(core) : nullptr;
    }
};

REGISTER_TENSORRT_PLUGIN(Flux2SparseAttnPluginCreator);

}  // namespace plugins
}  // namespace fluxrt
#endif
