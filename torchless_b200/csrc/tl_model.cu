// tl_model.cu -- device-resident Mistral model behind the model-level C ABI.
//
// Stands in for three reference types at once:
//   Parameters      (src/loader/parameters.cpp:95-155): parses the same binary
//                   header, but uploads every tensor once into HBM instead of
//                   keeping views into an mmap;
//   InferenceState  (src/model/mistral/inference_state.h): fp32 KV cache
//                   [L][KV][max_seq][hd] and all activations live on the
//                   device; `pos` is a device counter mirrored on the host;
//   Model<int8_t>   (src/model/mistral/modules.cpp:118-171): one decode step is
//                   a fixed sequence of 2 + 5 L kernel launches, captured once
//                   into a CUDA graph with programmatic dependent launch
//                   between kernels and replayed per token.
//
// HBM layout (per layer, 256-byte aligned blocks):
//   int8   [q_proj; k_proj; v_proj] rows concatenated   [(H + 2 KV) hd, D]
//          o_proj [D, H hd], gate_proj [F, D], up_proj [F, D], down_proj [D, F]
//   fp32   1/scale for each of the above (same order as the file's scales)
//          input/post-attention norm gains [D]
// global:  embedding [V, D], final norm [D], lm_head [V, D] (fp32, as exported)
//
// Per step: embed -> L x {qkv(+RMSNorm), attention(+RoPE, push_kv),
// o_proj(+residual), gate/up(+RMSNorm, SiLU*up), down_proj(+residual)}
// -> lm_head(+RMSNorm, argmax, pos++).
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cerrno>
#include <cmath>
#include <cstdio>
#include <array>
#include <cstring>
#include <functional>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "tl_common.cuh"
#include "tl_decode.cuh"
#include "tl_gemm.cuh"
#include "tl_prefill.cuh"
#include "tl_sample.cuh"
#include "tl_batch.cuh"
#include "tl_gemv.cuh"
#include "tl_json.h"
#include "tl_kernels.h"

namespace tl {
namespace {

// Cached positions + 1 from which the persistent decode step runs GQA
// attention (one CTA per kv group and split) instead of per-head attention.
constexpr int kGqaFromDefault = 1024;
constexpr int kGqaRowsDefault = 64;           // GQA attention: cached positions per split (at least)
constexpr int kSplitRowsDefault = 64;         // per-head attention: cached positions per split (at least)
constexpr int kKvPrefetchRowsDefault = 256;   // K (and V) rows per attention CTA hinted into L2

struct TensorRec {
    std::string dtype;
    std::vector<int64_t> shape;
    uint64_t offset = 0, scale_offset = 0, scale_size = 0;
    bool has_scales = false;
    uint64_t numel() const {
        uint64_t n = 1;
        for (auto d : shape) n *= static_cast<uint64_t>(d);
        return n;
    }
};

struct Header {
    tl_config cfg = {};
    std::map<std::string, TensorRec> tensors;
    const uint8_t* payload = nullptr;
    uint64_t payload_size = 0;
};

// std::stoi / std::stof semantics of Parameters::load_config
// (parameters.cpp:32-47): metadata values are strings.
bool meta_num(const JValue& m, const char* key, double& out) {
    const JValue* v = m.get(key);
    if (!v) return false;
    if (v->type == JValue::Str) {
        char* e = nullptr;
        out = std::strtod(v->s.c_str(), &e);
        return e != v->s.c_str();
    }
    if (v->is_num()) {
        out = v->f;
        return true;
    }
    return false;
}

tl_status parse_header(const uint8_t* data, size_t size, Header& h) {
    if (size < 8) return set_error(TL_ERR_FORMAT, "model binary shorter than its 8-byte header length");
    uint64_t hsize = 0;
    std::memcpy(&hsize, data, 8);
    if (hsize > size - 8) return set_error(TL_ERR_FORMAT, "header length %llu exceeds the file (%zu bytes)",
                                           static_cast<unsigned long long>(hsize), size);
    // The header is zero-padded to a 64-byte boundary (export_mistral.py:145-150);
    // the reference parses up to the first NUL (parameters.cpp:108-112).
    size_t jlen = 0;
    while (jlen < hsize && data[8 + jlen] != 0) jlen++;
    JValue root;
    std::string err;
    JsonParser parser(reinterpret_cast<const char*>(data + 8), jlen);
    if (!parser.parse(root, err)) return set_error(TL_ERR_FORMAT, "header JSON: %s", err.c_str());
    const JValue* meta = root.get("metadata");
    const JValue* tens = root.get("tensors");
    if (!meta || meta->type != JValue::Obj || !tens || tens->type != JValue::Obj)
        return set_error(TL_ERR_FORMAT, "header lacks metadata/tensors objects");

    double v[9];
    const char* keys[9] = {"hidden_size", "intermediate_size", "n_layers", "n_heads", "n_kv_heads",
                           "vocab_size", "max_position_embeddings", "rope_theta", "norm_eps"};
    for (int k = 0; k < 9; k++)
        if (!meta_num(*meta, keys[k], v[k])) return set_error(TL_ERR_FORMAT, "metadata.%s missing or not a number", keys[k]);
    tl_config& c = h.cfg;
    c.hidden_size = static_cast<size_t>(v[0]);
    c.intermediate_size = static_cast<size_t>(v[1]);
    c.n_layers = static_cast<size_t>(v[2]);
    c.n_heads = static_cast<size_t>(v[3]);
    c.n_kv_heads = static_cast<size_t>(v[4]);
    c.vocab_size = static_cast<size_t>(v[5]);
    c.max_position_embeddings = static_cast<size_t>(v[6]);
    c.rope_theta = static_cast<float>(v[7]);
    c.norm_eps = static_cast<float>(v[8]);
    double sw = 0;
    c.sliding_window = meta_num(*meta, "sliding_window", sw) ? static_cast<size_t>(sw) : 0;
    if (c.n_heads == 0 || c.hidden_size == 0) return set_error(TL_ERR_FORMAT, "hidden_size/n_heads must be positive");
    c.head_dim = c.hidden_size / c.n_heads;  // parameters.cpp:45
    const JValue* q = meta->get("quant");
    std::snprintf(c.quant, sizeof(c.quant), "%s", (q && q->type == JValue::Str) ? q->s.c_str() : "");

    for (const auto& kv : tens->obj) {
        const JValue& t = kv.second;
        TensorRec r;
        const JValue* dt = t.get("dtype");
        const JValue* sh = t.get("shape");
        const JValue* off = t.get("offset");
        if (!dt || dt->type != JValue::Str || !sh || sh->type != JValue::Arr || !off || !off->is_num())
            return set_error(TL_ERR_FORMAT, "tensor %s: missing dtype/shape/offset", kv.first.c_str());
        r.dtype = dt->s;
        for (const auto& d : sh->arr) {
            if (!d.is_num() || d.i <= 0) return set_error(TL_ERR_FORMAT, "tensor %s: bad shape", kv.first.c_str());
            r.shape.push_back(d.i);
        }
        r.offset = static_cast<uint64_t>(off->i);
        if (r.dtype == "int8") {
            const JValue* so = t.get("scale_offset");
            const JValue* ss = t.get("scale_size");
            if (!so || !so->is_num() || !ss || !ss->is_num())
                return set_error(TL_ERR_FORMAT, "tensor %s: int8 without scales", kv.first.c_str());
            r.scale_offset = static_cast<uint64_t>(so->i);
            r.scale_size = static_cast<uint64_t>(ss->i);
            r.has_scales = true;
        } else if (r.dtype != "f32" && r.dtype != "fp8") {
            return set_error(TL_ERR_FORMAT, "tensor %s: unknown dtype %s", kv.first.c_str(), r.dtype.c_str());
        }
        h.tensors[kv.first] = r;
    }
    h.payload = data + 8 + hsize;
    h.payload_size = size - 8 - hsize;
    return TL_OK;
}

// Bump allocator over one cudaMalloc, 256-byte aligned pieces.
// What a device error code (DeviceErr) means, for the host's message.
const char* device_err_text(unsigned code) {
    switch (code) {
        case kDevErrBarrier: return "decode grid barrier, readiness counter or tensor-parallel exchange";
        case kDevErrRingFull: return "decode weight tile arrival";
        case kDevErrRingEmpty: return "decode ring slot release";
        case kDevErrBatchXchg: return "batched tensor-parallel exchange (a peer's row did not arrive)";
        case kDevErrAttnLoad: return "prefill attention K/V load";
        case kDevErrAttnMma: return "prefill attention MMA issue";
        case kDevErrAttnS: return "prefill attention scores";
        case kDevErrAttnPv: return "prefill attention P V";
        case kDevErrAttnEpi: return "prefill attention epilogue";
        case kGemmErrSlot: return "GEMM stage slot release";
        case kGemmErrStage: return "GEMM stage data arrival";
        case kGemmErrAccReady: return "GEMM accumulator ready";
        case kGemmErrAccFree: return "GEMM accumulator drained";
        default: return "unknown wait";
    }
}

// CUDA events for device timing, destroyed on every return path.
struct Events {
    std::vector<cudaEvent_t> ev;
    tl_status create(size_t n) {
        ev.assign(n, nullptr);
        for (auto& e : ev) {
            const cudaError_t r = cudaEventCreate(&e);
            if (r != cudaSuccess) {
                e = nullptr;
                return set_error(TL_ERR_CUDA, "cudaEventCreate: %s", cudaGetErrorString(r));
            }
        }
        return TL_OK;
    }
    cudaEvent_t operator[](size_t i) const { return ev[i]; }
    ~Events() {
        for (auto e : ev)
            if (e) cudaEventDestroy(e);
    }
};

struct DeviceArena {
    char* base = nullptr;
    size_t cap = 0, used = 0;
    tl_status reserve(size_t bytes) {
        cap = bytes;
        cudaError_t e = cudaMalloc(&base, bytes > 0 ? bytes : 256);
        if (e != cudaSuccess) {
            base = nullptr;
            return set_error(e == cudaErrorMemoryAllocation ? TL_ERR_OUT_OF_MEMORY : TL_ERR_CUDA,
                             "cudaMalloc(%zu) failed: %s", bytes, cudaGetErrorString(e));
        }
        return TL_OK;
    }
    template <typename T>
    T* take(size_t count) {
        const size_t bytes = (count * sizeof(T) + 255) & ~static_cast<size_t>(255);
        if (used + bytes > cap) return nullptr;
        T* p = reinterpret_cast<T*>(base + used);
        used += bytes;
        return p;
    }
    static size_t pad(size_t bytes) { return (bytes + 255) & ~static_cast<size_t>(255); }
    void release() {
        if (base) cudaFree(base);
        base = nullptr;
    }
};

__global__ void k_invert(float* s, size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        s[i] = 1.0f / s[i];
}

struct LayerW {
    int8_t *wqkv = nullptr, *wo = nullptr, *w1 = nullptr, *w3 = nullptr, *w2 = nullptr;  // int8 or e5m2 bytes
    float *sqkv = nullptr, *so = nullptr, *s1 = nullptr, *s3 = nullptr, *s2 = nullptr;  // 1 / s (int8 only)
    float *g_in = nullptr, *g_post = nullptr;
};

struct Step {
    std::string name;
    std::function<double()> bytes;  // algorithmic bytes of this launch
    std::function<tl_status(cudaStream_t, bool)> launch;
};

}  // namespace
}  // namespace tl

using namespace tl;

struct tl_model {
    tl_config cfg = {};
    int device = 0;
    size_t max_seq = 0;
    int splits = 4;
    bool use_graph = true;
    bool pdl = true;
    float temperature = 0.f;   // > 0: decode steps sample (main.cpp:23-43) instead of sample_max
    uint64_t sample_seed = 0;  // uniform draw of position p: sample_uniform(sample_seed, p)
    cudaStream_t stream = nullptr;
    DeviceArena weights, state;
    std::vector<LayerW> layers;
    float *embed = nullptr, *norm = nullptr, *lm_head = nullptr;
    int n_batches = 0;  // live tl_batch objects on this model
    int window = 0;     // > 0: sliding-window attention over the last `window` positions (opt-in)
    bool w_f8 = false;  // projection weights are fp8 (e5m2) bytes without scales, not int8 + scales
    // lm_head stored in the projections' 8-bit format (format extension): lm_q
    // (int8 or e5m2 bytes) and, for int8, lm_s (1 / s) instead of lm_head
    bool lm_8bit = false;
    int8_t* lm_q = nullptr;
    float* lm_s = nullptr;
    float *kc = nullptr, *vc = nullptr, *cos_tab = nullptr, *sin_tab = nullptr;
    float *h = nullptr, *qkv = nullptr, *ctx = nullptr, *act = nullptr, *logits = nullptr;
    float *attn_part = nullptr, *am_v = nullptr;
    unsigned *attn_cnt = nullptr, *am_cnt = nullptr, *d_pos = nullptr;
    unsigned* qkv_cnt = nullptr;  // persistent kernel: q/k/v rows written per kv group
    uint8_t* act_dig = nullptr;   // persistent kernel: act published as staged digits
    int* act_k = nullptr;         // ... the exponent per layer (< -999: none yet)
    unsigned* act_ovf = nullptr;  // ... epoch + 1 of a step in which a value did not fit
    uint32_t *am_i = nullptr, *d_token = nullptr, *d_hist = nullptr, *d_prompt = nullptr;
    uint32_t* h_pinned = nullptr;  // [2]: token in, token out
    size_t pos = 0;
    std::vector<Step> steps;
    std::vector<DecodeLayer> layers_host_tmp;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t graph_exec = nullptr;
    // persistent decode kernel (tl_decode.cu)
    bool persistent = false;
    DeviceArena tiles;
    DecodeLayer* d_layers = nullptr;
    DecodeArgs dargs = {};
    int grid = 0, stages = 0, mega_splits = 0;
    size_t mega_smem = 0;
    unsigned *bar = nullptr, *ticket = nullptr;
    int* err = nullptr;
    int* dbg = nullptr;  // self-check build: {site, v0, v1}
    float2* stats = nullptr;  // persistent kernel: phase hand-over statistics [2][kStatsCap]
    // tensor parallelism: rank `rank` of `tp`; local head / kv head / F / vocab counts
    int tp = 1, rank = 0;
    int64_t lH = 0, lKV = 0, lF = 0, lV = 0;
    unsigned* epoch = nullptr;    // steps run (tp exchange counters)
    uint8_t* xbuf = nullptr;      // this rank's exchange buffer (tp), cudaMalloc'd for IPC
    uint8_t* xpeer_open[kMaxTp] = {};  // peer buffers opened with cudaIpcOpenMemHandle
    bool connected = false;
    bool broken = false;  // tp: a device-side wait gave up; the ranks' exchange state is lost
    // batched prompt pass (tl_model_prefill): fp16 weights dequantised on first
    // use (per layer q|k|v, o, gate|up in SwiGLU blocks, down) and row buffers
    DeviceArena scT, w16, rows;
    // per layer: q|k|v, o, gate|up, down as the dequantising GEMM reads them
    // (the int8 / e5m2 weights in place, their 1/s transposed into scT) ...
    std::vector<std::array<Q8Weights, 4>> lq8;
    // ... or, with tl_model_options.weights_f16, fp16 copies (gate|up in
    // blocks of 128 gate then 128 up rows) for the fp16 GEMM
    bool weights_f16 = false;
    std::vector<std::array<__half*, 4>> lw16;
    size_t rows_cap = 0;
    float *p_h = nullptr, *p_qkv = nullptr;
    __half *p_x16 = nullptr, *p_q16 = nullptr, *p_ctx16 = nullptr, *p_act16 = nullptr;
    __half *p_k16 = nullptr, *p_v16 = nullptr;  // fp16 copies of one layer's cache rows
    uint32_t* p_tok = nullptr;
    __half* lm16 = nullptr;  // fp16 lm_head for the batched logits GEMM (first batch use)
    DeviceArena lm16_arena;
    double bytes_per_step = 0;
};

namespace tl {
namespace {

size_t layer_kv_floats(const tl_model* m) { return m->lKV * m->max_seq * m->cfg.head_dim; }

tl_status check_shapes(const Header& h) {
    const tl_config& c = h.cfg;
    if (std::string(c.quant) != "int8" && std::string(c.quant) != "fp8")
        return set_error(TL_ERR_UNSUPPORTED,
                         "quant \"%s\": only int8 models (export_mistral.py --quant int8) and fp8 (e5m2) models "
                         "are built",
                         c.quant);
    if (c.n_heads != 4 * c.n_kv_heads)
        return set_error(TL_ERR_UNSUPPORTED,
                         "n_heads (%zu) != 4 * n_kv_heads (%zu): the reference hard-codes kv head = h/4",
                         c.n_heads, c.n_kv_heads);
    if (c.head_dim * c.n_heads != c.hidden_size)
        return set_error(TL_ERR_UNSUPPORTED, "hidden_size not divisible by n_heads");
    if (!(c.head_dim == 32 || c.head_dim == 64 || c.head_dim == 128 || c.head_dim == 256))
        return set_error(TL_ERR_UNSUPPORTED, "head_dim %zu not in {32, 64, 128, 256}", c.head_dim);
    if (c.hidden_size % 512 || c.intermediate_size % 512 || c.hidden_size > 16384 || c.intermediate_size > 16384)
        return set_error(TL_ERR_UNSUPPORTED,
                         "hidden_size (%zu) and intermediate_size (%zu) must be multiples of 512, <= 16384",
                         c.hidden_size, c.intermediate_size);
    if (c.n_layers == 0 || c.vocab_size == 0) return set_error(TL_ERR_FORMAT, "empty model");
    return TL_OK;
}

tl_status find(const Header& h, const std::string& name, const char* dtype, std::vector<int64_t> shape,
               const TensorRec*& out) {
    auto it = h.tensors.find(name);
    if (it == h.tensors.end()) return set_error(TL_ERR_FORMAT, "tensor %s not found", name.c_str());
    const TensorRec& r = it->second;
    if (r.dtype != dtype)
        return set_error(TL_ERR_FORMAT, "tensor %s has dtype %s, expected %s", name.c_str(), r.dtype.c_str(), dtype);
    if (r.shape != shape) return set_error(TL_ERR_FORMAT, "tensor %s has an unexpected shape", name.c_str());
    const uint64_t bytes = r.numel() * (r.dtype == "f32" ? 4 : 1);
    if (r.offset > h.payload_size || bytes > h.payload_size - r.offset)
        return set_error(TL_ERR_FORMAT, "tensor %s extends past the end of the file", name.c_str());
    if (r.has_scales) {
        if (r.scale_size * 64 != r.numel())
            return set_error(TL_ERR_UNSUPPORTED, "tensor %s: %llu scales for %llu weights (group 64 expected)",
                             name.c_str(), static_cast<unsigned long long>(r.scale_size),
                             static_cast<unsigned long long>(r.numel()));
        if (r.scale_offset > h.payload_size || r.scale_size * 4 > h.payload_size - r.scale_offset)
            return set_error(TL_ERR_FORMAT, "scales of %s extend past the end of the file", name.c_str());
    }
    out = &r;
    return TL_OK;
}

tl_status upload(void* dst, const Header& h, uint64_t offset, size_t bytes) {
    TL_CUDA_TRY(cudaMemcpy(dst, h.payload + offset, bytes, cudaMemcpyHostToDevice));
    return TL_OK;
}

// A cudaMemcpy from pageable host memory may return before its DMA has
// landed, and the model's kernels run on a non-blocking stream that is not
// ordered after it: wait for every upload before a kernel reads uploaded bytes.
tl_status uploads_landed() {
    TL_CUDA_TRY(cudaDeviceSynchronize());
    return TL_OK;
}

// Columns [col0, col0 + width) (in bytes) of every row of a row-major tensor.
tl_status upload_cols(void* dst, const Header& h, uint64_t offset, size_t rows, size_t row_bytes, size_t col0,
                      size_t width) {
    TL_CUDA_TRY(cudaMemcpy2D(dst, width, h.payload + offset + col0, row_bytes, width, rows, cudaMemcpyHostToDevice));
    return TL_OK;
}

tl_status build_steps(tl_model* m);
tl_status capture_graph(tl_model* m);

tl_status create_model(const uint8_t* data, size_t size, const tl_model_options* opts, tl_model** out) {
    Header h;
    TL_TRY(parse_header(data, size, h));
    TL_TRY(check_shapes(h));
    const tl_config& c = h.cfg;
    const int64_t D = c.hidden_size, F = c.intermediate_size, H = c.n_heads, KV = c.n_kv_heads,
                  HD = c.head_dim, V = c.vocab_size, L = c.n_layers;
    const int64_t NQKV = (H + 2 * KV) * HD;

    // Resolve and validate every tensor before touching the device.
    struct LayerRecs { const TensorRec *q, *k, *v, *o, *g, *u, *d, *ni, *np; };
    std::vector<LayerRecs> recs(L);
    const TensorRec *emb, *nrm, *lmh;
    TL_TRY(find(h, "model.embed_tokens.weight", "f32", {V, D}, emb));
    TL_TRY(find(h, "model.norm.weight", "f32", {D}, nrm));
    // Projection weights: int8 + per-64-group scales (export_mistral.py --quant
    // int8), or fp8 e5m2 bytes without scales (the format extension "fp8").
    const char* wdt = c.quant;
    const bool f8 = std::string(wdt) == "fp8";
    // lm_head: fp32 as export_mistral.py writes it (:119), or in the _proj
    // tensors' format (format extension; the header's dtype says which)
    const auto lm_it = h.tensors.find("lm_head.weight");
    const bool lm8 = lm_it != h.tensors.end() && lm_it->second.dtype == wdt;
    TL_TRY(find(h, "lm_head.weight", lm8 ? wdt : "f32", {V, D}, lmh));
    if (lm8 && !f8 && (!lmh->has_scales || D % 64))
        return set_error(TL_ERR_FORMAT, "int8 lm_head needs per-64-group scales");
    for (int64_t l = 0; l < L; l++) {
        const std::string p = "model.layers." + std::to_string(l) + ".";
        LayerRecs& r = recs[l];
        TL_TRY(find(h, p + "self_attn.q_proj.weight", wdt, {H * HD, D}, r.q));
        TL_TRY(find(h, p + "self_attn.k_proj.weight", wdt, {KV * HD, D}, r.k));
        TL_TRY(find(h, p + "self_attn.v_proj.weight", wdt, {KV * HD, D}, r.v));
        TL_TRY(find(h, p + "self_attn.o_proj.weight", wdt, {D, H * HD}, r.o));
        TL_TRY(find(h, p + "mlp.gate_proj.weight", wdt, {F, D}, r.g));
        TL_TRY(find(h, p + "mlp.up_proj.weight", wdt, {F, D}, r.u));
        TL_TRY(find(h, p + "mlp.down_proj.weight", wdt, {D, F}, r.d));
        TL_TRY(find(h, p + "input_layernorm.weight", "f32", {D}, r.ni));
        TL_TRY(find(h, p + "post_attention_layernorm.weight", "f32", {D}, r.np));
    }

    std::unique_ptr<tl_model> m(new tl_model());
    m->cfg = c;
    m->device = opts ? opts->device : 0;
    m->max_seq = (opts && opts->max_seq) ? opts->max_seq : 1024;
    // sliding window (opt-in; the reference attends to every position): 0 off,
    // < 0 the binary's sliding_window (parameters.cpp:41), > 0 that many positions
    if (opts && opts->sliding_window != 0) {
        const long long w = opts->sliding_window < 0 ? static_cast<long long>(c.sliding_window)
                                                     : static_cast<long long>(opts->sliding_window);
        TL_REQUIRE(w > 0 && w < (1ll << 30), "sliding_window: %lld positions (the binary says %zu)", w,
                   c.sliding_window);
        m->window = static_cast<int>(w);
    }
    m->use_graph = opts ? opts->use_graph != 0 : true;
    m->weights_f16 = opts && opts->weights_f16 != 0;
    // Tensor parallelism (Megatron split of modules.cpp's layers): this rank
    // keeps q heads / kv heads / F rows / vocab rows [rank n / tp, (rank + 1) n / tp).
    const int tp = (opts && opts->tp_size > 0) ? opts->tp_size : 1;
    const int rank = opts ? opts->tp_rank : 0;
    if (tp > 1) {
        if (!(tp == 2 || tp == 4 || tp == 8) || rank < 0 || rank >= tp)
            return set_error(TL_ERR_INVALID_ARGUMENT, "tp_size %d / tp_rank %d: tp_size must be 2, 4 or 8", tp, rank);
        if (KV % tp || V % tp || F % tp || (F / tp) % 64)
            return set_error(TL_ERR_UNSUPPORTED,
                             "tp_size %d must divide n_kv_heads (%lld) and vocab_size (%lld), and "
                             "intermediate_size (%lld) into multiples of 64",
                             tp, static_cast<long long>(KV), static_cast<long long>(V), static_cast<long long>(F));
        if (opts->kernel_mode != 0)
            return set_error(TL_ERR_UNSUPPORTED, "tensor parallelism runs the persistent decode kernel (kernel_mode 0)");
    }
    m->tp = tp;
    m->rank = rank;
    const int64_t Hl = H / tp, KVl = KV / tp, Fl = F / tp, Vl = V / tp;
    const int64_t NQKVl = (Hl + 2 * KVl) * HD;
    m->lH = Hl;
    m->lKV = KVl;
    m->lF = Fl;
    m->lV = Vl;
    if (const char* e = std::getenv("TL_NO_PDL")) m->pdl = (e[0] == '0');
    if (m->max_seq > (1u << 24))
        return set_error(TL_ERR_INVALID_ARGUMENT, "max_seq %zu too large (positions are exact in fp32 up to 2^24)",
                         m->max_seq);
    TL_CUDA_TRY(cudaSetDevice(m->device));
    TL_CUDA_TRY(cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking));
    m->splits = static_cast<int>(std::min<size_t>(32, std::max<size_t>(4, m->max_seq / 256)));

    // ---- weights arena (this rank's slices) ----
    using A = DeviceArena;
    // fp32 scales (int8 only): one per 64 weights
    auto sc_bytes = [&](int64_t numel) { return f8 ? size_t(0) : A::pad(numel / 64 * 4); };
    size_t wbytes = A::pad(V * D * 4) + (lm8 ? A::pad(Vl * D) + sc_bytes(Vl * D) : A::pad(Vl * D * 4)) +
                    A::pad(D * 4);
    const size_t per_layer = A::pad(NQKVl * D) + A::pad(D * Hl * HD) + 2 * A::pad(Fl * D) + A::pad(D * Fl) +
                             sc_bytes(NQKVl * D) + sc_bytes(D * Hl * HD) + 2 * sc_bytes(Fl * D) + sc_bytes(D * Fl) +
                             2 * A::pad(D * 4);
    wbytes += per_layer * L;
    TL_TRY(m->weights.reserve(wbytes));
    m->embed = m->weights.take<float>(V * D);
    m->w_f8 = f8;
    m->lm_8bit = lm8;
    if (lm8) {
        m->lm_q = m->weights.take<int8_t>(Vl * D);
        if (!f8) m->lm_s = m->weights.take<float>(Vl * D / 64);
    } else {
        m->lm_head = m->weights.take<float>(Vl * D);
    }
    m->norm = m->weights.take<float>(D);
    TL_TRY(upload(m->embed, h, emb->offset, V * D * 4));
    if (lm8) {  // this rank's vocabulary rows and (int8) their scales; stored s = 127/absmax becomes 1/s
        TL_TRY(upload(m->lm_q, h, lmh->offset + static_cast<uint64_t>(rank) * Vl * D, Vl * D));
        if (!f8) {
            TL_TRY(upload(m->lm_s, h, lmh->scale_offset + static_cast<uint64_t>(rank) * Vl * (D / 64) * 4,
                          Vl * (D / 64) * 4));
            TL_TRY(uploads_landed());
            k_invert<<<256, 256, 0, m->stream>>>(m->lm_s, static_cast<size_t>(Vl * D / 64));
            TL_TRY(check_launch("invert lm_head scales"));
        }
    } else {
        TL_TRY(upload(m->lm_head, h, lmh->offset + static_cast<uint64_t>(rank) * Vl * D * 4, Vl * D * 4));
    }
    TL_TRY(upload(m->norm, h, nrm->offset, D * 4));
    m->layers.resize(L);
    const int64_t G = D / 64;  // scale groups per row of a [*, D] tensor
    for (int64_t l = 0; l < L; l++) {
        LayerW& w = m->layers[l];
        const LayerRecs& r = recs[l];
        w.wqkv = m->weights.take<int8_t>(NQKVl * D);
        w.wo = m->weights.take<int8_t>(D * Hl * HD);
        w.w1 = m->weights.take<int8_t>(Fl * D);
        w.w3 = m->weights.take<int8_t>(Fl * D);
        w.w2 = m->weights.take<int8_t>(D * Fl);
        if (!f8) {  // fp8 weights have no scales (the pointers stay null)
            w.sqkv = m->weights.take<float>(NQKVl * D / 64);
            w.so = m->weights.take<float>(D * Hl * HD / 64);
            w.s1 = m->weights.take<float>(Fl * D / 64);
            w.s3 = m->weights.take<float>(Fl * D / 64);
            w.s2 = m->weights.take<float>(D * Fl / 64);
        }
        w.g_in = m->weights.take<float>(D);
        w.g_post = m->weights.take<float>(D);
        if (!w.g_post) return set_error(TL_ERR_OUT_OF_MEMORY, "weights arena too small (internal)");
        // q rows of this rank's heads, then its k and v rows: one GEMV produces [q | k | v].
        const int64_t q0 = rank * Hl * HD, k0 = rank * KVl * HD;
        TL_TRY(upload(w.wqkv, h, r.q->offset + q0 * D, Hl * HD * D));
        TL_TRY(upload(w.wqkv + Hl * HD * D, h, r.k->offset + k0 * D, KVl * HD * D));
        TL_TRY(upload(w.wqkv + (Hl + KVl) * HD * D, h, r.v->offset + k0 * D, KVl * HD * D));
        // o_proj: this rank's head columns of [D, H hd] (row-parallel)
        TL_TRY(upload_cols(w.wo, h, r.o->offset, D, H * HD, q0, Hl * HD));
        // gate/up: this rank's F rows; down_proj: its F columns (row-parallel)
        TL_TRY(upload(w.w1, h, r.g->offset + rank * Fl * D, Fl * D));
        TL_TRY(upload(w.w3, h, r.u->offset + rank * Fl * D, Fl * D));
        TL_TRY(upload_cols(w.w2, h, r.d->offset, D, F, rank * Fl, Fl));
        TL_TRY(upload(w.g_in, h, r.ni->offset, D * 4));
        TL_TRY(upload(w.g_post, h, r.np->offset, D * 4));
        if (!f8) {  // the int8 tensors' scales, sliced like their weights
            TL_TRY(upload(w.sqkv, h, r.q->scale_offset + q0 * G * 4, Hl * HD * G * 4));
            TL_TRY(upload(w.sqkv + Hl * HD * G, h, r.k->scale_offset + k0 * G * 4, KVl * HD * G * 4));
            TL_TRY(upload(w.sqkv + (Hl + KVl) * HD * G, h, r.v->scale_offset + k0 * G * 4, KVl * HD * G * 4));
            TL_TRY(upload_cols(w.so, h, r.o->scale_offset, D, H * HD / 64 * 4, q0 / 64 * 4, Hl * HD / 64 * 4));
            TL_TRY(upload(w.s1, h, r.g->scale_offset + rank * Fl * G * 4, Fl * G * 4));
            TL_TRY(upload(w.s3, h, r.u->scale_offset + rank * Fl * G * 4, Fl * G * 4));
            TL_TRY(upload_cols(w.s2, h, r.d->scale_offset, D, F / 64 * 4, rank * Fl / 64 * 4, Fl / 64 * 4));
            // Stored scales s = 127/absmax become 1/s: the GEMV multiplies.
            const size_t ns[5] = {static_cast<size_t>(NQKVl * D / 64), static_cast<size_t>(D * Hl * HD / 64),
                                  static_cast<size_t>(Fl * D / 64), static_cast<size_t>(Fl * D / 64),
                                  static_cast<size_t>(D * Fl / 64)};
            float* sp[5] = {w.sqkv, w.so, w.s1, w.s3, w.s2};
            TL_TRY(uploads_landed());
            for (int k = 0; k < 5; k++) k_invert<<<256, 256, 0, m->stream>>>(sp[k], ns[k]);
            TL_TRY(check_launch("invert scales"));
        }
    }

    TL_TRY(uploads_landed());  // the repack and dequant kernels read the uploaded weights

    // ---- persistent decode kernel: tiled weight copies ----
    const int kmode = opts ? opts->kernel_mode : 0;
    if (kmode == 0) {
        int max_smem = 0, dev_sms = 0, coop = 0;
        TL_CUDA_TRY(cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, m->device));
        TL_CUDA_TRY(cudaDeviceGetAttribute(&dev_sms, cudaDevAttrMultiProcessorCount, m->device));
        TL_CUDA_TRY(cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, m->device));
        int pbuf = 0;
        if (coop && decode_kernel_fits(static_cast<int>(D), static_cast<int>(Fl), static_cast<int>(Hl),
                                       static_cast<int>(KVl), static_cast<int>(HD), static_cast<int>(Vl),
                                       static_cast<int>(L), f8, dev_sms, max_smem, &m->stages, &m->mega_smem,
                                       &pbuf)) {
            m->persistent = true;
            m->grid = dev_sms;
            // Tuning knob: a shallower weight ring (fewer bytes in flight per SM).
            if (const char* e = std::getenv("TL_DECODE_STAGES")) {
                const int want = std::atoi(e);
                if (want >= 4 && want % 4 == 0 && want < m->stages) {  // slots keep their owner warps (x4)
                    m->mega_smem -= static_cast<size_t>(m->stages - want) * (2 * (f8 ? kTileBytesF8 : kTileBytesI8) + 16);
                    m->stages = want;
                }
            }
            m->mega_splits = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(dev_sms / Hl, 256 / Hl)));
            // GQA attention: one CTA per (kv group, split), up to one split per 64 positions
            if (HD == 128 && Hl == 4 * KVl) {
                m->dargs.gqa_splits = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(32, dev_sms / KVl)));
                m->dargs.gqa_from = kGqaFromDefault;
                m->dargs.gqa_rows = kGqaRowsDefault;
                // Tuning knobs: the position count from which GQA attention replaces per-head
                // attention, and the positions per split.
                if (const char* e = std::getenv("TL_DECODE_GQA_FROM")) m->dargs.gqa_from = std::atoi(e);
                if (const char* e = std::getenv("TL_DECODE_GQA_ROWS"))
                    m->dargs.gqa_rows = std::max(8, std::min(4096, std::atoi(e)));
            }
            m->dargs.kv_prefetch_rows = kKvPrefetchRowsDefault;
            // Tuning knob: cached K / V rows per attention CTA hinted into L2 ahead of attention.
            if (const char* e = std::getenv("TL_DECODE_KV_PREFETCH"))
                m->dargs.kv_prefetch_rows = std::max(0, std::min(1 << 20, std::atoi(e)));
            m->dargs.pbuf_floats = pbuf;
        }
    }
    if (tp > 1 && !m->persistent)
        return set_error(TL_ERR_UNSUPPORTED, "tensor parallelism needs the persistent decode kernel (shape or device)");
    if (m->persistent) {
        const size_t per = tiles_q_bytes(NQKVl, D, f8) + tiles_q_bytes(D, Hl * HD, f8) +
                           tiles_q_bytes(2 * Fl, D, f8) + tiles_q_bytes(D, Fl, f8);
        const size_t lm_tiles = lm8 ? tiles_q_bytes(Vl, D, f8) : tiles_f32_bytes(Vl, D);
        TL_TRY(m->tiles.reserve(per * L + lm_tiles + 256 * (4 * L + 1)));
        std::vector<DecodeLayer> dl(L);
        for (int64_t l = 0; l < L; l++) {
            const LayerW& w = m->layers[l];
            uint8_t* tq = m->tiles.take<uint8_t>(tiles_q_bytes(NQKVl, D, f8));
            uint8_t* to = m->tiles.take<uint8_t>(tiles_q_bytes(D, Hl * HD, f8));
            uint8_t* t13 = m->tiles.take<uint8_t>(tiles_q_bytes(2 * Fl, D, f8));
            uint8_t* t2 = m->tiles.take<uint8_t>(tiles_q_bytes(D, Fl, f8));
            TL_TRY(repack_i8(tq, w.wqkv, w.sqkv, NQKVl, D, m->stream));
            TL_TRY(repack_i8(to, w.wo, w.so, D, Hl * HD, m->stream));
            TL_TRY(repack_i8_swiglu(t13, w.w1, w.s1, w.w3, w.s3, Fl, D, m->stream));
            TL_TRY(repack_i8(t2, w.w2, w.s2, D, Fl, m->stream));
            dl[l] = DecodeLayer{tq, to, t13, t2, w.g_in, w.g_post, nullptr, nullptr};
        }
        uint8_t* tl = m->tiles.take<uint8_t>(lm_tiles);
        if (lm8) TL_TRY(repack_i8(tl, m->lm_q, m->lm_s, Vl, D, m->stream));
        else TL_TRY(repack_f32(tl, m->lm_head, Vl, D, m->stream));
        m->dargs.lm_head = tl;
        m->dargs.lm_8bit = lm8 ? 1 : 0;
        m->dargs.w_f8 = f8 ? 1 : 0;
        TL_CUDA_TRY(cudaMalloc(&m->d_layers, sizeof(DecodeLayer) * L));
        // KV pointers are filled once the state arena exists (below).
        m->dargs.layers = m->d_layers;
        m->layers_host_tmp = dl;
    }

    // ---- state arena: KV cache, RoPE tables, activations, scratch ----
    const size_t kv = L * layer_kv_floats(m.get());
    const size_t half = HD / 2;
    const int am_grid = std::max(gemv_f32_grid(V, D, true, true), m->grid);
    const int part_splits = std::max({m->splits, m->mega_splits, m->dargs.gqa_splits});
    size_t sbytes = 2 * A::pad(kv * 4) + 2 * A::pad(m->max_seq * half * 4) + A::pad(D * 4) + A::pad(NQKVl * 4) +
                    A::pad(Hl * HD * 4) + A::pad(Fl * 4) + A::pad(Vl * 4) + A::pad(Hl * part_splits * (HD + 4) * 4) +
                    A::pad(Hl * 4) * 2 + A::pad(am_grid * 4) * 2 + A::pad(4) * 6 + A::pad(16) + A::pad(m->max_seq * 4) * 2 +
                    A::pad(2 * kStatsCap * sizeof(float2)) + A::pad(D * 4) + A::pad(4) +
                    A::pad(3 * static_cast<size_t>(tile_slices(static_cast<int>(Fl)) * kTileCols)) + 2 * A::pad(L * 4);
    TL_TRY(m->state.reserve(sbytes));
    TL_CUDA_TRY(cudaMemsetAsync(m->state.base, 0, sbytes, m->stream));
    // The stream is non-blocking: the clear must land before the blocking
    // copies below (RoPE tables, layer table) write into the arena.
    TL_CUDA_TRY(cudaStreamSynchronize(m->stream));
    m->kc = m->state.take<float>(kv);
    m->vc = m->state.take<float>(kv);
    m->cos_tab = m->state.take<float>(m->max_seq * half);
    m->sin_tab = m->state.take<float>(m->max_seq * half);
    m->h = m->state.take<float>(D);
    m->qkv = m->state.take<float>(NQKVl);
    m->ctx = m->state.take<float>(Hl * HD);
    m->act = m->state.take<float>(Fl);
    m->logits = m->state.take<float>(Vl);
    m->attn_part = m->state.take<float>(Hl * part_splits * (HD + 4));
    m->attn_cnt = m->state.take<unsigned>(Hl);
    m->qkv_cnt = m->state.take<unsigned>(Hl);
    m->am_v = m->state.take<float>(am_grid);
    m->am_i = m->state.take<uint32_t>(am_grid);
    m->am_cnt = m->state.take<unsigned>(1);
    m->d_pos = m->state.take<unsigned>(1);
    m->d_token = m->state.take<uint32_t>(1);
    m->d_hist = m->state.take<uint32_t>(m->max_seq);
    m->d_prompt = m->state.take<uint32_t>(m->max_seq);
    m->bar = m->state.take<unsigned>(1);
    m->ticket = m->state.take<unsigned>(1);
    m->err = m->state.take<int>(1);
    m->dbg = m->state.take<int>(4);
    m->stats = m->state.take<float2>(2 * kStatsCap);
    m->epoch = m->state.take<unsigned>(1);
    m->act_dig = m->state.take<uint8_t>(3 * static_cast<size_t>(tile_slices(static_cast<int>(Fl)) * kTileCols));
    m->act_k = m->state.take<int>(L);
    m->act_ovf = m->state.take<unsigned>(L);
    if (!m->act_ovf) return set_error(TL_ERR_OUT_OF_MEMORY, "state arena too small (internal)");
    if (m->persistent) {
        for (int64_t l = 0; l < L; l++) {
            m->layers_host_tmp[l].k_cache = m->kc + static_cast<size_t>(l) * layer_kv_floats(m.get());
            m->layers_host_tmp[l].v_cache = m->vc + static_cast<size_t>(l) * layer_kv_floats(m.get());
        }
        TL_CUDA_TRY(cudaMemcpy(m->d_layers, m->layers_host_tmp.data(), sizeof(DecodeLayer) * L,
                               cudaMemcpyHostToDevice));
        DecodeArgs& d = m->dargs;
        d.n_layers = static_cast<int>(L);
        d.embed = m->embed; d.g_final = m->norm; d.cos_tab = m->cos_tab; d.sin_tab = m->sin_tab;
        d.h = m->h; d.qkv = m->qkv; d.attn_part = m->attn_part; d.act = m->act; d.logits = m->logits;
        d.ctx = m->ctx; d.attn_cnt = m->attn_cnt; d.qkv_cnt = m->qkv_cnt; d.stats = m->stats;
        if (tp == 1 && !f8) {  // act digits published by the gate/up epilogue
            std::vector<int> none(static_cast<size_t>(L), -1000);
            TL_CUDA_TRY(cudaMemcpy(m->act_k, none.data(), sizeof(int) * none.size(), cudaMemcpyHostToDevice));
            d.act_dig = m->act_dig; d.act_k = m->act_k; d.act_ovf = m->act_ovf;
        }
        // Tuning knob: tile pairs prefetched into L2 ahead of the ring.
        d.prefetch = 6;
        if (const char* e = std::getenv("TL_DECODE_PREFETCH")) d.prefetch = std::max(0, std::min(64, std::atoi(e)));
#ifdef TL_DECODE_CHECK
        d.dbg = m->dbg;
#endif
        d.am_v = m->am_v; d.am_i = m->am_i; d.ticket = m->ticket; d.bar = m->bar; d.err = m->err;
        d.token = m->d_token; d.pos = m->d_pos; d.history = m->d_hist;
        d.D = static_cast<int>(D); d.F = static_cast<int>(Fl); d.H = static_cast<int>(Hl);
        d.KV = static_cast<int>(KVl); d.HD = static_cast<int>(HD); d.V = static_cast<int>(Vl);
        d.tp_size = tp; d.tp_rank = rank; d.vocab_off = static_cast<int>(rank * Vl);
        d.epoch = m->epoch;
        // Bound of the kernel's waits on other CTAs and ranks (a peer that never
        // arrives ends the step with TL_ERR_TIMEOUT); TL_WAIT_TIMEOUT_MS shortens it.
        d.timeout_ns = 2000000000ull;
        if (const char* e = std::getenv("TL_WAIT_TIMEOUT_MS"))
            d.timeout_ns = static_cast<unsigned long long>(std::max(10, std::min(60000, std::atoi(e)))) * 1000000ull;
        if (tp > 1) {  // this rank's exchange buffer; peers are mapped by tl_model_tp_connect
            const size_t xb = xchg_bytes(tp, static_cast<int>(D));
            TL_CUDA_TRY(cudaMalloc(&m->xbuf, xb));
            TL_CUDA_TRY(cudaMemset(m->xbuf, 0, xb));
            d.xpeer[rank] = m->xbuf;
        }
        d.max_seq = static_cast<int>(m->max_seq); d.splits = m->mega_splits; d.window = m->window;
        // Tuning knob: positions per per-head attention split (more splits = more CTAs at short context).
        d.split_rows = kSplitRowsDefault;
        if (const char* e = std::getenv("TL_DECODE_SPLIT_ROWS")) d.split_rows = std::max(8, std::min(4096, std::atoi(e)));
        d.attn_scale = static_cast<float>(1.0 / std::sqrt(static_cast<double>(HD)));
    }

    // RotaryEmbedding::init_freq + ::forward (modules.cpp:12-27) with the
    // reference's float arithmetic and libm, for every position up front.
    {
        std::vector<float> inv(half), ct(m->max_seq * half), st(m->max_seq * half);
        for (size_t i = 0; i < half; i++)
            inv[i] = 1.0f / powf(c.rope_theta, static_cast<float>(i) / static_cast<float>(half));
        for (size_t p = 0; p < m->max_seq; p++)
            for (size_t i = 0; i < half; i++) {
                const float a = inv[i] * static_cast<float>(p);
                ct[p * half + i] = cosf(a);
                st[p * half + i] = sinf(a);
            }
        TL_CUDA_TRY(cudaMemcpy(m->cos_tab, ct.data(), ct.size() * 4, cudaMemcpyHostToDevice));
        TL_CUDA_TRY(cudaMemcpy(m->sin_tab, st.data(), st.size() * 4, cudaMemcpyHostToDevice));
    }
    TL_CUDA_TRY(cudaMallocHost(&m->h_pinned, 4 * sizeof(uint32_t)));
    TL_CUDA_TRY(cudaStreamSynchronize(m->stream));
    TL_TRY(uploads_landed());  // the layer table and RoPE tables, before any step reads them

    TL_TRY(build_steps(m.get()));
    if (m->use_graph) TL_TRY(capture_graph(m.get()));
    *out = m.release();
    return TL_OK;
}

// ---------------------------------------------------------------------------
// The launch sequence of one decode step.
// ---------------------------------------------------------------------------

void add_layer_steps(tl_model* m, int l, std::vector<Step>& steps) {
    const tl_config& c = m->cfg;
    const int D = c.hidden_size, F = c.intermediate_size, H = c.n_heads, KV = c.n_kv_heads, HD = c.head_dim;
    const int NQKV = (H + 2 * KV) * HD;
    const LayerW* w = &m->layers[l];
    const float eps = 1e-5f;  // RMSNorm::e, hard-coded in modules.h:24
    const double qb = m->w_f8 ? 1.0 : 1 + 4.0 / 64;  // bytes per weight, scales included
    const int f8 = m->w_f8 ? 1 : 0;

    steps.push_back({"gemv_qkv_rmsnorm",
                     [=] { return double(NQKV) * D * qb + 8.0 * D + 4.0 * NQKV; },
                     [=](cudaStream_t s, bool pdl) {
                         GemvI8Args a = {};
                         a.w = w->wqkv; a.s = w->sqkv; a.f8 = f8; a.x = m->h; a.g = w->g_in; a.eps = eps;
                         a.y = m->qkv; a.n = NQKV; a.d = D;
                         return launch_gemv_i8(a, I8Mode::Store, true, true, s, pdl);
                     }});
    steps.push_back({"attention_decode",
                     [=] {
                         const double npos = double(m->pos) + 1;
                         return 2.0 * KV * npos * HD * 4 + 4.0 * NQKV + 4.0 * H * HD;
                     },
                     [=](cudaStream_t s, bool pdl) {
                         AttnArgs a = {};
                         a.qkv = m->qkv;
                         a.k_cache = m->kc + static_cast<size_t>(l) * layer_kv_floats(m);
                         a.v_cache = m->vc + static_cast<size_t>(l) * layer_kv_floats(m);
                         a.cos_tab = m->cos_tab; a.sin_tab = m->sin_tab; a.pos = m->d_pos;
                         a.ctx = m->ctx; a.part = m->attn_part; a.counters = m->attn_cnt;
                         a.n_heads = H; a.n_kv_heads = KV; a.head_dim = HD;
                         a.max_seq = static_cast<int>(m->max_seq); a.splits = m->splits;
                         a.scale = static_cast<float>(1.0 / std::sqrt(static_cast<double>(HD)));
                         a.window = m->window;
                         return launch_attention(a, s, pdl);
                     }});
    steps.push_back({"gemv_o_residual",
                     [=] { return double(D) * H * HD * qb + 4.0 * H * HD + 8.0 * D; },
                     [=](cudaStream_t s, bool pdl) {
                         GemvI8Args a = {};
                         a.w = w->wo; a.s = w->so; a.f8 = f8; a.x = m->ctx; a.y = m->h; a.res = m->h;
                         a.n = D; a.d = H * HD;
                         return launch_gemv_i8(a, I8Mode::AddResidual, true, false, s, pdl);
                     }});
    steps.push_back({"gemv_gate_up_silu",
                     [=] { return 2.0 * F * D * qb + 8.0 * D + 4.0 * F; },
                     [=](cudaStream_t s, bool pdl) {
                         GemvI8Args a = {};
                         a.w = w->w1; a.s = w->s1; a.w2 = w->w3; a.s2 = w->s3; a.f8 = f8; a.x = m->h;
                         a.g = w->g_post;
                         a.eps = eps; a.y = m->act; a.n = F; a.d = D;
                         return launch_gemv_i8(a, I8Mode::SwiGLU, true, true, s, pdl);
                     }});
    steps.push_back({"gemv_down_residual",
                     [=] { return double(D) * F * qb + 4.0 * F + 8.0 * D; },
                     [=](cudaStream_t s, bool pdl) {
                         GemvI8Args a = {};
                         a.w = w->w2; a.s = w->s2; a.f8 = f8; a.x = m->act; a.y = m->h; a.res = m->h;
                         a.n = D; a.d = F;
                         return launch_gemv_i8(a, I8Mode::AddResidual, true, false, s, pdl);
                     }});
}

tl_status build_steps(tl_model* m) {
    const tl_config& c = m->cfg;
    const int D = c.hidden_size, V = c.vocab_size;
    m->steps.clear();
    if (m->persistent) {
        // this rank's bytes (all of them when tp = 1)
        const double F = m->lF, H = m->lH, KV = m->lKV, HD = c.head_dim, L = c.n_layers;
        const double NQKV = (H + 2 * KV) * HD;
        const double Vr = double(m->lV);
        // 8-bit weights (+ fp32 scales for int8) of every projection, the lm_head, norms,
        // one embedding row
        const double qb = m->w_f8 ? 1.0 : 1 + 4.0 / 64;
        const double per_layer = (NQKV * D + D * H * HD + 3.0 * F * D) * qb + 8.0 * D;
        const double fixed = per_layer * L + Vr * D * (m->lm_8bit ? qb : 4.0) + 8.0 * D;
        m->steps.push_back({"decode_step",
                            [=] { return fixed + 2.0 * L * KV * (double(m->pos) + 1) * HD * 4; },
                            [=](cudaStream_t s, bool) {
                                return launch_decode_step(m->dargs, m->grid, m->stages, m->mega_smem, s);
                            }});
        return TL_OK;
    }
    m->steps.push_back({"embed", [=] { return 8.0 * D; },
                        [=](cudaStream_t s, bool pdl) {
                            return launch_embed(m->h, m->embed, m->d_token, D, s, pdl);
                        }});
    for (int l = 0; l < static_cast<int>(c.n_layers); l++) add_layer_steps(m, l, m->steps);
    if (m->lm_8bit) {  // 8-bit lm_head: the projection GEMV with the final norm fused, then the argmax
        const double qb = m->w_f8 ? 1.0 : 1 + 4.0 / 64;
        m->steps.push_back({"gemv_lm_head_i8", [=] { return double(V) * D * qb + 8.0 * D + 4.0 * V; },
                            [=](cudaStream_t s, bool pdl) {
                                GemvI8Args a = {};
                                a.w = m->lm_q; a.s = m->lm_s; a.f8 = m->w_f8 ? 1 : 0; a.x = m->h; a.g = m->norm;
                                a.eps = 1e-5f;
                                a.y = m->logits; a.n = V; a.d = D;
                                return launch_gemv_i8(a, I8Mode::Store, true, true, s, pdl);
                            }});
        m->steps.push_back({"argmax", [=] { return 4.0 * V; },
                            [=](cudaStream_t s, bool) {
                                return argmax_step(m->d_token, m->d_hist, m->d_pos, m->logits, V, s);
                            }});
    } else
    m->steps.push_back({"gemv_lm_head_argmax", [=] { return double(V) * D * 4 + 8.0 * D + 4.0 * V; },
                        [=](cudaStream_t s, bool pdl) {
                            GemvF32Args a = {};
                            a.w = m->lm_head; a.x = m->h; a.g = m->norm; a.eps = 1e-5f; a.y = m->logits;
                            a.n = V; a.d = D;
                            a.part_v = m->am_v; a.part_i = m->am_i; a.counter = m->am_cnt;
                            a.out_token = m->d_token; a.history = m->d_hist; a.pos = m->d_pos;
                            return launch_gemv_f32(a, true, true, s, pdl);
                        }});
    if (m->temperature > 0.f)
        m->steps.push_back({"sample", [=] { return 3.0 * 4 * V; },
                            [=](cudaStream_t s, bool) {
                                return sample_step(m->d_token, m->d_hist, m->d_pos, m->logits, V, m->temperature,
                                                   m->sample_seed, s);
                            }});
    return TL_OK;
}

tl_status run_steps_eager(tl_model* m) {
    for (size_t i = 0; i < m->steps.size(); i++) TL_TRY(m->steps[i].launch(m->stream, m->pdl && i > 0));
    return TL_OK;
}

tl_status capture_graph(tl_model* m) {
    TL_CUDA_TRY(cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal));
    tl_status st = run_steps_eager(m);
    cudaGraph_t g = nullptr;
    cudaError_t e = cudaStreamEndCapture(m->stream, &g);
    if (m->persistent && (st != TL_OK || e != cudaSuccess)) {
        // One cooperative launch per step needs no graph: launch it directly.
        if (g) cudaGraphDestroy(g);
        cudaGetLastError();
        clear_error();
        return TL_OK;
    }
    if (st != TL_OK) {
        if (g) cudaGraphDestroy(g);
        return st;
    }
    if (e != cudaSuccess) return set_error(TL_ERR_CUDA, "graph capture failed: %s", cudaGetErrorString(e));
    e = cudaGraphInstantiate(&m->graph_exec, g, 0);
    if (e != cudaSuccess) {
        cudaGraphDestroy(g);
        return set_error(TL_ERR_CUDA, "graph instantiate failed: %s", cudaGetErrorString(e));
    }
    m->graph = g;
    return TL_OK;
}

// Steps and graph again, after a change of what a step's launches capture.
tl_status rebuild_steps(tl_model* m) {
    if (m->graph_exec) {
        cudaGraphExecDestroy(m->graph_exec);
        m->graph_exec = nullptr;
    }
    if (m->graph) {
        cudaGraphDestroy(m->graph);
        m->graph = nullptr;
    }
    TL_TRY(build_steps(m));
    if (m->use_graph) TL_TRY(capture_graph(m));
    return TL_OK;
}

tl_status run_step(tl_model* m) {
    if (m->graph_exec) {
        TL_CUDA_TRY(cudaGraphLaunch(m->graph_exec, m->stream));
        return TL_OK;
    }
    return run_steps_eager(m);
}

tl_status set_token(tl_model* m, uint32_t token) {
    if (token >= m->cfg.vocab_size)
        return set_error(TL_ERR_INVALID_ARGUMENT, "token %u >= vocab_size %zu", token, m->cfg.vocab_size);
    m->h_pinned[0] = token;
    TL_CUDA_TRY(cudaMemcpyAsync(m->d_token, m->h_pinned, 4, cudaMemcpyHostToDevice, m->stream));
    return TL_OK;
}

// A tensor-parallel model runs only once every rank's exchange buffer is mapped.
tl_status check_tp_ready(const tl_model* m) {
    if (m->tp > 1 && !m->connected)
        return set_error(TL_ERR_INVALID_ARGUMENT, "tensor-parallel model: call tl_model_tp_connect on every rank first");
    if (m->broken)
        return set_error(TL_ERR_TIMEOUT, "tensor-parallel exchange state was lost after a device-side timeout; "
                                         "reload the model on every rank");
    return TL_OK;
}

tl_status check_capacity(const tl_model* m, size_t steps) {
    if (m->pos + steps > m->max_seq)
        return set_error(TL_ERR_CAPACITY, "KV cache full: pos %zu + %zu steps > max_seq %zu", m->pos, steps,
                         m->max_seq);
    return TL_OK;
}

// A weight GEMM of the batched paths for layer l (which: 0 q|k|v, 1 o, 2
// gate|up, 3 down): the int8 weights in place (gemm_q8) or, with
// tl_model_options.weights_f16, their fp16 copies (gemm_f16).
tl_status layer_gemm(const tl_model* m, size_t l, int which, int epi, const __half* A, int M, int K, int N, void* C,
                     int ldc, cudaStream_t s) {
    if (m->weights_f16) return gemm_f16(epi, A, M, K, m->lw16[l][which], N, C, ldc, m->err, s);
    return gemm_q8(epi, A, M, K, m->lq8[l][which], N, C, ldc, m->err, s);
}
tl_status layer_gemm_splitk(const tl_model* m, size_t l, int which, const __half* A, int M, int K, int N,
                            float* part, size_t part_floats, int* ks, cudaStream_t s) {
    if (m->weights_f16) return gemm_f16_splitk(A, M, K, m->lw16[l][which], N, part, part_floats, ks, m->err, s);
    return gemm_q8_splitk(A, M, K, m->lq8[l][which], N, part, part_floats, ks, m->err, s);
}

// fp16 weights and row buffers of the batched prompt pass (first use / growth).
tl_status ensure_prefill(tl_model* m, size_t n) {
    const int64_t D = m->cfg.hidden_size, HD = m->cfg.head_dim, H = m->lH, KV = m->lKV, F = m->lF;
    const int64_t NQKV = (H + 2 * KV) * HD, L = m->cfg.n_layers;
    if (m->weights_f16 && m->lw16.empty()) {
        if (F % 128) return set_error(TL_ERR_UNSUPPORTED, "prefill: intermediate_size %lld not a multiple of 128",
                                      static_cast<long long>(F));
        using A = DeviceArena;
        const size_t per = A::pad(NQKV * D * 2) + A::pad(D * H * HD * 2) + A::pad(2 * F * D * 2) + A::pad(D * F * 2);
        TL_TRY(m->w16.reserve(per * L));
        m->lw16.resize(L);
        for (int64_t l = 0; l < L; l++) {
            const LayerW& w = m->layers[l];
            auto& W = m->lw16[l];
            W[0] = m->w16.take<__half>(NQKV * D);
            W[1] = m->w16.take<__half>(D * H * HD);
            W[2] = m->w16.take<__half>(2 * F * D);
            W[3] = m->w16.take<__half>(D * F);
            // the arena's scales are already 1/s; fp8 weights (null scales) convert exactly
            TL_TRY(dequant_f16(W[0], w.wqkv, w.sqkv, nullptr, nullptr, NQKV, D, false, m->stream));
            TL_TRY(dequant_f16(W[1], w.wo, w.so, nullptr, nullptr, D, H * HD, false, m->stream));
            TL_TRY(dequant_f16(W[2], w.w1, w.s1, w.w3, w.s3, F, D, true, m->stream));
            TL_TRY(dequant_f16(W[3], w.w2, w.s2, nullptr, nullptr, D, F, false, m->stream));
        }
    }
    if (!m->weights_f16 && m->lq8.empty()) {
        if (F % 128) return set_error(TL_ERR_UNSUPPORTED, "prefill: intermediate_size %lld not a multiple of 128",
                                      static_cast<long long>(F));
        using A = DeviceArena;
        const bool f8 = m->w_f8;  // e5m2 weights carry no scales
        if (!f8) {
            const size_t per = A::pad(NQKV * (D / 64) * 4) + A::pad(D * (H * HD / 64) * 4) +
                               2 * A::pad(F * (D / 64) * 4) + A::pad(D * (F / 64) * 4);
            TL_TRY(m->scT.reserve(per * L));
        }
        m->lq8.resize(L);
        for (int64_t l = 0; l < L; l++) {
            const LayerW& w = m->layers[l];
            auto& Q = m->lq8[l];
            Q[0].q = w.wqkv;
            Q[1].q = w.wo;
            Q[2].q = w.w1;
            Q[2].q2 = w.w3;
            Q[3].q = w.w2;
            if (f8) continue;
            // the arena's scales are already 1/s; [rows][groups] -> [groups][rows]
            auto tr = [&](const float* src, int64_t rows, int64_t cols, const float** dst) -> tl_status {
                float* t = m->scT.take<float>(rows * (cols / 64));
                *dst = t;
                return transpose_scales(t, src, static_cast<int>(rows), static_cast<int>(cols / 64), m->stream);
            };
            TL_TRY(tr(w.sqkv, NQKV, D, &Q[0].sT));
            TL_TRY(tr(w.so, D, H * HD, &Q[1].sT));
            TL_TRY(tr(w.s1, F, D, &Q[2].sT));
            TL_TRY(tr(w.s3, F, D, &Q[2].sT2));
            TL_TRY(tr(w.s2, D, F, &Q[3].sT));
        }
    }
    if (n > m->rows_cap) {
        m->rows.release();
        m->rows = DeviceArena();
        const size_t cap = std::max<size_t>(n, 64);
        using A = DeviceArena;
        // fp16 K and (transposed, rows padded to 64 keys) V of one layer's cache
        const size_t kvh = static_cast<size_t>(KV) * ((m->max_seq + 63) / 64 * 64) * HD;
        TL_TRY(m->rows.reserve(A::pad(cap * D * 4) + A::pad(cap * NQKV * 4) + A::pad(cap * D * 2) +
                               2 * A::pad(cap * H * HD * 2) + A::pad(cap * F * 2) + A::pad(cap * 4) +
                               2 * A::pad(kvh * 2)));
        m->p_h = m->rows.take<float>(cap * D);
        m->p_qkv = m->rows.take<float>(cap * NQKV);
        m->p_x16 = m->rows.take<__half>(cap * D);
        m->p_q16 = m->rows.take<__half>(cap * H * HD);
        m->p_ctx16 = m->rows.take<__half>(cap * H * HD);
        m->p_act16 = m->rows.take<__half>(cap * F);
        m->p_tok = m->rows.take<uint32_t>(cap);
        m->p_k16 = m->rows.take<__half>(kvh);
        m->p_v16 = m->rows.take<__half>(kvh);
        if (!m->p_v16) return set_error(TL_ERR_OUT_OF_MEMORY, "prefill row arena (internal)");
        m->rows_cap = cap;
    }
    return TL_OK;
}

tl_status sync(tl_model* m) {
    {  // the device error flag (bounded waits of the persistent step and the tensor-core kernels)
        cudaError_t e = cudaMemcpyAsync(m->h_pinned + 3, m->err, 4, cudaMemcpyDeviceToHost, m->stream);
        if (e != cudaSuccess) return set_error(TL_ERR_CUDA, "error-flag read: %s", cudaGetErrorString(e));
    }
    cudaError_t e = cudaStreamSynchronize(m->stream);
    if (e != cudaSuccess) return set_error(TL_ERR_CUDA, "decode step failed: %s", cudaGetErrorString(e));
    if (m->h_pinned[3] != 0) {
        const unsigned code = m->h_pinned[3];
        if (code >= 1000) {
            int dbg[4] = {0, 0, 0, 0};
            cudaMemcpy(dbg, m->dbg, sizeof(dbg), cudaMemcpyDeviceToHost);
            cudaMemsetAsync(m->err, 0, 4, m->stream);
            cudaMemsetAsync(m->dbg, 0, 16, m->stream);
            cudaStreamSynchronize(m->stream);
            m->h_pinned[3] = 0;
            return set_error(TL_ERR_INVALID_ARGUMENT, "decode kernel self-check: site %d values %d %d", dbg[0],
                             dbg[1], dbg[2]);
        }
        // A bounded wait inside the kernel gave up: clear the barrier and
        // ticket state so the next step starts clean, and report it.
        cudaMemsetAsync(m->bar, 0, 4, m->stream);
        cudaMemsetAsync(m->ticket, 0, 4, m->stream);
        cudaMemsetAsync(m->attn_cnt, 0, sizeof(unsigned) * m->cfg.n_heads, m->stream);
        if (m->qkv_cnt) cudaMemsetAsync(m->qkv_cnt, 0, sizeof(unsigned) * m->cfg.n_heads, m->stream);
        cudaMemsetAsync(m->err, 0, 4, m->stream);
        cudaStreamSynchronize(m->stream);
        m->h_pinned[3] = 0;
        if (code == kDevErrInput) return set_error(TL_ERR_INVALID_ARGUMENT, "decode kernel: token or position out of range");
        if (m->tp > 1) m->broken = true;
        return set_error(TL_ERR_TIMEOUT, "device wait timed out (code %u: %s)", code, device_err_text(code));
    }
    return TL_OK;
}

}  // namespace
}  // namespace tl

extern "C" {

tl_status tl_model_load_buffer(const void* data, size_t size, const tl_model_options* opts, tl_model** out) {
    clear_error();
    TL_REQUIRE(data && out, "tl_model_load_buffer: null argument");
    *out = nullptr;
    return create_model(static_cast<const uint8_t*>(data), size, opts, out);
}

tl_status tl_model_load(const char* path, const tl_model_options* opts, tl_model** out) {
    clear_error();
    TL_REQUIRE(path && out, "tl_model_load: null argument");
    *out = nullptr;
    // Parameters::map_file (parameters.cpp:10-29): read-only private mapping.
    const int fd = open(path, O_RDONLY);
    if (fd < 0) return set_error(TL_ERR_IO, "cannot open %s: %s", path, std::strerror(errno));
    struct stat st;
    if (fstat(fd, &st) < 0) {
        close(fd);
        return set_error(TL_ERR_IO, "cannot stat %s: %s", path, std::strerror(errno));
    }
    const size_t size = static_cast<size_t>(st.st_size);
    void* p = size ? mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0) : MAP_FAILED;
    close(fd);
    if (p == MAP_FAILED) return set_error(TL_ERR_IO, "cannot map %s (%zu bytes)", path, size);
    const tl_status s = create_model(static_cast<const uint8_t*>(p), size, opts, out);
    munmap(p, size);
    return s;
}

tl_status tl_model_destroy(tl_model* m) {
    clear_error();
    if (!m) return TL_OK;
    if (m->n_batches > 0)  // each holds the model; destroying it first would leave them dangling
        return set_error(TL_ERR_INVALID_ARGUMENT, "tl_model_destroy: %d batch(es) of this model still exist; "
                                                  "tl_batch_destroy them first", m->n_batches);
    cudaSetDevice(m->device);
    if (m->stream) cudaStreamSynchronize(m->stream);
    if (m->graph_exec) cudaGraphExecDestroy(m->graph_exec);
    if (m->graph) cudaGraphDestroy(m->graph);
    m->weights.release();
    m->state.release();
    m->tiles.release();
    m->scT.release();
    m->w16.release();
    m->rows.release();
    m->lm16_arena.release();
    if (m->d_layers) cudaFree(m->d_layers);
    if (m->h_pinned) cudaFreeHost(m->h_pinned);
    for (int q = 0; q < kMaxTp; q++)
        if (m->xpeer_open[q]) cudaIpcCloseMemHandle(m->xpeer_open[q]);
    if (m->xbuf) cudaFree(m->xbuf);
    if (m->stream) cudaStreamDestroy(m->stream);
    delete m;
    return TL_OK;
}

tl_status tl_model_config(const tl_model* m, tl_config* out) {
    clear_error();
    TL_REQUIRE(m && out, "tl_model_config: null argument");
    *out = m->cfg;
    return TL_OK;
}

tl_status tl_model_tp_handle(const tl_model* m, void* handle) {
    clear_error();
    TL_REQUIRE(m && handle, "tl_model_tp_handle: null argument");
    if (m->tp < 2) return set_error(TL_ERR_INVALID_ARGUMENT, "tl_model_tp_handle: model was not loaded with tp_size > 1");
    TL_CUDA_TRY(cudaSetDevice(m->device));
    cudaIpcMemHandle_t h;
    TL_CUDA_TRY(cudaIpcGetMemHandle(&h, m->xbuf));
    static_assert(sizeof(h) == TL_TP_HANDLE_BYTES, "IPC handle size");
    std::memcpy(handle, &h, sizeof(h));
    return TL_OK;
}

tl_status tl_model_tp_connect(tl_model* m, const void* handles) {
    clear_error();
    TL_REQUIRE(m && handles, "tl_model_tp_connect: null argument");
    if (m->tp < 2) return set_error(TL_ERR_INVALID_ARGUMENT, "tl_model_tp_connect: model was not loaded with tp_size > 1");
    if (m->connected) return set_error(TL_ERR_INVALID_ARGUMENT, "tl_model_tp_connect: already connected");
    TL_CUDA_TRY(cudaSetDevice(m->device));
    for (int q = 0; q < m->tp; q++) {
        if (q == m->rank) continue;
        cudaIpcMemHandle_t h;
        std::memcpy(&h, static_cast<const uint8_t*>(handles) + static_cast<size_t>(q) * TL_TP_HANDLE_BYTES, sizeof(h));
        void* p = nullptr;
        const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess)
            return set_error(TL_ERR_CUDA, "tl_model_tp_connect: opening rank %d's exchange buffer failed: %s", q,
                             cudaGetErrorString(e));
        m->xpeer_open[q] = static_cast<uint8_t*>(p);
        m->dargs.xpeer[q] = static_cast<uint8_t*>(p);
    }
    m->connected = true;
    // the step launch (and its graph) captured the arguments before the peers were known
    return rebuild_steps(m);
}

tl_status tl_model_set_sampling(tl_model* m, float temperature, uint64_t seed) {
    clear_error();
    TL_REQUIRE(m, "tl_model_set_sampling: null model");
    TL_REQUIRE(std::isfinite(temperature), "tl_model_set_sampling: temperature must be finite");
    if (temperature > 0.f && m->tp > 1)
        return set_error(TL_ERR_UNSUPPORTED, "tl_model_set_sampling: sampling needs the whole vocabulary on one "
                                             "rank (not available under tensor parallelism)");
    TL_CUDA_TRY(cudaSetDevice(m->device));
    TL_CUDA_TRY(cudaStreamSynchronize(m->stream));
    m->temperature = temperature > 0.f ? temperature : 0.f;
    m->sample_seed = seed;
    m->dargs.temperature = m->temperature;
    m->dargs.sample_seed = seed;
    return rebuild_steps(m);
}

tl_status tl_model_forward(tl_model* m, uint32_t token, float* logits, uint32_t* next_token) {
    clear_error();
    TL_REQUIRE(m, "tl_model_forward: null model");
    TL_TRY(check_tp_ready(m));
    TL_CUDA_TRY(cudaSetDevice(m->device));
    TL_TRY(check_capacity(m, 1));
    TL_TRY(set_token(m, token));
    TL_TRY(run_step(m));
    if (logits)
        TL_CUDA_TRY(cudaMemcpyAsync(logits, m->logits, m->lV * 4, cudaMemcpyDeviceToHost, m->stream));
    if (next_token)
        TL_CUDA_TRY(cudaMemcpyAsync(m->h_pinned + 1, m->d_token, 4, cudaMemcpyDeviceToHost, m->stream));
    TL_TRY(sync(m));
    m->pos++;
    if (next_token) *next_token = m->h_pinned[1];
    return TL_OK;
}

tl_status prefill_impl(tl_model* m, const uint32_t* tokens, size_t n, float* logits, uint32_t* next_token,
                       float* ms);

tl_status tl_model_prefill(tl_model* m, const uint32_t* tokens, size_t n, float* logits, uint32_t* next_token) {
    clear_error();
    return prefill_impl(m, tokens, n, logits, next_token, nullptr);
}

tl_status tl_model_time_prefill(tl_model* m, const uint32_t* tokens, size_t n, uint32_t* next_token, float* ms) {
    clear_error();
    TL_REQUIRE(ms, "tl_model_time_prefill: null ms");
    return prefill_impl(m, tokens, n, nullptr, next_token, ms);
}

tl_status prefill_impl(tl_model* m, const uint32_t* tokens, size_t n, float* logits, uint32_t* next_token,
                       float* ms_out) {
    TL_REQUIRE(m && tokens && n > 0, "tl_model_prefill: bad arguments");
    if (m->tp > 1) return set_error(TL_ERR_UNSUPPORTED, "tl_model_prefill: not available under tensor parallelism");
    TL_REQUIRE(n < (1u << 30), "tl_model_prefill: n too large");
    for (size_t i = 0; i < n; i++)
        TL_REQUIRE(tokens[i] < m->cfg.vocab_size, "token %u >= vocab_size %zu", tokens[i], m->cfg.vocab_size);
    TL_TRY(check_capacity(m, n));
    TL_CUDA_TRY(cudaSetDevice(m->device));
    TL_TRY(ensure_prefill(m, n));
    const int M = static_cast<int>(n), p0 = static_cast<int>(m->pos);
    const int D = static_cast<int>(m->cfg.hidden_size), HD = static_cast<int>(m->cfg.head_dim);
    const int H = static_cast<int>(m->lH), KV = static_cast<int>(m->lKV), F = static_cast<int>(m->lF);
    const int NQKV = (H + 2 * KV) * HD, V = static_cast<int>(m->lV);
    const int ms = static_cast<int>(m->max_seq);
    const float scale = static_cast<float>(1.0 / std::sqrt(static_cast<double>(HD)));  // modules.cpp:79-80
    cudaStream_t s = m->stream;
    TL_CUDA_TRY(cudaMemcpyAsync(m->p_tok, tokens, n * 4, cudaMemcpyHostToDevice, s));
    Events ev;
    if (ms_out) {  // device time of the whole pass, token ids resident
        TL_TRY(ev.create(2));
        TL_CUDA_TRY(cudaEventRecord(ev[0], s));
    }
    TL_TRY(embed_rows(m->p_h, m->embed, m->p_tok, M, D, s));
    for (size_t l = 0; l < m->cfg.n_layers; l++) {
        const LayerW& w = m->layers[l];
        float* kc = m->kc + l * layer_kv_floats(m);
        float* vc = m->vc + l * layer_kv_floats(m);
        TL_TRY(rmsnorm_rows_f16(m->p_x16, m->p_h, w.g_in, M, D, s));
        TL_TRY(layer_gemm(m, l, 0, kEpiStoreF32, m->p_x16, M, D, NQKV, m->p_qkv, NQKV, s));
        TL_TRY(rope_cache_rows(m->p_q16, m->p_qkv, kc, vc, m->cos_tab, m->sin_tab, M, p0, H, KV, HD, ms, s));
        if (HD == 128 && H == 4 * KV)  // tensor-core attention (tcgen05, tensor memory)
            TL_TRY(attention_prefill_tc(m->p_ctx16, m->p_q16, m->p_k16, m->p_v16, kc, vc, M, p0, H, KV, HD, ms,
                                        scale, m->window, m->err, s));
        else
            TL_TRY(attention_prefill(m->p_ctx16, m->p_q16, m->p_k16, m->p_v16, kc, vc, M, p0, H, KV, HD, ms, scale,
                                     m->window, s));
        TL_TRY(layer_gemm(m, l, 1, kEpiAddF32, m->p_ctx16, M, H * HD, D, m->p_h, D, s));
        TL_TRY(rmsnorm_rows_f16(m->p_x16, m->p_h, w.g_post, M, D, s));
        TL_TRY(layer_gemm(m, l, 2, kEpiSwiGluF16, m->p_x16, M, D, 2 * F, m->p_act16, F, s));
        TL_TRY(layer_gemm(m, l, 3, kEpiAddF32, m->p_act16, M, F, D, m->p_h, D, s));
    }
    // the last token's hidden state: final norm, lm_head, sample_max (modules.cpp:147-171, main.cpp:10-21)
    TL_CUDA_TRY(cudaMemcpyAsync(m->h, m->p_h + static_cast<size_t>(M - 1) * D, D * 4, cudaMemcpyDeviceToDevice, s));
    m->h_pinned[2] = static_cast<uint32_t>(p0 + M - 1);
    TL_CUDA_TRY(cudaMemcpyAsync(m->d_pos, m->h_pinned + 2, 4, cudaMemcpyHostToDevice, s));
    if (m->lm_8bit) {
        GemvI8Args a = {};
        a.w = m->lm_q; a.s = m->lm_s; a.f8 = m->w_f8 ? 1 : 0; a.x = m->h; a.g = m->norm; a.eps = 1e-5f;
        a.y = m->logits; a.n = V; a.d = D;
        TL_TRY(launch_gemv_i8(a, I8Mode::Store, true, true, s, false));
        TL_TRY(argmax_step(m->d_token, m->d_hist, m->d_pos, m->logits, V, s));
    } else {
        GemvF32Args a = {};
        a.w = m->lm_head; a.x = m->h; a.g = m->norm; a.eps = 1e-5f; a.y = m->logits;
        a.n = V; a.d = D;
        a.part_v = m->am_v; a.part_i = m->am_i; a.counter = m->am_cnt;
        a.out_token = m->d_token; a.history = m->d_hist; a.pos = m->d_pos;
        TL_TRY(launch_gemv_f32(a, true, true, s, false));
    }
    if (m->temperature > 0.f)
        TL_TRY(sample_step(m->d_token, m->d_hist, m->d_pos, m->logits, V, m->temperature, m->sample_seed, s));
    if (ms_out) TL_CUDA_TRY(cudaEventRecord(ev[1], s));
    if (logits) TL_CUDA_TRY(cudaMemcpyAsync(logits, m->logits, static_cast<size_t>(V) * 4, cudaMemcpyDeviceToHost, s));
    TL_CUDA_TRY(cudaMemcpyAsync(m->h_pinned + 1, m->d_token, 4, cudaMemcpyDeviceToHost, s));
    TL_TRY(sync(m));
    if (ms_out) TL_CUDA_TRY(cudaEventElapsedTime(ms_out, ev[0], ev[1]));
    m->pos = p0 + n;
    if (next_token) *next_token = m->h_pinned[1];
    return TL_OK;
}

tl_status tl_model_generate(tl_model* m, const uint32_t* prompt, size_t n_prompt, size_t n_new, uint32_t* out) {
    clear_error();
    TL_REQUIRE(m && prompt && n_prompt > 0 && (out || n_new == 0), "tl_model_generate: bad arguments");
    TL_REQUIRE(n_new > 0, "tl_model_generate: n_new must be positive (the last prompt token is forwarded by it)");
    TL_TRY(check_tp_ready(m));
    TL_CUDA_TRY(cudaSetDevice(m->device));
    TL_TRY(check_capacity(m, n_prompt - 1 + n_new));
    for (size_t i = 0; i < n_prompt; i++)
        TL_REQUIRE(prompt[i] < m->cfg.vocab_size, "prompt token %u >= vocab_size", prompt[i]);
    TL_CUDA_TRY(cudaMemcpyAsync(m->d_prompt, prompt, n_prompt * 4, cudaMemcpyHostToDevice, m->stream));
    // main.cpp:69-71: forward every prompt token but the last.
    for (size_t i = 0; i + 1 < n_prompt; i++) {
        TL_CUDA_TRY(cudaMemcpyAsync(m->d_token, m->d_prompt + i, 4, cudaMemcpyDeviceToDevice, m->stream));
        TL_TRY(run_step(m));
    }
    // main.cpp:73-77: t = last prompt token; n_new times t = argmax(forward(t)).
    TL_CUDA_TRY(cudaMemcpyAsync(m->d_token, m->d_prompt + n_prompt - 1, 4, cudaMemcpyDeviceToDevice, m->stream));
    const size_t first = m->pos + n_prompt - 1;
    for (size_t i = 0; i < n_new; i++) TL_TRY(run_step(m));
    TL_CUDA_TRY(cudaMemcpyAsync(out, m->d_hist + first, n_new * 4, cudaMemcpyDeviceToHost, m->stream));
    TL_TRY(sync(m));
    m->pos += n_prompt - 1 + n_new;
    return TL_OK;
}

tl_status tl_model_get_pos(const tl_model* m, size_t* pos) {
    clear_error();
    TL_REQUIRE(m && pos, "tl_model_get_pos: null argument");
    *pos = m->pos;
    return TL_OK;
}

tl_status tl_model_set_pos(tl_model* m, size_t pos) {
    clear_error();
    TL_REQUIRE(m, "tl_model_set_pos: null model");
    if (pos > m->max_seq) return set_error(TL_ERR_CAPACITY, "pos %zu > max_seq %zu", pos, m->max_seq);
    TL_CUDA_TRY(cudaSetDevice(m->device));
    m->h_pinned[2] = static_cast<uint32_t>(pos);
    TL_CUDA_TRY(cudaMemcpyAsync(m->d_pos, m->h_pinned + 2, 4, cudaMemcpyHostToDevice, m->stream));
    TL_TRY(sync(m));
    m->pos = pos;
    return TL_OK;
}

tl_status tl_model_layer_forward(tl_model* m, int layer, float* hidden) {
    clear_error();
    TL_REQUIRE(m && hidden, "tl_model_layer_forward: null argument");
    TL_REQUIRE(layer >= 0 && static_cast<size_t>(layer) < m->cfg.n_layers, "layer %d out of range", layer);
    if (m->tp > 1) return set_error(TL_ERR_UNSUPPORTED, "tl_model_layer_forward: not available under tensor parallelism");
    TL_TRY(check_capacity(m, 1));
    TL_CUDA_TRY(cudaSetDevice(m->device));
    const size_t D = m->cfg.hidden_size;
    TL_CUDA_TRY(cudaMemcpyAsync(m->h, hidden, D * 4, cudaMemcpyHostToDevice, m->stream));
    std::vector<Step> steps;
    add_layer_steps(m, layer, steps);
    for (auto& s : steps) TL_TRY(s.launch(m->stream, false));
    TL_CUDA_TRY(cudaMemcpyAsync(hidden, m->h, D * 4, cudaMemcpyDeviceToHost, m->stream));
    return sync(m);
}

tl_status tl_model_read_kv(const tl_model* m, int layer, size_t pos, float* k, float* v) {
    clear_error();
    TL_REQUIRE(m && k && v, "tl_model_read_kv: null argument");
    TL_REQUIRE(layer >= 0 && static_cast<size_t>(layer) < m->cfg.n_layers && pos < m->max_seq,
               "tl_model_read_kv: layer/pos out of range");
    TL_CUDA_TRY(cudaSetDevice(m->device));
    const size_t hd = m->cfg.head_dim;
    for (size_t kh = 0; kh < static_cast<size_t>(m->lKV); kh++) {
        const size_t off = layer * layer_kv_floats(m) + (kh * m->max_seq + pos) * hd;
        TL_CUDA_TRY(cudaMemcpyAsync(k + kh * hd, m->kc + off, hd * 4, cudaMemcpyDeviceToHost, m->stream));
        TL_CUDA_TRY(cudaMemcpyAsync(v + kh * hd, m->vc + off, hd * 4, cudaMemcpyDeviceToHost, m->stream));
    }
    return sync(const_cast<tl_model*>(m));
}

tl_status tl_model_time_decode(tl_model* m, uint32_t token, size_t n, uint32_t* out, float* ms) {
    clear_error();
    TL_REQUIRE(m && ms && n > 0, "tl_model_time_decode: bad arguments");
    TL_TRY(check_tp_ready(m));
    TL_CUDA_TRY(cudaSetDevice(m->device));
    TL_TRY(check_capacity(m, n));
    TL_TRY(set_token(m, token));
    Events ev;
    TL_TRY(ev.create(2));
    const size_t first = m->pos;
    tl_status st = TL_OK;
    cudaEventRecord(ev[0], m->stream);
    for (size_t i = 0; i < n && st == TL_OK; i++) st = run_step(m);
    cudaEventRecord(ev[1], m->stream);
    if (st == TL_OK) st = sync(m);
    if (st == TL_OK) {
        cudaEventElapsedTime(ms, ev[0], ev[1]);
        m->pos += n;
        if (out) {
            cudaMemcpy(out, m->d_hist + first, n * 4, cudaMemcpyDeviceToHost);
        }
    }
    return st;
}

tl_status tl_model_profile(tl_model* m, uint32_t token, size_t n, tl_kernel_time* kinds, int max_kinds,
                           int* n_kinds) {
    clear_error();
    TL_REQUIRE(m && kinds && n_kinds && n > 0 && max_kinds > 0, "tl_model_profile: bad arguments");
    TL_TRY(check_tp_ready(m));
    TL_CUDA_TRY(cudaSetDevice(m->device));
    TL_TRY(check_capacity(m, n));
    TL_TRY(set_token(m, token));
    const size_t S = m->steps.size();
    Events ev;
    TL_TRY(ev.create(S + 1));
    std::vector<std::string> names;
    std::vector<double> total_ms, bytes;
    std::vector<int> launches;
    tl_status st = TL_OK;
    for (size_t it = 0; it < n && st == TL_OK; it++) {
        std::vector<double> step_bytes(S);
        for (size_t i = 0; i < S; i++) step_bytes[i] = m->steps[i].bytes();
        cudaEventRecord(ev[0], m->stream);
        for (size_t i = 0; i < S && st == TL_OK; i++) {
            st = m->steps[i].launch(m->stream, false);
            cudaEventRecord(ev[i + 1], m->stream);
        }
        if (st == TL_OK) st = sync(m);
        if (st != TL_OK) break;
        m->pos++;
        for (size_t i = 0; i < S; i++) {
            float ms = 0.f;
            cudaEventElapsedTime(&ms, ev[i], ev[i + 1]);
            size_t k = 0;
            while (k < names.size() && names[k] != m->steps[i].name) k++;
            if (k == names.size()) {
                names.push_back(m->steps[i].name);
                total_ms.push_back(0);
                bytes.push_back(0);
                launches.push_back(0);
            }
            total_ms[k] += ms;
            bytes[k] += step_bytes[i];
            launches[k] += 1;
        }
    }
    if (st != TL_OK) return st;
    *n_kinds = static_cast<int>(std::min<size_t>(names.size(), max_kinds));
    for (int k = 0; k < *n_kinds; k++) {
        std::snprintf(kinds[k].name, sizeof(kinds[k].name), "%s", names[k].c_str());
        kinds[k].launches = launches[k];
        kinds[k].total_ms = total_ms[k];
        kinds[k].bytes_per_launch = bytes[k] / launches[k];
    }
    return TL_OK;
}

tl_status tl_model_trace_step(tl_model* m, uint32_t token, uint64_t* out, size_t cap, size_t* n_written) {
    clear_error();
    TL_REQUIRE(m && out && n_written, "tl_model_trace_step: null argument");
    if (!m->persistent) return set_error(TL_ERR_UNSUPPORTED, "tracing needs the persistent decode kernel");
    TL_TRY(check_tp_ready(m));
    TL_CUDA_TRY(cudaSetDevice(m->device));
    TL_TRY(check_capacity(m, 1));
    const size_t phases = 5 * m->cfg.n_layers + 1;
    const size_t n = static_cast<size_t>(m->grid) * phases * kTraceEvents;
    TL_REQUIRE(cap >= n + 2, "tl_model_trace_step: out holds %zu elements, %zu needed", cap, n + 2);
    unsigned long long* d_trace = nullptr;
    TL_CUDA_TRY(cudaMalloc(&d_trace, n * sizeof(unsigned long long)));
    tl_status st = TL_OK;
    if (cudaMemsetAsync(d_trace, 0, n * sizeof(unsigned long long), m->stream) != cudaSuccess)
        st = set_error(TL_ERR_CUDA, "trace buffer clear failed");
    if (st == TL_OK) st = set_token(m, token);
    if (st == TL_OK) {
        DecodeArgs a = m->dargs;
        a.trace = d_trace;
        st = launch_decode_step(a, m->grid, m->stages, m->mega_smem, m->stream);
    }
    if (st == TL_OK) st = sync(m);
    if (st == TL_OK) {
        m->pos++;
        out[0] = static_cast<uint64_t>(m->grid);
        out[1] = phases;
        if (cudaMemcpy(out + 2, d_trace, n * sizeof(unsigned long long), cudaMemcpyDeviceToHost) != cudaSuccess)
            st = set_error(TL_ERR_CUDA, "trace copy failed");
        *n_written = n + 2;
    }
    cudaFree(d_trace);
    return st;
}

// ---------------------------------------------------------------------------
// Batched decoding: B sequences with their own KV caches and positions.
// ---------------------------------------------------------------------------
}  // extern "C"

struct tl_batch {
    tl_model* m = nullptr;
    int B = 0, S = 1;
    size_t max_seq = 0;
    DeviceArena kv, rows;
    BatchKV bkv = {};
    float *hres = nullptr, *qf = nullptr, *part = nullptr, *logits = nullptr;
    __half *x16 = nullptr, *ctx16 = nullptr, *act16 = nullptr;
    uint32_t *tok = nullptr, *pos = nullptr, *next = nullptr;
    float* split = nullptr;  // split-K partials of the small-M GEMMs
    size_t split_floats = 0;
    // tensor parallelism: this rank's exchange buffer and the peers' (IPC)
    uint8_t* xbuf = nullptr;
    uint8_t* xpeer_open[kBatchMaxTp] = {};
    BatchXchg X = {};
    unsigned long long xseq = 0, aseq = 0;  // residual / argmax exchanges so far
    bool connected = false;
    uint32_t* h_pinned = nullptr;       // [B]
    std::vector<size_t> pos_host;
};

namespace tl {
namespace {

// One step of every sequence: token ids already in b->tok.
tl_status batch_step(tl_batch* b) {
    tl_model* m = b->m;
    cudaStream_t s = m->stream;
    const int B = b->B, D = static_cast<int>(m->cfg.hidden_size), HD = static_cast<int>(m->cfg.head_dim);
    const int H = static_cast<int>(m->lH), KV = static_cast<int>(m->lKV), F = static_cast<int>(m->lF);
    const int NQKV = (H + 2 * KV) * HD, V = static_cast<int>(m->lV);
    const float scale = static_cast<float>(1.0 / std::sqrt(static_cast<double>(HD)));  // modules.cpp:79-80
    size_t maxp = 0;
    for (size_t p : b->pos_host) maxp = std::max(maxp, p);
    const int S = std::max(1, std::min(b->S, static_cast<int>((maxp + 1 + 511) / 512)));  // >= 512 positions a split
    // q|k|v, o and down run split-K (B rows fill few output tiles); their
    // consumers (RoPE, residual + RMSNorm) sum the partials
    const size_t qkv_stride = static_cast<size_t>(B) * NQKV, d_stride = static_cast<size_t>(B) * D;
    int ks = 0;
    TL_TRY(embed_rows(b->hres, m->embed, b->tok, B, D, s));
    TL_TRY(residual_rmsnorm_rows(b->x16, b->hres, nullptr, 0, 0, m->layers[0].g_in, B, D, s));
    for (size_t l = 0; l < m->cfg.n_layers; l++) {
        const LayerW& w = m->layers[l];
        TL_TRY(layer_gemm_splitk(m, l, 0, b->x16, B, D, NQKV, b->split, b->split_floats, &ks, s));
        TL_TRY(rope_cache_batch(b->qf, b->split, ks, qkv_stride, b->bkv, static_cast<int>(l), b->pos, m->cos_tab,
                                m->sin_tab, B, H, KV, HD, s));
        TL_TRY(attention_decode_batch(b->part, b->qf, b->bkv, static_cast<int>(l), b->pos, B, H, KV, HD, S, scale,
                                      m->window, s));
        TL_TRY(attention_merge_batch(b->ctx16, b->part, B, H, HD, S, s));
        // under tensor parallelism the residual adds sum every rank's partial rows (exchange)
        auto residual = [&](const float* g) -> tl_status {
            if (m->tp > 1)
                return tp_residual_rmsnorm_rows(b->x16, b->hres, b->split, ks, d_stride, g, b->X, b->xseq++, m->err,
                                                s);
            return residual_rmsnorm_rows(b->x16, b->hres, b->split, ks, d_stride, g, B, D, s);
        };
        TL_TRY(layer_gemm_splitk(m, l, 1, b->ctx16, B, H * HD, D, b->split, b->split_floats, &ks, s));
        TL_TRY(residual(w.g_post));
        TL_TRY(layer_gemm_splitk(m, l, 2, b->x16, B, D, 2 * F, b->split, b->split_floats, &ks, s));
        TL_TRY(swiglu_rows(b->act16, b->split, ks, static_cast<size_t>(B) * 2 * F, B, static_cast<int>(F), s));
        TL_TRY(layer_gemm_splitk(m, l, 3, b->act16, B, F, D, b->split, b->split_floats, &ks, s));
        TL_TRY(residual(l + 1 < m->cfg.n_layers ? m->layers[l + 1].g_in : m->norm));
    }
    TL_TRY(gemm_f16(kEpiStoreF32, b->x16, B, D, m->lm16, V, b->logits, V, m->err, s));
    if (m->tp > 1)
        TL_TRY(tp_argmax_rows(b->next, b->logits, V, static_cast<int>(m->rank * m->lV), b->pos, b->X, b->aseq++,
                              m->err, s));
    else
        TL_TRY(argmax_rows(b->next, b->logits, B, V, b->pos, s));
    for (auto& p : b->pos_host) p++;
    return TL_OK;
}

tl_status batch_ready(const tl_batch* b, size_t steps) {
    TL_REQUIRE(b, "tl_batch: null batch");
    if (b->m->tp > 1) {
        if (!b->connected)
            return set_error(TL_ERR_INVALID_ARGUMENT, "tensor-parallel batch: call tl_batch_tp_connect on every rank");
        TL_TRY(check_tp_ready(b->m));
    }
    for (size_t p : b->pos_host)
        if (p + steps > b->max_seq)
            return set_error(TL_ERR_CAPACITY, "tl_batch: position %zu + %zu steps > max_seq %zu", p, steps, b->max_seq);
    return TL_OK;
}

}  // namespace
}  // namespace tl

extern "C" {

tl_status tl_batch_create(tl_model* m, int n_seq, size_t max_seq, tl_batch** out) {
    clear_error();
    TL_REQUIRE(m && out && n_seq > 0 && n_seq <= 4096, "tl_batch_create: bad arguments");
    *out = nullptr;
    if (m->tp > 1) {
        TL_REQUIRE(m->tp <= kBatchMaxTp, "tl_batch_create: tp %d > %d", m->tp, kBatchMaxTp);
        TL_TRY(check_tp_ready(m));
    }
    if (max_seq == 0) max_seq = m->max_seq;
    TL_REQUIRE(max_seq <= m->max_seq, "tl_batch_create: max_seq %zu > the model's %zu (RoPE tables)", max_seq,
               m->max_seq);
    TL_REQUIRE(m->cfg.head_dim == 128, "tl_batch_create: head_dim 128 is built");
    TL_CUDA_TRY(cudaSetDevice(m->device));
    TL_TRY(ensure_prefill(m, 1));  // fp16 weights
    const int64_t D = m->cfg.hidden_size, HD = m->cfg.head_dim, H = m->lH, KV = m->lKV, F = m->lF, V = m->lV;
    const int64_t L = m->cfg.n_layers, NQKV = (H + 2 * KV) * HD;
    if (!m->lm16) {
        TL_TRY(m->lm16_arena.reserve(DeviceArena::pad(V * D * 2)));
        m->lm16 = m->lm16_arena.take<__half>(V * D);
        if (m->lm_8bit) TL_TRY(dequant_f16(m->lm16, m->lm_q, m->lm_s, nullptr, nullptr, V, D, false, m->stream));
        else TL_TRY(f32_to_f16(m->lm16, m->lm_head, static_cast<size_t>(V) * D, m->stream));
    }
    std::unique_ptr<tl_batch> b(new tl_batch());
    b->m = m;
    b->B = n_seq;
    b->max_seq = max_seq;
    // most attention splits: about 16 CTAs per SM over the B x KV (sequence, kv head) pairs
    b->S = std::max(1, std::min(64, 16 * sm_count() / static_cast<int>(std::max<int64_t>(1, KV * n_seq))));
    const size_t layer = static_cast<size_t>(KV) * max_seq * HD;
    const size_t seq = layer * L;
    using A = DeviceArena;
    TL_TRY(b->kv.reserve(2 * A::pad(seq * n_seq * 4)));
    b->bkv.k = b->kv.take<float>(seq * n_seq);
    b->bkv.v = b->kv.take<float>(seq * n_seq);
    b->bkv.seq_stride = seq;
    b->bkv.layer_stride = layer;
    b->bkv.max_seq = static_cast<int>(max_seq);
    const size_t Bn = n_seq;
    // split-K partials: up to 16 K ranges of q|k|v / o / down, or 8 of the gate|up pairs
    b->split_floats = Bn * std::max<size_t>(16 * static_cast<size_t>(std::max<int64_t>(NQKV, D)),
                                            8 * 2 * static_cast<size_t>(F));
    TL_TRY(b->rows.reserve(A::pad(Bn * D * 4) + A::pad(Bn * H * HD * 4) +
                           A::pad(Bn * H * b->S * (HD + 4) * 4) + A::pad(Bn * V * 4) + A::pad(Bn * D * 2) +
                           A::pad(Bn * H * HD * 2) + A::pad(Bn * F * 2) + 3 * A::pad(Bn * 4) +
                           A::pad(b->split_floats * 4)));
    b->hres = b->rows.take<float>(Bn * D);
    b->qf = b->rows.take<float>(Bn * H * HD);
    b->part = b->rows.take<float>(Bn * H * b->S * (HD + 4));
    b->logits = b->rows.take<float>(Bn * V);
    b->x16 = b->rows.take<__half>(Bn * D);
    b->ctx16 = b->rows.take<__half>(Bn * H * HD);
    b->act16 = b->rows.take<__half>(Bn * F);
    b->tok = b->rows.take<uint32_t>(Bn);
    b->pos = b->rows.take<uint32_t>(Bn);
    b->next = b->rows.take<uint32_t>(Bn);
    b->split = b->rows.take<float>(b->split_floats);
    if (!b->split) return set_error(TL_ERR_OUT_OF_MEMORY, "tl_batch rows (internal)");
    TL_CUDA_TRY(cudaMemsetAsync(b->pos, 0, Bn * 4, m->stream));
    if (m->tp > 1) {  // exchange buffer (mapped by the peers in tl_batch_tp_connect)
        const size_t xb = bx_bytes(m->tp, n_seq, static_cast<int>(D));
        TL_CUDA_TRY(cudaMalloc(&b->xbuf, xb));
        TL_CUDA_TRY(cudaMemsetAsync(b->xbuf, 0, xb, m->stream));
        b->X.tp = m->tp;
        b->X.rank = m->rank;
        b->X.B = n_seq;
        b->X.D = static_cast<int>(D);
        b->X.buf[m->rank] = b->xbuf;
    }
    TL_CUDA_TRY(cudaMallocHost(&b->h_pinned, Bn * 4));
    b->pos_host.assign(Bn, 0);
    TL_CUDA_TRY(cudaStreamSynchronize(m->stream));
    m->n_batches++;
    *out = b.release();
    return TL_OK;
}

tl_status tl_batch_destroy(tl_batch* b) {
    clear_error();
    if (!b) return TL_OK;
    cudaSetDevice(b->m->device);
    cudaStreamSynchronize(b->m->stream);
    b->kv.release();
    b->rows.release();
    for (auto* p : b->xpeer_open)
        if (p) cudaIpcCloseMemHandle(p);
    if (b->xbuf) cudaFree(b->xbuf);
    if (b->h_pinned) cudaFreeHost(b->h_pinned);
    b->m->n_batches--;
    delete b;
    return TL_OK;
}

tl_status tl_batch_fill_kv_random(tl_batch* b, uint64_t seed, size_t n_pos) {
    clear_error();
    TL_REQUIRE(b && n_pos < b->max_seq && n_pos < (1u << 20), "tl_batch_fill_kv_random: bad arguments");
    tl_model* m = b->m;
    TL_CUDA_TRY(cudaSetDevice(m->device));
    TL_TRY(fill_kv_random(b->bkv, seed, b->B, static_cast<int>(m->cfg.n_layers), static_cast<int>(m->lKV),
                          static_cast<int>(m->cfg.head_dim), static_cast<int>(n_pos),
                          static_cast<int>(m->rank * m->lKV), static_cast<int>(m->cfg.n_kv_heads), m->stream));
    for (int i = 0; i < b->B; i++) b->h_pinned[i] = static_cast<uint32_t>(n_pos);
    TL_CUDA_TRY(cudaMemcpyAsync(b->pos, b->h_pinned, b->B * 4, cudaMemcpyHostToDevice, m->stream));
    TL_TRY(sync(m));
    b->pos_host.assign(b->B, n_pos);
    return TL_OK;
}

tl_status tl_batch_step(tl_batch* b, const uint32_t* tokens, float* logits, uint32_t* next_tokens) {
    clear_error();
    TL_TRY(batch_ready(b, 1));
    tl_model* m = b->m;
    TL_REQUIRE(tokens, "tl_batch_step: null tokens");
    for (int i = 0; i < b->B; i++)
        TL_REQUIRE(tokens[i] < m->cfg.vocab_size, "tl_batch_step: token %u >= vocab_size", tokens[i]);
    TL_CUDA_TRY(cudaSetDevice(m->device));
    std::memcpy(b->h_pinned, tokens, b->B * 4);
    TL_CUDA_TRY(cudaMemcpyAsync(b->tok, b->h_pinned, b->B * 4, cudaMemcpyHostToDevice, m->stream));
    TL_TRY(batch_step(b));
    if (logits)
        TL_CUDA_TRY(cudaMemcpyAsync(logits, b->logits, static_cast<size_t>(b->B) * m->lV * 4, cudaMemcpyDeviceToHost,
                                    m->stream));
    TL_CUDA_TRY(cudaMemcpyAsync(b->h_pinned, b->next, b->B * 4, cudaMemcpyDeviceToHost, m->stream));
    TL_TRY(sync(m));
    if (next_tokens) std::memcpy(next_tokens, b->h_pinned, b->B * 4);
    return TL_OK;
}

tl_status tl_batch_time_decode(tl_batch* b, const uint32_t* tokens, size_t n_steps, uint32_t* out, float* ms) {
    clear_error();
    TL_TRY(batch_ready(b, n_steps));
    TL_REQUIRE(tokens && ms && n_steps > 0, "tl_batch_time_decode: bad arguments");
    tl_model* m = b->m;
    TL_CUDA_TRY(cudaSetDevice(m->device));
    std::memcpy(b->h_pinned, tokens, b->B * 4);
    TL_CUDA_TRY(cudaMemcpyAsync(b->tok, b->h_pinned, b->B * 4, cudaMemcpyHostToDevice, m->stream));
    Events ev;
    TL_TRY(ev.create(2));
    TL_CUDA_TRY(cudaEventRecord(ev[0], m->stream));
    for (size_t i = 0; i < n_steps; i++) {
        TL_TRY(batch_step(b));
        // the argmax of this step is the next step's token (main.cpp:72-77 per sequence)
        TL_CUDA_TRY(cudaMemcpyAsync(b->tok, b->next, b->B * 4, cudaMemcpyDeviceToDevice, m->stream));
        if (out)
            TL_CUDA_TRY(cudaMemcpyAsync(out + i * b->B, b->next, b->B * 4, cudaMemcpyDeviceToHost, m->stream));
    }
    TL_CUDA_TRY(cudaEventRecord(ev[1], m->stream));
    TL_TRY(sync(m));
    TL_CUDA_TRY(cudaEventElapsedTime(ms, ev[0], ev[1]));
    return TL_OK;
}

tl_status tl_batch_tp_handle(const tl_batch* b, void* handle) {
    clear_error();
    TL_REQUIRE(b && handle, "tl_batch_tp_handle: null argument");
    if (b->m->tp < 2) return set_error(TL_ERR_INVALID_ARGUMENT, "tl_batch_tp_handle: model is not tensor-parallel");
    TL_CUDA_TRY(cudaSetDevice(b->m->device));
    cudaIpcMemHandle_t h;
    TL_CUDA_TRY(cudaIpcGetMemHandle(&h, b->xbuf));
    std::memcpy(handle, &h, sizeof(h));
    return TL_OK;
}

tl_status tl_batch_tp_connect(tl_batch* b, const void* handles) {
    clear_error();
    TL_REQUIRE(b && handles, "tl_batch_tp_connect: null argument");
    tl_model* m = b->m;
    if (m->tp < 2) return set_error(TL_ERR_INVALID_ARGUMENT, "tl_batch_tp_connect: model is not tensor-parallel");
    if (b->connected) return set_error(TL_ERR_INVALID_ARGUMENT, "tl_batch_tp_connect: already connected");
    TL_CUDA_TRY(cudaSetDevice(m->device));
    TL_CUDA_TRY(cudaStreamSynchronize(m->stream));  // the buffer's clear has landed
    for (int q = 0; q < m->tp; q++) {
        if (q == m->rank) continue;
        cudaIpcMemHandle_t h;
        std::memcpy(&h, static_cast<const uint8_t*>(handles) + static_cast<size_t>(q) * TL_TP_HANDLE_BYTES, sizeof(h));
        void* p = nullptr;
        const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess)
            return set_error(TL_ERR_CUDA, "tl_batch_tp_connect: opening rank %d's exchange buffer failed: %s", q,
                             cudaGetErrorString(e));
        b->xpeer_open[q] = static_cast<uint8_t*>(p);
        b->X.buf[q] = static_cast<uint8_t*>(p);
    }
    b->connected = true;
    return TL_OK;
}

tl_status tl_batch_read_kv(const tl_batch* b, int seq, int layer, size_t pos, float* k, float* v) {
    clear_error();
    TL_REQUIRE(b && k && v && seq >= 0 && seq < b->B && layer >= 0 &&
                   static_cast<size_t>(layer) < b->m->cfg.n_layers && pos < b->max_seq,
               "tl_batch_read_kv: bad arguments");
    const tl_model* m = b->m;
    TL_CUDA_TRY(cudaSetDevice(m->device));
    const size_t hd = m->cfg.head_dim;
    for (size_t kh = 0; kh < static_cast<size_t>(m->lKV); kh++) {
        const size_t off = seq * b->bkv.seq_stride + layer * b->bkv.layer_stride + (kh * b->max_seq + pos) * hd;
        TL_CUDA_TRY(cudaMemcpyAsync(k + kh * hd, b->bkv.k + off, hd * 4, cudaMemcpyDeviceToHost, m->stream));
        TL_CUDA_TRY(cudaMemcpyAsync(v + kh * hd, b->bkv.v + off, hd * 4, cudaMemcpyDeviceToHost, m->stream));
    }
    return sync(const_cast<tl_model*>(m));
}

tl_status tl_model_launches_per_step(const tl_model* m, int* launches) {
    clear_error();
    TL_REQUIRE(m && launches, "tl_model_launches_per_step: null argument");
    *launches = static_cast<int>(m->steps.size());
    return TL_OK;
}

}  // extern "C"
