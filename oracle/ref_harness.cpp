// ref_harness.cpp -- C entry points over the UNMODIFIED reference sources.
//
// TEST INFRASTRUCTURE ONLY.  oracle/Makefile compiles this file together with
// the reference's own src/*.cpp and main.cpp (renamed entry point) into
// oracle/_ref/libtorchless_ref.so.  Tests use it to pin the oracle
// restatement (tl_oracle.c) bit for bit, and bench.py's reference arm and
// cpu_baseline leg time the reference's own CPU code path through it.
//
// Nothing here re-implements reference arithmetic: every entry point builds
// the reference's Tensor views / InferenceState / Model<T> and calls the
// reference functions.  The only additions are the things the reference's
// CLI cannot do: load from an in-memory buffer, size MAX_SEQ_LEN, call
// RotaryEmbedding::init_freq (main.cpp never does, test_modules.cpp:169 does),
// and guard the KV cache bound (the reference overruns it silently under
// NDEBUG, inference_state.h:38-43).
#include <algorithm>
#include <chrono>
#include <cstdint>
#include <cstring>
#include <memory>
#include <random>
#include <string>
#include <vector>

#include "src/common/kernels.h"
#include "src/loader/parameters.h"
#include "src/model/mistral/inference_state.h"
#include "src/model/mistral/modules.h"
#include "src/tokenizer/tokenizer.h"

// main.cpp:10-21, linked from the reference's main.cpp (main renamed).
uint32_t sample_max(InferenceState& infer);
// main.cpp:23-43 and the generator it draws from (main.cpp:6-8).
uint32_t sample_multinomial(InferenceState& infer, float temp);
extern std::mt19937 gen;

namespace {

struct Session {
    std::shared_ptr<Parameters> params;
    std::unique_ptr<InferenceState> infer;
    std::unique_ptr<Model<int8_t>> model_i8;
    std::unique_ptr<Model<float>> model_f32;
    size_t max_seq = 0;
};

// Parameters::load_parameters (parameters.cpp:95-129) minus the file I/O:
// the same header parse and the same public load_config / Tokenizer::load /
// load_weights calls, pointed at a caller-owned buffer in the same layout.
bool load_from_buffer(Parameters& p, const char* buf, size_t size) {
    if (size < 8) return false;
    uint64_t header_size;
    std::memcpy(&header_size, buf, sizeof(header_size));
    if (header_size + 8 > size) return false;
    nlohmann::json header_json = nlohmann::json::parse(std::string(buf + 8, header_size));
    p.load_config(header_json);
    p.tokenizer.load(header_json["tokenizer"]);
    char* start = const_cast<char*>(buf) + header_size + sizeof(uint64_t);
    p.load_weights(start, header_json);
    return true;
}

Session* finish(std::shared_ptr<Parameters> params, size_t max_seq) {
    auto* s = new Session();
    s->params = std::move(params);
    s->max_seq = max_seq;
    MAX_SEQ_LEN = max_seq;  // inference_state.h:5, read by the constructor
    s->infer.reset(new InferenceState(s->params->config));
    RotaryEmbedding::init_freq(*s->infer, s->params->config);
    if (s->params->config.quant == "int8")
        s->model_i8.reset(new Model<int8_t>(s->params));
    else
        s->model_f32.reset(new Model<float>(s->params));
    return s;
}

template <typename T>
Tensor<T> view(T* p, std::vector<size_t> shape) { return Tensor<T>(p, shape); }

}  // namespace

extern "C" {

__attribute__((visibility("default"))) void* ref_load_file(const char* path, size_t max_seq) {
    auto params = std::make_shared<Parameters>();
    params->load_parameters(path);
    return finish(params, max_seq);
}

__attribute__((visibility("default"))) void* ref_load_buffer(const char* buf, size_t size,
                                                             size_t max_seq) {
    auto params = std::make_shared<Parameters>();
    if (!load_from_buffer(*params, buf, size)) return nullptr;
    return finish(params, max_seq);
}

__attribute__((visibility("default"))) void ref_free(void* h) { delete static_cast<Session*>(h); }

__attribute__((visibility("default"))) void ref_config(void* h, size_t* out9, float* outf2) {
    const Config& c = static_cast<Session*>(h)->params->config;
    out9[0] = c.hidden_size; out9[1] = c.intermediate_size; out9[2] = c.n_layers;
    out9[3] = c.n_heads; out9[4] = c.n_kv_heads; out9[5] = c.vocab_size;
    out9[6] = c.head_dim; out9[7] = c.sliding_window; out9[8] = c.max_position_embeddings;
    outf2[0] = c.rope_theta; outf2[1] = c.norm_eps;
}

// Model<T>::forward (modules.cpp:154-171).  Returns 1 instead of overrunning
// the KV cache.
__attribute__((visibility("default"))) int ref_forward(void* h, uint32_t token) {
    auto* s = static_cast<Session*>(h);
    if (s->infer->pos >= s->max_seq || token >= s->params->config.vocab_size) return 1;
    if (s->model_i8) s->model_i8->forward(*s->infer, token);
    else s->model_f32->forward(*s->infer, token);
    return 0;
}

__attribute__((visibility("default"))) const float* ref_logits(void* h) {
    return static_cast<Session*>(h)->infer->logits.data;
}
__attribute__((visibility("default"))) const float* ref_hidden(void* h) {
    return static_cast<Session*>(h)->infer->hidden_state.data;
}
__attribute__((visibility("default"))) uint32_t ref_sample_max(void* h) {
    return sample_max(*static_cast<Session*>(h)->infer);
}
// sample_multinomial (main.cpp:23-43) on the given logits (vocab_size of
// them, copied into infer.logits, which the call then divides by temp), with
// the generator seeded by `seed`; *r_out = the uniform draw the call takes
// (the same distribution applied to a copy of the seeded generator).
__attribute__((visibility("default"))) uint32_t ref_sample_logits(void* h, const float* logits, float temp,
                                                                  uint32_t seed, float* r_out) {
    auto* s = static_cast<Session*>(h);
    std::memcpy(s->infer->logits.data, logits, s->infer->logits.numel * sizeof(float));
    gen.seed(seed);
    std::mt19937 peek = gen;
    std::uniform_real_distribution<double> d(0.0, 1.0);
    *r_out = static_cast<float>(d(peek));
    return sample_multinomial(*s->infer, temp);
}
// Tokenizer::load (tokenizer.cpp:37-68) on a tokenizer object's JSON text;
// null if the JSON does not parse.
__attribute__((visibility("default"))) void* ref_tokenizer_new(const char* json, size_t len) {
    try {
        auto* t = new Tokenizer();
        t->load(nlohmann::json::parse(std::string(json, len)));
        return t;
    } catch (...) {
        return nullptr;
    }
}
__attribute__((visibility("default"))) void ref_tokenizer_free(void* t) { delete static_cast<Tokenizer*>(t); }
// Tokenizer::encode (tokenizer.cpp:121-177): the id count; the first `cap` ids to `ids`.
__attribute__((visibility("default"))) size_t ref_tokenizer_encode(void* t, const char* text, size_t len,
                                                                    uint32_t* ids, size_t cap) {
    const std::vector<uint32_t> v = static_cast<Tokenizer*>(t)->encode(std::string(text, len));
    std::memcpy(ids, v.data(), std::min(cap, v.size()) * sizeof(uint32_t));
    return v.size();
}
// Tokenizer::decode (tokenizer.cpp:203-209): the byte count; the first `cap` bytes to `out`.
__attribute__((visibility("default"))) size_t ref_tokenizer_decode(void* t, const uint32_t* ids, size_t n, char* out,
                                                                    size_t cap) {
    const std::string s = static_cast<Tokenizer*>(t)->decode(std::vector<uint32_t>(ids, ids + n));
    std::memcpy(out, s.data(), std::min(cap, s.size()));
    return s.size();
}
__attribute__((visibility("default"))) size_t ref_pos(void* h) {
    return static_cast<Session*>(h)->infer->pos;
}
__attribute__((visibility("default"))) void ref_set_pos(void* h, size_t pos) {
    static_cast<Session*>(h)->infer->pos = pos;
}

// Layer<T>::forward (modules.cpp:118-143) on a caller-provided hidden state
// (the pattern of test_modules.cpp:3-24).  h is read and written in place.
__attribute__((visibility("default"))) int ref_layer_forward(void* hs, int layer, float* h) {
    auto* s = static_cast<Session*>(hs);
    if (s->infer->pos >= s->max_seq) return 1;
    auto& hid = s->infer->hidden_state;
    std::memcpy(hid.data, h, hid.numel * sizeof(float));
    if (s->model_i8) s->model_i8->layers.at(layer).forward(*s->infer);
    else s->model_f32->layers.at(layer).forward(*s->infer);
    std::memcpy(h, hid.data, hid.numel * sizeof(float));
    return 0;
}

// Timing helper for the CPU baseline: one decode token through the
// reference's own modules, running `n_run` of the layers (first, first+1,
// ...) and returning seconds for {embedding, layers, final norm + lm_head}.
__attribute__((visibility("default"))) int ref_time_token(void* hs, uint32_t token, int first,
                                                          int n_run, double* out3) {
    auto* s = static_cast<Session*>(hs);
    if (!s->model_i8 || s->infer->pos >= s->max_seq) return 1;
    auto& m = *s->model_i8;
    auto& inf = *s->infer;
    using clk = std::chrono::steady_clock;
    auto t0 = clk::now();
    m.embedding.forward(inf, token);
    auto t1 = clk::now();
    const int L = static_cast<int>(m.layers.size());
    for (int i = 0; i < n_run; i++) m.layers.at((first + i) % L).forward(inf);
    auto t2 = clk::now();
    m.norm.forward(inf);
    m.lmHead.forward(inf);
    (void)sample_max(inf);
    auto t3 = clk::now();
    out3[0] = std::chrono::duration<double>(t1 - t0).count();
    out3[1] = std::chrono::duration<double>(t2 - t1).count();
    out3[2] = std::chrono::duration<double>(t3 - t2).count();
    return 0;
}

// ---- op-level wrappers over src/common/kernels.h (views, no copies) ----

__attribute__((visibility("default"))) void ref_matmul_i8(float* xout, int8_t* w, const float* scales,
                                                          size_t n_scales, float* x, size_t n,
                                                          size_t d) {
    Tensor<int8_t> W(w, std::vector<float>(scales, scales + n_scales), {n, d});
    auto X = view(x, {d});
    auto Y = view(xout, {n});
    matmul(Y, W, X);
}
__attribute__((visibility("default"))) void ref_matmul_f32(float* xout, float* w, float* x, size_t n,
                                                           size_t d) {
    auto W = view(w, {n, d});
    auto X = view(x, {d});
    auto Y = view(xout, {n});
    matmul(Y, W, X);
}
__attribute__((visibility("default"))) void ref_row_matmul(float* xout, float* x, float* w, size_t n,
                                                           size_t d) {
    auto W = view(w, {n, d});
    auto X = view(x, {n});
    auto Y = view(xout, {d});
    row_matmul(Y, X, W);
}
__attribute__((visibility("default"))) void ref_softmax(float* xout, float* x, size_t n) {
    auto X = view(x, {n});
    auto Y = view(xout, {n});
    softmax(Y, X);
}
__attribute__((visibility("default"))) void ref_rope(float* xout, float* x, float* c, float* s,
                                                     size_t n_heads, size_t head_dim) {
    auto X = view(x, {n_heads, head_dim});
    auto Y = view(xout, {n_heads, head_dim});
    auto C = view(c, {head_dim});
    auto S = view(s, {head_dim});
    rope(Y, X, C, S);
}
__attribute__((visibility("default"))) void ref_silu(float* xout, float* x, size_t n) {
    auto X = view(x, {n});
    auto Y = view(xout, {n});
    silu(Y, X);
}
__attribute__((visibility("default"))) void ref_rmsnorm(void* hs, float* x, float* g) {
    auto* s = static_cast<Session*>(hs);
    auto& hid = s->infer->hidden_state;
    std::memcpy(hid.data, x, hid.numel * sizeof(float));
    RMSNorm norm(view(g, {hid.numel}));
    norm.forward(*s->infer);
    std::memcpy(x, hid.data, hid.numel * sizeof(float));
}
__attribute__((visibility("default"))) void ref_rotary(void* hs, size_t pos, float* inv_freq,
                                                       float* cos_out, float* sin_out) {
    auto* s = static_cast<Session*>(hs);
    auto& inf = *s->infer;
    const size_t saved = inf.pos;
    inf.pos = pos;
    RotaryEmbedding::forward(inf);
    inf.pos = saved;
    std::memcpy(inv_freq, inf.inv_freq.data, inf.inv_freq.numel * sizeof(float));
    std::memcpy(cos_out, inf.cos.data, inf.cos.numel * sizeof(float));
    std::memcpy(sin_out, inf.sin.data, inf.sin.numel * sizeof(float));
}

}  // extern "C"
