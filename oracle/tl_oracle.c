/*
 * tl_oracle.c -- CPU restatement of the torchless int8 Mistral hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * path in torchless_b200/csrc.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline leg of bench.py may load it.  It is never part of the product
 * path, and the product never falls back to it.
 *
 * Every function restates one reference function operation by operation
 * (same operand order, same sequential fp32 accumulation, same divide-based
 * int8 dequantisation), so results are bit-identical to the reference CPU
 * backend built without FMA contraction (-O3 -DNDEBUG, no -march).  That
 * claim is checked against the reference compiled from its own sources
 * (oracle/_ref, see oracle/Makefile) in tests/test_oracle_pins.py.
 *
 * Build: gcc -std=c11 -O2 -ffp-contract=off -fno-fast-math -fopenmp -fPIC
 * (no -march: the reference's x86-64 baseline build has no FMA either).
 * OpenMP only parallelises across independent output rows; each row keeps
 * the reference's sequential order, so threading cannot change a bit.
 *
 * Reference file paths are relative to the ryansenn/torchless tree.
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define TLO_API __attribute__((visibility("default")))

/* ------------------------------------------------------------------------ */
/* Backend ops: src/backend/cpu/kernels.cpp, declared in src/common/kernels.h */
/* ------------------------------------------------------------------------ */

/* kernels.cpp:6-19  W (n,d) @ x (d,) -> xout (n,), sequential j per row. */
TLO_API void tlo_matmul_f32(float* xout, const float* w, const float* x,
                            size_t n, size_t d) {
    long long nn = (long long)n;
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < nn; i++) {
        const float* row = w + (size_t)i * d;
        float acc = 0.0f;
        for (size_t j = 0; j < d; j++) acc += row[j] * x[j];
        xout[i] = acc;
    }
}

/* kernels.cpp:21-33 with Tensor<int8_t>::get (tensor.cpp:101-104):
 *   get(i) = data[i] / scales[scales.size() * i / numel]
 * i.e. int8 -> fp32, divided by the stored scale (scale = 127/absmax),
 * then multiplied by x[j] and added to the running fp32 sum. */
TLO_API void tlo_matmul_i8(float* xout, const int8_t* w, const float* scales,
                           size_t n_scales, const float* x, size_t n, size_t d) {
    const size_t numel = n * d;
    long long nn = (long long)n;
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < nn; i++) {
        const size_t base = (size_t)i * d;
        float acc = 0.0f;
        for (size_t j = 0; j < d; j++) {
            const size_t e = base + j;
            const float wv = (float)w[e] / scales[n_scales * e / numel];
            acc += wv * x[j];
        }
        xout[i] = acc;
    }
}

/* fp8 export (format extension after the roadmap item README.md:160, "a cast
 * tensor.to(torch.float8_e5m2) during model export"): an e5m2 byte is sign,
 * 5 exponent bits (bias 15) and 2 mantissa bits; exponent 0 is subnormal
 * (m * 2^-16), exponent 31 is infinity (m = 0) or NaN.  Exact in fp32. */
TLO_API float tlo_fp8_to_f32(uint8_t b) {
    const int sign = b >> 7, e = (b >> 2) & 31, m = b & 3;
    float v;
    if (e == 31) v = m ? NAN : INFINITY;
    else if (e == 0) v = ldexpf((float)m, -16);
    else v = ldexpf((float)(4 + m), e - 17);
    return sign ? -v : v;
}

/* kernels.cpp:21-33 with the weight's get(i) = the e5m2 value of byte i:
 * converted to fp32, multiplied by x[j], added to the running fp32 sum. */
TLO_API void tlo_matmul_f8(float* xout, const uint8_t* w, const float* x, size_t n, size_t d) {
    long long nn = (long long)n;
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < nn; i++) {
        const uint8_t* row = w + (size_t)i * d;
        float acc = 0.0f;
        for (size_t j = 0; j < d; j++) acc += tlo_fp8_to_f32(row[j]) * x[j];
        xout[i] = acc;
    }
}

/* kernels.cpp:37-49  x (n,) @ W (n,d) -> xout (d,), sequential j. */
TLO_API void tlo_row_matmul(float* xout, const float* x, const float* w,
                            size_t n, size_t d) {
    for (size_t i = 0; i < d; i++) {
        float acc = 0.0f;
        for (size_t j = 0; j < n; j++) acc += w[j * d + i] * x[j];
        xout[i] = acc;
    }
}

/* Tensor<float>::max (tensor.cpp:71-78): std::max keeps the left operand
 * unless the right one is strictly greater. */
static float tlo_max(const float* x, size_t n) {
    float r = x[0];
    for (size_t i = 0; i < n; i++) r = (r < x[i]) ? x[i] : r;
    return r;
}

/* kernels.cpp:133-137 mul(xout, x, c). */
TLO_API void tlo_mul_scalar(float* xout, const float* x, float c, size_t n) {
    for (size_t i = 0; i < n; i++) xout[i] = x[i] * c;
}

/* kernels.cpp:55-63  exp(x - max), sequential total, then mul by 1/total. */
TLO_API void tlo_softmax(float* xout, const float* x, size_t n) {
    const float maxv = tlo_max(x, n);
    float total = 0.0f;
    for (size_t i = 0; i < n; i++) {
        xout[i] = expf(x[i] - maxv);
        total += xout[i];
    }
    tlo_mul_scalar(xout, xout, 1.0f / total, n);
}

/* kernels.cpp:78-95  half-split rotation of each head: (i, i+head_dim/2),
 * one cos/sin row shared by every head.  In place is allowed (xout == x). */
TLO_API void tlo_rope(float* xout, const float* x, const float* cosv,
                      const float* sinv, size_t n_heads, size_t head_dim) {
    const size_t half = head_dim / 2;
    for (size_t h = 0; h < n_heads; h++) {
        const size_t start = h * head_dim;
        for (size_t i = start; i < start + half; i++) {
            const float xi = x[i];
            const float yi = x[i + half];
            const float c = cosv[i - start];
            const float s = sinv[i - start];
            xout[i] = xi * c - yi * s;
            xout[i + half] = xi * s + yi * c;
        }
    }
}

/* kernels.cpp:98-102  x / (1 + exp(-x)). */
TLO_API void tlo_silu(float* xout, const float* x, size_t n) {
    for (size_t i = 0; i < n; i++) xout[i] = x[i] / (1.0f + expf(-x[i]));
}

/* kernels.cpp:106-112 */
TLO_API float tlo_sum(const float* x, size_t n) {
    float r = 0.0f;
    for (size_t i = 0; i < n; i++) r += x[i];
    return r;
}

/* kernels.cpp:114-119 */
TLO_API void tlo_add(float* xout, const float* x, const float* y, size_t n) {
    for (size_t i = 0; i < n; i++) xout[i] = x[i] + y[i];
}

/* kernels.cpp:122-125 */
TLO_API void tlo_add_scalar(float* xout, const float* x, float c, size_t n) {
    for (size_t i = 0; i < n; i++) xout[i] = x[i] + c;
}

/* kernels.cpp:127-131 */
TLO_API void tlo_mul(float* xout, const float* x, const float* y, size_t n) {
    for (size_t i = 0; i < n; i++) xout[i] = x[i] * y[i];
}

/* kernels.cpp:139-143: std::pow(float, int) promotes to double in C++11 and
 * the double result is stored back into a float. */
TLO_API void tlo_pow(float* xout, const float* x, int e, size_t n) {
    for (size_t i = 0; i < n; i++) xout[i] = (float)pow((double)x[i], (double)e);
}

/* kernels.cpp:145-149 */
TLO_API void tlo_sqrt(float* xout, const float* x, size_t n) {
    for (size_t i = 0; i < n; i++) xout[i] = sqrtf(x[i]);
}

/* ------------------------------------------------------------------------ */
/* Modules: src/model/mistral/modules.cpp                                    */
/* ------------------------------------------------------------------------ */

/* RMSNorm::forward (modules.cpp:31-46), in place on h[n].  The reference
 * hard-codes e = 1e-5f (modules.h:24) and ignores config.norm_eps.
 *   rms = sqrt(sum(h^2)/n + e); h *= 1/rms; h *= g  */
TLO_API void tlo_rmsnorm(float* h, const float* g, size_t n, float eps) {
    float squares = 0.0f;
    for (size_t i = 0; i < n; i++) squares += h[i] * h[i];
    const float rms = (float)sqrt((double)(squares / (float)n + eps));
    tlo_mul_scalar(h, h, 1.0f / rms, n);
    for (size_t i = 0; i < n; i++) h[i] = h[i] * g[i];
}

/* RotaryEmbedding::init_freq (modules.cpp:12-17):
 *   inv_freq[i] = 1 / powf(theta, i / n)  with n = head_dim/2 */
TLO_API void tlo_init_freq(float* inv_freq, size_t n, float theta) {
    for (size_t i = 0; i < n; i++)
        inv_freq[i] = 1.0f / powf(theta, (float)i / (float)n);
}

/* RotaryEmbedding::forward (modules.cpp:22-27):
 *   cos[i] = cosf(inv_freq[i % nf] * (float)pos), same for sin, i < head_dim */
TLO_API void tlo_rope_cos_sin(float* cosv, float* sinv, const float* inv_freq,
                              size_t n_freq, size_t head_dim, size_t pos) {
    for (size_t i = 0; i < head_dim; i++) {
        const float a = inv_freq[i % n_freq] * (float)pos;
        cosv[i] = cosf(a);
        sinv[i] = sinf(a);
    }
}

/* sample_max (main.cpp:10-21): first index holding the strict maximum,
 * starting from logits[0]. */
TLO_API uint32_t tlo_argmax(const float* logits, size_t n) {
    float max_val = logits[0];
    size_t res = 0;
    for (size_t i = 0; i < n; i++) {
        if (logits[i] > max_val) {
            res = i;
            max_val = logits[i];
        }
    }
    return (uint32_t)res;
}

/* sample_multinomial (main.cpp:23-43) with its uniform draw r supplied by the
 * caller (the reference draws r = (float)distr(gen), a uniform double in
 * [0, 1) from a global mt19937).  temp <= 0: sample_max.  temp > 0: every
 * logit divided by temp (the reference divides infer.logits in place; here a
 * copy is scaled), softmax (kernels.cpp:55-63), then the first index whose
 * running fp32 sum of probabilities reaches r; none: the last index. */
TLO_API uint32_t tlo_sample_multinomial(const float* logits, size_t n, float temp, float r) {
    if (!(temp > 0)) return tlo_argmax(logits, n);
    float* x = (float*)malloc(n * sizeof(float));
    float* p = (float*)malloc(n * sizeof(float));
    if (!x || !p) {
        free(x);
        free(p);
        return (uint32_t)(n - 1);
    }
    for (size_t i = 0; i < n; i++) x[i] = logits[i] / temp;
    tlo_softmax(p, x, n);
    float total = 0.0f;
    uint32_t res = (uint32_t)(n - 1);
    for (size_t i = 0; i < n; i++) {
        total += p[i];
        if (total >= r) {
            res = (uint32_t)i;
            break;
        }
    }
    free(x);
    free(p);
    return res;
}

/* The uniform draw of the library's device-side sampling for (seed, pos): the
 * splitmix64 finaliser of seed + (pos + 1) * 0x9E3779B97F4A7C15, top 24 bits
 * scaled by 2^-24 (exact in float, in [0, 1)).  Not the reference's draw
 * (an unseeded mt19937); a fixed function so that runs are reproducible. */
TLO_API float tlo_sample_uniform(uint64_t seed, uint64_t pos) {
    uint64_t z = seed + (pos + 1) * 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    z ^= z >> 31;
    return (float)(z >> 40) * (1.0f / 16777216.0f);
}

/* quantize (export_mistral.py:53-68) on fp32 input, torch CPU semantics:
 *   scale = 127 / max|x| over each group; torch evaluates int / tensor as
 *           reciprocal(tensor) * int, i.e. fl(fl(1/max) * 127)
 *   q     = round_half_even(x * scale) stored as int8 */
TLO_API void tlo_quantize(int8_t* q, float* scales, const float* x,
                          size_t numel, size_t group) {
    const size_t ng = numel / group;
    for (size_t g = 0; g < ng; g++) {
        const float* xs = x + g * group;
        float amax = 0.0f;
        for (size_t j = 0; j < group; j++) {
            const float a = fabsf(xs[j]);
            amax = (a > amax) ? a : amax;
        }
        const float r = 1.0f / amax;
        const float s = r * 127.0f;
        scales[g] = s;
        for (size_t j = 0; j < group; j++) q[g * group + j] = (int8_t)(int)rintf(xs[j] * s);
    }
}

/* ------------------------------------------------------------------------ */
/* Whole model: Model<T>::forward (modules.cpp:154-171) over InferenceState  */
/* (src/model/mistral/inference_state.h).                                    */
/* ------------------------------------------------------------------------ */

typedef struct {
    size_t hidden, inter, n_layers, n_heads, n_kv_heads, vocab, head_dim, max_seq;
    float rope_theta;
    /* 0: every cached position (the reference).  W > 0: sliding-window
     * attention over the last W positions (HF Mistral's sliding_window; the
     * reference parses it, parameters.cpp:41, and never uses it). */
    size_t window;
} tlo_config;

/* Tensor kinds, mirroring the names the reference looks up with
 * Parameters::get_tensor (modules.h:77-102). */
enum {
    TLO_EMBED = 0,     /* model.embed_tokens.weight            (global) */
    TLO_NORM = 1,      /* model.norm.weight                    (global) */
    TLO_LM_HEAD = 2,   /* lm_head.weight                       (global) */
    TLO_IN_NORM = 3,   /* input_layernorm.weight               (layer)  */
    TLO_POST_NORM = 4, /* post_attention_layernorm.weight      (layer)  */
    TLO_WQ = 5,        /* self_attn.q_proj.weight */
    TLO_WK = 6,        /* self_attn.k_proj.weight */
    TLO_WV = 7,        /* self_attn.v_proj.weight */
    TLO_WO = 8,        /* self_attn.o_proj.weight */
    TLO_W1 = 9,        /* mlp.gate_proj.weight */
    TLO_W2 = 10,       /* mlp.down_proj.weight */
    TLO_W3 = 11,       /* mlp.up_proj.weight */
    TLO_N_KINDS = 12
};

typedef struct {
    const void* data;      /* int8 when scales != NULL, e5m2 bytes when fp8, else fp32 */
    const float* scales;
    size_t n_scales;
    size_t rows, cols;
    int fp8;
} tlo_weight;

typedef struct {
    tlo_config c;
    tlo_weight global[3];
    tlo_weight* layer; /* [n_layers][TLO_N_KINDS] */
    float *kc, *vc;    /* [n_layers][n_kv_heads][max_seq][head_dim] */
    float *h, *residual, *q, *k, *v, *scores, *ctx, *gate, *up, *logits;
    float *inv_freq, *cosv, *sinv;
    size_t pos;
} tlo_model;

TLO_API tlo_model* tlo_model_new(const tlo_config* cfg) {
    tlo_model* m = (tlo_model*)calloc(1, sizeof(tlo_model));
    if (!m) return NULL;
    m->c = *cfg;
    const tlo_config* c = &m->c;
    m->layer = (tlo_weight*)calloc(c->n_layers * TLO_N_KINDS, sizeof(tlo_weight));
    const size_t kv = c->n_layers * c->n_kv_heads * c->max_seq * c->head_dim;
    m->kc = (float*)calloc(kv, sizeof(float));
    m->vc = (float*)calloc(kv, sizeof(float));
    m->h = (float*)calloc(c->hidden, sizeof(float));
    m->residual = (float*)calloc(c->hidden, sizeof(float));
    m->q = (float*)calloc(c->n_heads * c->head_dim, sizeof(float));
    m->k = (float*)calloc(c->n_kv_heads * c->head_dim, sizeof(float));
    m->v = (float*)calloc(c->n_kv_heads * c->head_dim, sizeof(float));
    m->scores = (float*)calloc(c->n_heads * c->max_seq, sizeof(float));
    m->ctx = (float*)calloc(c->n_heads * c->head_dim, sizeof(float));
    m->gate = (float*)calloc(c->inter, sizeof(float));
    m->up = (float*)calloc(c->inter, sizeof(float));
    m->logits = (float*)calloc(c->vocab, sizeof(float));
    m->inv_freq = (float*)calloc(c->head_dim / 2, sizeof(float));
    m->cosv = (float*)calloc(c->head_dim, sizeof(float));
    m->sinv = (float*)calloc(c->head_dim, sizeof(float));
    if (!m->layer || !m->kc || !m->vc || !m->h || !m->residual || !m->q || !m->k ||
        !m->v || !m->scores || !m->ctx || !m->gate || !m->up || !m->logits ||
        !m->inv_freq || !m->cosv || !m->sinv) {
        return NULL; /* test tooling: leak on OOM is acceptable */
    }
    /* The reference CLI never calls init_freq (main.cpp), the tests do
     * (test_modules.cpp:169); the oracle always does. */
    tlo_init_freq(m->inv_freq, c->head_dim / 2, c->rope_theta);
    return m;
}

TLO_API void tlo_model_free(tlo_model* m) {
    if (!m) return;
    free(m->layer); free(m->kc); free(m->vc); free(m->h); free(m->residual);
    free(m->q); free(m->k); free(m->v); free(m->scores); free(m->ctx);
    free(m->gate); free(m->up); free(m->logits); free(m->inv_freq);
    free(m->cosv); free(m->sinv); free(m);
}

/* layer < 0 selects a global tensor (Parameters::get_tensor, layer -1). */
TLO_API int tlo_model_set_tensor(tlo_model* m, int layer, int kind, const void* data,
                                 const float* scales, size_t n_scales, size_t rows,
                                 size_t cols) {
    tlo_weight w = {data, scales, n_scales, rows, cols, 0};
    if (layer < 0) {
        if (kind < 0 || kind > TLO_LM_HEAD) return 1;
        m->global[kind] = w;
        return 0;
    }
    if ((size_t)layer >= m->c.n_layers || kind < TLO_IN_NORM || kind >= TLO_N_KINDS) return 1;
    m->layer[(size_t)layer * TLO_N_KINDS + kind] = w;
    return 0;
}

/* An fp8 (e5m2) projection or lm_head: no scales. */
TLO_API int tlo_model_set_tensor_fp8(tlo_model* m, int layer, int kind, const uint8_t* data, size_t rows,
                                     size_t cols) {
    if (layer < 0 ? kind != TLO_LM_HEAD : kind < TLO_WQ) return 1;
    const int rc = tlo_model_set_tensor(m, layer, kind, data, NULL, 0, rows, cols);
    if (rc) return rc;
    if (layer < 0) m->global[kind].fp8 = 1;
    else m->layer[(size_t)layer * TLO_N_KINDS + kind].fp8 = 1;
    return 0;
}

TLO_API size_t tlo_model_pos(const tlo_model* m) { return m->pos; }
TLO_API void tlo_model_set_pos(tlo_model* m, size_t pos) { m->pos = pos; }
TLO_API float* tlo_model_logits(tlo_model* m) { return m->logits; }
TLO_API float* tlo_model_hidden(tlo_model* m) { return m->h; }
TLO_API float* tlo_model_k_cache(tlo_model* m) { return m->kc; }
TLO_API float* tlo_model_v_cache(tlo_model* m) { return m->vc; }

/* Dispatch on the stored dtype like matmul(Tensor<T>...) overloads. */
static void tlo_linear(float* y, const tlo_weight* w, const float* x) {
    if (w->fp8)
        tlo_matmul_f8(y, (const uint8_t*)w->data, x, w->rows, w->cols);
    else if (w->scales)
        tlo_matmul_i8(y, (const int8_t*)w->data, w->scales, w->n_scales, x, w->rows, w->cols);
    else
        tlo_matmul_f32(y, (const float*)w->data, x, w->rows, w->cols);
}

/* Attention<T>::forward (modules.cpp:49-92). */
static void tlo_attention(tlo_model* m, size_t l) {
    const tlo_config* c = &m->c;
    const tlo_weight* W = &m->layer[l * TLO_N_KINDS];
    const size_t hd = c->head_dim;
    tlo_linear(m->q, &W[TLO_WQ], m->h);
    tlo_linear(m->k, &W[TLO_WK], m->h);
    tlo_linear(m->v, &W[TLO_WV], m->h);
    tlo_rope_cos_sin(m->cosv, m->sinv, m->inv_freq, hd / 2, hd, m->pos);
    tlo_rope(m->q, m->q, m->cosv, m->sinv, c->n_heads, hd);
    tlo_rope(m->k, m->k, m->cosv, m->sinv, c->n_kv_heads, hd);
    /* InferenceState::push_kv (inference_state.h:38-43) */
    for (size_t kh = 0; kh < c->n_kv_heads; kh++) {
        const size_t off = ((l * c->n_kv_heads + kh) * c->max_seq + m->pos) * hd;
        memcpy(m->kc + off, m->k + kh * hd, hd * sizeof(float));
        memcpy(m->vc + off, m->v + kh * hd, hd * sizeof(float));
    }
    /* 1/sqrt(head_dim) is evaluated in double and passed as a float. */
    const float scale = (float)(1.0 / sqrt((double)hd));
    const size_t npos = m->pos + 1;
    const size_t lo = (c->window > 0 && npos > c->window) ? npos - c->window : 0;
    const size_t span = npos - lo; /* positions lo .. pos */
    for (size_t h = 0; h < c->n_heads; h++) {
        const size_t kh = h / 4; /* hard-coded GQA ratio, modules.cpp:70-71 */
        const float* kcache = m->kc + ((l * c->n_kv_heads + kh) * c->max_seq + lo) * hd;
        const float* vcache = m->vc + ((l * c->n_kv_heads + kh) * c->max_seq + lo) * hd;
        float* sc = m->scores + h * c->max_seq;
        tlo_matmul_f32(sc, kcache, m->q + h * hd, span, hd);
        tlo_mul_scalar(sc, sc, scale, span);
        tlo_softmax(sc, sc, span);
        tlo_row_matmul(m->ctx + h * hd, sc, vcache, span, hd);
    }
    tlo_linear(m->h, &W[TLO_WO], m->ctx);
}

/* MLP<T>::forward (modules.cpp:99-115). */
static void tlo_mlp(tlo_model* m, size_t l) {
    const tlo_config* c = &m->c;
    const tlo_weight* W = &m->layer[l * TLO_N_KINDS];
    tlo_linear(m->gate, &W[TLO_W1], m->h);
    tlo_silu(m->gate, m->gate, c->inter);
    tlo_linear(m->up, &W[TLO_W3], m->h);
    tlo_mul(m->gate, m->gate, m->up, c->inter);
    tlo_linear(m->h, &W[TLO_W2], m->gate);
}

/* Layer<T>::forward (modules.cpp:118-143) on the current hidden state. */
TLO_API int tlo_model_layer_forward(tlo_model* m, size_t l) {
    const tlo_config* c = &m->c;
    if (l >= c->n_layers || m->pos >= c->max_seq) return 1;
    const tlo_weight* W = &m->layer[l * TLO_N_KINDS];
    memcpy(m->residual, m->h, c->hidden * sizeof(float));
    tlo_rmsnorm(m->h, (const float*)W[TLO_IN_NORM].data, c->hidden, 1e-5f);
    tlo_attention(m, l);
    tlo_add(m->h, m->h, m->residual, c->hidden);
    memcpy(m->residual, m->h, c->hidden * sizeof(float));
    tlo_rmsnorm(m->h, (const float*)W[TLO_POST_NORM].data, c->hidden, 1e-5f);
    tlo_mlp(m, l);
    tlo_add(m->h, m->h, m->residual, c->hidden);
    return 0;
}

/* Model<T>::forward (modules.cpp:154-171): embedding row copy, every layer,
 * final norm, fp32 lm_head, pos++.  Returns nonzero when pos would overrun
 * the KV cache (the reference overruns silently under NDEBUG). */
TLO_API int tlo_model_forward(tlo_model* m, uint32_t token) {
    const tlo_config* c = &m->c;
    if (m->pos >= c->max_seq || token >= c->vocab) return 1;
    memcpy(m->h, (const float*)m->global[TLO_EMBED].data + (size_t)token * c->hidden,
           c->hidden * sizeof(float));
    for (size_t l = 0; l < c->n_layers; l++) tlo_model_layer_forward(m, l);
    tlo_rmsnorm(m->h, (const float*)m->global[TLO_NORM].data, c->hidden, 1e-5f);
    tlo_linear(m->logits, &m->global[TLO_LM_HEAD], m->h);
    m->pos++;
    return 0;
}
