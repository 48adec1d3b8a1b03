/*
 * torchless_b200.h -- C ABI of the B200 (sm_100a) torchless hot path.
 *
 * Drop-in boundary for the reference's CPU backend (ryansenn/torchless).
 * Every entry point cites the reference function it replaces.  Conventions:
 *
 *   - Output first, like the reference (src/common/kernels.h:11-29).
 *   - Op-level entry points take DEVICE pointers and a cudaStream_t passed as
 *     void* (NULL = the legacy default stream).  They are asynchronous.
 *     In-place use (xout == x) is allowed wherever the reference allows it
 *     (modules.cpp:61-62, 81, 105, 111).
 *   - Model-level entry points take HOST buffers and are synchronous.
 *   - Every call returns tl_status; nothing exits or aborts.  The reference
 *     asserts (compiled out under NDEBUG) or calls std::exit(1)
 *     (src/loader/parameters.cpp:13-26, 99-102); here the same conditions
 *     return TL_ERR_* and tl_last_error() holds the message.
 *   - Pointer/size arguments are plain C types; no torch types cross this ABI.
 */
#ifndef TORCHLESS_B200_H
#define TORCHLESS_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TL_API __attribute__((visibility("default")))

typedef enum tl_status {
    TL_OK = 0,
    TL_ERR_INVALID_ARGUMENT = 1, /* shape/pointer checks (reference: assert)            */
    TL_ERR_UNSUPPORTED = 2,      /* valid for the reference, not built here             */
    TL_ERR_IO = 3,               /* open/stat/read/mmap failed (reference: std::exit)   */
    TL_ERR_FORMAT = 4,           /* malformed header or tensor table                    */
    TL_ERR_CUDA = 5,             /* CUDA runtime error                                  */
    TL_ERR_OUT_OF_MEMORY = 6,
    TL_ERR_CAPACITY = 7,         /* KV cache full (reference overruns silently)         */
    TL_ERR_TIMEOUT = 8           /* a bounded device-side wait gave up                  */
} tl_status;

/* Message for the last failing call on this host thread ("" if none). */
TL_API const char* tl_last_error(void);
TL_API const char* tl_status_name(tl_status s);

/* ------------------------------------------------------------------------ */
/* Op level: src/common/kernels.h (bodies in src/backend/cpu/kernels.cpp).   */
/* ------------------------------------------------------------------------ */

/* kernels.h:11  matmul(Tensor<float>& xout, Tensor<float>& w, Tensor<float>& x)
 * xout[n] = W[n,d] @ x[d], fp32 (kernels.cpp:6-19). */
TL_API tl_status tl_matmul_f32(float* xout, const float* w, const float* x, size_t n, size_t d,
                               void* stream);

/* kernels.h:12  matmul(Tensor<float>& xout, Tensor<int8_t>& w, Tensor<float>& x)
 * xout[i] = sum_j (w[i,j] / scales[n_scales*(i*d+j)/(n*d)]) * x[j]
 * (kernels.cpp:21-33 with Tensor<int8_t>::get, tensor.cpp:101-104).
 * `scales` are the stored export scales (127/absmax), n_scales of them. */
TL_API tl_status tl_matmul_i8(float* xout, const int8_t* w, const float* scales, size_t n_scales,
                              const float* x, size_t n, size_t d, void* stream);

/* matmul(xout, W, x) with fp8 weights (format extension after the roadmap
 * item README.md:160, "fp8 with a cast tensor.to(torch.float8_e5m2)"): W is
 * [n, d] e5m2 bytes, each weight the e5m2 value itself (no scales);
 * xout[n] = W @ x[d] with fp32 sums (kernels.cpp:21-33 with that get()). */
TL_API tl_status tl_matmul_f8(float* xout, const uint8_t* w, const float* x, size_t n, size_t d, void* stream);

/* kernels.h:13  row_matmul(xout, x, w): xout[d] = x[n] @ W[n,d] (kernels.cpp:37-49). */
TL_API tl_status tl_row_matmul(float* xout, const float* x, const float* w, size_t n, size_t d,
                               void* stream);

/* kernels.h:15  softmax(xout, x) over n elements (kernels.cpp:55-63). */
TL_API tl_status tl_softmax(float* xout, const float* x, size_t n, void* stream);

/* kernels.h:16  rope(xout, x, cos, sin): x is [n_heads, head_dim]; pairs
 * (i, i + head_dim/2) of every head rotate by cos/sin[i] (kernels.cpp:78-95). */
TL_API tl_status tl_rope(float* xout, const float* x, const float* cos_, const float* sin_,
                         size_t n_heads, size_t head_dim, void* stream);

/* kernels.h:18  silu(xout, x) = x / (1 + exp(-x)) (kernels.cpp:98-102). */
TL_API tl_status tl_silu(float* xout, const float* x, size_t n, void* stream);

/* kernels.h:20  float sum(x); the result is written to *out (device). */
TL_API tl_status tl_sum(float* out, const float* x, size_t n, void* stream);

/* kernels.h:22-23  add(xout, x, y) and add(xout, x, c). */
TL_API tl_status tl_add(float* xout, const float* x, const float* y, size_t n, void* stream);
TL_API tl_status tl_add_scalar(float* xout, const float* x, float c, size_t n, void* stream);

/* kernels.h:25-26  mul(xout, x, y) and mul(xout, x, c). */
TL_API tl_status tl_mul(float* xout, const float* x, const float* y, size_t n, void* stream);
TL_API tl_status tl_mul_scalar(float* xout, const float* x, float c, size_t n, void* stream);

/* kernels.h:28-29  pow(xout, x, e) and sqrt(xout, x). */
TL_API tl_status tl_pow(float* xout, const float* x, int e, size_t n, void* stream);
TL_API tl_status tl_sqrt(float* xout, const float* x, size_t n, void* stream);

/* ------------------------------------------------------------------------ */
/* Module level pieces (src/model/mistral/modules.cpp, main.cpp,             */
/* export_mistral.py), as device ops.                                        */
/* ------------------------------------------------------------------------ */

/* RMSNorm::forward (modules.cpp:31-46): xout = x * (1/sqrt(sum(x^2)/n + eps)) * g.
 * The reference hard-codes eps = 1e-5f (modules.h:24). */
TL_API tl_status tl_rmsnorm(float* xout, const float* x, const float* g, size_t n, float eps,
                            void* stream);

/* RotaryEmbedding::forward (modules.cpp:22-27): cos/sin[i] of inv_freq[i % n_freq] * pos
 * for i < head_dim.  inv_freq from RotaryEmbedding::init_freq (modules.cpp:12-17). */
TL_API tl_status tl_rotary(float* cos_, float* sin_, const float* inv_freq, size_t n_freq,
                           size_t head_dim, size_t pos, void* stream);

/* sample_max (main.cpp:10-21): index of the first strict maximum of logits[n],
 * written to *out (device).  Its per-block partials live in scratch that is
 * allocated and freed stream-ordered (cudaMallocAsync / cudaFreeAsync) on
 * `stream` by every call. */
TL_API tl_status tl_argmax(uint32_t* out, const float* logits, size_t n, void* stream);

/* tl_argmax without any device allocation.  No counterpart in the reference
 * (its sample_max, main.cpp:10-21, is a host loop with no scratch); it exists
 * for callers that cannot allocate device memory at call time, such as a
 * serving loop that has given all free HBM to its KV-cache pool, where a
 * per-call allocation could fail or wait mid-generation.  Same result as
 * tl_argmax.  The partials live in a fixed 4 KB file-scope device array (512
 * partials of 1024 logits), so n must be <= 524288; larger n returns
 * TL_ERR_CAPACITY.  The first call on a device looks up that array's address
 * (cudaGetSymbolAddress, with that device current) and caches it; make that
 * first call before any stream capture begins.  The cached address belongs
 * to the device's primary context and is never looked up again: a process
 * that destroys that context (cudaDeviceReset) must not call this entry point
 * on that device afterwards.  The array is shared by all calls on a device:
 * calls whose kernels overlap in time (other streams or host threads) race on
 * it and must be serialised by the caller. */
TL_API tl_status tl_argmax_noalloc(uint32_t* out, const float* logits, size_t n, void* stream);

/* sample_multinomial (main.cpp:23-43) on device logits[n]; *out (device) gets
 * the index.  temperature <= 0: sample_max (main.cpp:10-21).  temperature > 0:
 * softmax(logits / temperature) (kernels.cpp:55-63) and the first index whose
 * running sum of probabilities reaches r; n - 1 if none does, or if a scaled
 * logit is NaN or +inf, or all are -inf (the reference's NaN then reaches
 * every probability).  r in [0, 1) replaces the reference's draw from its
 * global mt19937 (main.cpp:6-8, 35), so a call is reproducible.  The sums
 * run in parallel (per-thread chunks, then across chunks in order): the index
 * can differ from the reference's only where r is within rounding of a
 * running-sum boundary.  One block; no allocation. */
TL_API tl_status tl_sample_multinomial(uint32_t* out, const float* logits, size_t n, float temperature, float r,
                                       void* stream);

/* The uniform draw that device-side sampling (tl_model_set_sampling) uses for
 * the token at position pos: the splitmix64 finaliser of
 * seed + (pos + 1) * 0x9E3779B97F4A7C15, top 24 bits times 2^-24. */
TL_API float tl_sample_uniform(uint64_t seed, uint64_t pos);

/* MLP<T>::forward first half (modules.cpp:99-112), fused:
 * out[i] = silu(W1[i,:] @ x) * (W3[i,:] @ x), int8 W1/W3 [n, d] with stored scales. */
TL_API tl_status tl_mlp_gate_up(float* out, const int8_t* w1, const float* s1, const int8_t* w3,
                                const float* s3, const float* x, size_t n, size_t d,
                                void* stream);

/* Tensor-core GEMM of the batched paths (prefill, batched decode): no
 * counterpart in the reference, which runs one token at a time through
 * matmul (kernels.cpp:21-33).  c = a[m, k] b[n, k]^T with fp16 a and b
 * (row-major, k contiguous; the weights dequantised from int8), fp32
 * accumulation on the sm_100a tensor cores (tcgen05).  epilogue 0: c fp32
 * [m, ldc] = result; 1: c fp32 += result; 2: b rows come in blocks of 256 =
 * [128 gate rows | 128 up rows] and c is fp16 [m, ldc] with column
 * 128 block + j = silu(gate_j) * up_j (modules.cpp:99-112).  k must be a
 * multiple of 64; device pointers 16-byte aligned. */
TL_API tl_status tl_gemm_f16(void* c, const void* a, const void* b, size_t m, size_t n, size_t k, size_t ldc,
                             int epilogue, void* stream);

/* tl_gemm_f16 with 8-bit weights, dequantised inside the GEMM (the batched
 * paths' form; no counterpart in the reference, see tl_gemm_f16): b is int8
 * [n, k] (row-major, k contiguous) with inv_scales_t = 1 / s of each 64-column
 * group transposed to [k / 64][n] fp32, and each weight enters the tensor
 * cores as fp16(q) * fp16(1 / s) rounded to fp16 (tensor.cpp:101-104's
 * dequantisation in fp16 arithmetic); with inv_scales_t NULL, b
 * holds e5m2 bytes, widened exactly.  epilogue 0 / 1 as tl_gemm_f16; 2
 * (SwiGLU): b / inv_scales_t are the gate rows [n / 2, k] and b2 /
 * inv_scales_t2 the up rows, c is fp16 [m, ldc] with column 128 block + j =
 * silu(gate_j) * up_j over blocks of 128 rows.  k % 64 == 0, n % 4 == 0
 * (SwiGLU: n % 256 == 0); device pointers 16-byte aligned. */
TL_API tl_status tl_gemm_q8(void* c, const void* a, const void* b, const float* inv_scales_t, const void* b2,
                            const float* inv_scales_t2, size_t m, size_t n, size_t k, size_t ldc, int epilogue,
                            void* stream);

/* quantize (export_mistral.py:53-68): per group of `group` elements
 * scales[g] = fl(fl(1/max|x|) * 127), q = round_half_even(x * scales[g]). */
TL_API tl_status tl_quantize_i8(int8_t* q, float* scales, const float* x, size_t numel,
                                size_t group, void* stream);

/* ------------------------------------------------------------------------ */
/* Model level: Parameters + InferenceState + Model<T> on one device.        */
/* ------------------------------------------------------------------------ */

/* Config (src/loader/parameters.h:10-23). */
typedef struct tl_config {
    size_t hidden_size, intermediate_size, n_layers, n_heads, n_kv_heads, vocab_size, head_dim,
        sliding_window, max_position_embeddings;
    float rope_theta, norm_eps;
    char quant[16];
} tl_config;

typedef struct tl_model_options {
    int device;      /* CUDA device ordinal                                        */
    size_t max_seq;  /* KV cache capacity in positions; 0 -> 1024                  */
    int use_graph;   /* 1: each decode step is one CUDA-graph replay (default)    */
    int kernel_mode; /* 0: one persistent kernel per decode step when the shape   */
                     /*    fits (default), else per-op kernels; 1: per-op kernels */
    int tp_size;     /* tensor-parallel ranks (0 or 1: none; 2, 4, 8)              */
    int tp_rank;     /* this process's rank in [0, tp_size)                        */
    int sliding_window; /* 0: attend to every cached position, as the reference     */
                        /*    (modules.cpp:75-83) does (default); > 0: only the     */
                        /*    last W positions (HF Mistral's sliding window);       */
                        /*    < 0: W = the binary's sliding_window (its config      */
                        /*    field, parameters.cpp:41, unused by the reference).   */
                        /*    Opt-in: results then differ from the reference's past */
                        /*    W positions.                                          */
    int weights_f16;    /* batched paths (prefill, batched decode): 0 (default) read  */
                        /*    the int8 weights in place, dequantised inside the     */
                        /*    tensor-core GEMM; 1 keep an fp16 copy of every        */
                        /*    projection (2 bytes per parameter, made on first use):*/
                        /*    faster prefill for that memory.                       */
} tl_model_options;

/* Bytes of one rank's exchange-buffer handle (tl_model_tp_handle). */
#define TL_TP_HANDLE_BYTES 64

typedef struct tl_model tl_model;

/* Parameters::load_parameters (parameters.cpp:95-129) + InferenceState(Config&)
 * (inference_state.h:45-71) + Model<int8_t>(params) (modules.h:116-120).
 * Reads the export_mistral.py binary, uploads every weight once to HBM and
 * allocates the fp32 KV cache on the device.  opts may be NULL. */
TL_API tl_status tl_model_load(const char* path, const tl_model_options* opts, tl_model** out);

/* Same, from a host buffer holding the whole file (header + payload). */
TL_API tl_status tl_model_load_buffer(const void* data, size_t size, const tl_model_options* opts,
                                      tl_model** out);

/* Frees the model.  Its batches (tl_batch_create) must be destroyed first:
 * while any exists this returns TL_ERR_INVALID_ARGUMENT and frees nothing. */
TL_API tl_status tl_model_destroy(tl_model* m);
TL_API tl_status tl_model_config(const tl_model* m, tl_config* out);

/* Model<T>::forward (modules.cpp:154-171) for one token at the current
 * position, then pos++.  logits (host, vocab_size floats) and next_token
 * (host; sample_max of the logits, main.cpp:10-21) are optional outputs. */
TL_API tl_status tl_model_forward(tl_model* m, uint32_t token, float* logits, uint32_t* next_token);

/* The prompt loop of main.cpp:69-71 (Model<T>::forward once per token) as
 * one batched pass over tokens[0..n) at positions pos .. pos + n - 1: every
 * layer runs as tensor-core GEMMs over all n rows (fp16 weights dequantised
 * from int8 once, fp32 accumulation) with causal attention over the KV cache,
 * which receives the n new positions exactly as n forwards would write them.
 * logits (host, may be NULL) / *next_token (may be NULL) are those of the
 * last token (sample_max, main.cpp:10-21); pos advances by n and decoding
 * continues with tl_model_forward.  The first call allocates the fp16
 * weights (2 bytes per parameter).  Not available under tensor parallelism. */
TL_API tl_status tl_model_prefill(tl_model* m, const uint32_t* tokens, size_t n, float* logits,
                                  uint32_t* next_token);

/* tl_model_prefill with the device time of the pass (token ids resident,
 * CUDA events on the model's stream) in *ms (measurement aid). */
TL_API tl_status tl_model_time_prefill(tl_model* m, const uint32_t* tokens, size_t n, uint32_t* next_token,
                                       float* ms);

/* The greedy loop of main.cpp:69-77 on the device: forwards prompt[0..n_prompt-1]
 * then n_new times forwards the last argmax; writes the n_new generated ids
 * to out (host).  Only the ids cross the PCIe bus. */
TL_API tl_status tl_model_generate(tl_model* m, const uint32_t* prompt, size_t n_prompt,
                                   size_t n_new, uint32_t* out);

/* generate() with sample_multinomial(infer, temperature) (main.cpp:23-49) in
 * place of sample_max: from the next step on, every decode step of the model
 * (tl_model_forward, tl_model_generate, tl_model_time_decode, the last token
 * of tl_model_prefill) picks its token as tl_sample_multinomial does, with
 * r = tl_sample_uniform(seed, p) for the token computed at position p, on
 * the device (no host round trip).  temperature <= 0 restores sample_max.
 * The logits returned by the calls stay unscaled.  Not available under tensor
 * parallelism (TL_ERR_UNSUPPORTED): each rank holds a slice of the vocabulary. */
TL_API tl_status tl_model_set_sampling(tl_model* m, float temperature, uint64_t seed);

/* InferenceState::pos (inference_state.h:12). */
TL_API tl_status tl_model_get_pos(const tl_model* m, size_t* pos);
TL_API tl_status tl_model_set_pos(tl_model* m, size_t pos);

/* Layer<T>::forward (modules.cpp:118-143) on a host hidden state [hidden_size]
 * at the current position (pos is not advanced), as in test_modules.cpp:3-24. */
TL_API tl_status tl_model_layer_forward(tl_model* m, int layer, float* hidden);

/* Reads the KV cache rows written by push_kv (inference_state.h:38-43) for
 * (layer, pos): k and v are host buffers of n_kv_heads * head_dim floats. */
TL_API tl_status tl_model_read_kv(const tl_model* m, int layer, size_t pos, float* k, float* v);

/* Device time (ms, CUDA events on the model's stream) of n greedy decode steps
 * starting from `token` at the current position, graph replays back to back;
 * the generated ids go to out (host, may be NULL). */
TL_API tl_status tl_model_time_decode(tl_model* m, uint32_t token, size_t n, uint32_t* out,
                                      float* ms);

/* Per-kernel device times (ms per launch, averaged over n eager decode steps
 * with an event pair around every launch).  kinds[] receives up to max_kinds
 * entries of {name, launches, total_ms}; *n_kinds the count. */
typedef struct tl_kernel_time {
    char name[32];
    int launches;
    double total_ms;
    double bytes_per_launch; /* algorithmic bytes of one launch */
} tl_kernel_time;
TL_API tl_status tl_model_profile(tl_model* m, uint32_t token, size_t n, tl_kernel_time* kinds,
                                  int max_kinds, int* n_kinds);

/* Phase trace of one persistent-kernel decode step (tracing aid; the step is a
 * normal forward of `token` at the current position, launched without the
 * graph).  out[0] = CTAs, out[1] = phases (5 per layer + lm_head), then
 * %globaltimer ns stamps [cta][phase][8] = {phase begin, grid barrier passed,
 * activation staged, tiles done, epilogue done, staging loads landed,
 * producer's last issue, first tile of warp 0 done};
 * stamps a CTA does not reach stay 0.  cap is the capacity of out in
 * elements; *n_written receives the element count.  TL_ERR_UNSUPPORTED when
 * the model runs per-op kernels. */
TL_API tl_status tl_model_trace_step(tl_model* m, uint32_t token, uint64_t* out, size_t cap,
                                     size_t* n_written);

/* Tensor parallelism (Megatron-style split of the reference's layers,
 * modules.cpp:49-143): with tp_size > 1 in tl_model_options, rank r keeps q
 * heads, kv heads, gate/up rows, down_proj and o_proj columns and lm_head
 * rows of its slice [r n / tp, (r + 1) n / tp); o_proj and down_proj partials
 * are summed over the ranks inside the decode kernel through NVLink peer
 * memory (no collective library), the argmax is merged across ranks, and
 * every rank returns the same token.  logits arguments receive this rank's
 * vocab_size / tp_size slice.  Each process loads its rank, publishes
 * tl_model_tp_handle() (TL_TP_HANDLE_BYTES), gathers all ranks' handles in
 * rank order and calls tl_model_tp_connect(); every rank then runs the same
 * sequence of forward calls.  No reference counterpart (the reference is
 * single-process CPU code). */
TL_API tl_status tl_model_tp_handle(const tl_model* m, void* handle);
TL_API tl_status tl_model_tp_connect(tl_model* m, const void* handles);

/* Batched decoding: B independent sequences, each with its own fp32 KV
 * cache [L][KV][max_seq][hd] and position, one token per sequence per step.
 * No reference counterpart (the reference's InferenceState holds one
 * sequence); a step equals Model<int8_t>::forward (modules.cpp:118-171) plus
 * sample_max (main.cpp:10-21) run for every sequence, with the linear layers
 * as tensor-core GEMMs over the B rows (fp16 weights dequantised from int8,
 * fp32 accumulation, fp16 lm_head) and each sequence's attention over its own
 * cache.  The batch shares the model's weights and stream; max_seq (0: the
 * model's) must not exceed the model's.  Not available under tensor
 * parallelism. */
typedef struct tl_batch tl_batch;
TL_API tl_status tl_batch_create(tl_model* m, int n_seq, size_t max_seq, tl_batch** out);
TL_API tl_status tl_batch_destroy(tl_batch* b);
/* Cache rows [0, n_pos) of every sequence and layer = N(0, 1) draws of a
 * counter-based generator keyed (seed, sequence, layer, k/v, head, position,
 * dim), so any one sequence can be regenerated alone; every position := n_pos. */
TL_API tl_status tl_batch_fill_kv_random(tl_batch* b, uint64_t seed, size_t n_pos);
/* One step: tokens[B] (host) at each sequence's position; logits (host
 * [B][vocab_size], may be NULL) and next_tokens[B] (host, may be NULL). */
TL_API tl_status tl_batch_step(tl_batch* b, const uint32_t* tokens, float* logits, uint32_t* next_tokens);
/* n_steps greedy steps from tokens[B], each step feeding its argmaxes to the
 * next; out [n_steps][B] (host, may be NULL); *ms = device time (CUDA events). */
TL_API tl_status tl_batch_time_decode(tl_batch* b, const uint32_t* tokens, size_t n_steps, uint32_t* out,
                                      float* ms);
/* K and V rows of sequence `seq` at (layer, pos) into host k, v [n_kv_heads * head_dim]. */
TL_API tl_status tl_batch_read_kv(const tl_batch* b, int seq, int layer, size_t pos, float* k, float* v);

/* Batched decoding under tensor parallelism (a batch of a model loaded with
 * tp_size > 1, connected): every rank creates the batch with the same
 * sequences, then exchanges TL_TP_HANDLE_BYTES handles of its exchange buffer
 * in rank order (tl_batch_tp_handle, any host transport) and maps the others
 * (tl_batch_tp_connect) before the first step.  A step's o_proj and down_proj
 * partial rows are summed across ranks inside the residual + RMSNorm kernel
 * over NVLink peer memory (modules.cpp:128, 142), and the per-row argmax merges
 * the ranks' vocabulary slices.  tl_batch_step's logits are this rank's slice
 * [n_seq][vocab_size / tp]; tl_batch_read_kv returns this rank's kv heads.  A
 * peer that does not arrive within ~2 s fails the step with TL_ERR_TIMEOUT and
 * the model must be reloaded on every rank. */
TL_API tl_status tl_batch_tp_handle(const tl_batch* b, void* handle);
TL_API tl_status tl_batch_tp_connect(tl_batch* b, const void* handles);

/* Number of kernel launches one decode step issues (all of them this library's). */
TL_API tl_status tl_model_launches_per_step(const tl_model* m, int* launches);

/* ---- Tokenizer (host; tokenizer.cpp:1-209) ----
 * The Mistral BPE tokenizer stored in the model binary's header ("tokenizer":
 * {vocab, merges}): Metaspace pre-tokenisation, UTF-8 pieces with <0xXX> byte
 * fallback, repeated merges of the lowest-ranked adjacent pair, BOS (<s>)
 * prepended; decode concatenates the pieces with "\u2581" -> " " (byte
 * pieces stay as written, as in the reference).  Where the reference is
 * undefined (a byte piece or <s> missing, an id outside the vocabulary) these
 * return TL_ERR_FORMAT / TL_ERR_INVALID_ARGUMENT. */
typedef struct tl_tokenizer tl_tokenizer;

/* From a model binary on disk (reads its header only) or in memory. */
TL_API tl_status tl_tokenizer_load(const char* path, tl_tokenizer** out);
TL_API tl_status tl_tokenizer_load_buffer(const void* data, size_t size, tl_tokenizer** out);
/* From the tokenizer object's JSON text ({"vocab": {...}, "merges": [...]}). */
TL_API tl_status tl_tokenizer_load_json(const char* json, size_t len, tl_tokenizer** out);
TL_API tl_status tl_tokenizer_destroy(tl_tokenizer* t);
TL_API tl_status tl_tokenizer_vocab_size(const tl_tokenizer* t, size_t* n);
/* Tokenizer::encode (tokenizer.cpp:121-177) of text[len] into ids[cap];
 * *n_out = the id count (also when cap is too small: TL_ERR_CAPACITY). */
TL_API tl_status tl_tokenizer_encode(const tl_tokenizer* t, const char* text, size_t len, uint32_t* ids,
                                     size_t cap, size_t* n_out);
/* Tokenizer::decode (tokenizer.cpp:203-209) of ids[n] into out[cap] (NUL
 * appended); *len_out = the byte count (also on TL_ERR_CAPACITY). */
TL_API tl_status tl_tokenizer_decode(const tl_tokenizer* t, const uint32_t* ids, size_t n, char* out, size_t cap,
                                     size_t* len_out);

#ifdef __cplusplus
}
#endif

#endif /* TORCHLESS_B200_H */
