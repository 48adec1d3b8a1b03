// tl_batch.cuh -- kernels of batched decoding (tl_batch.cu): B independent
// sequences, one token each per step, with their own KV caches and positions.
// A step runs Model<int8_t>::forward (modules.cpp:118-171) for all B tokens:
// the linear layers as tensor-core GEMMs over the B rows (tl_gemm.cuh), the
// attention of each sequence over its own cache.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "torchless_b200.h"

namespace tl {

// Cache of sequence b, layer l: base + b * seq_stride + l * layer_stride
// floats, laid out [KV][max_seq][hd] like the model's own cache.
struct BatchKV {
    float *k, *v;
    size_t seq_stride, layer_stride;
    int max_seq;
};

// Row b of qkv [B, (H + 2 KV) hd] = part_0 + ... + part_{ks-1} (the q|k|v
// GEMM's split-K partials, part_r = part + r part_stride, summed in order) at
// position pos[b]: RoPE (kernels.cpp:78-95) on its q and k heads; k and v
// pushed into sequence b's cache of `layer` (inference_state.h:38-43); rotated
// q as fp32 qf [B, H hd].
tl_status rope_cache_batch(float* qf, const float* part, int ks, size_t part_stride, const BatchKV& kv, int layer,
                           const uint32_t* pos, const float* cos_tab, const float* sin_tab, int B, int H, int KV,
                           int HD, cudaStream_t s);

// Attention (modules.cpp:58-88) of each sequence's new query over its cache
// positions [0, pos[b]] in S splits; CTA (b, kv head g, split) serves the 4 q
// heads g * 4 .. g * 4 + 3 (kv head h / 4, modules.cpp:70), so every K / V row
// is read once.  part[(b H + h) S + split] = {max, sum, 0, 0, acc[hd]}.
tl_status attention_decode_batch(float* part, const float* qf, const BatchKV& kv, int layer, const uint32_t* pos,
                                 int B, int H, int KV, int HD, int S, float scale, cudaStream_t s);

// ctx16[b, h hd + i] = merge of the S split partials (fp16, the o_proj input).
tl_status attention_merge_batch(__half* ctx16, const float* part, int B, int H, int HD, int S, cudaStream_t s);

// out[b] = sample_max of logits[b, 0 .. V) (main.cpp:10-21: first strict max,
// NaN at index 0 keeps 0); pos[b]++ .
tl_status argmax_rows(uint32_t* out, const float* logits, int B, int V, uint32_t* pos, cudaStream_t s);

// Every sequence's cache rows [0, n_pos) of every layer = N(0, 1) draws of a
// counter-based generator keyed by (seed, sequence, layer, k/v, head, position,
// dim) (splitmix64 + Box-Muller), so any sequence can be regenerated alone.
tl_status fill_kv_random(const BatchKV& kv, uint64_t seed, int B, int L, int KV, int HD, int n_pos, cudaStream_t s);

// w16 = fp16(w) (fp32 lm_head for the batched logits GEMM).
tl_status f32_to_f16(__half* w16, const float* w, size_t n, cudaStream_t s);

}  // namespace tl
