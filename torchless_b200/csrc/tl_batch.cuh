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
// positions [0, pos[b]] (window > 0: the last `window` of them) in S splits; CTA (b, kv head g, split) serves the 4 q
// heads g * 4 .. g * 4 + 3 (kv head h / 4, modules.cpp:70), so every K / V row
// is read once.  part[(b H + h) S + split] = {max, sum, 0, 0, acc[hd]}.
tl_status attention_decode_batch(float* part, const float* qf, const BatchKV& kv, int layer, const uint32_t* pos,
                                 int B, int H, int KV, int HD, int S, float scale, int window, cudaStream_t s);

// ---- tensor parallelism (rank r of tp holds the Megatron-style slice the
// bs1 path uses: q/kv heads, gate/up rows and down columns of its F slice, o
// columns of its heads, lm_head rows [vocab_off, vocab_off + V)) ----
//
// Each rank's exchange buffer, mapped by its peers (CUDA IPC):
//   [0, 8 B)          u64 row arrivals of residual exchanges, one per sequence
//   [8 B, 16 B)       u64 row arrivals of argmax exchanges
//   bx_amslot         u64 [2][8][B] argmax candidates {value bits | global index << 32}
//   bx_recv           f32 [2][tp][B][D] o / down partial rows, per sender
// Counters only grow: exchange x of the batch's life is complete for row b
// once its counter reaches (x + 1) tp; buffers alternate by the parity of x.
constexpr int kBatchMaxTp = 8;
__host__ __device__ inline size_t bx_align(size_t x) { return (x + 255) / 256 * 256; }
__host__ __device__ inline size_t bx_amslot(int B) { return bx_align(16 * static_cast<size_t>(B)); }
__host__ __device__ inline size_t bx_recv(int B) { return bx_align(bx_amslot(B) + 2 * kBatchMaxTp * 8 * static_cast<size_t>(B)); }
__host__ __device__ inline size_t bx_bytes(int tp, int B, int D) { return bx_recv(B) + 2 * static_cast<size_t>(tp) * B * D * 4; }

struct BatchXchg {
    uint8_t* buf[kBatchMaxTp];  // every rank's buffer, own at [rank]
    int tp, rank, B, D;
};

// Residual exchange fused with the next RMSNorm (row b = one CTA): the row's
// sum of this rank's ks split-K partials goes to every rank's buffer (P2P
// stores over NVLink), then, once all tp ranks' rows have arrived, h[b] += the
// tp partial rows summed in rank order (bit-identical on every rank), and
// x16[b] = rmsnorm(h[b]) * g as residual_rmsnorm_rows.  `xseq` numbers the
// exchange; a wait that gives up (~2 s) sets *err = 6 and leaves the row.
tl_status tp_residual_rmsnorm_rows(__half* x16, float* h, const float* part, int ks, size_t part_stride,
                                   const float* g, const BatchXchg& X, unsigned long long xseq, int* err,
                                   cudaStream_t s);

// sample_max over the whole vocabulary of each row: every rank sends its
// slice's best {value, global index} (rank 0 flags a NaN logits[0]) to every
// rank, which merge them in rank order (= vocabulary order); out[b] = index,
// pos[b]++.  `aseq` numbers the argmax exchange; timeout as above.
tl_status tp_argmax_rows(uint32_t* out, const float* logits, int V, int vocab_off, uint32_t* pos, const BatchXchg& X,
                         unsigned long long aseq, int* err, cudaStream_t s);

// ctx16[b, h hd + i] = merge of the S split partials (fp16, the o_proj input).
tl_status attention_merge_batch(__half* ctx16, const float* part, int B, int H, int HD, int S, cudaStream_t s);

// out[b] = sample_max of logits[b, 0 .. V) (main.cpp:10-21: first strict max,
// NaN at index 0 keeps 0); pos[b]++ .
tl_status argmax_rows(uint32_t* out, const float* logits, int B, int V, uint32_t* pos, cudaStream_t s);

// Every sequence's cache rows [0, n_pos) of every layer = N(0, 1) draws of a
// counter-based generator keyed by (seed, sequence, layer, k/v, head, position,
// dim) (splitmix64 + Box-Muller), so any sequence can be regenerated alone.
// Under tensor parallelism the local kv heads are global heads kv_off ..
// kv_off + KV - 1 of KV_total, keyed by their global index: every split of the
// model sees the same cache contents.
tl_status fill_kv_random(const BatchKV& kv, uint64_t seed, int B, int L, int KV, int HD, int n_pos, int kv_off,
                         int KV_total, cudaStream_t s);

// w16 = fp16(w) (fp32 lm_head for the batched logits GEMM).
tl_status f32_to_f16(__half* w16, const float* w, size_t n, cudaStream_t s);

}  // namespace tl
