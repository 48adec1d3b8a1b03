// tl_prefill.cuh -- kernels of the batched prompt pass (tl_prefill.cu).
//
// A prompt of M tokens at positions p0 .. p0 + M - 1 runs each layer as
// whole-matrix steps (the GEMMs are tl_gemm.cuh):
//   rmsnorm_rows (fp16 out) -> GEMM q|k|v -> rope_cache_rows -> attention_prefill
//   -> GEMM o (+ residual) -> rmsnorm_rows -> GEMM gate|up (SwiGLU) -> GEMM down (+ residual)
// reproducing Model<int8_t>::forward run once per token (modules.cpp:118-171).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "torchless_b200.h"

namespace tl {

// w16[r, c] = fp16(q[r, c] * inv_s[r, c / 64]); rows re-ordered when `swiglu`:
// output block b of 256 rows = gate rows [128 b, 128 b + 128) then up rows of
// the same range (q1/inv1 gate, q3/inv3 up).  Null scales: the bytes are fp8
// e5m2 weights, converted exactly (w16 = the e5m2 value).
tl_status dequant_f16(__half* w16, const int8_t* q1, const float* inv1, const int8_t* q3, const float* inv3, int n,
                      int d, bool swiglu, cudaStream_t s);

// h[i, :] = embed[tokens[i], :]   (Embedding::forward, modules.cpp:5-7)
tl_status embed_rows(float* h, const float* embed, const uint32_t* tokens, int M, int D, cudaStream_t s);

// x16[i, :] = fp16(h[i, :] * (1 / sqrt(sum h^2 / D + 1e-5)) * g)   (RMSNorm, modules.cpp:31-46)
tl_status rmsnorm_rows_f16(__half* x16, const float* h, const float* g, int M, int D, cudaStream_t s);

// Residual add fused with the next RMSNorm: h[i, :] += part_0[i, :] + ... +
// part_{ks-1}[i, :] (split-K partials of the producing GEMM, part_r = part +
// r part_stride, summed in order; modules.cpp:128, 142), then x16 as in
// rmsnorm_rows_f16.  ks = 0 leaves h as it is.  D % 4 == 0, D <= 16384.
tl_status residual_rmsnorm_rows(__half* x16, float* h, const float* part, int ks, size_t part_stride, const float* g,
                                int M, int D, cudaStream_t s);

// Row i (position p0 + i) of qkv [M, (H + 2 KV) hd]: RoPE on its q and k heads
// (kernels.cpp:78-95, tables at the position), k and v rows pushed into the
// layer's cache (inference_state.h:38-43), rotated q written as fp16 q16 [M, H hd].
tl_status rope_cache_rows(__half* q16, const float* qkv, float* k_cache, float* v_cache, const float* cos_tab,
                          const float* sin_tab, int M, int p0, int H, int KV, int HD, int max_seq, cudaStream_t s);

// Causal GQA attention (modules.cpp:58-88) of the M new queries over cache
// positions [0, p0 + i] (window > 0: only the last `window` of them; kv head
// h / 4); ctx16 [M, H hd] fp16.  Cache rows
// [0, p0 + M) are first converted to fp16 scratch k16 / v16 [KV][p0 + M][hd];
// tensor cores (mma m16n8k16, fp16 inputs, fp32 accumulation and softmax).
tl_status attention_prefill(__half* ctx16, const __half* q16, __half* k16, __half* v16, const float* k_cache,
                            const float* v_cache, int M, int p0, int H, int KV, int HD, int max_seq, float scale,
                            int window, cudaStream_t s);

// The same attention on the 5th-generation tensor cores (tl_attn_tc.cu;
// head_dim 128, H = 4 KV): cache rows [0, p0 + M) become fp16 K [KV][T][hd]
// (k16) and V transposed [KV][hd][Tp] (vt16, Tp = T rounded up to 64, zero
// padded; room for Tp <= max_seq rounded up to 64), then one CTA per 32
// queries x kv group.  `err` receives a nonzero code if a bounded wait gave up.
tl_status attention_prefill_tc(__half* ctx16, const __half* q16, __half* k16, __half* vt16, const float* k_cache,
                               const float* v_cache, int M, int p0, int H, int KV, int HD, int max_seq, float scale,
                               int window, int* err, cudaStream_t s);

}  // namespace tl
