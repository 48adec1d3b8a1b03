// tl_kernels.h -- host-side launchers shared by the op-level ABI and the model.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "torchless_b200.h"

namespace tl {

struct GemvI8Args;
struct GemvF32Args;

// Launch modes for the fused int8 GEMV.
enum class I8Mode { Store, AddResidual, SwiGLU };

// True when (n, d, pointers) fit the fast int8 GEMV layout: d a multiple of
// 512 (so d/16 threads form whole warps), group size 64, 16-byte aligned rows.
bool gemv_i8_fast_ok(size_t n, size_t d, size_t n_scales, const void* w, const void* x);
bool gemv_f32_fast_ok(size_t n, size_t d, const void* w, const void* x);

// `inv` selects 1/s scales (model layout) versus stored s (reference layout).
// `pdl` launches with programmatic stream serialization.
tl_status launch_gemv_i8(const GemvI8Args& a, I8Mode mode, bool inv, bool norm, cudaStream_t s,
                         bool pdl);
tl_status launch_gemv_f32(const GemvF32Args& a, bool norm, bool argmax, cudaStream_t s, bool pdl);

// Grid size the f32 GEMV launcher uses for (n, d) (argmax partial count).
int gemv_f32_grid(size_t n, size_t d, bool norm, bool argmax);

// Decode attention for one layer (tl_attention.cu).
struct AttnArgs {
    const float* qkv;      // [q (H*hd) | k (KV*hd) | v (KV*hd)] un-rotated
    float* k_cache;        // this layer's [KV][max_seq][hd]
    float* v_cache;
    const float* cos_tab;  // [max_seq][hd/2]
    const float* sin_tab;
    const unsigned* pos;   // device position counter
    float* ctx;            // [H*hd]
    float* part;           // scratch: [H][S][hd + 2]
    unsigned* counters;    // scratch: [H], zero between launches
    int n_heads, n_kv_heads, head_dim, max_seq, splits;
    float scale;           // (float)(1/sqrt(head_dim))
    int window;            // > 0: attend to the last `window` positions only (sliding window)
};
tl_status launch_attention(const AttnArgs& a, cudaStream_t s, bool pdl);

// h = embed[token] (Embedding::forward, modules.cpp:5-7).
tl_status launch_embed(float* h, const float* table, const uint32_t* token, int hidden,
                       cudaStream_t s, bool pdl);

}  // namespace tl
