// tl_decode.cuh -- interface of the persistent decode-step kernel (tl_decode.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "torchless_b200.h"

namespace tl {

// Tiled weight layout streamed by the persistent kernel.
//
// int8 matrices ([n, d], row-major in the file) become tiles of 16 rows x 512
// columns (d a multiple of 64; the last tile of a row block is zero-padded).  A tile is 8192 bytes of weights followed by 512 bytes of fp32
// inverse scales; tiles are ordered row-block major ((rb, ks) -> rb*KS + ks),
// so the rows a CTA owns are one contiguous byte range.  Inside a tile,
// block w covers columns [64w, 64w+64) (one quantisation group):
//   byte  w*1024 + half*512 + lane*16 + j   holds  W[16 rb + 8 half + lane/4]
//                                                 [512 ks + 64 w + 16 (lane%4) + j]
// stored as the signed int8 q itself (the integer MMA's A operand);
//   float 2048 + rr*8 + w                    holds  1 / scale of row 16 rb + rr,
//                                                 group 8 ks + w.
// gate/up are interleaved: tile row rr < 8 is gate row 8 rb + rr, rr >= 8 is
// up row 8 rb + rr - 8, so one tile yields 8 SwiGLU outputs.
// fp8 matrices (e5m2 bytes, no scales) use the same 16 x 512 tiles and byte
// layout without the scale block: 8192 bytes per tile.
// The persistent kernel gives each tile to one consumer warp.
// fp32 lm_head tiles are 4 rows x 512 columns (8192 bytes):
//   float w*256 + (rr/2)*128 + lane*4 + (rr%2)*2 + e  holds
//   W[4 rb + rr][512 ks + 64 w + 2 lane + e].
constexpr int kTileCols = 512;
constexpr int kTileRowsI8 = 16;
constexpr int kTileBytesI8 = 8192 + 512;
constexpr int kTileBytesF8 = 8192;
constexpr int kTileRowsF32 = 4;
constexpr int kTileBytesF32 = 8192;
constexpr int kStatsCap = 1024;  // most CTAs / heads publishing statistics

// Tensor-parallel exchange buffer (one per rank, mapped into every rank's
// process over CUDA IPC), byte offsets:
constexpr size_t kXchgAmCnt = 8;     // u64: argmax candidate arrivals from all ranks
constexpr size_t kXchgAmSlot = 256;  // u64 [2][8]: {value bits | rank-local best index << 32}
constexpr size_t kXchgRecv = 512;    // u64 [2][tp][D]: {partial row value, exchange tag << 32} per sender
constexpr int kMaxTp = 8;
inline size_t xchg_bytes(int tp, int D) { return kXchgRecv + 2 * static_cast<size_t>(tp) * D * 8; }

struct DecodeLayer {
    const uint8_t* qkv;  // tiles of [q; k; v]   ((H + 2 KV) hd rows, d = D)
    const uint8_t* o;    // tiles of o_proj      (D rows, d = H hd)
    const uint8_t* w13;  // tiles of gate/up     (2F rows interleaved, d = D)
    const uint8_t* w2;   // tiles of down_proj   (D rows, d = F)
    const float* g_in;
    const float* g_post;
    float* k_cache;      // [KV][max_seq][hd]
    float* v_cache;
};

struct DecodeArgs {
    const DecodeLayer* layers;  // device array [n_layers]
    int n_layers;
    const float* embed;         // [V, D]
    const float* g_final;       // [D]
    const uint8_t* lm_head;     // fp32 tiles, or 8-bit tiles like the projections' when lm_8bit
    int lm_8bit;                // lm_head stored in the projections' format (format extension)
    int w_f8;                   // projection tiles hold fp8 (e5m2) weights, not int8 + scales
    const float* cos_tab;       // [max_seq][hd/2]
    const float* sin_tab;
    float* h;                   // residual stream [D]
    float* qkv;                 // [(H + 2 KV) hd]
    float* attn_part;           // [H][S][hd + 4] split partials {max, sum, 0, 0, acc}
    float* ctx;                 // [H hd] attention output (GQA attention; per-head attention leaves
                                // the merge of attn_part to the o_proj staging)
    unsigned* attn_cnt;         // [H] split tickets per kv group, zero between launches
    unsigned* qkv_cnt;          // [KV] q/k/v rows written per kv group, zero between launches
    float* act;                 // [F]
    float* logits;              // [V]
    float* am_v;                // [grid] argmax partials
    uint32_t* am_i;
    unsigned* ticket;           // zero between launches (last CTA resets it)
    unsigned* bar;              // grid barrier counter, zero between launches (last CTA resets it)
    int* err;                   // nonzero after a bounded wait gave up
    uint32_t* token;            // in: this step's token; out: argmax
    unsigned* pos;              // in: position; out: position + 1
    uint32_t* history;          // history[pos] = argmax
    int D, F, H, KV, HD, V, max_seq, splits;
    int split_rows;             // per-head attention: cached positions per split (at least)
    // GQA attention (hd 128, H = 4 KV): from position gqa_from - 1 on, one CTA
    // per (kv group, split) serves the group's 4 query heads, at most
    // gqa_splits splits; gqa_splits 0 = per-head attention only.
    int gqa_splits, gqa_from;
    int gqa_rows;               // GQA: cached positions per split (at least)
    int window;                 // > 0: attention over the last `window` positions (sliding window)
    // Sampling (main.cpp:23-43) in place of sample_max when temperature > 0:
    // the uniform draw of position pos is sample_uniform(sample_seed, pos).
    float temperature;
    unsigned long long sample_seed;
    int kv_prefetch_rows;       // K (and V) rows an attention CTA hints into L2 during q/k/v
    int pbuf_floats;            // per-phase partial-sum buffer (decode_kernel_fits)
    float attn_scale;
    // Phase hand-over statistics: [2][kStatsCap] {sum x^2, max |x|} of what
    // each CTA wrote in a phase, alternating buffers per phase.
    float2* stats;
    int prefetch;               // tile pairs prefetched into L2 ahead of the ring (0 = off)
    // act published as staged digits by the gate/up epilogue (one GPU, int8
    // tiles; null: off): the digits in the staging layout [3 * F padded],
    // per layer the exponent to use (set from the previous step's max with 2
    // bits of headroom; < -999: none yet), and the epoch + 1 of a step in
    // which some value did not fit (the down staging then converts act itself).
    uint8_t* act_dig;
    int* act_k;
    unsigned* act_ovf;
    // Tensor parallelism (tp_size > 1, modules.cpp layers split Megatron
    // style): this rank holds q heads and kv heads [rank H, (rank + 1) H)
    // (H, KV local), gate/up rows and down columns of its F slice, o_proj
    // columns of its heads, and lm_head rows [vocab_off, vocab_off + V).
    // o_proj and down_proj produce full-D partials that every rank sums in
    // rank order; xpeer[q] is rank q's exchange buffer (own at q = tp_rank).
    int tp_size, tp_rank, vocab_off;
    uint8_t* xpeer[kMaxTp];
    unsigned* epoch;            // steps run so far (numbers the tp exchanges and argmax rounds)
    unsigned long long timeout_ns;  // bound of every wait on other CTAs or ranks (then TL_ERR_TIMEOUT)
    // Optional phase trace (nullptr = off): per CTA, kTraceEvents %globaltimer
    // stamps for every phase, [cta][phase][event], phases = 5 per layer + lm_head.
    unsigned long long* trace;
    // Self-check build only (TL_DECODE_CHECK): first violated check as
    // {site, value0, value1}; the checked access is skipped.
    int* dbg;
};

// Trace events per phase: 0 begin, 1 grid barrier (or exchange) passed,
// 2 activation staged, 3 tiles done, 4 epilogue done, 5 staging loads
// landed, 6 producer's last issue of the phase, 7 warp 0's first tile done.
constexpr int kTraceEvents = 8;

// Shared-memory bytes, pipeline depth and partial-buffer size for a model
// shape on `grid` CTAs; false when the shape cannot run in the persistent kernel.
bool decode_kernel_fits(int D, int F, int H, int KV, int HD, int V, int n_layers, bool w_f8, int grid,
                        int max_smem, int* stages, size_t* smem_bytes, int* pbuf_floats);

// Launch one decode step (cooperative: every CTA resident on its own SM).
tl_status launch_decode_step(const DecodeArgs& a, int grid, int stages, size_t smem, cudaStream_t s);

// Weight repacking into the tiled layout (run once at model load).  Null
// scales: the bytes are fp8 (e5m2) weights and the tiles kTileBytesF8 long.
tl_status repack_i8(uint8_t* dst, const int8_t* w, const float* s, int n, int d, cudaStream_t st);
tl_status repack_i8_swiglu(uint8_t* dst, const int8_t* w1, const float* s1, const int8_t* w3,
                           const float* s3, int n, int d, cudaStream_t st);
tl_status repack_f32(uint8_t* dst, const float* w, int n, int d, cudaStream_t st);

// Tiles per row block: columns rounded up to whole tiles (padding is zero).
__host__ __device__ inline int tile_slices(int d) { return (d + kTileCols - 1) / kTileCols; }
inline size_t tiles_q_bytes(int n_rows, int d, bool f8) {
    return static_cast<size_t>((n_rows + kTileRowsI8 - 1) / kTileRowsI8) * tile_slices(d) *
           (f8 ? kTileBytesF8 : kTileBytesI8);
}
inline size_t tiles_f32_bytes(int n_rows, int d) {
    return static_cast<size_t>((n_rows + kTileRowsF32 - 1) / kTileRowsF32) * tile_slices(d) * kTileBytesF32;
}

}  // namespace tl
