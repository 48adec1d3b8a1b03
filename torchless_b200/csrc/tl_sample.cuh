// tl_sample.cuh -- sample_multinomial (main.cpp:23-43) on the device: the
// block-wide routine shared by the standalone op (tl_sample.cu), the
// persistent decode step's last CTA (tl_decode.cu) and the per-op / prefill
// steps (sample_step).
#pragma once

#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "torchless_b200.h"

namespace tl {

// The uniform draw of device-side sampling for (seed, position): the
// splitmix64 finaliser of seed + (pos + 1) * 0x9E3779B97F4A7C15, top 24 bits
// times 2^-24 (exact in float, in [0, 1)).  The reference draws from an
// unseeded mt19937 (main.cpp:6-8); a fixed counter function instead makes a
// sampled generation reproducible and checkable.
__host__ __device__ inline float sample_uniform(uint64_t seed, uint64_t pos) {
    uint64_t z = seed + (pos + 1) * 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    z ^= z >> 31;
    return static_cast<float>(z >> 40) * (1.0f / 16777216.0f);
}

// sample_multinomial over logits[0, n) at temperature temp > 0 with uniform
// draw r, by NT threads that all call it (thread t owns the contiguous chunk
// [t c, t c + c), c = ceil(n / NT)).  sm: NT / 32 floats of shared memory;
// sync(): a barrier of the NT threads.  Every thread gets the result:
//  * n - 1 if a scaled logit is NaN or +inf, or all are -inf: in the
//    reference a NaN then reaches the total and every probability, so no
//    running sum compares >= r and the loop falls through to the last index;
//  * else the first index whose running sum of probabilities reaches r, or
//    n - 1 if none does.
// Softmax as kernels.cpp:55-63: logits / temp, exp(x - max), total, times
// (1 / total).  The sums run over each thread's chunk and then across chunks
// in thread order (the reference sums sequentially), so the index can differ
// from the reference's only where r lies within rounding of a running-sum
// boundary.  Logits are read through L2 (they may be written by other CTAs
// of the same kernel).
template <int NT, typename Sync>
__device__ uint32_t sample_block(const float* logits, int n, float temp, float r, float* sm, Sync sync) {
    static_assert(NT % 32 == 0 && NT <= 1024, "whole warps");
    constexpr int NW = NT / 32;
    constexpr unsigned kAll = 0xffffffffu;
    const int t = threadIdx.x, lane = t & 31, w = t >> 5;
    const int c = (n + NT - 1) / NT;
    const int i0 = min(n, t * c), i1 = min(n, i0 + c);
    // pass 1: max of the scaled logits (Tensor::max, tensor.cpp:71-78), NaN / +inf
    float mx = -INFINITY;
    int bad = 0;
    for (int i = i0; i < i1; i++) {
        const float x = __ldcg(logits + i) / temp;
        bad |= (x != x) || (x == INFINITY);
        mx = fmaxf(mx, x);
    }
    bad = __any_sync(kAll, bad);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(kAll, mx, o));
    if (lane == 0) sm[w] = bad ? NAN : mx;
    sync();
    float M = -INFINITY;
    bool any_bad = false;
#pragma unroll
    for (int v = 0; v < NW; v++) {
        const float q = sm[v];
        if (q != q) any_bad = true;
        else M = fmaxf(M, q);
    }
    sync();
    if (any_bad || M == -INFINITY) return static_cast<uint32_t>(n - 1);
    // pass 2: total = sum of exp(x - max)
    float s = 0.f;
    for (int i = i0; i < i1; i++) s += expf(__ldcg(logits + i) / temp - M);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(kAll, s, o);
    if (lane == 0) sm[w] = s;
    sync();
    float total = 0.f;
#pragma unroll
    for (int v = 0; v < NW; v++) total += sm[v];
    sync();
    const float inv = 1.0f / total;  // mul(xout, xout, 1 / total)
    // pass 3: probability sum of each chunk, exclusive scan over the chunks
    float cs = 0.f;
    for (int i = i0; i < i1; i++) cs += expf(__ldcg(logits + i) / temp - M) * inv;
    float inc = cs;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const float y = __shfl_up_sync(kAll, inc, o);
        if (lane >= o) inc += y;
    }
    float pre = __shfl_up_sync(kAll, inc, 1);
    if (lane == 0) pre = 0.f;
    if (lane == 31) sm[w] = inc;
    sync();
    for (int v = 0; v < w; v++) pre += sm[v];
    sync();
    // the first index of this chunk whose running sum reaches r
    uint32_t hit = 0xffffffffu;
    float cum = pre;
    for (int i = i0; i < i1; i++) {
        cum += expf(__ldcg(logits + i) / temp - M) * inv;
        if (cum >= r) {
            hit = static_cast<uint32_t>(i);
            break;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) hit = min(hit, __shfl_xor_sync(kAll, hit, o));
    if (lane == 0) reinterpret_cast<uint32_t*>(sm)[w] = hit;
    sync();
    uint32_t res = 0xffffffffu;
#pragma unroll
    for (int v = 0; v < NW; v++) res = min(res, reinterpret_cast<const uint32_t*>(sm)[v]);
    sync();
    return res == 0xffffffffu ? static_cast<uint32_t>(n - 1) : res;
}

// sample_max (main.cpp:10-21) of logits[0, V) as one step's token: *token,
// history[*pos] = the index, then (*pos)++ (one CTA).
tl_status argmax_step(uint32_t* token, uint32_t* history, unsigned* pos, const float* logits, int V, cudaStream_t s);

// After a greedy lm_head step that wrote token / history[pos - 1] and
// advanced *pos: replaces the token with the sample at temperature temp of
// logits[0, V) using sample_uniform(seed, *pos - 1) (one CTA).
tl_status sample_step(uint32_t* token, uint32_t* history, const unsigned* pos, const float* logits, int V, float temp,
                      uint64_t seed, cudaStream_t s);

}  // namespace tl
