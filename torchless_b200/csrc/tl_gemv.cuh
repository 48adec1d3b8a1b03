// tl_gemv.cuh -- HBM-bound batch-1 matrix-vector kernels (int8 and fp32 weights).
//
// Replaces matmul(Tensor<float>&, Tensor<int8_t>&, Tensor<float>&) and
// matmul(Tensor<float>&, Tensor<float>&, Tensor<float>&)
// (src/backend/cpu/kernels.cpp:6-33) on the decode path, fused with the
// elementwise work around each call site in src/model/mistral/modules.cpp:
//   * RMSNorm prologue (modules.cpp:31-46) for q/k/v, gate/up and lm_head,
//   * residual-add epilogue (modules.cpp:128, 142) for o_proj and down_proj,
//   * SiLU(gate) * up epilogue (modules.cpp:99-112) for gate_proj/up_proj,
//   * logits store + argmax (main.cpp:10-21) for lm_head.
//
// Work decomposition.  A row of W (d columns) is split into 16-column chunks;
// thread t of the CTA owns chunks t, t + T, ... (C of them, T = d / (16 C)
// threads), so its slice of the activation vector lives in registers for the
// whole kernel and every weight byte is read once, with 16-byte streaming
// loads that are fully coalesced across the warp.  Each CTA walks a
// contiguous range of rows R at a time; per-row partial sums are reduced
// with a warp transpose-reduction and a shared-memory pass over warps.  The
// grid is one wave (SM count x resident CTAs), each CTA an equal row share.
//
// int8 dequantisation: the reference computes sum_j (q_j / s_g) x_j
// sequentially in fp32.  Here each 16-column chunk (inside one 64-column
// group) computes sum q_j x_j exactly-converted in fp32 and applies the
// group scale once (1/s precomputed at model upload, or a division for the
// op-level entry point that receives the stored scales).  This only reorders
// fp32 roundings (relative differences around 1e-6 per output), far inside
// the 1e-2 relative logit tolerance the parity tests enforce.
#pragma once

#include "tl_common.cuh"

namespace tl {

enum GemvEpi : int { kStore = 0, kAddResidual = 1, kSwiGLU = 2 };

struct GemvI8Args {
    const int8_t* w;   // [n, d] row-major (gate_proj in SwiGLU mode); e5m2 bytes when f8
    const float* s;    // [n * d / 64] group scales (inverted when INV); unused when f8
    const int8_t* w2;  // up_proj in SwiGLU mode
    const float* s2;
    const float* x;    // activation [d]; with NORM the un-normalised hidden state
    const float* g;    // RMSNorm gain [d] (NORM)
    float eps;
    float* y;          // output [n]
    const float* res;  // residual [n] (kAddResidual); may alias y
    int n, d;
    int f8;            // the weights are fp8 (e5m2) without scales (format extension)
};

// Loads 16 fp32 activations for chunk `ch` as 8 packed pairs.
__device__ __forceinline__ void load_x16(const float* x, int ch, float2 (&xp)[8]) {
    const float4* p = reinterpret_cast<const float4*>(x + 16 * ch);
#pragma unroll
    for (int k = 0; k < 4; k++) {
        const float4 v = p[k];
        xp[2 * k] = make_float2(v.x, v.y);
        xp[2 * k + 1] = make_float2(v.z, v.w);
    }
}

// RMSNorm of the activation slice held in registers (modules.cpp:31-46):
// x = (h * (1/rms)) * g with rms = sqrt(sum(h^2)/d + eps).  Every CTA
// recomputes the (cheap) sum of squares of the whole vector.
template <int C>
__device__ __forceinline__ void rmsnorm_slice(float2 (&xp)[C][8], const float* g, int T, int d,
                                              float eps, float* red) {
    float ss = 0.f;
#pragma unroll
    for (int c = 0; c < C; c++)
#pragma unroll
        for (int k = 0; k < 8; k++) ss += xp[c][k].x * xp[c][k].x + xp[c][k].y * xp[c][k].y;
    ss = block_sum(ss, red);
    const float rms = sqrtf(ss / static_cast<float>(d) + eps);
    const float inv = 1.0f / rms;
#pragma unroll
    for (int c = 0; c < C; c++) {
        float2 gp[8];
        load_x16(g, threadIdx.x + c * T, gp);
#pragma unroll
        for (int k = 0; k < 8; k++) {
            xp[c][k].x = (xp[c][k].x * inv) * gp[k].x;
            xp[c][k].y = (xp[c][k].y * inv) * gp[k].y;
        }
    }
}

// R rows per iteration, C chunks per thread.  Block size T = d / (16 C),
// a multiple of 32 and <= MAXT.  Dynamic shared memory: 32 + 2 * (T/32) * R
// floats.  F8: the weight bytes are e5m2 values, used as they are (no scale).
template <int R, int C, int MAXT, bool INV, bool NORM, int EPI, bool F8>
__global__ void __launch_bounds__(MAXT) gemv_i8_kernel(GemvI8Args a) {
    extern __shared__ float smem[];
    const int T = blockDim.x;
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5, nw = T >> 5;
    float* red = smem;        // 32 floats for block_sum
    float* part = smem + 32;  // [2][nw][R]
    const int gpr = a.d >> 6; // scale groups per row

    constexpr int OUT = (EPI == kSwiGLU) ? R / 2 : R;  // output rows per iteration
    const int units = (a.n + OUT - 1) / OUT;
    const int u0 = static_cast<int>((static_cast<long long>(units) * blockIdx.x) / gridDim.x);
    const int u1 = static_cast<int>((static_cast<long long>(units) * (blockIdx.x + 1)) / gridDim.x);

    // Row r of iteration u -> (matrix, row index).
    auto row_ptrs = [&](int u, int r, const int8_t*& wp, const float*& sp, int& row) {
        if (EPI == kSwiGLU) {
            row = u * OUT + (r % OUT);
            wp = (r < OUT) ? a.w : a.w2;
            sp = (r < OUT) ? a.s : a.s2;
        } else {
            row = u * OUT + r;
            wp = a.w;
            sp = a.s;
        }
    };

    uint4 wv[R][C];
    float sc[R][C];
    auto load_unit = [&](int u) {
#pragma unroll
        for (int r = 0; r < R; r++) {
            const int8_t* wp;
            const float* sp;
            int row;
            row_ptrs(u, r, wp, sp, row);
            const bool ok = row < a.n;
#pragma unroll
            for (int c = 0; c < C; c++) {
                const int ch = t + c * T;
                if (ok) {
                    wv[r][c] = ld_stream(wp + static_cast<size_t>(row) * a.d + 16 * ch);
                    sc[r][c] = F8 ? 1.f : __ldg(sp + static_cast<size_t>(row) * gpr + (ch >> 2));
                } else {
                    wv[r][c] = make_uint4(0, 0, 0, 0);
                    sc[r][c] = 1.f;
                }
            }
        }
    };

    // Weights do not depend on the previous kernel: start streaming them
    // before waiting on it.
    if (u0 < u1) load_unit(u0);
    pdl_wait();

    float2 xp[C][8];
#pragma unroll
    for (int c = 0; c < C; c++) load_x16(a.x, t + c * T, xp[c]);
    if (NORM) rmsnorm_slice<C>(xp, a.g, T, a.d, a.eps, red);
    pdl_launch_dependents();

    int buf = 0;
    for (int u = u0; u < u1; u++) {
        float p[R];
#pragma unroll
        for (int r = 0; r < R; r++) {
            float acc = 0.f;
#pragma unroll
            for (int c = 0; c < C; c++) {
                if (F8) {
                    acc += dot16_f8(wv[r][c], xp[c]);
                } else {
                    const float d16 = dot16_i8(wv[r][c], xp[c]);
                    acc += INV ? d16 * sc[r][c] : d16 / sc[r][c];
                }
            }
            p[r] = acc;
        }
        if (u + 1 < u1) load_unit(u + 1);

        warp_reduce_multi<R>(p);
        float* pb = part + buf * nw * R;
        if ((lane & (32 / R - 1)) == 0) pb[warp * R + lane / (32 / R)] = p[0];
        __syncthreads();
        if (t < OUT) {
            float v = 0.f;
            for (int w = 0; w < nw; w++) v += pb[w * R + t];
            const int row = u * OUT + t;
            if (row < a.n) {
                if (EPI == kStore) {
                    a.y[row] = v;
                } else if (EPI == kAddResidual) {
                    a.y[row] = v + a.res[row];
                } else {
                    float up = 0.f;
                    for (int w = 0; w < nw; w++) up += pb[w * R + OUT + t];
                    const float gate = v / (1.0f + expf(-v));  // silu, kernels.cpp:98-102
                    a.y[row] = gate * up;                      // mul, kernels.cpp:127-131
                }
            }
        }
        buf ^= 1;
    }
}

// ---------------------------------------------------------------------------
// fp32 weights (lm_head, modules.cpp:147-149; matmul(f32) kernels.cpp:6-19).
// ---------------------------------------------------------------------------

struct GemvF32Args {
    const float* w;     // [n, d]
    const float* x;     // activation [d] (hidden state when NORM)
    const float* g;     // RMSNorm gain (NORM)
    float eps;
    float* y;           // logits [n]
    int n, d;
    // Argmax (ARGMAX): per-CTA partials, a completion counter (zero before
    // the launch; the last CTA resets it), and the outputs.
    float* part_v;
    uint32_t* part_i;
    unsigned* counter;
    uint32_t* out_token;   // sample_max result
    uint32_t* history;     // optional: history[*pos] = token
    unsigned* pos;         // optional: ++*pos after the token is written
};

// Thread t owns 16 consecutive columns [16t, 16t+16): T = d/16 <= MAXT threads.
template <int R, int MAXT, bool NORM, bool ARGMAX>
__global__ void __launch_bounds__(MAXT) gemv_f32_kernel(GemvF32Args a) {
    extern __shared__ float smem[];
    const int T = blockDim.x;
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5, nw = T >> 5;
    float* red = smem;
    float* part = smem + 32;                      // [2][nw][R]
    __shared__ float bv_s[32];
    __shared__ uint32_t bi_s[32];

    const int units = (a.n + R - 1) / R;
    const int u0 = static_cast<int>((static_cast<long long>(units) * blockIdx.x) / gridDim.x);
    const int u1 = static_cast<int>((static_cast<long long>(units) * (blockIdx.x + 1)) / gridDim.x);

    float4 wv[R][4];
    auto load_unit = [&](int u) {
#pragma unroll
        for (int r = 0; r < R; r++) {
            const int row = u * R + r;
#pragma unroll
            for (int k = 0; k < 4; k++)
                wv[r][k] = (row < a.n) ? ld_stream_f4(a.w + static_cast<size_t>(row) * a.d + 16 * t + 4 * k)
                                       : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    };
    if (u0 < u1) load_unit(u0);
    pdl_wait();

    float2 xp[1][8];
    load_x16(a.x, t, xp[0]);
    if (NORM) rmsnorm_slice<1>(xp, a.g, T, a.d, a.eps, red);
    pdl_launch_dependents();

    float best_v = -INFINITY;
    uint32_t best_i = 0xffffffffu;
    int buf = 0;
    for (int u = u0; u < u1; u++) {
        float p[R];
#pragma unroll
        for (int r = 0; r < R; r++) {
            float2 acc0 = make_float2(0.f, 0.f), acc1 = make_float2(0.f, 0.f);
#pragma unroll
            for (int k = 0; k < 4; k++) {
                acc0 = ffma2(make_float2(wv[r][k].x, wv[r][k].y), xp[0][2 * k], acc0);
                acc1 = ffma2(make_float2(wv[r][k].z, wv[r][k].w), xp[0][2 * k + 1], acc1);
            }
            const float2 s = fadd2(acc0, acc1);
            p[r] = s.x + s.y;
        }
        if (u + 1 < u1) load_unit(u + 1);
        warp_reduce_multi<R>(p);
        float* pb = part + buf * nw * R;
        if ((lane & (32 / R - 1)) == 0) pb[warp * R + lane / (32 / R)] = p[0];
        __syncthreads();
        if (t < R) {
            float v = 0.f;
            for (int w = 0; w < nw; w++) v += pb[w * R + t];
            const int row = u * R + t;
            if (row < a.n) {
                a.y[row] = v;
                if (ARGMAX && better(v, row, best_v, best_i)) {
                    best_v = v;
                    best_i = row;
                }
            }
        }
        buf ^= 1;
    }

    if (!ARGMAX) return;
    // CTA argmax over the R candidate holders (threads 0..R-1).
    if (t < 32) {
        float v = (t < R) ? best_v : -INFINITY;
        uint32_t i = (t < R) ? best_i : 0xffffffffu;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(FULL, v, o);
            const uint32_t oi = __shfl_xor_sync(FULL, i, o);
            if (better(ov, oi, v, i)) { v = ov; i = oi; }
        }
        if (t == 0) {
            a.part_v[blockIdx.x] = v;
            a.part_i[blockIdx.x] = i;
        }
    }
    // Last CTA to finish combines the partials (threadfence reduction).
    __shared__ bool is_last;
    if (t == 0) {
        __threadfence();
        const unsigned done = atomicAdd(a.counter, 1u);
        is_last = (done == gridDim.x - 1);
    }
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    float v = -INFINITY;
    uint32_t i = 0xffffffffu;
    for (int b = t; b < static_cast<int>(gridDim.x); b += T) {
        const float ov = __ldcg(a.part_v + b);
        const uint32_t oi = __ldcg(a.part_i + b);
        if (better(ov, oi, v, i)) { v = ov; i = oi; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(FULL, v, o);
        const uint32_t oi = __shfl_xor_sync(FULL, i, o);
        if (better(ov, oi, v, i)) { v = ov; i = oi; }
    }
    if (lane == 0) { bv_s[warp] = v; bi_s[warp] = i; }
    __syncthreads();
    if (t == 0) {
        for (int w = 1; w < nw; w++)
            if (better(bv_s[w], bi_s[w], v, i)) { v = bv_s[w]; i = bi_s[w]; }
        // sample_max starts from logits[0] and only moves on a strict '>':
        // a NaN there (or no finite winner at all) leaves index 0.
        const float l0 = __ldcg(a.y);
        if (l0 != l0 || i == 0xffffffffu) i = 0;
        *a.out_token = i;
        if (a.pos) {
            const unsigned p = *a.pos;
            if (a.history) a.history[p] = i;
            *a.pos = p + 1;
        }
        *a.counter = 0;  // ready for the next launch
    }
}

}  // namespace tl
