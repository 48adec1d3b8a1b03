// tl_attention.cu -- batch-1 decode attention over the fp32 KV cache.
//
// Replaces, for one layer and one new token, the body of
// Attention<T>::forward between the q/k/v projections and o_proj
// (src/model/mistral/modules.cpp:58-88):
//   RotaryEmbedding::forward + rope(q) + rope(k)      (modules.cpp:58-62, 22-27;
//                                                      kernels.cpp:78-95)
//   InferenceState::push_kv                           (inference_state.h:38-43)
//   per head h, kv head h/4: scores = K[0..pos] q * 1/sqrt(head_dim),
//   softmax, context = p^T V                          (modules.cpp:70-88)
// The KV cache keeps the reference layout and dtype: fp32
// [n_kv_heads][max_seq][head_dim] per layer (inference_state.h:25-26).
//
// Flash-decoding: grid (n_heads, S).  CTA (h, s) takes one contiguous slice
// of positions 0..pos, each warp an interleaved subset of it, with an online
// softmax; the CTA writes (max, sum, unnormalised context) to a scratch
// partial, and the last CTA of head h (atomic ticket) merges the S partials.
// The new token's k (rotated) and v are used from shared memory for position
// `pos`; the CTA (4*kh, 0) writes them into the cache, so no CTA reads a
// cache row that is being written in the same launch.
//
// cos/sin come from a table filled on the host with the reference's own
// formula (cosf/sinf of powf-derived inv_freq times pos), so RoPE inputs are
// bit-identical to RotaryEmbedding::forward.
#include <math.h>

#include "tl_common.cuh"
#include "tl_kernels.h"

namespace tl {

namespace {

constexpr int kAttnWarps = 4;

template <int HD>
__global__ void __launch_bounds__(kAttnWarps * 32) attn_decode_kernel(AttnArgs a) {
    constexpr int VPL = HD / 32;  // values per lane
    constexpr int HALF = HD / 2;
    __shared__ float q_s[HD], k_s[HD], v_s[HD];
    __shared__ float wm[kAttnWarps], wl[kAttnWarps];
    __shared__ float wacc[kAttnWarps][HD];
    __shared__ bool is_last;

    const int h = blockIdx.x, s = blockIdx.y, S = gridDim.y;
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const int kh = h / 4;  // hard-coded GQA ratio of the reference (modules.cpp:70)

    pdl_wait();
    const unsigned pos = *a.pos;
    const float* qkv = a.qkv;
    const float* qh = qkv + h * HD;
    const float* kn = qkv + a.n_heads * HD + kh * HD;
    const float* vn = qkv + (a.n_heads + a.n_kv_heads) * HD + kh * HD;
    const float* ct = a.cos_tab + static_cast<size_t>(pos) * HALF;
    const float* st = a.sin_tab + static_cast<size_t>(pos) * HALF;
    for (int i = t; i < HALF; i += blockDim.x) {
        const float c = ct[i], sn = st[i];
        const float xq = qh[i], yq = qh[i + HALF];
        q_s[i] = xq * c - yq * sn;
        q_s[i + HALF] = xq * sn + yq * c;
        const float xk = kn[i], yk = kn[i + HALF];
        k_s[i] = xk * c - yk * sn;
        k_s[i + HALF] = xk * sn + yk * c;
        v_s[i] = vn[i];
        v_s[i + HALF] = vn[i + HALF];
    }
    __syncthreads();
    pdl_launch_dependents();

    float* kc = a.k_cache + static_cast<size_t>(kh) * a.max_seq * HD;
    float* vc = a.v_cache + static_cast<size_t>(kh) * a.max_seq * HD;
    if (s == 0 && (h & 3) == 0) {  // push_kv for this kv head
        for (int i = t; i < HD; i += blockDim.x) {
            kc[static_cast<size_t>(pos) * HD + i] = k_s[i];
            vc[static_cast<size_t>(pos) * HD + i] = v_s[i];
        }
    }

    const int npos = static_cast<int>(pos) + 1;
    const int lo = a.window > 0 ? max(0, npos - a.window) : 0;  // attended positions [lo, pos]
    const int chunk = (npos - lo + S - 1) / S;
    const int p0 = lo + s * chunk;
    const int p1 = min(npos, p0 + chunk);

    float q[VPL];
#pragma unroll
    for (int j = 0; j < VPL; j++) q[j] = q_s[lane * VPL + j];
    float m = -INFINITY, l = 0.f, acc[VPL];
#pragma unroll
    for (int j = 0; j < VPL; j++) acc[j] = 0.f;

    for (int p = p0 + warp; p < p1; p += kAttnWarps) {
        float kv[VPL], vv[VPL];
        if (p == static_cast<int>(pos)) {
#pragma unroll
            for (int j = 0; j < VPL; j++) {
                kv[j] = k_s[lane * VPL + j];
                vv[j] = v_s[lane * VPL + j];
            }
        } else {
            const float* kr = kc + static_cast<size_t>(p) * HD + lane * VPL;
            const float* vr = vc + static_cast<size_t>(p) * HD + lane * VPL;
            if constexpr (VPL % 4 == 0) {
#pragma unroll
                for (int j = 0; j < VPL; j += 4) {
                    const float4 k4 = *reinterpret_cast<const float4*>(kr + j);
                    const float4 v4 = *reinterpret_cast<const float4*>(vr + j);
                    kv[j] = k4.x; kv[j + 1] = k4.y; kv[j + 2] = k4.z; kv[j + 3] = k4.w;
                    vv[j] = v4.x; vv[j + 1] = v4.y; vv[j + 2] = v4.z; vv[j + 3] = v4.w;
                }
            } else {
#pragma unroll
                for (int j = 0; j < VPL; j++) {
                    kv[j] = kr[j];
                    vv[j] = vr[j];
                }
            }
        }
        float d = 0.f;
#pragma unroll
        for (int j = 0; j < VPL; j++) d += kv[j] * q[j];
        const float sc = warp_sum(d) * a.scale;
        const float mn = fmaxf(m, sc);
        const float corr = expf(m - mn);
        const float e = expf(sc - mn);
        l = l * corr + e;
#pragma unroll
        for (int j = 0; j < VPL; j++) acc[j] = acc[j] * corr + e * vv[j];
        m = mn;
    }

    if (lane == 0) { wm[warp] = m; wl[warp] = l; }
#pragma unroll
    for (int j = 0; j < VPL; j++) wacc[warp][lane * VPL + j] = acc[j];
    __syncthreads();

    float* part = a.part + (static_cast<size_t>(h) * S + s) * (HD + 2);
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kAttnWarps; w++) M = fmaxf(M, wm[w]);
    for (int i = t; i < HD; i += blockDim.x) {
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < kAttnWarps; w++)
            if (wl[w] > 0.f) v += wacc[w][i] * expf(wm[w] - M);
        part[2 + i] = v;
    }
    if (t == 0) {
        float L = 0.f;
#pragma unroll
        for (int w = 0; w < kAttnWarps; w++)
            if (wl[w] > 0.f) L += wl[w] * expf(wm[w] - M);
        part[0] = M;
        part[1] = L;
        __threadfence();
        is_last = (atomicAdd(a.counters + h, 1u) == static_cast<unsigned>(S) - 1);
    }
    __syncthreads();
    if (!is_last) return;
    __threadfence();

    // Merge the S partials of head h.
    const float* ph = a.part + static_cast<size_t>(h) * S * (HD + 2);
    float GM = -INFINITY;
    for (int j = 0; j < S; j++) {
        const float lj = __ldcg(ph + j * (HD + 2) + 1);
        if (lj > 0.f) GM = fmaxf(GM, __ldcg(ph + j * (HD + 2)));
    }
    float GL = 0.f;
    for (int j = 0; j < S; j++) {
        const float lj = __ldcg(ph + j * (HD + 2) + 1);
        if (lj > 0.f) GL += lj * expf(__ldcg(ph + j * (HD + 2)) - GM);
    }
    const float inv = 1.0f / GL;
    for (int i = t; i < HD; i += blockDim.x) {
        float v = 0.f;
        for (int j = 0; j < S; j++) {
            const float lj = __ldcg(ph + j * (HD + 2) + 1);
            if (lj > 0.f) v += __ldcg(ph + j * (HD + 2) + 2 + i) * expf(__ldcg(ph + j * (HD + 2)) - GM);
        }
        a.ctx[h * HD + i] = v * inv;
    }
    if (t == 0) a.counters[h] = 0;
}

__global__ void embed_kernel(float* h, const float* table, const uint32_t* token, int hidden) {
    pdl_wait();
    const size_t base = static_cast<size_t>(*token) * hidden;
    for (int i = threadIdx.x + blockIdx.x * blockDim.x; i < hidden; i += blockDim.x * gridDim.x)
        h[i] = table[base + i];
    pdl_launch_dependents();
}

template <typename K>
tl_status launch_ex(K kernel, dim3 grid, dim3 block, cudaStream_t s, bool pdl, const char* name,
                    void** args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    cudaError_t e = cudaLaunchKernelExC(&cfg, reinterpret_cast<const void*>(kernel), args);
    if (e != cudaSuccess)
        return set_error(TL_ERR_CUDA, "launch of %s failed: %s", name, cudaGetErrorString(e));
    return TL_OK;
}

}  // namespace

tl_status launch_attention(const AttnArgs& a, cudaStream_t s, bool pdl) {
    AttnArgs copy = a;
    void* args[] = {&copy};
    const dim3 grid(a.n_heads, a.splits), block(kAttnWarps * 32);
    switch (a.head_dim) {
        case 32: return launch_ex(attn_decode_kernel<32>, grid, block, s, pdl, "attention", args);
        case 64: return launch_ex(attn_decode_kernel<64>, grid, block, s, pdl, "attention", args);
        case 128: return launch_ex(attn_decode_kernel<128>, grid, block, s, pdl, "attention", args);
        case 256: return launch_ex(attn_decode_kernel<256>, grid, block, s, pdl, "attention", args);
    }
    return set_error(TL_ERR_UNSUPPORTED, "head_dim %d not supported (32, 64, 128, 256)", a.head_dim);
}

tl_status launch_embed(float* h, const float* table, const uint32_t* token, int hidden,
                       cudaStream_t s, bool pdl) {
    void* args[] = {&h, &table, &token, &hidden};
    return launch_ex(embed_kernel, dim3(1), dim3(512), s, pdl, "embed", args);
}

}  // namespace tl
