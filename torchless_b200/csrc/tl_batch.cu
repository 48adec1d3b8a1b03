// tl_batch.cu -- kernels of batched decoding (interface in tl_batch.cuh).
#include <math.h>

#include <algorithm>

#include "tl_batch.cuh"
#include "tl_common.cuh"

namespace tl {
namespace {

__global__ void k_rope_cache_batch(float* qf, const float* qkv, BatchKV kv, int layer, const uint32_t* pos,
                                   const float* cos_tab, const float* sin_tab, int H, int KV, int HD) {
    const int b = blockIdx.x, half = HD / 2;
    const int p = static_cast<int>(pos[b]);
    const float* row = qkv + static_cast<size_t>(b) * (H + 2 * KV) * HD;
    const float* ct = cos_tab + static_cast<size_t>(p) * half;
    const float* st = sin_tab + static_cast<size_t>(p) * half;
    float* kc = kv.k + b * kv.seq_stride + layer * kv.layer_stride;
    float* vc = kv.v + b * kv.seq_stride + layer * kv.layer_stride;
    for (int k = threadIdx.x; k < (H + KV) * half; k += blockDim.x) {
        const int hh = k / half, c = k % half;
        const float x = row[hh * HD + c], y = row[hh * HD + c + half];
        const float cc = ct[c], sn = st[c];
        const float xr = x * cc - y * sn, yr = x * sn + y * cc;
        float* dst = (hh < H) ? qf + (static_cast<size_t>(b) * H + hh) * HD
                              : kc + (static_cast<size_t>(hh - H) * kv.max_seq + p) * HD;
        dst[c] = xr;
        dst[c + half] = yr;
    }
    for (int k = threadIdx.x; k < KV * HD; k += blockDim.x) {
        const int kh = k / HD, c = k % HD;
        vc[(static_cast<size_t>(kh) * kv.max_seq + p) * HD + c] = row[(H + KV) * HD + k];
    }
}

constexpr int kBW = 8;  // warps per attention CTA
constexpr int kPF = 4;  // positions per warp in flight

template <int HD>
__global__ void __launch_bounds__(kBW * 32) k_attention_decode_batch(float* part, const float* qf, BatchKV kv,
                                                                     int layer, const uint32_t* pos, int H, int S,
                                                                     float scale) {
    constexpr int VPL = HD / 32, QPG = 4, W = HD + 2;
    __shared__ float q_s[QPG * HD];
    __shared__ float wp[kBW * QPG * W];
    const int s = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int npos = static_cast<int>(pos[b]) + 1;
    const int chunk = (npos + S - 1) / S;
    const int p0 = s * chunk, p1 = min(npos, p0 + chunk);
    for (int i = threadIdx.x; i < QPG * HD; i += blockDim.x)
        q_s[i] = qf[(static_cast<size_t>(b) * H + g * QPG) * HD + i];
    __syncthreads();
    const float* kc = kv.k + b * kv.seq_stride + layer * kv.layer_stride + static_cast<size_t>(g) * kv.max_seq * HD;
    const float* vc = kv.v + b * kv.seq_stride + layer * kv.layer_stride + static_cast<size_t>(g) * kv.max_seq * HD;
    float q[QPG][VPL], acc[QPG][VPL], m[QPG], l[QPG];
#pragma unroll
    for (int h = 0; h < QPG; h++) {
        m[h] = -INFINITY;
        l[h] = 0.f;
#pragma unroll
        for (int j = 0; j < VPL; j++) {
            q[h][j] = q_s[h * HD + lane * VPL + j];
            acc[h][j] = 0.f;
        }
    }
    for (int pb = p0 + warp; pb < p1; pb += kBW * kPF) {
        float kr[kPF][VPL], vr[kPF][VPL];
#pragma unroll
        for (int f = 0; f < kPF; f++) {
            const int p = pb + f * kBW;
            if (p < p1) {
                const float4 k4 = __ldcs(reinterpret_cast<const float4*>(kc + static_cast<size_t>(p) * HD) + lane);
                const float4 v4 = __ldcs(reinterpret_cast<const float4*>(vc + static_cast<size_t>(p) * HD) + lane);
                kr[f][0] = k4.x; kr[f][1] = k4.y; kr[f][2] = k4.z; kr[f][3] = k4.w;
                vr[f][0] = v4.x; vr[f][1] = v4.y; vr[f][2] = v4.z; vr[f][3] = v4.w;
            } else {
#pragma unroll
                for (int j = 0; j < VPL; j++) kr[f][j] = vr[f][j] = 0.f;
            }
        }
#pragma unroll
        for (int h = 0; h < QPG; h++) {
            float sc[kPF];
#pragma unroll
            for (int f = 0; f < kPF; f++) {
                float d = 0.f;
#pragma unroll
                for (int j = 0; j < VPL; j++) d += kr[f][j] * q[h][j];
                sc[f] = warp_sum(d) * scale;
            }
            float mn = m[h];
#pragma unroll
            for (int f = 0; f < kPF; f++)
                if (pb + f * kBW < p1) mn = fmaxf(mn, sc[f]);
            const float corr = expf(m[h] - mn);  // m = -inf first: exp(-inf) = 0
            l[h] *= corr;
#pragma unroll
            for (int j = 0; j < VPL; j++) acc[h][j] *= corr;
#pragma unroll
            for (int f = 0; f < kPF; f++) {
                if (pb + f * kBW < p1) {
                    const float e = expf(sc[f] - mn);
                    l[h] += e;
#pragma unroll
                    for (int j = 0; j < VPL; j++) acc[h][j] = fmaf(e, vr[f][j], acc[h][j]);
                }
            }
            m[h] = mn;
        }
    }
#pragma unroll
    for (int h = 0; h < QPG; h++) {
        float* mine = wp + (warp * QPG + h) * W;
        if (lane == 0) {
            mine[0] = m[h];
            mine[1] = l[h];
        }
#pragma unroll
        for (int j = 0; j < VPL; j++) mine[2 + lane * VPL + j] = acc[h][j];
    }
    __syncthreads();
    // this split's partial for each of the 4 heads: {M, L, 0, 0, acc[HD]}
    for (int k = threadIdx.x; k < QPG * (HD + 4); k += blockDim.x) {
        const int h = k / (HD + 4), i = k % (HD + 4);
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kBW; w++)
            if (wp[(w * QPG + h) * W + 1] > 0.f) M = fmaxf(M, wp[(w * QPG + h) * W]);
        float v = 0.f;
        if (i == 0) {
            v = M;
        } else if (i == 1 || i >= 4) {
            const int src = (i == 1) ? 1 : i - 2;
#pragma unroll
            for (int w = 0; w < kBW; w++) {
                const float* pw = wp + (w * QPG + h) * W;
                if (pw[1] > 0.f) v += pw[src] * expf(pw[0] - M);
            }
        }
        part[((static_cast<size_t>(b) * H + g * QPG + h) * S + s) * (HD + 4) + i] = v;
    }
}

__global__ void k_attention_merge_batch(__half* ctx16, const float* part, int H, int HD, int S) {
    const int bh = blockIdx.x, i = threadIdx.x;
    const float* ph = part + static_cast<size_t>(bh) * S * (HD + 4);
    float GM = -INFINITY;
    for (int s = 0; s < S; s++)
        if (ph[s * (HD + 4) + 1] > 0.f) GM = fmaxf(GM, ph[s * (HD + 4)]);
    float GL = 0.f, acc = 0.f;
    for (int s = 0; s < S; s++) {
        const float L = ph[s * (HD + 4) + 1];
        if (L > 0.f) {
            const float w = expf(ph[s * (HD + 4)] - GM);
            GL += L * w;
            acc += ph[s * (HD + 4) + 4 + i] * w;
        }
    }
    if (i < HD) ctx16[static_cast<size_t>(bh) * HD + i] = __float2half_rn(acc / GL);
}

__global__ void k_argmax_rows(uint32_t* out, const float* logits, int V, uint32_t* pos) {
    __shared__ float sv[32];
    __shared__ uint32_t si[32];
    const float* x = logits + static_cast<size_t>(blockIdx.x) * V;
    float v = -INFINITY;
    uint32_t idx = 0xffffffffu;
    for (int i = threadIdx.x; i < V; i += blockDim.x)
        if (better(x[i], static_cast<uint32_t>(i), v, idx)) {
            v = x[i];
            idx = static_cast<uint32_t>(i);
        }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(FULL, v, o);
        const uint32_t oi = __shfl_xor_sync(FULL, idx, o);
        if (better(ov, oi, v, idx)) {
            v = ov;
            idx = oi;
        }
    }
    if ((threadIdx.x & 31) == 0) {
        sv[threadIdx.x >> 5] = v;
        si[threadIdx.x >> 5] = idx;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < static_cast<int>(blockDim.x >> 5); w++)
            if (better(sv[w], si[w], v, idx)) {
                v = sv[w];
                idx = si[w];
            }
        if (x[0] != x[0] || idx == 0xffffffffu) idx = 0;  // sample_max keeps 0 (main.cpp:10-21)
        out[blockIdx.x] = idx;
        if (pos) pos[blockIdx.x]++;
    }
}

// splitmix64 (Vigna's published mixer).
__device__ __forceinline__ uint64_t splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

__global__ void k_fill_kv_random(BatchKV kv, uint64_t seed, int B, int L, int KV, int HD, int n_pos) {
    const size_t total = static_cast<size_t>(B) * L * 2 * KV * n_pos * HD;
    for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < total; e += (size_t)gridDim.x * blockDim.x) {
        size_t r = e;
        const int d = static_cast<int>(r % HD); r /= HD;
        const int p = static_cast<int>(r % n_pos); r /= n_pos;
        const int kh = static_cast<int>(r % KV); r /= KV;
        const int which = static_cast<int>(r % 2); r /= 2;
        const int l = static_cast<int>(r % L);
        const int b = static_cast<int>(r / L);
        // key independent of B and n_pos: (sequence, layer, k/v, head, position < 2^20, dim)
        const uint64_t key =
            ((((static_cast<uint64_t>(b) * L + l) * 2 + which) * KV + kh) * (1ull << 20) + p) * HD + d;
        const uint64_t rnd = splitmix64(seed ^ splitmix64(key >> 1));
        const float u1 = static_cast<float>((rnd >> 40) + 1) * 5.9604645e-8f;  // (0, 1]
        const float u2 = static_cast<float>((rnd >> 16) & 0xFFFFFF) * 5.9604645e-8f;
        const float rad = sqrtf(-2.0f * logf(u1));
        float sn, cs;
        sincospif(2.0f * u2, &sn, &cs);
        const float z = (key & 1) ? rad * sn : rad * cs;  // Box-Muller pair
        float* base = (which ? kv.v : kv.k) + b * kv.seq_stride + l * kv.layer_stride;
        base[(static_cast<size_t>(kh) * kv.max_seq + p) * HD + d] = z;
    }
}

__global__ void k_f32_to_f16(__half* w16, const float* w, size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        w16[i] = __float2half_rn(w[i]);
}

int grid_of(size_t n, int per) { return static_cast<int>(std::min<size_t>((n + per - 1) / per, 148 * 16)); }

}  // namespace

tl_status rope_cache_batch(float* qf, const float* qkv, const BatchKV& kv, int layer, const uint32_t* pos,
                           const float* cos_tab, const float* sin_tab, int B, int H, int KV, int HD, cudaStream_t s) {
    k_rope_cache_batch<<<B, 128, 0, s>>>(qf, qkv, kv, layer, pos, cos_tab, sin_tab, H, KV, HD);
    return check_launch("rope_cache_batch");
}

tl_status attention_decode_batch(float* part, const float* qf, const BatchKV& kv, int layer, const uint32_t* pos,
                                 int B, int H, int KV, int HD, int S, float scale, cudaStream_t s) {
    TL_REQUIRE(H == 4 * KV && S >= 1, "attention_decode_batch: H == 4 KV, S >= 1");
    const dim3 grid(S, KV, B);
    if (HD != 128) return set_error(TL_ERR_UNSUPPORTED, "attention_decode_batch: head_dim %d (128 built)", HD);
    k_attention_decode_batch<128><<<grid, kBW * 32, 0, s>>>(part, qf, kv, layer, pos, H, S, scale);
    return check_launch("attention_decode_batch");
}

tl_status attention_merge_batch(__half* ctx16, const float* part, int B, int H, int HD, int S, cudaStream_t s) {
    k_attention_merge_batch<<<B * H, HD, 0, s>>>(ctx16, part, H, HD, S);
    return check_launch("attention_merge_batch");
}

tl_status argmax_rows(uint32_t* out, const float* logits, int B, int V, uint32_t* pos, cudaStream_t s) {
    k_argmax_rows<<<B, 1024, 0, s>>>(out, logits, V, pos);
    return check_launch("argmax_rows");
}

tl_status fill_kv_random(const BatchKV& kv, uint64_t seed, int B, int L, int KV, int HD, int n_pos, cudaStream_t s) {
    const size_t total = static_cast<size_t>(B) * L * 2 * KV * n_pos * HD;
    k_fill_kv_random<<<grid_of(total, 256), 256, 0, s>>>(kv, seed, B, L, KV, HD, n_pos);
    return check_launch("fill_kv_random");
}

tl_status f32_to_f16(__half* w16, const float* w, size_t n, cudaStream_t s) {
    k_f32_to_f16<<<grid_of(n, 256), 256, 0, s>>>(w16, w, n);
    return check_launch("f32_to_f16");
}

}  // namespace tl
