// tl_prefill.cu -- row-wise kernels and causal attention of the batched
// prompt pass (interface and data flow in tl_prefill.cuh).
#include <math.h>

#include <algorithm>

#include "tl_common.cuh"
#include "tl_prefill.cuh"

namespace tl {
namespace {

__global__ void k_dequant_f16(__half* w16, const int8_t* q1, const float* inv1, const int8_t* q3, const float* inv3,
                              int n, int d, int swiglu) {
    const size_t rows = swiglu ? 2 * static_cast<size_t>(n) : n;
    const size_t chunks = rows * (d / 8);
    for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < chunks; idx += (size_t)gridDim.x * blockDim.x) {
        const size_t R = idx / (d / 8);
        const int c = static_cast<int>(idx % (d / 8)) * 8;
        const int8_t* q = q1;
        const float* inv = inv1;
        size_t r = R;
        if (swiglu) {  // block of 256 output rows = 128 gate rows, then the same 128 up rows
            const size_t b = R / 256, w = R % 256;
            if (w < 128) {
                r = b * 128 + w;
            } else {
                r = b * 128 + (w - 128);
                q = q3;
                inv = inv3;
            }
        }
        const int2 raw = *reinterpret_cast<const int2*>(q + r * d + c);
        if (!inv) {  // e5m2 bytes: each is the high byte of the same value's fp16 (exact)
            const uint32_t x = static_cast<uint32_t>(raw.x), y = static_cast<uint32_t>(raw.y);
            *reinterpret_cast<uint4*>(w16 + R * d + c) =
                make_uint4(__byte_perm(x, 0u, 0x1404), __byte_perm(x, 0u, 0x3424), __byte_perm(y, 0u, 0x1404),
                           __byte_perm(y, 0u, 0x3424));
            continue;
        }
        const float s = inv[(r * d + c) / 64];
        const int8_t* b8 = reinterpret_cast<const int8_t*>(&raw);
        __half2 out[4];
#pragma unroll
        for (int j = 0; j < 4; j++)
            out[j] = __floats2half2_rn(static_cast<float>(b8[2 * j]) * s, static_cast<float>(b8[2 * j + 1]) * s);
        *reinterpret_cast<uint4*>(w16 + R * d + c) = *reinterpret_cast<const uint4*>(out);
    }
}

__global__ void k_embed_rows(float* h, const float* embed, const uint32_t* tokens, int M, int D) {
    const size_t n4 = static_cast<size_t>(M) * D / 4;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
        const size_t row = i / (D / 4), c = i % (D / 4);
        reinterpret_cast<float4*>(h)[i] = reinterpret_cast<const float4*>(embed + static_cast<size_t>(tokens[row]) * D)[c];
    }
}

constexpr int kNormVec = 4;  // float4 columns a thread holds: rows up to 4 x 4 x 1024 = 16384 wide

// One CTA per row; thread t owns float4 columns t, t + blockDim, ...  With
// ks > 0 the row first takes its residual add: h += (part_0 + part_1 + ...).
__global__ void k_residual_rmsnorm_rows(__half* x16, float* h, const float* part, int ks, size_t part_stride,
                                        const float* g, int D) {
    __shared__ float red[32];
    const int n4 = D / 4;
    float4* hr = reinterpret_cast<float4*>(h + static_cast<size_t>(blockIdx.x) * D);
    const float4* pr = reinterpret_cast<const float4*>(part + static_cast<size_t>(blockIdx.x) * D);
    float4 v[kNormVec];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < kNormVec; j++) {
        const int c = threadIdx.x + j * blockDim.x;
        if (c >= n4) break;
        float4 x = hr[c];
        if (ks > 0) {
            float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int r = 0; r < ks; r++) {
                const float4 p = pr[r * (part_stride / 4) + c];
                a.x += p.x; a.y += p.y; a.z += p.z; a.w += p.w;
            }
            x.x += a.x; x.y += a.y; x.z += a.z; x.w += a.w;
            hr[c] = x;
        }
        v[j] = x;
        ss += x.x * x.x + x.y * x.y + x.z * x.z + x.w * x.w;
    }
    ss = block_sum(ss, red);
    const float inv = 1.0f / sqrtf(ss / static_cast<float>(D) + 1e-5f);
    uint2* y = reinterpret_cast<uint2*>(x16 + static_cast<size_t>(blockIdx.x) * D);
#pragma unroll
    for (int j = 0; j < kNormVec; j++) {
        const int c = threadIdx.x + j * blockDim.x;
        if (c >= n4) break;
        const float* gc = g + 4 * c;
        __half2 o[2] = {__floats2half2_rn((v[j].x * inv) * gc[0], (v[j].y * inv) * gc[1]),
                        __floats2half2_rn((v[j].z * inv) * gc[2], (v[j].w * inv) * gc[3])};
        y[c] = *reinterpret_cast<const uint2*>(o);
    }
}

// Block = row i (position p0 + i); its threads walk the (head slot, pair)
// items: rotated pair (c, c + hd / 2) of q / k head hh, or two v values of
// kv head hh - H - KV.
__global__ void k_rope_cache_rows(__half* q16, const float* qkv, float* kc, float* vc, const float* cos_tab,
                                  const float* sin_tab, int p0, int H, int KV, int HD, int max_seq) {
    const int i = blockIdx.x, pos = p0 + i, half = HD / 2;
    const float* ct = cos_tab + static_cast<size_t>(pos) * half;
    const float* st = sin_tab + static_cast<size_t>(pos) * half;
    const float* base = qkv + static_cast<size_t>(i) * (H + 2 * KV) * HD;
    for (int k = threadIdx.x; k < (H + 2 * KV) * half; k += blockDim.x) {
        const int hh = k / half, c = k % half;
        const float* row = base + hh * HD;
        const float x = row[c], y = row[c + half];
        if (hh < H + KV) {
            const float cc = ct[c], sn = st[c];
            const float xr = x * cc - y * sn, yr = x * sn + y * cc;
            if (hh < H) {
                __half* q = q16 + static_cast<size_t>(i) * H * HD + hh * HD;
                q[c] = __float2half_rn(xr);
                q[c + half] = __float2half_rn(yr);
            } else {
                float* kr = kc + (static_cast<size_t>(hh - H) * max_seq + pos) * HD;
                kr[c] = xr;
                kr[c + half] = yr;
            }
        } else {
            float* vr = vc + (static_cast<size_t>(hh - H - KV) * max_seq + pos) * HD;
            vr[c] = x;
            vr[c + half] = y;
        }
    }
}

// mma.m16n8k16 f16 x f16 -> f32 (A row-major 16x16, B col-major 16x8).
__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
}

__device__ __forceinline__ uint32_t su32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }
// Four 8x8 b16 matrices; lanes 8 i .. 8 i + 7 give the row addresses of matrix i.
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(su32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(su32(p)));
}
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(su32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__global__ void k_kv_to_f16(__half* k16, __half* v16, const float* kc, const float* vc, int KV, int T, int HD,
                            int max_seq) {
    const size_t n4 = static_cast<size_t>(KV) * T * HD / 4;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
        const size_t e = i * 4, kh = e / (static_cast<size_t>(T) * HD), rest = e % (static_cast<size_t>(T) * HD);
        const size_t src = kh * max_seq * HD + rest;
        const float4 a = *reinterpret_cast<const float4*>(kc + src);
        const float4 b = *reinterpret_cast<const float4*>(vc + src);
        const __half2 ka[2] = {__floats2half2_rn(a.x, a.y), __floats2half2_rn(a.z, a.w)};
        const __half2 vb[2] = {__floats2half2_rn(b.x, b.y), __floats2half2_rn(b.z, b.w)};
        *reinterpret_cast<uint2*>(k16 + e) = *reinterpret_cast<const uint2*>(ka);
        *reinterpret_cast<uint2*>(v16 + e) = *reinterpret_cast<const uint2*>(vb);
    }
}

// Flash attention, one CTA per (64 queries, head), 4 warps x 16 query rows.
// fp16 K and V blocks of 64 keys ([key][HD], rows padded) double-buffered with
// cp.async; S = Q K^T B fragments by ldmatrix, O += P V B fragments by
// ldmatrix.trans of the row-major V block.
constexpr int kAQ = 64, kAK = 64;
template <int HD>
__global__ void __launch_bounds__(128) k_attention_prefill(__half* ctx16, const __half* q16, const __half* k16,
                                                           const __half* v16, int M, int p0, int H, int T,
                                                           float scale, int window) {
    constexpr int KP = HD + 8;  // padded row (halves): 16-byte aligned, conflict-free ldmatrix
    extern __shared__ __align__(16) __half smem_h[];
    __half* Ks = smem_h;                 // [2][kAK][KP]
    __half* Vs = smem_h + 2 * kAK * KP;  // [2][kAK][KP]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int h = blockIdx.y, kh = h / 4;  // kv head h / 4 (modules.cpp:70)
    const int q0 = blockIdx.x * kAQ, qend = min(M, q0 + kAQ);
    const int r0 = q0 + warp * 16;
    const __half* kbase = k16 + static_cast<size_t>(kh) * T * HD;
    const __half* vbase = v16 + static_cast<size_t>(kh) * T * HD;

    uint32_t qa[HD / 16][4];
    {
        const int ra = r0 + g, rb = r0 + g + 8;
        const __half* qa_row = q16 + (static_cast<size_t>(ra) * H + h) * HD;
        const __half* qb_row = q16 + (static_cast<size_t>(rb) * H + h) * HD;
#pragma unroll
        for (int ks = 0; ks < HD / 16; ks++) {
            const int c = ks * 16 + 2 * t;
            qa[ks][0] = ra < M ? *reinterpret_cast<const uint32_t*>(qa_row + c) : 0u;
            qa[ks][1] = rb < M ? *reinterpret_cast<const uint32_t*>(qb_row + c) : 0u;
            qa[ks][2] = ra < M ? *reinterpret_cast<const uint32_t*>(qa_row + c + 8) : 0u;
            qa[ks][3] = rb < M ? *reinterpret_cast<const uint32_t*>(qb_row + c + 8) : 0u;
        }
    }
    float o[HD / 8][4];
#pragma unroll
    for (int j = 0; j < HD / 8; j++) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
    float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f;  // rows g and g + 8
    const int pos_a = p0 + r0 + g, pos_b = pos_a + 8;
    const bool row_a = (r0 + g) < M, row_b = (r0 + g + 8) < M;
    const int kmax = p0 + qend;  // keys [0, kmax) exist for this CTA
    const int nkb = (kmax + kAK - 1) / kAK;
    // sliding window: query at position p sees keys (p - window, p]; the CTA's
    // first query bounds the first key block any of its queries needs
    const int kb0 = window > 0 ? max(0, p0 + q0 - window + 1) / kAK : 0;

    auto stage = [&](int kb, int buf) {  // keys >= kmax are zero rows
        const int k0 = kb * kAK;
        __half* kd = Ks + buf * kAK * KP;
        __half* vd = Vs + buf * kAK * KP;
        for (int e = threadIdx.x; e < kAK * HD / 8; e += blockDim.x) {
            const int key = e / (HD / 8), c = (e % (HD / 8)) * 8;
            if (k0 + key < kmax) {
                cp_async16(kd + key * KP + c, kbase + static_cast<size_t>(k0 + key) * HD + c);
                cp_async16(vd + key * KP + c, vbase + static_cast<size_t>(k0 + key) * HD + c);
            } else {
                *reinterpret_cast<uint4*>(kd + key * KP + c) = make_uint4(0, 0, 0, 0);
                *reinterpret_cast<uint4*>(vd + key * KP + c) = make_uint4(0, 0, 0, 0);
            }
        }
        cp_async_commit();
    };
    stage(kb0, 0);
    const int mi = lane >> 3, mr = lane & 7;  // ldmatrix: matrix index, row within it
    for (int kb = kb0; kb < nkb; kb++) {
        const int buf = (kb - kb0) & 1, k0 = kb * kAK;
        if (kb + 1 < nkb) {
            stage(kb + 1, buf ^ 1);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        const __half* kd = Ks + buf * kAK * KP;
        const __half* vd = Vs + buf * kAK * KP;
        // S = Q K^T (16 x 64 per warp)
        float s[kAK / 8][4];
#pragma unroll
        for (int j = 0; j < kAK / 8; j++) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
        for (int ks = 0; ks < HD / 16; ks++) {
#pragma unroll
            for (int j = 0; j < kAK / 8; j += 2) {
                uint32_t b[4];  // b0, b1 of key tiles j and j + 1
                ldsm_x4(b, kd + (8 * j + 8 * (mi >> 1) + mr) * KP + 16 * ks + 8 * (mi & 1));
                mma_f16(s[j], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], b[0], b[1]);
                mma_f16(s[j + 1], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], b[2], b[3]);
            }
        }
        // scale, causal mask (key position <= query position), row max over the quad
        float mx_a = -INFINITY, mx_b = -INFINITY;
#pragma unroll
        for (int j = 0; j < kAK / 8; j++) {
#pragma unroll
            for (int e = 0; e < 2; e++) {
                const int key = k0 + j * 8 + 2 * t + e;
                const bool in_a = row_a && key <= pos_a && (window <= 0 || key > pos_a - window);
                const bool in_b = row_b && key <= pos_b && (window <= 0 || key > pos_b - window);
                s[j][e] = in_a ? s[j][e] * scale : -INFINITY;
                s[j][2 + e] = in_b ? s[j][2 + e] * scale : -INFINITY;
                mx_a = fmaxf(mx_a, s[j][e]);
                mx_b = fmaxf(mx_b, s[j][2 + e]);
            }
        }
        mx_a = fmaxf(mx_a, __shfl_xor_sync(FULL, mx_a, 1));
        mx_a = fmaxf(mx_a, __shfl_xor_sync(FULL, mx_a, 2));
        mx_b = fmaxf(mx_b, __shfl_xor_sync(FULL, mx_b, 1));
        mx_b = fmaxf(mx_b, __shfl_xor_sync(FULL, mx_b, 2));
        const float mn_a = fmaxf(m_a, mx_a), mn_b = fmaxf(m_b, mx_b);
        const float c_a = (mn_a == -INFINITY) ? 1.f : expf(m_a - mn_a);
        const float c_b = (mn_b == -INFINITY) ? 1.f : expf(m_b - mn_b);
        m_a = mn_a;
        m_b = mn_b;
        l_a *= c_a;
        l_b *= c_b;
#pragma unroll
        for (int j = 0; j < HD / 8; j++) {
            o[j][0] *= c_a;
            o[j][1] *= c_a;
            o[j][2] *= c_b;
            o[j][3] *= c_b;
        }
        // P = exp(S - m) as fp16 A fragments; O += P V
#pragma unroll
        for (int kk = 0; kk < kAK / 16; kk++) {
            float p[2][4];
#pragma unroll
            for (int u = 0; u < 2; u++) {
                const int j = 2 * kk + u;
                p[u][0] = (s[j][0] == -INFINITY) ? 0.f : expf(s[j][0] - mn_a);
                p[u][1] = (s[j][1] == -INFINITY) ? 0.f : expf(s[j][1] - mn_a);
                p[u][2] = (s[j][2] == -INFINITY) ? 0.f : expf(s[j][2] - mn_b);
                p[u][3] = (s[j][3] == -INFINITY) ? 0.f : expf(s[j][3] - mn_b);
                l_a += p[u][0] + p[u][1];
                l_b += p[u][2] + p[u][3];
            }
            const uint32_t a0 = pack_h2(p[0][0], p[0][1]), a1 = pack_h2(p[0][2], p[0][3]);
            const uint32_t a2 = pack_h2(p[1][0], p[1][1]), a3 = pack_h2(p[1][2], p[1][3]);
#pragma unroll
            for (int j = 0; j < HD / 8; j += 2) {
                uint32_t b[4];  // b0, b1 of dim tiles j and j + 1 (V transposed by ldmatrix)
                ldsm_x4_t(b, vd + (16 * kk + 8 * (mi & 1) + mr) * KP + 8 * j + 8 * (mi >> 1));
                mma_f16(o[j], a0, a1, a2, a3, b[0], b[1]);
                mma_f16(o[j + 1], a0, a1, a2, a3, b[2], b[3]);
            }
        }
        __syncthreads();  // everyone is done with `buf` before it is refilled
    }
    // row sums over the quad, normalise, store fp16 ctx
    l_a += __shfl_xor_sync(FULL, l_a, 1);
    l_a += __shfl_xor_sync(FULL, l_a, 2);
    l_b += __shfl_xor_sync(FULL, l_b, 1);
    l_b += __shfl_xor_sync(FULL, l_b, 2);
    const float ia = l_a > 0.f ? 1.0f / l_a : 0.f, ib = l_b > 0.f ? 1.0f / l_b : 0.f;
    __half* ya = ctx16 + (static_cast<size_t>(r0 + g) * H + h) * HD;
    __half* yb = ctx16 + (static_cast<size_t>(r0 + g + 8) * H + h) * HD;
#pragma unroll
    for (int j = 0; j < HD / 8; j++) {
        const int c = j * 8 + 2 * t;
        if (row_a) *reinterpret_cast<uint32_t*>(ya + c) = pack_h2(o[j][0] * ia, o[j][1] * ia);
        if (row_b) *reinterpret_cast<uint32_t*>(yb + c) = pack_h2(o[j][2] * ib, o[j][3] * ib);
    }
}

int grid_for(size_t n, int per) { return static_cast<int>(std::min<size_t>((n + per - 1) / per, 148 * 16)); }

}  // namespace

tl_status dequant_f16(__half* w16, const int8_t* q1, const float* inv1, const int8_t* q3, const float* inv3, int n,
                      int d, bool swiglu, cudaStream_t s) {
    TL_REQUIRE(d % 64 == 0 && (!swiglu || n % 128 == 0), "dequant_f16: shape");
    const size_t chunks = (swiglu ? 2 * static_cast<size_t>(n) : n) * (d / 8);
    k_dequant_f16<<<grid_for(chunks, 256), 256, 0, s>>>(w16, q1, inv1, q3, inv3, n, d, swiglu ? 1 : 0);
    return check_launch("dequant_f16");
}

tl_status embed_rows(float* h, const float* embed, const uint32_t* tokens, int M, int D, cudaStream_t s) {
    k_embed_rows<<<grid_for(static_cast<size_t>(M) * D / 4, 256), 256, 0, s>>>(h, embed, tokens, M, D);
    return check_launch("embed_rows");
}

tl_status rmsnorm_rows_f16(__half* x16, const float* h, const float* g, int M, int D, cudaStream_t s) {
    return residual_rmsnorm_rows(x16, const_cast<float*>(h), nullptr, 0, 0, g, M, D, s);
}

tl_status residual_rmsnorm_rows(__half* x16, float* h, const float* part, int ks, size_t part_stride, const float* g,
                                int M, int D, cudaStream_t s) {
    const int n4 = D / 4;
    // each thread holds up to kNormVec float4 columns: few threads per row keep
    // many rows resident per SM (the kernel is latency-bound, one row per CTA)
    const int threads = std::min(1024, std::max(32, ((n4 + kNormVec - 1) / kNormVec + 31) / 32 * 32));
    TL_REQUIRE(D % 4 == 0 && n4 <= kNormVec * threads, "rmsnorm rows: width %d (multiple of 4, at most %d)", D,
               kNormVec * 4 * 1024);
    TL_REQUIRE(((reinterpret_cast<uintptr_t>(h) | reinterpret_cast<uintptr_t>(part)) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(x16) & 7) == 0 && part_stride % 4 == 0 && (ks == 0 || part),
               "rmsnorm rows: alignment");
    k_residual_rmsnorm_rows<<<M, threads, 0, s>>>(x16, h, part, ks, part_stride, g, D);
    return check_launch("residual_rmsnorm_rows");
}

tl_status rope_cache_rows(__half* q16, const float* qkv, float* k_cache, float* v_cache, const float* cos_tab,
                          const float* sin_tab, int M, int p0, int H, int KV, int HD, int max_seq, cudaStream_t s) {
    TL_REQUIRE(HD % 2 == 0, "rope_cache_rows: head_dim %d", HD);
    k_rope_cache_rows<<<M, 256, 0, s>>>(q16, qkv, k_cache, v_cache, cos_tab, sin_tab, p0, H, KV, HD, max_seq);
    return check_launch("rope_cache_rows");
}

tl_status attention_prefill(__half* ctx16, const __half* q16, __half* k16, __half* v16, const float* k_cache,
                            const float* v_cache, int M, int p0, int H, int KV, int HD, int max_seq, float scale,
                            int window, cudaStream_t s) {
    TL_REQUIRE(H == 4 * KV, "attention_prefill: kv head h / 4 needs H == 4 KV");
    const int T = p0 + M;  // cached positions the queries can see
    const size_t n4 = static_cast<size_t>(KV) * T * HD / 4;
    k_kv_to_f16<<<grid_for(n4, 256), 256, 0, s>>>(k16, v16, k_cache, v_cache, KV, T, HD, max_seq);
    TL_TRY(check_launch("kv_to_f16"));
    const dim3 grid((M + kAQ - 1) / kAQ, H);
    switch (HD) {
        case 64: {
            const size_t smem = 4 * kAK * (64 + 8) * 2;
            k_attention_prefill<64><<<grid, 128, smem, s>>>(ctx16, q16, k16, v16, M, p0, H, T, scale, window);
            break;
        }
        case 128: {
            const size_t smem = 4 * kAK * (128 + 8) * 2;  // 69632 bytes
            static bool attr = false;
            if (!attr) {
                TL_CUDA_TRY(cudaFuncSetAttribute(k_attention_prefill<128>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
                attr = true;
            }
            k_attention_prefill<128><<<grid, 128, smem, s>>>(ctx16, q16, k16, v16, M, p0, H, T, scale, window);
            break;
        }
        default: return set_error(TL_ERR_UNSUPPORTED, "attention_prefill: head_dim %d", HD);
    }
    return check_launch("attention_prefill");
}

}  // namespace tl
