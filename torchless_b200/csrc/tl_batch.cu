// tl_batch.cu -- kernels of batched decoding (interface in tl_batch.cuh).
#include <math.h>

#include <algorithm>

#include "tl_batch.cuh"
#include "tl_common.cuh"

namespace tl {
namespace {

// Block (b, head slot hh), thread c < hd / 2: element pair (c, c + hd / 2) of
// q|k|v slot hh of row b, summed over the K-split partials in order.
__global__ void k_rope_cache_batch(float* qf, const float* part, int ks, size_t part_stride, BatchKV kv, int layer,
                                   const uint32_t* pos, const float* cos_tab, const float* sin_tab, int H, int KV,
                                   int HD) {
    const int b = blockIdx.x, hh = blockIdx.y, c = threadIdx.x, half = HD / 2;
    const int p = static_cast<int>(pos[b]);
    const float* row = part + static_cast<size_t>(b) * (H + 2 * KV) * HD + hh * HD;
    float x = 0.f, y = 0.f;
    for (int r = 0; r < ks; r++) {
        x += row[r * part_stride + c];
        y += row[r * part_stride + c + half];
    }
    const size_t cache = b * kv.seq_stride + layer * kv.layer_stride;
    if (hh < H + KV) {
        const float cc = cos_tab[static_cast<size_t>(p) * half + c], sn = sin_tab[static_cast<size_t>(p) * half + c];
        const float xr = x * cc - y * sn, yr = x * sn + y * cc;
        float* dst = (hh < H) ? qf + (static_cast<size_t>(b) * H + hh) * HD
                              : kv.k + cache + (static_cast<size_t>(hh - H) * kv.max_seq + p) * HD;
        dst[c] = xr;
        dst[c + half] = yr;
    } else {
        float* dst = kv.v + cache + (static_cast<size_t>(hh - H - KV) * kv.max_seq + p) * HD;
        dst[c] = x;
        dst[c + half] = y;
    }
}

constexpr int kBW = 8;  // warps per attention CTA

// Warp w takes groups of 8 positions; lane l holds dims 4 l .. 4 l + 3 of q,
// K, V and of the accumulators of the 4 heads.  The 32 partial dot products
// of a group (4 heads x 8 positions) are reduced together (transposed
// reduction, 31 shuffles); lane l then holds score(head l / 8, position l % 8),
// and the online softmax runs per 8-lane group.
template <int HD>
__global__ void __launch_bounds__(kBW * 32) k_attention_decode_batch(float* part, const float* qf, BatchKV kv,
                                                                     int layer, const uint32_t* pos, int H, int S,
                                                                     float scale, int window) {
    static_assert(HD == 128, "lane owns 4 of 128 dims");
    constexpr int QPG = 4, W = HD + 2, G = 8;  // heads per kv head, partial row, positions per group
    __shared__ float wp[kBW * QPG * W];
    const int s = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int npos = static_cast<int>(pos[b]) + 1;
    const int lo = window > 0 ? max(0, npos - window) : 0;  // attended positions [lo, pos]
    const int chunk = (npos - lo + S - 1) / S;
    const int p0 = lo + s * chunk, p1 = min(npos, p0 + chunk);
    const float* kc = kv.k + b * kv.seq_stride + layer * kv.layer_stride + static_cast<size_t>(g) * kv.max_seq * HD;
    const float* vc = kv.v + b * kv.seq_stride + layer * kv.layer_stride + static_cast<size_t>(g) * kv.max_seq * HD;
    float4 q[QPG], acc[QPG];
    float m[QPG];
#pragma unroll
    for (int h = 0; h < QPG; h++) {
        q[h] = reinterpret_cast<const float4*>(qf + (static_cast<size_t>(b) * H + g * QPG + h) * HD)[lane];
        acc[h] = make_float4(0.f, 0.f, 0.f, 0.f);
        m[h] = -INFINITY;
    }
    const int my_h = lane >> 3, my_f = lane & 7;
    float l_lane = 0.f;  // softmax denominator share of (head my_h, position slot my_f)
    for (int pb = p0 + warp * G; pb < p1; pb += kBW * G) {
        float4 kr[G], vr[G];
#pragma unroll
        for (int f = 0; f < G; f++) {
            if (pb + f < p1) {
                kr[f] = __ldcs(reinterpret_cast<const float4*>(kc + static_cast<size_t>(pb + f) * HD) + lane);
                vr[f] = __ldcs(reinterpret_cast<const float4*>(vc + static_cast<size_t>(pb + f) * HD) + lane);
            } else {
                kr[f] = vr[f] = make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
        float v[QPG * G];
#pragma unroll
        for (int h = 0; h < QPG; h++)
#pragma unroll
            for (int f = 0; f < G; f++)
                v[h * G + f] = q[h].x * kr[f].x + q[h].y * kr[f].y + q[h].z * kr[f].z + q[h].w * kr[f].w;
        warp_reduce_multi<QPG * G>(v);  // lane l: full dot of (head l / 8, position l % 8)
        const bool valid = pb + my_f < p1;
        const float sc = valid ? v[0] * scale : -INFINITY;
        float gm = sc;
        gm = fmaxf(gm, __shfl_xor_sync(FULL, gm, 1));
        gm = fmaxf(gm, __shfl_xor_sync(FULL, gm, 2));
        gm = fmaxf(gm, __shfl_xor_sync(FULL, gm, 4));
        float corr[QPG];
#pragma unroll
        for (int h = 0; h < QPG; h++) {
            const float mn = fmaxf(m[h], __shfl_sync(FULL, gm, h * G));  // position pb is valid: mn finite
            corr[h] = expf(m[h] - mn);  // first group: exp(-inf) = 0
            m[h] = mn;
            acc[h].x *= corr[h]; acc[h].y *= corr[h]; acc[h].z *= corr[h]; acc[h].w *= corr[h];
        }
        const float p = valid ? expf(sc - m[my_h]) : 0.f;
        l_lane = l_lane * corr[my_h] + p;
#pragma unroll
        for (int f = 0; f < G; f++) {
#pragma unroll
            for (int h = 0; h < QPG; h++) {
                const float ph = __shfl_sync(FULL, p, h * G + f);
                acc[h].x = fmaf(ph, vr[f].x, acc[h].x);
                acc[h].y = fmaf(ph, vr[f].y, acc[h].y);
                acc[h].z = fmaf(ph, vr[f].z, acc[h].z);
                acc[h].w = fmaf(ph, vr[f].w, acc[h].w);
            }
        }
    }
    // denominators: sum over each head's 8 lanes
    l_lane += __shfl_xor_sync(FULL, l_lane, 1);
    l_lane += __shfl_xor_sync(FULL, l_lane, 2);
    l_lane += __shfl_xor_sync(FULL, l_lane, 4);
#pragma unroll
    for (int h = 0; h < QPG; h++) {
        const float lh = __shfl_sync(FULL, l_lane, h * G);
        float* mine = wp + (warp * QPG + h) * W;
        if (lane == 0) {
            mine[0] = m[h];
            mine[1] = lh;
        }
        *reinterpret_cast<float2*>(mine + 2 + 4 * lane) = make_float2(acc[h].x, acc[h].y);
        *reinterpret_cast<float2*>(mine + 4 + 4 * lane) = make_float2(acc[h].z, acc[h].w);
    }
    __syncthreads();
    // this split's partial for each of the 4 heads: {M, L, 0, 0, acc[HD]}
    for (int k = threadIdx.x; k < QPG * (HD + 4); k += blockDim.x) {
        const int h = k / (HD + 4), i = k % (HD + 4);
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kBW; w++)
            if (wp[(w * QPG + h) * W + 1] > 0.f) M = fmaxf(M, wp[(w * QPG + h) * W]);
        float val = 0.f;
        if (i == 0) {
            val = M;
        } else if (i == 1 || i >= 4) {
            const int src = (i == 1) ? 1 : i - 2;
#pragma unroll
            for (int w = 0; w < kBW; w++) {
                const float* pw = wp + (w * QPG + h) * W;
                if (pw[1] > 0.f) val += pw[src] * expf(pw[0] - M);
            }
        }
        part[((static_cast<size_t>(b) * H + g * QPG + h) * S + s) * (HD + 4) + i] = val;
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

constexpr int kXVec = 4;                         // float4 columns a thread holds (D <= 16384)
constexpr unsigned long long kXchgTimeoutNs = 2000000000ull;

// Thread 0: adds this row's arrival to every rank's counter at `cnt_off`, then
// waits (bounded) for all tp arrivals of exchange `seq`; false on timeout or
// when an earlier wait of the step already failed (*err set): the kernels
// queued after a failed exchange then return at once instead of each
// spinning to its own timeout.
__device__ bool xchg_row_arrive_wait(const BatchXchg& X, size_t cnt_off, unsigned long long seq, int* err) {
    if (*reinterpret_cast<volatile int*>(err)) return false;
    fence_sys();  // this CTA's stores (ordered before by the caller's barrier) reach the peers first
    for (int q = 0; q < X.tp; q++) red_add_sys_u64(X.buf[q] + cnt_off, 1ull);
    const unsigned long long target = (seq + 1) * static_cast<unsigned long long>(X.tp);
    const unsigned long long t0 = globaltimer();
    for (unsigned i = 0;; i++) {
        if (ld_acquire_sys_u64(X.buf[X.rank] + cnt_off) >= target) return true;
        if ((i & 63) == 63) {
            if (*reinterpret_cast<volatile int*>(err)) return false;
            if (globaltimer() - t0 > kXchgTimeoutNs) {
                atomicCAS(err, 0, kDevErrBatchXchg);
                return false;
            }
        }
    }
}

__global__ void k_tp_residual_rmsnorm_rows(__half* x16, float* h, const float* part, int ks, size_t part_stride,
                                           const float* g, BatchXchg X, unsigned long long xseq, int* err) {
    __shared__ float red[32];
    __shared__ int ok;
    const int b = blockIdx.x, D = X.D, n4 = D / 4, par = static_cast<int>(xseq & 1);
    const size_t row_off = bx_recv(X.B) + (static_cast<size_t>(par) * X.tp * X.B + b) * D * 4;
    const size_t sender = static_cast<size_t>(X.B) * D * 4;  // bytes between senders' blocks
    const float4* pr = reinterpret_cast<const float4*>(part + static_cast<size_t>(b) * D);
    // this rank's partial row (its split-K partials summed in order) to every rank
#pragma unroll
    for (int j = 0; j < kXVec; j++) {
        const int c = threadIdx.x + j * blockDim.x;
        if (c >= n4) break;
        float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int r = 0; r < ks; r++) {
            const float4 p = pr[r * (part_stride / 4) + c];
            a.x += p.x; a.y += p.y; a.z += p.z; a.w += p.w;
        }
        for (int q = 0; q < X.tp; q++)
            reinterpret_cast<float4*>(X.buf[q] + row_off + X.rank * sender)[c] = a;
    }
    __syncthreads();
    if (threadIdx.x == 0) ok = xchg_row_arrive_wait(X, 8 * static_cast<size_t>(b), xseq, err);
    __syncthreads();
    if (!ok) return;
    // h += the tp partial rows in rank order, then RMSNorm
    float4* hr = reinterpret_cast<float4*>(h + static_cast<size_t>(b) * D);
    const uint8_t* mine = X.buf[X.rank] + row_off;
    float4 v[kXVec];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < kXVec; j++) {
        const int c = threadIdx.x + j * blockDim.x;
        if (c >= n4) break;
        float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int q = 0; q < X.tp; q++) {
            const float4 p = __ldcg(reinterpret_cast<const float4*>(mine + q * sender) + c);
            a.x += p.x; a.y += p.y; a.z += p.z; a.w += p.w;
        }
        float4 x = hr[c];
        x.x += a.x; x.y += a.y; x.z += a.z; x.w += a.w;
        hr[c] = x;
        v[j] = x;
        ss += x.x * x.x + x.y * x.y + x.z * x.z + x.w * x.w;
    }
    ss = block_sum(ss, red);
    const float inv = 1.0f / sqrtf(ss / static_cast<float>(D) + 1e-5f);
    uint2* y = reinterpret_cast<uint2*>(x16 + static_cast<size_t>(b) * D);
#pragma unroll
    for (int j = 0; j < kXVec; j++) {
        const int c = threadIdx.x + j * blockDim.x;
        if (c >= n4) break;
        const float* gc = g + 4 * c;
        __half2 o[2] = {__floats2half2_rn((v[j].x * inv) * gc[0], (v[j].y * inv) * gc[1]),
                        __floats2half2_rn((v[j].z * inv) * gc[2], (v[j].w * inv) * gc[3])};
        y[c] = *reinterpret_cast<const uint2*>(o);
    }
}

__global__ void k_tp_argmax_rows(uint32_t* out, const float* logits, int V, int vocab_off, uint32_t* pos,
                                 BatchXchg X, unsigned long long aseq, int* err) {
    __shared__ float sv[32];
    __shared__ uint32_t si[32];
    const int b = blockIdx.x;
    const float* x = logits + static_cast<size_t>(b) * V;
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
    if (threadIdx.x != 0) return;
    for (int w = 1; w < static_cast<int>(blockDim.x >> 5); w++)
        if (better(sv[w], si[w], v, idx)) {
            v = sv[w];
            idx = si[w];
        }
    uint32_t gi = idx == 0xffffffffu ? 0xffffffffu : idx + static_cast<uint32_t>(vocab_off);
    if (X.rank == 0 && x[0] != x[0]) gi = 0x80000000u;  // sample_max keeps 0 (main.cpp:10-21)
    const int par = static_cast<int>(aseq & 1);
    const unsigned long long slot = (static_cast<unsigned long long>(gi) << 32) | __float_as_uint(v);
    const size_t off = bx_amslot(X.B) + ((static_cast<size_t>(par) * kBatchMaxTp + X.rank) * X.B + b) * 8;
    for (int q = 0; q < X.tp; q++) st_relaxed_sys_u64(X.buf[q] + off, slot);
    if (!xchg_row_arrive_wait(X, 8 * static_cast<size_t>(X.B + b), aseq, err)) return;
    bool nan0 = false;
    float bv = -INFINITY;
    uint32_t bi = 0xffffffffu;
    for (int q = 0; q < X.tp; q++) {
        const unsigned long long s = ld_relaxed_sys_u64(
            X.buf[X.rank] + bx_amslot(X.B) + ((static_cast<size_t>(par) * kBatchMaxTp + q) * X.B + b) * 8);
        const uint32_t vi = static_cast<uint32_t>(s >> 32);
        if (vi == 0x80000000u) nan0 = true;
        else if (better(__uint_as_float(static_cast<uint32_t>(s)), vi, bv, bi)) {
            bv = __uint_as_float(static_cast<uint32_t>(s));
            bi = vi;
        }
    }
    out[b] = (nan0 || bi == 0xffffffffu) ? 0u : bi;
    pos[b]++;
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

__global__ void k_fill_kv_random(BatchKV kv, uint64_t seed, int B, int L, int KV, int HD, int n_pos, int kv_off,
                                 int KV_total) {
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
            ((((static_cast<uint64_t>(b) * L + l) * 2 + which) * KV_total + kh + kv_off) * (1ull << 20) + p) * HD + d;
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

tl_status rope_cache_batch(float* qf, const float* part, int ks, size_t part_stride, const BatchKV& kv, int layer,
                           const uint32_t* pos, const float* cos_tab, const float* sin_tab, int B, int H, int KV,
                           int HD, cudaStream_t s) {
    TL_REQUIRE(ks >= 1 && HD % 2 == 0 && HD <= 2048, "rope_cache_batch: ks %d, head_dim %d", ks, HD);
    k_rope_cache_batch<<<dim3(B, H + 2 * KV), HD / 2, 0, s>>>(qf, part, ks, part_stride, kv, layer, pos, cos_tab,
                                                               sin_tab, H, KV, HD);
    return check_launch("rope_cache_batch");
}

tl_status attention_decode_batch(float* part, const float* qf, const BatchKV& kv, int layer, const uint32_t* pos,
                                 int B, int H, int KV, int HD, int S, float scale, int window, cudaStream_t s) {
    TL_REQUIRE(H == 4 * KV && S >= 1, "attention_decode_batch: H == 4 KV, S >= 1");
    const dim3 grid(S, KV, B);
    if (HD != 128) return set_error(TL_ERR_UNSUPPORTED, "attention_decode_batch: head_dim %d (128 built)", HD);
    k_attention_decode_batch<128><<<grid, kBW * 32, 0, s>>>(part, qf, kv, layer, pos, H, S, scale, window);
    return check_launch("attention_decode_batch");
}

tl_status attention_merge_batch(__half* ctx16, const float* part, int B, int H, int HD, int S, cudaStream_t s) {
    k_attention_merge_batch<<<B * H, HD, 0, s>>>(ctx16, part, H, HD, S);
    return check_launch("attention_merge_batch");
}

tl_status tp_residual_rmsnorm_rows(__half* x16, float* h, const float* part, int ks, size_t part_stride,
                                   const float* g, const BatchXchg& X, unsigned long long xseq, int* err,
                                   cudaStream_t s) {
    const int D = X.D, n4 = D / 4;
    const int threads = std::min(1024, (n4 + 31) / 32 * 32);
    TL_REQUIRE(X.tp >= 2 && X.tp <= kBatchMaxTp && X.rank >= 0 && X.rank < X.tp && ks >= 1,
               "tp_residual_rmsnorm_rows: tp %d rank %d ks %d", X.tp, X.rank, ks);
    TL_REQUIRE(D % 4 == 0 && n4 <= kXVec * threads && part_stride % 4 == 0, "tp_residual_rmsnorm_rows: width %d", D);
    for (int q = 0; q < X.tp; q++) TL_REQUIRE(X.buf[q], "tp_residual_rmsnorm_rows: rank %d buffer not mapped", q);
    k_tp_residual_rmsnorm_rows<<<X.B, threads, 0, s>>>(x16, h, part, ks, part_stride, g, X, xseq, err);
    return check_launch("tp_residual_rmsnorm_rows");
}

tl_status tp_argmax_rows(uint32_t* out, const float* logits, int V, int vocab_off, uint32_t* pos, const BatchXchg& X,
                         unsigned long long aseq, int* err, cudaStream_t s) {
    TL_REQUIRE(X.tp >= 2 && X.tp <= kBatchMaxTp && V > 0, "tp_argmax_rows: tp %d V %d", X.tp, V);
    for (int q = 0; q < X.tp; q++) TL_REQUIRE(X.buf[q], "tp_argmax_rows: rank %d buffer not mapped", q);
    k_tp_argmax_rows<<<X.B, 1024, 0, s>>>(out, logits, V, vocab_off, pos, X, aseq, err);
    return check_launch("tp_argmax_rows");
}

tl_status argmax_rows(uint32_t* out, const float* logits, int B, int V, uint32_t* pos, cudaStream_t s) {
    k_argmax_rows<<<B, 1024, 0, s>>>(out, logits, V, pos);
    return check_launch("argmax_rows");
}

tl_status fill_kv_random(const BatchKV& kv, uint64_t seed, int B, int L, int KV, int HD, int n_pos, int kv_off,
                         int KV_total, cudaStream_t s) {
    TL_REQUIRE(kv_off >= 0 && kv_off + KV <= KV_total, "fill_kv_random: heads %d + %d of %d", kv_off, KV, KV_total);
    const size_t total = static_cast<size_t>(B) * L * 2 * KV * n_pos * HD;
    if (total == 0) return TL_OK;  // no cached positions to fill
    k_fill_kv_random<<<grid_of(total, 256), 256, 0, s>>>(kv, seed, B, L, KV, HD, n_pos, kv_off, KV_total);
    return check_launch("fill_kv_random");
}

tl_status f32_to_f16(__half* w16, const float* w, size_t n, cudaStream_t s) {
    k_f32_to_f16<<<grid_of(n, 256), 256, 0, s>>>(w16, w, n);
    return check_launch("f32_to_f16");
}

}  // namespace tl
