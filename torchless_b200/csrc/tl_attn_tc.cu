// tl_attn_tc.cu -- causal GQA attention of the prompt pass (modules.cpp:58-88
// for M new queries) on the 5th-generation tensor cores.
//
// CTA = 32 queries x the 4 query heads of one kv group (kv head h / 4,
// modules.cpp:70): 128 MMA rows, row r = query r / 4, head 4 g + r % 4, so
// every K / V tile is read once for the four heads.  Per key block of 64:
//   S[128 x 64]  = Q[128 x 128] K^T   tcgen05.mma kind::f16 into tensor memory
//                                      (two S buffers: block j + 1's MMA runs
//                                      while block j's softmax reads)
//   P            = exp(S scale - m)    8 softmax warps (a row's 64 scores split
//                                      between two), fp16 into tensor memory over
//                                      S's own columns: the A operand of the next MMA
//   O[128 x 128] += P V               tcgen05.mma, O accumulates in tensor memory
// The running maximum m of a row moves only when a block's maximum exceeds it
// by more than 8 (natural log): then O and the row sum are rescaled
// (tcgen05.ld / st); otherwise exponents up to e^8 stay within fp16 and the
// final O / l is exact all the same.
// Warp roles (320 threads): warp 0 TMA producer (K in two 64-dim boxes, V
// transposed: keys contiguous), warp 1 tensor-memory owner and MMA issuer,
// warps 2-9 softmax / epilogue (warp w reads tensor-memory lanes 32 (w % 4);
// warps w and w + 4 split a row's scores and output columns).
// Every mbarrier wait is bounded (~2 s): on expiry the kernel records an
// error, the roles stop, copies and MMAs in flight drain, tensor memory is
// freed.
#include <math.h>

#include <algorithm>
#include <mutex>

#include "tl_common.cuh"
#include "tl_prefill.cuh"
#include "tl_tc.cuh"

namespace tl {
namespace {

using namespace tc;

constexpr int kQ = 32;            // queries per CTA (x 4 heads = 128 MMA rows)
constexpr int kKB = 64;           // keys per block
constexpr int kHD = 128;          // head dim (two 64-column SWIZZLE_128B boxes)
constexpr int kNst = 2;           // K / V stages
constexpr int kThreads = 320;  // warp 0 TMA, warp 1 MMA, warps 2-9 softmax
constexpr float kRescale = 11.5f;  // lazy rescale threshold, log2 units (e^8)

constexpr int kQBytes = 2 * 128 * 128;  // Q: dims 0-63 and 64-127, 128 rows x 128 B each
constexpr int kKStage = 2 * 64 * 128;   // K: dims 0-63 and 64-127, 64 keys x 128 B each
constexpr int kVStage = 128 * 128;      // V^T: 128 dims x 64 keys (128 B)
constexpr int kXchFloats = 6 * 128;     // row max of each half [2 parities][2 halves], row sums [2 halves]
// ~100 KB: two CTAs share an SM (tensor memory: 256 of its 512 columns each)
constexpr size_t kSmem = 1024 + kQBytes + static_cast<size_t>(kNst) * (kKStage + kVStage) + 256 + kXchFloats * 4;

struct AttnTcArgs {
    __half* ctx16;        // [M][H][hd]
    const __half* q16;    // [M][H][hd], rotated
    int M, p0, H, T;      // queries, first query position, q heads, cached positions p0 + M
    int window;           // > 0: keys (pos - window, pos] only
    float scale;
    int* err;
};

// 2^x (hardware approximation, ~2 ulp; 2^-inf = +0)
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// 16-byte chunk c of row r of a SWIZZLE_128B K-major tile (rows of 128 bytes)
__device__ __forceinline__ uint32_t sw128(int r, int c) {
    return static_cast<uint32_t>(r * 128 + ((c ^ (r & 7)) << 4));
}

__global__ void __launch_bounds__(kThreads, 2)
    k_attn_prefill_tc(const __grid_constant__ CUtensorMap tma_k, const __grid_constant__ CUtensorMap tma_v,
                      AttnTcArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sQ = base;
    uint8_t* sK = sQ + kQBytes;
    uint8_t* sV = sK + kNst * kKStage;
    // K and V have their own rings: a K stage is free once its S MMA is done, a V
    // stage once its P V MMA is, so K loads run ahead of the softmax
    uint64_t* k_full = reinterpret_cast<uint64_t*>(sV + kNst * kVStage);
    uint64_t* k_empty = k_full + kNst;
    uint64_t* v_full = k_empty + kNst;
    uint64_t* v_empty = v_full + kNst;
    uint64_t* s_full = v_empty + kNst;   // [2] S buffer written
    uint64_t* p_full = s_full + 2;       // [2] P buffer written (8 softmax warps)
    uint64_t* pv_done = p_full + 2;      // [2] O += P V of the buffer's block finished
    uint64_t* q_ready = pv_done + 2;     // Q tile written (8 softmax warps)
    uint64_t* mma_done = q_ready + 1;    // every MMA issued has finished
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    float* xch = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(k_full) + 256);  // kXchFloats

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = blockIdx.y;
    const int q0 = (gridDim.x - 1 - blockIdx.x) * kQ;  // the longest (latest) query tiles start first
    const int qend = min(a.M, q0 + kQ);
    const int kmax = a.p0 + qend;  // keys [0, kmax) may be attended
    const int kb0 = a.window > 0 ? max(0, a.p0 + q0 - a.window + 1) / kKB : 0;
    const int nb = (kmax + kKB - 1) / kKB - kb0;  // key blocks of this CTA (>= 1)

    if (threadIdx.x == 0) {
        for (int s = 0; s < kNst; s++) {
            bar_init(&k_full[s], 1);
            bar_init(&k_empty[s], 1);
            bar_init(&v_full[s], 1);
            bar_init(&v_empty[s], 1);
        }
        for (int b = 0; b < 2; b++) {
            bar_init(&s_full[b], 1);
            bar_init(&p_full[b], 8);  // one arrival per softmax warp
            bar_init(&pv_done[b], 1);
        }
        bar_init(q_ready, 8);
        bar_init(mma_done, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {  // O: columns 0-127, S: 128-191 and 192-255
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(tmem_slot)),
                     "r"(256));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t tO = tmem, tS0 = tmem + 128;

    auto fail = [&](int code) {
        if (!*abort_flag && a.err) atomicCAS(a.err, 0, code);
        *abort_flag = 1;
    };
    // waits poll (test_wait) rather than suspend: the hand-offs here are short and frequent
    auto wait = [&](uint64_t* b, uint32_t parity) { return bar_spin_ab(b, parity, abort_flag); };

    if (warp == 0) {
        if (lane == 0) {  // ---- TMA producer: K_j, then V_(j-1) (K runs one block ahead) ----
            int nk = 0, nv = 0;  // loads issued
            auto load_k = [&](int j) -> bool {
                const int st = j % kNst;
                if (j >= kNst && !wait(&k_empty[st], ((j / kNst) - 1) & 1)) return false;
                const int key0 = (kb0 + j) * kKB;
                bar_expect_tx(&k_full[st], kKStage);
                tma_load_2d(sK + st * kKStage, &tma_k, 0, g * a.T + key0, &k_full[st]);
                tma_load_2d(sK + st * kKStage + 8192, &tma_k, 64, g * a.T + key0, &k_full[st]);
                nk++;
                return true;
            };
            auto load_v = [&](int j) -> bool {
                const int st = j % kNst;
                if (j >= kNst && !wait(&v_empty[st], ((j / kNst) - 1) & 1)) return false;
                bar_expect_tx(&v_full[st], kVStage);
                tma_load_2d(sV + st * kVStage, &tma_v, (kb0 + j) * kKB, g * kHD, &v_full[st]);
                nv++;
                return true;
            };
            bool ok = true;
            for (int j = 0; ok && j <= nb && !*abort_flag; j++) {
                if (j < nb) ok = load_k(j);
                if (ok && j >= 1) ok = load_v(j - 1);
            }
            if (!ok) fail(kDevErrAttnLoad);
            // every copy issued lands before the CTA exits
            for (int k = max(0, nk - kNst); k < nk; k++) bar_wait(&k_full[k % kNst], (k / kNst) & 1);
            for (int k = max(0, nv - kNst); k < nv; k++) bar_wait(&v_full[k % kNst], (k / kNst) & 1);
        }
    } else if (warp == 1) {
        if (lane == 0) {  // ---- MMA issuer ----
            const uint32_t id_s = idesc_f16<64>(), id_o = idesc_f16<128>();
            bool ok = wait(q_ready, 0);
            tc_fence_after();
            auto issue_s = [&](int j) -> bool {  // S[j & 1] = Q K_j^T
                const int st = j % kNst;
                if (!wait(&k_full[st], (j / kNst) & 1)) return false;
                tc_fence_after();
                const uint32_t ts = tS0 + static_cast<uint32_t>((j & 1) * 64);
#pragma unroll
                for (int d = 0; d < 2; d++) {
                    const uint64_t da = sdesc_k128(su32(sQ + d * 16384));
                    const uint64_t db = sdesc_k128(su32(sK + st * kKStage + d * 8192));
#pragma unroll
                    for (int k = 0; k < 4; k++) umma_f16(ts, da + 2 * k, db + 2 * k, id_s, (d | k) != 0);
                }
                umma_commit(&s_full[j & 1]);
                umma_commit(&k_empty[st]);  // K of this stage is read
                return true;
            };
            auto issue_pv = [&](int j) -> bool {  // O (+)= P_j V_j, P_j in tensor memory (S_j's columns)
                if (!wait(&p_full[j & 1], (j >> 1) & 1)) return false;
                const int st = j % kNst;
                if (!wait(&v_full[st], (j / kNst) & 1)) return false;
                tc_fence_after();
                const uint32_t tp = tS0 + static_cast<uint32_t>((j & 1) * 64);
                const uint64_t db = sdesc_k128(su32(sV + st * kVStage));
#pragma unroll
                for (int k = 0; k < 4; k++) umma_f16_ts(tO, tp + 8 * k, db + 2 * k, id_o, (j | k) != 0);
                umma_commit(&pv_done[j & 1]);
                umma_commit(&v_empty[st]);  // V of this stage is read
                return true;
            };
            if (ok) ok = issue_s(0);
            if (ok && nb > 1) ok = issue_s(1);
            for (int j = 0; ok && j < nb; j++) {
                ok = issue_pv(j);
                if (ok && j + 2 < nb) ok = issue_s(j + 2);
            }
            if (!ok) fail(kDevErrAttnMma);
            umma_commit(mma_done);  // completes once every MMA issued above has
            bar_wait(mma_done, 0);
        }
    } else {
        // ---- softmax / epilogue: 8 warps.  Warps w and w + 4 share tensor-memory
        // lanes 32 (w % 4) .. (rows r); half 0 takes scores 0-31 of a block and
        // output columns 0-63, half 1 the rest.  The halves combine a block's row
        // max through shared memory at one named barrier per block (double
        // buffered by block parity), and their row sums once at the end.  A warp
        // whose wait fails keeps stepping through the loop's barriers (doing no
        // work) so that the named barrier always sees all eight warps. ----
        const int quarter = warp & 3, half = (warp - 2) >> 2;
        const int r = quarter * 32 + lane;
        const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
        const int i = q0 + (r >> 2);                // query index
        const int h = 4 * g + (r & 3);               // head
        const bool row_ok = i < a.M;
        const int pos = a.p0 + i;
        auto pair_sync = [] { asm volatile("bar.sync 2, 256;" ::: "memory"); };
        {  // this half's 64 dims of the Q row into its swizzled K-major box
            const uint4* src = reinterpret_cast<const uint4*>(a.q16 + (static_cast<size_t>(i) * a.H + h) * kHD);
#pragma unroll
            for (int c = 0; c < 8; c++) {
                const uint4 v = row_ok ? src[8 * half + c] : make_uint4(0, 0, 0, 0);
                *reinterpret_cast<uint4*>(sQ + half * 16384 + sw128(r, c)) = v;
            }
            fence_proxy_async();
            __syncwarp();
            if (lane == 0) bar_arrive(q_ready);
        }
        const float sl = a.scale * 1.4426950408889634f;  // scores x 1/sqrt(hd) (modules.cpp:79-81), log2 units
        float m_used = -INFINITY, l = 0.f;
        bool ok = true;
        for (int j = 0; j < nb; j++) {
            const int key0 = (kb0 + j) * kKB + 32 * half;  // this half's 32 keys
            // every lane waits; the outcome is warp-uniform (tensor-memory access is warp-wide)
            const bool good = ok && __all_sync(FULL, wait(&s_full[j & 1], (j >> 1) & 1));
            float s[32];
            float mxh = -INFINITY;
            if (good) {
                tc_fence_after();
                tmem_ld32(tS0 + static_cast<uint32_t>((j & 1) * 64 + 32 * half) + lane_off, s);
                const bool full = row_ok && key0 + 31 <= pos && (a.window <= 0 || key0 > pos - a.window);
                if (full) {
#pragma unroll
                    for (int c = 0; c < 32; c++) s[c] *= sl;
                } else {  // causal / window mask (rows past M: everything)
#pragma unroll
                    for (int c = 0; c < 32; c++) {
                        const int key = key0 + c;
                        const bool in = row_ok && key <= pos && (a.window <= 0 || key > pos - a.window);
                        s[c] = in ? s[c] * sl : -INFINITY;
                    }
                }
                float mt[8];  // tree max
#pragma unroll
                for (int c = 0; c < 8; c++) mt[c] = fmaxf(fmaxf(s[4 * c], s[4 * c + 1]), fmaxf(s[4 * c + 2], s[4 * c + 3]));
#pragma unroll
                for (int w = 4; w > 0; w >>= 1)
#pragma unroll
                    for (int c = 0; c < w; c++) mt[c] = fmaxf(mt[c], mt[c + w]);
                mxh = mt[0];
            }
            xch[((j & 1) * 2 + half) * 128 + r] = mxh;
            tc_fence_before();  // both halves' S reads precede P's writes into those columns
            pair_sync();
            tc_fence_after();
            if (!good) {
                if (ok) fail(kDevErrAttnS);
                ok = false;
                continue;
            }
            const float mx = fmaxf(mxh, xch[((j & 1) * 2 + (half ^ 1)) * 128 + r]);
            // lazy rescale: the running max moves when the block's exceeds it by more than kRescale
            float f = 1.f;
            bool move = false;
            if (mx > m_used + kRescale || (m_used == -INFINITY && mx > -INFINITY)) {
                if (m_used != -INFINITY) f = ex2(m_used - mx);  // O holds earlier blocks
                move = true;
            }
            if (__any_sync(FULL, move && f != 1.f)) {  // this half's 64 O columns, warp-wide
                if (!__all_sync(FULL, wait(&pv_done[(j - 1) & 1], ((j - 1) >> 1) & 1))) {
                    fail(kDevErrAttnPv);
                    ok = false;
                    continue;
                }
                tc_fence_after();
#pragma unroll 1
                for (int q = 0; q < 2; q++) {
                    float o[32];
                    const uint32_t ta = tO + lane_off + static_cast<uint32_t>(64 * half + 32 * q);
                    tmem_ld32(ta, o);
#pragma unroll
                    for (int c = 0; c < 32; c++) o[c] *= f;
                    tmem_st32(ta, o);
                }
            }
            if (move) {
                l *= f;
                m_used = mx;
            }
            // P_j as fp16 pairs into S_j's first 32 columns (this half: 16 of them); the
            // P V MMA reads it from there, and S_{j+2} (issued after it) overwrites it
            const bool live = m_used != -INFINITY;  // else every score so far is masked: P = 0
            uint32_t pk[16];
            float ps[4];
#pragma unroll
            for (int c8 = 0; c8 < 4; c8++) {
                float e[8];
#pragma unroll
                for (int u = 0; u < 8; u++) e[u] = live ? ex2(s[8 * c8 + u] - m_used) : 0.f;  // 2^-inf = 0
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    const __half2 hv = __floats2half2_rn(e[2 * u], e[2 * u + 1]);
                    pk[4 * c8 + u] = *reinterpret_cast<const uint32_t*>(&hv);
                }
                ps[c8] = ((e[0] + e[1]) + (e[2] + e[3])) + ((e[4] + e[5]) + (e[6] + e[7]));
            }
            tmem_st16(tS0 + static_cast<uint32_t>((j & 1) * 64 + 16 * half) + lane_off, pk);
            l += (ps[0] + ps[1]) + (ps[2] + ps[3]);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) bar_arrive(&p_full[j & 1]);
        }
        // row sum = half 0 + half 1; then O / l for this half's 64 columns
        xch[4 * 128 + half * 128 + r] = l;
        pair_sync();
        const float lt = xch[4 * 128 + r] + xch[5 * 128 + r];
        if (ok && __all_sync(FULL, wait(&pv_done[(nb - 1) & 1], ((nb - 1) >> 1) & 1))) {
            tc_fence_after();
            const float inv = lt > 0.f ? 1.0f / lt : 0.f;
            uint4* dst = reinterpret_cast<uint4*>(a.ctx16 + (static_cast<size_t>(i) * a.H + h) * kHD) + 8 * half;
#pragma unroll 1
            for (int q = 0; q < 2; q++) {
                float o[32];
                tmem_ld32(tO + lane_off + static_cast<uint32_t>(64 * half + 32 * q), o);
                if (row_ok) {
#pragma unroll
                    for (int c8 = 0; c8 < 4; c8++) {
                        __half2 hv[4];
#pragma unroll
                        for (int u = 0; u < 4; u++)
                            hv[u] = __floats2half2_rn(o[8 * c8 + 2 * u] * inv, o[8 * c8 + 2 * u + 1] * inv);
                        dst[4 * q + c8] = *reinterpret_cast<const uint4*>(hv);
                    }
                }
            }
        } else if (ok) {
            fail(kDevErrAttnEpi);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(256));
    }
}

// fp32 cache rows [0, T) -> fp16 K [KV][T][hd] and V transposed [KV][hd][Tp]
// (keys contiguous; columns T .. Tp - 1 zero).  Block (32 keys, 32 dims, kv head).
__global__ void k_kv_to_f16_tc(__half* k16, __half* vt16, const float* kc, const float* vc, int T, int Tp, int HD,
                               int max_seq) {
    __shared__ float tile[32][33];
    const int t0 = blockIdx.x * 32, d0 = blockIdx.y * 32, kh = blockIdx.z;
    const int tx = threadIdx.x, ty = threadIdx.y;  // 32 x 8
    for (int k = ty; k < 32; k += 8) {
        const int t = t0 + k, d = d0 + tx;
        float kv = 0.f, vv = 0.f;
        if (t < T) {
            const size_t src = (static_cast<size_t>(kh) * max_seq + t) * HD + d;
            kv = kc[src];
            vv = vc[src];
            k16[(static_cast<size_t>(kh) * T + t) * HD + d] = __float2half_rn(kv);
        }
        tile[k][tx] = vv;
    }
    __syncthreads();
    for (int k = ty; k < 32; k += 8) {  // row d0 + k of V^T, keys t0 + tx
        const int d = d0 + k, t = t0 + tx;
        vt16[(static_cast<size_t>(kh) * HD + d) * Tp + t] = __float2half_rn(tile[tx][k]);
    }
}

}  // namespace

tl_status attention_prefill_tc(__half* ctx16, const __half* q16, __half* k16, __half* vt16, const float* k_cache,
                               const float* v_cache, int M, int p0, int H, int KV, int HD, int max_seq, float scale,
                               int window, int* err, cudaStream_t s) {
    TL_REQUIRE(HD == kHD && H == 4 * KV && M > 0 && p0 >= 0, "attention_prefill_tc: head_dim %d, H %d, KV %d", HD,
               H, KV);
    const int T = p0 + M, Tp = (T + kKB - 1) / kKB * kKB;
    TL_REQUIRE(Tp <= (max_seq + kKB - 1) / kKB * kKB, "attention_prefill_tc: %d positions", T);
    TL_REQUIRE(((reinterpret_cast<uintptr_t>(ctx16) | reinterpret_cast<uintptr_t>(q16) |
                 reinterpret_cast<uintptr_t>(k16) | reinterpret_cast<uintptr_t>(vt16)) & 15) == 0,
               "attention_prefill_tc: operands must be 16-byte aligned");
    k_kv_to_f16_tc<<<dim3(Tp / 32, HD / 32, KV), dim3(32, 8), 0, s>>>(k16, vt16, k_cache, v_cache, T, Tp, HD, max_seq);
    TL_TRY(check_launch("kv_to_f16_tc"));
    CUtensorMap tk, tv;
    TL_TRY(encode_2d(&tk, k16, KV * T, HD, HD, kKB));          // rows: (kv head, key), 64-key boxes
    TL_TRY(encode_2d(&tv, vt16, KV * HD, Tp, Tp, kHD));        // rows: (kv head, dim), 128-dim boxes
    static std::once_flag once;
    static cudaError_t attr = cudaSuccess;
    std::call_once(once, [] {
        attr = cudaFuncSetAttribute(k_attn_prefill_tc, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(kSmem));
    });
    if (attr != cudaSuccess) return set_error(TL_ERR_CUDA, "attention_prefill_tc smem: %s", cudaGetErrorString(attr));
    AttnTcArgs a{ctx16, q16, M, p0, H, T, window, scale, err};
    k_attn_prefill_tc<<<dim3((M + kQ - 1) / kQ, KV), kThreads, kSmem, s>>>(tk, tv, a);
    return check_launch("attention_prefill_tc");
}

}  // namespace tl
