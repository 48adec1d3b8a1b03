// tl_decode.cu -- one decode step of the whole model in one persistent kernel.
//
// Replaces Model<int8_t>::forward + sample_max (src/model/mistral/modules.cpp:
// 118-171, main.cpp:10-21) for batch 1 with a single cooperative launch:
// one CTA per SM, 8 consumer warps and 1 producer warp.
//
// Producer warp (one elected lane): streams every weight tile this CTA owns,
// phase after phase and layer after layer, into a shared-memory ring of
// `stages` slots with cp.async.bulk (non-multicast) completing on per-slot
// mbarriers.  Weights never depend on activations, so the producer runs ahead
// across phase boundaries and grid barriers; the ring (~160 KB per SM) keeps
// HBM busy while consumers wait for the previous phase's activations.
//
// Consumer warps: per phase, stage the activation vector as an fp16 hi/lo
// pair in shared memory (x*2^k = hi + lo, ~22 significant bits); then each
// warp takes whole tiles (round robin), converts the int8 weights to fp16
// with a byte-permute splice and runs mma.m16n8k16 (f16 inputs, f32
// accumulate) with B columns {x_hi, x_lo}: rows x (hi + lo) = W x to
// near-fp32 accuracy.  Each 64-column group is accumulated separately and
// scaled by its 1/s (tensor.cpp:101-104 dequantisation applied once per
// group).  Tile row sums go to a shared buffer and, after the phase, each
// row is summed over its tiles in a fixed order and the fused epilogue runs:
//   q/k/v                       -> qkv buffer         (modules.cpp:53-55)
//   o_proj + residual           -> h                  (modules.cpp:91, 128)
//   SiLU(gate) * up             -> act                (modules.cpp:99-112)
//   down_proj + residual        -> h                  (modules.cpp:113, 142)
//   lm_head (fp32 tiles, FFMA)  -> logits + argmax    (modules.cpp:147-149)
// RMSNorm (modules.cpp:31-46) is applied while staging x.  Attention
// (modules.cpp:58-88) runs between q/k/v and o_proj on H x S CTAs
// (flash-decoding partials; the o_proj phase merges them while staging x).
//
// Phases are separated by a grid barrier (monotonic counter, acquire/release).
// Every wait is bounded by ~2 s of %globaltimer; on expiry the kernel records
// an error code, the producer drains its in-flight copies, and all CTAs exit.
#include <cuda_fp16.h>
#include <math.h>

#include <algorithm>

#include "tl_common.cuh"
#include "tl_decode.cuh"

namespace tl {
namespace {

constexpr int kConsumerWarps = 8;
// Ring slot = two consecutive tiles fetched by ONE bulk copy: a copy costs a
// roughly fixed ~0.2 us per SM, so 17 KB copies stream at 7+ TB/s where
// single 8.7 KB tiles top out near 6 (4 once consumers read them).
constexpr int kTilesPerStage = 2;
constexpr int kStageBytes = kTilesPerStage * kTileBytesI8;
constexpr int kConsumers = kConsumerWarps * 32;
constexpr int kThreads = kConsumers + 32;
constexpr unsigned long long kTimeoutNs = 2000000000ull;

enum ErrCode : int { kErrBarrier = 1, kErrFull = 2, kErrEmpty = 3, kErrFetch = 4, kErrInput = 5 };

// ---------------------------------------------------------------------------
// PTX helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ unsigned long long globaltimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}
__device__ __forceinline__ bool mbar_test(uint64_t* b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(b)), "r"(parity), "r"(20000u)  // sleep up to 20 us instead of spinning
        : "memory");
    return ok != 0;
}
// Waits for the phase with `parity` to complete; false after ~2 s.
__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t parity) {
    if (mbar_test(b, parity)) return true;
    const unsigned long long t0 = globaltimer();
    for (unsigned i = 1;; i++) {
        if (mbar_test(b, parity)) return true;
        if ((i & 255) == 0 && globaltimer() - t0 > kTimeoutNs) return false;
    }
}
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }
// Orders this thread's earlier generic-proxy shared-memory accesses before
// later async-proxy (bulk copy) accesses to the same bytes.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ int ld_volatile(const int* p) { return *reinterpret_cast<const volatile int*>(p); }

__device__ __forceinline__ uint4 lds128(const void* p) { return *reinterpret_cast<const uint4*>(p); }

// int8 weights stored as q + 128: splice bytes into the mantissa of 1024.0h
// (0x6400 | u == 1024 + u exactly) and subtract 1152 = 1024 + 128.
__device__ __forceinline__ uint32_t u8x2_lo_to_h2(uint32_t w) {
    uint32_t r = __byte_perm(w, 0x64646464u, 0x5140);
    const __half2 h = __hsub2(*reinterpret_cast<__half2*>(&r), __half2(__float2half(1152.f), __float2half(1152.f)));
    return *reinterpret_cast<const uint32_t*>(&h);
}
__device__ __forceinline__ uint32_t u8x2_hi_to_h2(uint32_t w) {
    uint32_t r = __byte_perm(w, 0x64646464u, 0x5342);
    const __half2 h = __hsub2(*reinterpret_cast<__half2*>(&r), __half2(__float2half(1152.f), __float2half(1152.f)));
    return *reinterpret_cast<const uint32_t*>(&h);
}

// D = A(16x16 f16, row) * B(16x8 f16, col) + C (f32).
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Self-check build (TL_DECODE_CHECK): bounds/alignment checks that record the
// first violation in DecodeArgs::dbg and let the caller skip the access.
#ifdef TL_DECODE_CHECK
__device__ __noinline__ void tld_report(int* dbg, int* err, int site, long long v0, long long v1) {
    if (dbg && atomicCAS(dbg, 0, site) == 0) {
        dbg[1] = static_cast<int>(v0);
        dbg[2] = static_cast<int>(v1);
    }
    atomicCAS(err, 0, 1000 + site);
}
#define TLD_OK(cond, site, v0, v1) ((cond) ? true : (tld_report(a_dbg, a_err, (site), (v0), (v1)), false))
#else
#define TLD_OK(cond, site, v0, v1) true
#endif

// ---------------------------------------------------------------------------
// Shared memory map
// ---------------------------------------------------------------------------
struct Shared {
    uint8_t* ring;     // stages * kStageBytes
    uint8_t* xbuf;     // activation staging (fp16 hi|lo, fp32 for lm_head, or attention scratch)
    float* pbuf;       // per-tile row partial sums of the current phase
    float* scratch;    // 64 floats for block reductions
    float* mw;         // [256] attention merge data
    uint64_t* full;    // [stages]
    uint64_t* empty;   // [stages]
    uint64_t* abar;    // activation fetch (one bulk copy set per phase)
    int* flags;        // [0] abort, [1] last CTA (argmax), [2] last split (attention)
    uint32_t* info;    // [0] pos, [1] token
};

__host__ __device__ constexpr size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// fp32 activation (later fp16 hi|lo in place) + RMSNorm gain right after a
// length-D activation; or attention scratch.
__host__ __device__ inline size_t xbuf_bytes(int D, int F, int HD) {
    size_t x = 4 * static_cast<size_t>(D > F ? D : F);
    if (8 * static_cast<size_t>(D) > x) x = 8 * static_cast<size_t>(D);
    const size_t attn = (3 * HD + kConsumerWarps * (HD + 2)) * 4;  // q, k, v + warp partials
    if (attn > x) x = attn;
    return align_up(x, 128);
}

__host__ __device__ inline size_t fixed_bytes(int D, int F, int HD, int pbuf_floats) {
    return xbuf_bytes(D, F, HD) + align_up(static_cast<size_t>(pbuf_floats) * 4, 128) + 64 * 4 + 256 * 4 + 64;
}

__device__ Shared carve(uint8_t* base, int stages, const DecodeArgs& a) {
    Shared s;
    size_t off = 0;
    s.ring = base;
    off += static_cast<size_t>(stages) * kStageBytes;
    s.xbuf = base + off;
    off += xbuf_bytes(a.D, a.F, a.HD);
    s.pbuf = reinterpret_cast<float*>(base + off);
    off += align_up(static_cast<size_t>(a.pbuf_floats) * 4, 128);
    s.scratch = reinterpret_cast<float*>(base + off);
    off += 64 * 4;
    s.mw = reinterpret_cast<float*>(base + off);
    off += 256 * 4;
    s.flags = reinterpret_cast<int*>(base + off);
    s.info = reinterpret_cast<uint32_t*>(base + off + 16);
    off += 64;
    s.full = reinterpret_cast<uint64_t*>(base + off);
    s.empty = s.full + stages;
    s.abar = s.empty + stages;
    return s;
}

// ---------------------------------------------------------------------------
// Work split: CTA c of G owns row blocks [n*c/G, n*(c+1)/G).
// ---------------------------------------------------------------------------
__host__ __device__ inline void split_of(int n, int c, int g, int& b0, int& b1) {
    b0 = static_cast<int>(static_cast<long long>(n) * c / g);
    b1 = static_cast<int>(static_cast<long long>(n) * (c + 1) / g);
}
__device__ __forceinline__ void split(int n, int& b0, int& b1) { split_of(n, blockIdx.x, gridDim.x, b0, b1); }

// ---------------------------------------------------------------------------
// Producer
// ---------------------------------------------------------------------------
struct Producer {
    const Shared& sh;
    int stages;
    uint32_t it = 0;  // ring slots used so far
    int slot = 0;     // it % stages, kept incrementally
    uint32_t rnd = 0; // it / stages
    bool ok = true;
    int* a_dbg = nullptr;
    int* a_err = nullptr;
    unsigned long long* trace = nullptr;
    int n_phases = 0;

    __device__ Producer(const Shared& s, int st) : sh(s), stages(st) {}

    // Trace: time of the last issue of tiled phase `ph`.
    __device__ void stamp(int ph) const {
        if (trace) trace[(static_cast<size_t>(blockIdx.x) * n_phases + ph) * kTraceEvents + 6] = globaltimer();
    }

    // This CTA's tiles of one phase, kTilesPerStage per bulk copy.
    __device__ void range(const uint8_t* base, int n_rb, int ksn, uint32_t tile_bytes) {
        int b0, b1;
        split(n_rb, b0, b1);
        const uint8_t* src = base + static_cast<size_t>(b0) * ksn * tile_bytes;
        const int n = (b1 - b0) * ksn;
        for (int i = 0; i < n && ok; i += kTilesPerStage, it++) {
            const int s = slot;
            const uint32_t round = rnd;
            if (++slot == stages) {
                slot = 0;
                rnd++;
            }
            if (round > 0 && !mbar_wait(&sh.empty[s], (round - 1) & 1)) {
                ok = false;
                break;
            }
            if (*reinterpret_cast<volatile int*>(&sh.flags[0])) {
                ok = false;
                break;
            }
            const uint32_t bytes = static_cast<uint32_t>(min(kTilesPerStage, n - i)) * tile_bytes;
            const uint8_t* gsrc = src + static_cast<size_t>(i) * tile_bytes;
            if (!TLD_OK(s >= 0 && s < stages, 2, s, stages) ||
                !TLD_OK(bytes > 0 && bytes <= kStageBytes && (bytes & 15) == 0, 3, bytes, i) ||
                !TLD_OK(static_cast<size_t>(b0 * ksn + i) * tile_bytes + bytes <=
                            static_cast<size_t>(n_rb) * ksn * tile_bytes, 4, b0 * ksn + i, n_rb * ksn) ||
                !TLD_OK((reinterpret_cast<uintptr_t>(gsrc) & 15) == 0, 5, reinterpret_cast<uintptr_t>(gsrc) & 15, 0)) {
                ok = false;
                break;
            }
            mbar_expect_tx(&sh.full[s], bytes);
            bulk_load(sh.ring + static_cast<size_t>(s) * kStageBytes, src + static_cast<size_t>(i) * tile_bytes, bytes,
                      &sh.full[s]);
        }
    }

    // Every copy issued must land before the CTA exits.
    __device__ void drain() {
        for (int s = 0; s < stages; s++) {
            if (it <= static_cast<uint32_t>(s)) continue;
            const uint32_t last = s + stages * ((it - 1 - s) / stages);
            mbar_wait(&sh.full[s], (last / stages) & 1);
        }
    }
};

// ---------------------------------------------------------------------------
// Consumers.  Tiles of a phase are dealt round-robin to the 8 warps; each
// warp computes whole tiles (8 independent group accumulators) and leaves
// the 16 (or 4) row sums of each tile in pbuf[tile][row].  After the phase
// the rows are reduced over their tiles in a fixed order, so results do not
// depend on timing.
// ---------------------------------------------------------------------------
struct Consumer {
    const DecodeArgs& a;
    const Shared& sh;
    int stages;
    int t, lane, warp;
    int slot = 0;            // ring slot of the next tile pair
    uint32_t phase_bit = 0;  // parity of its current round
    unsigned barriers = 0;
    int* a_dbg;
    int* a_err;

    __device__ Consumer(const DecodeArgs& args, const Shared& s, int st)
        : a(args), sh(s), stages(st), t(threadIdx.x), lane(threadIdx.x & 31), warp(threadIdx.x >> 5),
          a_dbg(args.dbg), a_err(args.err) {}

    int phase = 0;  // trace slot of the current phase
    __device__ __forceinline__ void stamp(int ev) const {
        if (a.trace && t == 0) {
            const int n_phases = 5 * a.n_layers + 1;
            a.trace[(static_cast<size_t>(blockIdx.x) * n_phases + phase) * kTraceEvents + ev] = globaltimer();
        }
    }

    __device__ bool aborted() const { return *reinterpret_cast<volatile int*>(&sh.flags[0]) != 0; }

    __device__ void fail(int code) {
        atomicCAS(a.err, 0, code);
        *reinterpret_cast<volatile int*>(&sh.flags[0]) = 1;
    }

    // Block-wide (sum, max) of two values in one pass.
    __device__ float2 sum_max(float s, float m) {
        s = warp_sum(s);
        m = warp_max(m);
        if (lane == 0) {
            sh.scratch[warp] = s;
            sh.scratch[8 + warp] = m;
        }
        consumer_sync();
        float rs = 0.f, rm = 0.f;
#pragma unroll
        for (int w = 0; w < kConsumerWarps; w++) {
            rs += sh.scratch[w];
            rm = fmaxf(rm, sh.scratch[8 + w]);
        }
        consumer_sync();
        return make_float2(rs, rm);
    }

    // Thread 0: bring the next phase's activation (fp32, n floats) and, for a
    // normalised phase, its RMSNorm gain (D floats at byte 4 D) into xbuf
    // with bulk copies completing on sh.abar.  Called only after every
    // consumer warp is done with xbuf.
    __device__ void fetch(const float* act, int n, const float* g) {
        if (t != 0) return;
        const uint32_t bytes = static_cast<uint32_t>(n) * 4u + (g ? static_cast<uint32_t>(a.D) * 4u : 0u);
        if (!TLD_OK(static_cast<size_t>(n) * 4 <= (g ? 4 * static_cast<size_t>(a.D) : xbuf_bytes(a.D, a.F, a.HD)) &&
                        bytes <= xbuf_bytes(a.D, a.F, a.HD), 20, n, bytes) ||
            !TLD_OK(((reinterpret_cast<uintptr_t>(act) | reinterpret_cast<uintptr_t>(g)) & 15) == 0, 21,
                    reinterpret_cast<uintptr_t>(act) & 15, reinterpret_cast<uintptr_t>(g) & 15))
            return;
        // order this thread's acquire (generic proxy) before the async-proxy
        // reads of global memory, and the CTA's earlier generic accesses to
        // xbuf (made visible to this thread by the preceding bar.sync) before
        // the async-proxy writes into it
        asm volatile("fence.proxy.async.global;" ::: "memory");
        fence_proxy_async_smem();
        mbar_expect_tx(sh.abar, bytes);
        bulk_load(sh.xbuf, act, static_cast<uint32_t>(n) * 4u, sh.abar);
        if (g) bulk_load(sh.xbuf + 4 * static_cast<size_t>(a.D), g, static_cast<uint32_t>(a.D) * 4u, sh.abar);
    }
    uint32_t fetches = 0;

    // Grid-wide barrier over all CTAs' consumers, then (thread 0) the fetch of
    // the next phase's activation; false on error/abort.
    __device__ bool grid_barrier(const float* act = nullptr, int n = 0, const float* g = nullptr) {
        barriers++;
        const unsigned target = barriers * gridDim.x;
        consumer_sync();
        stamp(4);
        if (t == 0) {
            __threadfence();
            atomicAdd(a.bar, 1u);
            const unsigned long long t0 = globaltimer();
            bool ok = true;
            for (unsigned i = 0;; i++) {
                if (ld_acquire(a.bar) >= target) break;
                if (ld_volatile(a.err)) {
                    *reinterpret_cast<volatile int*>(&sh.flags[0]) = 1;
                    ok = false;
                    break;
                }
                if ((i & 63) == 63 && globaltimer() - t0 > kTimeoutNs) {
                    fail(kErrBarrier);
                    ok = false;
                    break;
                }
                __nanosleep(32);
            }
            if (ok && act) fetch(act, n, g);
        }
        consumer_sync();
        stamp(5);
        phase++;
        stamp(0);
        return !aborted();
    }

    // Waits for the fetched activation; false (uniform) on timeout.
    __device__ bool wait_fetch() {
        const bool ok = mbar_wait(sh.abar, fetches & 1);
        fetches++;
        if (!ok) fail(kErrFetch);
        consumer_sync();
        return !aborted();
    }

    // Stages the fetched activation in place (modules.cpp:31-46 RMSNorm with
    // the fetched gain when `norm`, e = 1e-5f from modules.h:24).
    //   kHalf: column c becomes the 4-byte word {hi, lo} (fp16) of x_c 2^k,
    //          k chosen so that max|x| 2^k < 2^14; returns 2^-k.
    //   kFp32: column c becomes the normalised fp32 x_c; returns 1.
    // Each thread rewrites only the columns it read, so no register copy of
    // the vector is needed.
    enum { kHalf = 0, kFp32 = 1 };
    __device__ float stage(int d, bool norm, int mode) {
        if (!TLD_OK(4 * static_cast<size_t>(d) <= xbuf_bytes(a.D, a.F, a.HD) && (!norm || d == a.D), 30, d, norm))
            return 1.0f;
        float* xs = reinterpret_cast<float*>(sh.xbuf);
        const float* gs = xs + a.D;
        float ss = 0.f, m = 0.f;
        for (int col = t; col < d; col += kConsumers) {
            const float x = xs[col];
            ss += x * x;
            m = fmaxf(m, fabsf(norm ? x * gs[col] : x));
        }
        stamp(1);
        const float2 r = sum_max(ss, m);
        const float inv = norm ? 1.0f / sqrtf(r.x / static_cast<float>(d) + 1e-5f) : 1.0f;
        const float amax = norm ? r.y * inv * 1.0001f : r.y;  // bound on max|x|
        int e = 0;
        if (amax > 0.f) frexpf(amax, &e);
        const int k = ::min(::max(14 - e, -120), 120);
        const float sc = (mode == kHalf) ? ldexpf(1.0f, k) : 1.0f;
        // kHalf layout: in each block of 16 columns [16 b, 16 b + 16), word
        // 16 b + m (m < 8) holds {hi[16 b + 2m], hi[16 b + 2m + 1]} and word
        // 16 b + 8 + m the lo pair: exactly the mma B-operand registers of the
        // x_hi (lanes 0-3) and x_lo (lanes 4-7) columns.  A block lies in one
        // warp (columns t + 256 i), so a warp sync separates reads from writes.
        uint32_t* xw = reinterpret_cast<uint32_t*>(xs);
        for (int col = t; col < d; col += kConsumers) {
            float x = xs[col];
            if (norm) x = (x * inv) * gs[col];
            if (mode == kFp32) {
                xs[col] = x;
            } else {
                const float xsc = x * sc;
                const __half hi = __float2half_rn(xsc);
                const __half lo = __float2half_rn(xsc - __half2float(hi));
                const unsigned short hb = __half_as_ushort(hi), lb = __half_as_ushort(lo);
                const unsigned short hp = __shfl_xor_sync(FULL, hb, 1), lp = __shfl_xor_sync(FULL, lb, 1);
                __syncwarp();
                const int j = col & 15;
                uint32_t* blk = xw + (col & ~15);
                if ((j & 1) == 0) blk[j >> 1] = static_cast<uint32_t>(hb) | (static_cast<uint32_t>(hp) << 16);
                else blk[8 + (j >> 1)] = static_cast<uint32_t>(lp) | (static_cast<uint32_t>(lb) << 16);
                __syncwarp();
            }
        }
        consumer_sync();
        stamp(2);
        return (mode == kHalf) ? ldexpf(1.0f, -k) : 1.0f;
    }

    // One int8 tile (16 rows x 512 columns) into pbuf[tile][0..15].
    __device__ __forceinline__ void tile_i8(const uint8_t* st, int ks, float* out) {
        const int r = lane >> 2, c = lane & 3;
        const float* sc = reinterpret_cast<const float*>(st + 8192);
        const float4 s0 = *reinterpret_cast<const float4*>(sc + r * 8);
        const float4 s1 = *reinterpret_cast<const float4*>(sc + r * 8 + 4);
        const float4 s8a = *reinterpret_cast<const float4*>(sc + (r + 8) * 8);
        const float4 s8b = *reinterpret_cast<const float4*>(sc + (r + 8) * 8 + 4);
        const float sr[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
        const float sr8[8] = {s8a.x, s8a.y, s8a.z, s8a.w, s8b.x, s8b.y, s8b.z, s8b.w};
        // B registers of columns 512 ks + 64 g + 16 c + [0, 16): lanes 0-3 the
        // hi pairs (words 0-7 of the block), lanes 4-7 the lo pairs (8-15).
        const uint32_t* xw =
            reinterpret_cast<const uint32_t*>(sh.xbuf) + ks * kTileCols + c * 16 + (lane >= 4 ? 8 : 0);
        float yr = 0.f, yr8 = 0.f;
#pragma unroll
        for (int g = 0; g < 8; g++) {
            const uint4 ar = lds128(st + g * 1024 + lane * 16);
            const uint4 ar8 = lds128(st + g * 1024 + 512 + lane * 16);
            uint4 b0 = make_uint4(0, 0, 0, 0), b1 = make_uint4(0, 0, 0, 0);
            if (lane < 8) {
                b0 = lds128(xw + g * 64);
                b1 = lds128(xw + g * 64 + 4);
            }
            float dacc[4] = {0.f, 0.f, 0.f, 0.f};
            mma16816(dacc, u8x2_lo_to_h2(ar.x), u8x2_lo_to_h2(ar8.x), u8x2_hi_to_h2(ar.x), u8x2_hi_to_h2(ar8.x),
                     b0.x, b0.y);
            mma16816(dacc, u8x2_lo_to_h2(ar.y), u8x2_lo_to_h2(ar8.y), u8x2_hi_to_h2(ar.y), u8x2_hi_to_h2(ar8.y),
                     b0.z, b0.w);
            mma16816(dacc, u8x2_lo_to_h2(ar.z), u8x2_lo_to_h2(ar8.z), u8x2_hi_to_h2(ar.z), u8x2_hi_to_h2(ar8.z),
                     b1.x, b1.y);
            mma16816(dacc, u8x2_lo_to_h2(ar.w), u8x2_lo_to_h2(ar8.w), u8x2_hi_to_h2(ar.w), u8x2_hi_to_h2(ar8.w),
                     b1.z, b1.w);
            // column 0 holds W x_hi, column 1 W x_lo (lanes with c == 0)
            yr = fmaf(dacc[0] + dacc[1], sr[g], yr);
            yr8 = fmaf(dacc[2] + dacc[3], sr8[g], yr8);
        }
        if (c == 0) {
            out[r] = yr;
            out[r + 8] = yr8;
        }
    }

    // One fp32 lm_head tile (4 rows x 512 columns) into pbuf[tile][0..3].
    __device__ __forceinline__ void tile_f32(const uint8_t* st, int ks, float* out) {
        const float* xf = reinterpret_cast<const float*>(sh.xbuf) + ks * kTileCols + 2 * lane;
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int g = 0; g < 8; g++) {
            const float4 wa = *reinterpret_cast<const float4*>(st + g * 1024 + lane * 16);
            const float4 wb = *reinterpret_cast<const float4*>(st + g * 1024 + 512 + lane * 16);
            const float2 xv = *reinterpret_cast<const float2*>(xf + g * 64);
            acc[0] = fmaf(wa.x, xv.x, fmaf(wa.y, xv.y, acc[0]));
            acc[1] = fmaf(wa.z, xv.x, fmaf(wa.w, xv.y, acc[1]));
            acc[2] = fmaf(wb.x, xv.x, fmaf(wb.y, xv.y, acc[2]));
            acc[3] = fmaf(wb.z, xv.x, fmaf(wb.w, xv.y, acc[3]));
        }
        warp_reduce_multi<4>(acc);  // lane l holds row l / 8
        if ((lane & 7) == 0) out[lane >> 3] = acc[0];
    }

    // All tiles of one phase: warp w computes the CTA's tiles w, w + 8, ...,
    // but every warp waits on and releases EVERY ring slot in order (the
    // empty barriers expect one arrival per consumer warp).  A warp therefore
    // never waits on a slot more than one round ahead of what it has seen
    // complete, which keeps the parity waits unambiguous even though bulk
    // copies may land out of order.
    // Returns the CTA's first row block, or -1 on error (uniform over warps).
    template <bool F32>
    __device__ int run_tiles(int n_rb, int ksn, int& n_rb_local) {
        int rb0, rb1;
        split(n_rb, rb0, rb1);
        n_rb_local = rb1 - rb0;
        const int n_tiles = n_rb_local * ksn;
        const int n_slots = (n_tiles + kTilesPerStage - 1) / kTilesPerStage;
        constexpr int ROWS = F32 ? kTileRowsF32 : kTileRowsI8;
        constexpr int TB = F32 ? kTileBytesF32 : kTileBytesI8;
        int my_i = warp;            // next tile of this warp
        int my_ks = warp % ksn;     // its k-slice, kept incrementally
        for (int j = 0; j < n_slots; j++) {
            const int s = slot;
            const uint32_t par = phase_bit;
            if (++slot == stages) {
                slot = 0;
                phase_bit ^= 1u;
            }
            if (!mbar_wait(&sh.full[s], par)) {
                fail(kErrFull);
                break;
            }
            if (my_i < n_tiles && my_i / kTilesPerStage == j) {
                if (TLD_OK((my_i + 1) * ROWS <= a.pbuf_floats, 12, my_i, a.pbuf_floats)) {
                    const uint8_t* st = sh.ring + static_cast<size_t>(s) * kStageBytes + (my_i % kTilesPerStage) * TB;
                    float* out = sh.pbuf + static_cast<size_t>(my_i) * ROWS;
                    if (F32) tile_f32(st, my_ks, out);
                    else tile_i8(st, my_ks, out);
                }
                my_i += kConsumerWarps;
                my_ks += kConsumerWarps;
                while (my_ks >= ksn) my_ks -= ksn;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&sh.empty[s]);
        }
        consumer_sync();
        stamp(3);
        return aborted() ? -1 : rb0;
    }

    // Row r (local) of the phase: sum of its ksn tile partials, fixed order.
    __device__ __forceinline__ float row_sum(int rbl, int rr, int ksn, int rows) const {
        const float* p = sh.pbuf + static_cast<size_t>(rbl) * ksn * rows + rr;
        float v = 0.f;
        for (int ks = 0; ks < ksn; ks++) v += p[ks * rows];
        return v;
    }

    // int8 phase; KIND 0 q/k/v, 1 o_proj (+res), 2 gate/up, 3 down (+res).
    template <int KIND>
    __device__ bool run_i8(int n_rows, int d, float unscale, const float* res) {
        const int ksn = d / kTileCols;
        const int n_rb = (n_rows + kTileRowsI8 - 1) / kTileRowsI8;
        int nrl = 0;
        const int rb0 = run_tiles<false>(n_rb, ksn, nrl);
        if (rb0 < 0) return false;
        if (KIND == 2) {
            for (int j = t; j < nrl * 8; j += kConsumers) {
                const int rbl = j / 8, o = j % 8;
                const int row = (rb0 + rbl) * 8 + o;
                if (row < n_rows / 2) {
                    const float gate = row_sum(rbl, o, ksn, 16) * unscale;
                    const float up = row_sum(rbl, o + 8, ksn, 16) * unscale;
                    a.act[row] = (gate / (1.0f + expf(-gate))) * up;  // silu * up, kernels.cpp:98-102, 127-131
                }
            }
        } else {
            for (int j = t; j < nrl * 16; j += kConsumers) {
                const int rbl = j / 16, rr = j % 16;
                const int row = (rb0 + rbl) * 16 + rr;
                if (row < n_rows) {
                    const float v = row_sum(rbl, rr, ksn, 16) * unscale;
                    if (KIND == 0) a.qkv[row] = v;
                    else a.h[row] = v + __ldcg(res + row);
                }
            }
        }
        return true;
    }

    // Attention for (head, split) = divmod(blockIdx.x, S) (modules.cpp:58-88).
    template <int HD>
    __device__ void attention(int layer, unsigned pos) {
        constexpr int VPL = HD / 32;
        constexpr int HALF = HD / 2;
        constexpr int PF = 4;  // positions per warp in flight
        const DecodeLayer& L = a.layers[layer];
        const int S = a.splits;
        const int u = blockIdx.x;
        if (u >= a.H * S) return;
        const int h = u / S, s = u % S, kh = h / 4;  // kv head h/4 (modules.cpp:70)
        if (!TLD_OK(pos < static_cast<unsigned>(a.max_seq) && kh < a.KV && h < a.H, 40, pos, kh)) return;
        if (!TLD_OK((3 * HD + kConsumerWarps * (HD + 2)) * 4 <= static_cast<int>(xbuf_bytes(a.D, a.F, a.HD)), 41, HD, 0))
            return;
        float* q_s = reinterpret_cast<float*>(sh.xbuf);
        float* k_s = q_s + HD;
        float* v_s = k_s + HD;
        float* wp = v_s + HD;  // [8][HD + 2]
        const float* qh = a.qkv + h * HD;
        const float* kn = a.qkv + a.H * HD + kh * HD;
        const float* vn = a.qkv + (a.H + a.KV) * HD + kh * HD;
        const float* ct = a.cos_tab + static_cast<size_t>(pos) * HALF;
        const float* st = a.sin_tab + static_cast<size_t>(pos) * HALF;
        for (int i = t; i < HALF; i += kConsumers) {
            const float cc = __ldg(ct + i), sn = __ldg(st + i);
            const float xq = __ldcg(qh + i), yq = __ldcg(qh + i + HALF);
            q_s[i] = xq * cc - yq * sn;
            q_s[i + HALF] = xq * sn + yq * cc;
            const float xk = __ldcg(kn + i), yk = __ldcg(kn + i + HALF);
            k_s[i] = xk * cc - yk * sn;
            k_s[i + HALF] = xk * sn + yk * cc;
            v_s[i] = __ldcg(vn + i);
            v_s[i + HALF] = __ldcg(vn + i + HALF);
        }
        consumer_sync();
        float* kc = L.k_cache + static_cast<size_t>(kh) * a.max_seq * HD;
        float* vc = L.v_cache + static_cast<size_t>(kh) * a.max_seq * HD;
        if (s == 0 && (h & 3) == 0) {  // push_kv (inference_state.h:38-43)
            for (int i = t; i < HD; i += kConsumers) {
                kc[static_cast<size_t>(pos) * HD + i] = k_s[i];
                vc[static_cast<size_t>(pos) * HD + i] = v_s[i];
            }
        }
        const int npos = static_cast<int>(pos) + 1;
        const int chunk = (npos + S - 1) / S;
        const int p0 = s * chunk, p1 = min(npos, p0 + chunk);
        float q[VPL], acc[VPL];
#pragma unroll
        for (int j = 0; j < VPL; j++) {
            q[j] = q_s[lane * VPL + j];
            acc[j] = 0.f;
        }
        float m = -INFINITY, l = 0.f;
        for (int pb = p0 + warp; pb < p1; pb += kConsumerWarps * PF) {
            float kv[PF][VPL], vv[PF][VPL];
#pragma unroll
            for (int f = 0; f < PF; f++) {
                const int p = pb + f * kConsumerWarps;
                if (p < p1 && p != static_cast<int>(pos)) {
                    const float* kr = kc + static_cast<size_t>(p) * HD + lane * VPL;
                    const float* vr = vc + static_cast<size_t>(p) * HD + lane * VPL;
#pragma unroll
                    for (int j = 0; j < VPL; j++) {
                        kv[f][j] = __ldcg(kr + j);
                        vv[f][j] = __ldcg(vr + j);
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < VPL; j++) {
                        kv[f][j] = k_s[lane * VPL + j];
                        vv[f][j] = v_s[lane * VPL + j];
                    }
                }
            }
#pragma unroll
            for (int f = 0; f < PF; f++) {
                const int p = pb + f * kConsumerWarps;
                if (p >= p1) break;
                float dsum = 0.f;
#pragma unroll
                for (int j = 0; j < VPL; j++) dsum += kv[f][j] * q[j];
                const float sc = warp_sum(dsum) * a.attn_scale;
                const float mn = fmaxf(m, sc);
                const float corr = expf(m - mn);
                const float e = expf(sc - mn);
                l = l * corr + e;
#pragma unroll
                for (int j = 0; j < VPL; j++) acc[j] = acc[j] * corr + e * vv[f][j];
                m = mn;
            }
        }
        float* mine = wp + warp * (HD + 2);
        if (lane == 0) {
            mine[0] = m;
            mine[1] = l;
        }
#pragma unroll
        for (int j = 0; j < VPL; j++) mine[2 + lane * VPL + j] = acc[j];
        consumer_sync();
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kConsumerWarps; w++)
            if (wp[w * (HD + 2) + 1] > 0.f) M = fmaxf(M, wp[w * (HD + 2)]);
        float* part = a.attn_part + static_cast<size_t>(u) * (HD + 2);
        for (int i = t; i < HD + 2; i += kConsumers) {
            float v = 0.f;
            if (i == 0) {
                v = M;
            } else {
#pragma unroll
                for (int w = 0; w < kConsumerWarps; w++) {
                    const float lw = wp[w * (HD + 2) + 1];
                    if (lw > 0.f) v += wp[w * (HD + 2) + i] * expf(wp[w * (HD + 2)] - M);
                }
            }
            part[i] = v;
        }
        // The last split of head h to finish merges the S partials into ctx.
        consumer_sync();
        if (t == 0) {
            __threadfence();
            sh.flags[2] = (atomicAdd(a.attn_cnt + h, 1u) == static_cast<unsigned>(S) - 1);
        }
        consumer_sync();
        if (!sh.flags[2]) return;  // uniform; flags[2] is next written after a later sync
        __threadfence();
        const float* ph = a.attn_part + static_cast<size_t>(h) * S * (HD + 2);
        if (t < HD) {
            float GM = -INFINITY;
            for (int j = 0; j < S; j++)
                if (__ldcg(ph + j * (HD + 2) + 1) > 0.f) GM = fmaxf(GM, __ldcg(ph + j * (HD + 2)));
            float GL = 0.f, acc_t = 0.f;
            for (int j = 0; j < S; j++) {
                const float lj = __ldcg(ph + j * (HD + 2) + 1);
                if (lj > 0.f) {
                    const float w = expf(__ldcg(ph + j * (HD + 2)) - GM);
                    GL += lj * w;
                    acc_t += __ldcg(ph + j * (HD + 2) + 2 + t) * w;
                }
            }
            a.ctx[h * HD + t] = acc_t / GL;
        }
        if (t == 0) a.attn_cnt[h] = 0;
    }

};

template <int HD>
__global__ void __launch_bounds__(kThreads, 1) decode_step_kernel(DecodeArgs a, int stages) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    const Shared sh = carve(smem_raw, stages, a);
#ifdef TL_DECODE_CHECK
    {
        unsigned dyn;
        asm volatile("mov.u32 %0, %%dynamic_smem_size;" : "=r"(dyn));
        const size_t end = reinterpret_cast<uint8_t*>(sh.abar + 1) - smem_raw;
        int* a_dbg = a.dbg;
        int* a_err = a.err;
        if (!TLD_OK(end <= dyn, 1, static_cast<long long>(end), dyn)) return;
    }
#endif
    if (threadIdx.x == 0) {
        for (int s = 0; s < stages; s++) {
            mbar_init(&sh.full[s], 1);
            mbar_init(&sh.empty[s], kConsumerWarps);
        }
        mbar_init(sh.abar, 1);
        sh.flags[0] = 0;
        sh.flags[1] = 0;
        sh.info[0] = __ldcg(a.pos);
        sh.info[1] = __ldcg(a.token);
        fence_mbar_init();
    }
    __syncthreads();
    // Never index with an out-of-range token or position: record and stop.
    if (sh.info[0] >= static_cast<unsigned>(a.max_seq) || sh.info[1] >= static_cast<unsigned>(a.V)) {
        if (threadIdx.x == 0) atomicCAS(a.err, 0, kErrInput);
        return;
    }

    const int D = a.D, F = a.F, NQKV = (a.H + 2 * a.KV) * a.HD;
    if (threadIdx.x >= kConsumers) {
        // ---------------- producer warp ----------------
        if (threadIdx.x != kConsumers) return;
        Producer p(sh, stages);
        p.a_dbg = a.dbg;
        p.a_err = a.err;
        p.trace = a.trace;
        p.n_phases = 5 * a.n_layers + 1;
        const int ksD = D / kTileCols, ksF = F / kTileCols;
        for (int l = 0; l < a.n_layers && p.ok; l++) {
            const DecodeLayer& L = a.layers[l];
            p.range(L.qkv, (NQKV + 15) / 16, ksD, kTileBytesI8);
            p.stamp(5 * l);
            p.range(L.o, (D + 15) / 16, (a.H * a.HD) / kTileCols, kTileBytesI8);
            p.stamp(5 * l + 2);
            p.range(L.w13, (2 * F + 15) / 16, ksD, kTileBytesI8);
            p.stamp(5 * l + 3);
            p.range(L.w2, (D + 15) / 16, ksF, kTileBytesI8);
            p.stamp(5 * l + 4);
        }
        if (p.ok) p.range(a.lm_head, (a.V + 3) / 4, ksD, kTileBytesF32);
        p.stamp(5 * a.n_layers);
        p.drain();
        return;
    }

    // ---------------- consumer warps ----------------
    Consumer cw(a, sh, stages);
    cw.stamp(0);
    const unsigned pos = sh.info[0];
    const uint32_t token = sh.info[1];
    const float* emb = a.embed + static_cast<size_t>(token) * D;
    cw.fetch(emb, D, a.layers[0].g_in);  // layer 0 reads the embedding row (modules.cpp:5-7)
    for (int l = 0; l < a.n_layers; l++) {
        const DecodeLayer& L = a.layers[l];
        const float* hin = (l == 0) ? emb : a.h;
        // q/k/v = W_qkv rmsnorm(h)
        if (!cw.wait_fetch()) return;
        float un = cw.stage(D, true, Consumer::kHalf);
        if (!cw.run_i8<0>(NQKV, D, un, nullptr)) return;
        if (!cw.grid_barrier()) return;
        // attention; the last split of each head writes ctx
        cw.attention<HD>(l, pos);
        if (!cw.grid_barrier(a.ctx, a.H * a.HD, nullptr)) return;
        // h = h + W_o ctx
        if (!cw.wait_fetch()) return;
        un = cw.stage(a.H * a.HD, false, Consumer::kHalf);
        if (!cw.run_i8<1>(D, a.H * a.HD, un, hin)) return;
        if (!cw.grid_barrier(a.h, D, L.g_post)) return;
        // act = silu(W1 x) * (W3 x), x = rmsnorm(h)
        if (!cw.wait_fetch()) return;
        un = cw.stage(D, true, Consumer::kHalf);
        if (!cw.run_i8<2>(2 * F, D, un, nullptr)) return;
        if (!cw.grid_barrier(a.act, F, nullptr)) return;
        // h = h + W2 act
        if (!cw.wait_fetch()) return;
        un = cw.stage(F, false, Consumer::kHalf);
        if (!cw.run_i8<3>(D, F, un, a.h)) return;
        const float* g_next = (l + 1 < a.n_layers) ? a.layers[l + 1].g_in : a.g_final;
        if (!cw.grid_barrier(a.h, D, g_next)) return;
    }
    // logits = lm_head rmsnorm(h); token = argmax (main.cpp:10-21)
    if (!cw.wait_fetch()) return;
    cw.stage(D, true, Consumer::kFp32);
    const int ksD = D / kTileCols;
    const int n_rb = (a.V + kTileRowsF32 - 1) / kTileRowsF32;
    int nrl = 0;
    const int rb0 = cw.run_tiles<true>(n_rb, ksD, nrl);
    if (rb0 < 0) return;
    float best_v = -INFINITY;
    uint32_t best_i = 0xffffffffu;
    const int t = threadIdx.x, lane = t & 31;
    for (int j = t; j < nrl * 4; j += kConsumers) {
        const int row = rb0 * 4 + j;
        if (row < a.V) {
            const float val = cw.row_sum(j / 4, j % 4, ksD, 4);
            a.logits[row] = val;
            if (better(val, row, best_v, best_i)) {
                best_v = val;
                best_i = row;
            }
        }
    }
    cw.stamp(4);
    // CTA argmax, then the last CTA to take a ticket merges all CTAs.
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(FULL, best_v, o);
        const uint32_t oi = __shfl_xor_sync(FULL, best_i, o);
        if (better(ov, oi, best_v, best_i)) { best_v = ov; best_i = oi; }
    }
    if (lane == 0) {
        sh.scratch[cw.warp] = best_v;
        reinterpret_cast<uint32_t*>(sh.scratch)[8 + cw.warp] = best_i;
    }
    consumer_sync();
    if (t == 0) {
        float bv = sh.scratch[0];
        uint32_t bi = reinterpret_cast<uint32_t*>(sh.scratch)[8];
        for (int w = 1; w < kConsumerWarps; w++) {
            const float ov = sh.scratch[w];
            const uint32_t oi = reinterpret_cast<uint32_t*>(sh.scratch)[8 + w];
            if (better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
        }
        a.am_v[blockIdx.x] = bv;
        a.am_i[blockIdx.x] = bi;
        __threadfence();
        sh.flags[1] = (atomicAdd(a.ticket, 1u) == gridDim.x - 1);
    }
    consumer_sync();
    if (!sh.flags[1]) return;
    __threadfence();
    float bv = -INFINITY;
    uint32_t bi = 0xffffffffu;
    for (int b = t; b < static_cast<int>(gridDim.x); b += kConsumers) {
        const float ov = __ldcg(a.am_v + b);
        const uint32_t oi = __ldcg(a.am_i + b);
        if (better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(FULL, bv, o);
        const uint32_t oi = __shfl_xor_sync(FULL, bi, o);
        if (better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
    }
    consumer_sync();  // every thread has read scratch above
    if (lane == 0) {
        sh.scratch[cw.warp] = bv;
        reinterpret_cast<uint32_t*>(sh.scratch)[8 + cw.warp] = bi;
    }
    consumer_sync();
    if (t == 0) {
        for (int w = 1; w < kConsumerWarps; w++) {
            const float ov = sh.scratch[w];
            const uint32_t oi = reinterpret_cast<uint32_t*>(sh.scratch)[8 + w];
            if (better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
        }
        const float l0 = __ldcg(a.logits);
        if (l0 != l0 || bi == 0xffffffffu) bi = 0;  // sample_max keeps 0 (main.cpp:10-21)
        *a.token = bi;
        a.history[pos] = bi;
        *a.pos = pos + 1;
        // Every CTA has passed every barrier and taken its ticket: reset both.
        *a.ticket = 0;
        *a.bar = 0;
        __threadfence();
    }
}

// ---------------------------------------------------------------------------
// Repacking kernels
// ---------------------------------------------------------------------------
__global__ void k_repack_i8(uint8_t* dst, const int8_t* w1, const float* s1, const int8_t* w3, const float* s3,
                            int n, int d, int swiglu) {
    const int ksn = d / kTileCols;
    const int n_rb = swiglu ? (2 * n + 15) / 16 : (n + 15) / 16;
    const size_t chunks = static_cast<size_t>(n_rb) * 16 * (d / 16);
    for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < chunks; idx += (size_t)gridDim.x * blockDim.x) {
        const int ch = static_cast<int>(idx % (d / 16));
        const int lrow = static_cast<int>(idx / (d / 16));
        const int rb = lrow / 16, rr = lrow % 16;
        const int8_t* src;
        int row;
        if (swiglu) {
            row = rb * 8 + (rr & 7);
            src = (rr < 8) ? w1 : w3;
        } else {
            row = lrow;
            src = w1;
        }
        const int col = ch * 16, ks = col / kTileCols, cc = col % kTileCols;
        const int w = cc / 64, c = (cc % 64) / 16, r = rr & 7, half = rr >> 3;
        const int lane = 4 * r + c;
        uint8_t* out = dst + (static_cast<size_t>(rb) * ksn + ks) * kTileBytesI8 + w * 1024 + half * 512 + lane * 16;
        uint4 v = make_uint4(0x80808080u, 0x80808080u, 0x80808080u, 0x80808080u);
        if (row < n) {
            v = *reinterpret_cast<const uint4*>(src + static_cast<size_t>(row) * d + col);
            v.x ^= 0x80808080u; v.y ^= 0x80808080u; v.z ^= 0x80808080u; v.w ^= 0x80808080u;
        }
        *reinterpret_cast<uint4*>(out) = v;
    }
    // scales (already 1/s): one per (logical row, group)
    const int gpr = d / 64;
    const size_t groups = static_cast<size_t>(n_rb) * 16 * gpr;
    for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < groups; idx += (size_t)gridDim.x * blockDim.x) {
        const int gi = static_cast<int>(idx % gpr);
        const int lrow = static_cast<int>(idx / gpr);
        const int rb = lrow / 16, rr = lrow % 16;
        const float* src;
        int row;
        if (swiglu) {
            row = rb * 8 + (rr & 7);
            src = (rr < 8) ? s1 : s3;
        } else {
            row = lrow;
            src = s1;
        }
        const int ks = gi / 8, w = gi % 8;
        float* out = reinterpret_cast<float*>(dst + (static_cast<size_t>(rb) * ksn + ks) * kTileBytesI8 + 8192);
        out[rr * 8 + w] = (row < n) ? src[static_cast<size_t>(row) * gpr + gi] : 0.f;
    }
}

__global__ void k_repack_f32(uint8_t* dst, const float* w, int n, int d) {
    const int ksn = d / kTileCols;
    const int n_rb = (n + 3) / 4;
    // one thread per (rb, row pair, ks, warp, lane) -> float4
    const size_t total = static_cast<size_t>(n_rb) * 2 * ksn * 8 * 32;
    for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < total; idx += (size_t)gridDim.x * blockDim.x) {
        size_t q = idx;
        const int lane = static_cast<int>(q % 32); q /= 32;
        const int wv = static_cast<int>(q % 8); q /= 8;
        const int ks = static_cast<int>(q % ksn); q /= ksn;
        const int rp = static_cast<int>(q % 2); q /= 2;
        const int rb = static_cast<int>(q);
        const int r0 = rb * 4 + rp * 2, col = ks * kTileCols + wv * 64 + 2 * lane;
        float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
        if (r0 < n) { o.x = w[static_cast<size_t>(r0) * d + col]; o.y = w[static_cast<size_t>(r0) * d + col + 1]; }
        if (r0 + 1 < n) { o.z = w[static_cast<size_t>(r0 + 1) * d + col]; o.w = w[static_cast<size_t>(r0 + 1) * d + col + 1]; }
        float* out = reinterpret_cast<float*>(dst + (static_cast<size_t>(rb) * ksn + ks) * kTileBytesF32);
        *reinterpret_cast<float4*>(out + wv * 256 + rp * 128 + lane * 4) = o;
    }
}

}  // namespace

bool decode_kernel_fits(int D, int F, int H, int KV, int HD, int V, int grid, int max_smem, int* stages,
                        size_t* smem_bytes, int* pbuf_floats) {
    if (D % kTileCols || F % kTileCols) return false;
    if (!(HD == 64 || HD == 128 || HD == 256) || H * HD != D || grid < 1) return false;
    // partial-sum buffer: the most tiles x rows any CTA owns in one phase
    auto need = [&](int n_rows, int rows_per_tile, int d) {
        const int n_rb = (n_rows + rows_per_tile - 1) / rows_per_tile;
        const int per_cta = (n_rb + grid - 1) / grid;
        return per_cta * (d / kTileCols) * rows_per_tile;
    };
    int pb = 512;  // also the attention-merge scratch (m and l of up to 256 heads x splits)
    pb = std::max(pb, need((H + 2 * KV) * HD, kTileRowsI8, D));
    pb = std::max(pb, need(D, kTileRowsI8, H * HD));
    pb = std::max(pb, need(2 * F, kTileRowsI8, D));
    pb = std::max(pb, need(D, kTileRowsI8, F));
    pb = std::max(pb, need(V, kTileRowsF32, D));
    const size_t fixed = fixed_bytes(D, F, HD, pb);
    if (static_cast<size_t>(max_smem) <= fixed) return false;
    int st = static_cast<int>((static_cast<size_t>(max_smem) - fixed - 16) / (kStageBytes + 16));
    st = st > 24 ? 24 : st;
    if (st < 4) return false;
    *stages = st;
    *pbuf_floats = pb;
    *smem_bytes = static_cast<size_t>(st) * kStageBytes + fixed + static_cast<size_t>(st) * 16 + 16;
    return true;
}

tl_status launch_decode_step(const DecodeArgs& a, int grid, int stages, size_t smem, cudaStream_t s) {
    DecodeArgs copy = a;
    void* args[] = {&copy, &stages};
    const void* fn = nullptr;
    switch (a.HD) {
        case 64: fn = reinterpret_cast<const void*>(decode_step_kernel<64>); break;
        case 128: fn = reinterpret_cast<const void*>(decode_step_kernel<128>); break;
        case 256: fn = reinterpret_cast<const void*>(decode_step_kernel<256>); break;
        default: return set_error(TL_ERR_UNSUPPORTED, "persistent decode: head_dim %d", a.HD);
    }
    int have = 0;
    cudaFuncAttributes fa;
    if (cudaFuncGetAttributes(&fa, fn) == cudaSuccess) have = fa.maxDynamicSharedSizeBytes;
    cudaError_t e = cudaSuccess;
    if (have < static_cast<int>(smem)) {
        e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return set_error(TL_ERR_CUDA, "decode_step smem attribute: %s", cudaGetErrorString(e));
    }
    e = cudaLaunchCooperativeKernel(fn, dim3(grid), dim3(kThreads), args, smem, s);
    if (e != cudaSuccess) return set_error(TL_ERR_CUDA, "decode_step launch: %s", cudaGetErrorString(e));
    return TL_OK;
}

tl_status repack_i8(uint8_t* dst, const int8_t* w, const float* s, int n, int d, cudaStream_t st) {
    k_repack_i8<<<1024, 256, 0, st>>>(dst, w, s, nullptr, nullptr, n, d, 0);
    return check_launch("repack_i8");
}

tl_status repack_i8_swiglu(uint8_t* dst, const int8_t* w1, const float* s1, const int8_t* w3, const float* s3,
                           int n, int d, cudaStream_t st) {
    k_repack_i8<<<1024, 256, 0, st>>>(dst, w1, s1, w3, s3, n, d, 1);
    return check_launch("repack_i8_swiglu");
}

tl_status repack_f32(uint8_t* dst, const float* w, int n, int d, cudaStream_t st) {
    k_repack_f32<<<1024, 256, 0, st>>>(dst, w, n, d);
    return check_launch("repack_f32");
}

}  // namespace tl
