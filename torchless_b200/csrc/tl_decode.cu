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
// across phase boundaries and grid barriers; it also prefetches the tiles a
// few slots beyond the ring into L2, so HBM keeps streaming while consumers
// wait at a barrier.
//
// Consumer warps: per phase, stage the activation vector as three int8
// digits of a 22-bit fixed-point value (x 2^k = 2^16 d0 + 2^8 d1 + d2); then
// each warp takes whole tiles (round robin) and runs integer tensor-core
// mma.m16n8k32 (s8 x s8 -> s32) with the raw int8 weights as A and the three
// digit vectors as B columns: each 64-column group's three dot products are
// exact integers, combined in fp32 and scaled by the group's 1/s
// (tensor.cpp:101-104 dequantisation applied once per group).  fp8 (e5m2)
// weights instead (a separate instantiation): x 2^k staged as two fp16 planes
// (hi + lo, 22 significant bits), the weight bytes widened to fp16 by byte
// permutes, and fp16 mma.m16n8k16 with fp32 accumulation (exact products).  Tile row sums
// go to a shared buffer and, after the phase, each row is summed over its
// tiles in a fixed order and the fused epilogue runs:
//   q/k/v                       -> qkv buffer         (modules.cpp:53-55)
//   o_proj + residual           -> h                  (modules.cpp:91, 128)
//   SiLU(gate) * up             -> act                (modules.cpp:99-112)
//   down_proj + residual        -> h                  (modules.cpp:113, 142)
//   lm_head (fp32 tiles, FFMA)  -> logits + argmax    (modules.cpp:147-149)
// Epilogues that write a vector another phase stages also publish, per CTA,
// its partial sum of squares and max magnitude, so that the stager gets the
// RMSNorm factor (modules.cpp:31-46) and the digit scale without another
// pass.  Attention (modules.cpp:58-88) runs between q/k/v and o_proj on
// H x S CTAs (flash-decoding partials; the last split of a head merges).
//
// Phases are separated by a grid barrier (monotonic counter, acquire/release).
// Every wait is bounded by ~2 s of %globaltimer; on expiry the kernel records
// an error code, the producer drains its in-flight copies, and all CTAs exit.
#include <math.h>

#include <algorithm>

#include "tl_common.cuh"
#include "tl_decode.cuh"
#include "tl_sample.cuh"

namespace tl {
namespace {

constexpr int kConsumerWarps = 8;
// Ring slot = two consecutive tiles fetched by ONE bulk copy: a copy costs a
// roughly fixed ~0.2 us per SM, so 17 KB copies stream at 7+ TB/s where
// single 8.7 KB tiles top out near 6.
constexpr int kTilesPerStage = 2;
constexpr int kStageBytes = kTilesPerStage * kTileBytesI8;
// Ring slot bytes for the weights' format (fp8 tiles carry no scale block;
// fp32 lm_head tiles, 8192 bytes, fit either).
__host__ __device__ constexpr int stage_bytes(bool f8) { return kTilesPerStage * (f8 ? kTileBytesF8 : kTileBytesI8); }
constexpr int kConsumers = kConsumerWarps * 32;
// Warps that own each ring slot (its tile positions); the ring has a multiple
// of kConsumerWarps / kWarpsPerSlot slots so that a slot keeps its owners.
constexpr int kWarpsPerSlot = kTilesPerStage;
constexpr int kSlotsPerOwnerCycle = kConsumerWarps / kWarpsPerSlot;
constexpr int kThreads = kConsumers + 32;
// Bound of the waits on this CTA's own weight copies; waits on other CTAs or
// ranks use DecodeArgs::timeout_ns.
constexpr unsigned long long kTimeoutNs = 2000000000ull;
// Staged digits of one 64-column group: d0 (x 2^16), d1 (x 2^8), d2 rows of 64 bytes.
constexpr int kGroupDigitBytes = 192;
// Staged fp16 planes of one 64-column group (fp8 weights): hi, lo rows of 64 halves.
constexpr int kGroupHalfBytes = 256;

constexpr int kErrBarrier = kDevErrBarrier, kErrFull = kDevErrRingFull, kErrEmpty = kDevErrRingEmpty,
              kErrInput = kDevErrInput;

// ---------------------------------------------------------------------------
// PTX helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
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
// Hint: bring [src, src + bytes) into L2 (no completion, no shared memory).
__device__ __forceinline__ void prefetch_l2(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }
struct ConsumerSync {
    __device__ void operator()() const { consumer_sync(); }
};
__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ int ld_volatile(const int* p) { return *reinterpret_cast<const volatile int*>(p); }

__device__ __forceinline__ uint4 lds128(const void* p) { return *reinterpret_cast<const uint4*>(p); }

// D = A(16x32 s8, row) * B(32x8 s8, col) + D (s32).
__device__ __forceinline__ void imma16832(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// D = A(16x16 f16, row) * B(16x8 f16, col) + D (f32).
__device__ __forceinline__ void hmma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
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
    uint8_t* ring;     // stages * stage_bytes(w_f8)
    uint8_t* xbuf;     // staged activation (int8 digits, fp32 for lm_head) or attention scratch
    float* pbuf;       // per-tile row partial sums of the current phase
    float* scratch;    // 64 floats for block reductions
    uint64_t* full;    // [stages]
    uint64_t* empty;   // [stages]
    int* flags;        // [0] abort, [1] last CTA (argmax), [2] last split (attention)
    uint32_t* info;    // [0] pos, [1] token
    DecodeLayer* layers;  // [n_layers] copy of the layer table (no global load at a phase switch)
    uint64_t* xbar;       // completion of the bulk copy of published act digits into xbuf
};

__host__ __device__ constexpr size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Digits of the longest staged vector (3 bytes per column; fp16 planes for
// fp8 weights: 4), the fp32 lm_head input, or the attention scratch.
__host__ __device__ inline size_t xbuf_bytes(int D, int F, int HD, bool f8) {
    const int Dp = tile_slices(D) * kTileCols, Fp = tile_slices(F) * kTileCols;
    size_t x = (f8 ? 4 : 3) * static_cast<size_t>(Dp > Fp ? Dp : Fp);
    if (4 * static_cast<size_t>(D) > x) x = 4 * static_cast<size_t>(D);
    const size_t attn = (3 * HD + kConsumerWarps * (HD + 2)) * 4;  // q, k, v + warp partials
    if (attn > x) x = attn;
    const size_t gqa = (6 * HD + kConsumerWarps * 4 * (HD + 2)) * 4;  // 4 q, k, v + 4 heads' warp partials
    if (HD == 128 && gqa > x) x = gqa;
    return align_up(x, 128);
}

__host__ __device__ inline size_t fixed_bytes(int D, int F, int HD, bool f8, int pbuf_floats, int n_layers) {
    return xbuf_bytes(D, F, HD, f8) + align_up(static_cast<size_t>(pbuf_floats) * 4, 128) + 64 * 4 + 64 +
           static_cast<size_t>(n_layers) * sizeof(DecodeLayer) + 16;
}

__device__ Shared carve(uint8_t* base, int stages, const DecodeArgs& a) {
    Shared s;
    size_t off = 0;
    s.ring = base;
    off += static_cast<size_t>(stages) * stage_bytes(a.w_f8 != 0);
    s.xbuf = base + off;
    off += xbuf_bytes(a.D, a.F, a.HD, a.w_f8 != 0);
    s.pbuf = reinterpret_cast<float*>(base + off);
    off += align_up(static_cast<size_t>(a.pbuf_floats) * 4, 128);
    s.scratch = reinterpret_cast<float*>(base + off);
    off += 64 * 4;
    s.flags = reinterpret_cast<int*>(base + off);
    s.info = reinterpret_cast<uint32_t*>(base + off + 16);
    off += 64;
    s.full = reinterpret_cast<uint64_t*>(base + off);
    s.empty = s.full + stages;
    s.layers = reinterpret_cast<DecodeLayer*>(s.empty + stages);
    s.xbar = reinterpret_cast<uint64_t*>(s.layers + a.n_layers);
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
// This CTA's byte range of one tiled phase ("segment"): 4 per layer
// (q/k/v, o, gate/up, down) and the lm_head.
struct Seg {
    const uint8_t* src;
    int n;        // tiles
    uint32_t tb;  // bytes per tile
    int n_rb, ksn, b0;
};

__device__ Seg seg_info(const DecodeArgs& a, const DecodeLayer* layers, int s) {
    const int NQKV = (a.H + 2 * a.KV) * a.HD;
    const int ksD = tile_slices(a.D);
    Seg g;
    const uint32_t tbq = a.w_f8 ? kTileBytesF8 : kTileBytesI8;  // 8-bit tile bytes
    if (s >= 4 * a.n_layers) {
        const int rows = a.lm_8bit ? kTileRowsI8 : kTileRowsF32;
        g.src = a.lm_head;
        g.n_rb = (a.V + rows - 1) / rows;
        g.ksn = ksD;
        g.tb = a.lm_8bit ? tbq : kTileBytesF32;
    } else {
        const DecodeLayer& L = layers[s >> 2];
        g.tb = tbq;
        switch (s & 3) {
            case 0: g.src = L.qkv; g.n_rb = (NQKV + 15) / 16; g.ksn = ksD; break;
            case 1: g.src = L.o; g.n_rb = (a.D + 15) / 16; g.ksn = tile_slices(a.H * a.HD); break;
            case 2: g.src = L.w13; g.n_rb = (2 * a.F + 15) / 16; g.ksn = ksD; break;
            default: g.src = L.w2; g.n_rb = (a.D + 15) / 16; g.ksn = tile_slices(a.F); break;
        }
    }
    int b1;
    split(g.n_rb, g.b0, b1);
    g.src += static_cast<size_t>(g.b0) * g.ksn * g.tb;
    g.n = (b1 - g.b0) * g.ksn;
    return g;
}

struct Producer {
    const DecodeArgs& a;
    const Shared& sh;
    int stages;
    uint32_t it = 0;   // ring slots used so far
    int slot = 0;      // it % stages, kept incrementally
    uint32_t rnd = 0;  // it / stages
    bool ok = true;
    int n_segs;
    int* a_dbg;
    int* a_err;
    // L2 prefetch cursor, `a.prefetch` slots ahead of the copies
    int pseg = 0, pi = 0;
    Seg pg;

    __device__ Producer(const DecodeArgs& args, const Shared& s, int st)
        : a(args), sh(s), stages(st), n_segs(4 * args.n_layers + 1), a_dbg(args.dbg), a_err(args.err) {}

    // Trace: time of the last issue of tiled phase `ph`.
    __device__ void stamp(int seg) const {
        if (!a.trace) return;
        const int n_phases = 5 * a.n_layers + 1;
        const int ph = (seg >= 4 * a.n_layers) ? 5 * a.n_layers : 5 * (seg >> 2) + ((seg & 3) == 0 ? 0 : (seg & 3) + 1);
        a.trace[(static_cast<size_t>(blockIdx.x) * n_phases + ph) * kTraceEvents + 6] = globaltimer();
    }

    // Prefetch the next slot of the prefetch cursor into L2.
    __device__ void prefetch_next() {
        while (pseg < n_segs && pi >= pg.n) {
            if (++pseg < n_segs) {
                pg = seg_info(a, sh.layers, pseg);
                pi = 0;
            }
        }
        if (pseg >= n_segs) return;
        const uint32_t bytes = static_cast<uint32_t>(min(kTilesPerStage, pg.n - pi)) * pg.tb;
        prefetch_l2(pg.src + static_cast<size_t>(pi) * pg.tb, bytes);
        pi += kTilesPerStage;
    }

    __device__ void run() {
        const int sb = stage_bytes(a.w_f8 != 0);  // ring slot bytes
        if (a.prefetch > 0) {
            pg = seg_info(a, sh.layers, 0);
            for (int j = 0; j < a.prefetch; j++) prefetch_next();
        }
        for (int sg = 0; sg < n_segs && ok; sg++) {
            const Seg g = seg_info(a, sh.layers, sg);
            for (int i = 0; i < g.n && ok; i += kTilesPerStage, it++) {
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
                const uint32_t bytes = static_cast<uint32_t>(min(kTilesPerStage, g.n - i)) * g.tb;
                const uint8_t* gsrc = g.src + static_cast<size_t>(i) * g.tb;
                if (!TLD_OK(bytes > 0 && bytes <= static_cast<uint32_t>(sb) && (bytes & 15) == 0, 3, bytes, i) ||
                    !TLD_OK(static_cast<size_t>(g.b0 * g.ksn + i) * g.tb + bytes <=
                                static_cast<size_t>(g.n_rb) * g.ksn * g.tb, 4, g.b0 * g.ksn + i, g.n_rb * g.ksn) ||
                    !TLD_OK((reinterpret_cast<uintptr_t>(gsrc) & 15) == 0, 5, reinterpret_cast<uintptr_t>(gsrc) & 15,
                            0)) {
                    ok = false;
                    break;
                }
                mbar_expect_tx(&sh.full[s], bytes);
                bulk_load(sh.ring + static_cast<size_t>(s) * sb, gsrc, bytes, &sh.full[s]);
                if (a.prefetch > 0) prefetch_next();
            }
            stamp(sg);
        }
        drain();
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
// TP: tensor-parallel exchange paths compiled in; F8: fp8 (e5m2) weight
// tiles and fp16-plane staging instead of int8 tiles and digits (a separate
// instantiation, so neither format's kernel carries the other's code).
template <bool TP, bool F8>
struct Consumer {
    const DecodeArgs& a;
    const Shared& sh;
    int stages;
    int t, lane, warp;
    uint32_t ring_it = 0;    // ring slots consumed so far by the CTA (same in every warp)
    int phase = 0;           // current phase: 5 per layer (qkv, attention, o, gate/up, down), then lm_head
    int arrivals = 0;        // grid barriers this CTA has arrived at (4 per layer)
    int* a_dbg;
    int* a_err;

    __device__ Consumer(const DecodeArgs& args, const Shared& s, int st)
        : a(args), sh(s), stages(st), t(threadIdx.x), lane(threadIdx.x & 31), warp(threadIdx.x >> 5),
          a_dbg(args.dbg), a_err(args.err) {}

    __device__ __forceinline__ void stamp(int ev) const {
        if (a.trace && t == 0) {
            const int n_phases = 5 * a.n_layers + 1;
            a.trace[(static_cast<size_t>(blockIdx.x) * n_phases + phase) * kTraceEvents + ev] = globaltimer();
        }
    }

    __device__ bool aborted() const { return *reinterpret_cast<volatile int*>(&sh.flags[0]) != 0; }

    // mbar_wait that also gives up once the CTA has aborted (a warp whose
    // slot will never be filled does not sit out the whole timeout).
    __device__ bool mbar_wait_ab(uint64_t* b, uint32_t parity) const {
        if (mbar_test(b, parity)) return true;
        const unsigned long long t0 = globaltimer();
        for (unsigned i = 1;; i++) {
            if (mbar_test(b, parity)) return true;
            if ((i & 255) == 0 && (aborted() || globaltimer() - t0 > kTimeoutNs)) return false;
        }
    }

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

    // ---- phase hand-over -------------------------------------------------
    // At the end of the attention, o, gate/up and down phases each CTA
    // publishes one entry {sum, max} of the vector it wrote (sum x^2,
    // max |x g| for h; max |x| for act and ctx) into buffer (barrier % 2),
    // then arrives at the grid barrier: a monotonic counter incremented with
    // a release by one thread per CTA (after a CTA-wide bar.sync), polled
    // with acquire loads.  Every CTA waits at every barrier, so the counter
    // reaches G b exactly when all G CTAs have arrived at barrier b, and no
    // CTA is ever more than one barrier ahead of another: two statistics
    // buffers suffice.  (q/k/v hands over to attention per kv group instead.)

    // Every thread: (sum vec^2, max |vec g|) computed by this CTA (layer 0's input).
    __device__ float2 local_stats(const float* vec, int d, const float* g) {
        float ss = 0.f, mx = 0.f;
        for (int i = t; i < d; i += kConsumers) {
            const float v = __ldg(vec + i);
            ss += v * v;
            mx = fmaxf(mx, fabsf(v * __ldg(g + i)));
        }
        return sum_max(ss, mx);
    }

    // Ends the current phase: publishes this CTA's partial and arrives (all
    // consumer threads call).
    __device__ void publish(float ss, float mx) {
        const float2 r = sum_max(ss, mx);  // ends with a bar.sync after all writes of the phase
        if (t == 0) {
            a.stats[static_cast<size_t>(arrivals & 1) * kStatsCap + blockIdx.x] = r;
            // release: the CTA's writes (ordered before by the bar.sync) become
            // visible to every CTA that acquires the count past this arrival
            asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(a.bar), "r"(1u) : "memory");
        }
        arrivals++;
        stamp(4);
        phase++;
        stamp(0);
    }

    // Waits until every CTA has arrived at this CTA's latest barrier; false
    // (uniform) on error or timeout.
    __device__ bool wait_all() {
        if (t == 0) {
            const unsigned target = static_cast<unsigned>(arrivals) * gridDim.x;
            const unsigned long long t0 = globaltimer();
            for (unsigned i = 0;; i++) {
                if (ld_acquire(a.bar) >= target) break;
                if ((i & 63) == 63) {
                    if (ld_volatile(a.err)) {
                        *reinterpret_cast<volatile int*>(&sh.flags[0]) = 1;
                        break;
                    }
                    if (globaltimer() - t0 > a.timeout_ns) {
                        fail(kErrBarrier);
                        break;
                    }
                }
            }
        }
        consumer_sync();
        stamp(1);
        return !aborted();
    }

    // Every thread: (sum of the sums, max of the maxima) of the previous
    // phase's G entries, reduced in a fixed order (bit-identical in all CTAs);
    // the first 256 are loaded together.  Call after wait_all().
    __device__ float2 read_stats() const {
        const float2* s = a.stats + static_cast<size_t>((arrivals - 1) & 1) * kStatsCap;
        const int n = gridDim.x;
        float2 v[8];
#pragma unroll
        for (int j = 0; j < 8; j++) v[j] = (lane + 32 * j < n) ? __ldcg(s + lane + 32 * j) : make_float2(0.f, 0.f);
        float ss = 0.f, mx = 0.f;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            ss += v[j].x;
            mx = fmaxf(mx, v[j].y);
        }
        for (int i = lane + 256; i < n; i += 32) {
            const float2 w = __ldcg(s + i);
            ss += w.x;
            mx = fmaxf(mx, w.y);
        }
        return make_float2(warp_sum(ss), warp_max(mx));
    }

    // Converts 16 staged columns (block b) to digits and stores them.
    // X = rint(v sc) with |X| <= 2^22 comes from one fma with 1.5 2^23: the
    // sum lies in [2^23, 2^24], where floats are the integers, so its bit
    // pattern is 0x4B400000 + X (round to nearest even, as __float2int_rn).
    // The balanced digits are bytes of shifted copies of X: d2 = byte 0 of X,
    // d1 = byte 1 of X + 128 (= (X + 128) >> 8), d0 = byte 2 of X + 32896
    // (= ((X + 128) >> 8 + 128) >> 8); adding 0x4B400000 changes bytes 0
    // and 1 of none of them and byte 2 only by 0x40, removed below.
    __device__ __forceinline__ void put_digits(int b, const float (&v)[16], float sc) {
        uint32_t w0[4], w1[4], w2[4];
#pragma unroll
        for (int q = 0; q < 4; q++) {
            uint32_t x[4], y[4], z[4];
#pragma unroll
            for (int j = 0; j < 4; j++) {
                x[j] = __float_as_uint(fmaf(v[4 * q + j], sc, 12582912.0f));  // 0x4B400000 + X
                y[j] = x[j] + 128u;
                z[j] = x[j] + (32896u - 0x400000u);
            }
            w2[q] = __byte_perm(__byte_perm(x[0], x[1], 0x0040), __byte_perm(x[2], x[3], 0x0040), 0x5410);
            w1[q] = __byte_perm(__byte_perm(y[0], y[1], 0x0051), __byte_perm(y[2], y[3], 0x0051), 0x5410);
            w0[q] = __byte_perm(__byte_perm(z[0], z[1], 0x0062), __byte_perm(z[2], z[3], 0x0062), 0x5410);
        }
        uint8_t* dst = sh.xbuf + (b >> 2) * kGroupDigitBytes + (b & 3) * 16;
        *reinterpret_cast<uint4*>(dst) = make_uint4(w0[0], w0[1], w0[2], w0[3]);
        *reinterpret_cast<uint4*>(dst + 64) = make_uint4(w1[0], w1[1], w1[2], w1[3]);
        *reinterpret_cast<uint4*>(dst + 128) = make_uint4(w2[0], w2[1], w2[2], w2[3]);
    }

    // fp8 weights: 16 staged columns (block b) as two fp16 planes of
    // X = x sc: hi = fp16(X), lo = fp16(X - hi).  Column 64 j + i of plane n
    // lands at byte 256 j + 128 n + 2 i, the B-operand rows of tile_f8.
    __device__ __forceinline__ void put_halves(int b, const float (&v)[16], float sc) {
        uint32_t hi[8], lo[8];
#pragma unroll
        for (int q = 0; q < 8; q++) {
            const float x0 = v[2 * q] * sc, x1 = v[2 * q + 1] * sc;
            const __half2 h = __floats2half2_rn(x0, x1);
            const float2 hf = __half22float2(h);
            const __half2 l = __floats2half2_rn(x0 - hf.x, x1 - hf.y);
            hi[q] = *reinterpret_cast<const uint32_t*>(&h);
            lo[q] = *reinterpret_cast<const uint32_t*>(&l);
        }
        uint8_t* dst = sh.xbuf + (b >> 2) * kGroupHalfBytes + (b & 3) * 32;
        *reinterpret_cast<uint4*>(dst) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        *reinterpret_cast<uint4*>(dst + 16) = make_uint4(hi[4], hi[5], hi[6], hi[7]);
        *reinterpret_cast<uint4*>(dst + 128) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
        *reinterpret_cast<uint4*>(dst + 144) = make_uint4(lo[4], lo[5], lo[6], lo[7]);
    }

    // Stages 16 columns (block b) for the weights' tile kind.
    __device__ __forceinline__ void put_x(int b, const float (&v)[16], float sc) {
        if constexpr (F8) put_halves(b, v, sc);
        else put_digits(b, v, sc);
    }

    // Zero staged columns of block b (padding columns: their weights are zero).
    __device__ __forceinline__ void zero_x(int b) {
        const uint4 z = make_uint4(0, 0, 0, 0);
        if constexpr (F8) {
            uint8_t* dst = sh.xbuf + (b >> 2) * kGroupHalfBytes + (b & 3) * 32;
            *reinterpret_cast<uint4*>(dst) = z;
            *reinterpret_cast<uint4*>(dst + 16) = z;
            *reinterpret_cast<uint4*>(dst + 128) = z;
            *reinterpret_cast<uint4*>(dst + 144) = z;
        } else {
            uint8_t* dst = sh.xbuf + (b >> 2) * kGroupDigitBytes + (b & 3) * 16;
            *reinterpret_cast<uint4*>(dst) = z;
            *reinterpret_cast<uint4*>(dst + 64) = z;
            *reinterpret_cast<uint4*>(dst + 128) = z;
        }
    }

    // Staging exponent k for a vector with max |x| <= amax: int8 digits hold
    // |x 2^k| <= 2^22; fp16 planes keep |x 2^k| < 2^14 (finite planes, and
    // products with e5m2 weights far inside fp32).
    __device__ __forceinline__ int stage_exp(float amax) const {
        int e = 0;
        if (amax > 0.f) frexpf(amax, &e);  // amax < 2^e
        return ::min(::max((F8 ? 14 : 22) - e, -120), 120);
    }

    // Staged bytes per column.
    static constexpr int x_bytes() { return F8 ? 4 : 3; }

    // Stages the phase input x into xbuf as int8 digits of X = rint(x 2^k):
    //   X = 2^16 d0 + 2^8 d1 + d2, |X| <= 2^22, so |d0| <= 64 and d1, d2 are
    //   the balanced base-256 digits in [-128, 127].
    // x = vec, or RMSNorm(vec) = (vec * inv) * g (modules.cpp:31-46, eps 1e-5f
    // from modules.h:24) when NORM; the whole vector's (sum vec^2, max |vec g|
    // or max |vec|) is *local (layer 0) or the previous phase's published
    // partials.  Column 64 j + i of digit n lands at byte 192 j + 64 n + i,
    // the B-operand rows of tile_i8.  The statistics and the first NB blocks
    // of 16 columns per thread are loaded together (one L2 round trip).
    // Returns 2^-k.
    template <bool NORM>
    __device__ float stage_digits(const float* vec, int d, const float* g, const float2* local) {
        constexpr int NB = NORM ? 2 : 4;
        const int dp = tile_slices(d) * kTileCols;  // padded to whole tiles
        if (!TLD_OK(x_bytes() * static_cast<size_t>(dp) <= xbuf_bytes(a.D, a.F, a.HD, F8) && d % 64 == 0, 30, d,
                    dp))
            return 1.0f;
        const int nb = d / 16;
        // staged padding columns (zero weights) must be finite: zero them
        for (int b = nb + t; b < dp / 16; b += kConsumers) zero_x(b);
        const float4* v4 = reinterpret_cast<const float4*>(vec);
        const float4* g4 = reinterpret_cast<const float4*>(g);
        float4 vb[NB][4], gb[NB][4];
#pragma unroll
        for (int i = 0; i < NB; i++) {
            const int b = t + i * kConsumers;
#pragma unroll
            for (int q = 0; q < 4; q++) {
                vb[i][q] = (b < nb) ? __ldcg(v4 + 4 * b + q) : make_float4(0.f, 0.f, 0.f, 0.f);
                if (NORM) gb[i][q] = (b < nb) ? __ldg(g4 + 4 * b + q) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
        const float2 st = local ? *local : read_stats();
        stamp(5);  // the statistics (loaded with the vector's first blocks) have landed
        const float inv = NORM ? 1.0f / sqrtf(st.x / static_cast<float>(d) + 1e-5f) : 1.0f;
        const float amax = NORM ? st.y * inv * 1.0001f : st.y;  // bound on max|x|
        const int k = stage_exp(amax);
        const float sc = ldexpf(1.0f, k);
        for (int base = 0;; base += NB * kConsumers) {
#pragma unroll
            for (int i = 0; i < NB; i++) {
                const int b = t + base + i * kConsumers;
                if (b < nb) {
                    float v[16];
#pragma unroll
                    for (int q = 0; q < 4; q++) {
                        float4 f = vb[i][q];
                        if (NORM) {
                            const float4 gg = gb[i][q];
                            f = make_float4((f.x * inv) * gg.x, (f.y * inv) * gg.y, (f.z * inv) * gg.z,
                                            (f.w * inv) * gg.w);
                        }
                        v[4 * q] = f.x; v[4 * q + 1] = f.y; v[4 * q + 2] = f.z; v[4 * q + 3] = f.w;
                    }
                    put_x(b, v, sc);
                }
            }
            if (base + NB * kConsumers >= nb) break;
            // longer vectors: next batch
#pragma unroll
            for (int i = 0; i < NB; i++) {
                const int b = t + base + NB * kConsumers + i * kConsumers;
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    vb[i][q] = (b < nb) ? __ldcg(v4 + 4 * b + q) : make_float4(0.f, 0.f, 0.f, 0.f);
                    if (NORM) gb[i][q] = (b < nb) ? __ldg(g4 + 4 * b + q) : make_float4(0.f, 0.f, 0.f, 0.f);
                }
            }
        }
        consumer_sync();
        stamp(2);
        return ldexpf(1.0f, -k);
    }

    // The down_proj staging when the gate/up epilogues published act as digits
    // (act_kp) and no value overflowed this step: one bulk copy of the digits
    // into xbuf.  Otherwise (or with TP / fp8 weights) the conversion of act.
    // CTA 0 sets the next step's exponent from this step's max |act| with 2
    // bits of headroom.  Returns 2^-k.
    __device__ float stage_act(int layer) {
        const int d = a.F;
        const bool dig = !TP && !F8 && a.act_dig != nullptr && act_kp > -1000 &&
                         __ldcg(a.act_ovf + layer) != epoch + 1;
        if (blockIdx.x == 0 && warp == 0 && !TP && !F8 && a.act_dig != nullptr) {
            const float2 st = read_stats();
            if (lane == 0) a.act_k[layer] = st.y > 0.f ? stage_exp(st.y) - 2 : -1000;
        }
        if (!dig) return stage_digits<false>(a.act, d, nullptr, nullptr);
        const uint32_t bytes = static_cast<uint32_t>(x_bytes() * tile_slices(d) * kTileCols);
        if (!TLD_OK(bytes <= xbuf_bytes(a.D, a.F, a.HD, F8) && (bytes & 15) == 0, 63, bytes, 0)) return 1.0f;
        if (t == 0) {
            mbar_expect_tx(sh.xbar, bytes);
            bulk_load(sh.xbuf, a.act_dig, bytes, sh.xbar);
        }
        if (!mbar_wait(sh.xbar, xbar_uses & 1u)) fail(kErrFull);  // a 43 KB copy: never near the bound
        xbar_uses++;
        stamp(5);
        consumer_sync();
        stamp(2);
        return ldexpf(1.0f, -act_kp);
    }

    // Stages RMSNorm(vec) (modules.cpp:31-46) as fp32 for the fp32 lm_head tiles.
    __device__ void stage_f32(const float* vec, int d, const float* g) {
        if (!TLD_OK(4 * static_cast<size_t>(d) <= xbuf_bytes(a.D, a.F, a.HD, F8) && d % 4 == 0, 31, d, 0)) return;
        const float2 st = read_stats();
        const float inv = 1.0f / sqrtf(st.x / static_cast<float>(d) + 1e-5f);
        float4* xs = reinterpret_cast<float4*>(sh.xbuf);
        for (int i = t; i < d / 4; i += kConsumers) {
            const float4 v = __ldcg(reinterpret_cast<const float4*>(vec) + i);
            const float4 gg = __ldg(reinterpret_cast<const float4*>(g) + i);
            xs[i] = make_float4((v.x * inv) * gg.x, (v.y * inv) * gg.y, (v.z * inv) * gg.z, (v.w * inv) * gg.w);
        }
        consumer_sync();
        stamp(2);
    }

    // One int8 tile (16 rows x 512 columns) into pbuf[tile][0..15].
    // Lane (r, c) = (lane / 4, lane % 4).  Per 64-column group, two
    // m16n8k32 integer MMAs: A = the raw weights (the lane's 16 bytes of rows
    // r and r + 8 are its A registers), B column n < 3 = digit n of x (lanes
    // with r = n load it), columns 3..7 zero.  The s32 results are exact;
    // lane c = 0 holds columns 0, 1 (d0, d1), lane c = 1 column 2 (d2).
    __device__ __forceinline__ void tile_i8(const uint8_t* st, int ks, float* out) {
        const int r = lane >> 2, c = lane & 3;
        const float* sc = reinterpret_cast<const float*>(st + 8192);
        const float4 s0 = *reinterpret_cast<const float4*>(sc + r * 8);
        const float4 s1 = *reinterpret_cast<const float4*>(sc + r * 8 + 4);
        const float4 s8a = *reinterpret_cast<const float4*>(sc + (r + 8) * 8);
        const float4 s8b = *reinterpret_cast<const float4*>(sc + (r + 8) * 8 + 4);
        // c = 0 lanes fold d0 in as (256 d0 + d1) * 256
        const float w = (c == 0) ? 256.f : 1.f;
        const int ms = (c == 0) ? 256 : 1;
        const float sr[8] = {s0.x * w, s0.y * w, s0.z * w, s0.w * w, s1.x * w, s1.y * w, s1.z * w, s1.w * w};
        const float sr8[8] = {s8a.x * w, s8a.y * w, s8a.z * w, s8a.w * w,
                              s8b.x * w, s8b.y * w, s8b.z * w, s8b.w * w};
        const uint8_t* xd = sh.xbuf + ks * (8 * kGroupDigitBytes) + (r < 3 ? r : 0) * 64 + c * 16;
        float yr = 0.f, yr8 = 0.f;
#pragma unroll
        for (int g = 0; g < 8; g++) {
            const uint4 ar = lds128(st + g * 1024 + lane * 16);
            const uint4 ar8 = lds128(st + g * 1024 + 512 + lane * 16);
            uint4 b = make_uint4(0, 0, 0, 0);
            if (r < 3) b = lds128(xd + g * kGroupDigitBytes);
            int dd[4] = {0, 0, 0, 0};
            imma16832(dd, ar.x, ar8.x, ar.y, ar8.y, b.x, b.y);
            imma16832(dd, ar.z, ar8.z, ar.w, ar8.w, b.z, b.w);
            yr = fmaf(static_cast<float>(dd[0] * ms + dd[1]), sr[g], yr);
            yr8 = fmaf(static_cast<float>(dd[2] * ms + dd[3]), sr8[g], yr8);
        }
        yr += __shfl_xor_sync(FULL, yr, 1);
        yr8 += __shfl_xor_sync(FULL, yr8, 1);
        if (c == 0) {
            out[r] = yr;
            out[r + 8] = yr8;
        }
    }

    // One fp8 tile (16 rows x 512 columns of e5m2 bytes in tile_i8's byte
    // layout, no scales) into pbuf[tile][0..15].  Lane (r, c) holds columns
    // [16 c, 16 c + 16) of rows r and r + 8 of each 64-column group.  Word m
    // of those 16 bytes (columns 16 c + 4 m ..) becomes two fp16 pairs by
    // byte permutes (an e5m2 byte is the high byte of the same value's fp16):
    // the A registers of m16n8k16 MMA m, whose k = {2c, 2c+1} / {2c+8, 2c+9}
    // stand for columns 16 c + 4 m + {0, 1} / {2, 3}.  B column 0 is the hi
    // plane of x, 1 the lo plane (lanes with r = 0 / 1 load the same columns
    // of them), 2..7 zero.  fp16 products are exact and accumulate in fp32;
    // lane c = 0 holds row r (d0 + d1) and row r + 8 (d2 + d3).  Each group
    // starts two fresh accumulators (even / odd m), so no MMA waits on more
    // than one other and the groups' chains overlap.
    __device__ __forceinline__ void tile_f8(const uint8_t* st, int ks, float* out) {
        const int r = lane >> 2, c = lane & 3;
        const uint8_t* xh = sh.xbuf + ks * (8 * kGroupHalfBytes) + (r < 2 ? r : 0) * 128 + c * 32;
        float yr = 0.f, yr8 = 0.f;
#pragma unroll
        for (int g = 0; g < 8; g++) {
            const uint4 ar = lds128(st + g * 1024 + lane * 16);
            const uint4 ar8 = lds128(st + g * 1024 + 512 + lane * 16);
            uint4 b0 = make_uint4(0, 0, 0, 0), b1 = make_uint4(0, 0, 0, 0);
            if (r < 2) {
                b0 = lds128(xh + g * kGroupHalfBytes);
                b1 = lds128(xh + g * kGroupHalfBytes + 16);
            }
            const uint32_t wa[4] = {ar.x, ar.y, ar.z, ar.w};
            const uint32_t wb[4] = {ar8.x, ar8.y, ar8.z, ar8.w};
            const uint32_t bx[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
            float d[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
            for (int m = 0; m < 4; m++)
                hmma16816(d[m & 1], __byte_perm(wa[m], 0u, 0x1404), __byte_perm(wb[m], 0u, 0x1404),
                          __byte_perm(wa[m], 0u, 0x3424), __byte_perm(wb[m], 0u, 0x3424), bx[2 * m], bx[2 * m + 1]);
            yr += (d[0][0] + d[0][1]) + (d[1][0] + d[1][1]);
            yr8 += (d[0][2] + d[0][3]) + (d[1][2] + d[1][3]);
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

    // All tiles of one phase.  Ring slots are owned by warps: slot counter j
    // (counted over the whole step, like the producer's) holds tile positions
    // 2 j and 2 j + 1, and position q belongs to warp q % 8, so warp w takes
    // position w & 1 of every slot j with j % 4 == w / 2.  The ring has a
    // multiple of 4 slots, so a slot is always used by the same two warps:
    // only they wait on its full barrier and release it (the empty barrier
    // expects two arrivals), and a warp waits on a slot only after releasing
    // that slot's previous round itself, which keeps the parity waits
    // unambiguous.  Tile i of the phase sits at position 2 j0 + i, j0 the
    // phase's first slot (a phase with an odd tile count leaves the second
    // position of its last slot empty).
    // Returns the CTA's first row block, or -1 on error (uniform over warps).
    template <bool F32>
    __device__ int run_tiles(int n_rb, int ksn, int& n_rb_local) {
        int rb0, rb1;
        split(n_rb, rb0, rb1);
        n_rb_local = rb1 - rb0;
        const int n_tiles = n_rb_local * ksn;
        const uint32_t n_slots = static_cast<uint32_t>((n_tiles + kTilesPerStage - 1) / kTilesPerStage);
        constexpr int ROWS = F32 ? kTileRowsF32 : kTileRowsI8;
        constexpr int TB = F32 ? kTileBytesF32 : (F8 ? kTileBytesF8 : kTileBytesI8);
        const uint32_t first = ring_it, end = ring_it + n_slots;
        const int pos_k = warp & 1;  // this warp's position in its slots
        static_assert(kWarpsPerSlot == 2 && kSlotsPerOwnerCycle == 4, "slot ownership below assumes 8 warps, 2 tiles");
        for (uint32_t j = first + ((static_cast<uint32_t>(warp >> 1) - first) & 3u); j < end; j += 4) {
            const int s = static_cast<int>(j % static_cast<uint32_t>(stages));
            const uint32_t par = (j / static_cast<uint32_t>(stages)) & 1u;
            if (!mbar_wait_ab(&sh.full[s], par)) {
                fail(kErrFull);
                break;
            }
            const int ti = 2 * static_cast<int>(j - first) + pos_k;
            if (ti < n_tiles && TLD_OK((ti + 1) * ROWS <= a.pbuf_floats, 12, ti, a.pbuf_floats)) {
                const uint8_t* st = sh.ring + static_cast<size_t>(s) * stage_bytes(F8) + pos_k * TB;
                float* out = sh.pbuf + static_cast<size_t>(ti) * ROWS;
                const int ks = ti % ksn;
                if constexpr (F32) tile_f32(st, ks, out);
                else if constexpr (F8) tile_f8(st, ks, out);
                else tile_i8(st, ks, out);
                if (j < first + 4) stamp(7);  // warp 0's first tile of the phase is done
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&sh.empty[s]);
        }
        ring_it = end;
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
    // Kinds 1 and 3 publish (sum h^2, max |h g_next|) of the rows they wrote,
    // kind 2 (0, max |act|); kind 0 instead adds its rows to each kv group's
    // ready count (qkv_cnt), which attention waits on.
    template <int KIND>
    __device__ bool run_i8(int n_rows, int d, float unscale, const float* res, const float* g_next, int layer = 0) {
        const int ksn = tile_slices(d);
        constexpr bool xchg = (KIND == 1 || KIND == 3) && TP;  // partial rows go to every rank
        const int n_rb = (n_rows + kTileRowsI8 - 1) / kTileRowsI8;
        // the first epilogue row's residual and next-norm gain, loaded before
        // the tiles so the epilogue does not wait on them
        float res0 = 0.f, g0 = 0.f;
        if (KIND == 1 || KIND == 3) {
            int b0, b1;
            split(n_rb, b0, b1);
            const int row = b0 * 16 + t;
            if (t < (b1 - b0) * 16 && row < n_rows) {
                res0 = __ldcg(res + row);
                g0 = __ldg(g_next + row);
            }
        }
        int nrl = 0;
        const int rb0 = run_tiles<false>(n_rb, ksn, nrl);
        if (rb0 < 0) return false;
        float ss = 0.f, mx = 0.f;
        if (KIND == 2) {
            // with a predicted exponent, also the act digits as the down staging
            // lays them out (put_digits' arithmetic), column c of digit n at byte
            // 192 (c / 64) + 64 n + c % 64
            act_kp = (!TP && !F8 && a.act_dig) ? a.act_k[layer] : -1000;
            const bool dig = act_kp > -1000;
            const float sc = dig ? ldexpf(1.0f, act_kp) : 0.f;
            bool ovf = false;
            for (int j = t; j < nrl * 8; j += kConsumers) {
                const int rbl = j / 8, o = j % 8;
                const int row = (rb0 + rbl) * 8 + o;
                if (row < n_rows / 2) {
                    const float gate = row_sum(rbl, o, ksn, 16) * unscale;
                    const float up = row_sum(rbl, o + 8, ksn, 16) * unscale;
                    const float v = (gate / (1.0f + expf(-gate))) * up;  // silu * up, kernels.cpp:98-102, 127-131
                    a.act[row] = v;
                    mx = fmaxf(mx, fabsf(v));
                    if (dig) {
                        if (!(fabsf(v * sc) <= 4194304.0f)) {  // |X| <= 2^22, and not NaN
                            ovf = true;
                        } else {
                            const uint32_t x = __float_as_uint(fmaf(v, sc, 12582912.0f));  // 0x4B400000 + X
                            uint8_t* dst = a.act_dig + 192 * (row / 64) + row % 64;
                            dst[0] = static_cast<uint8_t>((x + (32896u - 0x400000u)) >> 16);
                            dst[64] = static_cast<uint8_t>((x + 128u) >> 8);
                            dst[128] = static_cast<uint8_t>(x);
                        }
                    }
                }
            }
            if (ovf) a.act_ovf[layer] = epoch + 1;  // ordered before the arrival's release
        } else if (xchg) {
            // tensor parallel: this rank's partial rows to every rank, then
            // the CTA's rows summed over the ranks (every rank's CTA owns the
            // same rows, so each rank ends with the same h)
            const unsigned tag = xchg_tag();
            for (int j = t; j < nrl * 16; j += kConsumers) {
                const int row = (rb0 + j / 16) * 16 + j % 16;
                if (row < n_rows) xchg_send(row, row_sum(j / 16, j % 16, ksn, 16) * unscale, tag);
            }
            for (int j = t; j < nrl * 16; j += kConsumers) {
                const int row = (rb0 + j / 16) * 16 + j % 16;
                if (row < n_rows) {
                    const bool first = (j == t);
                    float hv = first ? res0 : __ldcg(res + row);
                    if (!xchg_gather(row, tag, hv)) break;
                    a.h[row] = hv;
                    ss += hv * hv;
                    mx = fmaxf(mx, fabsf(hv * (first ? g0 : __ldg(g_next + row))));
                }
            }
            xk++;
        } else {
            for (int j = t; j < nrl * 16; j += kConsumers) {
                const int rbl = j / 16, rr = j % 16;
                const int row = (rb0 + rbl) * 16 + rr;
                if (row < n_rows) {
                    const float v = row_sum(rbl, rr, ksn, 16) * unscale;
                    if (KIND == 0) {
                        a.qkv[row] = v;
                        // kv group of the row: q head / 4, or the k / v head
                        const int hh = row / a.HD;
                        const int grp = hh < a.H ? hh / 4 : (hh < a.H + a.KV ? hh - a.H : hh - a.H - a.KV);
                        atomicAdd(reinterpret_cast<unsigned*>(sh.scratch) + 32 + grp, 1u);
                    } else {
                        const bool first = (j == t);
                        const float hv = v + (first ? res0 : __ldcg(res + row));
                        a.h[row] = hv;
                        ss += hv * hv;
                        mx = fmaxf(mx, fabsf(hv * (first ? g0 : __ldg(g_next + row))));
                    }
                }
            }
        }
        if (KIND == 0) {
            // release each touched group's row count (after the bar.sync, so
            // every thread's rows are covered), then clear the counts
            consumer_sync();
            if (t < a.KV) {
                unsigned* cnt = reinterpret_cast<unsigned*>(sh.scratch) + 32 + t;
                if (*cnt) {
                    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(a.qkv_cnt + t), "r"(*cnt) : "memory");
                    *cnt = 0;
                }
            }
            stamp(4);
            phase++;
            stamp(0);
        } else {
            publish(ss, mx);
        }
        return !aborted();
    }

    // ---- tensor-parallel exchange (o_proj and down_proj partials) ----------
    // Exchange xk of a step (2 per layer): every rank's CTA c computes the
    // partial sums of the rows it owns (the same rows on every rank) over the
    // rank's slice of the inner dimension, and stores each into slot
    // [xk % 2][its rank][row] of every rank's receive buffer as one 8-byte
    // word {value, tag}, tag = the exchange's number in the whole run + 1
    // (single-copy atomic, so a reader sees either the old word or the new
    // one: no fence, no counter).  CTA c then polls its rows' tp words in its
    // own buffer until all carry the tag and sums them in rank order onto the
    // residual, so every rank holds bit-identical rows, and publishes its
    // statistics like the single-GPU epilogue; the local grid barrier follows.
    // Two slot sets suffice: a rank writes exchange x + 2 only after it has
    // gathered x + 1 from every rank, and every rank sends x + 1 only after
    // all its CTAs gathered x (its grid barrier lies between).
    int xk = 0;          // exchanges this CTA has completed in this step
    unsigned epoch = 0;  // steps run before this one
    int act_kp = -1000;  // exponent of the act digits the gate/up epilogue published (< -999: none)
    uint32_t xbar_uses = 0;

    __device__ __forceinline__ unsigned xchg_tag() const {
        return static_cast<unsigned>((static_cast<unsigned long long>(epoch) * 2 * a.n_layers + xk + 1) & 0xffffffffull);
    }
    __device__ __forceinline__ size_t xchg_off(int src_rank, int row) const {
        return kXchgRecv + ((static_cast<size_t>(xk & 1) * a.tp_size + src_rank) * a.D + row) * 8;
    }
    __device__ __forceinline__ void xchg_send(int row, float v, unsigned tag) const {
        const unsigned long long w = (static_cast<unsigned long long>(tag) << 32) | __float_as_uint(v);
        const size_t off = xchg_off(a.tp_rank, row);
        for (int q = 0; q < a.tp_size; q++) st_relaxed_sys_u64(a.xpeer[q] + off, w);
    }
    // acc += the tp partials of `row` in rank order; false (and the CTA
    // aborted) when a word has not arrived within the timeout.
    __device__ bool xchg_gather(int row, unsigned tag, float& acc) {
        const uint8_t* mine = a.xpeer[a.tp_rank];
        const unsigned long long t0 = globaltimer();
        for (int q = 0; q < a.tp_size; q++) {
            const size_t off = xchg_off(q, row);
            unsigned long long w = ld_relaxed_sys_u64(mine + off);
            for (unsigned i = 1; static_cast<unsigned>(w >> 32) != tag; i++) {
                if ((i & 63) == 0) {
                    if (aborted()) return false;
                    if (ld_volatile(a.err) || globaltimer() - t0 > a.timeout_ns) {
                        fail(kErrBarrier);
                        return false;
                    }
                }
                w = ld_relaxed_sys_u64(mine + off);
            }
            acc += __uint_as_float(static_cast<unsigned>(w));
        }
        return true;
    }

    // The query at `pos` attends to positions [attn_lo(pos), pos]: all of them
    // (modules.cpp:75-83), or the last a.window with a sliding window.
    __device__ int attn_lo(unsigned pos) const {
        return a.window > 0 ? ::max(0, static_cast<int>(pos) + 1 - a.window) : 0;
    }
    __device__ int attn_span(unsigned pos) const { return static_cast<int>(pos) + 1 - attn_lo(pos); }
    // GQA attention (attention_gqa) at this position?
    __device__ bool gqa(unsigned pos) const {
        return a.HD == 128 && a.gqa_splits > 0 && attn_span(pos) >= a.gqa_from;
    }
    // Splits over the attended positions: one per a.gqa_rows (GQA, at most
    // a.gqa_splits) or per a.split_rows (per head, at most a.splits).
    __device__ int attn_splits(unsigned pos) const {
        const int span = attn_span(pos);
        if (gqa(pos)) return ::min(a.gqa_splits, (span + a.gqa_rows - 1) / a.gqa_rows);
        return ::min(a.splits, (span + a.split_rows - 1) / a.split_rows);
    }

    // Thread 0 polls until kv group g's q, k and v rows of this layer are
    // written (qkv_cnt); every consumer thread returns false on error.
    __device__ bool wait_qkv(int g, int layer) {
        if (t == 0) {
            const unsigned target = static_cast<unsigned>(layer + 1) * 6 * a.HD;
            const unsigned long long t0 = globaltimer();
            for (unsigned i = 0;; i++) {
                if (ld_acquire(a.qkv_cnt + g) >= target) break;
                if ((i & 63) == 63) {
                    if (ld_volatile(a.err)) {
                        *reinterpret_cast<volatile int*>(&sh.flags[0]) = 1;
                        break;
                    }
                    if (globaltimer() - t0 > a.timeout_ns) {
                        fail(kErrBarrier);
                        break;
                    }
                }
            }
        }
        consumer_sync();
        return !aborted();
    }

    // Thread 0 of an attention CTA: hint its K and V position range of the
    // layer into L2, ahead of the attention phase (cached rows are from
    // earlier steps, so they can be fetched before q/k/v exist).
    template <int HD>
    __device__ void prefetch_kv(int layer, unsigned pos) const {
        const int S = attn_splits(pos);
        const int u = blockIdx.x;
        const int units = gqa(pos) ? a.KV * S : a.H * S;
        if (t != 0 || u >= units || pos == 0) return;
        const int s = u % S, kh = gqa(pos) ? u / S : (u / S) / 4;
        const int npos = static_cast<int>(pos);  // rows .. pos - 1 are cached
        const int chunk = (attn_span(pos) + S - 1) / S;
        const int p0 = attn_lo(pos) + s * chunk, p1 = min(npos, p0 + chunk);
        if (p1 <= p0) return;
        const DecodeLayer& L = sh.layers[layer];
        const size_t off = (static_cast<size_t>(kh) * a.max_seq + p0) * HD;
        const uint32_t bytes = static_cast<uint32_t>(::min(p1 - p0, a.kv_prefetch_rows)) * HD * 4;
        prefetch_l2(L.k_cache + off, bytes);
        prefetch_l2(L.v_cache + off, bytes);
    }

    // GQA attention (hd 128, H = 4 KV; modules.cpp:58-88, kv head h / 4):
    // CTA u < KV S takes kv group g = u / S and position split s = u % S for
    // the group's 4 query heads, so each K / V row is read once.  Warp w takes
    // groups of 8 positions; lane l holds dims 4 l .. 4 l + 3 of q, K, V and
    // of the 4 heads' accumulators.  The 32 dot products of a group (4 heads x
    // 8 positions) are reduced together (warp_reduce_multi): lane l then
    // holds the score of (head l / 8, position l % 8), and the online softmax
    // runs per 8-lane group.  With one split the CTA writes ctx of its 4
    // heads; otherwise each split writes its partial {M, L, 0, 0, acc} and the
    // last split of the group to finish (ticket attn_cnt[g]) merges them into
    // ctx.  mx = max |ctx| written by this thread (0 if none).
    template <int HD>
    __device__ bool attention_gqa(int layer, unsigned pos, float& mx) {
        mx = 0.f;
        if constexpr (HD != 128) {
            return true;
        } else {
            constexpr int QPG = 4, G = 8, W = HD + 2, HALF = HD / 2, PW = HD + 4;
            const DecodeLayer& L = sh.layers[layer];
            const int S = attn_splits(pos);
            const int u = blockIdx.x;
            if (u >= a.KV * S) return true;
            const int g = u / S, s = u % S;
            if (!TLD_OK(pos < static_cast<unsigned>(a.max_seq) && a.H == QPG * a.KV, 40, pos, g)) return true;
            if (!TLD_OK((6 * HD + kConsumerWarps * QPG * W) * 4 <= static_cast<int>(xbuf_bytes(a.D, a.F, a.HD, F8)), 41,
                        HD, 1))
                return true;
            if (!wait_qkv(g, layer)) return false;
            float* q_s = reinterpret_cast<float*>(sh.xbuf);  // [4][HD]
            float* k_s = q_s + QPG * HD;
            float* v_s = k_s + HD;
            float* wp = v_s + HD;  // [8 warps][4 heads][W]
            // RoPE (kernels.cpp:78-95) of the group's 4 q heads and its k head; v as is
            const float* ct = a.cos_tab + static_cast<size_t>(pos) * HALF;
            const float* st = a.sin_tab + static_cast<size_t>(pos) * HALF;
            for (int i = t; i < (QPG + 1) * HALF; i += kConsumers) {
                const int hh = i / HALF, c = i % HALF;
                const float* src = a.qkv + (hh < QPG ? (g * QPG + hh) * HD : a.H * HD + g * HD);
                float* dst = hh < QPG ? q_s + hh * HD : k_s;
                const float cc = __ldg(ct + c), sn = __ldg(st + c);
                const float x = __ldcg(src + c), y = __ldcg(src + c + HALF);
                dst[c] = x * cc - y * sn;
                dst[c + HALF] = x * sn + y * cc;
            }
            const float* vn = a.qkv + (a.H + a.KV) * HD + g * HD;
            for (int i = t; i < HD; i += kConsumers) v_s[i] = __ldcg(vn + i);
            consumer_sync();
            float* kc = L.k_cache + static_cast<size_t>(g) * a.max_seq * HD;
            float* vc = L.v_cache + static_cast<size_t>(g) * a.max_seq * HD;
            if (s == 0) {  // push_kv (inference_state.h:38-43)
                for (int i = t; i < HD; i += kConsumers) {
                    kc[static_cast<size_t>(pos) * HD + i] = k_s[i];
                    vc[static_cast<size_t>(pos) * HD + i] = v_s[i];
                }
            }
            const int npos = static_cast<int>(pos) + 1;
            const int chunk = (attn_span(pos) + S - 1) / S;
            const int p0 = attn_lo(pos) + s * chunk, p1 = min(npos, p0 + chunk);
            float4 q[QPG], acc[QPG];
            float m[QPG];
#pragma unroll
            for (int h = 0; h < QPG; h++) {
                q[h] = reinterpret_cast<const float4*>(q_s + h * HD)[lane];
                acc[h] = make_float4(0.f, 0.f, 0.f, 0.f);
                m[h] = -INFINITY;
            }
            const int my_h = lane >> 3, my_f = lane & 7;
            float l_lane = 0.f;  // softmax denominator share of (head my_h, position slot my_f)
            for (int pb = p0 + warp * G; pb < p1; pb += kConsumerWarps * G) {
                float4 kr[G], vr[G];
#pragma unroll
                for (int f = 0; f < G; f++) {
                    const int p = pb + f;
                    if (p < p1 && p != static_cast<int>(pos)) {
                        kr[f] = __ldcg(reinterpret_cast<const float4*>(kc + static_cast<size_t>(p) * HD) + lane);
                        vr[f] = __ldcg(reinterpret_cast<const float4*>(vc + static_cast<size_t>(p) * HD) + lane);
                    } else if (p == static_cast<int>(pos)) {  // this step's row: from shared memory
                        kr[f] = reinterpret_cast<const float4*>(k_s)[lane];
                        vr[f] = reinterpret_cast<const float4*>(v_s)[lane];
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
                warp_reduce_multi<QPG * G>(v);  // lane l: dot of (head l / 8, position l % 8)
                const bool valid = pb + my_f < p1;
                const float sc = valid ? v[0] * a.attn_scale : -INFINITY;
                float gm = sc;
                gm = fmaxf(gm, __shfl_xor_sync(FULL, gm, 1));
                gm = fmaxf(gm, __shfl_xor_sync(FULL, gm, 2));
                gm = fmaxf(gm, __shfl_xor_sync(FULL, gm, 4));
                float corr[QPG];
#pragma unroll
                for (int h = 0; h < QPG; h++) {
                    const float mn = fmaxf(m[h], __shfl_sync(FULL, gm, h * G));  // position pb valid: finite
                    corr[h] = expf(m[h] - mn);  // first group: exp(-inf) = 0
                    m[h] = mn;
                    acc[h].x *= corr[h]; acc[h].y *= corr[h]; acc[h].z *= corr[h]; acc[h].w *= corr[h];
                }
                // this lane's head: selects, not a dynamically indexed (local-memory) array
                const float m_my = my_h == 0 ? m[0] : my_h == 1 ? m[1] : my_h == 2 ? m[2] : m[3];
                const float c_my = my_h == 0 ? corr[0] : my_h == 1 ? corr[1] : my_h == 2 ? corr[2] : corr[3];
                const float pr = valid ? expf(sc - m_my) : 0.f;
                l_lane = l_lane * c_my + pr;
#pragma unroll
                for (int f = 0; f < G; f++) {
#pragma unroll
                    for (int h = 0; h < QPG; h++) {
                        const float ph = __shfl_sync(FULL, pr, h * G + f);
                        acc[h].x = fmaf(ph, vr[f].x, acc[h].x);
                        acc[h].y = fmaf(ph, vr[f].y, acc[h].y);
                        acc[h].z = fmaf(ph, vr[f].z, acc[h].z);
                        acc[h].w = fmaf(ph, vr[f].w, acc[h].w);
                    }
                }
            }
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
            consumer_sync();
            // this split over the 8 warps, per head: {M, L, 0, 0, acc}; one split: ctx = acc / L
            for (int k = t; k < QPG * PW; k += kConsumers) {
                const int h = k / PW, i = k % PW;
                float M = -INFINITY;
#pragma unroll
                for (int w = 0; w < kConsumerWarps; w++)
                    if (wp[(w * QPG + h) * W + 1] > 0.f) M = fmaxf(M, wp[(w * QPG + h) * W]);
                float Ls = 0.f, val = 0.f;
#pragma unroll
                for (int w = 0; w < kConsumerWarps; w++) {
                    const float* pw = wp + (w * QPG + h) * W;
                    if (pw[1] > 0.f) {
                        const float e = expf(pw[0] - M);
                        Ls += pw[1] * e;
                        if (i >= 4) val += pw[2 + (i - 4)] * e;
                    }
                }
                if (S == 1) {
                    if (i >= 4) {
                        const float c = val / Ls;
                        a.ctx[(g * QPG + h) * HD + (i - 4)] = c;
                        mx = fmaxf(mx, fabsf(c));
                    }
                } else {
                    a.attn_part[static_cast<size_t>((g * QPG + h) * S + s) * PW + i] =
                        i == 0 ? M : (i == 1 ? Ls : (i >= 4 ? val : 0.f));
                }
            }
            if (S == 1) return true;
            // the last split of the group to finish merges the S partials
            consumer_sync();  // every partial store of this CTA precedes thread 0's fence
            if (t == 0) {
                __threadfence();
                const unsigned target = static_cast<unsigned>(layer + 1) * S;
                sh.flags[2] = (atomicAdd(a.attn_cnt + g, 1u) + 1 == target);
            }
            consumer_sync();
            if (!sh.flags[2]) return true;
            __threadfence();
            // warp h (< 4): lane r < S loads split r's {M, L} of head h; all S in one round trip
            float* wsh = q_s;  // [4][32] merge weights e^(M_r - GM) / GL (q is no longer needed)
            if (warp < QPG) {
                const float* ph = a.attn_part + static_cast<size_t>(g * QPG + warp) * S * PW;
                const float2 ml = lane < S ? __ldcg(reinterpret_cast<const float2*>(ph + lane * PW))
                                           : make_float2(-INFINITY, 0.f);
                const bool ok = ml.y > 0.f;
                const float GM = warp_max(ok ? ml.x : -INFINITY);
                const float e = ok ? expf(ml.x - GM) : 0.f;
                const float GL = warp_sum(ml.y * e);
                wsh[warp * 32 + lane] = e / GL;
            }
            consumer_sync();
            for (int k = t; k < QPG * HALF; k += kConsumers) {  // (head, column pair)
                const int h = k / HALF, c = 2 * (k % HALF);
                const float* ph = a.attn_part + static_cast<size_t>(g * QPG + h) * S * PW + 4 + c;
                float c0 = 0.f, c1 = 0.f;
#pragma unroll 8
                for (int r = 0; r < S; r++) {  // every split wrote its row this step (empty: weight 0)
                    const float2 ac = __ldcg(reinterpret_cast<const float2*>(ph + r * PW));
                    const float w = wsh[h * 32 + r];
                    c0 = fmaf(ac.x, w, c0);
                    c1 = fmaf(ac.y, w, c1);
                }
                *reinterpret_cast<float2*>(a.ctx + (g * QPG + h) * HD + c) = make_float2(c0, c1);
                mx = fmaxf(mx, fmaxf(fabsf(c0), fabsf(c1)));
            }
            return true;
        }
    }

    // Attention for (head, split) = divmod(blockIdx.x, S) (modules.cpp:58-88):
    // writes the split's softmax partial {max, sum, acc}; the o_proj staging
    // merges the splits.  Starts as soon as kv group h / 4's q, k and v rows
    // are written (qkv_cnt, no grid barrier).  false (uniform) on error.
    template <int HD>
    __device__ bool attention(int layer, unsigned pos) {
        constexpr int VPL = HD / 32;
        constexpr int HALF = HD / 2;
        constexpr int PF = 4;  // positions per warp in flight
        const DecodeLayer& L = sh.layers[layer];
        const int S = attn_splits(pos);
        const int u = blockIdx.x;
        if (u >= a.H * S) return true;
        const int h = u / S, s = u % S, kh = h / 4;  // kv head h/4 (modules.cpp:70)
        if (!TLD_OK(pos < static_cast<unsigned>(a.max_seq) && kh < a.KV && h < a.H, 40, pos, kh)) return true;
        if (!TLD_OK((3 * HD + kConsumerWarps * (HD + 2)) * 4 <= static_cast<int>(xbuf_bytes(a.D, a.F, a.HD, F8)), 41, HD, 0))
            return true;
        if (!wait_qkv(kh, layer)) return false;
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
        const int chunk = (attn_span(pos) + S - 1) / S;
        const int p0 = attn_lo(pos) + s * chunk, p1 = min(npos, p0 + chunk);
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
            // scores of the PF positions, then one online-softmax rescale for all of them
            float sc[PF];
#pragma unroll
            for (int f = 0; f < PF; f++) {
                float dsum = 0.f;
#pragma unroll
                for (int j = 0; j < VPL; j++) dsum += kv[f][j] * q[j];
                sc[f] = warp_sum(dsum) * a.attn_scale;
            }
            float mn = m;
#pragma unroll
            for (int f = 0; f < PF; f++)
                if (pb + f * kConsumerWarps < p1) mn = fmaxf(mn, sc[f]);
            const float corr = expf(m - mn);
            l *= corr;
#pragma unroll
            for (int j = 0; j < VPL; j++) acc[j] *= corr;
#pragma unroll
            for (int f = 0; f < PF; f++) {
                if (pb + f * kConsumerWarps < p1) {
                    const float e = expf(sc[f] - mn);
                    l += e;
#pragma unroll
                    for (int j = 0; j < VPL; j++) acc[j] = fmaf(e, vv[f][j], acc[j]);
                }
            }
            m = mn;
        }
        float* mine = wp + warp * (HD + 2);
        if (lane == 0) {
            mine[0] = m;
            mine[1] = l;
        }
#pragma unroll
        for (int j = 0; j < VPL; j++) mine[2 + lane * VPL + j] = acc[j];
        consumer_sync();
        // this split's partial over the 8 warps: part[h S + s] = {M, L, 0, 0, acc[HD]}
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kConsumerWarps; w++)
            if (wp[w * (HD + 2) + 1] > 0.f) M = fmaxf(M, wp[w * (HD + 2)]);
        float* part = a.attn_part + static_cast<size_t>(h * S + s) * (HD + 4);
        for (int i = t; i < HD + 4; i += kConsumers) {
            float v = 0.f;
            if (i == 0) {
                v = M;
            } else if (i == 1 || i >= 4) {
                const int src = (i == 1) ? 1 : i - 2;  // l, or acc[i - 4] at warp offset 2 + (i - 4)
#pragma unroll
                for (int w = 0; w < kConsumerWarps; w++) {
                    const float* pw = wp + w * (HD + 2);
                    if (pw[1] > 0.f) v += pw[src] * expf(pw[0] - M);
                }
            }
            part[i] = v;
        }
        return true;
    }

    // Stages ctx = attention output (int8 digits or fp16 planes) for o_proj: merges, for
    // each head, the S split partials {M, L, acc} written by attention
    // (softmax over all positions = sum_s acc_s e^(M_s - M) / sum_s L_s e^(M_s - M),
    // M = max_s M_s), takes the CTA-wide max |ctx| for the digit scale and
    // stores the digits as stage_digits does.  Returns 2^-k.
    template <int HD>
    __device__ float stage_ctx_digits(unsigned pos) {
        const int S = attn_splits(pos);
        const int d = a.H * HD;
        const int nb = d / 16;
        const int dp = tile_slices(d) * kTileCols;  // padded to whole tiles
        if (!TLD_OK(x_bytes() * static_cast<size_t>(dp) <= xbuf_bytes(a.D, a.F, a.HD, F8), 32, d, dp)) return 1.0f;
        // fp16 planes of padding columns (zero weights) must be finite: zero them
        // (stale int8 digits are finite integers, 0 x anything = 0)
        if constexpr (F8)
            for (int b = nb + t; b < dp / 16; b += kConsumers) zero_x(b);
        // first block of 16 columns per thread (the only one when H hd <= 4096)
        float v[16];
        float mx = 0.f;
        const int b0 = t;
        if (b0 < nb) {
            merge_ctx_block<HD>(b0, S, v);
        } else {
#pragma unroll
            for (int j = 0; j < 16; j++) v[j] = 0.f;
        }
#pragma unroll
        for (int j = 0; j < 16; j++) mx = fmaxf(mx, fabsf(v[j]));
        for (int b = b0 + kConsumers; b < nb; b += kConsumers) {  // longer ctx: not kept, recomputed below
            float w[16];
            merge_ctx_block<HD>(b, S, w);
#pragma unroll
            for (int j = 0; j < 16; j++) mx = fmaxf(mx, fabsf(w[j]));
        }
        const float amax = sum_max(0.f, mx).y;
        const int k = stage_exp(amax);
        const float sc = ldexpf(1.0f, k);
        if (b0 < nb) put_x(b0, v, sc);
        for (int b = b0 + kConsumers; b < nb; b += kConsumers) {
            float w[16];
            merge_ctx_block<HD>(b, S, w);
            put_x(b, w, sc);
        }
        consumer_sync();
        stamp(2);
        return ldexpf(1.0f, -k);
    }

    // ctx columns [16 b, 16 b + 16) (one head): merge of the S split partials,
    // all of a group of 4 splits loaded before any is used, combined with a
    // running maximum in split order.
    template <int HD>
    __device__ __forceinline__ void merge_ctx_block(int b, int S, float (&v)[16]) const {
        const int h = (16 * b) / HD, i0 = (16 * b) % HD;
        const float* ph = a.attn_part + static_cast<size_t>(h) * S * (HD + 4);
        float GM = -INFINITY, GL = 0.f;
#pragma unroll
        for (int j = 0; j < 16; j++) v[j] = 0.f;
        for (int s0 = 0; s0 < S; s0 += 4) {
            float2 ml[4];
            float4 ac[4][4];
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const float* pp = ph + static_cast<size_t>(s0 + u) * (HD + 4);
                const bool ok = s0 + u < S;
                ml[u] = ok ? __ldcg(reinterpret_cast<const float2*>(pp)) : make_float2(-INFINITY, 0.f);
#pragma unroll
                for (int q = 0; q < 4; q++)
                    ac[u][q] = ok ? __ldcg(reinterpret_cast<const float4*>(pp + 4 + i0) + q)
                                  : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int u = 0; u < 4; u++) {
                if (!(ml[u].y > 0.f)) continue;
                if (ml[u].x > GM) {  // rescale what was merged so far
                    const float c = expf(GM - ml[u].x);
                    GL *= c;
#pragma unroll
                    for (int j = 0; j < 16; j++) v[j] *= c;
                    GM = ml[u].x;
                }
                const float w = expf(ml[u].x - GM);
                GL = fmaf(ml[u].y, w, GL);
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    v[4 * q] = fmaf(ac[u][q].x, w, v[4 * q]);
                    v[4 * q + 1] = fmaf(ac[u][q].y, w, v[4 * q + 1]);
                    v[4 * q + 2] = fmaf(ac[u][q].z, w, v[4 * q + 2]);
                    v[4 * q + 3] = fmaf(ac[u][q].w, w, v[4 * q + 3]);
                }
            }
        }
        const float inv = 1.0f / GL;
#pragma unroll
        for (int j = 0; j < 16; j++) v[j] *= inv;
    }
};

template <int HD, bool TP, bool F8>
__global__ void __launch_bounds__(kThreads, 1) decode_step_kernel(DecodeArgs a, int stages) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    const Shared sh = carve(smem_raw, stages, a);
#ifdef TL_DECODE_CHECK
    {
        unsigned dyn;
        asm volatile("mov.u32 %0, %%dynamic_smem_size;" : "=r"(dyn));
        const size_t end = reinterpret_cast<uint8_t*>(sh.xbar + 1) - smem_raw;
        int* a_dbg = a.dbg;
        int* a_err = a.err;
        if (!TLD_OK(end <= dyn, 1, static_cast<long long>(end), dyn)) return;
    }
#endif
    if (threadIdx.x == 0) {
        for (int s = 0; s < stages; s++) {
            mbar_init(&sh.full[s], 1);
            mbar_init(&sh.empty[s], kWarpsPerSlot);
        }
        mbar_init(sh.xbar, 1);
        sh.flags[0] = 0;
        sh.flags[1] = 0;
        for (int i = 32; i < 64; i++) reinterpret_cast<unsigned*>(sh.scratch)[i] = 0u;  // kv group row counts
        sh.info[0] = __ldcg(a.pos);
        sh.info[1] = __ldcg(a.token);
        sh.info[2] = __ldcg(a.epoch);
        fence_mbar_init();
    }
    static_assert(sizeof(DecodeLayer) % 8 == 0, "layer table copied in 8-byte words");
    for (int i = threadIdx.x; i < a.n_layers * static_cast<int>(sizeof(DecodeLayer) / 8); i += blockDim.x)
        reinterpret_cast<uint64_t*>(sh.layers)[i] = __ldg(reinterpret_cast<const unsigned long long*>(a.layers) + i);
    __syncthreads();
    // Never index with an out-of-range token or position: record and stop.
    // (a.V is this rank's vocabulary slice; tokens index the whole vocabulary)
    if (sh.info[0] >= static_cast<unsigned>(a.max_seq) || sh.info[1] >= static_cast<unsigned>(a.V * a.tp_size)) {
        if (threadIdx.x == 0) atomicCAS(a.err, 0, kErrInput);
        return;
    }

    const int D = a.D, F = a.F, NQKV = (a.H + 2 * a.KV) * a.HD;
    if (threadIdx.x >= kConsumers) {
        // ---------------- producer warp ----------------
        if (threadIdx.x != kConsumers) return;
        Producer p(a, sh, stages);
        p.run();
        return;
    }

    // ---------------- consumer warps ----------------
    Consumer<TP, F8> cw(a, sh, stages);
    cw.stamp(0);
    const unsigned pos = sh.info[0];
    const uint32_t token = sh.info[1];
    const float* emb = a.embed + static_cast<size_t>(token) * D;  // Embedding::forward (modules.cpp:5-7)
    cw.epoch = sh.info[2];
    const float2 st0 = cw.local_stats(emb, D, sh.layers[0].g_in);
    for (int l = 0; l < a.n_layers; l++) {
        const DecodeLayer& L = sh.layers[l];
        const float* hin = (l == 0) ? emb : a.h;
        // q/k/v = W_qkv rmsnorm(h)
        float un;
        if (l == 0) {
            un = cw.template stage_digits<true>(emb, D, L.g_in, &st0);
        } else {
            if (!cw.wait_all()) return;
            un = cw.template stage_digits<true>(a.h, D, L.g_in, nullptr);
        }
        cw.template prefetch_kv<HD>(l, pos);
        if (!cw.template run_i8<0>(NQKV, D, un, nullptr, nullptr)) return;
        // attention: ctx (GQA), or split partials merged by the o_proj staging
        const bool gqa = cw.gqa(pos);
        float ctx_max = 0.f;
        if (gqa) {
            if (!cw.template attention_gqa<HD>(l, pos, ctx_max) || cw.aborted()) return;
        } else {
            if (!cw.template attention<HD>(l, pos) || cw.aborted()) return;
        }
        cw.publish(0.f, ctx_max);
        // h = h + W_o ctx
        if (!cw.wait_all()) return;
        un = gqa ? cw.template stage_digits<false>(a.ctx, a.H * a.HD, nullptr, nullptr)
                 : cw.template stage_ctx_digits<HD>(pos);
        if (cw.t == 0) prefetch_l2(L.g_post, static_cast<uint32_t>(D) * 4u);  // staged after this phase
        if (!cw.template run_i8<1>(D, a.H * a.HD, un, hin, L.g_post)) return;
        // act = silu(W1 x) * (W3 x), x = rmsnorm(h)
        if (!cw.wait_all()) return;
        un = cw.template stage_digits<true>(a.h, D, L.g_post, nullptr);
        if (!cw.template run_i8<2>(2 * F, D, un, nullptr, nullptr, l)) return;
        // h = h + W2 act
        if (!cw.wait_all()) return;
        un = cw.stage_act(l);
        const float* g_next = (l + 1 < a.n_layers) ? sh.layers[l + 1].g_in : a.g_final;
        if (cw.t == 0) prefetch_l2(g_next, static_cast<uint32_t>(D) * 4u);  // staged after this phase
        if (!cw.template run_i8<3>(D, F, un, a.h, g_next)) return;
    }
    // logits = lm_head rmsnorm(h); token = argmax (main.cpp:10-21).  An 8-bit
    // lm_head runs like a projection: RMSNorm fused into the staging, the
    // projections' tiles of 16 rows.
    const bool lm8 = a.lm_8bit != 0;
    float lm_un = 1.0f;
    if (!cw.wait_all()) return;
    if (lm8) lm_un = cw.template stage_digits<true>(a.h, D, a.g_final, nullptr);
    else cw.stage_f32(a.h, D, a.g_final);
    const int ksD = tile_slices(D);
    const int lm_rows = lm8 ? kTileRowsI8 : kTileRowsF32;
    const int n_rb = (a.V + lm_rows - 1) / lm_rows;
    int nrl = 0;
    const int rb0 = lm8 ? cw.template run_tiles<false>(n_rb, ksD, nrl) : cw.template run_tiles<true>(n_rb, ksD, nrl);
    if (rb0 < 0) return;
    float best_v = -INFINITY;
    uint32_t best_i = 0xffffffffu;
    const int t = threadIdx.x, lane = t & 31;
    for (int j = t; j < nrl * lm_rows; j += kConsumers) {
        const int row = rb0 * lm_rows + j;
        if (row < a.V) {
            const float val = lm8 ? cw.row_sum(j / kTileRowsI8, j % kTileRowsI8, ksD, kTileRowsI8) * lm_un
                                  : cw.row_sum(j / kTileRowsF32, j % kTileRowsF32, ksD, kTileRowsF32);
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
        if (TP) {
            // Every rank sends its best {value, global index} (bit 31: this
            // rank's logits[0] is NaN) to every rank, then merges all of them
            // in rank order, i.e. in vocabulary order.
            const unsigned ep = sh.info[2];
            uint32_t gi = (bi == 0xffffffffu) ? 0xffffffffu : bi + static_cast<uint32_t>(a.vocab_off);
            if (a.tp_rank == 0 && l0 != l0) gi = 0x80000000u;
            const unsigned long long slot = (static_cast<unsigned long long>(gi) << 32) | __float_as_uint(bv);
            const size_t off = kXchgAmSlot + (static_cast<size_t>(ep & 1) * kMaxTp + a.tp_rank) * 8;
            for (int q = 0; q < a.tp_size; q++) st_relaxed_sys_u64(a.xpeer[q] + off, slot);
            fence_sys();
            for (int q = 0; q < a.tp_size; q++) red_add_sys_u64(a.xpeer[q] + kXchgAmCnt, 1ull);
            const unsigned long long target = (static_cast<unsigned long long>(ep) + 1) * a.tp_size;
            const unsigned long long t0 = globaltimer();
            bool ok = true;
            for (unsigned i = 0;; i++) {
                if (ld_acquire_sys_u64(a.xpeer[a.tp_rank] + kXchgAmCnt) >= target) break;
                if ((i & 63) == 63 && globaltimer() - t0 > a.timeout_ns) {
                    atomicCAS(a.err, 0, static_cast<int>(kErrBarrier));
                    ok = false;
                    break;
                }
            }
            bool nan0 = false;
            bv = -INFINITY;
            bi = 0xffffffffu;
            for (int q = 0; ok && q < a.tp_size; q++) {
                const unsigned long long v = ld_relaxed_sys_u64(
                    a.xpeer[a.tp_rank] + kXchgAmSlot + (static_cast<size_t>(ep & 1) * kMaxTp + q) * 8);
                const uint32_t vi = static_cast<uint32_t>(v >> 32);
                if (vi == 0x80000000u) nan0 = true;
                else if (better(__uint_as_float(static_cast<uint32_t>(v)), vi, bv, bi)) {
                    bv = __uint_as_float(static_cast<uint32_t>(v));
                    bi = vi;
                }
            }
            if (nan0 || bi == 0xffffffffu) bi = 0;  // sample_max keeps 0 (main.cpp:10-21)
        } else if (l0 != l0 || bi == 0xffffffffu) {
            bi = 0;  // sample_max keeps 0 (main.cpp:10-21)
        }
        sh.info[3] = bi;
    }
    consumer_sync();
    uint32_t tok = sh.info[3];
    if (a.temperature > 0.f)  // sample_multinomial (main.cpp:23-43); a whole-vocabulary rank only
        tok = sample_block<kConsumers>(a.logits, a.V, a.temperature, sample_uniform(a.sample_seed, pos), sh.scratch,
                                       ConsumerSync{});
    if (t == 0) {
        *a.token = tok;
        a.history[pos] = tok;
        *a.pos = pos + 1;
        *a.epoch = sh.info[2] + 1;
        // Every CTA has passed every barrier and taken its ticket: reset the
        // counters for the next step.
        *a.ticket = 0;
        *a.bar = 0;
        for (int g = 0; g < a.KV; g++) {
            a.qkv_cnt[g] = 0;
            a.attn_cnt[g] = 0;
        }
        __threadfence();
    }
}

// ---------------------------------------------------------------------------
// Repacking kernels
// ---------------------------------------------------------------------------
// Tiles of kTileBytesI8 (int8 + scales) or, with null scales, kTileBytesF8
// (the e5m2 bytes in the same layout).
__global__ void k_repack_i8(uint8_t* dst, const int8_t* w1, const float* s1, const int8_t* w3, const float* s3,
                            int n, int d, int swiglu) {
    const size_t tb = s1 ? kTileBytesI8 : kTileBytesF8;
    const int ksn = tile_slices(d), dp = ksn * kTileCols;  // columns >= d: zero padding
    const int n_rb = swiglu ? (2 * n + 15) / 16 : (n + 15) / 16;
    const size_t chunks = static_cast<size_t>(n_rb) * 16 * (dp / 16);
    for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < chunks; idx += (size_t)gridDim.x * blockDim.x) {
        const int ch = static_cast<int>(idx % (dp / 16));
        const int lrow = static_cast<int>(idx / (dp / 16));
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
        uint8_t* out = dst + (static_cast<size_t>(rb) * ksn + ks) * tb + w * 1024 + half * 512 + lane * 16;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (row < n && col < d) v = *reinterpret_cast<const uint4*>(src + static_cast<size_t>(row) * d + col);
        *reinterpret_cast<uint4*>(out) = v;
    }
    // scales (already 1/s): one per (logical row, group); padding groups 0
    if (!s1) return;
    const int gpr = d / 64, gprp = dp / 64;
    const size_t groups = static_cast<size_t>(n_rb) * 16 * gprp;
    for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < groups; idx += (size_t)gridDim.x * blockDim.x) {
        const int gi = static_cast<int>(idx % gprp);
        const int lrow = static_cast<int>(idx / gprp);
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
        out[rr * 8 + w] = (row < n && gi < gpr) ? src[static_cast<size_t>(row) * gpr + gi] : 0.f;
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

bool decode_kernel_fits(int D, int F, int H, int KV, int HD, int V, int n_layers, bool w_f8, int grid,
                        int max_smem, int* stages, size_t* smem_bytes, int* pbuf_floats) {
    if (D % kTileCols || F % 64 || (H * HD) % 64) return false;
    // H: this rank's q heads (H hd == D on one GPU, D / tp under tensor parallelism)
    if (!(HD == 64 || HD == 128 || HD == 256) || H * HD > D || grid < 1) return false;
    if (H != 4 * KV || KV > 32) return false;  // kv head h / 4; group row counts in smem
    // statistics entries; the barrier counter reaches grid x (5 L + 1)
    if (grid > kStatsCap || static_cast<long long>(grid) * (5 * n_layers + 1) >= (1ll << 31)) return false;
    // partial-sum buffer: the most tiles x rows any CTA owns in one phase
    auto need = [&](int n_rows, int rows_per_tile, int d) {
        const int n_rb = (n_rows + rows_per_tile - 1) / rows_per_tile;
        const int per_cta = (n_rb + grid - 1) / grid;
        return per_cta * tile_slices(d) * rows_per_tile;
    };
    int pb = 512;
    pb = std::max(pb, need((H + 2 * KV) * HD, kTileRowsI8, D));
    pb = std::max(pb, need(D, kTileRowsI8, H * HD));
    pb = std::max(pb, need(2 * F, kTileRowsI8, D));
    pb = std::max(pb, need(D, kTileRowsI8, F));
    pb = std::max(pb, need(V, kTileRowsF32, D));
    pb = std::max(pb, need(V, kTileRowsI8, D));  // 8-bit lm_head
    const size_t fixed = fixed_bytes(D, F, HD, w_f8, pb, n_layers);
    if (static_cast<size_t>(max_smem) <= fixed) return false;
    int st = static_cast<int>((static_cast<size_t>(max_smem) - fixed) / (stage_bytes(w_f8) + 16));
    st = st > 24 ? 24 : st;
    st -= st % kSlotsPerOwnerCycle;  // slots keep their owner warps
    if (st < kSlotsPerOwnerCycle) return false;
    *stages = st;
    *pbuf_floats = pb;
    *smem_bytes = static_cast<size_t>(st) * stage_bytes(w_f8) + fixed + static_cast<size_t>(st) * 16;
    return true;
}

tl_status launch_decode_step(const DecodeArgs& a, int grid, int stages, size_t smem, cudaStream_t s) {
    DecodeArgs copy = a;
    void* args[] = {&copy, &stages};
    const void* fn = nullptr;
    const int v = (a.tp_size > 1 ? 1 : 0) + (a.w_f8 ? 2 : 0);  // (TP, F8) instantiation
    auto pick = [&](auto k00, auto k10, auto k01, auto k11) {
        const void* ks[4] = {reinterpret_cast<const void*>(k00), reinterpret_cast<const void*>(k10),
                             reinterpret_cast<const void*>(k01), reinterpret_cast<const void*>(k11)};
        return ks[v];
    };
    switch (a.HD) {
        case 64: fn = pick(decode_step_kernel<64, false, false>, decode_step_kernel<64, true, false>,
                           decode_step_kernel<64, false, true>, decode_step_kernel<64, true, true>); break;
        case 128: fn = pick(decode_step_kernel<128, false, false>, decode_step_kernel<128, true, false>,
                            decode_step_kernel<128, false, true>, decode_step_kernel<128, true, true>); break;
        case 256: fn = pick(decode_step_kernel<256, false, false>, decode_step_kernel<256, true, false>,
                            decode_step_kernel<256, false, true>, decode_step_kernel<256, true, true>); break;
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
