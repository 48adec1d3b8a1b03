// tl_gemm_q8.cu -- tcgen05 GEMM with 8-bit weights dequantised in shared
// memory: C = A B^T, A fp16 activations, B the model's int8 weights (with the
// per-64-group 1/s) or e5m2 bytes, fp32 accumulation in tensor memory.
//
// The batched paths (prefill, batched decode) read the weights in their
// stored 8-bit form, so a GEMM streams 1 byte (+ 1/16 byte of scale) per
// weight instead of an fp16 copy's 2, and no fp16 copy of the model is kept.
// Per K block of 64 (one quantisation group):
//   warp 0      TMA of the weights: the BN x 64 int8 B box (plain rows of 64
//               bytes) and BN scales of that group from a transposed scale
//               array [K / 64][N] (one 4-byte scale per B row, contiguous),
//               into a deep ring (the copies come from HBM);
//   last warp   TMA of the 128 x 64 fp16 A box (SWIZZLE_128B) into its own
//               shorter ring;
//   8 warps     convert: w = fp16(q) * fp16(1/s) in packed fp16 arithmetic
//               (tensor.cpp:101-104's dequantisation with the scale rounded
//               to fp16; e5m2 bytes widen exactly) into one of two fp16 B buffers in
//               the SWIZZLE_128B K-major layout the MMA reads, then
//               fence.proxy.async and arrive;
//   warp 1      tcgen05.mma kind::f16 (M 128, N BN, K 16; 4 per block) on the
//               A stage and the converted B buffer; commits free both;
//   warps 2..    epilogue (shared with the fp16 GEMM; 4 warps, 8 for SwiGLU,
//               two per lane quarter each taking half the columns): store,
//               residual add or SwiGLU, and split-K partials.
// A SwiGLU B tile is 128 gate rows then the same 128 up rows: two B boxes and
// two scale boxes.  Every wait is bounded (~2 s); on expiry the kernel records
// an error code, drains what it issued, waits for its MMAs and frees its
// tensor memory.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <math.h>

#include <algorithm>
#include <mutex>

#include "tl_common.cuh"
#include "tl_gemm.cuh"
#include "tl_gemm_epi.cuh"
#include "tl_tc.cuh"

namespace tl {
namespace {

using namespace tc;
constexpr int kQBM = 128, kQBK = 64;
constexpr int kConvWarps = 8;
// Warps: 0 weight producer, 1 MMA, then EW epilogue warps (4: one per tensor-
// memory lane quarter; 8 for the SwiGLU epilogue, whose exp / divide per
// output would otherwise hold the MMAs of the next 256-row tile), then the 8
// converters, then the activation producer.
template <int EW>
struct Q8Warps {
    static constexpr int kConv0 = 2 + EW;
    static constexpr int kAProd = kConv0 + kConvWarps;
    static constexpr int kThreads = 32 * (kAProd + 1);
};
template <int EPI>
constexpr int q8_epi_warps() { return EPI == kEpiSwiGluF16 ? 8 : 4; }

// MT: 128-row M tiles per CTA tile, sharing each converted B block (1 for few
// rows; 2 for many, so the conversion is paid once per 256 rows).  Tiles are
// MT x 128 rows by 256 columns; MT = 1 double-buffers its accumulator (the
// epilogue of a tile overlaps the next tile's MMAs), MT = 2 fills the 512
// tensor-memory columns with its two accumulators and does not.
template <int MT>
struct Q8Cfg {
    static constexpr int BN = 256;
    static constexpr int kAcc = MT == 1 ? 2 : 1;  // accumulator sets in tensor memory
    // weights (int8 rows of 64 bytes + the block's 1/s of each row) and
    // activations have separate rings: the weight ring runs deep for few rows,
    // because its copies come from HBM; the activation boxes come from L2.
    static constexpr int kBStages = MT == 1 ? 5 : 3;
    static constexpr int kAStages = MT == 1 ? 4 : 3;
    static constexpr int kABytes = MT * kQBM * kQBK * 2;  // fp16 A boxes, SWIZZLE_128B
    static constexpr int kQBytes = BN * kQBK;             // 8-bit B rows of 64 bytes
    static constexpr int kSBytes = BN * 4;                // 1/s of each B row for the block's group
    static constexpr int kBStageBytes = kQBytes + kSBytes;
    static constexpr int kHBytes = BN * kQBK * 2;         // converted fp16 B, SWIZZLE_128B
    static constexpr int kHBufs = 2;
    static constexpr int kTmemCols = kAcc * MT * BN;
    static constexpr size_t kSmem = 1024 + static_cast<size_t>(kAStages) * kABytes +
                                    static_cast<size_t>(kHBufs) * kHBytes +
                                    static_cast<size_t>(kBStages) * kBStageBytes + 512;
    static_assert(kABytes % 1024 == 0 && kHBytes % 1024 == 0, "SWIZZLE_128B operands stay 1024-byte aligned");
    static_assert(kBStageBytes % 128 == 0, "weight stages stay 128-byte aligned");
    static_assert(kTmemCols == 512, "the accumulators fill tensor memory");
};

// One 16-byte chunk (16 weights) of B row `row` -> two fp16 chunks (elements
// 16 j .. 16 j + 15) of the SWIZZLE_128B row: chunk c of row r sits at 16-byte
// position c ^ (r % 8) of the row's 128 bytes.
template <bool F8>
__device__ __forceinline__ void convert_chunk(const uint8_t* q, float s, uint8_t* h, int row, int j) {
    const uint4 raw = *reinterpret_cast<const uint4*>(q + row * kQBK + 16 * j);
    uint32_t o[8];
    if constexpr (F8) {  // e5m2: each byte is the high byte of the same value's fp16
        const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
        for (int k = 0; k < 4; k++) {
            o[2 * k] = __byte_perm(w[k], 0u, 0x1404);
            o[2 * k + 1] = __byte_perm(w[k], 0u, 0x3424);
        }
    } else {
        // q -> fp16 in packed pairs, exactly: with u = q + 128 (the byte with
        // its top bit flipped), the fp16 with bits 0x64uu is 1024 + u, and
        // (1024 + u) - 1152 = q; then one fp16 product with fp16(1/s).
        const __half2 off = __float2half2_rn(1152.0f);
        const __half2 s2 = __float2half2_rn(s);
        const uint32_t w[4] = {raw.x ^ 0x80808080u, raw.y ^ 0x80808080u, raw.z ^ 0x80808080u, raw.w ^ 0x80808080u};
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const uint32_t lo = __byte_perm(w[k], 0x64646464u, 0x4140), hi = __byte_perm(w[k], 0x64646464u, 0x4342);
            const __half2 v0 = __hmul2(__hsub2(*reinterpret_cast<const __half2*>(&lo), off), s2);
            const __half2 v1 = __hmul2(__hsub2(*reinterpret_cast<const __half2*>(&hi), off), s2);
            o[2 * k] = *reinterpret_cast<const uint32_t*>(&v0);
            o[2 * k + 1] = *reinterpret_cast<const uint32_t*>(&v1);
        }
    }
    uint8_t* rowp = h + row * 128;
    const int sw = row & 7;
    *reinterpret_cast<uint4*>(rowp + (((2 * j) ^ sw) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
    *reinterpret_cast<uint4*>(rowp + (((2 * j + 1) ^ sw) << 4)) = make_uint4(o[4], o[5], o[6], o[7]);
}

// PAIRS: a B tile is 128 gate rows then the same 128 up rows (two boxes), for
// the SwiGLU epilogue or for split-K partials that a SwiGLU pass combines.
template <int EPI, bool F8, bool PAIRS, int MT>
__global__ void __launch_bounds__(Q8Warps<q8_epi_warps<EPI>()>::kThreads, 1)
    gemm_q8_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_q,
                   const __grid_constant__ CUtensorMap tma_q2, const __grid_constant__ CUtensorMap tma_s,
                   const __grid_constant__ CUtensorMap tma_s2, GemmArgs g) {
    using Cfg = Q8Cfg<MT>;
    constexpr int SA = Cfg::kAStages, SB = Cfg::kBStages, NB = Cfg::kHBufs, BN = Cfg::BN, TBM = MT * kQBM;
    constexpr int NACC = Cfg::kAcc;
    constexpr int kEpiWarps = q8_epi_warps<EPI>();
    constexpr int kConvWarp0 = Q8Warps<kEpiWarps>::kConv0, kAProdWarp = Q8Warps<kEpiWarps>::kAProd;
    constexpr bool swiglu = PAIRS;
    constexpr int QROWS = swiglu ? BN / 2 : BN;  // rows per B box
    extern __shared__ uint8_t smem_raw[];
    uint8_t* abase = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* hbase = abase + SA * Cfg::kABytes;
    uint8_t* bbase = hbase + NB * Cfg::kHBytes;
    uint64_t* fullA = reinterpret_cast<uint64_t*>(bbase + SB * Cfg::kBStageBytes);
    uint64_t* emptyA = fullA + SA;    // [SA] activation stage read by the MMAs (commit)
    uint64_t* fullB = emptyA + SA;    // [SB] weight stage landed
    uint64_t* emptyB = fullB + SB;    // [SB] weight stage converted (converter warps)
    uint64_t* bready = emptyB + SB;   // [NB] converted B buffer filled (converter warps)
    uint64_t* bfree = bready + NB;    // [NB] converted B buffer read by the MMAs (commit)
    uint64_t* tfull = bfree + NB;     // [NACC] accumulator ready
    uint64_t* tempty = tfull + 2;     // [NACC] accumulator drained by the epilogue
    uint64_t* mma_done = tempty + 2;  // every MMA issued has completed
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tm = (g.M + TBM - 1) / TBM, tn = (g.N + BN - 1) / BN, n_tiles = tm * tn * g.ksplit;
    const int nk_all = g.K / kQBK, nk_per = (nk_all + g.ksplit - 1) / g.ksplit;
    auto tile_of = [&](int t, int& m0, int& n0, int& kb0, int& nk) {
        m0 = (t % tm) * TBM;
        const int r = t / tm;
        n0 = (r % tn) * BN;
        kb0 = (r / tn) * nk_per;
        nk = max(0, min(nk_all, kb0 + nk_per) - kb0);
    };

    if (threadIdx.x == 0) {
        for (int s = 0; s < SA; s++) {
            bar_init(&fullA[s], 1);
            bar_init(&emptyA[s], 1);
        }
        for (int s = 0; s < SB; s++) {
            bar_init(&fullB[s], 1);
            bar_init(&emptyB[s], kConvWarps);
        }
        for (int b = 0; b < NB; b++) {
            bar_init(&bready[b], kConvWarps);
            bar_init(&bfree[b], 1);
        }
        for (int b = 0; b < NACC; b++) {
            bar_init(&tfull[b], 1);
            bar_init(&tempty[b], kEpiWarps);
        }
        bar_init(mma_done, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(tmem_slot)),
                     "r"(Cfg::kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    auto fail = [&](int code) {
        if (!*abort_flag && g.err) atomicCAS(g.err, 0, code);
        *abort_flag = 1;
    };

    if (warp == 0) {  // weight producer
        if (lane == 0) {
            uint32_t it = 0;
            const uint32_t bytes = Cfg::kQBytes + (F8 ? 0 : Cfg::kSBytes);
            for (int tile = blockIdx.x; tile < n_tiles && !*abort_flag; tile += gridDim.x) {
                int m0, n0, kb0, nk;
                tile_of(tile, m0, n0, kb0, nk);
                const int nq = swiglu ? n0 / 2 : n0;  // first B row of the box(es)
                for (int kb = kb0; kb < kb0 + nk; kb++, it++) {
                    const int s = it % SB;
                    if (it >= SB && !bar_wait_ab(&emptyB[s], ((it / SB) - 1) & 1, abort_flag)) {
                        fail(kGemmErrSlot);
                        break;
                    }
                    uint8_t* st = bbase + s * Cfg::kBStageBytes;
                    bar_expect_tx(&fullB[s], bytes);
                    tma_load_2d(st, &tma_q, kb * kQBK, nq, &fullB[s]);
                    if (swiglu) tma_load_2d(st + QROWS * kQBK, &tma_q2, kb * kQBK, nq, &fullB[s]);
                    if (!F8) {
                        tma_load_2d(st + Cfg::kQBytes, &tma_s, nq, kb, &fullB[s]);
                        if (swiglu) tma_load_2d(st + Cfg::kQBytes + QROWS * 4, &tma_s2, nq, kb, &fullB[s]);
                    }
                }
            }
            // every copy issued lands before the CTA exits
            const uint32_t first = it > static_cast<uint32_t>(SB) ? it - SB : 0;
            for (uint32_t k = first; k < it; k++) bar_wait(&fullB[k % SB], (k / SB) & 1);
        }
    } else if (warp == kAProdWarp) {  // activation producer
        if (lane == 0) {
            uint32_t it = 0;
            for (int tile = blockIdx.x; tile < n_tiles && !*abort_flag; tile += gridDim.x) {
                int m0, n0, kb0, nk;
                tile_of(tile, m0, n0, kb0, nk);
                for (int kb = kb0; kb < kb0 + nk; kb++, it++) {
                    const int s = it % SA;
                    if (it >= SA && !bar_wait_ab(&emptyA[s], ((it / SA) - 1) & 1, abort_flag)) {
                        fail(kGemmErrSlot);
                        break;
                    }
                    bar_expect_tx(&fullA[s], Cfg::kABytes);
#pragma unroll
                    for (int h = 0; h < MT; h++)
                        tma_load_2d(abase + s * Cfg::kABytes + h * (kQBM * kQBK * 2), &tma_a, kb * kQBK, m0 + h * kQBM,
                                    &fullA[s]);
                }
            }
            const uint32_t first = it > static_cast<uint32_t>(SA) ? it - SA : 0;
            for (uint32_t k = first; k < it; k++) bar_wait(&fullA[k % SA], (k / SA) & 1);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idesc = idesc_f16<BN>();
            uint32_t it = 0;
            int i = 0;
            for (int tile = blockIdx.x; tile < n_tiles && !*abort_flag; tile += gridDim.x, i++) {
                const int buf = i % NACC;
                if (i >= NACC && !bar_wait_ab(&tempty[buf], ((i / NACC) - 1) & 1, abort_flag)) {
                    fail(kGemmErrAccFree);
                    break;
                }
                tc_fence_after();
                const uint32_t dt = tmem + static_cast<uint32_t>(buf * MT * BN);
                int m0, n0, kb0, nk;
                tile_of(tile, m0, n0, kb0, nk);
                bool ok = true;
                for (int kb = 0; kb < nk; kb++, it++) {
                    const int sa = it % SA, hb = it % NB;
                    // busy polls: both are usually ready or about to be (no suspend / wake-up delay)
                    if (!bar_spin_ab(&fullA[sa], (it / SA) & 1, abort_flag) ||
                        !bar_spin_ab(&bready[hb], (it / NB) & 1, abort_flag)) {
                        fail(kGemmErrStage);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t db = sdesc_k128(su32(hbase + hb * Cfg::kHBytes));
#pragma unroll
                    for (int h = 0; h < MT; h++) {
                        const uint64_t da = sdesc_k128(su32(abase + sa * Cfg::kABytes + h * (kQBM * kQBK * 2)));
#pragma unroll
                        for (int k = 0; k < kQBK / 16; k++)
                            umma_f16(dt + static_cast<uint32_t>(h * BN), da + 2 * k, db + 2 * k, idesc, (kb | k) != 0);
                    }
                    umma_commit(&emptyA[sa]);
                    umma_commit(&bfree[hb]);
                }
                umma_commit(&tfull[buf]);  // accumulator ready (also on abort: frees the epilogue)
                if (!ok) break;
            }
            umma_commit(mma_done);  // tensor memory is freed only after every issued MMA wrote it
            bar_wait(mma_done, 0);
        }
    } else if (warp < kConvWarp0) {
        const int sub = warp & 3, part = (warp - 2) / 4;  // lane quarter (warp % 4) and column half
        int i = 0;
        for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, i++) {
            const int buf = i % NACC;
            if (!bar_wait_ab(&tfull[buf], (i / NACC) & 1, abort_flag)) {
                fail(kGemmErrAccReady);
                break;
            }
            tc_fence_after();
            if (*abort_flag) break;
            int m0, n0, kb0, nk;
            tile_of(tile, m0, n0, kb0, nk);
            GemmArgs gs = g;
            if (g.ksplit > 1) gs.C = static_cast<float*>(g.C) + static_cast<size_t>(kb0 / nk_per) * g.M * g.ldc;
#pragma unroll
            for (int h = 0; h < MT; h++)
                gemm_epilogue<BN, EPI>(gs, tmem + static_cast<uint32_t>((buf * MT + h) * BN), m0 + h * kQBM, n0, sub,
                                       lane, part, kEpiWarps / 4);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) bar_arrive(&tempty[buf]);
        }
    } else {
        // converter warps: thread ct takes 16-byte chunk ct % 4 of rows ct / 4, ct / 4 + 64, ...
        const int ct = threadIdx.x - 32 * kConvWarp0;
        const int j = ct & 3;
        uint32_t it = 0;
        for (int tile = blockIdx.x; tile < n_tiles && !*abort_flag; tile += gridDim.x) {
            int m0, n0, kb0, nk;
            tile_of(tile, m0, n0, kb0, nk);
            bool ok = true;
            for (int kb = 0; kb < nk; kb++, it++) {
                const int sb = it % SB, hb = it % NB;
                if (!bar_wait_ab(&fullB[sb], (it / SB) & 1, abort_flag) ||
                    (it >= NB && !bar_spin_ab(&bfree[hb], ((it / NB) - 1) & 1, abort_flag))) {
                    fail(kGemmErrStage);
                    ok = false;
                    break;
                }
                const uint8_t* q = bbase + sb * Cfg::kBStageBytes;
                const float* sc = reinterpret_cast<const float*>(q + Cfg::kQBytes);
                uint8_t* h = hbase + hb * Cfg::kHBytes;
#pragma unroll 4
                for (int row = ct >> 2; row < BN; row += 32 * kConvWarps / 4)
                    convert_chunk<F8>(q, F8 ? 1.0f : sc[row], h, row, j);
                fence_proxy_async();  // the tensor cores read what the generic proxy wrote
                __syncwarp();
                if (lane == 0) {
                    bar_arrive(&emptyB[sb]);
                    bar_arrive(&bready[hb]);
                }
            }
            if (!ok) break;
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(Cfg::kTmemCols));
    }
}

// 8-bit [rows][K] (K-major), box {64 bytes, box_rows}, no swizzle.
tl_status encode_q8(CUtensorMap* map, const void* ptr, int rows, int K, int box_rows) {
    auto fn = encode_fn();
    if (!fn) return set_error(TL_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(K)};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(kQBK), static_cast<cuuint32_t>(box_rows)};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(TL_ERR_CUDA, "cuTensorMapEncodeTiled (int8) failed (%d)", static_cast<int>(r));
    return TL_OK;
}

// fp32 transposed scales [groups][n], box {box_n, 1}.
tl_status encode_scales(CUtensorMap* map, const float* ptr, int n, int groups, int box_n) {
    auto fn = encode_fn();
    if (!fn) return set_error(TL_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(n), static_cast<cuuint64_t>(groups)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(n) * 4};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(box_n), 1u};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(ptr), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(TL_ERR_CUDA, "cuTensorMapEncodeTiled (scales) failed (%d)", static_cast<int>(r));
    return TL_OK;
}

template <int EPI, bool F8, bool PAIRS, int MT>
tl_status launch_q8(const __half* A, int M, int K, const Q8Weights& B, int N, void* C, int ldc, int* err,
                    cudaStream_t s, int ksplit) {
    using Cfg = Q8Cfg<MT>;
    const int qrows = PAIRS ? Cfg::BN / 2 : Cfg::BN;
    const int n_src = PAIRS ? N / 2 : N;  // rows of each source matrix
    CUtensorMap ta, tq, tq2, ts, ts2;
    TL_TRY(encode_kmajor(&ta, A, M, K, kQBM));
    TL_TRY(encode_q8(&tq, B.q, n_src, K, qrows));
    tq2 = tq;
    if (PAIRS) TL_TRY(encode_q8(&tq2, B.q2, n_src, K, qrows));
    ts = tq;
    ts2 = tq;
    if (!F8) {
        TL_TRY(encode_scales(&ts, B.sT, n_src, K / kQBK, qrows));
        ts2 = ts;
        if (PAIRS) TL_TRY(encode_scales(&ts2, B.sT2, n_src, K / kQBK, qrows));
    }
    auto kern = gemm_q8_kernel<EPI, F8, PAIRS, MT>;
    static std::once_flag once;  // per instantiation
    static cudaError_t attr_err = cudaSuccess;
    std::call_once(once, [&] {
        attr_err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        static_cast<int>(Cfg::kSmem));
    });
    if (attr_err != cudaSuccess) return set_error(TL_ERR_CUDA, "gemm_q8 smem attribute: %s", cudaGetErrorString(attr_err));
    const int tiles = ((N + Cfg::BN - 1) / Cfg::BN) * ((M + MT * kQBM - 1) / (MT * kQBM)) * ksplit;
    const int grid = std::min(tiles, sm_count());
    GemmArgs g{M, N, K, C, ldc, err, ksplit};
    kern<<<grid, Q8Warps<q8_epi_warps<EPI>()>::kThreads, Cfg::kSmem, s>>>(ta, tq, tq2, ts, ts2, g);
    return check_launch("gemm_q8");
}

// 256-row tiles (MT = 2) once there are more than 128 rows; e5m2 weights when sT is null.
bool use_mt2(int M, int /*N*/) { return M > kQBM; }

template <int EPI, bool PAIRS>
tl_status dispatch_q8(const __half* A, int M, int K, const Q8Weights& B, int N, void* C, int ldc, int* err,
                      cudaStream_t s, int ksplit) {
    if (use_mt2(M, N))
        return B.sT ? launch_q8<EPI, false, PAIRS, 2>(A, M, K, B, N, C, ldc, err, s, ksplit)
                    : launch_q8<EPI, true, PAIRS, 2>(A, M, K, B, N, C, ldc, err, s, ksplit);
    return B.sT ? launch_q8<EPI, false, PAIRS, 1>(A, M, K, B, N, C, ldc, err, s, ksplit)
                : launch_q8<EPI, true, PAIRS, 1>(A, M, K, B, N, C, ldc, err, s, ksplit);
}

// out[m][j] (fp16) = silu(sum_r P_r[m][g]) * sum_r P_r[m][g + 128], g = 256 (j / 128) + j % 128:
// the split-K partials of a gate|up GEMM of 1 x 256 tiles (128 gate then 128
// up columns) summed in order r = 0, 1, ... (modules.cpp:99-112).
__global__ void k_swiglu_rows(__half* out, const float* part, int ks, size_t stride, int M, int F) {
    const size_t total = static_cast<size_t>(M) * F;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const size_t m = i / F;
        const int j = static_cast<int>(i % F);
        const size_t gcol = static_cast<size_t>(j / 128) * 256 + j % 128;
        const float* row = part + m * 2 * static_cast<size_t>(F);
        float gv = 0.f, uv = 0.f;
        for (int r = 0; r < ks; r++) {
            gv += row[r * stride + gcol];
            uv += row[r * stride + gcol + 128];
        }
        out[m * F + j] = __float2half_rn((gv / (1.0f + expf(-gv))) * uv);
    }
}

// Split count for few output tiles: the K ranges (1..16, each >= 4 blocks)
// whose (tile, range) pairs fill the SMs best, fewest ranges on a tie.
int pick_ksplit(int tiles, int nk, size_t per_split_floats, size_t part_floats) {
    const int sms = sm_count();
    int best = 1;
    double best_eff = 0.0;
    for (int ks = 1; ks <= 16; ks++) {
        if (ks > 1 && nk / ks < 4) break;
        if (static_cast<size_t>(ks) * per_split_floats > part_floats) break;
        const int units = tiles * ks;
        const int waves = (units + sms - 1) / sms;
        const double eff = static_cast<double>(units) / (static_cast<double>(waves) * sms);
        if (eff > best_eff + 1e-9) {
            best_eff = eff;
            best = ks;
        }
    }
    // equal ranges that cover nk
    const int per = (nk + best - 1) / best;
    return (nk + per - 1) / per;
}

__global__ void k_transpose_scales(float* dst, const float* src, int n, int groups) {
    const size_t total = static_cast<size_t>(n) * groups;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const size_t row = i / groups, gi = i % groups;
        dst[gi * n + row] = src[i];
    }
}

tl_status check_q8(const __half* A, int M, int K, const Q8Weights& B, int N, const void* C) {
    TL_REQUIRE(A && B.q && C && M > 0 && N > 0 && K > 0, "gemm_q8: bad arguments");
    TL_REQUIRE(K % kQBK == 0, "gemm_q8: K = %d must be a multiple of %d", K, kQBK);
    TL_REQUIRE(((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(B.q) | reinterpret_cast<uintptr_t>(C) |
                 reinterpret_cast<uintptr_t>(B.q2) | reinterpret_cast<uintptr_t>(B.sT) |
                 reinterpret_cast<uintptr_t>(B.sT2)) & 15) == 0,
               "gemm_q8: operands must be 16-byte aligned");
    TL_REQUIRE(N % 4 == 0, "gemm_q8: N = %d must be a multiple of 4 (scale rows of 16 bytes)", N);
    return TL_OK;
}

}  // namespace

tl_status gemm_q8(int epi, const __half* A, int M, int K, const Q8Weights& B, int N, void* C, int ldc, int* err,
                  cudaStream_t s) {
    TL_TRY(check_q8(A, M, K, B, N, C));
    switch (epi) {
        case kEpiStoreF32:
            TL_REQUIRE(ldc >= N && ldc % 4 == 0, "gemm_q8: ldc");
            return dispatch_q8<kEpiStoreF32, false>(A, M, K, B, N, C, ldc, err, s, 1);
        case kEpiAddF32:
            TL_REQUIRE(ldc >= N && ldc % 4 == 0, "gemm_q8: ldc");
            return dispatch_q8<kEpiAddF32, false>(A, M, K, B, N, C, ldc, err, s, 1);
        case kEpiSwiGluF16:
            TL_REQUIRE(B.q2 && (B.sT2 || !B.sT) && N % 256 == 0 && ldc >= N / 2 && ldc % 8 == 0,
                       "gemm_q8 swiglu: up weights, N %% 256, ldc %% 8");
            return dispatch_q8<kEpiSwiGluF16, true>(A, M, K, B, N, C, ldc, err, s, 1);
        default:
            return set_error(TL_ERR_INVALID_ARGUMENT, "gemm_q8: unknown epilogue %d", epi);
    }
}

tl_status gemm_q8_splitk(const __half* A, int M, int K, const Q8Weights& B, int N, float* part, size_t part_floats,
                         int* ksplit, int* err, cudaStream_t s) {
    TL_TRY(check_q8(A, M, K, B, N, part));
    TL_REQUIRE(ksplit, "gemm_q8_splitk: null ksplit");
    TL_REQUIRE(static_cast<size_t>(M) * N <= part_floats, "gemm_q8_splitk: part holds %zu floats, %zu needed",
               part_floats, static_cast<size_t>(M) * N);
    // 128 x 256 tiles (the pair layout swiglu_rows reads)
    const int tiles = ((N + 255) / 256) * ((M + kQBM - 1) / kQBM);
    const int ks = pick_ksplit(tiles, K / kQBK, static_cast<size_t>(M) * N, part_floats);
    *ksplit = ks;
    const bool f8 = !B.sT;
    if (B.q2) {
        TL_REQUIRE((B.sT2 || f8) && N % 256 == 0, "gemm_q8_splitk pairs: up weights, N %% 256");
        return f8 ? launch_q8<kEpiStoreF32, true, true, 1>(A, M, K, B, N, part, N, err, s, ks)
                  : launch_q8<kEpiStoreF32, false, true, 1>(A, M, K, B, N, part, N, err, s, ks);
    }
    return f8 ? launch_q8<kEpiStoreF32, true, false, 1>(A, M, K, B, N, part, N, err, s, ks)
              : launch_q8<kEpiStoreF32, false, false, 1>(A, M, K, B, N, part, N, err, s, ks);
}

tl_status swiglu_rows(__half* out, const float* part, int ks, size_t stride, int M, int F, cudaStream_t s) {
    TL_REQUIRE(out && part && ks > 0 && M > 0 && F % 128 == 0, "swiglu_rows: bad arguments");
    const size_t total = static_cast<size_t>(M) * F;
    const int grid = static_cast<int>(std::min<size_t>(4 * sm_count(), (total + 255) / 256));
    k_swiglu_rows<<<grid, 256, 0, s>>>(out, part, ks, stride, M, F);
    return check_launch("swiglu_rows");
}

tl_status transpose_scales(float* dst, const float* src, int n, int groups, cudaStream_t s) {
    TL_REQUIRE(dst && src && n > 0 && groups > 0, "transpose_scales: bad arguments");
    const size_t total = static_cast<size_t>(n) * groups;
    const int grid = static_cast<int>(std::min<size_t>(4096, (total + 255) / 256));
    k_transpose_scales<<<grid, 256, 0, s>>>(dst, src, n, groups);
    return check_launch("transpose_scales");
}

}  // namespace tl

using namespace tl;

extern "C" {

tl_status tl_gemm_q8(void* c, const void* a, const void* b, const float* inv_scales_t, const void* b2,
                     const float* inv_scales_t2, size_t m, size_t n, size_t k, size_t ldc, int epilogue,
                     void* stream) {
    clear_error();
    TL_REQUIRE(m < (1u << 30) && n < (1u << 30) && k < (1u << 30) && ldc < (1u << 30), "tl_gemm_q8: sizes");
    Q8Weights w;
    w.q = b;
    w.sT = inv_scales_t;
    w.q2 = b2;
    w.sT2 = inv_scales_t2;
    return gemm_q8(epilogue, static_cast<const __half*>(a), static_cast<int>(m), static_cast<int>(k), w,
                   static_cast<int>(n), c, static_cast<int>(ldc), nullptr, as_stream(stream));
}

}  // extern "C"
