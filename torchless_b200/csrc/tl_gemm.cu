// tl_gemm.cu -- tcgen05 GEMM (sm_100a): C = A B^T, fp16 operands, fp32
// accumulation in tensor memory, fused epilogues.
//
// Persistent: one CTA per SM walks 128 x BN tiles of C.  Warp roles (192 threads):
//   warp 0      TMA producer: 128-row A and BN-row B boxes of 64 K-elements
//               (128 bytes, SWIZZLE_128B) into a ring of shared-memory stages,
//               completing on per-stage `full` mbarriers;
//   warp 1      allocates 2 x BN tensor-memory columns (two accumulators) and
//               issues tcgen05.mma (kind::f16, M 128, N BN, K 16; 4 per stage)
//               from one thread; tcgen05.commit frees each stage (`empty`) and
//               signals a finished accumulator (`tfull`);
//   warps 2-5   epilogue: tcgen05.ld of the accumulator rows (warp w reads
//               tensor-memory lanes 32 (w % 4) ..), fused op, global stores,
//               then hand the accumulator back (`tempty`) while the next
//               tile's MMAs already run in the other one.
// Every mbarrier wait is bounded by ~2 s of %globaltimer; on expiry the
// kernel records an error code, stops issuing, lets the work in flight drain
// (bounded), frees its tensor memory and returns.
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
constexpr int kBM = 128, kBK = 64;
constexpr int kGemmThreads = 192;

template <int BN>
struct GemmCfg {
    static constexpr int kStages = BN == 256 ? 4 : 6;
    static constexpr int kABytes = kBM * kBK * 2;
    static constexpr int kBBytes = BN * kBK * 2;
    static constexpr int kStageBytes = kABytes + kBBytes;
    // 1024-byte alignment slack (SWIZZLE_128B destinations) + stages + barriers
    static constexpr size_t kSmem = 1024 + static_cast<size_t>(kStages) * kStageBytes + 256;
    static_assert(2 * BN <= 512, "two accumulators must fit the 512 tensor-memory columns");
};

// Persistent: CTA c takes tiles c, c + G, ... (m fastest, so the CTAs that
// run together share B blocks: each weight block is read from HBM once).
// Two accumulators (2 x BN tensor-memory columns) let the epilogue of tile i
// run while the MMAs of tile i + 1 accumulate.
template <int BN, int EPI>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b, GemmArgs g) {
    using Cfg = GemmCfg<BN>;
    constexpr int S = Cfg::kStages;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(base + S * Cfg::kStageBytes);
    uint64_t* empty = full + S;
    uint64_t* tfull = empty + S;   // [2] accumulator ready
    uint64_t* tempty = tfull + 2;  // [2] accumulator drained by the epilogue
    uint64_t* mma_done = tempty + 2;  // every MMA this CTA issued has completed (before dealloc)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tm = (g.M + kBM - 1) / kBM, tn = (g.N + BN - 1) / BN, n_tiles = tm * tn * g.ksplit;
    const int nk_all = g.K / kBK, nk_per = (nk_all + g.ksplit - 1) / g.ksplit;
    // tile -> (m tile fastest, n tile, K split); its K-block range [kb0, kb0 + nk)
    auto tile_of = [&](int t, int& m0, int& n0, int& kb0, int& nk) {
        m0 = (t % tm) * kBM;
        const int r = t / tm;
        n0 = (r % tn) * BN;
        kb0 = (r / tn) * nk_per;
        nk = max(0, min(nk_all, kb0 + nk_per) - kb0);
    };

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) {
            bar_init(&full[s], 1);
            bar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; b++) {
            bar_init(&tfull[b], 1);
            bar_init(&tempty[b], 4);  // one arrival per epilogue warp
        }
        bar_init(mma_done, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {  // two accumulators: 2 BN fp32 columns x 128 lanes
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(tmem_slot)),
                     "r"(2 * BN));
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

    if (warp == 0) {
        if (lane == 0) {
            uint32_t it = 0;
            for (int tile = blockIdx.x; tile < n_tiles && !*abort_flag; tile += gridDim.x) {
                int m0, n0, kb0, nk;
                tile_of(tile, m0, n0, kb0, nk);
                for (int kb = kb0; kb < kb0 + nk; kb++, it++) {
                    const int s = it % S;
                    if (it >= S && !bar_wait_ab(&empty[s], ((it / S) - 1) & 1, abort_flag)) {
                        fail(kGemmErrSlot);
                        break;
                    }
                    uint8_t* sa = base + s * Cfg::kStageBytes;
                    bar_expect_tx(&full[s], Cfg::kStageBytes);
                    tma_load_2d(sa, &tma_a, kb * kBK, m0, &full[s]);
                    tma_load_2d(sa + Cfg::kABytes, &tma_b, kb * kBK, n0, &full[s]);
                }
            }
            // every copy issued lands before the CTA exits
            const uint32_t first = it > static_cast<uint32_t>(S) ? it - S : 0;
            for (uint32_t k = first; k < it; k++) bar_wait(&full[k % S], (k / S) & 1);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idesc = idesc_f16<BN>();
            uint32_t it = 0;
            int i = 0;
            for (int tile = blockIdx.x; tile < n_tiles && !*abort_flag; tile += gridDim.x, i++) {
                const int buf = i & 1;
                if (i >= 2 && !bar_wait_ab(&tempty[buf], ((i / 2) - 1) & 1, abort_flag)) {
                    fail(kGemmErrAccFree);
                    break;
                }
                tc_fence_after();
                const uint32_t dt = tmem + static_cast<uint32_t>(buf * BN);
                int m0, n0, kb0, nk;
                tile_of(tile, m0, n0, kb0, nk);
                bool ok = true;
                for (int kb = 0; kb < nk; kb++, it++) {
                    const int s = it % S;
                    if (!bar_wait_ab(&full[s], (it / S) & 1, abort_flag)) {
                        fail(kGemmErrStage);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sa = su32(base + s * Cfg::kStageBytes);
                    const uint64_t da = sdesc_k128(sa), db = sdesc_k128(sa + Cfg::kABytes);
#pragma unroll
                    for (int k = 0; k < kBK / 16; k++)  // K 16 per MMA = 32 bytes along the swizzled row
                        umma_f16(dt, da + 2 * k, db + 2 * k, idesc, (kb | k) != 0);
                    umma_commit(&empty[s]);  // stage free once these MMAs have read it
                }
                umma_commit(&tfull[buf]);  // accumulator ready (also on abort: frees the epilogue)
                if (!ok) break;
            }
            // also on abort: tensor memory is freed only after every issued MMA has written it
            umma_commit(mma_done);
            bar_wait(mma_done, 0);
        }
    } else {
        const int sub = warp & 3;  // tensor-memory lanes 32 sub .. (tcgen05.ld lane quarter of this warp)
        int i = 0;
        for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, i++) {
            const int buf = i & 1;
            if (!bar_wait_ab(&tfull[buf], (i / 2) & 1, abort_flag)) {
                fail(kGemmErrAccReady);
                break;
            }
            tc_fence_after();
            if (*abort_flag) break;
            int m0, n0, kb0, nk;
            tile_of(tile, m0, n0, kb0, nk);
            GemmArgs gs = g;  // a K split stores into its own slice
            if (g.ksplit > 1)
                gs.C = static_cast<float*>(g.C) + static_cast<size_t>(kb0 / nk_per) * g.M * g.ldc;
            gemm_epilogue<BN, EPI>(gs, tmem + static_cast<uint32_t>(buf * BN), m0, n0, sub, lane);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(&tempty[buf])) : "memory");
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * BN));
    }
}

template <int BN, int EPI>
tl_status launch_gemm(const __half* A, int M, int K, const __half* B, int N, void* C, int ldc, int* err,
                      cudaStream_t s, int ksplit = 1) {
    CUtensorMap ta, tb;
    TL_TRY(encode_kmajor(&ta, A, M, K, kBM));
    TL_TRY(encode_kmajor(&tb, B, N, K, BN));
    auto kern = gemm_tc_kernel<BN, EPI>;
    static std::once_flag once;  // per instantiation
    static cudaError_t attr_err = cudaSuccess;
    std::call_once(once, [&] {
        attr_err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        static_cast<int>(GemmCfg<BN>::kSmem));
    });
    if (attr_err != cudaSuccess)
        return set_error(TL_ERR_CUDA, "gemm smem attribute: %s", cudaGetErrorString(attr_err));
    const int tiles = ((N + BN - 1) / BN) * ((M + kBM - 1) / kBM) * ksplit;
    const int grid = std::min(tiles, sm_count());
    GemmArgs g{M, N, K, C, ldc, err, ksplit};
    kern<<<grid, kGemmThreads, GemmCfg<BN>::kSmem, s>>>(ta, tb, g);
    return check_launch("gemm_tc");
}

}  // namespace

tl_status gemm_f16(int epi, const __half* A, int M, int K, const __half* B, int N, void* C, int ldc, int* err,
                   cudaStream_t s) {
    TL_REQUIRE(A && B && C && M > 0 && N > 0 && K > 0, "gemm: bad arguments");
    TL_REQUIRE(K % kBK == 0, "gemm: K = %d must be a multiple of %d", K, kBK);
    TL_REQUIRE(((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(B) | reinterpret_cast<uintptr_t>(C)) &
                15) == 0,
               "gemm: operands must be 16-byte aligned");
    switch (epi) {
        case kEpiStoreF32:
            TL_REQUIRE(ldc >= N && ldc % 4 == 0, "gemm: ldc");
            return launch_gemm<256, kEpiStoreF32>(A, M, K, B, N, C, ldc, err, s);
        case kEpiAddF32:
            TL_REQUIRE(ldc >= N && ldc % 4 == 0, "gemm: ldc");
            return launch_gemm<256, kEpiAddF32>(A, M, K, B, N, C, ldc, err, s);
        case kEpiSwiGluF16:
            TL_REQUIRE(N % 256 == 0 && ldc >= N / 2 && ldc % 8 == 0, "gemm swiglu: N %% 256, ldc %% 8");
            return launch_gemm<256, kEpiSwiGluF16>(A, M, K, B, N, C, ldc, err, s);
        default:
            return set_error(TL_ERR_INVALID_ARGUMENT, "gemm: unknown epilogue %d", epi);
    }
}

tl_status gemm_f16_splitk(const __half* A, int M, int K, const __half* B, int N, float* part, size_t part_floats,
                          int* ksplit, int* err, cudaStream_t s) {
    TL_REQUIRE(A && B && part && ksplit && M > 0 && N > 0 && K > 0, "gemm splitk: bad arguments");
    TL_REQUIRE(K % kBK == 0 && N % 4 == 0, "gemm splitk: K = %d (multiple of %d), N = %d (multiple of 4)", K, kBK, N);
    TL_REQUIRE(((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(B) | reinterpret_cast<uintptr_t>(part)) &
                15) == 0,
               "gemm splitk: operands must be 16-byte aligned");
    TL_REQUIRE(static_cast<size_t>(M) * N <= part_floats, "gemm splitk: part holds %zu floats, %zu needed",
               part_floats, static_cast<size_t>(M) * N);
    // enough (output tile, K range) pairs for every SM; each range >= 4 K blocks and none empty
    const int tiles = ((N + 255) / 256) * ((M + kBM - 1) / kBM);
    const int nk = K / kBK;
    int ks = std::max(1, std::min({8, sm_count() / std::max(1, tiles), nk / 4}));
    while (ks > 1 && static_cast<size_t>(ks) * M * N > part_floats) ks--;
    const int per = (nk + ks - 1) / ks;
    ks = (nk + per - 1) / per;
    *ksplit = ks;
    return launch_gemm<256, kEpiStoreF32>(A, M, K, B, N, part, N, err, s, ks);
}

}  // namespace tl

using namespace tl;

extern "C" {

tl_status tl_gemm_f16(void* c, const void* a, const void* b, size_t m, size_t n, size_t k, size_t ldc, int epilogue,
                      void* stream) {
    clear_error();
    TL_REQUIRE(m < (1u << 30) && n < (1u << 30) && k < (1u << 30) && ldc < (1u << 30), "tl_gemm_f16: sizes");
    return gemm_f16(epilogue, static_cast<const __half*>(a), static_cast<int>(m), static_cast<int>(k),
                    static_cast<const __half*>(b), static_cast<int>(n), c, static_cast<int>(ldc), nullptr,
                    as_stream(stream));
}

}  // extern "C"
