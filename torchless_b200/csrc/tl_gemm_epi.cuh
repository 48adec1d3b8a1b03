// tl_gemm_epi.cuh -- the epilogue shared by the tcgen05 GEMMs (tl_gemm.cu,
// tl_gemm_q8.cu): one 128 x BN fp32 accumulator from tensor memory to global
// memory, stored, added to a residual, or through SiLU(gate) * up.
#pragma once

#include <cuda_fp16.h>
#include <math.h>
#include <stdint.h>

#include "tl_gemm.cuh"
#include "tl_tc.cuh"

namespace tl {

struct GemmArgs {
    int M, N, K;
    void* C;
    int ldc;
    int* err;
    int ksplit;  // K-block ranges per output tile (1: none); split s stores into C + s * M * ldc
};

// The epilogue of one 128 x BN accumulator (tensor-memory columns tcol ..)
// for tile rows m0 .., columns n0 ..; warp `sub` (tensor-memory lanes
// 32 sub ..) of the epilogue warps.  Column part `part` of `parts`: the warp
// takes accumulator columns [part, part + 1) x BN / parts (SwiGLU: output
// columns [part, part + 1) x BN / (2 parts)), so 8 warps can share a tile.
template <int BN, int EPI>
__device__ __forceinline__ void gemm_epilogue(const GemmArgs& g, uint32_t tcol, int m0, int n0, int sub, int lane,
                                              int part = 0, int parts = 1) {
    const int row = m0 + sub * 32 + lane;
    const uint32_t tl = tcol + (static_cast<uint32_t>(sub * 32) << 16);
    if (EPI == kEpiSwiGluF16) {
        __half* out = static_cast<__half*>(g.C);
        const int span = BN / 2 / parts;
#pragma unroll 1
        for (int c0 = part * span; c0 < (part + 1) * span; c0 += 32) {
            float gv[32], uv[32];
            tc::tmem_ld32(tl + c0, gv);
            tc::tmem_ld32(tl + BN / 2 + c0, uv);
            const int col = n0 / 2 + c0;
            if (row < g.M && col < g.N / 2) {
                __half2 h[16];
#pragma unroll
                for (int j = 0; j < 32; j += 2) {
                    const float a0 = (gv[j] / (1.0f + expf(-gv[j]))) * uv[j];  // silu * up (kernels.cpp:98-102)
                    const float a1 = (gv[j + 1] / (1.0f + expf(-gv[j + 1]))) * uv[j + 1];
                    h[j / 2] = __floats2half2_rn(a0, a1);
                }
                uint4* dst = reinterpret_cast<uint4*>(out + static_cast<size_t>(row) * g.ldc + col);
#pragma unroll
                for (int q = 0; q < 4; q++) dst[q] = reinterpret_cast<const uint4*>(h)[q];
            }
        }
    } else {
        float* out = static_cast<float*>(g.C);
        const int span = BN / parts;
#pragma unroll 1
        for (int c0 = part * span; c0 < (part + 1) * span; c0 += 32) {
            float v[32];
            tc::tmem_ld32(tl + c0, v);
            if (row < g.M) {
                float* dst = out + static_cast<size_t>(row) * g.ldc + n0 + c0;
                const int rem = g.N - (n0 + c0);
                if (rem >= 32) {
#pragma unroll
                    for (int j = 0; j < 32; j += 4) {
                        float4 x = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
                        if (EPI == kEpiAddF32) {
                            const float4 r = *reinterpret_cast<const float4*>(dst + j);
                            x.x += r.x; x.y += r.y; x.z += r.z; x.w += r.w;
                        }
                        *reinterpret_cast<float4*>(dst + j) = x;
                    }
                } else {
                    for (int j = 0; j < rem; j++) dst[j] = (EPI == kEpiAddF32) ? dst[j] + v[j] : v[j];
                }
            }
        }
    }
}

}  // namespace tl
