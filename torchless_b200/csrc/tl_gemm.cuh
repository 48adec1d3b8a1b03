// tl_gemm.cuh -- tcgen05 tensor-core GEMM for the batched paths (prefill,
// batched decode): C[M, N] = A[M, K] B[N, K]^T, A and B fp16 row-major
// (both K-contiguous), fp32 accumulation in tensor memory (tl_gemm.cu).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "torchless_b200.h"

namespace tl {

enum GemmEpilogue : int {
    kEpiStoreF32 = 0,  // C (fp32, row stride ldc) = A B^T
    kEpiAddF32 = 1,    // C += A B^T (residual add, modules.cpp:128, 142)
    kEpiSwiGluF16 = 2, // B rows in blocks of 256 = [128 gate rows | 128 up rows]; C (fp16, row stride
                       // ldc) column n0 / 2 + j = silu(gate_j) * up_j (modules.cpp:99-112)
};

// Shapes: K % 64 == 0, A / B / C 16-byte aligned; any M, N (tails masked).
// `err` (device int, may be null) receives a nonzero code if a bounded
// device-side wait gave up.
tl_status gemm_f16(int epilogue, const __half* A, int M, int K, const __half* B, int N, void* C, int ldc, int* err,
                   cudaStream_t s);

// Split-K for few output tiles (small M): K is cut into *ksplit ranges (chosen
// here, 1..8, so that the (tile, range) pairs fill the SMs) and range r stores
// its product into part + r M N ([M, N] row-major fp32).  The consumer sums
// the ranges in order r = 0, 1, ... (fused into its own kernel).
tl_status gemm_f16_splitk(const __half* A, int M, int K, const __half* B, int N, float* part, size_t part_floats,
                          int* ksplit, int* err, cudaStream_t s);

// 8-bit weights for the dequantising GEMM (tl_gemm_q8.cu): B [N, K] int8
// (row-major, K contiguous) with sT = 1/s transposed to [K / 64][N], or e5m2
// bytes with sT null.  SwiGLU: q / sT are the gate rows and q2 / sT2 the up
// rows of the same shape [N / 2, K]; B tile rows 0..127 are gate rows and
// 128..255 the same up rows.
struct Q8Weights {
    const void* q = nullptr;
    const float* sT = nullptr;
    const void* q2 = nullptr;
    const float* sT2 = nullptr;
};

// C = A B^T with B dequantised in shared memory (w = fp16(q) * fp16(1/s),
// rounded to fp16; e5m2 widened exactly), same epilogues and split-K
// contract as gemm_f16 / gemm_f16_splitk.  N % 4 == 0 (SwiGLU: N % 256 == 0).
tl_status gemm_q8(int epilogue, const __half* A, int M, int K, const Q8Weights& B, int N, void* C, int ldc, int* err,
                  cudaStream_t s);
tl_status gemm_q8_splitk(const __half* A, int M, int K, const Q8Weights& B, int N, float* part, size_t part_floats,
                         int* ksplit, int* err, cudaStream_t s);
// With B.q2 set (gate / up pairs), gemm_q8_splitk stores the pair tiles' split
// partials (columns 256 b .. 256 b + 127 gate, then 128 up) and swiglu_rows
// combines them: out[m][j] = silu(gate) * up as fp16 (modules.cpp:99-112).
tl_status swiglu_rows(__half* out, const float* part, int ks, size_t stride, int M, int F, cudaStream_t s);
// dst[g][i] = src[i][g] for a [n][groups] scale array.
tl_status transpose_scales(float* dst, const float* src, int n, int groups, cudaStream_t s);

}  // namespace tl
