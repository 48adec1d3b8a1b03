// tl_gemv.cu -- launch configuration for the fused GEMV kernels (tl_gemv.cuh).
#include <algorithm>

#include "tl_gemv.cuh"
#include "tl_kernels.h"

namespace tl {

namespace {

constexpr int kRowsI8 = 8;   // rows per iteration, int8 kernels
constexpr int kRowsF32 = 4;  // rows per iteration, fp32 kernels

// Chunks per thread for a row of d int8 columns: keep T = d/(16C) <= 512.
int chunks_for(size_t d) { return (d / 16 <= 512) ? 1 : 2; }

template <typename K>
tl_status launch(K kernel, int grid, int block, size_t smem, cudaStream_t s, bool pdl,
                 const char* name, void* arg) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(block);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    void* args[] = {arg};
    cudaError_t e = cudaLaunchKernelExC(&cfg, reinterpret_cast<const void*>(kernel), args);
    if (e != cudaSuccess)
        return set_error(TL_ERR_CUDA, "launch of %s failed: %s", name, cudaGetErrorString(e));
    return TL_OK;
}

// One wave of co-resident CTAs, at most one per work unit.
template <typename K>
int wave_grid(K kernel, int block, size_t smem, int units) {
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, block, smem) != cudaSuccess ||
        per_sm < 1)
        per_sm = 1;
    return std::max(1, std::min(units, per_sm * sm_count()));
}

template <int C, int MAXT, bool INV, bool NORM, int EPI, bool F8>
tl_status run_i8(GemvI8Args a, cudaStream_t s, bool pdl) {
    auto k = gemv_i8_kernel<kRowsI8, C, MAXT, INV, NORM, EPI, F8>;
    const int T = a.d / (16 * C);
    const int out_rows = (EPI == kSwiGLU) ? kRowsI8 / 2 : kRowsI8;
    const int units = (a.n + out_rows - 1) / out_rows;
    const size_t smem = (32 + 2 * (T / 32) * kRowsI8) * sizeof(float);
    const int grid = wave_grid(k, T, smem, units);
    return launch(k, grid, T, smem, s, pdl, "gemv_i8", &a);
}

template <bool INV, bool NORM, int EPI, bool F8 = false>
tl_status dispatch_i8(const GemvI8Args& a, cudaStream_t s, bool pdl) {
    const int C = chunks_for(a.d);
    const int T = a.d / (16 * C);
    if (C == 1) {
        if (T <= 128) return run_i8<1, 128, INV, NORM, EPI, F8>(a, s, pdl);
        if (T <= 256) return run_i8<1, 256, INV, NORM, EPI, F8>(a, s, pdl);
        return run_i8<1, 512, INV, NORM, EPI, F8>(a, s, pdl);
    }
    return run_i8<2, 512, INV, NORM, EPI, F8>(a, s, pdl);
}

template <int MAXT, bool NORM, bool ARGMAX>
int grid_f32(const GemvF32Args& a) {
    auto k = gemv_f32_kernel<kRowsF32, MAXT, NORM, ARGMAX>;
    const int T = a.d / 16;
    const size_t smem = (32 + 2 * (T / 32) * kRowsF32) * sizeof(float);
    return wave_grid(k, T, smem, (a.n + kRowsF32 - 1) / kRowsF32);
}

template <int MAXT, bool NORM, bool ARGMAX>
tl_status run_f32(GemvF32Args a, cudaStream_t s, bool pdl) {
    auto k = gemv_f32_kernel<kRowsF32, MAXT, NORM, ARGMAX>;
    const int T = a.d / 16;
    const size_t smem = (32 + 2 * (T / 32) * kRowsF32) * sizeof(float);
    const int grid = grid_f32<MAXT, NORM, ARGMAX>(a);
    return launch(k, grid, T, smem, s, pdl, "gemv_f32", &a);
}

template <bool NORM, bool ARGMAX>
tl_status dispatch_f32(const GemvF32Args& a, cudaStream_t s, bool pdl) {
    const int T = a.d / 16;
    if (T <= 128) return run_f32<128, NORM, ARGMAX>(a, s, pdl);
    if (T <= 256) return run_f32<256, NORM, ARGMAX>(a, s, pdl);
    if (T <= 512) return run_f32<512, NORM, ARGMAX>(a, s, pdl);
    return run_f32<1024, NORM, ARGMAX>(a, s, pdl);
}

template <bool NORM, bool ARGMAX>
int dispatch_grid_f32(const GemvF32Args& a) {
    const int T = a.d / 16;
    if (T <= 128) return grid_f32<128, NORM, ARGMAX>(a);
    if (T <= 256) return grid_f32<256, NORM, ARGMAX>(a);
    if (T <= 512) return grid_f32<512, NORM, ARGMAX>(a);
    return grid_f32<1024, NORM, ARGMAX>(a);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

bool gemv_i8_fast_ok(size_t n, size_t d, size_t n_scales, const void* w, const void* x) {
    if (n == 0 || d == 0 || d % 512 != 0 || d > 16384) return false;
    if (n_scales * 64 != n * d) return false;
    if (n > 0x7fffffff) return false;
    const int C = chunks_for(d);
    if ((d / (16 * C)) % 32 != 0) return false;
    return aligned16(w) && aligned16(x);
}

bool gemv_f32_fast_ok(size_t n, size_t d, const void* w, const void* x) {
    if (n == 0 || d == 0 || d % 512 != 0 || d / 16 > 1024 || n > 0x7fffffff) return false;
    return aligned16(w) && aligned16(x);
}

tl_status launch_gemv_i8(const GemvI8Args& a, I8Mode mode, bool inv, bool norm, cudaStream_t s,
                         bool pdl) {
    if (a.f8) {  // fp8 weights (model paths: the fused modes of the decode step)
        switch (mode) {
            case I8Mode::Store:
                return norm ? dispatch_i8<true, true, kStore, true>(a, s, pdl)
                            : dispatch_i8<true, false, kStore, true>(a, s, pdl);
            case I8Mode::AddResidual: return dispatch_i8<true, false, kAddResidual, true>(a, s, pdl);
            case I8Mode::SwiGLU: return dispatch_i8<true, true, kSwiGLU, true>(a, s, pdl);
        }
        return set_error(TL_ERR_INVALID_ARGUMENT, "unknown GEMV mode");
    }
    switch (mode) {
        case I8Mode::Store:
            if (inv) return norm ? dispatch_i8<true, true, kStore>(a, s, pdl)
                                 : dispatch_i8<true, false, kStore>(a, s, pdl);
            return norm ? dispatch_i8<false, true, kStore>(a, s, pdl)
                        : dispatch_i8<false, false, kStore>(a, s, pdl);
        case I8Mode::AddResidual:
            if (inv) return dispatch_i8<true, false, kAddResidual>(a, s, pdl);
            return dispatch_i8<false, false, kAddResidual>(a, s, pdl);
        case I8Mode::SwiGLU:
            if (inv) return norm ? dispatch_i8<true, true, kSwiGLU>(a, s, pdl)
                                 : dispatch_i8<true, false, kSwiGLU>(a, s, pdl);
            return dispatch_i8<false, false, kSwiGLU>(a, s, pdl);
    }
    return set_error(TL_ERR_INVALID_ARGUMENT, "unknown GEMV mode");
}

tl_status launch_gemv_f32(const GemvF32Args& a, bool norm, bool argmax, cudaStream_t s, bool pdl) {
    if (norm) return argmax ? dispatch_f32<true, true>(a, s, pdl) : dispatch_f32<true, false>(a, s, pdl);
    return argmax ? dispatch_f32<false, true>(a, s, pdl) : dispatch_f32<false, false>(a, s, pdl);
}

int gemv_f32_grid(size_t n, size_t d, bool norm, bool argmax) {
    GemvF32Args a = {};
    a.n = static_cast<int>(n);
    a.d = static_cast<int>(d);
    if (norm) return argmax ? dispatch_grid_f32<true, true>(a) : dispatch_grid_f32<true, false>(a);
    return argmax ? dispatch_grid_f32<false, true>(a) : dispatch_grid_f32<false, false>(a);
}

}  // namespace tl
