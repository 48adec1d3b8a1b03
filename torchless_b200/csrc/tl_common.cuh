// tl_common.cuh -- shared host/device helpers for the sm_100a kernels.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "torchless_b200.h"

namespace tl {

// Codes a kernel writes into the model's device error word when a bounded
// wait gives up (or an input is out of range); the host reads the word after
// each step.  1-5: persistent decode step, 6: batched tensor-parallel
// exchange, 11-16: tensor-core prefill attention, 21-24: tcgen05 GEMM.
enum DeviceErr : int {
    kDevErrBarrier = 1,      // decode: grid barrier, readiness counter or TP exchange
    kDevErrRingFull = 2,     // decode: a weight tile did not arrive
    kDevErrRingEmpty = 3,    // decode: a ring slot was not released
    kDevErrInput = 5,        // decode: token or position out of range
    kDevErrBatchXchg = 6,    // batched TP: a peer's row did not arrive
    kDevErrAttnLoad = 11,    // prefill attention: K / V load slot
    kDevErrAttnMma = 12,     // prefill attention: MMA issue waits
    kDevErrAttnS = 13,       // prefill attention: scores not ready
    kDevErrAttnPv = 14,      // prefill attention: P V not done
    kDevErrAttnEpi = 16,     // prefill attention: epilogue
    kGemmErrSlot = 21,       // GEMM: stage slot not freed
    kGemmErrStage = 22,      // GEMM: stage data did not arrive
    kGemmErrAccReady = 23,   // GEMM: accumulator not ready
    kGemmErrAccFree = 24,    // GEMM: accumulator not drained
};

// Records a formatted message for tl_last_error() and returns `s`.
tl_status set_error(tl_status s, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
void clear_error();

#define TL_CUDA_TRY(expr)                                                                  \
    do {                                                                                   \
        cudaError_t tl_e_ = (expr);                                                        \
        if (tl_e_ != cudaSuccess)                                                          \
            return ::tl::set_error(TL_ERR_CUDA, "%s failed: %s (%s:%d)", #expr,            \
                                   cudaGetErrorString(tl_e_), __FILE__, __LINE__);         \
    } while (0)

#define TL_TRY(expr)                         \
    do {                                     \
        tl_status tl_s_ = (expr);            \
        if (tl_s_ != TL_OK) return tl_s_;    \
    } while (0)

#define TL_REQUIRE(cond, ...)                                                      \
    do {                                                                           \
        if (!(cond)) return ::tl::set_error(TL_ERR_INVALID_ARGUMENT, __VA_ARGS__); \
    } while (0)

// Launch-time error check (configuration errors surface here, execution
// errors on the next synchronising call).
inline tl_status check_launch(const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess)
        return set_error(TL_ERR_CUDA, "launch of %s failed: %s", what, cudaGetErrorString(e));
    return TL_OK;
}

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// SM count of the current device (cached per device).
int sm_count();

// ---------------------------------------------------------------------------
// Device helpers
// ---------------------------------------------------------------------------

constexpr unsigned FULL = 0xffffffffu;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(FULL, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(FULL, v, o));
    return v;
}

// Block-wide sum; every thread gets the result.  `red` needs >= 32 floats.
__device__ __forceinline__ float block_sum(float v, float* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nw = (blockDim.x + 31) >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = (threadIdx.x < (unsigned)nw) ? red[threadIdx.x] : 0.0f;
    if (warp == 0) t = warp_sum(t);
    if (threadIdx.x == 0) red[0] = t;
    __syncthreads();
    return red[0];
}

// Reduce R per-lane values over the 32 lanes of a warp at once ("transpose
// reduction").  Afterwards lane l holds the full sum of value l / (32/R) in
// v[0].  R is a power of two <= 32.
template <int R>
__device__ __forceinline__ float warp_reduce_multi(float (&v)[R]) {
    const int lane = threadIdx.x & 31;
    int cnt = R;
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
        if (cnt > 1) {
            const bool upper = (lane & off) != 0;
            const int h = cnt >> 1;
#pragma unroll
            for (int i = 0; i < R / 2; i++) {
                if (i < h) {
                    const float send = upper ? v[i] : v[i + h];
                    const float keep = upper ? v[i + h] : v[i];
                    v[i] = keep + __shfl_xor_sync(FULL, send, off);
                }
            }
            cnt = h;
        } else {
            v[0] += __shfl_xor_sync(FULL, v[0], off);
        }
    }
    return v[0];
}

// Packed fp32x2 arithmetic (sm_100+): one instruction for two lanes of math.
__device__ __forceinline__ unsigned long long f2_bits(float2 a) {
    return (static_cast<unsigned long long>(__float_as_uint(a.y)) << 32) | __float_as_uint(a.x);
}
__device__ __forceinline__ float2 bits_f2(unsigned long long b) {
    return make_float2(__uint_as_float(static_cast<uint32_t>(b)),
                       __uint_as_float(static_cast<uint32_t>(b >> 32)));
}
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
    unsigned long long d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(f2_bits(a)), "l"(f2_bits(b)), "l"(f2_bits(c)));
    return bits_f2(d);
}
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
    unsigned long long d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(f2_bits(a)), "l"(f2_bits(b)));
    return bits_f2(d);
}

// Exact int8 -> fp32 for the four bytes of `w`: bias each byte to u = q + 128,
// splice it into the mantissa of 2^23 (giving 2^23 + u exactly), and let the
// caller subtract 2^23 + 128.  One byte-permute per value, no I2F.
constexpr float kI8Magic = 8388736.0f;  // 2^23 + 128
__device__ __forceinline__ void i8x4_biased(uint32_t w, float2& lo, float2& hi) {
    const uint32_t u = w ^ 0x80808080u;
    lo.x = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7540));
    lo.y = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7541));
    hi.x = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7542));
    hi.y = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7543));
}

// 16 int8 weights (one 16-byte chunk) dotted with 16 fp32 activations held as
// 8 float2 pairs; returns the fp32 sum (two packed accumulators).
__device__ __forceinline__ float dot16_i8(uint4 w, const float2 (&xp)[8]) {
    const float2 nb = make_float2(-kI8Magic, -kI8Magic);
    float2 acc0 = make_float2(0.f, 0.f), acc1 = make_float2(0.f, 0.f);
    const uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int j = 0; j < 4; j++) {
        float2 lo, hi;
        i8x4_biased(words[j], lo, hi);
        lo = fadd2(lo, nb);
        hi = fadd2(hi, nb);
        acc0 = ffma2(lo, xp[2 * j], acc0);
        acc1 = ffma2(hi, xp[2 * j + 1], acc1);
    }
    const float2 s = fadd2(acc0, acc1);
    return s.x + s.y;
}

// Sum over the 16 fp8 (e5m2) weights in w (byte j = column j) of weight * x:
// each byte is the high byte of the fp16 with the same value, so two byte
// permutes give the exact fp16 pairs of a word.
__device__ __forceinline__ float dot16_f8(uint4 w, const float2 (&xp)[8]) {
    float2 acc0 = make_float2(0.f, 0.f), acc1 = make_float2(0.f, 0.f);
    const uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const uint32_t p01 = __byte_perm(words[j], 0u, 0x1404), p23 = __byte_perm(words[j], 0u, 0x3424);
        const float2 lo = __half22float2(*reinterpret_cast<const __half2*>(&p01));
        const float2 hi = __half22float2(*reinterpret_cast<const __half2*>(&p23));
        acc0 = ffma2(lo, xp[2 * j], acc0);
        acc1 = ffma2(hi, xp[2 * j + 1], acc1);
    }
    const float2 s = fadd2(acc0, acc1);
    return s.x + s.y;
}

// Streaming 16-byte load that bypasses L1 allocation (weights are read once).
__device__ __forceinline__ uint4 ld_stream(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ float4 ld_stream_f4(const void* p) {
    uint4 r = ld_stream(p);
    return make_float4(__uint_as_float(r.x), __uint_as_float(r.y), __uint_as_float(r.z),
                       __uint_as_float(r.w));
}

// Programmatic dependent launch: wait for the producer grid's memory, and
// allow the next grid in the stream to start its prologue.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Argmax combine with the sample_max tie rule (main.cpp:10-21): larger value
// wins; equal values keep the smaller index.  NaN never wins.
__device__ __forceinline__ unsigned long long globaltimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// System scope (peer GPUs over NVLink): 64-bit counters and slots.
__device__ __forceinline__ void fence_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }
__device__ __forceinline__ void red_add_sys_u64(void* p, unsigned long long v) {
    asm volatile("red.relaxed.sys.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys_u64(const void* p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_relaxed_sys_u64(void* p, unsigned long long v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const void* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ bool better(float v, uint32_t i, float bv, uint32_t bi) {
    return v > bv || (v == bv && i < bi);
}

}  // namespace tl
