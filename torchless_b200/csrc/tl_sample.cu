// tl_sample.cu -- device sampling (interface in tl_sample.cuh and
// include/torchless_b200.h): the standalone sample_multinomial op and the
// step that samples a decode step's logits.
#include <math.h>

#include "tl_common.cuh"
#include "tl_sample.cuh"

namespace tl {
namespace {

constexpr int kSampleThreads = 1024;

struct BlockSync {
    __device__ void operator()() const { __syncthreads(); }
};

// sample_max (main.cpp:10-21) by one block: first index of the strict
// maximum; NaN at index 0 (or no comparable value) keeps 0.
__device__ uint32_t argmax_block(const float* logits, int n, float* sv, uint32_t* si) {
    float bv = -INFINITY;
    uint32_t bi = 0xffffffffu;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float v = __ldcg(logits + i);
        if (better(v, static_cast<uint32_t>(i), bv, bi)) {
            bv = v;
            bi = static_cast<uint32_t>(i);
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(FULL, bv, o);
        const uint32_t oi = __shfl_xor_sync(FULL, bi, o);
        if (better(ov, oi, bv, bi)) {
            bv = ov;
            bi = oi;
        }
    }
    if ((threadIdx.x & 31) == 0) {
        sv[threadIdx.x >> 5] = bv;
        si[threadIdx.x >> 5] = bi;
    }
    __syncthreads();
    bv = sv[0];
    bi = si[0];
    for (int w = 1; w < static_cast<int>(blockDim.x >> 5); w++)
        if (better(sv[w], si[w], bv, bi)) {
            bv = sv[w];
            bi = si[w];
        }
    const float l0 = __ldcg(logits);
    return (l0 != l0 || bi == 0xffffffffu) ? 0u : bi;
}

__global__ void __launch_bounds__(kSampleThreads) k_sample(uint32_t* out, const float* logits, int n, float temp,
                                                            float r) {
    __shared__ float sm[kSampleThreads / 32];
    __shared__ uint32_t si[kSampleThreads / 32];
    const uint32_t v = temp > 0.f ? sample_block<kSampleThreads>(logits, n, temp, r, sm, BlockSync{})
                                  : argmax_block(logits, n, sm, si);
    if (threadIdx.x == 0) *out = v;
}

__global__ void __launch_bounds__(kSampleThreads) k_sample_step(uint32_t* token, uint32_t* history,
                                                                 const unsigned* pos, const float* logits, int n,
                                                                 float temp, unsigned long long seed) {
    __shared__ float sm[kSampleThreads / 32];
    const unsigned p = *pos - 1;  // the position whose logits these are
    const uint32_t v = sample_block<kSampleThreads>(logits, n, temp, sample_uniform(seed, p), sm, BlockSync{});
    if (threadIdx.x == 0) {
        *token = v;
        history[p] = v;
    }
}

__global__ void __launch_bounds__(kSampleThreads) k_argmax_step(uint32_t* token, uint32_t* history, unsigned* pos,
                                                                 const float* logits, int n) {
    __shared__ float sv[kSampleThreads / 32];
    __shared__ uint32_t si[kSampleThreads / 32];
    const uint32_t v = argmax_block(logits, n, sv, si);
    if (threadIdx.x == 0) {
        const unsigned p = *pos;
        *token = v;
        history[p] = v;
        *pos = p + 1;
    }
}

}  // namespace

tl_status argmax_step(uint32_t* token, uint32_t* history, unsigned* pos, const float* logits, int V, cudaStream_t s) {
    TL_REQUIRE(V > 0, "argmax_step: V %d", V);
    k_argmax_step<<<1, kSampleThreads, 0, s>>>(token, history, pos, logits, V);
    return check_launch("argmax_step");
}

tl_status sample_step(uint32_t* token, uint32_t* history, const unsigned* pos, const float* logits, int V, float temp,
                      uint64_t seed, cudaStream_t s) {
    TL_REQUIRE(temp > 0.f && V > 0, "sample_step: temperature %g, V %d", static_cast<double>(temp), V);
    k_sample_step<<<1, kSampleThreads, 0, s>>>(token, history, pos, logits, V, temp, seed);
    return check_launch("sample_step");
}

}  // namespace tl

using namespace tl;

extern "C" {

tl_status tl_sample_multinomial(uint32_t* out, const float* logits, size_t n, float temperature, float r,
                                void* stream) {
    clear_error();
    TL_REQUIRE(out && logits && n > 0, "tl_sample_multinomial: bad arguments");
    TL_REQUIRE(n <= 0x7fffffffull, "tl_sample_multinomial: n = %zu too large", n);
    TL_REQUIRE(!(temperature != temperature) && !(r != r), "tl_sample_multinomial: NaN temperature or r");
    k_sample<<<1, kSampleThreads, 0, as_stream(stream)>>>(out, logits, static_cast<int>(n), temperature, r);
    return check_launch("sample_multinomial");
}

float tl_sample_uniform(uint64_t seed, uint64_t pos) { return sample_uniform(seed, pos); }

}  // extern "C"
