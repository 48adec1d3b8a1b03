// tl_ops.cu -- op-level C ABI mirroring src/common/kernels.h on device memory.
//
// Each entry point takes device pointers and a stream, validates shapes the
// way the reference asserts them (kernels.cpp:10, 25, 42), and launches a
// kernel.  Large aligned matmuls go to the fused GEMV kernels of tl_gemv.cuh;
// every other shape (the 2x3 / 3x2 known-answer cases of
// test_cpu_kernels.cpp, odd group layouts) to a warp-per-row kernel that
// follows the reference element formula exactly (including the generic
// scale index n_scales * i / numel of tensor.cpp:101-104).
#include <math.h>

#include <algorithm>
#include <mutex>

#include "tl_common.cuh"
#include "tl_gemv.cuh"
#include "tl_kernels.h"

// Scratch of tl_argmax_noalloc: 512 (value, index) partials, 4 KB per device.
static __device__ __align__(256) unsigned char g_noalloc_scratch[512 * 8];

namespace tl {
namespace {

constexpr int kBlock = 256;

int blocks_for(size_t n, int per_block = kBlock) {
    const size_t b = (n + per_block - 1) / per_block;
    return static_cast<int>(std::min<size_t>(std::max<size_t>(b, 1), 4096));
}

// ---- elementwise (kernels.cpp:98-149) ----
__global__ void k_silu(float* y, const float* x, size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        y[i] = x[i] / (1.0f + expf(-x[i]));
}
__global__ void k_add(float* y, const float* a, const float* b, size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        y[i] = a[i] + b[i];
}
__global__ void k_add_scalar(float* y, const float* a, float c, size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        y[i] = a[i] + c;
}
__global__ void k_mul(float* y, const float* a, const float* b, size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        y[i] = a[i] * b[i];
}
__global__ void k_mul_scalar(float* y, const float* a, float c, size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        y[i] = a[i] * c;
}
// std::pow(float, int) promotes to double (kernels.cpp:139-143).
__global__ void k_pow(float* y, const float* a, int e, size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        y[i] = static_cast<float>(pow(static_cast<double>(a[i]), static_cast<double>(e)));
}
__global__ void k_sqrt(float* y, const float* a, size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        y[i] = sqrtf(a[i]);
}

// ---- single-block reductions ----
__global__ void k_sum(float* out, const float* x, size_t n) {
    __shared__ float red[32];
    float v = 0.f;
    for (size_t i = threadIdx.x; i < n; i += blockDim.x) v += x[i];
    v = block_sum(v, red);
    if (threadIdx.x == 0) *out = v;
}

// softmax (kernels.cpp:55-63): e^(x - max) * (1/total).
__global__ void k_softmax(float* y, const float* x, size_t n) {
    __shared__ float red[32];
    float m = -INFINITY;
    for (size_t i = threadIdx.x; i < n; i += blockDim.x) m = fmaxf(m, x[i]);
    m = warp_max(m);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x < 32) {
        float t = (threadIdx.x < (blockDim.x + 31) / 32) ? red[threadIdx.x] : -INFINITY;
        t = warp_max(t);
        if (threadIdx.x == 0) red[0] = t;
    }
    __syncthreads();
    m = red[0];
    float s = 0.f;
    for (size_t i = threadIdx.x; i < n; i += blockDim.x) {
        const float e = expf(x[i] - m);
        y[i] = e;
        s += e;
    }
    s = block_sum(s, red);
    const float inv = 1.0f / s;
    for (size_t i = threadIdx.x; i < n; i += blockDim.x) y[i] = y[i] * inv;
}

// RMSNorm::forward (modules.cpp:31-46).
__global__ void k_rmsnorm(float* y, const float* x, const float* g, size_t n, float eps) {
    __shared__ float red[32];
    float ss = 0.f;
    for (size_t i = threadIdx.x; i < n; i += blockDim.x) ss += x[i] * x[i];
    ss = block_sum(ss, red);
    const float rms = sqrtf(ss / static_cast<float>(n) + eps);
    const float inv = 1.0f / rms;
    for (size_t i = threadIdx.x; i < n; i += blockDim.x) y[i] = (x[i] * inv) * g[i];
}

// rope (kernels.cpp:78-95): one thread per rotated pair.
__global__ void k_rope(float* y, const float* x, const float* c, const float* s, size_t n_heads,
                       size_t head_dim) {
    const size_t half = head_dim / 2;
    for (size_t k = blockIdx.x * (size_t)blockDim.x + threadIdx.x; k < n_heads * half;
         k += (size_t)gridDim.x * blockDim.x) {
        const size_t h = k / half, i = k % half, b = h * head_dim;
        const float xi = x[b + i], yi = x[b + i + half];
        y[b + i] = xi * c[i] - yi * s[i];
        y[b + i + half] = xi * s[i] + yi * c[i];
    }
}

// RotaryEmbedding::forward (modules.cpp:22-27).
__global__ void k_rotary(float* c, float* s, const float* inv_freq, size_t n_freq, size_t head_dim,
                         size_t pos) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < head_dim; i += (size_t)gridDim.x * blockDim.x) {
        const float a = inv_freq[i % n_freq] * static_cast<float>(pos);
        c[i] = cosf(a);
        s[i] = sinf(a);
    }
}

// ---- generic matmuls: one warp per output row (kernels.cpp:6-33) ----
__global__ void k_matmul_f32_rows(float* y, const float* w, const float* x, size_t n, size_t d) {
    const size_t row = blockIdx.x * (size_t)(blockDim.x / 32) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= n) return;
    const float* wr = w + row * d;
    float acc = 0.f;
    for (size_t j = lane; j < d; j += 32) acc += wr[j] * x[j];
    acc = warp_sum(acc);
    if (lane == 0) y[row] = acc;
}

__global__ void k_matmul_i8_rows(float* y, const int8_t* w, const float* scales, size_t n_scales,
                                 const float* x, size_t n, size_t d) {
    const size_t row = blockIdx.x * (size_t)(blockDim.x / 32) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= n) return;
    const size_t numel = n * d;
    float acc = 0.f;
    for (size_t j = lane; j < d; j += 32) {
        const size_t e = row * d + j;
        const float wv = static_cast<float>(w[e]) / scales[n_scales * e / numel];
        acc += wv * x[j];
    }
    acc = warp_sum(acc);
    if (lane == 0) y[row] = acc;
}

// fp8 (e5m2) weights: get(i) is the e5m2 value (the high byte of its fp16).
__global__ void k_matmul_f8_rows(float* y, const uint8_t* w, const float* x, size_t n, size_t d) {
    const size_t row = blockIdx.x * (size_t)(blockDim.x / 32) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= n) return;
    const uint8_t* wr = w + row * d;
    float acc = 0.f;
    for (size_t j = lane; j < d; j += 32) {
        const unsigned short bits = static_cast<unsigned short>(wr[j]) << 8;
        acc += __half2float(__ushort_as_half(bits)) * x[j];
    }
    acc = warp_sum(acc);
    if (lane == 0) y[row] = acc;
}

// row_matmul (kernels.cpp:37-49): one thread per output column, loop over rows.
__global__ void k_row_matmul(float* y, const float* x, const float* w, size_t n, size_t d) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < d; i += (size_t)gridDim.x * blockDim.x) {
        float acc = 0.f;
        for (size_t j = 0; j < n; j++) acc += w[j * d + i] * x[j];
        y[i] = acc;
    }
}

// Fused gate/up for shapes outside the GEMV fast path (modules.cpp:99-112).
__global__ void k_gate_up_rows(float* y, const int8_t* w1, const float* s1, const int8_t* w3,
                               const float* s3, const float* x, size_t n, size_t d) {
    const size_t row = blockIdx.x * (size_t)(blockDim.x / 32) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= n) return;
    const size_t numel = n * d, ns = numel / 64;
    float g = 0.f, u = 0.f;
    for (size_t j = lane; j < d; j += 32) {
        const size_t e = row * d + j;
        const size_t gi = ns * e / numel;
        g += (static_cast<float>(w1[e]) / s1[gi]) * x[j];
        u += (static_cast<float>(w3[e]) / s3[gi]) * x[j];
    }
    g = warp_sum(g);
    u = warp_sum(u);
    if (lane == 0) y[row] = (g / (1.0f + expf(-g))) * u;
}

// ---- argmax (sample_max, main.cpp:10-21) ----
// Pass 1: each block reduces a strided slice to (value, index).
__global__ void k_argmax_partial(float* pv, uint32_t* pi, const float* x, size_t n) {
    __shared__ float sv[32];
    __shared__ uint32_t si[32];
    float v = -INFINITY;
    uint32_t idx = 0xffffffffu;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        if (better(x[i], static_cast<uint32_t>(i), v, idx)) { v = x[i]; idx = static_cast<uint32_t>(i); }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(FULL, v, o);
        const uint32_t oi = __shfl_xor_sync(FULL, idx, o);
        if (better(ov, oi, v, idx)) { v = ov; idx = oi; }
    }
    if ((threadIdx.x & 31) == 0) { sv[threadIdx.x >> 5] = v; si[threadIdx.x >> 5] = idx; }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); w++)
            if (better(sv[w], si[w], v, idx)) { v = sv[w]; idx = si[w]; }
        pv[blockIdx.x] = v;
        pi[blockIdx.x] = idx;
    }
}
// Pass 2: one block merges the partials; NaN in logits[0] keeps index 0.
__global__ void k_argmax_final(uint32_t* out, const float* pv, const uint32_t* pi, int parts,
                               const float* x) {
    __shared__ float sv[32];
    __shared__ uint32_t si[32];
    float v = -INFINITY;
    uint32_t idx = 0xffffffffu;
    for (int i = threadIdx.x; i < parts; i += blockDim.x)
        if (better(pv[i], pi[i], v, idx)) { v = pv[i]; idx = pi[i]; }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(FULL, v, o);
        const uint32_t oi = __shfl_xor_sync(FULL, idx, o);
        if (better(ov, oi, v, idx)) { v = ov; idx = oi; }
    }
    if ((threadIdx.x & 31) == 0) { sv[threadIdx.x >> 5] = v; si[threadIdx.x >> 5] = idx; }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); w++)
            if (better(sv[w], si[w], v, idx)) { v = sv[w]; idx = si[w]; }
        const float x0 = x[0];
        if (x0 != x0 || idx == 0xffffffffu) idx = 0;
        *out = idx;
    }
}

// ---- quantize (export_mistral.py:53-68), one warp per group ----
__global__ void k_quantize(int8_t* q, float* scales, const float* x, size_t numel, size_t group) {
    const size_t ng = numel / group;
    const int lane = threadIdx.x & 31;
    for (size_t g = blockIdx.x * (size_t)(blockDim.x / 32) + (threadIdx.x >> 5); g < ng;
         g += (size_t)gridDim.x * (blockDim.x / 32)) {
        const float* xs = x + g * group;
        float m = 0.f;
        for (size_t j = lane; j < group; j += 32) m = fmaxf(m, fabsf(xs[j]));
        m = warp_max(m);
        // torch evaluates 127 / t as reciprocal(t) * 127: two IEEE roundings.
        const float s = __fmul_rn(__frcp_rn(m), 127.0f);
        if (lane == 0) scales[g] = s;
        for (size_t j = lane; j < group; j += 32)
            q[g * group + j] = static_cast<int8_t>(__float2int_rn(__fmul_rn(xs[j], s)));
    }
}

tl_status launched(const char* what) { return check_launch(what); }

}  // namespace
}  // namespace tl

using namespace tl;

extern "C" {

tl_status tl_matmul_f32(float* xout, const float* w, const float* x, size_t n, size_t d, void* stream) {
    clear_error();
    TL_REQUIRE(xout && w && x, "tl_matmul_f32: null pointer");
    TL_REQUIRE(n > 0 && d > 0, "tl_matmul_f32: empty shape (n=%zu, d=%zu)", n, d);
    cudaStream_t s = as_stream(stream);
    if (gemv_f32_fast_ok(n, d, w, x)) {
        GemvF32Args a = {};
        a.w = w; a.x = x; a.y = xout; a.n = static_cast<int>(n); a.d = static_cast<int>(d);
        return launch_gemv_f32(a, false, false, s, false);
    }
    k_matmul_f32_rows<<<static_cast<unsigned>((n + 7) / 8), 256, 0, s>>>(xout, w, x, n, d);
    return launched("matmul_f32");
}

tl_status tl_matmul_i8(float* xout, const int8_t* w, const float* scales, size_t n_scales,
                       const float* x, size_t n, size_t d, void* stream) {
    clear_error();
    TL_REQUIRE(xout && w && scales && x, "tl_matmul_i8: null pointer");
    TL_REQUIRE(n > 0 && d > 0 && n_scales > 0, "tl_matmul_i8: empty shape");
    TL_REQUIRE(n_scales <= n * d, "tl_matmul_i8: more scales (%zu) than weights", n_scales);
    cudaStream_t s = as_stream(stream);
    if (gemv_i8_fast_ok(n, d, n_scales, w, x)) {
        GemvI8Args a = {};
        a.w = w; a.s = scales; a.x = x; a.y = xout; a.n = static_cast<int>(n); a.d = static_cast<int>(d);
        return launch_gemv_i8(a, I8Mode::Store, false, false, s, false);
    }
    const size_t blocks = (n + 7) / 8;
    k_matmul_i8_rows<<<static_cast<unsigned>(blocks), 256, 0, s>>>(xout, w, scales, n_scales, x, n, d);
    return launched("matmul_i8");
}

tl_status tl_matmul_f8(float* xout, const uint8_t* w, const float* x, size_t n, size_t d, void* stream) {
    clear_error();
    TL_REQUIRE(xout && w && x, "tl_matmul_f8: null pointer");
    TL_REQUIRE(n > 0 && d > 0, "tl_matmul_f8: empty shape");
    cudaStream_t s = as_stream(stream);
    if (d % 64 == 0 && gemv_i8_fast_ok(n, d, n * d / 64, w, x)) {
        GemvI8Args a = {};
        a.w = reinterpret_cast<const int8_t*>(w); a.f8 = 1; a.x = x; a.y = xout;
        a.n = static_cast<int>(n); a.d = static_cast<int>(d);
        return launch_gemv_i8(a, I8Mode::Store, true, false, s, false);
    }
    k_matmul_f8_rows<<<static_cast<unsigned>((n + 7) / 8), 256, 0, s>>>(xout, w, x, n, d);
    return launched("matmul_f8");
}

tl_status tl_row_matmul(float* xout, const float* x, const float* w, size_t n, size_t d, void* stream) {
    clear_error();
    TL_REQUIRE(xout && x && w, "tl_row_matmul: null pointer");
    TL_REQUIRE(n > 0 && d > 0, "tl_row_matmul: empty shape");
    k_row_matmul<<<blocks_for(d), kBlock, 0, as_stream(stream)>>>(xout, x, w, n, d);
    return launched("row_matmul");
}

tl_status tl_softmax(float* xout, const float* x, size_t n, void* stream) {
    clear_error();
    TL_REQUIRE(xout && x && n > 0, "tl_softmax: bad arguments");
    k_softmax<<<1, 1024, 0, as_stream(stream)>>>(xout, x, n);
    return launched("softmax");
}

tl_status tl_rope(float* xout, const float* x, const float* c, const float* sn, size_t n_heads,
                  size_t head_dim, void* stream) {
    clear_error();
    TL_REQUIRE(xout && x && c && sn, "tl_rope: null pointer");
    TL_REQUIRE(n_heads > 0 && head_dim >= 2 && head_dim % 2 == 0, "tl_rope: bad shape");
    k_rope<<<blocks_for(n_heads * head_dim / 2), kBlock, 0, as_stream(stream)>>>(xout, x, c, sn, n_heads,
                                                                                 head_dim);
    return launched("rope");
}

tl_status tl_silu(float* xout, const float* x, size_t n, void* stream) {
    clear_error();
    TL_REQUIRE(xout && x, "tl_silu: null pointer");
    if (n == 0) return TL_OK;
    k_silu<<<blocks_for(n), kBlock, 0, as_stream(stream)>>>(xout, x, n);
    return launched("silu");
}

tl_status tl_sum(float* out, const float* x, size_t n, void* stream) {
    clear_error();
    TL_REQUIRE(out && (x || n == 0), "tl_sum: null pointer");
    k_sum<<<1, 1024, 0, as_stream(stream)>>>(out, x, n);
    return launched("sum");
}

tl_status tl_add(float* xout, const float* x, const float* y, size_t n, void* stream) {
    clear_error();
    TL_REQUIRE(xout && x && y, "tl_add: null pointer");
    if (n == 0) return TL_OK;
    k_add<<<blocks_for(n), kBlock, 0, as_stream(stream)>>>(xout, x, y, n);
    return launched("add");
}

tl_status tl_add_scalar(float* xout, const float* x, float c, size_t n, void* stream) {
    clear_error();
    TL_REQUIRE(xout && x, "tl_add_scalar: null pointer");
    if (n == 0) return TL_OK;
    k_add_scalar<<<blocks_for(n), kBlock, 0, as_stream(stream)>>>(xout, x, c, n);
    return launched("add_scalar");
}

tl_status tl_mul(float* xout, const float* x, const float* y, size_t n, void* stream) {
    clear_error();
    TL_REQUIRE(xout && x && y, "tl_mul: null pointer");
    if (n == 0) return TL_OK;
    k_mul<<<blocks_for(n), kBlock, 0, as_stream(stream)>>>(xout, x, y, n);
    return launched("mul");
}

tl_status tl_mul_scalar(float* xout, const float* x, float c, size_t n, void* stream) {
    clear_error();
    TL_REQUIRE(xout && x, "tl_mul_scalar: null pointer");
    if (n == 0) return TL_OK;
    k_mul_scalar<<<blocks_for(n), kBlock, 0, as_stream(stream)>>>(xout, x, c, n);
    return launched("mul_scalar");
}

tl_status tl_pow(float* xout, const float* x, int e, size_t n, void* stream) {
    clear_error();
    TL_REQUIRE(xout && x, "tl_pow: null pointer");
    if (n == 0) return TL_OK;
    k_pow<<<blocks_for(n), kBlock, 0, as_stream(stream)>>>(xout, x, e, n);
    return launched("pow");
}

tl_status tl_sqrt(float* xout, const float* x, size_t n, void* stream) {
    clear_error();
    TL_REQUIRE(xout && x, "tl_sqrt: null pointer");
    if (n == 0) return TL_OK;
    k_sqrt<<<blocks_for(n), kBlock, 0, as_stream(stream)>>>(xout, x, n);
    return launched("sqrt");
}

tl_status tl_rmsnorm(float* xout, const float* x, const float* g, size_t n, float eps, void* stream) {
    clear_error();
    TL_REQUIRE(xout && x && g && n > 0, "tl_rmsnorm: bad arguments");
    k_rmsnorm<<<1, 1024, 0, as_stream(stream)>>>(xout, x, g, n, eps);
    return launched("rmsnorm");
}

tl_status tl_rotary(float* c, float* sn, const float* inv_freq, size_t n_freq, size_t head_dim,
                    size_t pos, void* stream) {
    clear_error();
    TL_REQUIRE(c && sn && inv_freq && n_freq > 0 && head_dim > 0, "tl_rotary: bad arguments");
    k_rotary<<<blocks_for(head_dim), kBlock, 0, as_stream(stream)>>>(c, sn, inv_freq, n_freq, head_dim, pos);
    return launched("rotary");
}

// The partials live in a stream-ordered allocation made and released on the
// caller's stream for each call.
tl_status tl_argmax(uint32_t* out, const float* logits, size_t n, void* stream) {
    clear_error();
    TL_REQUIRE(out && logits && n > 0, "tl_argmax: bad arguments");
    TL_REQUIRE(n <= 0xffffffffull, "tl_argmax: n too large for 32-bit indices");
    cudaStream_t s = as_stream(stream);
    const int parts = std::min(blocks_for(n, 1024), 2 * sm_count());
    void* ws = nullptr;
    TL_CUDA_TRY(cudaMallocAsync(&ws, parts * (sizeof(float) + sizeof(uint32_t)), s));
    float* pv = static_cast<float*>(ws);
    uint32_t* pi = reinterpret_cast<uint32_t*>(pv + parts);
    k_argmax_partial<<<parts, 1024, 0, s>>>(pv, pi, logits, n);
    tl_status st = launched("argmax_partial");
    if (st == TL_OK) {
        k_argmax_final<<<1, 1024, 0, s>>>(out, pv, pi, parts, logits);
        st = launched("argmax_final");
    }
    cudaError_t e = cudaFreeAsync(ws, s);
    if (st == TL_OK && e != cudaSuccess)
        return set_error(TL_ERR_CUDA, "cudaFreeAsync failed: %s", cudaGetErrorString(e));
    return st;
}

}  // extern "C"

namespace tl {
namespace {

// ---- argmax without allocation ----
// For callers that cannot allocate device memory at call time: a serving loop
// that has handed all free HBM to its KV-cache pool at start-up has nothing
// left for a per-call allocation, and an allocation that fails (or waits on
// the pool) in the middle of a generation would end or stall the request.
// The partials live in this fixed file-scope array instead: one (value,
// index) pair per 1024 logits, so n is limited to kNoAllocMaxParts * 1024.
// Pass 1 writes every partial that pass 2 reads, so nothing in the array has
// to start at zero.  The array is shared by every call on a device: calls
// whose kernels overlap (two streams, or two host threads) race on it.
constexpr int kNoAllocMaxParts = 512;
constexpr size_t kNoAllocMaxLogits = static_cast<size_t>(kNoAllocMaxParts) * 1024;
constexpr int kNoAllocMaxDevices = 64;

static_assert(sizeof(g_noalloc_scratch) == kNoAllocMaxParts * (sizeof(float) + sizeof(uint32_t)),
              "scratch holds kNoAllocMaxParts (value, index) pairs");

// Device address of g_noalloc_scratch, looked up once per device (with that
// device current) on the first call made there.
std::mutex g_noalloc_mu;
unsigned char* g_noalloc_ptr[kNoAllocMaxDevices] = {};

tl_status noalloc_scratch(unsigned char** out) {
    int dev = -1;
    TL_CUDA_TRY(cudaGetDevice(&dev));
    TL_REQUIRE(dev >= 0 && dev < kNoAllocMaxDevices, "tl_argmax_noalloc: device %d out of range", dev);
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p)
            return set_error(TL_ERR_CUDA, "tl_argmax_noalloc: cudaGetSymbolAddress on device %d failed: %s", dev,
                             cudaGetErrorString(e));
        g_noalloc_ptr[dev] = static_cast<unsigned char*>(p);
    }
    *out = g_noalloc_ptr[dev];
    return TL_OK;
}

}  // namespace
}  // namespace tl

using namespace tl;

extern "C" {

tl_status tl_argmax_noalloc(uint32_t* out, const float* logits, size_t n, void* stream) {
    clear_error();
    TL_REQUIRE(out && logits && n > 0, "tl_argmax_noalloc: bad arguments");
    if (n > kNoAllocMaxLogits)
        return set_error(TL_ERR_CAPACITY,
                         "tl_argmax_noalloc: n = %zu exceeds the static scratch limit of %zu logits "
                         "(%d partials of 1024); use tl_argmax",
                         n, kNoAllocMaxLogits, kNoAllocMaxParts);
    unsigned char* ws = nullptr;
    TL_TRY(noalloc_scratch(&ws));
    float* pv = reinterpret_cast<float*>(ws);
    uint32_t* pi = reinterpret_cast<uint32_t*>(ws + kNoAllocMaxParts * sizeof(float));
    cudaStream_t s = as_stream(stream);
    const int parts = static_cast<int>((n + 1023) / 1024);
    k_argmax_partial<<<parts, 1024, 0, s>>>(pv, pi, logits, n);
    TL_TRY(launched("argmax_partial"));
    k_argmax_final<<<1, 1024, 0, s>>>(out, pv, pi, parts, logits);
    return launched("argmax_final");
}

tl_status tl_mlp_gate_up(float* out, const int8_t* w1, const float* s1, const int8_t* w3,
                         const float* s3, const float* x, size_t n, size_t d, void* stream) {
    clear_error();
    TL_REQUIRE(out && w1 && s1 && w3 && s3 && x, "tl_mlp_gate_up: null pointer");
    TL_REQUIRE(n > 0 && d > 0 && (n * d) % 64 == 0, "tl_mlp_gate_up: bad shape");
    cudaStream_t s = as_stream(stream);
    if (gemv_i8_fast_ok(n, d, n * d / 64, w1, x) && gemv_i8_fast_ok(n, d, n * d / 64, w3, x)) {
        GemvI8Args a = {};
        a.w = w1; a.s = s1; a.w2 = w3; a.s2 = s3; a.x = x; a.y = out;
        a.n = static_cast<int>(n); a.d = static_cast<int>(d);
        return launch_gemv_i8(a, I8Mode::SwiGLU, false, false, s, false);
    }
    k_gate_up_rows<<<static_cast<unsigned>((n + 7) / 8), 256, 0, s>>>(out, w1, s1, w3, s3, x, n, d);
    return launched("gate_up");
}

tl_status tl_quantize_i8(int8_t* q, float* scales, const float* x, size_t numel, size_t group,
                         void* stream) {
    clear_error();
    TL_REQUIRE(q && scales && x, "tl_quantize_i8: null pointer");
    TL_REQUIRE(group > 0 && numel % group == 0, "tl_quantize_i8: numel %zu not a multiple of group %zu",
               numel, group);
    if (numel == 0) return TL_OK;
    const size_t groups = numel / group;
    k_quantize<<<blocks_for(groups, 8), 256, 0, as_stream(stream)>>>(q, scales, x, numel, group);
    return launched("quantize");
}

}  // extern "C"
