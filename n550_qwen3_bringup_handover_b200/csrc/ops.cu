// Non-GEMM operators (ops.h:21-49) as CUDA kernels. Semantics follow the
// scalar reference ops_scalar.c:11-78; reductions run in parallel, so FP32
// results match within rounding (argmax and bf16_to_f32 are exact).
#include <math.h>

#include "common.cuh"
#include "launch.h"
#include "ops.h"

namespace n550 {

// RoPE inverse frequencies theta^(-2i/128), computed on the host with the
// C library's powf exactly as ops_scalar.c:21-25 does, so the device uses the
// reference's own table values.
__constant__ float c_inv_freq[64];

namespace {

template <int NT>
__device__ __forceinline__ float block_sum(float v, float *red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < NT / 32; i++) s += red[i];
    return s;
}

constexpr int RN_THREADS = 256;

// One CTA per row.
template <int OUT_BF16>
__global__ void __launch_bounds__(RN_THREADS)
rmsnorm_kernel(void *out, const float *__restrict__ x, const uint16_t *__restrict__ w,
               int n, float eps) {
    dep_wait();
    dep_launch();
    __shared__ float red[RN_THREADS / 32];
    const float *xr = x + (size_t)blockIdx.x * n;
    float ss = 0.f;
    for (int i = threadIdx.x; i < n; i += RN_THREADS) ss = fmaf(xr[i], xr[i], ss);
    ss = block_sum<RN_THREADS>(ss, red);
    const float scale = 1.0f / sqrtf(ss / (float)n + eps);
    for (int i = threadIdx.x; i < n; i += RN_THREADS) {
        const float v = xr[i] * scale * bf16_bits_to_f32(w[i]);
        if (OUT_BF16) ((uint16_t *)out)[(size_t)blockIdx.x * n + i] = f32_to_bf16_rne(v);
        else ((float *)out)[(size_t)blockIdx.x * n + i] = v;
    }
}

// One CTA per row, one thread per rotation pair (i, i+64) of one head.
__global__ void rope_kernel(float *v, int n_heads, int pos0) {
    dep_wait();
    dep_launch();
    const int pos = pos0 + blockIdx.x;
    float *row = v + (size_t)blockIdx.x * n_heads * 128;
    for (int t = threadIdx.x; t < n_heads * 64; t += blockDim.x) {
        const int h = t >> 6, i = t & 63;
        const float ang = (float)pos * c_inv_freq[i];
        float s, c;
        sincosf(ang, &s, &c);
        float *p = row + h * 128;
        const float a = p[i], b = p[i + 64];
        p[i] = a * c - b * s;
        p[i + 64] = b * c + a * s;
    }
}

__global__ void silu_mul_kernel(float *gate, const float *__restrict__ up, size_t n) {
    dep_wait();
    dep_launch();
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x) {
        const float g = gate[i];
        gate[i] = (g / (1.0f + expf(-g))) * up[i];
    }
}

__global__ void residual_add_kernel(float *x, const float *__restrict__ y, size_t n) {
    dep_wait();
    dep_launch();
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x)
        x[i] += y[i];
}

__global__ void bf16_to_f32_kernel(float *out, const uint16_t *__restrict__ in, size_t n) {
    dep_wait();
    dep_launch();
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x)
        out[i] = bf16_bits_to_f32(in[i]);
}

constexpr int SM_THREADS = 512;

__global__ void __launch_bounds__(SM_THREADS) softmax_kernel(float *x, int n) {
    dep_wait();
    dep_launch();
    __shared__ float red[SM_THREADS / 32];
    float *xr = x + (size_t)blockIdx.x * n;
    float mx = -INFINITY;
    for (int i = threadIdx.x; i < n; i += SM_THREADS) mx = fmaxf(mx, xr[i]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
    __syncthreads();
    mx = red[0];
#pragma unroll
    for (int i = 1; i < SM_THREADS / 32; i++) mx = fmaxf(mx, red[i]);
    float s = 0.f;
    for (int i = threadIdx.x; i < n; i += SM_THREADS) {
        const float e = expf(xr[i] - mx);
        xr[i] = e;
        s += e;
    }
    s = block_sum<SM_THREADS>(s, red);
    for (int i = threadIdx.x; i < n; i += SM_THREADS) xr[i] /= s;
}

}  // namespace

// (value, index) order of the reference argmax: larger value wins, equal
// values keep the lower index (strict > scan from index 0).
__device__ __forceinline__ void argmax_merge(float &bv, int &bi, float v, int i) {
    if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
}

__device__ void warp_argmax(float &bv, int &bi) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xFFFFFFFFu, bv, o);
        const int oi = __shfl_xor_sync(0xFFFFFFFFu, bi, o);
        argmax_merge(bv, bi, ov, oi);
    }
}

namespace {

constexpr int AM_THREADS = 1024;

__global__ void __launch_bounds__(AM_THREADS)
argmax_kernel(const float *__restrict__ v, int n, int ld, int32_t *idx) {
    dep_wait();
    dep_launch();
    __shared__ float sv[AM_THREADS / 32];
    __shared__ int si[AM_THREADS / 32];
    const float *r = v + (size_t)blockIdx.x * ld;
    float bv = -INFINITY;
    int bi = 0x7FFFFFFF;
    // 8 independent loads per thread in flight, merged in increasing index
    // order: the one-block row scan is bound by load latency, not bandwidth
    for (int i0 = threadIdx.x; i0 < n; i0 += 8 * AM_THREADS) {
        float x[8];
#pragma unroll
        for (int u = 0; u < 8; u++) {
            const int i = i0 + u * AM_THREADS;
            x[u] = i < n ? r[i] : -INFINITY;
        }
#pragma unroll
        for (int u = 0; u < 8; u++) {
            const int i = i0 + u * AM_THREADS;
            if (i < n) argmax_merge(bv, bi, x[u], i);
        }
    }
    warp_argmax(bv, bi);
    if ((threadIdx.x & 31) == 0) { sv[threadIdx.x >> 5] = bv; si[threadIdx.x >> 5] = bi; }
    __syncthreads();
    if (threadIdx.x < 32) {
        bv = sv[threadIdx.x];
        bi = si[threadIdx.x];
        warp_argmax(bv, bi);
        // All -inf (or NaN) rows: the reference returns index 0.
        if (threadIdx.x == 0) idx[blockIdx.x] = (bi == 0x7FFFFFFF) ? 0 : bi;
    }
}

constexpr int DOT_THREADS = 1024;

// Single-CTA dot product (qwen3_op_dot, ops_scalar.c:68-72).
__global__ void __launch_bounds__(DOT_THREADS)
dot_kernel(const float *__restrict__ a, const float *__restrict__ b, int n, float *out) {
    dep_wait();
    dep_launch();
    __shared__ float red[DOT_THREADS / 32];
    float s = 0.f;
    for (int i = threadIdx.x; i < n; i += DOT_THREADS) s = fmaf(a[i], b[i], s);
    s = block_sum<DOT_THREADS>(s, red);
    if (threadIdx.x == 0) *out = s;
}

// y += a * x (qwen3_op_axpy, ops_scalar.c:74-77).
__global__ void axpy_kernel(float *y, float a, const float *__restrict__ x, size_t n) {
    dep_wait();
    dep_launch();
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x)
        y[i] = __fadd_rn(y[i], __fmul_rn(a, x[i]));   // no FMA: bit-identical to the C loop
}

int grid_for(size_t n, int threads) {
    size_t g = (n + threads - 1) / threads;
    if (g > 148 * 32) g = 148 * 32;
    return g ? (int)g : 1;
}

bool g_freq_ready[64];

}  // namespace

int ensure_rope_table() {
    int dev = 0;
    N550_CUDA_TRY(cudaGetDevice(&dev));
    if (dev >= 0 && dev < 64 && g_freq_ready[dev]) return N550_OK;
    float f[64];
    for (int i = 0; i < 64; i++)
        f[i] = 1.0f / powf(1000000.0f, (float)(2 * i) / (float)128);
    N550_CUDA_TRY(cudaMemcpyToSymbol(c_inv_freq, f, sizeof f));
    if (dev >= 0 && dev < 64) g_freq_ready[dev] = true;
    return N550_OK;
}

int launch_rmsnorm(cudaStream_t st, void *out, int out_type, const float *x,
                   const uint16_t *w, int rows, int n, float eps) {
    if (rows <= 0 || n <= 0) return rows < 0 || n < 0 ? N550_ERR_ARG : N550_OK;
    if (out_type == N550_BF16)
        N550_CUDA_TRY(launch_k(rmsnorm_kernel<1>, rows, RN_THREADS, 0, st, out, x, w, n, eps));
    else if (out_type == N550_F32)
        N550_CUDA_TRY(launch_k(rmsnorm_kernel<0>, rows, RN_THREADS, 0, st, out, x, w, n, eps));
    else
        return N550_ERR_ARG;
    N550_LAUNCH_CHECK();
    return N550_OK;
}

int launch_rope(cudaStream_t st, float *v, int rows, int n_heads, int pos0) {
    if (rows <= 0 || n_heads <= 0) return rows < 0 || n_heads < 0 ? N550_ERR_ARG : N550_OK;
    int rc = ensure_rope_table();
    if (rc) return rc;
    N550_CUDA_TRY(launch_k(rope_kernel, rows, 256, 0, st, v, n_heads, pos0));
    N550_LAUNCH_CHECK();
    return N550_OK;
}

int launch_silu_mul(cudaStream_t st, float *gate, const float *up, size_t n) {
    if (!n) return N550_OK;
    N550_CUDA_TRY(launch_k(silu_mul_kernel, grid_for(n, 256), 256, 0, st, gate, up, n));
    N550_LAUNCH_CHECK();
    return N550_OK;
}

int launch_residual_add(cudaStream_t st, float *x, const float *y, size_t n) {
    if (!n) return N550_OK;
    N550_CUDA_TRY(launch_k(residual_add_kernel, grid_for(n, 256), 256, 0, st, x, y, n));
    N550_LAUNCH_CHECK();
    return N550_OK;
}

int launch_bf16_to_f32(cudaStream_t st, float *out, const uint16_t *in, size_t n) {
    if (!n) return N550_OK;
    N550_CUDA_TRY(launch_k(bf16_to_f32_kernel, grid_for(n, 256), 256, 0, st, out, in, n));
    N550_LAUNCH_CHECK();
    return N550_OK;
}

int launch_softmax(cudaStream_t st, float *x, int rows, int n) {
    if (rows <= 0 || n <= 0) return rows < 0 || n < 0 ? N550_ERR_ARG : N550_OK;
    N550_CUDA_TRY(launch_k(softmax_kernel, rows, SM_THREADS, 0, st, x, n));
    N550_LAUNCH_CHECK();
    return N550_OK;
}

int launch_argmax(cudaStream_t st, const float *v, int rows, int n, int ld, int32_t *idx) {
    if (rows <= 0 || n <= 0 || ld < n) return N550_ERR_ARG;
    N550_CUDA_TRY(launch_k(argmax_kernel, rows, AM_THREADS, 0, st, v, n, ld, idx));
    N550_LAUNCH_CHECK();
    return N550_OK;
}

int launch_dot(cudaStream_t st, const float *a, const float *b, int n, float *out) {
    if (n < 0) return N550_ERR_ARG;
    N550_CUDA_TRY(launch_k(dot_kernel, 1, DOT_THREADS, 0, st, a, b, n, out));
    N550_LAUNCH_CHECK();
    return N550_OK;
}

int launch_axpy(cudaStream_t st, float *y, float a, const float *x, size_t n) {
    if (!n) return N550_OK;
    N550_CUDA_TRY(launch_k(axpy_kernel, grid_for(n, 256), 256, 0, st, y, a, x, n));
    N550_LAUNCH_CHECK();
    return N550_OK;
}

}  // namespace n550
