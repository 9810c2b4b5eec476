// Internal launch interfaces of the non-GEMM kernels (not part of the C ABI).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace n550 {

extern __constant__ float c_inv_freq[64];
int ensure_rope_table();

int launch_rmsnorm(cudaStream_t st, void *out, int out_type, const float *x,
                   const uint16_t *w, int rows, int n, float eps);
int launch_rope(cudaStream_t st, float *v, int rows, int n_heads, int pos0);
int launch_silu_mul(cudaStream_t st, float *gate, const float *up, size_t n);
int launch_residual_add(cudaStream_t st, float *x, const float *y, size_t n);
int launch_bf16_to_f32(cudaStream_t st, float *out, const uint16_t *in, size_t n);
int launch_softmax(cudaStream_t st, float *x, int rows, int n);
int launch_argmax(cudaStream_t st, const float *v, int rows, int n, int ld, int32_t *idx);

int launch_dot(cudaStream_t st, const float *a, const float *b, int n, float *out);
int launch_axpy(cudaStream_t st, float *y, float a, const float *x, size_t n);

__device__ void warp_argmax(float &bv, int &bi);

}  // namespace n550
