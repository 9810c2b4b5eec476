// Internal launch interfaces of the GEMM kernels (not part of the C ABI).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace n550 {

// Epilogue variants of the tcgen05 GEMM.
enum {
    TC_EPI_F32 = 0,        // C (FP32) = acc
    TC_EPI_BF16 = 1,       // C (BF16) = rne(acc)
    TC_EPI_RESID_F32 = 2,  // C (FP32) += acc           (residual add fused)
    TC_EPI_SILU_BF16 = 3   // C (BF16) = silu(acc_gate) * acc_up (SwiGLU fused)
};

struct TcEpilogue {
    void *c;
    int ldc;
    int vec_ok;            // 16-byte vector stores allowed
};

// True when the tensor-core path takes these operands (TMA constraints).
bool tc_shape_ok(const void *a, int lda, const void *b, int ldb, int K);

// C = A[M,K] . B[N,K]^T on tcgen05 tensor cores. For TC_EPI_SILU_BF16, B
// holds the gate rows and b2 the up rows (each [N,K]); C is [M,N].
// bn is the tile width (128 or 256); max_ctas limits the persistent grid
// (0 = one CTA per SM).
int launch_gemm_tc(cudaStream_t st, int epi, int bn, const uint16_t *a, int lda,
                   const uint16_t *b, int ldb, const uint16_t *b2, void *c, int ldc,
                   int M, int N, int K, int max_ctas);

// Exact-mode (AME numerics) GEMM on CUDA cores.
int launch_gemm_exact(cudaStream_t st, const void *a, int a_type, int lda,
                      const uint16_t *b, int ldb, float *c, int ldc,
                      int M, int N, int K, int kblock);

// Fast-mode GEMM on CUDA cores (FP32 FMA) for shapes the TMA path cannot
// take; epi is TC_EPI_F32 / TC_EPI_BF16 / TC_EPI_RESID_F32.
int launch_gemm_simt(cudaStream_t st, int epi, const uint16_t *a, int lda,
                     const uint16_t *b, int ldb, void *c, int ldc, int M, int N, int K);

// Skinny-M GEMV (M <= 8): streams B once with 16-byte loads.
int launch_gemv(cudaStream_t st, int epi, const uint16_t *a, int lda,
                const uint16_t *b, int ldb, void *c, int ldc, int M, int N, int K);

// FP32 -> BF16 RNE staging copy of a row-major [rows, cols] matrix.
int launch_f32_to_bf16(cudaStream_t st, uint16_t *out, int ldo, const float *in, int ldi,
                       int rows, int cols);

}  // namespace n550
