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
    TC_EPI_SILU_BF16 = 3,  // C (BF16) = silu(acc_gate) * acc_up (SwiGLU fused)
    TC_EPI_QKV_ROPE = 4,   // per-head RMSNorm + RoPE of q/k, q out, k/v into the KV cache
    TC_EPI_ARGMAX = 5      // per row and tile: (max, lowest index of the max), no C written
};

// Operands of the fused QKV epilogue (qwen3.c:477-511): a 128-column tile is
// one head of the [q 16 | k 8 | v 8] x 128 qkv row.
struct TcQkv {
    uint16_t *q_bf16;          // [M, ldq] BF16 queries
    int ldq;
    uint16_t *kc, *vc;         // KV cache [seq][layer][kv_head][pos][128]
    int layer, max_len;
    const int32_t *tok_pos, *tok_seq;   // per row
    const uint16_t *q_norm, *k_norm;    // BF16 [128]
    const float2 *rope;        // [max_len][64] (cos, sin) of pos * inv_freq[i] (the epilogue
                               // evaluates the same values in registers)
    float eps;
};

struct TcEpilogue {
    void *c;
    int ldc;
    int vec_ok;            // 16-byte vector stores allowed
    int tma_resid;         // TC_EPI_RESID_F32 through TMA reduce-adds (C map given)
    TcQkv qkv;
    float *amax;           // TC_EPI_ARGMAX: [M][an] best value per row and N tile
    int32_t *aidx;         //                [M][an] its column
    int an;                //                number of N tiles
};

// Tile width (BN) used by the fast GEMMs for an M x N output: 128 or 256;
// g_tile_bn (n550_gemm_tile_config) overrides the automatic choice.
extern int g_tile_bn;
int n550_tile_bn(int M, int N);
// True when a bn = 256 tile runs as a 256 x 256 tile on a 2-CTA cluster.
bool tc_use_pair(int M, int bn);

// True when the tensor-core path takes these operands (TMA constraints: K >= 64,
// 16-byte aligned rows and bases).
bool tc_shape_ok(const void *a, int lda, const void *b, int ldb, int K);

// C = A[M,K] . B[N,K]^T on tcgen05 tensor cores. For TC_EPI_SILU_BF16, B
// holds the gate rows and b2 the up rows (each [N,K]); C is [M,N].
// bn is the tile width (128 or 256); max_ctas limits the persistent grid
// (0 = one CTA per SM).
int launch_gemm_tc(cudaStream_t st, int epi, int bn, const uint16_t *a, int lda,
                   const uint16_t *b, int ldb, const uint16_t *b2, void *c, int ldc,
                   int M, int N, int K, int max_ctas);

// Skinny-M variant (decode): the K loop is split over up to 8 CTAs per tile
// when the tile count alone cannot occupy the SMs; FP32 partials go to ws
// (ws_bytes large enough for splits x M x N floats, 2N for SwiGLU) and a
// reduce kernel sums them in slice order and applies the epilogue. Falls back
// to launch_gemm_tc when no split is worthwhile or ws is too small.
int launch_gemm_tc_splitk(cudaStream_t st, int epi, const uint16_t *a, int lda, const uint16_t *b,
                          int ldb, const uint16_t *b2, void *c, int ldc, int M, int N, int K,
                          float *ws, size_t ws_bytes);
// Only the partial-sum stage: ks_out slices of raw FP32 accumulators in ws
// ([slice][M][N], SwiGLU [slice][M][2N] with up at column N + n); epi is
// TC_EPI_F32 or TC_EPI_SILU_BF16. Consumers sum the slices in order.
int launch_gemm_tc_partials(cudaStream_t st, int epi, const uint16_t *a, int lda, const uint16_t *b,
                            int ldb, const uint16_t *b2, int M, int N, int K, float *ws,
                            size_t ws_bytes, int *ks_out);
int launch_splitk_reduce(cudaStream_t st, int epi, const float *ws, int ks, int M, int N, void *c,
                         int ldc);
// Number of K slices launch_gemm_tc_splitk uses (1 = no split).
int tc_splitk_plan(int M, int N, int K, int epi, int bn, int *kt_per);

// lm_head + argmax (qwen3.c:547-573 followed by qwen3_op_argmax): C = A . B^T
// is never written; each 128-column tile leaves (max, lowest index of the max)
// per row in amax/aidx ([M][ceil(N/128)], ws of at least M * ceil(N/128) * 8
// bytes), then one kernel merges the tiles into idx[M] with the rule of
// qwen3_op_argmax (first index of the maximum; rows without a finite maximum
// give 0).
int launch_gemm_tc_argmax(cudaStream_t st, const uint16_t *a, int lda, const uint16_t *b, int ldb,
                          int M, int N, int K, void *ws, size_t ws_bytes, int32_t *idx);

// The QKV projection with the fused per-head epilogue (N = 4096, BN = 128).
int launch_gemm_tc_qkv(cudaStream_t st, const uint16_t *a, int lda, const uint16_t *w,
                       const TcQkv &q, int M, int K, int max_ctas);

// Exact-mode (AME numerics) GEMM on CUDA cores.
int launch_gemm_exact(cudaStream_t st, const void *a, int a_type, int lda,
                      const uint16_t *b, int ldb, float *c, int ldc,
                      int M, int N, int K, int kblock);

// Fast-mode GEMM on CUDA cores (FP32 FMA) for shapes the TMA path cannot
// take; epi is TC_EPI_F32 / TC_EPI_BF16 / TC_EPI_RESID_F32.
int launch_gemm_simt(cudaStream_t st, int epi, const uint16_t *a, int lda,
                     const uint16_t *b, int ldb, void *c, int ldc, int M, int N, int K);

// Skinny-M GEMV (M <= 8): streams B once with 16-byte loads. x_ready (the
// RESID epilogue): no kernel still in flight writes c, so the K-split GEMV
// reads its residual rows before waiting for the previous kernel. nx != NULL
// (K = 1024, FP32 output): the A rows are bf16(rmsnorm(nx[m]) * nw), computed
// in the kernel exactly as the model's norm kernel computes them; a / lda are
// unused.
int launch_gemv(cudaStream_t st, int epi, const uint16_t *a, int lda,
                const uint16_t *b, int ldb, void *c, int ldc, int M, int N, int K,
                bool x_ready = false, const float *nx = nullptr, const uint16_t *nw = nullptr);
// h[m][n] = bf16(silu(a[m] . wg[n]) * (a[m] . wu[n])) for M <= 8 rows, one
// launch; nx / nw as in launch_gemv.
int launch_gemv_swiglu(cudaStream_t st, const uint16_t *a, int lda, const uint16_t *wg,
                       const uint16_t *wu, int ldb, uint16_t *h, int ldh, int M, int N, int K,
                       const float *nx = nullptr, const uint16_t *nw = nullptr);

// FP32 -> BF16 RNE staging copy of a row-major [rows, cols] matrix.
int launch_f32_to_bf16(cudaStream_t st, uint16_t *out, int ldo, const float *in, int ldi,
                       int rows, int cols);

}  // namespace n550
