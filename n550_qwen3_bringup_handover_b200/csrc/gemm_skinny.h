// Skinny-token tensor-core GEMM of the decode step (internal interface).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace n550 {

// Epilogues of the skinny GEMM (Y = X[T,K] . W[N,K]^T, T <= 128 tokens).
enum {
    SK_EPI_F32 = 0,     // out[t][n] = y                      (FP32)
    SK_EPI_RESID = 1,   // out[t][n] += y                     (residual add, qwen3.c:523/543)
    SK_EPI_SILU = 2,    // h[t][n] = silu(y_gate) * y_up      (BF16, W = gate rows, W2 = up rows)
    SK_EPI_QKV = 3      // per-head QK-norm + RoPE, q out, K/V into the cache (qwen3.c:477-511)
};

struct SkEpilogue {
    float *out;                 // F32 / RESID: [T][ldo] FP32
    int ldo;
    uint16_t *h;                // SILU: [T][ldh] BF16
    int ldh;
    // QKV: W is the [q 16 | k 8 | v 8] x 128 projection, one head per tile
    float *q_f32;               // [T][ldq] FP32 queries (either or both)
    uint16_t *q_bf16;           // [T][ldq] BF16 queries
    int ldq;
    uint16_t *kc, *vc;          // KV cache [seq][layer][kv_head][pos][128]
    int layer, max_len;
    const int32_t *tok_pos, *tok_seq;   // per token
    const uint16_t *q_norm, *k_norm;    // BF16 [128]
    const float2 *rope;         // [max_len][64] (cos, sin)
};

// n550_gemm_skinny_config: 0 = automatic (the skinny GEMM for M <=
// g_skinny_rows rows), 1-16 = the skinny GEMM for every M <= SK_MAX_T with that
// cluster size, -1 = off (such GEMMs take the split-K path).
extern int g_skinny_cs;

// Largest token count the skinny GEMM takes (tokens beyond 32 in 64-column
// tiles), and the largest it is chosen for automatically: measured on B200 in
// graph-replayed decode steps (1024-token context) it is ahead of the split-K
// GEMMs with their separate reduction kernels at 16 and 32 tokens (1.50 vs
// 1.72, 1.68 vs 1.77 ms per step) and behind from 64 on (2.43 vs 2.37, 4.09
// vs 3.63, 6.52 vs 6.30 ms at 64/128/256), where its per-CTA partial tiles
// and token-tile epilogues grow with the tokens.
constexpr int SK_MAX_T = 512;
extern int g_skinny_rows;     // n550_gemm_skinny_rows: automatic limit (default SK_AUTO_T)
constexpr int SK_AUTO_T = 32;

// Standalone FP32-output GEMMs (n550_gemm, qwen3_gemm) have no epilogue to
// fuse and pay for a separate reduction kernel on the split-K path: there the
// skinny GEMM is ahead up to 128 rows (measured on B200: the seven projection
// GEMMs of a layer at 128 rows, graph-replayed, 55.3 vs 61.7 us per layer).
constexpr int SK_AUTO_GEMM_T = 128;
extern int g_skinny_rows_gemm;

// Whether a fast-mode decoder layer of M rows takes the skinny GEMM.
inline bool skinny_route(int M) {
    return g_skinny_cs == 0 ? M <= g_skinny_rows : (g_skinny_cs > 0 && M <= SK_MAX_T);
}

// Whether a standalone FP32-output GEMM of M rows takes the skinny GEMM.
inline bool skinny_route_gemm(int M) {
    return g_skinny_cs == 0 ? M <= g_skinny_rows_gemm : (g_skinny_cs > 0 && M <= SK_MAX_T);
}

// Y = X . W^T for T <= SK_MAX_T tokens with epilogue `epi`. X BF16 [T][K]
// (row stride ldx), W (and W2 for SILU) BF16 [N][K] (row stride ldw).
// cs = K-split cluster size (0 = g_skinny_cs, else automatic). Returns N550_OK or an error.
int launch_gemm_skinny(cudaStream_t st, int epi, const uint16_t *x, int ldx, const uint16_t *w,
                       const uint16_t *w2, int ldw, int T, int N, int K, const SkEpilogue &ep,
                       int cs = 0);

}  // namespace n550
