// Persistent few-token decode step (internal interface).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace n550 {

constexpr int FD_MAX_TOKENS = 4;      // sequences per step the kernel takes
constexpr int FD_MAX_POS = 512;       // positions per attention unit
constexpr int FD_MAX_SPLITS = 32;     // attention splits per (token, KV head)
constexpr int FD_MAX_LEN = FD_MAX_POS * FD_MAX_SPLITS;   // longest context (8192)

// One decoder layer's tensors (QW3M order, qwen3_config.h:64-81).
struct FusedLayer {
    const uint16_t *in_norm, *wqkv, *q_norm, *k_norm, *wo, *post_norm, *wg, *wu, *wd;
};

struct FusedDecodeArgs {
    const FusedLayer *layers;     // [28], device memory
    const uint16_t *final_norm;
    uint16_t *kc, *vc;            // KV cache [seq][layer][kv_head][pos][128]
    int max_len;
    const float2 *rope;           // [max_len][64] (cos, sin)
    const int32_t *seq_ids, *pos; // per token
    int T;
    float *x;                     // [T][1024] residual stream (embedded tokens in, updated)
    float *qkv;                   // [T][4096] FP32 scratch
    uint16_t *attn;               // [T][2048] BF16 scratch
    uint16_t *h;                  // [T][3072] BF16 scratch
    float *part_m, *part_l, *part_o;   // attention split partials [T][16][FD_MAX_SPLITS]
    int *counters;                // [T][8] split arrivals, zero between uses
    unsigned *barrier;            // grid-barrier arrivals (zeroed by the launcher)
    uint16_t *xl;                 // [T][1024] out: final-normed rows for the lm_head
};

// Grid size (one CTA per SM) when the device can run the kernel, else 0.
int fused_decode_grid();

// Launches the 28 layers of a decode step of a.T <= FD_MAX_TOKENS sequences
// as one cooperative kernel. N550_ERR_UNSUPPORTED when the device cannot.
int launch_decode_fused(cudaStream_t st, const FusedDecodeArgs &a);

}  // namespace n550
