// Internal launch interfaces of the attention kernels (not part of the C ABI).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace n550 {

// Prefill: n_seqs sequences x L queries at positions pos0..pos0+L-1; the
// queries' own K/V are already in the cache. Q/out rows are [seq][L][2048].
struct AttnPrefillArgs {
    const uint16_t *q;        // BF16, row stride ldq elements
    const uint16_t *kc, *vc;  // KV cache base pointers
    uint16_t *out;            // BF16, row stride ldo
    const int32_t *seq_ids;   // [n_seqs] KV slots
    int ldq, ldo, L, pos0, layer, max_len;
    int kv_planes;            // slots x 28 layers x 8 KV heads in the cache
};

// Decode: one query per sequence at position pos[s] (attends 0..pos[s]).
struct AttnDecodeArgs {
    const float *q_f32;       // FP32 queries, or NULL to read q_bf16
    const uint16_t *q_bf16;
    const uint16_t *kc, *vc;
    uint16_t *out;
    const int32_t *seq_ids, *pos;
    int ldq, ldo, layer, max_len, splits;
    int kv_planes;            // slots x 28 layers x 8 KV heads in the cache
    float *part_m, *part_l, *part_o;   // split-KV partials (splits > 1)
    // splits > 1: per (sequence, KV head) arrival counters, zero between
    // calls; the CTA that completes a pair merges its splits (no separate
    // combine kernel). NULL: the combine kernel runs after the splits.
    int *counters;
    // Fused q/k/v preparation (qkv != NULL; q_f32 / q_bf16 are then unused):
    // raw q/k/v rows [s][qkv_ld] FP32, the sum of qkv_ks split-K slices
    // qkv_slice floats apart (qkv_ks <= 0: one row); each CTA applies the
    // per-head RMSNorm (q_norm, k_norm) and RoPE (rope table) to its two query
    // heads and its KV head, and the CTA whose positions include pos[s] writes
    // that position's K/V into the cache (qwen3.c:287-292, 498-511).
    const float *qkv;
    int qkv_ld, qkv_ks;
    size_t qkv_slice;
    const uint16_t *q_norm, *k_norm;
    const float2 *rope;
    uint16_t *kc_w, *vc_w;
};

int launch_attn_prefill(cudaStream_t st, const AttnPrefillArgs &a, int n_seqs);
int launch_attn_decode(cudaStream_t st, const AttnDecodeArgs &a, int n_seqs);
int attn_decode_splits(int n_seqs, int max_kv_len, int max_splits);

}  // namespace n550
