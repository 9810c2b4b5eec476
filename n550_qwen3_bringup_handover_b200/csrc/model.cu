// Qwen3-0.6B runtime on one B200: qwen3_init / qwen3_forward_batch /
// qwen3_forward / qwen3_argmax (qwen3.c:87-584) re-designed so that weights,
// KV cache and activations stay in HBM and many independent sequences share
// one pass.
//
// Per layer (prefill and decode alike):
//   rmsnorm(x) -> xb (BF16)                    qwen3.c:471-472
//   qkv = xb . [Wq;Wk;Wv]^T (one GEMM, N=4096)  qwen3.c:477-487
//   per-head RMSNorm + RoPE of q and k, K/V written to the cache (BF16)
//                                              qwen3.c:479-511
//   attention -> attn (BF16)                   qwen3.c:513-517
//   x += attn . Wo^T (residual fused in the GEMM epilogue)   qwen3.c:520-523
//   rmsnorm(x) -> xb                           qwen3.c:527
//   h = silu(xb . Wg^T) * (xb . Wu^T) (SwiGLU fused in the epilogue)
//                                              qwen3.c:531-537
//   x += h . Wd^T (residual fused)             qwen3.c:540-543
// then final RMSNorm of each sequence's last token and the tied lm_head
// (qwen3.c:547-573), followed by argmax (qwen3.c:582-584).
//
// BF16 activations exist only where the reference's AME GEMM rounds its FP32
// input to BF16 anyway (kernels_ame.c:220-236), so the GEMM inputs are the
// same values; the residual stream stays FP32. The KV cache is BF16.
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <vector>

#include "attention.h"
#include "common.cuh"
#include "decode_fused.h"
#include "gemm_skinny.h"
#include "gemm_tc.h"
#include "launch.h"
#include "ops.h"
#include "synth.cuh"

namespace n550 {
namespace {

constexpr int H = 1024, INTER = 3072, NLAYER = 28, NH = 16, NKVH = 8, HDIM = 128;
constexpr int VOCAB = 151936, QD = NH * HDIM, KVD = NKVH * HDIM, QKVD = QD + 2 * KVD;
constexpr int N_TENSORS = 1 + NLAYER * 11 + 1;
constexpr float EPS = 1e-6f;
constexpr int MAX_SPLITS = 32;

int32_t rd_i32(const uint8_t *p) {
    return (int32_t)((uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) |
                     ((uint32_t)p[3] << 24));
}
float rd_f32(const uint8_t *p) {
    int32_t v = rd_i32(p);
    float f;
    memcpy(&f, &v, 4);
    return f;
}
void wr_i32(uint8_t *p, int32_t v) {
    for (int i = 0; i < 4; i++) p[i] = (uint8_t)((uint32_t)v >> (8 * i));
}
void wr_f32(uint8_t *p, float f) {
    int32_t v;
    memcpy(&v, &f, 4);
    wr_i32(p, v);
}

// Elements of tensor idx in QW3M file order (qwen3_config.h:64-81).
size_t tensor_elems(int idx, bool *is_norm) {
    *is_norm = false;
    if (idx == 0) return (size_t)VOCAB * H;
    if (idx == N_TENSORS - 1) { *is_norm = true; return H; }
    switch ((idx - 1) % 11) {
    case 0: *is_norm = true; return H;
    case 1: return (size_t)QD * H;
    case 2: return (size_t)KVD * H;
    case 3: return (size_t)KVD * H;
    case 4: *is_norm = true; return HDIM;
    case 5: *is_norm = true; return HDIM;
    case 6: return (size_t)H * QD;
    case 7: *is_norm = true; return H;
    case 8: return (size_t)INTER * H;
    case 9: return (size_t)INTER * H;
    default: return (size_t)H * INTER;
    }
}

// Header checks in the order of qwen3_init (qwen3.c:93-146), same codes.
// Layouts: ROW, or TILE with 128 x 32 tiles -- the two the reference's
// qwen3_set_weight_layout accepts with the AME kernel (kernels_ame.c:188-207);
// *tiled reports which.
int parse_qw3m(const uint8_t *b, size_t size, size_t *offs, bool *tiled = nullptr) {
    if (size < 256) return N550_ERR_SIZE;
    if (b[0] != 'Q' || b[1] != 'W' || b[2] != '3' || b[3] != 'M') return N550_ERR_MAGIC;
    if (rd_i32(b + 4) != 1) return N550_ERR_VERSION;
    if (rd_i32(b + 44) != 1) return N550_ERR_DTYPE;
    if (rd_i32(b + 8) != H || rd_i32(b + 12) != INTER || rd_i32(b + 16) != NLAYER ||
        rd_i32(b + 20) != NH || rd_i32(b + 24) != NKVH || rd_i32(b + 28) != HDIM ||
        rd_i32(b + 32) != VOCAB)
        return N550_ERR_SHAPE;
    const int align = rd_i32(b + 72);
    if (align < 128 || (align & (align - 1)) != 0) return N550_ERR_SHAPE;
    const int layout = rd_i32(b + 76);
    const bool tile = layout == N550_LAYOUT_TILE && rd_i32(b + 80) == 128 && rd_i32(b + 84) == 32;
    if (layout != N550_LAYOUT_ROW && !tile) return N550_ERR_LAYOUT;
    if (tiled) *tiled = tile;
    if (rd_f32(b + 48) != 1000000.0f) return N550_ERR_SHAPE;
    if (rd_f32(b + 52) != 1e-06f) return N550_ERR_SHAPE;
    size_t pos = (size_t)(uint32_t)rd_i32(b + 68);
    for (int t = 0; t < N_TENSORS; t++) {
        bool nrm;
        const size_t n = tensor_elems(t, &nrm);
        const size_t p = (pos + (size_t)align - 1) & ~((size_t)align - 1);
        if (p + n * 2 > size) return N550_ERR_SIZE;
        offs[t] = p;
        pos = p + n * 2;
    }
    if (pos != size) return N550_ERR_SIZE;
    return N550_OK;
}

// True for the per-layer GEMM weights (q, k, v, o, gate, up, down), the
// tensors a tile-major export re-arranges; embed_tokens and the norms stay
// row-major (GET_WEIGHTS.md of the reference's L4 demo).
bool is_gemm_weight(int idx, int *N, int *K) {
    if (idx == 0 || idx == N_TENSORS - 1) return false;
    switch ((idx - 1) % 11) {
    case 1: *N = QD; *K = H; return true;
    case 2: case 3: *N = KVD; *K = H; return true;
    case 6: *N = H; *K = QD; return true;
    case 8: case 9: *N = INTER; *K = H; return true;
    case 10: *N = H; *K = INTER; return true;
    default: return false;
    }
}

// Tile-major [N/128][K/32][128][32] -> row-major [N][K] (the element offset of
// tile (n0, k0) is ((n0/128)*(K/32) + k0/32) * 4096, kernels_ame.c:212-215).
__global__ void untile_weight_kernel(uint16_t *__restrict__ dst, const uint16_t *__restrict__ src,
                                     int N, int K) {
    const size_t total = (size_t)N * K;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
         i += (size_t)gridDim.x * blockDim.x) {
        const int n = (int)(i / K), k = (int)(i % K);
        dst[i] = src[((size_t)(n >> 7) * (K >> 5) + (k >> 5)) * 4096 + (n & 127) * 32 + (k & 31)];
    }
}

// The random-init blob header: the fields a QW3M exporter writes for
// Qwen3-0.6B (qwen3_config.h:41-62), row layout, 128-byte alignment.
void make_header(uint8_t *h) {
    memset(h, 0, 256);
    memcpy(h, "QW3M", 4);
    wr_i32(h + 4, 1);
    wr_i32(h + 8, H); wr_i32(h + 12, INTER); wr_i32(h + 16, NLAYER);
    wr_i32(h + 20, NH); wr_i32(h + 24, NKVH); wr_i32(h + 28, HDIM);
    wr_i32(h + 32, VOCAB); wr_i32(h + 36, 40960); wr_i32(h + 40, 1);
    wr_i32(h + 44, 1);
    wr_f32(h + 48, 1000000.0f); wr_f32(h + 52, 1e-06f);
    wr_i32(h + 56, 151643); wr_i32(h + 60, 151645); wr_i32(h + 64, 151643);
    wr_i32(h + 68, 256); wr_i32(h + 72, 128);
}

size_t qw3m_row_size() {
    size_t pos = 256;
    for (int t = 0; t < N_TENSORS; t++) {
        bool nrm;
        pos = (pos + 127) & ~(size_t)127;
        pos += tensor_elems(t, &nrm) * 2;
    }
    return pos;
}

// ---------------------------------------------------------------- kernels

__global__ void synth_bf16_kernel(uint16_t *out, size_t n, uint64_t key, float scale) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x)
        out[i] = f32_to_bf16_rne(synth_normal(synth_u64(key, i), scale));
}

__global__ void fill_u16_kernel(uint16_t *out, size_t n, uint16_t v) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x)
        out[i] = v;
}

// Per-token (position, KV slot) of a prefill chunk: token t = i*Lc + j.
__global__ void setup_prefill_kernel(int32_t *tok_pos, int32_t *tok_seq, const int32_t *seq_ids,
                                     int Sc, int Lc, int p0) {
    dep_wait();
    dep_launch();
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= Sc * Lc) return;
    tok_pos[t] = p0 + t % Lc;
    tok_seq[t] = seq_ids[t / Lc];
}

// x[t] = embed[token] in FP32 (qwen3_embed, qwen3.c:276-279); the token of
// row t = i*Lc + j is tokens[i*ld + off + j]. A decode step (pos given) also
// records each row's position and KV slot for the layers.
__global__ void embed_kernel(float *x, const uint16_t *__restrict__ embed, const int32_t *tokens,
                             int Lc, int ld, int off, const int32_t *pos, const int32_t *seq_ids,
                             int32_t *tok_pos, int32_t *tok_seq) {
    dep_wait();
    dep_launch();
    const int t = blockIdx.x;
    if (pos && threadIdx.x == 0) {
        tok_pos[t] = pos[t];
        tok_seq[t] = seq_ids[t];
    }
    const int i = t / Lc, j = t % Lc;
    int tok = tokens[(size_t)i * ld + off + j];
    tok = min(max(tok, 0), VOCAB - 1);
    const uint2 *src = (const uint2 *)(embed + (size_t)tok * H);
    float4 *dst = (float4 *)(x + (size_t)t * H);
    for (int c = threadIdx.x; c < H / 4; c += blockDim.x) {
        const uint2 q = src[c];
        dst[c] = make_float4(__uint_as_float(q.x << 16), __uint_as_float(q.x & 0xFFFF0000u),
                             __uint_as_float(q.y << 16), __uint_as_float(q.y & 0xFFFF0000u));
    }
}

// Per-head RMSNorm of q and k (qk_norm, qwen3.c:287-292), RoPE at the
// token's position (ops_scalar.c:21-35), and the K/V cache write
// (qwen3.c:498-511). One warp per head; 32 heads per token
// ([q 16 | k 8 | v 8] x 128 is the qkv row).
// Sum of up to 8 split-K partial slices (issued together), or the plain row.
__device__ __forceinline__ float sum_slices(const float *p, int ks, size_t slice) {
    if (ks <= 0) return p[0];
    float v[8];
#pragma unroll
    for (int sk = 0; sk < 8; sk++) v[sk] = sk < ks ? p[sk * slice] : 0.f;
    float a = v[0];
#pragma unroll
    for (int sk = 1; sk < 8; sk++) a += v[sk];
    return a;
}

__global__ void __launch_bounds__(1024)
qknorm_rope_kv_kernel(const float *__restrict__ qkv, int ldqkv, int ks, size_t slice,
                      const uint16_t *__restrict__ qn, const uint16_t *__restrict__ kn,
                      const float2 *__restrict__ rope, const int32_t *__restrict__ tok_pos,
                      const int32_t *__restrict__ tok_seq, int layer, uint16_t *kc, uint16_t *vc,
                      int max_len, uint16_t *q_bf16, float *q_f32, int ldq) {
    dep_wait();
    dep_launch();
    // One warp per head (32 per token): qkv row t, or (ks > 0) the sum of ks
    // split-K partial slices of it; RoPE factors from the per-position table.
    const int t = blockIdx.x;
    const int hd = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int pos = tok_pos[t], seq = tok_seq[t];
    const float *row = qkv + (size_t)t * ldqkv + hd * HDIM + lane;
    float v[4];
#pragma unroll
    for (int j = 0; j < 4; j++) v[j] = sum_slices(row + 32 * j, ks, slice);
    if (hd < 24) {
        const uint16_t *w = hd < 16 ? qn : kn;
        float ss = v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, o);
        const float sc = 1.0f / sqrtf(ss / (float)HDIM + EPS);
#pragma unroll
        for (int j = 0; j < 4; j++) v[j] = v[j] * sc * bf16_bits_to_f32(w[lane + 32 * j]);
#pragma unroll
        for (int j = 0; j < 2; j++) {              // pairs (i, i + 64), i = lane + 32 j
            const float2 cs = rope[(size_t)pos * 64 + lane + 32 * j];
            const float a = v[j], b = v[j + 2];
            v[j] = a * cs.x - b * cs.y;
            v[j + 2] = b * cs.x + a * cs.y;
        }
    }
    if (hd < 16) {
        const size_t o = (size_t)t * ldq + hd * HDIM + lane;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            if (q_bf16) q_bf16[o + 32 * j] = f32_to_bf16_rne(v[j]);
            if (q_f32) q_f32[o + 32 * j] = v[j];
        }
    } else {
        const int kvh = (hd - 16) & 7;
        uint16_t *dst = (hd < 24 ? kc : vc) +
                        (((size_t)(seq * NLAYER + layer) * NKVH + kvh) * max_len + pos) * HDIM;
#pragma unroll
        for (int j = 0; j < 4; j++) dst[lane + 32 * j] = f32_to_bf16_rne(v[j]);
    }
}

// K/V rows (FP32, after QK-norm and RoPE) of T tokens of sequence slot 0 into
// the BF16 cache at positions pos0.. (the dump route's qwen3.c:498-511).
__global__ void dump_kv_kernel(uint16_t *kc, uint16_t *vc, const float *__restrict__ k,
                               const float *__restrict__ v, int layer, int max_len, int pos0) {
    dep_wait();
    dep_launch();
    const int t = blockIdx.x, i = threadIdx.x, kvh = i >> 7, d = i & 127;
    const size_t o = (((size_t)layer * NKVH + kvh) * max_len + pos0 + t) * HDIM + d;
    kc[o] = f32_to_bf16_rne(k[(size_t)t * KVD + i]);
    vc[o] = f32_to_bf16_rne(v[(size_t)t * KVD + i]);
}

// (cos, sin) of pos * inv_freq[i] for every position and rotation pair: the
// RoPE factors of ops_scalar.c:21-35, computed once per model with the same
// function the fused q/k/v GEMM epilogue evaluates in registers.
__global__ void rope_table_kernel(float2 *t, int max_len) {
    const int idx = blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= max_len * 64) return;
    float s, c;
    rope_sincos((float)(idx >> 6) * c_inv_freq[idx & 63], &s, &c);
    t[idx] = make_float2(c, s);
}

// After a decode step: record the chosen ids (row *counter of out) and feed
// them back as the next step's tokens at the next positions.
__global__ void decode_advance_kernel(const int32_t *next, int32_t *tokens, int32_t *pos,
                                      int32_t *out, int32_t *counter, int n) {
    dep_wait();
    dep_launch();
    const int step = *counter;
    for (int s = threadIdx.x; s < n; s += blockDim.x) {
        const int32_t id = next[s];
        out[(size_t)step * n + s] = id;
        tokens[s] = id;
        pos[s] += 1;
    }
    __syncthreads();
    if (threadIdx.x == 0) *counter = step + 1;
}

// x[t] += sum of ks split-K partial slices (the o / down projection, the
// residual add of qwen3.c:523/543), then, if w is given, out[t] =
// bf16(rmsnorm(x[t]) * w) for the next GEMM (qwen3.c:471/527/547). One CTA
// per row of 1024.
__global__ void __launch_bounds__(256)
resid_norm_rows_kernel(float *x, const float *__restrict__ ws, int ks, size_t slice,
                       const uint16_t *__restrict__ w, uint16_t *out) {
    // the norm weight is no kernel's output: read before the wait
    float wv[4];
#pragma unroll
    for (int j = 0; j < 4; j++) wv[j] = w ? bf16_bits_to_f32(w[threadIdx.x + 256 * j]) : 0.f;
    dep_wait();
    dep_launch();
    __shared__ float red[8];
    const int t = blockIdx.x;
    float *xr = x + (size_t)t * H;
    const float *pr = ws + (size_t)t * H;
    float xv[4];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const int c = threadIdx.x + 256 * j;
        xv[j] = xr[c] + sum_slices(pr + c, ks, slice);
        xr[c] = xv[j];
        ss = fmaf(xv[j], xv[j], ss);
    }
    if (!w) return;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    ss = 0.f;
#pragma unroll
    for (int i = 0; i < 8; i++) ss += red[i];
    const float sc = 1.0f / sqrtf(ss / (float)H + EPS);
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const int c = threadIdx.x + 256 * j;
        out[(size_t)t * H + c] = f32_to_bf16_rne(xv[j] * sc * wv[j]);
    }
}

// out[t] = bf16(rmsnorm(x[t]) * w) for rows of 1024 (qwen3.c:471/527, the
// normalised GEMM input): one warp per row, eight 16-byte loads per lane held
// in registers, warp-shuffle sum of squares, 8-byte stores. PRE_W (the few
// rows of a decode step, where the kernel is latency-bound): the norm weight,
// no kernel's output, is read before the programmatic-launch wait; a
// prefill's many rows keep the registers for loads in flight instead.
template <bool PRE_W>
__global__ void __launch_bounds__(256)
norm_rows_bf16_kernel(uint16_t *__restrict__ out, const float *__restrict__ x,
                      const uint16_t *__restrict__ w, int T) {
    // A prefill's rows are taken last to first: the residual GEMM before this
    // kernel wrote the last row blocks last, so those are still in L2, and
    // the GEMM after it reads the first rows first, which this order writes
    // last (measured on B200, 64 x 512 prefill: 2.30 -> 2.20 ms of norms per
    // step; the same bits either way)
    const int idx = blockIdx.x * 8 + (threadIdx.x >> 5);
    const int row = PRE_W ? idx : (int)gridDim.x * 8 - 1 - idx;
    const int lane = threadIdx.x & 31;
    const uint2 *wr = (const uint2 *)w;
    uint2 wv[8];
    if (PRE_W) {
#pragma unroll
        for (int i = 0; i < 8; i++) wv[i] = __ldg(wr + lane + 32 * i);
    }
    dep_wait();
    dep_launch();
    if (row >= T) return;
    const float4 *xr = (const float4 *)(x + (size_t)row * H);
    float4 v[8];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        v[i] = __ldg(xr + lane + 32 * i);
        ss = fmaf(v[i].x, v[i].x, ss);
        ss = fmaf(v[i].y, v[i].y, ss);
        ss = fmaf(v[i].z, v[i].z, ss);
        ss = fmaf(v[i].w, v[i].w, ss);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, o);
    const float sc = 1.0f / sqrtf(ss / (float)H + EPS);
    uint2 *orow = (uint2 *)(out + (size_t)row * H);
#pragma unroll
    for (int i = 0; i < 8; i++) {
        if (!PRE_W) wv[i] = __ldg(wr + lane + 32 * i);
        uint2 o;
        o.x = pack_bf16x2(v[i].x * sc * __uint_as_float(wv[i].x << 16),
                          v[i].y * sc * __uint_as_float(wv[i].x & 0xFFFF0000u));
        o.y = pack_bf16x2(v[i].z * sc * __uint_as_float(wv[i].y << 16),
                          v[i].w * sc * __uint_as_float(wv[i].y & 0xFFFF0000u));
        orow[lane + 32 * i] = o;
    }
}

// Final RMSNorm of the last token of each sequence (qwen3.c:547-573 only
// needs row NT-1): xl[i] = rmsnorm(x[i*Lc + Lc - 1]) in BF16.
__global__ void __launch_bounds__(256)
final_norm_kernel(uint16_t *xl, const float *__restrict__ x, const uint16_t *__restrict__ w, int Lc) {
    // the norm weight is no kernel's output: read before the wait
    float wv[4];
#pragma unroll
    for (int j = 0; j < 4; j++) wv[j] = bf16_bits_to_f32(w[threadIdx.x + 256 * j]);
    dep_wait();
    dep_launch();
    __shared__ float red[8];
    const float *xr = x + ((size_t)blockIdx.x * Lc + Lc - 1) * H;
    float xv[4];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < 4; j++) {
        xv[j] = xr[threadIdx.x + 256 * j];
        ss = fmaf(xv[j], xv[j], ss);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    ss = 0.f;
#pragma unroll
    for (int i = 0; i < 8; i++) ss += red[i];
    const float sc = 1.0f / sqrtf(ss / (float)H + EPS);
#pragma unroll
    for (int j = 0; j < 4; j++)
        xl[(size_t)blockIdx.x * H + threadIdx.x + 256 * j] = f32_to_bf16_rne(xv[j] * sc * wv[j]);
}

// h = silu(g) * u in BF16 (the unfused SwiGLU for the GEMV / exact paths).
__global__ void silu_mul_bf16_kernel(uint16_t *h, const float *__restrict__ g,
                                     const float *__restrict__ u, size_t n) {
    dep_wait();
    dep_launch();
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x) {
        const float gv = g[i];
        h[i] = f32_to_bf16_rne((gv / (1.0f + expf(-gv))) * u[i]);
    }
}

int grid1(size_t n) {
    size_t g = (n + 255) / 256;
    return (int)std::min<size_t>(std::max<size_t>(g, 1), 148 * 16);
}

}  // namespace
}  // namespace n550

using namespace n550;

// Per-kind kernel timing (n550_qwen3_profile): event pairs recorded on the
// launch stream around each launch while enabled.
struct ModelProf {
    bool on = false;
    std::vector<cudaEvent_t> pool;
    size_t used = 0;
    std::vector<std::pair<int, size_t>> marks;   // (kind, index of the start event)
    long long launches[N550_PROF_KINDS] = {};
    cudaEvent_t next_event() {
        if (used == pool.size()) {
            cudaEvent_t e;
            if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
            pool.push_back(e);
        }
        return pool[used++];
    }
};

struct n550_model {
    ModelProf prof;
    int dev = 0;
    n550_model_config cfg{};
    uint8_t *blob = nullptr;
    size_t blob_size = 0;
    size_t off[N_TENSORS] = {};
    const uint16_t *t[N_TENSORS] = {};
    uint16_t *fused_qkv = nullptr;          // only if q/k/v are not contiguous
    const uint16_t *wqkv[NLAYER] = {};
    uint16_t *kc = nullptr, *vc = nullptr;
    float *x = nullptr, *qkv = nullptr, *qf = nullptr, *logits = nullptr;
    uint16_t *xb = nullptr, *qb = nullptr, *attn = nullptr, *h = nullptr, *xl = nullptr;
    float *tmp_a = nullptr, *tmp_b = nullptr;
    size_t tmp_rows = 0;
    int32_t *tok_pos = nullptr, *tok_seq = nullptr, *next = nullptr, *host_tok = nullptr,
            *zero_seq = nullptr;
    float *part_m = nullptr, *part_l = nullptr, *part_o = nullptr;
    float2 *rope = nullptr;                 // [max_len][64] (cos, sin)
    float *ws = nullptr;                    // split-K partials of skinny GEMMs
    size_t ws_bytes = 0;
    n550_dump_fn dump = nullptr;            // per-op tensor dump (n550_qwen3_set_dump)
    void *dump_ctx = nullptr;
    FusedLayer *fd_layers = nullptr;        // layer tensors for the persistent decode kernel
    int *fd_counters = nullptr;             // its attention-split arrivals [FD_MAX_TOKENS][8]
    int *attn_counters = nullptr;           // decode attention split arrivals [max_seqs][8]
    unsigned *fd_barrier = nullptr;         // its grid-barrier counter
    // captured decode step (n550_qwen3_decode_steps)
    cudaGraphExec_t graph = nullptr;
    int g_n = 0;
    const void *g_key[4] = {};
    int32_t *step_counter = nullptr;
    // captured prefill of the last repeated call (n550_qwen3_prefill)
    cudaGraphExec_t pgraph = nullptr;
    long long pg_key[7] = {};               // key of the captured call
    long long pg_last[7] = {};              // key of the previous eager call
    cudaStream_t cap_stream = nullptr;      // capture/replay stream (the legacy
    cudaEvent_t ev_in = nullptr, ev_out = nullptr;   // stream cannot be captured)
};

namespace {

const uint16_t *W(const n550_model *m, int layer, int j) { return m->t[1 + 11 * layer + j]; }

// Token counts from which a layer's GEMMs run as whole tiles with their fused
// epilogues (q/k/v with QK-norm, RoPE and the KV write; residual adds by TMA
// reduce-add; SwiGLU); below, down to 9 tokens, the K loop is split and the
// partial sums are finished by row kernels (n550_qwen3_split_rows).
int g_split_rows = 1024;

// Decode steps of up to FD_MAX_TOKENS sequences run as one persistent kernel
// (n550_qwen3_fused_decode).
bool g_fused_decode = false;

int run_layers_fused(n550_model *m, cudaStream_t st, int T, const int32_t *seq_ids, const int32_t *pos) {
    FusedDecodeArgs a{};
    a.layers = m->fd_layers;
    a.final_norm = m->t[N_TENSORS - 1];
    a.kc = m->kc; a.vc = m->vc; a.max_len = m->cfg.max_len;
    a.rope = m->rope;
    a.seq_ids = seq_ids; a.pos = pos; a.T = T;
    a.x = m->x; a.qkv = m->qkv; a.attn = m->attn; a.h = m->h;
    a.part_m = m->part_m; a.part_l = m->part_l; a.part_o = m->part_o;
    a.counters = m->fd_counters;
    a.barrier = m->fd_barrier;
    a.xl = m->xl;
    return launch_decode_fused(st, a);
}

// Brackets the kernels launched in its scope with an event pair of `kind`
// (n kernels counted) while profiling is enabled.
struct ProfScope {
    n550_model *m;
    cudaStream_t st;
    int kind;
    cudaEvent_t e1 = nullptr;
    ProfScope(n550_model *m_, cudaStream_t st_, int kind_, int n = 1) : m(m_), st(st_), kind(kind_) {
        if (!m->prof.on) return;
        m->prof.launches[kind] += n;
        const size_t idx = m->prof.used;
        cudaEvent_t e0 = m->prof.next_event();
        e1 = m->prof.next_event();
        if (!e0 || !e1) { e1 = nullptr; return; }
        cudaEventRecord(e0, st);
        m->prof.marks.push_back({kind, idx});
    }
    ~ProfScope() { if (e1) cudaEventRecord(e1, st); }
};

void model_release(n550_model *m) {
    if (!m) return;
    if (m->graph) cudaGraphExecDestroy(m->graph);
    if (m->pgraph) cudaGraphExecDestroy(m->pgraph);
    if (m->step_counter) cudaFree(m->step_counter);
    if (m->cap_stream) cudaStreamDestroy(m->cap_stream);
    if (m->ev_in) cudaEventDestroy(m->ev_in);
    if (m->ev_out) cudaEventDestroy(m->ev_out);
    for (cudaEvent_t e : m->prof.pool) cudaEventDestroy(e);
    void *ptrs[] = {m->blob, m->fused_qkv, m->kc, m->vc, m->x, m->qkv, m->qf, m->logits, m->xb,
                    m->qb, m->attn, m->h, m->xl, m->tmp_a, m->tmp_b, m->tok_pos, m->tok_seq,
                    m->next, m->host_tok, m->zero_seq, m->part_m, m->part_l, m->part_o, m->rope, m->ws,
                    m->fd_layers, m->fd_counters, m->fd_barrier, m->attn_counters};
    for (void *p : ptrs) if (p) cudaFree(p);
    delete m;
}

// Allocations that depend on the config; the blob must already be on device.
int model_setup(n550_model *m) {
    const n550_model_config &c = m->cfg;
    for (int i = 0; i < N_TENSORS; i++) m->t[i] = (const uint16_t *)(m->blob + m->off[i]);
    bool contiguous = true;
    for (int l = 0; l < NLAYER; l++)
        contiguous = contiguous && W(m, l, 2) == W(m, l, 1) + (size_t)QD * H &&
                     W(m, l, 3) == W(m, l, 2) + (size_t)KVD * H;
    if (contiguous) {
        for (int l = 0; l < NLAYER; l++) m->wqkv[l] = W(m, l, 1);
    } else {
        N550_CUDA_TRY(cudaMalloc(&m->fused_qkv, (size_t)NLAYER * QKVD * H * 2));
        for (int l = 0; l < NLAYER; l++) {
            uint16_t *d = m->fused_qkv + (size_t)l * QKVD * H;
            N550_CUDA_TRY(cudaMemcpy(d, W(m, l, 1), (size_t)QD * H * 2, cudaMemcpyDeviceToDevice));
            N550_CUDA_TRY(cudaMemcpy(d + (size_t)QD * H, W(m, l, 2), (size_t)KVD * H * 2,
                                     cudaMemcpyDeviceToDevice));
            N550_CUDA_TRY(cudaMemcpy(d + (size_t)(QD + KVD) * H, W(m, l, 3), (size_t)KVD * H * 2,
                                     cudaMemcpyDeviceToDevice));
            m->wqkv[l] = d;
        }
    }
    const size_t T = (size_t)c.max_tokens, S = (size_t)c.max_seqs;
    const size_t kv = (size_t)c.max_seqs * NLAYER * NKVH * (size_t)c.max_len * HDIM;
#define ALLOC(p, bytes) N550_CUDA_TRY(cudaMalloc((void **)&(p), (bytes)))
    ALLOC(m->kc, kv * 2);
    ALLOC(m->vc, kv * 2);
    ALLOC(m->x, T * H * 4);
    ALLOC(m->xb, T * H * 2);
    ALLOC(m->qkv, T * QKVD * 4);
    ALLOC(m->qb, T * QD * 2);
    ALLOC(m->qf, S * QD * 4);
    ALLOC(m->attn, T * QD * 2);
    ALLOC(m->h, T * INTER * 2);
    // last-token rows; n550_qwen3_forward_rows normalises every row of a
    // call of up to N550_ROWS_MAX tokens into the same buffer
    const size_t head_rows = std::max(S, std::min(T, (size_t)N550_ROWS_MAX));
    ALLOC(m->xl, head_rows * H * 2);
    ALLOC(m->logits, head_rows * (size_t)VOCAB * 4);
    m->tmp_rows = c.gemm_mode == N550_MODE_EXACT ? T : 8;
    ALLOC(m->tmp_a, m->tmp_rows * INTER * 4);
    ALLOC(m->tmp_b, m->tmp_rows * INTER * 4);
    ALLOC(m->tok_pos, T * 4);
    ALLOC(m->tok_seq, T * 4);
    ALLOC(m->next, S * 4);
    ALLOC(m->host_tok, (T + N550_ROWS_MAX) * 4);
    ALLOC(m->zero_seq, 4);
    const size_t slots = S * NH * MAX_SPLITS;
    ALLOC(m->part_m, slots * 4);
    ALLOC(m->part_l, slots * 4);
    ALLOC(m->part_o, slots * HDIM * 4);
    ALLOC(m->rope, (size_t)c.max_len * 64 * sizeof(float2));
    // split-K workspace: up to 8 slices of [rows < 1024][2 x 3072] FP32
    m->ws_bytes = (size_t)8 * std::min<size_t>(T, 1023) * 2 * INTER * 4;
    ALLOC(m->ws, m->ws_bytes);
    ALLOC(m->step_counter, 4);
    ALLOC(m->fd_layers, NLAYER * sizeof(FusedLayer));
    ALLOC(m->fd_counters, FD_MAX_TOKENS * NKVH * sizeof(int));
    ALLOC(m->fd_barrier, sizeof(unsigned));
    ALLOC(m->attn_counters, S * NKVH * sizeof(int));
    N550_CUDA_TRY(cudaStreamCreateWithFlags(&m->cap_stream, cudaStreamNonBlocking));
    N550_CUDA_TRY(cudaEventCreateWithFlags(&m->ev_in, cudaEventDisableTiming));
    N550_CUDA_TRY(cudaEventCreateWithFlags(&m->ev_out, cudaEventDisableTiming));
#undef ALLOC
    N550_CUDA_TRY(cudaMemset(m->zero_seq, 0, 4));
    N550_CUDA_TRY(cudaMemset(m->fd_counters, 0, FD_MAX_TOKENS * NKVH * sizeof(int)));
    N550_CUDA_TRY(cudaMemset(m->attn_counters, 0, S * NKVH * sizeof(int)));
    {
        FusedLayer fl[NLAYER];
        for (int l = 0; l < NLAYER; l++)
            fl[l] = FusedLayer{W(m, l, 0), m->wqkv[l], W(m, l, 4), W(m, l, 5), W(m, l, 6),
                               W(m, l, 7), W(m, l, 8), W(m, l, 9), W(m, l, 10)};
        N550_CUDA_TRY(cudaMemcpy(m->fd_layers, fl, sizeof fl, cudaMemcpyHostToDevice));
    }
    N550_CUDA_TRY(cudaMemset(m->kc, 0, kv * 2));
    N550_CUDA_TRY(cudaMemset(m->vc, 0, kv * 2));
    int rc = ensure_rope_table();
    if (rc) return rc;
    rope_table_kernel<<<(c.max_len * 64 + 255) / 256, 256>>>(m->rope, c.max_len);
    N550_LAUNCH_CHECK();
    N550_CUDA_TRY(cudaDeviceSynchronize());
    return N550_OK;
}

int check_cfg(const n550_model_config *c) {
    if (!c || c->max_seqs < 1 || c->max_len < 1 || c->max_tokens < 1) return N550_ERR_ARG;
    if (c->gemm_mode != N550_MODE_FAST && c->gemm_mode != N550_MODE_EXACT) return N550_ERR_ARG;
    if (c->gemm_mode == N550_MODE_EXACT && c->kblock != 16 && c->kblock != 32) return N550_ERR_ARG;
    return N550_OK;
}

// A [M,K] BF16 . W[N,K]^T with epilogue `epi` into c (ldc). SILU takes W2.
// x_ready: see launch_gemv (the decoder layer's o and down projections).
int mgemm(n550_model *m, cudaStream_t st, int epi, const uint16_t *a, int lda, const uint16_t *w,
          const uint16_t *w2, void *c, int ldc, int M, int N, int K, bool x_ready = false) {
    if (m->cfg.gemm_mode == N550_MODE_EXACT) {
        if (epi == TC_EPI_F32)
            return launch_gemm_exact(st, a, N550_BF16, lda, w, K, (float *)c, ldc, M, N, K, m->cfg.kblock);
        if (epi == TC_EPI_RESID_F32) {
            int rc = launch_gemm_exact(st, a, N550_BF16, lda, w, K, m->tmp_a, N, M, N, K, m->cfg.kblock);
            if (rc) return rc;
            return launch_residual_add(st, (float *)c, m->tmp_a, (size_t)M * N);
        }
        if (epi == TC_EPI_SILU_BF16) {
            int rc = launch_gemm_exact(st, a, N550_BF16, lda, w, K, m->tmp_a, N, M, N, K, m->cfg.kblock);
            if (!rc) rc = launch_gemm_exact(st, a, N550_BF16, lda, w2, K, m->tmp_b, N, M, N, K, m->cfg.kblock);
            if (rc) return rc;
            N550_CUDA_TRY(launch_k(silu_mul_bf16_kernel, grid1((size_t)M * N), 256, 0, st, (uint16_t *)c,
                                   m->tmp_a, m->tmp_b, (size_t)M * N));
            N550_LAUNCH_CHECK();
            return N550_OK;
        }
        return N550_ERR_ARG;
    }
    if (M <= 8) {
        if (epi != TC_EPI_SILU_BF16) return launch_gemv(st, epi, a, lda, w, K, c, ldc, M, N, K, x_ready);
        // gate, up and SiLU . mul in one GEMV launch
        return launch_gemv_swiglu(st, a, lda, w, w2, K, (uint16_t *)c, ldc, M, N, K);
    }
    if (M < g_split_rows)   // skinny (decode, short prompts): split the K loop over more SMs
        return launch_gemm_tc_splitk(st, epi, a, lda, w, K, w2, c, ldc, M, N, K, m->ws, m->ws_bytes);
    return launch_gemm_tc(st, epi, n550_tile_bn(M, epi == TC_EPI_SILU_BF16 ? 2 * N : N), a, lda, w, K, w2, c,
                          ldc, M, N, K, 0);
}

int launch_qknorm_rope_kv(n550_model *m, cudaStream_t st, int T, int l, bool decode,
                          const float *src = nullptr, int ks = 0) {
    N550_CUDA_TRY(launch_k(qknorm_rope_kv_kernel, T, 1024, 0, st, src ? src : m->qkv, QKVD, ks,
                           (size_t)T * QKVD, W(m, l, 4), W(m, l, 5), m->rope, m->tok_pos, m->tok_seq, l,
                           m->kc, m->vc, m->cfg.max_len, decode ? nullptr : m->qb,
                           decode ? m->qf : nullptr, QD));
    N550_LAUNCH_CHECK();
    return N550_OK;
}

int launch_resid_norm(cudaStream_t st, float *x, const float *ws, int ks, int T,
                      const uint16_t *w, uint16_t *out) {
    N550_CUDA_TRY(launch_k(resid_norm_rows_kernel, T, 256, 0, st, x, ws, ks, (size_t)T * H, w, out));
    N550_LAUNCH_CHECK();
    return N550_OK;
}

// Split-K partial sums of A . W^T into m->ws (fast mode, skinny M).
int partials(n550_model *m, cudaStream_t st, const uint16_t *a, int lda, const uint16_t *w, int M,
             int N, int K, int *ks) {
    return launch_gemm_tc_partials(st, TC_EPI_F32, a, lda, w, K, nullptr, M, N, K, m->ws,
                                   m->ws_bytes, ks);
}

int launch_norm_rows(cudaStream_t st, uint16_t *out, const float *x, const uint16_t *w, int T) {
    if (T <= 0) return N550_OK;
    if (T <= 64)
        N550_CUDA_TRY(launch_k(norm_rows_bf16_kernel<true>, (T + 7) / 8, 256, 0, st, out, x, w, T));
    else
        N550_CUDA_TRY(launch_k(norm_rows_bf16_kernel<false>, (T + 7) / 8, 256, 0, st, out, x, w, T));
    N550_LAUNCH_CHECK();
    return N550_OK;
}

int launch_final_norm(cudaStream_t st, uint16_t *xl, const float *x, const uint16_t *w, int Sc, int Lc) {
    N550_CUDA_TRY(launch_k(final_norm_kernel, Sc, 256, 0, st, xl, x, w, Lc));
    N550_LAUNCH_CHECK();
    return N550_OK;
}

// All 28 layers over T tokens already embedded in m->x, with tok_pos/tok_seq
// set. decode: one token per sequence (seq_ids/pos arrays of n_seqs = T).
#define STEP(kind, nk, expr)                          \
    do {                                              \
        ProfScope ps_(m, st, (kind), (nk));           \
        if ((rc = (expr))) return rc;                 \
    } while (0)

// Decode attention takes the q/k/v rows before QK-norm and RoPE and finishes
// them itself (the K/V write included) instead of a separate row kernel
// (n550_qwen3_fused_attention_prep).
bool g_fused_prep = true;

int run_attention(n550_model *m, cudaStream_t st, int T, bool decode, const int32_t *seq_ids,
                  const int32_t *pos, int Sc, int Lc, int p0, int l, bool q_in_bf16 = false,
                  const float *raw_qkv = nullptr, int ks = 0) {
    const n550_model_config &c = m->cfg;
    int rc = N550_OK;
    if (decode) {
        AttnDecodeArgs a{};
        a.q_f32 = q_in_bf16 ? nullptr : m->qf;
        a.q_bf16 = m->qb;
        a.kc = m->kc; a.vc = m->vc; a.out = m->attn;
        a.seq_ids = seq_ids; a.pos = pos;
        a.ldq = QD; a.ldo = QD; a.layer = l; a.max_len = c.max_len;
        a.kv_planes = c.max_seqs * NLAYER * NKVH;
        a.splits = attn_decode_splits(T, c.max_len, MAX_SPLITS);
        a.part_m = m->part_m; a.part_l = m->part_l; a.part_o = m->part_o;
        a.counters = m->attn_counters;
        if (raw_qkv) {
            a.qkv = raw_qkv; a.qkv_ld = QKVD; a.qkv_ks = ks; a.qkv_slice = (size_t)T * QKVD;
            a.q_norm = W(m, l, 4); a.k_norm = W(m, l, 5); a.rope = m->rope;
            a.kc_w = m->kc; a.vc_w = m->vc;
        }
        STEP(N550_PROF_ATTN, 1, launch_attn_decode(st, a, T));
    } else {
        AttnPrefillArgs a{};
        a.q = m->qb; a.kc = m->kc; a.vc = m->vc; a.out = m->attn; a.seq_ids = seq_ids;
        a.ldq = QD; a.ldo = QD; a.L = Lc; a.pos0 = p0; a.layer = l; a.max_len = c.max_len;
        a.kv_planes = c.max_seqs * NLAYER * NKVH;
        STEP(N550_PROF_ATTN, 1, launch_attn_prefill(st, a, Sc));
    }
    return N550_OK;
}

// Skinny token counts (8 < T < 1024: decode, short prompts). Every projection
// is a split-K tensor-core GEMM whose partial sums feed a fused row kernel:
// QKV -> sum + QK-norm + RoPE + K/V write; o and down -> sum + residual add +
// the next RMSNorm (input_layernorm of the next layer, or the final norm for
// decode, whose rows are all last tokens); gate/up -> sum + SwiGLU.
// Sets *xl_ready when the final norm was applied to all T rows (into m->xl).
int run_layers_split(n550_model *m, cudaStream_t st, int T, bool decode, const int32_t *seq_ids,
                     const int32_t *pos, int Sc, int Lc, int p0, bool *xl_ready) {
    int rc = N550_OK, ks = 0, kt;
    const int gu_kernels = tc_splitk_plan(T, INTER, H, TC_EPI_SILU_BF16, 64, &kt) > 1 ? 2 : 1;
    STEP(N550_PROF_RMSNORM, 1, launch_norm_rows(st, m->xb, m->x, W(m, 0, 0), T));
    for (int l = 0; l < NLAYER; l++) {
        STEP(N550_PROF_GEMM_QKV, 1, partials(m, st, m->xb, H, m->wqkv[l], T, QKVD, H, &ks));
        if (decode && g_fused_prep) {
            if ((rc = run_attention(m, st, T, decode, seq_ids, pos, Sc, Lc, p0, l, false, m->ws, ks))) return rc;
        } else {
            STEP(N550_PROF_QKNORM_ROPE, 1, launch_qknorm_rope_kv(m, st, T, l, decode, m->ws, ks));
            if ((rc = run_attention(m, st, T, decode, seq_ids, pos, Sc, Lc, p0, l))) return rc;
        }
        STEP(N550_PROF_GEMM_O, 1, partials(m, st, m->attn, QD, W(m, l, 6), T, H, QD, &ks));
        STEP(N550_PROF_RMSNORM, 1, launch_resid_norm(st, m->x, m->ws, ks, T, W(m, l, 7), m->xb));
        STEP(N550_PROF_GEMM_GATEUP, gu_kernels,
             mgemm(m, st, TC_EPI_SILU_BF16, m->xb, H, W(m, l, 8), W(m, l, 9), m->h, INTER, T, INTER, H));
        STEP(N550_PROF_GEMM_DOWN, 1, partials(m, st, m->h, INTER, W(m, l, 10), T, H, INTER, &ks));
        const uint16_t *wn = l + 1 < NLAYER ? W(m, l + 1, 0) : (decode ? m->t[N_TENSORS - 1] : nullptr);
        uint16_t *dst = l + 1 < NLAYER ? m->xb : m->xl;
        STEP(N550_PROF_RMSNORM, 1, launch_resid_norm(st, m->x, m->ws, ks, T, wn, dst));
    }
    *xl_ready = decode;
    return N550_OK;
}

// Token counts above 8 that skinny_route() gives to the weight-streaming GEMM
// (the decode step of 9-32 sequences by default): every projection is one GEMM
// whose epilogue finishes the op -- QKV with QK-norm, RoPE and the K/V write;
// o and down with the residual add; gate/up with SwiGLU -- so a layer is 4
// GEMMs, attention and 2 RMSNorms.
int run_layers_skinny(n550_model *m, cudaStream_t st, int T, bool decode, const int32_t *seq_ids,
                      const int32_t *pos, int Sc, int Lc, int p0, bool *xl_ready) {
    const n550_model_config &c = m->cfg;
    int rc = N550_OK;
    STEP(N550_PROF_RMSNORM, 1, launch_norm_rows(st, m->xb, m->x, W(m, 0, 0), T));
    SkEpilogue resid{};
    resid.out = m->x;
    resid.ldo = H;
    SkEpilogue swiglu{};
    swiglu.h = m->h;
    swiglu.ldh = INTER;
    for (int l = 0; l < NLAYER; l++) {
        SkEpilogue q{};
        q.q_f32 = decode ? m->qf : nullptr;       // decode attention reads FP32 queries
        q.q_bf16 = decode ? nullptr : m->qb;      // the tcgen05 prefill attention BF16
        q.ldq = QD;
        q.kc = m->kc; q.vc = m->vc; q.layer = l; q.max_len = c.max_len;
        q.tok_pos = m->tok_pos; q.tok_seq = m->tok_seq;
        q.q_norm = W(m, l, 4); q.k_norm = W(m, l, 5);
        q.rope = m->rope;
        STEP(N550_PROF_GEMM_QKV, 1,
             launch_gemm_skinny(st, SK_EPI_QKV, m->xb, H, m->wqkv[l], nullptr, H, T, QKVD, H, q));
        if ((rc = run_attention(m, st, T, decode, seq_ids, pos, Sc, Lc, p0, l))) return rc;
        STEP(N550_PROF_GEMM_O, 1,
             launch_gemm_skinny(st, SK_EPI_RESID, m->attn, QD, W(m, l, 6), nullptr, QD, T, H, QD, resid));
        STEP(N550_PROF_RMSNORM, 1, launch_norm_rows(st, m->xb, m->x, W(m, l, 7), T));
        STEP(N550_PROF_GEMM_GATEUP, 1,
             launch_gemm_skinny(st, SK_EPI_SILU, m->xb, H, W(m, l, 8), W(m, l, 9), H, T, INTER, H, swiglu));
        STEP(N550_PROF_GEMM_DOWN, 1,
             launch_gemm_skinny(st, SK_EPI_RESID, m->h, INTER, W(m, l, 10), nullptr, INTER, T, H, INTER,
                                resid));
        // input norm of the next layer; after the last, the final norm (decode:
        // every row is a last token; prefill normalises its last rows later)
        const uint16_t *wn = l + 1 < NLAYER ? W(m, l + 1, 0) : (decode ? m->t[N_TENSORS - 1] : nullptr);
        uint16_t *dst = l + 1 < NLAYER ? m->xb : m->xl;
        if (wn) STEP(N550_PROF_RMSNORM, 1, launch_norm_rows(st, dst, m->x, wn, T));
    }
    *xl_ready = decode;
    return N550_OK;
}

// All 28 layers over T tokens already embedded in m->x, with tok_pos/tok_seq
// set. decode: one token per sequence (seq_ids/pos arrays of n_seqs = T).
int run_layers(n550_model *m, cudaStream_t st, int T, bool decode, const int32_t *seq_ids,
               const int32_t *pos, int Sc, int Lc, int p0, bool *xl_ready) {
    const n550_model_config &c = m->cfg;
    int rc = N550_OK;
    *xl_ready = false;
    const bool exact = c.gemm_mode == N550_MODE_EXACT;
    // A decode step of a few sequences: all 28 layers in one persistent kernel
    if (!exact && decode && g_fused_decode && T <= FD_MAX_TOKENS && c.max_len <= FD_MAX_LEN &&
        T <= c.max_seqs && fused_decode_grid() > 0) {
        ProfScope ps(m, st, N550_PROF_GEMM_QKV, 1);
        if ((rc = run_layers_fused(m, st, T, seq_ids, pos))) return rc;
        *xl_ready = true;
        return N550_OK;
    }
    // Up to 8 tokens the GEMV path (5 kernels per layer up to 4 tokens, 7
    // from 5: the norms then run as their own kernels) is ahead of the skinny
    // GEMMs (7 kernels with their cluster exchanges). Measured on B200,
    // graph-replayed decode steps at a 1024-token context: 2, 3, 4, 6, 8
    // sequences 836 / 935 / 1029 / 1130 / 1424 us (GEMV) vs 839 / 932 / 1235 /
    // 1263 / 1445 us (skinny) per step.
    if (!exact && T > 8 && skinny_route(T))
        return run_layers_skinny(m, st, T, decode, seq_ids, pos, Sc, Lc, p0, xl_ready);
    if (!exact && T > 8 && T < g_split_rows)
        return run_layers_split(m, st, T, decode, seq_ids, pos, Sc, Lc, p0, xl_ready);
    const bool fused_qkv = !exact && T >= g_split_rows;
    // the GEMV route of up to 4 rows normalises its input rows inside the q/k/v
    // and gate/up GEMVs (no norm launches)
    const bool gv_norm = !exact && T <= 4;
    const int gu_kernels = exact ? 3 : 1;
    const int res_kernels = exact ? 2 : 1;
    for (int l = 0; l < NLAYER; l++) {
        if (!gv_norm) STEP(N550_PROF_RMSNORM, 1, launch_norm_rows(st, m->xb, m->x, W(m, l, 0), T));
        if (gv_norm) {
            STEP(N550_PROF_GEMM_QKV, 1,
                 launch_gemv(st, TC_EPI_F32, nullptr, 0, m->wqkv[l], H, m->qkv, QKVD, T, QKVD, H, false, m->x,
                             W(m, l, 0)));
            if (!(decode && g_fused_prep))
                STEP(N550_PROF_QKNORM_ROPE, 1, launch_qknorm_rope_kv(m, st, T, l, decode));
        } else if (fused_qkv) {
            // One tcgen05 GEMM with QK-norm, RoPE and the K/V cache write in its epilogue.
            TcQkv q{};
            q.q_bf16 = m->qb;
            q.ldq = QD;
            q.kc = m->kc; q.vc = m->vc; q.layer = l; q.max_len = c.max_len;
            q.tok_pos = m->tok_pos; q.tok_seq = m->tok_seq;
            q.q_norm = W(m, l, 4); q.k_norm = W(m, l, 5);
            q.rope = m->rope; q.eps = EPS;
            STEP(N550_PROF_GEMM_QKV, 1, launch_gemm_tc_qkv(st, m->xb, H, m->wqkv[l], q, T, H, 0));
        } else {
            STEP(N550_PROF_GEMM_QKV, 1,
                 mgemm(m, st, TC_EPI_F32, m->xb, H, m->wqkv[l], nullptr, m->qkv, QKVD, T, QKVD, H));
            if (!(decode && g_fused_prep))
                STEP(N550_PROF_QKNORM_ROPE, 1, launch_qknorm_rope_kv(m, st, T, l, decode));
        }
        // the fused QKV epilogue leaves BF16 queries (decode attention reads either);
        // otherwise decode attention may finish the raw q/k/v rows itself
        const float *raw = !fused_qkv && decode && g_fused_prep ? m->qkv : nullptr;
        if ((rc = run_attention(m, st, T, decode, seq_ids, pos, Sc, Lc, p0, l, fused_qkv, raw, 0)))
            return rc;
        // o and down: the residual rows x were last written two or more kernels
        // back (the embedding or the previous residual GEMM), never by the
        // attention or the gate/up GEMM that precede them
        STEP(N550_PROF_GEMM_O, res_kernels,
             mgemm(m, st, TC_EPI_RESID_F32, m->attn, QD, W(m, l, 6), nullptr, m->x, H, T, H, QD, true));
        if (gv_norm) {
            STEP(N550_PROF_GEMM_GATEUP, 1,
                 launch_gemv_swiglu(st, nullptr, 0, W(m, l, 8), W(m, l, 9), H, m->h, INTER, T, INTER, H, m->x,
                                    W(m, l, 7)));
        } else {
            STEP(N550_PROF_RMSNORM, 1, launch_norm_rows(st, m->xb, m->x, W(m, l, 7), T));
            STEP(N550_PROF_GEMM_GATEUP, gu_kernels,
                 mgemm(m, st, TC_EPI_SILU_BF16, m->xb, H, W(m, l, 8), W(m, l, 9), m->h, INTER, T, INTER, H));
        }
        STEP(N550_PROF_GEMM_DOWN, res_kernels,
             mgemm(m, st, TC_EPI_RESID_F32, m->h, INTER, W(m, l, 10), nullptr, m->x, H, T, H, INTER, true));
    }
    return N550_OK;
}

// Last-token logits and argmax for Sc sequences whose rows are i*Lc + Lc - 1.
// logits == nullptr: the caller wants only the next tokens. In fast mode the
// lm_head GEMM then carries the argmax in its epilogue (per-tile maxima merged
// by one small kernel) and the [Sc, 151936] FP32 logits are never written.
int run_head(n550_model *m, cudaStream_t st, int Sc, int Lc, float *logits, int32_t *next,
             bool xl_ready = false) {
    int rc = N550_OK;
    if (!xl_ready)
        STEP(N550_PROF_RMSNORM, 1, launch_final_norm(st, m->xl, m->x, m->t[N_TENSORS - 1], Sc, Lc));
    if (!logits && next && m->cfg.gemm_mode == N550_MODE_FAST && Sc >= 4) {
        STEP(N550_PROF_GEMM_LMHEAD, 2,
             launch_gemm_tc_argmax(st, m->xl, H, m->t[0], H, Sc, VOCAB, H, m->ws, m->ws_bytes, next));
        return N550_OK;
    }
    if (!logits) logits = m->logits;
    STEP(N550_PROF_GEMM_LMHEAD, 1,
         mgemm(m, st, TC_EPI_F32, m->xl, H, m->t[0], nullptr, logits, VOCAB, Sc, VOCAB, H));
    if (next) STEP(N550_PROF_OTHER, 1, launch_argmax(st, logits, Sc, VOCAB, VOCAB, next));
    return N550_OK;
}

// The forward of T tokens of slot 0 op by op with every intermediate tensor
// materialised in FP32 and handed to the dump callback under the reference's
// names and in its order (qwen3.c:464-575, the EMIT points). The GEMMs take
// BF16 inputs and give FP32 as the runtime's; norms, RoPE, SiLU . mul and the
// residual adds are the op kernels of the C ABI; attention is the tcgen05
// prefill attention on the BF16 cache. For locating numerical drift, not speed.
int dump_forward(n550_model *m, cudaStream_t st, const int32_t *tokens, int T, int pos0) {
    const n550_model_config &c = m->cfg;
    float *q = nullptr, *k = nullptr, *v = nullptr, *g = nullptr, *u = nullptr, *o = nullptr,
          *att = nullptr, *host = nullptr;
    uint16_t *bf = nullptr, *attn = nullptr;
    int rc = N550_OK;
    auto emit = [&](int layer, const char *name, const float *d, size_t n) -> int {
        N550_CUDA_TRY(cudaMemcpyAsync(host, d, n * 4, cudaMemcpyDeviceToHost, st));
        N550_CUDA_TRY(cudaStreamSynchronize(st));
        m->dump(m->dump_ctx, layer, name, host, n);
        return N550_OK;
    };
    const size_t Tn = (size_t)T;
#define DTRY(expr) do { if ((rc = (expr))) goto done; } while (0)
#define DALLOC(p, bytes) do { if (cudaMalloc((void **)&(p), (bytes)) != cudaSuccess) { \
        (void)cudaGetLastError(); rc = N550_ERR_OOM; goto done; } } while (0)
    DALLOC(q, Tn * QD * 4); DALLOC(k, Tn * KVD * 4); DALLOC(v, Tn * KVD * 4);
    DALLOC(g, Tn * INTER * 4); DALLOC(u, Tn * INTER * 4); DALLOC(o, Tn * H * 4);
    DALLOC(att, Tn * QD * 4); DALLOC(bf, Tn * INTER * 2); DALLOC(attn, Tn * QD * 2);
    if (cudaMallocHost((void **)&host, (size_t)VOCAB * 4 + Tn * INTER * 4) != cudaSuccess) {
        (void)cudaGetLastError();
        host = nullptr;
        rc = N550_ERR_OOM;
        goto done;
    }
    if (launch_k(setup_prefill_kernel, (T + 255) / 256, 256, 0, st, m->tok_pos, m->tok_seq,
                 m->zero_seq, 1, T, pos0) != cudaSuccess ||
        launch_k(embed_kernel, T, 128, 0, st, m->x, m->t[0], tokens, T, T, 0, nullptr, nullptr,
                 nullptr, nullptr) != cudaSuccess) { rc = N550_ERR_CUDA; goto done; }
    DTRY(emit(-1, "embed_out", m->x, Tn * H));
    for (int l = 0; l < NLAYER; l++) {
        // xb = rmsnorm(x) (FP32 dumped, BF16 into the GEMMs)
        DTRY(launch_rmsnorm(st, o, N550_F32, m->x, W(m, l, 0), T, H, EPS));
        DTRY(emit(l, "input_layernorm_out", o, Tn * H));
        DTRY(launch_f32_to_bf16(st, bf, H, o, H, T, H));
        DTRY(mgemm(m, st, TC_EPI_F32, bf, H, W(m, l, 1), nullptr, q, QD, T, QD, H));
        DTRY(emit(l, "q_proj_out", q, Tn * QD));
        DTRY(launch_rmsnorm(st, q, N550_F32, q, W(m, l, 4), T * NH, HDIM, EPS));
        DTRY(emit(l, "q_norm_out", q, Tn * QD));
        DTRY(mgemm(m, st, TC_EPI_F32, bf, H, W(m, l, 2), nullptr, k, KVD, T, KVD, H));
        DTRY(emit(l, "k_proj_out", k, Tn * KVD));
        DTRY(launch_rmsnorm(st, k, N550_F32, k, W(m, l, 5), T * NKVH, HDIM, EPS));
        DTRY(emit(l, "k_norm_out", k, Tn * KVD));
        DTRY(mgemm(m, st, TC_EPI_F32, bf, H, W(m, l, 3), nullptr, v, KVD, T, KVD, H));
        DTRY(emit(l, "v_proj_out", v, Tn * KVD));
        DTRY(launch_rope(st, q, T, NH, pos0));
        DTRY(emit(l, "q_rope_out", q, Tn * QD));
        DTRY(launch_rope(st, k, T, NKVH, pos0));
        DTRY(emit(l, "k_rope_out", k, Tn * KVD));
        if (launch_k(dump_kv_kernel, T, KVD, 0, st, m->kc, m->vc, (const float *)k, (const float *)v, l,
                     c.max_len, pos0) != cudaSuccess) { rc = N550_ERR_CUDA; goto done; }
        DTRY(launch_f32_to_bf16(st, bf, QD, q, QD, T, QD));      // BF16 queries, as the runtime's
        {
            AttnPrefillArgs a{};
            a.q = bf; a.kc = m->kc; a.vc = m->vc; a.out = attn; a.seq_ids = m->zero_seq;
            a.ldq = QD; a.ldo = QD; a.L = T; a.pos0 = pos0; a.layer = l; a.max_len = c.max_len;
            a.kv_planes = c.max_seqs * NLAYER * NKVH;
            DTRY(launch_attn_prefill(st, a, 1));
        }
        DTRY(launch_bf16_to_f32(st, att, attn, Tn * QD));
        DTRY(emit(l, "attn_out", att, Tn * QD));
        DTRY(mgemm(m, st, TC_EPI_F32, attn, QD, W(m, l, 6), nullptr, o, H, T, H, QD));
        DTRY(emit(l, "o_proj_out", o, Tn * H));
        DTRY(launch_residual_add(st, m->x, o, Tn * H));
        DTRY(emit(l, "x_after_attn_residual", m->x, Tn * H));
        DTRY(launch_rmsnorm(st, o, N550_F32, m->x, W(m, l, 7), T, H, EPS));
        DTRY(emit(l, "post_attn_norm_out", o, Tn * H));
        DTRY(launch_f32_to_bf16(st, bf, H, o, H, T, H));
        DTRY(mgemm(m, st, TC_EPI_F32, bf, H, W(m, l, 8), nullptr, g, INTER, T, INTER, H));
        DTRY(emit(l, "gate_proj_out", g, Tn * INTER));
        DTRY(mgemm(m, st, TC_EPI_F32, bf, H, W(m, l, 9), nullptr, u, INTER, T, INTER, H));
        DTRY(emit(l, "up_proj_out", u, Tn * INTER));
        DTRY(launch_silu_mul(st, g, u, Tn * INTER));
        DTRY(emit(l, "silu_gate_mul_up", g, Tn * INTER));
        DTRY(launch_f32_to_bf16(st, bf, INTER, g, INTER, T, INTER));
        DTRY(mgemm(m, st, TC_EPI_F32, bf, INTER, W(m, l, 10), nullptr, o, H, T, H, INTER));
        DTRY(emit(l, "down_proj_out", o, Tn * H));
        DTRY(launch_residual_add(st, m->x, o, Tn * H));
        DTRY(emit(l, "layer_out", m->x, Tn * H));
    }
    DTRY(launch_rmsnorm(st, o, N550_F32, m->x, m->t[N_TENSORS - 1], T, H, EPS));
    DTRY(emit(-1, "final_norm_out", o, Tn * H));
    DTRY(launch_f32_to_bf16(st, bf, H, o + (Tn - 1) * H, H, 1, H));
    DTRY(mgemm(m, st, TC_EPI_F32, bf, H, m->t[0], nullptr, m->logits, VOCAB, 1, VOCAB, H));
    DTRY(emit(-1, "logits", m->logits, VOCAB));
done:
#undef DTRY
#undef DALLOC
    cudaStreamSynchronize(st);
    for (void *p : {(void *)q, (void *)k, (void *)v, (void *)g, (void *)u, (void *)o, (void *)att,
                    (void *)bf, (void *)attn})
        if (p) cudaFree(p);
    if (host) cudaFreeHost(host);
    return rc;
}

}  // namespace

extern "C" {

int n550_qwen3_init(n550_model_t **out, const void *blob, size_t blob_size,
                    const n550_model_config *cfg) {
    if (!out || !blob) return N550_ERR_ARG;
    *out = nullptr;
    int rc = check_cfg(cfg);
    if (rc) return rc;
    n550_model *m = new n550_model();
    m->cfg = *cfg;
    bool tiled = false;
    rc = parse_qw3m((const uint8_t *)blob, blob_size, m->off, &tiled);
    if (rc) { model_release(m); return rc; }
    cudaGetDevice(&m->dev);
    m->blob_size = blob_size;
    if (cudaMalloc(&m->blob, blob_size) != cudaSuccess) { model_release(m); return N550_ERR_OOM; }
    if (cudaMemcpy(m->blob, blob, blob_size, cudaMemcpyHostToDevice) != cudaSuccess) {
        model_release(m);
        return N550_ERR_CUDA;
    }
    if (tiled) {
        // Tile-major GEMM weights are put back into row-major order in place
        // (through a scratch copy), so every kernel sees one layout.
        uint16_t *tmp = nullptr;
        if (cudaMalloc(&tmp, (size_t)INTER * H * 2) != cudaSuccess) { model_release(m); return N550_ERR_OOM; }
        for (int t = 0; t < N_TENSORS && !rc; t++) {
            int N = 0, K = 0;
            if (!is_gemm_weight(t, &N, &K)) continue;
            uint16_t *w = (uint16_t *)(m->blob + m->off[t]);
            if (cudaMemcpy(tmp, w, (size_t)N * K * 2, cudaMemcpyDeviceToDevice) != cudaSuccess) {
                rc = N550_ERR_CUDA;
                break;
            }
            untile_weight_kernel<<<1184, 256>>>(w, tmp, N, K);
            if (cudaGetLastError() != cudaSuccess) rc = N550_ERR_CUDA;
        }
        if (!rc && cudaDeviceSynchronize() != cudaSuccess) rc = N550_ERR_CUDA;
        cudaFree(tmp);
        if (rc) { model_release(m); return rc; }
    }
    rc = model_setup(m);
    if (rc) { model_release(m); return rc; }
    *out = m;
    return N550_OK;
}

int n550_qwen3_init_random(n550_model_t **out, uint64_t seed, double sigma,
                           const n550_model_config *cfg) {
    if (!out) return N550_ERR_ARG;
    *out = nullptr;
    int rc = check_cfg(cfg);
    if (rc) return rc;
    n550_model *m = new n550_model();
    m->cfg = *cfg;
    uint8_t hdr[256];
    make_header(hdr);
    m->blob_size = qw3m_row_size();
    rc = parse_qw3m(hdr, m->blob_size, m->off);
    if (rc) { model_release(m); return rc; }
    cudaGetDevice(&m->dev);
    if (cudaMalloc(&m->blob, m->blob_size) != cudaSuccess) { model_release(m); return N550_ERR_OOM; }
    if (cudaMemset(m->blob, 0, m->blob_size) != cudaSuccess ||
        cudaMemcpy(m->blob, hdr, 256, cudaMemcpyHostToDevice) != cudaSuccess) {
        model_release(m);
        return N550_ERR_CUDA;
    }
    const float scale = synth_normal_scale(sigma);
    for (int t = 0; t < N_TENSORS; t++) {
        bool nrm;
        const size_t n = tensor_elems(t, &nrm);
        uint16_t *dst = (uint16_t *)(m->blob + m->off[t]);
        if (nrm) fill_u16_kernel<<<grid1(n), 256>>>(dst, n, (uint16_t)0x3F80);
        else synth_bf16_kernel<<<148 * 16, 256>>>(dst, n, synth_key(seed, (uint64_t)t), scale);
        if (cudaPeekAtLastError() != cudaSuccess) { model_release(m); return N550_ERR_CUDA; }
    }
    rc = model_setup(m);
    if (rc) { model_release(m); return rc; }
    *out = m;
    return N550_OK;
}

void n550_qwen3_free(n550_model_t *m) {
    if (m) cudaDeviceSynchronize();
    model_release(m);
}

static int prefill_eager(n550_model_t *m, cudaStream_t st, const int32_t *tokens,
                         const int32_t *seq_ids, int n_seqs, int seq_len, int pos0, float *logits,
                         int32_t *next_token);

// A call that repeats the previous call's buffers and shape (a serving loop
// over a fixed batch, a benchmark) is captured into a CUDA graph on its second
// occurrence and replayed from then on: the ~1000 launches and tensor-map
// encodings of a prefill leave the host. The first occurrence runs eagerly, so
// one-time setup (kernel attributes) never enters a capture. With the
// profiler on, every call runs eagerly.
int n550_qwen3_prefill(n550_model_t *m, void *stream, const int32_t *tokens, const int32_t *seq_ids,
                       int n_seqs, int seq_len, int pos0, float *logits, int32_t *next_token) {
    if (!m || !tokens || !seq_ids || n_seqs < 1 || seq_len < 1 || pos0 < 0) return N550_ERR_ARG;
    const n550_model_config &c = m->cfg;
    if (pos0 + seq_len > c.max_len) return N550_ERR_ARG;
    cudaStream_t st = (cudaStream_t)stream;
    if (m->prof.on) return prefill_eager(m, st, tokens, seq_ids, n_seqs, seq_len, pos0, logits, next_token);
    const long long key[7] = {(long long)(uintptr_t)tokens, (long long)(uintptr_t)seq_ids,
                              (long long)(uintptr_t)logits, (long long)(uintptr_t)next_token,
                              n_seqs, seq_len, pos0};
    const bool replay = m->pgraph && !memcmp(key, m->pg_key, sizeof key);
    const bool capture = !replay && !memcmp(key, m->pg_last, sizeof key);
    if (!replay && !capture) {
        memcpy(m->pg_last, key, sizeof key);
        return prefill_eager(m, st, tokens, seq_ids, n_seqs, seq_len, pos0, logits, next_token);
    }
    const cudaStream_t cs = m->cap_stream;
    N550_CUDA_TRY(cudaEventRecord(m->ev_in, st));
    N550_CUDA_TRY(cudaStreamWaitEvent(cs, m->ev_in, 0));
    int rc = N550_OK;
    if (capture) {
        if (m->pgraph) { cudaGraphExecDestroy(m->pgraph); m->pgraph = nullptr; }
        cudaGraph_t g = nullptr;
        if (cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
            rc = N550_ERR_CUDA;
        } else {
            rc = prefill_eager(m, cs, tokens, seq_ids, n_seqs, seq_len, pos0, logits, next_token);
            const cudaError_t ce = cudaStreamEndCapture(cs, &g);
            if (!rc && ce != cudaSuccess) rc = N550_ERR_CUDA;
        }
        if (!rc && cudaGraphInstantiate(&m->pgraph, g, 0) != cudaSuccess) {
            m->pgraph = nullptr;
            rc = N550_ERR_CUDA;
        }
        if (g) cudaGraphDestroy(g);
        (void)cudaGetLastError();
        if (!rc) memcpy(m->pg_key, key, sizeof key);
        else memset(m->pg_last, 0, sizeof m->pg_last);
    }
    if (!rc && cudaGraphLaunch(m->pgraph, cs) != cudaSuccess) rc = N550_ERR_CUDA;
    N550_CUDA_TRY(cudaEventRecord(m->ev_out, cs));
    N550_CUDA_TRY(cudaStreamWaitEvent(st, m->ev_out, 0));
    if (rc) return rc;
    return N550_OK;
}

static int prefill_eager(n550_model_t *m, cudaStream_t st, const int32_t *tokens,
                         const int32_t *seq_ids, int n_seqs, int seq_len, int pos0, float *logits,
                         int32_t *next_token) {
    const n550_model_config &c = m->cfg;
    const int Lmax = std::min(seq_len, c.max_tokens);
    int rc;
    for (int s0 = 0; s0 < n_seqs;) {
        const int Sc = std::max(1, std::min({n_seqs - s0, c.max_tokens / Lmax, c.max_seqs}));
        for (int j0 = 0; j0 < seq_len; j0 += Lmax) {
            const int Lc = std::min(Lmax, seq_len - j0);
            const int T = Sc * Lc;
            const int p0 = pos0 + j0;
            {
                ProfScope ps(m, st, N550_PROF_OTHER, 2);
                N550_CUDA_TRY(launch_k(setup_prefill_kernel, (T + 255) / 256, 256, 0, st, m->tok_pos,
                                       m->tok_seq, seq_ids + s0, Sc, Lc, p0));
                N550_CUDA_TRY(launch_k(embed_kernel, T, 128, 0, st, m->x, m->t[0],
                                       tokens + (size_t)s0 * seq_len, Lc, seq_len, j0, nullptr,
                                       nullptr, nullptr, nullptr));
                N550_LAUNCH_CHECK();
            }
            bool xl_ready = false;
            if ((rc = run_layers(m, st, T, false, seq_ids + s0, nullptr, Sc, Lc, p0, &xl_ready))) return rc;
            if (j0 + Lc == seq_len) {
                float *lg = logits ? logits + (size_t)s0 * VOCAB : nullptr;
                if ((rc = run_head(m, st, Sc, Lc, lg, next_token ? next_token + s0 : nullptr)))
                    return rc;
            }
        }
        s0 += Sc;
    }
    return N550_OK;
}

int n550_qwen3_decode(n550_model_t *m, void *stream, const int32_t *tokens, const int32_t *seq_ids,
                      const int32_t *pos, int n_seqs, float *logits, int32_t *next_token) {
    if (!m || !tokens || !seq_ids || !pos || n_seqs < 1) return N550_ERR_ARG;
    const n550_model_config &c = m->cfg;
    if (n_seqs > c.max_tokens || n_seqs > c.max_seqs) return N550_ERR_ARG;
    cudaStream_t st = (cudaStream_t)stream;
    {
        ProfScope ps(m, st, N550_PROF_OTHER, 1);
        N550_CUDA_TRY(launch_k(embed_kernel, n_seqs, 128, 0, st, m->x, m->t[0], tokens, 1, 1, 0, pos,
                               seq_ids, m->tok_pos, m->tok_seq));
        N550_LAUNCH_CHECK();
    }
    bool xl_ready = false;
    int rc = run_layers(m, st, n_seqs, true, seq_ids, pos, n_seqs, 1, 0, &xl_ready);
    if (rc) return rc;
    return run_head(m, st, n_seqs, 1, logits, next_token, xl_ready);
}

int n550_qwen3_decode_steps(n550_model_t *m, void *stream, int32_t *tokens, const int32_t *seq_ids,
                            int32_t *pos, int n_seqs, int steps, int32_t *out_ids, int use_graph) {
    if (!m || !tokens || !seq_ids || !pos || !out_ids || n_seqs < 1 || steps < 0) return N550_ERR_ARG;
    if (n_seqs > m->cfg.max_tokens || n_seqs > m->cfg.max_seqs) return N550_ERR_ARG;
    cudaStream_t st = (cudaStream_t)stream;
    N550_CUDA_TRY(cudaMemsetAsync(m->step_counter, 0, 4, st));   // ordered before the capture stream joins
    auto one_step = [&]() -> int {
        int rc = n550_qwen3_decode(m, st, tokens, seq_ids, pos, n_seqs, nullptr, m->next);
        if (rc) return rc;
        N550_CUDA_TRY(launch_k(decode_advance_kernel, 1, 256, 0, st, m->next, tokens, pos, out_ids,
                               m->step_counter, n_seqs));
        N550_LAUNCH_CHECK();
        return N550_OK;
    };
    if (!use_graph) {
        for (int i = 0; i < steps; i++) {
            int rc = one_step();
            if (rc) return rc;
        }
        return N550_OK;
    }
    // Capture and replay on the model's own stream, ordered after the
    // caller's stream and joined back to it with events.
    const cudaStream_t cs = m->cap_stream;
    N550_CUDA_TRY(cudaEventRecord(m->ev_in, st));
    N550_CUDA_TRY(cudaStreamWaitEvent(cs, m->ev_in, 0));
    auto step_on = [&](cudaStream_t s_) -> int {
        int rc = n550_qwen3_decode(m, s_, tokens, seq_ids, pos, n_seqs, nullptr, m->next);
        if (rc) return rc;
        N550_CUDA_TRY(launch_k(decode_advance_kernel, 1, 256, 0, s_, m->next, tokens, pos, out_ids,
                               m->step_counter, n_seqs));
        N550_LAUNCH_CHECK();
        return N550_OK;
    };
    int rc = N550_OK;
    const void *key[4] = {tokens, seq_ids, pos, out_ids};
    const bool same = m->graph && m->g_n == n_seqs && !memcmp(key, m->g_key, sizeof key);
    if (!same && steps > 0) {
        if (m->graph) { cudaGraphExecDestroy(m->graph); m->graph = nullptr; }
        // Step 0 runs uncaptured: first launches set kernel attributes, and
        // the capture below must not contain one-time work.
        rc = step_on(cs);
        steps--;
        if (!rc) {
            const bool prof = m->prof.on;
            m->prof.on = false;
            cudaGraph_t g = nullptr;
            if (cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
                rc = N550_ERR_CUDA;
            } else {
                rc = step_on(cs);
                const cudaError_t ce = cudaStreamEndCapture(cs, &g);
                if (!rc && ce != cudaSuccess) rc = N550_ERR_CUDA;
            }
            m->prof.on = prof;
            if (!rc && cudaGraphInstantiate(&m->graph, g, 0) != cudaSuccess) {
                m->graph = nullptr;
                rc = N550_ERR_CUDA;
            }
            if (g) cudaGraphDestroy(g);
            (void)cudaGetLastError();
            if (!rc) {
                m->g_n = n_seqs;
                memcpy(m->g_key, key, sizeof key);
            }
        }
    }
    for (int i = 0; i < steps && !rc; i++)
        if (cudaGraphLaunch(m->graph, cs) != cudaSuccess) rc = N550_ERR_CUDA;
    N550_CUDA_TRY(cudaEventRecord(m->ev_out, cs));
    N550_CUDA_TRY(cudaStreamWaitEvent(st, m->ev_out, 0));
    return rc;
}

int n550_qwen3_fused_attention_prep(int on) {
    g_fused_prep = on != 0;
    return N550_OK;
}

int n550_qwen3_fused_decode(int on) {
    g_fused_decode = on != 0;
    return N550_OK;
}

int n550_qwen3_split_rows(int rows) {
    if (rows < 9 || rows > 1024) return N550_ERR_ARG;
    g_split_rows = rows;
    return N550_OK;
}

int n550_qwen3_get_config(const n550_model_t *m, n550_model_config *cfg) {
    if (!m || !cfg) return N550_ERR_ARG;
    *cfg = m->cfg;
    return N550_OK;
}

int n550_qwen3_forward_rows(n550_model_t *m, void *stream, const int32_t *tokens,
                            const int32_t *seq_id, int n_token, int pos0, float *logits,
                            int32_t *next_ids) {
    if (!m || !tokens || !seq_id || n_token < 1 || n_token > N550_ROWS_MAX || pos0 < 0 ||
        (!logits && !next_ids))
        return N550_ERR_ARG;
    const n550_model_config &c = m->cfg;
    if (pos0 + n_token > c.max_len || n_token > c.max_tokens) return N550_ERR_ARG;
    cudaStream_t st = (cudaStream_t)stream;
    {
        ProfScope ps(m, st, N550_PROF_OTHER, 2);
        N550_CUDA_TRY(launch_k(setup_prefill_kernel, (n_token + 255) / 256, 256, 0, st, m->tok_pos,
                               m->tok_seq, seq_id, 1, n_token, pos0));
        N550_CUDA_TRY(launch_k(embed_kernel, n_token, 128, 0, st, m->x, m->t[0], tokens, n_token,
                               n_token, 0, nullptr, nullptr, nullptr, nullptr));
        N550_LAUNCH_CHECK();
    }
    bool xl_ready = false;
    int rc = run_layers(m, st, n_token, false, seq_id, nullptr, 1, n_token, pos0, &xl_ready);
    if (rc) return rc;
    // every row is a "last token" of its own (qwen3.c:556-566): the final norm
    // and the lm_head (+ argmax) over all n_token rows
    return run_head(m, st, n_token, 1, logits, next_ids);
}

int n550_qwen3_forward_rows_host(n550_model_t *m, const int32_t *tokens, int n_token, int pos0,
                                 int32_t *next_ids_host, float *logits_host) {
    if (!m || !tokens || !next_ids_host || n_token < 1 || n_token > N550_ROWS_MAX) return N550_ERR_ARG;
    if (n_token > m->cfg.max_tokens) return N550_ERR_ARG;
    cudaStream_t st = 0;
    N550_CUDA_TRY(cudaMemcpyAsync(m->host_tok, tokens, (size_t)n_token * 4, cudaMemcpyHostToDevice, st));
    int rc = n550_qwen3_forward_rows(m, st, m->host_tok, m->zero_seq, n_token, pos0,
                                     logits_host ? m->logits : nullptr, m->host_tok + n_token);
    if (rc) return rc;
    N550_CUDA_TRY(cudaMemcpyAsync(next_ids_host, m->host_tok + n_token, (size_t)n_token * 4,
                                  cudaMemcpyDeviceToHost, st));
    if (logits_host)
        N550_CUDA_TRY(cudaMemcpyAsync(logits_host, m->logits, (size_t)n_token * VOCAB * 4,
                                      cudaMemcpyDeviceToHost, st));
    N550_CUDA_TRY(cudaStreamSynchronize(st));
    return N550_OK;
}

int n550_qwen3_set_dump(n550_model_t *m, n550_dump_fn fn, void *ctx) {
    if (!m) return N550_ERR_ARG;
    m->dump = fn;
    m->dump_ctx = ctx;
    return N550_OK;
}

int n550_qwen3_forward_batch_host(n550_model_t *m, const int32_t *tokens, int n_token, int pos0,
                                  float *logits_host) {
    if (!m || !tokens || n_token < 1) return N550_ERR_ARG;
    if (n_token > m->cfg.max_tokens) return N550_ERR_ARG;
    cudaStream_t st = 0;
    N550_CUDA_TRY(cudaMemcpyAsync(m->host_tok, tokens, (size_t)n_token * 4, cudaMemcpyHostToDevice, st));
    if (m->dump) {
        if (pos0 < 0 || pos0 + n_token > m->cfg.max_len) return N550_ERR_ARG;
        int rc = dump_forward(m, st, m->host_tok, n_token, pos0);
        if (rc) return rc;
        int32_t best = 0;
        N550_CUDA_TRY(launch_argmax(st, m->logits, 1, VOCAB, VOCAB, m->next) ? cudaErrorUnknown : cudaSuccess);
        N550_CUDA_TRY(cudaMemcpyAsync(&best, m->next, 4, cudaMemcpyDeviceToHost, st));
        if (logits_host)
            N550_CUDA_TRY(cudaMemcpyAsync(logits_host, m->logits, (size_t)VOCAB * 4, cudaMemcpyDeviceToHost, st));
        N550_CUDA_TRY(cudaStreamSynchronize(st));
        return best;
    }
    int rc = n550_qwen3_prefill(m, st, m->host_tok, m->zero_seq, 1, n_token, pos0, m->logits, m->next);
    if (rc) return rc;
    int32_t best = 0;
    N550_CUDA_TRY(cudaMemcpyAsync(&best, m->next, 4, cudaMemcpyDeviceToHost, st));
    if (logits_host)
        N550_CUDA_TRY(cudaMemcpyAsync(logits_host, m->logits, (size_t)VOCAB * 4, cudaMemcpyDeviceToHost, st));
    N550_CUDA_TRY(cudaStreamSynchronize(st));
    return best;
}

int n550_qwen3_profile(n550_model_t *m, int enable) {
    if (!m) return N550_ERR_ARG;
    if (enable) {
        m->prof.used = 0;
        m->prof.marks.clear();
        for (long long &v : m->prof.launches) v = 0;
    }
    m->prof.on = enable != 0;
    return N550_OK;
}

int n550_qwen3_profile_read(n550_model_t *m, double *ms, int64_t *launches, int n_kinds) {
    if (!m || n_kinds < 0) return N550_ERR_ARG;
    N550_CUDA_TRY(cudaDeviceSynchronize());
    double acc[N550_PROF_KINDS] = {};
    for (const auto &mk : m->prof.marks) {
        float t = 0.f;
        N550_CUDA_TRY(cudaEventElapsedTime(&t, m->prof.pool[mk.second], m->prof.pool[mk.second + 1]));
        acc[mk.first] += t;
    }
    for (int k = 0; k < n_kinds && k < N550_PROF_KINDS; k++) {
        if (ms) ms[k] = acc[k];
        if (launches) launches[k] = m->prof.launches[k];
    }
    return N550_OK;
}

const uint16_t *n550_qwen3_weight(const n550_model_t *m, int which, size_t *elems) {
    if (!m || which < 0 || which >= N_TENSORS) return nullptr;
    bool nrm;
    if (elems) *elems = tensor_elems(which, &nrm);
    return m->t[which];
}

int n550_rope_table(void *stream, float *table, int max_len) {
    if (max_len < 0 || (max_len && !table) || ((uintptr_t)table & 7)) return N550_ERR_ARG;
    if (max_len == 0) return N550_OK;
    int rc = ensure_rope_table();
    if (rc) return rc;
    rope_table_kernel<<<(max_len * 64 + 255) / 256, 256, 0, (cudaStream_t)stream>>>((float2 *)table,
                                                                                    max_len);
    N550_LAUNCH_CHECK();
    return N550_OK;
}

// The decoder layer's q/k/v step on the route the runtime takes for M rows
// (run_layers): tile GEMM with the fused epilogue from 1024 rows (BF16
// queries), the weight-streaming GEMM with the fused epilogue for 9 rows on
// where skinny_route(M), else FP32 q/k/v rows (GEMV up to 8 rows, split-K partials
// otherwise, in a stream-ordered workspace) finished by qknorm_rope_kv_kernel.
int n550_qkv_rope_kv(void *stream, const uint16_t *x, int ldx, const uint16_t *wqkv,
                     const uint16_t *q_norm, const uint16_t *k_norm, const float *rope_table,
                     const int32_t *tok_seq, const int32_t *tok_pos, int M, void *q_out,
                     int q_type, int ldq, uint16_t *k_cache, uint16_t *v_cache, int max_len,
                     int layer) {
    cudaStream_t st = (cudaStream_t)stream;
    if (M < 0 || max_len <= 0 || layer < 0 || layer >= NLAYER) return N550_ERR_ARG;
    if (M == 0) return N550_OK;
    if (!x || !wqkv || !q_norm || !k_norm || !rope_table || !tok_seq || !tok_pos || !q_out ||
        !k_cache || !v_cache || ldx < H || ldq < QD || (q_type != N550_F32 && q_type != N550_BF16))
        return N550_ERR_ARG;
    int rc = ensure_rope_table();
    if (rc) return rc;
    const float2 *rope = (const float2 *)rope_table;
    uint16_t *qb = q_type == N550_BF16 ? (uint16_t *)q_out : nullptr;
    float *qf = q_type == N550_F32 ? (float *)q_out : nullptr;
    if (M >= 1024 && qb && tc_shape_ok(x, ldx, wqkv, H, H)) {
        TcQkv q{};
        q.q_bf16 = qb; q.ldq = ldq;
        q.kc = k_cache; q.vc = v_cache; q.layer = layer; q.max_len = max_len;
        q.tok_pos = tok_pos; q.tok_seq = tok_seq;
        q.q_norm = q_norm; q.k_norm = k_norm; q.rope = rope; q.eps = EPS;
        return launch_gemm_tc_qkv(st, x, ldx, wqkv, q, M, H, 0);
    }
    if (M > 8 && skinny_route(M) && tc_shape_ok(x, ldx, wqkv, H, H)) {
        SkEpilogue q{};
        q.q_f32 = qf; q.q_bf16 = qb; q.ldq = ldq;
        q.kc = k_cache; q.vc = v_cache; q.layer = layer; q.max_len = max_len;
        q.tok_pos = tok_pos; q.tok_seq = tok_seq;
        q.q_norm = q_norm; q.k_norm = k_norm; q.rope = rope;
        rc = launch_gemm_skinny(st, SK_EPI_QKV, x, ldx, wqkv, nullptr, H, M, QKVD, H, q);
        if (rc != N550_ERR_UNSUPPORTED) return rc;
    }
    int ks = 0, kt;
    const bool split = M > 8 && tc_shape_ok(x, ldx, wqkv, H, H);
    const size_t bytes = (size_t)(split ? 8 : 1) * M * QKVD * 4;
    float *ws = nullptr;
    if (cudaMallocAsync((void **)&ws, bytes, st) != cudaSuccess) {
        (void)cudaGetLastError();
        return N550_ERR_OOM;
    }
    if (split && tc_splitk_plan(M, QKVD, H, TC_EPI_F32, 64, &kt) > 0)
        rc = launch_gemm_tc_partials(st, TC_EPI_F32, x, ldx, wqkv, H, nullptr, M, QKVD, H, ws, bytes, &ks);
    else if (M <= 8)
        rc = launch_gemv(st, TC_EPI_F32, x, ldx, wqkv, H, ws, QKVD, M, QKVD, H);
    else
        rc = launch_gemm_simt(st, TC_EPI_F32, x, ldx, wqkv, H, ws, QKVD, M, QKVD, H);
    if (!rc) {
        if (launch_k(qknorm_rope_kv_kernel, M, 1024, 0, st, (const float *)ws, QKVD, ks,
                     (size_t)M * QKVD, q_norm, k_norm, rope, tok_pos, tok_seq, layer, k_cache, v_cache,
                     max_len, qb, qf, ldq) != cudaSuccess)
            rc = N550_ERR_CUDA;
        (void)cudaGetLastError();
    }
    cudaFreeAsync(ws, st);
    return rc;
}

}  // extern "C"
