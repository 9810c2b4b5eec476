/* n550 Qwen3-0.6B hot path on NVIDIA B200 (sm_100a) -- the C ABI.
 *
 * libn550_qwen3.so exports two layers:
 *
 * 1. The reference's operator plug points, same names and meaning, taking
 *    HOST pointers (drop-in for the KERNEL=ame / OPS=rvv backends): each call
 *    copies its operands to the current CUDA device, runs the CUDA kernel and
 *    copies the result back before returning, so on return the output is
 *    globally visible, as kernels_ame.c:438-444 guarantees. Like the
 *    reference these functions return nothing; a failed call leaves the output
 *    untouched (the reference's silent-return contract, kernels_ame.c:221) and
 *    records a status readable with n550_last_status().
 *
 * 2. A device-pointer, stream-ordered API (n550_*) with the same math that
 *    returns a status code, plus the model runtime that keeps the weights, the
 *    KV cache and all activations in HBM.
 *
 * No torch types, no C++ types: plain pointers and sizes. Streams are passed
 * as `void *` holding a cudaStream_t (NULL = legacy default stream).
 */
#ifndef N550_QWEN3_H
#define N550_QWEN3_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* The library is built with hidden visibility; everything declared here is
 * exported. */
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

/* ---------------------------------------------------------------------------
 * Status codes. Model-loader codes equal the reference's QWEN3_ERR_* values
 * (qwen3.h:190-201); the n550 codes are below -100.
 * ------------------------------------------------------------------------- */
enum {
    N550_OK               = 0,
    N550_ERR_MAGIC        = -1,   /* QWEN3_ERR_MAGIC   */
    N550_ERR_VERSION      = -2,   /* QWEN3_ERR_VERSION */
    N550_ERR_DTYPE        = -3,   /* QWEN3_ERR_DTYPE   */
    N550_ERR_SHAPE        = -4,   /* QWEN3_ERR_SHAPE   */
    N550_ERR_SIZE         = -5,   /* QWEN3_ERR_SIZE    */
    N550_ERR_OOM          = -6,   /* QWEN3_ERR_OOM     */
    N550_ERR_LAYOUT       = -7,   /* QWEN3_ERR_LAYOUT  */
    N550_ERR_ARG          = -101, /* argument outside the documented contract */
    N550_ERR_CUDA         = -102, /* a CUDA runtime call failed               */
    N550_ERR_UNSUPPORTED  = -103, /* shape/alignment this build does not take */
    N550_ERR_TIMEOUT      = -104  /* a bounded device-side wait expired       */
};

/* GEMM numerics. */
enum {
    N550_MODE_EXACT = 0,  /* AME golden numerics, bit-exact: exact sum per
                             K-block, binary64 then binary32 RNE per block */
    N550_MODE_FAST  = 1   /* tcgen05 tensor cores, BF16 x BF16 -> FP32     */
};

/* Element types for the device API. */
enum { N550_F32 = 0, N550_BF16 = 1 };

/* Weight layouts (kernels.h:67-68). */
#define N550_LAYOUT_ROW  0
#define N550_LAYOUT_TILE 1

/* ===========================================================================
 * 1. Reference plug points, host pointers
 * ========================================================================= */

/* C[M,N] = bf16_rne(A[M,K]) . B[N,K]^T; A FP32, B BF16 [out,in], C FP32,
 * all row-major. Replaces kernels.h:56-57 (qwen3_gemm) as implemented by
 * kernels_ame.c:448-451. Numerics follow n550_set_gemm_mode (default: exact
 * AME numerics, K-block 16). */
void qwen3_gemm(float *c, const float *a, const uint16_t *b, int M, int K, int N);

/* Same contract with B always row-major (kernels.h:79-80, kernels_ame.c:456-459). */
void qwen3_gemm_row(float *c, const float *a, const uint16_t *b, int M, int K, int N);

/* Accepts QW3M_LAYOUT_ROW (0) and QW3M_LAYOUT_TILE (1) with tile 128x32;
 * returns 0 when accepted, -1 otherwise (kernels.h:89, kernels_ame.c:188-207). */
int qwen3_set_weight_layout(int layout, int tile_n, int tile_k);

/* Name of this backend (kernels.h:92). */
const char *qwen3_kernel_name(void);

/* Non-GEMM ops (ops.h:21-49), host pointers, FP32. */
void  qwen3_op_rmsnorm(float *out, const float *x, const uint16_t *w, int n);
void  qwen3_op_rope(float *v, int n_heads, int pos);
void  qwen3_op_softmax(float *x, int n);
void  qwen3_op_silu_mul(float *gate, const float *up, int n);
void  qwen3_op_residual_add(float *x, const float *y, int n);
int   qwen3_op_argmax(const float *v, int n);       /* lowest index on ties */
void  qwen3_op_bf16_to_f32(float *out, const uint16_t *in, int n);
float qwen3_op_dot(const float *a, const float *b, int n);
void  qwen3_op_axpy(float *y, float a, const float *x, int n);
const char *qwen3_ops_name(void);

/* Numerics of qwen3_gemm / qwen3_gemm_row: mode N550_MODE_EXACT with kblock
 * 16 or 32, or N550_MODE_FAST (kblock ignored). No counterpart in the
 * reference, where numerics are chosen at link time (Makefile:14-21). */
int n550_set_gemm_mode(int mode, int kblock);

/* Status of the last host-pointer call on this thread (N550_OK or an error). */
int n550_last_status(void);
const char *n550_strerror(int status);

/* ===========================================================================
 * 2. Device-pointer, stream-ordered API
 * ========================================================================= */

/* C = A . B^T with element strides lda/ldb/ldc.
 *   mode EXACT: a_type F32 (rounded to BF16 RNE on load, kernels_ame.c:235)
 *               or BF16; c_type F32; kblock 16 or 32; any M, N, K >= 0.
 *   mode FAST:  a_type BF16 (or F32, staged to BF16 RNE first); c_type F32 or
 *               BF16. Tensor-core path needs K % 8 == 0, lda/ldb % 8 == 0 and
 *               16-byte aligned A/B; other shapes take a CUDA-core kernel.
 * Replaces gemm_impl (kernels_ame.c:217-445) for device-resident operands. */
int n550_gemm(void *stream, int mode, int kblock,
              const void *a, int a_type, int lda,
              const uint16_t *b, int ldb,
              void *c, int c_type, int ldc,
              int M, int N, int K);

/* Fast-mode C = bf16_rne(A) . B^T for callers that cannot allocate device
 * memory: runtimes that keep the reference's no-malloc discipline (a fixed
 * arena sized up front, qwen3.h:39-58) and hosts that must not let a call
 * synchronise the device, as cudaMalloc/cudaFree do. It computes what
 * n550_gemm(MODE_FAST, a_type = N550_F32) computes, with the BF16 staging copy
 * of A held in a fixed 8 MiB array that this library places in every GPU
 * that loads it (for as long as the process lives) instead of a per-call
 * allocation. Routing: up to 8 rows the GEMV, then the weight-streaming GEMM
 * (FP32 output, up to 128 rows by default, n550_gemm_skinny_rows), otherwise
 * the tile GEMM in one pass -- n550_gemm's split-K route for BF16 output and
 * for 129-1023 rows is not taken (its partial sums would need a second
 * array), so those shapes run slower here than through n550_gemm. No
 * counterpart in the reference.
 *   Limit: M * round_up(K, 8) <= 4,194,304 (e.g. 4096 x 1024, 1365 x 3072);
 *   larger calls return N550_ERR_ARG and touch nothing.
 *   The first call on each device looks up the array's device address; make
 *   that first call before capturing the stream into a CUDA graph. The address
 *   is kept for the life of the process: after cudaDeviceReset (or a release
 *   of the device's primary context) this entry point must not be called.
 *   All calls share the one array: calls that can overlap on the GPU (other
 *   streams, other threads) race on it and must be serialised by the caller.
 *   c_type is N550_F32 or N550_BF16; other arguments as in n550_gemm. */
int n550_gemm_f32a_noalloc(void *stream, const float *a, int lda,
                           const uint16_t *b, int ldb, void *c, int c_type, int ldc,
                           int M, int N, int K);

/* Tile shape of the fast-mode tensor-core GEMMs: 128 or 256 output columns
 * per single-CTA 128-row tile, 512 for 256 x 256 tiles computed by 2-CTA
 * clusters (tcgen05 cta_group::2), or 0 for the automatic choice (default:
 * pairs for M >= 12288 and N >= 1024). A tuning knob for profiling; results do
 * not depend on it beyond FP32 summation order. */
int n550_gemm_tile_config(int bn);

/* The skinny-token GEMM of the decode step: weights as the MMA's 128-row side,
 * the M rows (tokens) as its N side, K split over a thread-block cluster whose
 * partial tiles are summed on chip, the residual / SwiGLU / q-k-v epilogues
 * fused. 0 (default): decoder layers with 9 <= M <= 32 rows (up to 8 take the
 * GEMVs) and FP32-output GEMMs (n550_gemm, qwen3_gemm) with M <= 128 rows
 * (n550_gemm_skinny_rows) take it;
 * 1-16: every M <= 512 takes it with that cluster size; -1: off
 * (such GEMMs split K into FP32 partials in global memory). A tuning knob;
 * results change only by FP32 summation order. */
int n550_gemm_skinny_config(int cs);

/* Largest M (0-512) that takes the skinny-token GEMM automatically
 * (n550_gemm_skinny_config 0): by default 32 for decoder layers and 128 for
 * FP32-output GEMMs; a call sets both to m. A tuning knob. */
int n550_gemm_skinny_rows(int m);

/* Programmatic dependent launch (default on): every kernel of the library is
 * launched so that it may start while the previous kernel of its stream
 * finishes -- its launch, barrier/TMEM setup and weight loads overlap that
 * kernel's tail, and it waits for the previous kernels' results before
 * touching them. 0 launches with plain stream order. Results are identical
 * either way; a profiling knob. Applies to launches made (and CUDA graphs
 * captured) after the call. */
int n550_set_pdl(int on);

/* Fused fast-mode GEMMs of the decoder layer (A BF16, weights BF16 [N,K]):
 *   n550_gemm_residual: x[M,N] += A . B^T in FP32 -- qwen3_gemm followed by
 *     qwen3_op_residual_add (qwen3.c:520-523, 540-543);
 *   n550_gemm_swiglu:  h[M,N] = bf16(silu(A . Wg^T) * (A . Wu^T)) -- the gate
 *     and up qwen3_gemm calls followed by qwen3_op_silu_mul (qwen3.c:531-537). */
int n550_gemm_residual(void *stream, const uint16_t *a, int lda, const uint16_t *b, int ldb,
                       float *x, int ldx, int M, int N, int K);
int n550_gemm_swiglu(void *stream, const uint16_t *a, int lda, const uint16_t *wg,
                     const uint16_t *wu, int ldw, uint16_t *h, int ldh, int M, int N, int K);

/* RoPE factor table of the fused q/k/v step: table[pos][i] = (cos, sin) of
 * pos * inv_freq[i] as FP32 pairs, pos < max_len, i < 64, inv_freq[i] =
 * 1 / powf(1e6, 2i / 128) as ops_scalar.c:24 computes it; table holds
 * max_len * 128 floats (8-byte aligned). */
int n550_rope_table(void *stream, float *table, int max_len);

/* One decoder layer's q/k/v step (qwen3.c:477-511): qkv = x . Wqkv^T with
 * Wqkv = [Wq; Wk; Wv] BF16 [4096, 1024] and x BF16 [M, ldx >= 1024]; then per
 * head the RMSNorm over 128 with q_norm / k_norm (qk_norm, qwen3.c:287-292),
 * RoPE of q and k at tok_pos[r] (ops_scalar.c:21-35, factors from
 * n550_rope_table), the 16 query heads to q_out (q_type F32 or BF16, [M, ldq
 * >= 2048]) and the 8 K and 8 V heads, rounded to BF16, to the caches at
 * [tok_seq[r]][layer][kv_head][tok_pos[r]][128] (planes of max_len
 * positions, 28 layers per sequence slot). Rows must name distinct (seq,
 * pos). Route as the runtime's: the tile GEMM with this epilogue from 1024
 * rows (BF16 q_out), the weight-streaming GEMM with it where
 * n550_gemm_skinny_rows admits M (4 rows on), else FP32 q/k/v rows (GEMV up
 * to 8 rows, split-K partials beyond, in a stream-ordered workspace) finished
 * by one row kernel. */
int n550_qkv_rope_kv(void *stream, const uint16_t *x, int ldx, const uint16_t *wqkv,
                     const uint16_t *q_norm, const uint16_t *k_norm, const float *rope_table,
                     const int32_t *tok_seq, const int32_t *tok_pos, int M,
                     void *q_out, int q_type, int ldq, uint16_t *k_cache, uint16_t *v_cache,
                     int max_len, int layer);

/* Row-wise RMSNorm: out[r] = x[r] * rsqrt(mean(x[r]^2) + eps) * w
 * (ops_scalar.c:11-15). out_type F32 or BF16. */
int n550_rmsnorm(void *stream, void *out, int out_type, const float *x,
                 const uint16_t *w, int rows, int n, float eps);

/* Rotate-half RoPE in place on rows of n_heads x 128 FP32, row r at position
 * pos0 + r, theta 1e6 (ops_scalar.c:21-35). */
int n550_rope(void *stream, float *v, int rows, int n_heads, int pos0);

/* gate = silu(gate) * up over n elements (ops_scalar.c:46-51). */
int n550_silu_mul(void *stream, float *gate, const float *up, size_t n);

/* Row-wise softmax in place (ops_scalar.c:37-44). */
int n550_softmax(void *stream, float *x, int rows, int n);

/* Row-wise argmax, first index of the maximum (ops_scalar.c:57-62):
 * idx[r] = argmax(v[r*ld .. r*ld+n)). */
int n550_argmax(void *stream, const float *v, int rows, int n, int ld, int32_t *idx);

/* x += y (ops_scalar.c:53-55); out = bf16 -> f32 (ops_scalar.c:64-66). */
int n550_residual_add(void *stream, float *x, const float *y, size_t n);
int n550_bf16_to_f32(void *stream, float *out, const uint16_t *in, size_t n);

/* Causal GQA attention (qwen3.c:374-436, which the reference inlines in
 * qwen3_forward_batch) over the BF16 KV cache, device pointers, stream-ordered.
 * 16 query heads share 8 KV heads (head h reads KV head h/2), head_dim 128,
 * scores scaled by 0.08838834764831845, softmax over positions 0..p.
 *   k_cache, v_cache  [n_slots][28 layers][8 kv heads][max_len][128] BF16;
 *                     sequence s reads slot seq_ids[s] (device int32 array)
 * Prefill: n_seqs x L queries at positions pos0 .. pos0+L-1, whose K/V are
 * already in the cache; q [n_seqs*L][ldq], out [n_seqs*L][ldo], head h at
 * columns h*128 .. h*128+127. tcgen05 tensor cores (P rounded to BF16).
 * Decode: one query per sequence at position pos[s] (device int32 array);
 * q [n_seqs][ldq], out [n_seqs][ldo]. workspace may be NULL (one CTA per
 * sequence and KV head) or n550_attention_decode_workspace(n_seqs, max_len)
 * bytes of device memory for split-KV partials. */
int n550_attention_prefill(void *stream, const uint16_t *q, int ldq, const uint16_t *k_cache,
                           const uint16_t *v_cache, int n_slots, int max_len, int layer,
                           const int32_t *seq_ids, int n_seqs, int L, int pos0, uint16_t *out,
                           int ldo);
int n550_attention_decode(void *stream, const uint16_t *q, int ldq, const uint16_t *k_cache,
                          const uint16_t *v_cache, int n_slots, int max_len, int layer,
                          const int32_t *seq_ids, const int32_t *pos, int n_seqs, uint16_t *out,
                          int ldo, void *workspace, size_t workspace_bytes);
size_t n550_attention_decode_workspace(int n_seqs, int max_len);

/* Device status word written by bounded waits inside kernels; returns it and
 * clears it (N550_OK, or N550_ERR_TIMEOUT). Synchronises the device. */
int n550_device_status(void);

/* Health check of the failure path: one warp waits `cycles` SM clock cycles
 * (1 .. 2e9) on an mbarrier that nothing arrives on, with both of the
 * library's bounded waits in turn (the polling one and the one whose tries
 * sleep); each gives up, records N550_ERR_TIMEOUT in the device status word
 * and the kernel returns, leaving the context usable. Enqueued
 * on `stream`; read the result with n550_device_status(). No counterpart in
 * the reference. */
int n550_check_wait_expiry(void *stream, long long cycles);

/* ===========================================================================
 * 3. Model runtime (qwen3.h:203-257 re-designed for HBM): weights, KV cache
 *    and activations live on one GPU; many independent sequences share it.
 * ========================================================================= */
typedef struct n550_model n550_model_t;

typedef struct {
    int    max_seqs;     /* sequences with their own KV cache              */
    int    max_len;      /* positions per sequence (QWEN3_MAX_SEQ)          */
    int    max_tokens;   /* tokens per forward call (activation capacity)   */
    int    gemm_mode;    /* N550_MODE_FAST or N550_MODE_EXACT               */
    int    kblock;       /* exact-mode K-block (16 or 32)                   */
} n550_model_config;

/* Parses a QW3M blob in host memory (qwen3.c:87-146: same header checks and
 * error codes) and uploads it to the current device. */
int n550_qwen3_init(n550_model_t **out, const void *blob, size_t blob_size,
                    const n550_model_config *cfg);

/* Random-init weights generated on the device: linear weights from the
 * seeded integer generator (approximately N(0, sigma^2)), norms 1.0;
 * bit-identical to the same seed written as a QW3M blob. */
int n550_qwen3_init_random(n550_model_t **out, uint64_t seed, double sigma,
                           const n550_model_config *cfg);

void n550_qwen3_free(n550_model_t *m);

/* Batched prefill: n_seqs sequences of seq_len tokens each, tokens
 * [n_seqs][seq_len] and seq_ids [n_seqs] (KV slots) in device memory, all at
 * positions pos0..pos0+seq_len-1. Writes last-token logits [n_seqs][151936]
 * FP32 (may be NULL) and their argmax [n_seqs] (may be NULL).
 * qwen3_forward_batch (qwen3.c:455-576) generalised to many sequences. */
int n550_qwen3_prefill(n550_model_t *m, void *stream, const int32_t *tokens,
                       const int32_t *seq_ids, int n_seqs, int seq_len, int pos0,
                       float *logits, int32_t *next_token);

/* One decode step for n_seqs sequences: token[i] at position pos[i] of
 * sequence seq_ids[i] (device arrays). Greedy next token -> next_token[i];
 * logits [n_seqs][151936] optional. qwen3_forward + qwen3_argmax
 * (qwen3.c:578-584) generalised to many sequences. */
int n550_qwen3_decode(n550_model_t *m, void *stream, const int32_t *tokens,
                      const int32_t *seq_ids, const int32_t *pos, int n_seqs,
                      float *logits, int32_t *next_token);

/* `steps` greedy decode steps (the generation loop of main.c:240-256 for many
 * sequences): step i feeds tokens[s] at pos[s], writes the argmax to
 * out_ids[i * n_seqs + s], then sets tokens[s] = that id and pos[s] += 1 on
 * the device (tokens and pos are advanced in place). use_graph = 1 captures
 * one step (all its kernels) into a CUDA graph on first use and replays it
 * (one launch per step); the capture is rebuilt when n_seqs or a pointer
 * changes. Do not call it while the stream is being captured. */
int n550_qwen3_decode_steps(n550_model_t *m, void *stream, int32_t *tokens,
                            const int32_t *seq_ids, int32_t *pos, int n_seqs, int steps,
                            int32_t *out_ids, int use_graph);

/* Reference-shaped convenience on sequence slot 0 with HOST buffers:
 * tokens[n_token] at pos0.., last-token logits copied to logits_host
 * (151936 floats, may be NULL); returns the argmax (>= 0) or an error (< 0). */
int n550_qwen3_forward_batch_host(n550_model_t *m, const int32_t *tokens,
                                  int n_token, int pos0, float *logits_host);

/* Token count (9..1024, default 1024) from which the runtime's decoder layers
 * take whole-tile GEMMs with fused epilogues instead of split-K partial sums
 * finished by row kernels. A tuning knob; results do not depend on it beyond
 * FP32 summation order. */
int n550_qwen3_split_rows(int rows);

/* Decode steps that take the split-K or GEMV q/k/v route: the decode attention
 * kernel applies QK-norm and RoPE to the raw q/k/v rows and writes the new K/V
 * itself (1, default) or a separate row kernel does (0). Bit-identical
 * results either way. */
int n550_qwen3_fused_attention_prep(int on);

/* Decode steps of 1-4 sequences as one persistent kernel (1) or as the
 * per-layer kernel sequence (0, the default: measured faster on B200). The
 * persistent kernel runs the 28 layers on one CTA per SM, separated by bounded
 * grid barriers, with the next phase's weights streamed into shared memory
 * ahead of use (contexts up to 8192 positions). Results agree within FP32
 * summation order. */
int n550_qwen3_fused_decode(int on);

/* Per-op tensor dump (qwen3_set_dump / EMIT, qwen3.h:169-184, qwen3.c:464-575):
 * while fn is set, n550_qwen3_forward_batch_host runs the forward op by op with
 * every intermediate tensor materialised and calls fn(ctx, layer, name, data,
 * n) with an FP32 host copy of each, under the reference's names and in its
 * order ("embed_out", per layer "input_layernorm_out" ... "layer_out",
 * "final_norm_out", "logits"; layer -1 outside the layers). A debugging route
 * for locating numerical drift against the reference's own dump; it
 * allocates its buffers and synchronises per tensor. NULL turns it off. */
typedef void (*n550_dump_fn)(void *ctx, int layer, const char *name, const float *data, size_t n);
int n550_qwen3_set_dump(n550_model_t *m, n550_dump_fn fn, void *ctx);

/* The configuration a model was created with. */
int n550_qwen3_get_config(const n550_model_t *m, n550_model_config *cfg);

/* Most tokens per n550_qwen3_forward_rows call: QWEN3_SPEC_BATCH =
 * QWEN3_MAX_BATCH (qwen3.h:82-88, 145-146). */
#define N550_ROWS_MAX 128

/* One sequence's n_token (1..N550_ROWS_MAX) tokens at positions
 * pos0..pos0+n_token-1 of KV slot *seq_id (device int32), with the logits of
 * EVERY row (qwen3_forward_batch built with QWEN3_SPECULATIVE, qwen3.c:556-566:
 * row j's logits are the prediction after tokens[0..j]): logits
 * [n_token][151936] FP32 (may be NULL) and their argmax next_ids[n_token]
 * (may be NULL, not both). Device buffers, stream-ordered. */
int n550_qwen3_forward_rows(n550_model_t *m, void *stream, const int32_t *tokens,
                            const int32_t *seq_id, int n_token, int pos0, float *logits,
                            int32_t *next_ids);

/* The same on sequence slot 0 with HOST buffers (synchronous): next_ids_host
 * [n_token] receives every row's argmax, logits_host [n_token][151936] every
 * row's logits (may be NULL). Requires n_token <= the model's max_tokens. */
int n550_qwen3_forward_rows_host(n550_model_t *m, const int32_t *tokens, int n_token, int pos0,
                                 int32_t *next_ids_host, float *logits_host);

/* Prompt-lookup drafting (lookup_draft, main_baremetal.c:567-584): the last
 * `ngram` tokens of hist[n_hist] are searched for earlier in hist, newest
 * match first; the up to max_k tokens that followed the match go to draft.
 * Returns how many (0 when there is no match), or N550_ERR_ARG. */
int n550_lookup_draft(const int32_t *hist, int n_hist, int ngram, int32_t *draft, int max_k);

typedef struct {
    int64_t rounds;      /* forward_rows calls after the prefill              */
    int64_t drafted;     /* draft tokens proposed                             */
    int64_t accepted;    /* draft tokens equal to the model's own choice      */
} n550_spec_stats;

/* Greedy generation with prompt-lookup speculative verification (the
 * QWEN3_SPECULATIVE chat loop, main_baremetal.c:636-690) on sequence slot 0:
 * prefill the prompt (n_prompt <= max_tokens) at position 0, then per round
 * feed [next, draft...] (max_draft <= 127 drafts from n550_lookup_draft with
 * `ngram`) through n550_qwen3_forward_rows and keep the drafts up to the first
 * one that differs from the model's argmax. Stops after max_new tokens, at
 * the end of the KV cache, or when the next token is one of eos[n_eos] (not
 * emitted). out[max_new] receives the tokens, *n_out their count. With
 * max_draft = 0 it is plain greedy decoding. */
int n550_qwen3_generate_lookup(n550_model_t *m, const int32_t *prompt, int n_prompt, int max_new,
                               int max_draft, int ngram, const int32_t *eos, int n_eos,
                               int32_t *out, int *n_out, n550_spec_stats *stats);

/* Seeded synthetic token ids (the benchmark's inputs), host memory:
 * out[i] = u64(seed, stream, i) mod vocab with the generator of
 * n550_qwen3_init_random. No counterpart in the reference (its prompts come
 * from the tokenizer, which needs the unshipped tokenizer.bin). */
int n550_synth_tokens(int32_t *out, size_t n, uint64_t seed, uint64_t stream, int vocab);

/* Seeded synthetic BF16 values (the benchmark's GEMM operands), host memory:
 * out[i] = bf16_rne(normal(sigma)) of u64(seed, stream, i), the generator
 * n550_qwen3_init_random fills the weights with. No counterpart in the
 * reference. */
int n550_synth_normal_bf16(uint16_t *out, size_t n, uint64_t seed, uint64_t stream, double sigma);

/* Device buffers of one weight tensor, for tests: which = 0 embed,
 * 1 + 11*l + j for layer l tensor j in QW3M order, 309 final norm.
 * Returns a device pointer to the BF16 data in QW3M [out,in] order, or NULL. */
const uint16_t *n550_qwen3_weight(const n550_model_t *m, int which, size_t *elems);

/* Kernel-time accounting of one model, for benchmarks: while enabled, every
 * kernel the runtime launches is counted and bracketed by CUDA events on its
 * stream, accumulated per kind below. enable = 1 resets and starts, 0 stops.
 * n550_qwen3_profile_read synchronises, then fills ms[k] (device time) and
 * launches[k] for k < n_kinds. No counterpart in the reference (its only
 * instrumentation is the mcycle timing of main_baremetal.c:636,733-754). */
enum {
    N550_PROF_GEMM_QKV = 0, N550_PROF_GEMM_O, N550_PROF_GEMM_GATEUP, N550_PROF_GEMM_DOWN,
    N550_PROF_GEMM_LMHEAD, N550_PROF_ATTN, N550_PROF_QKNORM_ROPE, N550_PROF_RMSNORM,
    N550_PROF_OTHER, N550_PROF_KINDS
};
int n550_qwen3_profile(n550_model_t *m, int enable);
int n550_qwen3_profile_read(n550_model_t *m, double *ms, int64_t *launches, int n_kinds);

/* ===========================================================================
 * 4. Tokenizer and chat template (tokenizer.h, main.c:124-185): host code.
 * ========================================================================= */
typedef struct n550_tok n550_tok_t;

/* Error codes of the tokenizer (QWEN3_TOK_ERR_*, tokenizer.h:47-54). */
#define N550_TOK_ERR_MAGIC    (-1)
#define N550_TOK_ERR_VERSION  (-2)
#define N550_TOK_ERR_SIZE     (-3)
#define N550_TOK_ERR_OVERFLOW (-5)

/* Loads a QW3T v1 vocabulary (the reference's tok.bin: byte-level BPE
 * vocabulary, ranked merges, Unicode letter/digit ranges, special tokens;
 * qwen3_tok_init, tokenizer.c:65-110) from host memory; the bytes are copied.
 * Returns N550_OK or an N550_TOK_ERR_* code. */
int n550_tok_init(n550_tok_t **out, const void *blob, size_t size);
void n550_tok_free(n550_tok_t *t);
int n550_tok_vocab_size(const n550_tok_t *t);

/* UTF-8 text -> token ids (qwen3_tok_encode, tokenizer.c:313-345): special
 * tokens matched whole, the rest split by the GPT-style pre-tokenizer and
 * byte-level BPE. Returns the count, or N550_TOK_ERR_OVERFLOW when more than
 * max_out ids (or a piece longer than 2048 bytes) would result. */
int n550_tok_encode(const n550_tok_t *t, const char *text, size_t len, int32_t *out, int max_out);

/* Token ids -> bytes, '\0'-terminated (qwen3_tok_decode, tokenizer.c:347-358).
 * Returns the bytes written (without the '\0') or N550_TOK_ERR_OVERFLOW.
 * Ids outside the vocabulary decode to nothing. */
int n550_tok_decode(const n550_tok_t *t, const int32_t *ids, int n, char *out, size_t max_out);

/* The bytes of one token (qwen3_tok_piece), for streaming output. */
const uint8_t *n550_tok_piece(const n550_tok_t *t, int id, size_t *len);

/* Many texts at once on up to n_threads host threads (0: all cores): text i
 * -> out[i * max_out ..], counts[i] its id count. The prompts of a
 * data-parallel batch. No counterpart in the reference (one prompt at a time). */
int n550_tok_encode_batch(const n550_tok_t *t, const char *const *texts, const size_t *lens,
                          int n_texts, int32_t *out, int max_out, int32_t *counts, int n_threads);

/* A user turn in Qwen3's chat template with thinking disabled
 * (main.c:124-131): "<|im_start|>user\n" prompt
 * "<|im_end|>\n<|im_start|>assistant\n<think>\n\n</think>\n\n", encoded. */
int n550_chat_encode(const n550_tok_t *t, const char *prompt, size_t len, int32_t *out, int max_out);

/* Chat end to end (chat_mode, main.c:137-185; with max_draft > 0 the
 * speculative loop of main_baremetal.c:636-690): the prompt in the chat
 * template (n550_chat_encode, at most max_tokens ids) on sequence slot 0 from
 * position 0, up to max_new greedy tokens until an EOS (151645, 151643) or
 * the end of the KV cache, ids[max_new] and *n_ids, and their text in
 * text[max_text] ('\0'-terminated). Returns the text's length or an error. */
int n550_qwen3_chat(n550_model_t *m, const n550_tok_t *tok, const char *prompt, size_t len,
                    int max_new, int max_draft, char *text, size_t max_text, int32_t *ids,
                    int *n_ids);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif
#endif /* N550_QWEN3_H */
