/* CPU oracle for the n550 Qwen3 hot path -- TEST INFRASTRUCTURE ONLY.
 *
 * This library restates, in plain C, the reference algorithms that the
 * B200 kernels must reproduce. It is linked by tests/, by
 * __graft_entry__.smoke() and by bench.py's cpu_baseline leg, always as the
 * checker or the timed CPU baseline, never as the product path. The product
 * (n550_qwen3_bringup_handover_b200/csrc) never links or calls it.
 *
 * Parity pin: the AME exact GEMM below reproduces every c_ref.bin / c_peak.bin
 * of the 12 shipped AME golden cases bit-exactly at K-block 16
 * (rtl_verification/cases/*, checked by tests/test_oracle_golden.py), and the
 * forward restatement matches the reference's own qwen3.c compiled into
 * oracle/_ref/ bit-for-bit (tests/test_oracle_ref.py).
 */
#ifndef N550_ORACLE_H
#define N550_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- BF16 <-> FP32 (reference: qwen3.h:24-37, kernels_hwsim.c:45-51) ---- */
float    oracle_bf16_to_f32(uint16_t b);
uint16_t oracle_f32_to_bf16_rne(float f);
void     oracle_f32_to_bf16_array(uint16_t *out, const float *in, size_t n);

/* ---- GEMMs: C[M,N] = A[M,K] . B[N,K]^T, row-major with element strides ---- */

/* AME golden semantics (rtl_verification/golden_src/40_gen_ame_vectors.py:103-143):
 * per K-block the exact rational sum of acc + the block's bf16 x bf16
 * products, rounded to binary64 (RNE) and then to binary32 (RNE).
 * kblock is 16 (what the shipped vectors pin) or 32 (the generator as shipped).
 * c_bits receives FP32 bit patterns; peak (may be NULL) receives
 * max over blocks of |acc| after each rounding (the c_peak.bin definition).
 * Non-finite inputs are unpinned by the reference; they are summed in IEEE
 * binary64 and rounded to binary32. Returns 0, or -1 for bad arguments. */
int oracle_gemm_ame_exact(uint32_t *c_bits, int ldc, float *peak,
                          const uint16_t *a, int lda,
                          const uint16_t *b, int ldb,
                          int M, int N, int K, int kblock);

/* Same, with FP32 activations rounded to BF16 RNE first (kernels_ame.c:220-236). */
int oracle_gemm_ame_exact_f32a(float *c, const float *a, const uint16_t *b,
                               int M, int K, int N, int kblock);

/* kernels_hwsim.c:56-79 -- RNE staging of A, double sum per 16-block. */
void oracle_gemm_hwsim(float *c, const float *a, const uint16_t *b,
                       int M, int K, int N);

/* kernels_scalar.c:9-21 -- FP32 sequential sum, A not rounded. */
void oracle_gemm_scalar(float *c, const float *a, const uint16_t *b,
                        int M, int K, int N);

/* test_kernels.c:19-29 -- double-precision reference (the unit test's gemm_ref). */
void oracle_gemm_f64(float *c, const float *a, const uint16_t *b,
                     int M, int K, int N);

/* ---- non-GEMM ops (ops_scalar.c:11-78) ---- */
void  oracle_op_rmsnorm(float *out, const float *x, const uint16_t *w, int n);
void  oracle_op_rope(float *v, int n_heads, int pos);
void  oracle_op_softmax(float *x, int n);
void  oracle_op_silu_mul(float *gate, const float *up, int n);
void  oracle_op_residual_add(float *x, const float *y, int n);
int   oracle_op_argmax(const float *v, int n);
void  oracle_op_bf16_to_f32(float *out, const uint16_t *in, int n);
float oracle_op_dot(const float *a, const float *b, int n);
void  oracle_op_axpy(float *y, float a, const float *x, int n);

/* ---- seeded synthetic data (shared definition with the product's generator) ----
 * u64(seed, stream, i) = splitmix64(key + i*0xD1B54A32D192ED03),
 * key = splitmix64(seed ^ splitmix64(stream)).
 * normal: four 16-bit lanes of u64 summed (Irwin-Hall n=4), centred, times
 * sigma*sqrt(3)/65536 in FP32 -- an integer-exact approximation of N(0, sigma^2)
 * that the GPU reproduces bit-for-bit (no transcendental functions). */
uint64_t oracle_synth_u64(uint64_t seed, uint64_t stream, uint64_t i);
float    oracle_synth_normal_scale(double sigma);
void     oracle_synth_normal_bf16(uint16_t *out, size_t n, uint64_t seed,
                                  uint64_t stream, double sigma);
void     oracle_synth_normal_f32(float *out, size_t n, uint64_t seed,
                                 uint64_t stream, double sigma);
void     oracle_synth_tokens(int32_t *out, size_t n, uint64_t seed,
                             uint64_t stream, int vocab);

/* ---- QW3M weight blob (qwen3_config.h:41-81, qwen3.c:87-146) ---- */
size_t oracle_qw3m_size(void);            /* 1,192,100,096 for the row layout */
/* Writes a complete random-init row-layout blob: linear weights
 * ~N(0, sigma^2) (stream = tensor index in file order), norm weights 1.0. */
int    oracle_qw3m_write(uint8_t *blob, size_t size, uint64_t seed, double sigma);

/* ---- forward restatement (qwen3.c:455-584, non-OPT attention :374-436) ---- */
enum { ORACLE_GEMM_SCALAR = 0, ORACLE_GEMM_HWSIM = 1,
       ORACLE_GEMM_EXACT16 = 2, ORACLE_GEMM_EXACT32 = 3 };
typedef struct oracle_model oracle_model_t;
oracle_model_t *oracle_model_create(const uint8_t *blob, size_t size,
                                    int max_seq, int gemm_kind, int *err);
void  oracle_model_destroy(oracle_model_t *m);
/* n_token <= 128 (QWEN3_MAX_BATCH); logits of the last token only. */
int   oracle_model_forward_batch(oracle_model_t *m, const int32_t *tokens,
                                 int n_token, int pos0);
const float *oracle_model_logits(const oracle_model_t *m);

#ifdef __cplusplus
}
#endif
#endif
