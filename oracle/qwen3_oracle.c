/* CPU oracle: Qwen3-0.6B forward -- TEST INFRASTRUCTURE ONLY (see oracle.h).
 *
 * Restates qwen3_init's tensor slicing (fpga_bringup/src/src/qwen3.c:87-146)
 * and qwen3_forward_batch (qwen3.c:455-576) with the default (non-QWEN3_OPT)
 * attention (qwen3.c:374-436), op for op and in the same order, so that with
 * the scalar GEMM it is bit-identical to the reference compiled in
 * oracle/_ref. The GEMM is selectable: scalar (kernels_scalar.c), hwsim
 * (kernels_hwsim.c) or the AME exact rule at K-block 16/32.
 * KV cache: FP32 [layer][kv_head][pos][head_dim] (qwen3.h:62-76).
 */
#include <stdlib.h>
#include <string.h>

#include "oracle.h"

#define H       1024
#define IN      3072
#define NL      28
#define NH      16
#define NKV     8
#define HD      128
#define VOCAB   151936
#define QD      (NH * HD)
#define KVD     (NKV * HD)
#define GROUP   2
#define MAXB    128
#define ATTN_SCALE 0.08838834764831845f

typedef struct {
    const uint16_t *ln1, *wq, *wk, *wv, *qn, *kn, *wo, *ln2, *wg, *wu, *wd;
} layer_w;

struct oracle_model {
    const uint16_t *embed, *final_norm;
    layer_w L[NL];
    int max_seq, gemm_kind;
    float *x, *xb, *xb2, *q, *k, *v, *attn_out, *att, *hb, *hb2, *logits;
    float *kc, *vc;
};

static int32_t rd_i32(const uint8_t *p) {
    return (int32_t)((uint32_t)p[0] | ((uint32_t)p[1] << 8) |
                     ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24));
}

typedef struct { const uint8_t *base; size_t size, pos, align; int err; } cur_t;

static const uint16_t *take(cur_t *c, size_t n) {
    if (c->err) return NULL;
    size_t p = (c->pos + c->align - 1) & ~(c->align - 1);
    if (p + n * 2 > c->size) { c->err = -5; return NULL; }
    c->pos = p + n * 2;
    return (const uint16_t *)(c->base + p);
}

void oracle_model_destroy(oracle_model_t *m) {
    if (!m) return;
    free(m->x); free(m->xb); free(m->xb2); free(m->q); free(m->k); free(m->v);
    free(m->attn_out); free(m->att); free(m->hb); free(m->hb2); free(m->logits);
    free(m->kc); free(m->vc);
    free(m);
}

oracle_model_t *oracle_model_create(const uint8_t *b, size_t size, int max_seq,
                                    int gemm_kind, int *err) {
    *err = 0;
    if (size < 256 || memcmp(b, "QW3M", 4) != 0) { *err = -1; return NULL; }
    if (rd_i32(b + 4) != 1) { *err = -2; return NULL; }
    if (rd_i32(b + 44) != 1) { *err = -3; return NULL; }
    if (rd_i32(b + 8) != H || rd_i32(b + 12) != IN || rd_i32(b + 16) != NL ||
        rd_i32(b + 20) != NH || rd_i32(b + 24) != NKV || rd_i32(b + 28) != HD ||
        rd_i32(b + 32) != VOCAB) { *err = -4; return NULL; }
    const int align = rd_i32(b + 72);
    if (align < 128 || (align & (align - 1))) { *err = -4; return NULL; }
    if (rd_i32(b + 76) != 0) { *err = -7; return NULL; }

    oracle_model_t *m = (oracle_model_t *)calloc(1, sizeof *m);
    if (!m) { *err = -6; return NULL; }
    cur_t c = { b, size, (size_t)rd_i32(b + 68), (size_t)align, 0 };
    m->embed = take(&c, (size_t)VOCAB * H);
    for (int l = 0; l < NL; l++) {
        layer_w *w = &m->L[l];
        w->ln1 = take(&c, H);
        w->wq = take(&c, (size_t)QD * H);
        w->wk = take(&c, (size_t)KVD * H);
        w->wv = take(&c, (size_t)KVD * H);
        w->qn = take(&c, HD);
        w->kn = take(&c, HD);
        w->wo = take(&c, (size_t)H * QD);
        w->ln2 = take(&c, H);
        w->wg = take(&c, (size_t)IN * H);
        w->wu = take(&c, (size_t)IN * H);
        w->wd = take(&c, (size_t)H * IN);
    }
    m->final_norm = take(&c, H);
    if (c.err || c.pos != size) { *err = -5; oracle_model_destroy(m); return NULL; }

    m->max_seq = max_seq;
    m->gemm_kind = gemm_kind;
    m->x = malloc(sizeof(float) * MAXB * H);
    m->xb = malloc(sizeof(float) * MAXB * H);
    m->xb2 = malloc(sizeof(float) * MAXB * H);
    m->q = malloc(sizeof(float) * MAXB * QD);
    m->k = malloc(sizeof(float) * MAXB * KVD);
    m->v = malloc(sizeof(float) * MAXB * KVD);
    m->attn_out = malloc(sizeof(float) * MAXB * QD);
    m->att = malloc(sizeof(float) * NH * (size_t)max_seq);
    m->hb = malloc(sizeof(float) * MAXB * IN);
    m->hb2 = malloc(sizeof(float) * MAXB * IN);
    m->logits = malloc(sizeof(float) * VOCAB);
    m->kc = calloc((size_t)NL * max_seq * KVD, sizeof(float));
    m->vc = calloc((size_t)NL * max_seq * KVD, sizeof(float));
    if (!m->x || !m->xb || !m->xb2 || !m->q || !m->k || !m->v || !m->attn_out ||
        !m->att || !m->hb || !m->hb2 || !m->logits || !m->kc || !m->vc) {
        *err = -6; oracle_model_destroy(m); return NULL;
    }
    return m;
}

static void gemm(const oracle_model_t *m, float *c, const float *a,
                 const uint16_t *b, int M, int K, int N) {
    switch (m->gemm_kind) {
    case ORACLE_GEMM_HWSIM:   oracle_gemm_hwsim(c, a, b, M, K, N); break;
    case ORACLE_GEMM_EXACT16: oracle_gemm_ame_exact_f32a(c, a, b, M, K, N, 16); break;
    case ORACLE_GEMM_EXACT32: oracle_gemm_ame_exact_f32a(c, a, b, M, K, N, 32); break;
    default:                  oracle_gemm_scalar(c, a, b, M, K, N); break;
    }
}

static size_t kv_off(const oracle_model_t *m, int layer, int kvh, int pos) {
    return (size_t)layer * NKV * m->max_seq * HD + (size_t)kvh * m->max_seq * HD
         + (size_t)pos * HD;
}

static void qk_norm(float *v, const uint16_t *w, int n_heads) {
    for (int h = 0; h < n_heads; h++) {
        float *p = v + (size_t)h * HD;
        oracle_op_rmsnorm(p, p, w, HD);
    }
}

static void attention(oracle_model_t *m, int layer, int n_token, int pos0) {
    for (int i = 0; i < n_token; i++) {
        const int pos = pos0 + i;
        const float *qrow = m->q + (size_t)i * QD;
        float *orow = m->attn_out + (size_t)i * QD;
        for (int kvh = 0; kvh < NKV; kvh++) {
            const int h0 = kvh * GROUP;
            for (int t = 0; t <= pos; t++) {
                const float *kh = m->kc + kv_off(m, layer, kvh, t);
                for (int g = 0; g < GROUP; g++) {
                    const int h = h0 + g;
                    m->att[(size_t)h * m->max_seq + t] =
                        oracle_op_dot(qrow + (size_t)h * HD, kh, HD) * ATTN_SCALE;
                }
            }
            for (int g = 0; g < GROUP; g++) {
                const int h = h0 + g;
                oracle_op_softmax(m->att + (size_t)h * m->max_seq, pos + 1);
                memset(orow + (size_t)h * HD, 0, HD * sizeof(float));
            }
            for (int t = 0; t <= pos; t++) {
                const float *vh = m->vc + kv_off(m, layer, kvh, t);
                for (int g = 0; g < GROUP; g++) {
                    const int h = h0 + g;
                    oracle_op_axpy(orow + (size_t)h * HD,
                                   m->att[(size_t)h * m->max_seq + t], vh, HD);
                }
            }
        }
    }
}

int oracle_model_forward_batch(oracle_model_t *m, const int32_t *tokens,
                               int n_token, int pos0) {
    const int NT = n_token;
    if (NT <= 0 || NT > MAXB || pos0 < 0 || pos0 + NT > m->max_seq) return -1;
    for (int t = 0; t < NT; t++)
        oracle_op_bf16_to_f32(m->x + (size_t)t * H, m->embed + (size_t)tokens[t] * H, H);

    for (int l = 0; l < NL; l++) {
        const layer_w *w = &m->L[l];
        for (int r = 0; r < NT; r++)
            oracle_op_rmsnorm(m->xb + (size_t)r * H, m->x + (size_t)r * H, w->ln1, H);
        gemm(m, m->q, m->xb, w->wq, NT, H, QD);
        for (int r = 0; r < NT; r++) qk_norm(m->q + (size_t)r * QD, w->qn, NH);
        gemm(m, m->k, m->xb, w->wk, NT, H, KVD);
        for (int r = 0; r < NT; r++) qk_norm(m->k + (size_t)r * KVD, w->kn, NKV);
        gemm(m, m->v, m->xb, w->wv, NT, H, KVD);
        for (int r = 0; r < NT; r++) oracle_op_rope(m->q + (size_t)r * QD, NH, pos0 + r);
        for (int r = 0; r < NT; r++) oracle_op_rope(m->k + (size_t)r * KVD, NKV, pos0 + r);
        for (int t = 0; t < NT; t++)
            for (int kvh = 0; kvh < NKV; kvh++) {
                const size_t dst = kv_off(m, l, kvh, pos0 + t);
                const size_t src = (size_t)t * KVD + (size_t)kvh * HD;
                memcpy(m->kc + dst, m->k + src, HD * sizeof(float));
                memcpy(m->vc + dst, m->v + src, HD * sizeof(float));
            }
        attention(m, l, NT, pos0);
        gemm(m, m->xb2, m->attn_out, w->wo, NT, QD, H);
        for (int r = 0; r < NT; r++)
            oracle_op_residual_add(m->x + (size_t)r * H, m->xb2 + (size_t)r * H, H);
        for (int r = 0; r < NT; r++)
            oracle_op_rmsnorm(m->xb + (size_t)r * H, m->x + (size_t)r * H, w->ln2, H);
        gemm(m, m->hb, m->xb, w->wg, NT, H, IN);
        gemm(m, m->hb2, m->xb, w->wu, NT, H, IN);
        oracle_op_silu_mul(m->hb, m->hb2, NT * IN);
        gemm(m, m->xb2, m->hb, w->wd, NT, IN, H);
        oracle_op_residual_add(m->x, m->xb2, NT * H);
    }
    for (int r = 0; r < NT; r++)
        oracle_op_rmsnorm(m->x + (size_t)r * H, m->x + (size_t)r * H, m->final_norm, H);
    gemm(m, m->logits, m->x + (size_t)(NT - 1) * H, m->embed, 1, H, VOCAB);
    return 0;
}

const float *oracle_model_logits(const oracle_model_t *m) { return m->logits; }
