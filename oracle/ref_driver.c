/* Thin driver around the reference runtime, compiled together with the
 * reference's own sources (qwen3.c + kernels_*.c + ops_scalar.c, built where
 * they lie by oracle/Makefile) into oracle/_ref/libref_<kernel>.so.
 * TEST INFRASTRUCTURE ONLY: gives tests a handle-free C entry into
 * qwen3_init / qwen3_forward_batch / qwen3_last_logits (qwen3.h:206-245).
 */
#include <stdlib.h>

#include "kernels.h"
#include "ops.h"
#include "qwen3.h"

static qwen3_t g_model;
static void   *g_scratch;

int ref_model_init(const void *blob, size_t size) {
    if (!g_scratch) g_scratch = malloc(qwen3_scratch_bytes());
    if (!g_scratch) return QWEN3_ERR_OOM;
    return qwen3_init(&g_model, blob, size, g_scratch, qwen3_scratch_bytes());
}

void ref_forward_batch(const int *tokens, int n_token, int pos0) {
    qwen3_forward_batch(&g_model, tokens, n_token, pos0);
}

const float *ref_logits(void) { return qwen3_last_logits(&g_model); }

/* Rows of logits the last call left: all rows of a call of up to
 * QWEN3_SPEC_BATCH tokens in a QWEN3_SPECULATIVE build (qwen3.c:556-566),
 * otherwise the last row only. */
int ref_n_logits(void) { return g_model.s.n_logits; }

const float *ref_logits_row(int i) { return qwen3_logits_at(&g_model, i); }

int ref_max_seq(void) { return QWEN3_MAX_SEQ; }

/* The reference's per-op dump (qwen3_set_dump, qwen3.c:238-247): fn receives
 * every EMIT point of the following forward calls; NULL turns it off. */
void ref_set_dump(qwen3_dump_fn fn, void *ctx) { qwen3_set_dump(&g_model, fn, ctx); }

const char *ref_kernel_name(void) { return qwen3_kernel_name(); }
