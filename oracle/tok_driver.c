/* Thin driver around the reference's own tokenizer.c, compiled together with
 * it (where it lies) into oracle/_ref/libref_tok.so by oracle/Makefile.
 * TEST INFRASTRUCTURE ONLY: a handle-free C entry into qwen3_tok_init /
 * qwen3_tok_encode / qwen3_tok_decode (tokenizer.h:56-77) for the tests that
 * check this project's tokenizer against it. The blob must stay alive while
 * the tokenizer is used (the reference borrows it).
 */
#include <stdlib.h>

#include "tokenizer.h"

static qwen3_tok_t g_tok;
static void       *g_htab;

int ref_tok_init(const void *blob, size_t size) {
    if (!g_htab) g_htab = malloc(qwen3_tok_scratch_bytes());
    if (!g_htab) return QWEN3_TOK_ERR_OOM;
    return qwen3_tok_init(&g_tok, blob, size, g_htab, qwen3_tok_scratch_bytes());
}

int ref_tok_encode(const char *text, size_t len, int *out, int max_out) {
    return qwen3_tok_encode(&g_tok, text, len, out, max_out);
}

int ref_tok_decode(const int *ids, int n, char *out, size_t max_out) {
    return qwen3_tok_decode(&g_tok, ids, n, out, max_out);
}
