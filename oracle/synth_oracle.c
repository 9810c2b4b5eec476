/* CPU oracle: seeded synthetic inputs and the random-init QW3M blob --
 * TEST INFRASTRUCTURE ONLY (see oracle.h).
 *
 * The generator is this project's own definition (the reference ships no
 * weights: fpga_bringup/L2_L3_fullmodel/GET_WEIGHTS.md); the product's device
 * generator (csrc/synth.cuh) implements the same integer-exact formula, and
 * tests compare the two bit-for-bit.
 *
 * The blob layout restates the exporter contract the reference parses:
 * 256-byte header (qwen3_config.h:41-62, plus the layout word at +76 and tile
 * sizes at +80/+84 read by qwen3.c:114-116), then the 310 tensors in the
 * order of qwen3_config.h:64-81, each aligned to 128 bytes (qwen3.c:75-85).
 */
#define _GNU_SOURCE
#include <math.h>
#include <pthread.h>
#include <string.h>
#include <unistd.h>

#include "oracle.h"

#define HIDDEN  1024
#define INTER   3072
#define LAYERS  28
#define NHEADS  16
#define NKV     8
#define HDIM    128
#define VOCAB   151936
#define QDIM    (NHEADS * HDIM)
#define KVDIM   (NKV * HDIM)

static uint64_t smix(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

uint64_t oracle_synth_u64(uint64_t seed, uint64_t stream, uint64_t i) {
    const uint64_t key = smix(seed ^ smix(stream));
    return smix(key + i * 0xD1B54A32D192ED03ull);
}

float oracle_synth_normal_scale(double sigma) {
    return (float)(sigma * 1.7320508075688772 / 65536.0);
}

static float synth_normal_one(uint64_t r, float scale) {
    const int s = (int)(r & 0xFFFF) + (int)((r >> 16) & 0xFFFF)
                + (int)((r >> 32) & 0xFFFF) + (int)(r >> 48);
    return (float)(s - 131070) * scale;
}

typedef struct { uint16_t *out; size_t lo, hi; uint64_t key; float sc; } bf16_job;

static void *bf16_worker(void *p) {
    const bf16_job *j = (const bf16_job *)p;
    for (size_t i = j->lo; i < j->hi; i++)
        j->out[i] = oracle_f32_to_bf16_rne(
            synth_normal_one(smix(j->key + (uint64_t)i * 0xD1B54A32D192ED03ull), j->sc));
    return NULL;
}

/* Counter-based, so the split across threads does not change any value. */
void oracle_synth_normal_bf16(uint16_t *out, size_t n, uint64_t seed,
                              uint64_t stream, double sigma) {
    enum { MAXT = 64 };
    const float sc = oracle_synth_normal_scale(sigma);
    const uint64_t key = smix(seed ^ smix(stream));
    long nt = sysconf(_SC_NPROCESSORS_ONLN);
    if (nt < 1) nt = 1;
    if (nt > MAXT) nt = MAXT;
    if (n < ((size_t)1 << 20)) nt = 1;
    bf16_job jobs[MAXT];
    pthread_t th[MAXT];
    for (long t = 0; t < nt; t++) {
        jobs[t].out = out; jobs[t].key = key; jobs[t].sc = sc;
        jobs[t].lo = n * (size_t)t / (size_t)nt;
        jobs[t].hi = n * (size_t)(t + 1) / (size_t)nt;
    }
    for (long t = 1; t < nt; t++)
        if (pthread_create(&th[t], NULL, bf16_worker, &jobs[t]) != 0) {
            bf16_worker(&jobs[t]);
            th[t] = 0;
        }
    bf16_worker(&jobs[0]);
    for (long t = 1; t < nt; t++) if (th[t]) pthread_join(th[t], NULL);
}

void oracle_synth_normal_f32(float *out, size_t n, uint64_t seed,
                             uint64_t stream, double sigma) {
    const float sc = oracle_synth_normal_scale(sigma);
    const uint64_t key = smix(seed ^ smix(stream));
    for (size_t i = 0; i < n; i++)
        out[i] = synth_normal_one(smix(key + (uint64_t)i * 0xD1B54A32D192ED03ull), sc);
}

void oracle_synth_tokens(int32_t *out, size_t n, uint64_t seed, uint64_t stream,
                         int vocab) {
    for (size_t i = 0; i < n; i++)
        out[i] = (int32_t)(oracle_synth_u64(seed, stream, i) % (uint64_t)vocab);
}

/* ---- QW3M ---- */

static void wr_i32(uint8_t *p, int32_t v) {
    uint32_t u = (uint32_t)v;
    p[0] = (uint8_t)u; p[1] = (uint8_t)(u >> 8); p[2] = (uint8_t)(u >> 16); p[3] = (uint8_t)(u >> 24);
}
static void wr_f32(uint8_t *p, float f) { int32_t v; memcpy(&v, &f, 4); wr_i32(p, v); }

/* Elements per tensor, in file order; kind 1 = norm weight (all ones). */
static size_t tensor_elems(int idx, int *is_norm) {
    *is_norm = 0;
    if (idx == 0) return (size_t)VOCAB * HIDDEN;
    if (idx == 1 + LAYERS * 11) { *is_norm = 1; return HIDDEN; }
    switch ((idx - 1) % 11) {
    case 0:  *is_norm = 1; return HIDDEN;             /* input_layernorm */
    case 1:  return (size_t)QDIM * HIDDEN;            /* q_proj */
    case 2:  return (size_t)KVDIM * HIDDEN;           /* k_proj */
    case 3:  return (size_t)KVDIM * HIDDEN;           /* v_proj */
    case 4:  *is_norm = 1; return HDIM;               /* q_norm */
    case 5:  *is_norm = 1; return HDIM;               /* k_norm */
    case 6:  return (size_t)HIDDEN * QDIM;            /* o_proj */
    case 7:  *is_norm = 1; return HIDDEN;             /* post_attention_layernorm */
    case 8:  return (size_t)INTER * HIDDEN;           /* gate_proj */
    case 9:  return (size_t)INTER * HIDDEN;           /* up_proj */
    default: return (size_t)HIDDEN * INTER;           /* down_proj */
    }
}

#define N_TENSORS (1 + LAYERS * 11 + 1)
#define ALIGN 128

size_t oracle_qw3m_size(void) {
    size_t pos = 256;
    for (int t = 0; t < N_TENSORS; t++) {
        int nrm;
        pos = (pos + ALIGN - 1) & ~(size_t)(ALIGN - 1);
        pos += tensor_elems(t, &nrm) * 2;
    }
    return pos;
}

int oracle_qw3m_write(uint8_t *blob, size_t size, uint64_t seed, double sigma) {
    if (size != oracle_qw3m_size()) return -1;
    memset(blob, 0, 256);
    memcpy(blob, "QW3M", 4);
    wr_i32(blob + 4, 1);
    wr_i32(blob + 8, HIDDEN);  wr_i32(blob + 12, INTER); wr_i32(blob + 16, LAYERS);
    wr_i32(blob + 20, NHEADS); wr_i32(blob + 24, NKV);   wr_i32(blob + 28, HDIM);
    wr_i32(blob + 32, VOCAB);  wr_i32(blob + 36, 40960); wr_i32(blob + 40, 1);
    wr_i32(blob + 44, 1);
    wr_f32(blob + 48, 1000000.0f); wr_f32(blob + 52, 1e-06f);
    wr_i32(blob + 56, 151643); wr_i32(blob + 60, 151645); wr_i32(blob + 64, 151643);
    wr_i32(blob + 68, 256); wr_i32(blob + 72, ALIGN);
    wr_i32(blob + 76, 0); wr_i32(blob + 80, 0); wr_i32(blob + 84, 0);
    size_t pos = 256;
    for (int t = 0; t < N_TENSORS; t++) {
        int nrm;
        size_t n = tensor_elems(t, &nrm);
        size_t p = (pos + ALIGN - 1) & ~(size_t)(ALIGN - 1);
        memset(blob + pos, 0, p - pos);
        uint16_t *dst = (uint16_t *)(blob + p);
        if (nrm) for (size_t i = 0; i < n; i++) dst[i] = 0x3F80;   /* 1.0 */
        else oracle_synth_normal_bf16(dst, n, seed, (uint64_t)t, sigma);
        pos = p + n * 2;
    }
    return 0;
}
