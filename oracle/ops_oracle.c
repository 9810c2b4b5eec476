/* CPU oracle: non-GEMM ops -- TEST INFRASTRUCTURE ONLY (see oracle.h).
 *
 * Restates fpga_bringup/src/src/ops_scalar.c:11-78 operation by operation
 * (same evaluation order, FP32 throughout, libm sqrtf/expf/powf/sinf/cosf),
 * so that with the same compiler flags it is bit-identical to the reference.
 * Constants from qwen3_config.h:17-28.
 */
#include <math.h>
#include <string.h>

#include "oracle.h"

static inline float bf16f(uint16_t b) {
    uint32_t u = (uint32_t)b << 16;
    float f;
    memcpy(&f, &u, sizeof f);
    return f;
}

#define HEAD_DIM   128
#define RMS_EPS    1e-06f
#define ROPE_THETA 1000000.0f

void oracle_op_rmsnorm(float *out, const float *x, const uint16_t *w, int n) {
    float ss = 0.0f;
    for (int i = 0; i < n; i++) ss += x[i] * x[i];
    float scale = 1.0f / sqrtf(ss / (float)n + RMS_EPS);
    for (int i = 0; i < n; i++) out[i] = x[i] * scale * bf16f(w[i]);
}

/* rotate-half pairs (i, i + 64); inv_freq = theta^(-2i/128). */
void oracle_op_rope(float *v, int n_heads, int pos) {
    const int half = HEAD_DIM / 2;
    for (int i = 0; i < half; i++) {
        float inv_freq = 1.0f / powf(ROPE_THETA, (float)(2 * i) / (float)HEAD_DIM);
        float ang = (float)pos * inv_freq;
        float c = cosf(ang), s = sinf(ang);
        for (int h = 0; h < n_heads; h++) {
            float *p = v + (size_t)h * HEAD_DIM;
            float a = p[i], b = p[i + half];
            p[i]        = a * c - b * s;
            p[i + half] = b * c + a * s;
        }
    }
}

void oracle_op_softmax(float *x, int n) {
    float mx = x[0];
    for (int i = 1; i < n; i++) if (x[i] > mx) mx = x[i];
    float sum = 0.0f;
    for (int i = 0; i < n; i++) { x[i] = expf(x[i] - mx); sum += x[i]; }
    for (int i = 0; i < n; i++) x[i] /= sum;
}

void oracle_op_silu_mul(float *gate, const float *up, int n) {
    for (int i = 0; i < n; i++) {
        float g = gate[i];
        gate[i] = (g / (1.0f + expf(-g))) * up[i];
    }
}

void oracle_op_residual_add(float *x, const float *y, int n) {
    for (int i = 0; i < n; i++) x[i] += y[i];
}

/* First index of the maximum (strict >): ops_scalar.c:57-62. */
int oracle_op_argmax(const float *v, int n) {
    int best = 0;
    float bv = v[0];
    for (int i = 1; i < n; i++) if (v[i] > bv) { bv = v[i]; best = i; }
    return best;
}

void oracle_op_bf16_to_f32(float *out, const uint16_t *in, int n) {
    for (int i = 0; i < n; i++) out[i] = oracle_bf16_to_f32(in[i]);
}

float oracle_op_dot(const float *a, const float *b, int n) {
    float s = 0.0f;
    for (int i = 0; i < n; i++) s += a[i] * b[i];
    return s;
}

void oracle_op_axpy(float *y, float a, const float *x, int n) {
    for (int i = 0; i < n; i++) y[i] += a * x[i];
}
