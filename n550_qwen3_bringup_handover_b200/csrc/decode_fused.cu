// Decode step of 1-4 sequences as one persistent kernel (qwen3_forward,
// qwen3.c:455-545 for all 28 layers; the lm_head follows as its own GEMV).
//
// Why: at a few tokens a decode step is a 1.19 GB weight stream (183 us at
// the measured HBM bandwidth), but as ~250 dependent kernels it is bound by
// their launches and ramp-ups (~850 us). Here one cooperative grid of one CTA
// per SM walks the layers in five phases separated by grid barriers:
//
//   A  rmsnorm(x) into shared memory (every CTA, redundantly), q/k/v GEMV of
//      this CTA's columns -> qkv (FP32)
//   B  attention units (token, KV head, split): QK-norm + RoPE of the two
//      query heads and of k, the K/V write of split 0 into the cache, scores,
//      softmax and P.V on CUDA cores; several splits are merged by the unit
//      that finishes last -> attn (BF16)
//   C  o GEMV of this CTA's columns, x += (the residual)
//   D  rmsnorm(x) again, gate/up GEMV with SiLU . mul -> h (BF16)
//   E  down GEMV, x += (the residual)
//
// Every CTA owns a contiguous range of output columns in each GEMV; their
// weight rows are copied into shared memory by bulk copies issued as soon as
// the buffer is free, so the weights of the next phases stream while this
// phase computes and while the grid waits at a barrier. Data another CTA
// wrote inside the kernel is read with ld.global.cg (L1 is not coherent).
// Grid barriers and mbarrier waits are bounded: on expiry the kernel records
// N550_ERR_TIMEOUT in the device status word and every CTA returns.
#include "common.cuh"
#include "decode_fused.h"

namespace n550 {
namespace {

constexpr int H = 1024, QD = 2048, QKVD = 4096, INTER = 3072, NL = 28, NKV = 8, HD = 128;
constexpr float EPS = 1e-6f;
constexpr float kScale = 0.08838834764831845f;     // qwen3.c:296
constexpr int THREADS = 512, WARPS = THREADS / 32;
constexpr int WBUF = 88 * 1024;                    // one weight buffer (a CTA's rows of one phase)
constexpr int ACT = FD_MAX_TOKENS * INTER * 2;     // BF16 activations [T][<= 3072]
constexpr int SMEM = 2 * WBUF + ACT + 2 * FD_MAX_POS * 4 + WARPS * 256 * 4 + 4 * HD * 4 + 64 * 4 + 64;

__device__ __forceinline__ float ldcg(const float *p) { return __ldcg(p); }
__device__ __forceinline__ unsigned ld_acquire(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

struct Smem {
    uint8_t *wbuf[2];
    uint16_t *act;         // [T][K] BF16 GEMV input
    float *sc;             // [2][FD_MAX_POS] scores / probabilities
    float *ored;           // [WARPS][256] partial P.V sums
    float *hv;             // [4][128] q(2g), q(2g+1), k, v of an attention unit
    float *red;            // [64] block reductions
    uint64_t *bar;         // [3] weight-buffer mbarriers, K rows of an attention unit
    int *flag;             // barrier/abort flag
};

// Grid barrier over gridDim.x CTAs: a monotonic arrival counter (zeroed before
// the launch); `target` is the count that completes this barrier. Returns
// false (device status set) if the wait expired.
__device__ bool grid_sync(unsigned *ctr, unsigned target, int *flag) {
    __syncthreads();
    if (threadIdx.x == 0) {
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(ctr) : "memory");
        int ok = 1;
        if (ld_acquire(ctr) < target) {
            const long long t0 = clock64();
            while (ld_acquire(ctr) < target) {
                if (clock64() - t0 > kWaitCycles) { report_timeout(); ok = 0; break; }
            }
        }
        __threadfence();
        *flag = ok;
    }
    __syncthreads();
    return *flag != 0;
}

// Block-wide sum of one float per thread (all threads get the result).
__device__ float block_sum(float v, float *red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < WARPS; i++) s += red[i];
    return s;
}

__device__ float block_max(float v, float *red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float s = red[0];
#pragma unroll
    for (int i = 1; i < WARPS; i++) s = fmaxf(s, red[i]);
    return s;
}

// act[t][0..1024) = bf16(rmsnorm(x[t]) * w) for the T token rows (qwen3.c:471/527).
__device__ void norm_to_smem(const float *x, const uint16_t *w, uint16_t *act, int T, float *red) {
    for (int t = 0; t < T; t++) {
        const float *xr = x + (size_t)t * H;
        const int c = threadIdx.x * 2;
        const float a = ldcg(xr + c), b = ldcg(xr + c + 1);
        const float ss = block_sum(fmaf(a, a, b * b), red);
        const float s = 1.0f / sqrtf(ss / (float)H + EPS);
        act[t * H + c] = f32_to_bf16_rne(a * s * bf16_bits_to_f32(w[c]));
        act[t * H + c + 1] = f32_to_bf16_rne(b * s * bf16_bits_to_f32(w[c + 1]));
    }
}

// Columns [c0, c1) of an N-column GEMV that CTA b of G owns.
__device__ __forceinline__ void col_range(int N, int &c0, int &c1) {
    c0 = (int)(((long long)N * blockIdx.x) / gridDim.x);
    c1 = (int)(((long long)N * (blockIdx.x + 1)) / gridDim.x);
}

// Thread 0: bulk copies of weight rows [c0, c1) of W (and W2) into a buffer.
__device__ void issue_rows(const Smem &s, int buf, const uint16_t *W, const uint16_t *W2, int N, int K) {
    if (threadIdx.x != 0) return;
    int c0, c1;
    col_range(N, c0, c1);
    const uint32_t row = (uint32_t)K * 2, nrow = (uint32_t)(c1 - c0);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    mbar_arrive_expect_tx(&s.bar[buf], row * nrow * (W2 ? 2 : 1));
    // rows [c0, c1) of a row-major [N][K] matrix are one contiguous range
    bulk_load(s.wbuf[buf], W + (size_t)c0 * K, row * nrow, &s.bar[buf]);
    if (W2) bulk_load(s.wbuf[buf] + nrow * row, W2 + (size_t)c0 * K, row * nrow, &s.bar[buf]);
}

// Dot products of one weight row (shared memory, K BF16) with the T rows of
// act: this lane's partial sums (lane covers k = 8 lane + 256 j).
template <int K>
__device__ __forceinline__ void row_dot(const uint16_t *w, const uint16_t *act, int T, float (&acc)[FD_MAX_TOKENS]) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int t = 0; t < FD_MAX_TOKENS; t++) acc[t] = 0.f;
#pragma unroll 4
    for (int k = lane * 8; k < K; k += 256) {
        const uint4 wq = *(const uint4 *)(w + k);
        const float w0 = __uint_as_float(wq.x << 16), w1 = __uint_as_float(wq.x & 0xFFFF0000u),
                    w2 = __uint_as_float(wq.y << 16), w3 = __uint_as_float(wq.y & 0xFFFF0000u),
                    w4 = __uint_as_float(wq.z << 16), w5 = __uint_as_float(wq.z & 0xFFFF0000u),
                    w6 = __uint_as_float(wq.w << 16), w7 = __uint_as_float(wq.w & 0xFFFF0000u);
#pragma unroll
        for (int t = 0; t < FD_MAX_TOKENS; t++) {
            if (t >= T) break;
            const uint4 aq = *(const uint4 *)(act + t * K + k);
            float a = acc[t];
            a = fmaf(__uint_as_float(aq.x << 16), w0, a);
            a = fmaf(__uint_as_float(aq.x & 0xFFFF0000u), w1, a);
            a = fmaf(__uint_as_float(aq.y << 16), w2, a);
            a = fmaf(__uint_as_float(aq.y & 0xFFFF0000u), w3, a);
            a = fmaf(__uint_as_float(aq.z << 16), w4, a);
            a = fmaf(__uint_as_float(aq.z & 0xFFFF0000u), w5, a);
            a = fmaf(__uint_as_float(aq.w << 16), w6, a);
            a = fmaf(__uint_as_float(aq.w & 0xFFFF0000u), w7, a);
            acc[t] = a;
        }
    }
#pragma unroll
    for (int t = 0; t < FD_MAX_TOKENS; t++) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc[t] += __shfl_xor_sync(0xFFFFFFFFu, acc[t], o);
    }
}

// GEMV phase over this CTA's columns, one warp per column; out(t, n, value).
template <int K, class Out>
__device__ void gemv_phase(const Smem &s, int buf, int N, int T, Out out) {
    int c0, c1;
    col_range(N, c0, c1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint16_t *w = (const uint16_t *)s.wbuf[buf];
    for (int r = warp; r < c1 - c0; r += WARPS) {
        float acc[FD_MAX_TOKENS];
        row_dot<K>(w + (size_t)r * K, s.act, T, acc);
        if (lane < T) {
            float v = acc[0];
#pragma unroll
            for (int t = 1; t < FD_MAX_TOKENS; t++) if (lane == t) v = acc[t];
            out(lane, c0 + r, v);
        }
    }
}

// Gate/up phase: rows [0, nc) gate, [nc, 2 nc) up; h = bf16(silu(g) * u).
__device__ void swiglu_phase(const Smem &s, int buf, int T, uint16_t *h) {
    int c0, c1;
    col_range(INTER, c0, c1);
    const int nc = c1 - c0;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint16_t *w = (const uint16_t *)s.wbuf[buf];
    for (int r = warp; r < nc; r += WARPS) {
        float g[FD_MAX_TOKENS], u[FD_MAX_TOKENS];
        row_dot<H>(w + (size_t)r * H, s.act, T, g);
        row_dot<H>(w + (size_t)(nc + r) * H, s.act, T, u);
        if (lane < T) {
            float gv = g[0], uv = u[0];
#pragma unroll
            for (int t = 1; t < FD_MAX_TOKENS; t++) if (lane == t) { gv = g[t]; uv = u[t]; }
            __stcg(h + (size_t)lane * INTER + c0 + r, f32_to_bf16_rne((gv / (1.0f + expf(-gv))) * uv));
        }
    }
}

// BF16 rows [T][K] written by other CTAs -> shared memory.
__device__ void load_act(uint16_t *act, const uint16_t *src, int T, int K) {
    const int n = T * K / 8;
    for (int i = threadIdx.x; i < n; i += THREADS)
        ((uint4 *)act)[i] = __ldcg((const uint4 *)src + i);
}

// Rows of K a unit copies into shared memory (the activation buffer, free
// during the attention phase): 96 x 256 bytes.
constexpr int KSM_ROWS = ACT / (HD * 2);

// Splits of the attention over positions [0, pos]: up to 96 positions per
// unit while that takes at most FD_MAX_SPLITS units per (token, KV head), so
// that a unit's K rows arrive by one bulk copy; longer contexts take 32 units
// of up to 256 positions (the V rows a warp holds in registers) and read K
// directly.
__device__ __forceinline__ int attn_splits(int pos) {
    const int s = (pos + 1 + KSM_ROWS - 1) / KSM_ROWS;
    return s < FD_MAX_SPLITS ? s : FD_MAX_SPLITS;
}

// One attention unit: token t, KV head g, split sp of S (qwen3.c:287-292,
// 374-436 and 498-511 for that head pair).
__device__ void attn_unit(const FusedDecodeArgs &a, const Smem &s, int l, int t, int g, int sp, int S,
                          uint32_t &kphase) {
    const int pos = a.pos[t], seq = a.seq_ids[t];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const FusedLayer &L = a.layers[l];
    const int n = pos + 1;
    const int p0 = (int)((long long)n * sp / S), p1 = (int)((long long)n * (sp + 1) / S);
    const uint16_t *kbase = a.kc + ((size_t)(seq * NL + l) * NKV + g) * a.max_len * HD;
    const uint16_t *vbase = a.vc + ((size_t)(seq * NL + l) * NKV + g) * a.max_len * HD;
    // K rows [p0, p1) are contiguous in the cache: one bulk copy into shared
    // memory (the row at pos is not written yet; its scores use the new k)
    const bool k_smem = p1 - p0 <= KSM_ROWS;
    if (k_smem && threadIdx.x == 0) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        mbar_arrive_expect_tx(&s.bar[2], (uint32_t)(p1 - p0) * HD * 2);
        bulk_load(s.act, kbase + (size_t)p0 * HD, (uint32_t)(p1 - p0) * HD * 2, &s.bar[2]);
    }
    // V rows of this warp's positions (at most 16: a unit spans <= 256) are
    // requested first, so that their latency overlaps the head vectors and scores
    constexpr int VP = 256 / WARPS;
    uint2 vq[VP];
#pragma unroll
    for (int i = 0; i < VP; i++) {
        const int p = p0 + warp + WARPS * i;
        vq[i] = (p < p1 && p != pos) ? *(const uint2 *)(vbase + (size_t)p * HD + 4 * lane) : make_uint2(0, 0);
    }
    // q heads 2g, 2g+1, k head g, v head g: per-head RMSNorm and RoPE (q, k)
    if (warp < 4) {
        const int col = warp < 2 ? (2 * g + warp) * HD : (warp == 2 ? QD + g * HD : QD + 1024 + g * HD);
        const float *src = a.qkv + (size_t)t * QKVD + col;
        float v[4];
#pragma unroll
        for (int j = 0; j < 4; j++) v[j] = ldcg(src + lane + 32 * j);
        if (warp < 3) {
            const uint16_t *nw = warp < 2 ? L.q_norm : L.k_norm;
            float ss = v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, o);
            const float sc = 1.0f / sqrtf(ss / (float)HD + EPS);
#pragma unroll
            for (int j = 0; j < 4; j++) v[j] = v[j] * sc * bf16_bits_to_f32(nw[lane + 32 * j]);
#pragma unroll
            for (int j = 0; j < 2; j++) {               // pairs (i, i + 64)
                const float2 cs = a.rope[(size_t)pos * 64 + lane + 32 * j];
                const float x0 = v[j], x1 = v[j + 2];
                v[j] = x0 * cs.x - x1 * cs.y;
                v[j + 2] = x1 * cs.x + x0 * cs.y;
            }
        }
        if (warp >= 2) {            // k, v as the cache holds them (BF16)
            uint16_t *dst = (warp == 2 ? a.kc : a.vc) +
                            (((size_t)(seq * NL + l) * NKV + g) * a.max_len + pos) * HD;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const uint16_t b = f32_to_bf16_rne(v[j]);
                if (sp == 0) dst[lane + 32 * j] = b;
                v[j] = bf16_bits_to_f32(b);
            }
        }
#pragma unroll
        for (int j = 0; j < 4; j++) s.hv[warp * HD + lane + 32 * j] = v[j];
    }
    __syncthreads();
    if (k_smem) {
        mbar_wait(&s.bar[2], kphase);       // on expiry the status is set; the copy still lands here
        kphase ^= 1;
    }
    // scores, one position per thread
    float m0 = -INFINITY, m1 = -INFINITY;
    for (int p = p0 + (int)threadIdx.x; p < p1; p += THREADS) {
        float d0 = 0.f, d1 = 0.f;
        if (p == pos) {
            for (int d = 0; d < HD; d++) {
                const float k = s.hv[2 * HD + d];
                d0 = fmaf(s.hv[d], k, d0);
                d1 = fmaf(s.hv[HD + d], k, d1);
            }
        } else {
            const uint4 *kr = k_smem ? (const uint4 *)(s.act + (size_t)(p - p0) * HD)
                                     : (const uint4 *)(kbase + (size_t)p * HD);
            const int rot = k_smem ? (lane & 7) : 0;     // spreads the rows of 8 lanes over the banks
#pragma unroll 4
            for (int cc = 0; cc < 16; cc++) {
                const int c = (cc + rot) & 15;
                const uint4 q = kr[c];
                const uint32_t wv[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    const int d = c * 8 + 2 * e;
                    const float k0 = __uint_as_float(wv[e] << 16), k1 = __uint_as_float(wv[e] & 0xFFFF0000u);
                    d0 = fmaf(s.hv[d], k0, fmaf(s.hv[d + 1], k1, d0));
                    d1 = fmaf(s.hv[HD + d], k0, fmaf(s.hv[HD + d + 1], k1, d1));
                }
            }
        }
        d0 *= kScale;
        d1 *= kScale;
        s.sc[p - p0] = d0;
        s.sc[FD_MAX_POS + p - p0] = d1;
        m0 = fmaxf(m0, d0);
        m1 = fmaxf(m1, d1);
    }
    m0 = block_max(m0, s.red);
    m1 = block_max(m1, s.red + 32);
    float l0 = 0.f, l1 = 0.f;
    for (int p = p0 + (int)threadIdx.x; p < p1; p += THREADS) {
        const float e0 = expf(s.sc[p - p0] - m0), e1 = expf(s.sc[FD_MAX_POS + p - p0] - m1);
        s.sc[p - p0] = e0;
        s.sc[FD_MAX_POS + p - p0] = e1;
        l0 += e0;
        l1 += e1;
    }
    l0 = block_sum(l0, s.red);
    l1 = block_sum(l1, s.red + 32);
    // P.V: lane owns dims 4 lane .. 4 lane + 3, warps split the positions
    float o0[4] = {0.f, 0.f, 0.f, 0.f}, o1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int i = 0; i < VP; i++) {
        const int p = p0 + warp + WARPS * i;
        if (p >= p1) break;
        float v[4];
        if (p == pos) {
#pragma unroll
            for (int j = 0; j < 4; j++) v[j] = s.hv[3 * HD + 4 * lane + j];
        } else {
            v[0] = __uint_as_float(vq[i].x << 16); v[1] = __uint_as_float(vq[i].x & 0xFFFF0000u);
            v[2] = __uint_as_float(vq[i].y << 16); v[3] = __uint_as_float(vq[i].y & 0xFFFF0000u);
        }
        const float e0 = s.sc[p - p0], e1 = s.sc[FD_MAX_POS + p - p0];
#pragma unroll
        for (int j = 0; j < 4; j++) {
            o0[j] = fmaf(e0, v[j], o0[j]);
            o1[j] = fmaf(e1, v[j], o1[j]);
        }
    }
#pragma unroll
    for (int j = 0; j < 4; j++) {
        s.ored[warp * 256 + 4 * lane + j] = o0[j];
        s.ored[warp * 256 + 128 + 4 * lane + j] = o1[j];
    }
    __syncthreads();
    if (threadIdx.x < 256) {
        float o = 0.f;
#pragma unroll
        for (int w = 0; w < WARPS; w++) o += s.ored[w * 256 + threadIdx.x];
        const int hh = threadIdx.x >> 7, d = threadIdx.x & 127;
        const int head = 2 * g + hh;
        if (S == 1) {
            __stcg(a.attn + (size_t)t * QD + head * HD + d, f32_to_bf16_rne(o / (hh ? l1 : l0)));
        } else {
            const size_t slot = ((size_t)t * 16 + head) * FD_MAX_SPLITS + sp;
            __stcg(a.part_o + slot * HD + d, o);
            if (d == 0) {
                __stcg(a.part_m + slot, hh ? m1 : m0);
                __stcg(a.part_l + slot, hh ? l1 : l0);
            }
        }
    }
    if (S == 1) {
        __syncthreads();
        return;
    }
    // the unit that completes the (token, KV head) last merges the splits
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        const int prev = atomicAdd(a.counters + t * NKV + g, 1);
        s.flag[1] = prev == S - 1;
        if (prev == S - 1) {
            a.counters[t * NKV + g] = 0;        // ready for the next layer
            __threadfence();
        }
    }
    __syncthreads();
    if (!s.flag[1]) return;
    if (threadIdx.x < 256) {
        const int hh = threadIdx.x >> 7, d = threadIdx.x & 127;
        const int head = 2 * g + hh;
        const size_t base = ((size_t)t * 16 + head) * FD_MAX_SPLITS;
        float mx = -INFINITY;
        for (int k = 0; k < S; k++) mx = fmaxf(mx, ldcg(a.part_m + base + k));
        float den = 0.f, num = 0.f;
        for (int k = 0; k < S; k++) {
            const float f = expf(ldcg(a.part_m + base + k) - mx);
            den = fmaf(ldcg(a.part_l + base + k), f, den);
            num = fmaf(ldcg(a.part_o + (base + k) * HD + d), f, num);
        }
        __stcg(a.attn + (size_t)t * QD + head * HD + d, f32_to_bf16_rne(num / den));
    }
    __syncthreads();
}

__global__ void __launch_bounds__(THREADS, 1) decode_fused_kernel(FusedDecodeArgs a) {
    extern __shared__ __align__(1024) uint8_t smem[];
    Smem s;
    s.wbuf[0] = smem;
    s.wbuf[1] = smem + WBUF;
    s.act = (uint16_t *)(smem + 2 * WBUF);
    s.sc = (float *)(smem + 2 * WBUF + ACT);
    s.ored = s.sc + 2 * FD_MAX_POS;
    s.hv = s.ored + WARPS * 256;
    s.red = s.hv + 4 * HD;
    s.bar = (uint64_t *)(s.red + 64);
    s.flag = (int *)(s.bar + 3);
    const int T = a.T;
    if (threadIdx.x == 0) {
        mbar_init(&s.bar[0], 1);
        mbar_init(&s.bar[1], 1);
        mbar_init(&s.bar[2], 1);
        fence_mbar_init();
    }
    __syncthreads();
    uint32_t phase[2] = {0, 0}, kphase = 0;
    int pending[2] = {0, 0};            // copies issued into a buffer and not yet waited for
    unsigned target = 0;
    const unsigned G = gridDim.x;
    auto wait_buf = [&](int b) {
        const bool ok = mbar_wait(&s.bar[b], phase[b]);
        phase[b] ^= 1;
        pending[b]--;
        return ok;
    };
    // before leaving on an expired wait: the copies in flight land first (bounded)
    auto drain = [&]() {
        for (int b = 0; b < 2; b++)
            while (pending[b] > 0) wait_buf(b);
    };
    auto sync = [&]() {
        target += G;
        if (grid_sync(a.barrier, target, s.flag)) return true;
        drain();
        return false;
    };
    auto issue = [&](int b, const uint16_t *W, const uint16_t *W2, int N, int K) {
        issue_rows(s, b, W, W2, N, K);
        pending[b]++;
    };
    auto wait = [&](int b) {
        if (wait_buf(b)) return true;
        drain();
        return false;
    };
    issue(0, a.layers[0].wqkv, nullptr, QKVD, H);
    issue(1, a.layers[0].wo, nullptr, H, QD);
    // total attention units of a layer (the same on every CTA)
    int units = 0;
    for (int t = 0; t < T; t++) units += NKV * attn_splits(a.pos[t]);

    for (int l = 0; l < NL; l++) {
        const FusedLayer &L = a.layers[l];
        // ---- A: q/k/v ----
        norm_to_smem(a.x, L.in_norm, s.act, T, s.red);
        __syncthreads();
        if (!wait(0)) return;
        gemv_phase<H>(s, 0, QKVD, T, [&](int t, int n, float v) { __stcg(a.qkv + (size_t)t * QKVD + n, v); });
        __syncthreads();
        issue(0, L.wg, L.wu, INTER, H);
        if (!sync()) return;
        // ---- B: attention ----
        for (int u = blockIdx.x; u < units; u += G) {
            int t = 0, r = u;
            while (r >= NKV * attn_splits(a.pos[t])) { r -= NKV * attn_splits(a.pos[t]); t++; }
            const int S = attn_splits(a.pos[t]);
            attn_unit(a, s, l, t, r / S, r % S, S, kphase);
        }
        if (!sync()) return;
        // ---- C: o projection + residual ----
        load_act(s.act, a.attn, T, QD);
        __syncthreads();
        if (!wait(1)) return;
        gemv_phase<QD>(s, 1, H, T, [&](int t, int n, float v) {
            float *p = a.x + (size_t)t * H + n;
            __stcg(p, ldcg(p) + v);
        });
        __syncthreads();
        issue(1, L.wd, nullptr, H, INTER);
        if (!sync()) return;
        // ---- D: gate / up with SwiGLU ----
        norm_to_smem(a.x, L.post_norm, s.act, T, s.red);
        __syncthreads();
        if (!wait(0)) return;
        swiglu_phase(s, 0, T, a.h);
        __syncthreads();
        if (l + 1 < NL) issue(0, a.layers[l + 1].wqkv, nullptr, QKVD, H);
        if (!sync()) return;
        // ---- E: down projection + residual ----
        load_act(s.act, a.h, T, INTER);
        __syncthreads();
        if (!wait(1)) return;
        gemv_phase<INTER>(s, 1, H, T, [&](int t, int n, float v) {
            float *p = a.x + (size_t)t * H + n;
            __stcg(p, ldcg(p) + v);
        });
        __syncthreads();
        if (l + 1 < NL) issue(1, a.layers[l + 1].wo, nullptr, H, QD);
        if (!sync()) return;
    }
    // final norm of every row (each is its sequence's last token) for the lm_head
    if ((int)blockIdx.x < T) {
        const int t = blockIdx.x;
        const float *xr = a.x + (size_t)t * H;
        const int c = threadIdx.x * 2;
        const float v0 = ldcg(xr + c), v1 = ldcg(xr + c + 1);
        const float ss = block_sum(fmaf(v0, v0, v1 * v1), s.red);
        const float sc = 1.0f / sqrtf(ss / (float)H + EPS);
        a.xl[(size_t)t * H + c] = f32_to_bf16_rne(v0 * sc * bf16_bits_to_f32(a.final_norm[c]));
        a.xl[(size_t)t * H + c + 1] = f32_to_bf16_rne(v1 * sc * bf16_bits_to_f32(a.final_norm[c + 1]));
    }
}

}  // namespace

int fused_decode_grid() {
    static int grid[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
    if (grid[dev]) return grid[dev] > 0 ? grid[dev] : 0;
    int sms = 0, coop = 0, per_sm = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev) != cudaSuccess ||
        cudaFuncSetAttribute(decode_fused_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM) !=
            cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_fused_kernel, THREADS, SMEM) !=
            cudaSuccess) {
        (void)cudaGetLastError();
        grid[dev] = -1;
        return 0;
    }
    // one CTA per SM; each CTA's weight rows of a phase must fit one buffer
    const int g = sms;
    const bool fits = coop && per_sm >= 1 && (long long)((INTER + g - 1) / g) * 2 * H * 2 <= WBUF &&
                      (long long)((QKVD + g - 1) / g) * H * 2 <= WBUF;
    grid[dev] = fits ? g : -1;
    return fits ? g : 0;
}

int launch_decode_fused(cudaStream_t st, const FusedDecodeArgs &a) {
    if (a.T < 1 || a.T > FD_MAX_TOKENS) return N550_ERR_ARG;
    const int g = fused_decode_grid();
    if (!g) return N550_ERR_UNSUPPORTED;
    N550_CUDA_TRY(cudaMemsetAsync(a.barrier, 0, sizeof(unsigned), st));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(g);
    cfg.blockDim = dim3(THREADS);
    cfg.dynamicSmemBytes = SMEM;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    N550_CUDA_TRY(cudaLaunchKernelEx(&cfg, decode_fused_kernel, a));
    return N550_OK;
}

}  // namespace n550
