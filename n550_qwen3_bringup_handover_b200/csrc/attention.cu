// GQA causal attention over the BF16 KV cache (qwen3.c:374-436 re-designed).
//
// Reference semantics: for query position p and head h (KV head h/2, an
// integer division, qwen3.c:299), scores s_t = (q . k_t) * 0.08838834764831845
// for t = 0..p, softmax over t, out = sum_t softmax_t * v_t.
//
// KV cache layout in HBM: [seq][layer][kv_head][pos][128] BF16 for K and for
// V -- one (seq, layer, kv_head) is a contiguous run of positions, the
// kvh-major order of qwen3.h:62-76, so decode streams it with coalesced loads.
//
// This file is the decode side: one query per sequence, split-KV, the dot
// products on mma.sync tensor-core fragments fed by a TMA shared-memory ring;
// the partial (max, sum, out) of each split are merged by a combine kernel. Prefill runs on the tcgen05
// tensor cores (attn_prefill_tc.cu).
#include <cuda.h>

#include "attention.h"
#include "common.cuh"
#include "launch.h"
#include "tmap.h"

namespace n550 {
namespace {

constexpr int HD = 128;
constexpr int NKV = 8;
constexpr int NL = 28;
constexpr float kScale = 0.08838834764831845f;     // qwen3.c:296
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kEps = 1e-6f;                      // RMSNorm epsilon (qwen3_config.h)

// ---------------------------------------------------------------------------
// decode (split-KV; q.K^T and P.V on mma.sync tensor-core fragments)
// ---------------------------------------------------------------------------
constexpr int DC_THREADS = 128;     // 4 warps
constexpr int DC_WARPS = DC_THREADS / 32;
constexpr int DC_TP = 64;           // positions per tile
constexpr int DC_PPW = DC_TP / DC_WARPS;       // positions of a tile per warp (16)
constexpr int DC_STAGES = 3;        // tiles in flight per CTA
constexpr int DC_BOX = 64 * 64 * 2;            // 64 positions x 64 dims BF16, 128-byte swizzle
constexpr int DC_STAGE_BYTES = 4 * DC_BOX;     // K dims 0-63 | K 64-127 | V 0-63 | V 64-127
constexpr int DC_SMEM = DC_STAGES * DC_STAGE_BYTES + 1024 + 64;
static_assert(DC_PPW == 16, "one 16-position MMA k-step of P.V per warp and tile");

// Byte offset of the 16-byte chunk (position p, dims d..d+7; d a multiple of
// 8) in a tile held as two 128-byte-swizzled boxes of 64 dims: chunk c of a
// 128-byte row r sits at chunk c ^ (r & 7), so the 8 rows of an 8 x 8
// ldmatrix tile fall in 8 different bank groups.
__device__ __forceinline__ uint32_t dc_off(int p, int d) {
    return (uint32_t)((d >> 6) * DC_BOX + p * 128 + ((((d & 63) >> 3) ^ (p & 7)) << 4));
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}
// D (16 x 8, FP32) += A (16 x 16 BF16, rows 8-15 zero) . B (16 x 8 BF16)
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a2, uint32_t b0,
                                               uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
}

// One CTA per (split, kv head, sequence); its two query heads are rows 0-1
// of 16-row MMA tiles (rows 2-15 zero). K and V tiles of 64 positions stream
// through a 3-stage ring of TMA loads (3-D maps over the cache, 128-byte
// swizzle). Warp w owns positions 16w..16w+15 of every tile: S = q.K^T over
// them (2 x 8 MMAs of m16n8k16), an online softmax per head on the S
// fragments, then O += P.V (16 MMAs, the S fragments reused as the A
// operand in BF16, V read transposed by ldmatrix). The four warps' (max, sum,
// O) are merged at the end.
__global__ void __launch_bounds__(DC_THREADS)
attn_decode_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                   AttnDecodeArgs p) {
    extern __shared__ uint8_t dsm[];
    uint8_t *ring = (uint8_t *)(((uintptr_t)dsm + 1023) & ~(uintptr_t)1023);
    uint64_t *full = (uint64_t *)(ring + DC_STAGES * DC_STAGE_BYTES);
    uint64_t *empty = full + DC_STAGES;
    __shared__ float wm[DC_WARPS][2], wl[DC_WARPS][2];
    __shared__ __align__(16) float wo[DC_WARPS][2][HD];
    __shared__ __align__(16) float hv[4][HD];      // fused mode: q (2 heads), k, v of this KV head

    // The sequence ids and positions are inputs of the whole step (written
    // before the kernels this one depends on; read through L2), and cache
    // positions below pos[s] hold K/V of earlier steps. Only position pos[s]
    // and the queries come from the kernel this launch depends on.
    const int split = blockIdx.x, kvh = blockIdx.y, s = blockIdx.z;
    const int seq = __ldcg(p.seq_ids + s);
    const int kv_len = __ldcg(p.pos + s) + 1;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // Splits that hold positions: with the merge in this kernel (counters set)
    // a context takes floor(sqrt(kv_len / 32)) splits (1 up to 127 positions,
    // 4 at 512, 8 at 2048, 16 at 8192; at most the grid's), and the other CTAs
    // of the (sequence, KV head) return at once. Streaming a split costs its
    // positions, merging costs the split count: measured on B200 (graph-
    // replayed steps of 1-4 sequences at 64-2048 positions) this beats fixed
    // minimum split lengths of 128, 256 and 512 positions, and a one-sequence
    // step at a short context runs one CTA per KV head instead of merging
    // mostly empty splits (batch-1 decode 883 -> 657 us per token). Every CTA
    // of the pair computes the same count from pos[s].
    const int eff = p.counters ? max(1, min(p.splits, (int)sqrtf((float)kv_len * (1.0f / 32.0f))))
                               : p.splits;
    if (split >= eff) return;
    int chunk = (kv_len + eff - 1) / eff;
    chunk = (chunk + DC_TP - 1) / DC_TP * DC_TP;
    const int start = split * chunk, end = min(kv_len, start + chunk);
    const int n_tiles = end > start ? (end - start + DC_TP - 1) / DC_TP : 0;
    const int plane = (seq * NL + p.layer) * NKV + kvh;

    if (threadIdx.x == 0) {
        for (int i = 0; i < DC_STAGES; i++) { mbar_init(&full[i], 1); mbar_init(&empty[i], DC_WARPS); }
        fence_mbar_init();
        tma_prefetch_desc(&tmK);
        tma_prefetch_desc(&tmV);
    }
    __syncthreads();
    auto issue = [&](int tile) {
        const int st = tile % DC_STAGES;
        const int t0 = start + tile * DC_TP;
        uint8_t *b = ring + st * DC_STAGE_BYTES;
        mbar_arrive_expect_tx(&full[st], DC_STAGE_BYTES);
        tma_load_3d(b, &tmK, &full[st], 0, t0, plane);
        tma_load_3d(b + DC_BOX, &tmK, &full[st], 64, t0, plane);
        tma_load_3d(b + 2 * DC_BOX, &tmV, &full[st], 0, t0, plane);
        tma_load_3d(b + 3 * DC_BOX, &tmV, &full[st], 64, t0, plane);
    };
    // Tiles that end before position pos[s] are requested before waiting for
    // the previous kernel, so their latency overlaps its tail. In fused mode
    // every tile is: the row at pos[s] is replaced in shared memory by the K/V
    // this kernel computes.
    const bool fused = p.qkv != nullptr;
    const int pos = kv_len - 1;
    int pre = 0;
    if (threadIdx.x == 0)
        while (pre < min(DC_STAGES, n_tiles) && (fused || start + (pre + 1) * DC_TP <= pos)) issue(pre++);
    // Fused mode: the QK-norm weights and the RoPE factors of position pos[s]
    // are no output of the kernel this one depends on either.
    float nw[4] = {0.f, 0.f, 0.f, 0.f};
    float2 rcs[2] = {};
    if (fused && warp < 3) {
        const uint16_t *w = warp < 2 ? p.q_norm : p.k_norm;
#pragma unroll
        for (int j = 0; j < 4; j++) nw[j] = bf16_bits_to_f32(w[lane + 32 * j]);
#pragma unroll
        for (int j = 0; j < 2; j++) rcs[j] = p.rope[(size_t)pos * 64 + lane + 32 * j];
    }
    dep_wait();
    dep_launch();
    if (threadIdx.x == 0)
        for (int i = pre; i < min(DC_STAGES, n_tiles); i++) issue(i);
    if (fused) {
        // warp 0 / 1: query heads 2 kvh, 2 kvh + 1; warp 2: K head kvh; warp 3: V head kvh
        const int col = warp < 2 ? (kvh * 2 + warp) * HD : (warp == 2 ? 16 * HD + kvh * HD : 24 * HD + kvh * HD);
        const float *src = p.qkv + (size_t)s * p.qkv_ld + col + lane;
        float v[4];
#pragma unroll
        for (int j = 0; j < 4; j++) {          // the split-K slices summed in order
            if (p.qkv_ks <= 0) {
                v[j] = src[32 * j];
            } else {
                float a[8];
#pragma unroll
                for (int k = 0; k < 8; k++) a[k] = k < p.qkv_ks ? src[32 * j + k * p.qkv_slice] : 0.f;
                float acc = a[0];
#pragma unroll
                for (int k = 1; k < 8; k++) acc += a[k];
                v[j] = acc;
            }
        }
        if (warp < 3) {
            float ss = v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, o);
            const float sc = 1.0f / sqrtf(ss / (float)HD + kEps);
#pragma unroll
            for (int j = 0; j < 4; j++) v[j] = v[j] * sc * nw[j];
#pragma unroll
            for (int j = 0; j < 2; j++) {      // rotate-half pairs (i, i + 64)
                const float2 cs = rcs[j];
                const float a = v[j], b = v[j + 2];
                v[j] = a * cs.x - b * cs.y;
                v[j + 2] = b * cs.x + a * cs.y;
            }
        }
        if (warp >= 2) {                       // K and V as the cache holds them
            uint16_t *dst = (warp == 2 ? p.kc_w : p.vc_w) + ((size_t)plane * p.max_len + pos) * HD;
            const bool writer = start <= pos && pos < end;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const uint16_t b = f32_to_bf16_rne(v[j]);
                if (writer) dst[lane + 32 * j] = b;
                v[j] = bf16_bits_to_f32(b);
            }
        }
#pragma unroll
        for (int j = 0; j < 4; j++) hv[warp][lane + 32 * j] = v[j];
        __syncthreads();
    }

    // A fragments of q (x scale x log2 e, BF16): row g = lane / 4 is query
    // head 2 kvh + g for g < 2, zero otherwise; columns 16 kk + 2 tq (+1, +8).
    const int g = lane >> 2, tq = lane & 3;
    uint32_t qa[8][2];
#pragma unroll
    for (int kk = 0; kk < 8; kk++)
#pragma unroll
        for (int h8 = 0; h8 < 2; h8++) {
            float v0 = 0.f, v1 = 0.f;
            if (g < 2 && fused) {
                v0 = hv[g][16 * kk + 8 * h8 + 2 * tq];
                v1 = hv[g][16 * kk + 8 * h8 + 2 * tq + 1];
            } else if (g < 2) {
                const size_t o = (size_t)s * p.ldq + (size_t)(kvh * 2 + g) * HD + 16 * kk + 8 * h8 + 2 * tq;
                v0 = p.q_f32 ? p.q_f32[o] : bf16_bits_to_f32(p.q_bf16[o]);
                v1 = p.q_f32 ? p.q_f32[o + 1] : bf16_bits_to_f32(p.q_bf16[o + 1]);
            }
            qa[kk][h8] = pack_bf16x2(v0 * (kScale * kLog2e), v1 * (kScale * kLog2e));
        }
    float m_r = -INFINITY, l_r = 0.f;        // softmax state of row g (log2 units)
    float o[16][4];                           // O row g: dims 8 nt + 2 tq (+1)
#pragma unroll
    for (int nt = 0; nt < 16; nt++) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.f;
    bool ok = true;
    const int p0 = warp * DC_PPW;            // this warp's rows of every tile

    for (int tile = 0; tile < n_tiles && ok; tile++) {
        const int st = tile % DC_STAGES;
        const uint32_t par = (uint32_t)((tile / DC_STAGES) & 1);
        if (!mbar_wait(&full[st], par)) { ok = false; break; }
        uint8_t *kt = ring + st * DC_STAGE_BYTES;
        const uint32_t kb = smem_u32(kt), vb = kb + 2 * DC_BOX;
        const int t0 = start + tile * DC_TP + p0;              // this warp's first position
        // fused mode: the row at pos[s] (loaded stale) takes this kernel's K and V
        if (fused && pos >= t0 && pos < t0 + DC_PPW) {
            const int r = p0 + (pos - t0), c = lane & 15, which = lane >> 4;
            const float *src = hv[2 + which] + 8 * c;
            uint4 q;
            q.x = pack_bf16x2(src[0], src[1]);
            q.y = pack_bf16x2(src[2], src[3]);
            q.z = pack_bf16x2(src[4], src[5]);
            q.w = pack_bf16x2(src[6], src[7]);
            *(uint4 *)(kt + which * 2 * DC_BOX + dc_off(r, 8 * c)) = q;
            __syncwarp();
        }
        // V rows past the end of the range may hold anything (stale cache):
        // zero them so that 0-weights do not meet NaN.
        if (t0 + DC_PPW > end) {
            for (int idx = lane; idx < DC_PPW * 16; idx += 32) {
                const int r = idx >> 4, c = idx & 15;
                if (t0 + r >= end)
                    *(uint4 *)(kt + 2 * DC_BOX + (c >> 3) * DC_BOX + (p0 + r) * 128 + (c & 7) * 16) =
                        make_uint4(0u, 0u, 0u, 0u);
            }
            __syncwarp();
        }
        // S = q . K^T, positions p0 + 8 nt + (col): n-tiles of 8 positions
        float sc[2][4];
#pragma unroll
        for (int nt = 0; nt < 2; nt++) {
            sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
#pragma unroll
            for (int k2 = 0; k2 < 4; k2++) {        // 32 dims per ldmatrix.x4
                uint32_t b[4];
                ldsm_x4(kb + dc_off(p0 + 8 * nt + (lane & 7), 32 * k2 + 8 * (lane >> 3)), b);
                mma_bf16_16816(sc[nt], qa[2 * k2][0], qa[2 * k2][1], b[0], b[1]);
                mma_bf16_16816(sc[nt], qa[2 * k2 + 1][0], qa[2 * k2 + 1][1], b[2], b[3]);
            }
        }
        // online softmax of row g over this warp's 16 positions (4 per lane)
        float sv[2][2];
        float mx = -INFINITY;
#pragma unroll
        for (int nt = 0; nt < 2; nt++)
#pragma unroll
            for (int j = 0; j < 2; j++) {
                const bool valid = t0 + 8 * nt + 2 * tq + j < end;
                sv[nt][j] = valid ? sc[nt][j] : -INFINITY;
                mx = fmaxf(mx, sv[nt][j]);
            }
        mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, 2));
        const float mn = fmaxf(m_r, mx);
        const float corr = (mn == -INFINITY) ? 1.f : exp2f(m_r - mn);
        float sum = 0.f;
#pragma unroll
        for (int nt = 0; nt < 2; nt++)
#pragma unroll
            for (int j = 0; j < 2; j++) {
                const float e = (sv[nt][j] == -INFINITY) ? 0.f : exp2f(sv[nt][j] - mn);
                sv[nt][j] = e;
                sum += e;
            }
        sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 1);
        sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 2);
        l_r = l_r * corr + sum;
        m_r = mn;
#pragma unroll
        for (int nt = 0; nt < 16; nt++) { o[nt][0] *= corr; o[nt][1] *= corr; }
        // P as the A operand: columns 2 tq (+1) from n-tile 0, +8 from n-tile 1
        const uint32_t pa0 = pack_bf16x2(sv[0][0], sv[0][1]);
        const uint32_t pa2 = pack_bf16x2(sv[1][0], sv[1][1]);
        // O += P . V: B fragments of V [position][dim] through ldmatrix.trans
#pragma unroll
        for (int dn = 0; dn < 8; dn++) {            // 16 dims per ldmatrix.x4
            const int i = lane >> 3;
            uint32_t b[4];
            ldsm_x4_t(vb + dc_off(p0 + (lane & 7) + 8 * (i & 1), 16 * dn + 8 * (i >> 1)), b);
            mma_bf16_16816(o[2 * dn], pa0, pa2, b[0], b[1]);
            mma_bf16_16816(o[2 * dn + 1], pa0, pa2, b[2], b[3]);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
        // refill this stage with tile + STAGES once every warp has released it
        if (threadIdx.x == 0 && tile + DC_STAGES < n_tiles) {
            if (!mbar_wait(&empty[st], par)) ok = false;
            else issue(tile + DC_STAGES);
        }
    }
    // Copies issued but never consumed (only after an expired wait): let them land.
    if (!ok && threadIdx.x == 0)
        for (int i = 0; i < min(DC_STAGES, n_tiles); i++) mbar_wait(&full[i], 0);

    if (g < 2) {
        if (tq == 0) { wm[warp][g] = m_r; wl[warp][g] = l_r; }
#pragma unroll
        for (int nt = 0; nt < 16; nt++) {
            wo[warp][g][8 * nt + 2 * tq] = o[nt][0];
            wo[warp][g][8 * nt + 2 * tq + 1] = o[nt][1];
        }
    }
    __syncthreads();

    for (int i = threadIdx.x; i < 2 * HD; i += DC_THREADS) {
        const int h = i >> 7, d = i & 127;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < DC_WARPS; w++) M = fmaxf(M, wm[w][h]);
        float L = 0.f, O = 0.f;
#pragma unroll
        for (int w = 0; w < DC_WARPS; w++) {
            const float f = (wm[w][h] == -INFINITY) ? 0.f : exp2f(wm[w][h] - M);
            L += wl[w][h] * f;
            O += wo[w][h][d] * f;
        }
        const int head = kvh * 2 + h;
        if (eff == 1) {
            p.out[(size_t)s * p.ldo + head * HD + d] = f32_to_bf16_rne(O / L);
        } else {
            const size_t slot = ((size_t)s * 16 + head) * p.splits + split;
            p.part_o[slot * HD + d] = O;
            if (d == 0) { p.part_m[slot] = M; p.part_l[slot] = L; }
        }
    }
    if (eff == 1 || !p.counters) return;
    // The CTA that completes this (sequence, KV head) merges the splits of its
    // two heads, in split order (the combine kernel's arithmetic).
    __shared__ int last;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        int *ctr = p.counters + s * NKV + kvh;
        last = atomicAdd(ctr, 1) == eff - 1;
        if (last) {
            *ctr = 0;                              // ready for the next call
            __threadfence();
        }
    }
    __syncthreads();
    if (!last) return;
    for (int i = threadIdx.x; i < 2 * HD; i += DC_THREADS) {
        const int head = kvh * 2 + (i >> 7), d = i & 127;
        const size_t slot0 = ((size_t)s * 16 + head) * p.splits;
        float M = -INFINITY;
        for (int k = 0; k < eff; k++) M = fmaxf(M, __ldcg(p.part_m + slot0 + k));
        float L = 0.f, O = 0.f;
        for (int k = 0; k < eff; k++) {
            const float mi = __ldcg(p.part_m + slot0 + k);
            const float f = (mi == -INFINITY) ? 0.f : exp2f(mi - M);
            L += __ldcg(p.part_l + slot0 + k) * f;
            O += __ldcg(p.part_o + (slot0 + k) * HD + d) * f;
        }
        p.out[(size_t)s * p.ldo + head * HD + d] = f32_to_bf16_rne(O / L);
    }
}

__global__ void attn_combine_kernel(AttnDecodeArgs p) {
    dep_wait();
    dep_launch();
    const int head = blockIdx.x, s = blockIdx.y, d = threadIdx.x;
    const size_t slot0 = ((size_t)s * 16 + head) * p.splits;
    float M = -INFINITY;
    for (int i = 0; i < p.splits; i++) M = fmaxf(M, p.part_m[slot0 + i]);
    float L = 0.f, O = 0.f;
    for (int i = 0; i < p.splits; i++) {
        const float mi = p.part_m[slot0 + i];
        const float f = (mi == -INFINITY) ? 0.f : exp2f(mi - M);
        L += p.part_l[slot0 + i] * f;
        O += p.part_o[(slot0 + i) * HD + d] * f;
    }
    p.out[(size_t)s * p.ldo + head * HD + d] = f32_to_bf16_rne(O / L);
}

}  // namespace

int attn_decode_splits(int n_seqs, int max_kv_len, int max_splits) {
    // Split the positions only when the (sequence, KV head) CTAs would leave
    // more than half of the 148 SMs idle: from 10 sequences up one CTA per
    // pair streams its positions faster than split CTAs plus the combine
    // kernel (measured on B200 at 16-256 sequences x 1024 positions). Split CTAs
    // cover the SMs twice (2 resident per SM); splits are rounded to whole
    // 64-position tiles inside the kernel.
    if (2 * n_seqs * NKV > 148) return 1;
    int splits = (2 * 148 + n_seqs * NKV - 1) / (n_seqs * NKV);
    const int by_len = (max_kv_len + 63) / 64;
    if (splits > by_len) splits = by_len;
    if (splits > max_splits) splits = max_splits;
    return splits < 1 ? 1 : splits;
}

int launch_attn_decode(cudaStream_t st, const AttnDecodeArgs &a, int n_seqs) {
    if (n_seqs <= 0) return N550_OK;
    if (a.splits < 1) return N550_ERR_ARG;
    if (a.splits > 1 && (!a.part_m || !a.part_l || !a.part_o)) return N550_ERR_ARG;
    if (a.kv_planes < 1) return N550_ERR_ARG;
    static bool dc_attr[64];
    int dev = 0;
    N550_CUDA_TRY(cudaGetDevice(&dev));
    if (dev >= 0 && dev < 64 && !dc_attr[dev]) {
        N550_CUDA_TRY(cudaFuncSetAttribute(attn_decode_kernel,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, DC_SMEM));
        dc_attr[dev] = true;
    }
    // K and V as [planes][max_len][128] with 64 x 64 boxes (two per tile row)
    CUtensorMap tk, tv;
    int rc = tmap_bf16_sw128_3d(&tk, a.kc, (uint64_t)a.max_len, HD, HD, DC_TP, (uint64_t)a.kv_planes,
                                (uint64_t)a.max_len * HD);
    if (!rc) rc = tmap_bf16_sw128_3d(&tv, a.vc, (uint64_t)a.max_len, HD, HD, DC_TP, (uint64_t)a.kv_planes,
                                     (uint64_t)a.max_len * HD);
    if (rc) return rc;
    dim3 grid(a.splits, NKV, n_seqs);
    N550_CUDA_TRY(launch_k(attn_decode_kernel, grid, DC_THREADS, DC_SMEM, st, tk, tv, a));
    N550_LAUNCH_CHECK();
    if (a.splits > 1 && !a.counters) {
        N550_CUDA_TRY(launch_k(attn_combine_kernel, dim3(16, n_seqs), HD, 0, st, a));
        N550_LAUNCH_CHECK();
    }
    return N550_OK;
}

}  // namespace n550
