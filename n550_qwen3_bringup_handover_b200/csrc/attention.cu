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
// This file is the decode side: one query per sequence, split-KV on CUDA
// cores fed by a bulk-copy shared-memory ring; the partial (max, sum, out) of
// each split are merged by a combine kernel. Prefill runs on the tcgen05
// tensor cores (attn_prefill_tc.cu).
#include "attention.h"
#include "common.cuh"
#include "launch.h"

namespace n550 {
namespace {

constexpr int HD = 128;
constexpr int NKV = 8;
constexpr int NL = 28;
constexpr float kScale = 0.08838834764831845f;     // qwen3.c:296
constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ size_t kv_base(int seq, int layer, int kvh, int max_len) {
    return ((size_t)(seq * NL + layer) * NKV + kvh) * (size_t)max_len * HD;
}

// ---------------------------------------------------------------------------
// decode (CUDA cores, split-KV)
// ---------------------------------------------------------------------------
constexpr int DC_THREADS = 256;     // 8 warps
constexpr int DC_WARPS = DC_THREADS / 32;
constexpr int DC_TP = 64;           // positions per tile
constexpr int DC_PPW = DC_TP / DC_WARPS;     // positions of a tile per warp (8)
constexpr int DC_PASSES = DC_PPW / 4;        // 4 positions (8 lanes each) per pass
static_assert(DC_PASSES * 4 == DC_PPW, "whole passes per warp");
constexpr int DC_STAGES = 3;        // tiles in flight per CTA
constexpr int DC_TILE_BYTES = DC_TP * HD * 2;   // 16 KB of K (and of V)
constexpr int DC_SMEM = DC_STAGES * 2 * DC_TILE_BYTES + 1024;

__device__ __forceinline__ void bf16x8(const uint4 q, float (&f)[8]) {
    f[0] = __uint_as_float(q.x << 16); f[1] = __uint_as_float(q.x & 0xFFFF0000u);
    f[2] = __uint_as_float(q.y << 16); f[3] = __uint_as_float(q.y & 0xFFFF0000u);
    f[4] = __uint_as_float(q.z << 16); f[5] = __uint_as_float(q.z & 0xFFFF0000u);
    f[6] = __uint_as_float(q.w << 16); f[7] = __uint_as_float(q.w & 0xFFFF0000u);
}

// One CTA per (split, kv head, sequence). K and V tiles of 64 positions
// (16 KB each, contiguous in the cache) stream through a 3-stage shared
// ring by bulk copies; warp w owns positions 8w..8w+7 of every tile and
// keeps its own online-softmax state, merged with the others at the end.
// Eight warps per CTA (two CTAs per SM) keep enough independent work in
// flight to stream the cache near HBM speed even when there are fewer CTAs
// than SM slots (small decode batches).
__global__ void __launch_bounds__(DC_THREADS)
attn_decode_kernel(AttnDecodeArgs p) {
    extern __shared__ __align__(128) uint8_t dsm[];
    uint8_t *ring = (uint8_t *)(((uintptr_t)dsm + 127) & ~(uintptr_t)127);
    uint64_t *full = (uint64_t *)(ring + DC_STAGES * 2 * DC_TILE_BYTES);
    uint64_t *empty = full + DC_STAGES;
    __shared__ __align__(16) float ps[DC_WARPS][2][DC_PPW];
    __shared__ float wm[DC_WARPS][2], wl[DC_WARPS][2];
    __shared__ __align__(16) float wo[DC_WARPS][2][HD];

    dep_wait();
    dep_launch();
    const int split = blockIdx.x, kvh = blockIdx.y, s = blockIdx.z;
    const int seq = p.seq_ids[s];
    const int kv_len = p.pos[s] + 1;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int chunk = (kv_len + p.splits - 1) / p.splits;
    chunk = (chunk + DC_TP - 1) / DC_TP * DC_TP;
    const int start = split * chunk, end = min(kv_len, start + chunk);
    const int n_tiles = end > start ? (end - start + DC_TP - 1) / DC_TP : 0;
    const uint16_t *kbase = p.kc + kv_base(seq, p.layer, kvh, p.max_len);
    const uint16_t *vbase = p.vc + kv_base(seq, p.layer, kvh, p.max_len);

    if (threadIdx.x == 0) {
        for (int i = 0; i < DC_STAGES; i++) { mbar_init(&full[i], 1); mbar_init(&empty[i], DC_WARPS); }
        fence_mbar_init();
    }
    __syncthreads();
    auto issue = [&](int tile) {
        const int st = tile % DC_STAGES;
        const int t0 = start + tile * DC_TP;
        const uint32_t bytes = (uint32_t)min(DC_TP, end - t0) * HD * 2;
        uint8_t *kd = ring + st * 2 * DC_TILE_BYTES;
        mbar_arrive_expect_tx(&full[st], 2 * bytes);
        bulk_load(kd, kbase + (size_t)t0 * HD, bytes, &full[st]);
        bulk_load(kd + DC_TILE_BYTES, vbase + (size_t)t0 * HD, bytes, &full[st]);
    };
    if (threadIdx.x == 0)
        for (int i = 0; i < min(DC_STAGES, n_tiles); i++) issue(i);

    // q . k: 8 lanes per position, lane g8 = lane & 7 owns dims 16*g8 .. +15.
    const int g8 = lane & 7;
    float q0[16], q1[16];
    {
        const size_t qo = (size_t)s * p.ldq + (size_t)(kvh * 2) * HD + 16 * g8;
#pragma unroll
        for (int j = 0; j < 16; j++) {
            const float a = p.q_f32 ? p.q_f32[qo + j] : bf16_bits_to_f32(p.q_bf16[qo + j]);
            const float b = p.q_f32 ? p.q_f32[qo + HD + j] : bf16_bits_to_f32(p.q_bf16[qo + HD + j]);
            q0[j] = a * (kScale * kLog2e);
            q1[j] = b * (kScale * kLog2e);
        }
    }
    float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
    float acc[2][4] = {};                 // p . v: lane owns dims 4*lane .. +3
    bool ok = true;

    for (int tile = 0; tile < n_tiles && ok; tile++) {
        const int st = tile % DC_STAGES;
        const uint32_t par = (uint32_t)((tile / DC_STAGES) & 1);
        if (!mbar_wait(&full[st], par)) { ok = false; break; }
        const uint8_t *kt = ring + st * 2 * DC_TILE_BYTES;
        const uint8_t *vt = kt + DC_TILE_BYTES;
        const int t0 = start + tile * DC_TP + warp * DC_PPW;    // this warp's first position
        float sc[2][DC_PASSES];
#pragma unroll
        for (int pass = 0; pass < DC_PASSES; pass++) {
            const int r = warp * DC_PPW + pass * 4 + (lane >> 3);  // row in the tile
            const uint4 *kr = (const uint4 *)(kt + r * (HD * 2) + 32 * g8);
            float kf[16];
            bf16x8(kr[0], *(float(*)[8])kf);
            bf16x8(kr[1], *(float(*)[8])(kf + 8));
            float a0 = 0.f, a1 = 0.f;
#pragma unroll
            for (int j = 0; j < 16; j++) { a0 = fmaf(q0[j], kf[j], a0); a1 = fmaf(q1[j], kf[j], a1); }
#pragma unroll
            for (int o = 4; o > 0; o >>= 1) {
                a0 += __shfl_xor_sync(0xFFFFFFFFu, a0, o);
                a1 += __shfl_xor_sync(0xFFFFFFFFu, a1, o);
            }
            const bool valid = t0 + pass * 4 + (lane >> 3) < end;
            sc[0][pass] = valid ? a0 : -INFINITY;
            sc[1][pass] = valid ? a1 : -INFINITY;
        }
        // online softmax over this warp's DC_PPW positions (DC_PASSES per lane group)
#pragma unroll
        for (int h = 0; h < 2; h++) {
            float mx = sc[h][0];
#pragma unroll
            for (int pass = 1; pass < DC_PASSES; pass++) mx = fmaxf(mx, sc[h][pass]);
            mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, 8));
            mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, 16));
            const float mn = fmaxf(m[h], mx);
            const float c = (mn == -INFINITY) ? 1.f : exp2f(m[h] - mn);
            float sum = 0.f;
#pragma unroll
            for (int pass = 0; pass < DC_PASSES; pass++) {
                const float e = (sc[h][pass] == -INFINITY) ? 0.f : exp2f(sc[h][pass] - mn);
                sc[h][pass] = e;
                sum += e;
            }
            sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 8);
            sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 16);
            l[h] = l[h] * c + sum;
            m[h] = mn;
#pragma unroll
            for (int d = 0; d < 4; d++) acc[h][d] *= c;
        }
        if (g8 == 0) {
#pragma unroll
            for (int pass = 0; pass < DC_PASSES; pass++) {
                ps[warp][0][pass * 4 + (lane >> 3)] = sc[0][pass];
                ps[warp][1][pass * 4 + (lane >> 3)] = sc[1][pass];
            }
        }
        __syncwarp();
        const int nvalid = min(DC_PPW, end - t0);
        for (int j = 0; j < nvalid; j++) {
            const uint2 v2 = *(const uint2 *)(vt + (warp * DC_PPW + j) * (HD * 2) + 8 * lane);
            const float w0 = ps[warp][0][j], w1 = ps[warp][1][j];
            const float v0 = __uint_as_float(v2.x << 16), v1 = __uint_as_float(v2.x & 0xFFFF0000u);
            const float v2f = __uint_as_float(v2.y << 16), v3 = __uint_as_float(v2.y & 0xFFFF0000u);
            acc[0][0] = fmaf(w0, v0, acc[0][0]); acc[0][1] = fmaf(w0, v1, acc[0][1]);
            acc[0][2] = fmaf(w0, v2f, acc[0][2]); acc[0][3] = fmaf(w0, v3, acc[0][3]);
            acc[1][0] = fmaf(w1, v0, acc[1][0]); acc[1][1] = fmaf(w1, v1, acc[1][1]);
            acc[1][2] = fmaf(w1, v2f, acc[1][2]); acc[1][3] = fmaf(w1, v3, acc[1][3]);
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

    if (lane == 0) { wm[warp][0] = m[0]; wm[warp][1] = m[1]; wl[warp][0] = l[0]; wl[warp][1] = l[1]; }
#pragma unroll
    for (int d = 0; d < 4; d++) { wo[warp][0][4 * lane + d] = acc[0][d]; wo[warp][1][4 * lane + d] = acc[1][d]; }
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
        if (p.splits == 1) {
            p.out[(size_t)s * p.ldo + head * HD + d] = f32_to_bf16_rne(O / L);
        } else {
            const size_t slot = ((size_t)s * 16 + head) * p.splits + split;
            p.part_o[slot * HD + d] = O;
            if (d == 0) { p.part_m[slot] = M; p.part_l[slot] = L; }
        }
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
    // Enough CTAs to cover the SMs twice (2 resident per SM); splits are
    // rounded to whole 64-position tiles inside the kernel.
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
    static bool dc_attr[64];
    int dev = 0;
    N550_CUDA_TRY(cudaGetDevice(&dev));
    if (dev >= 0 && dev < 64 && !dc_attr[dev]) {
        N550_CUDA_TRY(cudaFuncSetAttribute(attn_decode_kernel,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, DC_SMEM));
        dc_attr[dev] = true;
    }
    dim3 grid(a.splits, NKV, n_seqs);
    N550_CUDA_TRY(launch_k(attn_decode_kernel, grid, DC_THREADS, DC_SMEM, st, a));
    N550_LAUNCH_CHECK();
    if (a.splits > 1) {
        N550_CUDA_TRY(launch_k(attn_combine_kernel, dim3(16, n_seqs), HD, 0, st, a));
        N550_LAUNCH_CHECK();
    }
    return N550_OK;
}

}  // namespace n550
