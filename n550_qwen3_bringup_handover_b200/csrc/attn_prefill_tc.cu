// Prefill attention on the 5th-generation tensor cores (tcgen05, TMEM, TMA).
//
// Reference semantics (qwen3.c:374-436): for query position p and head h (KV
// head h/2, qwen3.c:299), s_t = (q . k_t) * 0.08838834764831845 for
// t = 0..p, softmax over t, out = sum_t softmax_t * v_t.
//
// One CTA = 128 consecutive queries of one sequence x the two query heads of
// one KV head (the GQA pair), so each 128-key K/V block is read once for both
// heads.
//   warp 0     TMA producer: Q of both heads once, then K and V blocks into a
//              2-stage ring (128-byte swizzle; V is the MN-major B operand).
//   warp 1     allocates TMEM (512 columns); one thread issues the MMAs:
//              S_h = Q_h K^T (A and B in shared memory) and O_h += P_h V
//              (A = P read from TMEM, B = V from shared memory).
//   warps 2-5  softmax and output of head 0, warps 6-9 of head 1; a thread
//              owns one query row. Scores are taken in the log2 domain; P is
//              written back into TMEM over its S as packed BF16. O is rescaled
//              in TMEM only when a row's running maximum grows by more than 8
//              (a factor 256): the exponentials use the stale maximum
//              otherwise, which leaves O / l unchanged.
// MMA issue order S0(0) S1(0) | PV0(j) S0(j+1) PV1(j) S1(j+1) | ... keeps the
// tensor core on one head while the other head's softmax runs.
// TMEM columns: S0/P0 [0,128), S1/P1 [128,256), O0 [256,384), O1 [384,512).
// Every wait is bounded and reports N550_ERR_TIMEOUT through the device status
// word.
#include <cuda.h>

#include "attention.h"
#include "common.cuh"
#include "tmap.h"

namespace n550 {
namespace {

constexpr int HD = 128;
constexpr int NKV = 8;
constexpr int NL = 28;
constexpr int BQ = 128;                      // queries per CTA (per head)
constexpr int BKV = 128;                     // keys per block
constexpr int THREADS = 320;                 // 10 warps
constexpr int TILE_BYTES = 128 * HD * 2;     // 32 KB: 128 rows x 128 BF16
constexpr int HALF_BYTES = TILE_BYTES / 2;   // one 64-column TMA box (16 KB)
constexpr int STAGES = 2;
constexpr int SMEM_BYTES = (2 + 2 * STAGES) * TILE_BYTES + 1024 + 256;
constexpr float kScaleLog2 = 0.08838834764831845f * 1.4426950408889634f;   // qwen3.c:296
constexpr float kRescale = 8.0f;

struct PfParams {
    uint16_t *out;
    const int32_t *seq_ids;
    int ldo, L, pos0, layer, max_len, n_qblocks;
};

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// (lo, hi) -> packed BF16x2, round to nearest even.
__device__ __forceinline__ uint32_t cvt_bf16x2(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

// All 32 lanes wait; the result is warp-uniform so that the .sync.aligned
// tcgen05 loads/stores after it run converged.
__device__ __forceinline__ bool warp_wait(uint64_t *bar, uint32_t parity) {
    const bool ok = mbar_wait(bar, parity);
    return __all_sync(0xFFFFFFFFu, ok);
}

__device__ __forceinline__ void tmem_ld_row128(uint32_t taddr, uint32_t (&r)[128]) {
    uint32_t(&r0)[32] = *reinterpret_cast<uint32_t(*)[32]>(&r[0]);
    uint32_t(&r1)[32] = *reinterpret_cast<uint32_t(*)[32]>(&r[32]);
    uint32_t(&r2)[32] = *reinterpret_cast<uint32_t(*)[32]>(&r[64]);
    uint32_t(&r3)[32] = *reinterpret_cast<uint32_t(*)[32]>(&r[96]);
    tmem_ld_32x32b_x32(taddr, r0);
    tmem_ld_32x32b_x32(taddr + 32, r1);
    tmem_ld_32x32b_x32(taddr + 64, r2);
    tmem_ld_32x32b_x32(taddr + 96, r3);
    tmem_ld_wait();
}

__global__ void __launch_bounds__(THREADS, 1)
attn_prefill_tc_kernel(const __grid_constant__ CUtensorMap tmQ,
                       const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, const PfParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *base = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t *sQ = base;                              // [2 heads][TILE]
    uint8_t *sKV = base + 2 * TILE_BYTES;            // [STAGES][K TILE | V TILE]
    uint64_t *bars = (uint64_t *)(base + (2 + 2 * STAGES) * TILE_BYTES);
    uint64_t *q_full = bars;          // [1]
    uint64_t *k_full = bars + 1;      // [STAGES]
    uint64_t *v_full = bars + 3;      // [STAGES]
    uint64_t *kv_empty = bars + 5;    // [STAGES]
    uint64_t *s_full = bars + 7;      // [2 heads]
    uint64_t *p_full = bars + 9;      // [2 heads]
    uint64_t *o_full = bars + 11;     // [2 heads]
    uint64_t *done = bars + 13;       // [1]
    uint32_t *tmem_slot = (uint32_t *)(bars + 14);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int qb = p.n_qblocks - 1 - (int)blockIdx.x;   // longest rows first
    const int kvh = blockIdx.y, s = blockIdx.z;
    const int seq = p.seq_ids[s];
    const int q0 = qb * BQ;
    const int q_last = min(p.L, q0 + BQ) - 1;
    const int nblk = (p.pos0 + q_last) / BKV + 1;       // key blocks 0..nblk-1
    const int plane = (seq * NL + p.layer) * NKV + kvh;  // (slot, layer, kv head)

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int i = 0; i < 2; i++) {
            mbar_init(&k_full[i], 1);
            mbar_init(&v_full[i], 1);
            mbar_init(&kv_empty[i], 1);
            mbar_init(&s_full[i], 1);
            mbar_init(&p_full[i], 128);
            mbar_init(&o_full[i], 1);
        }
        mbar_init(done, 1);
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmQ);
        tma_prefetch_desc(&tmK);
        tma_prefetch_desc(&tmV);
    }
    if (warp == 1) { tmem_alloc(tmem_slot, 512); tmem_relinquish(); }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            mbar_arrive_expect_tx(q_full, 2 * TILE_BYTES);
            for (int h = 0; h < 2; h++)
                for (int half = 0; half < 2; half++)
                    tma_load_3d(sQ + h * TILE_BYTES + half * HALF_BYTES, &tmQ, q_full,
                                (2 * kvh + h) * HD + half * 64, q0, s);
            int issued = 0;
            for (int j = 0; j < nblk; j++) {
                const int st = j & 1;
                if (!mbar_wait(&kv_empty[st], ((j >> 1) & 1) ^ 1)) break;
                uint8_t *sK = sKV + st * 2 * TILE_BYTES;
                uint8_t *sV = sK + TILE_BYTES;
                // Positions at or beyond pos0 + L are outside the map: zeros.
                const int row = j * BKV;
                mbar_arrive_expect_tx(&k_full[st], TILE_BYTES);
                tma_load_3d(sK, &tmK, &k_full[st], 0, row, plane);
                tma_load_3d(sK + HALF_BYTES, &tmK, &k_full[st], 64, row, plane);
                mbar_arrive_expect_tx(&v_full[st], TILE_BYTES);
                tma_load_3d(sV, &tmV, &v_full[st], 0, row, plane);
                tma_load_3d(sV + HALF_BYTES, &tmV, &v_full[st], 64, row, plane);
                issued = j + 1;
            }
            // Drain: every load issued must have landed before the CTA exits.
            mbar_wait(q_full, 0);
            for (int j = issued > STAGES ? issued - STAGES : 0; j < issued; j++) {
                mbar_wait(&k_full[j & 1], (j >> 1) & 1);
                mbar_wait(&v_full[j & 1], (j >> 1) & 1);
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            constexpr uint32_t id_s = umma_idesc_bf16(128, 128);
            constexpr uint32_t id_o = umma_idesc_bf16(128, 128) | (1u << 16);   // V MN-major
            const uint32_t aQ = smem_u32(sQ), aKV = smem_u32(sKV);
            // S_t = Q_t . K^T over the 128 head dimensions (8 x K=16).
            auto issue_s = [&](int t, int st) {
                const uint32_t q = aQ + t * TILE_BYTES, k = aKV + st * 2 * TILE_BYTES;
#pragma unroll
                for (int kk = 0; kk < 8; kk++) {
                    const uint32_t off = (kk >> 2) * HALF_BYTES + (kk & 3) * 32;
                    umma_bf16(tmem + t * 128, umma_desc_sw128(q + off), umma_desc_sw128(k + off),
                              id_s, kk > 0 ? 1u : 0u);
                }
                umma_commit(&s_full[t]);
            };
            bool ok = mbar_wait(q_full, 0) && mbar_wait(&k_full[0], 0);
            if (ok) {
                tc_fence_after();
                issue_s(0, 0);
                issue_s(1, 0);
            }
            for (int j = 0; j < nblk && ok; j++) {
                const int st = j & 1;
                const uint32_t v = aKV + st * 2 * TILE_BYTES + TILE_BYTES;
                for (int t = 0; t < 2; t++) {
                    if (!(ok = mbar_wait(&p_full[t], j & 1))) break;
                    if (t == 0 && !(ok = mbar_wait(&v_full[st], (j >> 1) & 1))) break;
                    tc_fence_after();
                    // O_t += P_t . V over the 128 keys of the block (8 x K=16):
                    // P columns 8 kk .. 8 kk + 7, V rows 16 kk .. 16 kk + 15.
#pragma unroll
                    for (int kk = 0; kk < 8; kk++)
                        umma_bf16_ts(tmem + 256 + t * 128, tmem + t * 128 + kk * 8,
                                     umma_desc_sw128_mn(v + kk * 2048, HALF_BYTES), id_o,
                                     (j > 0 || kk > 0) ? 1u : 0u);
                    if (t == 1) umma_commit(&kv_empty[st]);
                    if (j + 1 < nblk) {
                        if (t == 0 && !(ok = mbar_wait(&k_full[st ^ 1], ((j + 1) >> 1) & 1))) break;
                        tc_fence_after();
                        issue_s(t, st ^ 1);
                    } else {
                        umma_commit(&o_full[t]);
                    }
                }
            }
            // Drain all MMAs of this thread before TMEM is released.
            umma_commit(done);
            mbar_wait(done, 0);
        }
    } else {
        // ---------------- softmax + output (warps 2..9) ----------------
        const int t = (warp - 2) >> 2;                  // head of the GQA pair
        const int qw = warp & 3;                        // TMEM lane quarter
        const int row = qw * 32 + lane;                 // query row in the block
        const int qpos = p.pos0 + q0 + row;
        const uint32_t lane_off = (uint32_t)(qw * 32) << 16;
        const uint32_t tS = tmem + lane_off + t * 128;
        const uint32_t tO = tmem + lane_off + 256 + t * 128;
        float m_run = -INFINITY, l_run = 0.f;
        bool ok = true;
        for (int j = 0; j < nblk; j++) {
            if (!(ok = warp_wait(&s_full[t], j & 1))) break;
            tc_fence_after();
            uint32_t r[128];
            tmem_ld_row128(tS, r);
            const int k0 = j * BKV;
            if (k0 + BKV - 1 > p.pos0 + q0) {           // the block crosses the diagonal
#pragma unroll
                for (int i = 0; i < 128; i++)
                    if (k0 + i > qpos) r[i] = 0xFF800000u;   // -inf
            }
            float mx0 = -INFINITY, mx1 = -INFINITY, mx2 = -INFINITY, mx3 = -INFINITY;
#pragma unroll
            for (int i = 0; i < 128; i += 4) {
                mx0 = fmaxf(mx0, __uint_as_float(r[i]));
                mx1 = fmaxf(mx1, __uint_as_float(r[i + 1]));
                mx2 = fmaxf(mx2, __uint_as_float(r[i + 2]));
                mx3 = fmaxf(mx3, __uint_as_float(r[i + 3]));
            }
            const float mx = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3)) * kScaleLog2;
            float m_use = m_run;
            bool resc = false;
            if (j == 0) {
                m_use = mx;
            } else if (mx > m_run + kRescale) {
                m_use = mx;
                resc = true;
            }
            const float corr = resc ? ex2(m_run - m_use) : 1.0f;
            float l0 = 0.f, l1 = 0.f;
            uint32_t pk[64];
#pragma unroll
            for (int c = 0; c < 64; c++) {
                const float a = ex2(fmaf(__uint_as_float(r[2 * c]), kScaleLog2, -m_use));
                const float b = ex2(fmaf(__uint_as_float(r[2 * c + 1]), kScaleLog2, -m_use));
                l0 += a;
                l1 += b;
                pk[c] = cvt_bf16x2(a, b);
            }
            tmem_st_32x32b_x32(tS, *reinterpret_cast<uint32_t(*)[32]>(&pk[0]));
            tmem_st_32x32b_x32(tS + 32, *reinterpret_cast<uint32_t(*)[32]>(&pk[32]));
            l_run = l_run * corr + (l0 + l1);
            m_run = m_use;
            if (__any_sync(0xFFFFFFFFu, resc)) {
                // O_t holds blocks 0..j-1 (complete: s_full(j) was committed
                // after PV_t(j-1)); PV_t(j) is not issued before p_full.
#pragma unroll 1
                for (int c = 0; c < 4; c++) {
                    uint32_t o[32];
                    tmem_ld_32x32b_x32(tO + 32 * c, o);
                    tmem_ld_wait();
#pragma unroll
                    for (int i = 0; i < 32; i++) o[i] = __float_as_uint(__uint_as_float(o[i]) * corr);
                    tmem_st_32x32b_x32(tO + 32 * c, o);
                }
            }
            tmem_st_wait();
            tc_fence_before();
            mbar_arrive(&p_full[t]);
        }
        if (ok) ok = warp_wait(&o_full[t], 0);
        if (ok) {
            tc_fence_after();
            const float inv = 1.0f / l_run;
            // Stage the BF16 row in this head's Q tile (no longer read: every
            // S_t MMA completed before o_full), 16-byte chunk cc of row r at
            // chunk cc ^ (r & 7), then store whole rows.
            uint8_t *stg = sQ + t * TILE_BYTES;
#pragma unroll 1
            for (int c = 0; c < 4; c++) {
                uint32_t o[32];
                tmem_ld_32x32b_x32(tO + 32 * c, o);
                tmem_ld_wait();
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    const int cc = c * 4 + k;
                    uint4 w;
                    w.x = cvt_bf16x2(__uint_as_float(o[8 * k]) * inv, __uint_as_float(o[8 * k + 1]) * inv);
                    w.y = cvt_bf16x2(__uint_as_float(o[8 * k + 2]) * inv, __uint_as_float(o[8 * k + 3]) * inv);
                    w.z = cvt_bf16x2(__uint_as_float(o[8 * k + 4]) * inv, __uint_as_float(o[8 * k + 5]) * inv);
                    w.w = cvt_bf16x2(__uint_as_float(o[8 * k + 6]) * inv, __uint_as_float(o[8 * k + 7]) * inv);
                    *(uint4 *)(stg + row * 256 + ((cc ^ (row & 7)) << 4)) = w;
                }
            }
            __syncwarp();
            const int head = 2 * kvh + t;
#pragma unroll 4
            for (int it = 0; it < 16; it++) {
                const int rr = qw * 32 + it * 2 + (lane >> 4), cc = lane & 15;
                const int qi = q0 + rr;
                if (qi < p.L) {
                    const uint4 w = *(const uint4 *)(stg + rr * 256 + ((cc ^ (rr & 7)) << 4));
                    *(uint4 *)(p.out + ((size_t)s * p.L + qi) * p.ldo + head * HD + cc * 8) = w;
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

bool g_attr[64];

}  // namespace

int launch_attn_prefill(cudaStream_t st, const AttnPrefillArgs &a, int n_seqs) {
    if (n_seqs <= 0 || a.L <= 0) return N550_OK;
    if (!a.q || !a.kc || !a.vc || !a.out || !a.seq_ids || a.pos0 < 0 || a.layer < 0 ||
        a.layer >= NL || a.max_len < a.pos0 + a.L || (a.ldq % 8) || (a.ldo % 8) ||
        a.ldq < 16 * HD || a.ldo < 16 * HD || ((uintptr_t)a.out & 15) || a.kv_planes <= 0 ||
        (long long)a.kv_planes * a.max_len * HD > (1LL << 40))
        return N550_ERR_ARG;
    // Q as [seq][L][ldq]; K and V as [plane][pos < pos0 + L][128], so that the
    // TMA reads zeros for query rows past L and for key positions past the
    // attended range instead of whatever the buffers hold there.
    CUtensorMap tq, tk, tv;
    int rc;
    const uint64_t kv_len = (uint64_t)(a.pos0 + a.L);
    if ((rc = tmap_bf16_sw128_3d(&tq, a.q, a.L, 16 * HD, a.ldq, BQ, n_seqs, (uint64_t)a.L * a.ldq)))
        return rc;
    if ((rc = tmap_bf16_sw128_3d(&tk, a.kc, kv_len, HD, HD, BKV, a.kv_planes, (uint64_t)a.max_len * HD)))
        return rc;
    if ((rc = tmap_bf16_sw128_3d(&tv, a.vc, kv_len, HD, HD, BKV, a.kv_planes, (uint64_t)a.max_len * HD)))
        return rc;
    int dev = 0;
    N550_CUDA_TRY(cudaGetDevice(&dev));
    if (dev >= 0 && dev < 64 && !g_attr[dev]) {
        N550_CUDA_TRY(cudaFuncSetAttribute(attn_prefill_tc_kernel,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
        g_attr[dev] = true;
    }
    PfParams p;
    p.out = a.out;
    p.seq_ids = a.seq_ids;
    p.ldo = a.ldo;
    p.L = a.L;
    p.pos0 = a.pos0;
    p.layer = a.layer;
    p.max_len = a.max_len;
    p.n_qblocks = (a.L + BQ - 1) / BQ;
    dim3 grid(p.n_qblocks, NKV, n_seqs);
    attn_prefill_tc_kernel<<<grid, THREADS, SMEM_BYTES, st>>>(tq, tk, tv, p);
    N550_LAUNCH_CHECK();
    return N550_OK;
}

}  // namespace n550
