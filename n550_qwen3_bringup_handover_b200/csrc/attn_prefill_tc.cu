// Prefill attention on the 5th-generation tensor cores (tcgen05, TMEM, TMA).
//
// Reference semantics (qwen3.c:374-436): for query position p and head h (KV
// head h/2, qwen3.c:299), s_t = (q . k_t) * 0.08838834764831845 for
// t = 0..p, softmax over t, out = sum_t softmax_t * v_t.
//
// Persistent kernel: one CTA per SM walks work items (longest first); an item
// is 128 consecutive queries of one sequence x the two query heads of one KV
// head (the GQA pair), so every 128-key K/V block is read once for both heads.
//   warp 0      TMA producer: Q of both heads per item, then K and V blocks
//               into a 2-stage ring (128-byte swizzle; V is consumed as the
//               MN-major B operand).
//   warp 1      allocates TMEM (512 columns) and issues the MMAs: the whole
//               warp walks the issue loop and one elected lane (elect.sync)
//               executes each tcgen05.mma, which keeps addresses and
//               descriptors warp-uniform (measured: 8 MMAs issued in ~460-700
//               cycles instead of ~740-850 from a lone lane-0 thread):
//               S_h = Q_h K^T (A and B in shared memory) and O_h += P_h V
//               (A = P read from TMEM, B = V from shared memory), in the order
//               S0 S1 | PV0(j) S0(j+1) PV1(j) S1(j+1) | ... so the tensor core
//               works on one head while the other head's softmax runs.
//   warps 2-17  softmax and output: 8 warps per head, a pair of warps per
//               32-row TMEM lane quarter, each warp owning 64 of the 128 key
//               columns of its rows (and 64 of the 128 output dimensions); the
//               pair exchanges row maxima and sums through shared memory
//               behind a 64-thread named barrier. Scores are in the log2
//               domain; P is written back into TMEM over its S as packed BF16;
//               O is rescaled in TMEM only when a row's running maximum grows
//               by more than 8 (a factor 256), otherwise the stale maximum is
//               kept, which leaves O / l unchanged.
// TMEM columns: S0/P0 [0,128), S1/P1 [128,256), O0 [256,384), O1 [384,512).
// Every wait is bounded and reports N550_ERR_TIMEOUT through the device status
// word.
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
constexpr int BQ = 128;                      // queries per item (per head)
constexpr int BKV = 128;                     // keys per block
constexpr int THREADS = 576;                 // 18 warps
constexpr int TILE_BYTES = 128 * HD * 2;     // 32 KB: 128 rows x 128 BF16
constexpr int HALF_BYTES = TILE_BYTES / 2;   // one 64-column TMA box (16 KB)
constexpr int STAGES = 2;
constexpr int XCH_BYTES = (2 * 2 * 2 * 128 + 2 * 2 * 128) * 4;   // row max (x2 parity) + row sum
constexpr int SMEM_BYTES = (2 + 2 * STAGES) * TILE_BYTES + XCH_BYTES + 1024 + 256;
static_assert(SMEM_BYTES <= 232448, "shared memory per CTA");
constexpr float kScaleLog2 = 0.08838834764831845f * 1.4426950408889634f;   // qwen3.c:296
constexpr float kRescale = 8.0f;

struct PfParams {
    uint16_t *out;
    const int32_t *seq_ids;
    int ldo, L, pos0, layer, max_len, n_qblocks, n_seqs, n_items;
    int snake;     // hand out every other round of items in reverse CTA order
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

// Named barrier over the two warps (64 threads) of a softmax pair.
__device__ __forceinline__ void pair_sync(int id) {
    asm volatile("bar.sync %0, 64;" ::"r"(id) : "memory");
}

template <int N>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, uint32_t (&r)[N]) {
#pragma unroll
    for (int c = 0; c < N / 32; c++)
        tmem_ld_32x32b_x32(taddr + 32 * c, *reinterpret_cast<uint32_t(*)[32]>(&r[32 * c]));
    tmem_ld_wait();
}

// Work item k (longest first): q block n_qblocks - 1 - k / (8 n_seqs), then
// KV head k % 8 of sequence n_seqs - 1 - (k % (8 n_seqs)) / 8.
struct Item {
    int s, kvh, q0, nblk, plane;
};

__device__ __forceinline__ Item decode_item(const PfParams &p, int k, bool with_plane = false) {
    Item it;
    const int per_q = NKV * p.n_seqs;
    const int qb = p.n_qblocks - 1 - k / per_q;
    const int rest = k % per_q;
    // last sequences first within a query block: the q/k/v GEMM wrote their
    // rows last, so they are still in L2 (attention 4.71 -> 4.60 ms per 64 x
    // 512-token prefill step on B200)
    it.s = p.n_seqs - 1 - rest / NKV;
    it.kvh = rest % NKV;
    it.q0 = qb * BQ;
    const int q_last = min(p.L, it.q0 + BQ) - 1;
    it.nblk = (p.pos0 + q_last) / BKV + 1;                      // key blocks 0..nblk-1
    // (slot, layer, kv head); only the producer needs it (a global load)
    it.plane = with_plane ? (p.seq_ids[it.s] * NL + p.layer) * NKV + it.kvh : 0;
    return it;
}

// The item after item k for this CTA: the next round of gridDim.x items in
// the longest-first order. With p.snake (few items per CTA: a prefill of a
// few sequences on one GPU) every other round is handed out in reverse CTA
// order, so that a CTA that took one of a round's longest items takes one of
// the next round's shortest and the CTAs finish closer together. Only the
// last round is partial, so an index past n_items ends the walk.
__device__ __forceinline__ int next_item(int k, const PfParams &p) {
    const int G = (int)gridDim.x;
    if (!p.snake) return k + G;
    const int r = k / G + 1, c = (int)blockIdx.x;
    return r * G + ((r & 1) ? G - 1 - c : c);
}

__global__ void __launch_bounds__(THREADS, 1)
attn_prefill_tc_kernel(const __grid_constant__ CUtensorMap tmQ,
                       const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, const PfParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *base = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t *sQ = base;                              // [2 heads][TILE]
    uint8_t *sKV = base + 2 * TILE_BYTES;            // [STAGES][K TILE | V TILE]
    float *xmax = (float *)(base + (2 + 2 * STAGES) * TILE_BYTES);   // [parity][head][half][row]
    float *xsum = xmax + 2 * 2 * 2 * 128;                             // [head][half][row]
    uint64_t *bars = (uint64_t *)((uint8_t *)xmax + XCH_BYTES);
    uint64_t *q_full = bars;          // [1]
    uint64_t *q_empty = bars + 1;     // [1] every S MMA of the item has read Q
    uint64_t *k_full = bars + 2;      // [STAGES]
    uint64_t *v_full = bars + 4;      // [STAGES]
    uint64_t *kv_empty = bars + 6;    // [STAGES]
    uint64_t *s_full = bars + 8;      // [2 heads]
    uint64_t *p_full = bars + 10;     // [2 heads]
    uint64_t *o_full = bars + 12;     // [2 heads] the item's last P.V done
    uint64_t *o_free = bars + 14;     // [2 heads] O read out of TMEM
    uint64_t *done = bars + 16;       // [1]
    uint32_t *tmem_slot = (uint32_t *)(bars + 17);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        mbar_init(q_empty, 1);
        for (int i = 0; i < 2; i++) {
            mbar_init(&k_full[i], 1);
            mbar_init(&v_full[i], 1);
            mbar_init(&kv_empty[i], 1);
            mbar_init(&s_full[i], 1);
            mbar_init(&p_full[i], 256);
            mbar_init(&o_full[i], 1);
            mbar_init(&o_free[i], 256);
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
    // the TMEM is held: the next kernel may start; q and the cache come from
    // the previous kernels
    dep_launch();
    dep_wait();

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            int kv_iter = 0, item_i = 0, q_loads = 0;
            bool ok = true;
            for (int k = blockIdx.x; k < p.n_items && ok; k = next_item(k, p), item_i++) {
                const Item it = decode_item(p, k, true);
                if (!(ok = mbar_wait(q_empty, (item_i & 1) ^ 1))) break;
                mbar_arrive_expect_tx(q_full, 2 * TILE_BYTES);
                q_loads++;
                for (int h = 0; h < 2; h++)
                    for (int half = 0; half < 2; half++)
                        tma_load_3d(sQ + h * TILE_BYTES + half * HALF_BYTES, &tmQ, q_full,
                                    (2 * it.kvh + h) * HD + half * 64, it.q0, it.s);
                // The next item's Q can only be loaded once this item's last S
                // MMA has read the buffer; bring it into L2 now so that load
                // does not wait on HBM.
                if (next_item(k, p) < p.n_items) {
                    const Item nx = decode_item(p, next_item(k, p));
                    for (int h = 0; h < 2; h++)
                        for (int half = 0; half < 2; half++)
                            tma_prefetch_3d(&tmQ, (2 * nx.kvh + h) * HD + half * 64, nx.q0, nx.s);
                }
                for (int j = 0; j < it.nblk; j++, kv_iter++) {
                    const int st = kv_iter & 1;
                    if (!(ok = mbar_wait(&kv_empty[st], ((kv_iter >> 1) & 1) ^ 1))) break;
                    uint8_t *sK = sKV + st * 2 * TILE_BYTES;
                    uint8_t *sV = sK + TILE_BYTES;
                    // Positions at or beyond pos0 + L are outside the map: zeros.
                    const int row = j * BKV;
                    mbar_arrive_expect_tx(&k_full[st], TILE_BYTES);
                    tma_load_3d(sK, &tmK, &k_full[st], 0, row, it.plane);
                    tma_load_3d(sK + HALF_BYTES, &tmK, &k_full[st], 64, row, it.plane);
                    mbar_arrive_expect_tx(&v_full[st], TILE_BYTES);
                    tma_load_3d(sV, &tmV, &v_full[st], 0, row, it.plane);
                    tma_load_3d(sV + HALF_BYTES, &tmV, &v_full[st], 64, row, it.plane);
                }
            }
            // Drain: every load issued must have landed before the CTA exits
            // (the last Q and the last two K/V stages; older ones were consumed).
            if (q_loads > 0) mbar_wait(q_full, (q_loads - 1) & 1);
            for (int j = kv_iter > STAGES ? kv_iter - STAGES : 0; j < kv_iter; j++) {
                mbar_wait(&k_full[j & 1], (j >> 1) & 1);
                mbar_wait(&v_full[j & 1], (j >> 1) & 1);
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        // The whole warp walks the loop and waits; one elected lane issues
        // each MMA and commit, so addresses and descriptors stay warp-uniform.
        {
            constexpr uint32_t id_s = umma_idesc_bf16(128, 128);
            constexpr uint32_t id_o = umma_idesc_bf16(128, 128) | (1u << 16);   // V MN-major
            const uint32_t aQ = smem_u32(sQ), aKV = smem_u32(sKV);
            // S_t = Q_t . K^T over the 128 head dimensions (8 x K=16).
            auto issue_s = [&](int t, int st) {
                const uint32_t q = aQ + t * TILE_BYTES, k = aKV + st * 2 * TILE_BYTES;
#pragma unroll
                for (int kk = 0; kk < 8; kk++) {
                    const uint32_t off = (kk >> 2) * HALF_BYTES + (kk & 3) * 32;
                    if (elect_one_sync())
                        umma_bf16(tmem + t * 128, umma_desc_sw128(q + off), umma_desc_sw128(k + off),
                                  id_s, kk > 0 ? 1u : 0u);
                }
                if (elect_one_sync()) umma_commit(&s_full[t]);
                __syncwarp();
            };
            int kv_iter = 0, item_i = 0, bj = 0;
            bool ok = true;
            for (int k = blockIdx.x; k < p.n_items && ok; k = next_item(k, p), item_i++) {
                const Item it = decode_item(p, k);
                // S columns are free: the previous item's P.V MMAs, which read
                // P there, were issued earlier and execute in order.
                if (!(ok = warp_wait(q_full, item_i & 1) && warp_wait(&k_full[kv_iter & 1], (kv_iter >> 1) & 1)))
                    break;
                tc_fence_after();
                issue_s(0, kv_iter & 1);
                issue_s(1, kv_iter & 1);
                if (it.nblk == 1 && elect_one_sync()) umma_commit(q_empty);
                __syncwarp();
                for (int j = 0; j < it.nblk && ok; j++, bj++) {
                    const int st = (kv_iter + j) & 1;
                    const uint32_t v = aKV + st * 2 * TILE_BYTES + TILE_BYTES;
                    for (int t = 0; t < 2; t++) {
                        if (!(ok = warp_wait(&p_full[t], bj & 1))) break;
                        if (t == 0 && !(ok = warp_wait(&v_full[st], ((kv_iter + j) >> 1) & 1))) break;
                        // the first P.V of an item overwrites O: the previous
                        // item's output must have been read out of TMEM
                        if (j == 0 && !(ok = warp_wait(&o_free[t], (item_i & 1) ^ 1))) break;
                        tc_fence_after();
                        // O_t += P_t . V over the 128 keys of the block (8 x K=16):
                        // P columns 8 kk .. 8 kk + 7, V rows 16 kk .. 16 kk + 15.
#pragma unroll
                        for (int kk = 0; kk < 8; kk++)
                            if (elect_one_sync())
                                umma_bf16_ts(tmem + 256 + t * 128, tmem + t * 128 + kk * 8,
                                             umma_desc_sw128_mn(v + kk * 2048, HALF_BYTES), id_o,
                                             (j > 0 || kk > 0) ? 1u : 0u);
                        if (t == 1 && elect_one_sync()) umma_commit(&kv_empty[st]);
                        __syncwarp();
                        if (j + 1 < it.nblk) {
                            if (t == 0 && !(ok = warp_wait(&k_full[st ^ 1], ((kv_iter + j + 1) >> 1) & 1)))
                                break;
                            tc_fence_after();
                            issue_s(t, st ^ 1);
                            if (t == 1 && j + 2 == it.nblk && elect_one_sync()) umma_commit(q_empty);
                            __syncwarp();
                        } else {
                            if (elect_one_sync()) umma_commit(&o_full[t]);
                            __syncwarp();
                        }
                    }
                }
                kv_iter += it.nblk;
            }
            // Drain all MMAs of this warp before TMEM is released.
            if (elect_one_sync()) umma_commit(done);
            __syncwarp();
            warp_wait(done, 0);
        }
    } else {
        // ---------------- softmax + output (warps 2..17) ----------------
        const int sw = warp - 2;
        const int t = sw >> 3;                          // head of the GQA pair
        const int half = (sw >> 2) & 1;                 // key columns / output dims 64*half..
        const int qw = warp & 3;                        // TMEM lane quarter
        const int row = qw * 32 + lane;                 // query row in the item
        const int bar_id = 1 + t * 4 + qw;              // this pair's named barrier
        const uint32_t lane_off = (uint32_t)(qw * 32) << 16;
        const uint32_t tS = tmem + lane_off + t * 128;  // S (and P) of head t, this lane quarter
        const uint32_t tO = tmem + lane_off + 256 + t * 128 + half * 64;
        float *my_sum = xsum + (t * 2 + half) * 128 + row;
        const float *other_sum = xsum + (t * 2 + (half ^ 1)) * 128 + row;
        int bj = 0;
        bool ok = true;
        for (int k = blockIdx.x, i = 0; k < p.n_items && ok; k = next_item(k, p), i++) {
            const Item it = decode_item(p, k);
            const int qpos = p.pos0 + it.q0 + row;
            float m_run = -INFINITY, l_run = 0.f;
            for (int j = 0; j < it.nblk; j++, bj++) {
                if (!(ok = warp_wait(&s_full[t], bj & 1))) break;
                tc_fence_after();
                // Causal mask: key column e of this half is valid for e <= lim.
                // lim grows with the lane, so each 32-column chunk is, for the
                // whole warp, all valid (state 0), all masked (1) or mixed (2).
                const int k0 = j * BKV;
                const bool diag = k0 + BKV - 1 > p.pos0 + it.q0;
                const int lim = qpos - k0 - half * 64;
                const int lim_lo = __shfl_sync(0xFFFFFFFFu, lim, 0);
                const int lim_hi = __shfl_sync(0xFFFFFFFFu, lim, 31);
                auto chunk_state = [&](int c) -> int {
                    if (!diag || 32 * c + 31 <= lim_lo) return 0;
                    return 32 * c > lim_hi ? 1 : 2;
                };
                // pass 1: maximum over this warp's 64 columns, 32 at a time
                float mx0 = -INFINITY, mx1 = -INFINITY, mx2 = -INFINITY, mx3 = -INFINITY;
#pragma unroll
                for (int c = 0; c < 2; c++) {
                    const int cs = chunk_state(c);
                    if (cs == 1) continue;
                    uint32_t v[32];
                    tmem_ld_32x32b_x32(tS + half * 64 + 32 * c, v);
                    tmem_ld_wait();
                    if (cs == 2) {
#pragma unroll
                        for (int e = 0; e < 32; e++)
                            if (32 * c + e > lim) v[e] = 0xFF800000u;   // -inf
                    }
#pragma unroll
                    for (int e = 0; e < 32; e += 4) {
                        mx0 = fmaxf(mx0, __uint_as_float(v[e]));
                        mx1 = fmaxf(mx1, __uint_as_float(v[e + 1]));
                        mx2 = fmaxf(mx2, __uint_as_float(v[e + 2]));
                        mx3 = fmaxf(mx3, __uint_as_float(v[e + 3]));
                    }
                }
                // Row maximum over both halves. The exchange slot alternates
                // with the block parity, so a slot is rewritten only after the
                // partner has passed the next barrier (and so read it). After
                // this barrier both warps have also finished reading the S
                // columns P overwrites (P of this half lands on S columns
                // 32*half.., read in pass 1 by half 0).
                float *xm = xmax + (((bj & 1) * 2 + t) * 2) * 128;
                xm[half * 128 + row] = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3));
                pair_sync(bar_id);
                const float mx = fmaxf(xm[row], xm[128 + row]) * kScaleLog2;
                float m_use = m_run;
                bool resc = false;
                if (j == 0) {
                    m_use = mx;
                } else if (mx > m_run + kRescale) {
                    m_use = mx;
                    resc = true;
                }
                const float corr = resc ? ex2(m_run - m_use) : 1.0f;
                // pass 2: P for keys 64*half + 32c .. +31 as 16 packed words at
                // P columns 32*half + 16c. Half 1's P overwrites S columns of
                // half 0's first chunk pair (32..63), which half 0 re-reads in
                // its own pass 2 -- so both halves re-read S before the second
                // barrier and write P only after it.
                uint32_t pk[2][16];
                float l0 = 0.f, l1 = 0.f;
#pragma unroll
                for (int c = 0; c < 2; c++) {
                    const int cs = chunk_state(c);
                    if (cs == 1) {
#pragma unroll
                        for (int e = 0; e < 16; e++) pk[c][e] = 0u;
                        continue;
                    }
                    uint32_t v[32];
                    tmem_ld_32x32b_x32(tS + half * 64 + 32 * c, v);
                    tmem_ld_wait();
#pragma unroll
                    for (int e = 0; e < 16; e++) {
                        float a = ex2(fmaf(__uint_as_float(v[2 * e]), kScaleLog2, -m_use));
                        float b = ex2(fmaf(__uint_as_float(v[2 * e + 1]), kScaleLog2, -m_use));
                        if (cs == 2) {
                            if (32 * c + 2 * e > lim) a = 0.f;
                            if (32 * c + 2 * e + 1 > lim) b = 0.f;
                        }
                        l0 += a;
                        l1 += b;
                        pk[c][e] = cvt_bf16x2(a, b);
                    }
                }
                pair_sync(bar_id);
                tmem_st_32x32b_x16(tS + half * 32, pk[0]);
                tmem_st_32x32b_x16(tS + half * 32 + 16, pk[1]);
                l_run = l_run * corr + (l0 + l1);
                m_run = m_use;
                if (__any_sync(0xFFFFFFFFu, resc)) {
                    // O_t holds blocks 0..j-1 (complete: s_full(j) was committed
                    // after PV_t(j-1)); PV_t(j) is not issued before p_full.
#pragma unroll 1
                    for (int c = 0; c < 2; c++) {
                        uint32_t o[32];
                        tmem_ld_32x32b_x32(tO + 32 * c, o);
                        tmem_ld_wait();
#pragma unroll
                        for (int e = 0; e < 32; e++) o[e] = __float_as_uint(__uint_as_float(o[e]) * corr);
                        tmem_st_32x32b_x32(tO + 32 * c, o);
                    }
                }
                tmem_st_wait();
                tc_fence_before();
                mbar_arrive(&p_full[t]);
            }
            if (ok) ok = warp_wait(&o_full[t], i & 1);
            if (!ok) break;
            tc_fence_after();
            // row sum over both halves; the slot is rewritten only an item later
            *my_sum = l_run;
            pair_sync(bar_id);
            const float inv = 1.0f / (l_run + *other_sum);
            // O / l of this row as BF16: 64 output dims = 8 chunks of 16 bytes
            uint32_t ch[8][4];
#pragma unroll
            for (int c = 0; c < 2; c++) {
                uint32_t o[32];
                tmem_ld_32x32b_x32(tO + 32 * c, o);
                tmem_ld_wait();
                if (c == 1) {
                    // O is read out: the next item's first P.V may overwrite it
                    tc_fence_before();
                    mbar_arrive(&o_free[t]);
                }
#pragma unroll
                for (int cc = 0; cc < 4; cc++)
#pragma unroll
                    for (int w = 0; w < 4; w++)
                        ch[c * 4 + cc][w] = cvt_bf16x2(__uint_as_float(o[8 * cc + 2 * w]) * inv,
                                                        __uint_as_float(o[8 * cc + 2 * w + 1]) * inv);
            }
            // Transpose the chunks within each group of 8 lanes (= 8 rows) in
            // three butterfly exchange stages, so that store k has lane 8g + j
            // write chunk j of row 8g + k: each store instruction covers four
            // whole 128-byte row pieces instead of 16 bytes of 32 rows (which
            // cost the L1 one pass per row).
            const int j8 = lane & 7;
#pragma unroll
            for (int m = 1; m < 8; m <<= 1) {
                const bool up = (j8 & m) != 0;
#pragma unroll
                for (int c = 0; c < 8; c++) {
                    if (c & m) continue;
#pragma unroll
                    for (int w = 0; w < 4; w++) {
                        const uint32_t send = up ? ch[c][w] : ch[c | m][w];
                        const uint32_t recv = __shfl_xor_sync(0xFFFFFFFFu, send, m);
                        if (up) ch[c][w] = recv;
                        else ch[c | m][w] = recv;
                    }
                }
            }
            const int rbase = qw * 32 + (lane & ~7);          // first row of this lane's group
#pragma unroll
            for (int k = 0; k < 8; k++) {
                const int qk = it.q0 + rbase + k;
                if (qk < p.L) {
                    uint4 *d = (uint4 *)(p.out + ((size_t)it.s * p.L + qk) * p.ldo + (2 * it.kvh + t) * HD +
                                         half * 64);
                    d[j8] = make_uint4(ch[k][0], ch[k][1], ch[k][2], ch[k][3]);
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
    p.n_seqs = n_seqs;
    p.n_items = p.n_qblocks * NKV * n_seqs;
    int sms = 148;
    N550_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    // persistent: one CTA per SM walks the items
    const int grid = p.n_items < sms ? p.n_items : sms;
    // measured on B200 (prefill of 512-token sequences): the reversed rounds
    // take 8 sequences' attention 0.82 -> 0.75 ms; from 16 sequences (3.5
    // rounds and more) the plain order is as fast or faster
    p.snake = p.n_items < 3 * grid;
    N550_CUDA_TRY(launch_k(attn_prefill_tc_kernel, grid, THREADS, SMEM_BYTES, st, tq, tk, tv, p));
    N550_LAUNCH_CHECK();
    return N550_OK;
}

}  // namespace n550
