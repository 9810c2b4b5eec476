// Fast-mode GEMM on the 5th-generation tensor cores (tcgen05, sm_100a).
//
// C[M,N] = A[M,K] . B[N,K]^T, A/B BF16 K-major (row-major [rows, K], the
// layout of kernels.h:44-57: B is the PyTorch [out, in] weight), FP32
// accumulation in TMEM. Replaces the AME tile loop of kernels_ame.c:272-422
// (mlae16/mlbe16 tile loads -> mfmacc.s.bf16 -> msce32 store).
//
// Structure (one persistent CTA per SM, 192 threads):
//   warp 0      TMA producer: 128x64 A and BNx64 B tiles into a STAGES-deep
//               shared-memory ring (128-byte swizzle), mbarrier complete_tx.
//   warp 1      allocates TMEM; one thread issues tcgen05.mma (M=128, N=BN,
//               K=16 per instruction) into one of two TMEM accumulators and
//               tcgen05.commit's the stage back to the producer.
//   warps 2-5   epilogue: tcgen05.ld 32 lanes x 32 columns per warp, fused
//               output transform, stores; then release the accumulator.
// The two accumulators let the epilogue of tile i overlap the MMAs of tile
// i+1. Every wait is bounded (common.cuh: mbar_wait) and reports
// N550_ERR_TIMEOUT through the device status word instead of hanging.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <string.h>

#include "common.cuh"
#include "gemm_tc.h"
#include "launch.h"
#include "ops.h"
#include "tmap.h"

namespace n550 {
namespace {

constexpr int BM = 128;
constexpr int BK = 64;            // one 128-byte swizzle row of BF16
constexpr int UMMA_K = 16;
// Epilogue warps: 4 (one per TMEM lane quarter); the two-head QKV tile gets
// 8 (one head each), because its per-row RMSNorm + RoPE work is latency-bound.
__host__ __device__ constexpr int tc_epi_warps(int BN, int EPI) {
    return (EPI == TC_EPI_QKV_ROPE && BN == 256) ? 16 : 4;
}

// Staging tiles per epilogue warp: the residual epilogue double-buffers the
// tiles its TMA reduce-adds read.
__host__ __device__ constexpr int tc_stg_tiles(int EPI) { return EPI == TC_EPI_RESID_F32 ? 2 : 1; }

// PAIR: a 2-CTA cluster computes a 256 x BN tile with tcgen05 cta_group::2;
// each CTA holds its 128 rows of A and half (BN/2 rows) of B.
template <int BN, int NEPI = 4, int STG = 1, bool PAIR = false>
struct TcCfg {
    static constexpr int B_ROWS = PAIR ? BN / 2 : BN;
    // (16 epilogue warps stage 64 KB: fewer operand stages fit)
    static constexpr int STAGES = PAIR ? (NEPI == 16 ? 4 : 6)
                                       : ((BN >= 256) ? (NEPI == 16 ? 3 : 4) : (BN >= 128 ? 6 : 8));
    static constexpr int THREADS = 64 + 32 * NEPI;
    static constexpr int A_BYTES = BM * BK * 2;
    static constexpr int B_BYTES = B_ROWS * BK * 2;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int TMEM_COLS = 2 * BN;
    static constexpr int EPI_BYTES = NEPI * STG * 32 * 32 * 4;   // 32x32-word tiles per epilogue warp
    // + 512 B: the q/k norm weights of the fused QKV epilogue; + 4 KB: its
    // sum-of-squares exchange between warp pairs ([tile parity][head][half][row])
    static constexpr int SMEM_BYTES =
        STAGES * STAGE_BYTES + EPI_BYTES + 1024 + 256 + 512 + (NEPI == 16 ? 4096 : 0);
    static_assert(SMEM_BYTES <= 232448, "shared memory per CTA");
};

// silu(g) * u (ops_scalar.c:46-51) with the fast exponential and divide: the
// fused SwiGLU epilogue is tolerance-checked (relative error ~1e-6).
__device__ __forceinline__ float silu_mul_f(float g, float u) {
    return __fdividef(g, 1.0f + __expf(-g)) * u;
}

// ---- epilogue staging -------------------------------------------------------
// Each epilogue warp owns a 32 x 32-word shared tile. After tcgen05.ld, lane r
// holds 32 consecutive columns of row r; the tile turns that into stores of
// whole 128-byte (FP32) or 64-byte (BF16) row segments, 4 or 8 rows per
// instruction. 16-byte chunk c of row r is placed so that the 8 lanes of a
// quarter-warp always hit 8 different bank groups, on the write and the read.
__device__ __forceinline__ int f32_word(int r, int c) { return r * 32 + ((c ^ (r & 7)) << 2); }
__device__ __forceinline__ int b16_word(int r, int c) {
    return r * 32 + (((c ^ ((r >> 1) & 3)) + 4 * (r & 1)) << 2);
}

__device__ __forceinline__ void stage_f32(uint32_t *stg, int lane, const uint32_t (&v)[32]) {
#pragma unroll
    for (int c = 0; c < 8; c++)
        *(uint4 *)(stg + f32_word(lane, c)) = make_uint4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
}

__device__ __forceinline__ void stage_bf16(uint32_t *stg, int lane, const float (&v)[32]) {
#pragma unroll
    for (int c = 0; c < 4; c++)
        *(uint4 *)(stg + b16_word(lane, c)) =
            make_uint4(pack_bf16x2(v[8 * c], v[8 * c + 1]), pack_bf16x2(v[8 * c + 2], v[8 * c + 3]),
                       pack_bf16x2(v[8 * c + 4], v[8 * c + 5]), pack_bf16x2(v[8 * c + 6], v[8 * c + 7]));
}

__device__ __forceinline__ float wf(uint32_t w) { return __uint_as_float(w); }

// Rows row0 + r (r < 32) of an FP32 destination; 4 columns per lane. For the
// residual, all 8 reads of x are issued before any store so that they overlap.
template <bool RESID>
__device__ __forceinline__ void flush_f32(const uint32_t *stg, int lane, float *C, int ldc, int row0,
                                          int M, int n, int N, bool vec_ok) {
    const int c = lane & 7;
    const int col = n + 4 * c;
    const bool vec = vec_ok && col + 4 <= N;
    float4 xv[8];
    if (RESID) {
#pragma unroll
        for (int it = 0; it < 8; it++) {
            const int m = row0 + it * 4 + (lane >> 3);
            xv[it] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (m < M && vec) xv[it] = __ldcs((const float4 *)(C + (size_t)m * ldc + col));
        }
    }
#pragma unroll
    for (int it = 0; it < 8; it++) {
        const int r = it * 4 + (lane >> 3);
        const uint4 q = *(const uint4 *)(stg + f32_word(r, c));
        const int m = row0 + r;
        if (m >= M) continue;
        float *dst = C + (size_t)m * ldc + col;
        if (vec) {
            if (RESID)
                *(float4 *)dst = make_float4(xv[it].x + wf(q.x), xv[it].y + wf(q.y),
                                             xv[it].z + wf(q.z), xv[it].w + wf(q.w));
            else
                *(float4 *)dst = make_float4(wf(q.x), wf(q.y), wf(q.z), wf(q.w));
        } else {
            const float v[4] = {wf(q.x), wf(q.y), wf(q.z), wf(q.w)};
#pragma unroll
            for (int e = 0; e < 4; e++)
                if (col + e < N) { if (RESID) dst[e] += v[e]; else dst[e] = v[e]; }
        }
    }
}

// Rows of a BF16 destination; rowptr(r) gives the address of column `n` of
// tile row r (or nullptr to skip the row); 8 columns per lane.
// A 32 x 32-word staging tile holds 32 rows x 32 BF16 in one half of each
// 128-byte row; alt = 16 selects the other half, a second tile in the same
// words (b16_word(r, c) ^ 16 keeps the bank spread of b16_word).
template <class RowPtr>
__device__ __forceinline__ void flush_bf16(const uint32_t *stg, int lane, RowPtr rowptr, int n,
                                           int N, bool vec_ok, int alt = 0) {
    const int c = lane & 3;
    const int col = n + 8 * c;
#pragma unroll
    for (int it = 0; it < 4; it++) {
        const int r = it * 8 + (lane >> 2);
        const uint4 q = *(const uint4 *)(stg + (b16_word(r, c) ^ alt));
        uint16_t *dst = rowptr(r);
        if (!dst) continue;
        dst += 8 * c;
        if (vec_ok && col + 8 <= N) {
            *(uint4 *)dst = q;
        } else {
            const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
            for (int e = 0; e < 8; e++)
                if (col + e < N) dst[e] = (uint16_t)((e & 1) ? (w[e >> 1] >> 16) : (w[e >> 1] & 0xFFFFu));
        }
    }
}

__device__ __forceinline__ void load_chunk(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    tmem_ld_32x32b_x32(taddr, r);
    tmem_ld_wait();
#pragma unroll
    for (int j = 0; j < 32; j++) v[j] = __uint_as_float(r[j]);
}

// Hands a TMEM accumulator back to the MMA thread after this warp's last
// tcgen05.ld of it. Single CTA: every epilogue thread arrives on the local
// barrier. CTA pair: one arrival per warp on the leader CTA's barrier (cbar,
// a shared::cluster address), whose MMAs write both CTAs' accumulators.
struct AccRelease {
    uint64_t *bar;
    uint32_t cbar;     // 0: single CTA
};
__device__ __forceinline__ void acc_release(const AccRelease &r, int lane) {
    tc_fence_before();
    if (!r.cbar) { mbar_arrive(r.bar); return; }
    __syncwarp();
    if (lane == 0) mbar_arrive_cluster(r.cbar);
}

// 16 values of one row (lane) as BF16 into 16-byte chunks c16 * 2, c16 * 2 + 1
// of a 32-column staging tile (alt selects the tile, as in flush_bf16).
// (lo, hi) -> packed BF16x2 with one cvt.rn (round to nearest even; the q/k/v
// values are finite).
__device__ __forceinline__ uint32_t cvt_rn_bf16x2(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

__device__ __forceinline__ void stage_bf16_16(uint32_t *stg, int lane, int c16, int alt,
                                              const float (&v)[16]) {
#pragma unroll
    for (int k = 0; k < 2; k++)
        *(uint4 *)(stg + (b16_word(lane, c16 * 2 + k) ^ alt)) =
            make_uint4(cvt_rn_bf16x2(v[8 * k], v[8 * k + 1]), cvt_rn_bf16x2(v[8 * k + 2], v[8 * k + 3]),
                       cvt_rn_bf16x2(v[8 * k + 4], v[8 * k + 5]), cvt_rn_bf16x2(v[8 * k + 6], v[8 * k + 7]));
}

__device__ __forceinline__ void load_chunk16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    tmem_ld_32x32b_x16(taddr, r);
    tmem_ld_wait();
#pragma unroll
    for (int j = 0; j < 16; j++) v[j] = __uint_as_float(r[j]);
}

// (cos, sin) of rotation pairs i and i + 1 at position pos: the expression the
// model's RoPE table is filled with (rope_sincos of pos * inv_freq[i]),
// evaluated in registers and so bit-identical to the table. Reading the table
// instead costs every lane its own 512-byte row -- uncoalesced L1 traffic
// that, in the epilogue of a persistent GEMM, slowed its tensor core (measured
// on B200 for the 32768 x 4096 x 1024 q/k/v GEMM: 0.297 -> 0.258 ms on CTA
// pairs).
__device__ __forceinline__ float4 rope_cs2(int pos, int i) {
    float s0, c0, s1, c1;
    rope_sincos((float)pos * c_inv_freq[i], &s0, &c0);
    rope_sincos((float)pos * c_inv_freq[i + 1], &s1, &c1);
    return make_float4(c0, s0, c1, s1);
}

// Fused QKV epilogue (qwen3.c:477-511). A 128-column tile is one head of the
// [q 16 | k 8 | v 8] x 128 qkv row. q and k heads: RMSNorm over the head
// (qk_norm, qwen3.c:287-292; four partial sums of squares), RoPE pairs
// (i, i + 64) from the (cos, sin) table (ops_scalar.c:21-35); q goes to the
// BF16 query buffer, k to the KV cache; v heads go to the cache unchanged. The
// accumulator is read from TMEM twice (sum of squares, then 16 rotation pairs
// at a time) to keep register use low. Lane r owns tile row r: it reads that
// row's token position / slot once, and the store loops take other rows'
// destination addresses from their owners by shuffle.
__device__ __forceinline__ void epilogue_qkv(const TcQkv &p, uint32_t *stg, int lane, uint32_t taddr,
                                             int row0, int M, int head, const AccRelease *rel,
                                             const uint16_t *norm_w) {
    const int m = row0 + lane;
    const bool row_ok = m < M;
    const int mc = row_ok ? m : M - 1;
    const int pos = p.tok_pos[mc];
    const bool normed = head < 24;
    // norm weights staged in shared memory at kernel start
    const uint16_t *w = head < 16 ? norm_w : norm_w + 128;
    uint16_t *dst_row;                     // column 0 of this head in the destination row
    if (head < 16) {
        dst_row = p.q_bf16 + (size_t)mc * p.ldq + head * 128;
    } else {
        const int kvh = (head - 16) & 7;
        uint16_t *cache = head < 24 ? p.kc : p.vc;
        const size_t slot = ((size_t)p.tok_seq[mc] * 28 + p.layer) * 8 + kvh;
        dst_row = cache + (slot * p.max_len + pos) * 128;
    }
    if (!row_ok) dst_row = nullptr;
    float scale = 1.f;
    if (normed) {
        float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll 1
        for (int c = 0; c < 4; c++) {
            float v[32];
            load_chunk(taddr + 32 * c, v);
#pragma unroll
            for (int j = 0; j < 32; j += 4) {
                s0 = fmaf(v[j], v[j], s0);
                s1 = fmaf(v[j + 1], v[j + 1], s1);
                s2 = fmaf(v[j + 2], v[j + 2], s2);
                s3 = fmaf(v[j + 3], v[j + 3], s3);
            }
        }
        scale = 1.0f / sqrtf(((s0 + s1) + (s2 + s3)) / 128.0f + p.eps);
    }
#pragma unroll 1
    for (int c = 0; c < 4; c++) {
        // rotation pairs (16c + j, 64 + 16c + j), j < 16
        float a[16], b[16];
        load_chunk16(taddr + 16 * c, a);
        load_chunk16(taddr + 64 + 16 * c, b);
        if (c == 3 && rel) acc_release(*rel, lane);
        if (normed) {
            // (cos, sin) of this row's position for rotation pairs 16c .. 16c + 15
            float4 cs4[8];
#pragma unroll
            for (int e = 0; e < 8; e++) cs4[e] = rope_cs2(pos, 16 * c + 2 * e);
            // 8 norm weights per 16-byte shared load
            const uint4 *w_lo = (const uint4 *)(w + 16 * c);
            const uint4 *w_hi = (const uint4 *)(w + 64 + 16 * c);
#pragma unroll
            for (int j8 = 0; j8 < 2; j8++) {
                const uint4 wl = w_lo[j8], wh = w_hi[j8];
                const uint32_t wlw[4] = {wl.x, wl.y, wl.z, wl.w}, whw[4] = {wh.x, wh.y, wh.z, wh.w};
#pragma unroll
                for (int j2 = 0; j2 < 4; j2++) {
                    const float4 t = cs4[j8 * 4 + j2];
#pragma unroll
                    for (int e = 0; e < 2; e++) {
                        const int j = j8 * 8 + j2 * 2 + e;
                        const float wa = __uint_as_float(e ? (wlw[j2] & 0xFFFF0000u) : (wlw[j2] << 16));
                        const float wb = __uint_as_float(e ? (whw[j2] & 0xFFFF0000u) : (whw[j2] << 16));
                        const float cs = e ? t.z : t.x, sn = e ? t.w : t.y;
                        const float x0 = a[j] * scale * wa;
                        const float x1 = b[j] * scale * wb;
                        a[j] = x0 * cs - x1 * sn;
                        b[j] = x1 * cs + x0 * sn;
                    }
                }
            }
        }
        // dims 16c.. go to the first staging tile, dims 64 + 16c.. to the second
        stage_bf16_16(stg, lane, c & 1, 0, a);
        stage_bf16_16(stg, lane, c & 1, 16, b);
        if (c & 1) {
            __syncwarp();
#pragma unroll
            for (int half = 0; half < 2; half++) {
                const int d0 = 32 * (c >> 1) + 64 * half;
                flush_bf16(stg, lane, [&](int r) -> uint16_t * {
                    uint16_t *d = (uint16_t *)__shfl_sync(0xFFFFFFFFu, (unsigned long long)dst_row, r);
                    return d ? d + d0 : nullptr;
                }, 0, 32, true, half ? 16 : 0);
            }
            __syncwarp();
        }
    }
}

// Half of the fused QKV epilogue for one head: this warp owns rotation pairs
// 32*half .. 32*half + 31, i.e. TMEM columns 32*half.. and 64 + 32*half.. of the
// head. The two halves of a row exchange partial sums of squares through
// shared memory (xss, [parity][head][half][128 rows], parity alternating per
// tile so a slot is rewritten only after the partner passed the next
// barrier) behind the pair's 64-thread named barrier bar_id.
__device__ __forceinline__ void epilogue_qkv_half(const TcQkv &p, uint32_t *stg, int lane, uint32_t taddr,
                                                  int row0, int M, int head, const AccRelease *rel,
                                                  const uint16_t *norm_w, int half, int hh, int qrow,
                                                  float *xss, int parity, int bar_id) {
    const int m = row0 + lane;
    const bool row_ok = m < M;
    const int mc = row_ok ? m : M - 1;
    const int pos = p.tok_pos[mc];
    const bool normed = head < 24;
    const uint16_t *w = head < 16 ? norm_w : norm_w + 128;
    uint16_t *dst_row;
    if (head < 16) {
        dst_row = p.q_bf16 + (size_t)mc * p.ldq + head * 128;
    } else {
        const int kvh = (head - 16) & 7;
        uint16_t *cache = head < 24 ? p.kc : p.vc;
        const size_t slot = ((size_t)p.tok_seq[mc] * 28 + p.layer) * 8 + kvh;
        dst_row = cache + (slot * p.max_len + pos) * 128;
    }
    if (!row_ok) dst_row = nullptr;
    float scale = 1.f;
    if (normed) {
        float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll 1
        for (int c = 0; c < 2; c++) {
            float v[32];
            load_chunk(taddr + 64 * c + 32 * half, v);
#pragma unroll
            for (int j = 0; j < 32; j += 4) {
                s0 = fmaf(v[j], v[j], s0);
                s1 = fmaf(v[j + 1], v[j + 1], s1);
                s2 = fmaf(v[j + 2], v[j + 2], s2);
                s3 = fmaf(v[j + 3], v[j + 3], s3);
            }
        }
        float *x = xss + ((parity * 2 + hh) * 2) * 128 + qrow;
        x[half * 128] = (s0 + s1) + (s2 + s3);
        asm volatile("bar.sync %0, 64;" ::"r"(bar_id) : "memory");
        const float ss = x[0] + x[128];
        scale = 1.0f / sqrtf(ss / 128.0f + p.eps);
    }
#pragma unroll 1
    for (int c = 0; c < 2; c++) {
        // rotation pairs (32*half + 16c + j, 64 + 32*half + 16c + j), j < 16
        const int col = 32 * half + 16 * c;
        float a[16], b[16];
        load_chunk16(taddr + col, a);
        load_chunk16(taddr + 64 + col, b);
        if (c == 1 && rel) acc_release(*rel, lane);
        if (normed) {
            const uint4 *w_lo = (const uint4 *)(w + col);
            const uint4 *w_hi = (const uint4 *)(w + 64 + col);
#pragma unroll
            for (int j8 = 0; j8 < 2; j8++) {
                const uint4 wl = w_lo[j8], wh = w_hi[j8];
                const uint32_t wlw[4] = {wl.x, wl.y, wl.z, wl.w}, whw[4] = {wh.x, wh.y, wh.z, wh.w};
#pragma unroll
                for (int j2 = 0; j2 < 4; j2++) {
                    const float4 t = rope_cs2(pos, 2 * (16 * half + 8 * c + 4 * j8 + j2));
#pragma unroll
                    for (int e = 0; e < 2; e++) {
                        const int j = j8 * 8 + j2 * 2 + e;
                        const float wa = __uint_as_float(e ? (wlw[j2] & 0xFFFF0000u) : (wlw[j2] << 16));
                        const float wb = __uint_as_float(e ? (whw[j2] & 0xFFFF0000u) : (whw[j2] << 16));
                        const float cs = e ? t.z : t.x, sn = e ? t.w : t.y;
                        const float x0 = a[j] * scale * wa;
                        const float x1 = b[j] * scale * wb;
                        a[j] = x0 * cs - x1 * sn;
                        b[j] = x1 * cs + x0 * sn;
                    }
                }
            }
        }
        // dims col.. to the first staging tile, 64 + col.. to the second
        stage_bf16_16(stg, lane, c, 0, a);
        stage_bf16_16(stg, lane, c, 16, b);
    }
    __syncwarp();
#pragma unroll
    for (int hi = 0; hi < 2; hi++) {
        const int d0 = 32 * half + 64 * hi;
        flush_bf16(stg, lane, [&](int r) -> uint16_t * {
            uint16_t *d = (uint16_t *)__shfl_sync(0xFFFFFFFFu, (unsigned long long)dst_row, r);
            return d ? d + d0 : nullptr;
        }, 0, 32, true, hi ? 16 : 0);
    }
    __syncwarp();
}

template <int BN, int EPI, bool PAIR>
__global__ void __launch_bounds__(TcCfg<BN, tc_epi_warps(BN, EPI)>::THREADS, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA,
               const __grid_constant__ CUtensorMap tmB,
               const __grid_constant__ CUtensorMap tmB2,
               const __grid_constant__ CUtensorMap tmC,
               const TcEpilogue ep, int M, int N, int K, int m_fast, int ksplit,
               int kt_per, float *ws, bool partials) {
    constexpr int NEPI = tc_epi_warps(BN, EPI);
    constexpr int STG = tc_stg_tiles(EPI);
    using Cfg = TcCfg<BN, NEPI, STG, PAIR>;
    constexpr int STAGES = Cfg::STAGES;
    constexpr int BMT = PAIR ? 2 * BM : BM;            // output rows per tile
    static_assert(!PAIR || BN == 256, "CTA pairs use 256-wide tiles");
    constexpr bool SILU = (EPI == TC_EPI_SILU_BF16);
    // Output columns per tile: SILU tiles hold BN/2 gate + BN/2 up columns.
    constexpr int OUT_N = SILU ? BN / 2 : BN;

    extern __shared__ uint8_t smem_raw[];
    uint8_t *base = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    // [stage ring][epilogue staging tiles][barriers]
    uint64_t *full = (uint64_t *)(base + STAGES * Cfg::STAGE_BYTES + Cfg::EPI_BYTES);
    uint64_t *empty = full + STAGES;
    uint64_t *tfull = empty + STAGES;       // [2]
    uint64_t *tempty = tfull + 2;           // [2]
    uint64_t *done = tempty + 2;            // [1] MMA drain at exit
    uint32_t *tmem_slot = (uint32_t *)(done + 1);
    uint16_t *norm_w = (uint16_t *)((uint8_t *)full + 256);   // [q_norm 128 | k_norm 128]
    float *xss = (float *)((uint8_t *)full + 768);              // QKV sum-of-squares exchange

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    // CTA pairs: cluster c (CTAs 2c, 2c+1) walks the tiles; CTA `rank` owns
    // rows rank*128.. of each 256-row tile.
    const int rank = PAIR ? (int)cluster_ctarank() : 0;
    const int u0 = PAIR ? (int)blockIdx.x / 2 : (int)blockIdx.x;
    const int ustep = PAIR ? (int)gridDim.x / 2 : (int)gridDim.x;
    const int num_m = (M + BMT - 1) / BMT;
    const int num_n = (N + OUT_N - 1) / OUT_N;
    const int num_k = (K + BK - 1) / BK;
    // Work unit u = (tile u / ksplit, K slice u % ksplit); with ksplit > 1 each
    // unit stores its FP32 partial tile into ws[slice] and a reduce kernel
    // applies the epilogue.
    const int total = num_m * num_n * ksplit;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        for (int b = 0; b < 2; b++) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], PAIR ? 2 * NEPI : 32 * NEPI);
        }
        mbar_init(done, 1);
        fence_mbar_init();
    }
    if (EPI == TC_EPI_QKV_ROPE && warp >= 2 && threadIdx.x - 64 < 32) {
        // 32 threads copy the two norm weight vectors (2 x 256 B) once
        const int i = threadIdx.x - 64;
        ((uint4 *)norm_w)[i] = i < 16 ? ((const uint4 *)ep.qkv.q_norm)[i]
                                      : ((const uint4 *)ep.qkv.k_norm)[i - 16];
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
        if (SILU) tma_prefetch_desc(&tmB2);
    }
    if (warp == 1) {
        if (PAIR) { tmem_alloc_pair(tmem_slot, Cfg::TMEM_COLS); tmem_relinquish_pair(); }
        else { tmem_alloc(tmem_slot, Cfg::TMEM_COLS); tmem_relinquish(); }
    }
    tc_fence_before();
    __syncthreads();
    // the peer's loads signal the leader's barriers and the leader's MMAs write
    // the peer's TMEM: both CTAs must be initialised first
    if (PAIR) cluster_sync();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    // TMEM is held: the next kernel of the stream may start its prologue
    dep_launch();

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            long long issued = 0;
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            // B is a weight operand that no kernel writes: the B tiles of the
            // first ring pass are requested before waiting for the previous
            // kernel, whose output A is.
            auto load_b = [&](uint8_t *sB, int kt, int nb) {
                if (SILU) {
                    tma_load_2d(sB, &tmB, &full[stage], kt * BK, nb * (BN / 2));
                    tma_load_2d(sB + (BN / 2) * BK * 2, &tmB2, &full[stage], kt * BK, nb * (BN / 2));
                } else {
                    tma_load_2d(sB, &tmB, &full[stage], kt * BK, nb * BN);
                }
            };
            int pre = 0;
            if (!PAIR && u0 < total) {
                const int t = u0 / ksplit, sk = u0 - t * ksplit;
                const int nb = m_fast ? t / num_m : t % num_n;
                const int kt0 = sk * kt_per, kt1 = min(num_k, kt0 + kt_per);
                pre = min(kt1 - kt0, STAGES);
                for (stage = 0; stage < pre; stage++) {
                    mbar_arrive_expect_tx(&full[stage], Cfg::STAGE_BYTES);
                    load_b(base + stage * Cfg::STAGE_BYTES + Cfg::A_BYTES, kt0 + stage, nb);
                }
                stage = 0;
            }
            dep_wait();
            for (int u = u0; u < total && ok; u += ustep) {
                const int t = u / ksplit, sk = u - t * ksplit;
                const int mb = m_fast ? t % num_m : t / num_n, nb = m_fast ? t / num_m : t % num_n;
                const int kt0 = sk * kt_per, kt1 = min(num_k, kt0 + kt_per);
                for (int kt = kt0; kt < kt1; kt++) {
                    uint8_t *sA = base + stage * Cfg::STAGE_BYTES;
                    uint8_t *sB = sA + Cfg::A_BYTES;
                    if (issued < pre) {
                        // first ring pass: the slot is free and B is on its way
                        tma_load_2d(sA, &tmA, &full[stage], kt * BK, mb * BM);
                        issued++;
                        if (++stage == STAGES) { stage = 0; phase ^= 1; }
                        continue;
                    }
                    if (!mbar_wait_sleep(&empty[stage], phase ^ 1)) { ok = false; break; }
                    if (PAIR) {
                        // both CTAs' bytes complete on the leader's barrier
                        const uint32_t cb = mapa_shared(smem_u32(&full[stage]), 0);
                        if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * Cfg::STAGE_BYTES);
                        tma_load_2d_pair(sA, &tmA, cb, kt * BK, mb * BMT + rank * BM);
                        if (SILU)   // the pair's B tile: gate rows (rank 0) | up rows (rank 1)
                            tma_load_2d_pair(sB, rank ? &tmB2 : &tmB, cb, kt * BK, nb * (BN / 2));
                        else
                            tma_load_2d_pair(sB, &tmB, cb, kt * BK, nb * BN + rank * (BN / 2));
                        issued++;
                        if (++stage == STAGES) { stage = 0; phase ^= 1; }
                        continue;
                    }
                    mbar_arrive_expect_tx(&full[stage], Cfg::STAGE_BYTES);
                    tma_load_2d(sA, &tmA, &full[stage], kt * BK, mb * BM);
                    load_b(sB, kt, nb);
                    issued++;
                    if (++stage == STAGES) { stage = 0; phase ^= 1; }
                }
            }
            // Drain: every load issued must have landed before the CTA exits
            // (pair: the leader's barriers count both CTAs' loads, and the
            // peer leaves only after the final cluster barrier).
            long long first = issued > STAGES ? issued - STAGES : 0;
            if (!PAIR || rank == 0)
                for (long long i = first; i < issued; i++)
                    if (!mbar_wait_sleep(&full[i % STAGES], (uint32_t)((i / STAGES) & 1))) break;
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        // (pair: only the leader issues; the peer's MMA warp only holds TMEM)
        if (lane == 0 && (!PAIR || rank == 0)) {
            constexpr uint32_t idesc = umma_idesc_bf16(BMT, BN);
            int stage = 0;
            uint32_t phase = 0;
            int ab = 0;
            uint32_t aphase = 0;
            bool ok = true;
            for (int u = u0; u < total && ok; u += ustep) {
                const int sk = u % ksplit;
                const int kt0 = sk * kt_per, kt1 = min(num_k, kt0 + kt_per);
                if (!(PAIR ? mbar_wait_cluster(&tempty[ab], aphase ^ 1) : mbar_wait_sleep(&tempty[ab], aphase ^ 1)))
                    break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + (uint32_t)(ab * BN);
                for (int kt = kt0; kt < kt1; kt++) {
                    if (!mbar_wait_sleep(&full[stage], phase)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t a0 = smem_u32(base + stage * Cfg::STAGE_BYTES);
                    const uint32_t b0 = a0 + Cfg::A_BYTES;
#pragma unroll
                    for (int ks = 0; ks < BK / UMMA_K; ks++) {
                        if (PAIR)
                            umma_bf16_pair(d_tmem, umma_desc_sw128(a0 + ks * UMMA_K * 2),
                                           umma_desc_sw128(b0 + ks * UMMA_K * 2), idesc,
                                           (kt != kt0 || ks != 0) ? 1u : 0u);
                        else
                            umma_bf16(d_tmem, umma_desc_sw128(a0 + ks * UMMA_K * 2),
                                      umma_desc_sw128(b0 + ks * UMMA_K * 2), idesc,
                                      (kt != kt0 || ks != 0) ? 1u : 0u);
                    }
                    if (PAIR) umma_commit_pair_mc(&empty[stage], 3);
                    else umma_commit(&empty[stage]);
                    if (++stage == STAGES) { stage = 0; phase ^= 1; }
                }
                if (!ok) break;
                if (PAIR) umma_commit_pair_mc(&tfull[ab], 3);
                else umma_commit(&tfull[ab]);
                if (++ab == 2) { ab = 0; aphase ^= 1; }
            }
            // Drain all MMAs of this thread before TMEM is released.
            if (PAIR) umma_commit_pair_mc(done, 1);
            else umma_commit(done);
            mbar_wait_sleep(done, 0);
        }
    } else {
        // ---------------- epilogue (warps 2..5) ----------------
        dep_wait();                              // outputs and tables of earlier kernels
        const int q = warp & 3;                 // TMEM lane quarter of this warp
        uint32_t *stg = (uint32_t *)(base + STAGES * Cfg::STAGE_BYTES) + (warp - 2) * STG * 32 * 32;
        int chunks = 0;                          // residual chunks handed to the TMA
        int ab_tiles = 0;                        // tiles drained (QKV exchange parity)
        int ab = 0;
        uint32_t aphase = 0;
        for (int u = u0; u < total; u += ustep) {
            const int t = u / ksplit, sk = u - t * ksplit;
            const int mb = m_fast ? t % num_m : t / num_n, nb = m_fast ? t / num_m : t % num_n;
            if (!mbar_wait_sleep(&tfull[ab], aphase)) break;
            tc_fence_after();
            const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(ab * BN);
            const int row0 = mb * BMT + rank * BM + q * 32;   // first row of this warp's quarter
            AccRelease rel;
            rel.bar = &tempty[ab];
            rel.cbar = PAIR ? mapa_shared(smem_u32(&tempty[ab]), 0) : 0u;
            if (ksplit > 1 || partials) {
                // Partial sums of K slice sk: raw FP32 accumulators into
                // ws[sk][M][ldw]; SwiGLU tiles put gate at column n, up at N + n.
                const int ldw = SILU ? 2 * N : N;
                float *slice = ws + (size_t)sk * M * ldw;
#pragma unroll 1
                for (int cch = 0; cch < BN; cch += 32) {
                    uint32_t r[32];
                    tmem_ld_32x32b_x32(taddr + cch, r);
                    tmem_ld_wait();
                    if (cch + 32 == BN) acc_release(rel, lane);
                    const int n = SILU ? (cch < OUT_N ? nb * OUT_N + cch : N + nb * OUT_N + cch - OUT_N)
                                       : nb * BN + cch;
                    const int nlim = SILU ? (cch < OUT_N ? N : 2 * N) : N;
                    stage_f32(stg, lane, r);
                    __syncwarp();
                    flush_f32<false>(stg, lane, slice, ldw, row0, M, n, nlim,
                                     (ldw % 4) == 0 && (n % 4) == 0);
                    __syncwarp();
                }
            } else if (EPI == TC_EPI_QKV_ROPE) {
                if (NEPI == 16) {
                    // warps 2-9: first head of the tile, 10-17: second; within
                    // a head, warps 2-5 / 10-13 take rotation pairs 0-31 and
                    // 6-9 / 14-17 pairs 32-63 of their lane quarter
                    const int sw = warp - 2;
                    const int hh = sw >> 3, half = (sw >> 2) & 1;
                    epilogue_qkv_half(ep.qkv, stg, lane, taddr + hh * 128, row0, M, nb * 2 + hh, &rel,
                                      norm_w, half, hh, q * 32 + lane, xss, ab_tiles & 1,
                                      1 + hh * 4 + q);
                    ab_tiles++;
                } else {
#pragma unroll 1
                    for (int hh = 0; hh < BN / 128; hh++)
                        epilogue_qkv(ep.qkv, stg, lane, taddr + hh * 128, row0, M,
                                     nb * (BN / 128) + hh, hh + 1 == BN / 128 ? &rel : nullptr, norm_w);
                }
            } else if (EPI == TC_EPI_ARGMAX) {
                // running (max, lowest column of the max) of this row over the
                // tile's columns, in increasing column order
                float bv = -INFINITY;
                int bi = 0x7FFFFFFF;
#pragma unroll 1
                for (int cch = 0; cch < BN; cch += 32) {
                    uint32_t r[32];
                    tmem_ld_32x32b_x32(taddr + cch, r);
                    tmem_ld_wait();
                    if (cch + 32 == BN) acc_release(rel, lane);
                    const int n0 = nb * BN + cch;
#pragma unroll
                    for (int j = 0; j < 32; j++) {
                        const float v = __uint_as_float(r[j]);
                        if (n0 + j < N && (v > bv || (v == bv && n0 + j < bi))) { bv = v; bi = n0 + j; }
                    }
                }
                const int m = row0 + lane;
                if (m < M) {
                    ep.amax[(size_t)m * ep.an + nb] = bv;
                    ep.aidx[(size_t)m * ep.an + nb] = bi;
                }
            } else if (SILU) {
#pragma unroll 1
                for (int cch = 0; cch < OUT_N; cch += 32) {
                    float g[32], u[32];
                    load_chunk(taddr + cch, g);
                    load_chunk(taddr + OUT_N + cch, u);
                    if (cch + 32 == OUT_N) acc_release(rel, lane);
                    float h[32];
#pragma unroll
                    for (int j = 0; j < 32; j++) h[j] = silu_mul_f(g[j], u[j]);
                    stage_bf16(stg, lane, h);
                    __syncwarp();
                    const int n = nb * OUT_N + cch;
                    uint16_t *C = (uint16_t *)ep.c;
                    flush_bf16(stg, lane, [&](int r) -> uint16_t * {
                        const int m = row0 + r;
                        return m < M ? C + (size_t)m * ep.ldc + n : nullptr;
                    }, n, N, ep.vec_ok);
                    __syncwarp();
                }
            } else if (EPI == TC_EPI_RESID_F32 && ep.tma_resid) {
                // x += acc: each 32 x 32 chunk is staged in the 128-byte
                // swizzled layout of the FP32 tensor map and reduce-added into
                // x by the TMA (L2 does the read-modify-write, one add per
                // element), two staging tiles alternating.
#pragma unroll 1
                for (int cch = 0; cch < BN; cch += 32) {
                    uint32_t r[32];
                    tmem_ld_32x32b_x32(taddr + cch, r);
                    tmem_ld_wait();
                    if (cch + 32 == BN) acc_release(rel, lane);
                    const int n = nb * BN + cch;
                    uint32_t *sb = stg + (chunks & 1) * 32 * 32;
                    if (lane == 0) bulk_wait_group_read<1>();   // the reduce that last read sb
                    __syncwarp();
                    stage_f32(sb, lane, r);
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0 && n < N && row0 < M) {
                        tma_reduce_add_2d(&tmC, sb, n, row0);
                        bulk_commit_group();
                    }
                    chunks++;
                }
            } else {
#pragma unroll 1
                for (int cch = 0; cch < BN; cch += 32) {
                    uint32_t r[32];
                    tmem_ld_32x32b_x32(taddr + cch, r);
                    tmem_ld_wait();
                    if (cch + 32 == BN) acc_release(rel, lane);
                    const int n = nb * BN + cch;
                    if (EPI == TC_EPI_BF16) {
                        float v[32];
#pragma unroll
                        for (int j = 0; j < 32; j++) v[j] = __uint_as_float(r[j]);
                        stage_bf16(stg, lane, v);
                        __syncwarp();
                        uint16_t *C = (uint16_t *)ep.c;
                        flush_bf16(stg, lane, [&](int rr) -> uint16_t * {
                            const int m = row0 + rr;
                            return m < M ? C + (size_t)m * ep.ldc + n : nullptr;
                        }, n, N, ep.vec_ok);
                    } else {
                        stage_f32(stg, lane, r);
                        __syncwarp();
                        flush_f32<EPI == TC_EPI_RESID_F32>(stg, lane, (float *)ep.c, ep.ldc, row0, M, n, N,
                                                           ep.vec_ok);
                    }
                    __syncwarp();
                }
            }
            if (++ab == 2) { ab = 0; aphase ^= 1; }
        }
        // Reduce-adds still in flight read this CTA's shared memory and must
        // land before the kernel completes.
        if (EPI == TC_EPI_RESID_F32 && lane == 0) bulk_wait_group<0>();
    }

    tc_fence_before();
    __syncthreads();
    // pair: the leader's MMAs wrote the peer's TMEM and the peer's loads were
    // counted on the leader's barriers -- neither CTA leaves before both are done
    if (PAIR) cluster_sync();
    if (warp == 1) {
        tc_fence_after();
        if (PAIR) tmem_dealloc_pair(tmem_base, Cfg::TMEM_COLS);
        else tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
    }
}

// ---------------- host side ----------------

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

int get_encoder() {
    if (g_encode) return N550_OK;
    cudaDriverEntryPointQueryResult q;
    void *fn = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000,
                                         cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn)
        return N550_ERR_CUDA;
    g_encode = (PFN_cuTensorMapEncodeTiled_v12000)fn;
    return N550_OK;
}

// K-major BF16 matrix [rows, K] with row stride ld elements; box = box_rows x 64.
int make_tmap(CUtensorMap *tm, const void *ptr, int rows, int K, int ld, int box_rows) {
    cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
    cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = g_encode(tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(ptr),
                          dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? N550_OK : N550_ERR_UNSUPPORTED;
}

// FP32 output [rows, cols] (row stride ld elements) for TMA stores/reduces of
// 32 x 32 staging tiles (128-byte rows, 128-byte swizzle).
int make_tmap_f32_out(CUtensorMap *tm, void *ptr, int rows, int cols, int ld) {
    if (get_encoder()) return N550_ERR_CUDA;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)ld * 4};
    cuuint32_t box[2] = {32, 32};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = g_encode(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, ptr, dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? N550_OK : N550_ERR_UNSUPPORTED;
}

int g_num_sms[64];

int num_sms() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (!g_num_sms[dev]) {
        int v = 0;
        cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
        g_num_sms[dev] = v > 0 ? v : 148;
    }
    return g_num_sms[dev];
}

template <int BN, int EPI, bool PAIR = false>
int launch_impl(cudaStream_t st, const CUtensorMap &ta, const CUtensorMap &tb,
                const CUtensorMap &tb2, const TcEpilogue &ep, int M, int N, int K,
                int max_ctas, int ksplit = 1, int kt_per = 1 << 30, float *ws = nullptr,
                bool partials = false, const CUtensorMap *tc = nullptr) {
    using Cfg = TcCfg<BN, tc_epi_warps(BN, EPI), tc_stg_tiles(EPI), PAIR>;
    if (PAIR && (ksplit != 1 || partials)) return N550_ERR_ARG;
    CUtensorMap tmc;
    if (tc) tmc = *tc;
    else memset(&tmc, 0, sizeof tmc);
    static bool attr_done[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr_done[dev]) {
        N550_CUDA_TRY(cudaFuncSetAttribute(gemm_tc_kernel<BN, EPI, PAIR>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           Cfg::SMEM_BYTES));
        attr_done[dev] = true;
    }
    constexpr int OUT_N = (EPI == TC_EPI_SILU_BF16) ? BN / 2 : BN;
    constexpr int BMT = PAIR ? 2 * BM : BM;
    const long long tiles = (long long)((M + BMT - 1) / BMT) * ((N + OUT_N - 1) / OUT_N) * ksplit;
    int grid = num_sms();
    if (max_ctas > 0 && max_ctas < grid) grid = max_ctas;
    const long long ctas = PAIR ? 2 * tiles : tiles;
    if (ctas < grid) grid = (int)ctas;
    if (PAIR) grid &= ~1;
    if (grid < 1) return N550_ERR_ARG;
    // Resident CTAs work on consecutive tiles: walk M fastest when the weight
    // operand is the larger one (e.g. the 311 MB lm_head), so each B tile is
    // fetched from HBM once and reused from L2 by the CTAs of all M tiles;
    // otherwise walk N fastest so that A rows are shared.
    const int m_fast = (long long)N * (EPI == TC_EPI_SILU_BF16 ? 2 : 1) > (long long)M;
    if constexpr (!PAIR) {
        N550_CUDA_TRY(launch_k(gemm_tc_kernel<BN, EPI, false>, grid, Cfg::THREADS, Cfg::SMEM_BYTES, st,
                               ta, tb, tb2, tmc, ep, M, N, K, m_fast, ksplit, kt_per, ws, partials));
        return N550_OK;
    } else {
    // 2-CTA clusters: consecutive CTAs (2c, 2c+1) form pair c.
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(Cfg::THREADS);
    cfg.dynamicSmemBytes = Cfg::SMEM_BYTES;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    // persistent pairs: no more clusters than can be resident at once (SMs
    // of a GPC that cannot be paired stay out)
    static int max_clusters[64] = {};
    if (dev >= 0 && dev < 64) {
        if (!max_clusters[dev]) {
            int n = 0;
            if (cudaOccupancyMaxActiveClusters(&n, gemm_tc_kernel<BN, EPI, true>, &cfg) != cudaSuccess || n < 1) {
                (void)cudaGetLastError();
                n = num_sms() / 2;
            }
            max_clusters[dev] = n;
        }
        if (grid > 2 * max_clusters[dev]) grid = 2 * max_clusters[dev];
        cfg.gridDim = dim3(grid);
    }
    cfg.numAttrs = g_pdl ? 2 : 1;
    N550_CUDA_TRY(cudaLaunchKernelEx(&cfg, gemm_tc_kernel<BN, EPI, true>, ta, tb, tb2, tmc, ep, M, N, K,
                                     m_fast, ksplit, kt_per, ws, partials));
    return N550_OK;
    }
}

// Sum of the ksplit partial tiles in slice order, then the epilogue.
template <int EPI>
__global__ void splitk_reduce_kernel(const float *__restrict__ ws, int ksplit, int M, int N, void *c,
                                     int ldc) {
    dep_wait();
    dep_launch();
    const int ldw = EPI == TC_EPI_SILU_BF16 ? 2 * N : N;
    const size_t slice = (size_t)M * ldw, total = (size_t)M * N;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
         i += (size_t)gridDim.x * blockDim.x) {
        const int m = (int)(i / N), n = (int)(i % N);
        const float *p = ws + (size_t)m * ldw + n;
        float acc = 0.f;
        for (int sk = 0; sk < ksplit; sk++) acc += p[sk * slice];
        if (EPI == TC_EPI_SILU_BF16) {
            float up = 0.f;
            for (int sk = 0; sk < ksplit; sk++) up += p[sk * slice + N];
            ((uint16_t *)c)[(size_t)m * ldc + n] = f32_to_bf16_rne(silu_mul_f(acc, up));
        } else if (EPI == TC_EPI_BF16) {
            ((uint16_t *)c)[(size_t)m * ldc + n] = f32_to_bf16_rne(acc);
        } else if (EPI == TC_EPI_RESID_F32) {
            ((float *)c)[(size_t)m * ldc + n] += acc;
        } else {
            ((float *)c)[(size_t)m * ldc + n] = acc;
        }
    }
}

}  // namespace

namespace {
int encode_sw128(CUtensorMap *tm, const void *ptr, cuuint32_t rank, const cuuint64_t *dims,
                 const cuuint64_t *strides, int box_rows) {
    int rc = get_encoder();
    if (rc) return rc;
    cuuint32_t box[3] = {64, (cuuint32_t)box_rows, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = g_encode(tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, const_cast<void *>(ptr), dims,
                          strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? N550_OK : N550_ERR_UNSUPPORTED;
}
}  // namespace

int tmap_bf16_sw128(CUtensorMap *tm, const void *ptr, uint64_t rows, uint64_t cols, uint64_t ld,
                    int box_rows) {
    if (!ptr || ((uintptr_t)ptr & 15) || (ld * 2) % 16 || cols < 64 || rows < 1 || box_rows < 1 ||
        box_rows > 256)
        return N550_ERR_ARG;
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
    return encode_sw128(tm, ptr, 2, dims, strides, box_rows);
}

int tmap_bf16_sw128_3d(CUtensorMap *tm, const void *ptr, uint64_t rows, uint64_t cols,
                       uint64_t ld, int box_rows, uint64_t planes, uint64_t plane_ld) {
    if (!ptr || ((uintptr_t)ptr & 15) || (ld * 2) % 16 || cols < 64 || rows < 1 || box_rows < 1 ||
        box_rows > 256 || planes < 1 || (plane_ld * 2) % 16 || plane_ld < rows * ld)
        return N550_ERR_ARG;
    const cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)rows, (cuuint64_t)planes};
    const cuuint64_t strides[2] = {(cuuint64_t)ld * 2, (cuuint64_t)plane_ld * 2};
    return encode_sw128(tm, ptr, 3, dims, strides, box_rows);
}

int launch_gemm_tc_qkv(cudaStream_t st, const uint16_t *a, int lda, const uint16_t *w,
                       const TcQkv &q, int M, int K, int max_ctas) {
    if (M <= 0) return N550_OK;
    if (!tc_shape_ok(a, lda, w, K, K)) return N550_ERR_UNSUPPORTED;
    if (!q.q_bf16 || !q.kc || !q.vc || !q.tok_pos || !q.tok_seq || !q.rope ||
        (q.ldq % 8))
        return N550_ERR_ARG;
    int rc = get_encoder();
    if (rc) return rc;
    const int bn = n550_tile_bn(M, 4096);
    CUtensorMap ta, tb;
    if ((rc = make_tmap(&ta, a, M, K, lda, BM))) return rc;
    if ((rc = make_tmap(&tb, w, 4096, K, K, bn))) return rc;
    TcEpilogue ep{};
    ep.qkv = q;
    ep.vec_ok = 1;
    // Pair tiles from M >= 12288 as for the other projections: in the model's
    // prefill step they are ahead of single-CTA tiles for this GEMM too
    // (measured on B200, 64 x 512 tokens: 32.4-32.7 vs 33.1 ms per step,
    // although an isolated launch favours single-CTA tiles, 0.246 vs 0.258 ms).
    if (bn == 256 && tc_use_pair(M, bn)) {
        // pair tiles: each CTA's B box is one head (128 rows)
        if ((rc = make_tmap(&tb, w, 4096, K, K, 128))) return rc;
        return launch_impl<256, TC_EPI_QKV_ROPE, true>(st, ta, tb, tb, ep, M, 4096, K, max_ctas);
    }
    if (bn == 256) return launch_impl<256, TC_EPI_QKV_ROPE>(st, ta, tb, tb, ep, M, 4096, K, max_ctas);
    return launch_impl<128, TC_EPI_QKV_ROPE>(st, ta, tb, tb, ep, M, 4096, K, max_ctas);
}

// 0: automatic; 128 / 256: single-CTA tiles of that width; 512: 256 x 256
// tiles on 2-CTA clusters.
int g_tile_bn = 0;
bool g_pdl = true;

bool tc_use_pair(int M, int bn) {
    if (bn != 256 || g_tile_bn == 256) return false;
    // Measured on B200 (prefill projection shapes): pairs are 0-10 % faster
    // from M = 16384 rows, even at 8192 and 4-14 % slower at 4096, where the
    // single-CTA 128 x 256 tiles ramp up faster.
    return g_tile_bn == 512 || M >= 12288;
}

int n550_tile_bn(int M, int N) {
    if (g_tile_bn == 512) return 256;
    if (g_tile_bn) return g_tile_bn;
    // 256-wide tiles halve the operand traffic per MMA (measured on prefill
    // shapes: 1.3 PFLOP/s vs 0.85); narrow outputs and skinny M keep 128 so
    // that there are enough tiles to occupy the SMs.
    return (M >= 1024 && N >= 1024) ? 256 : 128;
}

int tc_splitk_plan(int M, int N, int K, int epi, int bn, int *kt_per) {
    const int out_n = epi == TC_EPI_SILU_BF16 ? bn / 2 : bn;
    const long long tiles = (long long)((M + BM - 1) / BM) * ((N + out_n - 1) / out_n);
    const int num_k = (K + BK - 1) / BK;
    const int sms = num_sms();
    int ks = (int)(sms / (tiles > 0 ? tiles : 1));
    ks = std::min(ks, std::min(num_k / 2, 8));
    if (ks < 2) { *kt_per = num_k; return 1; }
    *kt_per = (num_k + ks - 1) / ks;
    return (num_k + *kt_per - 1) / *kt_per;
}

int launch_gemm_tc_partials(cudaStream_t st, int epi, const uint16_t *a, int lda, const uint16_t *b,
                            int ldb, const uint16_t *b2, int M, int N, int K, float *ws,
                            size_t ws_bytes, int *ks_out) {
    *ks_out = 0;
    if (M <= 0 || N <= 0) return N550_OK;
    if (!tc_shape_ok(a, lda, b, ldb, K)) return N550_ERR_UNSUPPORTED;
    if (epi != TC_EPI_F32 && epi != TC_EPI_SILU_BF16) return N550_ERR_ARG;
    // 64-wide tiles: twice the tiles of 128 for the same N, so half the K
    // slices (and half the partial-sum traffic) reach the same SM count.
    const int bn = 64;
    int kt_per = 0;
    const int ks = tc_splitk_plan(M, N, K, epi, bn, &kt_per);
    const size_t need = (size_t)ks * M * (epi == TC_EPI_SILU_BF16 ? 2 * N : N) * 4;
    if (!ws || need > ws_bytes) return N550_ERR_ARG;
    int rc = get_encoder();
    if (rc) return rc;
    const int brows = (epi == TC_EPI_SILU_BF16) ? bn / 2 : bn;
    CUtensorMap ta, tb, tb2;
    if ((rc = make_tmap(&ta, a, M, K, lda, BM))) return rc;
    if ((rc = make_tmap(&tb, b, N, K, ldb, brows))) return rc;
    if (epi == TC_EPI_SILU_BF16) {
        if ((rc = make_tmap(&tb2, b2, N, K, ldb, brows))) return rc;
    } else {
        tb2 = tb;
    }
    TcEpilogue ep{};
    // The split path of the kernel stores raw partials (also for ks == 1).
    if (epi == TC_EPI_SILU_BF16)
        rc = launch_impl<64, TC_EPI_SILU_BF16>(st, ta, tb, tb2, ep, M, N, K, 0, ks, kt_per, ws, true);
    else
        rc = launch_impl<64, TC_EPI_F32>(st, ta, tb, tb2, ep, M, N, K, 0, ks, kt_per, ws, true);
    if (!rc) *ks_out = ks;
    return rc;
}

int launch_splitk_reduce(cudaStream_t st, int epi, const float *ws, int ks, int M, int N, void *c,
                         int ldc) {
    const size_t total = (size_t)M * N;
    if (!total) return N550_OK;
    const int grid = (int)std::min<size_t>((total + 255) / 256, 148 * 8);
    auto go = [&](auto kernel) { return launch_k(kernel, grid, 256, 0, st, ws, ks, M, N, c, ldc); };
    cudaError_t e;
    switch (epi) {
    case TC_EPI_F32: e = go(splitk_reduce_kernel<TC_EPI_F32>); break;
    case TC_EPI_BF16: e = go(splitk_reduce_kernel<TC_EPI_BF16>); break;
    case TC_EPI_RESID_F32: e = go(splitk_reduce_kernel<TC_EPI_RESID_F32>); break;
    case TC_EPI_SILU_BF16: e = go(splitk_reduce_kernel<TC_EPI_SILU_BF16>); break;
    default: return N550_ERR_ARG;
    }
    N550_CUDA_TRY(e);
    return N550_OK;
}

int launch_gemm_tc_splitk(cudaStream_t st, int epi, const uint16_t *a, int lda, const uint16_t *b,
                          int ldb, const uint16_t *b2, void *c, int ldc, int M, int N, int K,
                          float *ws, size_t ws_bytes) {
    if (M <= 0 || N <= 0) return N550_OK;
    int kt_per = 0;
    const int ks = tc_splitk_plan(M, N, K, epi, 64, &kt_per);
    const size_t need = (size_t)ks * M * (epi == TC_EPI_SILU_BF16 ? 2 * N : N) * 4;
    if (ks == 1 || !ws || need > ws_bytes)
        return launch_gemm_tc(st, epi, 128, a, lda, b, ldb, b2, c, ldc, M, N, K, 0);
    if (epi != TC_EPI_F32 && epi != TC_EPI_BF16 && epi != TC_EPI_RESID_F32 && epi != TC_EPI_SILU_BF16)
        return N550_ERR_ARG;
    int got = 0;
    const int pe = epi == TC_EPI_SILU_BF16 ? TC_EPI_SILU_BF16 : TC_EPI_F32;
    int rc = launch_gemm_tc_partials(st, pe, a, lda, b, ldb, b2, M, N, K, ws, ws_bytes, &got);
    if (rc) return rc;
    return launch_splitk_reduce(st, epi, ws, got, M, N, c, ldc);
}

namespace {
// Merge the per-tile (max, index) pairs of a row (tiles in increasing column
// order): larger value wins, ties keep the lower index; a row whose values
// are all -inf or NaN gives index 0 (qwen3_op_argmax returns 0 there).
__global__ void __launch_bounds__(256)
argmax_tiles_kernel(const float *__restrict__ amax, const int32_t *__restrict__ aidx, int an,
                    int32_t *idx) {
    dep_wait();
    dep_launch();
    __shared__ float sv[8];
    __shared__ int si[8];
    const float *rv = amax + (size_t)blockIdx.x * an;
    const int32_t *ri = aidx + (size_t)blockIdx.x * an;
    float bv = -INFINITY;
    int bi = 0x7FFFFFFF;
    for (int t = threadIdx.x; t < an; t += 256) {
        const float v = rv[t];
        const int i = ri[t];
        if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xFFFFFFFFu, bv, o);
        const int oi = __shfl_xor_sync(0xFFFFFFFFu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    if ((threadIdx.x & 31) == 0) { sv[threadIdx.x >> 5] = bv; si[threadIdx.x >> 5] = bi; }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < 8; w++)
            if (sv[w] > sv[0] || (sv[w] == sv[0] && si[w] < si[0])) { sv[0] = sv[w]; si[0] = si[w]; }
        idx[blockIdx.x] = si[0] == 0x7FFFFFFF ? 0 : si[0];
    }
}
}  // namespace

int launch_gemm_tc_argmax(cudaStream_t st, const uint16_t *a, int lda, const uint16_t *b, int ldb,
                          int M, int N, int K, void *ws, size_t ws_bytes, int32_t *idx) {
    if (M <= 0) return N550_OK;
    if (N <= 0 || !idx) return N550_ERR_ARG;
    if (!tc_shape_ok(a, lda, b, ldb, K)) return N550_ERR_UNSUPPORTED;
    constexpr int BNA = 128;
    const int an = (N + BNA - 1) / BNA;
    if (!ws || ws_bytes < (size_t)M * an * 8 || ((uintptr_t)ws & 15)) return N550_ERR_ARG;
    int rc = get_encoder();
    if (rc) return rc;
    CUtensorMap ta, tb;
    if ((rc = make_tmap(&ta, a, M, K, lda, BM))) return rc;
    if ((rc = make_tmap(&tb, b, N, K, ldb, BNA))) return rc;
    TcEpilogue ep{};
    ep.amax = (float *)ws;
    ep.aidx = (int32_t *)((float *)ws + (size_t)M * an);
    ep.an = an;
    if ((rc = launch_impl<BNA, TC_EPI_ARGMAX>(st, ta, tb, tb, ep, M, N, K, 0))) return rc;
    N550_CUDA_TRY(launch_k(argmax_tiles_kernel, M, 256, 0, st, ep.amax, ep.aidx, an, idx));
    return N550_OK;
}

bool tc_shape_ok(const void *a, int lda, const void *b, int ldb, int K) {
    // K >= 64: the tensor maps' boxes are 64 elements wide
    return K >= 64 && (K % 8) == 0 && (lda % 8) == 0 && (ldb % 8) == 0 &&
           (((uintptr_t)a) & 15) == 0 && (((uintptr_t)b) & 15) == 0;
}

int launch_gemm_tc(cudaStream_t st, int epi, int bn, const uint16_t *a, int lda,
                   const uint16_t *b, int ldb, const uint16_t *b2, void *c, int ldc,
                   int M, int N, int K, int max_ctas) {
    if (M <= 0 || N <= 0) return N550_OK;
    if (!tc_shape_ok(a, lda, b, ldb, K)) return N550_ERR_UNSUPPORTED;
    if (epi == TC_EPI_SILU_BF16 && (!b2 || (((uintptr_t)b2) & 15))) return N550_ERR_ARG;
    int rc = get_encoder();
    if (rc) return rc;
    if (bn != 128 && bn != 256) bn = 128;
    const bool pair = tc_use_pair(M, bn);
    // B rows per CTA and TMA box: SwiGLU tiles hold bn/2 gate + bn/2 up rows,
    // pair tiles split a tile's bn rows between the two CTAs
    const int brows = (epi == TC_EPI_SILU_BF16 || pair) ? bn / 2 : bn;
    CUtensorMap ta, tb, tb2;
    if ((rc = make_tmap(&ta, a, M, K, lda, BM))) return rc;
    if ((rc = make_tmap(&tb, b, N, K, ldb, brows))) return rc;
    if (epi == TC_EPI_SILU_BF16) {
        if ((rc = make_tmap(&tb2, b2, N, K, ldb, brows))) return rc;
    } else {
        tb2 = tb;
    }
    TcEpilogue ep{};
    ep.c = c;
    ep.ldc = ldc;
    const int esz = (epi == TC_EPI_BF16 || epi == TC_EPI_SILU_BF16) ? 2 : 4;
    ep.vec_ok = ((((uintptr_t)c) & 15) == 0) && ((ldc * esz) % 16 == 0);
    CUtensorMap tc;
    const CUtensorMap *tcp = nullptr;
    if (epi == TC_EPI_RESID_F32 && ep.vec_ok && make_tmap_f32_out(&tc, c, M, N, ldc) == N550_OK) {
        ep.tma_resid = 1;
        tcp = &tc;
    }
#define N550_TC_CASE(BNV, EV)                                                                   \
    if (bn == BNV && epi == EV) {                                                               \
        if constexpr (BNV == 256)                                                               \
            if (pair)                                                                           \
                return launch_impl<256, EV, true>(st, ta, tb, tb2, ep, M, N, K, max_ctas, 1,      \
                                                  1 << 30, nullptr, false, tcp);                \
        return launch_impl<BNV, EV>(st, ta, tb, tb2, ep, M, N, K, max_ctas, 1, 1 << 30, nullptr,  \
                                    false, tcp);                                                \
    }
    N550_TC_CASE(128, TC_EPI_F32)
    N550_TC_CASE(128, TC_EPI_BF16)
    N550_TC_CASE(128, TC_EPI_RESID_F32)
    N550_TC_CASE(128, TC_EPI_SILU_BF16)
    N550_TC_CASE(256, TC_EPI_F32)
    N550_TC_CASE(256, TC_EPI_BF16)
    N550_TC_CASE(256, TC_EPI_RESID_F32)
    N550_TC_CASE(256, TC_EPI_SILU_BF16)
#undef N550_TC_CASE
    return N550_ERR_ARG;
}

}  // namespace n550
