// Skinny-token tcgen05 GEMM of the decode step: Y[T,N] = X[T,K] . W[N,K]^T for
// T <= 128 tokens (the qwen3_gemm calls of qwen3.c:477-545 when one token per
// sequence is in flight), with the residual add, SwiGLU or the q/k/v
// epilogue (QK-norm, RoPE, K/V cache write) fused.
//
// At a handful of tokens the projections are weight streams: 30 MB of BF16
// weights per layer against a few hundred KB of activations. The layout is
// chosen for that:
//  * the weight rows are the MMA's M side (128 output features per tile, one
//    TMEM lane each) and the tokens its N side (TN = 32 columns for up to 32
//    tokens, else 64-column token tiles), so every tcgen05.mma covers a whole
//    token tile;
//  * K is split over a thread-block cluster of CS CTAs (CS <= 16) until
//    ~128-256 CTAs stream weights in parallel; each CTA's k-tiles (16 KB of
//    weights + TN x 128 B of activations each) go through a ring of up to 8
//    stages -- usually all of them at once -- and the first ring pass of
//    weight tiles is requested before the programmatic-dependent-launch wait
//    (no kernel writes weights), so it streams while the previous kernel
//    finishes;
//  * the CS partial accumulators are summed through distributed shared
//    memory: CTA r owns token columns [r*tno, (r+1)*tno) of the tile, every
//    CTA writes each column of its partial into the owner's receive slots,
//    and the owner adds the slices in rank (= K) order -- a fixed order, so
//    results are deterministic -- and applies the epilogue. No partial sums
//    go through global memory and no separate reduction kernel runs.
#include <cuda.h>

#include <algorithm>

#include "common.cuh"
#include "gemm_skinny.h"
#include "gemm_tc.h"
#include "launch.h"
#include "tmap.h"

namespace n550 {
namespace {

constexpr int SK_THREADS = 192;        // warp 0 TMA, warp 1 MMA, warps 2-5 epilogue
constexpr int SK_BK = 64;              // K per stage (one 128-byte swizzle row)
constexpr int SK_MAX_STAGES = 8;       // operand ring depth
constexpr int SK_W_BYTES = 128 * SK_BK * 2;
constexpr int SK_MAX_CS = 16;
constexpr int SK_SMEM_MAX = 232448;    // opt-in shared memory per CTA
constexpr int SK_BAR_BYTES = 8 * (2 * SK_MAX_STAGES + 2) + 16;
constexpr int HEAD = 128;
constexpr int N_LAYERS = 28, N_KV_HEADS = 8;
constexpr float NORM_EPS = 1e-6f;

template <int TN>
struct SkCfg {
    static constexpr int X_BYTES = TN * SK_BK * 2;
    static constexpr int STAGE = SK_W_BYTES + X_BYTES;     // multiple of 1024
    static_assert(STAGE % 1024 == 0, "swizzle atoms need 1024-byte aligned stages");
};

struct SkParams {
    int T, N, K;
    int kt_per;         // k-tiles per CTA of the cluster
    int stages;         // operand ring depth (<= SK_MAX_STAGES)
    int n_ttiles;       // token tiles
    int recv_off;       // shared-memory offset of the receive slots
    int aux_off;        // QKV: positions, slots and RoPE rows of the owned tokens
    int bar_off;        // shared-memory offset of the barriers
    SkEpilogue ep;
};

// silu(g) * u (ops_scalar.c:46-51), as in the tcgen05 GEMM epilogue.
__device__ __forceinline__ float sk_silu_mul(float g, float u) {
    return __fdividef(g, 1.0f + __expf(-g)) * u;
}

template <int TN, int EPI>
__global__ void __launch_bounds__(SK_THREADS, 1)
gemm_skinny_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmW2,
                   const __grid_constant__ CUtensorMap tmX, const SkParams p) {
    using Cfg = SkCfg<TN>;
    constexpr bool SILU = EPI == SK_EPI_SILU;
    // Global reads of the epilogue are issued before the accumulator wait:
    // residual values of up to PF owned columns per thread (RESID), and the
    // positions, slots and RoPE rows of the owned tokens into shared memory
    // (QKV).
    constexpr int PF = EPI == SK_EPI_RESID ? 32 : 1;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *base = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    float *stage = (float *)base;                         // [TN][128] own partial, after the MMAs
    float *recv = (float *)(base + p.recv_off);           // [cs][tno][128] peers' partials
    uint64_t *full = (uint64_t *)(base + p.bar_off);      // [SK_MAX_STAGES] operands landed
    uint64_t *empty = full + SK_MAX_STAGES;               // [SK_MAX_STAGES] operands consumed
    uint64_t *tfull = empty + SK_MAX_STAGES;              // accumulator complete
    uint64_t *rfull = tfull + 1;                          // peers' slices received
    uint32_t *tmem_slot = (uint32_t *)(rfull + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int cs = (int)cluster_nctarank();
    const int r = (int)cluster_ctarank();
    const int tile = blockIdx.x / cs;
    const int ft = tile / p.n_ttiles, tt = tile - ft * p.n_ttiles;
    const int num_k = (p.K + SK_BK - 1) / SK_BK;
    const int kt0 = r * p.kt_per, nkt = max(0, min(num_k, kt0 + p.kt_per) - kt0);
    const int tno = (TN + cs - 1) / cs;                   // token columns per owner
    auto ncols = [&](int o) { return max(0, min(TN, (o + 1) * tno) - o * tno); };
    const int c_beg = r * tno, c_end = c_beg + ncols(r);

    if (threadIdx.x == 0) {
        for (int s = 0; s < SK_MAX_STAGES; s++) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        mbar_init(tfull, 1);
        mbar_init(rfull, 1);
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmW);
        if (SILU) tma_prefetch_desc(&tmW2);
        tma_prefetch_desc(&tmX);
    }
    if (warp == 1) { tmem_alloc(tmem_slot, TN); tmem_relinquish(); }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    dep_launch();
    // the peers' slices of the owned columns will land on rfull
    if (threadIdx.x == 0) mbar_arrive_expect_tx(rfull, (uint32_t)((cs - 1) * (c_end - c_beg) * 512));
    cluster_arrive();                                     // (1) barriers initialised

    bool ok = true;
    float xv[PF];
    float qw[4];
    int *apos = (int *)(base + p.aux_off);                // QKV: [tno] positions
    int *aseq = apos + tno;                               //      [tno] KV slots
    float2 *arope = (float2 *)(base + p.aux_off + ((tno * 8 + 15) & ~15));   // [tno][64]
    if (warp == 0) {
        if (lane == 0) {
            auto load_w = [&](int i) {
                const int st = i % p.stages;
                uint8_t *sW = base + st * Cfg::STAGE;
                const int k = (kt0 + i) * SK_BK;
                mbar_arrive_expect_tx(&full[st], Cfg::STAGE);
                if (SILU) {   // 64 gate rows over 64 up rows of the same features
                    tma_load_2d(sW, &tmW, &full[st], k, ft * 64);
                    tma_load_2d(sW + 64 * 128, &tmW2, &full[st], k, ft * 64);
                } else {
                    tma_load_2d(sW, &tmW, &full[st], k, ft * 128);
                }
            };
            // the first ring pass of weight tiles, before the wait for the
            // previous kernel
            const int pre = min(nkt, p.stages);
            for (int i = 0; i < pre; i++) load_w(i);
            dep_wait();
            for (int i = 0; i < nkt && ok; i++) {
                const int st = i % p.stages;
                if (i >= pre) {
                    if (!(ok = mbar_wait(&empty[st], (uint32_t)(((i / p.stages) & 1) ^ 1)))) break;
                    load_w(i);
                }
                tma_load_2d(base + st * Cfg::STAGE + SK_W_BYTES, &tmX, &full[st], (kt0 + i) * SK_BK, tt * TN);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = umma_idesc_bf16(128, TN);
            for (int i = 0; i < nkt && ok; i++) {
                const int st = i % p.stages;
                if (!(ok = mbar_wait(&full[st], (uint32_t)((i / p.stages) & 1)))) break;
                tc_fence_after();
                const uint32_t a0 = smem_u32(base + st * Cfg::STAGE);
                const uint32_t b0 = a0 + SK_W_BYTES;
#pragma unroll
                for (int ks = 0; ks < SK_BK / 16; ks++)
                    umma_bf16(tmem, umma_desc_sw128(a0 + ks * 32), umma_desc_sw128(b0 + ks * 32), idesc,
                              (i | ks) != 0 ? 1u : 0u);
                umma_commit(&empty[st]);
            }
            umma_commit(tfull);
        }
    } else {
        dep_wait();
        if (EPI == SK_EPI_RESID && c_end - c_beg <= PF) {
            // the residual rows this thread adds to, fetched while the MMAs run
            const int n = ft * 128 + (threadIdx.x - 64);
#pragma unroll
            for (int j = 0; j < PF; j++) {
                const int t = tt * TN + c_beg + j;
                xv[j] = (c_beg + j < c_end && t < p.T && n < p.N) ? p.ep.out[(size_t)t * p.ep.ldo + n] : 0.f;
            }
        }
        if (EPI == SK_EPI_QKV) {
            // positions and slots of the owned tokens, then their RoPE rows
            // (64 (cos, sin) pairs = 512 B each) into shared memory
            const int i = threadIdx.x - 64;
            for (int c = c_beg + i; c < c_end; c += 128) {
                const int t = tt * TN + c;
                apos[c - c_beg] = t < p.T ? p.ep.tok_pos[t] : 0;
                aseq[c - c_beg] = t < p.T ? p.ep.tok_seq[t] : 0;
            }
            named_bar_sync(1, 128);
            if (ft < 24) {
                const uint16_t *w = ft < 16 ? p.ep.q_norm : p.ep.k_norm;
#pragma unroll
                for (int j = 0; j < 4; j++) qw[j] = bf16_bits_to_f32(w[lane + 32 * j]);
                const int n16 = (c_end - c_beg) * 32;         // 16-byte pieces
#pragma unroll 4
                for (int idx = i; idx < n16; idx += 128) {
                    const int k = idx >> 5, piece = idx & 31;
                    ((uint4 *)(arope + k * 64))[piece] = ((const uint4 *)(p.ep.rope + (size_t)apos[k] * 64))[piece];
                }
            }
        }
        ok = mbar_wait(tfull, 0);
        tc_fence_after();
        // own partial: lane = feature f (TMEM lane), 32 token columns per load
        const int q = warp & 3;
        const int f = q * 32 + lane;
#pragma unroll 1
        for (int c0 = 0; c0 < TN; c0 += 32) {
            uint32_t v[32];
            tmem_ld_32x32b_x32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)c0, v);
            tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 32; j++) stage[(c0 + j) * 128 + f] = __uint_as_float(v[j]);
        }
        fence_proxy_async_smem();                         // the bulk copies read `stage`
        named_bar_sync(1, 128);
    }
    __syncwarp();
    cluster_wait();                                       // (1) every peer's rfull is armed
    if (threadIdx.x == 64 && cs > 1) {
        // columns of owner o -> its slot [r]: one bulk copy per peer
        const uint32_t slot = smem_u32(recv) + (uint32_t)(r * tno * 512);
        const uint32_t bar = smem_u32(rfull);
        for (int o = 0; o < cs; o++) {
            const int n = ncols(o);
            if (o == r || n == 0) continue;
            bulk_copy_to_cluster(mapa_shared(slot, (uint32_t)o), stage + o * tno * 128, (uint32_t)(n * 512),
                                 mapa_shared(bar, (uint32_t)o));
        }
    }
    if (warp >= 2 && !mbar_wait_cluster(rfull, 0)) ok = false;
    tc_fence_before();
    cluster_arrive_relaxed();                             // (2) this CTA has all its slices
    if (warp >= 2 && ok) {
        // ---- owner: sum the cs slices in K order, then the epilogue ----
        const int i = threadIdx.x - 64;                   // 0..127
        const SkEpilogue &ep = p.ep;
        // acc[j] = sum over the cs K slices, in slice order, of column c + j
        // (j < CB, columns < c_end) for feature feat; the CB loads of a slice
        // are independent.
        auto sum_cols = [&](auto &acc, int c, int feat) {
            constexpr int CB = sizeof(acc) / sizeof(acc[0]);
#pragma unroll
            for (int j = 0; j < CB; j++) acc[j] = 0.f;
            for (int s = 0; s < cs; s++) {
                const float *src = s == r ? stage + c * 128 + feat : recv + (s * tno + c - c_beg) * 128 + feat;
#pragma unroll
                for (int j = 0; j < CB; j++)
                    if (c + j < c_end) acc[j] += src[j * 128];
            }
        };
        if (EPI == SK_EPI_F32 || EPI == SK_EPI_RESID) {
            const int n = ft * 128 + i;
            if (n < p.N) {
                // y + x for 8 columns from c (x8: this pass's residual values)
                auto pass = [&](int c, const float (&x8)[8]) {
                    float y[8];
                    sum_cols(y, c, i);
#pragma unroll
                    for (int j = 0; j < 8; j++) {
                        const int t = tt * TN + c + j;
                        if (c + j >= c_end || t >= p.T) break;
                        float *o = ep.out + (size_t)t * ep.ldo + n;
                        *o = EPI == SK_EPI_RESID ? x8[j] + y[j] : y[j];
                    }
                };
                if (EPI == SK_EPI_RESID && c_end - c_beg <= PF) {
#pragma unroll
                    for (int k = 0; k < PF; k += 8) {          // prefetched: static indices
                        if (c_beg + k >= c_end) break;
                        float x8[8];
#pragma unroll
                        for (int j = 0; j < 8; j++) x8[j] = xv[k + j];
                        pass(c_beg + k, x8);
                    }
                } else {
#pragma unroll 1
                    for (int c = c_beg; c < c_end; c += 8) {
                        float x8[8];
#pragma unroll
                        for (int j = 0; j < 8; j++) {              // loads issued together
                            const int t = tt * TN + c + j;
                            x8[j] = EPI == SK_EPI_RESID && c + j < c_end && t < p.T
                                        ? ep.out[(size_t)t * ep.ldo + n] : 0.f;
                        }
                        pass(c, x8);
                    }
                }
            }
        } else if (EPI == SK_EPI_SILU) {
            const int fi = i & 63;
            const int n = ft * 64 + fi;
            if (n < p.N) {
                // threads 0-63 take columns c_beg.., 64-127 the next 4 of every 8
#pragma unroll 1
                for (int c = c_beg + (i >> 6) * 4; c < c_end; c += 8) {
                    float g[4], u[4];
                    sum_cols(g, c, fi);
                    sum_cols(u, c, 64 + fi);
#pragma unroll
                    for (int j = 0; j < 4; j++) {
                        const int t = tt * TN + c + j;
                        if (c + j >= c_end || t >= p.T) break;
                        ep.h[(size_t)t * ep.ldh + n] = f32_to_bf16_rne(sk_silu_mul(g[j], u[j]));
                    }
                }
            }
        } else {
            // QKV: the tile is head ft of [q 16 | k 8 | v 8]; one warp per
            // token, lane holds features lane + 32 j (RoPE pairs j, j + 2), as
            // in the unfused per-head kernel.
            const int hd = ft;
#pragma unroll 1
            for (int c = c_beg + (warp - 2); c < c_end; c += 4) {
                const int t = tt * TN + c;
                if (t >= p.T) break;
                const int pos = apos[c - c_beg], seq = aseq[c - c_beg];
                float2 rp[2];
                if (hd < 24)
                    for (int j = 0; j < 2; j++) rp[j] = arope[(c - c_beg) * 64 + lane + 32 * j];
                float v[4] = {0.f, 0.f, 0.f, 0.f};
                for (int s = 0; s < cs; s++) {
                    const float *src = s == r ? stage + c * 128 : recv + (s * tno + c - c_beg) * 128;
#pragma unroll
                    for (int j = 0; j < 4; j++) v[j] += src[lane + 32 * j];
                }
                if (hd < 24) {
                    float ss = v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3];
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, o);
                    const float sc = 1.0f / sqrtf(ss / (float)HEAD + NORM_EPS);
#pragma unroll
                    for (int j = 0; j < 4; j++) v[j] = v[j] * sc * qw[j];
#pragma unroll
                    for (int j = 0; j < 2; j++) {
                        const float2 cs2 = rp[j];
                        const float a = v[j], b = v[j + 2];
                        v[j] = a * cs2.x - b * cs2.y;
                        v[j + 2] = b * cs2.x + a * cs2.y;
                    }
                }
                if (hd < 16) {
                    const size_t o = (size_t)t * ep.ldq + hd * HEAD + lane;
#pragma unroll
                    for (int j = 0; j < 4; j++) {
                        if (ep.q_f32) ep.q_f32[o + 32 * j] = v[j];
                        if (ep.q_bf16) ep.q_bf16[o + 32 * j] = f32_to_bf16_rne(v[j]);
                    }
                } else {
                    const int kvh = (hd - 16) & 7;
                    uint16_t *dst = (hd < 24 ? ep.kc : ep.vc) +
                                    (((size_t)(seq * N_LAYERS + ep.layer) * N_KV_HEADS + kvh) * ep.max_len +
                                     pos) * HEAD;
#pragma unroll
                    for (int j = 0; j < 4; j++) dst[lane + 32 * j] = f32_to_bf16_rne(v[j]);
                }
            }
        }
    }
    // (2) no CTA leaves while a peer's copy may still read its `stage` or
    // write its `recv`
    __syncwarp();
    cluster_wait();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, TN);
}

// Shared memory: [operand ring | own partial [TN][128] FP32 once the MMAs are
// done][receive slots [cs][tno][128] FP32][QKV: positions, slots, RoPE rows of
// the owned tokens][barriers].
struct SkLayout {
    int stage_region, recv_off, aux_off, bar_off, smem;
};
SkLayout sk_layout(int tn, int stages, int cs, int epi) {
    SkLayout l;
    const int stage = 128 * SK_BK * 2 + tn * SK_BK * 2;
    const int tno = (tn + cs - 1) / cs;
    l.stage_region = std::max(stages * stage, tn * 128 * 4);
    l.recv_off = l.stage_region;
    l.aux_off = l.recv_off + (cs > 1 ? cs * tno * 128 * 4 : 0);
    const int aux = epi == SK_EPI_QKV ? ((tno * 8 + 15) & ~15) + tno * 64 * 8 : 0;
    l.bar_off = (l.aux_off + aux + 15) & ~15;
    l.smem = 1024 + l.bar_off + SK_BAR_BYTES;
    return l;
}

void sk_config(cudaLaunchConfig_t *cfg, cudaLaunchAttribute *attr, cudaStream_t st, int ctas, int cs,
               int smem) {
    *cfg = {};
    cfg->gridDim = dim3(ctas);
    cfg->blockDim = dim3(SK_THREADS);
    cfg->dynamicSmemBytes = smem;
    cfg->stream = st;
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = cs;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg->attrs = attr;
    cfg->numAttrs = g_pdl ? 2 : 1;
}

template <int TN, int EPI>
int sk_prepare() {
    static bool attr_done[64] = {};
    int dev = 0;
    N550_CUDA_TRY(cudaGetDevice(&dev));
    if (dev >= 0 && dev < 64 && !attr_done[dev]) {
        N550_CUDA_TRY(cudaFuncSetAttribute(gemm_skinny_kernel<TN, EPI>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, SK_SMEM_MAX));
        N550_CUDA_TRY(cudaFuncSetAttribute(gemm_skinny_kernel<TN, EPI>,
                                           cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
        attr_done[dev] = true;
    }
    return N550_OK;
}

// Whether clusters of cs CTAs with this shared memory fit the GPU (cached).
template <int TN, int EPI>
bool sk_cluster_fits(int cs, int smem) {
    if (cs <= 8) return true;
    static int cache[64][SK_MAX_CS + 1][8];   // 0 unknown, 1 fits, 2 does not; smem in 32 KB steps
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return false;
    int &c = cache[dev][cs][std::min(7, smem >> 15)];
    if (!c) {
        cudaLaunchConfig_t cfg;
        cudaLaunchAttribute attr[2];
        // the largest shared memory of the 32 KB step decides
        sk_config(&cfg, attr, 0, cs, cs, std::min(SK_SMEM_MAX, ((smem >> 15) + 1) << 15));
        cfg.numAttrs = 1;
        int n = 0;
        c = (sk_prepare<TN, EPI>() == N550_OK &&
             cudaOccupancyMaxActiveClusters(&n, gemm_skinny_kernel<TN, EPI>, &cfg) == cudaSuccess && n > 0)
                ? 1 : 2;
        (void)cudaGetLastError();
    }
    return c == 1;
}

template <int TN, int EPI>
int sk_launch(cudaStream_t st, const CUtensorMap &tw, const CUtensorMap &tw2, const CUtensorMap &tx,
              const SkParams &p, int ctas, int cs, int smem) {
    int rc = sk_prepare<TN, EPI>();
    if (rc) return rc;
    cudaLaunchConfig_t cfg;
    cudaLaunchAttribute attr[2];
    sk_config(&cfg, attr, st, ctas, cs, smem);
    N550_CUDA_TRY(cudaLaunchKernelEx(&cfg, gemm_skinny_kernel<TN, EPI>, tw, tw2, tx, p));
    return N550_OK;
}

template <int TN>
int sk_dispatch(cudaStream_t st, int epi, const CUtensorMap &tw, const CUtensorMap &tw2,
                const CUtensorMap &tx, const SkParams &p, int ctas, int cs, int smem) {
    switch (epi) {
    case SK_EPI_F32: return sk_launch<TN, SK_EPI_F32>(st, tw, tw2, tx, p, ctas, cs, smem);
    case SK_EPI_RESID: return sk_launch<TN, SK_EPI_RESID>(st, tw, tw2, tx, p, ctas, cs, smem);
    case SK_EPI_SILU: return sk_launch<TN, SK_EPI_SILU>(st, tw, tw2, tx, p, ctas, cs, smem);
    case SK_EPI_QKV: return sk_launch<TN, SK_EPI_QKV>(st, tw, tw2, tx, p, ctas, cs, smem);
    default: return N550_ERR_ARG;
    }
}

bool sk_fits(int tn, int epi, int cs, int smem) {
    switch (tn * 4 + epi) {
    case 32 * 4 + SK_EPI_F32: return sk_cluster_fits<32, SK_EPI_F32>(cs, smem);
    case 32 * 4 + SK_EPI_RESID: return sk_cluster_fits<32, SK_EPI_RESID>(cs, smem);
    case 32 * 4 + SK_EPI_SILU: return sk_cluster_fits<32, SK_EPI_SILU>(cs, smem);
    case 32 * 4 + SK_EPI_QKV: return sk_cluster_fits<32, SK_EPI_QKV>(cs, smem);
    case 64 * 4 + SK_EPI_F32: return sk_cluster_fits<64, SK_EPI_F32>(cs, smem);
    case 64 * 4 + SK_EPI_RESID: return sk_cluster_fits<64, SK_EPI_RESID>(cs, smem);
    case 64 * 4 + SK_EPI_SILU: return sk_cluster_fits<64, SK_EPI_SILU>(cs, smem);
    case 64 * 4 + SK_EPI_QKV: return sk_cluster_fits<64, SK_EPI_QKV>(cs, smem);
    default: return false;
    }
}

int sk_num_sms() {
    static int n = 0;
    if (!n) {
        int dev = 0, v = 0;
        if (cudaGetDevice(&dev) == cudaSuccess &&
            cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && v > 0)
            n = v;
        else
            n = 148;
    }
    return n;
}

// K split and ring depth for `tiles` output tiles: cs CTAs per tile with
// kt_per k-tiles each (none empty), `stages` ring slots -- all k-tiles when
// they fit, fewer so that two CTAs share an SM when the grid exceeds the SMs.
bool sk_plan(int tn, int epi, int tiles, int num_k, int *cs, int *kt_per, int *stages, SkLayout *lay) {
    int c = std::min(std::min(std::max(*cs, 1), SK_MAX_CS), num_k);
    const int kt = (num_k + c - 1) / c;
    c = (num_k + kt - 1) / kt;
    if (c > tn) return false;                             // every rank owns a column
    const int limit = tiles * c > sk_num_sms() ? (233472 - 2 * 1024) / 2 : SK_SMEM_MAX;
    int sg = std::min(kt, SK_MAX_STAGES);
    while (sg > 2 && sk_layout(tn, sg, c, epi).smem > limit) sg--;
    const SkLayout l = sk_layout(tn, sg, c, epi);
    if (l.smem > SK_SMEM_MAX) return false;
    *cs = c;
    *kt_per = kt;
    *stages = sg;
    *lay = l;
    return true;
}

}  // namespace

int g_skinny_cs = 0;
int g_skinny_rows = SK_AUTO_T;
int g_skinny_rows_gemm = SK_AUTO_GEMM_T;

int launch_gemm_skinny(cudaStream_t st, int epi, const uint16_t *x, int ldx, const uint16_t *w,
                       const uint16_t *w2, int ldw, int T, int N, int K, const SkEpilogue &ep, int cs) {
    if (T <= 0 || N <= 0) return N550_OK;
    if (T > SK_MAX_T || K <= 0 || epi < SK_EPI_F32 || epi > SK_EPI_QKV) return N550_ERR_ARG;
    if (!tc_shape_ok(x, ldx, w, ldw, K)) return N550_ERR_UNSUPPORTED;
    const bool silu = epi == SK_EPI_SILU;
    if (silu && (!w2 || (((uintptr_t)w2) & 15) || !ep.h)) return N550_ERR_ARG;
    if ((epi == SK_EPI_F32 || epi == SK_EPI_RESID) && !ep.out) return N550_ERR_ARG;
    if (epi == SK_EPI_QKV && (N != 32 * HEAD || !ep.kc || !ep.vc || !ep.tok_pos || !ep.tok_seq ||
                              !ep.rope || !ep.q_norm || !ep.k_norm || (!ep.q_f32 && !ep.q_bf16)))
        return N550_ERR_ARG;
    const int tn = T <= 32 ? 32 : 64;
    const int n_tt = (T + tn - 1) / tn;
    const int rows = silu ? 64 : 128;
    const int tiles = (N + rows - 1) / rows * n_tt;
    const int num_k = (K + SK_BK - 1) / SK_BK;
    if (cs <= 0 && g_skinny_cs > 0) cs = g_skinny_cs;
    if (cs <= 0) {
        // enough CTAs to stream the weights from ~all SMs
        cs = 1;
        while (cs < SK_MAX_CS && tiles * cs < 120 && 2 * cs <= num_k) cs *= 2;
    }
    int kt_per = 0, stages = 0;
    SkLayout lay;
    if (!sk_plan(tn, epi, tiles, num_k, &cs, &kt_per, &stages, &lay)) return N550_ERR_UNSUPPORTED;
    if (!sk_fits(tn, epi, cs, lay.smem)) {
        cs = 8;      // portable cluster size
        if (!sk_plan(tn, epi, tiles, num_k, &cs, &kt_per, &stages, &lay) || cs > 8)
            return N550_ERR_UNSUPPORTED;
    }
    int rc = N550_OK;
    CUtensorMap tw, tw2, tx;
    if ((rc = tmap_bf16_sw128(&tw, w, (uint64_t)N, (uint64_t)K, (uint64_t)ldw, rows))) return rc;
    if (silu) {
        if ((rc = tmap_bf16_sw128(&tw2, w2, (uint64_t)N, (uint64_t)K, (uint64_t)ldw, rows))) return rc;
    } else {
        tw2 = tw;
    }
    if ((rc = tmap_bf16_sw128(&tx, x, (uint64_t)T, (uint64_t)K, (uint64_t)ldx, tn))) return rc;
    SkParams p;
    p.T = T;
    p.N = N;
    p.K = K;
    p.kt_per = kt_per;
    p.stages = stages;
    p.n_ttiles = n_tt;
    p.recv_off = lay.recv_off;
    p.aux_off = lay.aux_off;
    p.bar_off = lay.bar_off;
    p.ep = ep;
    if (tn == 32) return sk_dispatch<32>(st, epi, tw, tw2, tx, p, tiles * cs, cs, lay.smem);
    return sk_dispatch<64>(st, epi, tw, tw2, tx, p, tiles * cs, cs, lay.smem);
}

}  // namespace n550
