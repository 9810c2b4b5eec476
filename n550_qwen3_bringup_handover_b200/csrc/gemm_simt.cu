// CUDA-core GEMM paths of fast mode:
//  * gemm_simt: FP32-FMA tiled GEMM for shapes the TMA tensor-core path cannot
//    take (K % 8 != 0, unaligned strides or pointers) -- same contract.
//  * gemv: skinny M (decode, M <= 8): one warp per output column n streams
//    B[n, :] once with 16-byte loads; A rows come through L1. At M <= 8 the
//    FMA work per weight byte is below the B200 FP32 rate, so this stays
//    HBM-bound (the decode GEMV of kernels_ame.c at mtilem = 1).
//  * f32_to_bf16: RNE staging of FP32 activations (kernels_ame.c:220-236).
#include "common.cuh"
#include "gemm_tc.h"
#include "launch.h"

namespace n550 {
namespace {

constexpr int ST = 64, SK = 16, STHREADS = 256;

template <int EPI>
__device__ __forceinline__ void epi_store(void *c, int ldc, int m, int n, float v) {
    if (EPI == TC_EPI_F32) ((float *)c)[(size_t)m * ldc + n] = v;
    else if (EPI == TC_EPI_BF16) ((uint16_t *)c)[(size_t)m * ldc + n] = f32_to_bf16_rne(v);
    else ((float *)c)[(size_t)m * ldc + n] += v;
}

template <int EPI>
__global__ void __launch_bounds__(STHREADS)
gemm_simt_kernel(const uint16_t *__restrict__ a, int lda, const uint16_t *__restrict__ b, int ldb,
                 void *c, int ldc, int M, int N, int K) {
    dep_wait();
    dep_launch();
    __shared__ float As[SK][ST + 1];
    __shared__ float Bs[SK][ST + 1];
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int m0 = blockIdx.y * ST, n0 = blockIdx.x * ST;
    float acc[4][4] = {};
    for (int k0 = 0; k0 < K; k0 += SK) {
        for (int e = threadIdx.x; e < ST * SK; e += STHREADS) {
            const int r = e / SK, kk = e % SK, k = k0 + kk;
            As[kk][r] = (m0 + r < M && k < K) ? bf16_bits_to_f32(a[(size_t)(m0 + r) * lda + k]) : 0.f;
            Bs[kk][r] = (n0 + r < N && k < K) ? bf16_bits_to_f32(b[(size_t)(n0 + r) * ldb + k]) : 0.f;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < SK; kk++) {
            float av[4], bv[4];
#pragma unroll
            for (int i = 0; i < 4; i++) av[i] = As[kk][ty + 16 * i];
#pragma unroll
            for (int j = 0; j < 4; j++) bv[j] = Bs[kk][tx + 16 * j];
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int m = m0 + ty + 16 * i;
        if (m >= M) continue;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int n = n0 + tx + 16 * j;
            if (n < N) epi_store<EPI>(c, ldc, m, n, acc[i][j]);
        }
    }
}

constexpr int GV_WARPS = 8;
constexpr int GV_MAXM = 8;

__device__ __forceinline__ void bf16x8_to_f32(const uint4 q, float (&f)[8]) {
    f[0] = __uint_as_float(q.x << 16); f[1] = __uint_as_float(q.x & 0xFFFF0000u);
    f[2] = __uint_as_float(q.y << 16); f[3] = __uint_as_float(q.y & 0xFFFF0000u);
    f[4] = __uint_as_float(q.z << 16); f[5] = __uint_as_float(q.z & 0xFFFF0000u);
    f[6] = __uint_as_float(q.w << 16); f[7] = __uint_as_float(q.w & 0xFFFF0000u);
}

// 16-byte loads of one lane's step of a weight row: 4 independent loads of 8
// BF16 at k0, k0 + 256, k0 + 512, k0 + 768 (zeros past K).
__device__ __forceinline__ void gv_load_step(uint4 (&q)[4], const uint16_t *row, int k0, int K) {
#pragma unroll
    for (int u = 0; u < 4; u++) {
        const int k = k0 + u * 256;
        q[u] = (k < K) ? __ldcs((const uint4 *)(row + k)) : make_uint4(0, 0, 0, 0);
    }
}

// One warp per output column n; requires K % 8 == 0 and 16-byte aligned rows.
// The weights do not depend on the previous kernel, so rows of up to 3072
// elements (every projection of the model) are requested whole -- 12 16-byte
// loads per lane in flight -- before the programmatic-launch wait, and overlap
// that kernel's tail; the activations are read after it. Longer rows continue
// in steps of 4 loads per lane. The summation order does not depend on it.
constexpr int GV_PRE = 3;           // steps of 1024 elements held in registers

// Input RMSNorm fused into the GEMV (NORM; rows of K = 1024): the block
// normalises the FP32 rows nx[m] into shared memory before its dot products,
// rounded to BF16 -- one warp per row with the loads, sum order and
// arithmetic of norm_rows_bf16_kernel (the model's rmsnorm, qwen3.c:471/527,
// ops_scalar.c:11-15) -- so the products see exactly the activations that
// kernel would write, and the few-row decode layer needs no norm launches.
// The norm weight, no kernel's output, is copied to shared memory before the
// programmatic-launch wait, like the weight rows.
constexpr int GV_NORM_K = 1024;
constexpr int GV_NORM_MAXM = 4;     // rows (the decode step's GEMV route takes up to 3)
constexpr float GV_NORM_EPS = 1e-6f;

__device__ __forceinline__ float bf16_round_f32(float v) { return bf16_bits_to_f32(f32_to_bf16_rne(v)); }

__device__ __forceinline__ void gv_norm_weight(uint16_t *nws, const uint16_t *__restrict__ nw) {
    if (threadIdx.x < GV_NORM_K / 8) ((uint4 *)nws)[threadIdx.x] = __ldg((const uint4 *)nw + threadIdx.x);
}

// Warp m < MM normalises row m (after the wait). The row is read twice, the
// second time from L1, so that it is not held in registers beside the weight
// rows prefetched before the wait.
template <int MM>
__device__ __forceinline__ void gv_norm_rows(float (*xs)[GV_NORM_K], const float *__restrict__ nx,
                                             const uint16_t *nws) {
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();                         // nws complete
    if (w < MM) {
        const float4 *xr = (const float4 *)(nx + (size_t)w * GV_NORM_K);
        float ss = 0.f;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const float4 v = __ldg(xr + lane + 32 * i);
            ss = fmaf(v.x, v.x, ss);
            ss = fmaf(v.y, v.y, ss);
            ss = fmaf(v.z, v.z, ss);
            ss = fmaf(v.w, v.w, ss);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, o);
        const float sc = 1.0f / sqrtf(ss / (float)GV_NORM_K + GV_NORM_EPS);
        const uint2 *wr = (const uint2 *)nws;
        float4 *dst = (float4 *)xs[w];
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const float4 v = __ldg(xr + lane + 32 * i);
            const uint2 wv = wr[lane + 32 * i];
            float4 o;
            o.x = bf16_round_f32(v.x * sc * __uint_as_float(wv.x << 16));
            o.y = bf16_round_f32(v.y * sc * __uint_as_float(wv.x & 0xFFFF0000u));
            o.z = bf16_round_f32(v.z * sc * __uint_as_float(wv.y << 16));
            o.w = bf16_round_f32(v.w * sc * __uint_as_float(wv.y & 0xFFFF0000u));
            dst[lane + 32 * i] = o;
        }
    }
    __syncthreads();
}

// Eight activations a[m][k .. k + 8) as FP32: BF16 rows in global memory, or
// (NORM) the block's normalised rows in shared memory.
template <bool NORM>
__device__ __forceinline__ void gv_a8(float (&af)[8], const uint16_t *__restrict__ a, int lda,
                                      const float (*xs)[GV_NORM_K], int m, int k) {
    if constexpr (NORM) {
        const float4 lo = *(const float4 *)&xs[m][k], hi = *(const float4 *)&xs[m][k + 4];
        af[0] = lo.x; af[1] = lo.y; af[2] = lo.z; af[3] = lo.w;
        af[4] = hi.x; af[5] = hi.y; af[6] = hi.z; af[7] = hi.w;
    } else {
        bf16x8_to_f32(__ldg((const uint4 *)(a + (size_t)m * lda + k)), af);
    }
}

template <int MM, bool NORM = false>
__device__ __forceinline__ void gv_consume(const uint4 (&q)[4], const uint16_t *__restrict__ a, int lda,
                                           int k0, int K, float (&acc)[MM],
                                           const float (*xs)[GV_NORM_K] = nullptr) {
#pragma unroll
    for (int u = 0; u < 4; u++) {
        const int k = k0 + u * 256;
        if (k >= K) break;
        float bf[8];
        bf16x8_to_f32(q[u], bf);
#pragma unroll
        for (int m = 0; m < MM; m++) {
            float af[8];
            gv_a8<NORM>(af, a, lda, xs, m, k);
#pragma unroll
            for (int j = 0; j < 8; j++) acc[m] = fmaf(af[j], bf[j], acc[m]);
        }
    }
}

// NORM (K = 1024, one step): 4 blocks per SM (64 registers) hold the 512
// blocks of the q/k/v projection in one wave.
template <int MM, int EPI, bool NORM = false>
__global__ void __launch_bounds__(GV_WARPS * 32, NORM ? 4 : 1)
gemv_kernel(const uint16_t *__restrict__ a, int lda, const uint16_t *__restrict__ b, int ldb,
            void *c, int ldc, int N, int K, const float *__restrict__ nx, const uint16_t *__restrict__ nw) {
    __shared__ __align__(16) float xs[NORM ? MM : 1][GV_NORM_K];
    __shared__ __align__(16) uint16_t nws[NORM ? GV_NORM_K : 8];
    const int lane = threadIdx.x & 31;
    const int n = blockIdx.x * GV_WARPS + (threadIdx.x >> 5);
    const uint16_t *brow = b + (size_t)(n < N ? n : 0) * ldb;
    const int k_first = n < N ? lane * 8 : K;
    constexpr int PRE = NORM ? 1 : GV_PRE;
    uint4 bq[PRE][4];
#pragma unroll
    for (int s = 0; s < PRE; s++) gv_load_step(bq[s], brow, k_first + s * 1024, K);
    if constexpr (NORM) gv_norm_weight(nws, nw);
    dep_wait();
    dep_launch();
    if constexpr (NORM) gv_norm_rows<MM>(xs, nx, nws);
    if (n >= N) return;
    float acc[MM];
#pragma unroll
    for (int m = 0; m < MM; m++) acc[m] = 0.f;
#pragma unroll
    for (int s = 0; s < PRE; s++) gv_consume<MM, NORM>(bq[s], a, lda, lane * 8 + s * 1024, K, acc, xs);
    for (int k0 = lane * 8 + PRE * 1024; k0 < K; k0 += 1024) {
        uint4 q[4];
        gv_load_step(q, brow, k0, K);
        gv_consume<MM, NORM>(q, a, lda, k0, K, acc, xs);
    }
#pragma unroll
    for (int m = 0; m < MM; m++) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc[m] += __shfl_xor_sync(0xFFFFFFFFu, acc[m], o);
    }
    if (lane < MM) {
        float v = acc[0];
#pragma unroll
        for (int m = 1; m < MM; m++) if (lane == m) v = acc[m];
        epi_store<EPI>(c, ldc, lane, n, v);
    }
}

// Wide few-row GEMV with K = 1024 (the lm_head: 151,936 columns, 311 MB of
// weights, an HBM stream): each warp takes two adjacent columns, so 8
// 16-byte loads per lane are in flight before the dependency wait, and the
// block keeps a 64-register budget (4 resident blocks per SM), enough bytes
// in flight to stream at the copy rate. Per column the loads, FMA order and
// reduction are gemv_kernel's, so the results are the same bits.
template <int MM, int EPI>
__global__ void __launch_bounds__(GV_WARPS * 32, 4)
gemv_wide_kernel(const uint16_t *__restrict__ a, int lda, const uint16_t *__restrict__ b, int ldb,
                 void *c, int ldc, int N) {
    constexpr int K = 1024;
    const int lane = threadIdx.x & 31;
    const int n0 = 2 * (blockIdx.x * GV_WARPS + (threadIdx.x >> 5));
    uint4 bq[2][4];
#pragma unroll
    for (int j = 0; j < 2; j++) {
        const int n = n0 + j;
        gv_load_step(bq[j], b + (size_t)(n < N ? n : 0) * ldb, n < N ? lane * 8 : K, K);
    }
    dep_wait();
    dep_launch();
    if (n0 >= N) return;
    float acc[2][MM];
#pragma unroll
    for (int j = 0; j < 2; j++)
#pragma unroll
        for (int m = 0; m < MM; m++) acc[j][m] = 0.f;
#pragma unroll
    for (int j = 0; j < 2; j++) gv_consume<MM>(bq[j], a, lda, lane * 8, K, acc[j]);
#pragma unroll
    for (int j = 0; j < 2; j++) {
#pragma unroll
        for (int m = 0; m < MM; m++) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) acc[j][m] += __shfl_xor_sync(0xFFFFFFFFu, acc[j][m], o);
        }
        const int n = n0 + j;
        if (lane < MM && n < N) {
            float v = acc[j][0];
#pragma unroll
            for (int m = 1; m < MM; m++) if (lane == m) v = acc[j][m];
            epi_store<EPI>(c, ldc, lane, n, v);
        }
    }
}

// Rows of 2048-4096 elements (the o and down projections) with the K loop
// split over KS warps per output column, one 1024-element step each, partial
// sums added in step order: 4x the warps of gemv_kernel in flight for the
// same N, so that the few-row decode step's narrow projections (1024
// outputs) are not held back by one 8-warp block per SM. Each warp's weights
// are requested before the programmatic-launch wait; with x_ready (the
// caller's guarantee that no kernel still in flight writes c: in the decode
// layer the residual rows were last written two or more kernels back, which
// completed before the previous kernel passed its own wait) so are the
// residual rows of the RESID epilogue, through L2.
constexpr int GVK_COLS = 4;         // output columns per block

template <int MM, int EPI, int KS>
__global__ void __launch_bounds__(GVK_COLS * KS * 32)
gemv_ksplit_kernel(const uint16_t *__restrict__ a, int lda, const uint16_t *__restrict__ b, int ldb,
                   void *c, int ldc, int N, int K, int x_ready) {
    __shared__ float part[GVK_COLS][KS][MM];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int col = warp / KS, kp = warp % KS;
    const int n = blockIdx.x * GVK_COLS + col;
    const uint16_t *brow = b + (size_t)(n < N ? n : 0) * ldb;
    const int k0 = n < N ? kp * 1024 + lane * 8 : K;
    uint4 q[4];
    gv_load_step(q, brow, k0, K);
    const bool pre_x = EPI == TC_EPI_RESID_F32 && x_ready && kp == 0 && lane < MM && n < N;
    float xo = 0.f;
    if (pre_x) xo = __ldcg((const float *)c + (size_t)lane * ldc + n);
    dep_wait();
    dep_launch();
    float acc[MM];
#pragma unroll
    for (int m = 0; m < MM; m++) acc[m] = 0.f;
    if (n < N) gv_consume<MM>(q, a, lda, k0, K, acc);
#pragma unroll
    for (int m = 0; m < MM; m++) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc[m] += __shfl_xor_sync(0xFFFFFFFFu, acc[m], o);
    }
    if (lane == 0) {
#pragma unroll
        for (int m = 0; m < MM; m++) part[col][kp][m] = acc[m];
    }
    __syncthreads();
    if (kp == 0 && lane < MM && n < N) {
        float v = part[col][0][lane];
#pragma unroll
        for (int k = 1; k < KS; k++) v += part[col][k][lane];
        if (pre_x) ((float *)c)[(size_t)lane * ldc + n] = xo + v;
        else epi_store<EPI>(c, ldc, lane, n, v);
    }
}

// Gate and up rows of output n in one warp (h = silu(x . wg[n]) * (x . wu[n])
// as BF16, ops_scalar.c:46-51): the SwiGLU of the few-token decode step in one
// launch instead of two GEMVs and an elementwise kernel. Same per-row loop and
// reduction order as gemv_kernel, so g and u are the values those GEMVs give.
// NORM: 3 blocks per SM (85 registers) hold the 384 blocks of the model's
// gate/up projection in one wave.
template <int MM, bool NORM = false>
__global__ void __launch_bounds__(GV_WARPS * 32, NORM ? 3 : 1)
gemv_swiglu_kernel(const uint16_t *__restrict__ a, int lda, const uint16_t *__restrict__ wg,
                   const uint16_t *__restrict__ wu, int ldb, uint16_t *h, int ldh, int N, int K,
                   const float *__restrict__ nx, const uint16_t *__restrict__ nw) {
    __shared__ __align__(16) float xs[NORM ? MM : 1][GV_NORM_K];
    __shared__ __align__(16) uint16_t nws[NORM ? GV_NORM_K : 8];
    const int lane = threadIdx.x & 31;
    const int n = blockIdx.x * GV_WARPS + (threadIdx.x >> 5);
    const size_t row = (size_t)(n < N ? n : 0) * ldb;
    const uint16_t *grow = wg + row, *urow = wu + row;
    // first step's gate and up weights before the programmatic-launch wait
    uint4 gq[4], uq[4];
    gv_load_step(gq, grow, n < N ? lane * 8 : K, K);
    gv_load_step(uq, urow, n < N ? lane * 8 : K, K);
    if constexpr (NORM) gv_norm_weight(nws, nw);
    dep_wait();
    dep_launch();
    if constexpr (NORM) gv_norm_rows<MM>(xs, nx, nws);
    if (n >= N) return;
    float ag[MM], au[MM];
#pragma unroll
    for (int m = 0; m < MM; m++) ag[m] = au[m] = 0.f;
    for (int k0 = lane * 8; k0 < K; k0 += 32 * 8 * 4) {
        if (k0 != lane * 8) {
            gv_load_step(gq, grow, k0, K);
            gv_load_step(uq, urow, k0, K);
        }
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const int k = k0 + u * 256;
            if (k >= K) break;
            float gf[8], uf[8];
            bf16x8_to_f32(gq[u], gf);
            bf16x8_to_f32(uq[u], uf);
#pragma unroll
            for (int m = 0; m < MM; m++) {
                float af[8];
                gv_a8<NORM>(af, a, lda, xs, m, k);
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    ag[m] = fmaf(af[j], gf[j], ag[m]);
                    au[m] = fmaf(af[j], uf[j], au[m]);
                }
            }
        }
    }
#pragma unroll
    for (int m = 0; m < MM; m++) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            ag[m] += __shfl_xor_sync(0xFFFFFFFFu, ag[m], o);
            au[m] += __shfl_xor_sync(0xFFFFFFFFu, au[m], o);
        }
    }
    if (lane < MM) {
        float g = ag[0], u = au[0];
#pragma unroll
        for (int m = 1; m < MM; m++)
            if (lane == m) { g = ag[m]; u = au[m]; }
        h[(size_t)lane * ldh + n] = f32_to_bf16_rne((g / (1.0f + expf(-g))) * u);
    }
}

template <int MM>
int gemv_swiglu_dispatch(cudaStream_t st, const uint16_t *a, int lda, const uint16_t *wg,
                         const uint16_t *wu, int ldb, uint16_t *h, int ldh, int N, int K,
                         const float *nx, const uint16_t *nw) {
    const int grid = (N + GV_WARPS - 1) / GV_WARPS;
    if (nx) {
        if constexpr (MM <= GV_NORM_MAXM)
            N550_CUDA_TRY(launch_k(gemv_swiglu_kernel<MM, true>, grid, GV_WARPS * 32, 0, st, a, lda, wg, wu,
                                   ldb, h, ldh, N, K, nx, nw));
        else
            return N550_ERR_UNSUPPORTED;
    } else
        N550_CUDA_TRY(launch_k(gemv_swiglu_kernel<MM, false>, grid, GV_WARPS * 32, 0, st, a, lda, wg, wu, ldb,
                               h, ldh, N, K, nx, nw));
    return N550_OK;
}

__global__ void f32_to_bf16_kernel(uint16_t *out, int ldo, const float *in, int ldi,
                                   int rows, int cols) {
    dep_wait();
    dep_launch();
    const size_t total = (size_t)rows * cols;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
         i += (size_t)gridDim.x * blockDim.x) {
        const size_t r = i / cols, cc = i % cols;
        out[r * ldo + cc] = f32_to_bf16_rne(in[r * ldi + cc]);
    }
}

template <int MM>
int gemv_dispatch(cudaStream_t st, int epi, const uint16_t *a, int lda, const uint16_t *b,
                  int ldb, void *c, int ldc, int N, int K, bool x_ready, const float *nx,
                  const uint16_t *nw) {
    if (nx) {               // fused input norm: K = 1024, FP32 output, up to 4 rows
        if constexpr (MM <= GV_NORM_MAXM) {
            if (epi != TC_EPI_F32) return N550_ERR_UNSUPPORTED;
            N550_CUDA_TRY(launch_k(gemv_kernel<MM, TC_EPI_F32, true>, (N + GV_WARPS - 1) / GV_WARPS,
                                   GV_WARPS * 32, 0, st, a, lda, b, ldb, c, ldc, N, K, nx, nw));
            return N550_OK;
        } else {
            return N550_ERR_UNSUPPORTED;
        }
    }
    // 2-4 steps of 1024 and at most 2048 columns: one warp per step
    if (K > 1024 && K <= 4096 && N <= 2048) {
        const int ks = (K + 1023) / 1024;
        const int grid = (N + GVK_COLS - 1) / GVK_COLS;
        auto go = [&](auto kernel) {
            return launch_k(kernel, grid, GVK_COLS * ks * 32, 0, st, a, lda, b, ldb, c, ldc, N, K,
                            x_ready ? 1 : 0);
        };
        cudaError_t e;
        if (ks == 2) {
            if (epi == TC_EPI_F32) e = go(gemv_ksplit_kernel<MM, TC_EPI_F32, 2>);
            else if (epi == TC_EPI_BF16) e = go(gemv_ksplit_kernel<MM, TC_EPI_BF16, 2>);
            else if (epi == TC_EPI_RESID_F32) e = go(gemv_ksplit_kernel<MM, TC_EPI_RESID_F32, 2>);
            else return N550_ERR_ARG;
        } else if (ks == 3) {
            if (epi == TC_EPI_F32) e = go(gemv_ksplit_kernel<MM, TC_EPI_F32, 3>);
            else if (epi == TC_EPI_BF16) e = go(gemv_ksplit_kernel<MM, TC_EPI_BF16, 3>);
            else if (epi == TC_EPI_RESID_F32) e = go(gemv_ksplit_kernel<MM, TC_EPI_RESID_F32, 3>);
            else return N550_ERR_ARG;
        } else {
            if (epi == TC_EPI_F32) e = go(gemv_ksplit_kernel<MM, TC_EPI_F32, 4>);
            else if (epi == TC_EPI_BF16) e = go(gemv_ksplit_kernel<MM, TC_EPI_BF16, 4>);
            else if (epi == TC_EPI_RESID_F32) e = go(gemv_ksplit_kernel<MM, TC_EPI_RESID_F32, 4>);
            else return N550_ERR_ARG;
        }
        N550_CUDA_TRY(e);
        return N550_OK;
    }
    if (K == 1024 && N >= 65536) {          // the lm_head: an HBM stream
        const int grid = (N + 2 * GV_WARPS - 1) / (2 * GV_WARPS);
        auto gw = [&](auto kernel) {
            return launch_k(kernel, grid, GV_WARPS * 32, 0, st, a, lda, b, ldb, c, ldc, N);
        };
        cudaError_t e;
        if (epi == TC_EPI_F32) e = gw(gemv_wide_kernel<MM, TC_EPI_F32>);
        else if (epi == TC_EPI_BF16) e = gw(gemv_wide_kernel<MM, TC_EPI_BF16>);
        else if (epi == TC_EPI_RESID_F32) e = gw(gemv_wide_kernel<MM, TC_EPI_RESID_F32>);
        else return N550_ERR_ARG;
        N550_CUDA_TRY(e);
        return N550_OK;
    }
    const int grid = (N + GV_WARPS - 1) / GV_WARPS;
    auto go = [&](auto kernel) {
        return launch_k(kernel, grid, GV_WARPS * 32, 0, st, a, lda, b, ldb, c, ldc, N, K,
                        (const float *)nullptr, (const uint16_t *)nullptr);
    };
    cudaError_t e;
    if (epi == TC_EPI_F32) e = go(gemv_kernel<MM, TC_EPI_F32>);
    else if (epi == TC_EPI_BF16) e = go(gemv_kernel<MM, TC_EPI_BF16>);
    else if (epi == TC_EPI_RESID_F32) e = go(gemv_kernel<MM, TC_EPI_RESID_F32>);
    else return N550_ERR_ARG;
    N550_CUDA_TRY(e);
    return N550_OK;
}

}  // namespace

int launch_gemm_simt(cudaStream_t st, int epi, const uint16_t *a, int lda,
                     const uint16_t *b, int ldb, void *c, int ldc, int M, int N, int K) {
    if (M <= 0 || N <= 0) return N550_OK;
    const long long gy = (M + ST - 1) / ST;
    if (gy > 65535) return N550_ERR_UNSUPPORTED;
    dim3 grid((N + ST - 1) / ST, (unsigned)gy);
    auto go = [&](auto kernel) {
        return launch_k(kernel, grid, STHREADS, 0, st, a, lda, b, ldb, c, ldc, M, N, K);
    };
    cudaError_t e;
    if (epi == TC_EPI_F32) e = go(gemm_simt_kernel<TC_EPI_F32>);
    else if (epi == TC_EPI_BF16) e = go(gemm_simt_kernel<TC_EPI_BF16>);
    else if (epi == TC_EPI_RESID_F32) e = go(gemm_simt_kernel<TC_EPI_RESID_F32>);
    else return N550_ERR_ARG;
    N550_CUDA_TRY(e);
    return N550_OK;
}

// The fused input norm's requirements: rows of K = 1024, 16-byte aligned
// rows and norm weight.
bool gv_norm_ok(int K, const float *nx, const uint16_t *nw) {
    return K == GV_NORM_K && nw && !(((uintptr_t)nx) & 15) && !(((uintptr_t)nw) & 15);
}

int launch_gemv(cudaStream_t st, int epi, const uint16_t *a, int lda,
                const uint16_t *b, int ldb, void *c, int ldc, int M, int N, int K, bool x_ready,
                const float *nx, const uint16_t *nw) {
    if (M <= 0 || N <= 0) return N550_OK;
    if (M > GV_MAXM || (K % 8) || (ldb % 8) || (((uintptr_t)b) & 15)) return N550_ERR_UNSUPPORTED;
    if (nx ? !gv_norm_ok(K, nx, nw) : ((lda % 8) || (((uintptr_t)a) & 15))) return N550_ERR_UNSUPPORTED;
    switch (M) {
    case 1: return gemv_dispatch<1>(st, epi, a, lda, b, ldb, c, ldc, N, K, x_ready, nx, nw);
    case 2: return gemv_dispatch<2>(st, epi, a, lda, b, ldb, c, ldc, N, K, x_ready, nx, nw);
    case 3: return gemv_dispatch<3>(st, epi, a, lda, b, ldb, c, ldc, N, K, x_ready, nx, nw);
    case 4: return gemv_dispatch<4>(st, epi, a, lda, b, ldb, c, ldc, N, K, x_ready, nx, nw);
    case 5: return gemv_dispatch<5>(st, epi, a, lda, b, ldb, c, ldc, N, K, x_ready, nx, nw);
    case 6: return gemv_dispatch<6>(st, epi, a, lda, b, ldb, c, ldc, N, K, x_ready, nx, nw);
    case 7: return gemv_dispatch<7>(st, epi, a, lda, b, ldb, c, ldc, N, K, x_ready, nx, nw);
    default: return gemv_dispatch<8>(st, epi, a, lda, b, ldb, c, ldc, N, K, x_ready, nx, nw);
    }
}

int launch_gemv_swiglu(cudaStream_t st, const uint16_t *a, int lda, const uint16_t *wg,
                       const uint16_t *wu, int ldb, uint16_t *h, int ldh, int M, int N, int K,
                       const float *nx, const uint16_t *nw) {
    if (M <= 0 || N <= 0) return N550_OK;
    if (M > GV_MAXM || (K % 8) || (ldb % 8) || (((uintptr_t)wg) & 15) || (((uintptr_t)wu) & 15) || !h)
        return N550_ERR_UNSUPPORTED;
    if (nx ? !gv_norm_ok(K, nx, nw) : ((lda % 8) || (((uintptr_t)a) & 15))) return N550_ERR_UNSUPPORTED;
    switch (M) {
    case 1: return gemv_swiglu_dispatch<1>(st, a, lda, wg, wu, ldb, h, ldh, N, K, nx, nw);
    case 2: return gemv_swiglu_dispatch<2>(st, a, lda, wg, wu, ldb, h, ldh, N, K, nx, nw);
    case 3: return gemv_swiglu_dispatch<3>(st, a, lda, wg, wu, ldb, h, ldh, N, K, nx, nw);
    case 4: return gemv_swiglu_dispatch<4>(st, a, lda, wg, wu, ldb, h, ldh, N, K, nx, nw);
    case 5: return gemv_swiglu_dispatch<5>(st, a, lda, wg, wu, ldb, h, ldh, N, K, nx, nw);
    case 6: return gemv_swiglu_dispatch<6>(st, a, lda, wg, wu, ldb, h, ldh, N, K, nx, nw);
    case 7: return gemv_swiglu_dispatch<7>(st, a, lda, wg, wu, ldb, h, ldh, N, K, nx, nw);
    default: return gemv_swiglu_dispatch<8>(st, a, lda, wg, wu, ldb, h, ldh, N, K, nx, nw);
    }
}

int launch_f32_to_bf16(cudaStream_t st, uint16_t *out, int ldo, const float *in, int ldi,
                       int rows, int cols) {
    if (rows <= 0 || cols <= 0) return N550_OK;
    const size_t total = (size_t)rows * cols;
    int grid = (int)((total + 255) / 256);
    if (grid > 148 * 16) grid = 148 * 16;
    N550_CUDA_TRY(launch_k(f32_to_bf16_kernel, grid, 256, 0, st, out, ldo, in, ldi, rows, cols));
    return N550_OK;
}

}  // namespace n550
