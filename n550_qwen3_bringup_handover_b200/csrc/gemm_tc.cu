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

#include "common.cuh"
#include "gemm_tc.h"

namespace n550 {
namespace {

constexpr int BM = 128;
constexpr int BK = 64;            // one 128-byte swizzle row of BF16
constexpr int UMMA_K = 16;
constexpr int THREADS = 192;

template <int BN>
struct TcCfg {
    static constexpr int STAGES = (BN >= 256) ? 4 : 6;
    static constexpr int A_BYTES = BM * BK * 2;
    static constexpr int B_BYTES = BN * BK * 2;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int TMEM_COLS = 2 * BN;
    static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 256;
};

__device__ __forceinline__ float silu_mul_f(float g, float u) {
    return (g / (1.0f + expf(-g))) * u;   // ops_scalar.c:46-51
}

// Epilogue for one 32-column chunk of one row. `v` holds FP32 accumulators.
template <int EPI>
__device__ __forceinline__ void store_chunk(const TcEpilogue &ep, int m, int n, int ncols_valid,
                                            const float (&v)[32]) {
    if (EPI == TC_EPI_F32) {
        float *dst = (float *)ep.c + (size_t)m * ep.ldc + n;
        if (ncols_valid == 32 && ep.vec_ok) {
#pragma unroll
            for (int j = 0; j < 32; j += 4)
                *(float4 *)(dst + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
        } else {
            for (int j = 0; j < ncols_valid; j++) dst[j] = v[j];
        }
    } else if (EPI == TC_EPI_BF16) {
        uint16_t *dst = (uint16_t *)ep.c + (size_t)m * ep.ldc + n;
        if (ncols_valid == 32 && ep.vec_ok) {
#pragma unroll
            for (int j = 0; j < 32; j += 8) {
                uint4 q;
                q.x = pack_bf16x2(v[j], v[j + 1]);
                q.y = pack_bf16x2(v[j + 2], v[j + 3]);
                q.z = pack_bf16x2(v[j + 4], v[j + 5]);
                q.w = pack_bf16x2(v[j + 6], v[j + 7]);
                *(uint4 *)(dst + j) = q;
            }
        } else {
            for (int j = 0; j < ncols_valid; j++) dst[j] = f32_to_bf16_rne(v[j]);
        }
    } else if (EPI == TC_EPI_RESID_F32) {
        // x += y in FP32 (ops_scalar.c:53-55), y = this GEMM's output.
        float *dst = (float *)ep.c + (size_t)m * ep.ldc + n;
        if (ncols_valid == 32 && ep.vec_ok) {
#pragma unroll
            for (int j = 0; j < 32; j += 4) {
                float4 x = *(float4 *)(dst + j);
                x.x += v[j]; x.y += v[j + 1]; x.z += v[j + 2]; x.w += v[j + 3];
                *(float4 *)(dst + j) = x;
            }
        } else {
            for (int j = 0; j < ncols_valid; j++) dst[j] += v[j];
        }
    }
}

template <int BN, int EPI>
__global__ void __launch_bounds__(THREADS, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA,
               const __grid_constant__ CUtensorMap tmB,
               const __grid_constant__ CUtensorMap tmB2,
               const TcEpilogue ep, int M, int N, int K) {
    using Cfg = TcCfg<BN>;
    constexpr int STAGES = Cfg::STAGES;
    constexpr bool SILU = (EPI == TC_EPI_SILU_BF16);
    // Output columns per tile: SILU tiles hold BN/2 gate + BN/2 up columns.
    constexpr int OUT_N = SILU ? BN / 2 : BN;

    extern __shared__ uint8_t smem_raw[];
    uint8_t *base = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t *full = (uint64_t *)(base + STAGES * Cfg::STAGE_BYTES);
    uint64_t *empty = full + STAGES;
    uint64_t *tfull = empty + STAGES;       // [2]
    uint64_t *tempty = tfull + 2;           // [2]
    uint64_t *done = tempty + 2;            // [1] MMA drain at exit
    uint32_t *tmem_slot = (uint32_t *)(done + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    const int num_m = (M + BM - 1) / BM;
    const int num_n = (N + OUT_N - 1) / OUT_N;
    const int total = num_m * num_n;
    const int num_k = (K + BK - 1) / BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        for (int b = 0; b < 2; b++) { mbar_init(&tfull[b], 1); mbar_init(&tempty[b], 128); }
        mbar_init(done, 1);
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
        if (SILU) tma_prefetch_desc(&tmB2);
    }
    if (warp == 1) { tmem_alloc(tmem_slot, Cfg::TMEM_COLS); tmem_relinquish(); }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            long long issued = 0;
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
                const int mb = t / num_n, nb = t % num_n;
                for (int kt = 0; kt < num_k; kt++) {
                    if (!mbar_wait(&empty[stage], phase ^ 1)) { ok = false; break; }
                    uint8_t *sA = base + stage * Cfg::STAGE_BYTES;
                    uint8_t *sB = sA + Cfg::A_BYTES;
                    mbar_arrive_expect_tx(&full[stage], Cfg::STAGE_BYTES);
                    tma_load_2d(sA, &tmA, &full[stage], kt * BK, mb * BM);
                    if (SILU) {
                        tma_load_2d(sB, &tmB, &full[stage], kt * BK, nb * (BN / 2));
                        tma_load_2d(sB + (BN / 2) * BK * 2, &tmB2, &full[stage], kt * BK,
                                    nb * (BN / 2));
                    } else {
                        tma_load_2d(sB, &tmB, &full[stage], kt * BK, nb * BN);
                    }
                    issued++;
                    if (++stage == STAGES) { stage = 0; phase ^= 1; }
                }
            }
            // Drain: every load issued must have landed before the CTA exits.
            long long first = issued > STAGES ? issued - STAGES : 0;
            for (long long i = first; i < issued; i++)
                if (!mbar_wait(&full[i % STAGES], (uint32_t)((i / STAGES) & 1))) break;
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            constexpr uint32_t idesc = umma_idesc_bf16(BM, BN);
            int stage = 0;
            uint32_t phase = 0;
            int ab = 0;
            uint32_t aphase = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
                if (!mbar_wait(&tempty[ab], aphase ^ 1)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + (uint32_t)(ab * BN);
                for (int kt = 0; kt < num_k; kt++) {
                    if (!mbar_wait(&full[stage], phase)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t a0 = smem_u32(base + stage * Cfg::STAGE_BYTES);
                    const uint32_t b0 = a0 + Cfg::A_BYTES;
#pragma unroll
                    for (int ks = 0; ks < BK / UMMA_K; ks++) {
                        umma_bf16(d_tmem, umma_desc_sw128(a0 + ks * UMMA_K * 2),
                                  umma_desc_sw128(b0 + ks * UMMA_K * 2), idesc,
                                  (kt | ks) != 0);
                    }
                    umma_commit(&empty[stage]);
                    if (++stage == STAGES) { stage = 0; phase ^= 1; }
                }
                if (!ok) break;
                umma_commit(&tfull[ab]);
                if (++ab == 2) { ab = 0; aphase ^= 1; }
            }
            // Drain all MMAs of this thread before TMEM is released.
            umma_commit(done);
            mbar_wait(done, 0);
        }
    } else {
        // ---------------- epilogue (warps 2..5) ----------------
        const int q = warp & 3;                 // TMEM lane quarter of this warp
        const int row = q * 32 + lane;
        int ab = 0;
        uint32_t aphase = 0;
        for (int t = blockIdx.x; t < total; t += gridDim.x) {
            const int mb = t / num_n, nb = t % num_n;
            if (!mbar_wait(&tfull[ab], aphase)) break;
            tc_fence_after();
            const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(ab * BN);
            const int m = mb * BM + row;
            if (SILU) {
#pragma unroll 1
                for (int cch = 0; cch < OUT_N; cch += 32) {
                    uint32_t rg[32], ru[32];
                    tmem_ld_32x32b_x32(taddr + cch, rg);
                    tmem_ld_32x32b_x32(taddr + OUT_N + cch, ru);
                    tmem_ld_wait();
                    const int n = nb * OUT_N + cch;
                    if (m < M && n < N) {
                        float v[32];
#pragma unroll
                        for (int j = 0; j < 32; j++)
                            v[j] = silu_mul_f(__uint_as_float(rg[j]), __uint_as_float(ru[j]));
                        store_chunk<TC_EPI_BF16>(ep, m, n, min(32, N - n), v);
                    }
                }
            } else {
#pragma unroll 1
                for (int cch = 0; cch < BN; cch += 32) {
                    uint32_t r[32];
                    tmem_ld_32x32b_x32(taddr + cch, r);
                    tmem_ld_wait();
                    const int n = nb * BN + cch;
                    if (m < M && n < N) {
                        float v[32];
#pragma unroll
                        for (int j = 0; j < 32; j++) v[j] = __uint_as_float(r[j]);
                        store_chunk<EPI>(ep, m, n, min(32, N - n), v);
                    }
                }
            }
            tc_fence_before();
            mbar_arrive(&tempty[ab]);
            if (++ab == 2) { ab = 0; aphase ^= 1; }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
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

template <int BN, int EPI>
int launch_impl(cudaStream_t st, const CUtensorMap &ta, const CUtensorMap &tb,
                const CUtensorMap &tb2, const TcEpilogue &ep, int M, int N, int K,
                int max_ctas) {
    using Cfg = TcCfg<BN>;
    static bool attr_done[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr_done[dev]) {
        N550_CUDA_TRY(cudaFuncSetAttribute(gemm_tc_kernel<BN, EPI>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           Cfg::SMEM_BYTES));
        attr_done[dev] = true;
    }
    constexpr int OUT_N = (EPI == TC_EPI_SILU_BF16) ? BN / 2 : BN;
    const long long tiles = (long long)((M + BM - 1) / BM) * ((N + OUT_N - 1) / OUT_N);
    int grid = num_sms();
    if (max_ctas > 0 && max_ctas < grid) grid = max_ctas;
    if (tiles < grid) grid = (int)tiles;
    gemm_tc_kernel<BN, EPI><<<grid, THREADS, Cfg::SMEM_BYTES, st>>>(ta, tb, tb2, ep, M, N, K);
    N550_LAUNCH_CHECK();
    return N550_OK;
}

}  // namespace

bool tc_shape_ok(const void *a, int lda, const void *b, int ldb, int K) {
    return K > 0 && (K % 8) == 0 && (lda % 8) == 0 && (ldb % 8) == 0 &&
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
    const int brows = (epi == TC_EPI_SILU_BF16) ? bn / 2 : bn;
    CUtensorMap ta, tb, tb2;
    if ((rc = make_tmap(&ta, a, M, K, lda, BM))) return rc;
    if ((rc = make_tmap(&tb, b, N, K, ldb, brows))) return rc;
    if (epi == TC_EPI_SILU_BF16) {
        if ((rc = make_tmap(&tb2, b2, N, K, ldb, brows))) return rc;
    } else {
        tb2 = tb;
    }
    TcEpilogue ep;
    ep.c = c;
    ep.ldc = ldc;
    const int esz = (epi == TC_EPI_BF16 || epi == TC_EPI_SILU_BF16) ? 2 : 4;
    ep.vec_ok = ((((uintptr_t)c) & 15) == 0) && ((ldc * esz) % 16 == 0);
#define N550_TC_CASE(BNV, EV) \
    if (bn == BNV && epi == EV) return launch_impl<BNV, EV>(st, ta, tb, tb2, ep, M, N, K, max_ctas);
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
