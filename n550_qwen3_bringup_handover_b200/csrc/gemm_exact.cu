// Exact-mode GEMM: the AME golden numerics, bit-for-bit.
//
// Rule (rtl_verification/golden_src/40_gen_ame_vectors.py:121-143 with
// K_BLOCK = kblock; the shipped c_ref.bin files pin kblock = 16, matching
// kernels_hwsim.c:31 HW_ROUND_K): per output and per K-block,
//     acc <- binary32_rne( binary64_rne( acc + sum_k a_k * b_k ) )
// with the block sum exact. A is BF16 (or FP32 rounded to BF16 RNE on load,
// as kernels_ame.c:220-236 stages it), B is BF16, C is FP32.
//
// How it is exact on CUDA cores: every bf16 x bf16 product has at most 16
// significant bits and is exact in binary64. The block is summed as a
// TwoSum chain s <- s + p; the chain's rounding errors are accumulated as
// |err|. If all errors are zero the binary64 s IS the exact sum, the first
// rounding is the identity, and one binary32 rounding finishes the rule.
// Otherwise (wide dynamic range inside one block, e.g. the +-6912 outliers
// of case 008) that output's block is recomputed in an integer
// superaccumulator and rounded twice exactly like the generator.
// An exactly-zero block result is +0.0 (a Fraction has no signed zero).
// Non-finite inputs are unpinned by the reference; they are summed in IEEE
// binary64.
#include "common.cuh"
#include "launch.h"

namespace n550 {

__device__ int g_device_status = 0;

namespace {

constexpr int THREADS = 256;
constexpr int MAXKB = 32;

// ---- integer superaccumulator (bit 0 = 2^-XBIAS), 20 x 32-bit limbs ----
constexpr int XLIMBS = 20;
constexpr int XBIAS = 288;

__device__ __forceinline__ void xadd(long long (&L)[XLIMBS], int neg,
                                     unsigned long long mant, int exp) {
    if (!mant) return;
    const int p = exp + XBIAS;
    const int li = p >> 5, off = p & 31;
    const unsigned long long v = mant << off;
    long long lo = (long long)(v & 0xFFFFFFFFull), hi = (long long)(v >> 32);
    if (neg) { lo = -lo; hi = -hi; }
    L[li] += lo;
    L[li + 1] += hi;
}

// Exact sum -> binary64 round-half-even (exact zero -> +0.0).
__device__ double xround_f64(long long (&L)[XLIMBS]) {
    unsigned long long U[XLIMBS];
    long long carry = 0;
#pragma unroll
    for (int i = 0; i < XLIMBS; i++) {
        long long v = L[i] + carry;
        carry = v >> 32;                      // arithmetic shift: floor(v / 2^32)
        U[i] = (unsigned long long)(v & 0xFFFFFFFFll);
    }
    const bool neg = carry < 0;
    if (neg) {
        unsigned long long c = 1;
#pragma unroll
        for (int i = 0; i < XLIMBS; i++) {
            unsigned long long v = ((~U[i]) & 0xFFFFFFFFull) + c;
            U[i] = v & 0xFFFFFFFFull;
            c = v >> 32;
        }
    }
    int t = XLIMBS - 1;
    while (t >= 0 && U[t] == 0) t--;
    if (t < 0) return 0.0;
    const int msb = 32 * t + (31 - __clz((unsigned)U[t]));
    const int start = msb - 63;
    unsigned long long W;
    bool sticky = false;
    if (start <= 0) {
        W = (U[0] | (U[1] << 32)) << (-start);
    } else {
        const int li = start >> 5, off = start & 31;
        const unsigned long long l0 = U[li];
        const unsigned long long l1 = (li + 1 < XLIMBS) ? U[li + 1] : 0ull;
        const unsigned long long l2 = (li + 2 < XLIMBS) ? U[li + 2] : 0ull;
        W = (l0 >> off) | (l1 << (32 - off));
        if (off) W |= l2 << (64 - off);
        for (int i = 0; i < li; i++) sticky |= (U[i] != 0);
        sticky |= (l0 & ((1ull << off) - 1ull)) != 0;
    }
    unsigned long long mant = W >> 11;
    const bool rbit = (W >> 10) & 1ull;
    sticky |= (W & 0x3FFull) != 0;
    int e = start + 11 - XBIAS;
    if (rbit && (sticky || (mant & 1ull))) {
        mant++;
        if (mant == (1ull << 53)) { mant >>= 1; e++; }
    }
    const double d = scalbn((double)mant, e);
    return neg ? -d : d;
}

// One block of the rule, exactly: operands are BF16 values held as FP32 in
// shared memory (a[k*stride], b[k*stride]).
__device__ __noinline__ float exact_block(float acc, const float *a, const float *b,
                                          int sa, int sb, int len) {
    bool finite = isfinite(acc);
    for (int k = 0; k < len; k++)
        finite = finite && isfinite(a[k * sa]) && isfinite(b[k * sb]);
    if (!finite) {
        double s = (double)acc;
        for (int k = 0; k < len; k++)
            s = __dadd_rn(s, __dmul_rn((double)a[k * sa], (double)b[k * sb]));
        return __double2float_rn(s);
    }
    long long L[XLIMBS];
#pragma unroll
    for (int i = 0; i < XLIMBS; i++) L[i] = 0;
    {
        const uint32_t u = __float_as_uint(acc);
        const int ex = (u >> 23) & 0xFF;
        const unsigned long long m = ex ? (0x800000u | (u & 0x7FFFFFu)) : (u & 0x7FFFFFu);
        xadd(L, (int)(u >> 31), m, ex ? ex - 150 : -149);
    }
    for (int k = 0; k < len; k++) {
        const uint32_t ua = __float_as_uint(a[k * sa]) >> 16;
        const uint32_t ub = __float_as_uint(b[k * sb]) >> 16;
        const int ea = (ua >> 7) & 0xFF, eb = (ub >> 7) & 0xFF;
        const unsigned long long ma = ea ? (128u + (ua & 0x7Fu)) : (ua & 0x7Fu);
        const unsigned long long mb = eb ? (128u + (ub & 0x7Fu)) : (ub & 0x7Fu);
        xadd(L, (int)((ua ^ ub) >> 15) & 1, ma * mb,
             (ea ? ea - 134 : -133) + (eb ? eb - 134 : -133));
    }
    return __double2float_rn(xround_f64(L));
}

// CH consecutive K-blocks of KB products for one output (operands a[k * SA],
// b[k * SB]), as independent TwoSum chains: the first from the accumulator, the
// others from zero. They are then applied in order: an error-free chain is the
// exact block sum, so one binary64 addition to the accumulator is the rule's
// binary64_rne(acc + block); a chain with an error goes to exact_block. The
// independent chains hide the FP64 latency of a thread's single output.
// Returns the K elements consumed (whole groups of CH blocks within len).
template <int CH, int KB, int SA, int SB>
__device__ __forceinline__ int exact_chains(float &acc, const float *a, const float *b, int len) {
    int kb0 = 0;
    for (; kb0 + CH * KB <= len; kb0 += CH * KB) {
        double s[CH], e[CH];
#pragma unroll
        for (int q = 0; q < CH; q++) { s[q] = q == 0 ? (double)acc : 0.0; e[q] = 0.0; }
#pragma unroll
        for (int kk = 0; kk < KB; kk++) {
#pragma unroll
            for (int q = 0; q < CH; q++) {
                const int k = kb0 + q * KB + kk;
                const double p = __dmul_rn((double)a[k * SA], (double)b[k * SB]);      // exact
                const double t = __dadd_rn(s[q], p);
                const double bp = __dsub_rn(t, s[q]);
                const double err = __dadd_rn(__dsub_rn(s[q], __dsub_rn(t, bp)), __dsub_rn(p, bp));
                s[q] = t;
                e[q] = __dadd_rn(e[q], fabs(err));
            }
        }
#pragma unroll
        for (int q = 0; q < CH; q++) {
            if (e[q] != 0.0 || !isfinite(s[q])) {
                acc = exact_block(acc, a + (kb0 + q * KB) * SA, b + (kb0 + q * KB) * SB, SA, SB, KB);
            } else if (q == 0) {
                acc = (s[q] == 0.0) ? 0.0f : __double2float_rn(s[q]);
            } else {
                const double t = __dadd_rn((double)acc, s[q]);
                acc = (t == 0.0) ? 0.0f : __double2float_rn(t);
            }
        }
    }
    return kb0;
}

// TM x TN outputs per CTA, RM x RN per thread (THREADS = TM/RM x TN/RN): 64 x 64
// tiles of 4 x 4 for many rows, 16 x 16 tiles of one output per thread for
// few rows (decode, BASELINE configs[0]'s 16 rows), so that such GEMMs spread
// over 8x more CTAs instead of computing mostly padding rows.
// KC: K elements staged in shared memory at a time (a multiple of 32, so whole
// K-blocks of 16 or 32); the small tiles stage 256 so that the global loads of
// 16 K-blocks are in flight together.
// CH > 1 (one output per thread only): whole groups of CH K-blocks go through
// exact_chains, the rest of a stage block by block.
template <bool A_F32, int TM, int TN, int RM, int RN, int KC, int CH = 1>
__global__ void __launch_bounds__(THREADS)
gemm_exact_kernel(const void *__restrict__ a_ptr, int lda,
                  const uint16_t *__restrict__ b, int ldb,
                  float *__restrict__ c, int ldc, int M, int N, int K, int kblock) {
    static_assert((TM / RM) * (TN / RN) == THREADS, "one thread per RM x RN outputs");
    constexpr int CX = TN / RN, CY = TM / RM;
    dep_wait();
    dep_launch();
    static_assert(KC % MAXKB == 0, "whole K-blocks per stage");
    __shared__ float As[KC][TM];
    __shared__ float Bs[KC][TN];
    const int tx = threadIdx.x % CX, ty = threadIdx.x / CX;
    const int m0 = blockIdx.y * TM, n0 = blockIdx.x * TN;

    float acc[RM][RN];
#pragma unroll
    for (int i = 0; i < RM; i++)
#pragma unroll
        for (int j = 0; j < RN; j++) acc[i][j] = 0.0f;

    for (int kc0 = 0; kc0 < K; kc0 += KC) {
        const int clen = min(KC, K - kc0);
        // Stage K elements [kc0, kc0 + clen) of rows m0.. of A and n0.. of B.
        for (int e = threadIdx.x; e < TM * KC; e += THREADS) {
            const int r = e / KC, kk = e - r * KC;
            float av = 0.0f;
            if (kk < clen && m0 + r < M) {
                if (A_F32) {
                    const float *ar = (const float *)a_ptr + (size_t)(m0 + r) * lda;
                    av = bf16_bits_to_f32(f32_to_bf16_rne(ar[kc0 + kk]));
                } else {
                    const uint16_t *ar = (const uint16_t *)a_ptr + (size_t)(m0 + r) * lda;
                    av = bf16_bits_to_f32(ar[kc0 + kk]);
                }
            }
            As[kk][r] = av;
        }
        for (int e = threadIdx.x; e < TN * KC; e += THREADS) {
            const int r = e / KC, kk = e - r * KC;
            float bv = 0.0f;
            if (kk < clen && n0 + r < N) bv = bf16_bits_to_f32(b[(size_t)(n0 + r) * ldb + kc0 + kk]);
            Bs[kk][r] = bv;
        }
        __syncthreads();
      int kb_done = 0;                    // K elements of this stage already applied
      if constexpr (CH > 1) {
        static_assert(RM == 1 && RN == 1, "chains of one output per thread");
        kb_done = kblock == 16 ? exact_chains<CH, 16, TM, TN>(acc[0][0], &As[0][ty], &Bs[0][tx], clen)
                               : exact_chains<CH, 32, TM, TN>(acc[0][0], &As[0][ty], &Bs[0][tx], clen);
      }
      for (int kb0 = kb_done; kb0 < clen; kb0 += kblock) {
        const int len = min(kblock, clen - kb0);

        double s[RM][RN], e[RM][RN];
#pragma unroll
        for (int i = 0; i < RM; i++)
#pragma unroll
            for (int j = 0; j < RN; j++) { s[i][j] = (double)acc[i][j]; e[i][j] = 0.0; }

        for (int kk = 0; kk < len; kk++) {
            double av[RM], bv[RN];
#pragma unroll
            for (int i = 0; i < RM; i++) av[i] = (double)As[kb0 + kk][ty + CY * i];
#pragma unroll
            for (int j = 0; j < RN; j++) bv[j] = (double)Bs[kb0 + kk][tx + CX * j];
#pragma unroll
            for (int i = 0; i < RM; i++)
#pragma unroll
                for (int j = 0; j < RN; j++) {
                    const double p = __dmul_rn(av[i], bv[j]);          // exact
                    const double t = __dadd_rn(s[i][j], p);
                    const double bp = __dsub_rn(t, s[i][j]);
                    const double err = __dadd_rn(__dsub_rn(s[i][j], __dsub_rn(t, bp)),
                                                 __dsub_rn(p, bp));
                    s[i][j] = t;
                    e[i][j] = __dadd_rn(e[i][j], fabs(err));
                }
        }
#pragma unroll
        for (int i = 0; i < RM; i++)
#pragma unroll
            for (int j = 0; j < RN; j++) {
                if (e[i][j] == 0.0 && isfinite(s[i][j])) {
                    acc[i][j] = (s[i][j] == 0.0) ? 0.0f : __double2float_rn(s[i][j]);
                } else {
                    acc[i][j] = exact_block(acc[i][j], &As[kb0][ty + CY * i],
                                            &Bs[kb0][tx + CX * j], TM, TN, len);
                }
            }
      }
        __syncthreads();
    }

#pragma unroll
    for (int i = 0; i < RM; i++) {
        const int m = m0 + ty + CY * i;
        if (m >= M) continue;
#pragma unroll
        for (int j = 0; j < RN; j++) {
            const int n = n0 + tx + CX * j;
            if (n < N) c[(size_t)m * ldc + n] = acc[i][j];
        }
    }
}

}  // namespace

int launch_gemm_exact(cudaStream_t st, const void *a, int a_type, int lda,
                      const uint16_t *b, int ldb, float *c, int ldc,
                      int M, int N, int K, int kblock) {
    if (M < 0 || N < 0 || K < 0) return N550_ERR_ARG;
    if (kblock != 16 && kblock != 32) return N550_ERR_ARG;
    if (M == 0 || N == 0) return N550_OK;
    if (lda < K || ldb < K || ldc < N) return N550_ERR_ARG;
    if (!c || (K && (!a || !b))) return N550_ERR_ARG;
    if (a_type != N550_F32 && a_type != N550_BF16) return N550_ERR_ARG;
    const bool few = M <= 16;
    const int tm = few ? 16 : 64, tn = few ? 16 : 64;
    const long long gy = (M + tm - 1) / tm, gx = (N + tn - 1) / tn;
    if (gy > 65535 || gx > 0x7FFFFFFF) return N550_ERR_UNSUPPORTED;
    dim3 grid((unsigned)gx, (unsigned)gy);
    const bool f32 = a_type == N550_F32;
    auto kern = few ? (f32 ? gemm_exact_kernel<true, 16, 16, 1, 1, 256, 4> : gemm_exact_kernel<false, 16, 16, 1, 1, 256, 4>)
                    : (f32 ? gemm_exact_kernel<true, 64, 64, 4, 4, MAXKB> : gemm_exact_kernel<false, 64, 64, 4, 4, MAXKB>);
    N550_CUDA_TRY(launch_k(kern, grid, THREADS, 0, st, a, lda, b, ldb, c, ldc, M, N, K, kblock));
    return N550_OK;
}

}  // namespace n550
