// Shared device/host helpers for the n550 B200 kernels (sm_100a only).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "../../include/n550_qwen3.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "n550 kernels are written for sm_100a (B200) only"
#endif

namespace n550 {

// ---------------------------------------------------------------------------
// Status plumbing
// ---------------------------------------------------------------------------
#define N550_CUDA_TRY(expr)                                                   \
    do {                                                                      \
        cudaError_t _e = (expr);                                              \
        if (_e != cudaSuccess) return (int)N550_ERR_CUDA;                     \
    } while (0)

#define N550_LAUNCH_CHECK()                                                   \
    do {                                                                      \
        if (cudaPeekAtLastError() != cudaSuccess) {                           \
            (void)cudaGetLastError();                                         \
            return (int)N550_ERR_CUDA;                                        \
        }                                                                     \
    } while (0)

// Device-side error word: bounded waits that expire record N550_ERR_TIMEOUT
// here and return instead of hanging. Read (and cleared) by
// n550_device_status().
extern __device__ int g_device_status;

__device__ __forceinline__ void report_timeout() {
    atomicExch(&g_device_status, N550_ERR_TIMEOUT);
}

// Upper bound of any spin-wait, in SM clock cycles (~1 s at 2 GHz).
constexpr long long kWaitCycles = 2000000000ll;

// ---------------------------------------------------------------------------
// Programmatic dependent launch. Kernels launched by launch_k() (launch.h)
// may start while the previous kernel of the stream is still running:
// dep_wait() blocks until every earlier grid has completed and its memory is
// visible, so it must precede the first access to any buffer another kernel
// writes or reads (only weights, tensor maps and constant tables may be read
// before it). dep_launch() lets the next kernel start its own prologue; in
// kernels that allocate TMEM it comes after the allocation (a dependent CTA
// on the same SM must not take the columns this CTA still waits for).
// Both are no-ops for a kernel launched without the attribute.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------------------
// BF16 bit helpers (no dependency on cuda_bf16 operator overloads)
// ---------------------------------------------------------------------------
__host__ __device__ __forceinline__ float bf16_bits_to_f32(uint16_t b) {
#ifdef __CUDA_ARCH__
    return __uint_as_float(((uint32_t)b) << 16);
#else
    uint32_t u = ((uint32_t)b) << 16;
    float f;
    __builtin_memcpy(&f, &u, 4);
    return f;
#endif
}

// FP32 -> BF16 round-half-even; Inf/NaN truncated (kernels_hwsim.c:45-51).
__host__ __device__ __forceinline__ uint16_t f32_to_bf16_rne(float f) {
#ifdef __CUDA_ARCH__
    uint32_t u = __float_as_uint(f);
#else
    uint32_t u;
    __builtin_memcpy(&u, &f, 4);
#endif
    if ((u & 0x7F800000u) == 0x7F800000u) return (uint16_t)(u >> 16);
    u += 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

// sin and cos of a RoPE angle x = pos * inv_freq (ops_scalar.c:21-35; x >= 0): Cody-Waite
// reduction x = k * pi/2 + r with pi/2 split into P1 (13 significant bits, so
// k * P1 is exact for k < 2^11) and P2 = fl32(pi/2 - P1), then the hardware
// sine/cosine approximations on |r| <= pi/4 (absolute error ~2^-21) and the
// quadrant k mod 4. Reduction error <= 3e-8 for x <= 3200 (checked against
// binary64 over every position < 3200 and all 64 frequencies); beyond that
// sincosf. About 10 instructions instead of sincosf's ~40: the fused q/k/v
// GEMM evaluates 32 of these per thread and tile, and every instruction its
// epilogue saves is power the power-capped tensor cores get back (measured on
// B200: 32.21 -> 31.89 ms per 64 x 512-token prefill step).
__device__ __forceinline__ void rope_sincos(float x, float *s, float *c) {
    if (!(fabsf(x) <= 3200.0f)) {
        sincosf(x, s, c);
        return;
    }
    const float k = rintf(x * 0.636619772367581343f);          // 2 / pi
    float r = fmaf(-k, 1.57080078125f, x);                     // P1 = 0x1.922p+0
    r = fmaf(-k, -4.454454938240815e-06f, r);                  // P2 = -0x1.2aeef4p-18
    const float sr = __sinf(r), cr = __cosf(r);
    const int q = (int)k & 3;
    const float sv = (q & 1) ? cr : sr, cv = (q & 1) ? sr : cr;
    *s = (q & 2) ? -sv : sv;
    *c = ((q + 1) & 2) ? -cv : cv;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    return (uint32_t)f32_to_bf16_rne(lo) | ((uint32_t)f32_to_bf16_rne(hi) << 16);
}

// ---------------------------------------------------------------------------
// Shared-memory address / mbarrier / TMA / tcgen05 wrappers (inline PTX)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
                 ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
    return ok != 0;
}

// try_wait with a suspend-time hint of 1 ms: the waiting thread sleeps until
// the phase completes (or the hint expires) instead of returning after the
// hardware's short default and polling again.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity), "r"(1000000u) : "memory");
    return ok != 0;
}

// Bounded wait: true when the phase completed, false (and the device status
// set to N550_ERR_TIMEOUT) after `limit` cycles (kWaitCycles unless a health
// check asks for less).
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, long long limit = kWaitCycles) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (clock64() - t0 > limit) { report_timeout(); return false; }
    }
    return true;
}

// mbar_wait whose polls sleep (mbar_try_wait_sleep). For the tensor-core GEMM,
// which runs at the board's power cap in a prefill: waiting warps that poll
// spend issue slots and power the MMAs could use (measured on B200, 64 x 512
// prefill step: 32.50 -> 31.84 ms median); latency-critical waits keep
// mbar_wait.
__device__ __forceinline__ bool mbar_wait_sleep(uint64_t *bar, uint32_t parity, long long limit = kWaitCycles) {
    if (mbar_try_wait_sleep(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait_sleep(bar, parity)) {
        if (clock64() - t0 > limit) { report_timeout(); return false; }
    }
    return true;
}

// 2-D tiled TMA load global -> shared, completion on an mbarrier.
// c0 is the innermost (contiguous) coordinate in elements; callers keep
// c0 * sizeof(elem) a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_2d(void *dst, const void *tmap, uint64_t *bar,
                                            int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];"
        ::"r"(smem_u32(dst)), "l"(tmap), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
        : "memory");
}

// 3-D tiled TMA load (c0 innermost, same alignment rule as tma_load_2d).
__device__ __forceinline__ void tma_load_3d(void *dst, const void *tmap, uint64_t *bar,
                                            int c0, int c1, int c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5}], [%2];"
        ::"r"(smem_u32(dst)), "l"(tmap), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
}

// L2 prefetch of one 3-D tensor-map box (no shared-memory destination).
__device__ __forceinline__ void tma_prefetch_3d(const void *tmap, int c0, int c1, int c2) {
    asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];"
                 ::"l"(tmap), "r"(c0), "r"(c1), "r"(c2) : "memory");
}

// Non-tensor bulk copy global -> shared (16-byte aligned addresses, size a
// multiple of 16), completion counted on an mbarrier.
__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}

// 2-D tiled TMA reduce-add shared -> global (element type from the tensor
// map; out-of-range rows/columns of the box are skipped), tracked by the
// issuing thread's bulk async-groups.
__device__ __forceinline__ void tma_reduce_add_2d(const void *tmap, const void *src, int c0, int c1) {
    asm volatile(
        "cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3}], [%1];"
        ::"l"(tmap), "r"(smem_u32(src)), "r"(c0), "r"(c1) : "memory");
}
__device__ __forceinline__ void bulk_commit_group() {
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Wait until at most N bulk async-groups of this thread still read shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_group_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// Wait until at most N bulk async-groups of this thread are incomplete.
template <int N>
__device__ __forceinline__ void bulk_wait_group() {
    asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}
// Make this thread's generic-proxy shared-memory writes visible to the async
// proxy (TMA) before a bulk copy reads them.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Named barrier `id` (1-15; 0 is __syncthreads) over `n` threads (multiple of 32).
__device__ __forceinline__ void named_bar_sync(int id, int n) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

__device__ __forceinline__ void tma_prefetch_desc(const void *tmap) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

// --- tcgen05 (5th-generation tensor core, accumulators in TMEM) ---
__device__ __forceinline__ void tmem_alloc(uint32_t *dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 ::"r"(smem_u32(dst_smem)), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;"
                 ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] . B[smem]^T ; M=128, N from idesc, K=16 (bf16).
__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// D[tmem] (+)= A[tmem] . B[smem]^T ; the A operand (M=128 rows = TMEM lanes,
// K=16 BF16 packed two per 32-bit column, 8 columns) is read from TMEM.
__device__ __forceinline__ void umma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                             uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
        ::"r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive on an mbarrier once all previously issued tcgen05.mma of this thread
// have completed.
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
        ::"r"(smem_u32(bar)) : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread t of the warp receives
// row (lane base + t), columns col..col+31.
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
          "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]),
          "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]),
          "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
          "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}
// 32 lanes x 16 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
          "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]),
          "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Store counterpart of tmem_ld_32x32b_x32: thread t writes row (lane base + t).
__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
        ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]),
          "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]),
          "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]),
          "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]),
          "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}
__device__ __forceinline__ void tmem_st_32x32b_x16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
        ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]),
          "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]),
          "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}
__device__ __forceinline__ void tmem_st_wait() {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// UMMA shared-memory descriptor, K-major operand in the 128-byte swizzle
// canonical layout: rows of 128 B, 8-row groups 1024 B apart (SBO = 1024),
// descriptor version 1 (sm_100), layout type 2 = SWIZZLE_128B.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t smem_addr) {
    uint64_t d = 0;
    d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);          // start address
    d |= (uint64_t)1 << 16;                                // LBO (unused for SW128 K-major)
    d |= (uint64_t)(1024 >> 4) << 32;                      // SBO
    d |= (uint64_t)1 << 46;                                // version
    d |= (uint64_t)2 << 61;                                // SWIZZLE_128B
    return d;
}

// UMMA shared-memory descriptor, MN-major operand in the 128-byte swizzle
// canonical layout: 64-element (128-byte) MN runs, 8 K rows 128 B apart form a
// 1024-byte atom; atoms along K are 1024 B apart (SBO), atoms along MN are
// `lbo` bytes apart (LBO).
__device__ __forceinline__ uint64_t umma_desc_sw128_mn(uint32_t smem_addr, uint32_t lbo) {
    uint64_t d = 0;
    d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);
    d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)(1024 >> 4) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)2 << 61;
    return d;
}

// Instruction descriptor, kind::f16: D FP32, A/B BF16, both K-major
// (bit 16 set = B MN-major).
__host__ __device__ constexpr uint32_t umma_idesc_bf16(int M, int N) {
    return (1u << 4)                       // D format F32
         | (1u << 7)                       // A format BF16
         | (1u << 10)                      // B format BF16
         | ((uint32_t)(N >> 3) << 17)      // N / 8
         | ((uint32_t)(M >> 4) << 24);     // M / 16
}

__device__ __forceinline__ int elect_one_lane() { return (threadIdx.x & 31) == 0; }

// One lane of the converged warp (elect.sync): the warp runs an MMA issue loop
// together -- its descriptors and addresses stay warp-uniform -- and only the
// elected lane executes each single-thread tcgen05 instruction.
__device__ __forceinline__ bool elect_one_sync() {
    uint32_t pred = 0;
    asm volatile(
        "{\n\t.reg .pred P;\n\t"
        "elect.sync _|P, 0xFFFFFFFF;\n\t"
        "selp.b32 %0, 1, 0, P;\n\t}"
        : "=r"(pred));
    return pred != 0;
}

// ---------------------------------------------------------------------------
// CTA pairs (2-CTA clusters, tcgen05 cta_group::2)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cluster_nctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
    return r;
}
// 32-bit store into the shared memory of a CTA of the cluster (address from
// mapa_shared); visible to that CTA after the next cluster_sync.
__device__ __forceinline__ void st_cluster_f32(uint32_t cluster_addr, float v) {
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(cluster_addr), "f"(v) : "memory");
}
// Split cluster barrier: every thread of every CTA arrives (release), and
// later waits (acquire) for the phase; work in between overlaps it.
__device__ __forceinline__ void cluster_arrive() {
    asm volatile("barrier.cluster.arrive.release;" ::: "memory");
}
// Arrival without memory ordering (for a barrier that only keeps CTAs alive).
__device__ __forceinline__ void cluster_arrive_relaxed() {
    asm volatile("barrier.cluster.arrive.relaxed;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
    asm volatile("barrier.cluster.wait.acquire;" ::: "memory");
}
// Bulk copy of `bytes` (multiple of 16, 16-byte aligned) from this CTA's shared
// memory into the shared memory of a CTA of the cluster (dst and its mbarrier
// given as shared::cluster addresses); completion counted on that mbarrier.
__device__ __forceinline__ void bulk_copy_to_cluster(uint32_t dst_cluster, const void *src, uint32_t bytes,
                                                     uint32_t bar_cluster) {
    asm volatile(
        "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(dst_cluster), "r"(smem_u32(src)), "r"(bytes), "r"(bar_cluster) : "memory");
}
// All threads of all CTAs of the cluster.
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;"
                 ::: "memory");
}
// Shared::cluster address of the variable at local shared address `addr` in
// CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}
// Arrive on an mbarrier given by a shared::cluster address (possibly in the
// peer CTA), releasing this thread's prior writes at cluster scope.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];"
                 ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
    return ok != 0;
}
// Bounded wait with cluster-scope acquire (arrivals from the peer CTA).
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t *bar, uint32_t parity) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait_cluster(bar, parity)) {
        if (clock64() - t0 > kWaitCycles) { report_timeout(); return false; }
    }
    return true;
}
// 2-D TMA load into this CTA's shared memory whose completion is counted on
// an mbarrier of either CTA of the pair (cluster address). No multicast.
__device__ __forceinline__ void tma_load_2d_pair(void *dst, const void *tmap, uint32_t bar_cluster,
                                                 int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];"
        ::"r"(smem_u32(dst)), "l"(tmap), "r"(bar_cluster), "r"(c0), "r"(c1)
        : "memory");
}
// TMEM allocation shared by the CTA pair (one warp of each CTA executes it).
__device__ __forceinline__ void tmem_alloc_pair(uint32_t *dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;"
                 ::"r"(smem_u32(dst_smem)), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;"
                 ::"r"(taddr), "r"(ncols) : "memory");
}
// D (+)= A . B^T over the CTA pair: M = 256 (rows 0..127 from this CTA's A
// tile into its TMEM, 128..255 from the peer's), B split across the two CTAs'
// shared memory at the same offset. Issued by the pair's leader only.
__device__ __forceinline__ void umma_bf16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                               uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrive on the mbarrier at this shared offset in every CTA of `mask` once the
// pair's previously issued MMAs have completed.
__device__ __forceinline__ void umma_commit_pair_mc(uint64_t *bar, uint16_t mask) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
        " [%0], %1;" ::"r"(smem_u32(bar)), "h"(mask) : "memory");
}

}  // namespace n550
