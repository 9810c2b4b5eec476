// The exported C ABI (include/n550_qwen3.h): the reference's operator plug
// points over host pointers, and the device-pointer stream-ordered API.
#include <mutex>
#include <string.h>

#include "attention.h"
#include "common.cuh"
#include "gemm_skinny.h"
#include "gemm_tc.h"
#include "launch.h"
#include "ops.h"
#include "synth.cuh"

namespace n550 {
namespace {

thread_local int t_status = N550_OK;
int g_mode = N550_MODE_EXACT;
int g_kblock = 16;
int g_b_tiled = 0;        // qwen3_set_weight_layout(TILE) accepted

// ---- host-shim device workspace: one growing buffer per slot and device ----
enum { WS_A = 0, WS_B, WS_C, WS_T, WS_SLOTS };
struct Ws { void *p = nullptr; size_t cap = 0; };
std::mutex g_ws_mu;
Ws g_ws[64][WS_SLOTS];

void *ws_get(int slot, size_t bytes) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    Ws &w = g_ws[dev][slot];
    if (bytes <= w.cap) return w.p;
    if (w.p) cudaFree(w.p);
    w.p = nullptr;
    w.cap = 0;
    size_t cap = bytes < 4096 ? 4096 : bytes + bytes / 4;
    if (cudaMalloc(&w.p, cap) != cudaSuccess) { (void)cudaGetLastError(); return nullptr; }
    w.cap = cap;
    return w.p;
}

// Tile-major weights (kernels_ame.c:212-215): 128x32 tiles, n-tile major,
// k-tile minor, each tile row-major with a 32-element row stride.
__global__ void untile_kernel(uint16_t *dst, const uint16_t *src, int N, int K) {
    const size_t total = (size_t)N * K;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
         i += (size_t)gridDim.x * blockDim.x) {
        const int n = (int)(i / K), k = (int)(i % K);
        const size_t tile = (size_t)(n / 128) * (K / 32) + (k / 32);
        dst[i] = src[tile * 4096 + (size_t)(n % 128) * 32 + (k % 32)];
    }
}

// C = A . B^T in FP32 through the skinny-token GEMM (M <= SK_MAX_T).
int skinny_f32(cudaStream_t st, const uint16_t *a, int lda, const uint16_t *b, int ldb, float *c,
               int ldc, int M, int N, int K) {
    SkEpilogue ep{};
    ep.out = c;
    ep.ldo = ldc;
    return launch_gemm_skinny(st, SK_EPI_F32, a, lda, b, nullptr, ldb, M, N, K, ep);
}

int device_gemm(cudaStream_t st, int mode, int kblock, const void *a, int a_type, int lda,
                const uint16_t *b, int ldb, void *c, int c_type, int ldc, int M, int N, int K) {
    if (M < 0 || N < 0 || K < 0) return N550_ERR_ARG;
    if (M == 0 || N == 0) return N550_OK;
    if (!c || (K && (!a || !b)) || lda < K || ldb < K || ldc < N) return N550_ERR_ARG;
    if (mode == N550_MODE_EXACT) {
        if (c_type != N550_F32) return N550_ERR_ARG;
        return launch_gemm_exact(st, a, a_type, lda, b, ldb, (float *)c, ldc, M, N, K, kblock);
    }
    if (mode != N550_MODE_FAST) return N550_ERR_ARG;
    if (c_type != N550_F32 && c_type != N550_BF16) return N550_ERR_ARG;
    const int esz = c_type == N550_F32 ? 4 : 2;
    if (K == 0) {
        N550_CUDA_TRY(cudaMemset2DAsync(c, (size_t)ldc * esz, 0, (size_t)N * esz, M, st));
        return N550_OK;
    }
    const uint16_t *abf = (const uint16_t *)a;
    uint16_t *staged = nullptr;
    int ldab = lda;
    if (a_type == N550_F32) {
        ldab = (K + 7) & ~7;
        N550_CUDA_TRY(cudaMallocAsync((void **)&staged, (size_t)M * ldab * 2, st));
        int rc = launch_f32_to_bf16(st, staged, ldab, (const float *)a, lda, M, K);
        if (rc) { cudaFreeAsync(staged, st); return rc; }
        abf = staged;
    } else if (a_type != N550_BF16) {
        return N550_ERR_ARG;
    }
    const int epi = c_type == N550_F32 ? TC_EPI_F32 : TC_EPI_BF16;
    int rc;
    int kt;
    if (M <= 8 && launch_gemv(st, epi, abf, ldab, b, ldb, c, ldc, M, N, K) == N550_OK) {
        rc = N550_OK;
    } else if (skinny_route_gemm(M) && epi == TC_EPI_F32 &&
               tc_shape_ok(abf, ldab, b, ldb, K) &&
               (rc = skinny_f32(st, abf, ldab, b, ldb, (float *)c, ldc, M, N, K)) != N550_ERR_UNSUPPORTED) {
        // weight-streaming GEMM (rc set)
    } else if (M < 1024 && tc_shape_ok(abf, ldab, b, ldb, K) &&
               tc_splitk_plan(M, N, K, epi, 64, &kt) > 1) {
        // skinny M: split the K loop, partials in a stream-ordered workspace
        const size_t ws_bytes = (size_t)8 * M * N * 4;
        float *ws = nullptr;
        if (cudaMallocAsync((void **)&ws, ws_bytes, st) != cudaSuccess) {
            (void)cudaGetLastError();
            if (staged) cudaFreeAsync(staged, st);
            return N550_ERR_OOM;
        }
        rc = launch_gemm_tc_splitk(st, epi, abf, ldab, b, ldb, nullptr, c, ldc, M, N, K, ws, ws_bytes);
        cudaFreeAsync(ws, st);
    } else if (tc_shape_ok(abf, ldab, b, ldb, K)) {
        rc = launch_gemm_tc(st, epi, n550_tile_bn(M, N), abf, ldab, b, ldb, nullptr, c, ldc, M, N, K, 0);
    } else {
        rc = launch_gemm_simt(st, epi, abf, ldab, b, ldb, c, ldc, M, N, K);
    }
    if (staged) cudaFreeAsync(staged, st);
    return rc;
}

// Host-pointer GEMM: copy in, compute on the current device, copy out.
int host_gemm(float *c, const float *a, const uint16_t *b, int M, int K, int N, int tiled) {
    if (M < 0 || K < 0 || N < 0 || (M && N && (!c || (K && (!a || !b))))) return N550_ERR_ARG;
    if (M == 0 || N == 0) return N550_OK;
    if (tiled && ((N % 128) || (K % 32))) return N550_ERR_UNSUPPORTED;
    std::lock_guard<std::mutex> lk(g_ws_mu);
    const size_t abytes = (size_t)M * K * 4, bbytes = (size_t)N * K * 2, cbytes = (size_t)M * N * 4;
    float *da = (float *)ws_get(WS_A, abytes + 16);
    uint16_t *db = (uint16_t *)ws_get(WS_B, bbytes + 16);
    float *dc = (float *)ws_get(WS_C, cbytes + 16);
    if (!da || !db || !dc) return N550_ERR_OOM;
    cudaStream_t st = 0;
    if (K) {
        N550_CUDA_TRY(cudaMemcpyAsync(da, a, abytes, cudaMemcpyHostToDevice, st));
        if (tiled) {
            uint16_t *dt = (uint16_t *)ws_get(WS_T, bbytes + 16);
            if (!dt) return N550_ERR_OOM;
            N550_CUDA_TRY(cudaMemcpyAsync(dt, b, bbytes, cudaMemcpyHostToDevice, st));
            untile_kernel<<<148 * 8, 256, 0, st>>>(db, dt, N, K);
            N550_LAUNCH_CHECK();
        } else {
            N550_CUDA_TRY(cudaMemcpyAsync(db, b, bbytes, cudaMemcpyHostToDevice, st));
        }
    }
    int rc = device_gemm(st, g_mode, g_kblock, da, N550_F32, K, db, K, dc, N550_F32, N, M, N, K);
    if (rc) return rc;
    N550_CUDA_TRY(cudaMemcpyAsync(c, dc, cbytes, cudaMemcpyDeviceToHost, st));
    N550_CUDA_TRY(cudaStreamSynchronize(st));
    return N550_OK;
}

// Run an in-place float op on host data: x[n] (+ optional second input).
template <class F>
int host_op(float *x_out, const float *x_in, size_t nx, const void *y, size_t ybytes, F launch) {
    std::lock_guard<std::mutex> lk(g_ws_mu);
    float *dx = (float *)ws_get(WS_A, nx * 4 + 16);
    void *dy = ybytes ? ws_get(WS_B, ybytes + 16) : nullptr;
    if (!dx || (ybytes && !dy)) return N550_ERR_OOM;
    cudaStream_t st = 0;
    if (nx) N550_CUDA_TRY(cudaMemcpyAsync(dx, x_in, nx * 4, cudaMemcpyHostToDevice, st));
    if (ybytes) N550_CUDA_TRY(cudaMemcpyAsync(dy, y, ybytes, cudaMemcpyHostToDevice, st));
    int rc = launch(st, dx, dy);
    if (rc) return rc;
    if (nx && x_out) N550_CUDA_TRY(cudaMemcpyAsync(x_out, dx, nx * 4, cudaMemcpyDeviceToHost, st));
    N550_CUDA_TRY(cudaStreamSynchronize(st));
    return N550_OK;
}

inline void set_status(int s) { t_status = s; }

// Tensor-core GEMM with epilogue `epi`; skinny M (< 1024) splits the K loop
// with its partials in a stream-ordered workspace.
int skinny_or_full(cudaStream_t st, int epi, const uint16_t *a, int lda, const uint16_t *b, int ldb,
                   const uint16_t *b2, void *c, int ldc, int M, int N, int K) {
    if (skinny_route(M) &&
        (epi == TC_EPI_F32 || epi == TC_EPI_RESID_F32 || epi == TC_EPI_SILU_BF16)) {
        // weight-streaming GEMM, K split over a cluster, reduced on chip
        SkEpilogue ep{};
        if (epi == TC_EPI_SILU_BF16) { ep.h = (uint16_t *)c; ep.ldh = ldc; }
        else { ep.out = (float *)c; ep.ldo = ldc; }
        const int sk = epi == TC_EPI_SILU_BF16 ? SK_EPI_SILU : (epi == TC_EPI_F32 ? SK_EPI_F32 : SK_EPI_RESID);
        const int rc = launch_gemm_skinny(st, sk, a, lda, b, b2, ldb, M, N, K, ep);
        if (rc != N550_ERR_UNSUPPORTED) return rc;
    }
    int kt;
    if (M < 1024 && tc_splitk_plan(M, N, K, epi, 64, &kt) > 1) {
        const size_t ws_bytes = (size_t)8 * M * N * (epi == TC_EPI_SILU_BF16 ? 2 : 1) * 4;
        float *ws = nullptr;
        if (cudaMallocAsync((void **)&ws, ws_bytes, st) != cudaSuccess) {
            (void)cudaGetLastError();
            return N550_ERR_OOM;
        }
        const int rc = launch_gemm_tc_splitk(st, epi, a, lda, b, ldb, b2, c, ldc, M, N, K, ws, ws_bytes);
        cudaFreeAsync(ws, st);
        return rc;
    }
    return launch_gemm_tc(st, epi, n550_tile_bn(M, epi == TC_EPI_SILU_BF16 ? 2 * N : N), a, lda, b, ldb,
                          b2, c, ldc, M, N, K, 0);
}

// ---- staging area of n550_gemm_f32a_noalloc ----
// 4 Mi BF16 elements (8 MiB) in every GPU that loads the library. Its host
// symbol is only a stand-in: kernels get the device address looked up below.
constexpr size_t kNoAllocStageElems = (size_t)4 << 20;
static __device__ __align__(256) uint16_t g_noalloc_stage[kNoAllocStageElems];
std::mutex g_noalloc_mu;
uint16_t *g_noalloc_ptr[64];

// Device address of the staging array on the current device (looked up once
// per device, with that device current); nullptr on failure.
uint16_t *noalloc_stage() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        void *p = nullptr;
        if (cudaGetSymbolAddress(&p, g_noalloc_stage) != cudaSuccess) {
            (void)cudaGetLastError();
            return nullptr;
        }
        g_noalloc_ptr[dev] = (uint16_t *)p;
    }
    return g_noalloc_ptr[dev];
}

// One warp waits on an mbarrier that nothing arrives on, for at most `cycles`,
// first polling (mbar_wait) and then with suspended tries (mbar_wait_sleep, the
// tensor-core GEMM's waits): the expiry path of every bounded wait in the
// library (status word set to N550_ERR_TIMEOUT, kernel returns).
__global__ void wait_expiry_kernel(long long cycles) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_mbar_init();
    }
    __syncwarp();
    mbar_wait(&bar, 0, cycles);
    mbar_wait_sleep(&bar, 0, cycles);
}

}  // namespace
}  // namespace n550

using namespace n550;

extern "C" {

// ---------------- reference plug points (host pointers) ----------------

void qwen3_gemm(float *c, const float *a, const uint16_t *b, int M, int K, int N) {
    set_status(host_gemm(c, a, b, M, K, N, g_b_tiled));
}

void qwen3_gemm_row(float *c, const float *a, const uint16_t *b, int M, int K, int N) {
    set_status(host_gemm(c, a, b, M, K, N, 0));
}

int qwen3_set_weight_layout(int layout, int tile_n, int tile_k) {
    if (layout == N550_LAYOUT_ROW) { g_b_tiled = 0; return 0; }
    if (layout != N550_LAYOUT_TILE) return -1;
    if (tile_n != 128 || tile_k != 32) return -1;
    g_b_tiled = 1;
    return 0;
}

const char *qwen3_kernel_name(void) {
    if (g_mode == N550_MODE_FAST) return "n550-b200 tcgen05 (fast)";
    return g_kblock == 32 ? "n550-b200 exact (AME K-block 32)" : "n550-b200 exact (AME K-block 16)";
}

int n550_set_gemm_mode(int mode, int kblock) {
    if (mode == N550_MODE_EXACT) {
        if (kblock != 16 && kblock != 32) return N550_ERR_ARG;
        g_mode = mode;
        g_kblock = kblock;
        return N550_OK;
    }
    if (mode == N550_MODE_FAST) { g_mode = mode; return N550_OK; }
    return N550_ERR_ARG;
}

void qwen3_op_rmsnorm(float *out, const float *x, const uint16_t *w, int n) {
    if (n <= 0 || !out || !x || !w) { set_status(n == 0 ? N550_OK : N550_ERR_ARG); return; }
    set_status(host_op(out, x, (size_t)n, w, (size_t)n * 2, [&](cudaStream_t st, float *dx, void *dw) {
        return launch_rmsnorm(st, dx, N550_F32, dx, (const uint16_t *)dw, 1, n, 1e-6f);
    }));
}

void qwen3_op_rope(float *v, int n_heads, int pos) {
    if (n_heads <= 0 || !v) { set_status(n_heads == 0 ? N550_OK : N550_ERR_ARG); return; }
    set_status(host_op(v, v, (size_t)n_heads * 128, nullptr, 0, [&](cudaStream_t st, float *dv, void *) {
        return launch_rope(st, dv, 1, n_heads, pos);
    }));
}

void qwen3_op_softmax(float *x, int n) {
    if (n <= 0 || !x) { set_status(n == 0 ? N550_OK : N550_ERR_ARG); return; }
    set_status(host_op(x, x, (size_t)n, nullptr, 0, [&](cudaStream_t st, float *dx, void *) {
        return launch_softmax(st, dx, 1, n);
    }));
}

void qwen3_op_silu_mul(float *gate, const float *up, int n) {
    if (n <= 0 || !gate || !up) { set_status(n == 0 ? N550_OK : N550_ERR_ARG); return; }
    set_status(host_op(gate, gate, (size_t)n, up, (size_t)n * 4, [&](cudaStream_t st, float *dg, void *du) {
        return launch_silu_mul(st, dg, (const float *)du, (size_t)n);
    }));
}

void qwen3_op_residual_add(float *x, const float *y, int n) {
    if (n <= 0 || !x || !y) { set_status(n == 0 ? N550_OK : N550_ERR_ARG); return; }
    set_status(host_op(x, x, (size_t)n, y, (size_t)n * 4, [&](cudaStream_t st, float *dx, void *dy) {
        return launch_residual_add(st, dx, (const float *)dy, (size_t)n);
    }));
}

int qwen3_op_argmax(const float *v, int n) {
    if (n <= 0 || !v) { set_status(N550_ERR_ARG); return 0; }
    int32_t best = 0;
    int rc = host_op(nullptr, v, (size_t)n, nullptr, 0, [&](cudaStream_t st, float *dv, void *) {
        int32_t *di = (int32_t *)ws_get(WS_C, 16);
        if (!di) return (int)N550_ERR_OOM;
        int r = launch_argmax(st, dv, 1, n, n, di);
        if (r) return r;
        N550_CUDA_TRY(cudaMemcpyAsync(&best, di, 4, cudaMemcpyDeviceToHost, st));
        return (int)N550_OK;
    });
    set_status(rc);
    return rc ? 0 : (int)best;
}

void qwen3_op_bf16_to_f32(float *out, const uint16_t *in, int n) {
    if (n <= 0 || !out || !in) { set_status(n == 0 ? N550_OK : N550_ERR_ARG); return; }
    set_status(host_op(out, out, 0, in, (size_t)n * 2, [&](cudaStream_t st, float *, void *din) {
        float *dout = (float *)ws_get(WS_C, (size_t)n * 4 + 16);
        if (!dout) return (int)N550_ERR_OOM;
        int r = launch_bf16_to_f32(st, dout, (const uint16_t *)din, (size_t)n);
        if (r) return r;
        N550_CUDA_TRY(cudaMemcpyAsync(out, dout, (size_t)n * 4, cudaMemcpyDeviceToHost, st));
        return (int)N550_OK;
    }));
}

float qwen3_op_dot(const float *a, const float *b, int n) {
    if (n <= 0 || !a || !b) { set_status(n == 0 ? N550_OK : N550_ERR_ARG); return 0.0f; }
    float r = 0.0f;
    int rc = host_op(nullptr, a, (size_t)n, b, (size_t)n * 4, [&](cudaStream_t st, float *da, void *db) {
        float *dr = (float *)ws_get(WS_C, 16);
        if (!dr) return (int)N550_ERR_OOM;
        int e = launch_dot(st, da, (const float *)db, n, dr);
        if (e) return e;
        N550_CUDA_TRY(cudaMemcpyAsync(&r, dr, 4, cudaMemcpyDeviceToHost, st));
        return (int)N550_OK;
    });
    set_status(rc);
    return rc ? 0.0f : r;
}

void qwen3_op_axpy(float *y, float a, const float *x, int n) {
    if (n <= 0 || !y || !x) { set_status(n == 0 ? N550_OK : N550_ERR_ARG); return; }
    set_status(host_op(y, y, (size_t)n, x, (size_t)n * 4, [&](cudaStream_t st, float *dy, void *dx) {
        return launch_axpy(st, dy, a, (const float *)dx, (size_t)n);
    }));
}

const char *qwen3_ops_name(void) { return "n550-b200 cuda"; }

int n550_last_status(void) { return t_status; }

const char *n550_strerror(int s) {
    switch (s) {
    case N550_OK: return "ok";
    case N550_ERR_MAGIC: return "bad magic (not a QW3M weight file)";
    case N550_ERR_VERSION: return "QW3M version mismatch";
    case N550_ERR_DTYPE: return "QW3M dtype is not BF16";
    case N550_ERR_SHAPE: return "QW3M shape/hyper-parameters do not match Qwen3-0.6B";
    case N550_ERR_SIZE: return "QW3M size mismatch";
    case N550_ERR_OOM: return "out of device memory";
    case N550_ERR_LAYOUT: return "weight layout not supported";
    case N550_ERR_ARG: return "invalid argument";
    case N550_ERR_CUDA: return "CUDA runtime error";
    case N550_ERR_UNSUPPORTED: return "unsupported shape or alignment";
    case N550_ERR_TIMEOUT: return "bounded device wait expired";
    default: return "unknown";
    }
}

// ---------------- device-pointer API ----------------

int n550_gemm(void *stream, int mode, int kblock, const void *a, int a_type, int lda,
              const uint16_t *b, int ldb, void *c, int c_type, int ldc, int M, int N, int K) {
    return device_gemm((cudaStream_t)stream, mode, kblock, a, a_type, lda, b, ldb, c, c_type,
                       ldc, M, N, K);
}

int n550_gemm_tile_config(int bn) {
    if (bn != 0 && bn != 128 && bn != 256 && bn != 512) return N550_ERR_ARG;
    g_tile_bn = bn;
    return N550_OK;
}

int n550_gemm_skinny_config(int cs) {
    if (cs < -1 || cs > 16) return N550_ERR_ARG;
    g_skinny_cs = cs;
    return N550_OK;
}

int n550_gemm_skinny_rows(int m) {
    if (m < 0 || m > SK_MAX_T) return N550_ERR_ARG;
    g_skinny_rows = m;
    g_skinny_rows_gemm = m;
    return N550_OK;
}

int n550_set_pdl(int on) {
    g_pdl = on != 0;
    return N550_OK;
}

int n550_gemm_residual(void *stream, const uint16_t *a, int lda, const uint16_t *b, int ldb,
                       float *x, int ldx, int M, int N, int K) {
    cudaStream_t st = (cudaStream_t)stream;
    if (M < 0 || N < 0 || K < 0 || (M && N && (!x || (K && (!a || !b)))) || lda < K || ldb < K ||
        ldx < N)
        return N550_ERR_ARG;
    if (M == 0 || N == 0 || K == 0) return N550_OK;
    if (M <= 8 && launch_gemv(st, TC_EPI_RESID_F32, a, lda, b, ldb, x, ldx, M, N, K) == N550_OK)
        return N550_OK;
    if (tc_shape_ok(a, lda, b, ldb, K))
        return skinny_or_full(st, TC_EPI_RESID_F32, a, lda, b, ldb, nullptr, x, ldx, M, N, K);
    return launch_gemm_simt(st, TC_EPI_RESID_F32, a, lda, b, ldb, x, ldx, M, N, K);
}

int n550_gemm_swiglu(void *stream, const uint16_t *a, int lda, const uint16_t *wg,
                     const uint16_t *wu, int ldw, uint16_t *h, int ldh, int M, int N, int K) {
    cudaStream_t st = (cudaStream_t)stream;
    if (M < 0 || N < 0 || K <= 0 || (M && N && (!h || !a || !wg || !wu)) || lda < K || ldw < K ||
        ldh < N)
        return N550_ERR_ARG;
    if (M == 0 || N == 0) return N550_OK;
    // up to 8 rows: gate, up and SiLU . mul in one GEMV launch (as the other
    // few-row GEMMs of this interface)
    if (M <= 8 && launch_gemv_swiglu(st, a, lda, wg, wu, ldw, h, ldh, M, N, K) == N550_OK)
        return N550_OK;
    if (!tc_shape_ok(a, lda, wg, ldw, K) || !tc_shape_ok(a, lda, wu, ldw, K))
        return N550_ERR_UNSUPPORTED;
    return skinny_or_full(st, TC_EPI_SILU_BF16, a, lda, wg, ldw, wu, h, ldh, M, N, K);
}

int n550_rmsnorm(void *stream, void *out, int out_type, const float *x, const uint16_t *w,
                 int rows, int n, float eps) {
    return launch_rmsnorm((cudaStream_t)stream, out, out_type, x, w, rows, n, eps);
}

int n550_rope(void *stream, float *v, int rows, int n_heads, int pos0) {
    return launch_rope((cudaStream_t)stream, v, rows, n_heads, pos0);
}

int n550_silu_mul(void *stream, float *gate, const float *up, size_t n) {
    return launch_silu_mul((cudaStream_t)stream, gate, up, n);
}

int n550_softmax(void *stream, float *x, int rows, int n) {
    return launch_softmax((cudaStream_t)stream, x, rows, n);
}

int n550_argmax(void *stream, const float *v, int rows, int n, int ld, int32_t *idx) {
    return launch_argmax((cudaStream_t)stream, v, rows, n, ld, idx);
}

int n550_residual_add(void *stream, float *x, const float *y, size_t n) {
    return launch_residual_add((cudaStream_t)stream, x, y, n);
}

int n550_bf16_to_f32(void *stream, float *out, const uint16_t *in, size_t n) {
    return launch_bf16_to_f32((cudaStream_t)stream, out, in, n);
}

int n550_gemm_f32a_noalloc(void *stream, const float *a, int lda, const uint16_t *b, int ldb,
                           void *c, int c_type, int ldc, int M, int N, int K) {
    cudaStream_t st = (cudaStream_t)stream;
    if (M < 0 || N < 0 || K < 0) return N550_ERR_ARG;
    if (M == 0 || N == 0) return N550_OK;
    if (!c || (K && (!a || !b)) || lda < K || ldb < K || ldc < N) return N550_ERR_ARG;
    if (c_type != N550_F32 && c_type != N550_BF16) return N550_ERR_ARG;
    const int ldab = (K + 7) & ~7;
    if ((size_t)M * (size_t)ldab > kNoAllocStageElems) return N550_ERR_ARG;
    const int esz = c_type == N550_F32 ? 4 : 2;
    if (K == 0) {
        N550_CUDA_TRY(cudaMemset2DAsync(c, (size_t)ldc * esz, 0, (size_t)N * esz, M, st));
        return N550_OK;
    }
    uint16_t *stage = noalloc_stage();
    if (!stage) return N550_ERR_CUDA;
    // Every element the GEMM reads ([0, M) x [0, K)) is rewritten here; the
    // padding columns [K, ldab) are never read (the TMA box and the CUDA-core
    // paths stop at K), so the array needs no clearing between calls.
    int rc = launch_f32_to_bf16(st, stage, ldab, a, lda, M, K);
    if (rc) return rc;
    const int epi = c_type == N550_F32 ? TC_EPI_F32 : TC_EPI_BF16;
    if (M <= 8 && launch_gemv(st, epi, stage, ldab, b, ldb, c, ldc, M, N, K) == N550_OK) return N550_OK;
    if (!tc_shape_ok(stage, ldab, b, ldb, K))
        return launch_gemm_simt(st, epi, stage, ldab, b, ldb, c, ldc, M, N, K);
    // the weight-streaming GEMM keeps its partial tiles on chip, as in n550_gemm
    if (skinny_route_gemm(M) && epi == TC_EPI_F32) {
        rc = skinny_f32(st, stage, ldab, b, ldb, (float *)c, ldc, M, N, K);
        if (rc != N550_ERR_UNSUPPORTED) return rc;
    }
    // no split-K here: its FP32 partials would need a second, larger array
    return launch_gemm_tc(st, epi, n550_tile_bn(M, N), stage, ldab, b, ldb, nullptr, c, ldc, M, N, K, 0);
}

int n550_synth_tokens(int32_t *out, size_t n, uint64_t seed, uint64_t stream, int vocab) {
    if ((n && !out) || vocab <= 0) return N550_ERR_ARG;
    const uint64_t key = synth_key(seed, stream);
    for (size_t i = 0; i < n; i++) out[i] = (int32_t)(synth_u64(key, i) % (uint64_t)vocab);
    return N550_OK;
}

int n550_synth_normal_bf16(uint16_t *out, size_t n, uint64_t seed, uint64_t stream, double sigma) {
    if (n && !out) return N550_ERR_ARG;
    const uint64_t key = synth_key(seed, stream);
    const float scale = synth_normal_scale(sigma);
    for (size_t i = 0; i < n; i++) out[i] = f32_to_bf16_rne(synth_normal(synth_u64(key, i), scale));
    return N550_OK;
}

int n550_attention_prefill(void *stream, const uint16_t *q, int ldq, const uint16_t *k_cache,
                           const uint16_t *v_cache, int n_slots, int max_len, int layer,
                           const int32_t *seq_ids, int n_seqs, int L, int pos0, uint16_t *out,
                           int ldo) {
    if (n_seqs < 0 || L < 0 || n_slots <= 0 || max_len <= 0) return N550_ERR_ARG;
    AttnPrefillArgs a{};
    a.q = q; a.kc = k_cache; a.vc = v_cache; a.out = out; a.seq_ids = seq_ids;
    a.ldq = ldq; a.ldo = ldo; a.L = L; a.pos0 = pos0; a.layer = layer; a.max_len = max_len;
    a.kv_planes = n_slots * 28 * 8;
    return launch_attn_prefill((cudaStream_t)stream, a, n_seqs);
}

static const int kDecodeMaxSplits = 32;

size_t n550_attention_decode_workspace(int n_seqs, int max_len) {
    if (n_seqs <= 0 || max_len <= 0) return 0;
    const int splits = attn_decode_splits(n_seqs, max_len, kDecodeMaxSplits);
    return (size_t)n_seqs * 16 * splits * (2 + 128) * sizeof(float);
}

int n550_attention_decode(void *stream, const uint16_t *q, int ldq, const uint16_t *k_cache,
                          const uint16_t *v_cache, int n_slots, int max_len, int layer,
                          const int32_t *seq_ids, const int32_t *pos, int n_seqs, uint16_t *out,
                          int ldo, void *workspace, size_t workspace_bytes) {
    if (n_seqs == 0) return N550_OK;
    if (n_seqs < 0 || n_slots <= 0 || max_len <= 0 || layer < 0 || layer >= 28 || !q || !k_cache ||
        !v_cache || !seq_ids || !pos || !out || ldq < 16 * 128 || ldo < 16 * 128)
        return N550_ERR_ARG;
    AttnDecodeArgs a{};
    a.q_bf16 = q; a.kc = k_cache; a.vc = v_cache; a.out = out; a.seq_ids = seq_ids; a.pos = pos;
    a.ldq = ldq; a.ldo = ldo; a.layer = layer; a.max_len = max_len;
    a.kv_planes = n_slots * 28 * 8;
    a.splits = 1;
    const size_t need = n550_attention_decode_workspace(n_seqs, max_len);
    if (workspace && workspace_bytes >= need && ((uintptr_t)workspace & 15) == 0) {
        a.splits = attn_decode_splits(n_seqs, max_len, kDecodeMaxSplits);
        const size_t slots = (size_t)n_seqs * 16 * a.splits;
        a.part_o = (float *)workspace;
        a.part_m = a.part_o + slots * 128;
        a.part_l = a.part_m + slots;
    }
    return launch_attn_decode((cudaStream_t)stream, a, n_seqs);
}

int n550_check_wait_expiry(void *stream, long long cycles) {
    if (cycles < 1 || cycles > kWaitCycles) return N550_ERR_ARG;
    wait_expiry_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(cycles);
    N550_CUDA_TRY(cudaGetLastError());
    return N550_OK;
}

int n550_device_status(void) {
    if (cudaDeviceSynchronize() != cudaSuccess) return N550_ERR_CUDA;
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_device_status, sizeof v) != cudaSuccess) return N550_ERR_CUDA;
    const int zero = 0;
    if (cudaMemcpyToSymbol(g_device_status, &zero, sizeof zero) != cudaSuccess) return N550_ERR_CUDA;
    return v;
}

}  // extern "C"
