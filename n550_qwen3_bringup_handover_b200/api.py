"""Python bindings of the C ABI: reference-named host functions (numpy in,
numpy out, like the reference's ops over host buffers) and device functions
over torch CUDA tensors (torch is only the allocator and stream holder)."""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import BF16, F32, MODE_EXACT, MODE_FAST, check, lib

__all__ = [
    "qwen3_gemm", "qwen3_gemm_row", "qwen3_set_weight_layout", "qwen3_op_rmsnorm",
    "qwen3_op_rope", "qwen3_op_softmax", "qwen3_op_silu_mul", "qwen3_op_residual_add",
    "qwen3_op_argmax", "qwen3_op_bf16_to_f32", "qwen3_op_dot", "qwen3_op_axpy",
    "last_status", "gemm", "rmsnorm", "rope", "silu_mul", "softmax", "argmax",
    "residual_add", "bf16_to_f32", "device_status", "stream_ptr", "gemm_residual", "gemm_swiglu",
    "attention_prefill", "attention_decode",
]


def _np(a):
    return a.ctypes.data_as(C.c_void_p)


def last_status() -> int:
    return lib().n550_last_status()


# ---------------- reference plug points over host buffers ----------------

def qwen3_gemm(a: np.ndarray, b: np.ndarray, row: bool = False) -> np.ndarray:
    """C[M,N] = A[M,K] . B[N,K]^T with A FP32, B BF16 bits (uint16)."""
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.uint16)
    M, K = a.shape
    N = b.shape[0]
    c = np.zeros((M, N), np.float32)
    fn = lib().qwen3_gemm_row if row else lib().qwen3_gemm
    fn(_np(c), _np(a), _np(b), M, K, N)
    check(last_status(), "qwen3_gemm")
    return c


def qwen3_gemm_row(a, b):
    return qwen3_gemm(a, b, row=True)


def qwen3_set_weight_layout(layout: int, tile_n: int, tile_k: int) -> int:
    return lib().qwen3_set_weight_layout(layout, tile_n, tile_k)


def qwen3_op_rmsnorm(x, w):
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty_like(x)
    lib().qwen3_op_rmsnorm(_np(out), _np(x), _np(np.ascontiguousarray(w, np.uint16)), x.size)
    check(last_status(), "qwen3_op_rmsnorm")
    return out


def qwen3_op_rope(v, n_heads, pos):
    v = np.array(v, np.float32, copy=True)
    lib().qwen3_op_rope(_np(v), n_heads, pos)
    check(last_status(), "qwen3_op_rope")
    return v


def qwen3_op_softmax(x):
    x = np.array(x, np.float32, copy=True)
    lib().qwen3_op_softmax(_np(x), x.size)
    check(last_status(), "qwen3_op_softmax")
    return x


def qwen3_op_silu_mul(g, u):
    g = np.array(g, np.float32, copy=True)
    lib().qwen3_op_silu_mul(_np(g), _np(np.ascontiguousarray(u, np.float32)), g.size)
    check(last_status(), "qwen3_op_silu_mul")
    return g


def qwen3_op_residual_add(x, y):
    x = np.array(x, np.float32, copy=True)
    lib().qwen3_op_residual_add(_np(x), _np(np.ascontiguousarray(y, np.float32)), x.size)
    check(last_status(), "qwen3_op_residual_add")
    return x


def qwen3_op_argmax(v) -> int:
    v = np.ascontiguousarray(v, np.float32)
    r = lib().qwen3_op_argmax(_np(v), v.size)
    check(last_status(), "qwen3_op_argmax")
    return int(r)


def qwen3_op_bf16_to_f32(b):
    b = np.ascontiguousarray(b, np.uint16)
    out = np.empty(b.shape, np.float32)
    lib().qwen3_op_bf16_to_f32(_np(out), _np(b), b.size)
    check(last_status(), "qwen3_op_bf16_to_f32")
    return out


def qwen3_op_dot(a, b) -> float:
    a = np.ascontiguousarray(a, np.float32)
    r = lib().qwen3_op_dot(_np(a), _np(np.ascontiguousarray(b, np.float32)), a.size)
    check(last_status(), "qwen3_op_dot")
    return float(r)


def qwen3_op_axpy(y, a, x):
    y = np.array(y, np.float32, copy=True)
    lib().qwen3_op_axpy(_np(y), float(a), _np(np.ascontiguousarray(x, np.float32)), y.size)
    check(last_status(), "qwen3_op_axpy")
    return y


# ---------------- device API over torch tensors ----------------

def stream_ptr(stream=None):
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return C.c_void_p(s.cuda_stream)


def _dp(t):
    return C.c_void_p(t.data_ptr())


def _dtype_code(t):
    import torch
    if t.dtype == torch.float32:
        return F32
    if t.dtype in (torch.bfloat16, torch.int16, torch.uint16):
        return BF16
    raise TypeError(f"unsupported dtype {t.dtype}")


def gemm(a, b, mode=MODE_FAST, kblock=16, out=None, out_dtype=None, M=None, N=None, K=None):
    """C = A . B^T on the current device; A [M,K] (f32 or bf16), B [N,K] bf16."""
    import torch
    M = a.shape[0] if M is None else M
    N = b.shape[0] if N is None else N
    K = a.shape[1] if K is None else K
    if out is None:
        dt = out_dtype or torch.float32
        out = torch.empty((M, N), dtype=dt, device=a.device)
    check(lib().n550_gemm(stream_ptr(), mode, kblock, _dp(a), _dtype_code(a), a.stride(0),
                          _dp(b), b.stride(0), _dp(out), _dtype_code(out), out.stride(0),
                          M, N, K), "n550_gemm")
    return out


def gemm_residual(a, b, x):
    """x += A . B^T (FP32 x, BF16 A and B) with the fused residual epilogue."""
    M, K = a.shape
    N = b.shape[0]
    check(lib().n550_gemm_residual(stream_ptr(), _dp(a), a.stride(0), _dp(b), b.stride(0), _dp(x),
                                   x.stride(0), M, N, K), "n550_gemm_residual")
    return x


def gemm_swiglu(a, wg, wu, out=None):
    """h = silu(A . Wg^T) * (A . Wu^T) in BF16 with the fused SwiGLU epilogue."""
    import torch
    M, K = a.shape
    N = wg.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=a.device)
    check(lib().n550_gemm_swiglu(stream_ptr(), _dp(a), a.stride(0), _dp(wg), _dp(wu), wg.stride(0),
                                 _dp(out), out.stride(0), M, N, K), "n550_gemm_swiglu")
    return out


def rmsnorm(x, w, eps=1e-6, out_dtype=None):
    import torch
    out = torch.empty(x.shape, dtype=out_dtype or torch.float32, device=x.device)
    n = x.shape[-1]
    check(lib().n550_rmsnorm(stream_ptr(), _dp(out), _dtype_code(out), _dp(x), _dp(w),
                             x.numel() // n, n, eps), "n550_rmsnorm")
    return out


def rope(v, n_heads, pos0):
    rows = v.numel() // (n_heads * 128)
    check(lib().n550_rope(stream_ptr(), _dp(v), rows, n_heads, pos0), "n550_rope")
    return v


def silu_mul(g, u):
    check(lib().n550_silu_mul(stream_ptr(), _dp(g), _dp(u), g.numel()), "n550_silu_mul")
    return g


def softmax(x):
    n = x.shape[-1]
    check(lib().n550_softmax(stream_ptr(), _dp(x), x.numel() // n, n), "n550_softmax")
    return x


def argmax(v):
    import torch
    v2 = v.reshape(-1, v.shape[-1])
    idx = torch.empty(v2.shape[0], dtype=torch.int32, device=v.device)
    check(lib().n550_argmax(stream_ptr(), _dp(v2), v2.shape[0], v2.shape[1], v2.stride(0),
                            _dp(idx)), "n550_argmax")
    return idx


def residual_add(x, y):
    check(lib().n550_residual_add(stream_ptr(), _dp(x), _dp(y), x.numel()), "n550_residual_add")
    return x


def bf16_to_f32(b):
    import torch
    out = torch.empty(b.shape, dtype=torch.float32, device=b.device)
    check(lib().n550_bf16_to_f32(stream_ptr(), _dp(out), _dp(b), b.numel()), "n550_bf16_to_f32")
    return out


def _cache_dims(k_cache):
    if k_cache.dim() != 5 or tuple(k_cache.shape[1:3]) != (28, 8) or k_cache.shape[4] != 128:
        raise ValueError("KV cache must be [slots, 28, 8, max_len, 128]")
    return k_cache.shape[0], k_cache.shape[3]


def attention_prefill(q, k_cache, v_cache, seq_ids, L, pos0, layer, out=None):
    """Causal GQA attention of len(seq_ids) sequences x L queries (rows of q,
    BF16 [n_seqs*L, >=2048]) at positions pos0.. over the BF16 KV cache."""
    import torch
    n_slots, max_len = _cache_dims(k_cache)
    n_seqs = seq_ids.numel()
    if out is None:
        out = torch.empty((n_seqs * L, 2048), dtype=torch.bfloat16, device=q.device)
    check(lib().n550_attention_prefill(stream_ptr(), _dp(q), q.stride(0), _dp(k_cache), _dp(v_cache),
                                       n_slots, max_len, layer, _dp(seq_ids), n_seqs, L, pos0,
                                       _dp(out), out.stride(0)), "n550_attention_prefill")
    return out


def attention_decode(q, k_cache, v_cache, seq_ids, pos, layer, out=None, split=True):
    """One query per sequence (rows of q, BF16) at position pos[s]; split=True
    passes a split-KV workspace, split=False runs one CTA per (seq, KV head)."""
    import torch
    n_slots, max_len = _cache_dims(k_cache)
    n_seqs = seq_ids.numel()
    if out is None:
        out = torch.empty((n_seqs, 2048), dtype=torch.bfloat16, device=q.device)
    ws, nbytes = None, 0
    if split:
        nbytes = lib().n550_attention_decode_workspace(n_seqs, max_len)
        ws = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=q.device)
    check(lib().n550_attention_decode(stream_ptr(), _dp(q), q.stride(0), _dp(k_cache), _dp(v_cache),
                                      n_slots, max_len, layer, _dp(seq_ids), _dp(pos), n_seqs,
                                      _dp(out), out.stride(0), _dp(ws) if ws is not None else None,
                                      nbytes), "n550_attention_decode")
    return out


def device_status() -> int:
    return lib().n550_device_status()
