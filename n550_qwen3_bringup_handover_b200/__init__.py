"""n550 Qwen3-0.6B hot path on B200 -- Python host-side mirror of the C ABI.

The product is libn550_qwen3.so (csrc/, built in-tree by build.py for
sm_100a); this module only binds it with ctypes so tests, bench.py and Python
callers can reach the same entry points a C caller links against
(include/n550_qwen3.h). There is no fallback: if the library is missing the
import fails.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libn550_qwen3.so"
HEADER = PKG.parent / "include" / "n550_qwen3.h"

# Status codes (include/n550_qwen3.h)
OK = 0
ERR_MAGIC, ERR_VERSION, ERR_DTYPE, ERR_SHAPE, ERR_SIZE, ERR_OOM, ERR_LAYOUT = -1, -2, -3, -4, -5, -6, -7
ERR_ARG, ERR_CUDA, ERR_UNSUPPORTED, ERR_TIMEOUT = -101, -102, -103, -104
MODE_EXACT, MODE_FAST = 0, 1
N550_TOK_ERR_MAGIC, N550_TOK_ERR_VERSION, N550_TOK_ERR_SIZE, N550_TOK_ERR_OVERFLOW = -1, -2, -3, -5
F32, BF16 = 0, 1
LAYOUT_ROW, LAYOUT_TILE = 0, 1

_lib = None


class N550Error(RuntimeError):
    def __init__(self, status: int, what: str = ""):
        self.status = status
        super().__init__(f"{what}: {strerror(status)} ({status})" if what else strerror(status))


class SpecStats(C.Structure):
    _fields_ = [("rounds", C.c_int64), ("drafted", C.c_int64), ("accepted", C.c_int64)]


class ModelConfig(C.Structure):
    _fields_ = [("max_seqs", C.c_int), ("max_len", C.c_int), ("max_tokens", C.c_int),
                ("gemm_mode", C.c_int), ("kblock", C.c_int)]


def lib() -> C.CDLL:
    """Load libn550_qwen3.so (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise ImportError(f"{LIB_PATH} is missing; build it with "
                          "`python -m n550_qwen3_bringup_handover_b200.build`")
    L = C.CDLL(str(LIB_PATH))
    vp, i, f, sz, u16p = C.c_void_p, C.c_int, C.c_float, C.c_size_t, C.c_void_p
    sig = {
        "qwen3_gemm": (None, [vp, vp, vp, i, i, i]),
        "qwen3_gemm_row": (None, [vp, vp, vp, i, i, i]),
        "qwen3_set_weight_layout": (i, [i, i, i]),
        "qwen3_kernel_name": (C.c_char_p, []),
        "qwen3_op_rmsnorm": (None, [vp, vp, vp, i]),
        "qwen3_op_rope": (None, [vp, i, i]),
        "qwen3_op_softmax": (None, [vp, i]),
        "qwen3_op_silu_mul": (None, [vp, vp, i]),
        "qwen3_op_residual_add": (None, [vp, vp, i]),
        "qwen3_op_argmax": (i, [vp, i]),
        "qwen3_op_bf16_to_f32": (None, [vp, vp, i]),
        "qwen3_op_dot": (f, [vp, vp, i]),
        "qwen3_op_axpy": (None, [vp, f, vp, i]),
        "qwen3_ops_name": (C.c_char_p, []),
        "n550_set_gemm_mode": (i, [i, i]),
        "n550_last_status": (i, []),
        "n550_strerror": (C.c_char_p, [i]),
        "n550_gemm": (i, [vp, i, i, vp, i, i, vp, i, vp, i, i, i, i, i]),
        "n550_rmsnorm": (i, [vp, vp, i, vp, vp, i, i, f]),
        "n550_gemm_residual": (i, [vp, vp, i, vp, i, vp, i, i, i, i]),
        "n550_gemm_tile_config": (i, [i]),
        "n550_set_pdl": (i, [i]),
        "n550_gemm_skinny_config": (i, [i]),
        "n550_gemm_skinny_rows": (i, [i]),
        "n550_check_wait_expiry": (i, [vp, C.c_longlong]),
        "n550_gemm_swiglu": (i, [vp, vp, i, vp, vp, i, vp, i, i, i, i]),
        "n550_rope": (i, [vp, vp, i, i, i]),
        "n550_silu_mul": (i, [vp, vp, vp, sz]),
        "n550_softmax": (i, [vp, vp, i, i]),
        "n550_argmax": (i, [vp, vp, i, i, i, vp]),
        "n550_residual_add": (i, [vp, vp, vp, sz]),
        "n550_bf16_to_f32": (i, [vp, vp, vp, sz]),
        "n550_device_status": (i, []),
        "n550_attention_prefill": (i, [vp, vp, i, vp, vp, i, i, i, vp, i, i, i, vp, i]),
        "n550_attention_decode": (i, [vp, vp, i, vp, vp, i, i, i, vp, vp, i, vp, i, vp, sz]),
        "n550_attention_decode_workspace": (sz, [i, i]),
        "n550_rope_table": (i, [vp, vp, i]),
        "n550_qkv_rope_kv": (i, [vp, vp, i, vp, vp, vp, vp, vp, vp, i, vp, i, i, vp, vp, i, i]),
    }
    optional = {
        "n550_qwen3_init": (i, [C.POINTER(vp), vp, sz, C.POINTER(ModelConfig)]),
        "n550_qwen3_init_random": (i, [C.POINTER(vp), C.c_uint64, C.c_double, C.POINTER(ModelConfig)]),
        "n550_qwen3_free": (None, [vp]),
        "n550_qwen3_prefill": (i, [vp, vp, vp, vp, i, i, i, vp, vp]),
        "n550_qwen3_decode": (i, [vp, vp, vp, vp, vp, i, vp, vp]),
        "n550_qwen3_forward_batch_host": (i, [vp, vp, i, i, vp]),
        "n550_qwen3_decode_steps": (i, [vp, vp, vp, vp, vp, i, i, vp, i]),
        "n550_qwen3_weight": (vp, [vp, i, C.POINTER(sz)]),
        "n550_qwen3_profile": (i, [vp, i]),
        "n550_qwen3_profile_read": (i, [vp, vp, vp, i]),
        "n550_synth_tokens": (i, [vp, sz, C.c_uint64, C.c_uint64, i]),
        "n550_qwen3_get_config": (i, [vp, C.POINTER(ModelConfig)]),
        "n550_qwen3_split_rows": (i, [i]),
        "n550_qwen3_set_dump": (i, [vp, vp, vp]),
        "n550_qwen3_fused_decode": (i, [i]),
        "n550_qwen3_fused_attention_prep": (i, [i]),
        "n550_qwen3_forward_rows": (i, [vp, vp, vp, vp, i, i, vp, vp]),
        "n550_qwen3_forward_rows_host": (i, [vp, vp, i, i, vp, vp]),
        "n550_lookup_draft": (i, [vp, i, i, vp, i]),
        "n550_qwen3_generate_lookup": (i, [vp, vp, i, i, i, i, vp, i, vp, C.POINTER(C.c_int),
                                           C.POINTER(SpecStats)]),
        "n550_tok_init": (i, [C.POINTER(vp), vp, sz]),
        "n550_tok_free": (None, [vp]),
        "n550_tok_vocab_size": (i, [vp]),
        "n550_tok_encode": (i, [vp, C.c_char_p, sz, vp, i]),
        "n550_tok_decode": (i, [vp, vp, i, C.c_char_p, sz]),
        "n550_tok_piece": (vp, [vp, i, C.POINTER(sz)]),
        "n550_tok_encode_batch": (i, [vp, vp, vp, i, vp, i, vp, i]),
        "n550_chat_encode": (i, [vp, C.c_char_p, sz, vp, i]),
        "n550_qwen3_chat": (i, [vp, vp, C.c_char_p, sz, i, i, C.c_char_p, sz, vp, C.POINTER(C.c_int)]),
        "n550_synth_normal_bf16": (i, [vp, sz, C.c_uint64, C.c_uint64, C.c_double]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype, fn.argtypes = res, args
    for name, (res, args) in optional.items():
        if hasattr(L, name):
            fn = getattr(L, name)
            fn.restype, fn.argtypes = res, args
    _lib = L
    return L


def strerror(status: int) -> str:
    return lib().n550_strerror(status).decode()


def check(status: int, what: str = "") -> None:
    if status != OK:
        raise N550Error(status, what)


def kernel_name() -> str:
    return lib().qwen3_kernel_name().decode()


def synth_tokens(n: int, seed: int, stream: int, vocab: int = 151936):
    """Seeded synthetic token ids (numpy int32), the library's generator."""
    import numpy as np
    out = np.empty(n, np.int32)
    check(lib().n550_synth_tokens(out.ctypes.data_as(C.c_void_p), n, seed, stream, vocab),
          "n550_synth_tokens")
    return out


def synth_normal_bf16(shape, seed: int, stream: int, sigma: float):
    """Seeded synthetic BF16 bits (numpy uint16), the library's generator."""
    import numpy as np
    out = np.empty(shape, np.uint16)
    check(lib().n550_synth_normal_bf16(out.ctypes.data_as(C.c_void_p), out.size, seed, stream, sigma),
          "n550_synth_normal_bf16")
    return out


def lookup_draft(hist, ngram: int = 3, max_k: int = 127):
    """Prompt-lookup draft tokens for the history `hist` (n550_lookup_draft)."""
    import numpy as np
    h = np.ascontiguousarray(hist, np.int32)
    out = np.empty(max(max_k, 1), np.int32)
    k = lib().n550_lookup_draft(h.ctypes.data_as(C.c_void_p), h.size, ngram,
                                out.ctypes.data_as(C.c_void_p), max_k)
    if k < 0:
        check(k, "n550_lookup_draft")
    return out[:k].copy()


def set_gemm_mode(mode: int, kblock: int = 16) -> None:
    check(lib().n550_set_gemm_mode(mode, kblock), "n550_set_gemm_mode")


from .api import *  # noqa: E402,F401,F403
from .model import Model  # noqa: E402,F401
from .tokenizer import Tokenizer  # noqa: E402,F401
