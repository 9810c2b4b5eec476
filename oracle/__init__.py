"""CPU oracle for the n550 Qwen3 hot path -- TEST INFRASTRUCTURE ONLY.

Importable only by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
leg, where it is the checker or the timed CPU baseline. The product package
never imports it.

  liboracle.so   this project's C restatement (oracle/*.c, built by `make -C oracle`)
  _ref/libref_<kernel>.so  the reference's own qwen3.c + kernels_<kernel>.c +
                 ops_scalar.c (built by `make -C oracle ref` where the reference
                 sources exist; the built files travel with the repository)
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "liboracle.so"
REF_DIR = HERE / "_ref"

GEMM_SCALAR, GEMM_HWSIM, GEMM_EXACT16, GEMM_EXACT32 = 0, 1, 2, 3
VOCAB = 151936
QW3M_SIZE = 1_192_100_096

_lib = None


def _p(a):
    return a.ctypes.data_as(C.c_void_p)


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} missing: run `make -C oracle`")
        L = C.CDLL(str(LIB_PATH))
        vp, i, sz, u64, f, d = C.c_void_p, C.c_int, C.c_size_t, C.c_uint64, C.c_float, C.c_double
        L.oracle_gemm_ame_exact.argtypes = [vp, i, vp, vp, i, vp, i, i, i, i, i]
        L.oracle_gemm_ame_exact_f32a.argtypes = [vp, vp, vp, i, i, i, i]
        for n in ("oracle_gemm_hwsim", "oracle_gemm_scalar", "oracle_gemm_f64"):
            getattr(L, n).argtypes = [vp, vp, vp, i, i, i]
        L.oracle_f32_to_bf16_rne.argtypes = [f]
        L.oracle_f32_to_bf16_rne.restype = C.c_uint16
        L.oracle_f32_to_bf16_array.argtypes = [vp, vp, sz]
        L.oracle_op_rmsnorm.argtypes = [vp, vp, vp, i]
        L.oracle_op_rope.argtypes = [vp, i, i]
        L.oracle_op_softmax.argtypes = [vp, i]
        L.oracle_op_silu_mul.argtypes = [vp, vp, i]
        L.oracle_op_residual_add.argtypes = [vp, vp, i]
        L.oracle_op_argmax.argtypes = [vp, i]
        L.oracle_op_argmax.restype = i
        L.oracle_op_bf16_to_f32.argtypes = [vp, vp, i]
        L.oracle_op_dot.argtypes = [vp, vp, i]
        L.oracle_op_dot.restype = f
        L.oracle_op_axpy.argtypes = [vp, f, vp, i]
        L.oracle_synth_u64.argtypes = [u64, u64, u64]
        L.oracle_synth_u64.restype = u64
        L.oracle_synth_normal_bf16.argtypes = [vp, sz, u64, u64, d]
        L.oracle_synth_normal_f32.argtypes = [vp, sz, u64, u64, d]
        L.oracle_synth_tokens.argtypes = [vp, sz, u64, u64, i]
        L.oracle_qw3m_size.restype = sz
        L.oracle_qw3m_write.argtypes = [vp, sz, u64, d]
        L.oracle_model_create.argtypes = [vp, sz, i, i, C.POINTER(i)]
        L.oracle_model_create.restype = vp
        L.oracle_model_destroy.argtypes = [vp]
        L.oracle_model_forward_batch.argtypes = [vp, vp, i, i]
        L.oracle_model_logits.argtypes = [vp]
        L.oracle_model_logits.restype = C.POINTER(C.c_float)
        _lib = L
    return _lib


# ---------------- GEMMs ----------------

def gemm_ame_exact(a_bf16, b_bf16, kblock=16, M=None, N=None, K=None, lda=None, ldb=None):
    """C bits (uint32 [M,N]) and peak (float32 [M,N]) under the AME exact rule."""
    a = np.ascontiguousarray(a_bf16, dtype=np.uint16)
    b = np.ascontiguousarray(b_bf16, dtype=np.uint16)
    M = a.shape[0] if M is None else M
    N = b.shape[0] if N is None else N
    lda = a.shape[1] if lda is None else lda
    ldb = b.shape[1] if ldb is None else ldb
    K = min(lda, ldb) if K is None else K
    c = np.zeros((M, N), np.uint32)
    pk = np.zeros((M, N), np.float32)
    rc = lib().oracle_gemm_ame_exact(_p(c), N, _p(pk), _p(a), lda, _p(b), ldb, M, N, K, kblock)
    if rc:
        raise ValueError("oracle_gemm_ame_exact: bad arguments")
    return c, pk


def gemm_ame_exact_f32a(a_f32, b_bf16, kblock=16):
    a = np.ascontiguousarray(a_f32, dtype=np.float32)
    b = np.ascontiguousarray(b_bf16, dtype=np.uint16)
    M, K = a.shape
    N = b.shape[0]
    c = np.zeros((M, N), np.float32)
    lib().oracle_gemm_ame_exact_f32a(_p(c), _p(a), _p(b), M, K, N, kblock)
    return c


def _gemm(name, a_f32, b_bf16):
    a = np.ascontiguousarray(a_f32, dtype=np.float32)
    b = np.ascontiguousarray(b_bf16, dtype=np.uint16)
    M, K = a.shape
    N = b.shape[0]
    c = np.zeros((M, N), np.float32)
    getattr(lib(), name)(_p(c), _p(a), _p(b), M, K, N)
    return c


def gemm_hwsim(a, b):
    return _gemm("oracle_gemm_hwsim", a, b)


def gemm_scalar(a, b):
    return _gemm("oracle_gemm_scalar", a, b)


def gemm_f64(a, b):
    return _gemm("oracle_gemm_f64", a, b)


# ---------------- conversions / synthetic data ----------------

def f32_to_bf16(x):
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.zeros(x.shape, np.uint16)
    lib().oracle_f32_to_bf16_array(_p(out), _p(x), x.size)
    return out


def bf16_to_f32(b):
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def synth_normal_bf16(shape, seed, stream, sigma):
    out = np.zeros(shape, np.uint16)
    lib().oracle_synth_normal_bf16(_p(out), out.size, seed, stream, sigma)
    return out


def synth_normal_f32(shape, seed, stream, sigma):
    out = np.zeros(shape, np.float32)
    lib().oracle_synth_normal_f32(_p(out), out.size, seed, stream, sigma)
    return out


def synth_tokens(n, seed, stream, vocab=VOCAB):
    out = np.zeros(n, np.int32)
    lib().oracle_synth_tokens(_p(out), n, seed, stream, vocab)
    return out


def qw3m_blob(seed=0, sigma=0.02):
    size = lib().oracle_qw3m_size()
    blob = np.empty(size, np.uint8)
    if lib().oracle_qw3m_write(_p(blob), size, seed, sigma):
        raise RuntimeError("oracle_qw3m_write failed")
    return blob


# ---------------- ops ----------------

def rmsnorm(x, w):
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty_like(x)
    w = np.ascontiguousarray(w, np.uint16)
    n = x.shape[-1]
    xs, os_ = x.reshape(-1, n), out.reshape(-1, n)
    for r in range(xs.shape[0]):
        lib().oracle_op_rmsnorm(_p(os_[r]), _p(xs[r]), _p(w), n)
    return out


def rope(v, n_heads, pos):
    v = np.array(v, np.float32, copy=True)
    lib().oracle_op_rope(_p(v), n_heads, pos)
    return v


def softmax(x):
    x = np.array(x, np.float32, copy=True)
    lib().oracle_op_softmax(_p(x), x.size)
    return x


def silu_mul(g, u):
    g = np.array(g, np.float32, copy=True)
    u = np.ascontiguousarray(u, np.float32)
    lib().oracle_op_silu_mul(_p(g), _p(u), g.size)
    return g


def argmax(v):
    v = np.ascontiguousarray(v, np.float32)
    return int(lib().oracle_op_argmax(_p(v), v.size))


def dot(a, b):
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    return float(lib().oracle_op_dot(_p(a), _p(b), a.size))


def axpy(y, a, x):
    y = np.array(y, np.float32, copy=True)
    x = np.ascontiguousarray(x, np.float32)
    lib().oracle_op_axpy(_p(y), a, _p(x), y.size)
    return y


# ---------------- forward ----------------

class OracleModel:
    """The C restatement of qwen3_forward_batch on a QW3M blob."""

    def __init__(self, blob, max_seq=256, gemm_kind=GEMM_SCALAR):
        self._blob = blob
        err = C.c_int(0)
        self._h = lib().oracle_model_create(_p(blob), blob.size, max_seq, gemm_kind, C.byref(err))
        if not self._h:
            raise RuntimeError(f"oracle_model_create failed: {err.value}")

    def forward_batch(self, tokens, pos0):
        t = np.ascontiguousarray(tokens, np.int32)
        if lib().oracle_model_forward_batch(self._h, _p(t), t.size, pos0):
            raise ValueError("forward_batch: bad arguments")
        return np.ctypeslib.as_array(lib().oracle_model_logits(self._h), (VOCAB,)).copy()

    def close(self):
        if self._h:
            lib().oracle_model_destroy(self._h)
            self._h = None

    def __del__(self):
        self.close()


class RefModel:
    """The reference's own qwen3.c (+ kernels_<kernel>.c) built in oracle/_ref.

    One model per library (the reference keeps a static model instance)."""

    def __init__(self, blob, kernel="scalar"):
        path = REF_DIR / f"libref_{kernel}.so"
        if not path.exists():
            raise FileNotFoundError(path)
        L = C.CDLL(str(path), mode=os.RTLD_LOCAL)
        L.ref_model_init.argtypes = [C.c_void_p, C.c_size_t]
        L.ref_forward_batch.argtypes = [C.c_void_p, C.c_int, C.c_int]
        L.ref_logits.restype = C.POINTER(C.c_float)
        L.ref_logits_row.restype = C.POINTER(C.c_float)
        L.ref_logits_row.argtypes = [C.c_int]
        L.ref_kernel_name.restype = C.c_char_p
        self.L = L
        self._blob = blob
        rc = L.ref_model_init(_p(blob), blob.size)
        if rc:
            raise RuntimeError(f"qwen3_init failed: {rc}")
        self.max_seq = L.ref_max_seq()

    def forward_batch(self, tokens, pos0):
        t = np.ascontiguousarray(tokens, np.int32)
        self.L.ref_forward_batch(_p(t), t.size, pos0)
        return np.ctypeslib.as_array(self.L.ref_logits(), (VOCAB,)).copy()

    def forward_dump(self, tokens, pos0):
        """forward_batch with the reference's per-op dump on: the list of
        (layer, name, FP32 array) of every EMIT point, in order."""
        out = []
        fn_t = C.CFUNCTYPE(None, C.c_void_p, C.c_int, C.c_char_p, C.POINTER(C.c_float), C.c_size_t)

        def cb(ctx, layer, name, data, n):
            out.append((layer, name.decode(), np.ctypeslib.as_array(data, (n,)).copy()))

        f = fn_t(cb)
        self.L.ref_set_dump.argtypes = [fn_t, C.c_void_p]
        self.L.ref_set_dump(f, None)
        try:
            self.forward_batch(tokens, pos0)
        finally:
            self.L.ref_set_dump(fn_t(0), None)
        return out

    def logits_rows(self):
        """Every row of logits the last call left ([n_logits, VOCAB]); all rows
        of the call in the QWEN3_SPECULATIVE build (libref_spec.so)."""
        n = self.L.ref_n_logits()
        return np.stack([np.ctypeslib.as_array(self.L.ref_logits_row(i), (VOCAB,)).copy()
                         for i in range(n)])

    def gemm(self, a_f32, b_bf16):
        a = np.ascontiguousarray(a_f32, np.float32)
        b = np.ascontiguousarray(b_bf16, np.uint16)
        M, K = a.shape
        N = b.shape[0]
        c = np.zeros((M, N), np.float32)
        self.L.qwen3_gemm.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int]
        self.L.qwen3_gemm(_p(c), _p(a), _p(b), M, K, N)
        return c


_ref_libs = {}


def ref_gemm(kernel, a_f32, b_bf16):
    """The reference's own qwen3_gemm from kernels_<kernel>.c (oracle/_ref)."""
    if kernel not in _ref_libs:
        L = C.CDLL(str(REF_DIR / f"libref_{kernel}.so"), mode=os.RTLD_LOCAL)
        L.qwen3_gemm.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int]
        _ref_libs[kernel] = L
    a = np.ascontiguousarray(a_f32, np.float32)
    b = np.ascontiguousarray(b_bf16, np.uint16)
    M, K = a.shape
    N = b.shape[0]
    c = np.zeros((M, N), np.float32)
    _ref_libs[kernel].qwen3_gemm(_p(c), _p(a), _p(b), M, K, N)
    return c


def ref_available(kernel="scalar"):
    return (REF_DIR / f"libref_{kernel}.so").exists()


# ---------------- prompt-lookup speculative decoding ----------------

def lookup_draft(hist, ngram, max_k):
    """Restates lookup_draft (main_baremetal.c:567-584): the last `ngram`
    tokens of hist are searched for earlier, newest match first; up to max_k
    tokens that followed the match are returned ([] without a match)."""
    n = len(hist)
    if n < ngram + 1 or max_k <= 0:
        return []
    pat = list(hist[n - ngram:])
    for i in range(n - ngram - 1, -1, -1):
        if list(hist[i:i + ngram]) != pat:
            continue
        out = list(hist[i + ngram:i + ngram + max_k])
        if out:
            return out
    return []


def speculative_generate(model, prompt, max_new, max_draft, ngram=3, eos=(151645, 151643),
                         max_seq=2048):
    """Restates the QWEN3_SPECULATIVE generation loop (main_baremetal.c:636-690)
    on a RefModel of libref_spec.so (all-row logits): returns (tokens,
    rounds, drafted, accepted)."""
    hist = [int(t) for t in prompt]
    logits = model.forward_batch(np.asarray(prompt, np.int32), 0)
    nxt = argmax(logits)
    limit = min(max_new, max_seq - len(prompt))
    pos, out = len(prompt), []
    rounds = drafted = accepted = 0
    while len(out) < limit:
        if nxt in eos:
            break
        draft = lookup_draft(hist, ngram, max_draft)[:max(0, limit - len(out) - 1)]
        batch = np.asarray([nxt] + draft, np.int32)
        model.forward_batch(batch, pos)
        rows = model.logits_rows()
        rounds += 1
        drafted += len(draft)
        out.append(nxt)
        hist.append(nxt)
        kept, done = 1, False
        for j, d in enumerate(draft):
            if len(out) >= limit:
                break
            pred = argmax(rows[j])
            if pred != d:
                nxt, done = pred, True
                break
            accepted += 1
            if pred in eos:
                nxt, done = pred, True
                break
            out.append(pred)
            hist.append(pred)
            kept += 1
        if not done:
            nxt = argmax(rows[len(draft)])
        pos += kept
    return out, rounds, drafted, accepted


# ---------------- tokenizer ----------------

TOK_PATH = REF_DIR / "tok.bin"


class RefTokenizer:
    """The reference's own tokenizer.c (oracle/_ref/libref_tok.so) on a QW3T
    vocabulary; one instance per process (the reference keeps static state)."""

    def __init__(self, blob=None):
        L = C.CDLL(str(REF_DIR / "libref_tok.so"), mode=os.RTLD_LOCAL)
        L.ref_tok_init.argtypes = [C.c_void_p, C.c_size_t]
        L.ref_tok_encode.argtypes = [C.c_char_p, C.c_size_t, C.c_void_p, C.c_int]
        L.ref_tok_decode.argtypes = [C.c_void_p, C.c_int, C.c_char_p, C.c_size_t]
        self.L = L
        self._blob = np.frombuffer(TOK_PATH.read_bytes() if blob is None else blob, np.uint8).copy()
        self.rc = L.ref_tok_init(_p(self._blob), self._blob.size)

    def encode(self, data: bytes, max_out=4096):
        out = np.zeros(max_out, np.int32)
        n = self.L.ref_tok_encode(data, len(data), _p(out), max_out)
        return n if n < 0 else out[:n].copy()

    def decode(self, ids, max_out=1 << 16):
        ids = np.ascontiguousarray(ids, np.int32)
        buf = C.create_string_buffer(max_out)
        n = self.L.ref_tok_decode(_p(ids), ids.size, buf, max_out)
        return n if n < 0 else buf.raw[:n]


def tokenizer_available():
    return TOK_PATH.exists() and (REF_DIR / "libref_tok.so").exists()
