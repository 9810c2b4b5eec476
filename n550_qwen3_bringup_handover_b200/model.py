"""Model runtime binding: the reference's qwen3_init / qwen3_forward_batch /
qwen3_forward / qwen3_argmax (qwen3.h:206-248) as one handle over
libn550_qwen3.so, extended to many sequences per call."""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import MODE_FAST, ModelConfig, SpecStats, check, lib

VOCAB = 151936
EOS_IDS = (151645, 151643)          # QWEN3_EOS_TOKEN_ID_0 / _1 (qwen3_config.h:29-30)


class Model:
    """Weights, KV cache and activations of Qwen3-0.6B on the current CUDA device."""

    def __init__(self, *, blob: np.ndarray | None = None, seed: int = 0, sigma: float = 0.02,
                 max_seqs: int = 1, max_len: int = 2048, max_tokens: int = 512,
                 gemm_mode: int = MODE_FAST, kblock: int = 16):
        self.cfg = ModelConfig(max_seqs, max_len, max_tokens, gemm_mode, kblock)
        # held for close(): at interpreter exit the module's globals may be gone
        self._lib = lib()
        h = C.c_void_p()
        if blob is not None:
            b = np.ascontiguousarray(blob, np.uint8)
            rc = lib().n550_qwen3_init(C.byref(h), b.ctypes.data_as(C.c_void_p), b.size,
                                       C.byref(self.cfg))
        else:
            rc = lib().n550_qwen3_init_random(C.byref(h), seed, sigma, C.byref(self.cfg))
        check(rc, "n550_qwen3_init")
        self._h = h

    @property
    def handle(self):
        return self._h

    def close(self):
        if getattr(self, "_h", None):
            self._lib.n550_qwen3_free(self._h)
            self._h = None

    def __del__(self):
        self.close()

    # ---- reference-shaped host path (sequence slot 0) ----
    def forward_batch(self, tokens, pos0: int, want_logits: bool = True):
        """qwen3_forward_batch on host tokens: (argmax, last-token logits or None)."""
        t = np.ascontiguousarray(tokens, np.int32)
        logits = np.empty(VOCAB, np.float32) if want_logits else None
        r = lib().n550_qwen3_forward_batch_host(
            self._h, t.ctypes.data_as(C.c_void_p), t.size, pos0,
            logits.ctypes.data_as(C.c_void_p) if want_logits else None)
        if r < 0:
            check(r, "n550_qwen3_forward_batch_host")
        return int(r), logits

    def forward_dump(self, tokens, pos0: int):
        """forward_batch on slot 0 with the per-op dump (n550_qwen3_set_dump):
        (next id, [(layer, name, FP32 array), ...] in the reference's order)."""
        out = []
        fn_t = C.CFUNCTYPE(None, C.c_void_p, C.c_int, C.c_char_p, C.POINTER(C.c_float), C.c_size_t)

        def cb(ctx, layer, name, data, n):
            out.append((layer, name.decode(), np.ctypeslib.as_array(data, (n,)).copy()))

        f = fn_t(cb)
        check(lib().n550_qwen3_set_dump(self._h, f, None), "n550_qwen3_set_dump")
        try:
            nxt, _ = self.forward_batch(tokens, pos0)
        finally:
            lib().n550_qwen3_set_dump(self._h, fn_t(0), None)
        return nxt, out

    def forward_rows(self, tokens, pos0: int, want_logits: bool = False):
        """Every row's argmax (and logits) of one call on slot 0: the
        QWEN3_SPECULATIVE qwen3_forward_batch (n550_qwen3_forward_rows_host)."""
        t = np.ascontiguousarray(tokens, np.int32)
        ids = np.empty(t.size, np.int32)
        logits = np.empty((t.size, VOCAB), np.float32) if want_logits else None
        check(lib().n550_qwen3_forward_rows_host(
            self._h, t.ctypes.data_as(C.c_void_p), t.size, pos0, ids.ctypes.data_as(C.c_void_p),
            logits.ctypes.data_as(C.c_void_p) if want_logits else None), "n550_qwen3_forward_rows_host")
        return ids, logits

    def generate_lookup(self, prompt, max_new: int, max_draft: int = 127, ngram: int = 3,
                        eos=EOS_IDS):
        """Greedy generation with prompt-lookup speculative verification on
        slot 0 (n550_qwen3_generate_lookup): (tokens, stats dict)."""
        p = np.ascontiguousarray(prompt, np.int32)
        e = np.ascontiguousarray(eos, np.int32)
        out = np.empty(max(max_new, 1), np.int32)
        n = C.c_int(0)
        st = SpecStats()
        check(lib().n550_qwen3_generate_lookup(
            self._h, p.ctypes.data_as(C.c_void_p), p.size, max_new, max_draft, ngram,
            e.ctypes.data_as(C.c_void_p), e.size, out.ctypes.data_as(C.c_void_p), C.byref(n),
            C.byref(st)), "n550_qwen3_generate_lookup")
        return out[:n.value].copy(), {"rounds": st.rounds, "drafted": st.drafted,
                                       "accepted": st.accepted}

    def chat(self, tokenizer, prompt, max_new: int = 64, max_draft: int = 0,
             max_text: int = 1 << 16):
        """One chat turn (n550_qwen3_chat): (reply bytes, generated ids)."""
        data = prompt.encode() if isinstance(prompt, str) else bytes(prompt)
        ids = np.empty(max(max_new, 1), np.int32)
        n = C.c_int(0)
        buf = C.create_string_buffer(max_text)
        r = lib().n550_qwen3_chat(self._h, tokenizer.handle, data, len(data), max_new, max_draft,
                                  buf, max_text, ids.ctypes.data_as(C.c_void_p), C.byref(n))
        if r < 0:
            check(r, "n550_qwen3_chat")
        return buf.raw[:r], ids[:n.value].copy()

    # ---- batched device path (torch CUDA tensors) ----
    def prefill(self, tokens, seq_ids, pos0=0, logits=None, next_token=None, stream=None):
        from .api import stream_ptr
        S, L = tokens.shape
        check(lib().n550_qwen3_prefill(
            self._h, stream_ptr(stream), C.c_void_p(tokens.data_ptr()), C.c_void_p(seq_ids.data_ptr()),
            S, L, pos0, C.c_void_p(logits.data_ptr()) if logits is not None else None,
            C.c_void_p(next_token.data_ptr()) if next_token is not None else None), "n550_qwen3_prefill")

    def decode(self, tokens, seq_ids, pos, logits=None, next_token=None, stream=None):
        from .api import stream_ptr
        check(lib().n550_qwen3_decode(
            self._h, stream_ptr(stream), C.c_void_p(tokens.data_ptr()), C.c_void_p(seq_ids.data_ptr()),
            C.c_void_p(pos.data_ptr()), tokens.shape[0],
            C.c_void_p(logits.data_ptr()) if logits is not None else None,
            C.c_void_p(next_token.data_ptr()) if next_token is not None else None), "n550_qwen3_decode")

    def decode_steps(self, tokens, seq_ids, pos, steps, out_ids, use_graph=True, stream=None):
        """`steps` greedy steps; tokens/pos (device int32) advance in place,
        out_ids[steps, n_seqs] receives the chosen ids."""
        from .api import stream_ptr
        check(lib().n550_qwen3_decode_steps(
            self._h, stream_ptr(stream), C.c_void_p(tokens.data_ptr()), C.c_void_p(seq_ids.data_ptr()),
            C.c_void_p(pos.data_ptr()), tokens.shape[0], steps, C.c_void_p(out_ids.data_ptr()),
            1 if use_graph else 0), "n550_qwen3_decode_steps")

    def weight_bits(self, which: int) -> np.ndarray:
        """Copy of one QW3M tensor (BF16 bits) from the device."""
        import torch
        n = C.c_size_t(0)
        p = lib().n550_qwen3_weight(self._h, which, C.byref(n))
        if not p:
            raise IndexError(which)
        view = torch.as_tensor(_DeviceArray(p, n.value), device="cuda")
        return view.cpu().numpy().view(np.uint16)


class _DeviceArray:
    """Zero-copy CUDA array interface over a device pointer of int16."""

    def __init__(self, ptr: int, n: int):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<i2", "data": (ptr, False),
                                         "version": 3, "strides": None}
