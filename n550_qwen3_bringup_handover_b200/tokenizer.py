"""Host tokenizer binding (n550_tok_*, include/n550_qwen3.h section 4): the
Qwen3 byte-level BPE over a QW3T vocabulary file (the reference's tok.bin),
and the chat template of the reference's chat mode (main.c:124-131)."""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np

from . import check, lib


class Tokenizer:
    """QW3T vocabulary loaded into the library (the bytes are copied)."""

    def __init__(self, blob: bytes | str | Path):
        if isinstance(blob, (str, Path)):
            blob = Path(blob).read_bytes()
        buf = np.frombuffer(blob, np.uint8)
        self._lib = lib()          # held for close() at interpreter exit
        h = C.c_void_p()
        check(lib().n550_tok_init(C.byref(h), buf.ctypes.data_as(C.c_void_p), buf.size),
              "n550_tok_init")
        self._h = h

    def close(self):
        if getattr(self, "_h", None):
            self._lib.n550_tok_free(self._h)
            self._h = None

    def __del__(self):
        self.close()

    @property
    def handle(self):
        return self._h

    @property
    def vocab_size(self) -> int:
        return lib().n550_tok_vocab_size(self._h)

    def encode(self, text: str | bytes, max_out: int = 8192) -> np.ndarray:
        data = text.encode() if isinstance(text, str) else bytes(text)
        out = np.empty(max_out, np.int32)
        n = lib().n550_tok_encode(self._h, data, len(data), out.ctypes.data_as(C.c_void_p), max_out)
        if n < 0:
            check(n, "n550_tok_encode")
        return out[:n].copy()

    def chat(self, prompt: str | bytes, max_out: int = 8192) -> np.ndarray:
        """Token ids of one user turn in Qwen3's chat template (thinking off)."""
        data = prompt.encode() if isinstance(prompt, str) else bytes(prompt)
        out = np.empty(max_out, np.int32)
        n = lib().n550_chat_encode(self._h, data, len(data), out.ctypes.data_as(C.c_void_p), max_out)
        if n < 0:
            check(n, "n550_chat_encode")
        return out[:n].copy()

    def encode_batch(self, texts, max_out: int = 4096, threads: int = 0):
        """Many texts on host threads: a list of id arrays."""
        datas = [t.encode() if isinstance(t, str) else bytes(t) for t in texts]
        n = len(datas)
        ptrs = (C.c_char_p * max(n, 1))(*datas)
        lens = (C.c_size_t * max(n, 1))(*[len(d) for d in datas])
        out = np.empty((max(n, 1), max_out), np.int32)
        counts = np.empty(max(n, 1), np.int32)
        check(lib().n550_tok_encode_batch(self._h, ptrs, lens, n, out.ctypes.data_as(C.c_void_p),
                                          max_out, counts.ctypes.data_as(C.c_void_p), threads),
              "n550_tok_encode_batch")
        return [out[i, :counts[i]].copy() for i in range(n)]

    def decode(self, ids, max_out: int = 1 << 20) -> bytes:
        a = np.ascontiguousarray(ids, np.int32)
        buf = C.create_string_buffer(max_out)
        n = lib().n550_tok_decode(self._h, a.ctypes.data_as(C.c_void_p), a.size, buf, max_out)
        if n < 0:
            check(n, "n550_tok_decode")
        return buf.raw[:n]

    def piece(self, token_id: int) -> bytes:
        n = C.c_size_t(0)
        p = lib().n550_tok_piece(self._h, token_id, C.byref(n))
        return C.string_at(p, n.value) if p and n.value else b""
