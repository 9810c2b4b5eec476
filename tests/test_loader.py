"""QW3M loader checks of n550_qwen3_init (qwen3.c:93-146): same order, same
error codes. The header is validated before any device call, so these run
without a GPU."""
import ctypes as C

import numpy as np
import pytest

import n550_qwen3_bringup_handover_b200 as n5

QW3M_SIZE = 1_192_100_096


def header(**over):
    h = np.zeros(256, np.uint8)
    h[:4] = np.frombuffer(b"QW3M", np.uint8)
    vals = dict(version=1, hidden=1024, inter=3072, layers=28, heads=16, kv=8, hd=128,
                vocab=151936, max_pos=40960, tie=1, dtype=1, bos=151643, eos0=151645,
                eos1=151643, data_start=256, align=128, layout=0, tile_n=0, tile_k=0)
    vals.update(over)
    off = dict(version=4, hidden=8, inter=12, layers=16, heads=20, kv=24, hd=28, vocab=32,
               max_pos=36, tie=40, dtype=44, bos=56, eos0=60, eos1=64, data_start=68,
               align=72, layout=76, tile_n=80, tile_k=84)
    for k, o in off.items():
        h[o:o + 4] = np.frombuffer(np.int32(vals[k]).tobytes(), np.uint8)
    h[48:52] = np.frombuffer(np.float32(over.get("theta", 1000000.0)).tobytes(), np.uint8)
    h[52:56] = np.frombuffer(np.float32(over.get("eps", 1e-6)).tobytes(), np.uint8)
    return h


def init_status(blob, size=None):
    cfg = n5.ModelConfig(1, 64, 16, n5.MODE_FAST, 16)
    h = C.c_void_p()
    size = blob.size if size is None else size
    return n5.lib().n550_qwen3_init(C.byref(h), blob.ctypes.data_as(C.c_void_p), size, C.byref(cfg))


@pytest.mark.parametrize("mutation,code", [
    (dict(), n5.ERR_SIZE),                       # header only: tensors run past the end
    (dict(version=2), n5.ERR_VERSION),
    (dict(dtype=2), n5.ERR_DTYPE),
    (dict(hidden=896), n5.ERR_SHAPE),
    (dict(vocab=151000), n5.ERR_SHAPE),
    (dict(align=96), n5.ERR_SHAPE),
    (dict(align=64), n5.ERR_SHAPE),
    (dict(layout=1), n5.ERR_LAYOUT),             # tile-major without a tile shape
    (dict(layout=1, tile_n=64, tile_k=32), n5.ERR_LAYOUT),
    (dict(layout=2, tile_n=128, tile_k=32), n5.ERR_LAYOUT),
    (dict(layout=1, tile_n=128, tile_k=32, align=4096), n5.ERR_SIZE),   # accepted; header only
    (dict(theta=10000.0), n5.ERR_SHAPE),
    (dict(eps=1e-5), n5.ERR_SHAPE),
])
def test_header_error_codes(mutation, code):
    assert init_status(header(**mutation)) == code


def test_bad_magic_and_short_blob():
    h = header()
    h[0] = ord("X")
    assert init_status(h) == n5.ERR_MAGIC
    assert init_status(header(), size=100) == n5.ERR_SIZE


def test_config_validation():
    h = C.c_void_p()
    blob = header()
    for cfg in (n5.ModelConfig(0, 64, 16, n5.MODE_FAST, 16), n5.ModelConfig(1, 64, 16, 7, 16),
                n5.ModelConfig(1, 64, 16, n5.MODE_EXACT, 24)):
        assert n5.lib().n550_qwen3_init(C.byref(h), blob.ctypes.data_as(C.c_void_p), blob.size,
                                        C.byref(cfg)) == n5.ERR_ARG
