"""CPU checks of the C ABI: the library loads, exports every function the
public header declares, and its host-only logic (layout negotiation, mode
selection, status strings) behaves like the reference interface."""
import re
import subprocess

import pytest

import n550_qwen3_bringup_handover_b200 as n5


def declared_functions():
    text = n5.HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", " ", text, flags=re.S)
    names = re.findall(r"\b((?:qwen3|n550)_[A-Za-z0-9_]+)\s*\(", text)
    return sorted(set(names))


def test_header_declares_reference_plug_points():
    names = set(declared_functions())
    # kernels.h:56-92 and ops.h:21-49
    for ref in ["qwen3_gemm", "qwen3_gemm_row", "qwen3_set_weight_layout", "qwen3_kernel_name",
                "qwen3_op_rmsnorm", "qwen3_op_rope", "qwen3_op_softmax", "qwen3_op_silu_mul",
                "qwen3_op_residual_add", "qwen3_op_argmax", "qwen3_op_bf16_to_f32",
                "qwen3_op_dot", "qwen3_op_axpy", "qwen3_ops_name"]:
        assert ref in names


def test_library_exports_every_declared_symbol():
    out = subprocess.run(["nm", "-D", "--defined-only", str(n5.LIB_PATH)],
                         capture_output=True, text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    missing = [f for f in declared_functions() if f not in exported]
    assert not missing, missing


def test_library_loads_and_binds():
    L = n5.lib()
    for f in declared_functions():
        assert hasattr(L, f)


def test_weight_layout_negotiation():
    # kernels_ame.c:188-207: ROW always, TILE only with 128x32 tiles
    assert n5.qwen3_set_weight_layout(n5.LAYOUT_ROW, 0, 0) == 0
    assert n5.qwen3_set_weight_layout(n5.LAYOUT_TILE, 128, 32) == 0
    assert n5.qwen3_set_weight_layout(n5.LAYOUT_TILE, 64, 32) != 0
    assert n5.qwen3_set_weight_layout(7, 128, 32) != 0
    assert n5.qwen3_set_weight_layout(n5.LAYOUT_ROW, 0, 0) == 0


def test_gemm_mode_selection_and_names():
    try:
        n5.set_gemm_mode(n5.MODE_EXACT, 32)
        assert "32" in n5.kernel_name()
        n5.set_gemm_mode(n5.MODE_FAST)
        assert "fast" in n5.kernel_name()
        with pytest.raises(n5.N550Error):
            n5.set_gemm_mode(n5.MODE_EXACT, 24)
        with pytest.raises(n5.N550Error):
            n5.set_gemm_mode(9, 16)
    finally:
        n5.set_gemm_mode(n5.MODE_EXACT, 16)
    assert "16" in n5.kernel_name()
    assert n5.lib().qwen3_ops_name().decode()


def test_status_strings():
    for s in (n5.OK, n5.ERR_MAGIC, n5.ERR_LAYOUT, n5.ERR_ARG, n5.ERR_CUDA, n5.ERR_TIMEOUT):
        assert n5.strerror(s) and n5.strerror(s) != "unknown"
    assert n5.strerror(12345) == "unknown"


def test_device_entry_points_reject_bad_arguments():
    """Argument checks of the stream-ordered entry points run on the host
    before any CUDA call (so this runs without a GPU): invalid shapes, strides,
    layers and knob values give N550_ERR_ARG, empty problems N550_OK."""
    L = n5.lib()
    assert L.n550_gemm_tile_config(7) == n5.ERR_ARG
    assert L.n550_gemm_tile_config(0) == n5.OK
    assert L.n550_gemm_skinny_config(17) == n5.ERR_ARG
    assert L.n550_gemm_skinny_config(-2) == n5.ERR_ARG
    assert L.n550_gemm_skinny_config(0) == n5.OK
    # n550_gemm_residual(stream, a, lda, b, ldb, x, ldx, M, N, K)
    assert L.n550_gemm_residual(None, None, 8, None, 8, None, 8, -1, 8, 8) == n5.ERR_ARG
    assert L.n550_gemm_residual(None, None, 4, None, 8, None, 8, 0, 8, 8) == n5.ERR_ARG   # lda < K
    assert L.n550_gemm_residual(None, None, 8, None, 8, None, 8, 0, 8, 8) == n5.OK        # M = 0
    # n550_gemm_swiglu(stream, a, lda, wg, wu, ldw, h, ldh, M, N, K)
    assert L.n550_gemm_swiglu(None, None, 8, None, None, 8, None, 8, -1, 8, 8) == n5.ERR_ARG
    assert L.n550_gemm_swiglu(None, None, 8, None, None, 8, None, 4, 2, 8, 8) == n5.ERR_ARG  # ldh < N
    # attention: no KV slots, a layer past the 28th, null buffers
    assert L.n550_attention_prefill(None, None, 2048, None, None, 0, 64, 0, None, 1, 8, 0, None,
                                    2048) == n5.ERR_ARG
    assert L.n550_attention_decode(None, None, 2048, None, None, 1, 64, 28, None, None, 1, None,
                                   2048, None, 0) == n5.ERR_ARG
    assert L.n550_attention_decode(None, None, 2048, None, None, 1, 64, 0, None, None, 0, None,
                                   2048, None, 0) == n5.OK                                 # no sequences
    # n550_qkv_rope_kv(stream, x, ldx, wqkv, qn, kn, rope, seq, pos, M, q, q_type, ldq, kc, vc,
    #                  max_len, layer): a layer past the 28th, ldq below 2048, no rows
    assert L.n550_qkv_rope_kv(None, None, 1024, None, None, None, None, None, None, 4, None, n5.F32,
                              2048, None, None, 64, 28) == n5.ERR_ARG
    assert L.n550_qkv_rope_kv(None, None, 1024, None, None, None, None, None, None, 4, None, n5.F32,
                              1024, None, None, 64, 0) == n5.ERR_ARG
    assert L.n550_qkv_rope_kv(None, None, 1024, None, None, None, None, None, None, 0, None, n5.F32,
                              2048, None, None, 64, 0) == n5.OK
    assert L.n550_rope_table(None, None, -1) == n5.ERR_ARG
    assert L.n550_rope_table(None, None, 0) == n5.OK
    # the failure-path health check: limits outside 1 .. 2e9 cycles launch nothing
    assert L.n550_check_wait_expiry(None, 0) == n5.ERR_ARG
    assert L.n550_check_wait_expiry(None, 2_000_000_001) == n5.ERR_ARG


def test_synth_normal_matches_oracle_generator():
    """The library's seeded BF16 generator (bench.py's GEMM operands) is
    bit-identical to the oracle's, which made the config-1 golden fixture."""
    import numpy as np
    import oracle
    for shape, seed, stream, sigma in [((16, 1024), 0, 0x41, 1.0), ((2048, 1024), 0, 0x42, 0.02),
                                       ((3, 5), 7, 9, 0.5)]:
        assert np.array_equal(n5.synth_normal_bf16(shape, seed, stream, sigma),
                              oracle.synth_normal_bf16(shape, seed, stream, sigma))
