"""libleafq.so loads, exports every symbol include/leafq.h declares, and
rejects invalid arguments on the host before touching a device."""
import ctypes

import pytest

from leaf_b200 import _lib


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    declared = _lib.declared_symbols()
    assert declared, "no declarations found in include/leafq.h"
    for name in declared:
        assert hasattr(lib, name), f"{name} declared but not exported"
    assert set(declared) == set(_lib._SIGNATURES)


def test_version_and_error_text():
    lib = _lib.load()
    assert lib.leafq_version() == 100
    assert isinstance(lib.leafq_last_error(), bytes)


def test_workspace_sizes():
    lib = _lib.load()
    # Decode GEMV (per-row INT8, <= 8 tokens) needs no workspace.
    assert lib.leafq_linear_workspace_bytes(1, 2048, 8, 2048, 8) == 0
    assert lib.leafq_linear_workspace_bytes(8, 5632, 8, 5632, 8) == 0
    # Prefill: codes + token scales, each rounded to 256 bytes.
    assert lib.leafq_linear_workspace_bytes(512, 2048, 8, 2048, 8) == 512 * 2048 + 2048
    # Grouped / INT4 always go through codes in the workspace.
    assert lib.leafq_linear_workspace_bytes(1, 256, 4, 32, 8) == 256 + 256
    # Weight-only paths need none.
    assert lib.leafq_linear_workspace_bytes(1, 4096, 4, 32, 32) == 0


@pytest.mark.parametrize("bits,group,abits,cols", [(5, 32, 8, 64), (8, 0, 8, 64), (8, 30, 8, 64),
                                                   (4, 3, 8, 66), (8, 64, 16, 64)])
def test_invalid_descriptors_rejected_on_host(bits, group, abits, cols):
    lib = _lib.load()
    dummy = ctypes.c_void_p(16)
    status = lib.leafq_linear(None, dummy, 1, cols, dummy, dummy, 4, bits, group, abits, None, dummy,
                              None, 0, 0)
    assert status == _lib.LEAFQ_ERR_INVALID
    assert lib.leafq_last_error()


def test_graph_quantize_rejects_bad_scale_on_host():
    lib = _lib.load()
    dummy = ctypes.c_void_p(16)
    for scale in (0.0, -1.0, float("inf"), float("nan")):
        assert lib.leafq_graph_quantize(None, dummy, 4, scale, dummy, None) == _lib.LEAFQ_ERR_INVALID


def test_gemm_rejects_bad_activation_and_huge_k():
    lib = _lib.load()
    dummy = ctypes.c_void_p(16)
    assert lib.leafq_gemm_i8_per_channel(None, dummy, dummy, None, 1.0, dummy, dummy, 2, 4, 4, 2) \
        == _lib.LEAFQ_ERR_INVALID
    assert lib.leafq_gemm_i8_per_channel(None, dummy, dummy, None, 1.0, dummy, dummy, 2, 200000, 4, 0) \
        == _lib.LEAFQ_ERR_UNSUPPORTED


def test_zero_sized_calls_are_no_ops():
    lib = _lib.load()
    assert lib.leafq_linear(None, None, 0, 64, None, None, 8, 8, 64, 8, None, None, None, 0, 0) == 0
    assert lib.leafq_quantize_act(None, None, 0, 64, None, None) == 0


def test_decoder_ops_reject_bad_shapes_on_host():
    lib = _lib.load()
    d = ctypes.c_void_p(16)
    assert lib.leafq_rmsnorm(None, d, None, 0, 2, 0, d, 1e-5, d) == _lib.LEAFQ_ERR_INVALID
    assert lib.leafq_rmsnorm(None, d, None, 0, 2, 20000, d, 1e-5, d) == _lib.LEAFQ_ERR_INVALID
    assert lib.leafq_rotary_append(None, d, 1, 6, 4, 64, 64, d, d, d, d, d, d, 8) == _lib.LEAFQ_ERR_INVALID
    assert lib.leafq_rotary_append(None, d, 1, 8, 2, 64, 65, d, d, d, d, d, d, 8) == _lib.LEAFQ_ERR_INVALID
    assert lib.leafq_attention(None, d, d, d, 1, 8, 3, 64, d, 8, 0.5, d) == _lib.LEAFQ_ERR_INVALID
    assert lib.leafq_attention(None, d, d, d, 1, 8, 2, 64, d, 8, 0.0, d) == _lib.LEAFQ_ERR_INVALID
    assert lib.leafq_silu_gate(None, d, 1, 0, d) == _lib.LEAFQ_ERR_INVALID
    assert lib.leafq_argmax(None, d, 1, 0, d) == _lib.LEAFQ_ERR_INVALID
    assert lib.leafq_embed(None, d, 1, d, None, 8, 64, 10, 64, 1.0, d, None) == _lib.LEAFQ_ERR_INVALID
    assert lib.leafq_advance_position(None, None, 1) == _lib.LEAFQ_ERR_INVALID
    # Zero tokens are no-ops.
    assert lib.leafq_silu_gate(None, None, 0, 8, None) == 0
    assert lib.leafq_attention(None, None, None, None, 0, 8, 2, 64, None, 8, 0.5, None) == 0


def test_rope_tables_match_libm_on_host():
    import numpy as np

    from oracle.decoder import rope_tables

    lib = _lib.load()
    cos = np.empty((40, 32), np.float32)
    sin = np.empty_like(cos)
    assert lib.leafq_rope_tables(ctypes.c_float(10000.0), 64, 40, cos.ctypes.data, sin.ctypes.data) == 0
    c, s = rope_tables(10000.0, 64, 40)
    assert np.array_equal(cos.view(np.uint32), c.view(np.uint32))
    assert np.array_equal(sin.view(np.uint32), s.view(np.uint32))


def test_plans_reject_bad_arguments_on_host():
    lib = _lib.load()
    out = ctypes.c_void_p()
    handle = (ctypes.c_uint8 * _lib.LEAFQ_IPC_HANDLE_BYTES)()
    assert lib.leafq_allgather_init(0, 9, 16, ctypes.byref(out), handle) == _lib.LEAFQ_ERR_INVALID
    assert lib.leafq_allgather_init(2, 2, 16, ctypes.byref(out), handle) == _lib.LEAFQ_ERR_INVALID
    assert lib.leafq_allgather_run(None, None, None, 1, 1, 0, 1, None) == _lib.LEAFQ_ERR_INVALID
    assert lib.leafq_model_plan_create(None, ctypes.byref(out)) == _lib.LEAFQ_ERR_INVALID
    desc = _lib.ModelDesc()
    desc.layers = 1
    desc.layer = ctypes.c_void_p(16)
    desc.hidden, desc.intermediate, desc.heads, desc.kv_heads = 100, 256, 4, 2  # hidden % 16 != 0
    desc.head_dim, desc.vocab, desc.capacity, desc.attn_scale = 25, 10, 8, 0.5
    assert lib.leafq_model_plan_create(ctypes.byref(desc), ctypes.byref(out)) == _lib.LEAFQ_ERR_UNSUPPORTED
    assert lib.leafq_model_plan_run(None, None) == _lib.LEAFQ_ERR_INVALID
    assert lib.leafq_model_plan_destroy(None) == 0
