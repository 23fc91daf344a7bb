"""The CPU restatement (oracle/) against golden vectors the reference produced.

Runs everywhere (no GPU, no reference tree needed): this is what pins the
oracle on the GPU box.
"""
import numpy as np
import pytest

import oracle
from conftest import bits_equal, golden, linear_cases


def test_act_quant_matches_reference_codes_and_scales():
    g = golden("act_quant")
    q, sx = oracle.quantize_act(g["x"])
    assert np.array_equal(sx.view(np.uint32), g["sx"].view(np.uint32))
    assert np.array_equal(q.astype(np.int16), g["q16"])
    # The VNNI container holds the same code + 128.
    assert np.array_equal(q.astype(np.int16) + 128, g["qu8"].astype(np.int16))
    qr, sxr = oracle.quantize_act(g["x_ragged"])
    assert np.array_equal(qr.astype(np.int16), g["q16_ragged"])
    assert bits_equal(sxr, g["sx_ragged"])


def test_act_quant_edge_rows():
    g = golden("act_quant")
    # all-zero row: scale floor 1e-12, every code 0
    assert g["sx"][2] == np.float32(1e-12) and not g["q16"][2].any()
    # tiny row: floor applies, codes stay within [-127, 127]
    assert g["sx"][3] == np.float32(1e-12)
    assert np.abs(g["q16"]).max() <= 127


@pytest.mark.parametrize("bits,group", [(8, 256), (8, 64), (4, 32), (4, 64)])
def test_weight_codec_matches_exporter(bits, group):
    g = golden("codec")
    payload, scales = oracle.quantize_weight(g["w"], bits, group)
    assert np.array_equal(payload, g[f"payload_{bits}_{group}"])
    assert bits_equal(scales, g[f"scales_{bits}_{group}"])


def test_int4_unpack_roundtrip():
    g = golden("codec")
    payload = g["payload_4_32"]
    codes = oracle.unpack_int4(payload)
    repacked = (codes[:, 0::2].astype(np.uint8) & 15) | ((codes[:, 1::2].astype(np.uint8) & 15) << 4)
    assert np.array_equal(repacked, payload)
    assert codes.min() >= -7 and codes.max() <= 7


@pytest.mark.parametrize("case", linear_cases())
def test_linear_matches_reference(case):
    g = golden(case)
    bits, group = int(g["bits"]), int(g["group"])
    bias = g.get("bias")
    if case.startswith(("w4a32", "w8a32")):
        y = oracle.linear_float(g["x"], g["w"], g["scales"], bits, group, bias)
        assert bits_equal(y, g["y"])
        return
    y, acc = oracle.linear_int(g["x"], g["w"], g["scales"], bits, group, bias, want_acc=True)
    assert bits_equal(y, g["y"])
    q, sx = oracle.quantize_act(g["x"])
    assert np.array_equal(q, g["q"]) and bits_equal(sx, g["sx"])
    # The decoder's own dispatch: VNNI tile (two roundings per group) for
    # several INT8 tokens on an AVX-VNNI CPU, the AVX2 kernels otherwise.
    vnni = g["x"].shape[0] > 1 and bits == 8
    y_dispatch = oracle.linear_int(g["x"], g["w"], g["scales"], bits, group, bias, fused=not vnni)
    assert bits_equal(y_dispatch, g["y_dispatch"])
    # int32 accumulators are exact: recompute from codes in int64.
    codes = g["w"] if bits == 8 else oracle.unpack_int4(g["w"])
    m, k = g["x"].shape
    ref_acc = np.einsum("mgk,ngk->mng", q.reshape(m, k // group, group).astype(np.int64),
                        codes.reshape(-1, k // group, group).astype(np.int64))
    assert np.array_equal(acc, ref_acc)


def test_graph_gemm_matches_reference():
    g = golden("graph_gemm")
    for n in (8, 23, 35, 40):
        a, b = g[f"a_{n}"], g[f"b_{n}"]
        out = oracle.gemm_i8_per_channel(a, b, g[f"bias_{n}"], 0.003, g[f"scales_{n}"], relu=True)
        assert bits_equal(out, g[f"out_relu_{n}"])
        assert bits_equal(out, g[f"out_reference_relu_{n}"])
        out = oracle.gemm_i8_per_channel(a, b, None, 0.003, g[f"scales_{n}"], relu=False)
        assert bits_equal(out, g[f"out_{n}"])


def test_graph_quantize_matches_reference():
    g = golden("graph_quantize")
    q = oracle.graph_quantize(g["x"], g["scale"])
    assert np.array_equal(q, g["q"])
    # half-to-even ties: 0.5 -> 0, 1.5 -> 2, -2.5 -> -2
    assert list(q[:3]) == [0, 2, -2]


def test_graph_quantize_rejects_non_finite():
    with pytest.raises(ValueError):
        oracle.graph_quantize(np.array([1.0, np.nan], dtype=np.float32), 0.1)
    with pytest.raises(ValueError):
        oracle.graph_quantize(np.array([1.0], dtype=np.float32), 0.0)
