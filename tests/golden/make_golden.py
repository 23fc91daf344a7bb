"""Generate the golden vectors in this directory from the reference itself.

Run in a checkout where the reference tree is available (LEAF_REFERENCE, or a
``reference`` directory beside this repository) and the reference kernels are
built (oracle.build(ref=True)):

    python tests/golden/make_golden.py

Weights are quantised by the reference's own exporter function
(tools/export_decoder.py:91-105, imported from the reference tree) and every
output comes from the reference's compiled CPU kernels (oracle/_ref,
compiled unmodified from engine/src/decoder.cpp, kernels/gemm.cpp and
executor.cpp).  Inputs are seeded numpy draws with the BASELINE shapes' value
distributions (x ~ N(0, 1) with a few x20 outliers, W ~ N(0, 0.02),
bias ~ N(0, 0.01)), cut down to sizes that keep each file small.
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO))
import oracle as _oracle  # noqa: E402

REF = _oracle.reference_root() or Path(os.environ.get("LEAF_REFERENCE", "reference"))
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(REF))

import oracle  # noqa: E402
from tools.export_decoder import quantize as reference_quantize  # noqa: E402


def activations(rng, m, k, outliers=True):
    x = rng.standard_normal((m, k)).astype(np.float32)
    if outliers:
        mask = rng.random((m, k)) < 0.01
        x[mask] *= 20
    return x


def linear_case(rng, name, m, k, n, bits, group, float_act=False, bias=True):
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    payload, scales = reference_quantize(w, bits, group)
    x = activations(rng, m, k, outliers=not float_act)
    b = (rng.standard_normal(n) * 0.01).astype(np.float32) if bias else None
    case = dict(x=x, w=payload, scales=scales, bits=np.int32(bits), group=np.int32(group))
    if b is not None:
        case["bias"] = b
    if float_act:
        case["y"] = oracle.ref_linear_float(x, payload, scales, bits, group, b, mode=0)
    else:
        # mode 1: the AVX2 kernels (decode and INT4 dispatch, fused groups);
        # mode 0: the decoder's own dispatch on an AVX-VNNI CPU (VNNI tile
        # for tokens > 1 and INT8 weights).
        case["y"] = oracle.ref_linear_int(x, payload, scales, bits, group, b, mode=1)
        case["y_dispatch"] = oracle.ref_linear_int(x, payload, scales, bits, group, b, mode=0)
        q16, sx = oracle.ref_quantize_i16(x)
        case["q"] = q16.astype(np.int8)
        case["sx"] = sx
    np.savez_compressed(HERE / f"{name}.npz", **case)


def main():
    if not oracle.ref_available():
        raise SystemExit("build the reference kernels first: make -C oracle ref")
    assert oracle.ref().leafref_has_vnni() == 1, "golden dispatch outputs assume an AVX-VNNI CPU"
    rng = np.random.default_rng(20241201)

    # Activation quantiser: normal rows, outliers, an all-zero row, a row of
    # tiny values (scale floor 1e-12), ragged widths (AVX tail).
    x = activations(rng, 6, 2048)
    x[2] = 0.0
    x[3] = (rng.standard_normal(2048) * 1e-14).astype(np.float32)
    x[4, 5] = 1e4
    q16, sx = oracle.ref_quantize_i16(x)
    qu8, sx8 = oracle.ref_quantize_u8(x)
    assert np.array_equal(sx, sx8)
    xr = activations(rng, 3, 37)
    qr16, sxr = oracle.ref_quantize_i16(xr)
    np.savez_compressed(HERE / "act_quant.npz", x=x, q16=q16, qu8=qu8, sx=sx, x_ragged=xr,
                        q16_ragged=qr16, sx_ragged=sxr)

    # Weight codec.
    w = (rng.standard_normal((24, 256)) * 0.02).astype(np.float32)
    codec = {"w": w}
    for bits, group in ((8, 256), (8, 64), (4, 32), (4, 64)):
        payload, scales = reference_quantize(w, bits, group)
        codec[f"payload_{bits}_{group}"] = payload
        codec[f"scales_{bits}_{group}"] = scales
    np.savez_compressed(HERE / "codec.npz", **codec)

    # W8A8 per-row (config-0 row width), decode and prefill-tile token counts.
    linear_case(rng, "w8a8_row_m1", 1, 2048, 40, 8, 2048)
    linear_case(rng, "w8a8_row_m5", 5, 2048, 37, 8, 2048)
    linear_case(rng, "w8a8_row_m13_nobias", 13, 512, 33, 8, 512, bias=False)
    # Grouped INT8 (int8_group_size) and W4A8.
    linear_case(rng, "w8a8_g64_m1", 1, 256, 24, 8, 64)
    linear_case(rng, "w8a8_g64_m3", 3, 256, 24, 8, 64)
    linear_case(rng, "w4a8_g32_m1", 1, 256, 20, 4, 32)
    linear_case(rng, "w4a8_g32_m6", 6, 256, 20, 4, 32)
    # Weight-only fp32-activation paths (config-1 row width for INT4 g32).
    linear_case(rng, "w4a32_g32_m1", 1, 4096, 16, 4, 32, float_act=True)
    linear_case(rng, "w4a32_g64_m6", 6, 512, 12, 4, 64, float_act=True)
    linear_case(rng, "w4a32_g48_m1", 1, 480, 9, 4, 48, float_act=True)
    linear_case(rng, "w8a32_g36_m2", 2, 360, 7, 8, 36, float_act=True)
    linear_case(rng, "w8a32_row_m1", 1, 2048, 8, 8, 2048, float_act=True)

    # Graph executor INT8 GEMM: the shapes and value recipe of
    # tests/native/test_kernels.cpp:43-66 (m=4, k=31, n in {8,23,35,40},
    # codes in [-127, 127], bias i*0.01, scales 0.002 + i*1e-5, s_in 0.003),
    # drawn with numpy instead of mt19937.
    gemm = {}
    for n in (8, 23, 35, 40):
        a = rng.integers(-127, 128, (4, 31)).astype(np.int8)
        b = rng.integers(-127, 128, (31, n)).astype(np.int8)
        bias = (np.arange(n, dtype=np.float32) * np.float32(0.01)).astype(np.float32)
        scales = (np.float32(0.002) + np.arange(n, dtype=np.float32) * np.float32(0.00001)).astype(np.float32)
        gemm[f"a_{n}"], gemm[f"b_{n}"] = a, b
        gemm[f"bias_{n}"], gemm[f"scales_{n}"] = bias, scales
        gemm[f"out_relu_{n}"] = oracle.ref_gemm_i8_per_channel(a, b, bias, 0.003, scales, relu=True)
        gemm[f"out_{n}"] = oracle.ref_gemm_i8_per_channel(a, b, None, 0.003, scales, relu=False)
        gemm[f"out_reference_relu_{n}"] = oracle.ref_gemm_i8_per_channel(
            a, b, bias, 0.003, scales, relu=True, reference=True)
    np.savez_compressed(HERE / "graph_gemm.npz", **gemm)

    # Graph executor static quantiser, including exact .5 ties.
    scale = np.float32(0.01)
    xq = (rng.standard_normal(4096) * 0.5).astype(np.float32)
    xq[:6] = np.array([0.005, 0.015, -0.025, 2.0, -2.0, 0.0], dtype=np.float32)
    np.savez_compressed(HERE / "graph_quantize.npz", x=xq, scale=scale,
                        q=oracle.ref_graph_quantize(xq, scale))
    print("golden vectors written to", HERE)


if __name__ == "__main__":
    main()
