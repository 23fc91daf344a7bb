"""The graph executor's INT8 GEMM on the tensor cores (graph_gemm_tc_kernel:
tcgen05.mma kind::i8, TMA operands, the [k, n] weight read MN-major or the
transB [n, k] weight K-major) against the CPU restatement of
leaf::kernels::gemm_i8_per_channel (kernels/gemm.cpp:99-166) and of the
Gemm / MatMul node (executor.cpp:524-614), bit for bit.  Every shape here
has row strides that are multiples of 16 bytes, which is what routes it to
the tensor cores; ragged m / n / k tails, both tile widths (128 and 256
output columns) and the node glue (C broadcasts, alpha / beta, Relu, Silu, Gelu)
are covered."""
import numpy as np
import pytest
import torch

import leaf_b200 as lq
import oracle
from conftest import bits_equal

pytestmark = pytest.mark.gpu


def _dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


@pytest.mark.parametrize("m,k,n", [(1, 128, 16), (70, 304, 144), (300, 2048, 1024), (129, 1040, 272),
                                   (2048, 256, 2560)])
@pytest.mark.parametrize("with_bias,relu", [(True, True), (False, False)])
def test_gemm_i8_per_channel_tensor_cores(cuda_device, m, k, n, with_bias, relu):
    rng = np.random.default_rng(m * 7 + k + n)
    a = rng.integers(-127, 128, (m, k)).astype(np.int8)
    b = rng.integers(-127, 128, (k, n)).astype(np.int8)
    bias = (rng.standard_normal(n) * 0.1).astype(np.float32) if with_bias else None
    scales = (rng.random(n) * 0.01 + 1e-4).astype(np.float32)
    got = lq.gemm_i8_per_channel(_dev(a), _dev(b), None if bias is None else _dev(bias), 0.0031, _dev(scales),
                                 relu=relu).cpu().numpy()
    expect = oracle.gemm_i8_per_channel(a, b, bias, 0.0031, scales, relu=relu)
    assert bits_equal(got, expect)


def test_gemm_i8_per_channel_extreme_codes(cuda_device):
    # Every product at +-127 * +-127 over the whole k: the int32 sums' extremes.
    m, k, n = 130, 2048, 128
    a = np.full((m, k), 127, dtype=np.int8)
    a[1::2] = -127
    b = np.full((k, n), 127, dtype=np.int8)
    b[:, 1::3] = -127
    scales = np.full(n, 1.0, dtype=np.float32)
    got = lq.gemm_i8_per_channel(_dev(a), _dev(b), None, 1.0, _dev(scales)).cpu().numpy()
    expect = oracle.gemm_i8_per_channel(a, b, None, 1.0, scales, relu=False)
    assert bits_equal(got, expect)
    assert float(got[0, 0]) == 127.0 * 127.0 * k


@pytest.mark.parametrize("trans_a,trans_b", [(0, 0), (1, 0), (0, 1), (1, 1)])
@pytest.mark.parametrize("c_kind,activation", [(None, None), ("row", "Relu"), ("full", "Silu"),
                                               ("scalar", "Gelu")])
def test_gemm_node_tensor_cores(cuda_device, trans_a, trans_b, c_kind, activation):
    rng = np.random.default_rng(hash((trans_a, trans_b, c_kind, activation, "tc")) % 2**32)
    m, k, n = 150, 256, 96
    a = (rng.standard_normal((k, m) if trans_a else (m, k)) * 2).astype(np.float32)
    a[rng.random(a.shape) < 0.01] *= 30
    w = rng.integers(-127, 128, (n, k) if trans_b else (k, n)).astype(np.int8)
    ws = (rng.random(n).astype(np.float32) * 0.02 + 0.001).astype(np.float32)
    c = {None: None, "scalar": np.float32([0.75]), "row": rng.standard_normal(n).astype(np.float32),
         "full": rng.standard_normal((m, n)).astype(np.float32)}[c_kind]
    alpha, beta, scale = 0.9, -1.3, 0.05
    expect = oracle.graph_linear(a, w, ws, scale, "Gemm", trans_a, trans_b, alpha, beta, c, activation)
    got = lq.graph_linear(_dev(a), _dev(w), _dev(ws), scale, "Gemm", bool(trans_a), bool(trans_b), alpha, beta,
                          None if c is None else _dev(c), activation).cpu().numpy()
    assert bits_equal(got, expect)


def test_matmul_node_tensor_cores_batched(cuda_device):
    rng = np.random.default_rng(31)
    a = rng.standard_normal((4, 40, 512)).astype(np.float32)
    w = rng.integers(-127, 128, (512, 384)).astype(np.int8)
    ws = (rng.random(384).astype(np.float32) * 0.01 + 0.001).astype(np.float32)
    expect = oracle.graph_linear(a, w, ws, 0.02, "MatMul")
    got = lq.graph_linear(_dev(a), _dev(w), _dev(ws), 0.02, "MatMul").cpu().numpy()
    assert got.shape == (4, 40, 384)
    assert bits_equal(got, expect)
