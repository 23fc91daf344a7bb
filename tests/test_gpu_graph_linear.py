"""The graph executor's quantised Gemm / MatMul node (execute_quant_linear,
executor.cpp:524-614) through leafq_graph_linear against the CPU
restatement (whose quantiser and per-channel GEMM are pinned to the
reference's own kernels in tests/test_oracle.py), bit for bit: transA /
transB, every C broadcast, alpha / beta, the fused activations, batched
MatMul inputs, and the reference's rejections."""
import numpy as np
import pytest
import torch

import leaf_b200 as lq
import oracle
from leaf_b200._lib import LeafError

pytestmark = pytest.mark.gpu


def _case(rng, m, k, n, trans_a, trans_b):
    a = (rng.standard_normal((k, m) if trans_a else (m, k)) * 2).astype(np.float32)
    a[rng.random(a.shape) < 0.01] *= 30  # some codes saturate
    w = rng.integers(-127, 128, (n, k) if trans_b else (k, n)).astype(np.int8)
    ws = (rng.random(n).astype(np.float32) * 0.02 + 0.001).astype(np.float32)
    return a, w, ws


@pytest.mark.parametrize("trans_a,trans_b", [(0, 0), (1, 0), (0, 1), (1, 1)])
@pytest.mark.parametrize("c_kind", [None, "scalar", "row", "full"])
@pytest.mark.parametrize("activation", [None, "Relu", "Silu", "Gelu"])
def test_gemm_node_bit_exact(cuda_device, trans_a, trans_b, c_kind, activation):
    rng = np.random.default_rng(hash((trans_a, trans_b, c_kind, activation)) % 2**32)
    m, k, n = 37, 200, 70
    a, w, ws = _case(rng, m, k, n, trans_a, trans_b)
    c = {None: None, "scalar": np.float32([0.75]), "row": rng.standard_normal(n).astype(np.float32),
         "full": rng.standard_normal((m, n)).astype(np.float32)}[c_kind]
    alpha, beta, scale = 0.9, -1.3, 0.05
    expect = oracle.graph_linear(a, w, ws, scale, "Gemm", trans_a, trans_b, alpha, beta, c, activation)
    got = lq.graph_linear(torch.from_numpy(a).cuda(), torch.from_numpy(w).cuda(), torch.from_numpy(ws).cuda(),
                          scale, "Gemm", bool(trans_a), bool(trans_b), alpha, beta,
                          None if c is None else torch.from_numpy(c).cuda(), activation).cpu().numpy()
    assert got.shape == expect.shape
    assert np.array_equal(got.view(np.uint32), expect.view(np.uint32))


def test_matmul_node_batched(cuda_device):
    rng = np.random.default_rng(3)
    a = rng.standard_normal((3, 5, 96)).astype(np.float32)
    w = rng.integers(-127, 128, (96, 130)).astype(np.int8)
    ws = (rng.random(130).astype(np.float32) * 0.01 + 0.001).astype(np.float32)
    expect = oracle.graph_linear(a, w, ws, 0.02, "MatMul")
    got = lq.graph_linear(torch.from_numpy(a).cuda(), torch.from_numpy(w).cuda(), torch.from_numpy(ws).cuda(),
                          0.02, "MatMul").cpu().numpy()
    assert got.shape == (3, 5, 130)
    assert np.array_equal(got.view(np.uint32), expect.view(np.uint32))


def test_graph_linear_rejections(cuda_device):
    rng = np.random.default_rng(4)
    a, w, ws = _case(rng, 4, 32, 8, 0, 0)
    A, W, WS = (torch.from_numpy(t).cuda() for t in (a, w, ws))
    with pytest.raises(LeafError, match="broadcast"):
        lq.graph_linear(A, W, WS, 0.1, c=torch.zeros(3, device="cuda"))
    with pytest.raises(LeafError, match="activation scale"):
        lq.graph_linear(A, W, WS, 0.0)
    with pytest.raises(LeafError, match="unsupported fused activation"):
        lq.graph_linear(A, W, WS, 0.1, activation="Tanh")
    bad = A.clone()
    bad[1, 3] = float("nan")
    with pytest.raises(LeafError, match="non-finite"):
        lq.graph_linear(bad, W, WS, 0.1)
    with pytest.raises(LeafError, match="transA"):
        lq.graph_linear(A.reshape(2, 2, 32), W, WS, 0.1, trans_a=True)


@pytest.mark.parametrize("k,n", [(100, 4141), (256, 4144)])  # CUDA cores (rows not 16-byte) and tensor cores
def test_gelu_over_sixty_binades(cuda_device, k, n):
    # Weight scales log-uniform over 1e-30 .. 1e3 put the Gelu's tanhf argument
    # in every branch of the algorithm (tiny, |x| < 1, |x| >= 1, saturated)
    # with both signs; the last columns overflow to +-inf before the
    # activation: Gelu(+inf) = +inf, Gelu(-inf) = -inf * 0 = NaN.  Bits are
    # compared everywhere except the NaNs' payloads (the x86 default NaN and
    # the GPU's canonical NaN differ in sign and payload, not in being NaN).
    rng = np.random.default_rng(k)
    m = 300
    a = (rng.standard_normal((m, k)) * 2).astype(np.float32)
    w = rng.integers(-127, 128, (k, n)).astype(np.int8)
    ws = np.exp(rng.uniform(np.log(1e-30), np.log(1e3), n)).astype(np.float32)
    ws[-8:] = np.float32(3e38)
    expect = oracle.graph_linear(a, w, ws, 0.05, "MatMul", activation="Gelu")
    got = lq.graph_linear(torch.from_numpy(a).cuda(), torch.from_numpy(w).cuda(), torch.from_numpy(ws).cuda(),
                          0.05, "MatMul", activation="Gelu").cpu().numpy()
    nan = np.isnan(expect)
    assert nan.any() and np.isinf(expect).any()
    assert np.array_equal(np.isnan(got), nan)
    assert np.array_equal(got[~nan].view(np.uint32), expect[~nan].view(np.uint32))
