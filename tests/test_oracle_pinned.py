"""The CPU restatement against the reference's own compiled kernels on fresh
seeded cases (where oracle/_ref was built: this container, and the GPU box
when the built library travels with the snapshot)."""
import numpy as np
import pytest

import oracle
from conftest import bits_equal

pytestmark = pytest.mark.skipif(not oracle.ref_available(), reason="reference kernels not built")


def _weight(rng, n, k, bits, group):
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    return oracle.quantize_weight(w, bits, group)


@pytest.mark.parametrize("m", [1, 2, 3, 5, 8])
@pytest.mark.parametrize("bits,group,k,n", [(8, 2048, 2048, 67), (8, 64, 256, 40), (4, 32, 256, 41),
                                            (4, 128, 512, 9), (8, 100, 300, 10), (4, 30, 90, 7)])
def test_integer_linear_all_dispatch_modes(m, bits, group, k, n):
    rng = np.random.default_rng(1000 * m + k + n)
    payload, scales = _weight(rng, n, k, bits, group)
    x = rng.standard_normal((m, k)).astype(np.float32)
    bias = (rng.standard_normal(n) * 0.01).astype(np.float32)
    fused = oracle.linear_int(x, payload, scales, bits, group, bias, fused=True)
    unfused = oracle.linear_int(x, payload, scales, bits, group, bias, fused=False)
    for threads in (1, 3):
        assert bits_equal(fused, oracle.ref_linear_int(x, payload, scales, bits, group, bias, threads, mode=1))
        vnni = m > 1 and bits == 8
        assert bits_equal(unfused if vnni else fused,
                          oracle.ref_linear_int(x, payload, scales, bits, group, bias, threads, mode=0))
    if group == k:  # one group per row: every reference path agrees
        assert bits_equal(fused, unfused)


@pytest.mark.parametrize("m", [1, 2, 4, 5, 6])
@pytest.mark.parametrize("bits,group,k,n", [(4, 32, 4096, 9), (4, 64, 512, 5), (8, 2048, 2048, 7),
                                            (4, 48, 480, 5), (8, 36, 360, 3), (32, 0, 264, 4),
                                            (4, 10, 100, 3)])
def test_float_activation_linear(m, bits, group, k, n):
    rng = np.random.default_rng(7 * m + k + n)
    if bits == 32:
        payload = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
        scales = None
    else:
        payload, scales = _weight(rng, n, k, bits, group)
    x = rng.standard_normal((m, k)).astype(np.float32)
    bias = (rng.standard_normal(n) * 0.01).astype(np.float32)
    y = oracle.linear_float(x, payload, scales, bits, group, bias)
    assert bits_equal(y, oracle.ref_linear_float(x, payload, scales, bits, group, bias, threads=2))


def test_quantizer_containers():
    rng = np.random.default_rng(3)
    x = rng.standard_normal((7, 1000)).astype(np.float32) * 3
    q, sx = oracle.quantize_act(x)
    q16, sx16 = oracle.ref_quantize_i16(x)
    q8, sx8 = oracle.ref_quantize_u8(x)
    assert np.array_equal(q.astype(np.int16), q16)
    assert np.array_equal(q.astype(np.int16) + 128, q8.astype(np.int16))
    assert bits_equal(sx, sx16) and bits_equal(sx, sx8)


def test_graph_paths():
    rng = np.random.default_rng(5)
    a = rng.integers(-127, 128, (9, 70)).astype(np.int8)
    b = rng.integers(-127, 128, (70, 33)).astype(np.int8)
    bias = (rng.standard_normal(33) * 0.1).astype(np.float32)
    scales = (rng.random(33) * 0.01).astype(np.float32)
    for relu in (False, True):
        for bb in (None, bias):
            assert bits_equal(oracle.gemm_i8_per_channel(a, b, bb, 0.0031, scales, relu),
                              oracle.ref_gemm_i8_per_channel(a, b, bb, 0.0031, scales, relu))
    x = (rng.standard_normal(5000) * 2).astype(np.float32)
    assert np.array_equal(oracle.graph_quantize(x, 0.013), oracle.ref_graph_quantize(x, 0.013))


def test_graph_activations():
    # apply_activation (executor.cpp:232-242) of the reference against the
    # restatement, over values spanning every float binade, both signs, zeros
    # and infinities; NaN results compared by position.
    rng = np.random.default_rng(11)
    bits = rng.integers(0, 2**32, 400000, dtype=np.uint64).astype(np.uint32)
    x = bits.view(np.float32)
    x = np.concatenate([x[np.isfinite(x)], (rng.standard_normal(100000) * 4).astype(np.float32),
                        np.float32([0.0, -0.0, np.inf, -np.inf, 1e-40, -1e-40, 9.0, -9.0, 22.0, -22.0])])
    for activation in (None, "Relu", "Silu", "Gelu"):
        got, ref = oracle.graph_activation(x, activation), oracle.ref_graph_activation(x, activation)
        nan = np.isnan(ref)
        assert np.array_equal(np.isnan(got), nan), activation
        assert np.array_equal(got[~nan].view(np.uint32), ref[~nan].view(np.uint32)), activation
    with pytest.raises(ValueError, match="unsupported fused activation"):
        oracle.ref_graph_activation(x[:4], "Tanh")
