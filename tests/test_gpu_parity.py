"""CUDA path (libleafq.so through the C ABI) against the reference.

Golden-size cases compare with vectors the reference's own kernels produced;
BASELINE-size cases compare with the pinned CPU restatement (oracle/) on the
same seeded inputs, all rows where the oracle is fast and a seeded sample of
weight rows (rows are independent) where it is not.  The bar is bit-exact
everywhere: int8 codes, int32 accumulators and fp32 outputs.
"""
import numpy as np
import pytest
import torch

import leaf_b200 as lq
import oracle
from conftest import bits_equal, golden, linear_cases

pytestmark = pytest.mark.gpu


def dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None and t.dtype != dtype:
        t = t.view(dtype) if t.element_size() == torch.empty(0, dtype=dtype).element_size() else t.to(dtype)
    return t.cuda()


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def weight_of(g):
    bits, group = int(g["bits"]), int(g["group"])
    rows = g["scales"].shape[0]
    cols = g["x"].shape[1]
    return lq.QuantWeight.from_host(g["w"], g["scales"], rows, cols, bits, group, g.get("bias"))


def make_weight(rng, n, k, bits, group):
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    payload, scales = oracle.quantize_weight(w, bits, group)
    return payload, scales


def activations(rng, m, k, outliers=True):
    x = rng.standard_normal((m, k)).astype(np.float32)
    if outliers:
        x[rng.random((m, k)) < 0.01] *= 20
    return x


# ---------------------------------------------------------------- golden
def test_act_quant_golden(cuda_device):
    g = golden("act_quant")
    q, sx = lq.quantize_act(dev(g["x"]))
    assert np.array_equal(host(q).astype(np.int16), g["q16"])
    assert bits_equal(host(sx), g["sx"])
    q, sx = lq.quantize_act(dev(g["x_ragged"]))
    assert np.array_equal(host(q).astype(np.int16), g["q16_ragged"])
    assert bits_equal(host(sx), g["sx_ragged"])


@pytest.mark.parametrize("case", linear_cases())
def test_linear_golden(cuda_device, case):
    g = golden(case)
    w = weight_of(g)
    abits = 32 if case.startswith(("w4a32", "w8a32")) else 8
    y = lq.linear(dev(g["x"]), w, activation_bits=abits)
    assert bits_equal(host(y), g["y"]), f"{case}: max |diff| {np.abs(host(y) - g['y']).max()}"
    if abits == 8:
        # The decoder's own dispatch on this CPU (VNNI tile for several INT8
        # tokens) is reproduced with the VNNI rounding flag.
        vnni = g["x"].shape[0] > 1 and int(g["bits"]) == 8
        flags = lq.LEAFQ_FLAG_VNNI_ROUNDING if vnni else 0
        y = lq.linear(dev(g["x"]), w, activation_bits=8, flags=flags)
        assert bits_equal(host(y), g["y_dispatch"])
        # Accumulators through the codes entry point.
        yq, acc = lq.linear_int_q(dev(g["q"]), dev(g["sx"]), w, want_acc=True)
        assert bits_equal(host(yq), g["y"])
        _, ref_acc = oracle.linear_int_q(g["q"], g["sx"], g["w"], g["scales"], int(g["bits"]),
                                         int(g["group"]), g.get("bias"), want_acc=True)
        assert np.array_equal(host(acc), ref_acc)


def test_graph_gemm_golden(cuda_device):
    g = golden("graph_gemm")
    for n in (8, 23, 35, 40):
        a, b = dev(g[f"a_{n}"]), dev(g[f"b_{n}"])
        out = lq.gemm_i8_per_channel(a, b, dev(g[f"bias_{n}"]), 0.003, dev(g[f"scales_{n}"]), relu=True)
        assert bits_equal(host(out), g[f"out_relu_{n}"])
        out = lq.gemm_i8_per_channel(a, b, None, 0.003, dev(g[f"scales_{n}"]), relu=False)
        assert bits_equal(host(out), g[f"out_{n}"])


def test_graph_quantize_golden(cuda_device):
    g = golden("graph_quantize")
    assert np.array_equal(host(lq.graph_quantize(dev(g["x"]), float(g["scale"]))), g["q"])
    bad = dev(np.array([1.0, np.inf, 2.0], dtype=np.float32))
    with pytest.raises(lq.LeafError):
        lq.graph_quantize(bad, 0.1)


# ------------------------------------------------------- BASELINE sizes
@pytest.mark.parametrize("m", [1, 2, 3, 4, 5, 8])
def test_w8a8_decode_gemv_config0(cuda_device, m):
    """Config 0: M=1, K=2048, N=5632 (and small decode batches)."""
    rng = np.random.default_rng(100 + m)
    payload, scales = make_weight(rng, 5632, 2048, 8, 2048)
    x = activations(rng, m, 2048)
    bias = (rng.standard_normal(5632) * 0.01).astype(np.float32)
    w = lq.QuantWeight.from_host(payload, scales, 5632, 2048, 8, 2048, bias)
    y = host(lq.linear(dev(x), w))
    assert bits_equal(y, oracle.linear_int(x, payload, scales, 8, 2048, bias))


@pytest.mark.parametrize("k,n", [(5632, 2048), (2048, 2560), (2048, 32000), (48, 7), (4112, 33)])
def test_w8a8_decode_gemv_shapes(cuda_device, k, n):
    """down_proj, fused qkv, lm_head rows and ragged chunking (K > 4096)."""
    rng = np.random.default_rng(k + n)
    payload, scales = make_weight(rng, n, k, 8, k)
    x = activations(rng, 1, k)
    w = lq.QuantWeight.from_host(payload, scales, n, k, 8, k, None)
    y = host(lq.linear(dev(x), w))
    assert bits_equal(y, oracle.linear_int(x, payload, scales, 8, k, None))


def test_w4a32_gemv_config1(cuda_device):
    """Config 1: INT4 weight-only, K=4096, N=11008, groups of 32."""
    rng = np.random.default_rng(11)
    payload, scales = make_weight(rng, 11008, 4096, 4, 32)
    x = activations(rng, 1, 4096, outliers=False)
    w = lq.QuantWeight.from_host(payload, scales, 11008, 4096, 4, 32)
    y = host(lq.linear(dev(x), w, activation_bits=32))
    assert bits_equal(y, oracle.linear_float(x, payload, scales, 4, 32, None))


@pytest.mark.parametrize("m,k,n,group", [(1, 4096, 300, 64), (1, 4096, 300, 128), (3, 512, 40, 32),
                                         (5, 1024, 17, 64)])
def test_w4a32_other_groups_and_tokens(cuda_device, m, k, n, group):
    rng = np.random.default_rng(m * k + n + group)
    payload, scales = make_weight(rng, n, k, 4, group)
    x = activations(rng, m, k, outliers=False)
    bias = (rng.standard_normal(n) * 0.01).astype(np.float32)
    w = lq.QuantWeight.from_host(payload, scales, n, k, 4, group, bias)
    y = host(lq.linear(dev(x), w, activation_bits=32))
    assert bits_equal(y, oracle.linear_float(x, payload, scales, 4, group, bias))


@pytest.mark.parametrize("k,n", [(2048, 5632), (8192, 300), (128, 1000), (4096, 33), (1024, 16 * 148 + 5)])
def test_w4a32_group32_widths(cuda_device, k, n):
    """The 32-column kernel over 4..256 groups per row (so 128..2 row slots
    per stage), ragged row counts, every nibble value, a bias, and x with
    exact zeros, subnormals, tiny and large values."""
    rng = np.random.default_rng(k * 7 + n)
    payload = rng.integers(0, 256, size=(n, k // 2), dtype=np.uint8)
    scales = (rng.random((n, k // 32)) * 1e-2 + 1e-4).astype(np.float32)
    scales[0, 0] = 3e4
    x = activations(rng, 1, k)
    x[0, ::17] = 0.0
    x[0, 5::97] = np.float32(1.5e-42)
    x[0, 7::89] = np.float32(-3e-39)
    x[0, 9::61] *= np.float32(1e25)
    bias = (rng.standard_normal(n) * 0.01).astype(np.float32)
    w = lq.QuantWeight.from_host(payload, scales, n, k, 4, 32, bias)
    y = host(lq.linear(dev(x), w, activation_bits=32))
    assert bits_equal(y, oracle.linear_float(x, payload, scales, 4, 32, bias))


@pytest.mark.parametrize("n", [5632, 2048])
def test_w8a8_prefill_gemm_config2(cuda_device, n):
    """Config 2: M=512, K=2048, N in {5632, 2048}, 1% x20 outliers; the
    oracle checks a seeded sample of 192 weight rows for all 512 tokens."""
    rng = np.random.default_rng(200 + n)
    payload, scales = make_weight(rng, n, 2048, 8, 2048)
    x = activations(rng, 512, 2048)
    bias = (rng.standard_normal(n) * 0.01).astype(np.float32)
    w = lq.QuantWeight.from_host(payload, scales, n, 2048, 8, 2048, bias)
    y = host(lq.linear(dev(x), w))
    rows = np.sort(rng.choice(n, 192, replace=False))
    expect = oracle.linear_int(x, payload[rows], scales[rows], 8, 2048, bias[rows])
    assert bits_equal(y[:, rows], expect)


def test_w8a8_prefill_gemm_down_proj(cuda_device):
    rng = np.random.default_rng(31)
    payload, scales = make_weight(rng, 2048, 5632, 8, 5632)
    x = activations(rng, 512, 5632)
    w = lq.QuantWeight.from_host(payload, scales, 2048, 5632, 8, 5632)
    y = host(lq.linear(dev(x), w))
    rows = np.sort(rng.choice(2048, 96, replace=False))
    assert bits_equal(y[:, rows], oracle.linear_int(x, payload[rows], scales[rows], 8, 5632, None))


@pytest.mark.parametrize("m,k,n", [(9, 1040, 300), (200, 2064, 257), (129, 128, 513), (640, 512, 256),
                                   (16, 256, 9500), (64, 2048, 2560), (64, 512, 20000), (40, 256, 38000),
                                   (12, 512, 1001), (33, 528, 4098), (17, 4096, 5000)])
def test_w8a8_prefill_gemm_ragged(cuda_device, m, k, n):
    """Tiles cut by M, N and K edges (K a multiple of 16 but not of 128), and
    every tile width (on 148 SMs: 32, 64, 128 and 256 rows per tile), with
    the thin code tiles of launches of at most 64 tokens."""
    rng = np.random.default_rng(m + k + n)
    payload, scales = make_weight(rng, n, k, 8, k)
    x = activations(rng, m, k)
    bias = (rng.standard_normal(n) * 0.01).astype(np.float32)
    w = lq.QuantWeight.from_host(payload, scales, n, k, 8, k, bias)
    y = host(lq.linear(dev(x), w))
    assert bits_equal(y, oracle.linear_int(x, payload, scales, 8, k, bias))


@pytest.mark.parametrize("m", [256, 64, 47, 9])
def test_tensor_core_accumulators_exact(cuda_device, m):
    """With unit scales and no bias the epilogue returns float(acc) exactly
    (|acc| < 2^24), so the tcgen05 int32 accumulators are checked directly:
    128-row MMAs, and the 64-row MMAs of launches of at most 64 tokens (every
    accumulator row of each TMEM sub-partition's 16 lanes)."""
    rng = np.random.default_rng(5 + m)
    k, n = 2048, 512
    q = rng.integers(-127, 128, (m, k)).astype(np.int8)
    w = rng.integers(-127, 128, (n, k)).astype(np.int8)
    ones_t = np.ones(m, dtype=np.float32)
    ones_w = np.ones((n, 1), dtype=np.float32)
    qw = lq.QuantWeight.from_host(w, ones_w, n, k, 8, k)
    y = host(lq.linear_int_q(dev(q), dev(ones_t), qw))
    acc = q.astype(np.int64) @ w.astype(np.int64).T
    assert np.abs(acc).max() < 2 ** 24
    assert np.array_equal(y.astype(np.int64), acc)


@pytest.mark.parametrize("m", [1, 4, 40])
@pytest.mark.parametrize("bits,group", [(8, 64), (4, 32), (4, 128), (8, 128)])
def test_grouped_integer_paths(cuda_device, m, bits, group):
    rng = np.random.default_rng(m + bits + group)
    k, n = 1024, 96
    payload, scales = make_weight(rng, n, k, bits, group)
    x = activations(rng, m, k)
    bias = (rng.standard_normal(n) * 0.01).astype(np.float32)
    w = lq.QuantWeight.from_host(payload, scales, n, k, bits, group, bias)
    y = host(lq.linear(dev(x), w))
    assert bits_equal(y, oracle.linear_int(x, payload, scales, bits, group, bias, fused=True))
    y = host(lq.linear(dev(x), w, flags=lq.LEAFQ_FLAG_VNNI_ROUNDING))
    assert bits_equal(y, oracle.linear_int(x, payload, scales, bits, group, bias, fused=False))


def test_act_quant_large_and_odd(cuda_device):
    rng = np.random.default_rng(9)
    # At least as many rows as SMs, with at most 2048 aligned floats each: the
    # warp-per-row kernel (every register width: 64, 200, 500, 1000, 2044, 2048
    # columns); fewer rows, or other widths: the block-per-row kernel.
    for m, k in ((512, 2048), (3, 5632), (2, 1), (5, 33), (4096, 2048), (100, 64), (70, 1000), (9, 2044),
                 (33, 2052), (160, 64), (150, 200), (149, 500), (200, 1000), (150, 2044), (147, 2048)):
        x = activations(rng, m, k)
        q, sx = lq.quantize_act(dev(x))
        eq, esx = oracle.quantize_act(x)
        assert np.array_equal(host(q), eq) and bits_equal(host(sx), esx)


def test_graph_gemm_random(cuda_device):
    rng = np.random.default_rng(13)
    a = rng.integers(-127, 128, (70, 300)).astype(np.int8)
    b = rng.integers(-127, 128, (300, 130)).astype(np.int8)
    bias = (rng.standard_normal(130) * 0.1).astype(np.float32)
    scales = (rng.random(130) * 0.01).astype(np.float32)
    out = lq.gemm_i8_per_channel(dev(a), dev(b), dev(bias), 0.0031, dev(scales), relu=True)
    assert bits_equal(host(out), oracle.gemm_i8_per_channel(a, b, bias, 0.0031, scales, relu=True))


def test_pdl_chain_matches_serial(cuda_device):
    """A chain of dependent linears launched with programmatic dependent
    launch gives the same bits as the plain launches."""
    rng = np.random.default_rng(17)
    ws = []
    for n, k in ((2560, 2048), (2048, 2048), (5632, 2048), (2048, 5632)):
        payload, scales = make_weight(rng, n, k, 8, k)
        ws.append(lq.QuantWeight.from_host(payload, scales, n, k, 8, k))
    x0 = dev(activations(rng, 1, 2048))

    def chain(flags):
        x = x0
        x = lq.linear(x, ws[0], flags=flags)[:, :2048].contiguous()
        x = lq.linear(x, ws[1], flags=flags)
        x = lq.linear(x, ws[2], flags=flags)
        return lq.linear(x, ws[3], flags=flags)

    assert bits_equal(host(chain(0)), host(chain(lq.LEAFQ_FLAG_PDL)))
    assert lq.load().leafq_device_status() == 0


def test_streams_are_independent(cuda_device):
    rng = np.random.default_rng(19)
    payload, scales = make_weight(rng, 4096, 2048, 8, 2048)
    w = lq.QuantWeight.from_host(payload, scales, 4096, 2048, 8, 2048)
    xs = [activations(rng, 1, 2048) for _ in range(4)]
    streams = [torch.cuda.Stream() for _ in xs]
    outs = []
    for s, x in zip(streams, xs):
        with torch.cuda.stream(s):
            outs.append(lq.linear(dev(x), w))
    torch.cuda.synchronize()
    for x, y in zip(xs, outs):
        assert bits_equal(y.cpu().numpy(), oracle.linear_int(x, payload, scales, 8, 2048, None))


@pytest.mark.parametrize("m", [1, 5, 40])
@pytest.mark.parametrize("bits,group,abits", [(8, 512, 8), (8, 64, 8), (4, 32, 8), (4, 32, 32), (8, 512, 32)])
def test_smoothquant_input_scale(cuda_device, m, bits, group, abits):
    """A weight with a calibrated input_scale (decoder.cpp:1008-1019): the
    input times the factors (one float rounding) is what the linear sees;
    leafq_linear_smooth fuses the scaling into the quantiser."""
    rng = np.random.default_rng(m * 100 + bits + group + abits)
    k, n = 512, 96
    payload, scales = make_weight(rng, n, k, bits, group)
    x = activations(rng, m, k)
    factors = (rng.random(k) * 1.5 + 0.5).astype(np.float32)
    w = lq.QuantWeight.from_host(payload, scales, n, k, bits, group, None, factors)
    y = host(lq.linear(dev(x), w, abits))
    xs = (x * factors[None, :]).astype(np.float32)
    if abits == 8:
        expect = oracle.linear_int(xs, payload, scales, bits, group, None)
    else:
        expect = oracle.linear_float(xs, payload, scales, bits, group, None)
    assert bits_equal(y, expect)
