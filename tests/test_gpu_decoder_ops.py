"""Decoder operators through the C ABI against the CPU restatement
(oracle/decoder.py, itself bit-exact against the reference decoder):
RMSNorm (sum of squares in the reference's left-to-right order, on inputs
built to stress rounding: ties, zeros, subnormal squares, overflow), RoPE +
KV append, attention and the SiLU gate, bit for bit."""
import ctypes

import numpy as np
import pytest
import torch

import leaf_b200 as lq
import oracle
from oracle import decoder as od

pytestmark = pytest.mark.gpu


def _s():
    return torch.cuda.current_stream().cuda_stream


def _vectors(rng, kind, rows, width):
    g = rng.standard_normal((rows, width)).astype(np.float32)
    if kind == "normal":
        return g
    if kind == "outliers":
        g[rng.random(g.shape) < 0.01] *= 100
        return g
    if kind == "grid":  # exact low-precision values: many rounding ties
        return (np.floor(g * 4) / 4).astype(np.float32)
    if kind == "zeros":
        g[rng.random(g.shape) < 0.3] = 0
        return g
    if kind == "tiny":  # squares in the subnormal range
        return (g * np.float32(1e-20)).astype(np.float32)
    if kind == "huge":  # sums overflow to inf
        return (g * np.float32(1e18)).astype(np.float32)
    if kind == "pow2":
        return np.ldexp(np.float32(1), rng.integers(-10, 10, size=g.shape)).astype(np.float32)
    if kind == "ones":  # partial sums land exactly on powers of two
        return np.sign(g).astype(np.float32)
    if kind == "growing":  # the running sum changes binade at almost every element
        e = (np.arange(width) % 48) - 40
        return (np.ldexp(np.float32(1), e)[None, :] * (1 + np.abs(g) * 0.01)).astype(np.float32)
    raise ValueError(kind)


@pytest.mark.parametrize("width", [64, 100, 102, 2048, 3000, 4096])
@pytest.mark.parametrize("kind", ["normal", "outliers", "grid", "zeros", "tiny", "huge", "pow2", "ones", "growing"])
def test_rmsnorm_bit_exact(cuda_device, kind, width):
    rng = np.random.default_rng(hash((kind, width)) % 2**32)
    rows = 512 if kind == "normal" and width == 2048 else 48
    x = _vectors(rng, kind, rows, width)
    delta = rng.standard_normal((rows, width)).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(width)).astype(np.float32)
    # No residual first (the built inputs reach the norm as they are), then
    # with the residual added, with and without the "+ 0.0f" of the delta.
    for use_delta, add_zero in ((False, 0), (True, 0), (True, 1)):
        h = torch.from_numpy(x).cuda()
        d = torch.from_numpy(delta).cuda()
        d_ptr = d.data_ptr() if use_delta else None
        out = torch.empty_like(h)
        lq._lib.check(lq.load().leafq_rmsnorm(_s(), h.data_ptr(), d_ptr, add_zero, rows, width,
                                              torch.from_numpy(w).cuda().data_ptr(), ctypes.c_float(1e-5),
                                              out.data_ptr()))
        hx = x + ((delta + np.float32(0)) if add_zero else delta) if use_delta else x
        assert np.array_equal(h.cpu().numpy().view(np.uint32), hx.view(np.uint32))
        with np.errstate(over="ignore", invalid="ignore"):
            expect = od.rmsnorm(hx, w, 1e-5)
        got = out.cpu().numpy()
        assert np.array_equal(got.view(np.uint32), expect.view(np.uint32)), kind
        if width % 4 == 0 and kind != "huge":
            # The same norm with the per-token INT8 quantisation fused in.
            h = torch.from_numpy(x).cuda()
            codes = torch.empty((rows, width), dtype=torch.int8, device="cuda")
            sx = torch.empty(rows, device="cuda")
            lq._lib.check(lq.load().leafq_rmsnorm_quantize(
                _s(), h.data_ptr(), d_ptr, add_zero, rows, width, torch.from_numpy(w).cuda().data_ptr(),
                ctypes.c_float(1e-5), None, codes.data_ptr(), sx.data_ptr()))
            eq, esx = oracle.quantize_act(expect)
            assert np.array_equal(codes.cpu().numpy(), eq), kind
            assert np.array_equal(sx.cpu().numpy().view(np.uint32), esx.view(np.uint32)), kind


def test_rotary_attention_silu_bit_exact(cuda_device):
    rng = np.random.default_rng(7)
    heads, kv, dim, cap, tokens, start = 8, 2, 64, 256, 5, 37
    c = od.rope_tables(10000.0, dim, cap)
    cos, sin = (torch.from_numpy(t).cuda() for t in c)
    qkv = rng.standard_normal((tokens, (heads + 2 * kv) * dim)).astype(np.float32)
    kc = rng.standard_normal((kv, cap, dim)).astype(np.float32)
    vc = rng.standard_normal((kv, cap, dim)).astype(np.float32)
    pos = torch.tensor([start], dtype=torch.int32, device="cuda")
    q_heads = torch.empty((heads, tokens, dim), device="cuda")
    kd, vd = torch.from_numpy(kc).cuda(), torch.from_numpy(vc).cuda()
    lib = lq.load()
    lq._lib.check(lib.leafq_rotary_append(_s(), torch.from_numpy(qkv).cuda().data_ptr(), tokens, heads, kv,
                                          dim, dim, cos.data_ptr(), sin.data_ptr(), pos.data_ptr(),
                                          q_heads.data_ptr(), kd.data_ptr(), vd.data_ptr(), cap))
    # oracle: the same rotation and append
    dec = od.OracleDecoder.__new__(od.OracleDecoder)
    dec.c = type("C", (), {"head_dim": dim, "rotary_dim": dim})()
    dec.cos, dec.sin = c
    qh = dec._rotate(qkv[:, :heads * dim], tokens, heads, start)
    kh = dec._rotate(qkv[:, heads * dim:(heads + kv) * dim], tokens, kv, start)
    vh = qkv[:, (heads + kv) * dim:].reshape(tokens, kv, dim).transpose(1, 0, 2)
    kc[:, start:start + tokens] = kh
    vc[:, start:start + tokens] = vh
    assert np.array_equal(q_heads.cpu().numpy().view(np.uint32), qh.view(np.uint32))
    assert np.array_equal(kd.cpu().numpy().view(np.uint32), kc.view(np.uint32))
    assert np.array_equal(vd.cpu().numpy().view(np.uint32), vc.view(np.uint32))
    scale = float(np.float32(1) / np.sqrt(np.sqrt(np.float32(dim))))
    out = torch.empty((tokens, heads * dim), device="cuda")
    lq._lib.check(lib.leafq_attention(_s(), q_heads.data_ptr(), kd.data_ptr(), vd.data_ptr(), tokens, heads,
                                      kv, dim, pos.data_ptr(), cap, ctypes.c_float(scale), out.data_ptr()))
    sc = np.float32(scale)
    expect = np.zeros((tokens, heads * dim), np.float32)
    for h in range(heads):
        for t in range(tokens):
            n = start + t + 1
            s = (od.attention_dot(qh[h, t], kc[h // (heads // kv), :n]) * sc) * sc
            e = oracle.expf(s - s.max())
            expect[t, h * dim:(h + 1) * dim] = od.seq_sum((e / od.seq_sum(e))[:, None] * vc[h // (heads // kv), :n],
                                                          axis=0)
    assert np.array_equal(out.cpu().numpy().view(np.uint32), expect.view(np.uint32))
    # SiLU gate over interleaved gate / up rows.
    gu = (rng.standard_normal((3, 2 * 1000)) * 4).astype(np.float32)
    act = torch.empty((3, 1000), device="cuda")
    lq._lib.check(lib.leafq_silu_gate(_s(), torch.from_numpy(gu).cuda().data_ptr(), 3, 1000, act.data_ptr()))
    g, u = gu[:, 0::2], gu[:, 1::2]
    expect = u * (g / (np.float32(1) + oracle.expf(-g)))
    assert np.array_equal(act.cpu().numpy().view(np.uint32), expect.view(np.uint32))
    # The same gate with the down projection's INT8 quantisation fused in.
    act2 = torch.empty((3, 1000), device="cuda")
    codes = torch.empty((3, 1000), dtype=torch.int8, device="cuda")
    sx = torch.empty(3, device="cuda")
    lq._lib.check(lib.leafq_silu_gate_quantize(_s(), torch.from_numpy(gu).cuda().data_ptr(), 3, 1000,
                                               act2.data_ptr(), codes.data_ptr(), sx.data_ptr()))
    eq, esx = oracle.quantize_act(expect)
    assert np.array_equal(act2.cpu().numpy().view(np.uint32), expect.view(np.uint32))
    assert np.array_equal(codes.cpu().numpy(), eq)
    assert np.array_equal(sx.cpu().numpy().view(np.uint32), esx.view(np.uint32))


@pytest.mark.parametrize("tokens,width", [(64, 5632), (1, 6144), (5, 1001), (2, 3), (150, 5632), (147, 4097)])
def test_silu_gate_quantize_shapes(cuda_device, tokens, width):
    """The fused SiLU gate + INT8 quantisation: fewer tokens than SMs take
    four CTAs per token (row maximum through distributed shared memory), more
    take one block per token; both against the restatement, bit for bit."""
    rng = np.random.default_rng(tokens * 7 + width)
    gu = (rng.standard_normal((tokens, 2 * width)) * 4).astype(np.float32)
    gu[0, 0:2 * width:7] *= np.float32(30.0)
    act = torch.empty((tokens, width), device="cuda")
    codes = torch.empty((tokens, width), dtype=torch.int8, device="cuda")
    sx = torch.empty(tokens, device="cuda")
    lib = lq.load()
    lq._lib.check(lib.leafq_silu_gate_quantize(_s(), torch.from_numpy(gu).cuda().data_ptr(), tokens, width,
                                               act.data_ptr(), codes.data_ptr(), sx.data_ptr()))
    g, u = gu[:, 0::2], gu[:, 1::2]
    expect = u * (g / (np.float32(1) + oracle.expf(-g)))
    eq, esx = oracle.quantize_act(expect)
    assert np.array_equal(act.cpu().numpy().view(np.uint32), expect.view(np.uint32))
    assert np.array_equal(codes.cpu().numpy(), eq)
    assert np.array_equal(sx.cpu().numpy().view(np.uint32), esx.view(np.uint32))
    assert lib.leafq_device_status() == 0
