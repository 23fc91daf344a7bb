"""Batched decoding (several independent requests per forward, the shape of
config 4): the batched rotary / attention operators against the CPU
restatement, and the batched decoder against the reference decoder's
recorded tokens and the single-sequence decoder, bit for bit."""
import ctypes
import json

import numpy as np
import pytest
import torch

import leaf_b200 as lq
import oracle
from oracle import decoder as od
from conftest import GOLDEN
import decoder_fixture as fx  # tests/golden
from test_gpu_decoder import _artifact, _close

pytestmark = pytest.mark.gpu


def _s():
    return torch.cuda.current_stream().cuda_stream


def _rotate(qkv_part, tokens, heads, start, dim, tables):
    dec = od.OracleDecoder.__new__(od.OracleDecoder)
    dec.c = type("C", (), {"head_dim": dim, "rotary_dim": dim})()
    dec.cos, dec.sin = tables
    return dec._rotate(qkv_part, tokens, heads, start)


def _attention(q, kc, vc, start, tokens, heads, kv, scale):
    """q [heads][tokens][dim], caches [kv][cap][dim] -> [tokens][heads*dim]."""
    dim = q.shape[-1]
    sc = np.float32(scale)
    out = np.zeros((tokens, heads * dim), np.float32)
    for h in range(heads):
        for t in range(tokens):
            n = start + t + 1
            s = (od.attention_dot(q[h, t], kc[h // (heads // kv), :n]) * sc) * sc
            e = oracle.expf(s - s.max())
            out[t, h * dim:(h + 1) * dim] = od.seq_sum((e / od.seq_sum(e))[:, None] * vc[h // (heads // kv), :n],
                                                      axis=0)
    return out


@pytest.mark.parametrize("heads,kv,dim,tokens", [(8, 2, 64, 1), (8, 2, 64, 5), (32, 4, 64, 40),
                                                 (4, 2, 32, 70), (32, 4, 64, 16), (8, 8, 32, 17)])
def test_batched_rotary_attention_bit_exact(cuda_device, heads, kv, dim, tokens):
    _batched_rotary_attention(heads, kv, dim, tokens, 192, [0, 37, 100], heads * 1000 + tokens)


@pytest.mark.parametrize("heads,kv,dim,tokens,cap,starts", [
    # 20 sequences x 4 kv heads: one block per kv head serving 8 query heads,
    # caches of 1 to 599 keys across the kernel's staged key and value chunks
    (32, 4, 64, 1, 600, [0, 62, 63, 64, 126, 127, 128, 129, 254, 255, 256, 383, 384, 447, 510, 511, 512, 513,
                         575, 598]),
    (16, 2, 32, 3, 400, [5, 60, 61, 125, 126, 127, 189, 250, 253, 254, 300, 318, 319, 320, 350, 381, 382, 383,
                         390, 396]),
    # few blocks: each kv head's query heads split over two blocks
    (8, 2, 64, 2, 520, [300, 450, 517]),
    (32, 8, 64, 1, 700, [699, 0, 640]),
])
def test_batched_decode_attention_long_caches(cuda_device, heads, kv, dim, tokens, cap, starts):
    _batched_rotary_attention(heads, kv, dim, tokens, cap, starts, heads * 1000 + tokens + cap)


def _batched_rotary_attention(heads, kv, dim, tokens, cap, starts, seed):
    rng = np.random.default_rng(seed)
    S = len(starts)
    tables = od.rope_tables(10000.0, dim, cap)
    cos, sin = (torch.from_numpy(t).cuda() for t in tables)
    width = (heads + 2 * kv) * dim
    qkv = rng.standard_normal((S, tokens, width)).astype(np.float32)
    kc = rng.standard_normal((S, kv, cap, dim)).astype(np.float32)
    vc = rng.standard_normal((S, kv, cap, dim)).astype(np.float32)
    pos = torch.tensor(starts, dtype=torch.int32, device="cuda")
    q_heads = torch.empty((S, heads, tokens, dim), device="cuda")
    kd, vd = torch.from_numpy(kc).cuda(), torch.from_numpy(vc).cuda()
    lib = lq.load()
    lq._lib.check(lib.leafq_rotary_append_batch(_s(), torch.from_numpy(qkv).cuda().data_ptr(), S, tokens, heads,
                                                kv, dim, dim, cos.data_ptr(), sin.data_ptr(), pos.data_ptr(),
                                                q_heads.data_ptr(), kd.data_ptr(), vd.data_ptr(), cap))
    scale = float(np.float32(1) / np.sqrt(np.sqrt(np.float32(dim))))
    need = lib.leafq_attention_workspace_bytes(S, tokens, heads, kv, dim, cap)
    assert (need > 0) == (tokens >= 16)
    ws = torch.empty(max(need, 16), dtype=torch.uint8, device="cuda")
    out = torch.empty((S * tokens, heads * dim), device="cuda")
    lq._lib.check(lib.leafq_attention_batch(_s(), q_heads.data_ptr(), kd.data_ptr(), vd.data_ptr(), S, tokens,
                                            heads, kv, dim, pos.data_ptr(), cap, cap, ctypes.c_float(scale),
                                            out.data_ptr(), ws.data_ptr(), ws.numel()))
    got_q, got_k, got_v = q_heads.cpu().numpy(), kd.cpu().numpy(), vd.cpu().numpy()
    got = out.cpu().numpy().reshape(S, tokens, heads * dim)
    for s, start in enumerate(starts):
        qh = _rotate(qkv[s, :, :heads * dim], tokens, heads, start, dim, tables)
        kh = _rotate(qkv[s, :, heads * dim:(heads + kv) * dim], tokens, kv, start, dim, tables)
        vh = qkv[s, :, (heads + kv) * dim:].reshape(tokens, kv, dim).transpose(1, 0, 2)
        kc[s, :, start:start + tokens] = kh
        vc[s, :, start:start + tokens] = vh
        assert np.array_equal(got_q[s].view(np.uint32), qh.view(np.uint32)), s
        assert np.array_equal(got_k[s].view(np.uint32), kc[s].view(np.uint32)), s
        assert np.array_equal(got_v[s].view(np.uint32), vc[s].view(np.uint32)), s
        expect = _attention(qh, kc[s], vc[s], start, tokens, heads, kv, scale)
        ok, err = _close(got[s], expect)
        assert ok, f"sequence {s}: attention differs by {err}"
    assert lq.load().leafq_device_status() == 0


def test_attention_position_past_cache_is_reported(cuda_device):
    """A start position whose tokens do not fit the cache is skipped on the
    device and reported by leafq_device_status (no out-of-bounds access)."""
    lib = lq.load()
    heads, kv, dim, cap, tokens = 8, 2, 64, 64, 20
    pos = torch.tensor([0, cap - 4], dtype=torch.int32, device="cuda")
    qkv = torch.zeros((2 * tokens, (heads + 2 * kv) * dim), device="cuda")
    q_heads = torch.zeros((2, heads, tokens, dim), device="cuda")
    kc = torch.zeros((2, kv, cap, dim), device="cuda")
    vc = torch.zeros_like(kc)
    c = torch.zeros((cap, dim // 2), device="cuda")
    lq._lib.check(lib.leafq_rotary_append_batch(_s(), qkv.data_ptr(), 2, tokens, heads, kv, dim, dim,
                                                c.data_ptr(), c.data_ptr(), pos.data_ptr(), q_heads.data_ptr(),
                                                kc.data_ptr(), vc.data_ptr(), cap))
    assert lib.leafq_device_status() == lq._lib.LEAFQ_ERR_INVALID
    need = lib.leafq_attention_workspace_bytes(2, tokens, heads, kv, dim, cap)
    ws = torch.empty(need, dtype=torch.uint8, device="cuda")
    out = torch.empty((2 * tokens, heads * dim), device="cuda")
    lq._lib.check(lib.leafq_attention_batch(_s(), q_heads.data_ptr(), kc.data_ptr(), vc.data_ptr(), 2, tokens,
                                            heads, kv, dim, pos.data_ptr(), cap, cap, ctypes.c_float(0.5),
                                            out.data_ptr(), ws.data_ptr(), ws.numel()))
    assert lib.leafq_device_status() == lq._lib.LEAFQ_ERR_INVALID
    assert lib.leafq_device_status() == 0


def _prompts(golden, vocab, count, seed):
    prompt = golden["prompt"].tolist()
    rng = np.random.default_rng(seed)
    return [prompt] + [rng.integers(0, vocab, size=len(prompt)).tolist() for _ in range(count - 1)]


@pytest.mark.parametrize("name", ["tiny_w8", "tiny_w4"])
def test_tiny_batch_matches_single_sequences(cuda_device, tmp_path, name):
    from leaf_b200.decoder import Decoder

    path, golden = _artifact(tmp_path, name, fx.TINY)
    generated = golden["generated"].tolist()
    prompts = _prompts(golden, fx.TINY.vocab, 3, 11)
    batch = Decoder(path, sequences=3)
    logits = batch.forward_batch(prompts).cpu().numpy()
    ok, err = _close(logits[0], golden["prefill_logits"][-1])
    assert ok, f"batched prefill logits differ from the reference by {err}"
    single = Decoder(path)
    for s, p in enumerate(prompts[1:], 1):
        single.reset()
        ok, err = _close(logits[s], single.forward(p).cpu().numpy()[0])
        assert ok, f"sequence {s}: batched prefill logits differ by {err}"
    batch.reset()
    got = batch.generate_batch(prompts, len(generated))
    assert got[0] == generated
    for s, p in enumerate(prompts[1:], 1):
        single.reset()
        assert got[s] == single.generate(p, len(generated)), s
    assert batch.device_status() == 0


def test_tinyllama_batch_tokens(cuda_device, tmp_path):
    """Two TinyLlama-shape requests decoded together: the first is the
    reference's recorded request (identical tokens), the second a different
    random prompt (tokens of the single-sequence decoder)."""
    from leaf_b200.decoder import Decoder

    path, golden = _artifact(tmp_path, "tinyllama_w8", fx.TINYLLAMA)
    generated = golden["generated"].tolist()
    prompts = _prompts(golden, fx.TINYLLAMA.vocab, 2, 5)
    n = len(prompts[0]) + len(generated)
    batch = Decoder(path, sequences=2, capacity=n)
    got = batch.generate_batch(prompts, len(generated))
    assert got[0] == generated, next(i for i, (a, b) in enumerate(zip(got[0], generated)) if a != b)
    assert batch.device_status() == 0
    del batch
    single = Decoder(path, capacity=n)
    path.unlink()
    assert got[1] == single.generate(prompts[1], len(generated))
