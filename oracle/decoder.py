"""CPU restatement of Leaf's decoder forward (TEST INFRASTRUCTURE ONLY).

Follows ``Decoder::Impl::forward_into`` (engine/src/decoder.cpp:1282-1452) for
the Llama family (RMSNorm, RoPE, gated SiLU, sequential residual), in numpy
float32 with the reference's operation order:

* embedding: float(q) * scale (Weight::value, decoder.cpp:241-250) * embedding_scale;
* RMSNorm (norm(), decoder.cpp:706-727): sum of v*v accumulated sequentially
  (np.cumsum in float32 rounds after every addition), scale =
  1 / sqrt(sum / width + eps), out = (v * scale) * w + 0;
* RoPE tables with libm cosf / sinf / powf (decoder.cpp:929-933, 1248-1256),
  rotation a*c - b*s, b*c + a*s (:1259-1281);
* attention (KVCache::attend -> transformer.cpp:93-145; quantised artifacts
  take this path for prefill and decode, the vector kernel is FP32-artifact
  only, decoder.cpp:942-947): q.k summed sequentially (scalar_dot: the
  reference build has no -mavx2 for transformer.cpp), score =
  (dot * scale) * scale, softmax with libm expf, denominator and
  probability-weighted values summed sequentially over keys;
* SiLU gate up * (g / (1 + expf(-g))) (decoder.cpp:982-988, 1414; the vector
  SiLU kernel is enabled for W8A8 on Windows builds only,
  decoder_config.h:5-11);
* linears through the oracle's integer kernels (``linear_int``), or the
  reference's compiled kernels when ``use_ref`` (faster at full size).
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import expf, linear_int, ref_linear_int, unpack_int4

_libm = ctypes.CDLL("libm.so.6")
for _name in ("cosf", "sinf"):
    getattr(_libm, _name).restype = ctypes.c_float
    getattr(_libm, _name).argtypes = [ctypes.c_float]
_libm.powf.restype = ctypes.c_float
_libm.powf.argtypes = [ctypes.c_float, ctypes.c_float]

F = np.float32
_COEFFICIENTS = [1.0 / 479001600.0, 1.0 / 39916800.0, 1.0 / 3628800.0, 1.0 / 362880.0,
                 1.0 / 40320.0, 1.0 / 5040.0, 1.0 / 720.0, 1.0 / 120.0, 1.0 / 24.0, 1.0 / 6.0,
                 0.5, 1.0, 1.0]


def exp_reference(x: np.ndarray) -> np.ndarray:
    """attention_vector.h:22-53 / silu_gate.h:45-70 for x in [-80, 80];
    libm-equivalent double exp outside."""
    x = np.asarray(x, dtype=np.float32)
    xd = x.astype(np.float64)
    n = np.rint(xd * 1.4426950408889634074)
    r = xd - n * 0.69314718036912381649
    r = r - n * 1.9082149292705877000e-10
    p = np.full_like(xd, 1.0 / 6227020800.0)
    for c in _COEFFICIENTS:
        p = p * r + c
    scale = np.ldexp(1.0, np.where(np.isfinite(n), n, 0).astype(np.int64))
    out = (p * scale).astype(np.float32)
    outside = ~((x >= -80.0) & (x <= 80.0))
    if outside.any():
        with np.errstate(over="ignore", under="ignore"):
            out[outside] = np.exp(xd[outside]).astype(np.float32)
    return out


def seq_sum(values: np.ndarray, axis: int = -1) -> np.ndarray:
    """Left-to-right float32 sum (every addition rounded)."""
    return np.cumsum(np.asarray(values, dtype=np.float32), axis=axis, dtype=np.float32).take(-1, axis=axis)


def rmsnorm(v: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    v = np.asarray(v, dtype=np.float32)
    width = v.shape[-1]
    sq = seq_sum(v * v)
    scale = F(1.0) / np.sqrt(sq / F(width) + F(eps))
    return (v * scale[..., None]) * w + F(0.0)


def rope_tables(theta: float, rotary_dim: int, positions: int):
    half = rotary_dim // 2
    cos = np.empty((positions, half), np.float32)
    sin = np.empty_like(cos)
    for i in range(half):
        freq = F(1.0) / F(_libm.powf(F(theta), F(2 * i) / F(rotary_dim)))
        for p in range(positions):
            angle = F(p) * freq
            cos[p, i] = _libm.cosf(angle)
            sin[p, i] = _libm.sinf(angle)
    return cos, sin


def attention_dot(q: np.ndarray, keys: np.ndarray) -> np.ndarray:
    """q.k for one query against [n, dim] keys.  transformer.cpp is compiled
    without -mavx2 by the reference's build (leaf/cli.py:66), so fast_dot
    (:65-79) is its scalar_dot (:60-64): one sequential sum over dim."""
    return seq_sum(keys * q, axis=1)


class OracleDecoder:
    """forward(ids) over an ``Artifact`` (leaf_b200.artifact is a file parser;
    the oracle reads the tensors through it)."""

    def __init__(self, artifact, use_ref: bool = False, threads: int = 1):
        self.art = artifact
        c = artifact.config
        self.c = c
        self.use_ref, self.threads = use_ref, threads
        self.cos, self.sin = rope_tables(c.theta, c.rotary_dim, c.max_positions)
        self.scale = F(1.0) / np.sqrt(np.sqrt(F(c.head_dim)))
        self.reset()

    def reset(self):
        c = self.c
        self.k = [np.zeros((c.kv_heads, 0, c.head_dim), np.float32) for _ in range(c.layers)]
        self.v = [np.zeros((c.kv_heads, 0, c.head_dim), np.float32) for _ in range(c.layers)]
        self.length = 0

    def _linear(self, x, name):
        """Decoder::Impl::linear (decoder.cpp:994-1233): the input times the
        calibrated ``input_scale`` when the artifact has one (:1008-1019, one
        float multiply per element), the integer linear, then + bias (:1229)."""
        t = self.art.get(name)
        base = name[:-len(".weight")]
        scale = self.art.get(base + ".input_scale")
        bias = self.art.get(base + ".bias")
        if scale is not None:
            x = (np.asarray(x, dtype=np.float32) * scale.data.reshape(1, -1)).astype(np.float32)
        b = None if bias is None else np.ascontiguousarray(bias.data.reshape(-1), dtype=np.float32)
        if self.use_ref:
            return ref_linear_int(x, t.data, t.scales, t.bits, t.group, b, threads=self.threads)
        return linear_int(x, t.data, t.scales, t.bits, t.group, b)

    def _rotate(self, x, tokens, nheads, pos):
        c = self.c
        d, half = c.head_dim, c.rotary_dim // 2
        x = x.reshape(tokens, nheads, d).transpose(1, 0, 2).copy()  # [heads][tokens][dim]
        cos = self.cos[pos:pos + tokens][None, :, :]
        sin = self.sin[pos:pos + tokens][None, :, :]
        a, b = x[..., :half].copy(), x[..., half:2 * half].copy()
        x[..., :half] = a * cos - b * sin
        x[..., half:2 * half] = b * cos + a * sin
        return x

    def forward(self, ids, all_logits: bool = False) -> np.ndarray:
        c, art = self.c, self.art
        tokens, pos = len(ids), self.length
        emb = art.get("model.embed_tokens.weight")
        rows = np.asarray(ids, dtype=np.int64)
        table = emb.data[rows]
        if emb.bits == 4:
            table = unpack_int4(table)
        q = table.astype(np.float32)
        if emb.bits == 32:
            values = q
        else:
            values = q * emb.scales[rows].reshape(tokens, -1).repeat(emb.group, axis=1)
        hidden = values * F(c.embedding_scale)
        for layer in range(c.layers):
            p = f"model.layers.{layer}."
            x = rmsnorm(hidden, art.get(p + "input_layernorm.weight").data.reshape(-1), c.epsilon)
            qv = self._linear(x, p + "self_attn.q_proj.weight")
            kv = self._linear(x, p + "self_attn.k_proj.weight")
            vv = self._linear(x, p + "self_attn.v_proj.weight")
            qh = self._rotate(qv, tokens, c.heads, pos)
            kh = self._rotate(kv, tokens, c.kv_heads, pos)
            vh = vv.reshape(tokens, c.kv_heads, c.head_dim).transpose(1, 0, 2)
            self.k[layer] = np.concatenate([self.k[layer], kh], axis=1)
            self.v[layer] = np.concatenate([self.v[layer], vh], axis=1)
            attn = np.zeros((tokens, c.heads * c.head_dim), np.float32)
            group = c.heads // c.kv_heads
            for h in range(c.heads):
                K, V = self.k[layer][h // group], self.v[layer][h // group]
                for t in range(tokens):
                    n = pos + t + 1
                    s = (attention_dot(qh[h, t], K[:n]) * self.scale) * self.scale
                    e = expf(s - s.max())
                    prob = e / seq_sum(e)
                    attn[t, h * c.head_dim:(h + 1) * c.head_dim] = seq_sum(prob[:, None] * V[:n], axis=0)
            o = self._linear(attn, p + "self_attn.o_proj.weight")
            hidden = hidden + o
            x = rmsnorm(hidden, art.get(p + "post_attention_layernorm.weight").data.reshape(-1), c.epsilon)
            up = self._linear(x, p + "mlp.up_proj.weight")
            gate = self._linear(x, p + "mlp.gate_proj.weight")
            act = up * (gate / (F(1.0) + expf(-gate)))
            down = self._linear(act, p + "mlp.down_proj.weight")
            hidden = hidden + (down + F(0.0))
        x = rmsnorm(hidden, art.get("model.norm.weight").data.reshape(-1), c.epsilon)
        self.length += tokens
        rows = x if all_logits else x[-1:]
        return self._linear(np.ascontiguousarray(rows), "lm_head.weight")
