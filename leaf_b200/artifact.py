"""Reader for Leaf's mapped decoder artifacts (LEAFDC02, 03, 04, 07).

Restates the reference loader's parse and checks (decoder.cpp:787-904): the
header (magic, version, tensor count, 64-byte aligned data base, 10 uint32
dimensions, theta, epsilon, 8 uint32 operator fields, embedding scale), the
LEAFDC07 operator metadata (storage policy, Q/K norm flag, static RoPE
frequencies), the EOS list (LEAFDC04/05/06/07), then one descriptor per
tensor (name, rank 2, rows, cols, bits, group, payload offset and size, scale
offset and count) with the same range and metadata checks.  Payloads are
numpy views of one read-only memory map; ``to_device`` uploads a tensor as a
``QuantWeight`` in the same layout (no repacking).  The source-BF16 storage
versions (LEAFDC05/06, FP32-compute artifacts) are rejected: this library's
path is the quantised one.
"""
from __future__ import annotations

import math
import struct
from dataclasses import dataclass, field
from pathlib import Path
from typing import Optional

import numpy as np

from . import _lib
from ._lib import LeafError

_HEADER = struct.Struct("<8sIIQ10Iff8If")
_DESCRIPTOR = struct.Struct("<5I4Q")
_VERSIONS = {b"LEAFDC02": 2, b"LEAFDC03": 3, b"LEAFDC04": 4, b"LEAFDC05": 5, b"LEAFDC06": 6,
             b"LEAFDC07": 7}


def _check(condition: bool, message: str) -> None:
    if not condition:
        raise LeafError(_lib.LEAFQ_ERR_INVALID, message)


@dataclass
class DecoderConfig:
    hidden: int
    intermediate: int
    heads: int
    kv_heads: int
    layers: int
    vocab: int
    max_positions: int
    eos: int
    head_dim: int
    sliding_window: int
    theta: float
    epsilon: float
    norm_kind: int
    activation: int
    position_kind: int
    gated: int
    parallel: int
    rotary_dim: int
    position_offset: int
    final_norm: int
    embedding_scale: float
    qk_norm: bool = False
    rope_frequencies: list = field(default_factory=list)
    eos_tokens: list = field(default_factory=list)


@dataclass
class HostTensor:
    """One artifact tensor: data is the payload (int8 [rows, cols], packed
    uint8 [rows, cols/2] or float32 [rows, cols]); scales float32
    [rows, cols/group] for bits 8/4."""

    name: str
    rows: int
    cols: int
    bits: int
    group: int
    data: np.ndarray
    scales: Optional[np.ndarray]


class Artifact:
    def __init__(self, path):
        self.path = Path(path)
        blob = np.memmap(self.path, dtype=np.uint8, mode="r")
        self._blob = blob
        size = blob.size
        _check(size >= _HEADER.size, "unsupported artifact magic")
        raw = bytes(blob[:_HEADER.size])
        magic = raw[:8]
        _check(magic in _VERSIONS, "unsupported artifact magic")
        fields = _HEADER.unpack(raw)
        version, count, base = fields[1], fields[2], fields[3]
        _check(version == _VERSIONS[magic], "unsupported decoder artifact version")
        _check(version not in (5, 6), "source-BF16 storage artifacts (FP32 compute) are not on the "
               "quantised GPU path")
        (h, f, heads, kv, layers, vocab, maxpos, eos, dim, window) = fields[4:14]
        theta, eps = fields[14], fields[15]
        (norm_kind, activation, position_kind, gated, parallel, rotary_dim, offset,
         final_norm) = fields[16:24]
        escale = fields[24]
        _check(version in (3, 4, 7) or window == 0, "invalid sliding-window artifact configuration")
        _check(all((h, f, heads, kv, layers, vocab, dim, maxpos)) and heads % kv == 0 and
               norm_kind <= 1 and activation <= 3 and position_kind <= 2 and gated <= 1 and
               parallel <= 1 and rotary_dim <= dim and rotary_dim % 2 == 0 and
               (position_kind != 0 or rotary_dim > 0) and final_norm <= 1 and
               math.isfinite(escale) and escale > 0 and math.isfinite(theta) and theta > 0 and
               math.isfinite(eps) and eps > 0, "invalid decoder configuration")
        _check(base % 64 == 0 and base <= size and count <= size // 56, "invalid tensor table")
        _check(eos < vocab or eos == 0xFFFFFFFF, "invalid EOS token")
        pos = _HEADER.size

        def u32():
            nonlocal pos
            _check(pos + 4 <= size, "truncated decoder artifact")
            v = struct.unpack_from("<I", blob, pos)[0]
            pos += 4
            return v

        def f32():
            nonlocal pos
            _check(pos + 4 <= size, "truncated decoder artifact")
            v = struct.unpack_from("<f", blob, pos)[0]
            pos += 4
            return v

        qk_norm, frequencies = False, []
        if version == 7:
            _check(pos <= base and base - pos >= 12, "truncated decoder operator metadata")
            storage, qk, nfreq = u32(), u32(), u32()
            _check(storage in (0, 5, 6), "invalid decoder storage policy")
            _check(storage == 0, "source-BF16 storage artifacts are not on the quantised GPU path")
            _check((qk or nfreq) and qk <= 1 and position_kind == 0 and (not qk or norm_kind == 0) and
                   (not nfreq or nfreq == rotary_dim // 2) and nfreq <= (base - pos) // 4,
                   "invalid decoder operator metadata")
            qk_norm = bool(qk)
            for _ in range(nfreq):
                fr = f32()
                _check(math.isfinite(fr) and 0 < fr <= 1, "invalid static RoPE frequency")
                frequencies.append(fr)
        _check(qk_norm or heads * dim == h, "invalid decoder head geometry")
        eos_tokens = []
        if version in (4, 7):
            _check(pos <= base and base - pos >= 4, "truncated EOS metadata")
            n = u32()
            _check((version == 7 or n >= 2) and n <= 1024 and n <= vocab and n <= (base - pos) // 4,
                   "invalid multi-EOS token count")
            for _ in range(n):
                token = u32()
                _check(token < vocab and token not in eos_tokens, "invalid or duplicate EOS token")
                eos_tokens.append(token)
            _check((eos == 0xFFFFFFFF) if not eos_tokens else eos == eos_tokens[0],
                   "multi-EOS primary token mismatch")
        elif eos < vocab:
            eos_tokens.append(eos)
        self.config = DecoderConfig(h, f, heads, kv, layers, vocab, maxpos, eos, dim, window, theta,
                                    eps, norm_kind, activation, position_kind, gated, parallel,
                                    rotary_dim, offset, final_norm, escale, qk_norm, frequencies,
                                    eos_tokens)
        self.tensors: dict[str, HostTensor] = {}
        for _ in range(count):
            n = u32()
            _check(pos + n <= size, "truncated decoder artifact")
            name = bytes(blob[pos:pos + n]).decode("utf-8")
            pos += n
            _check(pos + _DESCRIPTOR.size <= size, "truncated decoder artifact")
            rank, rows, cols, bits, group, off, nbytes, soff, scount = _DESCRIPTOR.unpack_from(blob, pos)
            pos += _DESCRIPTOR.size
            _check(rank == 2 and rows and cols and bits in (32, 8, 4), "invalid tensor " + name)
            elements = rows * cols
            _check((bits != 4 or cols % 2 == 0) and nbytes == elements * bits // 8 and off % 64 == 0 and
                   off <= size - base and nbytes <= size - base - off, "invalid tensor data range " + name)
            start = base + off
            if bits == 32:
                _check(scount == 0 and group == 0, "unexpected FP32 quantization metadata")
                data = blob[start:start + nbytes].view(np.float32).reshape(rows, cols)
                scales = None
            else:
                _check(group and cols % group == 0 and (bits != 4 or group % 2 == 0) and
                       scount == rows * (cols // group) and soff % 64 == 0 and soff <= size - base and
                       scount <= (size - base - soff) // 4, "invalid quantization metadata " + name)
                width = cols if bits == 8 else cols // 2
                data = blob[start:start + nbytes].view(np.int8 if bits == 8 else np.uint8)
                data = data.reshape(rows, width)
                s0 = base + soff
                scales = blob[s0:s0 + 4 * scount].view(np.float32).reshape(rows, cols // group)
                _check(bool(np.all(np.isfinite(scales)) and np.all(scales > 0)), "invalid quantization scale")
            if name.endswith(".input_scale"):
                _check(bits == 32 and rows == 1, "invalid calibrated input scale tensor")
                _check(bool(np.all(np.isfinite(data)) and np.all(data > 0)),
                       "invalid calibrated input scale value")
            _check(name not in self.tensors, "duplicate tensor " + name)
            self.tensors[name] = HostTensor(name, rows, cols, bits, group, data, scales)
        _check(pos <= base, "metadata overlaps tensor payload")
        self._require("model.embed_tokens.weight", vocab, h)
        self._require("lm_head.weight", vocab, h)
        if final_norm:
            self._require("model.norm.weight", 1, h)
        q = heads * dim
        for i in range(layers):
            p = f"model.layers.{i}."
            self._require(p + "input_layernorm.weight", 1, h)
            self._require(p + "post_attention_layernorm.weight", 1, h)
            self._require(p + "self_attn.q_proj.weight", q, h)
            self._require(p + "self_attn.k_proj.weight", kv * dim, h)
            self._require(p + "self_attn.v_proj.weight", kv * dim, h)
            self._require(p + "self_attn.o_proj.weight", h, q)
            if gated:
                self._require(p + "mlp.gate_proj.weight", f, h)
            self._require(p + "mlp.up_proj.weight", f, h)
            self._require(p + "mlp.down_proj.weight", h, f)

    def _require(self, name: str, rows: int, cols: int) -> HostTensor:
        t = self.tensors.get(name)
        _check(t is not None and t.rows == rows and t.cols == cols,
               "missing or incompatible tensor " + name)
        return t

    def get(self, name: str) -> Optional[HostTensor]:
        return self.tensors.get(name)


def load(path) -> Artifact:
    return Artifact(path)
