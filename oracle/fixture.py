"""Seeded random Llama decoders in the reference's artifact format.  TEST
INFRASTRUCTURE ONLY: the decoder parity fixtures and the CPU baseline's model
file; the product never imports it.

``llama_tensors`` draws every tensor of a Llama-architecture decoder from one
seeded numpy generator in a fixed order (weights N(0, 0.02), RMSNorm weights
1 or 1 + N(0, norm_noise)), so the same seed gives the same model on every
machine with this numpy.  ``write_artifact`` writes those tensors as a
LEAFDC02 decoder artifact, restating the reference exporter
(tools/export_decoder.py:214-413): header struct ``<8sIIQ10Iff8If`` with the
config values of tools/decoder_plan.py:330-376, one ``<I`` name length + name
+ ``<5I4Q`` descriptor per tensor in tools/decoder_plan.py:408-427 order,
payloads and scales 64-byte aligned after a 64-byte aligned data base,
matrices with more than one row quantised by export_decoder.quantize
(:91-105), one-row tensors fp32.  ``tests/golden/make_decoder_golden.py``
checks that this writer and the reference exporter produce identical bytes
(and ``tests/test_artifact.py`` checks the recorded digests).
"""
from __future__ import annotations

import json
import struct
from dataclasses import dataclass
from pathlib import Path

import numpy as np

HEADER = struct.Struct("<8sIIQ10Iff8If")
DESCRIPTOR = struct.Struct("<5I4Q")
NO_EOS = 0xFFFFFFFF


@dataclass(frozen=True)
class LlamaShape:
    hidden: int
    intermediate: int
    heads: int
    kv_heads: int
    layers: int
    vocab: int
    max_positions: int
    theta: float = 10000.0
    epsilon: float = 1e-5

    @property
    def head_dim(self) -> int:
        return self.hidden // self.heads

    def hf_config(self) -> dict:
        """A Hugging Face config.json the reference's plan builder accepts
        (llama adapter, no EOS so greedy generation never stops early)."""
        return dict(model_type="llama", architectures=["LlamaForCausalLM"],
                    hidden_size=self.hidden, intermediate_size=self.intermediate,
                    num_attention_heads=self.heads, num_key_value_heads=self.kv_heads,
                    num_hidden_layers=self.layers, vocab_size=self.vocab,
                    max_position_embeddings=self.max_positions, rms_norm_eps=self.epsilon,
                    rope_theta=self.theta, hidden_act="silu", tie_word_embeddings=False,
                    eos_token_id=None)

    def tensor_order(self):
        """(name, rows, cols) in the order of tools/decoder_plan.py:408-427."""
        h, f, kv, d = self.hidden, self.intermediate, self.kv_heads, self.head_dim
        q = self.heads * d
        out = [("model.embed_tokens.weight", self.vocab, h), ("lm_head.weight", self.vocab, h),
               ("model.norm.weight", 1, h)]
        for i in range(self.layers):
            p = f"model.layers.{i}."
            out += [(p + "input_layernorm.weight", 1, h), (p + "post_attention_layernorm.weight", 1, h),
                    (p + "self_attn.q_proj.weight", q, h), (p + "self_attn.k_proj.weight", kv * d, h),
                    (p + "self_attn.v_proj.weight", kv * d, h), (p + "self_attn.o_proj.weight", h, q),
                    (p + "mlp.up_proj.weight", f, h), (p + "mlp.down_proj.weight", h, f),
                    (p + "mlp.gate_proj.weight", f, h)]
        return out


TINY = LlamaShape(hidden=128, intermediate=256, heads=4, kv_heads=2, layers=2, vocab=256,
                  max_positions=256)
TINYLLAMA = LlamaShape(hidden=2048, intermediate=5632, heads=32, kv_heads=4, layers=22,
                       vocab=32000, max_positions=2048)


def llama_tensors(shape: LlamaShape, seed: int, norm_noise: float = 0.0):
    """Yield (name, float32 array [rows, cols] or [cols]) in tensor order."""
    rng = np.random.default_rng(seed)
    for name, rows, cols in shape.tensor_order():
        if rows == 1:
            w = np.ones(cols, dtype=np.float32)
            if norm_noise:
                w += (rng.standard_normal(cols, dtype=np.float32) * np.float32(norm_noise))
            yield name, w
        else:
            yield name, rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(0.02)


def prompt_ids(shape: LlamaShape, seed: int, length: int) -> np.ndarray:
    return np.random.default_rng(seed).integers(0, shape.vocab, size=length).astype(np.uint32)


def quantize(array: np.ndarray, bits: int, group: int):
    """tools/export_decoder.py:91-105 (same numpy expressions)."""
    rows, cols = array.shape
    grouped = array.reshape(rows, cols // group, group)
    limit = (1 << (bits - 1)) - 1
    scales = np.maximum(np.max(np.abs(grouped), axis=-1) / limit, 1e-12).astype("<f4")
    values = np.clip(np.rint(grouped / scales[..., None]), -limit, limit).astype(np.int8)
    values = values.reshape(rows, cols)
    if bits == 4:
        nibbles = values.astype(np.uint8) & 15
        values = nibbles[:, 0::2] | (nibbles[:, 1::2] << 4)
    return np.ascontiguousarray(values), np.ascontiguousarray(scales)


def _align64(v: int) -> int:
    return (v + 63) & ~63


def header_values(shape: LlamaShape):
    """config_values() of the llama plan (tools/decoder_plan.py:195-240, 330-376)."""
    d = shape.head_dim
    return (shape.hidden, shape.intermediate, shape.heads, shape.kv_heads, shape.layers, shape.vocab,
            shape.max_positions, NO_EOS, d, 0, float(shape.theta), float(shape.epsilon),
            0, 0, 0, 1, 0, d, 0, 1, 1.0)


def smooth_variant(shape: LlamaShape, tensors, seed: int, biases: bool = True):
    """The same decoder with the extra tensors the reference decoder looks up
    for every linear (Decoder::Impl::linear, decoder.cpp:1003-1019): per-column
    SmoothQuant factors -- each projection's weight columns multiplied by
    factors f and ``<proj>.input_scale`` = 1 / f (fp32 [1, cols]), as
    tools/export_decoder.py:383-390 exports a calibrated model -- and, with
    `biases`, q / k / v projection biases ``<proj>.bias`` (fp32 [1, rows], as
    a Qwen2 export carries).  Returns (tensors, extras): the modified tensors
    in tensor order and the extra one-row tensors (name, array)."""
    rng = np.random.default_rng(seed)
    smoothed = ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj",
                "mlp.gate_proj", "mlp.up_proj", "mlp.down_proj")
    out, extras = [], []
    for name, array in tensors:
        base = name[:-len(".weight")] if name.endswith(".weight") else name
        if name.startswith("model.layers.") and base.split(".", 3)[3] in smoothed:
            cols = array.shape[1]
            factors = np.clip(np.exp(rng.standard_normal(cols, dtype=np.float32) * np.float32(0.5)),
                              np.float32(1e-4), np.float32(1e4)).astype(np.float32)
            array = (array * factors[None, :]).astype(np.float32)
            extras.append((base + ".input_scale", (np.float32(1.0) / factors).astype(np.float32)))
            if biases and base.split(".", 3)[3] in smoothed[:3]:
                extras.append((base + ".bias", (rng.standard_normal(array.shape[0], dtype=np.float32)
                                                * np.float32(0.1)).astype(np.float32)))
        out.append((name, array))
    return out, extras


def write_artifact(path: Path, shape: LlamaShape, tensors, bits: int = 8, group_size: int = 64, extras=()):
    """Write the LEAFDC02 artifact the reference exporter writes for these
    tensors at `bits` (8: per-row INT8; 4: INT4 in groups of min(group_size,
    cols)).  `tensors` is an iterable of (name, array) in tensor order;
    `extras` are one-row fp32 tensors (input scales, biases) written after
    them (the reference decoder finds tensors by name)."""
    extras = [(name, np.asarray(array, dtype=np.float32).reshape(-1)) for name, array in extras]
    order = shape.tensor_order() + [(name, 1, array.size) for name, array in extras]
    tensors = list(tensors) + extras
    descriptors, offset = [], 0
    for name, rows, cols in order:
        precision = bits if rows > 1 else 32
        group = cols if precision == 8 else min(group_size, cols) if precision == 4 else 0
        size = rows * cols * precision // 8
        offset = _align64(offset)
        start = offset
        offset += size
        scales = rows * (cols // group) if precision in (4, 8) else 0
        offset = _align64(offset)
        scale_start = offset
        offset += scales * 4
        descriptors.append((name, rows, cols, precision, group, start, size, scale_start, scales))
    metadata = HEADER.size + sum(4 + len(d[0].encode()) + DESCRIPTOR.size for d in descriptors)
    base = _align64(metadata)
    path = Path(path)
    with path.open("wb") as out:
        out.write(HEADER.pack(b"LEAFDC02", 2, len(descriptors), base, *header_values(shape)))
        for name, rows, cols, precision, group, start, size, scale_start, scales in descriptors:
            encoded = name.encode()
            out.write(struct.pack("<I", len(encoded)))
            out.write(encoded)
            out.write(DESCRIPTOR.pack(2, rows, cols, precision, group, start, size, scale_start, scales))
        by_name = {d[0]: d for d in descriptors}
        for name, array in tensors:
            _, rows, cols, precision, group, start, _, scale_start, scales = by_name[name]
            array = np.ascontiguousarray(np.asarray(array, dtype=np.float32).reshape(rows, cols))
            if precision == 32:
                payload, scale_array = array.astype("<f4", copy=False), None
            else:
                payload, scale_array = quantize(array, precision, group)
            out.seek(base + start)
            out.write(payload.tobytes())
            if scales:
                out.seek(base + scale_start)
                out.write(scale_array.tobytes())


def write_snapshot(directory: Path, shape: LlamaShape, tensors) -> None:
    """A Hugging Face snapshot (config.json + one F32 safetensors file) for
    the reference exporter."""
    directory = Path(directory)
    directory.mkdir(parents=True, exist_ok=True)
    (directory / "config.json").write_text(json.dumps(shape.hf_config()))
    entries, payloads, offset = {}, [], 0
    for name, array in tensors:
        data = np.ascontiguousarray(array, dtype="<f4").tobytes()
        entries[name] = {"dtype": "F32", "shape": list(array.shape),
                         "data_offsets": [offset, offset + len(data)]}
        payloads.append(data)
        offset += len(data)
    header = json.dumps(entries).encode()
    with (directory / "model.safetensors").open("wb") as out:
        out.write(struct.pack("<Q", len(header)))
        out.write(header)
        for data in payloads:
            out.write(data)
