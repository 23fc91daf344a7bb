"""Device-resident W8A8 linear stack of a TinyLlama-1.1B-shaped decoder.

One decode step runs every quantised Linear of one token in the order the
reference's forward loop calls them (decoder.cpp:1321-1441): per layer
q/k/v (one launch over the row-concatenated [q; k; v] matrix -- rows are
independent, so each output is bit-identical to the separate calls), o,
gate/up (one launch over [gate; up]) and down, then lm_head.  Each linear's
input is the previous one's output, so the launches form the same
dependency chain as the decoder's; the non-linear glue between them (norms,
RoPE, attention, SiLU, residuals) is not part of this stack.

The step is captured once into a CUDA graph whose kernels are launched with
programmatic dependent launch, so each GEMV starts streaming its weights
while the previous one finishes.  Weights are read-only inside the step,
which is what makes that overlap valid.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from ._lib import LEAFQ_FLAG_PDL
from .linear import QuantWeight, linear


@dataclass(frozen=True)
class StackShape:
    hidden: int = 2048
    heads: int = 32
    kv_heads: int = 4
    intermediate: int = 5632
    layers: int = 22
    vocab: int = 32000

    @property
    def head_dim(self) -> int:
        return self.hidden // self.heads

    @property
    def qkv_rows(self) -> int:
        return self.hidden + 2 * self.kv_heads * self.head_dim

    def linears(self):
        """(name, rows, cols) of one layer's fused launches, then lm_head."""
        h, f = self.hidden, self.intermediate
        layer = [("qkv", self.qkv_rows, h), ("o", h, h), ("gate_up", 2 * f, h), ("down", h, f)]
        return layer, ("lm_head", self.vocab, h)

    def weight_bytes(self) -> int:
        layer, head = self.linears()
        per_layer = sum(r * c for _, r, c in layer)
        return self.layers * per_layer + head[1] * head[2]

    def scale_bytes(self) -> int:
        layer, head = self.linears()
        return 4 * (self.layers * sum(r for _, r, _ in layer) + head[1])

    def activation_bytes(self, tokens: int = 1) -> int:
        layer, head = self.linears()
        per_layer = sum(4 * tokens * (r + c) for _, r, c in layer)
        return self.layers * per_layer + 4 * tokens * (head[1] + head[2])

    def step_bytes(self, tokens: int = 1) -> int:
        """Algorithmic HBM bytes of one step: every weight byte, scale and
        activation read or written once."""
        return self.weight_bytes() + self.scale_bytes() + self.activation_bytes(tokens)


def random_w8_weight(rows: int, cols: int, generator: torch.Generator, device) -> QuantWeight:
    """Per-row INT8 weight quantised from N(0, 0.02) with the exporter's
    formula (tools/export_decoder.py:91-105), generated on the device."""
    w = torch.randn((rows, cols), generator=generator, device=device, dtype=torch.float32) * 0.02
    scale = torch.clamp(w.abs().amax(dim=1, keepdim=True) / 127.0, min=1e-12)
    codes = torch.clamp(torch.round(w / scale), -127, 127).to(torch.int8)
    del w
    return QuantWeight(codes.contiguous(), scale.contiguous(), rows, cols, 8, cols)


class LinearStack:
    """All W8A8 linears of one decode step, replayable as a CUDA graph."""

    def __init__(self, shape: StackShape = StackShape(), tokens: int = 1, seed: int = 0,
                 device="cuda"):
        self.shape = shape
        self.tokens = tokens
        self.device = torch.device(device)
        gen = torch.Generator(device=self.device)
        gen.manual_seed(seed)
        layer, head = shape.linears()
        self.layers = [{name: random_w8_weight(r, c, gen, self.device) for name, r, c in layer}
                       for _ in range(shape.layers)]
        self.lm_head = random_w8_weight(head[1], head[2], gen, self.device)
        t, h, f = tokens, shape.hidden, shape.intermediate
        self.x = torch.randn((t, h), generator=gen, device=self.device, dtype=torch.float32)
        self.qkv = torch.empty((t, shape.qkv_rows), device=self.device)
        self.attn = torch.empty((t, h), device=self.device)
        self.o = torch.empty((t, h), device=self.device)
        self.gate_up = torch.empty((t, 2 * f), device=self.device)
        self.up = torch.empty((t, f), device=self.device)
        self.down = torch.empty((t, h), device=self.device)
        self.logits = torch.empty((t, shape.vocab), device=self.device)
        self.graph = None

    def launches_per_step(self, persistent: bool = True) -> int:
        return 1 if persistent else 4 * self.shape.layers + 1

    def plan_ops(self):
        """The step as a decode-plan chain (same dependencies as _step)."""
        from .decode import DecodeOp

        f = self.shape.intermediate
        ops = []
        for i, layer in enumerate(self.layers):
            base = len(ops)
            if i == 0:
                ops.append(DecodeOp(layer["qkv"], x=self.x))
            else:
                ops.append(DecodeOp(layer["qkv"], wait=base - 1))
            ops.append(DecodeOp(layer["o"], wait=base))                    # q slice of q|k|v
            ops.append(DecodeOp(layer["gate_up"], wait=base + 1))
            ops.append(DecodeOp(layer["down"], wait=base + 2, x_offset=f))  # up half of gate|up
        ops.append(DecodeOp(self.lm_head, wait=len(ops) - 1, y=self.logits))
        return ops

    def run_persistent(self) -> torch.Tensor:
        """One step as a single persistent launch (the bench path)."""
        from .decode import DecodePlan

        if getattr(self, "plan", None) is None:
            if self.tokens != 1:
                raise ValueError("the persistent decode kernel runs one token per step")
            self.plan = DecodePlan(self.plan_ops())
        self.plan.run()
        return self.logits

    def capture_persistent(self) -> None:
        self.run_persistent()  # plan creation and kernel attributes outside capture
        torch.cuda.synchronize(self.device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.plan.run()
        torch.cuda.synchronize(self.device)

    def _step(self, flags: int) -> None:
        h, f = self.shape.hidden, self.shape.intermediate
        x = self.x
        for layer in self.layers:
            linear(x, layer["qkv"], out=self.qkv, flags=flags)
            # The attention output has the query width; the chain feeds the
            # query slice forward in its place.  With one token the slice is
            # already contiguous memory; with several it is gathered first.
            a_in = self.qkv[:, :h]
            if self.tokens > 1:
                self.attn.copy_(a_in)
                a_in = self.attn
            linear(a_in, layer["o"], out=self.o, flags=flags)
            linear(self.o, layer["gate_up"], out=self.gate_up, flags=flags)
            u_in = self.gate_up[:, f:]
            if self.tokens > 1:
                self.up.copy_(u_in)
                u_in = self.up
            linear(u_in, layer["down"], out=self.down, flags=flags)
            x = self.down
        linear(x, self.lm_head, out=self.logits, flags=flags)

    def run_eager(self, pdl: bool = True) -> torch.Tensor:
        self._step(LEAFQ_FLAG_PDL if pdl else 0)
        return self.logits

    def capture(self, pdl: bool = True) -> None:
        self.run_eager(pdl)  # first calls set kernel attributes outside capture
        torch.cuda.synchronize(self.device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self._step(LEAFQ_FLAG_PDL if pdl else 0)
        torch.cuda.synchronize(self.device)

    def replay(self) -> torch.Tensor:
        if self.graph is None:
            self.capture()
        self.graph.replay()
        return self.logits


class _DeviceTensor:
    """One tensor of a device-resident model in artifact layout."""

    def __init__(self, name, rows, cols, bits, group, data, scales):
        self.name, self.rows, self.cols, self.bits, self.group = name, rows, cols, bits, group
        self.data, self.scales = data, scales


class RandomDecoderModel:
    """A Llama-shaped W8A8 decoder with random weights generated on the GPU,
    with the ``config`` / ``get(name)`` interface of ``leaf_b200.artifact.Artifact``:
    weights N(0, 0.02) quantised per row by the exporter's formula
    (tools/export_decoder.py:91-105), embedding and lm_head per-row INT8,
    RMSNorm weights 1, no EOS."""

    def __init__(self, shape: StackShape, seed: int = 0, max_positions: int = 2048, device="cuda"):
        from .artifact import DecoderConfig

        h, f, heads, kv = shape.hidden, shape.intermediate, shape.heads, shape.kv_heads
        d = h // heads
        self.config = DecoderConfig(h, f, heads, kv, shape.layers, shape.vocab, max_positions,
                                    0xFFFFFFFF, d, 0, 10000.0, float(np.float32(1e-5)), 0, 0, 0, 1, 0, d,
                                    0, 1, 1.0)
        gen = torch.Generator(device=device)
        gen.manual_seed(seed)
        self._tensors = {}

        def mat(name, rows, cols):
            w = random_w8_weight(rows, cols, gen, device)
            self._tensors[name] = _DeviceTensor(name, rows, cols, 8, cols, w.data, w.scales.reshape(rows, 1))

        def norm(name):
            self._tensors[name] = _DeviceTensor(name, 1, h, 32, 0,
                                                torch.ones((1, h), dtype=torch.float32, device=device), None)

        mat("model.embed_tokens.weight", shape.vocab, h)
        mat("lm_head.weight", shape.vocab, h)
        norm("model.norm.weight")
        for i in range(shape.layers):
            p = f"model.layers.{i}."
            norm(p + "input_layernorm.weight")
            norm(p + "post_attention_layernorm.weight")
            mat(p + "self_attn.q_proj.weight", heads * d, h)
            mat(p + "self_attn.k_proj.weight", kv * d, h)
            mat(p + "self_attn.v_proj.weight", kv * d, h)
            mat(p + "self_attn.o_proj.weight", h, heads * d)
            mat(p + "mlp.gate_proj.weight", f, h)
            mat(p + "mlp.up_proj.weight", f, h)
            mat(p + "mlp.down_proj.weight", h, f)

    def get(self, name):
        return self._tensors.get(name)

    def release(self) -> None:
        """Drop the per-matrix copies once a Decoder has fused them."""
        self._tensors.clear()


def decoder_step_bytes(shape: StackShape, position: int) -> int:
    """Algorithmic HBM bytes of one whole-model decode step at cache length
    `position`: every INT8 weight and row scale once, the embedding row, the
    norm weights, the cached keys and values read (positions 0..position-1)
    and this token's written, the hand-off vectors and the logits."""
    h, f, heads, kv, layers = shape.hidden, shape.intermediate, shape.heads, shape.kv_heads, shape.layers
    d = h // heads
    layer, head = shape.linears()
    weights = layers * sum(r * c + 4 * r for _, r, c in layer) + head[1] * (head[2] + 4)
    embed = h + 4
    norms = 4 * h * (2 * layers + 1)
    kv_bytes = layers * 2 * kv * d * 4 * (position + 1)
    handoff = layers * 8 * (shape.qkv_rows + h + h + f + h)
    return weights + embed + norms + kv_bytes + handoff + 4 * shape.vocab
