"""Host-side mirror of Leaf's quantised-linear operator interface.

The reference keeps its weights in a mapped artifact and runs
``Decoder::Impl::linear(input, tokens, name, output)`` (decoder.cpp:994-1233)
for a weight looked up by name, raising ``std::runtime_error("Leaf decoder:
...")`` on bad input.  ``QuantLinearSet`` keeps the same contract over
device-resident weights: ``linear(x, name)`` looks up ``name.weight``,
``name.bias`` and ``name.input_scale`` and runs the leafq C ABI on the current
CUDA stream.  PyTorch tensors are only containers for device memory and the
stream; every arithmetic step runs in libleafq.so.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch

from . import _lib
from ._lib import LeafError, check, load

_ALIGN = 256


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _require_cuda(t: torch.Tensor, name: str) -> None:
    if not t.is_cuda:
        raise LeafError(_lib.LEAFQ_ERR_INVALID, f"{name} must be a CUDA tensor")
    if not t.is_contiguous():
        raise LeafError(_lib.LEAFQ_ERR_INVALID, f"{name} must be contiguous")


@dataclass
class QuantWeight:
    """One quantised matrix in the reference's Weight layout (decoder.cpp:236-251).

    data: int8 [rows, cols] (bits 8), uint8 [rows, cols / 2] (bits 4, low
    nibble = even column) or float32 [rows, cols] (bits 32); scales: float32
    [rows, cols / group] (None for bits 32).
    """

    data: torch.Tensor
    scales: Optional[torch.Tensor]
    rows: int
    cols: int
    bits: int
    group: int
    bias: Optional[torch.Tensor] = None
    input_scale: Optional[torch.Tensor] = None

    @classmethod
    def from_host(cls, data, scales, rows, cols, bits, group, bias=None, input_scale=None,
                  device="cuda"):
        """Upload a weight in artifact layout (numpy arrays or tensors)."""
        def up(a, dtype):
            if a is None:
                return None
            t = torch.as_tensor(a)
            if dtype is not None:
                t = t.view(dtype) if t.dtype.itemsize == dtype.itemsize else t.to(dtype)
            return t.contiguous().to(device)
        dtype = {8: torch.int8, 4: torch.uint8, 32: torch.float32}[bits]
        return cls(up(data, dtype), up(scales, torch.float32), rows, cols, bits,
                   group if bits != 32 else 0, up(bias, torch.float32),
                   up(input_scale, torch.float32))

    def check(self) -> None:
        expected = {8: self.rows * self.cols, 4: self.rows * self.cols // 2,
                    32: self.rows * self.cols}[self.bits]
        if self.data.numel() * self.data.element_size() != expected * (4 if self.bits == 32 else 1):
            raise LeafError(_lib.LEAFQ_ERR_INVALID, "invalid tensor data range")
        if self.bits != 32:
            if self.group <= 0 or self.cols % self.group:
                raise LeafError(_lib.LEAFQ_ERR_INVALID, "invalid quantization metadata")
            if self.scales is None or self.scales.numel() != self.rows * (self.cols // self.group):
                raise LeafError(_lib.LEAFQ_ERR_INVALID, "invalid quantization metadata")
        if self.bias is not None and self.bias.numel() != self.rows:
            raise LeafError(_lib.LEAFQ_ERR_INVALID, "incompatible linear bias")
        if self.input_scale is not None and self.input_scale.numel() != self.cols:
            raise LeafError(_lib.LEAFQ_ERR_INVALID, "incompatible calibrated input scale")


class Workspace:
    """Caller-owned device scratch for the two-kernel linear paths (codes and
    token scales).  Grown on demand outside the hot path; reuse it across
    calls on one stream."""

    def __init__(self, device="cuda"):
        self.device = torch.device(device)
        self.buffer = torch.empty(0, dtype=torch.uint8, device=self.device)

    def get(self, nbytes: int) -> torch.Tensor:
        if nbytes > self.buffer.numel():
            self.buffer = torch.empty(max(nbytes, 2 * self.buffer.numel()), dtype=torch.uint8,
                                      device=self.device)
        return self.buffer


def quantize_act(x: torch.Tensor):
    """Per-token dynamic INT8 quantisation (decoder.cpp:1028-1038).
    Returns (codes int8 [tokens, cols], scales float32 [tokens])."""
    _require_cuda(x, "input")
    if x.dtype != torch.float32 or x.dim() != 2:
        raise LeafError(_lib.LEAFQ_ERR_INVALID, "input must be float32 [tokens, cols]")
    tokens, cols = x.shape
    q = torch.empty((tokens, cols), dtype=torch.int8, device=x.device)
    sx = torch.empty(tokens, dtype=torch.float32, device=x.device)
    check(load().leafq_quantize_act(_stream(x.device), x.data_ptr(), tokens, cols, q.data_ptr(),
                                    sx.data_ptr()))
    return q, sx


def linear(x: torch.Tensor, weight: QuantWeight, activation_bits: int = 8,
           out: Optional[torch.Tensor] = None, workspace: Optional[Workspace] = None,
           flags: int = 0) -> torch.Tensor:
    """y[tokens, rows] = quantised linear of x[tokens, cols] -- the body of
    Decoder::Impl::linear for one weight (SmoothQuant pre-scale, quantise,
    integer or weight-only dot, bias)."""
    _require_cuda(x, "input")
    if x.dtype != torch.float32 or x.dim() != 2 or x.shape[1] != weight.cols:
        raise LeafError(_lib.LEAFQ_ERR_INVALID, "input must be float32 [tokens, cols]")
    tokens = x.shape[0]
    if out is None:
        out = torch.empty((tokens, weight.rows), dtype=torch.float32, device=x.device)
    lib = load()
    if weight.input_scale is not None:
        # decoder.cpp:1008-1019: x * input_scale (one IEEE multiply per
        # element), fused into the quantiser.
        need = lib.leafq_linear_smooth_workspace_bytes(tokens, weight.cols, activation_bits)
        buf = (workspace or Workspace(x.device)).get(need)
        check(lib.leafq_linear_smooth(_stream(x.device), x.data_ptr(), weight.input_scale.data_ptr(), tokens,
                                      weight.cols, weight.data.data_ptr(), _ptr(weight.scales), weight.rows,
                                      weight.bits, weight.group, activation_bits, _ptr(weight.bias),
                                      out.data_ptr(), buf.data_ptr(), buf.numel(), flags))
        return out
    need = lib.leafq_linear_workspace_bytes(tokens, weight.cols, weight.bits, weight.group,
                                            activation_bits)
    ws_ptr, ws_bytes = None, 0
    if need:
        workspace = workspace or Workspace(x.device)
        buf = workspace.get(need)
        ws_ptr, ws_bytes = buf.data_ptr(), buf.numel()
    check(lib.leafq_linear(_stream(x.device), x.data_ptr(), tokens, weight.cols,
                           weight.data.data_ptr(), _ptr(weight.scales), weight.rows, weight.bits,
                           weight.group, activation_bits, _ptr(weight.bias), out.data_ptr(), ws_ptr,
                           ws_bytes, flags))
    return out


def linear_int_q(q: torch.Tensor, sx: torch.Tensor, weight: QuantWeight, want_acc: bool = False,
                 flags: int = 0):
    """Integer linear from codes; optionally returns the int32 group sums
    [tokens, rows, groups] the reference accumulates."""
    _require_cuda(q, "codes")
    tokens, cols = q.shape
    y = torch.empty((tokens, weight.rows), dtype=torch.float32, device=q.device)
    acc = None
    if want_acc:
        acc = torch.empty((tokens, weight.rows, cols // weight.group), dtype=torch.int32,
                          device=q.device)
    check(load().leafq_linear_int_q(_stream(q.device), q.data_ptr(), sx.data_ptr(), tokens, cols,
                                    weight.data.data_ptr(), _ptr(weight.scales), weight.rows,
                                    weight.bits, weight.group, _ptr(weight.bias), y.data_ptr(),
                                    _ptr(acc), flags))
    return (y, acc) if want_acc else y


def graph_quantize(x: torch.Tensor, scale: float):
    """Static INT8 quantiser of the graph executor (executor.cpp:220-230).
    Raises like the reference when the input holds a non-finite value."""
    _require_cuda(x, "input")
    q = torch.empty(x.shape, dtype=torch.int8, device=x.device)
    flag = torch.zeros(1, dtype=torch.int32, device=x.device)
    check(load().leafq_graph_quantize(_stream(x.device), x.data_ptr(), x.numel(), float(scale),
                                      q.data_ptr(), flag.data_ptr()))
    if int(flag.item()) != 0:
        raise LeafError(_lib.LEAFQ_ERR_NONFINITE, "INT8 input contains a non-finite value")
    return q


def gemm_i8_per_channel(a: torch.Tensor, b: torch.Tensor, bias: Optional[torch.Tensor],
                        input_scale: float, weight_scales: torch.Tensor, relu: bool = False):
    """leaf::kernels::gemm_i8_per_channel: a int8 [m, k], b int8 [k, n]."""
    _require_cuda(a, "a")
    _require_cuda(b, "b")
    m, k = a.shape
    n = b.shape[1]
    out = torch.empty((m, n), dtype=torch.float32, device=a.device)
    check(load().leafq_gemm_i8_per_channel(_stream(a.device), a.data_ptr(), b.data_ptr(), _ptr(bias),
                                           float(input_scale), weight_scales.data_ptr(),
                                           out.data_ptr(), m, k, n, 1 if relu else 0))
    return out


_ACTIVATIONS = {None: 0, "": 0, "Relu": 1, "Silu": 2, "Gelu": 3}


def graph_linear(a: torch.Tensor, weight: torch.Tensor, weight_scales: torch.Tensor, input_scale: float,
                 op_type: str = "Gemm", trans_a: bool = False, trans_b: bool = False, alpha: float = 1.0,
                 beta: float = 1.0, c: Optional[torch.Tensor] = None, activation: Optional[str] = None):
    """A quantised Gemm / MatMul node of the graph executor
    (execute_quant_linear, executor.cpp:524-614) on the GPU.

    a: fp32 input ([..., k]; [k, m] with trans_a, Gemm only); weight: int8
    initializer [k, n] ([n, k] with trans_b); weight_scales: fp32 [n];
    c: the Gemm's optional third input (one value, [n] or the output shape).
    MatMul nodes ignore alpha / beta / C as the reference does.  Raises like
    the reference on a non-finite input or an unsupported broadcast."""
    _require_cuda(a, "input")
    _require_cuda(weight, "weight")
    gemm = op_type == "Gemm"
    if not gemm:
        trans_a = trans_b = False
        alpha, beta, c = 1.0, 0.0, None
    if a.dim() < 2:
        raise LeafError(_lib.LEAFQ_ERR_INVALID, "INT8 linear input must be a matrix or batched matrix")
    if trans_a and a.dim() != 2:
        raise LeafError(_lib.LEAFQ_ERR_INVALID, "batched INT8 Gemm transA is unsupported")
    if weight.dim() != 2 or weight.dtype != torch.int8:
        raise LeafError(_lib.LEAFQ_ERR_INVALID, "INT8 linear weight must be a rank-2 initializer")
    m = a.shape[1] if trans_a else a.numel() // a.shape[-1]
    k = a.shape[0] if trans_a else a.shape[-1]
    n = weight.shape[0] if trans_b else weight.shape[1]
    if (weight.shape[1] if trans_b else weight.shape[0]) != k:
        raise LeafError(_lib.LEAFQ_ERR_INVALID, "INT8 linear K dimensions do not match")
    if weight_scales.numel() != n:
        raise LeafError(_lib.LEAFQ_ERR_INVALID, "INT8 weight scales do not match output channels")
    out_shape = (m, n) if trans_a else tuple(a.shape[:-1]) + (n,)
    c_kind = 0
    if c is not None:
        _require_cuda(c, "C")
        if c.numel() == 1:
            c_kind = 1
        elif c.dim() == 1 and c.shape[0] == n:
            c_kind = 2
        elif tuple(c.shape) == out_shape:
            c_kind = 3
        else:
            raise LeafError(_lib.LEAFQ_ERR_INVALID, "unsupported INT8 Gemm C broadcast shape")
        c = c.to(torch.float32).contiguous()
    if activation not in _ACTIVATIONS:
        raise LeafError(_lib.LEAFQ_ERR_INVALID, f"leaf::Executor: unsupported fused activation: {activation}")
    a = a.to(torch.float32).contiguous()
    out = torch.empty(out_shape, dtype=torch.float32, device=a.device)
    lib = load()
    ws = torch.empty(max(lib.leafq_graph_linear_workspace_bytes(m, k), 1), dtype=torch.uint8, device=a.device)
    flag = torch.zeros(1, dtype=torch.int32, device=a.device)
    check(lib.leafq_graph_linear(_stream(a.device), a.data_ptr(), m, k, int(trans_a), weight.data_ptr(), n,
                                 int(trans_b), float(input_scale), weight_scales.contiguous().data_ptr(),
                                 float(alpha), float(beta), _ptr(c), c_kind, _ACTIVATIONS[activation],
                                 out.data_ptr(), ws.data_ptr(), ws.numel(), flag.data_ptr()))
    if int(flag.item()) != 0:
        raise LeafError(_lib.LEAFQ_ERR_NONFINITE, "INT8 input contains a non-finite value")
    return out


class QuantLinearSet:
    """Named quantised linears, looked up like Decoder::Impl::weights.

    ``linear(x, "model.layers.0.mlp.up_proj")`` finds ``<name>.weight`` (and
    its bias / input_scale) and returns y [tokens, rows]."""

    def __init__(self, activation_bits: int = 8, device="cuda"):
        if activation_bits not in (8, 32):
            raise LeafError(_lib.LEAFQ_ERR_INVALID, "activation bits must be 8 or 32")
        self.activation_bits = activation_bits
        self.device = torch.device(device)
        self.weights: dict[str, QuantWeight] = {}
        self.workspace = Workspace(self.device)

    def add(self, name: str, weight: QuantWeight) -> None:
        weight.check()
        if name in self.weights:
            raise LeafError(_lib.LEAFQ_ERR_INVALID, f"duplicate tensor {name}.weight")
        self.weights[name] = weight

    def linear(self, x: torch.Tensor, name: str, out: Optional[torch.Tensor] = None,
               flags: int = 0) -> torch.Tensor:
        weight = self.weights.get(name)
        if weight is None:
            raise LeafError(_lib.LEAFQ_ERR_INVALID, f"missing or incompatible tensor {name}.weight")
        return linear(x, weight, self.activation_bits, out=out, workspace=self.workspace,
                      flags=flags)
