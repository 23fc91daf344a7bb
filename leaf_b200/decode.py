"""Persistent decode plans: a chain of per-row W8A8 linears run as one launch.

A plan mirrors the reference forward loop's sequence of ``linear()`` calls
(decoder.cpp:1321-1441).  Each op is ``DecodeOp(weight, x=..., wait=...,
x_offset=..., y=...)``: its input is either a CUDA fp32 tensor ready before
the run (``x``) or the output of an earlier op (``wait`` = that op's index,
starting at element ``x_offset``); ``y`` optionally receives a plain fp32
copy of the output.  ``run()`` executes the chain with
``leafq_decode_plan_run`` on the current stream; results are bit-identical
to calling ``leaf_b200.linear`` op by op.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Optional, Sequence

import torch

from . import _lib
from ._lib import LeafError, check, load
from .linear import QuantWeight


@dataclass
class DecodeOp:
    weight: QuantWeight
    x: Optional[torch.Tensor] = None
    wait: int = -1
    x_offset: int = 0
    y: Optional[torch.Tensor] = None


class DecodePlan:
    def __init__(self, ops: Sequence[DecodeOp], tokens: int = 1, device=None):
        if not ops:
            raise LeafError(_lib.LEAFQ_ERR_INVALID, "a decode plan needs at least one op")
        table = (_lib.DecodeOp * len(ops))()
        self._keep = []
        for j, op in enumerate(ops):
            w = op.weight
            if w.bits != 8 or w.group != w.cols:
                raise LeafError(_lib.LEAFQ_ERR_UNSUPPORTED,
                                "decode plans take per-row INT8 weights (group == cols)")
            for name, t, n in (("x", op.x, w.cols), ("y", op.y, w.rows)):
                if t is None:
                    continue
                if t.dtype != torch.float32 or not t.is_cuda or not t.is_contiguous():
                    raise LeafError(_lib.LEAFQ_ERR_INVALID, f"op {j}: {name} must be contiguous CUDA float32")
                if t.numel() != tokens * n:
                    raise LeafError(_lib.LEAFQ_ERR_INVALID, f"op {j}: {name} size does not match the weight")
            table[j] = _lib.DecodeOp(None if op.x is None else op.x.data_ptr(),
                                     None if op.y is None else op.y.data_ptr(), w.data.data_ptr(),
                                     w.scales.data_ptr(), None if w.bias is None else w.bias.data_ptr(),
                                     w.rows, w.cols, int(op.wait), int(op.x_offset))
            self._keep.append(op)
        self.device = torch.device(device) if device is not None else ops[0].weight.data.device
        self._handle = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            check(load().leafq_decode_plan_create(ctypes.cast(table, ctypes.c_void_p), len(ops), tokens,
                                                  ctypes.byref(self._handle)))

    def run(self) -> None:
        check(load().leafq_decode_plan_run(torch.cuda.current_stream(self.device).cuda_stream,
                                           self._handle))

    def close(self) -> None:
        if self._handle:
            load().leafq_decode_plan_destroy(self._handle)
            self._handle = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass
