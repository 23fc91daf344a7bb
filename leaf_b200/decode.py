"""Persistent decode plans: a chain of per-row W8A8 linears run as one launch.

``DecodePlan([(x, weight, y, wait), ...])`` mirrors the reference forward
loop's sequence of ``linear()`` calls (decoder.cpp:1321-1441): op j reads x
(fp32 [1, cols]) and writes y (fp32 [1, rows]); ``wait`` names the earlier op
whose output x is (or -1 when x is ready before the run).  ``run()`` executes
the whole chain with ``leafq_decode_plan_run`` on the current stream; results
are bit-identical to calling ``leaf_b200.linear`` op by op.
"""
from __future__ import annotations

import ctypes
from typing import Optional, Sequence, Tuple

import torch

from . import _lib
from ._lib import DecodeOp, LeafError, check, load
from .linear import QuantWeight

OpSpec = Tuple[torch.Tensor, QuantWeight, torch.Tensor, int]


class DecodePlan:
    def __init__(self, ops: Sequence[OpSpec], tokens: int = 1):
        if not ops:
            raise LeafError(_lib.LEAFQ_ERR_INVALID, "a decode plan needs at least one op")
        table = (DecodeOp * len(ops))()
        self._keep = []
        for j, (x, w, y, wait) in enumerate(ops):
            if w.bits != 8 or w.group != w.cols:
                raise LeafError(_lib.LEAFQ_ERR_UNSUPPORTED,
                                "decode plans take per-row INT8 weights (group == cols)")
            if x.dtype != torch.float32 or y.dtype != torch.float32 or not x.is_cuda or not y.is_cuda:
                raise LeafError(_lib.LEAFQ_ERR_INVALID, f"op {j}: x and y must be CUDA float32")
            if x.numel() != tokens * w.cols or y.numel() != tokens * w.rows:
                raise LeafError(_lib.LEAFQ_ERR_INVALID, f"op {j}: x/y sizes do not match the weight")
            table[j] = DecodeOp(x.data_ptr(), y.data_ptr(), w.data.data_ptr(), w.scales.data_ptr(),
                                None if w.bias is None else w.bias.data_ptr(), w.rows, w.cols,
                                int(wait), 0)
            self._keep.append((x, w, y))
        self.device = ops[0][0].device
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
