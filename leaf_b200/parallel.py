"""N-sharded quantised linear over one process per GPU (tensor parallel along N).

Every output row of a Leaf linear is independent: the reference splits the
rows of one call into grains of 32 over its worker threads
(decoder.cpp:1109, host_support.h:151-178) and each row's int32 dot and fp32
epilogue touch only that row.  Splitting the rows over GPUs is therefore
bit-exact for any GPU count: rank g owns rows [g*N//G, (g+1)*N//G) of every
weight, quantises the full activation row itself (absmax is order-free, so
every rank derives the identical token scale), runs its slice through
``leafq_linear`` and the slices are all-gathered along N.

``RowShards`` is the partition, ``shard_host_weight`` cuts an artifact-layout
weight to one rank's rows, ``RowGather`` reassembles [tokens, N] from the
per-rank [tokens, n_g] slices with one all-gather (NCCL on GPUs, gloo on CPU),
and ``ShardedLinear`` is the operator.  The peer-memory all-gather without
NCCL is ``leafq_allgather_*`` in the C ABI (``PeerAllGather`` below).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Optional

import numpy as np
import torch
import torch.distributed as dist

from . import _lib
from ._lib import LeafError, check, load
from .linear import QuantWeight, Workspace, _ptr, _require_cuda, _stream, linear


@dataclass(frozen=True)
class RowShards:
    """Contiguous split of `rows` output rows over `world` ranks."""

    rows: int
    world: int

    def __post_init__(self):
        if self.world < 1 or self.rows < 0:
            raise LeafError(_lib.LEAFQ_ERR_INVALID, "invalid row partition")

    def begin(self, rank: int) -> int:
        return rank * self.rows // self.world

    def end(self, rank: int) -> int:
        return (rank + 1) * self.rows // self.world

    def count(self, rank: int) -> int:
        return self.end(rank) - self.begin(rank)

    @property
    def widest(self) -> int:
        return max(self.count(r) for r in range(self.world))

    @property
    def even(self) -> bool:
        return self.rows % self.world == 0


def shard_host_weight(data, scales, bias, rows: int, cols: int, bits: int, group: int,
                      rank: int, world: int):
    """One rank's rows of a weight in the reference artifact layout
    (export_decoder.py:91-105): INT8 [rows, cols], INT4 [rows, cols/2],
    fp32 [rows, cols]; scales [rows, cols/group]; bias [rows].  Returns
    (data, scales, bias, begin, end) as contiguous numpy arrays."""
    part = RowShards(rows, world)
    b, e = part.begin(rank), part.end(rank)
    width = {8: cols, 4: cols // 2, 32: cols}[bits]
    d = np.ascontiguousarray(np.asarray(data).reshape(rows, width)[b:e])
    s = None
    if scales is not None:
        s = np.ascontiguousarray(np.asarray(scales).reshape(rows, -1)[b:e])
    bb = None if bias is None else np.ascontiguousarray(np.asarray(bias).reshape(rows)[b:e])
    return d, s, bb, b, e


class RowGather:
    """All-gather of per-rank [tokens, n_g] slices into [tokens, rows].

    With one token and rows divisible by the world size the slices land in
    the output directly (one collective, no copy).  Otherwise every rank
    sends a [tokens, widest] block (padded) and the blocks are placed by row
    range after the collective."""

    def __init__(self, rows: int, group=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.part = RowShards(rows, self.world)

    def __call__(self, local: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        part = self.part
        tokens = local.shape[0]
        if local.shape != (tokens, part.count(self.rank)):
            raise LeafError(_lib.LEAFQ_ERR_INVALID, "local slice does not match the partition")
        if out is None:
            out = torch.empty((tokens, part.rows), dtype=local.dtype, device=local.device)
        if tokens == 1 and part.even:
            dist.all_gather_into_tensor(out.view(-1), local.contiguous().view(-1), group=self.group)
            return out
        w = part.widest
        send = torch.zeros((tokens, w), dtype=local.dtype, device=local.device)
        send[:, : local.shape[1]] = local
        buf = torch.empty((self.world, tokens, w), dtype=local.dtype, device=local.device)
        dist.all_gather_into_tensor(buf.view(-1), send.view(-1), group=self.group)
        for r in range(self.world):
            out[:, part.begin(r):part.end(r)] = buf[r, :, : part.count(r)]
        return out


class PeerAllGather:
    """The C ABI's peer-memory all-gather (``leafq_allgather_*``) on a process
    group of one process per GPU.

    Creation is collective: every rank allocates its receive buffer for up to
    `max_elements` gathered floats and the CUDA IPC handles are exchanged
    over the group.  Every rank must then make the same sequence of
    ``run`` / ``linear`` calls (same tokens and rows); they may be captured
    in a CUDA graph.  ``close`` is collective too."""

    def __init__(self, max_elements: int, group=None):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.device = torch.device("cuda", torch.cuda.current_device())
        self.max_elements = int(max_elements)
        lib = load()
        handle = (ctypes.c_uint8 * _lib.LEAFQ_IPC_HANDLE_BYTES)()
        ag = ctypes.c_void_p()
        check(lib.leafq_allgather_init(self.rank, self.world, self.max_elements, ctypes.byref(ag),
                                       handle))
        self._ag = ag
        on = self.device if dist.get_backend(group) == "nccl" else torch.device("cpu")
        mine = torch.tensor(list(bytes(handle)), dtype=torch.uint8, device=on)
        every = torch.empty(self.world * _lib.LEAFQ_IPC_HANDLE_BYTES, dtype=torch.uint8, device=on)
        dist.all_gather_into_tensor(every, mine, group=group)
        table = (ctypes.c_uint8 * every.numel())(*every.cpu().tolist())
        check(lib.leafq_allgather_connect(self._ag, table))

    def run(self, local: torch.Tensor, row_begin: int, rows: int,
            out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Gather [tokens, local_rows] slices (this rank's at row_begin) into
        [tokens, rows] on every rank."""
        _require_cuda(local, "local rows")
        tokens, local_rows = local.shape
        if out is None:
            out = torch.empty((tokens, rows), dtype=torch.float32, device=local.device)
        check(load().leafq_allgather_run(_stream(local.device), self._ag, local.data_ptr(), tokens,
                                         local_rows, row_begin, rows, out.data_ptr()))
        return out

    def linear(self, x: torch.Tensor, shard: QuantWeight, row_begin: int, rows: int,
               activation_bits: int = 8, out: Optional[torch.Tensor] = None,
               workspace: Optional[Workspace] = None, flags: int = 0) -> torch.Tensor:
        """This rank's rows of the linear, gathered into [tokens, rows] on
        every rank; the decode GEMV stores into the peers from its epilogue."""
        _require_cuda(x, "input")
        if x.dtype != torch.float32 or x.dim() != 2 or x.shape[1] != shard.cols:
            raise LeafError(_lib.LEAFQ_ERR_INVALID, "input must be float32 [tokens, cols]")
        if shard.input_scale is not None:  # decoder.cpp:1008-1019
            scaled = torch.empty_like(x)
            check(load().leafq_scale_columns(_stream(x.device), x.contiguous().data_ptr(), x.shape[0], shard.cols,
                                             shard.input_scale.data_ptr(), scaled.data_ptr()))
            x = scaled
        tokens = x.shape[0]
        if out is None:
            out = torch.empty((tokens, rows), dtype=torch.float32, device=x.device)
        lib = load()
        need = lib.leafq_linear_workspace_bytes(tokens, shard.cols, shard.bits, shard.group,
                                                activation_bits)
        ws_ptr, ws_bytes = None, 0
        if need:
            workspace = workspace or Workspace(x.device)
            buf = workspace.get(need)
            ws_ptr, ws_bytes = buf.data_ptr(), buf.numel()
        check(lib.leafq_linear_allgather(
            _stream(x.device), self._ag, x.data_ptr(), tokens, shard.cols, shard.data.data_ptr(),
            _ptr(shard.scales), shard.rows, row_begin, rows, shard.bits, shard.group,
            activation_bits, _ptr(shard.bias), out.data_ptr(), ws_ptr, ws_bytes, flags))
        return out

    def close(self) -> None:
        if self._ag is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)  # no rank may still store into a buffer being freed
        check(load().leafq_allgather_destroy(self._ag))
        self._ag = None


class ShardedLinear:
    """``Decoder::Impl::linear`` for one weight, N-sharded over a process group.

    Each rank holds rows [begin, end) of the weight on its own GPU; ``__call__``
    takes the full activation [tokens, cols] on every rank and returns the
    full output [tokens, rows] on every rank, bit-identical to the unsharded
    call.  The gather is an NCCL all-gather (``RowGather``) or, given a
    ``PeerAllGather``, the C ABI's peer-memory gather fused into the kernel."""

    def __init__(self, shard: QuantWeight, rows: int, activation_bits: int = 8, group=None,
                 peer: Optional[PeerAllGather] = None):
        self.gather = RowGather(rows, group)
        rank = self.gather.rank
        if shard.rows != self.gather.part.count(rank):
            raise LeafError(_lib.LEAFQ_ERR_INVALID, "weight shard does not match the partition")
        self.shard = shard
        self.rows = rows
        self.cols = shard.cols
        self.row_begin = self.gather.part.begin(rank)
        self.activation_bits = activation_bits
        self.peer = peer
        self.workspace = Workspace(shard.data.device)

    @classmethod
    def from_host(cls, data, scales, rows, cols, bits, group_size, bias=None, input_scale=None,
                  activation_bits: int = 8, group=None, device="cuda",
                  peer: Optional[PeerAllGather] = None):
        """Cut the full artifact-layout weight to this rank's rows and upload them."""
        world, rank = dist.get_world_size(group), dist.get_rank(group)
        d, s, b, lo, hi = shard_host_weight(data, scales, bias, rows, cols, bits, group_size,
                                            rank, world)
        shard = QuantWeight.from_host(d, s, hi - lo, cols, bits, group_size, b, input_scale,
                                      device=device)
        shard.check()
        return cls(shard, rows, activation_bits, group, peer)

    def __call__(self, x: torch.Tensor, out: Optional[torch.Tensor] = None,
                 flags: int = 0) -> torch.Tensor:
        if self.peer is not None:
            return self.peer.linear(x, self.shard, self.row_begin, self.rows, self.activation_bits,
                                    out=out, workspace=self.workspace, flags=flags)
        local = linear(x, self.shard, self.activation_bits, workspace=self.workspace, flags=flags)
        return self.gather(local, out)
