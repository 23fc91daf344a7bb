"""GPU port of Leaf's decoder (``leaf::runtime::Decoder``, decoder.h) for
Llama-family artifacts with quantised linears.

``Decoder(artifact).forward(ids)`` follows ``Impl::forward_into``
(decoder.cpp:1282-1452) op for op: embedding, per layer RMSNorm -> q|k|v ->
RoPE + KV append -> attention -> o -> residual + RMSNorm -> gate|up -> SiLU
gate -> down -> residual (+ next RMSNorm), final RMSNorm, lm_head on the last
row.  Every linear is ``leafq_linear`` (W8A8 / W4A8 with activation_bits 8,
weight-only with 32); the other operators are the library's decoder kernels.
q, k and v run as one linear over their stacked rows, gate and up as one
linear over their interleaved rows (gate_0, up_0, gate_1, ...) -- rows are
independent, so the outputs are bit-identical to the separate calls the
reference makes.  ``generate`` is the greedy loop of
main_decoder.cpp:95-113: one prefill forward, then one CUDA-graph replay per
token with the argmax, the next embedding and the position update on the
device (no host round trip per token).

Supported artifacts: RMSNorm, RoPE, gated SiLU, sequential residual, no
sliding window, no Q/K norm (the Llama / Mistral-without-window / Qwen2
family); anything else raises.  Linear biases (q / k / v in Qwen2 exports) are
added in the linears' epilogues; SmoothQuant input scales
(``<proj>.input_scale``, decoder.cpp:1008-1019) are applied inside each
projection's quantiser, which runs q / k / v and gate / up as separate
linears (their inputs are scaled differently).  Such artifacts take the
per-operator path; the one-launch step needs the plain per-row INT8 export.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import numpy as np
import torch

from . import _lib
from ._lib import LEAFQ_FLAG_PDL, LeafError, check, load
from .artifact import Artifact, HostTensor
from .linear import QuantWeight, Workspace


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _on(a, device: torch.device) -> torch.Tensor:
    """A payload (numpy view of the mapped artifact, or a tensor) on the device."""
    if isinstance(a, torch.Tensor):
        return a.to(device)
    return torch.from_numpy(np.array(a)).to(device)


def _concat_rows(parts: list[HostTensor], device: torch.device, interleave: bool = False,
                 biases=None, input_scale=None) -> QuantWeight:
    """Rows of several equally quantised matrices as one weight: stacked
    (q | k | v) or, with interleave, alternating (gate_0, up_0, gate_1, ...).
    biases: one HostTensor or None per part (a missing bias adds 0.0f, as the
    reference's output = result + 0 would not: only parts with a bias get
    one, so a stack mixing both is rejected); input_scale: the calibrated
    SmoothQuant factors of a single part."""
    bits, group, cols = parts[0].bits, parts[0].group, parts[0].cols
    if any(p.bits != bits or p.group != group or p.cols != cols for p in parts):
        raise LeafError(_lib.LEAFQ_ERR_UNSUPPORTED, "fused projections need one precision and group")
    datas = [_on(p.data, device) for p in parts]
    scales = None if bits == 32 else [_on(p.scales, device) for p in parts]
    if interleave:
        data = torch.stack(datas, dim=1).reshape(-1, datas[0].shape[1])
        scales = None if scales is None else torch.stack(scales, dim=1).reshape(-1, scales[0].shape[1])
    else:
        data = torch.cat(datas, dim=0)
        scales = None if scales is None else torch.cat(scales, dim=0)
    rows = sum(p.rows for p in parts)
    bias = None
    if biases is not None and any(b is not None for b in biases):
        if any(b is None for b in biases):
            raise LeafError(_lib.LEAFQ_ERR_UNSUPPORTED, "stacked projections with and without biases")
        vecs = [_on(b.data, device).to(torch.float32).reshape(-1) for b in biases]
        bias = (torch.stack(vecs, dim=1).reshape(-1) if interleave else torch.cat(vecs)).contiguous()
    scale = None if input_scale is None else _on(input_scale.data, device).to(torch.float32).reshape(-1).contiguous()
    w = QuantWeight(data.contiguous(), None if scales is None else scales.contiguous(), rows, cols, bits,
                    group if bits != 32 else 0, bias, scale)
    w.check()
    return w


class Decoder:
    def __init__(self, artifact, activation_bits: int = 8, device="cuda",
                 capacity: Optional[int] = None, sequences: int = 1, group=None,
                 gather: str = "nccl"):
        """artifact: a path, an ``Artifact``, or any object with the same
        ``config`` / ``get(name)`` interface whose payloads are tensors
        (``leaf_b200.stack.RandomDecoderModel``).

        sequences > 1 decodes that many independent requests together (one
        KV cache and position per sequence, every linear over all of their
        rows): ``forward_batch`` / ``generate_batch`` give each sequence the
        tokens the single-sequence decoder gives it, bit for bit -- the
        reference serves the same requests one after another
        (main_decoder.cpp:233-300).

        group: a torch.distributed process group of one process per GPU.
        Every linear's weight is then split by output rows over the group
        (rank r keeps rows [r*N/G, (r+1)*N/G)), each rank computes its rows
        and the slices are all-gathered (NCCL) into the full output on every
        rank; the other operators run on every rank.  Rows are independent,
        so the results are the unsharded ones bit for bit.  Every rank must
        make the same calls.  gather="peer" gathers the decode steps' outputs
        with the library's own peer-memory all-gather over NVLink
        (``leafq_allgather_*``), which lets the step be one CUDA graph; the
        prompt's gathers stay NCCL."""
        art = artifact if hasattr(artifact, "get") else Artifact(artifact)
        cfg = art.config
        if not (cfg.norm_kind == 0 and cfg.position_kind == 0 and cfg.gated == 1 and
                cfg.activation == 0 and cfg.parallel == 0 and cfg.sliding_window == 0 and
                not cfg.qk_norm and not cfg.rope_frequencies and cfg.position_offset == 0):
            raise LeafError(_lib.LEAFQ_ERR_UNSUPPORTED,
                            "GPU decoder supports RMSNorm / RoPE / gated SiLU decoders without "
                            "sliding window or Q/K norm")
        if activation_bits not in (8, 32):
            raise LeafError(_lib.LEAFQ_ERR_INVALID, "activation bits must be 8 or 32")
        if sequences < 1:
            raise LeafError(_lib.LEAFQ_ERR_INVALID, "sequences must be positive")
        self.cfg = cfg
        self.sequences = int(sequences)
        self.group = group
        if group is not None:
            import torch.distributed as dist
            self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
        else:
            self.world, self.rank = 1, 0
        self._full_rows: dict[int, int] = {}
        self._gather_bufs: dict = {}
        if gather not in ("nccl", "peer"):
            raise LeafError(_lib.LEAFQ_ERR_INVALID, "gather must be 'nccl' or 'peer'")
        self._peer = None
        self._peer_kind = gather if self.world > 1 else "nccl"
        self.activation_bits = activation_bits
        self.device = torch.device(device)
        self.capacity = int(capacity or cfg.max_positions)
        self.lib = load()
        dev = self.device

        def f32(t: HostTensor):
            return _on(t.data, dev).to(torch.float32).reshape(-1).contiguous()

        def weight(parts, interleave=False, biases=None, input_scale=None):
            return self._shard(_concat_rows(parts, dev, interleave, biases, input_scale))

        emb = art.get("model.embed_tokens.weight")
        self.embed_table = _on(emb.data, dev).contiguous()
        self.embed_scales = None if emb.scales is None else _on(emb.scales, dev).contiguous()
        self.embed_bits, self.embed_group = emb.bits, emb.group
        # SmoothQuant artifacts (decoder.cpp:1008-1019) carry per-projection
        # input scales: q, k, v (and gate, up) then cannot share one
        # quantisation of their common input and run as separate linears.
        self.smooth = any(art.get(f"model.layers.{i}.{n}.input_scale") is not None for i in range(cfg.layers)
                          for n in ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj",
                                    "mlp.gate_proj", "mlp.up_proj", "mlp.down_proj"))
        self.has_bias = False
        self.layers = []
        for i in range(cfg.layers):
            p = f"model.layers.{i}."
            get = art.get
            names = {n: p + m for n, m in (("q", "self_attn.q_proj"), ("k", "self_attn.k_proj"),
                                           ("v", "self_attn.v_proj"), ("o", "self_attn.o_proj"),
                                           ("gate", "mlp.gate_proj"), ("up", "mlp.up_proj"),
                                           ("down", "mlp.down_proj"))}
            wt = {n: get(b + ".weight") for n, b in names.items()}
            bias = {n: get(b + ".bias") for n, b in names.items()}
            scale = {n: get(b + ".input_scale") for n, b in names.items()}
            self.has_bias |= any(b is not None for b in bias.values())
            layer = dict(input_norm=f32(get(p + "input_layernorm.weight")),
                         post_norm=f32(get(p + "post_attention_layernorm.weight")),
                         o=weight([wt["o"]], biases=[bias["o"]], input_scale=scale["o"]),
                         down=weight([wt["down"]], biases=[bias["down"]], input_scale=scale["down"]))
            if self.smooth:
                for n in ("q", "k", "v", "gate", "up"):
                    layer[n] = weight([wt[n]], biases=[bias[n]], input_scale=scale[n])
            else:
                layer["qkv"] = weight([wt["q"], wt["k"], wt["v"]], biases=[bias["q"], bias["k"], bias["v"]])
                layer["gate_up"] = weight([wt["gate"], wt["up"]], interleave=True,
                                          biases=[bias["gate"], bias["up"]])
            self.layers.append(layer)
        self.final_norm = f32(art.get("model.norm.weight")) if cfg.final_norm else None
        self.lm_head = weight([art.get("lm_head.weight")], biases=[art.get("lm_head.bias")])
        self.has_bias |= self.lm_head.bias is not None
        d, kv = cfg.head_dim, cfg.kv_heads
        S = self.sequences
        self.k_cache = [torch.zeros((S, kv, self.capacity, d), dtype=torch.float32, device=dev)
                        for _ in range(cfg.layers)]
        self.v_cache = [torch.zeros_like(k) for k in self.k_cache]
        half = cfg.rotary_dim // 2
        cos = np.empty((self.capacity, half), dtype=np.float32)
        sin = np.empty_like(cos)
        check(self.lib.leafq_rope_tables(ctypes.c_float(cfg.theta), cfg.rotary_dim, self.capacity,
                                         cos.ctypes.data, sin.ctypes.data))
        self.cos = torch.from_numpy(cos).to(dev)
        self.sin = torch.from_numpy(sin).to(dev)
        # decoder.cpp:1348: both q and k are scaled by 1/sqrt(sqrt(dim)).
        self.scale = float(np.float32(1.0) / np.sqrt(np.sqrt(np.float32(d))))
        self.position = torch.zeros(S, dtype=torch.int32, device=dev)
        self.error_flag = torch.zeros(1, dtype=torch.int32, device=dev)
        self.length = 0
        self._buffers: dict[int, dict] = {}
        self.graph: Optional[torch.cuda.CUDAGraph] = None
        self.token = torch.zeros(S, dtype=torch.int32, device=dev)
        self.history = torch.zeros(self.capacity + 1, dtype=torch.int32, device=dev)
        self.step_logits = torch.zeros(cfg.vocab, dtype=torch.float32, device=dev)
        self._plan = None
        self._plan_refs = None
        self._step_ready = False

    # ------------------------------------------------------------ buffers
    def _bufs(self, tokens: int) -> dict:
        """Buffers of one forward of `tokens` tokens per sequence."""
        b = self._buffers.get(tokens)
        if b is None:
            c = self.cfg
            q = c.heads * c.head_dim
            dev = self.device
            S = self.sequences
            rows = S * tokens
            e = lambda *s: torch.empty(s, dtype=torch.float32, device=dev)  # noqa: E731
            b = dict(ids=torch.zeros(rows, dtype=torch.int32, device=dev), hidden=e(rows, c.hidden),
                     normalized=e(rows, c.hidden), qkv=e(rows, q + 2 * c.kv_heads * c.head_dim),
                     q_heads=e(S, c.heads, tokens, c.head_dim), attn=e(rows, q), o=e(rows, c.hidden),
                     gate_up=e(rows, 2 * c.intermediate), act=e(rows, c.intermediate),
                     down=e(rows, c.hidden), last=e(S, c.hidden), logits=e(S, c.vocab),
                     workspace=Workspace(dev),
                     q=e(rows, q), k=e(rows, c.kv_heads * c.head_dim), v=e(rows, c.kv_heads * c.head_dim),
                     gate=e(rows, c.intermediate), up=e(rows, c.intermediate),
                     codes=torch.empty((rows, c.hidden), dtype=torch.int8, device=dev),
                     codes_mlp=torch.empty((rows, c.intermediate), dtype=torch.int8, device=dev),
                     code_scales=e(rows))
            # Each chunk size owns its workspace, sized once: a captured graph
            # keeps its pointers, so nothing it uses may be reallocated.
            for w in self._weights():
                for r in (rows, S):
                    need = self._workspace_bytes(w, r)
                    if need:
                        b["workspace"].get(need)
            need = self.lib.leafq_attention_workspace_bytes(S, tokens, c.heads, c.kv_heads, c.head_dim,
                                                            self.capacity)
            b["attention_ws"] = torch.empty(max(need, 16), dtype=torch.uint8, device=dev)
            self._buffers[tokens] = b
        return b

    def _weights(self):
        for layer in self.layers:
            for n in ("qkv", "q", "k", "v", "o", "gate_up", "gate", "up", "down"):
                if n in layer:
                    yield layer[n]
        yield self.lm_head

    # ------------------------------------------------------- row sharding
    def _shard(self, w: QuantWeight) -> QuantWeight:
        """This rank's rows of a weight (the whole weight without a group)."""
        if self.world == 1:
            return w
        from .parallel import RowShards

        part = RowShards(w.rows, self.world)
        if not part.even:
            raise LeafError(_lib.LEAFQ_ERR_UNSUPPORTED,
                            f"{w.rows} rows do not split evenly over {self.world} ranks")
        b, e = part.begin(self.rank), part.end(self.rank)
        shard = QuantWeight(w.data[b:e].clone(), None if w.scales is None else w.scales[b:e].clone(), e - b,
                            w.cols, w.bits, w.group, None if w.bias is None else w.bias[b:e].clone(),
                            w.input_scale)
        self._full_rows[id(shard)] = w.rows
        return shard

    def _sharded_out(self, w: QuantWeight, out: torch.Tensor, tokens: int):
        """(buffer this rank's rows are written to, gather step or None)."""
        if self.world == 1:
            return out, None
        n = w.rows
        key = (tokens, n)
        bufs = self._gather_bufs.get(key)
        if bufs is None:
            local = torch.empty((tokens, n), dtype=torch.float32, device=self.device)
            stacked = torch.empty((self.world, tokens, n), dtype=torch.float32, device=self.device)
            bufs = self._gather_bufs[key] = (local, stacked)
        local, stacked = bufs

        def gather():
            import torch.distributed as dist

            if self._peer is not None and tokens == self.sequences:
                # Decode step: this rank's rows stored into every rank's
                # buffer over NVLink, collected in row order (graph-capturable).
                self._peer.run(local, self.rank * n, self.world * n, out)
                return
            if tokens == 1:  # [world][n] is already the row order of [1, world * n]
                dist.all_gather_into_tensor(out.view(-1), local.view(-1), group=self.group)
            else:
                dist.all_gather_into_tensor(stacked.view(-1), local.view(-1), group=self.group)
                out.view(tokens, self.world, n).copy_(stacked.permute(1, 0, 2))
        return local, gather

    # -------------------------------------------------------------- ops
    # Linears are launched with programmatic dependent launch: their kernels
    # wait on the previous kernel before reading its output, and start
    # streaming weights (which nothing in the step writes) before that.
    def _workspace_bytes(self, w: QuantWeight, tokens: int) -> int:
        if w.input_scale is not None:
            return self.lib.leafq_linear_smooth_workspace_bytes(tokens, w.cols, self.activation_bits)
        return self.lib.leafq_linear_workspace_bytes(tokens, w.cols, w.bits, w.group, self.activation_bits)

    def _linear(self, x: torch.Tensor, w: QuantWeight, out: torch.Tensor, tokens: int,
                workspace: Workspace) -> None:
        """Decoder::Impl::linear for one (stacked) weight: input scale, linear,
        bias (decoder.cpp:994-1233)."""
        lib = self.lib
        need = self._workspace_bytes(w, tokens)
        ws = workspace.buffer if need else None
        if ws is not None and ws.numel() < need:
            raise LeafError(_lib.LEAFQ_ERR_INVALID, "decoder workspace too small")
        dst, gather = self._sharded_out(w, out, tokens)
        bias = None if w.bias is None else w.bias.data_ptr()
        scales = None if w.scales is None else w.scales.data_ptr()
        wsp, wsn = (None, 0) if ws is None else (ws.data_ptr(), ws.numel())
        if w.input_scale is not None:
            check(lib.leafq_linear_smooth(_stream(), x.data_ptr(), w.input_scale.data_ptr(), tokens, w.cols,
                                          w.data.data_ptr(), scales, w.rows, w.bits, w.group, self.activation_bits,
                                          bias, dst.data_ptr(), wsp, wsn, LEAFQ_FLAG_PDL))
        else:
            check(lib.leafq_linear(_stream(), x.data_ptr(), tokens, w.cols, w.data.data_ptr(), scales, w.rows,
                                   w.bits, w.group, self.activation_bits, bias, dst.data_ptr(), wsp, wsn,
                                   LEAFQ_FLAG_PDL))
        if gather is not None:
            gather()

    def _forward_device(self, b: dict, tokens: int) -> None:
        """One forward of `tokens` ids per sequence already in b["ids"] at
        the device positions; logits of each sequence's last row in
        b["logits"]; positions advanced."""
        c, lib, s = self.cfg, self.lib, _stream()
        S = self.sequences
        rows = S * tokens
        check(lib.leafq_embed(s, b["ids"].data_ptr(), rows, self.embed_table.data_ptr(),
                              None if self.embed_scales is None else self.embed_scales.data_ptr(),
                              self.embed_bits, self.embed_group, c.vocab, c.hidden,
                              ctypes.c_float(c.embedding_scale), b["hidden"].data_ptr(),
                              self.error_flag.data_ptr()))
        # With more than 8 rows the W8A8 linears take codes: the RMSNorm
        # before q|k|v and gate|up quantises its output in the same pass
        # (leafq_rmsnorm_quantize), which is what leafq_linear's own
        # quantiser would produce from the fp32 rows.
        fuse = self.activation_bits == 8 and rows > 8 and c.hidden % 4 == 0 and c.hidden <= 4096 and not self.smooth

        def norm(delta, add_zero, weight, codes):
            d = None if delta is None else delta.data_ptr()
            if codes:
                check(lib.leafq_rmsnorm_quantize(s, b["hidden"].data_ptr(), d, add_zero, rows, c.hidden,
                                                 weight.data_ptr(), ctypes.c_float(c.epsilon), None,
                                                 b["codes"].data_ptr(), b["code_scales"].data_ptr()))
            else:
                check(lib.leafq_rmsnorm(s, b["hidden"].data_ptr(), d, add_zero, rows, c.hidden,
                                        weight.data_ptr(), ctypes.c_float(c.epsilon), b["normalized"].data_ptr()))

        def normed_linear(w, out):
            if fuse:
                dst, gather = self._sharded_out(w, out, rows)
                check(lib.leafq_linear_int_q(s, b["codes"].data_ptr(), b["code_scales"].data_ptr(), rows, w.cols,
                                             w.data.data_ptr(), w.scales.data_ptr(), w.rows, w.bits, w.group,
                                             None if w.bias is None else w.bias.data_ptr(), dst.data_ptr(), None,
                                             LEAFQ_FLAG_PDL))
                if gather is not None:
                    gather()
            else:
                self._linear(b["normalized"], w, out, rows, b["workspace"])

        norm(None, 0, self.layers[0]["input_norm"], fuse)
        ws = b["attention_ws"]
        for i, layer in enumerate(self.layers):
            if self.smooth:
                # Each projection on its own input scale, then q | k | v
                # side by side in every row as the stacked linear writes them.
                for n in ("q", "k", "v"):
                    self._linear(b["normalized"], layer[n], b[n], rows, b["workspace"])
                torch.cat((b["q"], b["k"], b["v"]), dim=1, out=b["qkv"])
            else:
                normed_linear(layer["qkv"], b["qkv"])
            check(lib.leafq_rotary_append_batch(s, b["qkv"].data_ptr(), S, tokens, c.heads, c.kv_heads,
                                                c.head_dim, c.rotary_dim, self.cos.data_ptr(),
                                                self.sin.data_ptr(), self.position.data_ptr(),
                                                b["q_heads"].data_ptr(), self.k_cache[i].data_ptr(),
                                                self.v_cache[i].data_ptr(), self.capacity))
            check(lib.leafq_attention_batch(s, b["q_heads"].data_ptr(), self.k_cache[i].data_ptr(),
                                            self.v_cache[i].data_ptr(), S, tokens, c.heads, c.kv_heads,
                                            c.head_dim, self.position.data_ptr(), self.capacity,
                                            self.capacity, ctypes.c_float(self.scale), b["attn"].data_ptr(),
                                            ws.data_ptr(), ws.numel()))
            self._linear(b["attn"], layer["o"], b["o"], rows, b["workspace"])
            norm(b["o"], 0, layer["post_norm"], fuse)
            if self.smooth:
                # gate and up on their own input scales, interleaved as the
                # SiLU kernel reads them (gate_0, up_0, gate_1, ...).
                self._linear(b["normalized"], layer["gate"], b["gate"], rows, b["workspace"])
                self._linear(b["normalized"], layer["up"], b["up"], rows, b["workspace"])
                torch.stack((b["gate"], b["up"]), dim=2, out=b["gate_up"].view(rows, c.intermediate, 2))
            else:
                normed_linear(layer["gate_up"], b["gate_up"])
            if fuse and c.intermediate <= 6144:
                # SiLU gate and the down projection's quantisation in one pass.
                check(lib.leafq_silu_gate_quantize(s, b["gate_up"].data_ptr(), rows, c.intermediate, None,
                                                   b["codes_mlp"].data_ptr(), b["code_scales"].data_ptr()))
                w = layer["down"]
                dst, gather = self._sharded_out(w, b["down"], rows)
                check(lib.leafq_linear_int_q(s, b["codes_mlp"].data_ptr(), b["code_scales"].data_ptr(), rows,
                                             w.cols, w.data.data_ptr(), w.scales.data_ptr(), w.rows, w.bits,
                                             w.group, None if w.bias is None else w.bias.data_ptr(),
                                             dst.data_ptr(), None, LEAFQ_FLAG_PDL))
                if gather is not None:
                    gather()
            else:
                check(lib.leafq_silu_gate(s, b["gate_up"].data_ptr(), rows, c.intermediate,
                                          b["act"].data_ptr()))
                self._linear(b["act"], layer["down"], b["down"], rows, b["workspace"])
            last = i + 1 == len(self.layers)
            if last and self.final_norm is None:
                # no final norm: the logits would read the residual stream itself
                raise LeafError(_lib.LEAFQ_ERR_UNSUPPORTED, "artifacts without a final norm")
            norm(b["down"], 1, self.final_norm if last else self.layers[i + 1]["input_norm"], fuse and not last)
        if tokens == 1:
            last_rows = b["normalized"]
        elif S == 1:
            last_rows = b["normalized"][tokens - 1:tokens]
        else:  # each sequence's last row, gathered into consecutive rows
            b["last"].copy_(b["normalized"].view(S, tokens, c.hidden)[:, tokens - 1])
            last_rows = b["last"]
        self._linear(last_rows, self.lm_head, b["logits"], S, b["workspace"])
        check(lib.leafq_advance_positions(s, self.position.data_ptr(), S, tokens))

    # ----------------------------------------------------------- public API
    def reset(self) -> None:
        """Decoder::reset: empty every KV cache."""
        self.length = 0
        self.position.zero_()

    def forward(self, ids) -> torch.Tensor:
        """Decoder::forward_into(ids, logits) with all_logits = false: the
        last position's logits [1, vocab] (a device tensor reused by later
        calls)."""
        if self.sequences != 1:
            raise LeafError(_lib.LEAFQ_ERR_INVALID, "a batched decoder runs forward_batch")
        ids = [int(i) for i in ids]
        if not ids:
            raise LeafError(_lib.LEAFQ_ERR_INVALID, "input tokens are empty")
        if self.length + len(ids) > min(self.cfg.max_positions, self.capacity):
            raise LeafError(_lib.LEAFQ_ERR_INVALID, "context length exceeds artifact limit")
        if any(i < 0 or i >= self.cfg.vocab for i in ids):
            raise LeafError(_lib.LEAFQ_ERR_INVALID, "token id exceeds vocabulary")
        b = self._bufs(len(ids))
        b["ids"].copy_(torch.tensor(ids, dtype=torch.int32))
        self._forward_device(b, len(ids))
        self.length += len(ids)
        return b["logits"]

    def _decode_step(self) -> None:
        """One decode step of every sequence from the ids of the previous
        argmax (the captured graph, or its launches when not captured)."""
        if self.graph is not None:
            self.graph.replay()
            return
        b = self._bufs(1)
        self._forward_device(b, 1)
        check(self.lib.leafq_argmax(_stream(), b["logits"].data_ptr(), self.sequences, self.cfg.vocab,
                                    b["ids"].data_ptr()))

    def capture_decode(self) -> None:
        """Capture one decode step (ids from the previous step's argmax) as
        a CUDA graph.  A sharded decoder steps without a graph (its NCCL
        gathers run eagerly)."""
        if self.world > 1 and self._peer_kind == "nccl":
            self._bufs(1)
            self._step_ready = True
            return
        if self.world > 1 and self._peer is None:
            from .parallel import PeerAllGather

            widest = max(self._full_rows.values())
            self._peer = PeerAllGather(self.sequences * widest, group=self.group)
        b = self._bufs(1)
        stream = torch.cuda.Stream(self.device)
        stream.wait_stream(torch.cuda.current_stream(self.device))
        saved = self.position.clone()
        with torch.cuda.stream(stream):
            self._forward_device(b, 1)  # warm-up outside capture (lazy loads, smem attributes)
            check(self.lib.leafq_argmax(_stream(), b["logits"].data_ptr(), self.sequences, self.cfg.vocab,
                                        b["ids"].data_ptr()))
        torch.cuda.current_stream(self.device).wait_stream(stream)
        torch.cuda.synchronize(self.device)
        self.position.copy_(saved)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            self._forward_device(b, 1)
            check(self.lib.leafq_argmax(_stream(), b["logits"].data_ptr(), self.sequences, self.cfg.vocab,
                                        b["ids"].data_ptr()))
        self.graph = graph
        self._step_ready = True

    def generate(self, prompt, max_new: int) -> list[int]:
        """main_decoder.cpp:95-113 greedy continuation without EOS handling
        on the device: prefill, then one graph replay per further token."""
        if not self._step_ready:
            self.capture_decode()
        if self.length + len(prompt) + max_new - 1 > min(self.cfg.max_positions, self.capacity):
            raise LeafError(_lib.LEAFQ_ERR_INVALID, "context length exceeds artifact limit")
        logits = self.forward(prompt)
        step = self._bufs(1)
        check(self.lib.leafq_argmax(_stream(), logits.data_ptr(), 1, self.cfg.vocab,
                                    step["ids"].data_ptr()))
        out = torch.empty(max_new, dtype=torch.int32, device=self.device)
        out[0:1].copy_(step["ids"])
        eos = set(self.cfg.eos_tokens)
        produced = max_new
        for i in range(1, max_new):
            if eos and int(out[i - 1].item()) in eos:
                produced = i
                break
            self._decode_step()
            self.length += 1
            out[i:i + 1].copy_(step["ids"])
        return [int(t) for t in out[:produced].tolist()]

    def forward_batch(self, prompts) -> torch.Tensor:
        """forward() for every sequence of the batch at once: prompts is one
        list of ids per sequence, all of the same length; returns each
        sequence's last-position logits [sequences, vocab] (a device tensor
        reused by later calls)."""
        prompts = [[int(i) for i in p] for p in prompts]
        if len(prompts) != self.sequences:
            raise LeafError(_lib.LEAFQ_ERR_INVALID, "one prompt per sequence")
        tokens = len(prompts[0])
        if tokens == 0 or any(len(p) != tokens for p in prompts):
            raise LeafError(_lib.LEAFQ_ERR_INVALID, "batched prompts must be non-empty and of equal length")
        if self.length + tokens > min(self.cfg.max_positions, self.capacity):
            raise LeafError(_lib.LEAFQ_ERR_INVALID, "context length exceeds artifact limit")
        if any(i < 0 or i >= self.cfg.vocab for p in prompts for i in p):
            raise LeafError(_lib.LEAFQ_ERR_INVALID, "token id exceeds vocabulary")
        b = self._bufs(tokens)
        b["ids"].copy_(torch.tensor(prompts, dtype=torch.int32).reshape(-1))
        self._forward_device(b, tokens)
        self.length += tokens
        return b["logits"]

    def generate_batch(self, prompts, max_new: int) -> list[list[int]]:
        """generate() for every sequence of the batch: one prefill over all
        prompts, then one graph replay per token for all sequences.  A
        sequence that reaches an EOS id stops there (its later tokens are
        computed with the batch and dropped), as the reference's loop does."""
        if max_new < 1:
            raise LeafError(_lib.LEAFQ_ERR_INVALID, "max_new must be positive")
        if not self._step_ready:
            self.capture_decode()
        tokens = len(prompts[0]) if prompts else 0
        if self.length + tokens + max_new - 1 > min(self.cfg.max_positions, self.capacity):
            raise LeafError(_lib.LEAFQ_ERR_INVALID, "context length exceeds artifact limit")
        logits = self.forward_batch(prompts)
        step = self._bufs(1)
        check(self.lib.leafq_argmax(_stream(), logits.data_ptr(), self.sequences, self.cfg.vocab,
                                    step["ids"].data_ptr()))
        out = torch.empty((max_new, self.sequences), dtype=torch.int32, device=self.device)
        out[0].copy_(step["ids"])
        for i in range(1, max_new):
            self._decode_step()
            out[i].copy_(step["ids"])
        self.length += max_new - 1
        eos = set(self.cfg.eos_tokens)
        result = []
        for seq in out.t().tolist():
            for i, t in enumerate(seq):
                if t in eos:
                    seq = seq[:i + 1]
                    break
            result.append(seq)
        return result

    # ------------------------------------------------ whole-step kernel
    def fused_supported(self) -> bool:
        """The one-launch decode step needs per-row INT8 weights and
        embedding, W8A8, and a cache of at most 4096 rows."""
        per_row = all(w.bits == 8 and w.group == w.cols for w in self._weights())
        return (per_row and not self.smooth and not self.has_bias and "qkv" in self.layers[0] and
                self.sequences == 1 and self.world == 1 and self.activation_bits == 8 and
                self.embed_bits == 8 and
                self.embed_group == self.cfg.hidden and self.capacity <= 4096 and
                self.final_norm is not None)

    def build_fused(self) -> None:
        """Create the leafq_model_plan for this decoder (one cooperative
        launch per generated token)."""
        if not self.fused_supported():
            raise LeafError(_lib.LEAFQ_ERR_UNSUPPORTED,
                            "one-launch decode needs per-row INT8 weights, W8A8 and capacity <= 4096")
        c, ptr = self.cfg, (lambda t: t.data_ptr())
        layers = (_lib.ModelLayer * c.layers)()
        for i, L in enumerate(self.layers):
            layers[i] = _lib.ModelLayer(
                ptr(L["input_norm"]), ptr(L["post_norm"]), ptr(L["qkv"].data), ptr(L["qkv"].scales),
                ptr(L["o"].data), ptr(L["o"].scales), ptr(L["gate_up"].data), ptr(L["gate_up"].scales),
                ptr(L["down"].data), ptr(L["down"].scales), ptr(self.k_cache[i]), ptr(self.v_cache[i]))
        desc = _lib.ModelDesc(
            c.layers, c.hidden, c.intermediate, c.heads, c.kv_heads, c.head_dim, c.vocab, self.capacity,
            c.epsilon, c.embedding_scale, self.scale, ptr(self.embed_table), ptr(self.embed_scales),
            ptr(self.final_norm), ptr(self.lm_head.data), ptr(self.lm_head.scales), ptr(self.cos),
            ptr(self.sin), ctypes.cast(layers, ctypes.c_void_p), ptr(self.token), ptr(self.position),
            ptr(self.history), ptr(self.step_logits))
        plan = ctypes.c_void_p()
        check(self.lib.leafq_model_plan_create(ctypes.byref(desc), ctypes.byref(plan)))
        self._plan = plan
        self._plan_refs = (layers, desc)

    def step_fused(self) -> None:
        """One decode step of the token in self.token at the device position
        (one launch); the argmax replaces self.token."""
        check(self.lib.leafq_model_plan_run(_stream(), self._plan))

    def capture_stream_step(self, token_in: torch.Tensor, token_out: torch.Tensor) -> "torch.cuda.CUDAGraph":
        """One streaming decode step as a CUDA graph, for a server that sends
        every token to its client: copy the input token id from pinned host
        memory (``token_in``, int32 [1]), run step_fused(), copy the produced
        token id into pinned host memory (``token_out``).  Replay it, then
        synchronise the stream before reading ``token_out``.  The two may be
        the same pinned word: each replay then reads the previous step's token
        and leaves its own there.  The graph holds the plan's buffers: delete
        it before close()."""
        if self._plan is None:
            self.build_fused()
        for t in (token_in, token_out):
            if t.device.type != "cpu" or not t.is_pinned() or t.dtype != torch.int32 or t.numel() != 1:
                raise LeafError(_lib.LEAFQ_ERR_INVALID, "stream tokens must be pinned int32 [1] host tensors")
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            self.token.copy_(token_in, non_blocking=True)
            self.step_fused()
            token_out.copy_(self.token, non_blocking=True)
        return graph

    def generate_fused(self, prompt, max_new: int) -> list[int]:
        """Greedy continuation as generate(), with every decode step one
        launch of the whole-model kernel."""
        if self._plan is None:
            self.build_fused()
        n = self.length + len(prompt)
        if n + max_new - 1 > min(self.cfg.max_positions, self.capacity):
            raise LeafError(_lib.LEAFQ_ERR_INVALID, "context length exceeds artifact limit")
        logits = self.forward(prompt)
        check(self.lib.leafq_argmax(_stream(), logits.data_ptr(), 1, self.cfg.vocab,
                                    self.token.data_ptr()))
        self.history[n:n + 1].copy_(self.token)
        for _ in range(max_new - 1):
            self.step_fused()
        self.length += max_new - 1
        out = [int(t) for t in self.history[n:n + max_new].tolist()]
        eos = set(self.cfg.eos_tokens)
        for i, t in enumerate(out):
            if t in eos:
                return out[:i + 1]
        return out

    def close(self) -> None:
        if self._peer is not None:
            self.graph = None  # the graph holds the peer kernels
            self._peer.close()
            self._peer = None
        if self._plan is not None:
            torch.cuda.synchronize(self.device)
            check(self.lib.leafq_model_plan_destroy(self._plan))
            self._plan = None

    def device_status(self) -> int:
        bad = int(self.error_flag.item())
        if bad:
            raise LeafError(_lib.LEAFQ_ERR_INVALID, "token id exceeds vocabulary")
        return self.lib.leafq_device_status()
