"""leaf_b200: B200-native (sm_100a) quantised-linear operators for Leaf.

The hot path -- per-token INT8 activation quantisation, the W8A8 / W4A8 /
W4A32 decode GEMV, the W8A8 tcgen05 prefill GEMM, the dequant + bias
epilogue and the graph executor's INT8 GEMM -- runs in libleafq.so (C ABI in
include/leafq.h).  This package is the host-side mirror of the reference's
operator interface plus the N-sharded multi-GPU wrapper.
"""
from ._lib import LeafError, LEAFQ_FLAG_PDL, LEAFQ_FLAG_VNNI_ROUNDING, load
from .linear import (QuantLinearSet, QuantWeight, Workspace, gemm_i8_per_channel,
                     graph_linear, graph_quantize, linear, linear_int_q, quantize_act)

__all__ = [
    "LeafError", "LEAFQ_FLAG_PDL", "LEAFQ_FLAG_VNNI_ROUNDING", "load", "QuantLinearSet",
    "QuantWeight", "Workspace", "gemm_i8_per_channel", "graph_linear", "graph_quantize", "linear",
    "linear_int_q", "quantize_act",
]
