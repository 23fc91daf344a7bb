"""ctypes binding of libleafq.so (the C ABI declared in include/leafq.h).

The library must be present and loadable: there is no CPU or PyTorch
fallback for any leafq operation.  A missing library raises immediately.
"""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
LIBRARY = PACKAGE / "libleafq.so"
HEADER = PACKAGE.parent / "include" / "leafq.h"

LEAFQ_OK = 0
LEAFQ_ERR_INVALID = 1
LEAFQ_ERR_CUDA = 2
LEAFQ_ERR_UNSUPPORTED = 3
LEAFQ_ERR_TIMEOUT = 4
LEAFQ_ERR_NONFINITE = 5

LEAFQ_FLAG_VNNI_ROUNDING = 0x1
LEAFQ_FLAG_PDL = 0x2

LEAFQ_IPC_HANDLE_BYTES = 64

_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_int = ctypes.c_int
_u32 = ctypes.c_uint32
_f32 = ctypes.c_float
_size = ctypes.c_size_t

_SIGNATURES = {
    "leafq_last_error": ([], ctypes.c_char_p),
    "leafq_version": ([], _int),
    "leafq_device_status": ([], _int),
    "leafq_set_wait_limit_ns": ([ctypes.c_uint64], _int),
    "leafq_quantize_act": ([_vp, _vp, _i64, _i64, _vp, _vp], _int),
    "leafq_linear_workspace_bytes": ([_i64, _i64, _int, _i64, _int], _size),
    "leafq_linear": ([_vp, _vp, _i64, _i64, _vp, _vp, _i64, _int, _i64, _int, _vp, _vp, _vp, _size,
                      _u32], _int),
    "leafq_linear_int_q": ([_vp, _vp, _vp, _i64, _i64, _vp, _vp, _i64, _int, _i64, _vp, _vp, _vp,
                            _u32], _int),
    "leafq_graph_quantize": ([_vp, _vp, _i64, _f32, _vp, _vp], _int),
    "leafq_linear_smooth_workspace_bytes": ([_i64, _i64, _int], ctypes.c_size_t),
    "leafq_scale_columns": ([_vp, _vp, _i64, _i64, _vp, _vp], _int),
    "leafq_linear_smooth": ([_vp, _vp, _vp, _i64, _i64, _vp, _vp, _i64, _int, _i64, _int, _vp, _vp, _vp,
                             ctypes.c_size_t, ctypes.c_uint32], _int),
    "leafq_graph_linear_workspace_bytes": ([_i64, _i64], ctypes.c_size_t),
    "leafq_graph_linear": ([_vp, _vp, _i64, _i64, _int, _vp, _i64, _int, _f32, _vp, _f32, _f32, _vp, _int,
                            _int, _vp, _vp, ctypes.c_size_t, _vp], _int),
    "leafq_gemm_i8_per_channel": ([_vp, _vp, _vp, _vp, _f32, _vp, _vp, _i64, _i64, _i64, _int],
                                  _int),
    "leafq_linear_w8a8_static_scratch": ([_vp, _vp, _i64, _i64, _vp, _vp, _i64, _vp, _vp, _u32],
                                         _int),
    "leafq_decode_plan_create": ([_vp, _int, _int, _vp], _int),
    "leafq_decode_plan_run": ([_vp, _vp], _int),
    "leafq_decode_plan_destroy": ([_vp], _int),
    "leafq_allgather_init": ([_int, _int, _i64, _vp, _vp], _int),
    "leafq_allgather_connect": ([_vp, _vp], _int),
    "leafq_allgather_run": ([_vp, _vp, _vp, _i64, _i64, _i64, _i64, _vp], _int),
    "leafq_linear_allgather": ([_vp, _vp, _vp, _i64, _i64, _vp, _vp, _i64, _i64, _i64, _int, _i64,
                                _int, _vp, _vp, _vp, _size, _u32], _int),
    "leafq_allgather_destroy": ([_vp], _int),
    "leafq_model_plan_create": ([_vp, _vp], _int),
    "leafq_model_plan_run": ([_vp, _vp], _int),
    "leafq_model_plan_destroy": ([_vp], _int),
    "leafq_embed": ([_vp, _vp, _i64, _vp, _vp, _int, _i64, _i64, _i64, _f32, _vp, _vp], _int),
    "leafq_rmsnorm": ([_vp, _vp, _vp, _int, _i64, _i64, _vp, _f32, _vp], _int),
    "leafq_rmsnorm_quantize": ([_vp, _vp, _vp, _int, _i64, _i64, _vp, _f32, _vp, _vp, _vp], _int),
    "leafq_rope_tables": ([_f32, _int, _i64, _vp, _vp], _int),
    "leafq_rotary_append": ([_vp, _vp, _i64, _int, _int, _int, _int, _vp, _vp, _vp, _vp, _vp, _vp,
                             _i64], _int),
    "leafq_attention": ([_vp, _vp, _vp, _vp, _i64, _int, _int, _int, _vp, _i64, _f32, _vp], _int),
    "leafq_rotary_append_batch": ([_vp, _vp, _int, _i64, _int, _int, _int, _int, _vp, _vp, _vp, _vp, _vp,
                                   _vp, _i64], _int),
    "leafq_attention_workspace_bytes": ([_int, _i64, _int, _int, _int, _i64], _i64),
    "leafq_attention_batch": ([_vp, _vp, _vp, _vp, _int, _i64, _int, _int, _int, _vp, _i64, _i64, _f32, _vp,
                               _vp, _i64], _int),
    "leafq_silu_gate": ([_vp, _vp, _i64, _i64, _vp], _int),
    "leafq_silu_gate_quantize": ([_vp, _vp, _i64, _i64, _vp, _vp, _vp], _int),
    "leafq_argmax": ([_vp, _vp, _i64, _i64, _vp], _int),
    "leafq_expf": ([_vp, _vp, _i64, _vp], _int),
    "leafq_advance_position": ([_vp, _vp, ctypes.c_int32], _int),
    "leafq_advance_positions": ([_vp, _vp, _int, ctypes.c_int32], _int),
}


class DecodeOp(ctypes.Structure):
    """leafq_decode_op (include/leafq.h)."""

    _fields_ = [("x", _vp), ("y", _vp), ("weight", _vp), ("weight_scales", _vp), ("bias", _vp),
                ("rows", _i64), ("cols", _i64), ("wait", ctypes.c_int32),
                ("x_offset", ctypes.c_int32)]



class ModelLayer(ctypes.Structure):
    """leafq_model_layer (include/leafq.h)."""

    _fields_ = [(name, _vp) for name in (
        "input_norm", "post_norm", "qkv", "qkv_scales", "o", "o_scales", "gate_up",
        "gate_up_scales", "down", "down_scales", "k_cache", "v_cache")]


class ModelDesc(ctypes.Structure):
    """leafq_model_desc (include/leafq.h)."""

    _fields_ = [("layers", ctypes.c_int32), ("hidden", ctypes.c_int32),
                ("intermediate", ctypes.c_int32), ("heads", ctypes.c_int32),
                ("kv_heads", ctypes.c_int32), ("head_dim", ctypes.c_int32),
                ("vocab", ctypes.c_int32), ("capacity", _i64), ("epsilon", _f32),
                ("embedding_scale", _f32), ("attn_scale", _f32)] + [
        (name, _vp) for name in ("embed", "embed_scales", "final_norm", "lm_head", "lm_head_scales",
                                 "cos_table", "sin_table", "layer", "ids", "position", "history",
                                 "logits")]


_lib = None


class LeafError(RuntimeError):
    """A leafq call failed; mirrors the reference's std::runtime_error."""

    def __init__(self, status: int, message: str):
        super().__init__(f"Leaf decoder: {message} (leafq status {status})")
        self.status = status


def declared_symbols() -> list[str]:
    """Every function name include/leafq.h declares."""
    text = HEADER.read_text()
    return sorted(set(re.findall(r"\b(leafq_[a-z0-9_]+)\s*\(", text)))


def load() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIBRARY.exists():
            raise LeafError(LEAFQ_ERR_UNSUPPORTED,
                            f"{LIBRARY} is missing; build it with `python -m leaf_b200.build`")
        lib = ctypes.CDLL(str(LIBRARY))
        for name, (args, restype) in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = restype
        _lib = lib
    return _lib


def check(status: int) -> None:
    if status != LEAFQ_OK:
        message = load().leafq_last_error().decode(errors="replace")
        raise LeafError(status, message or "unknown failure")
