"""CPU oracle for Leaf's quantised-linear path.  TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU legs import
this package, and only as the checker / CPU baseline.  The product
(``leaf_b200``) never imports it and has no CPU fallback.

Two checkers live here:

* ``liboracle.so`` -- our own plain-C restatement (``leafq_oracle.c``), plus the
  numpy weight codec below.  Built from this repository alone.
* ``_ref/libleafref.so`` -- the reference's own CPU kernels compiled unmodified
  from the reference tree by ``Makefile`` (present wherever it was built; the
  built file travels with the repository snapshot).

Parity status: the restatement is pinned against the reference's compiled
kernels (tests/test_oracle_pinned.py, run wherever ``_ref`` exists) and against
golden vectors that the reference produced (tests/golden/, checked on every
machine).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
_ORACLE = HERE / "liboracle.so"
_REF = HERE / "_ref" / "libleafref.so"
REF_DECODER = HERE / "_ref" / "leaf_decoder"

_c_size = ctypes.c_size_t
_vp = ctypes.c_void_p

_lib = None
_ref = None


def reference_root():
    """The reference checkout the ``_ref`` recipe compiles from: the
    LEAF_REFERENCE environment variable, else a ``reference`` directory beside
    this repository; None when neither holds the engine sources."""
    env = os.environ.get("LEAF_REFERENCE")
    for root in ([Path(env)] if env else []) + [HERE.parent.parent / "reference"]:
        if (root / "engine" / "src" / "decoder.cpp").exists():
            return root
    return None


def build(ref: bool = False) -> None:
    """Compile the C restatement (and, when the reference tree is present, the
    reference kernels)."""
    subprocess.run(["make", "-s", "-C", str(HERE), "oracle"], check=True)
    if ref:
        root = reference_root()
        if root is None:
            raise FileNotFoundError("no reference tree: set LEAF_REFERENCE")
        subprocess.run(["make", "-s", "-C", str(HERE), "ref", f"REF={root}"], check=True)


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not _ORACLE.exists():
            build()
        _lib = ctypes.CDLL(str(_ORACLE))
        _lib.oq_quantize_act.argtypes = [_vp, _c_size, _c_size, _vp, _vp]
        _lib.oq_linear_int_q.argtypes = [_vp, _vp, _c_size, _c_size, _vp, _vp, _c_size,
                                         ctypes.c_uint, _c_size, _vp, _vp, _vp, ctypes.c_int]
        _lib.oq_linear_int.argtypes = [_vp, _c_size, _c_size, _vp, _vp, _c_size, ctypes.c_uint,
                                       _c_size, _vp, _vp, _vp, ctypes.c_int]
        _lib.oq_expf.argtypes = [_vp, _vp, _c_size]
        _lib.oq_gelu.argtypes = [_vp, _vp, _c_size]
        _lib.oq_tanhf.argtypes = [_vp, _vp, _c_size]
        _lib.oq_linear_float.argtypes = [_vp, _c_size, _c_size, _vp, _vp, _c_size, ctypes.c_uint,
                                         _c_size, _vp, _vp]
        _lib.oq_graph_quantize.argtypes = [_vp, _c_size, ctypes.c_float, _vp]
        _lib.oq_gemm_i8_per_channel.argtypes = [_vp, _vp, _vp, ctypes.c_float, _vp, _vp, _c_size,
                                                _c_size, _c_size, ctypes.c_int]
        _lib.oq_gemm_i8_per_channel.restype = None
    return _lib


def ref_available() -> bool:
    return _REF.exists()


def ref() -> ctypes.CDLL:
    global _ref
    if _ref is None:
        if not _REF.exists():
            raise FileNotFoundError(f"reference kernels not built: {_REF}")
        _ref = ctypes.CDLL(str(_REF))
        _ref.leafref_last_error.restype = ctypes.c_char_p
        _ref.leafref_quantize_i16.argtypes = [_vp, _c_size, _c_size, _vp, _vp]
        _ref.leafref_quantize_u8.argtypes = [_vp, _c_size, _c_size, _vp, _vp]
        _ref.leafref_linear_int.argtypes = [_vp, _c_size, _c_size, _vp, _vp, _c_size, ctypes.c_uint,
                                            _c_size, _vp, _vp, ctypes.c_uint, ctypes.c_int]
        _ref.leafref_linear_float.argtypes = [_vp, _c_size, _c_size, _vp, _vp, _c_size,
                                              ctypes.c_uint, _c_size, _vp, _vp, ctypes.c_uint,
                                              ctypes.c_int]
        for name in ("leafref_gemm_i8_per_channel", "leafref_gemm_i8_reference"):
            getattr(_ref, name).argtypes = [_vp, _vp, _vp, ctypes.c_float, _vp, _vp, _c_size,
                                            _c_size, _c_size, ctypes.c_int]
        _ref.leafref_graph_quantize.argtypes = [_vp, _c_size, ctypes.c_float, _vp]
        _ref.leafref_graph_activation.argtypes = [_vp, _c_size, ctypes.c_char_p, _vp]
        _ref.leafref_graph_last_error.restype = ctypes.c_char_p
    return _ref


def _p(array):
    return None if array is None else array.ctypes.data


def _f32(array):
    return np.ascontiguousarray(array, dtype=np.float32)


# --------------------------------------------------------------------------
# weight codec (tools/export_decoder.py:91-105), restated in numpy
# --------------------------------------------------------------------------
def quantize_weight(weight: np.ndarray, bits: int, group: int):
    """Symmetric weight quantiser of tools/export_decoder.py:91-105.

    scale = max(max|w| / L, 1e-12) in fp32 per (row, group), L = 2**(bits-1)-1;
    code = clip(rint(w / scale), -L, L); int4 codes are packed two per byte,
    low nibble = even column.  Returns (payload, scales[rows, cols/group]).
    """
    weight = np.ascontiguousarray(weight, dtype=np.float32)
    rows, cols = weight.shape
    if cols % group:
        raise ValueError(f"group {group} does not divide width {cols}")
    grouped = weight.reshape(rows, cols // group, group)
    limit = (1 << (bits - 1)) - 1
    scales = np.maximum(np.max(np.abs(grouped), axis=-1) / np.float32(limit),
                        np.float32(1e-12)).astype(np.float32)
    codes = np.clip(np.rint(grouped / scales[..., None]), -limit, limit).astype(np.int8)
    codes = codes.reshape(rows, cols)
    if bits == 4:
        nibbles = codes.astype(np.uint8) & 15
        codes = nibbles[:, 0::2] | (nibbles[:, 1::2] << 4)
    return np.ascontiguousarray(codes), np.ascontiguousarray(scales)


def unpack_int4(packed: np.ndarray) -> np.ndarray:
    """Signed int4 codes [rows, cols] from the packed [rows, cols/2] bytes."""
    low = (packed & 15).astype(np.int8)
    high = (packed >> 4).astype(np.int8)
    codes = np.empty((packed.shape[0], packed.shape[1] * 2), dtype=np.int8)
    codes[:, 0::2] = np.where(low >= 8, low - 16, low)
    codes[:, 1::2] = np.where(high >= 8, high - 16, high)
    return codes


# --------------------------------------------------------------------------
# our C restatement
# --------------------------------------------------------------------------
def quantize_act(x: np.ndarray):
    """(q int8 [M,K], sx fp32 [M]) -- decoder.cpp:1028-1038 / 618-627."""
    x = _f32(x)
    m, k = x.shape
    q = np.empty((m, k), dtype=np.int8)
    sx = np.empty(m, dtype=np.float32)
    lib().oq_quantize_act(_p(x), m, k, _p(q), _p(sx))
    return q, sx


def linear_int(x, weight, scales, bits, group, bias=None, want_acc=False, fused=True):
    """W8A8 / W4A8 linear (the integer branch of Decoder::Impl::linear).

    fused=True restates the AVX2 kernels (decode and INT4 paths); fused=False
    the VNNI prefill tile.  They differ only with several groups per row.
    """
    x = _f32(x)
    m, k = x.shape
    n = scales.shape[0]
    y = np.empty((m, n), dtype=np.float32)
    acc = np.empty((m, n, k // group), dtype=np.int32) if want_acc else None
    weight = np.ascontiguousarray(weight)
    scales = _f32(scales)
    bias = None if bias is None else _f32(bias)
    status = lib().oq_linear_int(_p(x), m, k, _p(weight), _p(scales), n, bits, group, _p(bias),
                                 _p(y), _p(acc), int(fused))
    if status:
        raise ValueError(f"oq_linear_int failed ({status})")
    return (y, acc) if want_acc else y


def linear_int_q(q, sx, weight, scales, bits, group, bias=None, want_acc=False, fused=True):
    q = np.ascontiguousarray(q, dtype=np.int8)
    sx = _f32(sx)
    m, k = q.shape
    n = scales.shape[0]
    y = np.empty((m, n), dtype=np.float32)
    acc = np.empty((m, n, k // group), dtype=np.int32) if want_acc else None
    weight = np.ascontiguousarray(weight)
    scales = _f32(scales)
    bias = None if bias is None else _f32(bias)
    status = lib().oq_linear_int_q(_p(q), _p(sx), m, k, _p(weight), _p(scales), n, bits, group,
                                   _p(bias), _p(y), _p(acc), int(fused))
    if status:
        raise ValueError(f"oq_linear_int_q failed ({status})")
    return (y, acc) if want_acc else y


def linear_float(x, weight, scales, bits, group, bias=None):
    """Weight-only linear with fp32 activations in dot_avx order."""
    x = _f32(x)
    m, k = x.shape
    n = weight.shape[0]
    y = np.empty((m, n), dtype=np.float32)
    weight = np.ascontiguousarray(weight)
    scales = None if scales is None else _f32(scales)
    bias = None if bias is None else _f32(bias)
    status = lib().oq_linear_float(_p(x), m, k, _p(weight), _p(scales), n, bits, group or 0,
                                   _p(bias), _p(y))
    if status:
        raise ValueError(f"oq_linear_float failed ({status})")
    return y


def expf(x):
    """libm expf elementwise (float32 in, float32 out)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty_like(x)
    lib().oq_expf(_p(x), _p(y), x.size)
    return y


def gelu(x):
    """The graph executor's fused Gelu, tanh form (executor.cpp:236-240):
    (0.5f * v) * (1 + tanhf(c * (v + ((0.044715f * v) * v) * v))), each step
    one float32 rounding, libm tanhf."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty_like(x)
    lib().oq_gelu(_p(x), _p(y), x.size)
    return y


def tanhf(x):
    """libm tanhf elementwise (float32 in, float32 out)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty_like(x)
    lib().oq_tanhf(_p(x), _p(y), x.size)
    return y


def graph_activation(v, activation):
    """apply_activation (executor.cpp:232-242): None / "" identity, Relu as
    std::max(value, 0.0f), Silu v / (1 + expf(-v)), Gelu as gelu()."""
    f = np.float32
    v = _f32(v)
    if activation in (None, ""):
        return v.copy()
    if activation == "Relu":
        return np.where(v < 0, f(0), v).astype(np.float32)
    if activation == "Silu":
        return (v / (f(1) + expf(-v))).astype(np.float32)
    if activation == "Gelu":
        return gelu(v)
    raise ValueError(f"leaf::Executor: unsupported fused activation: {activation}")


def graph_quantize(x, scale):
    x = _f32(x).reshape(-1)
    q = np.empty(x.shape, dtype=np.int8)
    if lib().oq_graph_quantize(_p(x), x.size, float(scale), _p(q)):
        raise ValueError("non-finite input or scale")
    return q


def gemm_i8_per_channel(a, b, bias, input_scale, weight_scales, relu=False):
    a = np.ascontiguousarray(a, dtype=np.int8)
    b = np.ascontiguousarray(b, dtype=np.int8)
    m, k = a.shape
    n = b.shape[1]
    out = np.empty((m, n), dtype=np.float32)
    bias = None if bias is None else _f32(bias)
    weight_scales = _f32(weight_scales)
    lib().oq_gemm_i8_per_channel(_p(a), _p(b), _p(bias), float(input_scale), _p(weight_scales),
                                 _p(out), m, k, n, int(relu))
    return out


def graph_linear(a, weight, weight_scales, input_scale, op_type="Gemm", trans_a=False, trans_b=False,
                 alpha=1.0, beta=1.0, c=None, activation=None):
    """execute_quant_linear (engine/src/executor.cpp:524-614) restated: the
    input transposed first with transA (:549-556), quantize_input (:220-230),
    the weight transposed to [k, n] with transB (:559-568),
    gemm_i8_per_channel (:574-576), then per element
    value = alpha * value; value += beta * C[index]; apply_activation
    (:593-613, :232-242), each step one float32 rounding."""
    gemm = op_type == "Gemm"
    if not gemm:
        trans_a = trans_b = False
        alpha, beta, c = 1.0, 0.0, None
    a = _f32(a)
    if trans_a:
        a2 = np.ascontiguousarray(a.T)
        out_shape = (a2.shape[0], None)
    else:
        a2 = a.reshape(-1, a.shape[-1])
        out_shape = tuple(a.shape[:-1]) + (None,)
    w = np.asarray(weight, dtype=np.int8)
    wk = np.ascontiguousarray(w.T) if trans_b else w
    m, k = a2.shape
    n = wk.shape[1]
    out_shape = out_shape[:-1] + (n,)
    qa = graph_quantize(a2, input_scale).reshape(m, k)
    v = gemm_i8_per_channel(qa, wk, None, input_scale, weight_scales)
    f = np.float32
    v = (f(alpha) * v).astype(np.float32)
    if c is not None:
        c = _f32(c)
        if c.size == 1:
            cb = np.full((m, n), c.reshape(-1)[0], dtype=np.float32)
        elif c.ndim == 1 and c.shape[0] == n:
            cb = np.broadcast_to(c, (m, n))
        elif tuple(c.shape) == out_shape:
            cb = c.reshape(m, n)
        else:
            raise ValueError("unsupported INT8 Gemm C broadcast shape")
        v = (v + (f(beta) * cb).astype(np.float32)).astype(np.float32)
    v = graph_activation(v, activation)
    return v.reshape(out_shape)


# --------------------------------------------------------------------------
# the reference's own kernels (oracle/_ref)
# --------------------------------------------------------------------------
def ref_quantize_i16(x):
    x = _f32(x)
    m, k = x.shape
    q = np.empty((m, k), dtype=np.int16)
    sx = np.empty(m, dtype=np.float32)
    if ref().leafref_quantize_i16(_p(x), m, k, _p(q), _p(sx)):
        raise RuntimeError(ref().leafref_last_error().decode())
    return q, sx


def ref_quantize_u8(x):
    x = _f32(x)
    m, k = x.shape
    q = np.empty((m, k), dtype=np.uint8)
    sx = np.empty(m, dtype=np.float32)
    if ref().leafref_quantize_u8(_p(x), m, k, _p(q), _p(sx)):
        raise RuntimeError(ref().leafref_last_error().decode())
    return q, sx


def ref_linear_int(x, weight, scales, bits, group, bias=None, threads=1, mode=0):
    x = _f32(x)
    m, k = x.shape
    n = scales.shape[0]
    y = np.empty((m, n), dtype=np.float32)
    weight = np.ascontiguousarray(weight)
    scales = _f32(scales)
    bias = None if bias is None else _f32(bias)
    if ref().leafref_linear_int(_p(x), m, k, _p(weight), _p(scales), n, bits, group, _p(bias),
                                _p(y), threads, mode):
        raise RuntimeError(ref().leafref_last_error().decode())
    return y


def ref_linear_float(x, weight, scales, bits, group, bias=None, threads=1, mode=0):
    x = _f32(x)
    m, k = x.shape
    n = weight.shape[0]
    y = np.empty((m, n), dtype=np.float32)
    weight = np.ascontiguousarray(weight)
    scales = None if scales is None else _f32(scales)
    bias = None if bias is None else _f32(bias)
    if ref().leafref_linear_float(_p(x), m, k, _p(weight), _p(scales), n, bits, group or 0,
                                  _p(bias), _p(y), threads, mode):
        raise RuntimeError(ref().leafref_last_error().decode())
    return y


def ref_gemm_i8_per_channel(a, b, bias, input_scale, weight_scales, relu=False, reference=False):
    a = np.ascontiguousarray(a, dtype=np.int8)
    b = np.ascontiguousarray(b, dtype=np.int8)
    m, k = a.shape
    n = b.shape[1]
    out = np.empty((m, n), dtype=np.float32)
    bias = None if bias is None else _f32(bias)
    weight_scales = _f32(weight_scales)
    fn = ref().leafref_gemm_i8_reference if reference else ref().leafref_gemm_i8_per_channel
    fn(_p(a), _p(b), _p(bias), float(input_scale), _p(weight_scales), _p(out), m, k, n, int(relu))
    return out


def ref_graph_activation(x, activation):
    """The reference's own apply_activation (executor.cpp:232-242) over an
    array, through oracle/_ref."""
    x = _f32(x).reshape(-1)
    y = np.empty_like(x)
    if ref().leafref_graph_activation(_p(x), x.size, (activation or "").encode(), _p(y)):
        raise ValueError(ref().leafref_graph_last_error().decode())
    return y


def ref_graph_quantize(x, scale):
    x = _f32(x).reshape(-1)
    q = np.empty(x.shape, dtype=np.int8)
    if ref().leafref_graph_quantize(_p(x), x.size, float(scale), _p(q)):
        raise ValueError(ref().leafref_graph_last_error().decode())
    return q


def cpu_count() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1
