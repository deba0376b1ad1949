"""Lazy elementwise fusion: expression DAG -> CUDA C -> NVRTC -> launch.

The graph keeps the reference's shape (``src/macmetalpy/_fusion.py``):
``InputNode`` / ``UnaryOpNode`` / ``BinaryOpNode`` with ``_shape``,
``_dtype`` and ``_depth``, ``_MAX_DEPTH = 16``, the fuseable op sets
(``_fusion.py:272-290``), CSE by node identity and a kernel cache keyed by
topology (``_fusion.py:297-436``).  Changes for B200:

* the emitter writes CUDA C into a hand-written grid-stride skeleton with
  aligned vector loads/stores (two vectors in flight per thread) instead of
  MSL, and NVRTC compiles it once per topology + dtype + input-layout key;
* inputs may be broadcast or strided views: a broadcast dimension is a
  stride-0 dimension indexed in the kernel (32-bit magic-number division),
  so nothing is materialised first (the reference copies every broadcast
  operand to full size, ``ndarray.py:515-545``);
* Python scalars are ``ScalarNode`` kernel parameters, not filled buffers
  (the reference allocates ``creation.full(shape, scalar)``, ``ndarray.py:1026``);
* ``CastNode`` fuses dtype conversion (the reference runs ``cast_op``
  kernels, ``_kernel_cache.py:45-59``);
* a reduction (or axis reduction) of a lazy array fuses the expression into
  the reduction kernel: the expression's inputs are read once and the
  intermediate array is never written.
"""

from __future__ import annotations

import ctypes
import math
import os
import threading

import numpy as np

from . import _cuda_backend as _cb
from ._config import get_config

_CFG = get_config()
from ._dtypes import CUDA_TYPE_NAMES, MMP_CODES

__all__ = [
    "FusionNode",
    "InputNode",
    "ScalarNode",
    "UnaryOpNode",
    "BinaryOpNode",
    "CastNode",
    "SelectNode",
    "materialize",
    "run_elementwise",
    "run_reduce",
    "_MAX_DEPTH",
    "_FUSEABLE_UNARY_OPS",
    "_FUSEABLE_BINARY_OPS",
]

_MAX_DEPTH = 16
_MAX_NDIM = 8
_BLOCK = 256
_BLOCK3 = (ctypes.c_uint * 3)(_BLOCK, 1, 1)

_CSRC = os.path.join(os.path.dirname(os.path.abspath(__file__)), "csrc")


# ---------------------------------------------------------------------------
# nodes
# ---------------------------------------------------------------------------


# Every node also carries, from its construction:
#   _sig    -- the structure of its graph (op names and dtypes, leaves by
#              kind only): the identity of the generated code up to the
#              leaves' data layout;
#   _leaves -- its leaf nodes (inputs and scalars) in the post-order the
#              planner visits them, repeats included.
# A repeated expression then finds its compiled kernel and launch template
# from (_sig, the leaves' sharing pattern and layouts) without walking the
# graph again.  Graphs whose leaf list would pass _MAX_LEAVES (heavy sharing
# doubles it per level) carry None and take the full planner.
_MAX_LEAVES = 64


def _join_leaves(*parts):
    n = 0
    for p in parts:
        if p is None:
            return None
        n += len(p)
    if n > _MAX_LEAVES:
        return None
    out = parts[0]
    for p in parts[1:]:
        out = out + p
    return out


def _dt(x):
    return x if isinstance(x, np.dtype) else np.dtype(x)


class FusionNode:
    __slots__ = ("_shape", "_dtype", "_depth", "_sig", "_leaves")


class InputNode(FusionNode):
    """A materialised device array (any view: offset, strides, broadcast)."""

    __slots__ = ("_array",)

    def __init__(self, array):
        self._array = array
        self._shape = array._shape
        self._dtype = array._dtype
        self._depth = 0
        self._sig = ("in", self._dtype)
        self._leaves = (self,)


class ScalarNode(FusionNode):
    """A scalar broadcast to any shape; passed to the kernel by value."""

    __slots__ = ("_value",)

    def __init__(self, value, dtype):
        self._dtype = np.dtype(dtype)
        self._value = np.asarray(value).astype(self._dtype)[()]
        self._shape = ()
        self._depth = 0
        self._sig = ("sc", self._dtype)
        self._leaves = (self,)


class UnaryOpNode(FusionNode):
    """``_in_dtype`` is the loop dtype the operand is cast to (equal to
    ``_dtype`` except for predicates such as isnan, whose result is bool)."""

    __slots__ = ("_op_name", "_input", "_in_dtype")

    def __init__(self, op_name, input_node, shape, dtype, in_dtype=None):
        self._op_name = op_name
        self._input = input_node
        self._dtype = _dt(dtype)
        self._in_dtype = _dt(in_dtype) if in_dtype is not None else self._dtype
        self._shape = shape if shape.__class__ is tuple else tuple(shape)
        self._depth = input_node._depth + 1
        self._leaves = input_node._leaves
        self._sig = None if self._leaves is None else \
            ("un", op_name, self._dtype, self._in_dtype, input_node._sig)


class BinaryOpNode(FusionNode):
    """``_in_dtype`` is the loop dtype both operands are cast to (equal to
    ``_dtype`` except for comparisons, whose result is bool)."""

    __slots__ = ("_op_name", "_lhs", "_rhs", "_in_dtype")

    def __init__(self, op_name, lhs, rhs, shape, dtype, in_dtype=None):
        self._op_name = op_name
        self._lhs = lhs
        self._rhs = rhs
        self._shape = shape if shape.__class__ is tuple else tuple(shape)
        self._dtype = _dt(dtype)
        self._in_dtype = _dt(in_dtype) if in_dtype is not None else self._dtype
        self._depth = max(lhs._depth, rhs._depth) + 1
        self._leaves = _join_leaves(lhs._leaves, rhs._leaves)
        self._sig = None if self._leaves is None else \
            ("bin", op_name, self._dtype, self._in_dtype, lhs._sig, rhs._sig)


class SelectNode(FusionNode):
    """``where(cond, x, y)``: cond is bool, x and y already cast to _dtype."""

    __slots__ = ("_cond", "_x", "_y")

    def __init__(self, cond, x, y, shape, dtype):
        self._cond = cond
        self._x = x
        self._y = y
        self._shape = tuple(shape)
        self._dtype = np.dtype(dtype)
        self._depth = max(cond._depth, x._depth, y._depth) + 1
        self._leaves = _join_leaves(cond._leaves, x._leaves, y._leaves)
        self._sig = None if self._leaves is None else ("sel", self._dtype, cond._sig, x._sig, y._sig)


def unary_node(op_name, inp, shape, out_dt, loop_dt):
    """UnaryOpNode from values that are already normalised (np.dtype
    objects, a shape tuple): the elementwise fast path's constructor."""
    n = UnaryOpNode.__new__(UnaryOpNode)
    n._op_name = op_name
    n._input = inp
    n._dtype = out_dt
    n._in_dtype = loop_dt
    n._shape = shape
    n._depth = inp._depth + 1
    lv = inp._leaves
    n._leaves = lv
    n._sig = None if lv is None else ("un", op_name, out_dt, loop_dt, inp._sig)
    return n


def binary_node(op_name, lhs, rhs, shape, out_dt, loop_dt):
    """BinaryOpNode from normalised values (see unary_node)."""
    n = BinaryOpNode.__new__(BinaryOpNode)
    n._op_name = op_name
    n._lhs = lhs
    n._rhs = rhs
    n._dtype = out_dt
    n._in_dtype = loop_dt
    n._shape = shape
    dl, dr = lhs._depth, rhs._depth
    n._depth = (dl if dl > dr else dr) + 1
    a, b = lhs._leaves, rhs._leaves
    lv = a + b if (a is not None and b is not None and len(a) + len(b) <= _MAX_LEAVES) else None
    n._leaves = lv
    n._sig = None if lv is None else ("bin", op_name, out_dt, loop_dt, lhs._sig, rhs._sig)
    return n


class CastNode(FusionNode):
    __slots__ = ("_input",)

    def __init__(self, input_node, dtype):
        self._input = input_node
        self._shape = input_node._shape
        self._dtype = np.dtype(dtype)
        self._depth = input_node._depth + 1
        self._leaves = input_node._leaves
        self._sig = None if self._leaves is None else ("cast", self._dtype, input_node._sig)


# ---------------------------------------------------------------------------
# op tables: numpy ufunc + CUDA expression per op name
# ---------------------------------------------------------------------------

_UNARY_UFUNC = {
    "neg_op": np.negative, "negative_op": np.negative, "positive_op": np.positive,
    "abs_op": np.absolute, "sqrt_op": np.sqrt, "exp_op": np.exp, "log_op": np.log,
    "sin_op": np.sin, "cos_op": np.cos, "tan_op": np.tan, "asin_op": np.arcsin,
    "acos_op": np.arccos, "atan_op": np.arctan, "sinh_op": np.sinh, "cosh_op": np.cosh,
    "tanh_op": np.tanh, "log2_op": np.log2, "log10_op": np.log10, "exp2_op": np.exp2,
    "expm1_op": np.expm1, "log1p_op": np.log1p, "cbrt_op": np.cbrt,
    "reciprocal_op": np.reciprocal, "rint_op": np.rint, "trunc_op": np.trunc,
    "asinh_op": np.arcsinh, "acosh_op": np.arccosh, "atanh_op": np.arctanh,
    "degrees_op": np.degrees, "radians_op": np.radians, "sign_op": np.sign,
    "floor_op": np.floor, "ceil_op": np.ceil, "square_op": np.square,
    "isnan_op": np.isnan, "isinf_op": np.isinf, "isfinite_op": np.isfinite,
    "signbit_op": np.signbit, "logical_not_op": np.logical_not, "invert_op": np.invert,
}

_BINARY_UFUNC = {
    "add_op": np.add, "sub_op": np.subtract, "mul_op": np.multiply, "div_op": np.true_divide,
    "pow_op": np.power, "max_op": np.maximum, "min_op": np.minimum, "fmax_op": np.fmax,
    "fmin_op": np.fmin, "atan2_op": np.arctan2, "hypot_op": np.hypot,
    "floor_divide_op": np.floor_divide, "fmod_op": np.fmod, "mod_op": np.remainder,
    "copysign_op": np.copysign, "nextafter_op": np.nextafter, "logaddexp_op": np.logaddexp,
    "logaddexp2_op": np.logaddexp2, "heaviside_op": np.heaviside,
    "lt_op": np.less, "le_op": np.less_equal, "gt_op": np.greater, "ge_op": np.greater_equal,
    "eq_op": np.equal, "ne_op": np.not_equal,
    "logical_and_op": np.logical_and, "logical_or_op": np.logical_or,
    "logical_xor_op": np.logical_xor, "bitwise_and_op": np.bitwise_and,
    "bitwise_or_op": np.bitwise_or, "bitwise_xor_op": np.bitwise_xor,
    "left_shift_op": np.left_shift, "right_shift_op": np.right_shift,
}

_FUSEABLE_UNARY_OPS = frozenset(_UNARY_UFUNC)
_FUSEABLE_BINARY_OPS = frozenset(_BINARY_UFUNC)

_MATH1 = {
    "sqrt_op": "m_sqrt", "exp_op": "m_exp", "log_op": "m_log", "sin_op": "m_sin",
    "cos_op": "m_cos", "tan_op": "m_tan", "asin_op": "m_asin", "acos_op": "m_acos",
    "atan_op": "m_atan", "sinh_op": "m_sinh", "cosh_op": "m_cosh", "tanh_op": "m_tanh",
    "log2_op": "m_log2", "log10_op": "m_log10", "exp2_op": "m_exp2", "expm1_op": "m_expm1",
    "log1p_op": "m_log1p", "cbrt_op": "m_cbrt", "asinh_op": "m_asinh", "acosh_op": "m_acosh",
    "atanh_op": "m_atanh", "floor_op": "m_floor", "ceil_op": "m_ceil", "trunc_op": "m_trunc",
    "rint_op": "m_rint",
}

_MATH2 = {
    "atan2_op": "m_atan2", "hypot_op": "m_hypot", "copysign_op": "m_copysign",
    "nextafter_op": "m_nextafter", "logaddexp_op": "logaddexp", "logaddexp2_op": "logaddexp2",
    "heaviside_op": "heaviside",
}

_CMP = {"lt_op": "<", "le_op": "<=", "gt_op": ">", "ge_op": ">=", "eq_op": "==", "ne_op": "!="}


# bool predicates on the loop value (numpy: NaN is true, only zero is false)
_LOGIC = {"logical_and_op": "&&", "logical_or_op": "||", "logical_xor_op": "!="}
_BITS = {"bitwise_and_op": "&", "bitwise_or_op": "|", "bitwise_xor_op": "^"}
_PRED = {"isnan_op": "mmpd::isnan_", "isinf_op": "mmpf::isinf_", "isfinite_op": "mmpf::isfinite_",
         "signbit_op": "mmpf::signbit_"}

# Ops whose generated code is a library math call, a comparison, a select,
# a bit operation or one of the rn_* operations: an expression made only of
# these is compiled with --fmad=true (contraction inside the math library,
# which CUDA's documented error bounds assume).  Every other op -- the
# division family (floor_divide, mod, fmod), pow, logaddexp(2), hypot,
# atan2, heaviside, nextafter -- has helpers whose exactness relies on each
# + and * being rounded on its own, so expressions with them keep
# --fmad=false.
_FMAD_SAFE = frozenset(
    set(_MATH1) | {"neg_op", "negative_op", "positive_op", "abs_op", "sign_op", "square_op", "degrees_op",
                   "radians_op", "isnan_op", "isinf_op", "isfinite_op", "signbit_op", "logical_not_op",
                   "invert_op", "reciprocal_op", "add_op", "sub_op", "mul_op", "div_op", "max_op",
                   "min_op", "fmax_op", "fmin_op", "copysign_op", "left_shift_op", "right_shift_op"}
    | set(_CMP) | set(_LOGIC) | set(_BITS))


def _is_float(dt) -> bool:
    return dt.kind == "f"


def _arith_name(dt) -> str:
    return "float" if dt == np.float16 else CUDA_TYPE_NAMES[dt]


def _float_literal(v: float, dt) -> str:
    h = float(v).hex()
    return f"{h}f" if dt != np.float64 else h


def _unary_expr(op: str, dt, x: str) -> str:
    R = _arith_name(dt)
    f = _is_float(dt)
    if op in ("neg_op", "negative_op"):
        return f"(-{x})" if f else f"({R})({R}(0) - {x})"
    if op == "positive_op":
        return x
    if op == "abs_op":
        if dt == np.bool_:
            return x
        return f"mmpf::m_fabs({x})" if f else f"mmpf::i_abs<{R}>({x})"
    if op == "sign_op":
        return f"mmpf::sign_<{R}>({x})"
    if op == "square_op":
        return f"mmpf::rn_mul({x}, {x})" if f else f"({x} * {x})"
    if op == "reciprocal_op":
        return f"({R}(1) / {x})" if f else f"({x} == {R}(0) ? {R}(0) : ({R})({R}(1) / {x}))"
    if op == "degrees_op":
        c = np.array(180.0, dt) / np.array(np.pi, dt) if dt != np.float16 else np.float32(180) / np.float32(np.pi)
        return f"mmpf::rn_mul({x}, {_float_literal(float(c), dt if dt != np.float16 else np.dtype(np.float32))})"
    if op == "radians_op":
        c = np.array(np.pi, dt) / np.array(180.0, dt) if dt != np.float16 else np.float32(np.pi) / np.float32(180)
        return f"mmpf::rn_mul({x}, {_float_literal(float(c), dt if dt != np.float16 else np.dtype(np.float32))})"
    if op == "cast":
        return x
    if op in _PRED:
        return f"{_PRED[op]}({x})"
    if op == "logical_not_op":
        return f"(({x}) == {R}(0))"
    if op == "invert_op":
        if dt == np.bool_:
            return f"(!{x})"
        if f:
            raise TypeError(f"invert needs an integer or bool loop dtype, got {dt}")
        return f"({R})(~{x})"
    if op in _MATH1:
        if not f:
            raise TypeError(f"{op} needs a float loop dtype, got {dt}")
        return f"mmpf::{_MATH1[op]}({x})"
    raise ValueError(f"Unknown unary op for fusion: {op}")


def _binary_expr(op: str, dt, a: str, b: str) -> str:
    R = _arith_name(dt)
    f = _is_float(dt)
    isbool = dt == np.bool_
    if op == "add_op":
        return f"({a} || {b})" if isbool else (f"mmpf::rn_add({a}, {b})" if f else f"({a} + {b})")
    if op == "sub_op":
        return f"mmpf::rn_sub({a}, {b})" if f else f"({a} - {b})"
    if op == "mul_op":
        return f"({a} && {b})" if isbool else (f"mmpf::rn_mul({a}, {b})" if f else f"({a} * {b})")
    if op == "div_op":
        return f"({a} / {b})"
    if op == "floor_divide_op":
        if isbool:
            return f"({a} && {b})"
        return f"mmpf::floor_divide_f<{R}>({a}, {b})" if f else f"mmpf::floor_divide_i<{R}>({a}, {b})"
    if op == "mod_op":  # the reference's composite a - floor_divide(a, b) * b
        if isbool:
            return f"(({a}) && !({b}))"
        T = CUDA_TYPE_NAMES[dt]
        return f"mmpf::ref_mod_f<{T}, {R}>({a}, {b})" if f else f"mmpf::ref_mod_i<{R}>({a}, {b})"
    if op == "fmod_op":
        return f"mmpf::m_fmod({a}, {b})" if f else f"mmpf::i_fmod<{R}>({a}, {b})"
    if op == "pow_op":
        if isbool:
            return f"({a} || !{b})"
        return f"mmpf::m_pow({a}, {b})" if f else f"mmpf::i_power<{R}>({a}, {b})"
    if op == "max_op":
        return f"mmpf::maximum<{R}>({a}, {b})"
    if op == "min_op":
        return f"mmpf::minimum<{R}>({a}, {b})"
    if op == "fmax_op":
        return f"mmpf::fmax_<{R}>({a}, {b})"
    if op == "fmin_op":
        return f"mmpf::fmin_<{R}>({a}, {b})"
    if op in _CMP:
        return f"({a} {_CMP[op]} {b})"
    if op in _LOGIC:
        return f"((({a}) != {R}(0)) {_LOGIC[op]} (({b}) != {R}(0)))"
    if op in _BITS:
        if f:
            raise TypeError(f"{op} needs an integer or bool loop dtype, got {dt}")
        return f"({a} {_BITS[op]} {b})"
    if op in ("left_shift_op", "right_shift_op"):
        if f or isbool:
            raise TypeError(f"{op} needs an integer loop dtype, got {dt}")
        return f"mmpf::{'shl_' if op == 'left_shift_op' else 'shr_'}<{R}>({a}, {b})"
    if op in _MATH2:
        if not f:
            raise TypeError(f"{op} needs a float loop dtype, got {dt}")
        name = _MATH2[op]
        tmpl = f"<{R}>" if name in ("logaddexp", "logaddexp2", "heaviside") else ""
        return f"mmpf::{name}{tmpl}({a}, {b})"
    raise ValueError(f"Unknown binary op for fusion: {op}")


# ---------------------------------------------------------------------------
# layout analysis
# ---------------------------------------------------------------------------


def _fastdiv(d: int) -> tuple[int, int]:
    """(m, s) with q = (umulhi(n, m) + n) >> s == n // d for all 32-bit n
    (Granlund & Montgomery 1994)."""
    if d < 1:
        d = 1
    l = (d - 1).bit_length()  # ceil(log2(d))
    m = ((1 << 32) * ((1 << l) - d)) // d + 1
    return m & 0xFFFFFFFF, l


def _c_strides(shape):
    st = [1] * len(shape)
    for i in range(len(shape) - 2, -1, -1):
        st[i] = st[i + 1] * shape[i + 1]
    return tuple(st)


def _bcast_strides(shape, strides, target):
    nd = len(target) - len(shape)
    out = [0] * nd
    for s, st, t in zip(shape, strides, target[nd:]):
        out.append(0 if s == 1 else st)
    return out


def _collapse(shape, stride_lists):
    """Drop size-1 dims and merge adjacent dims that are contiguous for every
    operand.  Returns (shape, [strides per operand])."""
    dims = [i for i, s in enumerate(shape) if s != 1]
    shp = [shape[i] for i in dims]
    sts = [[st[i] for i in dims] for st in stride_lists]
    if not shp:
        return [1], [[0] for _ in stride_lists]
    out_shape = [shp[0]]
    out_st = [[st[0]] for st in sts]
    for d in range(1, len(shp)):
        mergeable = all(o[-1] == st[d] * shp[d] for o, st in zip(out_st, sts))
        if mergeable:
            out_shape[-1] *= shp[d]
            for o, st in zip(out_st, sts):
                o[-1] = st[d]
        else:
            out_shape.append(shp[d])
            for o, st in zip(out_st, sts):
                o.append(st[d])
    return out_shape, out_st


class _Plan:
    """Everything the emitter and the launcher need for one graph."""

    def __init__(self, root, out_shape, vec):
        self.root = root
        self.out_shape = tuple(out_shape)
        self.n = int(math.prod(self.out_shape)) if self.out_shape else 1
        self.order = []  # post-order nodes (CSE by id)
        self.ids = {}
        self.inputs = []  # list of ndarray views (dedup)
        self.input_key = {}
        self.scalars = []  # ScalarNode list
        self.topo = []  # per node, its part of the code key (built during the walk)
        self._visit(root)
        self.vec = vec
        self.fmad = all(t[0] not in ("un", "bin") or t[1] in _FMAD_SAFE for t in self.topo)
        self._layout()

    def _visit(self, node):
        nid = id(node)
        idx = self.ids.get(nid)
        if idx is not None:
            return idx
        if isinstance(node, InputNode):
            a = node._array
            key = (a._ptr, a._shape, a._strides, a._dtype)
            slot = self.input_key.get(key)
            if slot is None:
                slot = self.input_key[key] = len(self.inputs)
                self.inputs.append(a)
            t = ("in", slot, node._dtype)
        elif isinstance(node, ScalarNode):
            t = ("sc", len(self.scalars), node._dtype)
            self.scalars.append(node)
        elif isinstance(node, UnaryOpNode):
            t = ("un", node._op_name, node._dtype, node._in_dtype, self._visit(node._input))
        elif isinstance(node, CastNode):
            t = ("cast", node._dtype, self._visit(node._input))
        elif isinstance(node, BinaryOpNode):
            t = ("bin", node._op_name, node._dtype, node._in_dtype, self._visit(node._lhs), self._visit(node._rhs))
        elif isinstance(node, SelectNode):
            t = ("sel", node._dtype, self._visit(node._cond), self._visit(node._x), self._visit(node._y))
        else:
            raise TypeError(f"Unknown node type: {type(node)}")
        idx = len(self.order)
        self.order.append(node)
        self.topo.append(t)
        self.ids[nid] = idx
        return idx

    def _layout(self):
        shape = self.out_shape
        st_lists = [_bcast_strides(a._shape, a._strides, shape) for a in self.inputs]
        if self.n == 0:
            self.cshape, self.cstrides = [1], [[0] for _ in self.inputs]
        else:
            self.cshape, self.cstrides = _collapse(list(shape) if shape else [1], st_lists or [])
            if not st_lists:
                self.cstrides = []
        nd = len(self.cshape)
        cst = _c_strides(self.cshape)
        kinds = []
        V = self.vec
        inner = self.cshape[-1]
        for a, st in zip(self.inputs, self.cstrides):
            isz = a._dtype.itemsize
            ptr = a._ptr
            if all(s == 0 for s in st):
                kinds.append("bc")
            elif list(st) == list(cst):
                kinds.append("ct" if ptr % (V * isz) == 0 else "ctu")
            elif st[-1] == 1 and ptr % (V * isz) == 0 and all(s % V == 0 for s in st[:-1]):
                kinds.append("sv")
            elif st[-1] == 0:
                kinds.append("sb")
            else:
                kinds.append("sg")
        self.kinds = kinds
        has_strided = any(k in ("sv", "sb", "sg") for k in kinds)
        self.strided = has_strided
        self.nd = nd if has_strided else 1
        # vector path: contiguous inputs aligned; strided inputs need an
        # inner extent that is a multiple of V
        self.vec_ok = all(k != "ctu" for k in kinds) and (not has_strided or inner % V == 0)
        span = 0
        for a, st in zip(self.inputs, self.cstrides):
            span = max(span, sum(abs(s) * (e - 1) for s, e in zip(st, self.cshape)))
        self.idx64 = self.n >= (1 << 31) or span >= (1 << 31)

    # -- identity of the generated code (not of the data)
    def key(self):
        kinds = tuple((k, a._dtype) for k, a in zip(self.kinds, self.inputs))
        return (tuple(self.topo), kinds, self.nd if self.strided else 0, self.idx64, self.vec,
                bool(get_config().fast_math), self.fmad)


# ---------------------------------------------------------------------------
# CUDA source generation
# ---------------------------------------------------------------------------


def _ct(dt) -> str:
    return CUDA_TYPE_NAMES[np.dtype(dt)]


def _emit_loader(plan: _Plan) -> tuple[str, list[str]]:
    """Return (struct source, kernel parameter declarations in order)."""
    out_t = _ct(plan.root._dtype)
    I = "long long" if plan.idx64 else "int"
    U = "unsigned long long" if plan.idx64 else "unsigned"
    nd = plan.nd
    params = []
    members = []
    for k, a in enumerate(plan.inputs):
        t = _ct(a._dtype)
        params.append(f"const {t}* __restrict__ in{k}")
        members.append(f"  const {t}* in{k};")
        if plan.kinds[k] in ("sv", "sb", "sg"):
            for d in range(nd):
                params.append(f"long long st{k}_{d}")
            members.append(f"  {I} st{k}[{nd}];")
    for j, s in enumerate(plan.scalars):
        t = "unsigned short" if s._dtype == np.float16 else _ct(s._dtype)
        params.append(f"{t} sc{j}")
        members.append(f"  {_ct(s._dtype)} sc{j};")
    if plan.strided:
        for d in range(nd):
            params.append(f"long long dim{d}")
            params.append(f"unsigned fdm{d}")
            params.append(f"unsigned fds{d}")
        members.append(f"  {I} dim[{nd}];")
        members.append(f"  mmpd::FastDiv fd[{nd}];")
    params.append("int aligned")
    members.append("  int aligned;")

    # expression body: eval(a0, a1, ...) on raw input element values
    args = ", ".join(f"{_ct(a._dtype)} a{k}" for k, a in enumerate(plan.inputs))
    lines = []
    names = {}
    for i, node in enumerate(plan.order):
        t = _ct(node._dtype)
        nm = f"t{i}"
        names[id(node)] = nm
        if isinstance(node, InputNode):
            a = node._array
            k = plan.input_key[(a._ptr, a._shape, a._strides, a._dtype)]
            lines.append(f"    const {t} {nm} = a{k};")
        elif isinstance(node, ScalarNode):
            lines.append(f"    const {t} {nm} = sc{plan.scalars.index(node)};")
        elif isinstance(node, (UnaryOpNode, CastNode)):
            x = names[id(node._input)]
            if isinstance(node, CastNode):
                lines.append(f"    const {t} {nm} = mmpd::cvt<{t}>({x});")
            else:
                ldt = node._in_dtype
                R = _arith_name(ldt)
                xv = f"mmpd::cvt<{R}>(mmpd::cvt<{_ct(ldt)}>({x}))"
                lines.append(f"    const {R} x{i} = {xv};")
                lines.append(f"    const {t} {nm} = mmpd::cvt<{t}>({_unary_expr(node._op_name, ldt, 'x' + str(i))});")
        elif isinstance(node, SelectNode):
            c_, x_, y_ = names[id(node._cond)], names[id(node._x)], names[id(node._y)]
            lines.append(f"    const {t} {nm} = mmpd::cvt<bool>({c_}) ? mmpd::cvt<{t}>({x_}) : mmpd::cvt<{t}>({y_});")
        else:
            ldt = node._in_dtype
            lt = _ct(ldt)
            R = _arith_name(ldt)
            a_ = names[id(node._lhs)]
            b_ = names[id(node._rhs)]
            if ldt == np.float16:
                av = f"mmpd::cvt<float>(mmpd::cvt<__half>({a_}))"
                bv = f"mmpd::cvt<float>(mmpd::cvt<__half>({b_}))"
            else:
                av = f"mmpd::cvt<{lt}>({a_})"
                bv = f"mmpd::cvt<{lt}>({b_})"
            lines.append(f"    const {R} l{i} = {av};")
            lines.append(f"    const {R} r{i} = {bv};")
            lines.append(f"    const {t} {nm} = mmpd::cvt<{t}>({_binary_expr(node._op_name, ldt, f'l{i}', f'r{i}')});")
    root = names[id(plan.root)]
    body = "\n".join(lines)

    # index decomposition
    def offsets_code(var_i: str, need: list[int]) -> str:
        if not need:
            return ""
        c = [f"    {U} r_ = ({U})({var_i});"]
        for k in need:
            c.append(f"    {I} o{k} = 0;")
        for d in range(nd - 1, 0, -1):
            if plan.idx64:
                c.append(f"    {{ {U} q_ = r_ / ({U})dim[{d}]; {I} c_ = ({I})(r_ - q_ * ({U})dim[{d}]);")
            else:
                c.append(f"    {{ {U} q_ = fd[{d}].div(r_); {I} c_ = ({I})(r_ - q_ * ({U})dim[{d}]);")
            for k in need:
                c.append(f"      o{k} += c_ * st{k}[{d}];")
            c.append("      r_ = q_; }")
        for k in need:
            c.append(f"    o{k} += ({I})r_ * st{k}[0];")
        return "\n".join(c)

    strided_in = [k for k, kd in enumerate(plan.kinds) if kd in ("sv", "sb", "sg")]
    scalar_loads = []
    for k, kd in enumerate(plan.kinds):
        if kd in ("ct", "ctu"):
            scalar_loads.append(f"in{k}[i]")
        elif kd == "bc":
            scalar_loads.append(f"in{k}[0]")
        else:
            scalar_loads.append(f"in{k}[o{k}]")
    op_scalar = offsets_code("i", strided_in)

    V = plan.vec
    raw_members, load_lines, apply_args = [], [], []
    for k, kd in enumerate(plan.kinds):
        t = _ct(plan.inputs[k]._dtype)
        if kd in ("ct", "sv"):
            raw_members.append(f"    mmpd::Vec<{t}, V> v{k};")
            src_ = f"in{k} + i" if kd == "ct" else f"in{k} + o{k}"
            load_lines.append(f"    r.v{k} = mmpd::ldvec<{t}, V>({src_});")
            apply_args.append(f"r.v{k}.v[j]")
        elif kd in ("bc", "sb"):
            raw_members.append(f"    {t} b{k};")
            load_lines.append(f"    r.b{k} = in{k}[{'0' if kd == 'bc' else f'o{k}'}];")
            apply_args.append(f"r.b{k}")
        else:  # sg (gather) / ctu (unaligned contiguous)
            raw_members.append(f"    {t} g{k}[V];")
            if kd == "sg":
                load_lines.append(f"#pragma unroll\n    for (int j = 0; j < V; ++j) r.g{k}[j] = in{k}[o{k} + ({I})j * st{k}[{nd - 1}]];")
            else:
                load_lines.append(f"#pragma unroll\n    for (int j = 0; j < V; ++j) r.g{k}[j] = in{k}[i + j];")
            apply_args.append(f"r.g{k}[j]")
    op_vec = offsets_code("i", strided_in)
    raw_body = "\n".join(raw_members) if raw_members else "    int unused;"

    src = f"""
struct Loader {{
  typedef {out_t} value_type;
{chr(10).join(members)}
  template <int V>
  struct Raw {{
{raw_body}
  }};
  __device__ __forceinline__ {out_t} eval({args}) const {{
{body}
    return {root};
  }}
  __device__ __forceinline__ {out_t} operator()(long long i) const {{
{op_scalar}
    return eval({", ".join(scalar_loads)});
  }}
  // raw loads of V elements at i (no arithmetic, so several vectors of
  // loads can be in flight before any evaluation)
  template <int V>
  __device__ __forceinline__ void load(long long i, Raw<V> &r) const {{
{op_vec}
{chr(10).join(load_lines)}
  }}
  template <int V>
  __device__ __forceinline__ void apply(const Raw<V> &r, {out_t} (&out)[V]) const {{
#pragma unroll
    for (int j = 0; j < V; ++j) out[j] = eval({", ".join(apply_args)});
  }}
  template <int V>
  __device__ __forceinline__ void vec(long long i, {out_t} (&out)[V]) const {{
    Raw<V> r;
    load<V>(i, r);
    apply<V>(r, out);
  }}
}};
"""
    return src, params


def _loader_init(plan: _Plan) -> str:
    nd = plan.nd
    c = ["  Loader L;"]
    for k in range(len(plan.inputs)):
        c.append(f"  L.in{k} = in{k};")
        if plan.kinds[k] in ("sv", "sb", "sg"):
            for d in range(nd):
                c.append(f"  L.st{k}[{d}] = st{k}_{d};")
    for j, s in enumerate(plan.scalars):
        if s._dtype == np.float16:
            c.append(f"  L.sc{j} = __ushort_as_half(sc{j});")
        else:
            c.append(f"  L.sc{j} = sc{j};")
    if plan.strided:
        I = "long long" if plan.idx64 else "int"
        for d in range(nd):
            c.append(f"  L.dim[{d}] = ({I})dim{d}; L.fd[{d}].d = (unsigned)dim{d}; "
                     f"L.fd[{d}].m = fdm{d}; L.fd[{d}].s = fds{d};")
    c.append("  L.aligned = aligned;")
    return "\n".join(c)


_HEADER = """#include "mmp_device.cuh"
#include "mmp_fused_ops.cuh"
"""


def _ew_source(plan: _Plan, out_strided: bool) -> str:
    loader, params = _emit_loader(plan)
    out_t = _ct(plan.root._dtype)
    V = plan.vec
    p = ",\n    ".join(params + [f"{out_t}* __restrict__ out", "long long n"] +
                        ([f"long long ost{d}" for d in range(plan.nd)] if out_strided else []))
    if out_strided:
        I = "long long" if plan.idx64 else "int"
        U = "unsigned long long" if plan.idx64 else "unsigned"
        dec = [f"    {U} r_ = ({U})i; {I} oo = 0;"]
        for d in range(plan.nd - 1, 0, -1):
            dec.append(f"    {{ {U} q_ = r_ / ({U})dim{d}; {I} c_ = ({I})(r_ - q_ * ({U})dim{d}); "
                       f"oo += c_ * ({I})ost{d}; r_ = q_; }}")
        dec.append(f"    oo += ({I})r_ * ({I})ost0;")
        body = f"""  for (long long i = t; i < n; i += nth) {{
{chr(10).join(dec)}
    out[oo] = L(i);
  }}"""
    else:
        body = f"""  if (L.aligned) {{
    const long long nv = n / {V};
    long long v = t;
    // four vectors per thread per iteration: all loads first, then math
    for (; v + 3 * nth < nv; v += 4 * nth) {{
      Loader::Raw<{V}> r0, r1, r2, r3;
      L.load<{V}>(v * {V}, r0);
      L.load<{V}>((v + nth) * {V}, r1);
      L.load<{V}>((v + 2 * nth) * {V}, r2);
      L.load<{V}>((v + 3 * nth) * {V}, r3);
      mmpd::Vec<{out_t}, {V}> w0, w1, w2, w3;
      L.apply<{V}>(r0, w0.v);
      L.apply<{V}>(r1, w1.v);
      L.apply<{V}>(r2, w2.v);
      L.apply<{V}>(r3, w3.v);
      mmpd::stvec<{out_t}, {V}>(out + v * {V}, w0);
      mmpd::stvec<{out_t}, {V}>(out + (v + nth) * {V}, w1);
      mmpd::stvec<{out_t}, {V}>(out + (v + 2 * nth) * {V}, w2);
      mmpd::stvec<{out_t}, {V}>(out + (v + 3 * nth) * {V}, w3);
    }}
    for (; v < nv; v += nth) {{
      mmpd::Vec<{out_t}, {V}> w0;
      L.vec<{V}>(v * {V}, w0.v);
      mmpd::stvec<{out_t}, {V}>(out + v * {V}, w0);
    }}
    for (long long i = nv * {V} + t; i < n; i += nth) out[i] = L(i);
  }} else {{
    for (long long i = t; i < n; i += nth) out[i] = L(i);
  }}"""
    return f"""{_HEADER}
{loader}
extern "C" __global__ void __launch_bounds__({_BLOCK}) mmp_fused_ew(
    {p}) {{
{_loader_init(plan)}
  const long long nth = (long long)gridDim.x * {_BLOCK};
  const long long t = (long long)blockIdx.x * {_BLOCK} + threadIdx.x;
{body}
}}
"""


def _red_source(plan: _Plan, opc: int, kind: str, cv: int) -> str:
    """Reduction kernel over the expression: the templates of mmp_reduce.cuh
    instantiated with the generated loader."""
    loader, params = _emit_loader(plan)
    T = _ct(plan.root._dtype)
    if kind == "full":
        extra = ["long long n", "void* out", "int out_dt", "double ddof", "void* scratch",
                 "unsigned* ticket", "mmpd::PartialOut* part"]
        call = f"mmpd::reduce_full_body<{opc}, {T}, Loader>(L, n, out, out_dt, ddof, scratch, ticket, part);"
    elif kind == "rows_block":
        extra = ["long long rows", "long long k", "void* out", "int out_dt", "double ddof"]
        call = f"mmpd::reduce_rows_block_body<{opc}, {T}, Loader>(L, rows, k, out, out_dt, ddof);"
    elif kind == "rows_warp":
        extra = ["long long rows", "long long k", "void* out", "int out_dt", "double ddof"]
        call = f"mmpd::reduce_rows_warp_body<{opc}, {T}, Loader>(L, rows, k, out, out_dt, ddof);"
    else:
        extra = ["long long outer", "long long k", "long long inner", "long long kchunk", "void* out",
                 "int out_dt", "double ddof", "void* scratch", "unsigned* tickets"]
        call = (f"mmpd::reduce_cols_body<{opc}, {T}, Loader, {cv}>(L, outer, k, inner, kchunk, out, "
                f"out_dt, ddof, scratch, tickets);")
    plist = ",\n    ".join(params + extra)
    return f"""{_HEADER}#include "mmp_reduce.cuh"
{loader}
extern "C" __global__ void __launch_bounds__(mmpd::RBLOCK) mmp_fused_reduce(
    {plist}) {{
{_loader_init(plan)}
  {call}
}}
"""


# ---------------------------------------------------------------------------
# compile + launch
# ---------------------------------------------------------------------------

_cache: dict = {}
_cache_lock = threading.Lock()
_CUDA_INC = None


def _options(fmad: bool = False) -> bytes:
    global _CUDA_INC
    if _CUDA_INC is None:
        cands = [os.environ.get("CUDA_HOME", ""), "/usr/local/cuda"]
        _CUDA_INC = next((os.path.join(c, "include") for c in cands
                          if c and os.path.exists(os.path.join(c, "include", "cuda_fp16.h"))),
                         "/usr/local/cuda/include")
    opts = ["--gpu-architecture=sm_100a", "-std=c++17", f"-I{_CSRC}", f"-I{_CUDA_INC}",
            "--fmad=true" if fmad else "--fmad=false", "-lineinfo", "-default-device"]
    if get_config().fast_math:
        opts.append("--use_fast_math")
    return "\n".join(opts).encode()


def compile_kernel(src: str, name: str, fmad: bool = False) -> int:
    """NVRTC-compile ``src`` and return the handle of kernel ``name``."""
    fn = ctypes.c_void_p()
    log = ctypes.create_string_buffer(1 << 16)
    rc = _cb.lib.mmp_compile(src.encode(), name.encode(), _options(fmad), ctypes.byref(fn), log, len(log))
    if rc != 0:
        msg = _cb.lib.mmp_last_error().decode(errors="replace")
        raise RuntimeError(f"fused kernel compile failed: {msg}\n--- source ---\n{src}")
    return fn.value


def _get(key, make_src, name, fmad=False):
    with _cache_lock:
        fn = _cache.get(key)
    if fn is None:
        fn = compile_kernel(make_src(), name, fmad)
        with _cache_lock:
            _cache[key] = fn
    return fn


def _ctype_scalar(v, dt):
    dt = np.dtype(dt)
    if dt == np.float16:
        return ctypes.c_uint16(int(np.asarray(v, np.float16).view(np.uint16)))
    m = {
        np.dtype(np.bool_): ctypes.c_bool, np.dtype(np.int8): ctypes.c_int8,
        np.dtype(np.uint8): ctypes.c_uint8, np.dtype(np.int16): ctypes.c_int16,
        np.dtype(np.uint16): ctypes.c_uint16, np.dtype(np.int32): ctypes.c_int32,
        np.dtype(np.uint32): ctypes.c_uint32, np.dtype(np.int64): ctypes.c_int64,
        np.dtype(np.uint64): ctypes.c_uint64, np.dtype(np.float32): ctypes.c_float,
        np.dtype(np.float64): ctypes.c_double,
    }[dt]
    return m(v.item() if hasattr(v, "item") else v)


def _arg_template(plan: _Plan) -> list:
    """The loader's kernel arguments with the per-call values left as
    markers -- ("in", k): input k's pointer, ("sc", j, dtype): scalar j --
    and everything that follows from the layout built once."""
    t = []
    for k in range(len(plan.inputs)):
        t.append(("in", k))
        if plan.kinds[k] in ("sv", "sb", "sg"):
            for s in plan.cstrides[k]:
                t.append(ctypes.c_longlong(int(s)))
    for j, sc in enumerate(plan.scalars):
        t.append(("sc", j, sc._dtype))
    if plan.strided:
        for d in plan.cshape:
            m, sh = _fastdiv(int(d))
            t.append(ctypes.c_longlong(int(d)))
            t.append(ctypes.c_uint(m))
            t.append(ctypes.c_uint(sh))
    t.append(ctypes.c_int(1 if plan.vec_ok else 0))
    return t


def _fill(template, inputs, scalars) -> list:
    out = []
    for x in template:
        if x.__class__ is tuple:
            if x[0] == "in":
                out.append(ctypes.c_void_p(inputs[x[1]]._ptr))
            else:
                out.append(_ctype_scalar(scalars[x[1]]._value, x[2]))
        else:
            out.append(x)
    return out


def _loader_args(plan: _Plan) -> list:
    return _fill(_arg_template(plan), plan.inputs, plan.scalars)


# ---------------------------------------------------------------------------
# launch templates: a repeated expression skips the planner
# ---------------------------------------------------------------------------

_tmpl: dict = {}
_TMPL_MAX = 4096


def _leaf_key(node, V):
    """(distinct inputs, distinct scalars, key part) from the node's leaf
    list: the inputs are deduplicated by view (pointer, shape, strides,
    dtype) and the scalars by node, in first-occurrence order -- the order
    the planner assigns their kernel slots -- and the key records which
    leaf is which slot and each input's layout (what the planner's layout
    classification reads)."""
    ins, scal, pat = [], [], []
    ikeys, sids = {}, {}
    for lf in node._leaves:
        if lf.__class__ is InputNode:
            a = lf._array
            k = (a._ptr, a._shape, a._strides, a._dtype)
            slot = ikeys.get(k)
            if slot is None:
                slot = ikeys[k] = len(ins)
                ins.append(a)
            pat.append(slot)
        else:
            slot = sids.get(id(lf))
            if slot is None:
                slot = sids[id(lf)] = len(scal)
                scal.append(lf)
            pat.append(-1 - slot)
    lay = tuple((a._shape, a._strides, a._dtype, a._ptr % (V * a._dtype.itemsize) == 0) for a in ins)
    return ins, scal, (tuple(pat), lay)


def _same_slots(plan: _Plan, ins, scal) -> bool:
    return (len(plan.inputs) == len(ins) and all(p is q for p, q in zip(plan.inputs, ins))
            and len(plan.scalars) == len(scal) and all(p is q for p, q in zip(plan.scalars, scal)))


class _FullReduceLaunch:
    """A fused full reduction ready to launch again: the kernel, its grid
    and one argument array whose per-call slots (input pointers, scalar
    values, output, ddof, scratch) are rewritten under a lock before each
    launch (the launch copies the values, so the array is free right
    after)."""

    __slots__ = ("fn", "grid", "n", "args", "ptrs", "dyn", "lock", "acc_bytes", "nargs")

    def __init__(self, fn, grid, n, template):
        self.fn = ctypes.c_void_p(fn)
        self.grid = (ctypes.c_uint * 3)(int(grid), 1, 1)
        self.acc_bytes = 64 * int(grid)
        self.n = n
        objs, dyn = [], []
        for x in template:
            if x.__class__ is tuple:
                if x[0] == "in":
                    o = ctypes.c_void_p(0)
                    dyn.append((o, "in", x[1], None))
                else:
                    o = _ctype_scalar(0, x[2])
                    dyn.append((o, "sc", x[1], np.dtype(x[2])))
                objs.append(o)
            else:
                objs.append(x)
        self.dyn = dyn
        tail = [ctypes.c_longlong(n), ctypes.c_void_p(0), ctypes.c_int(0), ctypes.c_double(0.0),
                ctypes.c_void_p(0), ctypes.c_void_p(0), ctypes.c_void_p(0)]
        self.args = objs + tail
        self.nargs = len(self.args)
        self.ptrs = (ctypes.c_void_p * len(self.args))(*[ctypes.addressof(o) for o in self.args])
        self.lock = threading.Lock()

    def launch(self, ins, scal, out_ptr, code, ddof, scr=None, tick=None, part=0):
        """Launch; with scr None the library fills in its scratch region in
        the same call (mmp_launch_scratch)."""
        with self.lock:
            for o, kind, slot, dt in self.dyn:
                if kind == "in":
                    o.value = ins[slot]._ptr
                elif dt == np.float16:
                    o.value = int(np.asarray(scal[slot]._value, np.float16).view(np.uint16))
                else:
                    o.value = scal[slot]._value.item()
            a = self.args
            a[-6].value = out_ptr
            a[-5].value = code
            a[-4].value = ddof
            a[-1].value = part
            if scr is None:
                n = self.nargs
                rc = _cb.lib.mmp_launch_scratch(self.fn, self.grid, _BLOCK3, 0, self.ptrs, self.acc_bytes + 256,
                                                n - 3, n - 2)
            else:
                a[-3].value = scr
                a[-2].value = tick
                rc = _cb.lib.mmp_launch(self.fn, self.grid, _BLOCK3, 0, self.ptrs)
            if rc:
                _cb.check(rc, "fused kernel launch")


def _remember(key, value):
    if len(_tmpl) >= _TMPL_MAX:
        _tmpl.clear()
    _tmpl[key] = value


def _launch(fn, grid, args, block=_BLOCK):
    arr = (ctypes.c_void_p * len(args))(*[ctypes.addressof(x) for x in args])
    g = (ctypes.c_uint * 3)(int(grid[0]), int(grid[1]) if len(grid) > 1 else 1,
                             int(grid[2]) if len(grid) > 2 else 1)
    b = (ctypes.c_uint * 3)(int(block), 1, 1)
    _cb.check(_cb.lib.mmp_launch(ctypes.c_void_p(fn), g, b, 0, arr), "fused kernel launch")


_occ: dict = {}


def _resident_blocks(fn) -> int:
    """Blocks of _BLOCK threads that fit on the whole GPU at once."""
    r = _occ.get(fn)
    if r is None:
        per_sm = ctypes.c_int(0)
        _cb.check(_cb.lib.mmp_occupancy(ctypes.c_void_p(fn), _BLOCK, 0, ctypes.byref(per_sm)), "occupancy")
        r = max(1, per_sm.value) * _cb.CudaBackend().sm_count
        _occ[fn] = r
    return r


def _vec_width(dtypes) -> int:
    mx = max((np.dtype(d).itemsize for d in dtypes), default=4)
    return 8 if mx <= 2 else 4


def run_elementwise(node, out_ptr: int, out_shape, out_strides=None) -> None:
    """Evaluate ``node`` over ``out_shape`` into device memory ``out_ptr``
    (C-contiguous unless ``out_strides`` (elements) is given)."""
    out_shape = tuple(out_shape)
    tmp_plan = _Plan(node, out_shape, 4)
    V = _vec_width([a._dtype for a in tmp_plan.inputs] + [node._dtype])
    plan = tmp_plan if V == 4 else _Plan(node, out_shape, V)
    if plan.n == 0:
        return
    out_strided = out_strides is not None and tuple(out_strides) != _c_strides(out_shape)
    if out_strided:
        # decompose over the full (uncollapsed) output shape
        plan.strided = True
        shp = [s for s in out_shape] or [1]
        plan.cshape = list(shp)
        plan.nd = len(shp)
        plan.cstrides = [_bcast_strides(a._shape, a._strides, out_shape) or [0] for a in plan.inputs]
        plan.kinds = ["sg" if any(plan.cstrides[k]) else "bc" for k in range(len(plan.inputs))]
        plan.vec_ok = False
        plan.idx64 = True
    if not out_strided and out_ptr % (V * node._dtype.itemsize) != 0:
        plan.vec_ok = False
    key = ("ew", plan.key(), out_strided, V)
    fn = _get(key, lambda: _ew_source(plan, out_strided), "mmp_fused_ew", plan.fmad)
    args = _loader_args(plan) + [ctypes.c_void_p(out_ptr), ctypes.c_longlong(plan.n)]
    if out_strided:
        args += [ctypes.c_longlong(int(s)) for s in out_strides]
    per = _BLOCK * V * 4
    grid = max(1, min((plan.n + per - 1) // per, _resident_blocks(fn)))
    _launch(fn, (grid,), args)


def materialize(arr) -> None:
    """Evaluate ``arr``'s fusion graph into a new contiguous buffer."""
    node = arr._fusion_node
    if node is None:
        return
    buf = _cb.DeviceBuffer(max(arr.nbytes, 1))
    run_elementwise(node, buf.ptr, arr._shape)
    arr._buffer = buf
    arr._fusion_node = None
    arr._offset = 0
    arr._strides = _c_strides(arr._shape)


# ---------------------------------------------------------------------------
# fused reductions
# ---------------------------------------------------------------------------

_RED_V = {1: 8, 2: 8, 4: 4, 8: 2}
_occ_cache: dict = {}


def run_reduce(node, shape, opc: int, out_ptr: int, out_dt, ddof: float = 0.0,
               axis_split=None, want_partial: bool = False):
    """Reduce the expression ``node`` (logical C-order ``shape``).

    ``axis_split`` None reduces everything; otherwise (outer, k, inner) with
    the reduced extent k in the middle.  Returns an ``MmpPartial`` when
    ``want_partial`` (full reductions only).
    """
    T = node._dtype
    V = _RED_V[T.itemsize]
    code = MMP_CODES[out_dt if isinstance(out_dt, np.dtype) else np.dtype(out_dt)]
    if axis_split is None:
        t = tkey = None
        if node._leaves is not None:
            ins, scal, lk = _leaf_key(node, V)
            tkey = ("red", opc, node._sig, lk, shape if shape.__class__ is tuple else tuple(shape),
                    bool(_CFG.fast_math))
            t = _tmpl.get(tkey)
        if t is None:
            plan = _Plan(node, shape, V)
            n = plan.n
            key = ("red", opc, plan.key())

            def src():
                return _red_source(plan, opc, "full", 1)

            fn = _get(key, src, "mmp_fused_reduce", plan.fmad)
            per = _BLOCK * V * 4
            grid = max(1, min((n + per - 1) // per, _resident_blocks(fn)))
            t = _FullReduceLaunch(fn, grid, n, _arg_template(plan))
            if tkey is not None and _same_slots(plan, ins, scal):
                _remember(tkey, t)
            ins, scal = plan.inputs, plan.scalars
        if not want_partial:
            t.launch(ins, scal, out_ptr, code, float(ddof))
            return None
        acc_bytes = t.acc_bytes
        scr = ctypes.c_void_p()
        tick = ctypes.c_void_p()
        _cb.check(_cb.lib.mmp_scratch(acc_bytes + 256, ctypes.byref(scr), ctypes.byref(tick)))
        part_ptr = scr.value + acc_bytes
        t.launch(ins, scal, out_ptr, code, float(ddof), scr.value, tick.value, part_ptr)
        p = _cb.MmpPartial()
        _cb.check(_cb.lib.mmp_d2h(ctypes.byref(p), ctypes.c_void_p(part_ptr), ctypes.sizeof(p)))
        return p
    plan = _Plan(node, shape, V)
    be = _cb.CudaBackend()
    outer, kk, inner = (int(v) for v in axis_split)
    sms = be.sm_count
    if inner == 1:
        rows = outer
        kind = "rows_block" if (kk >= 2048 or rows < sms * 4) else "rows_warp"
        key = ("red", opc, kind, plan.key())
        fn = _get(key, lambda: _red_source(plan, opc, kind, 1), "mmp_fused_reduce", plan.fmad)
        grid = min(rows, sms * 8) if kind == "rows_block" else min((rows + 7) // 8, sms * 8)
        args = _loader_args(plan) + [ctypes.c_longlong(rows), ctypes.c_longlong(kk), ctypes.c_void_p(out_ptr),
                                     ctypes.c_int(code), ctypes.c_double(ddof)]
        _launch(fn, (max(grid, 1),), args)
        return None
    cv = min(V, 4)
    if not (plan.vec_ok and inner % cv == 0):
        cv = 1
    ctiles = (inner + 32 * cv - 1) // (32 * cv)
    gx = outer * ctiles
    target = sms * 6
    S = 1
    if gx <= 4096 and gx < target:
        S = max(1, min(-(-target // gx), -(-kk // 64), 65535))
    kchunk = max(1, -(-kk // S))
    S = max(1, -(-kk // kchunk))
    scr = ctypes.c_void_p()
    tick = ctypes.c_void_p()
    _cb.check(_cb.lib.mmp_scratch(S * outer * inner * 32 + 256, ctypes.byref(scr), ctypes.byref(tick)))
    key = ("red", opc, "cols", cv, plan.key())
    fn = _get(key, lambda: _red_source(plan, opc, "cols", cv), "mmp_fused_reduce", plan.fmad)
    args = _loader_args(plan) + [ctypes.c_longlong(outer), ctypes.c_longlong(kk), ctypes.c_longlong(inner),
                                 ctypes.c_longlong(kchunk), ctypes.c_void_p(out_ptr), ctypes.c_int(code),
                                 ctypes.c_double(ddof), ctypes.c_void_p(scr.value), ctypes.c_void_p(tick.value)]
    _launch(fn, (gx, S), args)
    return None
