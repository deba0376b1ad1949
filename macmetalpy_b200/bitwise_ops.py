"""Bitwise operations (mirrors ``src/macmetalpy/bitwise_ops.py:35-95``).

The reference casts both operands to int32 and returns int32 on both of
its paths (CPU: ``a_np.astype(np.int32)`` then the numpy function,
``bitwise_ops.py:37-45``; GPU: ``astype(np.int32)`` and an int32 shader,
``:46-56``), so ``bitwise_and(int64, int64)`` keeps the low 32 bits and
``invert(bool)`` is ``~int32(b)``.  The same casts and int32 results are
used here, each op one fused node.  Shifts follow numpy's int32 loop: a
count outside [0, 32) gives 0 (left) or the sign fill (right).

``ndarray`` operators dispatch as the reference does
(``ndarray.py:1670-1700, 2549-2590``): ``&``, ``|``, ``^``, ``~`` on integer
arrays are these int32 bitwise ops; on bool and float arrays ``&``, ``|``,
``^`` are logical ops with a bool result and ``~`` of bool is logical not;
``<<`` and ``>>`` are always the int32 shifts.
"""

from __future__ import annotations

import numpy as np

from .ndarray import ndarray

__all__ = ["bitwise_and", "bitwise_or", "bitwise_xor", "invert", "bitwise_not", "bitwise_invert",
           "left_shift", "right_shift"]


def _i32(x):
    from . import creation

    a = x if isinstance(x, ndarray) else creation.asarray(np.asarray(x))
    return a if a.dtype == np.int32 else a.astype(np.int32)


def _bin(op):
    def f(x1, x2, **kwargs):
        return ndarray._elementwise(op, _i32(x1), _i32(x2))
    f.__name__ = op[:-3]
    f.__doc__ = f"Elementwise {op[:-3]} on int32 casts of both operands (the reference's rule)."
    return f


bitwise_and = _bin("bitwise_and_op")
bitwise_or = _bin("bitwise_or_op")
bitwise_xor = _bin("bitwise_xor_op")
left_shift = _bin("left_shift_op")
right_shift = _bin("right_shift_op")


def invert(x, **kwargs):
    """``~int32(x)``."""
    return ndarray._elementwise("invert_op", _i32(x))


bitwise_not = invert
bitwise_invert = invert
