"""``maximum`` / ``minimum`` ufunc objects (mirrors ``src/macmetalpy/ufunc.py:10-49``).

``__call__`` is the fused device op; ``reduce`` is the device max/min
reduction; ``accumulate`` (CPU in the reference) is not on the device path
and runs on a host copy.
"""

from __future__ import annotations

import numpy as np

from .ndarray import ndarray

__all__ = ["ufunc", "maximum", "minimum"]


class ufunc:
    def __init__(self, name, op_name, np_ufunc, red):
        self.__name__ = name
        self._op = op_name
        self._np = np_ufunc
        self._red = red
        self.nin, self.nout = 2, 1

    def __call__(self, x1, x2, out=None, **kwargs):
        r = ndarray._elementwise(self._op, x1, x2)
        if out is not None:
            out[...] = r
            return out
        return r

    def reduce(self, a, axis=0, dtype=None, out=None, keepdims=False):
        from . import reductions
        return getattr(reductions, self._red)(a, axis=axis, out=out, keepdims=keepdims)

    def accumulate(self, a, axis=0, dtype=None, out=None):
        from .creation import asarray
        return asarray(self._np.accumulate(asarray(a).get(), axis=axis, dtype=dtype))

    def __repr__(self):
        return f"<ufunc '{self.__name__}'>"


maximum = ufunc("maximum", "max_op", np.maximum, "max")
minimum = ufunc("minimum", "min_op", np.minimum, "min")
