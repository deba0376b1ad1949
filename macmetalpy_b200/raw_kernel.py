"""User CUDA kernels (mirrors ``src/macmetalpy/raw_kernel.py:15-62``).

``RawKernel(source, func_name)`` keeps the reference's interface, but the
source is CUDA C (compiled once for sm_100a with NVRTC; ``extern "C"`` or
C++ names both work).  ``kernel(grid, args)``: ``grid`` is a THREAD count
(int or 1-3 tuple, ``ValueError`` otherwise) as in the reference; blocks of
``block`` threads (default 256 / 16x16 / 8x8x4) are launched to cover it,
so the kernel must bounds-check its global index.  ``args`` may hold
ndarrays (passed as device pointers), numpy scalars (their own type) and
Python scalars (``int`` -> 64-bit, which an ``int`` parameter reads
correctly for values that fit; ``float`` -> float32; ``bool`` -> bool).
"""

from __future__ import annotations

import ctypes
from typing import Sequence, Union

import numpy as np

from . import _cuda_backend as _cb
from . import _fusion as _fu
from .ndarray import ndarray

__all__ = ["RawKernel"]

_DEFAULT_BLOCK = {1: (256, 1, 1), 2: (16, 16, 1), 3: (8, 8, 4)}


class RawKernel:
    def __init__(self, source: str, func_name: str, options: tuple = (), **kwargs) -> None:
        self._source = source
        self._func_name = func_name
        self._options = tuple(options)
        self._fn = None

    @property
    def kernel(self) -> int:
        if self._fn is None:
            self._fn = _fu.compile_kernel(self._source, self._func_name)
        return self._fn

    @staticmethod
    def _arg(a):
        if isinstance(a, ndarray):
            return ctypes.c_void_p(a._ptr)
        if isinstance(a, np.generic):
            return _fu._ctype_scalar(a, a.dtype)
        if isinstance(a, bool):
            return ctypes.c_bool(a)
        if isinstance(a, int):
            return ctypes.c_int64(a)
        if isinstance(a, float):
            return ctypes.c_float(a)
        raise TypeError(f"unsupported kernel argument type {type(a).__name__}")

    def __call__(self, grid: Union[int, tuple], args: Sequence, block=None, shared_mem: int = 0) -> None:
        if isinstance(grid, (int, np.integer)):
            grid = (int(grid),)
        grid = tuple(int(g) for g in grid)
        if not 1 <= len(grid) <= 3:
            raise ValueError("grid tuple must have 1-3 elements")
        blk = tuple(block) if block is not None else _DEFAULT_BLOCK[len(grid)]
        blk = blk + (1,) * (3 - len(blk))
        g = [(grid[i] + blk[i] - 1) // blk[i] if i < len(grid) else 1 for i in range(3)]
        cargs = [self._arg(a) for a in args]
        ptrs = (ctypes.c_void_p * max(len(cargs), 1))(
            *[ctypes.addressof(x) for x in cargs])
        gg = (ctypes.c_uint * 3)(*g)
        bb = (ctypes.c_uint * 3)(*blk)
        _cb.check(_cb.lib.mmp_launch(ctypes.c_void_p(self.kernel), gg, bb, int(shared_mem), ptrs), "RawKernel")
