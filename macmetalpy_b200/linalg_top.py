"""``matmul`` (mirrors ``src/macmetalpy/linalg_top.py:94-111`` and
``ndarray.__matmul__``, ``ndarray.py:1398-1450``).

All sizes and ranks run on the GPU through ``mmp_gemm``: float32 on tcgen05
tensor cores with the 3xTF32 split (float32-level accuracy), float16 on
tensor cores with float32 accumulation, other dtypes on CUDA cores.  The
reference runs ``matmul`` on the CPU below 4,194,304 elements and for every
batched (3-D) input, and its ``@`` raises ``ValueError`` for 3-D operands
(``ndarray.py:1422``); here ``@`` and ``matmul`` follow numpy's batched
semantics (a deliberate divergence from that one reference test,
``tests/test_error_handling.py:116-121``).
"""

from __future__ import annotations

import ctypes
import math

import numpy as np

from . import _cuda_backend as _cb
from ._broadcasting import broadcast_shapes
from ._dtypes import MMP_CODES, resolve_dtype
from .ndarray import ndarray

__all__ = ["matmul", "GEMM_MODES"]

GEMM_MODES = {"auto": 0, "3xtf32": 1, "tf32": 2, "f16": 3, "simt": 4}


def _rowmajor(a: ndarray) -> ndarray:
    """a with C-contiguous trailing two dims and contiguous batch."""
    return a._ensure_contiguous()


def matmul(x1, x2, out=None, *, mode: str = "auto", **kwargs):
    """Matrix product with numpy semantics (1-D promotion, batch broadcast).
    A row-block distributed ``x1`` multiplies its block by the replicated
    ``x2`` (``distributed.DistArray.matmul``)."""
    from .creation import asarray

    if x1.__class__.__name__ == "DistArray":
        return x1.matmul(asarray(x2))

    a = asarray(x1)
    b = asarray(x2)
    if a.ndim == 0 or b.ndim == 0:
        raise ValueError("matmul: Input operand does not have enough dimensions")
    dt = resolve_dtype(np.matmul.resolve_dtypes((a.dtype, b.dtype, None))[-1])
    if a.dtype != dt:
        a = a.astype(dt)
    if b.dtype != dt:
        b = b.astype(dt)
    a1 = a.ndim == 1
    b1 = b.ndim == 1
    if a1:
        a = a.reshape(1, -1)
    if b1:
        b = b.reshape(-1, 1)
    M, K = a.shape[-2:]
    K2, N = b.shape[-2:]
    if K != K2:
        # the reference's message (ndarray.py:1426-1429), which its tests match
        raise ValueError(f"matmul shape mismatch: ({M},{K}) @ ({K2},{N})")
    batch_shape = broadcast_shapes(a.shape[:-2], b.shape[:-2])
    B = math.prod(batch_shape) if batch_shape else 1
    a = _rowmajor(a)
    b = _rowmajor(b)

    def bstride(x, rows, cols):
        xb = x.shape[:-2]
        if (math.prod(xb) if xb else 1) == B:
            if tuple(xb) != tuple(batch_shape):
                return None
            return rows * cols
        if (math.prod(xb) if xb else 1) == 1:
            return 0
        return None

    sa = bstride(a, M, K)
    sb = bstride(b, K, N)
    if sa is None:
        a = a.broadcast_to(batch_shape + (M, K)).copy()
        sa = M * K
    if sb is None:
        b = b.broadcast_to(batch_shape + (K, N)).copy()
        sb = K * N
    res = ndarray._empty(batch_shape + (M, N), dt)
    if res.size:
        _cb.check(_cb.lib.mmp_gemm(MMP_CODES[dt], GEMM_MODES[mode], B, M, N, K, ctypes.c_void_p(a._ptr), K, sa,
                                   ctypes.c_void_p(b._ptr), N, sb, ctypes.c_void_p(res._buffer.ptr), N, M * N),
                  "matmul")
    if a1 and b1:
        res = res.reshape(batch_shape)
    elif a1:
        res = res.reshape(batch_shape + (N,))
    elif b1:
        res = res.reshape(batch_shape + (M,))
    if out is not None:
        out[...] = res
        return out
    return res
