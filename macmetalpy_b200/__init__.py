"""macmetalpy_b200 -- B200 (sm_100a) backend for MacMetalPy's array hot path.

``import macmetalpy_b200 as cp`` gives the reference's ``import macmetalpy as
cp`` surface for the ndarray / ufunc / reduction / cumsum / matmul path and
the lazy fusion engine, backed by ``libmmp_cuda.so`` (C ABI in
``include/mmp_cuda.h``).  The reference's platform guard
(``src/macmetalpy/__init__.py:5-6``) is dropped; there is no CPU fallback.
"""

from __future__ import annotations

import numpy as _np

from . import _cuda_backend, cuda
from ._config import get_config, set_config
from ._cuda_backend import CudaBackend
from .bitwise_ops import *  # noqa: F401,F403
from .creation import *  # noqa: F401,F403
from .indexing import *  # noqa: F401,F403
from .linalg_top import matmul
from .logic_ops import *  # noqa: F401,F403
from .math_ops import *  # noqa: F401,F403
from .nan_ops import *  # noqa: F401,F403
from .order_stats import *  # noqa: F401,F403
from .ndarray import ndarray
from .raw_kernel import RawKernel
from .reductions import *  # noqa: F401,F403
from .sorting import *  # noqa: F401,F403
from .ufunc_ops import *  # noqa: F401,F403
from .ufunc import maximum, minimum  # ufunc objects (ufunc.py:10-49)

__version__ = "0.1.0"

bool_ = _np.bool_
int8, int16, int32, int64 = _np.int8, _np.int16, _np.int32, _np.int64
uint8, uint16, uint32, uint64 = _np.uint8, _np.uint16, _np.uint32, _np.uint64
float16, float32, float64 = _np.float16, _np.float32, _np.float64
dtype = _np.dtype
newaxis = None
pi, e, inf, nan = _np.pi, _np.e, _np.inf, _np.nan


def synchronize() -> None:
    """Wait for all queued device work (``__init__.py:233-236``); raises if a
    kernel reported a device-side error."""
    CudaBackend().synchronize()


def get_array_module(*args):
    import sys
    return sys.modules[__name__]
