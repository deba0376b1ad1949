"""dtype resolution (mirrors ``src/macmetalpy/_dtypes.py:77-146``) and the
numpy <-> CUDA C <-> libmmp_cuda dtype-code tables.

``resolve_dtype`` keeps the reference's rules: ``None`` -> the configured
default float; float64 -> float32 under ``float64_behavior="downcast"``
(with the optional warning), kept under ``"cpu_fallback"`` (computed on the
GPU here); complex128 -> complex64; int8/uint8 -> int16/uint16.
"""

from __future__ import annotations

import warnings

import numpy as np

from ._config import get_config

__all__ = [
    "resolve_dtype",
    "result_dtype",
    "is_float_dtype",
    "SUPPORTED_DTYPES",
    "CUDA_TYPE_NAMES",
    "MMP_CODES",
]

# dtype codes of include/mmp_cuda.h (enum mmp_dtype)
MMP_CODES: dict = {
    np.dtype(np.bool_): 0,
    np.dtype(np.int8): 1,
    np.dtype(np.uint8): 2,
    np.dtype(np.int16): 3,
    np.dtype(np.uint16): 4,
    np.dtype(np.int32): 5,
    np.dtype(np.uint32): 6,
    np.dtype(np.int64): 7,
    np.dtype(np.uint64): 8,
    np.dtype(np.float16): 9,
    np.dtype(np.float32): 10,
    np.dtype(np.float64): 11,
}

# C type used for each dtype inside generated CUDA code
CUDA_TYPE_NAMES: dict = {
    np.dtype(np.bool_): "bool",
    np.dtype(np.int8): "int8_t",
    np.dtype(np.uint8): "uint8_t",
    np.dtype(np.int16): "int16_t",
    np.dtype(np.uint16): "uint16_t",
    np.dtype(np.int32): "int32_t",
    np.dtype(np.uint32): "uint32_t",
    np.dtype(np.int64): "int64_t",
    np.dtype(np.uint64): "uint64_t",
    np.dtype(np.float16): "__half",
    np.dtype(np.float32): "float",
    np.dtype(np.float64): "double",
}

SUPPORTED_DTYPES = frozenset(
    np.dtype(d)
    for d in (np.bool_, np.int16, np.uint16, np.int32, np.uint32, np.int64, np.uint64,
              np.float16, np.float32, np.float64)
)

_PASSTHROUGH = frozenset(SUPPORTED_DTYPES - {np.dtype(np.float64)})
_F64 = np.dtype(np.float64)


def is_float_dtype(dtype) -> bool:
    """True if ``dtype`` is a floating-point type."""
    return np.issubdtype(np.dtype(dtype), np.floating)


def resolve_dtype(dtype) -> np.dtype:
    """Resolve a user-supplied dtype to one the device path computes in."""
    if dtype is None:
        return np.dtype(get_config().default_float_dtype)
    dtype = np.dtype(dtype)
    if dtype in _PASSTHROUGH:
        return dtype
    if dtype == _F64:
        cfg = get_config()
        if cfg.float64_behavior == "downcast":
            if cfg.warn_on_downcast:
                warnings.warn("float64 is downcast to float32 (float64_behavior='downcast').",
                              UserWarning, stacklevel=3)
            return np.dtype(cfg.default_float_dtype)
        return dtype
    if dtype == np.int8:
        return np.dtype(np.int16)
    if dtype == np.uint8:
        return np.dtype(np.uint16)
    if dtype == np.complex128 or dtype == np.complex64:
        raise TypeError(f"complex dtypes are not supported on the device path: {dtype}")
    if dtype == np.float128 if hasattr(np, "float128") else False:
        return resolve_dtype(_F64)
    raise TypeError(f"Unsupported dtype: {dtype}")


def result_dtype(dt1, dt2) -> np.dtype:
    """numpy promotion of two dtypes, then :func:`resolve_dtype`."""
    return resolve_dtype(np.result_type(dt1, dt2))
