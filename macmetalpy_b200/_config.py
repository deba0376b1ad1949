"""Global configuration (mirrors ``src/macmetalpy/_config.py:11-64``).

Keys and defaults are the reference's.  ``float64_behavior`` keeps its two
values; on B200 float64 is computed natively on the GPU, so
``"cpu_fallback"`` (the default) means "keep float64" and ``"downcast"``
means "compute in float32", which is how the reference resolves dtypes
(``_dtypes.resolve_dtype``).  ``fast_math`` compiles fused kernels with
``--use_fast_math``.  ``shard_threshold`` (not a reference key) is the size
above which host data uploaded on a multi-rank job is block-distributed.
"""

from __future__ import annotations

from typing import Literal

__all__ = ["MacMetalConfig", "get_config", "set_config"]

_CONFIG = None  # the one instance, made below at import


class MacMetalConfig:
    """The process's configuration.  Its one instance is made when this
    module is imported (under Python's import lock, so no lock of its own);
    calling the class returns that instance, as the reference's singleton
    does."""

    __slots__ = ("float64_behavior", "warn_on_downcast", "default_float_dtype", "fast_math", "shard_threshold")

    def __new__(cls) -> "MacMetalConfig":
        if _CONFIG is not None:
            return _CONFIG
        inst = super().__new__(cls)
        inst.float64_behavior = "cpu_fallback"
        inst.warn_on_downcast = True
        inst.default_float_dtype = "float32"
        inst.fast_math = False
        inst.shard_threshold = None
        return inst


_CONFIG = MacMetalConfig()


def get_config() -> MacMetalConfig:
    """Return the global configuration."""
    return _CONFIG


def set_config(
    *,
    float64_behavior: Literal["downcast", "cpu_fallback"] | None = None,
    warn_on_downcast: bool | None = None,
    default_float_dtype: str | None = None,
    fast_math: bool | None = None,
    shard_threshold: int | None = None,
) -> None:
    """Update global configuration values (the reference's keys, plus
    ``shard_threshold``: with ``distributed.init()`` done on more than one
    rank, ``array()`` / ``asarray()`` of host data with at least this many
    elements return this rank's row block as a ``distributed.DistArray``;
    0 turns it off again)."""
    cfg = get_config()
    if float64_behavior is not None:
        if float64_behavior not in ("downcast", "cpu_fallback"):
            raise ValueError(
                f"float64_behavior must be 'downcast' or 'cpu_fallback', got {float64_behavior!r}"
            )
        cfg.float64_behavior = float64_behavior
    if warn_on_downcast is not None:
        cfg.warn_on_downcast = warn_on_downcast
    if default_float_dtype is not None:
        cfg.default_float_dtype = default_float_dtype
    if fast_math is not None:
        cfg.fast_math = fast_math
    if shard_threshold is not None:
        if int(shard_threshold) < 0:
            raise ValueError(f"shard_threshold must be >= 0, got {shard_threshold!r}")
        cfg.shard_threshold = int(shard_threshold) or None
