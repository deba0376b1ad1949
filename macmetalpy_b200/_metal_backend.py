"""The reference's backend name, for code that reaches it directly.

The reference's tests and some callers use ``MetalBackend()`` itself
(``src/macmetalpy/_metal_backend.py:179-372``; e.g.
``tests/test_synchronize.py:11``) for ``synchronize()`` and the
``_has_pending`` flag.  Here the one device backend is ``CudaBackend``;
``MetalBackend`` is that singleton under the reference's name, with the same
``synchronize()`` and a ``_has_pending`` that is False once the stream has
drained (the reference clears it in ``synchronize``,
``_metal_backend.py:359-372``).  Buffer creation and kernel dispatch of the
Metal class (``create_buffer``, ``execute_kernel``) have no counterpart:
they are the ``mmp_malloc`` / ``mmp_launch`` entry points of the C ABI.
"""

from __future__ import annotations

import ctypes

from . import _cuda_backend as _cb

__all__ = ["MetalBackend"]


class MetalBackend:
    """Singleton view of the device backend under the reference's name."""

    _instance = None

    def __new__(cls):
        if cls._instance is None:
            inst = super().__new__(cls)
            inst._be = _cb.CudaBackend()
            cls._instance = inst
        return cls._instance

    def synchronize(self) -> None:
        self._be.synchronize()

    @property
    def _has_pending(self) -> bool:
        """True while work enqueued on the device stream has not finished."""
        busy = ctypes.c_int(0)
        _cb.check(_cb.lib.mmp_stream_query(None, ctypes.byref(busy)), "stream query")
        return bool(busy.value)
