"""Streams, events and pinned host memory (the ``cupy.cuda`` names a
CuPy-style program uses to overlap copies with compute).

The reference has one implicit queue (``MetalBackend``,
``_metal_backend.py:341-372``) and no counterpart.  Here kernels always run
on the library stream of the current device; a :class:`Stream` carries
asynchronous copies (``ndarray.set(arr, stream=s)``,
``ndarray.get(stream=s, out=pinned)``), which the two copy engines run
concurrently with kernels and with each other:

* ``get(stream=s)`` makes ``s`` wait for the kernels enqueued so far, then
  copies; the host must ``s.synchronize()`` before reading ``out``;
* ``set(arr, stream=s)`` copies on ``s`` and makes the library stream wait
  for that copy, so later kernels see the data; ``arr`` must stay unchanged
  until ``s`` has finished it;
* pinned host arrays (:func:`empty_pinned`) are needed for copies that do
  not block the host.

Device arrays used by a side stream must stay alive until its work is done.
"""

from __future__ import annotations

import ctypes
import weakref

import numpy as np

from . import _cuda_backend as _cb

__all__ = ["Stream", "Event", "empty_pinned", "get_current_stream"]


class Event:
    def __init__(self):
        _cb.CudaBackend()
        p = ctypes.c_void_p()
        _cb.check(_cb.lib.mmp_event_create(ctypes.byref(p)), "event")
        self.ptr = p.value
        weakref.finalize(self, _cb.lib.mmp_event_destroy, ctypes.c_void_p(self.ptr))

    def record(self, stream=None) -> "Event":
        _cb.check(_cb.lib.mmp_event_record_on(ctypes.c_void_p(self.ptr), _sp(stream)), "event record")
        return self

    def synchronize(self) -> None:
        ms = ctypes.c_float()
        # elapsed_ms waits for its end event (here the event itself)
        _cb.check(_cb.lib.mmp_event_elapsed_ms(ctypes.c_void_p(self.ptr), ctypes.c_void_p(self.ptr),
                                               ctypes.byref(ms)), "event synchronize")

    def elapsed_time(self, end: "Event") -> float:
        ms = ctypes.c_float()
        _cb.check(_cb.lib.mmp_event_elapsed_ms(ctypes.c_void_p(self.ptr), ctypes.c_void_p(end.ptr),
                                               ctypes.byref(ms)), "event elapsed")
        return float(ms.value)


class Stream:
    """A non-blocking stream for asynchronous copies.  ``Stream.null`` is the
    library stream that kernels run on."""

    null: "Stream"

    def __init__(self, non_blocking=True, _ptr=None, _own=True):
        if _ptr is not None or not _own:
            self.ptr = _ptr
            return
        _cb.CudaBackend()
        p = ctypes.c_void_p()
        _cb.check(_cb.lib.mmp_stream_create(ctypes.byref(p)), "stream")
        self.ptr = p.value
        weakref.finalize(self, _cb.lib.mmp_stream_destroy, ctypes.c_void_p(self.ptr))

    def synchronize(self) -> None:
        _cb.check(_cb.lib.mmp_stream_synchronize(_sp(self)), "stream synchronize")

    def wait_event(self, event: Event) -> None:
        _cb.check(_cb.lib.mmp_stream_wait_event(_sp(self), ctypes.c_void_p(event.ptr)), "stream wait")

    def record(self, event: Event | None = None) -> Event:
        return (event or Event()).record(self)


Stream.null = Stream(_ptr=None, _own=False)


def _sp(stream):
    """ctypes pointer of a stream (None: the library stream)."""
    if stream is None or stream.ptr is None:
        return None
    return ctypes.c_void_p(stream.ptr)


def get_current_stream() -> Stream:
    return Stream.null


def empty_pinned(shape, dtype=np.float32) -> np.ndarray:
    """numpy array in pinned (page-locked) host memory, freed when the array
    (and every view of it) is gone."""
    _cb.CudaBackend()
    dt = np.dtype(dtype)
    shape = (shape,) if isinstance(shape, (int, np.integer)) else tuple(shape)
    n = int(np.prod(shape)) * dt.itemsize
    p = ctypes.c_void_p()
    _cb.check(_cb.lib.mmp_host_alloc(n, ctypes.byref(p)), "pinned alloc")
    raw = np.ctypeslib.as_array((ctypes.c_char * max(n, 1)).from_address(p.value))
    # every view of the result keeps `raw` (the array wrapping the memory)
    # alive as its base, so the memory is freed with the last view
    weakref.finalize(raw, _cb.lib.mmp_host_free, ctypes.c_void_p(p.value))
    return raw[:n].view(dt).reshape(shape)
