"""ctypes binding of ``libmmp_cuda.so`` (the C ABI in ``include/mmp_cuda.h``).

Replaces the reference's ``MetalBackend`` singleton
(``src/macmetalpy/_metal_backend.py:179-372``): ``create_buffer`` /
``array_to_buffer`` become stream-ordered ``cudaMallocAsync`` + H2D copies,
``execute_kernel`` becomes NVRTC compile-once + launch on the device's
stream, ``synchronize`` a stream synchronisation.  Every failing call raises
``RuntimeError`` with the library's message (the reference surfaces no
device errors at all: ``runFunction`` returns ``void``,
``_metal_backend.py:250-257``).  There is no CPU fallback: if the library
or a GPU is missing, use raises.
"""

from __future__ import annotations

import ctypes
import os
import threading

import numpy as np

from ._dtypes import MMP_CODES

__all__ = ["lib", "CudaBackend", "DeviceBuffer", "check", "MmpPartial", "LIB_PATH"]

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("MMP_CUDA_LIB", os.path.join(_HERE, "_lib", "libmmp_cuda.so"))


class MmpPartial(ctypes.Structure):
    """Mirror of ``mmp_partial`` (include/mmp_cuda.h)."""

    _fields_ = [
        ("s1", ctypes.c_double),
        ("s2", ctypes.c_double),
        ("shift", ctypes.c_double),
        ("count", ctypes.c_int64),
        ("ival", ctypes.c_int64),
        ("index", ctypes.c_int64),
    ]


_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_int = ctypes.c_int
_sz = ctypes.c_size_t

# name -> (restype, argtypes); exactly the functions include/mmp_cuda.h declares
SIGNATURES = {
    "mmp_abi_version": (_int, []),
    "mmp_last_error": (ctypes.c_char_p, []),
    "mmp_device_count": (_int, [ctypes.POINTER(_int)]),
    "mmp_init": (_int, [_int]),
    "mmp_get_device": (_int, [ctypes.POINTER(_int)]),
    "mmp_sm_count": (_int, [ctypes.POINTER(_int)]),
    "mmp_get_stream": (_int, [ctypes.POINTER(_vp)]),
    "mmp_set_stream": (_int, [_vp]),
    "mmp_malloc": (_int, [_sz, ctypes.POINTER(_vp)]),
    "mmp_free": (_int, [_vp]),
    "mmp_memset": (_int, [_vp, _int, _sz]),
    "mmp_h2d": (_int, [_vp, _vp, _sz]),
    "mmp_d2h": (_int, [_vp, _vp, _sz]),
    "mmp_d2d": (_int, [_vp, _vp, _sz]),
    "mmp_host_alloc": (_int, [_sz, ctypes.POINTER(_vp)]),
    "mmp_host_free": (_int, [_vp]),
    "mmp_scratch": (_int, [_sz, ctypes.POINTER(_vp), ctypes.POINTER(_vp)]),
    "mmp_synchronize": (_int, []),
    "mmp_check_device_error": (_int, [ctypes.POINTER(_int)]),
    "mmp_event_create": (_int, [ctypes.POINTER(_vp)]),
    "mmp_event_destroy": (_int, [_vp]),
    "mmp_event_record": (_int, [_vp]),
    "mmp_event_elapsed_ms": (_int, [_vp, _vp, ctypes.POINTER(ctypes.c_float)]),
    "mmp_compile": (_int, [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_char_p, ctypes.POINTER(_vp),
                           ctypes.c_char_p, _sz]),
    "mmp_launch": (_int, [_vp, ctypes.POINTER(ctypes.c_uint), ctypes.POINTER(ctypes.c_uint),
                          ctypes.c_uint, ctypes.POINTER(_vp)]),
    "mmp_launch_scratch": (_int, [_vp, ctypes.POINTER(ctypes.c_uint), ctypes.POINTER(ctypes.c_uint), ctypes.c_uint,
                                   ctypes.POINTER(_vp), ctypes.c_size_t, _int, _int]),
    "mmp_occupancy": (_int, [_vp, _int, ctypes.c_uint, ctypes.POINTER(_int)]),
    "mmp_reduce": (_int, [_int, _int, _vp, _i64, _int, _vp, ctypes.c_double,
                          ctypes.POINTER(MmpPartial)]),
    "mmp_reduce_axis": (_int, [_int, _int, _vp, _i64, _i64, _i64, _int, _vp, ctypes.c_double]),
    "mmp_scan": (_int, [_int, _int, _vp, _int, _vp, _i64, _i64, _i64, _vp]),
    "mmp_scan_noalloc": (_int, [_int, _int, _vp, _int, _vp, _i64, _i64, _i64, _vp]),
    "mmp_gemm": (_int, [_int, _int, _i64, _i64, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _i64, _vp,
                        _i64, _i64]),
    "mmp_sort": (_int, [_int, _vp, _vp, _vp, _i64, _i64]),
    "mmp_searchsorted": (_int, [_int, _vp, _i64, _vp, _i64, _int, _vp, _vp]),
    "mmp_stream_create": (_int, [ctypes.POINTER(_vp)]),
    "mmp_stream_destroy": (_int, [_vp]),
    "mmp_stream_synchronize": (_int, [_vp]),
    "mmp_stream_query": (_int, [_vp, ctypes.POINTER(_int)]),
    "mmp_stream_wait_event": (_int, [_vp, _vp]),
    "mmp_event_record_on": (_int, [_vp, _vp]),
    "mmp_h2d_async": (_int, [_vp, _vp, _sz, _vp]),
    "mmp_d2h_async": (_int, [_vp, _vp, _sz, _vp]),
    "mmp_selftest_bounded_wait": (_int, [_int, ctypes.POINTER(ctypes.c_uint)]),
    "mmp_gather": (_int, [_int, _vp, _i64, _vp, _i64, _vp]),
    "mmp_scatter": (_int, [_int, _vp, _i64, _vp, _i64, _vp]),
    "mmp_compact_indices": (_int, [_vp, _vp, _i64, _i64, _vp]),
    "mmp_reduce_partial": (_int, [_int, _int, _vp, _i64, _i64, _vp]),
    "mmp_merge_partials": (_int, [_int, _int, _vp, _int, _int, _vp, ctypes.c_double, _vp]),
    "mmp_nccl_version": (_int, [ctypes.POINTER(_int)]),
    "mmp_comm_unique_id": (_int, [_vp]),
    "mmp_comm_init": (_int, [_int, _int, _vp, ctypes.c_double]),
    "mmp_comm_rank": (_int, [ctypes.POINTER(_int), ctypes.POINTER(_int)]),
    "mmp_comm_destroy": (_int, []),
    "mmp_comm_abort": (_int, []),
    "mmp_allreduce": (_int, [_vp, _vp, _sz, _int, _int]),
    "mmp_allgather": (_int, [_vp, _vp, _sz, _int]),
    "mmp_broadcast": (_int, [_vp, _vp, _sz, _int, _int]),
    "mmp_group_start": (_int, []),
    "mmp_group_end": (_int, []),
    "mmp_comm_synchronize": (_int, [ctypes.c_double]),
    "mmp_comm_peer_init": (_int, []),
    "mmp_reduce_allranks": (_int, [_int, _int, _vp, _i64, _i64, _int, _vp, ctypes.c_double]),
    "mmp_scan_allranks": (_int, [_int, _int, _vp, _int, _vp, _i64]),
    "mmp_allreduce_sum_peer": (_int, [_vp, _vp, ctypes.c_size_t, _int, _int]),
}


def _load():
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(
            f"libmmp_cuda.so not found at {LIB_PATH}; build it with "
            "`python macmetalpy_b200/csrc/build.py` or `__graft_entry__.build()` (there is no CPU fallback)"
        )
    L = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    return L


lib = _load()


def check(rc: int, what: str = "") -> None:
    """Raise ``RuntimeError`` if a library call failed."""
    if rc != 0:
        msg = lib.mmp_last_error().decode(errors="replace")
        raise RuntimeError(f"{what}: {msg}" if what else msg)


def dtype_code(dtype) -> int:
    return MMP_CODES[np.dtype(dtype)]


class CudaBackend:
    """Per-process device state (one stream per device, stream-ordered pool).

    Singleton like the reference's ``MetalBackend`` (``_metal_backend.py:179-195``).
    """

    _instance = None
    _lock = threading.Lock()

    def __new__(cls):
        with cls._lock:
            if cls._instance is None:
                inst = super().__new__(cls)
                inst._setup()
                cls._instance = inst
            return cls._instance

    def _setup(self) -> None:
        n = ctypes.c_int(0)
        rc = lib.mmp_device_count(ctypes.byref(n))
        if rc != 0 or n.value < 1:
            msg = lib.mmp_last_error().decode(errors="replace")
            raise RuntimeError(f"no CUDA device available for macmetalpy_b200 ({msg})")
        self.device_count = n.value
        dev = int(os.environ.get("LOCAL_RANK", os.environ.get("MMP_DEVICE", "0"))) % n.value
        check(lib.mmp_init(dev), "mmp_init")
        self.device = dev
        sms = ctypes.c_int(0)
        check(lib.mmp_sm_count(ctypes.byref(sms)))
        self.sm_count = sms.value

    # -- memory
    def malloc(self, nbytes: int) -> int:
        p = ctypes.c_void_p()
        check(lib.mmp_malloc(max(int(nbytes), 1), ctypes.byref(p)), "mmp_malloc")
        return p.value

    def synchronize(self) -> None:
        code = ctypes.c_int(0)
        check(lib.mmp_check_device_error(ctypes.byref(code)), "synchronize")
        if code.value:
            raise RuntimeError(f"a kernel reported device error code {code.value} "
                               "(a bounded wait ran out)")

    def stream_ptr(self) -> int:
        p = ctypes.c_void_p()
        check(lib.mmp_get_stream(ctypes.byref(p)))
        return p.value or 0


# Blocks of at most _SMALL bytes (0-d reduction results, scalars, partials)
# are recycled through a free list instead of a stream-ordered
# cudaMallocAsync / cudaFreeAsync pair per call (two driver calls that cost
# more than the small kernel that fills the block).  Reuse is ordered like
# the pool's own: a block goes back on the list when its last Python owner
# is gone, and whatever the library enqueues next on the same stream runs
# after every earlier use of it.  The process drives one device (the
# backend singleton's), so one list serves.
_SMALL = 256
_SMALL_KEEP = 4096
_small_free: list = []


class DeviceBuffer:
    """Owns one device allocation; freed (stream-ordered) when collected."""

    __slots__ = ("ptr", "nbytes", "__weakref__")

    def __init__(self, nbytes: int):
        if CudaBackend._instance is None:
            CudaBackend()
        self.nbytes = n = int(nbytes)
        if n <= _SMALL:
            try:
                self.ptr = _small_free.pop()
                return
            except IndexError:
                n = _SMALL
        p = ctypes.c_void_p()
        check(lib.mmp_malloc(n if n > 0 else 1, ctypes.byref(p)), "mmp_malloc")
        self.ptr = p.value

    def __del__(self):
        p = getattr(self, "ptr", None)
        if p:
            self.ptr = None
            if self.nbytes <= _SMALL and len(_small_free) < _SMALL_KEEP:
                _small_free.append(p)
                return
            try:
                lib.mmp_free(ctypes.c_void_p(p))
            except Exception:
                pass


class Event:
    """CUDA event on the library stream (for timing)."""

    def __init__(self):
        p = ctypes.c_void_p()
        check(lib.mmp_event_create(ctypes.byref(p)))
        self.ptr = p.value

    def record(self) -> None:
        check(lib.mmp_event_record(ctypes.c_void_p(self.ptr)))

    def elapsed_ms(self, end: "Event") -> float:
        ms = ctypes.c_float(0)
        check(lib.mmp_event_elapsed_ms(ctypes.c_void_p(self.ptr), ctypes.c_void_p(end.ptr),
                                       ctypes.byref(ms)))
        return float(ms.value)

    def __del__(self):
        if getattr(self, "ptr", None):
            try:
                lib.mmp_event_destroy(ctypes.c_void_p(self.ptr))
            except Exception:
                pass
            self.ptr = None
