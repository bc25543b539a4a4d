"""Device memory, pinned host memory, streams, events and graph replay for the host side.

Everything goes through the runtime entry points of libsalt_b200 (salt_malloc, salt_memcpy_async,
salt_stream_*, salt_event_*, salt_graph_*; include/salt_b200.h), so the package needs no GPU
framework: numpy arrays on the host, DeviceArray on the device.  Under JAX, XLA would own these
buffers and streams instead (the reference's setting).

Streams: every call of this package enqueues on the *current stream* of the calling thread, the
legacy default stream unless a `Stream` is made current with `use_stream`.  Device memory is
stream-ordered: it is allocated on the current stream and, when its last reference goes, freed
on the stream that allocated it.
"""
from __future__ import annotations

import contextlib
import ctypes
import threading
import weakref
from typing import NamedTuple

import numpy as np

from . import _lib
from .stream import PAD_TIME, EventStream

_tls = threading.local()


def _vp(x) -> ctypes.c_void_p:
    return ctypes.c_void_p(x)


def device_count() -> int:
    n = ctypes.c_int32(0)
    try:
        _lib.check(_lib.lib().salt_device_count(ctypes.byref(n)))
    except (OSError, RuntimeError):
        return 0
    return int(n.value)


def require_cuda() -> None:
    if device_count() < 1:
        raise RuntimeError("salt_b200 needs a CUDA device (B200, sm_100a); there is no CPU "
                           "fallback")


def set_device(index: int) -> None:
    _lib.check(_lib.lib().salt_set_device(int(index)))


def current_device() -> int:
    d = ctypes.c_int32(0)
    _lib.check(_lib.lib().salt_get_device(ctypes.byref(d)))
    return int(d.value)


def synchronize() -> None:
    """Waits for all work on the current device."""
    _lib.check(_lib.lib().salt_device_synchronize())


# ---------------------------------------------------------------- streams and events

class Stream:
    """A CUDA stream.  Stream() creates a non-blocking stream (high_priority=True: one whose
    blocks the scheduler prefers); Stream.default() is the legacy default stream (handle NULL)."""

    def __init__(self, _handle: int | None = None, _owned: bool = True,
                 high_priority: bool = False):
        if _handle is None and _owned:
            h = ctypes.c_void_p()
            make = (_lib.lib().salt_stream_create_high_priority if high_priority
                    else _lib.lib().salt_stream_create)
            _lib.check(make(ctypes.byref(h)))
            _handle = h.value
        self.handle = _handle or 0
        self._owned = bool(_owned and self.handle)
        if self._owned:
            weakref.finalize(self, _lib.lib().salt_stream_destroy, _vp(self.handle))

    @staticmethod
    def default() -> "Stream":
        return Stream(0, _owned=False)

    @property
    def ptr(self) -> ctypes.c_void_p:
        return _vp(self.handle)

    def synchronize(self) -> None:
        _lib.check(_lib.lib().salt_stream_synchronize(self.ptr))

    def wait_event(self, event: "Event") -> None:
        _lib.check(_lib.lib().salt_stream_wait_event(self.ptr, event.ptr))

    def wait_stream(self, other: "Stream") -> None:
        ev = Event()
        ev.record(other)
        self.wait_event(ev)


def current_stream() -> Stream:
    stack = getattr(_tls, "streams", None)
    return stack[-1] if stack else Stream.default()


def stream_handle() -> ctypes.c_void_p:
    """The current stream as the C ABI takes it."""
    return current_stream().ptr


@contextlib.contextmanager
def use_stream(stream: Stream):
    """Makes `stream` the calling thread's current stream inside the block."""
    stack = getattr(_tls, "streams", None)
    if stack is None:
        stack = _tls.streams = []
    stack.append(stream)
    try:
        yield stream
    finally:
        stack.pop()


class Event:
    """A CUDA event; timing=True allows elapsed_ms between two recorded events."""

    def __init__(self, timing: bool = False):
        h = ctypes.c_void_p()
        _lib.check(_lib.lib().salt_event_create(int(bool(timing)), ctypes.byref(h)))
        self.handle = h.value
        weakref.finalize(self, _lib.lib().salt_event_destroy, _vp(self.handle))

    @property
    def ptr(self) -> ctypes.c_void_p:
        return _vp(self.handle)

    def record(self, stream: Stream | None = None) -> "Event":
        _lib.check(_lib.lib().salt_event_record(self.ptr, (stream or current_stream()).ptr))
        return self

    def synchronize(self) -> None:
        _lib.check(_lib.lib().salt_event_synchronize(self.ptr))

    def query(self) -> bool:
        """True once the work before the last record has finished (does not wait)."""
        done = ctypes.c_int32(0)
        _lib.check(_lib.lib().salt_event_query(self.ptr, ctypes.byref(done)))
        return bool(done.value)

    def elapsed_ms(self, end: "Event") -> float:
        ms = ctypes.c_float(0.0)
        _lib.check(_lib.lib().salt_event_elapsed_ms(self.ptr, end.ptr, ctypes.byref(ms)))
        return float(ms.value)


class Graph:
    """Everything enqueued on a non-default stream while capturing, replayed with one launch.
    Usage: ``with Graph.capture(stream) as g: <enqueue work on stream>``, then ``g.replay()``."""

    def __init__(self):
        self.handle = None

    @staticmethod
    @contextlib.contextmanager
    def capture(stream: Stream):
        g = Graph()
        _lib.check(_lib.lib().salt_graph_begin_capture(stream.ptr))
        try:
            with use_stream(stream):
                yield g
        finally:
            h = ctypes.c_void_p()
            _lib.check(_lib.lib().salt_graph_end_capture(stream.ptr, ctypes.byref(h)))
            g.handle = h.value
            weakref.finalize(g, _lib.lib().salt_graph_destroy, _vp(g.handle))

    def replay(self, stream: Stream | None = None) -> None:
        _lib.check(_lib.lib().salt_graph_launch(_vp(self.handle),
                                                (stream or current_stream()).ptr))


# ---------------------------------------------------------------- device arrays

class _Allocation:
    """One device allocation, freed (stream-ordered) on the stream that made it."""
    __slots__ = ("ptr", "nbytes", "stream", "__weakref__")

    def __init__(self, nbytes: int):
        self.nbytes = int(nbytes)
        self.stream = current_stream()
        p = ctypes.c_void_p()
        _lib.check(_lib.lib().salt_malloc(ctypes.c_size_t(max(self.nbytes, 1)), self.stream.ptr,
                                          ctypes.byref(p)))
        self.ptr = int(p.value or 0)
        # the finalizer holds the Stream, so the stream outlives the allocation
        weakref.finalize(self, _free_on, self.ptr, self.stream)


def _free_on(ptr: int, stream: "Stream") -> None:
    _lib.lib().salt_free(_vp(ptr), stream.ptr)


class DeviceArray:
    """A C-contiguous array in device memory: shape, numpy dtype and a device pointer.
    Indexing the leading axis (an integer or a step-1 slice) gives a view sharing the memory."""
    __slots__ = ("ptr", "shape", "dtype", "_owner")

    def __init__(self, ptr: int, shape, dtype, owner):
        self.ptr = int(ptr)
        self.shape = tuple(int(v) for v in shape)
        self.dtype = np.dtype(dtype)
        self._owner = owner

    # construction
    @staticmethod
    def empty(shape, dtype) -> "DeviceArray":
        shape = (int(shape),) if np.isscalar(shape) else tuple(int(v) for v in shape)
        nbytes = int(np.prod(shape, dtype=np.int64)) * np.dtype(dtype).itemsize
        a = _Allocation(nbytes)
        return DeviceArray(a.ptr, shape, dtype, a)

    @staticmethod
    def zeros(shape, dtype) -> "DeviceArray":
        d = DeviceArray.empty(shape, dtype)
        d.fill_bytes(0)
        return d

    @staticmethod
    def full(shape, value, dtype) -> "DeviceArray":
        return DeviceArray.from_host(np.full(shape, value, dtype=dtype))

    @staticmethod
    def from_host(a, dtype=None) -> "DeviceArray":
        """A device copy of a host array (ordered on the current stream; the host array may be
        reused as soon as this returns)."""
        h = np.ascontiguousarray(np.asarray(a, dtype=dtype))
        d = DeviceArray.empty(h.shape, h.dtype)
        d.copy_from(h, sync=True)
        return d

    # properties
    @property
    def size(self) -> int:
        return int(np.prod(self.shape, dtype=np.int64))

    @property
    def nbytes(self) -> int:
        return self.size * self.dtype.itemsize

    @property
    def ndim(self) -> int:
        return len(self.shape)

    def data_ptr(self) -> int:
        return self.ptr

    def __len__(self) -> int:
        return self.shape[0]

    def __getitem__(self, idx) -> "DeviceArray":
        row = int(np.prod(self.shape[1:], dtype=np.int64)) * self.dtype.itemsize
        if isinstance(idx, (int, np.integer)):
            i = int(idx) + (self.shape[0] if idx < 0 else 0)
            if not 0 <= i < self.shape[0]:
                raise IndexError(idx)
            return DeviceArray(self.ptr + i * row, self.shape[1:], self.dtype, self)
        if isinstance(idx, slice):
            start, stop, step = idx.indices(self.shape[0])
            if step != 1:
                raise IndexError("device views take step-1 slices of the leading axis")
            n = max(0, stop - start)
            return DeviceArray(self.ptr + start * row, (n,) + self.shape[1:], self.dtype, self)
        raise IndexError("device views index the leading axis only")

    def view(self, dtype) -> "DeviceArray":
        dtype = np.dtype(dtype)
        if dtype.itemsize != self.dtype.itemsize:
            raise ValueError("view keeps the element size")
        return DeviceArray(self.ptr, self.shape, dtype, self)

    # transfers
    def copy_from(self, host, *, sync: bool = False, stream: Stream | None = None) -> None:
        """Host (numpy, ideally pinned) -> this array; asynchronous unless sync."""
        h = np.asarray(host)
        if h.nbytes != self.nbytes or not h.flags.c_contiguous:
            raise ValueError(f"copy_from: {h.shape} {h.dtype} into {self.shape} {self.dtype}")
        s = stream or current_stream()
        _lib.check(_lib.lib().salt_memcpy_async(_vp(self.ptr), _vp(h.ctypes.data),
                                                ctypes.c_size_t(self.nbytes), s.ptr))
        if sync:
            s.synchronize()

    def copy_from_device(self, other: "DeviceArray", stream: Stream | None = None) -> None:
        if other.nbytes != self.nbytes:
            raise ValueError("copy_from_device: sizes differ")
        _lib.check(_lib.lib().salt_memcpy_async(_vp(self.ptr), _vp(other.ptr),
                                                ctypes.c_size_t(self.nbytes),
                                                (stream or current_stream()).ptr))

    def copy_to(self, host, *, sync: bool = True, stream: Stream | None = None) -> None:
        """This array -> host (numpy, C-contiguous, same byte size)."""
        if host.nbytes != self.nbytes or not host.flags.c_contiguous:
            raise ValueError("copy_to: size or layout differs")
        s = stream or current_stream()
        _lib.check(_lib.lib().salt_memcpy_async(_vp(host.ctypes.data), _vp(self.ptr),
                                                ctypes.c_size_t(self.nbytes), s.ptr))
        if sync:
            s.synchronize()

    def numpy(self) -> np.ndarray:
        """A host copy (waits for the current stream)."""
        out = np.empty(self.shape, self.dtype)
        if self.nbytes:
            self.copy_to(out)
        return out

    def fill_bytes(self, value: int = 0, stream: Stream | None = None) -> None:
        _lib.check(_lib.lib().salt_memset_async(_vp(self.ptr), int(value),
                                                ctypes.c_size_t(self.nbytes),
                                                (stream or current_stream()).ptr))

    def __repr__(self) -> str:
        return f"DeviceArray(shape={self.shape}, dtype={self.dtype}, ptr=0x{self.ptr:x})"


def empty(shape, dtype) -> DeviceArray:
    return DeviceArray.empty(shape, dtype)


def zeros(shape, dtype) -> DeviceArray:
    return DeviceArray.zeros(shape, dtype)


def to_device(a, dtype) -> DeviceArray:
    return DeviceArray.from_host(a, dtype)


def ptr(a) -> ctypes.c_void_p | None:
    """Device (or host) pointer of an array for the C ABI; None for None.  Host numpy arrays pass
    their data pointer (only where the C ABI asks for host memory)."""
    if a is None:
        return None
    if isinstance(a, np.ndarray):
        return _vp(a.ctypes.data)
    return _vp(a.data_ptr())


def workspace(nbytes: int) -> DeviceArray:
    """A device buffer of at least nbytes (allocations are 256-byte aligned)."""
    return DeviceArray.empty((max(int(nbytes), 1),), np.uint8)


# ---------------------------------------------------------------- pinned host memory

class _PinnedBuffer:
    def __init__(self, nbytes: int):
        p = ctypes.c_void_p()
        _lib.check(_lib.lib().salt_host_alloc(ctypes.c_size_t(max(int(nbytes), 1)),
                                              ctypes.byref(p)))
        self.ptr = int(p.value)
        self.nbytes = int(nbytes)
        self.raw = (ctypes.c_uint8 * max(self.nbytes, 1)).from_address(self.ptr)
        weakref.finalize(self, _lib.lib().salt_host_free, _vp(self.ptr))


class PinnedArray(np.ndarray):
    """A numpy array in page-locked host memory; views keep the memory alive."""
    _pinned = None

    def __array_finalize__(self, obj):
        self._pinned = getattr(obj, "_pinned", None)


def pinned_empty(shape, dtype) -> PinnedArray:
    """A numpy array in page-locked host memory mapped for the device (what asynchronous copies
    and salt_stream_h2d_real need); the memory lives as long as the array or a view of it."""
    shape = (int(shape),) if np.isscalar(shape) else tuple(int(v) for v in shape)
    dt = np.dtype(dtype)
    buf = _PinnedBuffer(int(np.prod(shape, dtype=np.int64)) * dt.itemsize)
    arr = np.frombuffer(buf.raw, dtype=np.uint8, count=buf.nbytes).view(dt).reshape(shape)
    arr = arr.view(PinnedArray)
    arr._pinned = buf
    return arr


def pinned_copy(a, dtype=None) -> np.ndarray:
    h = np.asarray(a, dtype=dtype)
    out = pinned_empty(h.shape, h.dtype)
    out[...] = h
    return out


# ---------------------------------------------------------------- batched event streams

class DeviceStream(NamedTuple):
    """A batched event stream resident on the device: (B, capacity) times/sources, (B,) n_real.

    virtual_pads: entries at or beyond min(n_real, capacity) are pads that were not written
    (they read as time 1e12, source 0 — salt_core/stream.py:42-45).
    """
    times: DeviceArray
    src: DeviceArray
    n_real: DeviceArray
    virtual_pads: bool

    @property
    def batch(self) -> int:
        return int(self.times.shape[0])

    @property
    def capacity(self) -> int:
        return int(self.times.shape[1])

    @staticmethod
    def from_host(stream: EventStream) -> "DeviceStream":
        t = np.asarray(stream.event_times, dtype=np.float32)
        s = np.asarray(stream.event_source_idx)
        n = np.asarray(stream.n_real_events)
        if t.ndim == 1:
            t, s, n = t[None], s[None], n.reshape(1)
        return DeviceStream(to_device(t, np.float32), to_device(s, np.int32),
                            to_device(n, np.int32), False)

    def to_host(self) -> EventStream:
        """Batched EventStream with pads materialised as the reference writes them."""
        t = self.times.numpy()
        s = self.src.numpy()
        n = self.n_real.numpy().astype(np.int32)
        if self.virtual_pads:
            idx = np.arange(t.shape[1])[None, :]
            pad = idx >= np.minimum(n, t.shape[1])[:, None]
            t[pad] = PAD_TIME
            s[pad] = 0
        return EventStream(t, s, np.ones_like(t, dtype=np.float32), n)
