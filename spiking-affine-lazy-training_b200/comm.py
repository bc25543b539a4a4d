"""NCCL for the sharded forward, through its C API (libnccl.so.2, loaded with ctypes).

The only collective of the multi-GPU path is the all-gather of each rank's int32 logits (and
fits) after its shard's forward (samples are independent: the reference vmaps the network over
the batch, salt_core/network.py:179-183).  One process per GPU; the ranks agree on an NCCL
unique id through any key-value store with ``set(key, bytes)`` and a blocking ``get(key)``
(for example the TCP store a launcher already runs).

A rank that dies leaves its peers' collective waiting on the GPU.  ``NcclComm.wait`` bounds that
wait: it polls the collective's completion and NCCL's asynchronous error state, and past the
timeout aborts the communicator (which ends the pending kernels) and raises ``CommError``.
"""
from __future__ import annotations

import ctypes
import os
import sys
import time

import numpy as np

from .device import DeviceArray, Event, current_stream

_NCCL_DTYPES = {np.dtype(np.int8): 0, np.dtype(np.uint8): 1, np.dtype(np.int32): 2,
                np.dtype(np.uint32): 3, np.dtype(np.int64): 4, np.dtype(np.uint64): 5,
                np.dtype(np.float16): 6, np.dtype(np.float32): 7, np.dtype(np.float64): 8}
_IN_PROGRESS = 7
_nccl = None


class CommError(RuntimeError):
    pass


class _UniqueId(ctypes.Structure):
    _fields_ = [("internal", ctypes.c_char * 128)]

    @staticmethod
    def from_bytes(raw: bytes) -> "_UniqueId":
        if len(raw) != 128:
            raise ValueError("an NCCL unique id has 128 bytes")
        uid = _UniqueId()
        ctypes.memmove(ctypes.addressof(uid), raw, 128)   # (the field itself reads as a copy)
        return uid

    def to_bytes(self) -> bytes:
        return ctypes.string_at(ctypes.addressof(self), 128)


def nccl():
    """libnccl.so.2 (the copy already in the process if another library loaded one)."""
    global _nccl
    if _nccl is None:
        # by soname first: a process that already loaded an NCCL (another library's) shares it
        names = [os.environ.get("SALT_NCCL_LIBRARY") or "libnccl.so.2"]
        names += [os.path.join(p, "nvidia", "nccl", "lib", "libnccl.so.2") for p in sys.path
                  if p and os.path.exists(os.path.join(p, "nvidia", "nccl", "lib",
                                                       "libnccl.so.2"))]
        err = None
        for name in names:
            try:
                _nccl = ctypes.CDLL(name, mode=ctypes.RTLD_GLOBAL)
                break
            except OSError as e:
                err = e
        if _nccl is None:
            raise CommError(f"libnccl.so.2 could not be loaded: {err}")
        vp, ci = ctypes.c_void_p, ctypes.c_int
        sigs = {"ncclGetErrorString": (ctypes.c_char_p, [ci]),
                "ncclGetVersion": (ci, [ctypes.POINTER(ci)]),
                "ncclGetUniqueId": (ci, [ctypes.POINTER(_UniqueId)]),
                "ncclCommInitRank": (ci, [ctypes.POINTER(vp), ci, _UniqueId, ci]),
                "ncclAllGather": (ci, [vp, vp, ctypes.c_size_t, ci, vp, vp]),
                "ncclCommGetAsyncError": (ci, [vp, ctypes.POINTER(ci)]),
                "ncclCommAbort": (ci, [vp]),
                "ncclCommDestroy": (ci, [vp])}
        for name, (res, args) in sigs.items():
            fn = getattr(_nccl, name)
            fn.restype, fn.argtypes = res, args
    return _nccl


def _check(rc: int, what: str) -> None:
    if rc != 0:
        msg = nccl().ncclGetErrorString(rc).decode(errors="replace")
        raise CommError(f"{what}: NCCL error {rc} ({msg})")


def nccl_version() -> int:
    v = ctypes.c_int(0)
    _check(nccl().ncclGetVersion(ctypes.byref(v)), "ncclGetVersion")
    return int(v.value)


def new_unique_id() -> bytes:
    uid = _UniqueId()
    _check(nccl().ncclGetUniqueId(ctypes.byref(uid)), "ncclGetUniqueId")
    return uid.to_bytes()


class NcclComm:
    """One rank of an NCCL communicator on the current device."""

    def __init__(self, rank: int, world: int, unique_id: bytes):
        self.rank, self.world = int(rank), int(world)
        uid = _UniqueId.from_bytes(bytes(unique_id))
        comm = ctypes.c_void_p()
        _check(nccl().ncclCommInitRank(ctypes.byref(comm), self.world, uid, self.rank),
               "ncclCommInitRank")
        self._comm = comm
        self._done = Event()

    @classmethod
    def from_store(cls, store, rank: int, world: int, key: str = "salt_b200/nccl_id"):
        """Rank 0 makes the unique id and publishes it under `key`; the others read it."""
        if rank == 0:
            uid = new_unique_id()
            store.set(key, uid)
        else:
            uid = bytes(store.get(key))
        return cls(rank, world, uid)

    def all_gather(self, send: DeviceArray, recv: DeviceArray, stream=None) -> None:
        """recv (world * rows, ...) <- every rank's send (rows, ...), in rank order; enqueued on
        `stream` (the current stream by default), not waited for."""
        if recv.nbytes != send.nbytes * self.world or recv.dtype != send.dtype:
            raise ValueError("all_gather: recv must hold world x send of the same dtype")
        s = stream or current_stream()
        _check(nccl().ncclAllGather(ctypes.c_void_p(send.data_ptr()),
                                    ctypes.c_void_p(recv.data_ptr()),
                                    ctypes.c_size_t(send.size), _NCCL_DTYPES[send.dtype],
                                    self._comm, s.ptr), "ncclAllGather")
        self._done.record(s)

    def wait(self, timeout_s: float = 60.0) -> None:
        """Waits for the last collective; raises CommError (after aborting the communicator)
        when a peer's failure is reported or the timeout passes."""
        deadline = time.monotonic() + float(timeout_s)
        state = ctypes.c_int(0)
        while not self._done.query():
            _check(nccl().ncclCommGetAsyncError(self._comm, ctypes.byref(state)),
                   "ncclCommGetAsyncError")
            if state.value not in (0, _IN_PROGRESS):
                self.abort()
                raise CommError(f"a peer failed: NCCL async error {state.value}")
            if time.monotonic() > deadline:
                self.abort()
                raise CommError(f"collective did not finish within {timeout_s} s")
            time.sleep(0.0005)

    def abort(self) -> None:
        if self._comm:
            nccl().ncclCommAbort(self._comm)
            self._comm = ctypes.c_void_p()

    def close(self) -> None:
        if self._comm:
            _check(nccl().ncclCommDestroy(self._comm), "ncclCommDestroy")
            self._comm = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
