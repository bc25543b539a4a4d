"""Device memory and stream plumbing for the C ABI (PyTorch is used only as the CUDA allocator,
the stream/event handle and the NCCL process group; no torch operator computes anything on the
SALT path)."""
from __future__ import annotations

import ctypes
from typing import NamedTuple

import numpy as np

try:
    import torch
except ImportError:  # pragma: no cover - torch is part of the image
    torch = None

from .stream import PAD_TIME, EventStream


def require_cuda() -> None:
    if torch is None or not torch.cuda.is_available():
        raise RuntimeError("salt_b200 needs a CUDA device (B200, sm_100a); there is no CPU "
                           "fallback")


def ptr(t) -> ctypes.c_void_p | None:
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def current_stream() -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def to_device(a: np.ndarray, dtype) -> "torch.Tensor":
    return torch.from_numpy(np.array(a, dtype=dtype, copy=True, order="C")).cuda()


def workspace(nbytes: int) -> "torch.Tensor":
    """A device buffer of at least nbytes whose data pointer is 256-byte aligned."""
    buf = torch.empty(max(int(nbytes), 1) + 256, dtype=torch.uint8, device="cuda")
    off = (-buf.data_ptr()) % 256
    return buf[off:off + max(int(nbytes), 1)]


class DeviceStream(NamedTuple):
    """A batched event stream resident on the device: (B, capacity) times/sources, (B,) n_real.

    virtual_pads: entries at or beyond min(n_real, capacity) are pads that were not written
    (they read as time 1e12, source 0 — salt_core/stream.py:42-45).
    """
    times: "torch.Tensor"
    src: "torch.Tensor"
    n_real: "torch.Tensor"
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
        t = self.times.cpu().numpy().copy()
        s = self.src.cpu().numpy().copy()
        n = self.n_real.cpu().numpy().astype(np.int32)
        if self.virtual_pads:
            idx = np.arange(t.shape[1])[None, :]
            pad = idx >= np.minimum(n, t.shape[1])[:, None]
            t[pad] = PAD_TIME
            s[pad] = 0
        return EventStream(t, s, np.ones_like(t, dtype=np.float32), n)
