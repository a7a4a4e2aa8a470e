"""Device-resident tensors and per-GPU contexts.

``DeviceTensor`` is the device-storage counterpart of the reference's
``DenseTensor<T>`` (src/Lokad.Onnx.Tensors/DenseTensor.cs:31-278): a dense
row-major buffer plus its dimensions, living in one GPU's HBM.  Reshape is a
zero-copy view over the same buffer (DenseTensor.cs:231-242).
"""
from __future__ import annotations

import ctypes
import threading

import numpy as np

from . import _native as N

ONNX_DTYPE = {np.dtype(np.float32): 1, np.dtype(np.int64): 7, np.dtype(np.int32): 6,
              np.dtype(np.uint8): 2, np.dtype(np.bool_): 9, np.dtype(np.float64): 11}
NP_DTYPE = {v: k for k, v in ONNX_DTYPE.items()}


class Context:
    """One GPU: device, CUDA stream and caching allocator (lonnx_ctx)."""

    _default = {}
    _lock = threading.Lock()

    def __init__(self, device: int = 0):
        h = ctypes.c_void_p()
        N.check(N.lib.lonnx_ctx_create(device, ctypes.byref(h)))
        self.handle = h
        self.device = device

    @classmethod
    def default(cls, device: int = 0) -> "Context":
        with cls._lock:
            if device not in cls._default:
                cls._default[device] = cls(device)
            return cls._default[device]

    def sync(self):
        N.check(N.lib.lonnx_sync(self.handle))

    @property
    def launches(self) -> int:
        return int(N.lib.lonnx_launch_count(self.handle))

    @property
    def stream(self) -> int:
        return int(N.lib.lonnx_ctx_stream(self.handle) or 0)

    def close(self):
        if self.handle:
            N.lib.lonnx_ctx_destroy(self.handle)
            self.handle = None


class DeviceTensor:
    """A dense tensor in device memory (float32 activations, int64 indices)."""

    def __init__(self, ctx: Context, shape, dtype, ptr=None, owner=None):
        self.ctx = ctx
        self.shape = tuple(int(s) for s in shape)
        self.dtype = np.dtype(dtype)
        self.name = None
        self._owner = owner
        if ptr is None:
            p = ctypes.c_void_p()
            N.check(N.lib.lonnx_malloc(ctx.handle, max(self.nbytes, 1), ctypes.byref(p)))
            self.ptr = p.value
            self._owns = True
        else:
            self.ptr = ptr
            self._owns = False

    @property
    def size(self) -> int:
        return int(np.prod(self.shape)) if self.shape else 1

    @property
    def nbytes(self) -> int:
        return self.size * self.dtype.itemsize

    @property
    def rank(self) -> int:
        return len(self.shape)

    @classmethod
    def from_host(cls, ctx: Context, arr) -> "DeviceTensor":
        a = np.ascontiguousarray(arr)
        t = cls(ctx, a.shape, a.dtype)
        if a.nbytes:
            N.check(N.lib.lonnx_memcpy_h2d(ctx.handle, t.ptr, a.ctypes.data, a.nbytes))
            # pageable source: the copy is staged before returning, but keep the
            # array alive until the stream has consumed it
            t._host_ref = a
        return t

    def to_host(self) -> np.ndarray:
        out = np.empty(self.shape, self.dtype)
        if out.nbytes:
            N.check(N.lib.lonnx_memcpy_d2h(self.ctx.handle, out.ctypes.data, self.ptr, out.nbytes))
        return out

    def reshape(self, *shape) -> "DeviceTensor":
        if len(shape) == 1 and isinstance(shape[0], (tuple, list)):
            shape = tuple(shape[0])
        shape = list(shape)
        if -1 in shape:
            known = int(np.prod([s for s in shape if s != -1]))
            shape[shape.index(-1)] = self.size // known
        if int(np.prod(shape)) != self.size:
            raise ValueError(f"cannot reshape {self.shape} to {tuple(shape)}")
        return DeviceTensor(self.ctx, shape, self.dtype, ptr=self.ptr, owner=self)

    def __del__(self):
        try:
            if self._owns and self.ptr and self.ctx.handle:
                N.lib.lonnx_free(self.ctx.handle, self.ptr)
        except Exception:
            pass

    def __repr__(self):
        return f"DeviceTensor(shape={self.shape}, dtype={self.dtype}, device={self.ctx.device})"
