"""Device plumbing for the host mirror: device arrays, raw pointers, the stream.

All arithmetic runs in ``libcv3cuda.so``; this module only owns device memory.
Host NumPy inputs are uploaded, and results come back in the caller's container
type (NumPy in -> NumPy out, device array in -> device array out), which is how
the ``ops`` mirror keeps the reference's NumPy signatures while the model stages
stay device-resident.

Two memory providers:

* PyTorch (the default when it is importable): CUDA tensors, torch's caching
  allocator and current stream.  The model stages (CUDA graphs, batched engines)
  use this one.
* NumPy + ctypes only (``CV3_HOST=numpy``, or PyTorch not installed):
  :class:`DeviceArray` buffers from the library's own ``cv3_device_alloc`` /
  ``cv3_memcpy`` entry points on the default stream.  ``ops``, ``quant.qmatmul``
  and ``torch_rng`` then run with no GPU framework at all, as cv3cpu's NumPy
  host does.
"""

from __future__ import annotations

import ctypes
import os

import numpy as np

from ._lib import call

torch = None
if os.environ.get("CV3_HOST", "torch").lower() != "numpy":
    try:
        import torch  # noqa: F811
    except ImportError:  # pragma: no cover - exercised by the NumPy-host test
        torch = None

BACKEND = "torch" if torch is not None else "numpy"


class DeviceArray:
    """A contiguous device buffer with a shape and a NumPy dtype.

    Memory comes from ``cv3_device_alloc`` and is returned by ``cv3_device_free``
    when the owning array is collected (views keep their owner alive).  The
    subset of the tensor interface the ops layer uses is provided: ``shape``,
    ``dtype``, ``data_ptr()``, ``dim()``, ``numel()``, ``reshape``, ``unsqueeze``,
    integer indexing of the first axis, ``clone``, ``copy_``, ``cpu().numpy()``.
    """

    is_cuda = True

    def __init__(self, shape, dtype=np.float32, _ptr=None, _base=None):
        self.shape = tuple(int(s) for s in shape)
        self.dtype = np.dtype(dtype)
        self._base = _base
        if _ptr is None:
            p = ctypes.c_void_p(0)
            call("cv3_device_alloc", self.nbytes, ctypes.byref(p))
            self._ptr = p.value or 0
            self._owner = True
        else:
            self._ptr = int(_ptr)
            self._owner = False

    def __del__(self):
        if getattr(self, "_owner", False) and self._ptr:
            try:
                call("cv3_device_free", ctypes.c_void_p(self._ptr))
            except Exception:  # pragma: no cover - interpreter shutdown
                pass
            self._ptr = 0

    def __repr__(self):
        return f"DeviceArray(shape={self.shape}, dtype={self.dtype.name})"

    @property
    def nbytes(self) -> int:
        return self.numel() * self.dtype.itemsize

    def data_ptr(self) -> int:
        return self._ptr

    def dim(self) -> int:
        return len(self.shape)

    def numel(self) -> int:
        return int(np.prod(self.shape, dtype=np.int64)) if self.shape else 1

    def contiguous(self) -> "DeviceArray":
        return self

    def _view(self, shape, offset_bytes: int = 0) -> "DeviceArray":
        return DeviceArray(shape, self.dtype, self._ptr + offset_bytes, self._base or self)

    def reshape(self, *shape) -> "DeviceArray":
        if len(shape) == 1 and isinstance(shape[0], (tuple, list)):
            shape = tuple(shape[0])
        shape = list(int(s) for s in shape)
        if -1 in shape:
            i = shape.index(-1)
            rest = int(np.prod([s for j, s in enumerate(shape) if j != i], dtype=np.int64))
            shape[i] = self.numel() // max(rest, 1)
        if int(np.prod(shape, dtype=np.int64)) != self.numel():
            raise ValueError(f"cannot reshape {self.shape} to {tuple(shape)}")
        return self._view(shape)

    def unsqueeze(self, axis: int) -> "DeviceArray":
        shape = list(self.shape)
        shape.insert(axis if axis >= 0 else len(shape) + 1 + axis, 1)
        return self._view(shape)

    def __getitem__(self, i):
        if not isinstance(i, (int, np.integer)):
            raise TypeError("DeviceArray supports integer indexing of the first axis only")
        n = self.shape[0]
        i = int(i) + (n if i < 0 else 0)
        if not 0 <= i < n:
            raise IndexError(f"index {i} out of range for axis 0 of size {n}")
        sub = self.shape[1:]
        step = int(np.prod(sub, dtype=np.int64)) if sub else 1
        return self._view(sub, i * step * self.dtype.itemsize)

    def copy_(self, src) -> "DeviceArray":
        if src.nbytes != self.nbytes:
            raise ValueError("copy_: size mismatch")
        call("cv3_memcpy", ctypes.c_void_p(self._ptr), ctypes.c_void_p(src.data_ptr()), self.nbytes, 2, None)
        return self

    def clone(self) -> "DeviceArray":
        return DeviceArray(self.shape, self.dtype).copy_(self)

    def cpu(self) -> "DeviceArray":
        return self

    def numpy(self) -> np.ndarray:
        host = np.empty(self.shape, self.dtype)
        if host.nbytes:
            call("cv3_memcpy", host.ctypes.data_as(ctypes.c_void_p), ctypes.c_void_p(self._ptr), host.nbytes, 1, None)
            call("cv3_stream_synchronize", None)
        return host

    @staticmethod
    def from_numpy(a) -> "DeviceArray":
        a = np.ascontiguousarray(a)
        d = DeviceArray(a.shape, a.dtype)
        if a.nbytes:
            call("cv3_memcpy", ctypes.c_void_p(d.data_ptr()), a.ctypes.data_as(ctypes.c_void_p), a.nbytes, 0, None)
        return d


# element types, in the provider's own terms
if torch is not None:
    F32, F64, F16, I64, I32, I16, I8, U8 = (torch.float32, torch.float64, torch.float16, torch.int64, torch.int32,
                                            torch.int16, torch.int8, torch.uint8)
    _NP = {torch.float32: np.float32, torch.float64: np.float64, torch.int32: np.int32, torch.int64: np.int64,
           torch.int8: np.int8, torch.float16: np.float16, torch.int16: np.int16, torch.uint8: np.uint8}
else:
    F32, F64, F16, I64, I32, I16, I8, U8 = (np.float32, np.float64, np.float16, np.int64, np.int32, np.int16,
                                            np.int8, np.uint8)
    _NP = {t: t for t in (F32, F64, F16, I64, I32, I16, I8, U8)}


_device_seen = False


def require_cuda() -> None:
    global _device_seen
    if torch is not None:
        if not torch.cuda.is_available():
            raise RuntimeError("no CUDA device visible: the cv3 B200 kernels have no CPU path")
        return
    if _device_seen:
        return
    n = ctypes.c_int(0)
    try:
        call("cv3_device_info", ctypes.byref(n), None, None)
    except Exception as e:
        raise RuntimeError("no CUDA device visible: the cv3 B200 kernels have no CPU path") from e
    _device_seen = True


def is_device(x) -> bool:
    return isinstance(x, DeviceArray) or (torch is not None and isinstance(x, torch.Tensor))


def is_host(x) -> bool:
    return not is_device(x)


def is_half(x) -> bool:
    """A table of fp16 values (host array or device array)."""
    dt = x.dtype
    return dt == np.float16 or (torch is not None and dt == torch.float16)


def dev(x, dtype=None):
    """A contiguous device array of ``dtype`` (default float32) holding ``x`` (no copy if
    it already is one)."""
    dtype = F32 if dtype is None else dtype
    require_cuda()
    if torch is not None:
        if isinstance(x, torch.Tensor):
            if not x.is_cuda:
                x = x.cuda()
            if x.dtype != dtype:
                x = x.to(dtype)
            return x.contiguous()
        return torch.from_numpy(np.ascontiguousarray(np.asarray(x, dtype=_NP[dtype]))).cuda()
    if isinstance(x, DeviceArray):
        if x.dtype != np.dtype(dtype):
            raise TypeError(f"device array of {x.dtype} where {np.dtype(dtype)} is expected")
        return x
    return DeviceArray.from_numpy(np.asarray(x, dtype=_NP[dtype]))


def empty(shape, dtype=None):
    dtype = F32 if dtype is None else dtype
    require_cuda()
    shape = tuple(int(s) for s in shape)
    if torch is not None:
        return torch.empty(shape, dtype=dtype, device="cuda")
    return DeviceArray(shape, dtype)


def empty_like(x):
    if torch is not None and isinstance(x, torch.Tensor):
        return torch.empty_like(x)
    return DeviceArray(x.shape, x.dtype)


def zeros(shape, dtype=None):
    dtype = F32 if dtype is None else dtype
    require_cuda()
    shape = tuple(int(s) for s in shape)
    if torch is not None:
        return torch.zeros(shape, dtype=dtype, device="cuda")
    d = DeviceArray(shape, dtype)
    call("cv3_memset", ctypes.c_void_p(d.data_ptr()), 0, d.nbytes, None)
    return d


def ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream():
    """The stream the ops are ordered on: torch's current stream, or the default stream."""
    if torch is not None:
        return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    return None


def upload(a):
    """A device copy of the host array ``a`` with its own element type."""
    a = np.ascontiguousarray(a)
    require_cuda()
    if torch is not None:
        return torch.from_numpy(a).cuda()
    return DeviceArray.from_numpy(a)


def out(t, host: bool):
    if isinstance(t, np.ndarray):
        return t
    return t.cpu().numpy() if host else t
