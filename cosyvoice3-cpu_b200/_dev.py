"""Device plumbing for the host mirror: CUDA tensors, raw pointers, the stream.

PyTorch provides device memory and the current stream only; all arithmetic
runs in ``libcv3cuda.so``.  Host NumPy inputs are uploaded, and results are
returned in the caller's container type (NumPy in -> NumPy out, CUDA tensor in
-> CUDA tensor out), which is how the ``ops`` mirror keeps the reference's
NumPy signatures while the model stages stay device-resident.
"""

from __future__ import annotations

import ctypes

import numpy as np

try:
    import torch
except ImportError as e:  # pragma: no cover
    raise RuntimeError("the cv3 B200 build needs PyTorch for device memory") from e


def require_cuda() -> None:
    if not torch.cuda.is_available():
        raise RuntimeError("no CUDA device visible: the cv3 B200 kernels have no CPU path")


def is_host(x) -> bool:
    return not isinstance(x, torch.Tensor)


def dev(x, dtype=torch.float32) -> "torch.Tensor":
    """A contiguous CUDA tensor of ``dtype`` holding ``x`` (no copy if already one)."""
    require_cuda()
    if isinstance(x, torch.Tensor):
        if not x.is_cuda:
            x = x.cuda()
        if x.dtype != dtype:
            x = x.to(dtype)
        return x.contiguous()
    npdt = {torch.float32: np.float32, torch.float64: np.float64, torch.int32: np.int32,
            torch.int64: np.int64, torch.int8: np.int8, torch.float16: np.float16}[dtype]
    return torch.from_numpy(np.ascontiguousarray(np.asarray(x, dtype=npdt))).cuda()


def empty(shape, dtype=torch.float32) -> "torch.Tensor":
    require_cuda()
    return torch.empty(tuple(int(s) for s in shape), dtype=dtype, device="cuda")


def zeros(shape, dtype=torch.float32) -> "torch.Tensor":
    require_cuda()
    return torch.zeros(tuple(int(s) for s in shape), dtype=dtype, device="cuda")


def ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def out(t, host: bool):
    return t.cpu().numpy() if host else t
