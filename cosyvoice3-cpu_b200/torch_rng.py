"""PyTorch's CPU random stream, generated on the GPU; the surface of
``cv3cpu/torch_rng.py`` (``randn``, ``rand``, ``TorchMT19937``).

The arithmetic runs in ``libcv3cuda.so`` (``cv3_torch_rand``, ``cv3_torch_randn``,
``cv3_torch_u32``, ``cv3_torch_rand64``) and equals the reference bit for bit.  Results come back
as NumPy arrays unless ``device=True`` is passed.
"""

from __future__ import annotations

import numpy as np

from . import _dev as D
from ._lib import call

torch = D.torch


def _numel(shape):
    shape = (shape,) if isinstance(shape, int) else tuple(shape)
    return shape, (int(np.prod(shape)) if shape else 1)


def randn(shape, seed: int = 0, gen: "TorchMT19937 | None" = None, device: bool = False):
    """``torch.manual_seed(seed); torch.randn(shape)``; cv3cpu/torch_rng.py:117-142."""
    shape, n = _numel(shape)
    if gen is not None:
        return gen.randn(shape, device=device)
    out = D.empty((n,))
    scratch = D.empty((32,))
    call("cv3_torch_randn", seed & 0xFFFFFFFF, 0, n, D.ptr(out), D.ptr(scratch), D.stream())
    out = out.reshape(shape)
    return out if device else out.cpu().numpy()


def rand(shape, seed: int = 0, gen: "TorchMT19937 | None" = None, device: bool = False):
    """``torch.manual_seed(seed); torch.rand(shape)``; cv3cpu/torch_rng.py:145-150."""
    shape, n = _numel(shape)
    if gen is not None:
        return gen.rand(shape, device=device)
    out = D.empty((n,))
    call("cv3_torch_rand", seed & 0xFFFFFFFF, 0, n, D.ptr(out), D.stream())
    out = out.reshape(shape)
    return out if device else out.cpu().numpy()


class TorchMT19937:
    """A generator position in torch's stream (cv3cpu/torch_rng.py:27-102).

    The device kernel regenerates the stream from the seed and skips to the
    current position, so successive draws continue the same stream.
    """

    def __init__(self, seed: int = 0):
        self.seed = seed & 0xFFFFFFFF
        self.pos = 0

    def next_u32(self, n: int, device: bool = False):
        """The next ``n`` tempered 32-bit words (cv3cpu/torch_rng.py:71-86)."""
        out = D.empty((n,), D.I32)
        if n:
            call("cv3_torch_u32", self.seed, self.pos, n, D.ptr(out), D.stream())
        self.pos += n
        return out if device else out.cpu().numpy().view(np.uint32)

    def random_float64(self, n: int, device: bool = False):
        """``n`` double uniforms from word pairs, first word high (cv3cpu/torch_rng.py:93-102)."""
        out = D.empty((n,), D.F64)
        if n:
            call("cv3_torch_rand64", self.seed, self.pos, n, D.ptr(out), D.stream())
        self.pos += 2 * n
        return out if device else out.cpu().numpy()

    def random_float32(self, n: int, device: bool = False):
        out = D.empty((n,))
        if n:
            call("cv3_torch_rand", self.seed, self.pos, n, D.ptr(out), D.stream())
        self.pos += n
        return out if device else out.cpu().numpy()

    def rand(self, shape, device: bool = False):
        shape, n = _numel(shape)
        r = self.random_float32(n, device=True).reshape(shape)
        return r if device else r.cpu().numpy()

    def randn(self, shape, device: bool = False):
        shape, n = _numel(shape)
        out = D.empty((n,))
        scratch = D.empty((32,))
        if n:
            call("cv3_torch_randn", self.seed, self.pos, n, D.ptr(out), D.ptr(scratch), D.stream())
        self.pos += (n + (16 if n % 16 else 0)) if n >= 16 else 4 * ((n + 1) // 2)
        out = out.reshape(shape)
        return out if device else out.cpu().numpy()
