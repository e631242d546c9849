"""Block-quantised weights (q8 and q4) and the quantised linear, on the GPU.

q8 (the reference's "balanced" format, ``cv3cpu/quant.py:9-19``): a weight of
logical shape ``(N, K)`` is stored as an ``int8[N, Kp]`` payload, K padded with
zeros up to a multiple of 64, plus ``float16[N, Kp/64]`` scales, one per (row,
64-wide K block).  ``W[n, k] = float32(q[n, k]) * float32(s[n, k // 64])``.
q4 (the "tiny" profile's LM body, ``cv3cpu/quant.py:70-86``): 32-wide blocks,
``uint8[N, Kp/2]`` with byte j of a block holding code j (low nibble) and code
j + 16 (high nibble), ``W = (code - 8) * scale``.

``quantize_q8`` / ``quantize_q4`` are the format's writers (offline, host side,
identical in result to ``cv3cpu/quant.py:56-86``).  ``qmatmul`` -- the operation the models
run -- executes on the GPU through ``libcv3cuda.so`` and has no CPU path.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import numpy as np

Q8_BLOCK = 64
Q4_BLOCK = 32


@dataclass
class QTensor:
    """A q8 weight: payload, scales, logical shape; ``cv3cpu/quant.py:89-136``.

    ``q`` and ``scales`` may be host NumPy arrays (e.g. views into the weight
    file's mmap) or CUDA tensors; :func:`to_device` returns the device copy.
    """

    kind: str
    q: object
    scales: object
    shape: tuple
    block: int = Q8_BLOCK
    orig_shape: Optional[tuple] = None

    @property
    def kernel_size(self) -> Optional[int]:
        if self.orig_shape is not None and len(self.orig_shape) == 3:
            return int(self.orig_shape[2])
        return None

    @property
    def nbytes(self) -> int:
        return int(self.q.nbytes) + int(self.scales.nbytes)

    @property
    def padded_k(self) -> int:
        return int(self.scales.shape[1]) * self.block

    def to_device(self, device="cuda") -> "QTensor":
        from . import _dev as D
        if D.is_device(self.q):
            return self
        q = D.upload(np.asarray(self.q))
        s = D.upload(np.ascontiguousarray(self.scales).view(np.int16))
        return QTensor(self.kind, q, s, tuple(self.shape), self.block, self.orig_shape)

    def dequant_rows(self, r0: int, r1: int) -> np.ndarray:
        """Host fp32 rows (format inspection only; the GPU path never calls this)."""
        s = np.asarray(self.scales)[r0:r1]
        if s.dtype != np.float16:
            s = s.view(np.float16)
        nb = s.shape[1]
        if self.kind == "q4":   # byte j of a block: code j (low nibble), code j + 16 (high)
            b = np.asarray(self.q)[r0:r1].reshape(r1 - r0, nb, self.block // 2)
            q = np.concatenate([(b & 0x0F).astype(np.float32) - 8.0, (b >> 4).astype(np.float32) - 8.0], axis=2)
        else:
            q = np.asarray(self.q)[r0:r1].astype(np.float32)
        w = (q.reshape(r1 - r0, nb, self.block) * s.astype(np.float32)[:, :, None])
        return w.reshape(r1 - r0, nb * self.block)[:, : self.shape[1]]

    def dequant(self) -> np.ndarray:
        return self.dequant_rows(0, self.shape[0])


def quantize_q8(w: np.ndarray, block: int = Q8_BLOCK):
    """``(int8 [N, Kp], float16 [N, Kp/block], Kp)``: absmax/127 per block,
    round half to even, clip to +-127, zero blocks get scale 1."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    n, k = w.shape
    kp = -(-k // block) * block
    if kp != k:
        w = np.pad(w, ((0, 0), (0, kp - k)))
    b = w.reshape(n, kp // block, block)
    scale = (np.abs(b).max(axis=2) / 127.0).astype(np.float32)
    scale[scale == 0] = 1.0
    q = np.clip(np.rint(b / scale[:, :, None]), -127, 127).astype(np.int8)
    return q.reshape(n, kp), scale.astype(np.float16), kp


def quantize_q4(w: np.ndarray, block: int = Q4_BLOCK):
    """``(uint8 [N, Kp/2], float16 [N, Kp/block], Kp)``: the "tiny" profile's 4-bit
    format (``cv3cpu/quant.py:70-86``): per block the largest-magnitude element (first
    on ties) sets ``scale = ext / -8`` so it maps to code 0; codes ``rint(w / scale +
    8)`` clipped to [0, 15]; byte j packs code j (low nibble) and j + 16 (high)."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    n, k = w.shape
    kp = -(-k // block) * block
    if kp != k:
        w = np.pad(w, ((0, 0), (0, kp - k)))
    b = w.reshape(n, kp // block, block)
    ext = np.take_along_axis(b, np.abs(b).argmax(axis=2)[:, :, None], axis=2)[:, :, 0]
    scale = (ext / -8.0).astype(np.float32)
    scale[scale == 0] = 1.0
    code = np.clip(np.rint(b / scale[:, :, None] + 8.0), 0, 15).astype(np.uint8)
    half = block // 2
    packed = (code[:, :, :half] | (code[:, :, half:] << 4)).astype(np.uint8)
    return packed.reshape(n, kp // 2), scale.astype(np.float16), kp


def make_qtensor(w: np.ndarray, orig_shape=None, kind: str = "q8") -> QTensor:
    if kind not in ("q8", "q4"):
        raise ValueError(f"unknown quant kind {kind!r}")
    q, s, _ = (quantize_q4 if kind == "q4" else quantize_q8)(w.reshape(w.shape[0], -1))
    return QTensor(kind, q, s, (w.shape[0], int(np.prod(w.shape[1:]))), Q4_BLOCK if kind == "q4" else Q8_BLOCK,
                   tuple(orig_shape) if orig_shape is not None else tuple(w.shape))


def qmatmul(x, w, bias=None, tile_bytes=None, threads=None):
    """``x @ W.T (+ bias)`` on the GPU; signature of ``cv3cpu/quant.py:156``.

    ``tile_bytes`` and ``threads`` are accepted for signature compatibility:
    the CUDA kernel streams the payload once and its result does not depend
    on either.
    """
    from . import ops
    return ops.linear(x, w, bias)
