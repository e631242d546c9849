"""The cv3cpu ``.safetensors`` weight file: reader, writer and device cache.

Format (``cv3cpu/io/weights.py:1-14``, ``:60-86``; container
``cv3cpu/io/safetensors_io.py``): a standard safetensors file -- little-endian
u64 header length, JSON header, packed tensor data.  A q8 weight stores its
int8 payload under its own name (``I8``; a q4 weight its packed nibbles, ``U8``)
and its float16 scales under
``<name>.__scales__`` (``F16``); the JSON string ``__metadata__["cv3cpu"]``
holds ``{"version", "meta", "quant": {name: {kind, block, shape, mshape}}}``.

:class:`WeightFile` maps the file read-only and hands out NumPy views or
:class:`QTensor` objects, like the reference.  :class:`DeviceWeights` uploads
tensors once into HBM (keyed by name) and frees them on :meth:`evict`, the
device counterpart of the reference's ``MADV_DONTNEED`` stage release.
"""

from __future__ import annotations

import json
import mmap
import struct
from typing import Any, Dict, Iterable, Optional

import numpy as np

from .quant import QTensor

SCALES_SUFFIX = ".__scales__"
METADATA_KEY = "cv3cpu"
FORMAT_VERSION = 1

_DTYPES = {"F64": np.dtype("<f8"), "F32": np.dtype("<f4"), "F16": np.dtype("<f2"),
           "I64": np.dtype("<i8"), "I32": np.dtype("<i4"), "I16": np.dtype("<i2"),
           "I8": np.dtype("i1"), "U8": np.dtype("u1"), "BOOL": np.dtype("?")}
_TAGS = {v: k for k, v in _DTYPES.items()}


def write_weights(path: str, tensors: Dict[str, Any], meta: Dict[str, Any]) -> None:
    """Write ``name -> ndarray | QTensor`` as a cv3cpu-format ``.safetensors``."""
    index: Dict[str, Any] = {}
    quant: Dict[str, Any] = {}
    blobs = []
    pos = 0

    def add(name, arr):
        nonlocal pos
        arr = np.ascontiguousarray(arr)
        index[name] = {"dtype": _TAGS[arr.dtype],
                       "shape": list(arr.shape), "data_offsets": [pos, pos + arr.nbytes]}
        blobs.append(arr)
        pos += arr.nbytes

    for name in tensors:
        t = tensors[name]
        if isinstance(t, QTensor):
            # q8 payloads are int8 (I8); q4 payloads packed nibbles, uint8 (U8) as quant.py:70-86 makes them
            add(name, np.asarray(t.q).view(np.uint8 if t.kind == "q4" else np.int8))
            sc = np.asarray(t.scales)
            add(name + SCALES_SUFFIX, sc if sc.dtype == np.float16 else sc.view(np.float16))
            quant[name] = {"kind": t.kind, "block": t.block,
                           "shape": list(t.orig_shape if t.orig_shape is not None else t.shape),
                           "mshape": list(t.shape)}
        else:
            add(name, np.asarray(t))
    header = dict(index)
    header["__metadata__"] = {METADATA_KEY: json.dumps(
        {"version": FORMAT_VERSION, "meta": meta, "quant": quant}, separators=(",", ":"))}
    raw = json.dumps(header, separators=(",", ":")).encode("utf-8")
    raw += b" " * ((-len(raw)) % 8)
    with open(path, "wb") as fh:
        fh.write(struct.pack("<Q", len(raw)))
        fh.write(raw)
        for b in blobs:
            fh.write(b.tobytes())


class WeightFile:
    """Read side: ``get(name)`` -> ndarray view or :class:`QTensor` (host)."""

    def __init__(self, path: str):
        self.path = path
        self._fh = open(path, "rb")
        n = struct.unpack("<Q", self._fh.read(8))[0]
        header = json.loads(self._fh.read(n).decode("utf-8"))
        self._base = 8 + n
        md = header.pop("__metadata__", {}) or {}
        blob = json.loads(md.get(METADATA_KEY, "{}"))
        self.meta: Dict[str, Any] = blob.get("meta", {})
        self._quant: Dict[str, Any] = blob.get("quant", {})
        self._index = header
        self._mm = mmap.mmap(self._fh.fileno(), 0, access=mmap.ACCESS_READ)
        self._cache: Dict[str, Any] = {}

    def keys(self) -> Iterable[str]:
        return [k for k in self._index if not k.endswith(SCALES_SUFFIX)]

    def __contains__(self, name: str) -> bool:
        return name in self._index and not name.endswith(SCALES_SUFFIX)

    def _raw(self, name: str) -> np.ndarray:
        e = self._index[name]
        a, b = e["data_offsets"]
        arr = np.frombuffer(self._mm, dtype=_DTYPES[e["dtype"]], count=(b - a) // _DTYPES[e["dtype"]].itemsize,
                            offset=self._base + a).reshape(e["shape"])
        if arr.itemsize > 1 and arr.ctypes.data % arr.itemsize:
            arr = np.array(arr, copy=True)
        return arr

    def entry(self, name: str) -> Dict[str, Any]:
        if name not in self:
            raise KeyError(name)
        q = self._quant.get(name)
        if q is not None:
            return {"kind": q["kind"], "shape": list(q["shape"]), "block": q["block"],
                    "mshape": list(q["mshape"])}
        e = self._index[name]
        kind = {"F32": "f32", "F16": "f16", "I32": "i32", "I64": "i64", "I8": "i8", "U8": "u8"}.get(
            e["dtype"], e["dtype"].lower())
        return {"kind": kind, "shape": list(e["shape"])}

    def get(self, name: str, default=None):
        if name not in self:
            return default
        hit = self._cache.get(name)
        if hit is not None:
            return hit
        q = self._quant.get(name)
        if q is None:
            out = self._raw(name)
        else:
            if q["kind"] not in ("q8", "q4"):
                raise ValueError(f"{name}: quant kind {q['kind']!r} is not supported by the device build")
            out = QTensor(q["kind"], self._raw(name), self._raw(name + SCALES_SUFFIX),
                          tuple(q["mshape"]), int(q["block"]), tuple(q["shape"]))
        self._cache[name] = out
        return out

    def __getitem__(self, name: str):
        if name not in self:
            raise KeyError(name)
        return self.get(name)

    def close(self) -> None:
        self._cache.clear()
        try:
            self._mm.close()
        except BufferError:
            pass
        self._fh.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


class TensorDict(dict):
    """In-memory ``name -> tensor`` mapping with a ``meta`` attribute (synthetic models)."""

    def __init__(self, tensors: Dict[str, Any], meta: Dict[str, Any]):
        super().__init__(tensors)
        self.meta = meta

    def entry(self, name: str) -> Dict[str, Any]:
        t = self[name]
        if isinstance(t, QTensor):
            return {"kind": t.kind, "shape": list(t.orig_shape or t.shape), "mshape": list(t.shape)}
        return {"kind": str(np.asarray(t).dtype), "shape": list(np.shape(t))}


class DeviceWeights:
    """HBM copies of host weights, uploaded on first use and kept by name.

    ``f32(name)`` returns a float32 CUDA tensor (f16 tables widened exactly),
    ``q8(name)`` the device :class:`QTensor`, ``raw(name)`` the tensor in its
    stored dtype.  :meth:`evict` frees every cached tensor under a prefix and
    hands the freed device memory back to the driver (the device counterpart of
    the reference's ``WeightFile.evict``, cv3cpu/io/weights.py:182-205, which
    returns a stage's mmap pages to the OS).
    """

    def __init__(self, host, device: str = "cuda"):
        self.host = host
        self.meta = host.meta
        self.device = device
        self._cache: Dict[Any, Any] = {}

    def __contains__(self, name: str) -> bool:
        return name in self.host

    def entry(self, name: str):
        return self.host.entry(name)

    def _put(self, key, fn):
        hit = self._cache.get(key)
        if hit is None:
            hit = fn()
            self._cache[key] = hit
        return hit

    def host_tensor(self, name: str):
        return self.host[name] if not hasattr(self.host, "get") else self.host.get(name)

    def raw(self, name: str):
        import torch
        return self._put(("raw", name), lambda: torch.from_numpy(
            np.ascontiguousarray(np.asarray(self.host_tensor(name)))).to(self.device))

    def f32(self, name: str):
        import torch
        def up():
            t = self.host_tensor(name)
            if isinstance(t, QTensor):
                from .models._common import f32_of      # dequantised on the GPU
                return f32_of(self.weight(name))
            return torch.from_numpy(np.ascontiguousarray(np.asarray(t, dtype=np.float32))).to(self.device)
        return self._put(("f32", name), up)

    def weight(self, name: str):
        """Device form for a linear: a device QTensor for q8, else fp32."""
        t = self.host_tensor(name)
        if isinstance(t, QTensor):
            return self._put(("q8", name), lambda: t.to_device(self.device))
        return self.f32(name)

    def is_q8(self, name: str) -> bool:
        return isinstance(self.host_tensor(name), QTensor)

    def cache(self, key, fn):
        """Cache an arbitrary derived device tensor (fused or pre-split weights)."""
        return self._put(("derived",) + tuple(key if isinstance(key, tuple) else (key,)), fn)

    def evict(self, prefix: str = "", release: bool = True) -> int:
        """Drop every cached tensor whose name starts with ``prefix``; returns their bytes.

        With ``release`` the caching allocator's now-unused blocks go back to the driver
        (``cudaFree``), so another process or stage can use the HBM; callers must have
        dropped their own references to the stage (models, engines, CUDA graphs) first,
        as ``CosyVoice3CUDA._drop`` does."""
        freed = 0
        for k in list(self._cache):
            name = k[1] if len(k) > 1 and isinstance(k[1], str) else ""
            if name.startswith(prefix):
                v = self._cache.pop(k)
                freed += _nbytes(v)
        if release:
            release_device_memory()
        return freed


def release_device_memory() -> None:
    """Return the allocator's unused cached blocks to the driver (after collecting
    reference cycles that may still hold device tensors or graph memory pools)."""
    import gc
    import torch
    gc.collect()
    if torch.cuda.is_available() and torch.cuda.is_initialized():
        torch.cuda.synchronize()
        torch.cuda.empty_cache()


def _nbytes(v) -> int:
    if isinstance(v, QTensor):
        return v.nbytes
    if isinstance(v, (list, tuple)):
        return sum(_nbytes(x) for x in v)
    return int(getattr(v, "nbytes", 0) or (v.numel() * v.element_size() if hasattr(v, "numel") else 0))
