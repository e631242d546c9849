"""The cv3cpu kernel layer on B200: ``cv3cpu/ops.py``'s functions, same names and
signatures, executed by ``libcv3cuda.so``.

Every function accepts host NumPy arrays (and then returns NumPy, so existing
callers and the reference's tests work unchanged) or CUDA tensors (and then
returns CUDA tensors without leaving the device).  Argument checks raise the
reference's exception types: ``ValueError`` for GQA/shape mismatches and a
quantised conv without a kernel size, ``IndexError`` for embedding ids outside
the table.  There is no CPU path; without the library or a GPU they raise.

Constant tables (Hann window, linear-interpolation positions) are built on the
host in float64 exactly as the reference builds them, then used on the device.
"""

from __future__ import annotations

import math
from typing import Optional, Tuple, Union

import numpy as np

from . import _dev as D
from ._lib import call
from .quant import QTensor

torch = D.torch

Weight = Union[np.ndarray, QTensor, "torch.Tensor"]

TILE_BYTES = 8 << 20   # accepted for signature compatibility (cv3cpu/ops.py:23)

ACT = {"silu": 0, "sigmoid": 1, "gelu_tanh": 2, "gelu": 3, "mish": 4, "elu": 5,
       "leaky_relu": 6, "tanh": 7, "exp": 8}


def _unary(name: str, x, param: float = 0.0):
    host = D.is_host(x)
    xd = D.dev(x)
    y = D.empty_like(xd)
    call("cv3_unary", ACT[name], float(param), D.ptr(xd), xd.numel(), D.ptr(y), D.stream())
    return D.out(y, host)


def silu(x):                       # cv3cpu/ops.py:30
    return _unary("silu", x)


def sigmoid(x):                    # cv3cpu/ops.py:34
    return _unary("sigmoid", x)


def gelu_tanh(x):                  # cv3cpu/ops.py:41
    return _unary("gelu_tanh", x)


def gelu(x):                       # cv3cpu/ops.py:46
    return _unary("gelu", x)


def mish(x):                       # cv3cpu/ops.py:63
    return _unary("mish", x)


def elu(x, alpha: float = 1.0):    # cv3cpu/ops.py:69
    return _unary("elu", x, alpha)


def leaky_relu(x, slope: float = 0.01):   # cv3cpu/ops.py:73
    return _unary("leaky_relu", x, slope)


def snake(x, alpha, eps: float = 1e-9):
    """BigVGAN Snake over ``(C, T)``; cv3cpu/ops.py:77-81 (eps fixed at 1e-9)."""
    if eps != 1e-9:
        raise ValueError("the device snake is built for eps=1e-9")
    host = D.is_host(x)
    xd, ad = D.dev(x), D.dev(alpha).reshape(-1)
    c = xd.shape[0] if xd.dim() > 1 else 1
    if ad.numel() != c:
        raise ValueError(f"snake: {ad.numel()} alphas for {c} channels")
    y = D.empty_like(xd)
    call("cv3_snake", D.ptr(xd), D.ptr(ad), 1, c, xd.numel() // max(c, 1), D.ptr(y), D.stream())
    return D.out(y, host)


def _rows(x, axis):
    if axis not in (-1, x.dim() - 1):
        raise ValueError("the device reduction runs over the last axis")
    dim = x.shape[-1]
    return x.numel() // max(dim, 1), dim


def softmax(x, axis: int = -1):    # cv3cpu/ops.py:84
    host = D.is_host(x)
    xd = D.dev(x)
    rows, dim = _rows(xd, axis)
    y = D.empty_like(xd)
    call("cv3_softmax", D.ptr(xd), rows, dim, 0, D.ptr(y), D.stream())
    return D.out(y, host)


def log_softmax(x, axis: int = -1):   # cv3cpu/ops.py:90
    host = D.is_host(x)
    xd = D.dev(x)
    rows, dim = _rows(xd, axis)
    y = D.empty_like(xd)
    call("cv3_softmax", D.ptr(xd), rows, dim, 1, D.ptr(y), D.stream())
    return D.out(y, host)


def rms_norm(x, weight, eps: float = 1e-6):   # cv3cpu/ops.py:101
    host = D.is_host(x)
    xd, wd = D.dev(x), D.dev(weight)
    rows, dim = _rows(xd, -1)
    y = D.empty_like(xd)
    call("cv3_rms_norm", D.ptr(xd), D.ptr(wd), rows, dim, float(eps), D.ptr(y), D.stream())
    return D.out(y, host)


def layer_norm(x, weight=None, bias=None, eps: float = 1e-5):   # cv3cpu/ops.py:107
    host = D.is_host(x)
    xd = D.dev(x)
    wd = D.dev(weight) if weight is not None else None
    bd = D.dev(bias) if bias is not None else None
    rows, dim = _rows(xd, -1)
    y = D.empty_like(xd)
    call("cv3_layer_norm", D.ptr(xd), D.ptr(wd), D.ptr(bd), rows, dim, float(eps), D.ptr(y), D.stream())
    return D.out(y, host)


def _weight_dev(weight):
    """(kind, tensors...) for a linear weight: q8 / q4 device QTensor or fp32 matrix."""
    if isinstance(weight, QTensor):
        if weight.kind not in ("q8", "q4"):
            raise ValueError(f"quant kind {weight.kind!r} is not supported by the device build")
        return weight.to_device()
    return D.dev(weight)


def linear(x, weight: Weight, bias=None, residual=None, out=None):
    """``x @ weight.T + bias`` with ``weight`` ``(out, in)``; cv3cpu/ops.py:121-123.

    ``weight`` may be a q8 or q4 :class:`QTensor` (``cv3cpu/quant.py:156``) or a plain
    fp32/fp16 matrix.  ``residual`` (device extension) is added after the bias.
    """
    host = D.is_host(x)
    xd = D.dev(x)
    w = _weight_dev(weight)
    n, k = (int(w.shape[0]), int(w.shape[1]))
    if xd.shape[-1] != k:
        raise ValueError(f"linear: input has {xd.shape[-1]} features, weight expects {k}")
    lead = tuple(xd.shape[:-1])
    x2 = xd.reshape(-1, k)
    m = x2.shape[0]
    y = out if out is not None else D.empty(lead + (n,))
    bd = D.dev(bias).reshape(-1) if bias is not None else None
    rd = D.dev(residual) if residual is not None else None
    if isinstance(w, QTensor):
        call("cv3_q4_linear" if w.kind == "q4" else "cv3_q8_linear", D.ptr(x2), m, k, k, D.ptr(w.q),
             D.ptr(w.scales), n, w.padded_k, D.ptr(bd), D.ptr(rd), D.ptr(y), n, D.stream())
    elif m >= 16 and k % 4 == 0:
        # fp32 weights, enough rows: tensor cores (3xTF32, fp32-level accuracy)
        if rd is not None:
            y.copy_(rd.reshape(y.shape))
        call("cv3_tc_gemm", D.ptr(x2), k, D.ptr(w), k, D.ptr(y), n, m, n, k, 3 if rd is not None else 0,
             D.ptr(bd), None, 0, 0, D.stream())
    else:
        call("cv3_f32_linear", D.ptr(x2), m, k, k, D.ptr(w), n, k, D.ptr(bd), D.ptr(rd),
             D.ptr(y), n, D.stream())
    return D.out(y, host)


def _table_kind(table):
    if isinstance(table, QTensor):
        return 3 if table.kind == "q4" else 2
    t = table if D.is_device(table) else np.asarray(table)
    return 1 if D.is_half(t) else 0


def embedding(table: Weight, ids):
    """Row gather widened to fp32; IndexError outside the table; cv3cpu/ops.py:126-144."""
    host_ids = not D.is_device(ids)
    rows = int(table.shape[0])
    if host_ids:
        ids = np.asarray(ids)
        if ids.size and (int(ids.min()) < 0 or int(ids.max()) >= rows):
            raise IndexError(f"token id {int(ids.max())} is outside the {rows}-row embedding table")
    idd = D.dev(ids, D.I64).reshape(-1)
    kind = _table_kind(table)
    if kind >= 2:
        t = table.to_device()
        dim, kp = int(t.shape[1]), t.padded_k
        tab, sc = t.q, t.scales
    else:
        tab = D.dev(table, D.F16 if kind == 1 else D.F32)
        dim, kp, sc = int(tab.shape[1]), int(tab.shape[1]), None
    shape = tuple(ids.shape) if host_ids else tuple(ids.shape)
    y = D.empty((idd.numel(), dim))
    call("cv3_embedding", D.ptr(tab), kind, D.ptr(sc), rows, dim, kp, D.ptr(idd), idd.numel(),
         D.ptr(y), dim, None, D.stream())
    y = y.reshape(shape + (dim,))
    dev_table = D.is_device(table) or (isinstance(table, QTensor) and D.is_device(table.q))
    return D.out(y, host_ids and not dev_table)


def conv1d(x, weight: Weight, bias=None, stride: int = 1, dilation: int = 1, groups: int = 1,
           pad: Tuple[int, int] = (0, 0), kernel_size: Optional[int] = None,
           tile_bytes: int = TILE_BYTES):
    """``(C_in, T) -> (C_out, T_out)`` (or batched ``(B, C_in, T)``); cv3cpu/ops.py:165-219.

    A q8 weight is the folded ``(C_out, C_in/g * k)`` matrix and needs its kernel
    size (``kernel_size`` or the recorded original shape), as in the reference.
    """
    host = D.is_host(x)
    if isinstance(weight, QTensor):
        if weight.kind != "q8":
            raise ValueError(f"quantised conv weights of kind {weight.kind!r} are not supported")
        k = kernel_size or weight.kernel_size
        if k is None:
            raise ValueError("kernel_size is required for a quantised conv weight "
                             "that does not record its original 3-D shape")
        if groups != 1:
            raise ValueError("quantised grouped convs are not supported")
        wq = weight.to_device()
        cout, kk = int(wq.shape[0]), int(wq.shape[1])
        w = D.empty((cout, kk))
        call("cv3_q8_dequant", D.ptr(wq.q), D.ptr(wq.scales), cout, wq.padded_k, kk, D.ptr(w), D.stream())
        w = w.reshape(cout, kk // k, k)
    else:
        w = D.dev(weight)
    cout, cin_g, k = (int(s) for s in w.shape)
    xd = D.dev(x)
    batched = xd.dim() == 3
    xb = xd if batched else xd.unsqueeze(0)
    b, cin, t = (int(s) for s in xb.shape)
    if cin != cin_g * groups:
        raise ValueError(f"conv1d: input has {cin} channels, weight expects {cin_g} x {groups} groups")
    span = dilation * (k - 1) + 1
    t_out = (t + pad[0] + pad[1] - span) // stride + 1
    t_out = max(t_out, 0)
    y = D.empty((b, cout, t_out))
    bd = D.dev(bias).reshape(-1) if bias is not None else None
    if t_out:
        call("cv3_conv1d", D.ptr(xb), b, cin, t, D.ptr(w), cout, k, stride, dilation, groups,
             pad[0], pad[1], D.ptr(bd), D.ptr(y), t_out, D.stream())
    return D.out(y if batched else y[0], host)


def depthwise_conv1d(x, weight, bias=None, dilation: int = 1, pad=(0, 0)):
    """groups == C convolution; cv3cpu/ops.py:222-236."""
    w = D.dev(weight) if not D.is_host(weight) else np.asarray(weight, dtype=np.float32)
    if int(w.shape[1]) != 1:
        raise ValueError("depthwise weight must be (C, 1, k)")
    return conv1d(x, w, bias, dilation=dilation, groups=int(w.shape[0]), pad=pad)


def _mask_args(spec):
    if spec is None:
        return 0, 0, 0
    if spec[0] == "causal":
        return 1, int(spec[1]) if len(spec) > 1 else 0, 0
    if spec[0] == "chunk":
        return 2, int(spec[1]), int(spec[2])
    raise ValueError(f"unknown mask spec {spec}")


def sdpa(q, k, v, mask_spec=None, scale: Optional[float] = None, tile_bytes: int = TILE_BYTES):
    """Exact softmax attention over ``(H, N, D)``; GQA when k/v have fewer heads;
    cv3cpu/ops.py:267-300."""
    host = D.is_host(q)
    qd, kd, vd = D.dev(q), D.dev(k), D.dev(v)
    h, n, d = (int(s) for s in qd.shape)
    hk, m, _ = (int(s) for s in kd.shape)
    if hk != h and h % hk:
        raise ValueError(f"{h} query heads is not a multiple of {hk} kv heads")
    if scale is None:
        scale = 1.0 / math.sqrt(d)
    kind, a, b = _mask_args(mask_spec)
    o = D.empty((h, n, d))
    call("cv3_attention", D.ptr(qd), 0, n * d, d, D.ptr(kd), 0, m * d, d, D.ptr(vd), 0, m * d, d,
         D.ptr(o), 0, n * d, d, 1, h, hk, n, m, d, float(np.float32(scale)), kind, a, b, D.stream())
    return D.out(o, host)


def interpolate_nearest(x, scale: int):   # cv3cpu/ops.py:335-336
    host = D.is_host(x)
    xd = D.dev(x)
    t = int(xd.shape[-1])
    rows = xd.numel() // max(t, 1)
    y = D.empty(tuple(xd.shape[:-1]) + (t * scale,))
    call("cv3_interpolate_nearest", D.ptr(xd), rows, t, int(scale), D.ptr(y), D.stream())
    return D.out(y, host)


def interpolate_linear(x, size: int, align_corners: bool = False):   # cv3cpu/ops.py:318-332
    host = D.is_host(x)
    xd = D.dev(x)
    c, t = (int(s) for s in xd.shape)
    if t == size:
        return D.out(xd.clone(), host)
    if align_corners:
        pos = np.linspace(0.0, t - 1.0, size, dtype=np.float64)
    else:
        pos = np.clip((np.arange(size, dtype=np.float64) + 0.5) * (t / size) - 0.5, 0.0, t - 1.0)
    i0 = np.floor(pos).astype(np.int64)
    i1 = np.minimum(i0 + 1, t - 1)
    w = (pos - i0).astype(np.float32)
    y = D.empty((c, size))
    # keep every temporary alive until the launch is queued (a freed block could
    # otherwise be handed to the next temporary of the same call)
    i0d, i1d, wd = D.dev(i0, D.I64), D.dev(i1, D.I64), D.dev(w)
    call("cv3_interpolate_linear", D.ptr(xd), c, t, D.ptr(i0d), D.ptr(i1d), D.ptr(wd), size, D.ptr(y), D.stream())
    return D.out(y, host)


def hann_window(n: int, periodic: bool = True) -> np.ndarray:
    """Constant window table, float64 then float32; cv3cpu/ops.py:339-343."""
    denom = n if periodic else n - 1
    return (0.5 - 0.5 * np.cos(2.0 * np.pi * np.arange(n) / denom)).astype(np.float32)


def stft_stacked(x, n_fft: int, hop: int, win):
    """``(…, L) -> (…, n_fft+2, frames)``: real rows then imaginary rows (device)."""
    xd = D.dev(x)
    lead = tuple(xd.shape[:-1])
    L = int(xd.shape[-1])
    b = xd.numel() // max(L, 1)
    frames = 1 + L // hop
    nb = n_fft // 2 + 1
    out = D.empty(lead + (2 * nb, frames))
    wd = D.dev(win)
    call("cv3_stft", D.ptr(xd), b, L, n_fft, hop, D.ptr(wd), D.ptr(out), frames, D.stream())
    return out


def stft(x, n_fft: int, hop: int, win, center: bool = True, pad_mode: str = "reflect"):
    """``torch.stft`` (onesided, complex) for 1-D input; cv3cpu/ops.py:346-355."""
    if not center or pad_mode != "reflect":
        raise ValueError("the device stft is built for center=True, reflect padding")
    host = D.is_host(x)
    s = stft_stacked(x, n_fft, hop, win)
    nb = n_fft // 2 + 1
    if host:
        s = s.cpu().numpy()
        return (s[:nb] + 1j * s[nb:]).astype(np.complex64)
    if torch is None or not isinstance(s, torch.Tensor):
        raise TypeError("a complex device result needs PyTorch tensors: pass NumPy input (NumPy output) "
                        "or use stft_stacked")
    return torch.complex(s[:nb], s[nb:])


def istft_stacked(spec, n_fft: int, hop: int, win, mode: int = 0, limit: float = math.inf,
                  center: bool = True, length: Optional[int] = None):
    """Device iSTFT of a stacked ``(…, n_fft+2, frames)`` spectrum (mode 0: re/im,
    mode 1: the vocoder's log-magnitude/phase head)."""
    sd = D.dev(spec)
    lead = tuple(sd.shape[:-2])
    frames = int(sd.shape[-1])
    b = sd.numel() // max(frames * int(sd.shape[-2]), 1)
    total = (frames - 1) * hop + n_fft
    off = n_fft // 2 if center else 0
    n_out = total - 2 * off if center else total
    scratch = D.empty((b, frames, n_fft))
    y = D.empty(lead + (n_out,))
    wd = D.dev(win)
    call("cv3_istft", D.ptr(sd), mode, b, frames, n_fft, hop, D.ptr(wd), float(limit), off,
         D.ptr(scratch), D.ptr(y), n_out, D.stream())
    if length is not None and length != n_out:
        if torch is not None and isinstance(y, torch.Tensor):
            y = y[..., :length] if n_out >= length else torch.nn.functional.pad(y, (0, length - n_out))
        else:   # device arrays of the NumPy host: trimmed or padded on the host
            h = y.numpy()
            y = h[..., :length] if n_out >= length else np.pad(h, [(0, 0)] * (h.ndim - 1) + [(0, length - n_out)])
    return y


def istft(spec, n_fft: int, hop: int, win, center: bool = True, length: Optional[int] = None):
    """``torch.istft`` (onesided) for a ``(F, N)`` complex input; cv3cpu/ops.py:358-377."""
    host = D.is_host(spec)
    if host:
        spec = np.asarray(spec)
        stacked = np.concatenate([spec.real, spec.imag], axis=0).astype(np.float32)
    else:
        stacked = torch.cat([spec.real, spec.imag], dim=0).float()
    y = istft_stacked(stacked, n_fft, hop, win, 0, math.inf, center, length)
    return D.out(y, host)
