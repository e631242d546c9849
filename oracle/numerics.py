"""NumPy restatement of the reference kernel layer (test infrastructure only).

Covers ``cv3cpu/ops.py``, ``cv3cpu/quant.py`` (q8 path) and
``cv3cpu/torch_rng.py``.  The arithmetic, dtypes and order of floating-point
operations follow the reference line by line wherever that decides a rounding;
the loop structure, tiling and naming are this file's own.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional, Tuple

import numpy as np

F32 = np.float32

# ---------------------------------------------------------------------------
# q8 block quantisation                                  cv3cpu/quant.py:31-136
# ---------------------------------------------------------------------------

Q8_BLOCK = 64  # quant.py:31


@dataclass
class QTensor:
    """q8 weight: int8 ``q[N, Kp]``, float16 ``scales[N, Kp/64]``, logical ``shape``.

    Mirrors ``cv3cpu.quant.QTensor`` (quant.py:89-136).  Anything with the same
    attribute names is accepted by the functions below (duck typing), so the
    product package's weight objects can be handed in directly.
    """
    kind: str
    q: np.ndarray
    scales: np.ndarray
    shape: tuple
    block: int = Q8_BLOCK
    orig_shape: Optional[tuple] = None

    @property
    def kernel_size(self) -> Optional[int]:
        if self.orig_shape is not None and len(self.orig_shape) == 3:
            return int(self.orig_shape[2])
        return None


def is_quant(w) -> bool:
    return hasattr(w, "scales") and hasattr(w, "q")


def quantize_q8(w: np.ndarray, block: int = Q8_BLOCK):
    """Symmetric absmax/127 per (row, 64-wide K block); quant.py:56-67.

    Returns ``(int8 payload [N, Kp], float16 scales [N, Kp/block], Kp)``.  K is
    zero-padded up to a multiple of ``block``; an all-zero block gets scale 1.
    Rounding is NumPy's ``rint`` (half to even) before the clip to +-127.
    """
    w = np.ascontiguousarray(w, dtype=F32)
    rows, k = w.shape
    kp = -(-k // block) * block
    if kp != k:
        w = np.concatenate([w, np.zeros((rows, kp - k), F32)], axis=1)
    blk = w.reshape(rows, kp // block, block)
    scale = (np.abs(blk).max(axis=2) / 127.0).astype(F32)
    scale[scale == 0] = 1.0
    q = np.clip(np.rint(blk / scale[:, :, None]), -127, 127).astype(np.int8)
    return q.reshape(rows, kp), scale.astype(np.float16), kp


Q4_BLOCK = 32  # quant.py:32


def quantize_q4(w: np.ndarray, block: int = Q4_BLOCK):
    """llama.cpp-style Q4_0 per (row, 32-wide K block); quant.py:70-86.

    The block's largest-magnitude element (first on ties) fixes the scale
    ``s = ext / -8``, so it lands exactly on code 0; codes ``rint(w / s + 8)``
    clipped to [0, 15]; byte j of a block packs code j (low nibble) and code
    j + 16 (high nibble).  Returns ``(uint8 payload [N, Kp/2], float16 scales
    [N, Kp/block], Kp)``; an all-zero block gets scale 1.
    """
    w = np.ascontiguousarray(w, dtype=F32)
    rows, k = w.shape
    kp = -(-k // block) * block
    if kp != k:
        w = np.concatenate([w, np.zeros((rows, kp - k), F32)], axis=1)
    blk = w.reshape(rows, kp // block, block)
    pick = np.abs(blk).argmax(axis=2)
    ext = np.take_along_axis(blk, pick[:, :, None], axis=2)[:, :, 0]
    scale = (ext / -8.0).astype(F32)
    scale[scale == 0] = 1.0
    code = np.clip(np.rint(blk / scale[:, :, None] + 8.0), 0, 15).astype(np.uint8)
    half = block // 2
    packed = (code[:, :, :half] | (code[:, :, half:] << 4)).astype(np.uint8)
    return packed.reshape(rows, kp // 2), scale.astype(np.float16), kp


def dequant_rows(w, r0: int, r1: int) -> np.ndarray:
    """fp32 rows ``[r0, r1)`` of a q8 or q4 weight, padding sliced off; quant.py:110-133.

    q8: ``float32(q) * float32(scale)``; q4: ``(float32(code) - 8) * float32(scale)``,
    low nibbles first within each block.  Both are exact in fp32.
    """
    nb = w.scales.shape[1]
    blk = w.block
    rows = r1 - r0
    if getattr(w, "kind", "q8") == "q4":
        b = np.asarray(w.q[r0:r1]).reshape(rows, nb, blk // 2)
        wide = np.concatenate([(b & 0x0F).astype(F32) - F32(8.0), (b >> 4).astype(F32) - F32(8.0)], axis=2)
    else:
        wide = w.q[r0:r1].reshape(rows, nb, blk).astype(F32)
    wide *= w.scales[r0:r1].astype(F32)[:, :, None]
    return wide.reshape(rows, nb * blk)[:, : w.shape[1]]


def dequant(w) -> np.ndarray:
    return dequant_rows(w, 0, w.shape[0])


def qmatmul(x: np.ndarray, w, bias: Optional[np.ndarray] = None,
            tile_bytes: int = 1 << 20) -> np.ndarray:
    """``x @ W.T (+ bias)`` for a q8 or plain fp32 ``W`` of shape (N, K); quant.py:156-204.

    Plain weights go straight to one BLAS call (quant.py:165-170).  Quantised
    ones are widened one row tile at a time and multiplied tile by tile
    (quant.py:172-199); the result is independent of the tile size up to BLAS
    rounding.
    """
    if not is_quant(w):
        y = x.astype(F32, copy=False) @ np.asarray(w, dtype=F32).T
        if bias is not None:
            y += bias
        return y
    n, k = w.shape
    lead = x.shape[:-1]
    xf = np.ascontiguousarray(x, dtype=F32).reshape(-1, k)
    padded = w.scales.shape[1] * w.block
    step = max(1, min(n, tile_bytes // (padded * 4)))
    out = np.empty((n, xf.shape[0]), dtype=F32)
    for r0 in range(0, n, step):
        r1 = min(n, r0 + step)
        out[r0:r1] = dequant_rows(w, r0, r1) @ xf.T
    y = np.ascontiguousarray(out.T)
    if bias is not None:
        y += bias
    return y.reshape(*lead, n)


# ---------------------------------------------------------------------------
# elementwise                                              cv3cpu/ops.py:30-93
# ---------------------------------------------------------------------------

def silu(x):                                        # ops.py:30-31
    return x / (1.0 + np.exp(-x, dtype=F32))


def sigmoid(x):                                     # ops.py:34-35
    return 1.0 / (1.0 + np.exp(-x, dtype=F32))


_GELU_C = math.sqrt(2.0 / math.pi)


def gelu_tanh(x):                                   # ops.py:41-43
    return 0.5 * x * (1.0 + np.tanh(_GELU_C * (x + 0.044715 * x * x * x)))


def gelu(x):
    """Exact-erf GELU through Abramowitz & Stegun 7.1.26; ops.py:46-60."""
    z = x / math.sqrt(2.0)
    a = np.abs(z)
    t = 1.0 / (1.0 + 0.3275911 * a)
    poly = ((((1.061405429 * t - 1.453152027) * t) + 1.421413741) * t - 0.284496736) * t + 0.254829592
    erf = np.sign(z) * (1.0 - poly * t * np.exp(-a * a))
    return 0.5 * x * (1.0 + erf)


def mish(x):
    """x * tanh(softplus(x)), softplus guarded at 20; ops.py:63-66."""
    sp = np.where(x > 20.0, x, np.log1p(np.exp(np.minimum(x, 20.0))))
    return x * np.tanh(sp)


def elu(x, alpha: float = 1.0):                     # ops.py:69-70
    return np.where(x > 0, x, alpha * np.expm1(np.minimum(x, 0.0)))


def leaky_relu(x, slope: float = 0.01):             # ops.py:73-74
    return np.where(x >= 0, x, x * slope)


def snake(x, alpha, eps: float = 1e-9):
    """x + sin(a x)^2 / (a + eps) per channel of ``(C, T)``; ops.py:77-81."""
    a = np.asarray(alpha).reshape(-1, 1)
    s = np.sin(a * x)
    return x + (1.0 / (a + eps)) * (s * s)


def softmax(x, axis: int = -1):                     # ops.py:84-87
    e = np.exp(x - np.max(x, axis=axis, keepdims=True))
    return e / np.sum(e, axis=axis, keepdims=True)


def log_softmax(x, axis: int = -1):                 # ops.py:90-93
    z = x - np.max(x, axis=axis, keepdims=True)
    return z - np.log(np.sum(np.exp(z), axis=axis, keepdims=True))


# ---------------------------------------------------------------------------
# norms, linear, embedding                                ops.py:101-144
# ---------------------------------------------------------------------------

def rms_norm(x, weight, eps: float = 1e-6):         # ops.py:101-104
    x = x.astype(F32, copy=False)
    ms = np.mean(x * x, axis=-1, keepdims=True)
    return (x * (1.0 / np.sqrt(ms + eps))) * weight


def layer_norm(x, weight=None, bias=None, eps: float = 1e-5):   # ops.py:107-118
    x = x.astype(F32, copy=False)
    xc = x - np.mean(x, axis=-1, keepdims=True)
    y = xc / np.sqrt(np.mean(xc * xc, axis=-1, keepdims=True) + eps)
    if weight is not None:
        y = y * weight
    if bias is not None:
        y = y + bias
    return y


def linear(x, weight, bias=None):                   # ops.py:121-123
    return qmatmul(x, weight, bias)


def embedding(table, ids):
    """Row gather, widened to fp32, IndexError outside the table; ops.py:126-144."""
    ids = np.asarray(ids)
    rows = table.shape[0]
    if ids.size and (int(ids.min()) < 0 or int(ids.max()) >= rows):
        raise IndexError(f"token id {int(ids.max())} is outside the {rows}-row embedding table")
    if is_quant(table):
        flat = ids.reshape(-1)
        out = np.stack([dequant_rows(table, int(r), int(r) + 1)[0] for r in flat]) \
            if flat.size else np.zeros((0, table.shape[1]), F32)
        return out.reshape(*ids.shape, table.shape[1])
    return np.asarray(table[ids], dtype=F32)


# ---------------------------------------------------------------------------
# convolution                                               ops.py:152-236
# ---------------------------------------------------------------------------

def conv1d(x, weight, bias=None, stride: int = 1, dilation: int = 1, groups: int = 1,
           pad: Tuple[int, int] = (0, 0), kernel_size: Optional[int] = None,
           tile_frames: int = 4096):
    """``(C_in, T) -> (C_out, T_out)`` cross-correlation; ops.py:165-219.

    As in the reference, a plain weight and the input are cast to float32
    (ops.py:182, :190) -- so even a float64 caller computes in float32 -- and the
    product is an im2col matrix times the ``(C_out/g, C_in/g * k)`` weight.
    A q8 weight is a folded ``(C_out, C_in * k)`` matrix (groups must be 1).
    """
    if is_quant(weight):
        cout = weight.shape[0]
        k = kernel_size or weight.kernel_size
        if k is None:
            raise ValueError("kernel_size is required for a quantised conv weight "
                             "that does not record its original 3-D shape")
        cin_g = weight.shape[1] // k
        if groups != 1:
            raise ValueError("quantised grouped convs are not supported")
    else:
        weight = np.asarray(weight, dtype=F32)
        cout, cin_g, k = weight.shape
    if x.shape[0] != cin_g * groups:
        raise ValueError(f"conv1d: input has {x.shape[0]} channels, weight expects "
                         f"{cin_g} x {groups} groups")
    xp = np.pad(x, ((0, 0), pad)) if (pad[0] or pad[1]) else x
    xp = np.ascontiguousarray(xp, dtype=F32)
    span = dilation * (k - 1) + 1
    t_out = (xp.shape[1] - span) // stride + 1
    if t_out <= 0:
        return np.zeros((cout, 0), F32)
    out = np.empty((cout, t_out), F32)
    cout_g = cout // groups
    # time tiles sized like the reference's 8 MB im2col budget (ops.py:198-199)
    tile_frames = max(1, min(t_out, (8 << 20) // max(1, cin_g * k * 4)))
    for g in range(groups):
        xg = xp[g * cin_g:(g + 1) * cin_g]
        wg = weight if is_quant(weight) else \
            weight[g * cout_g:(g + 1) * cout_g].reshape(cout_g, cin_g * k)
        sc, stt = xg.strides
        for t0 in range(0, t_out, tile_frames):
            t1 = min(t_out, t0 + tile_frames)
            # column (c, j) of frame t reads xg[c, t*stride + j*dilation]: a strided view
            view = np.lib.stride_tricks.as_strided(xg[:, t0 * stride:], shape=(cin_g, k, t1 - t0),
                                                   strides=(sc, stt * dilation, stt * stride), writeable=False)
            cols = np.ascontiguousarray(view).reshape(cin_g * k, t1 - t0)
            if is_quant(wg):
                out[:, t0:t1] = qmatmul(cols.T, wg).T
            else:
                out[g * cout_g:(g + 1) * cout_g, t0:t1] = wg @ cols
    if bias is not None:
        out += np.asarray(bias, dtype=F32).reshape(-1, 1)
    return out


def depthwise_conv1d(x, weight, bias=None, dilation: int = 1, pad=(0, 0)):
    """groups == C convolution as k shifted multiply-adds; ops.py:222-236."""
    weight = np.asarray(weight, dtype=F32)
    c, one, k = weight.shape
    if one != 1:
        raise ValueError("depthwise weight must be (C, 1, k)")
    xp = np.pad(x, ((0, 0), pad)) if (pad[0] or pad[1]) else x
    t_out = xp.shape[1] - dilation * (k - 1)
    out = np.zeros((c, t_out), F32)
    for j in range(k):
        out += weight[:, 0, j:j + 1] * xp[:, j * dilation: j * dilation + t_out]
    if bias is not None:
        out += np.asarray(bias, dtype=F32).reshape(-1, 1)
    return out


# ---------------------------------------------------------------------------
# attention                                                 ops.py:244-310
# ---------------------------------------------------------------------------

def mask_block(q0, q1, k0, k1, spec):
    """Boolean allowed-mask for queries [q0,q1) x keys [k0,k1); ops.py:244-264."""
    if spec is None:
        return None
    qi = np.arange(q0, q1)[:, None]
    ki = np.arange(k0, k1)[None, :]
    if spec[0] == "causal":
        return ki <= qi + (spec[1] if len(spec) > 1 else 0)
    if spec[0] == "chunk":
        size, left = spec[1], spec[2]
        end = (qi // size + 1) * size
        start = np.zeros_like(qi) if left < 0 else np.maximum((qi // size - left) * size, 0)
        return (ki < end) & (ki >= start)
    raise ValueError(f"unknown mask spec {spec}")


def sdpa(q, k, v, mask_spec=None, scale=None, tile_q: int = 256):
    """Exact softmax attention over ``(H, N, D)``, GQA by head repeat; ops.py:267-300."""
    h, n, d = q.shape
    hk, m, _ = k.shape
    if hk != h:
        if h % hk:
            raise ValueError(f"{h} query heads is not a multiple of {hk} kv heads")
        k = np.repeat(k, h // hk, axis=0)
        v = np.repeat(v, h // hk, axis=0)
    if scale is None:
        scale = 1.0 / math.sqrt(d)
    kt = np.ascontiguousarray(np.swapaxes(k, 1, 2))
    out = np.empty((h, n, d), F32)
    for q0 in range(0, n, tile_q):
        q1 = min(n, q0 + tile_q)
        s = (q[:, q0:q1] * F32(scale)) @ kt
        allowed = mask_block(q0, q1, 0, m, mask_spec)
        if allowed is not None:
            add = np.zeros((1, q1 - q0, m), F32)
            add[0][~allowed] = -np.inf
            s += add
        s -= s.max(axis=-1, keepdims=True)
        np.exp(s, out=s)
        s /= s.sum(axis=-1, keepdims=True)
        out[:, q0:q1] = s @ v
    return out


# ---------------------------------------------------------------------------
# resampling and short-time Fourier transforms               ops.py:318-377
# ---------------------------------------------------------------------------

def interpolate_nearest(x, scale: int):             # ops.py:335-336
    return np.repeat(x, scale, axis=-1)


def interpolate_linear(x, size: int, align_corners: bool = False):   # ops.py:318-332
    c, t = x.shape
    if t == size:
        return x.astype(F32, copy=True)
    if align_corners:
        pos = np.linspace(0.0, t - 1.0, size, dtype=np.float64)
    else:
        pos = np.clip((np.arange(size, dtype=np.float64) + 0.5) * (t / size) - 0.5, 0.0, t - 1.0)
    i0 = np.floor(pos).astype(np.int64)
    i1 = np.minimum(i0 + 1, t - 1)
    w = (pos - i0).astype(F32)
    return x[:, i0] * (1.0 - w) + x[:, i1] * w


def hann_window(n: int, periodic: bool = True):     # ops.py:339-343
    denom = n if periodic else n - 1
    return (0.5 - 0.5 * np.cos(2.0 * np.pi * np.arange(n) / denom)).astype(F32)


def stft(x, n_fft: int, hop: int, win, center: bool = True):
    """Onesided complex STFT ``(n_fft/2+1, frames)`` with reflect padding; ops.py:346-355."""
    x = np.asarray(x, dtype=F32)
    if center:
        x = np.pad(x, (n_fft // 2, n_fft // 2), mode="reflect")
    frames = 1 + (len(x) - n_fft) // hop
    idx = np.arange(frames)[:, None] * hop + np.arange(n_fft)[None, :]
    return np.fft.rfft(x[idx] * win, n=n_fft, axis=1).T


def istft(spec, n_fft: int, hop: int, win, center: bool = True, length=None):
    """Inverse of :func:`stft` with window-square normalisation; ops.py:358-377."""
    frames = np.fft.irfft(spec, n=n_fft, axis=0).astype(F32) * win[:, None]
    n = frames.shape[1]
    total = (n - 1) * hop + n_fft
    y = np.zeros(total, F32)
    env = np.zeros(total, F32)
    w2 = (win * win).astype(F32)
    for j in range(n_fft):
        y[j: j + (n - 1) * hop + 1: hop] += frames[j]
        env[j: j + (n - 1) * hop + 1: hop] += w2[j]
    nz = np.abs(env) > 1e-11
    y[nz] /= env[nz]
    if center:
        y = y[n_fft // 2: total - n_fft // 2]
    if length is not None:
        y = y[:length] if len(y) >= length else np.pad(y, (0, length - len(y)))
    return y


# ---------------------------------------------------------------------------
# PyTorch's CPU generator                               cv3cpu/torch_rng.py
# ---------------------------------------------------------------------------

_MT_N, _MT_M = 624, 397
_MT_A = np.uint32(0x9908B0DF)
_HI = np.uint32(0x80000000)
_LO = np.uint32(0x7FFFFFFF)


class MT19937:
    """MT19937 seeded with ``init_genrand`` plus torch's output conventions.

    Follows torch_rng.py:27-102: seeding (:30-37), the state twist (:39-69),
    tempering (:81-86), float32 uniforms from the low 24 bits (:88-91) and
    float64 uniforms from two words, first word high (:93-102).
    """

    def __init__(self, seed: int = 0):
        st = [seed & 0xFFFFFFFF]
        for i in range(1, _MT_N):
            p = st[-1]
            st.append((1812433253 * (p ^ (p >> 30)) + i) & 0xFFFFFFFF)
        self.state = np.array(st, dtype=np.uint32)
        self.pos = _MT_N

    def _regenerate(self) -> None:
        old = self.state
        new = np.empty_like(old)
        # word i mixes old[i] (top bit), old[i+1] (low 31 bits) and word i+397,
        # which is old for i < 227 and already-regenerated for i >= 227.
        def mix(lo, hi, far):
            y = (old[lo:hi] & _HI) | (old[lo + 1:hi + 1] & _LO)
            new[lo:hi] = far ^ (y >> np.uint32(1)) ^ np.where(y & np.uint32(1), _MT_A, np.uint32(0))
        lag = _MT_N - _MT_M                      # 227
        mix(0, lag, old[_MT_M:_MT_N])
        for lo in range(lag, _MT_N - 1, lag):
            hi = min(lo + lag, _MT_N - 1)
            mix(lo, hi, new[lo - lag:hi - lag])
        y = (int(old[-1]) & 0x80000000) | (int(new[0]) & 0x7FFFFFFF)
        v = int(new[_MT_M - 1]) ^ (y >> 1) ^ (0x9908B0DF if y & 1 else 0)
        new[-1] = v & 0xFFFFFFFF
        self.state = new
        self.pos = 0

    def raw(self, n: int) -> np.ndarray:
        """``n`` untempered state words, regenerating as needed."""
        out = np.empty(n, dtype=np.uint32)
        done = 0
        while done < n:
            if self.pos >= _MT_N:
                self._regenerate()
            take = min(n - done, _MT_N - self.pos)
            out[done:done + take] = self.state[self.pos:self.pos + take]
            self.pos += take
            done += take
        return out

    def next_u32(self, n: int) -> np.ndarray:
        y = self.raw(n)
        y ^= y >> np.uint32(11)
        y ^= (y << np.uint32(7)) & np.uint32(0x9D2C5680)
        y ^= (y << np.uint32(15)) & np.uint32(0xEFC60000)
        y ^= y >> np.uint32(18)
        return y

    def random_float32(self, n: int) -> np.ndarray:
        return (self.next_u32(n) & np.uint32(0xFFFFFF)).astype(F32) * F32(1.0 / (1 << 24))

    def random_float64(self, n: int) -> np.ndarray:
        w = self.next_u32(2 * n).astype(np.uint64)
        v = ((w[0::2] << np.uint64(32)) | w[1::2]) & np.uint64((1 << 53) - 1)
        return v.astype(np.float64) * (1.0 / (1 << 53))


def box_muller16(u: np.ndarray) -> np.ndarray:
    """torch ``normal_fill_16``: element j pairs with j+8, math in float64; torch_rng.py:105-114."""
    d = u.astype(np.float64)
    r = np.sqrt(-2.0 * np.log(1.0 - d[..., :8]))
    th = 2.0 * np.pi * d[..., 8:]
    return np.concatenate([r * np.cos(th), r * np.sin(th)], axis=-1).astype(F32)


def randn(shape, seed: int = 0, gen: Optional[MT19937] = None) -> np.ndarray:
    """``torch.manual_seed(seed); torch.randn(shape)`` on CPU; torch_rng.py:117-142."""
    shape = (shape,) if isinstance(shape, int) else tuple(shape)
    n = int(np.prod(shape)) if shape else 1
    g = gen if gen is not None else MT19937(seed)
    if n < 16:
        # scalar normal_distribution<double>: theta from the first double
        # uniform of a pair, radius from the second (torch_rng.py:122-133)
        pairs = (n + 1) // 2
        u = g.random_float64(2 * pairs).reshape(pairs, 2)
        th = 2.0 * np.pi * u[:, 0]
        r = np.sqrt(-2.0 * np.log1p(-u[:, 1]))
        out = np.empty(2 * pairs, F32)
        out[0::2] = (r * np.cos(th)).astype(F32)
        out[1::2] = (r * np.sin(th)).astype(F32)
        return out[:n].reshape(shape)
    u = g.random_float32(n)
    out = np.empty(n, F32)
    whole = n - n % 16
    out[:whole] = box_muller16(u[:whole].reshape(-1, 16)).reshape(-1)
    if n % 16:
        # the last 16 outputs are redrawn from 16 fresh uniforms (torch_rng.py:138-141)
        out[n - 16:] = box_muller16(g.random_float32(16).reshape(1, 16)).reshape(-1)
    return out.reshape(shape)


def rand(shape, seed: int = 0, gen: Optional[MT19937] = None) -> np.ndarray:
    """``torch.manual_seed(seed); torch.rand(shape)``; torch_rng.py:145-150."""
    shape = (shape,) if isinstance(shape, int) else tuple(shape)
    n = int(np.prod(shape)) if shape else 1
    g = gen if gen is not None else MT19937(seed)
    return g.random_float32(n).reshape(shape)


# ---------------------------------------------------------------------------
# speech-token sampling                       cv3cpu/models/llm.py:37-49, :125-149
# ---------------------------------------------------------------------------

def nucleus_sampling(probs_sorted, idx_sorted, rng, top_p: float, top_k: int) -> int:   # llm.py:37-49
    cum, n = 0.0, 0
    for i in range(min(top_k, idx_sorted.shape[0])):
        if cum >= top_p:
            break
        cum += float(probs_sorted[i])
        n += 1
    p = probs_sorted[:n].astype(np.float64)
    p = p / p.sum()
    return int(idx_sorted[rng.choice(n, p=p)])


def sample_token(logp, decoded, rng, speech_token_size: int, ignore_eos: bool, strict_min_len: bool,
                 top_p: float = 0.8, top_k: int = 25, win_size: int = 10, tau_r: float = 0.1) -> int:
    """One step of CosyVoice3LM._sample (llm.py:125-149): stop ids masked below min_len,
    nucleus draw from softmax(scores), repetition-aware resample from the full distribution."""
    scores = np.array(logp, dtype=np.float32, copy=True)
    if ignore_eos:
        if strict_min_len:
            scores[speech_token_size:speech_token_size + 200] = -np.inf
        else:
            scores[speech_token_size] = -np.inf
    probs = softmax(scores)
    order = np.argsort(-probs, kind="stable")
    top = nucleus_sampling(probs[order], order, rng, top_p, top_k)
    window = list(decoded)[-win_size:]
    if sum(1 for t in window if t == top) >= win_size * tau_r:
        scores[top] = -np.inf
        p = softmax(scores).astype(np.float64)
        p /= p.sum()
        top = int(rng.choice(p.shape[0], p=p))
    return top
