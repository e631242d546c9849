"""Helpers shared by the device stages: fused weight preparation and raw launches.

The stages call the C ABI with raw device pointers (Python ints) so that a
step's launch sequence is cheap to issue and can be captured once into a CUDA
graph.  Weights are prepared once per process and cached in
:class:`~..weights.DeviceWeights` (fused QKV / gate-up matrices, pre-split
operands), so the per-step work is launches only.
"""

from __future__ import annotations

import numpy as np
import torch

from .. import _dev as D
from .._lib import call
from ..quant import QTensor

torch = D.torch


TC_MIN_ROWS = 16   # below this many rows the fp32 GEMV/SIMT path is used


class Lin:
    """A linear layer's device operands: q8 (payload, scales) or fp32 matrix, and bias."""

    __slots__ = ("q8", "q4", "w", "scales", "n", "k", "kp", "bias", "_keep", "_lo")

    def __init__(self, w, bias=None):
        self._keep = [w, bias]
        if isinstance(w, QTensor):
            self.q8 = True            # quantised (q8, or q4 when self.q4)
            self.q4 = w.kind == "q4"
            self.w, self.scales = w.q.data_ptr(), w.scales.data_ptr()
            self.n, self.k, self.kp = int(w.shape[0]), int(w.shape[1]), w.padded_k
        else:
            self.q8 = self.q4 = False
            self.w, self.scales = w.data_ptr(), None
            self.n, self.k = int(w.shape[0]), int(w.shape[1])
            self.kp = self.k
        self.bias = bias.data_ptr() if bias is not None else None
        self._lo = None

    def lo(self, stream=None) -> int:
        """Device pointer to W - tf32(W), the remainder the 3xTF32 GEMM pairs with W
        (made on first use and kept; must first be called outside stream capture)."""
        if self._lo is None:
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError("Lin.lo(): the weight remainder must be made before stream capture")
            w = self._keep[0]
            lo = D.empty(tuple(w.shape))
            s = stream if stream is not None else D.stream()
            call("cv3_tf32_lo", self.w, self.n * self.k, lo.data_ptr(), s)
            self._lo = lo
        return self._lo.data_ptr()

    def __call__(self, x: int, m: int, y: int, residual: int = None, ldx: int = None, ldy: int = None,
                 stream=None):
        """y = x W^T + bias (+ residual).  fp32 weights with >= TC_MIN_ROWS rows of x run
        on the tensor cores (3xTF32); q8 weights stream through the GEMV kernel."""
        s = stream if stream is not None else D.stream()
        ldx = self.k if ldx is None else ldx
        ldy = self.n if ldy is None else ldy
        if self.q8:
            call("cv3_q4_linear" if self.q4 else "cv3_q8_linear", x, m, self.k, ldx, self.w, self.scales, self.n,
                 self.kp, self.bias, residual, y, ldy, s)
        elif m >= TC_MIN_ROWS and self.k % 4 == 0 and ldx % 4 == 0:
            if residual is not None and residual != y:
                raise ValueError("tensor-core linear adds the residual in place (residual must alias y)")
            call("cv3_tc_gemm_split", x, ldx, self.w, self.lo(s), self.k, y, ldy, m, self.n, self.k,
                 3 if residual is not None else 0, self.bias, None, 0, 0, s)
        else:
            call("cv3_f32_linear", x, m, self.k, ldx, self.w, self.n, self.k, self.bias, residual, y, ldy, s)

    def tc(self, x: int, m: int, y: int, mode: int, gate: int = None, rows_per_group: int = 0,
           gate_stride: int = 0, stream=None):
        """Tensor-core linear with a fused epilogue (0 bias, 1 GELU-tanh, 2 gated residual
        into y, 3 residual into y); fp32 weights only."""
        if self.q8:
            raise ValueError("fused tensor-core epilogues need fp32 weights")
        s = stream if stream is not None else D.stream()
        call("cv3_tc_gemm_split", x, self.k, self.w, self.lo(s), self.k, y, self.n, m, self.n, self.k, mode,
             self.bias, gate, rows_per_group, gate_stride, s)


class LinQ8:
    """A q8 linear on the tensor cores with the int8 weights as stored (``cv3_tc_gemm_q8``):
    the payload as exact fp16 and the scales transposed, made once; fewer than
    TC_MIN_ROWS rows of x take the q8 GEMV instead."""

    __slots__ = ("q", "n", "k", "w16", "st", "bias", "_keep")

    def __init__(self, w: QTensor, bias=None, stream=None):
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("LinQ8: weights must be prepared before stream capture")
        self.n, self.k = int(w.shape[0]), int(w.shape[1])
        if w.kind != "q8" or w.padded_k != self.k or self.k % 64 or self.n % 128:
            raise ValueError("LinQ8 needs a q8 matrix with K a multiple of 64 and N of 128")
        self.q = Lin(w, bias)
        self.w16 = torch.empty((self.n, self.k), dtype=torch.float16, device="cuda")
        self.st = D.empty((self.k // 64, self.n))
        call("cv3_q8_gemm_prepare", w.q.data_ptr(), w.scales.data_ptr(), self.n, self.k, self.w16.data_ptr(),
             self.st.data_ptr(), stream if stream is not None else D.stream())
        self.bias = bias.data_ptr() if bias is not None else None
        self._keep = [w, bias]

    def __call__(self, x: int, m: int, y: int, residual: int = None, ldx: int = None, ldy: int = None,
                 stream=None):
        ldx = self.k if ldx is None else ldx
        ldy = self.n if ldy is None else ldy
        if m < TC_MIN_ROWS or ldx % 4 or x % 16:
            return self.q(x, m, y, residual=residual, ldx=ldx, ldy=ldy, stream=stream)
        if residual is not None and residual != y:
            raise ValueError("tensor-core linear adds the residual in place (residual must alias y)")
        self.tc(x, m, y, 3 if residual is not None else 0, ldx=ldx, ldy=ldy, stream=stream)

    def tc_planes(self, planes: int, exps: int, lde: int, m: int, y: int, mode: int, gate: int = None,
                  rows_per_group: int = 0, gate_stride: int = 0, stream=None, out_planes: int = None,
                  out_exps: int = None, out_lde: int = 0):
        """cv3_tc_gemm_q8_planes: x given as activation planes; modes as tc, plus 4 (GELU-tanh
        written as activation planes to out_planes / out_exps)."""
        s = stream if stream is not None else D.stream()
        call("cv3_tc_gemm_q8_planes", planes, exps, lde, self.w16.data_ptr(), self.st.data_ptr(), y, self.n, m,
             self.n, self.k, mode, self.bias, gate, rows_per_group, gate_stride, out_planes, out_exps, out_lde, s)

    def tc(self, x: int, m: int, y: int, mode: int, gate: int = None, rows_per_group: int = 0,
           gate_stride: int = 0, stream=None, ldx: int = None, ldy: int = None):
        """Fused epilogue as Lin.tc: 0 bias, 1 GELU-tanh, 2 gated residual into y, 3 residual into y."""
        s = stream if stream is not None else D.stream()
        call("cv3_tc_gemm_q8", x, self.k if ldx is None else ldx, self.w16.data_ptr(), self.st.data_ptr(), y,
             self.n if ldy is None else ldy, m, self.n, self.k, mode, self.bias, gate, rows_per_group, gate_stride, s)


class ConvTC:
    """A conv1d weight in the tensor-core layout (``cv3_conv_weight_tc``): Wt[C_out][ci_pad/32][k][32]
    plus the tf32 remainder when the weight is not exactly tf32 (fp16-stored weights are)."""

    __slots__ = ("wt", "lo", "cout", "cin_g", "k", "groups", "ci_pad", "bias")

    def __init__(self, w, bias=None, groups: int = 1, stream=None):
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("ConvTC: weights must be rearranged before stream capture")
        self.cout, self.cin_g, self.k = (int(v) for v in w.shape)
        self.groups = int(groups)
        self.ci_pad = (self.cin_g + 31) // 32 * 32
        s = stream if stream is not None else D.stream()
        self.wt = D.empty((self.cout, self.ci_pad // 32, self.k, 32))
        lo = D.empty((self.cout, self.ci_pad // 32, self.k, 32))
        w = w.contiguous()
        call("cv3_conv_weight_tc", w.data_ptr(), self.cout, self.cin_g, self.k, self.ci_pad, self.wt.data_ptr(),
             lo.data_ptr(), s)
        self.lo = lo if bool(torch.count_nonzero(lo)) else None
        self.bias = bias

    def __call__(self, x, y, batch: int, t_in: int, t_out: int, stride: int = 1, dilation: int = 1,
                 pad_left: int = 0, residual=None, xs=None, ys=None, act: int = -1, act_param: float = 0.0,
                 snake_alpha=None, stream=None):
        """x, y device tensors (or pointers with explicit strides ``xs``/``ys`` = (s_b, s_c, s_t));
        default strides are channel-major [batch][C][T].  Epilogue: bias, ``act`` (CV3_ACT_*),
        snake with per-channel ``snake_alpha``, + ``residual``."""
        s = stream if stream is not None else D.stream()
        cin, cout = self.cin_g * self.groups, self.cout
        xs = xs if xs is not None else (cin * t_in, t_in, 1)
        ys = ys if ys is not None else (cout * t_out, t_out, 1)
        xp = x if isinstance(x, int) else x.data_ptr()
        yp = y if isinstance(y, int) else y.data_ptr()
        rp = residual if (residual is None or isinstance(residual, int)) else residual.data_ptr()
        call("cv3_conv1d_tc", xp, xs[0], xs[1], xs[2], batch, cin, t_in, self.wt.data_ptr(),
             self.lo.data_ptr() if self.lo is not None else None, self.ci_pad, cout, self.k, stride, dilation,
             self.groups, pad_left, self.bias.data_ptr() if self.bias is not None else None, int(act),
             float(act_param), snake_alpha.data_ptr() if snake_alpha is not None else None, rp, yp,
             ys[0], ys[1], ys[2], t_out, s)


class DecodeGemv:
    """A q8 weight streamed by ``cv3_q8_decode_gemv_mma`` for <= 32 activation rows
    (``cv3_q8_decode_gemv`` for <= 8 where the tensor-core kernel does not apply).

    Small matrices split K over several CTAs so every SM streams part of the
    weight; the split needs a private partial-sum workspace and per-row-tile
    counters (zero, and left zero by the kernel), allocated here once.
    ``norm_w`` fuses an RMSNorm of x; ``swiglu`` expects rows interleaved
    gate/up and writes ``silu(gate) * up``.
    """

    def __init__(self, w: QTensor, bias=None, norm_w=None, eps: float = 1e-6, swiglu: bool = False,
                 target_ctas: int = 296, mma_splits: int = 1):
        self._keep = [w, bias, norm_w]
        self.n, self.k, self.kp = int(w.shape[0]), int(w.shape[1]), w.padded_k
        self.q, self.scales = w.q.data_ptr(), w.scales.data_ptr()
        self.bias = bias.data_ptr() if bias is not None else None
        self.norm = norm_w.data_ptr() if norm_w is not None else None
        self.eps = float(eps)
        self.swiglu = 1 if swiglu else 0
        # the tensor-core kernel takes every unpadded K up to 5120 (all of Qwen2's linears);
        # mma_splits > 1 splits K over CTAs (with a fused RMSNorm only as one cluster of at
        # most 8, whose first CTA adds the others' sums of squares).
        # Measured in the batch-8 decode graph: the down projection (896 rows, K 4864) gains
        # from 2 splits (112 CTAs instead of 56), 4 splits and the out projection lose.
        self.mma = self.kp == self.k and self.k % 64 == 0 and self.k <= 5120
        if self.mma:
            groups = self.k // 64
            self.splits = max(1, min(int(mma_splits), groups, 8 if norm_w is not None else groups))
            gs = -(-groups // self.splits)
            eff = -(-groups // gs)
            # the kernel's row tiles: 32 rows for n >= 4096 with <= 16 scale groups per CTA, else 16
            tiles = -(-self.n // (32 if self.n >= 4096 and gs <= 16 else 16))
        else:
            tiles = -(-self.n // 32)
            self.splits = max(1, min(64, -(-target_ctas // tiles), self.kp // 64))
            kps = -(-(self.kp // self.splits) // 16) * 16
            eff = -(-self.kp // kps)
        self.ws = D.empty((eff * (32 if self.mma else 8) * self.n,)) if eff > 1 else None
        self.cnt = torch.zeros(tiles, dtype=torch.int32, device="cuda") if eff > 1 else None

    def __call__(self, x: int, m: int, y: int, residual: int = None, ldx: int = None, ldy: int = None,
                 stream=None):
        s = stream if stream is not None else D.stream()
        ldx = self.k if ldx is None else ldx
        ldy = (self.n // 2 if self.swiglu else self.n) if ldy is None else ldy
        if self.mma:
            if ldx % 4 or x % 16:
                raise ValueError("DecodeGemv: x must be 16-byte aligned rows")
            call("cv3_q8_decode_gemv_mma", x, m, self.k, ldx, self.q, self.scales, self.n, self.kp, self.bias,
                 residual, self.norm, self.eps, self.swiglu, y, ldy, self.splits,
                 self.ws.data_ptr() if self.ws is not None else None, self.ws.numel() if self.ws is not None else 0,
                 self.cnt.data_ptr() if self.cnt is not None else None, s)
            return
        call("cv3_q8_decode_gemv", x, m, self.k, ldx, self.q, self.scales, self.n, self.kp, self.bias, residual,
             self.norm, self.eps, self.swiglu, y, ldy, self.splits,
             self.ws.data_ptr() if self.ws is not None else None, self.ws.numel() if self.ws is not None else 0,
             self.cnt.data_ptr() if self.cnt is not None else None, s)


def interleave_rows(a: QTensor, b: QTensor) -> QTensor:
    """q8 rows a_0, b_0, a_1, b_1, ... (the SwiGLU pairing of cv3_q8_decode_gemv)."""
    n, kp = int(a.q.shape[0]), int(a.q.shape[1])
    q = torch.stack([a.q, b.q], dim=1).reshape(2 * n, kp).contiguous()
    s = torch.stack([a.scales, b.scales], dim=1).reshape(2 * n, -1).contiguous()
    return QTensor("q8", q, s, (2 * n, int(a.shape[1])), a.block, None)


def cat_rows(parts):
    """Stack weights along the output dimension (q8 payload + scales, or fp32)."""
    if all(isinstance(p, QTensor) for p in parts) and len({p.kind for p in parts}) == 1:
        k = parts[0].shape[1]
        q = torch.cat([p.q for p in parts], 0).contiguous()
        s = torch.cat([p.scales for p in parts], 0).contiguous()
        return QTensor(parts[0].kind, q, s, (int(q.shape[0]), k), parts[0].block, None)
    # mixed storage (small q8 and fp32 parts): stack fp32, dequantised exactly on the GPU
    return torch.cat([f32_of(p) for p in parts], 0).contiguous()


def f32_of(w):
    """fp32 device matrix of a device weight (q8 / q4 dequantised on the GPU, exactly)."""
    if isinstance(w, QTensor):
        n, k = int(w.shape[0]), int(w.shape[1])
        out = D.empty((n, k))
        call("cv3_q4_dequant" if w.kind == "q4" else "cv3_q8_dequant", w.q.data_ptr(), w.scales.data_ptr(), n,
             w.padded_k, k, out.data_ptr(), D.stream())
        return out
    return w


class Graph:
    """A captured launch sequence; counts its kernel nodes for the launch books."""

    def __init__(self):
        self.g = None
        self.nodes = 0

    def capture(self, fn) -> None:
        from .. import _lib
        start = _lib.launch_count()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=side):
            fn(D.stream())
        torch.cuda.current_stream().wait_stream(side)
        self.nodes = _lib.launch_count() - start
        _lib.note_capture(self.nodes)
        self.g = g

    def replay(self) -> None:
        from .. import _lib
        self.g.replay()
        _lib.note_replay(self.nodes)


def host_table(fn, *args):
    return torch.from_numpy(np.ascontiguousarray(fn(*args))).cuda()
