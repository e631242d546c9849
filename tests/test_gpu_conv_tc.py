"""Tensor-core conv1d (cv3_conv1d_tc) against the oracle's conv1d and activations.

The kernel is an implicit GEMM on tcgen05 with 3xTF32 products (two when the
weight is an exact tf32 value, as the vocoder's fp16-stored weights are).
Cases: the vocoder's resblock / upsample / source-down geometries (dilation,
stride, causal left pads), the DiT's grouped k=31 position conv in token-major
layout, input-channel counts that are not multiples of 32, short signals, and
each fused epilogue (activation, snake, residual in place).  Both kernels
run: the window kernel (stride 1 with a window of 128 + (k-1) dil <= 256
frames; A operands are shifted views of one staged window) and the gather kernel (forced with cv3_conv_tc_set_window(0),
and taken by itself otherwise); each case checks which kernel ran.  Bar: max |got - ref| / max |ref| <= 1e-5, the
fp32 bar; the error word must stay clear.
"""

import ctypes

import numpy as np
import pytest

from conftest import pkg, rel_err

import oracle.numerics as nx

pytestmark = pytest.mark.gpu

TOL = 1e-5


@pytest.fixture(params=[1, 0], ids=["window", "gather"])
def window(request):
    lib = pkg("_lib").load()
    lib.cv3_conv_tc_set_window(request.param)
    yield request.param
    lib.cv3_conv_tc_set_window(1)


def _last_path():
    p = ctypes.c_int(-9)
    pkg("_lib").load().cv3_conv_tc_last_path(ctypes.byref(p))
    return p.value


def _window_path(T, t_out, k, stride, dil, token_major, cin_g):
    """The kernel the host dispatch should pick with windows enabled (see cv3_conv1d_tc)."""
    frames = 128 + (k - 1) * dil
    if stride != 1:
        return 0
    if not token_major:
        return 1 if frames <= 256 else 0
    return 2 if frames <= 256 and cin_g % 4 == 0 else 0


def _conv_tc(x, w, bias, stride=1, dilation=1, groups=1, pad=(0, 0), act=-1, act_p=0.0, alpha=None,
             residual=None, token_major=False, fp16_weights=False, window=None):
    """Run the device conv on host arrays x (B, C_in, T); returns (B, C_out, T_out).
    With ``window`` given (the fixture's switch), checks the input path the launch took."""
    import torch
    common = pkg("models._common")
    B, cin, T = x.shape
    cout, cin_g, k = w.shape
    span = dilation * (k - 1) + 1
    t_out = (T + pad[0] + pad[1] - span) // stride + 1
    wd = torch.from_numpy(w).cuda()
    bd = torch.from_numpy(bias).cuda() if bias is not None else None
    cv = common.ConvTC(wd, bd, groups=groups)
    assert (cv.lo is None) == fp16_weights
    if token_major:
        xd = torch.from_numpy(np.ascontiguousarray(x.transpose(0, 2, 1))).cuda()
        xs = (T * cin, 1, cin)
        y = torch.from_numpy(np.ascontiguousarray(residual.transpose(0, 2, 1))).cuda() if residual is not None \
            else torch.full((B, t_out, cout), float("nan"), device="cuda")
        ys = (t_out * cout, 1, cout)
    else:
        xd = torch.from_numpy(x).cuda()
        xs = (cin * T, T, 1)
        y = torch.from_numpy(residual.copy()).cuda() if residual is not None \
            else torch.full((B, cout, t_out), float("nan"), device="cuda")
        ys = (cout * t_out, t_out, 1)
    ad = torch.from_numpy(alpha).cuda() if alpha is not None else None
    cv(xd, y, B, T, t_out, stride=stride, dilation=dilation, pad_left=pad[0],
       residual=y if residual is not None else None, xs=xs, ys=ys, act=act, act_param=act_p, snake_alpha=ad)
    torch.cuda.synchronize()
    if window is not None:
        want = _window_path(T, t_out, k, stride, dilation, token_major, cin_g) if window else 0
        assert _last_path() == want
    code = ctypes.c_int(-1)
    assert pkg("_lib").load().cv3_tc_conv_status(ctypes.byref(code)) == 0 and code.value == 0
    out = y.cpu().numpy()
    return out.transpose(0, 2, 1) if token_major else out


def _ref(x, w, bias, stride=1, dilation=1, groups=1, pad=(0, 0)):
    return np.stack([nx.conv1d(xb, w, bias, stride=stride, dilation=dilation, groups=groups, pad=pad) for xb in x])


def _data(rng, B, cin, T, cout, cin_g, k, fp16=False):
    x = rng.normal(size=(B, cin, T)).astype(np.float32)
    w = (rng.normal(size=(cout, cin_g, k)) / np.sqrt(cin_g * k)).astype(np.float32)
    if fp16:
        w = w.astype(np.float16).astype(np.float32)
    b = (rng.normal(size=cout) * 0.1).astype(np.float32)
    return x, w, b


@pytest.mark.parametrize("B,cin,T,cout,k,stride,dil,pad,fp16", [
    (2, 256, 300, 256, 7, 1, 3, (18, 0), True),     # resblock conv, dilated, causal pad
    (2, 128, 700, 128, 11, 1, 5, (50, 0), True),    # window: 178 frames, negative first coordinate
    (1, 64, 1000, 64, 3, 1, 1, (2, 0), True),       # BN = 64 tile
    (2, 80, 120, 512, 5, 1, 1, (0, 4), False),      # conv_pre: 80 channels (not a multiple of 32), right pad
    (2, 18, 601, 256, 14, 5, 1, (4, 0), True),      # strided source down-sampling (gather kernel)
    (1, 512, 50, 80, 7, 1, 1, (6, 0), False),       # few frames (odd row pitch), C_out not a tile multiple
    (3, 96, 129, 200, 1, 1, 1, (0, 0), False),      # 1x1, ragged frames and channels
    (2, 64, 1004, 64, 16, 1, 1, (15, 0), True),     # upsample conv (k = 16), last tile partial
    (1, 40, 200, 72, 3, 2, 1, (1, 0), False),       # stride 2 (gather kernel), 40 channels
    (2, 128, 64, 128, 11, 1, 5, (50, 0), True),     # one short tile
    (2, 64, 30001, 64, 11, 1, 5, (50, 0), True),    # vocoder's last stage: odd frame count, many tiles per CTA
    (1, 32, 500, 32, 3, 1, 65, (130, 0), True),     # window of 128 + 130 = 258 frames: gather kernel
    (1, 32, 500, 32, 3, 1, 64, (128, 0), True),     # 128 + 128 = 256 frames: the widest window
])
def test_conv_tc_channel_major(B, cin, T, cout, k, stride, dil, pad, fp16, window):
    rng = np.random.default_rng(cin * 7 + T)
    x, w, b = _data(rng, B, cin, T, cout, cin, k, fp16)
    got = _conv_tc(x, w, b, stride, dil, 1, pad, fp16_weights=fp16, window=window)
    assert rel_err(got, _ref(x, w, b, stride, dil, 1, pad)) < TOL


def test_conv_tc_grouped_token_major_position_conv(window):
    """The DiT's conv position embedding: 1024 channels, 16 groups, k = 31, causal pad,
    token-major (B, T, C) in and out, mish fused, residual added in place."""
    rng = np.random.default_rng(5)
    B, C, T, k, g = 2, 1024, 150, 31, 16
    x, w, b = _data(rng, B, C, T, C, C // g, k)
    h = rng.normal(size=(B, C, T)).astype(np.float32)
    got = _conv_tc(x, w, b, groups=g, pad=(k - 1, 0), act=4, residual=h, token_major=True, window=window)
    ref = h + nx.mish(_ref(x, w, b, groups=g, pad=(k - 1, 0)))
    assert rel_err(got, ref) < TOL


@pytest.mark.parametrize("B,C,T,k,g,act", [
    (1, 1024, 333, 31, 16, -1),   # three CTAs along time, no activation
    (3, 256, 40, 5, 4, 4),        # short signal, 64-channel groups
    (2, 96, 200, 3, 2, -1),       # 48-channel groups: the second channel block is partly masked
])
def test_conv_tc_token_major_shapes(B, C, T, k, g, act, window):
    rng = np.random.default_rng(T + k)
    x, w, b = _data(rng, B, C, T, C, C // g, k)
    got = _conv_tc(x, w, b, groups=g, pad=(k - 1, 0), act=act, token_major=True, window=window)
    ref = _ref(x, w, b, groups=g, pad=(k - 1, 0))
    assert rel_err(got, nx.mish(ref) if act == 4 else ref) < TOL


def test_conv_tc_grouped_channel_major(window):
    """Groups in channel-major layout: each group's window starts at its own channel."""
    rng = np.random.default_rng(21)
    x, w, b = _data(rng, 2, 96, 260, 64, 48, 5)
    got = _conv_tc(x, w, b, groups=2, pad=(4, 0), window=window)
    assert rel_err(got, _ref(x, w, b, groups=2, pad=(4, 0))) < TOL


@pytest.mark.parametrize("act,p,fn", [(4, 0.0, nx.mish), (5, 1.0, lambda v: nx.elu(v, 1.0)),
                                      (6, 0.1, lambda v: nx.leaky_relu(v, 0.1))])
def test_conv_tc_fused_activation(act, p, fn):
    rng = np.random.default_rng(act)
    x, w, b = _data(rng, 2, 128, 200, 128, 128, 5)
    got = _conv_tc(x, w, b, pad=(4, 0), act=act, act_p=p)
    assert rel_err(got, fn(_ref(x, w, b, pad=(4, 0)))) < TOL


def test_conv_tc_snake_and_residual():
    """resblock: x + conv2(snake(conv1(...))) with the snake after conv1 and the residual fused."""
    rng = np.random.default_rng(9)
    x, w, b = _data(rng, 2, 128, 333, 128, 128, 7, fp16=True)
    alpha = rng.uniform(0.2, 2.0, size=128).astype(np.float32)
    got = _conv_tc(x, w, b, dilation=3, pad=(18, 0), alpha=alpha, fp16_weights=True)
    ref = np.stack([nx.snake(r, alpha) for r in _ref(x, w, b, dilation=3, pad=(18, 0))])
    assert rel_err(got, ref) < TOL
    res = rng.normal(size=(2, 128, 333)).astype(np.float32)
    got = _conv_tc(x, w, b, pad=(6, 0), residual=res, fp16_weights=True)
    assert rel_err(got, res + _ref(x, w, b, pad=(6, 0))) < TOL


@pytest.mark.parametrize("cout", [64, 128])
def test_conv_tc_snake_large_arguments(cout):
    """Snake epilogue with alpha x beyond the branch-free sine's range (|alpha x| > 8192) in
    some chunks of a thread's channels and not in others: those chunks take CUDA's sinf."""
    rng = np.random.default_rng(cout)
    x, w, b = _data(rng, 2, cout, 500, cout, cout, 3, fp16=True)
    alpha = np.where(np.arange(cout) % 24 < 8, rng.uniform(3000, 9000, size=cout),
                     rng.uniform(0.2, 2.0, size=cout)).astype(np.float32)
    got = _conv_tc(x, w, b, dilation=3, pad=(6, 0), alpha=alpha, fp16_weights=True)
    pre = _ref(x, w, b, dilation=3, pad=(6, 0))
    assert (np.abs(alpha[None, :, None] * pre) > 8192).any()
    ref = np.stack([nx.snake(r, alpha) for r in pre])
    assert rel_err(got, ref) < TOL
