"""The tcgen05 3xTF32 GEMM against fp64 products of the same fp32 inputs.

Bar: max |got - ref| / max |ref| <= 1e-5 (measured 1.7e-6 at K=1024 and
3.1e-6 at K=2048 with the default accumulator layout; NumPy's fp32 BLAS is
~6e-7 on the same inputs).  Cases grow from one 128x128 tile to
the DiT's shapes, with row/column tails, K tails and every epilogue.  After
each case the kernel's error word (bounded-wait expiry) must be clear.

Both entry points run every case: cv3_tc_gemm (B split in the kernel) and
cv3_tc_gemm_split (B with its cv3_tf32_lo remainder; persistent tiles, four
accumulators, each tile's epilogue overlapped with the next tile's MMAs).
"""

import ctypes

import numpy as np
import pytest

from conftest import pkg, rel_err

pytestmark = pytest.mark.gpu


KINDS = ["in_kernel_split", "presplit_b"]


def _run(a, b, mode=0, bias=None, gate=None, c0=None, rows_per_group=0, kind="in_kernel_split"):
    import torch
    L = pkg("_lib")
    ad, bd = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
    m, k = a.shape
    n = b.shape[0]
    c = torch.from_numpy(c0.copy()).cuda() if c0 is not None else torch.zeros(m, n, device="cuda")
    bb = torch.from_numpy(bias).cuda() if bias is not None else None
    gg = torch.from_numpy(gate).cuda() if gate is not None else None
    st = torch.cuda.current_stream().cuda_stream
    bias_p = bb.data_ptr() if bb is not None else None
    gate_p = gg.data_ptr() if gg is not None else None
    if kind == "in_kernel_split":
        L.call("cv3_tc_gemm", ad.data_ptr(), k, bd.data_ptr(), k, c.data_ptr(), n, m, n, k, mode,
               bias_p, gate_p, rows_per_group, n if gate is not None else 0, st)
    else:
        lo = torch.empty_like(bd)
        L.call("cv3_tf32_lo", bd.data_ptr(), n * k, lo.data_ptr(), st)
        L.call("cv3_tc_gemm_split", ad.data_ptr(), k, bd.data_ptr(), lo.data_ptr(), k, c.data_ptr(), n, m, n, k,
               mode, bias_p, gate_p, rows_per_group, n if gate is not None else 0, st)
    torch.cuda.synchronize()
    code = ctypes.c_int()
    L.call("cv3_tc_gemm_status", ctypes.byref(code))
    assert code.value == 0, f"bounded wait expired (code {code.value})"
    return c.cpu().numpy()


def _gelu(x):
    return 0.5 * x * (1.0 + np.tanh(np.sqrt(2.0 / np.pi) * (x + 0.044715 * x ** 3)))


@pytest.mark.parametrize("m,n,k", [(128, 128, 32), (128, 128, 64), (256, 256, 256), (37, 100, 68),
                                   (1000, 1024, 1024), (10400, 3072, 1024), (10400, 1024, 320),
                                   (1000, 1024, 2048), (130, 80, 1024), (300, 200, 4)])
@pytest.mark.parametrize("kind", KINDS)
def test_plain_gemm(m, n, k, kind):
    rng = np.random.default_rng(m + n + k)
    a = rng.normal(size=(m, k)).astype(np.float32)
    b = (rng.normal(size=(n, k)) * 0.02).astype(np.float32)
    ref = a.astype(np.float64) @ b.astype(np.float64).T
    assert rel_err(_run(a, b, kind=kind), ref) < 1e-5


def test_tf32_lo_is_the_exact_remainder():
    import torch
    rng = np.random.default_rng(3)
    x = np.concatenate([rng.normal(size=5000), [0.0, -0.0, 1e-38, -3e38, 1.0, -1.0]]).astype(np.float32)
    xd = torch.from_numpy(x).cuda()
    lo = torch.empty_like(xd)
    pkg("_lib").call("cv3_tf32_lo", xd.data_ptr(), x.size, lo.data_ptr(), torch.cuda.current_stream().cuda_stream)
    hi = (x.view(np.uint32) & np.uint32(0xFFFFE000)).view(np.float32)
    assert np.array_equal(lo.cpu().numpy().view(np.uint32), (x - hi).view(np.uint32))


def test_presplit_strided_operands():
    """A with lda > k and C with ldc > n (column slices of wider buffers)."""
    import torch
    L = pkg("_lib")
    rng = np.random.default_rng(11)
    m, n, k, lda, ldc = 333, 200, 512, 600, 260
    abuf = rng.normal(size=(m, lda)).astype(np.float32)
    b = (rng.normal(size=(n, k)) * 0.05).astype(np.float32)
    ad, bd = torch.from_numpy(abuf).cuda(), torch.from_numpy(b).cuda()
    cd = torch.full((m, ldc), 7.0, device="cuda")
    lo = torch.empty_like(bd)
    st = torch.cuda.current_stream().cuda_stream
    L.call("cv3_tf32_lo", bd.data_ptr(), n * k, lo.data_ptr(), st)
    L.call("cv3_tc_gemm_split", ad.data_ptr(), lda, bd.data_ptr(), lo.data_ptr(), k, cd.data_ptr(), ldc, m, n, k,
           0, None, None, 0, 0, st)
    torch.cuda.synchronize()
    got = cd.cpu().numpy()
    ref = abuf[:, :k].astype(np.float64) @ b.astype(np.float64).T
    assert rel_err(got[:, :n], ref) < 1e-5
    assert np.all(got[:, n:] == 7.0)


@pytest.mark.parametrize("kind", KINDS)
def test_epilogues(kind):
    rng = np.random.default_rng(7)
    m, n, k = 650, 2048, 1024
    a = rng.normal(size=(m, k)).astype(np.float32)
    b = (rng.normal(size=(n, k)) * 0.02).astype(np.float32)
    bias = rng.normal(size=n).astype(np.float32)
    y = a.astype(np.float64) @ b.astype(np.float64).T + bias
    assert rel_err(_run(a, b, 0, bias, kind=kind), y) < 1e-5
    assert rel_err(_run(a, b, 1, bias, kind=kind), _gelu(y)) < 1e-5
    h = rng.normal(size=(m, n)).astype(np.float32)
    gate = rng.normal(size=(2, n)).astype(np.float32)
    rows = 325
    ref = h + np.repeat(gate, rows, axis=0) * y
    assert rel_err(_run(a, b, 2, bias, gate, h, rows_per_group=rows, kind=kind), ref) < 1e-5
    assert rel_err(_run(a, b, 3, bias, None, h, kind=kind), h + y) < 1e-5


# ---------------------------------------------------------------------------
# cv3_tc_gemm_q8: the int8 weights as stored (balanced DiT), against fp64 of A . (q * s)^T
# ---------------------------------------------------------------------------

def _run_q8(a, w, mode=0, bias=None, gate=None, c0=None, rows_per_group=0):
    import torch
    L = pkg("_lib")
    qt = pkg("quant").make_qtensor(w)
    n, k = w.shape
    m = a.shape[0]
    qd, sd = torch.from_numpy(qt.q).cuda(), torch.from_numpy(qt.scales.view(np.uint16)).cuda()
    w16 = torch.empty((n, k), dtype=torch.float16, device="cuda")
    stt = torch.empty((k // 64, n), dtype=torch.float32, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    L.call("cv3_q8_gemm_prepare", qd.data_ptr(), sd.data_ptr(), n, k, w16.data_ptr(), stt.data_ptr(), st)
    ad = torch.from_numpy(a).cuda()
    c = torch.from_numpy(c0.copy()).cuda() if c0 is not None else torch.zeros(m, n, device="cuda")
    bb = torch.from_numpy(bias).cuda() if bias is not None else None
    gg = torch.from_numpy(gate).cuda() if gate is not None else None
    L.call("cv3_tc_gemm_q8", ad.data_ptr(), k, w16.data_ptr(), stt.data_ptr(), c.data_ptr(), n, m, n, k, mode,
           bb.data_ptr() if bb is not None else None, gg.data_ptr() if gg is not None else None, rows_per_group,
           n if gate is not None else 0, st)
    torch.cuda.synchronize()
    code = ctypes.c_int()
    L.call("cv3_tc_gemm_q8_status", ctypes.byref(code))
    assert code.value == 0, f"bounded wait expired (code {code.value})"
    wd = qt.q.astype(np.float64) * np.repeat(qt.scales.astype(np.float64), 64, axis=1)[:, :k]
    return c.cpu().numpy(), wd


@pytest.mark.parametrize("m,n,k", [(128, 128, 64), (37, 128, 128), (300, 256, 1024), (1000, 1024, 2048),
                                   (10400, 2048, 1024), (1300, 3072, 1024)])
def test_q8_gemm_matches_fp64(m, n, k):
    rng = np.random.default_rng(m + n + k)
    a = rng.normal(size=(m, k)).astype(np.float32)
    a[: m // 3] *= 40.0   # rows of different magnitudes (per-row, per-group scaling)
    a[:, : k // 4] *= 1e-3
    w = (rng.normal(size=(n, k)) * 0.02).astype(np.float32)
    got, wd = _run_q8(a, w)
    ref = a.astype(np.float64) @ wd.T
    assert rel_err(got, ref) < 1e-5


@pytest.mark.parametrize("mode", [0, 1, 2, 3])
def test_q8_gemm_epilogues(mode):
    rng = np.random.default_rng(7 + mode)
    m, n, k = 650, 1024, 1024
    a = rng.normal(size=(m, k)).astype(np.float32)
    w = (rng.normal(size=(n, k)) * 0.03).astype(np.float32)
    bias = rng.normal(size=n).astype(np.float32)
    gate = rng.normal(size=(3, n)).astype(np.float32) if mode == 2 else None
    c0 = rng.normal(size=(m, n)).astype(np.float32) if mode >= 2 else None
    got, wd = _run_q8(a, w, mode, bias, gate, c0, rows_per_group=256 if mode == 2 else 0)
    y = a.astype(np.float64) @ wd.T + bias
    if mode == 1:
        y = _gelu(y)
    elif mode == 2:
        y = c0 + gate[np.arange(m) // 256] * y
    elif mode == 3:
        y = c0 + y
    assert rel_err(got, y) < 1e-5


# ---------------------------------------------------------------------------
# activation planes: split, the planes GEMM, GELU written as planes, LN as planes
# ---------------------------------------------------------------------------

def _planes_of(x):
    """Device activation planes of a host fp32 matrix (cv3_q8_split_rows)."""
    import torch
    L = pkg("_lib")
    m, k = x.shape
    lde = -(-m // 16) * 16
    xd = torch.from_numpy(x).cuda()
    pl = torch.empty((m, 2 * k), dtype=torch.float16, device="cuda")
    ex = torch.empty((k // 64, lde), dtype=torch.int8, device="cuda")
    L.call("cv3_q8_split_rows", xd.data_ptr(), k, m, k, pl.data_ptr(), ex.data_ptr(), lde,
           torch.cuda.current_stream().cuda_stream)
    return pl, ex, lde


def _unplanes(pl, ex, m, k):
    """fp64 values the planes carry: (hi + lo) * 2^-e."""
    p = pl.cpu().numpy().astype(np.float64).reshape(m, k // 64, 2, 64)
    e = ex.cpu().numpy()[:, :m].astype(np.float64).T          # [m][k/64]
    return ((p[:, :, 0] + p[:, :, 1]) * np.exp2(-e)[:, :, None]).reshape(m, k)


def _w16(w):
    import torch
    L = pkg("_lib")
    qt = pkg("quant").make_qtensor(w)
    n, k = w.shape
    qd, sd = torch.from_numpy(qt.q).cuda(), torch.from_numpy(qt.scales.view(np.uint16)).cuda()
    w16 = torch.empty((n, k), dtype=torch.float16, device="cuda")
    stt = torch.empty((k // 64, n), dtype=torch.float32, device="cuda")
    L.call("cv3_q8_gemm_prepare", qd.data_ptr(), sd.data_ptr(), n, k, w16.data_ptr(), stt.data_ptr(),
           torch.cuda.current_stream().cuda_stream)
    wd = qt.q.astype(np.float64) * np.repeat(qt.scales.astype(np.float64), 64, axis=1)[:, :k]
    return w16, stt, wd


def test_split_rows_carries_22_bits():
    import torch
    rng = np.random.default_rng(1)
    x = (rng.normal(size=(37, 256)) * np.exp(rng.normal(size=(37, 1)) * 4)).astype(np.float32)
    x[3, :64] = 0.0
    pl, ex, lde = _planes_of(x)
    torch.cuda.synchronize()
    back = _unplanes(pl, ex, 37, 256)
    assert np.all(np.abs(back - x) <= np.abs(x) * 2.0 ** -21 + 1e-30)


@pytest.mark.parametrize("m,n,k,mode", [(300, 256, 1024, 0), (10400, 2048, 1024, 0), (650, 1024, 2048, 2),
                                        (650, 1024, 1024, 3), (129, 128, 64, 0)])
def test_q8_planes_gemm_matches_fp64(m, n, k, mode):
    import torch
    L = pkg("_lib")
    rng = np.random.default_rng(m + k + mode)
    a = rng.normal(size=(m, k)).astype(np.float32)
    a[: m // 4] *= 30.0
    w = (rng.normal(size=(n, k)) * 0.02).astype(np.float32)
    bias = rng.normal(size=n).astype(np.float32)
    gate = rng.normal(size=(2, n)).astype(np.float32)
    c0 = rng.normal(size=(m, n)).astype(np.float32)
    pl, ex, lde = _planes_of(a)
    w16, stt, wd = _w16(w)
    c = torch.from_numpy(c0.copy()).cuda()
    gg = torch.from_numpy(gate).cuda()
    bb = torch.from_numpy(bias).cuda()
    L.call("cv3_tc_gemm_q8_planes", pl.data_ptr(), ex.data_ptr(), lde, w16.data_ptr(), stt.data_ptr(), c.data_ptr(),
           n, m, n, k, mode, bb.data_ptr(), gg.data_ptr() if mode == 2 else None, 400 if mode == 2 else 0,
           n if mode == 2 else 0, None, None, 0, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    code = ctypes.c_int()
    L.call("cv3_tc_gemm_q8_status", ctypes.byref(code))
    assert code.value == 0
    y = a.astype(np.float64) @ wd.T + bias
    if mode == 2:
        y = c0 + gate[np.arange(m) // 400] * y
    elif mode == 3:
        y = c0 + y
    assert rel_err(c.cpu().numpy(), y) < 1e-5


def test_q8_planes_gelu_chain_matches_fp64():
    """ff1 with GELU written as planes (mode 4), then ff2 reading them: the DiT feed-forward."""
    import torch
    L = pkg("_lib")
    rng = np.random.default_rng(5)
    m, d, f = 650, 1024, 2048
    a = rng.normal(size=(m, d)).astype(np.float32)
    w1 = (rng.normal(size=(f, d)) * 0.03).astype(np.float32)
    w2 = (rng.normal(size=(d, f)) * 0.03).astype(np.float32)
    b1 = rng.normal(size=f).astype(np.float32)
    pl, ex, lde = _planes_of(a)
    w16a, sta, wd1 = _w16(w1)
    w16b, stb, wd2 = _w16(w2)
    st = torch.cuda.current_stream().cuda_stream
    pl2 = torch.empty((m, 2 * f), dtype=torch.float16, device="cuda")
    ex2 = torch.empty((f // 64, lde), dtype=torch.int8, device="cuda")
    bb = torch.from_numpy(b1).cuda()
    L.call("cv3_tc_gemm_q8_planes", pl.data_ptr(), ex.data_ptr(), lde, w16a.data_ptr(), sta.data_ptr(), None, 0,
           m, f, d, 4, bb.data_ptr(), None, 0, 0, pl2.data_ptr(), ex2.data_ptr(), lde, st)
    c = torch.zeros((m, d), device="cuda")
    L.call("cv3_tc_gemm_q8_planes", pl2.data_ptr(), ex2.data_ptr(), lde, w16b.data_ptr(), stb.data_ptr(),
           c.data_ptr(), d, m, d, f, 0, None, None, 0, 0, None, None, 0, st)
    torch.cuda.synchronize()
    h = _gelu(a.astype(np.float64) @ wd1.T + b1)
    assert rel_err(_unplanes(pl2, ex2, m, f), h) < 1e-5
    assert rel_err(c.cpu().numpy(), h @ wd2.T) < 1e-5


def test_ln_modulate_planes_match_fp32():
    import torch
    L = pkg("_lib")
    rng = np.random.default_rng(9)
    rows, d = 300, 1024
    h = (rng.normal(size=(rows, d)) * 3 + 1).astype(np.float32)
    mods = rng.normal(size=(2, 2 * d)).astype(np.float32) * 0.3
    hd, md = torch.from_numpy(h).cuda(), torch.from_numpy(mods).cuda()
    st = torch.cuda.current_stream().cuda_stream
    y = torch.empty((rows, d), device="cuda")
    sc, sh = md.data_ptr(), md.data_ptr() + d * 4
    L.call("cv3_ln_modulate", hd.data_ptr(), rows, d, 1e-6, sc, sh, 160, 2 * d, y.data_ptr(), st)
    lde = 304
    pl = torch.empty((rows, 2 * d), dtype=torch.float16, device="cuda")
    ex = torch.empty((d // 64, lde), dtype=torch.int8, device="cuda")
    L.call("cv3_ln_modulate_planes", hd.data_ptr(), rows, d, 1e-6, sc, sh, 160, 2 * d, pl.data_ptr(), ex.data_ptr(),
           lde, st)
    torch.cuda.synchronize()
    ref = y.cpu().numpy().astype(np.float64)
    assert np.all(np.abs(_unplanes(pl, ex, rows, d) - ref) <= np.abs(ref) * 2.0 ** -21 + 1e-30)


@pytest.mark.parametrize("k,bound", [(1024, 3e-6), (2048, 5e-6), (4096, 1e-5)])
def test_split_gemm_error_growth_with_k(k, bound):
    """The precision claim behind the split GEMM's accumulator layout (two hi*hi chains of
    alternate K blocks plus the cross terms, added in fp32 by the epilogue): the error
    against fp64 grows slowly with K -- measured 0.9-1.9e-6 at the DiT shapes -- and stays
    inside the 1e-5 bar at K = 4096 (during development a single accumulator over all
    products measured 3.3e-5 there: the tensor core truncates each addition into it)."""
    rng = np.random.default_rng(k)
    a = rng.normal(size=(512, k)).astype(np.float32)
    b = (rng.normal(size=(384, k)) * 0.02).astype(np.float32)
    ref = a.astype(np.float64) @ b.astype(np.float64).T
    err = rel_err(_run(a, b, kind="presplit_b"), ref)
    print(f"K={k}: {err:.2e} of max")
    assert err < bound, err
