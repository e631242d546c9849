"""The tcgen05 3xTF32 GEMM against fp64 products of the same fp32 inputs.

Bar: max |got - ref| / max |ref| <= 1e-5 (measured 1.7e-6 at K=1024 and
3.1e-6 at K=2048 with the default accumulator layout; NumPy's fp32 BLAS is
~6e-7 on the same inputs).  Cases grow from one 128x128 tile to
the DiT's shapes, with row/column tails, K tails and every epilogue.  After
each case the kernel's error word (bounded-wait expiry) must be clear.
"""

import ctypes

import numpy as np
import pytest

from conftest import pkg, rel_err

pytestmark = pytest.mark.gpu


def _run(a, b, mode=0, bias=None, gate=None, c0=None, rows_per_group=0):
    import torch
    L = pkg("_lib")
    ad, bd = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
    m, k = a.shape
    n = b.shape[0]
    c = torch.from_numpy(c0.copy()).cuda() if c0 is not None else torch.zeros(m, n, device="cuda")
    bb = torch.from_numpy(bias).cuda() if bias is not None else None
    gg = torch.from_numpy(gate).cuda() if gate is not None else None
    L.call("cv3_tc_gemm", ad.data_ptr(), k, bd.data_ptr(), k, c.data_ptr(), n, m, n, k, mode,
           bb.data_ptr() if bb is not None else None, gg.data_ptr() if gg is not None else None,
           rows_per_group, n if gate is not None else 0, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    code = ctypes.c_int()
    L.call("cv3_tc_gemm_status", ctypes.byref(code))
    assert code.value == 0, f"bounded wait expired (code {code.value})"
    return c.cpu().numpy()


def _gelu(x):
    return 0.5 * x * (1.0 + np.tanh(np.sqrt(2.0 / np.pi) * (x + 0.044715 * x ** 3)))


@pytest.mark.parametrize("m,n,k", [(128, 128, 32), (128, 128, 64), (256, 256, 256), (37, 100, 68),
                                   (1000, 1024, 1024), (10400, 3072, 1024), (10400, 1024, 320),
                                   (1000, 1024, 2048), (130, 80, 1024)])
def test_plain_gemm(m, n, k):
    rng = np.random.default_rng(m + n + k)
    a = rng.normal(size=(m, k)).astype(np.float32)
    b = (rng.normal(size=(n, k)) * 0.02).astype(np.float32)
    ref = a.astype(np.float64) @ b.astype(np.float64).T
    assert rel_err(_run(a, b), ref) < 1e-5


def test_epilogues():
    rng = np.random.default_rng(7)
    m, n, k = 650, 2048, 1024
    a = rng.normal(size=(m, k)).astype(np.float32)
    b = (rng.normal(size=(n, k)) * 0.02).astype(np.float32)
    bias = rng.normal(size=n).astype(np.float32)
    y = a.astype(np.float64) @ b.astype(np.float64).T + bias
    assert rel_err(_run(a, b, 0, bias), y) < 1e-5
    assert rel_err(_run(a, b, 1, bias), _gelu(y)) < 1e-5
    h = rng.normal(size=(m, n)).astype(np.float32)
    gate = rng.normal(size=(2, n)).astype(np.float32)
    rows = 325
    ref = h + np.repeat(gate, rows, axis=0) * y
    assert rel_err(_run(a, b, 2, bias, gate, h, rows_per_group=rows), ref) < 1e-5
    assert rel_err(_run(a, b, 3, bias, None, h), h + y) < 1e-5
