"""The ops layer with no GPU framework: NumPy + ctypes only.

A child process blocks ``import torch`` and selects the NumPy host
(``CV3_HOST=numpy``); ``ops``, ``quant.qmatmul`` and ``torch_rng`` then allocate
and copy through the library's own ``cv3_device_alloc`` / ``cv3_memcpy`` entry
points, as a cv3cpu user's NumPy program would.  Each op is compared with the
oracle on the same seeded inputs (1e-5 for fp32 / int8 arithmetic, bit-exact for
the RNG draws), and the reference's exception types are raised for bad input.
"""

import json
import os
import subprocess
import sys

import pytest

from conftest import REPO

pytestmark = pytest.mark.gpu

CHILD = r"""
import importlib, json, os, sys
sys.modules["torch"] = None          # any `import torch` now raises ImportError
sys.path.insert(0, sys.argv[1])
import numpy as np

pkg = lambda n: importlib.import_module("cosyvoice3-cpu_b200." + n)
D, ops, quant, trng = pkg("_dev"), pkg("ops"), pkg("quant"), pkg("torch_rng")
import oracle.numerics as nx

def rel(got, ref):
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    assert got.shape == ref.shape, (got.shape, ref.shape)
    return float(np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-9))

rng = np.random.default_rng(0)
res = {"backend": D.BACKEND, "torch_loaded": sys.modules.get("torch") is not None}
w = (rng.normal(size=(512, 384)) * 0.02).astype(np.float32)
b = rng.normal(size=512).astype(np.float32)
qt = quant.make_qtensor(w)
oq = nx.QTensor("q8", qt.q, qt.scales, qt.shape, 64)
x = rng.normal(size=(5, 384)).astype(np.float32)
res["qmatmul"] = rel(quant.qmatmul(x, qt, b), nx.qmatmul(x, oq, b))
x2 = rng.normal(size=(40, 384)).astype(np.float32)
res["linear_f32"] = rel(ops.linear(x2, w, b), nx.linear(x2, w, b))
h = rng.normal(size=(7, 896)).astype(np.float32)
g = (1 + 0.1 * rng.normal(size=896)).astype(np.float32)
res["rms_norm"] = rel(ops.rms_norm(h, g), nx.rms_norm(h, g))
res["layer_norm"] = rel(ops.layer_norm(h, None, None, 1e-6), nx.layer_norm(h, None, None, 1e-6))
res["log_softmax"] = rel(ops.log_softmax(h), nx.log_softmax(h))
res["silu"] = rel(ops.silu(h), nx.silu(h))
a = np.abs(rng.normal(size=(7, 1))).astype(np.float32) + 0.5
res["snake"] = rel(ops.snake(h, a), nx.snake(h, a))
q = rng.normal(size=(14, 33, 64)).astype(np.float32)
k = rng.normal(size=(2, 33, 64)).astype(np.float32)
v = rng.normal(size=(2, 33, 64)).astype(np.float32)
res["sdpa_causal_gqa"] = rel(ops.sdpa(q, k, v, ("causal", 0)), nx.sdpa(q, k, v, ("causal", 0)))
xc = rng.normal(size=(16, 200)).astype(np.float32)
wc = (rng.normal(size=(24, 16, 7)) * 0.1).astype(np.float32)
res["conv1d"] = rel(ops.conv1d(xc, wc, None, dilation=3, pad=(18, 0)), nx.conv1d(xc, wc, None, dilation=3, pad=(18, 0)))
tab = (rng.normal(size=(300, 96)) * 0.02).astype(np.float32)
qtab = quant.make_qtensor(tab)
ids = np.array([[3, 299, 0], [17, 17, 150]])
res["embedding_q8"] = rel(ops.embedding(qtab, ids), nx.embedding(nx.QTensor("q8", qtab.q, qtab.scales, qtab.shape, 64), ids))
try:
    ops.embedding(qtab, np.array([300]))
    res["index_error"] = False
except IndexError:
    res["index_error"] = True
try:
    ops.sdpa(q, k[:1].repeat(3, 0), v[:1].repeat(3, 0))
    res["value_error"] = False
except ValueError:
    res["value_error"] = True
sig = rng.normal(size=4000).astype(np.float32)
win = ops.hann_window(16)
spec = ops.stft(sig, 16, 4, win)
res["stft"] = rel(np.concatenate([spec.real, spec.imag]), np.concatenate([nx.stft(sig, 16, 4, win).real, nx.stft(sig, 16, 4, win).imag]))
res["istft"] = rel(ops.istft(spec, 16, 4, win, length=4000), nx.istft(spec, 16, 4, win, length=4000))
res["interpolate_linear"] = rel(ops.interpolate_linear(xc, 333), nx.interpolate_linear(xc, 333))
res["randn_bitexact"] = bool(np.array_equal(trng.randn((1, 80, 700), 0), nx.randn((1, 80, 700), 0)))
res["rand_bitexact"] = bool(np.array_equal(trng.rand((9, 1000), 3), nx.rand((9, 1000), 3)))
free0 = D.ctypes.c_int64(0)
D.call("cv3_mem_get_info", D.ctypes.byref(free0), None)
big = D.empty((64 << 20,))                  # 256 MB from cv3_device_alloc
free1 = D.ctypes.c_int64(0)
D.call("cv3_mem_get_info", D.ctypes.byref(free1), None)
del big
free2 = D.ctypes.c_int64(0)
D.call("cv3_mem_get_info", D.ctypes.byref(free2), None)
res["alloc_mb"] = (free0.value - free1.value) / 2**20
res["freed_mb"] = (free2.value - free1.value) / 2**20
print("RESULT " + json.dumps(res))
"""


def test_ops_run_without_pytorch():
    env = dict(os.environ, CV3_HOST="numpy")
    p = subprocess.run([sys.executable, "-c", CHILD, REPO], capture_output=True, text=True, env=env, timeout=600)
    assert p.returncode == 0, p.stdout[-2000:] + p.stderr[-4000:]
    line = [ln for ln in p.stdout.splitlines() if ln.startswith("RESULT ")][-1]
    res = json.loads(line[len("RESULT "):])
    assert res.pop("backend") == "numpy"
    assert res.pop("torch_loaded") is False
    assert res.pop("index_error") is True and res.pop("value_error") is True
    assert res.pop("randn_bitexact") is True and res.pop("rand_bitexact") is True
    assert res.pop("alloc_mb") >= 255 and res.pop("freed_mb") >= 255
    for name, err in res.items():
        assert err < 1e-5, (name, err)
