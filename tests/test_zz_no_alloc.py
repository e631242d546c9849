"""cv3_istft_noalloc: the inverse STFT for callers that cannot allocate device
memory (a real-time audio callback that must not block on cudaMalloc, or a
host whose own pool already owns the GPU).  It must give cv3_istft's result
with its built-in frame buffer instead of a caller's, call after call.

This file is collected last (``zz``) so a run that stops at the first failure
has already run every other test; it also passes alone in a fresh process.
"""

import ctypes
import math

import numpy as np
import pytest

from conftest import pkg, rel_err

pytestmark = pytest.mark.gpu

TOL = 1e-5   # the fp32 bar used throughout the GPU tests


def _istft_pair(spec, mode, limit):
    import torch
    L = pkg("_lib")
    b, two_f, frames = spec.shape
    n_fft, hop = 16, 4
    win = torch.from_numpy(np.asarray(pkg("ops").hann_window(n_fft))).cuda()
    sd = torch.from_numpy(spec).cuda()
    out_len = (frames - 1) * hop
    st = torch.cuda.current_stream().cuda_stream
    ref = torch.empty(b, out_len, device="cuda")
    scratch = torch.empty(b, frames, n_fft, device="cuda")
    L.call("cv3_istft", sd.data_ptr(), mode, b, frames, n_fft, hop, win.data_ptr(), limit, n_fft // 2,
           scratch.data_ptr(), ref.data_ptr(), out_len, st)
    got = torch.empty(b, out_len, device="cuda")
    L.call("cv3_istft_noalloc", sd.data_ptr(), mode, b, frames, n_fft, hop, win.data_ptr(), limit, n_fft // 2,
           got.data_ptr(), out_len, st)
    torch.cuda.synchronize()
    return got.cpu().numpy(), ref.cpu().numpy()


def test_noalloc_istft_matches_the_allocating_entry_point_twice_in_a_row():
    rng = np.random.default_rng(11)
    # first call: one 10 s utterance's vocoder head (mode 1, clipped)
    spec1 = rng.normal(size=(1, 18, 60001)).astype(np.float32)
    got, ref = _istft_pair(spec1, 1, 0.99)
    assert got.shape == (1, 240000) and rel_err(got, ref) < TOL
    # second call, different shape and mode: nothing stale may leak through
    spec2 = rng.normal(size=(2, 18, 20001)).astype(np.float32)
    got, ref = _istft_pair(spec2, 0, math.inf)
    assert got.shape == (2, 80000) and rel_err(got, ref) < TOL


def test_noalloc_istft_rejects_sizes_beyond_its_buffer():
    import torch
    L = pkg("_lib")
    lib = L.load()
    y = torch.empty(1, device="cuda")
    rc = lib.cv3_istft_noalloc(None, 0, 2, 40000, 16, 4, None, ctypes.c_float(1.0), 8, y.data_ptr(), 1, None)
    assert rc == L.CV3_ERR_VALUE
    assert b"built-in" in lib.cv3_last_error()


_CAPTURE_CHILD = r"""
import sys
sys.path.insert(0, sys.argv[1])
import torch
from conftest import pkg
L = pkg("_lib")
lib = L.load()
y = torch.empty(64, device="cuda")
s = torch.cuda.Stream()
g = torch.cuda.CUDAGraph()
with torch.cuda.stream(s):
    g.capture_begin()
    rc = lib.cv3_istft_noalloc(None, 0, 1, 4, 16, 4, None, 1.0, 8, y.data_ptr(), 12, s.cuda_stream)
    msg = lib.cv3_last_error()
    g.capture_end()
print("RC", rc, msg.decode())
"""


def test_noalloc_first_call_inside_a_capture_is_refused(tmp_path):
    """In a fresh process (nothing looked up yet) the first call, made on a capturing
    stream, returns CV3_ERR_VALUE with a message instead of breaking the capture."""
    import os
    import subprocess
    import sys
    tests = os.path.dirname(os.path.abspath(__file__))
    script = tmp_path / "capture_child.py"
    script.write_text(_CAPTURE_CHILD)
    env = dict(os.environ, PYTHONPATH=tests + os.pathsep + os.environ.get("PYTHONPATH", ""))
    out = subprocess.run([sys.executable, str(script), tests], capture_output=True, text=True, timeout=300, env=env)
    assert out.returncode == 0, out.stderr[-2000:]
    line = [ln for ln in out.stdout.splitlines() if ln.startswith("RC ")][-1]
    assert line.split()[1] == str(pkg("_lib").CV3_ERR_VALUE), line
    assert "before any stream capture" in line
