"""Tensor-core attention (head dim 64) against the oracle's exact softmax attention.

cv3_attention sends head-dim-64 problems with 16-byte aligned rows and more
than 4 queries to the tcgen05 kernel (3xTF32 products, online softmax in
fp32).  These cases read q/k/v in the models' token-major layout (one fused
[batch][tokens][3 * heads * 64] buffer, as the DiT's QKV linear writes it) and
cover the mask kinds of cv3cpu/ops.py:244-264, GQA, ragged query/key counts,
several batches and key counts that are not tile multiples.  Tolerance 1e-5
of max |ref|, the fp32 bar.
"""

import math

import numpy as np
import pytest

from conftest import pkg, rel_err

import oracle.numerics as nx

pytestmark = pytest.mark.gpu

TOL = 1e-5
HD = 64


def _run(batch, h, hk, n, m, spec, seed):
    import torch
    lib = pkg("_lib")
    rng = np.random.default_rng(seed)
    # queries and keys in separate token-major buffers (n may differ from m)
    qbuf = (rng.normal(size=(batch, n, h * HD)) * 1.5).astype(np.float32)
    kvbuf = rng.normal(size=(batch, m, 2 * hk * HD)).astype(np.float32)
    qd = torch.from_numpy(qbuf).cuda()
    kvd = torch.from_numpy(kvbuf).cuda()
    out = torch.full((batch, n, h * HD), float("nan"), device="cuda")
    kind, a, b = pkg("ops")._mask_args(spec)
    scale = float(np.float32(1.0 / math.sqrt(HD)))
    q, k = qd.data_ptr(), kvd.data_ptr()
    v = k + hk * HD * 4
    lib.call("cv3_attention", q, n * h * HD, HD, h * HD,
             k, m * 2 * hk * HD, HD, 2 * hk * HD,
             v, m * 2 * hk * HD, HD, 2 * hk * HD,
             out.data_ptr(), n * h * HD, HD, h * HD,
             batch, h, hk, n, m, HD, scale, kind, a, b, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    import ctypes
    code = ctypes.c_int(-1)
    assert lib.load().cv3_tc_attention_status(ctypes.byref(code)) == 0 and code.value == 0
    got = out.cpu().numpy()
    for bi in range(batch):
        qh = qbuf[bi].reshape(n, h, HD).transpose(1, 0, 2)
        kh = kvbuf[bi, :, :hk * HD].reshape(m, hk, HD).transpose(1, 0, 2)
        vh = kvbuf[bi, :, hk * HD:].reshape(m, hk, HD).transpose(1, 0, 2)
        ref = nx.sdpa(np.ascontiguousarray(qh), np.ascontiguousarray(kh), np.ascontiguousarray(vh), spec)
        mine = got[bi].reshape(n, h, HD).transpose(1, 0, 2)
        assert np.isfinite(mine).all()
        assert rel_err(mine, ref) < TOL, (bi, float(np.abs(mine - ref).max()))


@pytest.mark.parametrize("batch,h,hk,n,m,spec", [
    (1, 16, 16, 650, 650, None),            # the DiT shape (per utterance, per CFG half)
    (2, 16, 16, 200, 200, ("chunk", 50, -1)),   # streaming DiT: all left chunks
    (1, 16, 16, 300, 300, ("chunk", 50, 1)),    # one chunk of left context (tiles skipped)
    (1, 16, 16, 97, 97, ("chunk", 7, 0)),
    (2, 14, 2, 137, 137, ("causal", 0)),        # Qwen2 prefill, GQA 7:1
    (1, 14, 2, 40, 180, ("causal", 140)),       # continuation: 40 new queries after 140 cached keys
    (1, 4, 4, 5, 70, None),                     # smallest query count on this path
    (3, 2, 1, 129, 63, None),                   # fewer keys than one tile, ragged queries
    (1, 8, 8, 64, 64, None),
    (1, 2, 2, 256, 1000, None),                 # many key tiles (ring wraps several times)
])
def test_tc_attention(batch, h, hk, n, m, spec):
    _run(batch, h, hk, n, m, spec, seed=batch * 1000 + n + m)


def test_tc_attention_large_batch_grid():
    # 16 utterance halves x 16 heads = 256 (batch, head) pairs, as in the CFG flow solve
    _run(16, 16, 16, 70, 70, None, seed=7)
