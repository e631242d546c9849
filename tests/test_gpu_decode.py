"""The fused decode GEMV (cv3_q8_decode_gemv) and the decode engine's fused path.

Kernel vs the oracle: RMSNorm-fused input, bias, residual, SwiGLU row pairs,
K split over CTAs (deterministic reduction), 1..32 rows (8-sequence column
blocks; a row's result does not depend on how many rows share the call);
tolerance 1e-5 (the int8 dequantisation is exact).  Engine: a small LM whose every linear is q8,
so the fused path runs, against the oracle's greedy decode.
"""

import ctypes

import numpy as np
import pytest

from conftest import pkg, rel_err

import oracle.numerics as nx
import oracle.stages as st

pytestmark = pytest.mark.gpu


def _dg(qt, **kw):
    return pkg("models._common").DecodeGemv(qt.to_device(), **kw)


@pytest.mark.parametrize("n,k", [(1152, 896), (896, 896), (896, 4864), (9728, 896), (6761, 896), (96, 100)])
@pytest.mark.parametrize("m", [1, 3, 8, 12, 32])
def test_decode_gemv_plain_and_residual(n, k, m):
    import torch
    if m > 8 and k % 64:
        pytest.skip("K not a multiple of 64: the CUDA-core GEMV, which takes up to 8 rows")
    rng = np.random.default_rng(n + k + m)
    w = (rng.normal(size=(n, k)) * 0.02).astype(np.float32)
    qt = pkg("quant").make_qtensor(w)
    oq = nx.QTensor("q8", qt.q, qt.scales, qt.shape, 64)
    x = rng.normal(size=(m, k)).astype(np.float32)
    b = rng.normal(size=n).astype(np.float32)
    r = rng.normal(size=(m, n)).astype(np.float32)
    g = _dg(qt, bias=torch.from_numpy(b).cuda(), mma_splits=5 if (k > 1024 and m > 8) else 1)
    xd, y = torch.from_numpy(x).cuda(), torch.from_numpy(r).cuda()
    for _ in range(2):                       # twice: the split counters must be left at zero
        y.copy_(torch.from_numpy(r))
        g(xd.data_ptr(), m, y.data_ptr(), residual=y.data_ptr())
        torch.cuda.synchronize()
        assert rel_err(y.cpu().numpy(), nx.qmatmul(x, oq, b) + r) < 1e-5


@pytest.mark.parametrize("m", [1, 5, 8, 20, 32])
def test_decode_gemv_fused_norm_and_swiglu(m):
    import torch
    C = pkg("models._common")
    rng = np.random.default_rng(m)
    k, inter = 896, 4864
    gate = (rng.normal(size=(inter, k)) * 0.02).astype(np.float32)
    up = (rng.normal(size=(inter, k)) * 0.02).astype(np.float32)
    qg, qu = pkg("quant").make_qtensor(gate), pkg("quant").make_qtensor(up)
    nw = (1 + 0.1 * rng.normal(size=k)).astype(np.float32)
    x = rng.normal(size=(m, k)).astype(np.float32)
    n = nx.rms_norm(x, nw, 1e-6)
    og = nx.qmatmul(n, nx.QTensor("q8", qg.q, qg.scales, qg.shape, 64))
    ou = nx.qmatmul(n, nx.QTensor("q8", qu.q, qu.scales, qu.shape, 64))
    ref = nx.silu(og) * ou
    inter_q = C.interleave_rows(qg.to_device(), qu.to_device())
    g = C.DecodeGemv(inter_q, norm_w=torch.from_numpy(nw).cuda(), eps=1e-6, swiglu=True)
    y = torch.empty(m, inter, device="cuda")
    g(torch.from_numpy(x).cuda().data_ptr(), m, y.data_ptr())
    torch.cuda.synchronize()
    assert rel_err(y.cpu().numpy(), ref) < 1e-5


def test_engine_fused_path_matches_oracle(small_weights):
    """Small LM with every linear quantised: the engine takes the fused path."""
    W0 = small_weights["f32"]
    Q = pkg("quant")
    tensors = dict(W0)
    for name, t in W0.items():
        if name.startswith("llm.") and ("proj.weight" in name or "llm_decoder.weight" in name):
            tensors[name] = Q.make_qtensor(t)
    W = pkg("weights").TensorDict(tensors, W0.meta)
    lm = pkg("models.llm").CosyVoice3LM(pkg("weights").DeviceWeights(W))
    olm = st.SpeechLM(W, W.meta)
    rng = np.random.default_rng(9)
    eop = W.meta["endofprompt_id"]
    prompts, oprompts = [], []
    for nn in (6, 11):
        text = [eop] + rng.integers(0, 2000, size=nn).tolist()
        prompts.append(lm.prompt_embedding(text, (), [1, 2, 3]))
        oprompts.append(olm.prompt_embedding(text, (), [1, 2, 3]))
    toks = lm.generate_greedy(prompts, 16).cpu().numpy()
    eng = lm.last_engine
    assert all(f is not None for f in eng.fast) and eng.fast_head is not None
    for b in range(2):
        ref, _ = olm.generate_greedy(oprompts[b], 16)
        assert toks[b].tolist() == ref


@pytest.mark.parametrize("n,k", [(1152, 896), (896, 4864), (6761, 896), (9728, 896), (48, 128)])
@pytest.mark.parametrize("m", [1, 8])
def test_tensor_core_and_cuda_core_gemvs_agree(n, k, m):
    """cv3_q8_decode_gemv_mma (warp MMA, three exact bf16 parts of x) against the CUDA-core
    kernel and the oracle on the same operands, with the RMSNorm fused in."""
    import torch
    L = pkg("_lib")
    rng = np.random.default_rng(n * 7 + k + m)
    w = (rng.normal(size=(n, k)) * 0.02).astype(np.float32)
    hq = pkg("quant").make_qtensor(w)
    qt = hq.to_device()
    nw = (1 + 0.1 * rng.normal(size=k)).astype(np.float32)
    x = (rng.normal(size=(m, k)) * 3.0).astype(np.float32)
    ref = nx.qmatmul(nx.rms_norm(x, nw, 1e-6), nx.QTensor("q8", hq.q, hq.scales, hq.shape, 64))
    xd, nwd = torch.from_numpy(x).cuda(), torch.from_numpy(nw).cuda()
    st = torch.cuda.current_stream().cuda_stream
    y1, y2 = torch.empty(m, n, device="cuda"), torch.empty(m, n, device="cuda")
    L.call("cv3_q8_decode_gemv_mma", xd.data_ptr(), m, k, k, qt.q.data_ptr(), qt.scales.data_ptr(), n, k, None, None,
           nwd.data_ptr(), 1e-6, 0, y1.data_ptr(), n, 1, None, 0, None, st)
    L.call("cv3_q8_decode_gemv", xd.data_ptr(), m, k, k, qt.q.data_ptr(), qt.scales.data_ptr(), n, k, None, None,
           nwd.data_ptr(), 1e-6, 0, y2.data_ptr(), n, 1, None, 0, None, st)
    torch.cuda.synchronize()
    assert rel_err(y1.cpu().numpy(), ref) < 1e-5
    assert rel_err(y1.cpu().numpy(), y2.cpu().numpy()) < 1e-5


@pytest.mark.parametrize("m,cap", [(1, 96), (3, 96), (8, 96), (3, 1024), (8, 1024), (32, 96), (32, 1024)])
def test_decode_rope_attention_matches_separate_kernels(m, cap):
    """cv3_decode_rope_attention (RoPE + cache append + attention in one launch) against
    cv3_rope_qkv_append followed by cv3_decode_attention on the same qkv rows and caches:
    bit-identical caches and outputs (every key's dot product takes the same column order
    whether its row was staged in shared memory or read from global memory), including a
    sequence whose position lies past the cache (its key and value are not stored by
    either), at cap 1024 positions past the rows that fit in shared memory, and at 32
    sequences several query heads per CTA."""
    import torch
    L = pkg("_lib")
    H, Hk, hd = 14, 2, 64
    n = (H + 2 * Hk) * hd
    rng = np.random.default_rng(70 + m)
    c, s = pkg("models.qwen2").rope_tables(cap, hd, 1e6)
    cosd, sind = torch.from_numpy(c).cuda(), torch.from_numpy(s).cuda()
    qkv = torch.from_numpy(rng.normal(size=(m, n)).astype(np.float32)).cuda()
    pos_h = rng.integers(10, cap, size=m).astype(np.int32)
    if m > 2:
        pos_h[1] = cap + 5
    lens_h = np.minimum(pos_h + 1, cap).astype(np.int32)
    pos, lens = torch.from_numpy(pos_h).cuda(), torch.from_numpy(lens_h).cuda()
    seqs = torch.arange(m, dtype=torch.int32, device="cuda")
    kc0 = torch.from_numpy(rng.normal(size=(m, Hk, cap, hd)).astype(np.float32)).cuda()
    vc0 = torch.from_numpy(rng.normal(size=(m, Hk, cap, hd)).astype(np.float32)).cuda()
    st = torch.cuda.current_stream().cuda_stream
    scale = float(np.float32(1.0 / np.sqrt(hd)))
    outs = []
    for fused in (True, False):
        kc, vc = kc0.clone(), vc0.clone()
        a = torch.zeros(m, H * hd, device="cuda")
        if fused:
            L.call("cv3_decode_rope_attention", qkv.data_ptr(), n, cosd.data_ptr(), sind.data_ptr(), pos.data_ptr(),
                   kc.data_ptr(), vc.data_ptr(), lens.data_ptr(), m, H, Hk, hd, cap, scale, a.data_ptr(), st)
        else:
            q = torch.empty(m, H * hd, device="cuda")
            L.call("cv3_rope_qkv_append", qkv.data_ptr(), m, n, cosd.data_ptr(), sind.data_ptr(), seqs.data_ptr(),
                   pos.data_ptr(), H, Hk, hd, q.data_ptr(), kc.data_ptr(), vc.data_ptr(), cap, st)
            L.call("cv3_decode_attention", q.data_ptr(), kc.data_ptr(), vc.data_ptr(), lens.data_ptr(), m, H, Hk, hd,
                   cap, scale, a.data_ptr(), st)
        torch.cuda.synchronize()
        outs.append((a.cpu().numpy(), kc.cpu().numpy(), vc.cpu().numpy()))
    for x, y in zip(outs[0], outs[1]):
        assert np.array_equal(x, y)
    code = ctypes.c_int(-1)
    L.load().cv3_decode_attention_status(ctypes.byref(code))
    assert code.value == 0


@pytest.mark.parametrize("m", [9, 17, 32])
def test_decode_gemv_rows_independent_of_batch(m):
    """Each row of an m-row call equals the same row computed alone, bit for bit (the
    batch-32 decode must choose the ids a sequence gets alone)."""
    import torch
    rng = np.random.default_rng(100 + m)
    n, k = 1152, 896
    w = (rng.normal(size=(n, k)) * 0.02).astype(np.float32)
    qt = pkg("quant").make_qtensor(w)
    nw = torch.from_numpy((1 + 0.1 * rng.normal(size=k)).astype(np.float32)).cuda()
    b = torch.from_numpy(rng.normal(size=n).astype(np.float32)).cuda()
    g = _dg(qt, bias=b, norm_w=nw, eps=1e-6)
    x = torch.from_numpy(rng.normal(size=(m, k)).astype(np.float32)).cuda()
    y = torch.empty(m, n, device="cuda")
    g(x.data_ptr(), m, y.data_ptr())
    y1 = torch.empty(1, n, device="cuda")
    for i in (0, m // 2, m - 1):
        g(x[i:i + 1].data_ptr(), 1, y1.data_ptr())
        torch.cuda.synchronize()
        assert torch.equal(y[i], y1[0]), i


def test_decode_gemv_long_k_many_rows_needs_splits():
    """32 rows of K = 4864 do not fit one CTA's shared memory unsplit: a ValueError, not a launch."""
    import torch
    rng = np.random.default_rng(5)
    qt = pkg("quant").make_qtensor((rng.normal(size=(896, 4864)) * 0.02).astype(np.float32))
    g = _dg(qt)
    x = torch.zeros(32, 4864, device="cuda")
    y = torch.zeros(32, 896, device="cuda")
    with pytest.raises(ValueError):
        g(x.data_ptr(), 32, y.data_ptr())


@pytest.mark.parametrize("cap", [256, 1024])
def test_decode_attention_sequence_independent_of_batch(cap):
    """A sequence's attention output is the same, bit for bit, alone (one query head per
    CTA) and among 32 sequences (four query heads per CTA, fewer rows staged)."""
    import torch
    L = pkg("_lib")
    H, Hk, hd, m = 14, 2, 64, 32
    rng = np.random.default_rng(cap)
    q = torch.from_numpy(rng.normal(size=(m, H * hd)).astype(np.float32)).cuda()
    kc = torch.from_numpy(rng.normal(size=(m, Hk, cap, hd)).astype(np.float32)).cuda()
    vc = torch.from_numpy(rng.normal(size=(m, Hk, cap, hd)).astype(np.float32)).cuda()
    lens = torch.from_numpy(rng.integers(1, cap + 1, size=m).astype(np.int32)).cuda()
    st = torch.cuda.current_stream().cuda_stream
    scale = float(np.float32(1.0 / np.sqrt(hd)))
    a = torch.zeros(m, H * hd, device="cuda")
    L.call("cv3_decode_attention", q.data_ptr(), kc.data_ptr(), vc.data_ptr(), lens.data_ptr(), m, H, Hk, hd, cap,
           scale, a.data_ptr(), st)
    a1 = torch.zeros(1, H * hd, device="cuda")
    for i in (0, 13, 31):
        L.call("cv3_decode_attention", q[i:i + 1].data_ptr(), kc[i:i + 1].data_ptr(), vc[i:i + 1].data_ptr(),
               lens[i:i + 1].data_ptr(), 1, H, Hk, hd, cap, scale, a1.data_ptr(), st)
        torch.cuda.synchronize()
        assert torch.equal(a[i], a1[0]), i


@pytest.mark.parametrize("m", [1, 8, 32])
@pytest.mark.parametrize("splits", [2, 4])
def test_decode_gemv_fused_norm_with_cluster_k_splits(m, splits):
    """The fused-RMSNorm GEMV with K split over a cluster (the decode step's qkv projection):
    each CTA folds its K range, the first adds the others' dot products and sums of squares
    in split order; against the oracle's rms_norm then q8 linear (1e-5), repeated twice."""
    import torch
    rng = np.random.default_rng(200 + m + splits)
    n, k = 1152, 896
    w = (rng.normal(size=(n, k)) * 0.02).astype(np.float32)
    qt = pkg("quant").make_qtensor(w)
    oq = nx.QTensor("q8", qt.q, qt.scales, qt.shape, 64)
    nw = (1 + 0.1 * rng.normal(size=k)).astype(np.float32)
    b = rng.normal(size=n).astype(np.float32)
    x = rng.normal(size=(m, k)).astype(np.float32)
    ref = nx.qmatmul(nx.rms_norm(x, nw, 1e-6), oq, b)
    g = _dg(qt, bias=torch.from_numpy(b).cuda(), norm_w=torch.from_numpy(nw).cuda(), eps=1e-6, mma_splits=splits)
    assert g.splits == splits
    xd, y = torch.from_numpy(x).cuda(), torch.empty(m, n, device="cuda")
    for _ in range(2):
        g(xd.data_ptr(), m, y.data_ptr())
        torch.cuda.synchronize()
        assert rel_err(y.cpu().numpy(), ref) < 1e-5
