"""Op-level parity: every CUDA kernel against the CPU oracle on the same seeded inputs.

Tolerances (max |got - ref| / max |ref|): fp32 ops 1e-5; the int8 path 1e-5 as
well (dequantisation is exact, only fp32 summation order differs); the RNG and
index work bit-exact.  Shapes cover the model's own (LM 896/4864/1152/6761, DiT
1024, HiFT source-down k30 s15 ...) plus ragged and tiny edge cases.
"""

import math

import numpy as np
import pytest

from conftest import pkg, rel_err

import oracle.numerics as nx

pytestmark = pytest.mark.gpu

TOL = 1e-5


@pytest.fixture(scope="module")
def ops():
    return pkg("ops")


@pytest.fixture
def rng():
    return np.random.default_rng(0)


def test_device_is_a_b200_class_gpu():
    import ctypes
    lib = pkg("_lib").load()
    sm, major, minor = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    assert lib.cv3_device_info(ctypes.byref(sm), ctypes.byref(major), ctypes.byref(minor)) == 0
    assert major.value == 10


@pytest.mark.parametrize("name", ["silu", "sigmoid", "gelu_tanh", "gelu", "mish", "elu"])
def test_activations(ops, rng, name):
    x = (rng.normal(size=(37, 129)) * 4).astype(np.float32)
    assert rel_err(getattr(ops, name)(x), getattr(nx, name)(x)) < 1e-6


def test_leaky_relu_and_mish_guard(ops):
    x = np.array([-50.0, -1.0, 0.0, 1.0, 20.0, 100.0, 1e4], dtype=np.float32)
    assert np.array_equal(ops.leaky_relu(x, 0.1), nx.leaky_relu(x, 0.1))
    got = ops.mish(x)
    assert np.isfinite(got).all() and rel_err(got, nx.mish(x)) < 1e-6


def test_snake(ops, rng):
    a = (np.abs(rng.normal(size=24)) + 0.5).astype(np.float32)
    x = rng.normal(size=(24, 1001)).astype(np.float32)
    assert rel_err(ops.snake(x, a), nx.snake(x, a)) < 1e-6


def test_snake_sine_against_cuda_sinf(ops, rng):
    """The snake's branch-free squared sine (|alpha x| <= 8192; CUDA's sinf beyond, and for
    inf / nan) against float64 and against the same formula on CUDA's sinf (torch.sin):
    per element within 2 ulp of the terms, and on the whole as accurate as sinf."""
    import torch
    a = np.exp(rng.uniform(np.log(1e-3), np.log(3e4), size=64)).astype(np.float32)
    x = (rng.normal(size=(64, 4097)) * np.exp(rng.uniform(-3, 3, size=(64, 4097)))).astype(np.float32)
    x[0, :4] = [np.inf, -np.inf, np.nan, 0.0]
    got = ops.snake(x, a)
    ad, xd = torch.from_numpy(a).cuda()[:, None], torch.from_numpy(x).cuda()
    cuda = (xd + (1.0 / (ad + 1e-9)) * torch.sin(ad * xd) ** 2).cpu().numpy()
    fin = np.isfinite(x)
    assert np.array_equal(np.isnan(got[~fin]), np.isnan(cuda[~fin]))
    a64 = a.astype(np.float64)[:, None]
    inv = 1.0 / (a64 + np.float32(1e-9))
    ref = x + inv * np.sin(np.float32(a)[:, None] * x).astype(np.float64) ** 2
    bound = 2.0 ** -22 * (np.abs(x) + inv)
    err, err_cuda = np.abs(got - ref)[fin], np.abs(cuda - ref)[fin]
    assert (err <= bound[fin]).all(), float((err / bound[fin]).max())
    assert err.mean() <= 1.5 * err_cuda.mean() and err.max() <= 2.0 * err_cuda.max()
    big = np.abs(np.float32(a)[:, None] * x) > 8192
    assert big.sum() > 1000 and (~big).sum() > 1000  # both forms ran


@pytest.mark.parametrize("rows,dim", [(1, 896), (7, 1024), (300, 17), (2, 6761)])
def test_norms_and_softmax(ops, rng, rows, dim):
    x = (rng.normal(size=(rows, dim)) * 3).astype(np.float32)
    w = rng.normal(size=dim).astype(np.float32)
    b = rng.normal(size=dim).astype(np.float32)
    assert rel_err(ops.rms_norm(x, w, 1e-6), nx.rms_norm(x, w, 1e-6)) < TOL
    assert rel_err(ops.layer_norm(x, None, None, 1e-6), nx.layer_norm(x, None, None, 1e-6)) < TOL
    assert rel_err(ops.layer_norm(x, w, b, 1e-5), nx.layer_norm(x, w, b, 1e-5)) < TOL
    assert rel_err(ops.softmax(x * 10), nx.softmax(x * 10)) < TOL
    assert rel_err(ops.log_softmax(x * 10), nx.log_softmax(x * 10)) < TOL


@pytest.mark.parametrize("n,k", [(4864, 896), (896, 4864), (1152, 896), (6761, 896), (128, 257), (9, 100), (64, 64)])
@pytest.mark.parametrize("m", [1, 2, 3, 8, 13])
def test_q8_linear(ops, rng, n, k, m):
    Q = pkg("quant")
    w = (rng.normal(size=(n, k)) * 0.02).astype(np.float32)
    qt = Q.make_qtensor(w)
    x = rng.normal(size=(m, k)).astype(np.float32)
    b = rng.normal(size=n).astype(np.float32)
    r = rng.normal(size=(m, n)).astype(np.float32)
    oq = nx.QTensor("q8", qt.q, qt.scales, qt.shape, 64)
    ref = nx.qmatmul(x, oq, b) + r
    got = ops.linear(x, qt, b, residual=r)
    assert got.shape == (m, n)
    assert rel_err(got, ref) < TOL


@pytest.mark.parametrize("m,n,k", [(1, 80, 192), (37, 100, 33), (1000, 1024, 1024), (130, 2048, 1024)])
def test_f32_linear(ops, rng, m, n, k):
    w = (rng.normal(size=(n, k)) * 0.02).astype(np.float32)
    x = rng.normal(size=(m, k)).astype(np.float32)
    b = rng.normal(size=n).astype(np.float32)
    assert rel_err(ops.linear(x, w, b), nx.qmatmul(x, w, b)) < TOL


def test_q8_dequant_is_exact(rng):
    Q = pkg("quant")
    qt = Q.make_qtensor(rng.normal(size=(33, 100)).astype(np.float32))
    ops = pkg("ops")
    x = np.eye(100, dtype=np.float32)
    got = ops.linear(x, qt)                       # columns of W^T through the kernel
    assert rel_err(got.T, nx.dequant(nx.QTensor("q8", qt.q, qt.scales, qt.shape, 64))) < 1e-7


@pytest.mark.parametrize("cin,cout,k,stride,dil,groups,T,pad", [
    (4, 6, 3, 1, 1, 1, 12, (1, 1)),
    (4, 6, 5, 1, 2, 1, 16, (4, 0)),
    (8, 8, 3, 1, 1, 4, 13, (2, 2)),
    (3, 6, 4, 2, 1, 1, 17, (0, 0)),
    (18, 8, 30, 15, 1, 1, 61, (14, 0)),
    (16, 16, 7, 1, 1, 4, 20, (6, 0)),
    (1024, 1024, 31, 1, 1, 16, 120, (30, 0)),
    (80, 512, 5, 1, 1, 1, 50, (0, 4)),
    (64, 64, 11, 1, 5, 1, 300, (50, 0)),
])
def test_conv1d(ops, rng, cin, cout, k, stride, dil, groups, T, pad):
    w = (rng.normal(size=(cout, cin // groups, k)) * 0.1).astype(np.float32)
    b = rng.normal(size=cout).astype(np.float32)
    x = rng.normal(size=(cin, T)).astype(np.float32)
    ref = nx.conv1d(x, w, b, stride=stride, dilation=dil, groups=groups, pad=pad)
    got = ops.conv1d(x, w, b, stride=stride, dilation=dil, groups=groups, pad=pad)
    assert got.shape == ref.shape
    assert rel_err(got, ref) < TOL


def test_conv1d_quantised_weight_and_errors(ops, rng):
    Q = pkg("quant")
    w = (rng.normal(size=(6, 4, 3)) * 0.1).astype(np.float32)
    qt = Q.make_qtensor(w.reshape(6, -1), orig_shape=(6, 4, 3))
    x = rng.normal(size=(4, 15)).astype(np.float32)
    ref = nx.conv1d(x, nx.QTensor("q8", qt.q, qt.scales, qt.shape, 64, (6, 4, 3)), None, pad=(2, 0))
    assert rel_err(ops.conv1d(x, qt, None, pad=(2, 0)), ref) < TOL
    bare = Q.QTensor("q8", qt.q, qt.scales, qt.shape, 64, None)
    with pytest.raises(ValueError, match="kernel_size"):
        ops.conv1d(x, bare)
    with pytest.raises(ValueError):
        ops.conv1d(x[:3], w)


def test_depthwise(ops, rng):
    w = rng.normal(size=(12, 1, 7)).astype(np.float32)
    b = rng.normal(size=12).astype(np.float32)
    x = rng.normal(size=(12, 20)).astype(np.float32)
    assert rel_err(ops.depthwise_conv1d(x, w, b, pad=(3, 3)), nx.depthwise_conv1d(x, w, b, pad=(3, 3))) < TOL


@pytest.mark.parametrize("h,hk,n,m,spec", [
    (4, 4, 23, 23, None), (4, 4, 23, 23, ("causal",)), (4, 4, 23, 23, ("chunk", 8, -1)),
    (4, 4, 23, 23, ("chunk", 8, 1)), (4, 4, 23, 23, ("chunk", 5, 0)), (4, 2, 19, 19, None),
    (14, 2, 1, 300, None), (14, 2, 1, 10, ("causal", 9)), (14, 2, 64, 64, ("causal", 0)),
    (16, 16, 500, 500, None), (2, 1, 3, 40, ("causal", 37)),
])
def test_sdpa(ops, rng, h, hk, n, m, spec):
    d = 64 if h >= 14 or n >= 64 else 16
    q = rng.normal(size=(h, n, d)).astype(np.float32)
    k = rng.normal(size=(hk, m, d)).astype(np.float32)
    v = rng.normal(size=(hk, m, d)).astype(np.float32)
    assert rel_err(ops.sdpa(q, k, v, spec), nx.sdpa(q, k, v, spec)) < TOL


def test_sdpa_gqa_mismatch_raises(ops, rng):
    q = rng.normal(size=(14, 1, 64)).astype(np.float32)
    k = rng.normal(size=(3, 5, 64)).astype(np.float32)
    with pytest.raises(ValueError, match="not a multiple"):
        ops.sdpa(q, k, k)


def test_stft_istft(ops, rng):
    win = nx.hann_window(16)
    sig = rng.normal(size=4003).astype(np.float32)
    ref = nx.stft(sig, 16, 4, win)
    got = ops.stft(sig, 16, 4, win)
    assert got.shape == ref.shape
    assert rel_err(np.stack([got.real, got.imag]), np.stack([ref.real, ref.imag])) < TOL
    back = ops.istft(ref, 16, 4, win)
    assert rel_err(back, nx.istft(ref, 16, 4, win)) < TOL
    assert len(ops.istft(ref, 16, 4, win, length=4003)) == 4003


def test_interpolation(ops, rng):
    x = rng.normal(size=(3, 5)).astype(np.float32)
    assert np.array_equal(ops.interpolate_nearest(x, 4), nx.interpolate_nearest(x, 4))
    y = np.arange(10, dtype=np.float32)[None, :]
    assert rel_err(ops.interpolate_linear(y, 5), nx.interpolate_linear(y, 5)) < 1e-7
    assert rel_err(ops.interpolate_linear(y, 23, True), nx.interpolate_linear(y, 23, True)) < 1e-6


def test_embedding(ops, rng):
    Q = pkg("quant")
    tab = rng.normal(size=(50, 33)).astype(np.float32)
    ids = np.array([[0, 49, 7], [7, 7, 1]])
    assert np.array_equal(ops.embedding(tab, ids), nx.embedding(tab, ids))
    t16 = tab.astype(np.float16)
    assert np.array_equal(ops.embedding(t16, ids), nx.embedding(t16, ids))
    qt = Q.make_qtensor(tab)
    assert np.array_equal(ops.embedding(qt, ids), nx.embedding(nx.QTensor("q8", qt.q, qt.scales, qt.shape, 64), ids))
    with pytest.raises(IndexError, match="outside"):
        ops.embedding(tab, np.array([50]))


# ---------------------------------------------------------------------------
# RNG: bit-exact
# ---------------------------------------------------------------------------

def test_flow_noise_buffer_is_bit_exact():
    R = pkg("torch_rng")
    assert np.array_equal(R.randn((1, 80, 15000), 0), nx.randn((1, 80, 15000), 0))


@pytest.mark.parametrize("seed", [0, 1, 42, 1986])
@pytest.mark.parametrize("n", [1, 5, 15, 16, 17, 1000, 4003])
def test_randn_bit_exact(seed, n):
    R = pkg("torch_rng")
    assert np.array_equal(R.randn((n,), seed), nx.randn((n,), seed))


def test_rand_and_shared_generator_bit_exact():
    R = pkg("torch_rng")
    assert np.array_equal(R.rand((480 * 500 * 9,), 0), nx.rand((480 * 500 * 9,), 0))
    g, h = R.TorchMT19937(0), nx.MT19937(0)
    assert np.array_equal(g.randn((1000,)), nx.randn((1000,), gen=h))
    assert np.array_equal(g.randn((1000,)), nx.randn((1000,), gen=h))
    assert np.array_equal(g.random_float32(37), h.random_float32(37))


@pytest.mark.parametrize("seed", [0, 1986])
def test_generator_words_and_doubles_bit_exact(seed):
    """TorchMT19937.next_u32 / random_float64 (cv3cpu/torch_rng.py:71-102), interleaved with
    the other draws across a state regeneration: the same words, doubles and stream position."""
    R = pkg("torch_rng")
    g, h = R.TorchMT19937(seed), nx.MT19937(seed)
    assert np.array_equal(g.next_u32(5), h.next_u32(5))
    assert np.array_equal(g.random_float64(3), h.random_float64(3))
    assert np.array_equal(g.rand((7,)), h.random_float32(7))
    assert np.array_equal(g.next_u32(1300), h.next_u32(1300))        # crosses 624-word regenerations
    assert np.array_equal(g.random_float64(700), h.random_float64(700))
    assert np.array_equal(g.randn((20,)), nx.randn((20,), gen=h))


@pytest.mark.parametrize("rows,dim,rpg", [(10400, 1024, 650), (37, 1024, 0), (300, 512, 100), (50, 80, 25)])
def test_ln_modulate(rng, rows, dim, rpg):
    """cv3_ln_modulate (the DiT's AdaLN: layer_norm(h) * (1 + scale[g]) + shift[g], g = row //
    rows_per_group) against the oracle's layer_norm: the warp-per-row kernel (dim 512 / 1024,
    aligned) and the generic one (dim 80)."""
    import torch
    L = pkg("_lib")
    groups = rows // rpg if rpg else 1
    h = (rng.normal(size=(rows, dim)) * 3 + 0.5).astype(np.float32)
    mods = rng.normal(size=(groups, 2, dim)).astype(np.float32) * 0.2   # [g][scale | shift]
    hd, md = torch.from_numpy(h).cuda(), torch.from_numpy(mods).cuda()
    y = torch.empty_like(hd)
    L.call("cv3_ln_modulate", hd.data_ptr(), rows, dim, 1e-6, md.data_ptr(), md.data_ptr() + dim * 4, rpg,
           2 * dim, y.data_ptr(), torch.cuda.current_stream().cuda_stream)
    g = np.arange(rows) // rpg if rpg else np.zeros(rows, dtype=np.int64)
    ref = nx.layer_norm(h, eps=1e-6) * (np.float32(1) + mods[g, 0]) + mods[g, 1]
    assert rel_err(y.cpu().numpy(), ref) < TOL
