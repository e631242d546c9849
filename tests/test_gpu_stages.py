"""Stage parity on the GPU: the DiT flow solve and the HiFT vocoder against the
reference's goldens and the oracle (small synthetic model, both profiles), plus
batching invariance (utterances solved together equal utterances solved alone).

Tolerance: 1e-5 max relative error for the fp32 stages;
the q8 ("balanced") path is checked at the same bar because dequantisation is
exact and only summation order differs.
"""

import numpy as np
import pytest

from conftest import pkg, rel_err

import oracle.numerics as nx
import oracle.stages as st

pytestmark = pytest.mark.gpu

TOL = 1e-5


def _device(W):
    return pkg("weights").DeviceWeights(W)


@pytest.mark.parametrize("profile", ["balanced", "f32"])
def test_flow_matches_reference_goldens(golden, small_weights, profile):
    W = small_weights[profile]
    g = lambda k: golden[f"{profile}/flow_{k}"]  # noqa: E731
    flow = pkg("models.flow").Flow(_device(W))
    mel = flow.inference(g("token"), g("prompt_token"), g("prompt_feat"), g("embedding"))
    assert mel.shape == g("mel").shape
    assert rel_err(mel, g("mel")) < TOL


def test_dit_forward_matches_oracle(small_weights):
    W = small_weights["f32"]
    rng = np.random.default_rng(3)
    B, N = 3, 37
    x, mu, cond = (rng.normal(size=(B, 80, N)).astype(np.float32) for _ in range(3))
    spk = rng.normal(size=(B, 80)).astype(np.float32)
    t = np.array([0.1, 0.5, 0.9], np.float32)
    got = pkg("models.dit").DiT(_device(W)).forward(x, mu, t, spk, cond)
    ref = st.DiT(W, W.meta).forward(x, mu, t, spk, cond)
    assert rel_err(got, ref) < TOL
    got_s = pkg("models.dit").DiT(_device(W)).forward(x, mu, t, spk, cond, streaming=True)
    assert rel_err(got_s, st.DiT(W, W.meta).forward(x, mu, t, spk, cond, streaming=True)) < TOL


def test_flow_batched_solve_equals_single(small_weights):
    W = small_weights["balanced"]
    flow = pkg("models.flow").Flow(_device(W))
    rng = np.random.default_rng(4)
    conds = []
    for s in range(3):
        tok = rng.integers(0, 256, size=15)
        conds.append(flow.conditioning(tok, rng.integers(0, 256, size=5), rng.normal(size=(10, 80)).astype(np.float32),
                                       rng.normal(size=192).astype(np.float32)))
    together = flow.solve_batch([c[0] for c in conds], [c[1] for c in conds], [c[2] for c in conds]).cpu().numpy()
    for u, c in enumerate(conds):
        alone = flow.solve_batch([c[0]], [c[1]], [c[2]], use_graph=False).cpu().numpy()[0]
        assert rel_err(together[u], alone) < TOL
    of = st.Flow(W, W.meta)
    ref = of.solve_euler(conds[1][0].cpu().numpy()[None], conds[1][1].cpu().numpy()[None],
                         conds[1][2].cpu().numpy()[None])
    assert rel_err(together[1], ref[0]) < TOL


@pytest.mark.parametrize("profile", ["balanced", "f32"])
def test_hift_matches_reference_goldens(golden, small_weights, profile):
    W = small_weights[profile]
    h = pkg("models.hift").HiFTGenerator(_device(W))
    mel = golden[f"{profile}/hift_mel"]
    assert rel_err(h.inference(mel, chunk=None), golden[f"{profile}/hift_wav"]) < TOL
    assert rel_err(h.inference(mel, chunk=4, context=64), golden[f"{profile}/hift_wav_chunked"]) < TOL


def test_hift_pieces_match_oracle(small_weights):
    W = small_weights["f32"]
    h = pkg("models.hift").HiFTGenerator(_device(W))
    oh = st.HiFT(W, W.meta)
    rng = np.random.default_rng(6)
    mel = np.clip(rng.normal(-5.0, 2.0, size=(80, 23)), -11.5, 2.0).astype(np.float32)
    D = pkg("_dev")
    f0 = h.f0_predict(D.dev(mel)[None])
    f0_ref = oh.f0_predict(mel).astype(np.float32)
    assert rel_err(f0.cpu().numpy()[0], f0_ref) < TOL
    src = h.excitation(D.dev(f0_ref)[None]).cpu().numpy()[0]
    assert rel_err(src, oh.excitation(f0_ref)) < TOL
    # batch of two equals two singles
    mels = np.stack([mel, mel[:, ::-1].copy()])
    both = h.inference_batch(mels).cpu().numpy()
    assert rel_err(both[1], oh.inference(mels[1], chunk=None)) < TOL


def test_hift_graph_replay_equals_eager():
    """The batched vocoder replayed from its CUDA graph (full geometry, batch 2): bit-identical
    to the eager pass on the input it was captured with and on a new input of the same shape,
    and every replay returns a fresh tensor."""
    import torch
    W = pkg("synth").synthetic_weights("f32", stages=("hift",))
    h = pkg("models.hift").HiFTGenerator(_device(W))
    rng = np.random.default_rng(11)
    mels = [torch.from_numpy(np.clip(rng.normal(-5.0, 2.0, size=(2, 80, 30)), -11.5, 2.0).astype(np.float32)).cuda()
            for _ in range(2)]
    eager = [h.inference_batch(m) for m in mels]
    outs = [h.inference_batch(mels[0], use_graph=True) for _ in range(3)]   # eager, capture, replay
    assert len(h._graphs) == 1
    for o in outs:
        assert torch.equal(o, eager[0])
    second = h.inference_batch(mels[1], use_graph=True)
    assert torch.equal(second, eager[1])
    assert torch.equal(outs[-1], eager[0])      # the earlier result was not overwritten


def test_hift_full_geometry_snake_and_vocoder_length(small_weights):
    W = pkg("synth").synthetic_weights("f32", stages=("hift",))
    h = pkg("models.hift").HiFTGenerator(_device(W))
    rng = np.random.default_rng(1)
    mel = np.clip(rng.normal(-5.0, 2.0, size=(80, 40)), -11.5, 2.0).astype(np.float32)
    got = h.inference(mel)
    assert got.shape == (480 * 40,) and np.abs(got).max() <= 0.99 + 1e-7
    assert rel_err(got, st.HiFT(W, W.meta).inference(mel, chunk=None)) < TOL


def test_balanced_dit_forward_full_size_q8_gemm_matches_oracle():
    """The released DiT geometry in the balanced profile: the block matrices run through
    cv3_tc_gemm_q8_planes on the stored int8 weights; one forward at batch 2 x 128 frames
    against the oracle (which dequantises to fp32, as the reference's qmatmul does) at
    the fp32 bar, and the dequantised 3xTF32 path agrees as well."""
    W = pkg("synth").synthetic_weights("balanced", stages=("flow",))
    rng = np.random.default_rng(12)
    B, N = 2, 128
    x, mu, cond = (rng.normal(size=(B, 80, N)).astype(np.float32) for _ in range(3))
    spk = rng.normal(size=(B, 80)).astype(np.float32)
    t = np.array([0.2, 0.8], np.float32)
    dev = pkg("models.dit").DiT(_device(W))
    dev.prepare()
    assert type(dev.blocks[0].ff1).__name__ == "LinQ8"
    got = dev.forward(x, mu, t, spk, cond)
    ref = st.DiT(W, W.meta).forward(x, mu, t, spk, cond)
    assert rel_err(got, ref) < TOL
    split = pkg("models.dit").DiT(_device(W))
    split.q8_planes = False  # fp32 rows split inside each GEMM instead of activation planes
    assert rel_err(split.forward(x, mu, t, spk, cond), ref) < TOL
    f32 = pkg("models.dit").DiT(_device(W))
    f32.q8_gemm = False
    assert rel_err(f32.forward(x, mu, t, spk, cond), ref) < TOL
