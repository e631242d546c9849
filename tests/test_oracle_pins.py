"""Pin the CPU oracle: against the reference's frozen goldens and the reference itself.

* torch RNG goldens (copied from the reference's ``tests/reference_values.json``)
  for every seed/shape the reference's own suite checks;
* stage goldens produced by running the reference on the small synthetic model
  (``tests/golden/make_golden.py``);
* when the reference checkout is present: op-by-op agreement with
  ``cv3cpu.ops``/``cv3cpu.quant``, and the frozen upstream outputs of
  ``tests/fixtures/reference_io.npz`` through the converted tiny checkpoint.
"""

import os
import sys

import numpy as np
import pytest

from conftest import REFERENCE, have_reference, pkg, rel_err

import oracle.numerics as nx
import oracle.stages as st


def _check_golden(g, arr):
    flat = np.asarray(arr, dtype=np.float64).reshape(-1)
    assert list(np.shape(arr)) == g["shape"]
    got = np.array([flat[i] for i in g["idx"]])
    assert np.abs(got - np.array(g["vals"])).max() < 1e-5
    assert abs(flat.sum() - g["sum"]) < 1e-2 * max(1.0, abs(g["sum"]))


@pytest.mark.parametrize("seed", [0, 1, 42, 1986])
@pytest.mark.parametrize("shape", [(5,), (17,), (1000,), (1, 80, 15000)])
def test_oracle_randn_matches_torch_goldens(rng_golden, seed, shape):
    _check_golden(rng_golden[f"randn_{seed}_{'x'.join(map(str, shape))}"], nx.randn(shape, seed))


@pytest.mark.parametrize("seed", [0, 1, 42, 1986])
def test_oracle_rand_matches_torch_goldens(rng_golden, seed):
    _check_golden(rng_golden[f"rand_{seed}_1000"], nx.rand((1000,), seed))


def test_oracle_shared_generator_advances(rng_golden):
    g = nx.MT19937(0)
    first = nx.randn((1000,), gen=g)
    _check_golden(rng_golden["randn_0_1000"], first)
    assert not np.array_equal(first, nx.randn((1000,), gen=g))


# ---------------------------------------------------------------------------
# stage goldens from the reference run on the small synthetic model
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("profile", ["balanced", "f32"])
def test_oracle_lm_matches_reference_goldens(golden, small_weights, profile):
    W = small_weights[profile]
    lm = st.SpeechLM(W, W.meta)
    x0 = lm.prompt_embedding(golden[f"{profile}/lm_text"], (), golden[f"{profile}/lm_prompt_speech"])
    toks, logps = lm.generate_greedy(x0, 8)
    assert toks == golden[f"{profile}/lm_tokens"].tolist()
    assert rel_err(logps, golden[f"{profile}/lm_logp"]) < 1e-5


@pytest.mark.parametrize("profile", ["balanced", "f32"])
def test_oracle_flow_matches_reference_goldens(golden, small_weights, profile):
    W = small_weights[profile]
    g = lambda k: golden[f"{profile}/flow_{k}"]  # noqa: E731
    mel = st.Flow(W, W.meta).inference(g("token"), g("prompt_token"), g("prompt_feat"), g("embedding"))
    assert mel.shape == g("mel").shape
    assert rel_err(mel, g("mel")) < 1e-5


@pytest.mark.parametrize("profile", ["balanced", "f32"])
def test_oracle_hift_matches_reference_goldens(golden, small_weights, profile):
    W = small_weights[profile]
    h = st.HiFT(W, W.meta)
    mel = golden[f"{profile}/hift_mel"]
    assert rel_err(h.inference(mel, chunk=None), golden[f"{profile}/hift_wav"]) < 1e-5
    assert rel_err(h.inference(mel, chunk=4, context=64), golden[f"{profile}/hift_wav_chunked"]) < 1e-5


# ---------------------------------------------------------------------------
# live reference (this container only)
# ---------------------------------------------------------------------------

needs_ref = pytest.mark.skipif(not have_reference(), reason="reference checkout not present")


@pytest.fixture(scope="module")
def ref():
    sys.path.insert(0, REFERENCE)
    import cv3cpu.ops as rops
    import cv3cpu.quant as rquant
    import cv3cpu.torch_rng as rrng
    return rops, rquant, rrng


@needs_ref
def test_oracle_ops_equal_reference_ops(ref):
    rops, rquant, _ = ref
    rng = np.random.default_rng(0)
    x = (rng.normal(size=(7, 33)) * 3).astype(np.float32)
    for name in ("silu", "sigmoid", "gelu_tanh", "gelu", "mish", "elu", "softmax", "log_softmax"):
        assert np.array_equal(getattr(nx, name)(x), getattr(rops, name)(x)), name
    assert np.array_equal(nx.leaky_relu(x, 0.1), rops.leaky_relu(x, 0.1))
    a = np.abs(rng.normal(size=7)).astype(np.float32) + 0.5
    assert np.array_equal(nx.snake(x, a), rops.snake(x, a))
    w = rng.normal(size=33).astype(np.float32)
    assert np.array_equal(nx.rms_norm(x, w), rops.rms_norm(x, w))
    assert np.array_equal(nx.layer_norm(x, None, None, 1e-6), rops.layer_norm(x, None, None, 1e-6))
    wq = rng.normal(size=(40, 100)).astype(np.float32)
    qa, sa, _ = nx.quantize_q8(wq)
    qb, sb, _ = rquant.quantize_q8(wq)
    assert np.array_equal(qa, qb) and np.array_equal(sa, sb)
    qt = rquant.QTensor("q8", qb, sb, (40, 100), 64)
    xx = rng.normal(size=(3, 100)).astype(np.float32)
    assert rel_err(nx.qmatmul(xx, qt), rquant.qmatmul(xx, qt)) < 1e-6
    xc = rng.normal(size=(18, 61)).astype(np.float32)
    wc = (rng.normal(size=(8, 18, 30)) * 0.1).astype(np.float32)
    assert rel_err(nx.conv1d(xc, wc, None, stride=15, pad=(14, 0)),
                   rops.conv1d(xc, wc, None, stride=15, pad=(14, 0))) < 1e-6
    qh, kh, vh = (rng.normal(size=(4, 23, 16)).astype(np.float32) for _ in range(3))
    for spec in (None, ("causal",), ("causal", 3), ("chunk", 5, 1)):
        assert rel_err(nx.sdpa(qh, kh, vh, spec), rops.sdpa(qh, kh, vh, spec)) < 1e-6
    win = nx.hann_window(16)
    sig = rng.normal(size=400).astype(np.float32)
    assert np.array_equal(nx.stft(sig, 16, 4, win), rops.stft(sig, 16, 4, win))
    spec = nx.stft(sig, 16, 4, win)
    assert np.array_equal(nx.istft(spec, 16, 4, win), rops.istft(spec, 16, 4, win))


@needs_ref
def test_oracle_rng_equals_reference_rng_on_the_flow_buffer(ref):
    _, _, rrng = ref
    assert np.array_equal(nx.randn((1, 80, 15000), 0), rrng.randn((1, 80, 15000), 0))
    assert np.array_equal(nx.MT19937(0).random_float32(4800 * 9), rrng.TorchMT19937(0).random_float32(4800 * 9))
    for n in (1, 5, 17, 33):
        assert np.array_equal(nx.randn((n,), 7), rrng.randn((n,), 7))


@needs_ref
def test_oracle_matches_frozen_upstream_outputs(tmp_path):
    """The reference's own pin (tests/test_reference.py:99-155): the converted tiny
    checkpoint through the oracle's stages against upstream PyTorch outputs."""
    sys.path.insert(0, REFERENCE)
    from cv3cpu.convert import convert
    from conftest import pkg
    path = str(tmp_path / "tiny.safetensors")
    convert(os.path.join(REFERENCE, "tests", "fixtures", "checkpoint"), path, profile="f32", verbose=False)
    W = pkg("weights").WeightFile(path)
    io = dict(np.load(os.path.join(REFERENCE, "tests", "fixtures", "reference_io.npz")))
    mel = st.Flow(W, W.meta).inference(io["token"], io["prompt_token"], io["prompt_feat"], io["embedding"])
    assert rel_err(mel, io["flow_mel"]) < 5e-4
    h = st.HiFT(W, W.meta)
    n = 480 * io["mel"].shape[1]
    h.set_source_noise(nx.MT19937(0).random_float32(n * 9).reshape(n, 9))
    assert rel_err(h.inference(io["mel"], chunk=None), io["hift_wav"]) < 2e-3
    lm = st.SpeechLM(W, W.meta)
    x = np.concatenate([lm.speech_emb([lm.sos]), lm.text_emb(io["text"]), lm.speech_emb([lm.task_id]),
                        lm.speech_emb(io["prompt_speech"])], axis=0)
    cache = lm.body.new_cache()
    forced = list(io["forced"])
    for i, refl in enumerate(io["llm_logits"]):
        got = lm.head(lm.body.forward(x, cache)[-1:])[0]
        assert rel_err(got, refl) < 1e-3, i
        if i < len(forced):
            x = lm.speech_emb([int(forced[i])])
    W.close()


@pytest.mark.skipif(not have_reference(), reason="reference checkout not present")
@pytest.mark.parametrize("strict", [False, True])
def test_oracle_sampler_matches_reference(strict):
    """The oracle's sampler against CosyVoice3LM._sample (llm.py:125-149) itself: same
    tokens and the same random stream over 300 steps with stops, masking and repeats."""
    sys.path.insert(0, REFERENCE)
    from cv3cpu.models import llm as rl
    sts = 6561
    ref = rl.CosyVoice3LM.__new__(rl.CosyVoice3LM)
    ref.speech_token_size = sts
    ref.stop_token_ids = set(range(sts, sts + 200))
    cfg = rl.SamplingConfig(seed=11)
    rng = np.random.default_rng(11)
    data = np.random.default_rng(5)
    decoded = []
    for i in range(300):
        logits = (data.normal(size=6761) * 3.0).astype(np.float32)
        logp = nx.log_softmax(logits)
        ign = i % 7 < 3
        a = ref._sample(logp, decoded, cfg, ign, strict)
        b = nx.sample_token(logp, decoded, rng, sts, ign, strict)
        assert a == b, i
        decoded.append(a)
    assert cfg.rng.bit_generator.state == rng.bit_generator.state


@pytest.mark.skipif(not have_reference(), reason="reference checkout not present")
def test_oracle_q4_matches_reference():
    """q4 ('tiny' profile) writer and expansion: byte-identical payload and scales to
    cv3cpu.quant.quantize_q4 (quant.py:70-86), identical rows to QTensor.dequant_rows."""
    sys.path.insert(0, REFERENCE)
    from cv3cpu import quant as rq
    rng = np.random.default_rng(8)
    for n, k in [(37, 96), (64, 100), (5, 31)]:
        w = (rng.normal(size=(n, k)) * 0.05).astype(np.float32)
        w[0, :5] = 0.0
        w[1, :32] = 0.0                       # an all-zero block
        w[2, 3] = -w[2, :32].__abs__().max()  # negative extreme
        q, s, kp = nx.quantize_q4(w)
        rq_q, rq_s, rq_kp = rq.quantize_q4(w)
        assert kp == rq_kp and np.array_equal(q, rq_q) and np.array_equal(s, rq_s)
        ref = rq.QTensor("q4", rq_q, rq_s, (n, k), rq.Q4_BLOCK).dequant()
        got = nx.dequant(nx.QTensor("q4", q, s, (n, k), nx.Q4_BLOCK))
        assert np.array_equal(ref, got)


@pytest.mark.skipif(not have_reference(), reason="reference checkout not present")
@pytest.mark.parametrize("profile", ["balanced", "f32"])
def test_oracle_sampled_generation_matches_reference(tmp_path, profile):
    """The oracle's sampling loop against CosyVoice3LM.generate (llm.py:80-123) on the small
    synthetic model read through the reference's own weight reader: identical tokens
    (stops, min/max lengths, repetition redraws) and the generator left in the same state."""
    sys.path.insert(0, REFERENCE)
    from cv3cpu.io.weights import WeightFile as RefWF
    from cv3cpu.models import llm as rl
    W = pkg("weights")
    syn = pkg("synth").synthetic_weights(profile, small=True, stages=("llm",))
    path = str(tmp_path / "lm.safetensors")
    W.write_weights(path, dict(syn), syn.meta)
    ref = rl.CosyVoice3LM(RefWF(path))
    olm = st.SpeechLM(syn, syn.meta)
    eop = syn.meta["endofprompt_id"]
    data = np.random.default_rng(2)
    total = 0
    # (min ratio, strict): the small model's 200 stop ids are a large share of its speech
    # vocabulary, so most trials mask all of them up to min_len to get long samples
    for trial, (lo, strict) in enumerate([(2.0, True), (3.0, True), (1.0, False), (2.5, True), (1.5, True)]):
        text = data.integers(0, 2000, size=6 + 3 * trial).tolist()
        prompt_text = [eop]
        speech = data.integers(0, 256, size=4).tolist()
        cfg = rl.SamplingConfig(seed=30 + trial, max_token_text_ratio=4.0, min_token_text_ratio=lo)
        want = list(ref.generate(text, prompt_text, speech, sampling=cfg, strict_min_len=strict))
        rng = np.random.default_rng(30 + trial)
        got = olm.generate_sampled(olm.prompt_embedding(text, prompt_text, speech), len(text), rng, lo, 4.0, strict)
        assert got == want, trial
        assert rng.bit_generator.state == cfg.rng.bit_generator.state
        total += len(want)
    assert total >= 60


# ---- the same pins from committed fixtures (tests/golden/sampling_small.npz, written by
# ---- make_golden.py from the reference): they run without the reference checkout

def _sampling_golden():
    from conftest import GOLDEN
    sys.path.insert(0, GOLDEN)
    import make_golden
    with np.load(os.path.join(GOLDEN, "sampling_small.npz")) as z:
        return {k: z[k] for k in z.files}, make_golden


def test_oracle_q4_matches_reference_golden():
    g, _ = _sampling_golden()
    q, s, kp = nx.quantize_q4(g["q4_w"])
    assert np.array_equal(q, g["q4_q"]) and np.array_equal(s, g["q4_scales"]) and kp == int(g["q4_kp"])


@pytest.mark.parametrize("strict", [False, True])
def test_oracle_sampler_matches_reference_golden(strict):
    g, mg = _sampling_golden()
    rng = np.random.default_rng(11)
    data = np.random.default_rng(5)
    decoded = []
    for i in range(200):
        logp = nx.log_softmax(mg.sampler_logits(data))
        decoded.append(nx.sample_token(logp, decoded, rng, 6561, i % 7 < 3, strict))
    assert decoded == g[f"sampler_{int(strict)}_tokens"].tolist()
    st = rng.bit_generator.state["state"]
    assert [str(st["state"]), str(st["inc"])] == g[f"sampler_{int(strict)}_state"].tolist()


def test_oracle_sampled_generation_matches_reference_golden():
    g, mg = _sampling_golden()
    syn = pkg("synth").synthetic_weights("balanced", small=True, stages=("llm",))
    olm = st.SpeechLM(syn, syn.meta)
    eop = syn.meta["endofprompt_id"]
    total = 0
    for trial, (lo, strict) in enumerate(mg.SAMPLED_TRIALS):
        text, speech = g[f"generate_{trial}_text"].tolist(), g[f"generate_{trial}_speech"].tolist()
        got = olm.generate_sampled(olm.prompt_embedding(text, [eop], speech), len(text),
                                   np.random.default_rng(30 + trial), lo, 4.0, strict)
        assert got == g[f"generate_{trial}_tokens"].tolist(), trial
        total += len(got)
    assert total >= 60


@pytest.mark.skipif(not have_reference(), reason="reference checkout not present")
def test_oracle_q4_lm_matches_reference(tmp_path):
    """The small LM with every body linear and the token table in q4 (the 'tiny' storage),
    written with this package's writer and run by the reference (cv3cpu.quant q4 path,
    quant.py:110-133 + 156-204) and by the oracle: log-probabilities within 1e-5 and the
    same greedy tokens over 8 steps."""
    sys.path.insert(0, REFERENCE)
    from cv3cpu import ops as rops
    from cv3cpu.io.weights import WeightFile as RefWF
    from cv3cpu.models import llm as rl
    Q, W = pkg("quant"), pkg("weights")
    syn = pkg("synth").synthetic_weights("f32", small=True, stages=("llm",))
    tensors = dict(syn)
    for name, t in syn.items():
        if name.startswith("llm.model.layers.") and name.endswith("proj.weight") or name == "llm.model.embed_tokens":
            tensors[name] = Q.make_qtensor(t, kind="q4")
    path = str(tmp_path / "tiny.safetensors")
    W.write_weights(path, tensors, syn.meta)
    ref = rl.CosyVoice3LM(RefWF(path))
    Wt = W.TensorDict(tensors, syn.meta)
    olm = st.SpeechLM(Wt, Wt.meta)
    eop = syn.meta["endofprompt_id"]
    text, speech = [eop] + list(range(30, 39)), [4, 5, 6]
    x = np.concatenate([ref._speech_emb([ref.sos]), ref._text_emb(text), ref._speech_emb([ref.task_id]),
                        ref._speech_emb(speech)], axis=0).astype(np.float32)
    assert rel_err(olm.prompt_embedding(text, (), speech), x) < 1e-6
    cache = ref.body.new_cache()
    toks, logps = [], []
    for _ in range(8):
        h = ref.body.forward(x, cache)
        logp = rops.log_softmax(ref._head(h[-1:]).astype(np.float32), axis=-1)[0]
        top = int(np.argmax(logp[: ref.speech_token_size]))
        toks.append(top)
        logps.append(logp)
        x = ref._speech_emb([top])
    otoks, ologps = olm.generate_greedy(olm.prompt_embedding(text, (), speech), 8)
    assert otoks == toks
    assert rel_err(ologps, np.stack(logps)) < 1e-5


# ---------------------------------------------------------------------------
# full benchmark geometry (tests/golden/full_size.npz, made by the reference)
# ---------------------------------------------------------------------------

@pytest.fixture(scope="module")
def full_golden():
    with np.load(os.path.join(os.path.dirname(__file__), "golden", "full_size.npz")) as z:
        return {k: z[k] for k in z.files}


def test_oracle_vocoder_matches_reference_at_500_frames(full_golden):
    """Config 3 (f32 vocoder, 500 frames): the oracle's F0 and waveform against the
    reference's, at the full geometry."""
    wl = pkg("workloads")
    W = pkg("synth").synthetic_weights("f32", stages=("hift",))
    h = st.HiFT(W, W.meta)
    mel = wl.vocoder_mel(1)
    f0 = h.f0_predict(mel)
    assert rel_err(f0, full_golden["c3_f0"]) < 1e-6
    assert np.array_equal(f0 > 10.0, full_golden["c3_f0"] > 10.0)
    assert rel_err(h.inference(mel), full_golden["c3_wav"]) < 1e-6


@needs_ref
def test_reference_f0_condnet_runs_in_float32():
    """The reference's F0 predictor hands float64 arrays to ``ops.conv1d``
    (cv3cpu/models/hift.py:56-72), but ``conv1d`` casts input and weight to float32
    and returns float32 (cv3cpu/ops.py:183, :186, :198), and ``elu`` keeps float32:
    the five condnet convolutions run in float32 and only the classifier dot product
    is float64.  The device path reproduces exactly that."""
    sys.path.insert(0, REFERENCE)
    from cv3cpu import ops as rops
    rng = np.random.default_rng(0)
    x = rng.normal(size=(80, 40))                       # float64, as f0_predict passes it
    w = rng.normal(size=(512, 80, 4))
    b = rng.normal(size=512)
    y = rops.conv1d(x, w, b, pad=(0, 3))
    assert y.dtype == np.float32 and rops.elu(y).dtype == np.float32
    y32 = rops.conv1d(x.astype(np.float32), w.astype(np.float32), b.astype(np.float32), pad=(0, 3))
    assert np.array_equal(y, y32)
