"""Parity at the benchmark geometry, against fixtures the reference itself made
(``tests/golden/full_size.npz``, written by ``make_golden.py --only full`` from
the same seeded weights and inputs).

* config 1 -- Qwen2-0.5B LM in the balanced int8 form: 250 greedy ids from a
  64-id prompt must be identical; log-probabilities at four steps within 1e-4
  (the int8 path's bar).  A differing id is reported with the reference's
  top-two log-prob margin at that step (near ties can flip under a different
  summation order; the margin shows whether that happened).
* config 2 -- f32 DiT, 22 x 1024: one forward at batch 2 x 500 frames within
  1e-5; the 10-step CFG flow solve of 250 tokens within 1e-5.
* config 3 -- f32 vocoder, 500 frames: F0 within 1e-5 with an identical voiced
  mask (F0 > 10), the waveform within 1e-5 (whole-utterance decode against the
  reference's default 250-frame chunked inference).
* config 4 -- one utterance through the balanced LM, flow and vocoder: ids
  identical, mel within 1e-4, waveform within 1e-4 (three stages compounded).
* config 5 -- the balanced DiT at CFG batch 2 x 1500 frames within 1e-5 of the
  reference; batch-32 greedy decode identical to batch-1 decode per sequence.
"""

import os

import numpy as np
import pytest

from conftest import GOLDEN, pkg, rel_err

pytestmark = pytest.mark.gpu

FP32_TOL = 1e-5
INT8_TOL = 1e-4


@pytest.fixture(scope="module")
def full():
    with np.load(os.path.join(GOLDEN, "full_size.npz")) as z:
        return {k: z[k] for k in z.files}


def _device(W):
    return pkg("weights").DeviceWeights(W)


def _greedy(lm, x0, steps, logp_steps=()):
    """Batch-1 greedy decode through the graph-replayed engine: ids and the log-prob rows."""
    eng = lm.engine(1, 1024, steps)
    eng.keep_logp = bool(logp_steps)
    eng.prefill([x0])
    rows = {}
    if 0 in logp_steps:
        rows[0] = eng.logp[0].cpu().numpy().copy()
    if eng.graph is None and steps > 1:
        state = (eng.h, eng.pos, eng.lens, eng.step_no, eng.next_ids, eng.history)
        saved = [t.clone() for t in state]
        eng.capture()
        for t, s in zip(state, saved):
            t.copy_(s)
    for i in range(1, steps):
        eng.step()
        if i in logp_steps:
            rows[i] = eng.logp[0].cpu().numpy().copy()
    return eng.history[0, :steps].cpu().numpy(), rows


def _first_flip(got, ref, margin):
    bad = np.nonzero(np.asarray(got) != np.asarray(ref))[0]
    if bad.size == 0:
        return ""
    i = int(bad[0])
    return (f"first differing id at step {i}: device {int(got[i])} vs reference {int(ref[i])}, "
            f"reference top-two log-prob margin there {float(margin[i]):.3e}")


def test_config1_lm_250_greedy_ids_and_logp(full):
    wl = pkg("workloads")
    W = pkg("synth").synthetic_weights("balanced", stages=("llm",))
    lm = pkg("models.llm").CosyVoice3LM(_device(W))
    x0 = lm._text_emb(wl.lm_prompt_ids(0, vocab=W.meta["qwen2"]["vocab_size"]))
    steps = [int(s) for s in full["c1_logp_steps"]]
    ids, rows = _greedy(lm, x0, wl.LM_STEPS, steps)
    assert ids.tolist() == full["c1_tokens"].tolist(), _first_flip(ids, full["c1_tokens"], full["c1_margin"])
    for j, s in enumerate(steps):
        assert rel_err(rows[s], full["c1_logp"][j]) < INT8_TOL, s


def test_config2_dit_forward_batch2_500_frames(full):
    wl = pkg("workloads")
    W = pkg("synth").synthetic_weights("f32", stages=("flow",))
    got = pkg("models.dit").DiT(_device(W)).forward(*wl.dit_inputs(2))
    assert got.shape == full["c2_dit_out"].shape
    assert rel_err(got, full["c2_dit_out"]) < FP32_TOL


def test_config2_flow_solve_250_tokens(full):
    wl = pkg("workloads")
    W = pkg("synth").synthetic_weights("f32", stages=("flow",))
    tokens, emb = wl.flow_inputs(0)
    mel = pkg("models.flow").Flow(_device(W)).inference(tokens, np.zeros(0, np.int64), np.zeros((0, 80), np.float32),
                                                        emb)
    assert mel.shape == full["c2_mel"].shape == (80, 500)
    assert rel_err(mel, full["c2_mel"]) < FP32_TOL


def test_config3_vocoder_500_frames_f0_and_waveform(full):
    wl = pkg("workloads")
    D = pkg("_dev")
    W = pkg("synth").synthetic_weights("f32", stages=("hift",))
    h = pkg("models.hift").HiFTGenerator(_device(W))
    mel = wl.vocoder_mel(1)
    f0 = h.f0_predict(D.dev(mel)[None]).cpu().numpy()[0]
    ref_f0 = full["c3_f0"]
    assert rel_err(f0, ref_f0) < FP32_TOL
    assert np.array_equal(f0 > 10.0, ref_f0 > 10.0)
    wav = h.inference(mel)
    assert wav.shape == full["c3_wav"].shape == (240000,)
    assert rel_err(wav, full["c3_wav"]) < FP32_TOL
    # the exact time-chunked decode (200-frame chunks, 64 frames of context) as well
    assert rel_err(h.inference(mel, chunk=200, context=64), full["c3_wav"]) < FP32_TOL


def test_config4_one_utterance_through_three_balanced_stages(full):
    wl = pkg("workloads")
    W = pkg("synth").synthetic_weights("balanced")
    tts = pkg("pipeline").CosyVoice3CUDA(W)
    req = wl.requests([0], W.meta)[0]
    wav, toks = tts.synthesize_greedy_batch([req], wl.LM_STEPS, to_host=True)
    assert toks[0].tolist() == full["c4_tokens"].tolist(), _first_flip(toks[0], full["c4_tokens"], full["c4_margin"])
    mel = tts.flow.inference(full["c4_tokens"], req.voice.speech_token, req.voice.mel, req.voice.embedding)
    assert rel_err(mel, full["c4_mel"]) < INT8_TOL
    assert wav.shape == (1, 240000)
    assert rel_err(wav[0], full["c4_wav"]) < INT8_TOL


def test_config1_persistent_decode_250_ids(full):
    """The persistent decode kernel (every step in one launch, weights streamed into shared
    memory ahead of the layer chain) on config 1: the reference's 250 greedy ids, and the
    last step's log-probabilities within 1e-4."""
    import ctypes
    wl = pkg("workloads")
    W = pkg("synth").synthetic_weights("balanced", stages=("llm",))
    lm = pkg("models.llm").CosyVoice3LM(_device(W))
    x0 = lm._text_emb(wl.lm_prompt_ids(0, vocab=W.meta["qwen2"]["vocab_size"]))
    eng = lm.engine(1, 512, wl.LM_STEPS)
    assert eng.persistent_ok
    eng.keep_logp = True
    ids = eng.run([x0], wl.LM_STEPS, persistent=True).cpu().numpy()[0]
    code = ctypes.c_int(-1)
    assert pkg("_lib").load().cv3_decode_status(ctypes.byref(code)) == 0 and code.value == 0
    assert ids.tolist() == full["c1_tokens"].tolist(), _first_flip(ids, full["c1_tokens"], full["c1_margin"])
    assert rel_err(eng.logp[0].cpu().numpy(), full["c1_logp"][-1]) < INT8_TOL


def test_config5_dit_forward_batch2_1500_frames():
    """Config 5's flow length: one forward of the balanced DiT (int8-weight GEMMs on
    activation planes, attention over 1500 keys) at CFG batch 2 x 1500 frames against the
    reference's own output (``config5_dit.npz``, ``make_golden.py --only c5``)."""
    wl = pkg("workloads")
    with np.load(os.path.join(GOLDEN, "config5_dit.npz")) as z:
        ref = z["c5_dit_out"]
    W = pkg("synth").synthetic_weights("balanced", stages=("flow",))
    dit = pkg("models.dit").DiT(_device(W))
    got = dit.forward(*wl.dit_inputs(5, 2, 1500))
    assert type(dit.blocks[0].ff1).__name__ == "LinQ8"
    assert got.shape == ref.shape == (2, 80, 1500)
    assert rel_err(got, ref) < FP32_TOL


def test_config5_lm_batch32_ids_equal_batch1():
    """Config 5 decodes 32 sequences per GPU: the full-size balanced LM on 32 prompts of
    40-80 text ids (one graph-replayed batch of 32: the decode GEMV streams each weight once
    for all 32 rows) gives every sequence exactly the ids it gets when decoded alone."""
    W = pkg("synth").synthetic_weights("balanced", stages=("llm",))
    lm = pkg("models.llm").CosyVoice3LM(_device(W))
    rng = np.random.default_rng(32)
    vocab = W.meta["qwen2"]["vocab_size"]
    prompts = [lm._text_emb(rng.integers(0, vocab, size=int(rng.integers(40, 81))).tolist()) for _ in range(32)]
    steps = 40
    batch = lm.generate_greedy(prompts, steps).cpu().numpy()
    assert batch.shape == (32, steps)
    for i, p in enumerate(prompts):
        alone = lm.generate_greedy([p], steps).cpu().numpy()[0]
        assert alone.tolist() == batch[i].tolist(), i
