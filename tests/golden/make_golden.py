"""Regenerate the golden fixtures in this directory from the reference itself.

Run in a checkout that has the reference project importable (its root on
``--reference``); the GPU box never runs this.  It writes:

* ``torch_rng.json`` -- the torch RNG samples the reference's own test suite
  pins (``tests/reference_values.json["torch_rng"]`` of the reference).
* ``stages_small.npz`` -- outputs of the reference's model classes on the
  small synthetic geometry (this package's ``synth.synthetic_weights(small=True)``,
  written with this package's writer and read back with the reference's
  ``WeightFile``): LM log-probabilities and greedy tokens over 8 decode steps,
  a flow mel, and vocoder waveforms (whole and time-chunked), for the
  ``balanced`` (q8) and ``f32`` profiles.  Inputs are seeded and stored beside
  the outputs.

* ``sampling_small.npz`` -- the reference's q4 writer on a seeded matrix
  (``quant.quantize_q4``), 200 steps of its sampler (``CosyVoice3LM._sample``
  on log-probabilities of seeded logits, with stops, min-length masking in both
  modes and repetition redraws) with the final generator state, and its sampled
  ``generate`` on the small ``balanced`` model.  The seeds that regenerate the
  inputs are stored beside the outputs.

* ``full_size.npz`` (``--only full``) -- the reference's model classes at the
  benchmark geometry, on the seeded inputs of this package's ``workloads``
  module: config 1 (balanced Qwen2-0.5B LM, 64-id prompt, 250 greedy steps:
  ids, the top-two log-prob margin of every step and four log-prob rows),
  config 2 (f32 DiT: one forward at batch 2 x 500 frames and the 10-step CFG
  flow solve of 250 tokens), config 3 (f32 vocoder, 500 frames: F0 and the
  waveform the default chunked inference returns) and one config-4 utterance
  through all three balanced stages (ids, mel, waveform).

* ``config5_dit.npz`` (``--only c5``) -- one forward of the reference's DiT in the
  balanced profile at config 5's flow length: CFG batch 2 x 1500 frames
  (``workloads.dit_inputs(5, 2, 1500)``).

It also asserts that the synthetic generator reproduces the reference's own
random-model generator tensor for tensor.

    python tests/golden/make_golden.py --reference /path/to/cosyvoice3-cpu [--only sampling|full|c5]
"""

from __future__ import annotations

import argparse
import importlib
import json
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))


def _pkg(name):
    sys.path.insert(0, REPO)
    return importlib.import_module(f"cosyvoice3-cpu_b200.{name}")


def lm_inputs(seed: int, vocab: int, eop: int, speech: int):
    rng = np.random.default_rng(seed)
    text = [eop] + rng.integers(0, vocab - 1, size=9).tolist()
    prompt_speech = rng.integers(0, speech, size=5).tolist()
    return np.array(text, np.int64), np.array(prompt_speech, np.int64)


def flow_inputs(seed: int, speech: int):
    rng = np.random.default_rng(seed)
    return (rng.integers(0, speech, size=12).astype(np.int64), rng.integers(0, speech, size=4).astype(np.int64),
            rng.normal(size=(8, 80)).astype(np.float32), rng.normal(size=192).astype(np.float32))


def hift_mel(seed: int, frames: int):
    rng = np.random.default_rng(seed)
    return np.clip(rng.normal(-5.0, 2.0, size=(80, frames)), -11.5, 2.0).astype(np.float32)


def sampler_logits(data, vocab: int = 6761):
    """Seeded, peaked logits of one sampler step (shared with the tests)."""
    x = (data.normal(size=vocab) * 3.0).astype(np.float32)
    x[data.integers(0, 40, size=4)] += 6.0
    return x


SAMPLED_TRIALS = [(2.0, True), (3.0, True), (1.0, False), (2.5, True), (1.5, True)]


def make_sampling(reference: str) -> None:
    from cv3cpu import ops, quant
    from cv3cpu.io.weights import WeightFile
    from cv3cpu.models import llm as rl
    out = {}
    # q4 writer
    w = (np.random.default_rng(8).normal(size=(37, 96)) * 0.05).astype(np.float32)
    w[1, :32] = 0.0
    q, sc, kp = quant.quantize_q4(w)
    out["q4_w"], out["q4_q"], out["q4_scales"], out["q4_kp"] = w, q, sc, np.int64(kp)
    # 200 sampler steps per mode: logits from data seed 5, generator seed 11, ignore_eos when i % 7 < 3
    sts = 6561
    ref = rl.CosyVoice3LM.__new__(rl.CosyVoice3LM)
    ref.speech_token_size = sts
    ref.stop_token_ids = set(range(sts, sts + 200))
    for strict in (False, True):
        cfg = rl.SamplingConfig(seed=11)
        data = np.random.default_rng(5)
        decoded = []
        for i in range(200):
            logp = ops.log_softmax(sampler_logits(data))
            decoded.append(ref._sample(logp, decoded, cfg, i % 7 < 3, strict))
        st = cfg.rng.bit_generator.state["state"]
        out[f"sampler_{int(strict)}_tokens"] = np.array(decoded, np.int64)
        out[f"sampler_{int(strict)}_state"] = np.array([str(st["state"]), str(st["inc"])])
    # sampled generation on the small balanced model (text / speech from data seed 2)
    syn = _pkg("synth").synthetic_weights("balanced", small=True, stages=("llm",))
    path = os.path.join(tempfile.mkdtemp(), "lm.safetensors")
    _pkg("weights").write_weights(path, dict(syn), syn.meta)
    lm = rl.CosyVoice3LM(WeightFile(path))
    eop = syn.meta["endofprompt_id"]
    data = np.random.default_rng(2)
    for trial, (lo, strict) in enumerate(SAMPLED_TRIALS):
        text = data.integers(0, 2000, size=6 + 3 * trial).tolist()
        speech = data.integers(0, 256, size=4).tolist()
        cfg = rl.SamplingConfig(seed=30 + trial, max_token_text_ratio=4.0, min_token_text_ratio=lo)
        toks = list(lm.generate(text, [eop], speech, sampling=cfg, strict_min_len=strict))
        out[f"generate_{trial}_text"] = np.array(text, np.int64)
        out[f"generate_{trial}_speech"] = np.array(speech, np.int64)
        out[f"generate_{trial}_tokens"] = np.array(toks, np.int64)
    np.savez_compressed(os.path.join(HERE, "sampling_small.npz"), **out)
    print("wrote sampling_small.npz", sorted(out))


LOGP_STEPS = (0, 1, 125, 249)


def greedy_reference(lm, x, steps: int):
    """The build's greedy decode written with the reference's pieces: body forward,
    ``_head``, ``log_softmax`` (llm.py:112-114), first argmax over the speech tokens,
    next input ``_speech_emb([top])``.  Returns ids, per-step top-two margins and the
    log-prob rows of LOGP_STEPS."""
    from cv3cpu import ops
    cache = lm.body.new_cache()
    ids, margins, rows = [], [], []
    for i in range(steps):
        h = lm.body.forward(x, cache)
        logp = ops.log_softmax(lm._head(h[-1:]).astype(np.float32), axis=-1)[0]
        sp = logp[: lm.speech_token_size]
        top = int(np.argmax(sp))
        two = np.partition(sp, -2)[-2:]
        ids.append(top)
        margins.append(float(two[1] - two[0]))
        if i in LOGP_STEPS:
            rows.append(logp.copy())
        x = lm._speech_emb([top])
        if i % 50 == 0:
            print(f"  greedy step {i}", flush=True)
    return np.array(ids, np.int64), np.array(margins, np.float32), np.stack(rows).astype(np.float32)


def make_full(reference: str) -> None:
    """Full-geometry fixtures (see the module docstring).  About 10 minutes of CPU."""
    from cv3cpu.io.weights import WeightFile
    from cv3cpu.models.dit import DiT
    from cv3cpu.models.flow import Flow
    from cv3cpu.models.hift import HiFTGenerator
    from cv3cpu.models.llm import CosyVoice3LM
    synth, weights, wl = _pkg("synth"), _pkg("weights"), _pkg("workloads")
    tmp = tempfile.mkdtemp()
    out = {}

    def written(profile, stages):
        W = synth.synthetic_weights(profile, stages=stages)
        path = os.path.join(tmp, f"{profile}_{'_'.join(stages)}.safetensors")
        weights.write_weights(path, dict(W), W.meta)
        return WeightFile(path), W.meta

    # ---- config 1: balanced LM, 64-id prompt, 250 greedy steps
    f, meta = written("balanced", ("llm",))
    lm = CosyVoice3LM(f, "llm.")
    ids = wl.lm_prompt_ids(0, vocab=meta["qwen2"]["vocab_size"])
    x0 = lm._text_emb(ids).astype(np.float32)
    print("config 1: LM", flush=True)
    toks, margins, rows = greedy_reference(lm, x0, wl.LM_STEPS)
    out["c1_tokens"], out["c1_margin"], out["c1_logp"] = toks, margins, rows
    out["c1_logp_steps"] = np.array(LOGP_STEPS, np.int64)
    f.close()

    # ---- config 2: f32 DiT forward at (2, 80, 500), and the 10-step flow solve
    f, meta = written("f32", ("flow",))
    print("config 2: DiT forward + flow solve", flush=True)
    dit = DiT(f, "flow.decoder.estimator.")
    out["c2_dit_out"] = dit.forward(*wl.dit_inputs(2)).astype(np.float32)
    tokens, emb = wl.flow_inputs(0)
    out["c2_mel"] = Flow(f, "flow.").inference(tokens, np.zeros(0, np.int64), np.zeros((0, 80), np.float32),
                                               emb).astype(np.float32)
    f.close()

    # ---- config 3: f32 vocoder, 500 frames
    f, meta = written("f32", ("hift",))
    print("config 3: vocoder", flush=True)
    hift = HiFTGenerator(f, "hift.")
    mel = wl.vocoder_mel(1)
    out["c3_f0"] = hift.f0_predict(mel)
    out["c3_wav"] = hift.inference(mel).astype(np.float32)
    f.close()

    # ---- config 4: one utterance (seed 0) through the three balanced stages
    f, meta = written("balanced", ("llm", "flow", "hift"))
    print("config 4: chain", flush=True)
    req = wl.requests([0], meta)[0]
    v = req.voice
    lm = CosyVoice3LM(f, "llm.")
    text = list(req.prompt_ids) + list(req.text_ids)
    x0 = np.concatenate([lm._speech_emb([lm.sos]), lm._text_emb(text), lm._speech_emb([lm.task_id]),
                         lm._speech_emb(v.speech_token.tolist())], axis=0).astype(np.float32)
    toks, margins, _ = greedy_reference(lm, x0, wl.LM_STEPS)
    out["c4_tokens"], out["c4_margin"] = toks, margins
    mel = Flow(f, "flow.").inference(toks, v.speech_token, v.mel, v.embedding).astype(np.float32)
    out["c4_mel"] = mel
    out["c4_wav"] = HiFTGenerator(f, "hift.").inference(mel).astype(np.float32)
    f.close()
    np.savez_compressed(os.path.join(HERE, "full_size.npz"), **out)
    print("wrote full_size.npz", {k: v.shape for k, v in out.items()})


def make_c5(reference: str) -> None:
    """Config 5's DiT length (one forward, balanced profile, batch 2 x 1500 frames)."""
    from cv3cpu.io.weights import WeightFile
    from cv3cpu.models.dit import DiT
    synth, weights, wl = _pkg("synth"), _pkg("weights"), _pkg("workloads")
    tmp = tempfile.mkdtemp()
    W = synth.synthetic_weights("balanced", stages=("flow",))
    path = os.path.join(tmp, "balanced_flow.safetensors")
    weights.write_weights(path, dict(W), W.meta)
    f = WeightFile(path)
    print("config 5: DiT forward at (2, 80, 1500)", flush=True)
    out = {"c5_dit_out": DiT(f, "flow.decoder.estimator.").forward(*wl.dit_inputs(5, 2, 1500)).astype(np.float32)}
    f.close()
    np.savez_compressed(os.path.join(HERE, "config5_dit.npz"), **out)
    print("wrote config5_dit.npz", {k: v.shape for k, v in out.items()})


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="root of the reference checkout")
    ap.add_argument("--only", choices=["sampling", "full", "c5"], help="regenerate only this fixture")
    a = ap.parse_args()
    sys.path.insert(0, a.reference)
    sys.path.insert(0, os.path.join(a.reference, "tools"))
    if a.only == "sampling":
        make_sampling(a.reference)
        return
    if a.only == "full":
        make_full(a.reference)
        return
    if a.only == "c5":
        make_c5(a.reference)
        return
    from cv3cpu.io.weights import WeightFile
    from cv3cpu.models.flow import Flow
    from cv3cpu.models.hift import HiFTGenerator
    from cv3cpu.models.llm import CosyVoice3LM
    from cv3cpu import ops
    import make_dummy_model

    synth = _pkg("synth")
    weights = _pkg("weights")

    with open(os.path.join(a.reference, "tests", "reference_values.json")) as fh:
        rv = json.load(fh)
    with open(os.path.join(HERE, "torch_rng.json"), "w") as fh:
        json.dump(rv["torch_rng"], fh, indent=0, sort_keys=True)

    out = {}
    tmp = tempfile.mkdtemp()
    for profile in ("balanced", "f32"):
        W = synth.synthetic_weights(profile, small=True)
        path = os.path.join(tmp, f"{profile}.safetensors")
        weights.write_weights(path, dict(W), W.meta)
        ref_path = os.path.join(tmp, f"ref_{profile}.safetensors")
        make_dummy_model.build(ref_path, profile, small=True)
        mine, theirs = WeightFile(path), WeightFile(ref_path)
        assert sorted(mine.keys()) == sorted(theirs.keys())
        for name in theirs.keys():
            x, y = mine.get_f32(name), theirs.get_f32(name)
            assert x.shape == y.shape and np.array_equal(x, y), name
            assert mine.entry(name)["kind"] == theirs.entry(name)["kind"], name
        theirs.close()
        f = mine
        meta = f.meta
        # ---- LM: 8 greedy steps (argmax over the speech tokens, stop ids masked)
        lm = CosyVoice3LM(f, "llm.")
        text, pspeech = lm_inputs(1, meta["qwen2"]["vocab_size"], meta["endofprompt_id"], meta["speech_token_size"])
        x = np.concatenate([lm._speech_emb([lm.sos]), lm._text_emb(text), lm._speech_emb([lm.task_id]),
                            lm._speech_emb(pspeech)], axis=0).astype(np.float32)
        cache = lm.body.new_cache()
        toks, logps = [], []
        for _ in range(8):
            h = lm.body.forward(x, cache)
            logp = ops.log_softmax(lm._head(h[-1:]).astype(np.float32), axis=-1)[0]
            top = int(np.argmax(logp[: lm.speech_token_size]))
            toks.append(top)
            logps.append(logp)
            x = lm._speech_emb([top])
        out[f"{profile}/lm_text"] = text
        out[f"{profile}/lm_prompt_speech"] = pspeech
        out[f"{profile}/lm_tokens"] = np.array(toks, np.int64)
        out[f"{profile}/lm_logp"] = np.stack(logps).astype(np.float32)
        # ---- flow: 12 tokens + 4 prompt tokens, 8-frame prompt mel
        tok, ptok, pfeat, emb = flow_inputs(2, meta["speech_token_size"])
        mel = Flow(f, "flow.").inference(tok, ptok, pfeat, emb)
        out[f"{profile}/flow_token"] = tok
        out[f"{profile}/flow_prompt_token"] = ptok
        out[f"{profile}/flow_prompt_feat"] = pfeat
        out[f"{profile}/flow_embedding"] = emb
        out[f"{profile}/flow_mel"] = mel.astype(np.float32)
        # ---- vocoder: 10 mel frames, whole and chunked (chunk 4, context 64)
        m = hift_mel(3, 10)
        hift = HiFTGenerator(f, "hift.")
        out[f"{profile}/hift_mel"] = m
        out[f"{profile}/hift_wav"] = hift.inference(m, chunk=None).astype(np.float32)
        out[f"{profile}/hift_wav_chunked"] = hift.inference(m, chunk=4, context=64).astype(np.float32)
        f.close()
    np.savez_compressed(os.path.join(HERE, "stages_small.npz"), **out)
    print("wrote", sorted(out))
    make_sampling(a.reference)


if __name__ == "__main__":
    main()
