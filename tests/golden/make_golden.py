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

It also asserts that the synthetic generator reproduces the reference's own
random-model generator tensor for tensor.

    python tests/golden/make_golden.py --reference /path/to/cosyvoice3-cpu
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


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="root of the reference checkout")
    a = ap.parse_args()
    sys.path.insert(0, a.reference)
    sys.path.insert(0, os.path.join(a.reference, "tools"))
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


if __name__ == "__main__":
    main()
