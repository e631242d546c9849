"""Seeded synthetic inputs for the benchmark configurations.

No dataset or checkpoint is involved: every input below is random data with
the shapes and value distributions the configurations name, drawn from
``numpy.random.default_rng(seed)``.  The golden-fixture script, the GPU parity
tests and ``bench.py`` all take their inputs from here, so a fixture made by
running the reference on these inputs checks exactly what the bench times.

* config 1 -- LM decode: a 64-id random text prompt, then 250 greedy steps.
* config 2 -- flow: 250 speech tokens in [0, 6561) (mu at 500 frames after the
  x2 upsampling), a random 192-d speaker vector, no prompt (cond = 0).
* config 3 -- vocoder: an 80 x 500 log-mel, N(-5, 2^2) clipped to [-11.5, 2].
* config 4 -- end to end: per seed, 40..80 text ids, a prompt text ending in
  <|endofprompt|>, 75 prompt speech tokens with 150 prompt mel frames and a
  192-d speaker vector.
* config 5 -- throughput sweep: as config 4 with 120..240 text ids and 750
  generated tokens per utterance.
"""

from __future__ import annotations

from typing import List, Sequence

import numpy as np

LM_PROMPT_IDS = 64
LM_STEPS = 250
FLOW_TOKENS = 250
VOCODER_FRAMES = 500
PROMPT_TOKENS = 75


def lm_prompt_ids(seed: int = 0, n: int = LM_PROMPT_IDS, vocab: int = 151936) -> np.ndarray:
    """Config 1: ``n`` random text ids (the prompt is their ``embed_tokens`` rows)."""
    return np.random.default_rng(seed).integers(0, vocab, size=n).astype(np.int64)


def flow_inputs(seed: int = 0, n_tokens: int = FLOW_TOKENS, speech_tokens: int = 6561):
    """Config 2: speech tokens and a speaker vector (no prompt)."""
    rng = np.random.default_rng(seed)
    tokens = rng.integers(0, speech_tokens, size=n_tokens).astype(np.int64)
    embedding = rng.normal(size=192).astype(np.float32)
    return tokens, embedding


def dit_inputs(seed: int = 2, batch: int = 2, frames: int = 2 * FLOW_TOKENS):
    """One DiT forward at the config-2 CFG shape: x, mu, cond ``(B, 80, N)``, spk ``(B, 80)``, t ``(B,)``."""
    rng = np.random.default_rng(seed)
    x, mu, cond = (rng.normal(size=(batch, 80, frames)).astype(np.float32) for _ in range(3))
    spk = rng.normal(size=(batch, 80)).astype(np.float32)
    t = rng.uniform(0.05, 0.95, size=batch).astype(np.float32)
    return x, mu, t, spk, cond


def vocoder_mel(seed: int = 1, frames: int = VOCODER_FRAMES) -> np.ndarray:
    """Config 3: an ``(80, frames)`` log-mel, N(-5, 2^2) clipped to [-11.5, 2]."""
    rng = np.random.default_rng(seed)
    return np.clip(rng.normal(-5.0, 2.0, size=(80, frames)), -11.5, 2.0).astype(np.float32)


def requests(seeds: Sequence[int], meta: dict, text_len=(40, 80)) -> List:
    """Config 4 (``text_len`` 40..80) and config 5 (120..240) utterances, one per seed."""
    from .pipeline import Request
    from .voice import VoicePack
    eop = int(meta.get("endofprompt_id", 151646))
    vocab = int(meta["qwen2"]["vocab_size"])
    sts = int(meta.get("speech_token_size", 6561))
    out = []
    for s in seeds:
        rng = np.random.default_rng(s)
        n = int(rng.integers(text_len[0], text_len[1] + 1))
        text = rng.integers(0, vocab, size=n).tolist()
        prompt_text = rng.integers(0, vocab, size=8).tolist() + [eop]
        voice = VoicePack(speech_token=rng.integers(0, sts, size=PROMPT_TOKENS),
                          mel=rng.normal(size=(2 * PROMPT_TOKENS, 80)).astype(np.float32),
                          embedding=rng.normal(size=192).astype(np.float32), name=f"seed{s}")
        out.append(Request(text, prompt_text, voice))
    return out
