"""End-to-end parity of the batched greedy synthesis path on the small model:
tokens exact; waveforms within 5e-5 of the oracle's LM -> flow -> vocoder chain.
Each stage alone is held to 1e-5 (tests/test_gpu_stages.py); chained, the flow's
fp32 reordering differences (~1e-6 of the mel) pass through the vocoder, so the
chain gets a 5x looser bar."""

import numpy as np
import pytest

from conftest import pkg, rel_err

import oracle.stages as st

pytestmark = pytest.mark.gpu


def _requests(meta, n=3, prompt_tokens=6):
    VoicePack, Request = pkg("voice").VoicePack, pkg("pipeline").Request
    out = []
    for s in range(n):
        rng = np.random.default_rng(100 + s)
        text = rng.integers(0, 2000, size=int(rng.integers(5, 12))).tolist()
        prompt = [meta["endofprompt_id"]] + rng.integers(0, 2000, size=3).tolist()
        voice = VoicePack(speech_token=rng.integers(0, 256, size=prompt_tokens),
                          mel=rng.normal(size=(2 * prompt_tokens, 80)).astype(np.float32),
                          embedding=rng.normal(size=192).astype(np.float32))
        out.append(Request(text, prompt, voice))
    return out


@pytest.mark.parametrize("profile", ["balanced", "f32"])
def test_greedy_batch_synthesis_matches_oracle(small_weights, profile):
    W = small_weights[profile]
    tts = pkg("pipeline").CosyVoice3CUDA(W)
    reqs = _requests(W.meta)
    wav, toks = tts.synthesize_greedy_batch(reqs, n_tokens=10)
    assert wav.shape == (3, 2 * 480 * 10) and np.abs(wav).max() <= 0.99 + 1e-7
    lm, flow, hift = st.SpeechLM(W, W.meta), st.Flow(W, W.meta), st.HiFT(W, W.meta)
    for u, r in enumerate(reqs):
        x0 = lm.prompt_embedding(r.text_ids, r.prompt_ids, r.voice.speech_token.tolist())
        ref_toks, _ = lm.generate_greedy(x0, 10)
        assert toks[u].tolist() == ref_toks, u
        mel = flow.inference(ref_toks, r.voice.speech_token, r.voice.mel, r.voice.embedding)
        assert rel_err(wav[u], hift.inference(mel, chunk=None)) < 5e-5, u


def test_sampled_synthesis_runs_and_matches_reference_contract(small_weights):
    W = small_weights["balanced"]
    SamplingConfig = pkg("models.llm").SamplingConfig
    tts = pkg("pipeline").CosyVoice3CUDA(W, seed=7)
    r = _requests(W.meta, 1)[0]
    sampling = SamplingConfig(seed=7, max_token_text_ratio=3.0, min_token_text_ratio=1.0, strict_min_len=True)
    out = tts.synthesize_ids([r.text_ids], r.prompt_ids, r.voice, sampling=sampling)
    assert out.sample_rate == 24000 and out.audio.dtype == np.float32
    assert len(out.audio) == 2 * 480 * len(out.speech_tokens[0])
    assert np.isfinite(out.audio).all() and np.abs(out.audio).max() <= 0.99 + 1e-6


def test_release_stages_gives_the_llm_hbm_back():
    """With ``release_stages`` the LM stage's weights, engines and graphs are dropped after
    the LM runs and the memory goes back to the driver (free HBM rises by at least the
    int8 LM's 375 MB of layer weights) -- the device form of the reference's eviction
    (cv3cpu/pipeline.py:81-86, io/weights.py:182-205)."""
    import torch
    W = pkg("synth").synthetic_weights("balanced", stages=("llm",))
    tts = pkg("pipeline").CosyVoice3CUDA(W, release_stages=True)
    lm = tts.llm
    eop = W.meta["endofprompt_id"]
    prompt = lm.prompt_embedding([eop, 11, 12, 13], (), [1, 2, 3])
    toks = lm.generate_greedy([prompt], 4).cpu()
    assert toks.shape == (1, 4)
    del lm, prompt
    torch.cuda.synchronize()
    free_before = torch.cuda.mem_get_info()[0]
    tts._drop("llm")
    free_after = torch.cuda.mem_get_info()[0]
    assert tts._llm is None
    assert free_after - free_before > 375e6, (free_before, free_after)
