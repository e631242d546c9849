"""Device sampler (cv3_sample_select) against the oracle's restatement of the
reference's sampler (cv3cpu/models/llm.py:37-49, :125-149; pinned to the
reference itself in test_oracle_pins.py): the same tokens, stop decisions and
numpy PCG64 stream.  The device computes exp with CUDA's expf, numpy with its
own float32 exp, so probabilities may differ in the last place; everything else
(pairwise sums, float64 nucleus and cumulative sums, the draws) is done in the
reference's order, and the seeded cases below agree token for token.
"""

import numpy as np
import pytest

from conftest import pkg

import oracle.numerics as nx

pytestmark = pytest.mark.gpu


def _words(rng):
    s = rng.bit_generator.state["state"]
    m = (1 << 64) - 1
    w = [(s["state"] >> 64) & m, s["state"] & m, (s["inc"] >> 64) & m, s["inc"] & m]
    return [v - (1 << 64) if v >= (1 << 63) else v for v in w]


@pytest.mark.parametrize("strict", [False, True])
def test_sample_select_matches_oracle(strict):
    import torch
    L = pkg("_lib")
    B, V, sts, steps, hist = 3, 6761, 6561, 80, 96
    seeds = [3, 4, 5]
    rngs = [np.random.default_rng(s) for s in seeds]
    rng_state = torch.tensor([_words(r) for r in rngs], dtype=torch.int64, device="cuda")
    min_len = torch.tensor([10, 0, 30], dtype=torch.int32, device="cuda")
    max_len = torch.tensor([70, 80, 50], dtype=torch.int32, device="cuda")
    count = torch.zeros(B, dtype=torch.int32, device="cuda")
    done = torch.zeros(B, dtype=torch.int32, device="cuda")
    next_ids = torch.zeros(B, dtype=torch.int64, device="cuda")
    pos = torch.zeros(B, dtype=torch.int32, device="cuda")
    lens = torch.zeros(B, dtype=torch.int32, device="cuda")
    history = torch.zeros((B, hist), dtype=torch.int64, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    data = np.random.default_rng(99)
    ref_tok = [[] for _ in range(B)]
    ref_done = [False] * B
    mins, maxs = min_len.cpu().tolist(), max_len.cpu().tolist()
    for i in range(steps):
        # peaked logits: nucleus sets of a few tokens, frequent repeats and occasional stops
        logits = (data.normal(size=(B, V)) * 3.0).astype(np.float32)
        logits[:, data.integers(0, 40, size=4)] += 6.0
        lg = torch.from_numpy(logits).cuda()   # kept alive past the launch
        L.call("cv3_sample_select", lg.data_ptr(), B, V, sts, min_len.data_ptr(),
               max_len.data_ptr(), int(strict), 0.8, 25, 10, 0.1, rng_state.data_ptr(), next_ids.data_ptr(),
               pos.data_ptr(), lens.data_ptr(), history.data_ptr(), hist, count.data_ptr(), done.data_ptr(), None, st)
        for b in range(B):
            if ref_done[b]:
                continue
            n = len(ref_tok[b])
            if n >= maxs[b]:
                ref_done[b] = True
                continue
            top = nx.sample_token(nx.log_softmax(logits[b]), ref_tok[b], rngs[b], sts, n < mins[b], strict)
            if sts <= top < sts + 200:
                ref_done[b] = True
            else:
                ref_tok[b].append(top)
                ref_done[b] = len(ref_tok[b]) >= maxs[b]
    torch.cuda.synchronize()
    cnt, hs = count.cpu().tolist(), history.cpu().numpy()
    for b in range(B):
        assert hs[b, :cnt[b]].tolist() == ref_tok[b], b
        assert bool(done[b].item()) == ref_done[b]
        assert rng_state[b].cpu().tolist() == _words(rngs[b]), b
    assert pos.cpu().tolist() == cnt and lens.cpu().tolist() == cnt


@pytest.mark.parametrize("profile", ["balanced", "f32"])
def test_generate_device_sampler_matches_host_sampler(small_weights, profile):
    """CosyVoice3LM.generate with the device sampler (graph-replayed steps) against the
    host-sampler path (a device forward per token, numpy sampling): same tokens, and the
    generator left in the same state."""
    W = small_weights[profile]
    llm = pkg("models.llm")
    lm = llm.CosyVoice3LM(pkg("weights").DeviceWeights(W))
    eop = W.meta["endofprompt_id"]
    rng = np.random.default_rng(21)
    for trial in range(3):
        text = [eop] + rng.integers(0, 2000, size=12 + 5 * trial).tolist()
        sp = rng.integers(0, 256, size=5).tolist()
        kw = dict(seed=40 + trial, max_token_text_ratio=4.0, min_token_text_ratio=1.0, strict_min_len=trial == 1)
        a, b = llm.SamplingConfig(**kw), llm.SamplingConfig(**kw)
        dev = list(lm.generate(text, (), sp, sampling=a))
        host = list(lm.generate(text, (), sp, sampling=b, device_sampler=False))
        assert dev == host, trial
        assert a.rng.bit_generator.state == b.rng.bit_generator.state


@pytest.mark.parametrize("profile", ["balanced", "f32"])
def test_generate_matches_oracle_sampled_generation(small_weights, profile):
    """CosyVoice3LM.generate (graph-replayed steps, device sampler) against the oracle's
    restatement of the reference's sampling loop (pinned to CosyVoice3LM.generate itself):
    the same tokens, stops and min/max lengths, and the generator left in the same state."""
    import oracle.stages as st
    W = small_weights[profile]
    llm = pkg("models.llm")
    lm = llm.CosyVoice3LM(pkg("weights").DeviceWeights(W))
    olm = st.SpeechLM(W, W.meta)
    eop = W.meta["endofprompt_id"]
    data = np.random.default_rng(2)
    total = 0
    for trial, (lo, strict) in enumerate([(2.0, True), (3.0, True), (1.0, False), (2.5, True)]):
        text = data.integers(0, 2000, size=6 + 3 * trial).tolist()
        speech = data.integers(0, 256, size=4).tolist()
        cfg = llm.SamplingConfig(seed=30 + trial, max_token_text_ratio=4.0, min_token_text_ratio=lo,
                                 strict_min_len=strict)
        got = list(lm.generate(text, [eop], speech, sampling=cfg))
        rng = np.random.default_rng(30 + trial)
        want = olm.generate_sampled(olm.prompt_embedding(text, [eop], speech), len(text), rng, lo, 4.0, strict)
        assert got == want, trial
        assert cfg.rng.bit_generator.state == rng.bit_generator.state
        total += len(want)
    assert total >= 40
