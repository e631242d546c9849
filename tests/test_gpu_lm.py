"""LM stage parity: the device Qwen2 body, head and greedy decode against the
oracle and the reference's goldens (small synthetic model), plus the full
Qwen2-0.5B geometry for a few teacher-forced steps.

Tolerances: log-probabilities 1e-5 (small f32 and q8 models: the int8
dequantisation is exact, only summation order differs) and 1e-4 at full size
(the int8 path's bar); greedy ids exact.
"""

import numpy as np
import pytest

from conftest import pkg, rel_err

import oracle.stages as st

pytestmark = pytest.mark.gpu


def _device(W):
    return pkg("weights").DeviceWeights(W)


@pytest.mark.parametrize("profile", ["balanced", "f32"])
def test_greedy_decode_matches_reference_goldens(golden, small_weights, profile):
    W = small_weights[profile]
    lm = pkg("models.llm").CosyVoice3LM(_device(W))
    x0 = lm.prompt_embedding(golden[f"{profile}/lm_text"], (), golden[f"{profile}/lm_prompt_speech"])
    eng = lm.engine(1, 256, 8)
    eng.keep_logp = True
    eng.prefill([x0])
    logps = [eng.logp[0].cpu().numpy().copy()]
    for _ in range(7):
        eng.step()
        logps.append(eng.logp[0].cpu().numpy().copy())
    toks = eng.history[0, :8].cpu().numpy().tolist()
    assert toks == golden[f"{profile}/lm_tokens"].tolist()
    assert rel_err(np.stack(logps), golden[f"{profile}/lm_logp"]) < 1e-5


@pytest.mark.parametrize("profile", ["balanced", "f32"])
def test_graph_decode_equals_eager_and_oracle(small_weights, profile):
    W = small_weights[profile]
    lm = pkg("models.llm").CosyVoice3LM(_device(W))
    olm = st.SpeechLM(W, W.meta)
    rng = np.random.default_rng(5)
    eop = W.meta["endofprompt_id"]
    prompts, oprompts = [], []
    for n in (7, 19, 12):
        text = [eop] + rng.integers(0, 2000, size=n).tolist()
        sp = rng.integers(0, 256, size=4).tolist()
        prompts.append(lm.prompt_embedding(text, (), sp))
        oprompts.append(olm.prompt_embedding(text, (), sp))
    graph = lm.generate_greedy(prompts, 20, persistent=False).cpu().numpy()
    eager = lm.generate_greedy(prompts, 20, use_graph=False, persistent=False).cpu().numpy()
    assert np.array_equal(graph, eager)
    for b in range(3):
        toks, _ = olm.generate_greedy(oprompts[b], 20)
        assert graph[b].tolist() == toks, b


def test_incremental_decoding_equals_one_full_pass(small_weights):
    """cv3cpu tests/test_reference.py:158-169 on the device body."""
    W = small_weights["f32"]
    lm = pkg("models.llm").CosyVoice3LM(_device(W))
    rng = np.random.default_rng(0)
    x = rng.normal(size=(17, lm.cfg.hidden_size)).astype(np.float32) * 0.2
    full = lm.body.forward(x)
    cache = lm.body.new_cache(1, 64)
    parts = [lm.body.forward(x[:5], cache)] + [lm.body.forward(x[i:i + 1], cache) for i in range(5, 17)]
    assert rel_err(np.concatenate(parts), full) < 5e-5
    assert rel_err(full, st.Qwen2(W, W.meta).forward(x)) < 1e-5


def test_full_size_lm_teacher_forced():
    """Qwen2-0.5B geometry, balanced q8: prefill 64 rows + 4 forced steps vs the oracle."""
    W = pkg("synth").synthetic_weights("balanced", stages=("llm",))
    lm = pkg("models.llm").CosyVoice3LM(_device(W))
    olm = st.SpeechLM(W, W.meta)
    rng = np.random.default_rng(0)
    x = (rng.normal(size=(64, 896)) * 0.1).astype(np.float32)
    forced = rng.integers(0, 6561, size=4).tolist()
    _, ref_logp = olm.generate_greedy(x, 5, forced=forced)
    eng = lm.engine(1, 256, 5)
    eng.keep_logp = True
    eng.prefill([x])
    got = [eng.logp[0].cpu().numpy().copy()]
    for t in forced:
        eng.next_ids.fill_(t)
        eng.h.copy_(pkg("_dev").dev(olm.speech_emb([t])))
        eng.step()
        got.append(eng.logp[0].cpu().numpy().copy())
    assert rel_err(np.stack(got), ref_logp) < 1e-4


def _decode_status_clear():
    import ctypes
    code = ctypes.c_int(-1)
    assert pkg("_lib").load().cv3_decode_status(ctypes.byref(code)) == 0 and code.value == 0


def test_persistent_decode_equals_graph_steps():
    """cv3_decode_steps (every step in one cooperative launch) against the per-step graph at
    the released geometry (every layer q8, as the persistent kernel requires): identical
    greedy ids for a ragged batch, per-step log-probs within 1e-5."""
    W = pkg("synth").synthetic_weights("balanced", stages=("llm",))
    lm = pkg("models.llm").CosyVoice3LM(_device(W))
    rng = np.random.default_rng(11)
    hid = lm.cfg.hidden_size
    prompts = [(rng.normal(size=(n, hid)) * 0.1).astype(np.float32) for n in (9, 30, 17)]
    eng = lm.engine(3, 256, 24)
    assert eng.persistent_ok
    mk = eng.run(prompts, 24, persistent=True).cpu().numpy()
    _decode_status_clear()
    gr = eng.run(prompts, 24, persistent=False).cpu().numpy()
    assert np.array_equal(mk, gr)
    # step by step with log-probs
    eng.keep_logp = True
    eng.prefill(prompts)
    a = []
    for _ in range(6):
        eng.steps_persistent(1)
        a.append(eng.logp.cpu().numpy().copy())
    eng.graph = None
    eng.prefill(prompts)
    b = []
    for _ in range(6):
        eng.step()
        b.append(eng.logp.cpu().numpy().copy())
    assert rel_err(np.stack(a), np.stack(b)) < 1e-5
    _decode_status_clear()


def test_persistent_decode_bench_batch():
    """Eight sequences (the benchmark's batch) at the released geometry: the persistent
    launch reproduces the graph's 40 greedy tokens exactly."""
    W = pkg("synth").synthetic_weights("balanced", stages=("llm",))
    lm = pkg("models.llm").CosyVoice3LM(_device(W))
    rng = np.random.default_rng(3)
    prompts = [(rng.normal(size=(60 + 3 * i, 896)) * 0.1).astype(np.float32) for i in range(8)]
    mk = lm.generate_greedy(prompts, 40, persistent=True).cpu().numpy()
    gr = lm.generate_greedy(prompts, 40, persistent=False).cpu().numpy()
    assert np.array_equal(mk, gr)
    _decode_status_clear()
