"""The q4 "tiny" profile on the device (cv3cpu/quant.py:70-86 format, :124-131
expansion, :156-204 qmatmul with a q4 QTensor) against the oracle: the
dequantisation and the embedding gather are exact (bit-equal), the linear is
within 1e-5 of the oracle's widen-then-matmul (fp32 summation order only), and a
small LM whose body linears and token embedding are q4 decodes the oracle's
greedy tokens.
"""

import numpy as np
import pytest

from conftest import pkg, rel_err

import oracle.numerics as nx
import oracle.stages as st

pytestmark = pytest.mark.gpu


def _q4(w):
    t = pkg("quant").make_qtensor(w, kind="q4")
    return t, nx.QTensor("q4", t.q, t.scales, t.shape, nx.Q4_BLOCK)


@pytest.mark.parametrize("n,k", [(1152, 896), (896, 4864), (6761, 896), (37, 70)])
@pytest.mark.parametrize("m", [1, 3, 8, 21])
def test_q4_linear(n, k, m):
    import torch
    rng = np.random.default_rng(n + k + m)
    qt, oq = _q4((rng.normal(size=(n, k)) * 0.02).astype(np.float32))
    x = rng.normal(size=(m, k)).astype(np.float32)
    b = rng.normal(size=n).astype(np.float32)
    r = rng.normal(size=(m, n)).astype(np.float32)
    got = pkg("ops").linear(torch.from_numpy(x).cuda(), qt, torch.from_numpy(b).cuda(),
                            residual=torch.from_numpy(r).cuda())
    torch.cuda.synchronize()
    assert rel_err(got.cpu().numpy(), nx.qmatmul(x, oq, b) + r) < 1e-5
    assert rel_err(pkg("quant").qmatmul(x, qt), nx.qmatmul(x, oq)) < 1e-5   # host arrays in, host out


def test_q4_dequant_and_embedding_are_exact():
    import torch
    rng = np.random.default_rng(4)
    qt, oq = _q4((rng.normal(size=(300, 100)) * 0.05).astype(np.float32))
    d = qt.to_device()
    out = torch.empty(300, 100, device="cuda")
    pkg("_lib").call("cv3_q4_dequant", d.q.data_ptr(), d.scales.data_ptr(), 300, d.padded_k, 100, out.data_ptr(),
                     torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy(), nx.dequant(oq))
    ids = rng.integers(0, 300, size=(3, 7))
    assert np.array_equal(pkg("ops").embedding(qt, ids), nx.embedding(oq, ids))
    with pytest.raises(IndexError):
        pkg("ops").embedding(qt, [300])


def test_tiny_profile_lm_greedy_matches_oracle(small_weights):
    """Small LM in the 'tiny' storage: every body linear and the token embedding q4 (the
    small geometry is below the profile's size threshold, so they are quantised here),
    speech embedding and head q8.  The decode engine runs its generic q4 path."""
    W0 = small_weights["f32"]
    Q = pkg("quant")
    tensors = dict(W0)
    for name, t in W0.items():
        if name.startswith("llm.model.layers.") and name.endswith("proj.weight") or name == "llm.model.embed_tokens":
            tensors[name] = Q.make_qtensor(t, kind="q4")
        elif name in ("llm.llm_decoder.weight", "llm.speech_embedding"):
            tensors[name] = Q.make_qtensor(t)
    W = pkg("weights").TensorDict(tensors, W0.meta)
    lm = pkg("models.llm").CosyVoice3LM(pkg("weights").DeviceWeights(W))
    olm = st.SpeechLM(W, W.meta)
    rng = np.random.default_rng(12)
    eop = W.meta["endofprompt_id"]
    prompts, oprompts = [], []
    for nn in (6, 11):
        text = [eop] + rng.integers(0, 2000, size=nn).tolist()
        prompts.append(lm.prompt_embedding(text, (), [1, 2, 3]))
        oprompts.append(olm.prompt_embedding(text, (), [1, 2, 3]))
        assert rel_err(prompts[-1].cpu().numpy(), oprompts[-1]) < 1e-6
    toks = lm.generate_greedy(prompts, 16).cpu().numpy()
    assert all(f is None for f in lm.last_engine.fast)
    for b in range(2):
        ref, _ = olm.generate_greedy(oprompts[b], 16)
        assert toks[b].tolist() == ref
