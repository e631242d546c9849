"""Host-side logic on the CPU: the weight format, the q8 writer and the synthetic model."""

import os
import sys

import numpy as np
import pytest

from conftest import REFERENCE, have_reference, pkg

import oracle.numerics as nx


def test_quantize_q8_matches_the_oracle():
    rng = np.random.default_rng(3)
    for shape in [(9, 100), (64, 64), (128, 257), (4, 64)]:
        w = rng.normal(size=shape).astype(np.float32)
        a = pkg("quant").quantize_q8(w)
        b = nx.quantize_q8(w)
        assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1]) and a[2] == b[2]


def test_zero_blocks_get_unit_scale():
    q, s, _ = pkg("quant").quantize_q8(np.zeros((4, 64), np.float32))
    assert np.all(s == 1.0) and np.all(q == 0)


def test_weight_file_round_trip(tmp_path):
    Q = pkg("quant")
    W = pkg("weights")
    rng = np.random.default_rng(0)
    t = {"a.weight": Q.make_qtensor(rng.normal(size=(6, 4, 3)).astype(np.float32), orig_shape=(6, 4, 3)),
         "a.bias": rng.normal(size=6).astype(np.float32),
         "b": rng.normal(size=(5, 7)).astype(np.float16)}
    path = str(tmp_path / "w.safetensors")
    W.write_weights(path, t, {"x": 1})
    f = W.WeightFile(path)
    assert f.meta == {"x": 1}
    assert sorted(f.keys()) == sorted(t)
    qt = f.get("a.weight")
    assert isinstance(qt, Q.QTensor) and qt.kernel_size == 3 and qt.shape == (6, 12)
    assert np.array_equal(qt.q, t["a.weight"].q) and np.array_equal(qt.scales, t["a.weight"].scales)
    assert np.array_equal(f.get("a.bias"), t["a.bias"]) and f.get("b").dtype == np.float16
    assert f.entry("a.weight")["kind"] == "q8" and f.entry("b")["kind"] == "f16"
    assert "missing" not in f and f.get("missing") is None
    f.close()


@pytest.mark.skipif(not have_reference(), reason="reference checkout not present")
def test_reference_reads_our_files(tmp_path):
    sys.path.insert(0, REFERENCE)
    from cv3cpu.io.weights import WeightFile as RefWF
    W = pkg("weights")
    syn = pkg("synth").synthetic_weights("balanced", small=True, stages=("llm",))
    path = str(tmp_path / "s.safetensors")
    W.write_weights(path, dict(syn), syn.meta)
    r = RefWF(path)
    name = "llm.model.embed_tokens"                      # q8 even in the small model
    assert np.array_equal(r.get_f32(name), syn[name].dequant())
    assert np.array_equal(r.get_f32("llm.model.layers.0.mlp.gate_proj.weight"),
                          syn["llm.model.layers.0.mlp.gate_proj.weight"])
    assert r.meta["qwen2"]["hidden_size"] == 128
    r.close()


def test_synthetic_storage_kinds_follow_the_balanced_profile():
    k = pkg("synth").storage_kind
    assert k("llm.model.layers.0.mlp.up_proj.weight", (4864, 896), "balanced") == "q8"
    assert k("llm.llm_decoder.weight", (6761, 896), "balanced") == "q8"
    assert k("flow.decoder.estimator.transformer_blocks.0.attn.to_q.weight", (1024, 1024), "balanced") == "q8"
    assert k("flow.decoder.estimator.proj_out.weight", (80, 1024), "balanced") == "f16"
    assert k("flow.decoder.estimator.input_embed.conv_pos_embed.conv1.0.weight", (1024, 64, 31), "balanced") == "f32"
    assert k("hift.ups.0.weight", (256, 512, 16), "balanced") == "f16"
    assert k("hift.f0_predictor.condnet.0.weight", (512, 80, 4), "balanced") == "f32"
    assert k("llm.model.layers.0.input_layernorm", (896,), "balanced") == "f32"
    assert k("llm.model.layers.0.mlp.up_proj.weight", (4864, 896), "f32") == "f32"


def test_synthetic_small_model_geometry():
    syn = pkg("synth").synthetic_weights("balanced", small=True)
    assert syn.meta["qwen2"]["hidden_size"] == 128 and syn.meta["speech_token_size"] == 256
    assert syn["llm.llm_decoder.weight"].shape == (456, 128)
    assert syn["hift.conv_pre.weight"].shape == (64, 80, 5)
    assert syn["hift.f0_predictor.condnet.1.weight"].shape == (512, 512, 3)
