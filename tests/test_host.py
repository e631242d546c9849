"""Host-side logic on the CPU: the weight format, the q8 writer and the synthetic model."""

import os
import sys

import numpy as np
import pytest

from conftest import REFERENCE, REPO, have_reference, pkg

import oracle.numerics as nx


def test_quantize_q8_matches_the_oracle():
    rng = np.random.default_rng(3)
    for shape in [(9, 100), (64, 64), (128, 257), (4, 64)]:
        w = rng.normal(size=shape).astype(np.float32)
        a = pkg("quant").quantize_q8(w)
        b = nx.quantize_q8(w)
        assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1]) and a[2] == b[2]


def test_quantize_q4_matches_the_oracle():
    """The 'tiny' profile's 4-bit writer: payload, scales and padded K equal the oracle's
    (itself pinned byte-for-byte to cv3cpu.quant.quantize_q4), negative extremes land on
    code 0, zero blocks get scale 1, and the host expansion equals the oracle's."""
    rng = np.random.default_rng(7)
    for shape in [(9, 100), (64, 64), (33, 31), (4, 32)]:
        w = rng.normal(size=shape).astype(np.float32)
        w[0, :32] = 0.0
        a = pkg("quant").quantize_q4(w)
        b = nx.quantize_q4(w)
        assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1]) and a[2] == b[2]
        assert np.all(a[1][0, 0] == 1.0)
        t = pkg("quant").make_qtensor(w, kind="q4")
        assert t.kind == "q4" and t.padded_k == b[2] and t.q.shape == (shape[0], b[2] // 2)
        assert np.array_equal(t.dequant(), nx.dequant(nx.QTensor("q4", b[0], b[1], shape, nx.Q4_BLOCK)))


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


def test_q4_weight_file_round_trip_and_reference_reader(tmp_path):
    """A 'tiny' file: the q4 token table is written with its kind and block, read back
    bit-equal by this package's reader and, when the reference checkout is present, by
    cv3cpu's own reader with the same expansion."""
    W = pkg("weights")
    syn = pkg("synth").synthetic_weights("tiny", small=True, stages=("llm",))
    name = "llm.model.embed_tokens"                      # q4 in the small tiny model
    assert syn[name].kind == "q4"
    path = str(tmp_path / "t.safetensors")
    W.write_weights(path, dict(syn), syn.meta)
    f = W.WeightFile(path)
    qt = f.get(name)
    assert qt.kind == "q4" and qt.block == 32 and f.entry(name)["kind"] == "q4"
    assert np.array_equal(qt.q, syn[name].q) and np.array_equal(qt.scales, syn[name].scales)
    assert np.array_equal(qt.dequant(), syn[name].dequant())
    f.close()
    if have_reference():
        sys.path.insert(0, REFERENCE)
        from cv3cpu.io.weights import WeightFile as RefWF
        r = RefWF(path)
        assert np.array_equal(r.get_f32(name), syn[name].dequant())
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


def test_synthetic_storage_kinds_follow_the_tiny_profile():
    """'tiny' (convert.py PROFILES): the LM body and its token table 4-bit, the rest as balanced."""
    k = pkg("synth").storage_kind
    assert k("llm.model.layers.0.mlp.up_proj.weight", (4864, 896), "tiny") == "q4"
    assert k("llm.model.embed_tokens", (151936, 896), "tiny") == "q4"
    assert k("llm.llm_decoder.weight", (6761, 896), "tiny") == "q8"
    assert k("llm.speech_embedding", (6761, 896), "tiny") == "q8"
    assert k("flow.decoder.estimator.transformer_blocks.0.attn.to_q.weight", (1024, 1024), "tiny") == "q8"
    assert k("hift.ups.0.weight", (256, 512, 16), "tiny") == "f16"
    assert k("llm.model.layers.0.input_layernorm", (896,), "tiny") == "f32"


def test_synthetic_small_model_geometry():
    syn = pkg("synth").synthetic_weights("balanced", small=True)
    assert syn.meta["qwen2"]["hidden_size"] == 128 and syn.meta["speech_token_size"] == 256
    assert syn["llm.llm_decoder.weight"].shape == (456, 128)
    assert syn["hift.conv_pre.weight"].shape == (64, 80, 5)
    assert syn["hift.f0_predictor.condnet.1.weight"].shape == (512, 512, 3)


def test_ops_import_without_pytorch_and_fail_loudly_without_a_device():
    """The NumPy host: with ``import torch`` blocked, ops / quant / torch_rng import and pick
    the library's own device memory; on a machine without a GPU an op raises (there is no
    CPU path)."""
    import subprocess
    import sys
    child = (
        "import importlib, sys\n"
        "sys.modules['torch'] = None\n"
        "sys.path.insert(0, sys.argv[1])\n"
        "import numpy as np\n"
        "D = importlib.import_module('cosyvoice3-cpu_b200._dev')\n"
        "ops = importlib.import_module('cosyvoice3-cpu_b200.ops')\n"
        "importlib.import_module('cosyvoice3-cpu_b200.quant')\n"
        "importlib.import_module('cosyvoice3-cpu_b200.torch_rng')\n"
        "assert D.BACKEND == 'numpy' and D.torch is None\n"
        "try:\n"
        "    ops.silu(np.ones(4, np.float32))\n"
        "    print('RAN')\n"
        "except RuntimeError as e:\n"
        "    print('RAISED', e)\n")
    p = subprocess.run([sys.executable, "-c", child, REPO], capture_output=True, text=True, timeout=300)
    assert p.returncode == 0, p.stderr[-3000:]
    out = p.stdout.strip().splitlines()[-1]
    # without a GPU the op must raise; on a GPU machine it runs
    assert out.startswith("RAISED no CUDA device") or out == "RAN", out


def test_device_array_views_without_a_device():
    """The NumPy host's device arrays: shapes, views and byte offsets (no memory touched:
    an array made on a given address owns nothing and frees nothing)."""
    D = pkg("_dev")
    a = D.DeviceArray((4, 3, 5), np.float32, _ptr=0x10000)
    assert a.numel() == 60 and a.nbytes == 240 and a.dim() == 3
    r = a.reshape(-1, 5)
    assert r.shape == (12, 5) and r.data_ptr() == 0x10000
    assert a.reshape((2, 30)).shape == (2, 30)
    with pytest.raises(ValueError):
        a.reshape(7, -1, 3)
    assert a.unsqueeze(0).shape == (1, 4, 3, 5) and a.unsqueeze(-1).shape == (4, 3, 5, 1)
    assert a[2].shape == (3, 5) and a[2].data_ptr() == 0x10000 + 2 * 15 * 4
    assert a[-1].data_ptr() == 0x10000 + 3 * 15 * 4
    with pytest.raises(IndexError):
        a[4]
    with pytest.raises(TypeError):
        a[1:2]
    h = D.DeviceArray((8,), np.float16, _ptr=0x20000)
    assert h.nbytes == 16 and D.is_half(h) and D.is_device(h) and not D.is_host(h)
