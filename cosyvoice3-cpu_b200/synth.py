"""Synthetic CosyVoice 3 weights with the released geometry (random values).

The tensor names, shapes, per-profile storage kinds and value distribution
follow the reference's random-model generator
(``tools/make_dummy_model.py:25-181``) and its kind rules
(``cv3cpu/convert.py:25-49``, ``:255-265``, ``:300-302``): every tensor is
``N(0, 1) * 0.02`` float32 drawn from ``numpy.random.default_rng(crc32(name))``
(norm scales and Snake alphas are ones), then stored as q8, float16 or float32
according to the profile.  Because the seed is the name, the values equal the
reference generator's tensor for tensor, which lets the golden tests cross-check
against the reference reading the same file.

There is no public dataset or checkpoint involved; everything here is seeded
random data of the benchmark's shapes.
"""

from __future__ import annotations

import re
import zlib
from typing import Any, Dict, Tuple

import numpy as np

from .quant import make_qtensor
from .weights import TensorDict

QWEN = dict(hidden_size=896, num_hidden_layers=24, num_attention_heads=14,
            num_key_value_heads=2, intermediate_size=4864, rms_norm_eps=1e-6,
            rope_theta=1000000.0, vocab_size=151936)
SMALL_QWEN = dict(hidden_size=128, num_hidden_layers=2, num_attention_heads=2,
                  num_key_value_heads=1, intermediate_size=256, rms_norm_eps=1e-6,
                  rope_theta=1000000.0, vocab_size=2048)
DIT = {"dim": 1024, "depth": 22, "heads": 16, "dim_head": 64, "static_chunk_size": 50,
       "num_decoding_left_chunks": -1, "conv_pos_kernel": 31, "conv_pos_groups": 16}
SMALL_DIT = dict(DIT, dim=128, depth=2, heads=2, dim_head=64)
FLOW = {"token_mel_ratio": 2, "pre_lookahead_len": 3, "output_size": 80,
        "inference_cfg_rate": 0.7, "n_timesteps": 10}
HIFT = {"upsample_rates": [8, 5, 3], "upsample_kernel_sizes": [16, 11, 7],
        "resblock_kernel_sizes": [3, 7, 11], "resblock_dilation_sizes": [[1, 3, 5]] * 3,
        "source_resblock_kernel_sizes": [7, 7, 11],
        "source_resblock_dilation_sizes": [[1, 3, 5]] * 3,
        "istft_n_fft": 16, "istft_hop_len": 4, "lrelu_slope": 0.1, "audio_limit": 0.99,
        "sampling_rate": 24000, "nb_harmonics": 8, "nsf_alpha": 0.1, "nsf_sigma": 0.003,
        "nsf_voiced_threshold": 10.0, "conv_pre_look_right": 4}

# storage kind per profile: (default kind, LM body kind, min elements to quantise)
PROFILES = {"balanced": ("q8", "q8", 1 << 16), "tiny": ("q8", "q4", 1 << 16), "f32": ("f32", "f32", 1 << 62)}
_KEEP_F32 = re.compile(r"(\.bias$)|(layernorm)|(\.norm$)|(alpha)|(f0_predictor)|(l_linear)|"
                       r"(spk_embed_affine)|(conv_pos_embed)")
_KEEP_F16 = re.compile(r"^hift\.|(flow\.input_embedding$)|(proj_out)|(time_embed)|(pre_lookahead)")


def storage_kind(name: str, shape, profile: str) -> str:
    """q8 / q4 / f16 / f32 for one tensor; the rules of convert.py:255-265 and :300-302."""
    default, lm_kind, min_numel = PROFILES[profile]
    if len(shape) == 1 or _KEEP_F32.search(name) or int(np.prod(shape)) < min_numel:
        return "f32"
    if _KEEP_F16.search(name):
        return "f32" if default == "f32" else "f16"
    kind = lm_kind if (name.startswith("llm.model.layers.") or name == "llm.model.embed_tokens") else default
    if kind == "q8" and len(shape) == 3 and "conv_pos_embed" in name:
        kind = "f32"     # grouped convs never take the quantised GEMM
    return kind


def _tensor(name: str, shape, profile: str, ones: bool = False):
    arr = (np.ones(shape, np.float32) if ones else
           np.random.default_rng(zlib.crc32(name.encode())).standard_normal(shape, dtype=np.float32) * 0.02)
    kind = storage_kind(name, shape, profile)
    if kind in ("q8", "q4"):
        return make_qtensor(arr.reshape(arr.shape[0], -1), orig_shape=arr.shape, kind=kind)
    if kind == "f16":
        return arr.astype(np.float16)
    return arr


def _specs(small: bool, stages) -> Tuple[list, Dict[str, Any]]:
    q = SMALL_QWEN if small else QWEN
    dit = SMALL_DIT if small else DIT
    hb = 64 if small else 512
    sts = 256 if small else 6561
    head = sts + 200
    meta = {"source": "synthetic", "sample_rate": 24000, "qwen2": dict(q),
            "speech_token_size": sts, "endofprompt_id": (q["vocab_size"] - 1) if small else 151646,
            "flow": dict(FLOW), "dit": dict(dit), "hift": dict(HIFT)}
    S = []                                         # (name, shape, ones)
    h = q["hidden_size"]
    kv = q["num_key_value_heads"] * (h // q["num_attention_heads"])
    inter = q["intermediate_size"]
    if "llm" in stages:
        S.append(("llm.model.embed_tokens", (q["vocab_size"], h), False))
        for i in range(q["num_hidden_layers"]):
            p = f"llm.model.layers.{i}."
            S += [(p + "self_attn.q_proj.weight", (h, h), False), (p + "self_attn.q_proj.bias", (h,), False),
                  (p + "self_attn.k_proj.weight", (kv, h), False), (p + "self_attn.k_proj.bias", (kv,), False),
                  (p + "self_attn.v_proj.weight", (kv, h), False), (p + "self_attn.v_proj.bias", (kv,), False),
                  (p + "self_attn.o_proj.weight", (h, h), False),
                  (p + "mlp.gate_proj.weight", (inter, h), False), (p + "mlp.up_proj.weight", (inter, h), False),
                  (p + "mlp.down_proj.weight", (h, inter), False),
                  (p + "input_layernorm", (h,), True), (p + "post_attention_layernorm", (h,), True)]
        S += [("llm.model.norm", (h,), True), ("llm.llm_decoder.weight", (head, h), False),
              ("llm.speech_embedding", (head, h), False)]
    if "flow" in stages:
        d, depth = dit["dim"], dit["depth"]
        e = "flow.decoder.estimator."
        S += [("flow.input_embedding", (sts, 80), False),
              ("flow.spk_embed_affine_layer.weight", (80, 192), False),
              ("flow.spk_embed_affine_layer.bias", (80,), False),
              ("flow.pre_lookahead_layer.conv1.weight", (1024, 80, 4), False),
              ("flow.pre_lookahead_layer.conv1.bias", (1024,), False),
              ("flow.pre_lookahead_layer.conv2.weight", (80, 1024, 3), False),
              ("flow.pre_lookahead_layer.conv2.bias", (80,), False),
              (e + "time_embed.time_mlp.0.weight", (d, 256), False), (e + "time_embed.time_mlp.0.bias", (d,), False),
              (e + "time_embed.time_mlp.2.weight", (d, d), False), (e + "time_embed.time_mlp.2.bias", (d,), False),
              (e + "input_embed.proj.weight", (d, 320), False), (e + "input_embed.proj.bias", (d,), False)]
        for c in ("conv1", "conv2"):
            S += [(e + f"input_embed.conv_pos_embed.{c}.0.weight",
                   (d, d // dit["conv_pos_groups"], dit["conv_pos_kernel"]), False),
                  (e + f"input_embed.conv_pos_embed.{c}.0.bias", (d,), False)]
        for i in range(depth):
            b = e + f"transformer_blocks.{i}."
            S += [(b + "attn_norm.linear.weight", (6 * d, d), False), (b + "attn_norm.linear.bias", (6 * d,), False)]
            for n in ("to_q", "to_k", "to_v"):
                S += [(b + f"attn.{n}.weight", (d, d), False), (b + f"attn.{n}.bias", (d,), False)]
            S += [(b + "attn.to_out.0.weight", (d, d), False), (b + "attn.to_out.0.bias", (d,), False),
                  (b + "ff.ff.0.0.weight", (2 * d, d), False), (b + "ff.ff.0.0.bias", (2 * d,), False),
                  (b + "ff.ff.2.weight", (d, 2 * d), False), (b + "ff.ff.2.bias", (d,), False)]
        S += [(e + "norm_out.linear.weight", (2 * d, d), False), (e + "norm_out.linear.bias", (2 * d,), False),
              (e + "proj_out.weight", (80, d), False), (e + "proj_out.bias", (80,), False)]
    if "hift" in stages:
        m = HIFT
        S += [("hift.conv_pre.weight", (hb, 80, m["conv_pre_look_right"] + 1), False),
              ("hift.conv_pre.bias", (hb,), False)]
        chans = []
        for i, (u, k) in enumerate(zip(m["upsample_rates"], m["upsample_kernel_sizes"])):
            cin, cout = hb // (2 ** i), hb // (2 ** (i + 1))
            chans.append(cout)
            S += [(f"hift.ups.{i}.weight", (cout, cin, k), False), (f"hift.ups.{i}.bias", (cout,), False)]
        downs = list(np.cumprod([1] + m["upsample_rates"][::-1][:-1]))[::-1]
        for i, u in enumerate(downs):
            u = int(u)
            ks = 1 if u == 1 else 2 * u
            S += [(f"hift.source_downs.{i}.weight", (chans[i], m["istft_n_fft"] + 2, ks), False),
                  (f"hift.source_downs.{i}.bias", (chans[i],), False)]
            S += _resblock_specs(f"hift.source_resblocks.{i}", chans[i], m["source_resblock_kernel_sizes"][i],
                                 m["source_resblock_dilation_sizes"][i])
        for i in range(len(m["upsample_rates"])):
            for j, (k, dil) in enumerate(zip(m["resblock_kernel_sizes"], m["resblock_dilation_sizes"])):
                S += _resblock_specs(f"hift.resblocks.{i * 3 + j}", chans[i], k, dil)
        S += [("hift.conv_post.weight", (m["istft_n_fft"] + 2, chans[-1], 7), False),
              ("hift.conv_post.bias", (m["istft_n_fft"] + 2,), False),
              ("hift.m_source.l_linear.weight", (1, m["nb_harmonics"] + 1), False),
              ("hift.m_source.l_linear.bias", (1,), False)]
        for i in range(5):
            S += [(f"hift.f0_predictor.condnet.{i}.weight", (512, 80 if i == 0 else 512, 4 if i == 0 else 3), False),
                  (f"hift.f0_predictor.condnet.{i}.bias", (512,), False)]
        S += [("hift.f0_predictor.classifier.weight", (1, 512), False),
              ("hift.f0_predictor.classifier.bias", (1,), False)]
    return S, meta


def _resblock_specs(base, ch, k, dils):
    out = []
    for j, _ in enumerate(dils):
        out += [(f"{base}.convs1.{j}.weight", (ch, ch, k), False), (f"{base}.convs1.{j}.bias", (ch,), False),
                (f"{base}.convs2.{j}.weight", (ch, ch, k), False), (f"{base}.convs2.{j}.bias", (ch,), False),
                (f"{base}.activations1.{j}.alpha", (ch,), True), (f"{base}.activations2.{j}.alpha", (ch,), True)]
    return out


def synthetic_weights(profile: str = "balanced", small: bool = False,
                      stages=("llm", "flow", "hift")) -> TensorDict:
    """``name -> ndarray | QTensor`` with a ``.meta`` dict, built in memory."""
    if profile not in PROFILES:
        raise ValueError(f"unknown profile {profile!r}; pick one of {sorted(PROFILES)}")
    specs, meta = _specs(small, stages)
    meta["profile"] = profile
    return TensorDict({n: _tensor(n, s, profile, ones) for n, s, ones in specs}, meta)
