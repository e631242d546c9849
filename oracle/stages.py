"""NumPy restatement of the three CosyVoice 3 stages (test infrastructure only).

Qwen2 LM body and head (``cv3cpu/models/qwen2.py``, ``cv3cpu/models/llm.py``),
the DiT flow estimator and Euler/CFG solver (``cv3cpu/models/dit.py``,
``cv3cpu/models/flow.py``) and the HiFT vocoder (``cv3cpu/models/hift.py``),
each driven through :mod:`oracle.numerics`.

Weights are any mapping ``name -> ndarray | q8 weight`` (``W[name]``) plus the
metadata dict the reference keeps in the weight file (``meta["qwen2"]``,
``meta["dit"]``, ``meta["flow"]``, ``meta["hift"]``).
"""

from __future__ import annotations

import math
from typing import List, Optional, Sequence

import numpy as np

from . import numerics as nx

F32 = np.float32


def _kernel(w) -> int:
    """Last dimension of a conv weight, read from a q8 weight's original shape too."""
    if nx.is_quant(w):
        return int(w.orig_shape[-1])
    return int(np.shape(w)[-1])


# ---------------------------------------------------------------------------
# Qwen2 body                                           cv3cpu/models/qwen2.py
# ---------------------------------------------------------------------------

def qwen_rope_tables(positions: np.ndarray, dim: int, theta: float):
    """Half-split RoPE cos/sin, angles in float64 then cast; qwen2.py:46-61."""
    inv = 1.0 / (theta ** (np.arange(0, dim, 2, dtype=np.float64) / dim))
    ang = np.asarray(positions, dtype=np.float64)[:, None] * inv[None, :]
    ang = np.concatenate([ang, ang], axis=-1)
    return np.cos(ang).astype(F32), np.sin(ang).astype(F32)


def qwen_rope(x, cos, sin):
    """``x (H, T, D)``: x*cos + rotate_half(x)*sin; qwen2.py:64-71."""
    h = x.shape[-1] // 2
    rot = np.concatenate([-x[..., h:], x[..., :h]], axis=-1)
    return x * cos[None] + rot * sin[None]


class KV:
    """Per-layer fp32 (kv_heads, L, head_dim) cache; qwen2.py:74-121 (no growth policy needed)."""

    def __init__(self, layers: int):
        self.k: List[Optional[np.ndarray]] = [None] * layers
        self.v: List[Optional[np.ndarray]] = [None] * layers
        self.length = 0
        self.layers = layers

    def append(self, i, k, v):
        self.k[i] = k if self.k[i] is None else np.concatenate([self.k[i], k], axis=1)
        self.v[i] = v if self.v[i] is None else np.concatenate([self.v[i], v], axis=1)
        if i == self.layers - 1:
            self.length = self.k[i].shape[1]
        return self.k[i], self.v[i]


class Qwen2:
    """Decoder-only Qwen2 over embeddings; forward follows qwen2.py:139-179."""

    def __init__(self, W, meta, prefix: str = "llm.model."):
        c = meta["qwen2"]
        self.W, self.p = W, prefix
        self.hidden = int(c["hidden_size"])
        self.layers = int(c["num_hidden_layers"])
        self.heads = int(c["num_attention_heads"])
        self.kv_heads = int(c["num_key_value_heads"])
        self.head_dim = self.hidden // self.heads
        self.eps = float(c.get("rms_norm_eps", 1e-6))
        self.theta = float(c.get("rope_theta", 1e6))

    def t(self, name):
        return self.W[self.p + name]

    def new_cache(self) -> KV:
        return KV(self.layers)

    def forward(self, x, cache: Optional[KV] = None):
        T = x.shape[0]
        past = cache.length if cache is not None else 0
        cos, sin = qwen_rope_tables(np.arange(past, past + T), self.head_dim, self.theta)
        mask = ("causal", past) if T > 1 else None
        nh, nkv, hd = self.heads, self.kv_heads, self.head_dim
        h = x.astype(F32, copy=False)
        for i in range(self.layers):
            p = f"layers.{i}."
            n = nx.rms_norm(h, self.t(p + "input_layernorm"), self.eps)
            q = nx.linear(n, self.t(p + "self_attn.q_proj.weight"), self.t(p + "self_attn.q_proj.bias"))
            k = nx.linear(n, self.t(p + "self_attn.k_proj.weight"), self.t(p + "self_attn.k_proj.bias"))
            v = nx.linear(n, self.t(p + "self_attn.v_proj.weight"), self.t(p + "self_attn.v_proj.bias"))
            q = qwen_rope(np.ascontiguousarray(q.reshape(T, nh, hd).transpose(1, 0, 2)), cos, sin)
            k = qwen_rope(np.ascontiguousarray(k.reshape(T, nkv, hd).transpose(1, 0, 2)), cos, sin)
            v = np.ascontiguousarray(v.reshape(T, nkv, hd).transpose(1, 0, 2))
            if cache is not None:
                k, v = cache.append(i, k, v)
            a = nx.sdpa(q, k, v, mask).transpose(1, 0, 2).reshape(T, nh * hd)
            h = h + nx.linear(a, self.t(p + "self_attn.o_proj.weight"))
            n = nx.rms_norm(h, self.t(p + "post_attention_layernorm"), self.eps)
            g = nx.linear(n, self.t(p + "mlp.gate_proj.weight"))
            u = nx.linear(n, self.t(p + "mlp.up_proj.weight"))
            h = h + nx.linear(nx.silu(g) * u, self.t(p + "mlp.down_proj.weight"))
        return nx.rms_norm(h, self.t("norm"), self.eps)


class SpeechLM:
    """CosyVoice3LM pieces (llm.py:52-78) plus the build's greedy decode.

    Greedy selection: the reference only samples (llm.py:125-149).  The build
    defines greedy decoding as the argmax of the same ``log_softmax(head(h))``
    (llm.py:114) with every stop id masked -- what ``_sample`` does with
    ``ignore_eos`` and ``strict_min_len`` (llm.py:128-136) -- so a fixed-length
    run never stops early; ties resolve to the lowest id (``np.argmax``).
    """

    def __init__(self, W, meta, prefix: str = "llm."):
        self.W, self.p = W, prefix
        self.body = Qwen2(W, meta, prefix + "model.")
        self.speech_token_size = int(meta.get("speech_token_size", 6561))
        self.sos = self.speech_token_size
        self.task_id = self.speech_token_size + 2
        self.endofprompt_id = int(meta.get("endofprompt_id", 151646))

    def speech_emb(self, ids):
        return nx.embedding(self.W[self.p + "speech_embedding"], np.asarray(ids))

    def text_emb(self, ids):
        return nx.embedding(self.W[self.p + "model.embed_tokens"], np.asarray(ids))

    def head(self, h):
        b = self.W.get(self.p + "llm_decoder.bias") if hasattr(self.W, "get") else None
        return nx.linear(h, self.W[self.p + "llm_decoder.weight"], b)

    def prompt_embedding(self, text, prompt_text=(), prompt_speech=()):
        """``[sos, text, task, prompt speech]`` embeddings; llm.py:91-104."""
        text = list(prompt_text) + list(text)
        if self.endofprompt_id not in text:
            raise ValueError(f"CosyVoice 3 expects '<|endofprompt|>' (id {self.endofprompt_id}) "
                             f"somewhere in the prompt text")
        parts = [self.speech_emb([self.sos]), self.text_emb(text), self.speech_emb([self.task_id])]
        if len(prompt_speech):
            parts.append(self.speech_emb(list(prompt_speech)))
        return np.concatenate(parts, axis=0).astype(F32)

    def greedy(self, logp):
        return int(np.argmax(logp[: self.speech_token_size]))

    def generate_greedy(self, x0, n_tokens: int, forced: Optional[Sequence[int]] = None,
                        cache: Optional[KV] = None):
        """Decode ``n_tokens`` greedy tokens from prompt embeddings ``x0``.

        Returns ``(tokens, logps)``.  With ``forced`` the next input is the forced
        token (teacher forcing) while the greedy choice is still recorded.
        """
        cache = cache or self.body.new_cache()
        toks, logps = [], []
        x = x0
        for i in range(n_tokens):
            h = self.body.forward(x, cache)
            logp = nx.log_softmax(self.head(h[-1:]).astype(F32), axis=-1)[0]
            top = self.greedy(logp)
            toks.append(top)
            logps.append(logp)
            nxt = top if (forced is None or i >= len(forced)) else int(forced[i])
            x = self.speech_emb([nxt])
        return toks, np.stack(logps) if logps else np.zeros((0, 0), F32)

    def generate_sampled(self, x0, n_new_text: int, rng, min_ratio: float = 2.0, max_ratio: float = 20.0,
                         strict_min_len: bool = False, top_p: float = 0.8, top_k: int = 25,
                         win_size: int = 10, tau_r: float = 0.1):
        """The reference's sampling loop (llm.py:107-123) from prompt embeddings ``x0``:
        min / max lengths from the new text's length, one forward per step, the sampler of
        llm.py:125-149 (``nx.sample_token``) drawing from ``rng``; a stop id ends it."""
        min_len, max_len = int(n_new_text * min_ratio), int(n_new_text * max_ratio)
        cache = self.body.new_cache()
        out, x = [], x0
        sts = self.speech_token_size
        for i in range(max_len):
            h = self.body.forward(x, cache)
            logp = nx.log_softmax(self.head(h[-1:]).astype(F32), axis=-1)[0]
            top = nx.sample_token(logp, out, rng, sts, i < min_len, strict_min_len, top_p, top_k, win_size, tau_r)
            if sts <= top < sts + 200:
                break
            out.append(top)
            x = self.speech_emb([top])
        return out


# ---------------------------------------------------------------------------
# DiT estimator                                          cv3cpu/models/dit.py
# ---------------------------------------------------------------------------

def time_sinusoid(t, dim: int = 256, scale: float = 1000.0):
    """float32 sin/cos timestep features; dit.py:13-18."""
    half = dim // 2
    step = math.log(10000.0) / (half - 1)
    freqs = np.exp(np.arange(half, dtype=F32) * -step)
    ang = scale * np.asarray(t).reshape(-1, 1).astype(F32) * freqs[None, :]
    return np.concatenate([np.sin(ang), np.cos(ang)], axis=-1)


def dit_rope_angles(n: int, dim_head: int, theta: float = 10000.0):
    """Interleaved-pair rotary angles ``(n, dim_head)``, f64 -> f32; dit.py:21-29."""
    inv = 1.0 / (theta ** (np.arange(0, dim_head, 2, dtype=np.float64) / dim_head))
    ang = np.arange(n, dtype=np.float64)[:, None] * inv[None, :]
    return np.repeat(ang, 2, axis=-1).astype(F32)


def dit_partial_rope(x, ang):
    """Rotate channels ``[0, dim_head)`` of the whole projection, pairs (2i, 2i+1); dit.py:32-54."""
    r = ang.shape[-1]
    head = x[..., :r]
    c, s = np.cos(ang), np.sin(ang)
    pair = head.reshape(*head.shape[:-1], -1, 2)
    rot = np.stack([-pair[..., 1], pair[..., 0]], axis=-1).reshape(head.shape)
    return np.concatenate([head * c + rot * s, x[..., r:]], axis=-1)


class DiT:
    """F5-style DiT, forward as dit.py:144-180."""

    def __init__(self, W, meta, prefix: str = "flow.decoder.estimator."):
        m = meta.get("dit", {})
        self.W, self.p = W, prefix
        self.dim = int(m.get("dim", 1024))
        self.depth = int(m.get("depth", 22))
        self.heads = int(m.get("heads", 16))
        self.dim_head = int(m.get("dim_head", 64))
        self.chunk = int(m.get("static_chunk_size", 50))
        self.left = int(m.get("num_decoding_left_chunks", -1))
        self.kpos = int(m.get("conv_pos_kernel", 31))
        self.gpos = int(m.get("conv_pos_groups", 16))

    def t(self, name):
        return self.W[self.p + name]

    def time_embed(self, t):                                   # dit.py:86-90
        h = nx.linear(time_sinusoid(np.asarray(t, F32)), self.t("time_embed.time_mlp.0.weight"),
                      self.t("time_embed.time_mlp.0.bias"))
        return nx.linear(nx.silu(h), self.t("time_embed.time_mlp.2.weight"),
                         self.t("time_embed.time_mlp.2.bias"))

    def input_embed(self, x, cond, mu, spks):                  # dit.py:92-112
        b, n, _ = x.shape
        cat = np.concatenate([x, cond, mu, np.broadcast_to(spks[:, None, :], (b, n, spks.shape[1]))], -1)
        h = nx.linear(cat, self.t("input_embed.proj.weight"), self.t("input_embed.proj.bias"))
        pos = np.empty_like(h)
        pre = "input_embed.conv_pos_embed."
        for i in range(b):
            z = np.ascontiguousarray(h[i].T)
            for c in ("conv1", "conv2"):
                z = nx.mish(nx.conv1d(z, self.t(pre + c + ".0.weight"), self.t(pre + c + ".0.bias"),
                                      groups=self.gpos, pad=(self.kpos - 1, 0)))
            pos[i] = z.T
        return pos + h

    def attention(self, blk, x, ang, mask):                    # dit.py:114-129
        b, n, _ = x.shape
        q = nx.linear(x, self.t(blk + "attn.to_q.weight"), self.t(blk + "attn.to_q.bias"))
        k = nx.linear(x, self.t(blk + "attn.to_k.weight"), self.t(blk + "attn.to_k.bias"))
        v = nx.linear(x, self.t(blk + "attn.to_v.weight"), self.t(blk + "attn.to_v.bias"))
        q, k = dit_partial_rope(q, ang), dit_partial_rope(k, ang)
        h, d = self.heads, self.dim_head
        out = np.empty((b, n, h * d), F32)
        for i in range(b):
            split = lambda a: np.ascontiguousarray(a[i].reshape(n, h, d).transpose(1, 0, 2))  # noqa: E731
            out[i] = nx.sdpa(split(q), split(k), split(v), mask).transpose(1, 0, 2).reshape(n, h * d)
        return nx.linear(out, self.t(blk + "attn.to_out.0.weight"), self.t(blk + "attn.to_out.0.bias"))

    def feed_forward(self, blk, x):                            # dit.py:131-142
        h = nx.gelu_tanh(nx.linear(x, self.t(blk + "ff.ff.0.0.weight"), self.t(blk + "ff.ff.0.0.bias")))
        return nx.linear(h, self.t(blk + "ff.ff.2.weight"), self.t(blk + "ff.ff.2.bias"))

    def forward(self, x, mu, t, spks, cond, streaming: bool = False):
        """``x, mu, cond (B, 80, N)``, ``t (B,)``, ``spks (B, 80)`` -> ``(B, 80, N)``."""
        x = np.ascontiguousarray(np.swapaxes(x, 1, 2))
        mu = np.ascontiguousarray(np.swapaxes(mu, 1, 2))
        cond = np.ascontiguousarray(np.swapaxes(cond, 1, 2))
        n = x.shape[1]
        temb = self.time_embed(np.asarray(t, F32))
        h = self.input_embed(x, cond, mu, spks)
        ang = dit_rope_angles(n, self.dim_head)
        mask = ("chunk", self.chunk, self.left) if streaming else None
        st = nx.silu(temb)
        for i in range(self.depth):
            blk = f"transformer_blocks.{i}."
            mod = nx.linear(st, self.t(blk + "attn_norm.linear.weight"), self.t(blk + "attn_norm.linear.bias"))
            sh_a, sc_a, g_a, sh_f, sc_f, g_f = np.split(mod, 6, axis=1)
            z = nx.layer_norm(h, None, None, 1e-6) * (1.0 + sc_a[:, None]) + sh_a[:, None]
            h = h + g_a[:, None] * self.attention(blk, z, ang, mask)
            z = nx.layer_norm(h, None, None, 1e-6) * (1.0 + sc_f[:, None]) + sh_f[:, None]
            h = h + g_f[:, None] * self.feed_forward(blk, z)
        mod = nx.linear(st, self.t("norm_out.linear.weight"), self.t("norm_out.linear.bias"))
        scale, shift = np.split(mod, 2, axis=1)
        h = nx.layer_norm(h, None, None, 1e-6) * (1.0 + scale)[:, None] + shift[:, None]
        out = nx.linear(h, self.t("proj_out.weight"), self.t("proj_out.bias"))
        return np.ascontiguousarray(np.swapaxes(out, 1, 2))


# ---------------------------------------------------------------------------
# flow: token front end and the Euler/CFG solve          cv3cpu/models/flow.py
# ---------------------------------------------------------------------------

NOISE_SHAPE = (1, 80, 15000)                                   # flow.py:16


class Flow:
    def __init__(self, W, meta, prefix: str = "flow."):
        m = meta.get("flow", {})
        self.W, self.p, self.meta = W, prefix, meta
        self.ratio = int(m.get("token_mel_ratio", 2))
        self.look = int(m.get("pre_lookahead_len", 3))
        self.out_ch = int(m.get("output_size", 80))
        self.cfg = float(m.get("inference_cfg_rate", 0.7))
        self.steps = int(m.get("n_timesteps", 10))
        self.dit = DiT(W, meta, prefix + "decoder.estimator.")
        self._noise = None

    def t(self, name):
        return self.W[self.p + name]

    def noise(self, n: int):                                   # flow.py:36-43
        if self._noise is None:
            self._noise = nx.randn(NOISE_SHAPE, 0)
        if n > self._noise.shape[2]:
            raise ValueError(f"utterance needs {n} mel frames but the fixed CFM noise only has "
                             f"{self._noise.shape[2]}; split the text into shorter segments")
        return self._noise[:, :, :n]

    def pre_lookahead(self, e):                                # flow.py:46-56
        x = np.ascontiguousarray(e.T)
        h = nx.leaky_relu(nx.conv1d(x, self.t("pre_lookahead_layer.conv1.weight"),
                                    self.t("pre_lookahead_layer.conv1.bias"), pad=(0, self.look)), 0.01)
        k2 = _kernel(self.t("pre_lookahead_layer.conv2.weight"))
        h = nx.conv1d(h, self.t("pre_lookahead_layer.conv2.weight"),
                      self.t("pre_lookahead_layer.conv2.bias"), pad=(k2 - 1, 0))
        return h.T + e

    @staticmethod
    def schedule(steps: int):
        """Cosine t-span, float64 then float32; flow.py:68-69."""
        ts = 1.0 - np.cos(np.linspace(0.0, 1.0, steps + 1, dtype=np.float64) * 0.5 * np.pi)
        return ts.astype(F32)

    def solve_euler(self, mu, spks, cond, temperature: float = 1.0, streaming: bool = False):
        """Fixed-step Euler with CFG (slot 1 unconditioned); flow.py:58-93."""
        n = mu.shape[2]
        x = self.noise(n) * temperature
        ts = self.schedule(self.steps)
        mu_in = np.zeros((2, 80, n), F32)
        mu_in[0] = mu[0]
        spk_in = np.zeros((2, spks.shape[1]), F32)
        spk_in[0] = spks[0]
        cond_in = np.zeros((2, 80, n), F32)
        cond_in[0] = cond[0]
        t, dt = ts[0], ts[1] - ts[0]
        for step in range(1, len(ts)):
            d = self.dit.forward(np.broadcast_to(x, (2, 80, n)), mu_in, np.array([t, t], F32),
                                 spk_in, cond_in, streaming=streaming)
            x = x + dt * ((1.0 + self.cfg) * d[0:1] - self.cfg * d[1:2])
            t = t + dt
            if step < len(ts) - 1:
                dt = ts[step + 1] - t
        return x.astype(F32)

    def conditioning(self, token, prompt_token, prompt_feat, embedding):
        """``(mu, spks, cond, prompt_frames)`` for one utterance; flow.py:96-125."""
        emb = np.asarray(embedding, F32).reshape(1, -1)
        emb = emb / np.maximum(np.linalg.norm(emb, axis=1, keepdims=True), 1e-12)
        spk = nx.linear(emb, self.t("spk_embed_affine_layer.weight"), self.t("spk_embed_affine_layer.bias"))
        ids = np.maximum(np.concatenate([np.asarray(prompt_token, np.int64),
                                         np.asarray(token, np.int64)]), 0)
        h = np.repeat(self.pre_lookahead(nx.embedding(self.t("input_embedding"), ids)), self.ratio, axis=0)
        prompt_feat = np.asarray(prompt_feat, F32)
        p = prompt_feat.shape[0]
        if p > h.shape[0]:
            raise ValueError("prompt mel is longer than the token grid")
        cond = np.zeros((1, self.out_ch, h.shape[0]), F32)
        cond[0, :, :p] = prompt_feat.T
        return np.ascontiguousarray(h.T)[None], spk, cond, p

    def inference(self, token, prompt_token, prompt_feat, embedding, streaming: bool = False):
        mu, spk, cond, p = self.conditioning(token, prompt_token, prompt_feat, embedding)
        return self.solve_euler(mu, spk, cond, streaming=streaming)[0, :, p:]


# ---------------------------------------------------------------------------
# HiFT vocoder                                           cv3cpu/models/hift.py
# ---------------------------------------------------------------------------

def causal_pad(k: int, d: int = 1) -> int:                     # hift.py:14-16
    return int((k * d - d) / 2) * 2 + (k + 1) % 2


class HiFT:
    def __init__(self, W, meta, prefix: str = "hift."):
        m = meta.get("hift", {})
        self.W, self.p = W, prefix
        self.rates = list(m.get("upsample_rates", [8, 5, 3]))
        self.rb_k = list(m.get("resblock_kernel_sizes", [3, 7, 11]))
        self.rb_d = [list(d) for d in m.get("resblock_dilation_sizes", [[1, 3, 5]] * 3)]
        self.srb_k = list(m.get("source_resblock_kernel_sizes", [7, 7, 11]))
        self.srb_d = [list(d) for d in m.get("source_resblock_dilation_sizes", [[1, 3, 5]] * 3)]
        self.n_fft = int(m.get("istft_n_fft", 16))
        self.hop = int(m.get("istft_hop_len", 4))
        self.slope = float(m.get("lrelu_slope", 0.1))
        self.limit = float(m.get("audio_limit", 0.99))
        self.sr = int(m.get("sampling_rate", 24000))
        self.harm = int(m.get("nb_harmonics", 8)) + 1
        self.alpha = float(m.get("nsf_alpha", 0.1))
        self.sigma = float(m.get("nsf_sigma", 0.003))
        self.vthr = float(m.get("nsf_voiced_threshold", 10.0))
        self.look = int(m.get("conv_pre_look_right", 4))
        self.up = int(np.prod(self.rates)) * self.hop
        self.win = nx.hann_window(self.n_fft)
        self.noise_seed = int(m.get("noise_seed", 0))
        self._noise = None

    def t(self, name):
        return self.W[self.p + name]

    def k(self, name) -> int:
        return _kernel(self.t(name))

    def f0_predict(self, mel):
        """F0 head; hift.py:56-72.  The convs run in float32 (``conv1d`` casts),
        the classifier dot product in float64."""
        x = np.asarray(mel, dtype=np.float64)
        for i in range(5):
            w = np.asarray(self.t(f"f0_predictor.condnet.{i}.weight"), dtype=np.float64)
            b = np.asarray(self.t(f"f0_predictor.condnet.{i}.bias"), dtype=np.float64)
            kk = w.shape[-1]
            x = nx.elu(nx.conv1d(x, w, b, pad=(0, causal_pad(kk)) if i == 0 else (causal_pad(kk), 0)))
        cw = np.asarray(self.t("f0_predictor.classifier.weight"), dtype=np.float64)
        cb = np.asarray(self.t("f0_predictor.classifier.bias"), dtype=np.float64)
        return np.abs((x.T @ cw.T + cb)[:, 0])

    def noise(self, n: int):                                   # hift.py:75-81
        if self._noise is None or self._noise.shape[0] < n:
            need = max(n, 1)
            self._noise = nx.MT19937(self.noise_seed).random_float32(need * self.harm).reshape(need, self.harm)
        return self._noise[:n]

    def set_source_noise(self, buf):                           # hift.py:83-88
        self._noise = np.asarray(buf, dtype=F32)

    def excitation(self, f0):
        """NSF harmonic source ``(T,) -> (up*T,)``; hift.py:90-111."""
        T, up = f0.shape[0], self.up
        rad = (f0[:, None] * np.arange(1, self.harm + 1)[None, :] / self.sr) % 1.0
        phase = np.cumsum(rad, axis=0) * (2.0 * np.pi) * up
        sines = np.sin(np.repeat(phase, up, axis=0)).astype(F32)
        sines *= self.alpha
        uv = (np.repeat(f0, up) > self.vthr).astype(F32)[:, None]
        amp = uv * self.sigma + (1.0 - uv) * (self.alpha / 3.0)
        src = sines * uv + amp * self.noise(up * T)
        merged = nx.linear(src, self.t("m_source.l_linear.weight"), self.t("m_source.l_linear.bias"))
        return np.tanh(merged)[:, 0]

    def resblock(self, group, idx, x, kernel, dils):           # hift.py:114-129
        base = f"{group}.{idx}."
        for j, d in enumerate(dils):
            y = nx.snake(x, np.asarray(self.t(base + f"activations1.{j}.alpha"), F32))
            y = nx.conv1d(y, self.t(base + f"convs1.{j}.weight"), self.t(base + f"convs1.{j}.bias"),
                          dilation=d, pad=(causal_pad(kernel, d), 0))
            y = nx.snake(y, np.asarray(self.t(base + f"activations2.{j}.alpha"), F32))
            y = nx.conv1d(y, self.t(base + f"convs2.{j}.weight"), self.t(base + f"convs2.{j}.bias"),
                          pad=(causal_pad(kernel, 1), 0))
            x = y + x
        return x

    def spectral(self, mel, s_stft):
        """conv_pre .. conv_post, ``(80, T) -> (n_fft+2, up/hop*T + 1)``; hift.py:131-168."""
        x = nx.conv1d(mel, self.t("conv_pre.weight"), self.t("conv_pre.bias"),
                      pad=(0, causal_pad(self.k("conv_pre.weight"))))
        downs = list(np.cumprod([1] + self.rates[::-1][:-1]))[::-1]
        nk = len(self.rb_k)
        for i, r in enumerate(self.rates):
            x = nx.interpolate_nearest(nx.leaky_relu(x, self.slope), r)
            kk = self.k(f"ups.{i}.weight")
            x = nx.conv1d(x, self.t(f"ups.{i}.weight"), self.t(f"ups.{i}.bias"), pad=(kk - 1, 0))
            if i == len(self.rates) - 1:
                x = np.concatenate([x[:, 1:2], x], axis=1)
            u = int(downs[i])
            ks = self.k(f"source_downs.{i}.weight")
            if u == 1:
                si = nx.conv1d(s_stft, self.t(f"source_downs.{i}.weight"), self.t(f"source_downs.{i}.bias"),
                               pad=(causal_pad(ks), 0))
            else:
                si = nx.conv1d(s_stft, self.t(f"source_downs.{i}.weight"), self.t(f"source_downs.{i}.bias"),
                               stride=u, pad=(u - 1, 0))
            x = x + self.resblock("source_resblocks", i, si, self.srb_k[i], self.srb_d[i])
            acc = None
            for j in range(nk):
                r_ = self.resblock("resblocks", i * nk + j, x, self.rb_k[j], self.rb_d[j])
                acc = r_ if acc is None else acc + r_
            x = acc / nk
        x = nx.leaky_relu(x, 0.01)
        return nx.conv1d(x, self.t("conv_post.weight"), self.t("conv_post.bias"),
                         pad=(causal_pad(self.k("conv_post.weight")), 0))

    def spectral_chunked(self, mel, s_stft, chunk: int, context: int):
        """Exact time-chunked :meth:`spectral`; hift.py:170-194."""
        up = int(np.prod(self.rates))
        T = mel.shape[1]
        look = causal_pad(self.k("conv_pre.weight"))
        pieces = []
        for m0 in range(0, T, chunk):
            m1 = min(T, m0 + chunk)
            c0, c1 = max(0, m0 - context), min(T, m1 + look)
            sub = self.spectral(mel[:, c0:c1], s_stft[:, c0 * up: c1 * up + 1])
            lead, take = (m0 - c0) * up, (m1 - m0) * up
            pieces.append(sub[:, : 1 + take] if m0 == 0 else sub[:, 1 + lead: 1 + lead + take])
        return np.concatenate(pieces, axis=1)

    def source_stft(self, source):
        spec = nx.stft(source, self.n_fft, self.hop, self.win)
        return np.concatenate([spec.real, spec.imag], axis=0).astype(F32)

    def istft_head(self, x):
        """exp/clip magnitude, sin phase, iSTFT, clip; hift.py:204-210."""
        half = self.n_fft // 2 + 1
        mag = np.clip(np.exp(np.minimum(x[:half], 80.0)), None, 1e2)
        ph = np.sin(x[half:])
        y = nx.istft(mag * np.cos(ph) + 1j * mag * np.sin(ph), self.n_fft, self.hop, self.win)
        return np.clip(y, -self.limit, self.limit)

    def decode(self, mel, source, chunk=None, context: int = 64):   # hift.py:196-210
        s = self.source_stft(source)
        if chunk is None or mel.shape[1] <= chunk:
            x = self.spectral(mel, s)
        else:
            x = self.spectral_chunked(mel, s, chunk, context)
        return self.istft_head(x)

    def inference(self, mel, chunk=250, context: int = 64):    # hift.py:212-218
        mel = np.ascontiguousarray(mel, dtype=F32)
        f0 = self.f0_predict(mel)
        return self.decode(mel, self.excitation(f0.astype(F32)), chunk=chunk, context=context)
