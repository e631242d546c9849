"""Qwen2 decoder body on the GPU (mirror of ``cv3cpu/models/qwen2.py``).

``Qwen2Model.forward(x, cache)`` keeps the reference's contract (embeddings in,
final hidden states out, causal prefill, one-token steps see the whole cache)
for any number of rows of one sequence.  :class:`DecodeEngine` runs the
batched greedy decode: all sequences of a batch advance one token per step,
and a step -- 24 layers, the head, the greedy pick and the next input's
embedding -- is one CUDA graph replay with positions, cache lengths and token
ids kept in device memory.

Per-layer weights are fused once at load: q/k/v rows stacked into one
``(H + 2 Hk) * D``-row matrix with one bias, gate and up rows stacked into one
``2 * I``-row matrix; both keep the q8 layout, so a decode step streams each
int8 payload exactly once.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from .. import _dev as D
from .._lib import call
from ..quant import QTensor
from ._common import DecodeGemv, Graph, Lin, cat_rows, f32_of, interleave_rows

torch = D.torch


@dataclass
class Qwen2Config:
    hidden_size: int
    num_hidden_layers: int
    num_attention_heads: int
    num_key_value_heads: int
    intermediate_size: int
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1000000.0
    vocab_size: int = 151936

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_attention_heads

    @classmethod
    def from_meta(cls, meta: dict) -> "Qwen2Config":
        m = meta["qwen2"]
        return cls(**{k: m[k] for k in cls.__dataclass_fields__ if k in m})


def rope_tables(n: int, dim: int, theta: float):
    """Half-split RoPE tables, angles in float64 then cast (cv3cpu/models/qwen2.py:46-56)."""
    inv = 1.0 / (theta ** (np.arange(0, dim, 2, dtype=np.float64) / dim))
    ang = np.arange(n, dtype=np.float64)[:, None] * inv[None, :]
    ang = np.concatenate([ang, ang], axis=-1)
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


class KVCache:
    """Device KV cache for ``batch`` sequences: k/v ``[layer][seq][kv_head][cap][head_dim]`` fp32.

    ``len(cache)`` is the cached length of sequence 0 (the reference's one-sequence
    contract, cv3cpu/models/qwen2.py:74-121); capacity is reserved up front.
    """

    def __init__(self, layers: int, heads: int, head_dim: int, batch: int = 1, cap: int = 1024):
        self.layers, self.heads, self.head_dim, self.batch, self.cap = layers, heads, head_dim, batch, cap
        self.k = D.zeros((layers, batch, heads, cap, head_dim))
        self.v = D.zeros((layers, batch, heads, cap, head_dim))
        self.lengths = [0] * batch

    def __len__(self) -> int:
        return self.lengths[0]

    def layer_ptrs(self, i: int):
        return self.k[i].data_ptr(), self.v[i].data_ptr()

    def nbytes(self) -> int:
        return self.k.numel() * 4 * 2


class _Layer:
    __slots__ = ("qkv", "o", "gu", "down", "ln1", "ln2", "qkv32", "o32", "gu32", "down32")


class Qwen2Model:
    """Decoder-only Qwen2 over embeddings; forward follows cv3cpu/models/qwen2.py:139-179."""

    def __init__(self, weights, cfg: Qwen2Config, prefix: str = "llm.model."):
        self.w = weights
        self.cfg = cfg
        self.prefix = prefix
        self._layers = None
        self._rope = (0, None, None)

    # -- weights -----------------------------------------------------------------
    def _t(self, name):
        return self.w.weight(self.prefix + name)

    def layers(self):
        if self._layers is None:
            out = []
            for i in range(self.cfg.num_hidden_layers):
                p = f"layers.{i}."
                L = _Layer()
                qkv = self.w.cache((self.prefix + p + "qkv",), lambda p=p: cat_rows(
                    [self._t(p + f"self_attn.{n}_proj.weight") for n in "qkv"]))
                bqkv = self.w.cache((self.prefix + p + "qkv_bias",), lambda p=p: torch.cat(
                    [self.w.f32(self.prefix + p + f"self_attn.{n}_proj.bias") for n in "qkv"]).contiguous())
                gu = self.w.cache((self.prefix + p + "gate_up",), lambda p=p: cat_rows(
                    [self._t(p + "mlp.gate_proj.weight"), self._t(p + "mlp.up_proj.weight")]))
                L.qkv = Lin(qkv, bqkv)
                L.o = Lin(self._t(p + "self_attn.o_proj.weight"))
                L.gu = Lin(gu)
                L.down = Lin(self._t(p + "mlp.down_proj.weight"))
                L.ln1 = self.w.f32(self.prefix + p + "input_layernorm")
                L.ln2 = self.w.f32(self.prefix + p + "post_attention_layernorm")
                L.qkv32 = L.o32 = L.gu32 = L.down32 = None
                out.append(L)
            self._layers = out
        return self._layers

    def _wide(self, L: _Layer):
        """fp32 copies (dequantised on the GPU) for multi-row prefill GEMMs."""
        if L.qkv32 is None:
            L.qkv32 = Lin(f32_of(L.qkv._keep[0]), L.qkv._keep[1])
            L.o32 = Lin(f32_of(L.o._keep[0]))
            L.gu32 = Lin(f32_of(L.gu._keep[0]))
            L.down32 = Lin(f32_of(L.down._keep[0]))
        return L.qkv32, L.o32, L.gu32, L.down32

    def norm_w(self):
        return self.w.f32(self.prefix + "norm")

    def rope(self, n: int):
        if self._rope[0] < n:
            cap = max(n, 2 * self._rope[0], 1024)
            c, s = rope_tables(cap, self.cfg.head_dim, self.cfg.rope_theta)
            self._rope = (cap, torch.from_numpy(c).cuda(), torch.from_numpy(s).cuda())
        return self._rope[1], self._rope[2]

    def embed(self, ids):
        from .. import ops
        return ops.embedding(self.w.weight(self.prefix + "embed_tokens"), ids)

    def new_cache(self, batch: int = 1, cap: int = 1024) -> KVCache:
        c = self.cfg
        return KVCache(c.num_hidden_layers, c.num_key_value_heads, c.head_dim, batch, cap)

    # -- forward over T rows of one sequence ---------------------------------------
    def forward(self, x, cache: KVCache = None, seq: int = 0, tile_bytes: int = 0):
        """``x`` ``(T, hidden)`` -> final hidden states ``(T, hidden)`` (host in -> host out)."""
        host = D.is_host(x)
        h = D.dev(x).clone()
        T = int(h.shape[0])
        c = self.cfg
        H, Hk, hd, hid = c.num_attention_heads, c.num_key_value_heads, c.head_dim, c.hidden_size
        if cache is None:
            cache = self.new_cache(1, max(T, 1))
            seq = 0
        past = cache.lengths[seq]
        if past + T > cache.cap:
            raise ValueError(f"KV cache capacity {cache.cap} exceeded ({past} + {T})")
        cos, sin = self.rope(past + T)
        st = D.stream()
        n = D.empty((T, hid))
        qkv = D.empty((T, (H + 2 * Hk) * hd))
        q = D.empty((T, H * hd))
        a = D.empty((T, H * hd))
        gu = D.empty((T, 2 * c.intermediate_size))
        act = D.empty((T, c.intermediate_size))
        seqs = torch.full((T,), seq, dtype=torch.int32, device="cuda")
        pos = torch.arange(past, past + T, dtype=torch.int32, device="cuda")
        scale = float(np.float32(1.0 / np.sqrt(hd)))
        mask_kind = 1 if T > 1 else 0
        for i, L in enumerate(self.layers()):
            lq, lo, lg, ld = (L.qkv, L.o, L.gu, L.down) if T <= 8 else self._wide(L)
            kc, vc = cache.layer_ptrs(i)
            call("cv3_rms_norm", h.data_ptr(), L.ln1.data_ptr(), T, hid, c.rms_norm_eps, n.data_ptr(), st)
            lq(n.data_ptr(), T, qkv.data_ptr(), stream=st)
            call("cv3_rope_qkv_append", qkv.data_ptr(), T, qkv.shape[1], cos.data_ptr(), sin.data_ptr(),
                 seqs.data_ptr(), pos.data_ptr(), H, Hk, hd, q.data_ptr(), kc, vc, cache.cap, st)
            kseq = seq * Hk * cache.cap * hd * 4
            call("cv3_attention", q.data_ptr(), 0, hd, H * hd,
                 kc + kseq, 0, cache.cap * hd, hd, vc + kseq, 0, cache.cap * hd, hd,
                 a.data_ptr(), 0, hd, H * hd, 1, H, Hk, T, past + T, hd, scale, mask_kind, past, 0, st)
            lo(a.data_ptr(), T, h.data_ptr(), residual=h.data_ptr(), stream=st)
            call("cv3_rms_norm", h.data_ptr(), L.ln2.data_ptr(), T, hid, c.rms_norm_eps, n.data_ptr(), st)
            lg(n.data_ptr(), T, gu.data_ptr(), stream=st)
            call("cv3_swiglu", gu.data_ptr(), T, c.intermediate_size, act.data_ptr(), st)
            ld(act.data_ptr(), T, h.data_ptr(), residual=h.data_ptr(), stream=st)
        out = D.empty((T, hid))
        call("cv3_rms_norm", h.data_ptr(), self.norm_w().data_ptr(), T, hid, c.rms_norm_eps, out.data_ptr(), st)
        cache.lengths[seq] = past + T
        return D.out(out, host)


    def forward_batch(self, xs, cache: KVCache):
        """Prefill of several sequences in one pass: ``xs[b]`` ``(T_b, hidden)`` device
        embeddings of sequence b (cache row b, appended from position 0).  Rows of all
        sequences are stacked, so every GEMM runs once over all of them (each row's result
        is the same as in :meth:`forward`: a row's products do not depend on the other
        rows); RoPE and the cache append take per-row sequence ids and positions, and the
        causal attention runs per sequence.  Returns the final hidden states of each
        sequence's last row, ``(len(xs), hidden)``."""
        c = self.cfg
        H, Hk, hd, hid = c.num_attention_heads, c.num_key_value_heads, c.head_dim, c.hidden_size
        lens = [int(x.shape[0]) for x in xs]
        if max(lens) > cache.cap:
            raise ValueError(f"KV cache capacity {cache.cap} exceeded ({max(lens)})")
        offs = np.concatenate([[0], np.cumsum(lens)]).astype(np.int64)
        T = int(offs[-1])
        h = torch.cat([D.dev(x) for x in xs], 0).contiguous()
        cos, sin = self.rope(max(lens))
        st = D.stream()
        n = D.empty((T, hid))
        qkv = D.empty((T, (H + 2 * Hk) * hd))
        q = D.empty((T, H * hd))
        a = D.empty((T, H * hd))
        gu = D.empty((T, 2 * c.intermediate_size))
        act = D.empty((T, c.intermediate_size))
        seqs = torch.cat([torch.full((t,), b, dtype=torch.int32) for b, t in enumerate(lens)]).cuda()
        pos = torch.cat([torch.arange(t, dtype=torch.int32) for t in lens]).cuda()
        scale = float(np.float32(1.0 / np.sqrt(hd)))
        for i, L in enumerate(self.layers()):
            lq, lo, lg, ld = (L.qkv, L.o, L.gu, L.down) if T <= 8 else self._wide(L)
            kc, vc = cache.layer_ptrs(i)
            call("cv3_rms_norm", h.data_ptr(), L.ln1.data_ptr(), T, hid, c.rms_norm_eps, n.data_ptr(), st)
            lq(n.data_ptr(), T, qkv.data_ptr(), stream=st)
            call("cv3_rope_qkv_append", qkv.data_ptr(), T, qkv.shape[1], cos.data_ptr(), sin.data_ptr(),
                 seqs.data_ptr(), pos.data_ptr(), H, Hk, hd, q.data_ptr(), kc, vc, cache.cap, st)
            for b, t in enumerate(lens):
                kseq = b * Hk * cache.cap * hd * 4
                row = int(offs[b]) * H * hd * 4
                call("cv3_attention", q.data_ptr() + row, 0, hd, H * hd,
                     kc + kseq, 0, cache.cap * hd, hd, vc + kseq, 0, cache.cap * hd, hd,
                     a.data_ptr() + row, 0, hd, H * hd, 1, H, Hk, t, t, hd, scale, 1 if t > 1 else 0, 0, 0, st)
            lo(a.data_ptr(), T, h.data_ptr(), residual=h.data_ptr(), stream=st)
            call("cv3_rms_norm", h.data_ptr(), L.ln2.data_ptr(), T, hid, c.rms_norm_eps, n.data_ptr(), st)
            lg(n.data_ptr(), T, gu.data_ptr(), stream=st)
            call("cv3_swiglu", gu.data_ptr(), T, c.intermediate_size, act.data_ptr(), st)
            ld(act.data_ptr(), T, h.data_ptr(), residual=h.data_ptr(), stream=st)
        last = h[torch.as_tensor(offs[1:] - 1, device="cuda")].contiguous()
        out = D.empty((len(xs), hid))
        call("cv3_rms_norm", last.data_ptr(), self.norm_w().data_ptr(), len(xs), hid, c.rms_norm_eps,
             out.data_ptr(), st)
        for b, t in enumerate(lens):
            cache.lengths[b] = t
        return out


def pk_sm_count() -> int:
    return int(torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count)


class DecodeEngine:
    """Batched greedy decode, one CUDA graph per step.

    The fused qkv projection runs as ``QKV_SPLITS`` K splits of one cluster (its 1152 rows
    alone fill only half the SMs; the splits' sums of squares for the folded RMSNorm are
    added by the cluster's first CTA).

    Device state per sequence: ``pos`` (position of the token being fed),
    ``lens`` (cache length after it is appended), ``next_ids`` (token fed next)
    and ``history`` (tokens chosen so far).  A step runs every layer on the
    ``batch`` rows, the head GEMV, :c:func:`cv3_head_select` (log_softmax,
    first argmax over the speech tokens, bookkeeping) and the embedding gather
    of the chosen tokens into the next step's input.
    """

    QKV_SPLITS = 2

    def __init__(self, model: Qwen2Model, head_w, speech_emb, speech_tokens: int, batch: int, cap: int,
                 max_steps: int):
        c = model.cfg
        self.m, self.c, self.B, self.cap = model, c, batch, cap
        H, Hk, hd, hid = c.num_attention_heads, c.num_key_value_heads, c.head_dim, c.hidden_size
        self.cache = model.new_cache(batch, cap)
        self.head = Lin(head_w)
        self.vocab = self.head.n
        self.select = speech_tokens
        self.emb = speech_emb
        self.h = D.zeros((batch, hid))
        self.n = D.empty((batch, hid))
        self.qkv = D.empty((batch, (H + 2 * Hk) * hd))
        self.q = D.empty((batch, H * hd))
        self.a = D.empty((batch, H * hd))
        self.gu = D.empty((batch, 2 * c.intermediate_size))
        self.act = D.empty((batch, c.intermediate_size))
        self.logits = D.empty((batch, self.vocab))
        self.logp = D.empty((batch, self.vocab))
        self.next_ids = torch.zeros(batch, dtype=torch.int64, device="cuda")
        self.seqs = torch.arange(batch, dtype=torch.int32, device="cuda")
        self.pos = torch.zeros(batch, dtype=torch.int32, device="cuda")
        self.lens = torch.zeros(batch, dtype=torch.int32, device="cuda")
        self.step_no = torch.zeros(1, dtype=torch.int32, device="cuda")
        self.history = torch.zeros((batch, max_steps), dtype=torch.int64, device="cuda")
        self.max_steps = max_steps
        self.cos, self.sin = model.rope(cap)
        self.scale = float(np.float32(1.0 / np.sqrt(hd)))
        self.graph = None
        self.keep_logp = False
        self.sampling = None  # (top_p, top_k, win_size, tau_r, strict): device sampler instead of greedy
        # fused q8 decode GEMVs (RMSNorm in, residual / SwiGLU out) where the layer is q8
        self.fast = []
        for i, L in enumerate(model.layers()):
            p = f"layers.{i}."
            ws = [L.qkv._keep[0], L.o._keep[0], model._t(p + "mlp.gate_proj.weight"),
                  model._t(p + "mlp.up_proj.weight"), L.down._keep[0]]
            if all(isinstance(w, QTensor) and w.kind == "q8" for w in ws):   # (q4 layers: generic path)
                gu = model.w.cache((model.prefix + p + "gate_up_interleaved",), lambda ws=ws: interleave_rows(ws[2], ws[3]))
                self.fast.append((DecodeGemv(ws[0], L.qkv._keep[1], L.ln1, c.rms_norm_eps, mma_splits=self.QKV_SPLITS),
                                  DecodeGemv(ws[1]),
                                  DecodeGemv(gu, norm_w=L.ln2, eps=c.rms_norm_eps, swiglu=True),
                                  DecodeGemv(ws[4], mma_splits=5)))
            else:
                self.fast.append(None)
        self.fast_head = DecodeGemv(head_w, norm_w=model.norm_w(), eps=c.rms_norm_eps) \
            if isinstance(head_w, QTensor) and head_w.kind == "q8" else None
        self._mk = self._persistent_setup()

    # -- persistent decode (cv3_decode_steps): every step of a run in one launch ----------
    def _persistent_setup(self):
        """Parameter block and scratch of the persistent decode kernel, or None where it does
        not apply (a layer or the head not q8, head dim != 64, more than 8 sequences,
        hidden > 1216 or intermediate > 4864)."""
        from .. import _lib
        c, B = self.c, self.B
        hid, inter = c.hidden_size, c.intermediate_size
        e = self.emb
        if (B > 8 or c.head_dim != 64 or hid != c.num_attention_heads * 64 or hid % 64 or hid > 1216
                or self.cap > 1536
                or inter % 64 or inter > 4864 or c.num_attention_heads // c.num_key_value_heads > 8
                or self.fast_head is None or any(F is None for F in self.fast)
                or any(g.kp != g.k for F in self.fast for g in F) or self.fast_head.kp != hid
                or (isinstance(e, QTensor) and (e.kind != "q8" or e.padded_k != hid))):
            return None
        ptrs = []
        for i, F in enumerate(self.fast):
            kc, vc = self.cache.layer_ptrs(i)
            qkv, o, gu, dn = F
            ptrs += [qkv.q, qkv.scales, qkv.bias, qkv.norm, o.q, o.scales, gu.q, gu.scales, gu.norm, dn.q, dn.scales,
                     kc, vc]
        if any(v is None for v in ptrs):
            return None
        keep = []
        table = torch.tensor(ptrs, dtype=torch.int64, device="cuda")
        keep.append(table)
        # the head in whole 16-row tiles (zero rows past the vocabulary; never read back)
        if self.fast_head.bias is not None:
            return None
        hw = self.fast_head._keep[0]
        hq, hs = hw.q, hw.scales
        pad = (-self.vocab) % 16
        if pad:
            hq = torch.cat([hq, torch.zeros((pad, hq.shape[1]), dtype=hq.dtype, device="cuda")]).contiguous()
            hs = torch.cat([hs, torch.zeros((pad, hs.shape[1]), dtype=hs.dtype, device="cuda")]).contiguous()
        keep += [hq, hs]
        H, Hk = c.num_attention_heads, c.num_key_value_heads
        nch = -(-self.cap // 64)
        parts = -(-(inter // 64) // 19)
        h1 = D.empty((B, hid))
        attn_part = D.empty((B, H, nch, 66))
        ntf = -(-self.vocab // 16)
        part = D.empty((max((hid // 16) * parts * 16 * 8, 8 * ntf * 4),))
        lib = _lib.load()
        words = int(lib.cv3_decode_sync_words(len(self.fast), hid))
        sync = torch.zeros(words, dtype=torch.int32, device="cuda")
        keep += [h1, attn_part, part, sync]
        P = _lib.DecodeParams()
        P.layers = table.data_ptr()
        P.n_layers, P.batch, P.hidden = len(self.fast), B, hid
        P.heads, P.kv_heads, P.head_dim, P.inter = H, Hk, c.head_dim, inter
        P.eps, P.scale, P.cap = c.rms_norm_eps, self.scale, self.cap
        P.cos_table, P.sin_table = self.cos.data_ptr(), self.sin.data_ptr()
        P.final_norm = self.m.norm_w().data_ptr()
        P.head_q, P.head_s = hq.data_ptr(), hs.data_ptr()
        P.vocab, P.select = self.vocab, self.select
        if isinstance(e, QTensor):
            P.emb, P.emb_scales, P.emb_rows = e.q.data_ptr(), e.scales.data_ptr(), int(e.shape[0])
        else:
            P.emb, P.emb_scales, P.emb_rows = e.data_ptr(), None, int(e.shape[0])
        P.h, P.h1, P.qkv, P.attn_part = self.h.data_ptr(), h1.data_ptr(), self.qkv.data_ptr(), attn_part.data_ptr()
        P.part, P.part_floats, P.act = part.data_ptr(), int(part.numel()), self.act.data_ptr()
        P.attn = self.a.data_ptr()
        P.logits, P.logp = self.logits.data_ptr(), None
        P.pos, P.lens, P.next_ids = self.pos.data_ptr(), self.lens.data_ptr(), self.next_ids.data_ptr()
        P.history, P.hist_stride = self.history.data_ptr(), self.max_steps
        P.step, P.sync, P.sync_words = self.step_no.data_ptr(), sync.data_ptr(), words
        return {"params": P, "keep": keep, "sync": sync}

    @property
    def persistent_ok(self) -> bool:
        return self._mk is not None

    def steps_persistent(self, n: int, stream=None):
        """``n`` greedy decode steps in one cooperative launch (cv3_decode_steps)."""
        import ctypes
        if self._mk is None:
            raise RuntimeError("persistent decode needs q8 layers and head, head dim 64, <= 8 sequences")
        P = self._mk["params"]
        P.logp = self.logp.data_ptr() if self.keep_logp else None
        P.steps = int(n)
        call("cv3_decode_steps", ctypes.byref(P), stream if stream is not None else D.stream())

    def reset_persistent(self):
        """Zero the completion counters (after a reported wait failure left them uneven)."""
        if self._mk is not None:
            self._mk["sync"].zero_()

    def launches(self, st):
        """One decode step for every sequence (all pointers fixed -> graph-capturable)."""
        c, B = self.c, self.B
        H, Hk, hd, hid = c.num_attention_heads, c.num_key_value_heads, c.head_dim, c.hidden_size
        for i, L in enumerate(self.m.layers()):
            kc, vc = self.cache.layer_ptrs(i)
            F = self.fast[i]
            if F is not None:
                F[0](self.h.data_ptr(), B, self.qkv.data_ptr(), stream=st)
                # RoPE, cache append and attention in one launch (rows are the sequences in order)
                call("cv3_decode_rope_attention", self.qkv.data_ptr(), self.qkv.shape[1], self.cos.data_ptr(),
                     self.sin.data_ptr(), self.pos.data_ptr(), kc, vc, self.lens.data_ptr(), B, H, Hk, hd,
                     self.cap, self.scale, self.a.data_ptr(), st)
                F[1](self.a.data_ptr(), B, self.h.data_ptr(), residual=self.h.data_ptr(), stream=st)
                F[2](self.h.data_ptr(), B, self.act.data_ptr(), stream=st)
                F[3](self.act.data_ptr(), B, self.h.data_ptr(), residual=self.h.data_ptr(), stream=st)
                continue
            call("cv3_rms_norm", self.h.data_ptr(), L.ln1.data_ptr(), B, hid, c.rms_norm_eps, self.n.data_ptr(), st)
            L.qkv(self.n.data_ptr(), B, self.qkv.data_ptr(), stream=st)
            call("cv3_rope_qkv_append", self.qkv.data_ptr(), B, self.qkv.shape[1], self.cos.data_ptr(),
                 self.sin.data_ptr(), self.seqs.data_ptr(), self.pos.data_ptr(), H, Hk, hd, self.q.data_ptr(),
                 kc, vc, self.cap, st)
            call("cv3_decode_attention", self.q.data_ptr(), kc, vc, self.lens.data_ptr(), B, H, Hk, hd, self.cap,
                 self.scale, self.a.data_ptr(), st)
            L.o(self.a.data_ptr(), B, self.h.data_ptr(), residual=self.h.data_ptr(), stream=st)
            call("cv3_rms_norm", self.h.data_ptr(), L.ln2.data_ptr(), B, hid, c.rms_norm_eps, self.n.data_ptr(), st)
            L.gu(self.n.data_ptr(), B, self.gu.data_ptr(), stream=st)
            call("cv3_swiglu", self.gu.data_ptr(), B, c.intermediate_size, self.act.data_ptr(), st)
            L.down(self.act.data_ptr(), B, self.h.data_ptr(), residual=self.h.data_ptr(), stream=st)
        if self.fast_head is not None and B <= 32:
            self.fast_head(self.h.data_ptr(), B, self.logits.data_ptr(), stream=st)
            self.select_and_feed(st, logits_ready=True)
            return
        call("cv3_rms_norm", self.h.data_ptr(), self.m.norm_w().data_ptr(), B, hid, c.rms_norm_eps,
             self.n.data_ptr(), st)
        self.select_and_feed(st)

    def enable_sampling(self, top_p: float, top_k: int, win_size: int, tau_r: float, strict: bool):
        """Choose tokens with the device sampler (cv3_sample_select) instead of the greedy
        head: per-sequence numpy PCG64 states, token counts, min/max lengths and done flags
        live on the device, so a sampled step is graph-capturable like a greedy one."""
        B = self.B
        self.sampling = (float(top_p), int(top_k), int(win_size), float(tau_r), 1 if strict else 0)
        self.rng_state = torch.zeros((B, 4), dtype=torch.int64, device="cuda")
        self.min_len = torch.zeros(B, dtype=torch.int32, device="cuda")
        self.max_len = torch.zeros(B, dtype=torch.int32, device="cuda")
        self.count = torch.zeros(B, dtype=torch.int32, device="cuda")
        self.done = torch.zeros(B, dtype=torch.int32, device="cuda")
        self.graph = None

    def select_and_feed(self, st, logits_ready: bool = False):
        if not logits_ready:
            self.head(self.n.data_ptr(), self.B, self.logits.data_ptr(), stream=st)
        if self.sampling is not None:
            top_p, top_k, win, tau_r, strict = self.sampling
            call("cv3_sample_select", self.logits.data_ptr(), self.B, self.vocab, self.select,
                 self.min_len.data_ptr(), self.max_len.data_ptr(), strict, top_p, top_k, win, tau_r,
                 self.rng_state.data_ptr(), self.next_ids.data_ptr(), self.pos.data_ptr(), self.lens.data_ptr(),
                 self.history.data_ptr(), self.max_steps, self.count.data_ptr(), self.done.data_ptr(),
                 self.logp.data_ptr() if self.keep_logp else None, st)
            self._feed(st)
            return
        call("cv3_head_select", self.logits.data_ptr(), self.B, self.vocab, self.select,
             self.logp.data_ptr() if self.keep_logp else None, self.next_ids.data_ptr(), self.pos.data_ptr(),
             self.lens.data_ptr(), self.history.data_ptr(), self.max_steps, self.step_no.data_ptr(), st)
        self._feed(st)

    def _feed(self, st):
        """The chosen tokens' speech embeddings become the next step's input rows."""
        e = self.emb
        if isinstance(e, QTensor):
            call("cv3_embedding", e.q.data_ptr(), 3 if e.kind == "q4" else 2, e.scales.data_ptr(), int(e.shape[0]),
                 int(e.shape[1]),
                 e.padded_k, self.next_ids.data_ptr(), self.B, self.h.data_ptr(), int(e.shape[1]), None, st)
        else:
            call("cv3_embedding", e.data_ptr(), 0, None, int(e.shape[0]), int(e.shape[1]), int(e.shape[1]),
                 self.next_ids.data_ptr(), self.B, self.h.data_ptr(), int(e.shape[1]), None, st)

    def prefill(self, prompts):
        """Run each sequence's prompt rows, pick its first token, set positions."""
        if len(prompts) != self.B:
            raise ValueError(f"{len(prompts)} prompts for a batch of {self.B}")
        self.cache.lengths = [0] * self.B          # a new batch overwrites the cache from position 0
        last = self.m.forward_batch([D.dev(x) for x in prompts], self.cache)
        T = torch.tensor([int(np.shape(x)[0]) for x in prompts], dtype=torch.int32, device="cuda")
        self.pos.copy_(T - 1)       # head_select advances pos/lens by one
        self.lens.copy_(T)
        self.step_no.zero_()
        self.n.copy_(last)
        self.select_and_feed(D.stream())

    def capture(self):
        g = Graph()
        g.capture(self.launches)
        self.graph = g

    def step(self):
        if self.graph is None:
            self.launches(D.stream())
        else:
            self.graph.replay()

    def run_sampled(self, prompts, rng_states, min_lens, max_lens, poll: int = 8):
        """Sampled decode (enable_sampling first) until every sequence has drawn a stop id or
        reached its max length.  ``rng_states``: per sequence numpy PCG64 ``(state, inc)``.
        Steps run as graph replays; the done flags are read every ``poll`` steps (a finished
        sequence's steps change nothing).  Returns the token lists and the final states."""
        if self.sampling is None:
            raise RuntimeError("run_sampled needs enable_sampling()")
        B = self.B
        if not (len(prompts) == len(rng_states) == len(min_lens) == len(max_lens) == B):
            raise ValueError("one prompt, random state, min and max length per sequence")
        if max(max_lens) > self.max_steps:
            raise ValueError("max length exceeds the engine's max_steps")
        if max(int(np.shape(x)[0]) for x in prompts) + max(max_lens) > self.cap:
            raise ValueError("prompt + max length exceed the KV cache capacity")
        m64 = (1 << 64) - 1
        words = []
        for st_, inc in rng_states:
            for v in ((st_ >> 64) & m64, st_ & m64, (inc >> 64) & m64, inc & m64):
                words.append(v - (1 << 64) if v >= (1 << 63) else v)  # as int64 bit patterns
        self.rng_state.copy_(torch.tensor(words, dtype=torch.int64).view(B, 4))
        self.min_len.copy_(torch.tensor(list(min_lens), dtype=torch.int32))
        self.max_len.copy_(torch.tensor(list(max_lens), dtype=torch.int32))
        self.count.zero_()
        self.done.copy_(torch.tensor([1 if m <= 0 else 0 for m in max_lens], dtype=torch.int32))
        self.prefill(prompts)
        if self.graph is None:
            state = (self.h, self.pos, self.lens, self.step_no, self.next_ids, self.history, self.rng_state,
                     self.count, self.done)
            saved = [t.clone() for t in state]
            self.capture()
            for t, v in zip(state, saved):
                t.copy_(v)
        steps = 1
        while steps < max(max_lens) and not bool(self.done.all()):
            for _ in range(min(poll, max(max_lens) - steps)):
                self.step()
                steps += 1
        counts = self.count.cpu().tolist()
        hist = self.history.cpu().numpy()
        rs = self.rng_state.cpu().numpy().astype(np.uint64).tolist()
        out_states = [((int(r[0]) << 64) | int(r[1]), (int(r[2]) << 64) | int(r[3])) for r in rs]
        return [hist[b, :counts[b]].tolist() for b in range(B)], out_states

    def run(self, prompts, n_tokens: int, use_graph: bool = True, persistent: bool = False):
        """Greedy-decode ``n_tokens`` tokens for every prompt; returns ``[B][n_tokens]`` ids (device).
        The steps after the prefill run as one CUDA graph per step (``use_graph``), eager launches,
        or -- ``persistent`` -- one cooperative launch for all of them (cv3_decode_steps: the
        weights stream into shared memory ahead of the layer chain)."""
        if n_tokens > self.max_steps:
            raise ValueError("n_tokens exceeds max_steps")
        if max(int(np.shape(x)[0]) for x in prompts) + n_tokens > self.cap:
            raise ValueError("prompt + tokens exceed the KV cache capacity")
        self.prefill(prompts)
        if persistent and self.persistent_ok:
            if n_tokens > 1:
                self.steps_persistent(n_tokens - 1)
            return self.history[:, :n_tokens].clone()
        if use_graph and self.graph is None and n_tokens > 1:
            # capture replays from a snapshot of the state so capture's own launch has no effect
            saved = [t.clone() for t in (self.h, self.pos, self.lens, self.step_no, self.next_ids, self.history)]
            self.capture()
            for t, s in zip((self.h, self.pos, self.lens, self.step_no, self.next_ids, self.history), saved):
                t.copy_(s)
        for _ in range(n_tokens - 1):
            self.step()
        return self.history[:, :n_tokens].clone()
