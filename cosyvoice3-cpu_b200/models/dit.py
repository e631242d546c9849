"""The F5-style DiT flow estimator on the GPU (mirror of ``cv3cpu/models/dit.py``).

Activations are token-major ``[batch * frames, 1024]`` rows.  Per process the
weights are prepared once: q/k/v rows fused into one ``3072 x 1024`` matrix,
the 22 blocks' AdaLN matrices and ``norm_out`` stacked into one matrix (they
all multiply the same ``silu(temb)`` row), and q8 matrices dequantised on the
device for the dense GEMMs (exact: ``float(q) * float(scale)``).

Constant tables are built on the host exactly as the reference builds them:
the sinusoidal time features for a timestep (dit.py:13-18, float32 NumPy) and
the partial-RoPE angles (dit.py:21-29, float64 then float32, cos/sin taken in
float32).
"""

from __future__ import annotations

import math

import numpy as np

from .. import _dev as D
from .._lib import call
from ..quant import QTensor
from ._common import TC_MIN_ROWS, ConvTC, Lin, LinQ8, cat_rows, f32_of

torch = D.torch


def time_features(t, dim: int = 256, scale: float = 1000.0) -> np.ndarray:
    """Sinusoidal timestep features, float32 as dit.py:13-18 computes them."""
    half = dim // 2
    step = math.log(10000.0) / (half - 1)
    freqs = np.exp(np.arange(half, dtype=np.float32) * -step)
    emb = scale * np.asarray(t).reshape(-1, 1).astype(np.float32) * freqs[None, :]
    return np.concatenate([np.sin(emb), np.cos(emb)], axis=-1)


def rope_angle_tables(n: int, dim_head: int, theta: float = 10000.0):
    """cos/sin of the interleaved rotary angles (dit.py:21-29 and :51-52)."""
    inv = 1.0 / (theta ** (np.arange(0, dim_head, 2, dtype=np.float64) / dim_head))
    ang = np.repeat(np.outer(np.arange(n, dtype=np.float64), inv), 2, axis=-1).astype(np.float32)
    return np.cos(ang), np.sin(ang)


class _Block:
    __slots__ = ("qkv", "out", "ff1", "ff2")


class Workspace:
    """Activation buffers of one (batch, frames) shape; reused by every step."""

    def __init__(self, B: int, N: int, dim: int, ff: int, mel: int = 80, spk: int = 80):
        R = B * N
        self.B, self.N, self.R = B, N, R
        self.cat = D.empty((R, 3 * mel + spk))
        self.h = D.empty((R, dim))
        self.z = D.empty((R, dim))
        self.qkv = D.empty((R, 3 * dim))
        self.a = D.empty((R, dim))
        self.y = D.empty((R, dim))
        self.f1 = D.empty((R, ff))
        self.c2 = D.empty((B, dim, N))
        self.out = D.empty((R, mel))
        self.dim, self.ff = dim, ff
        self.zp = None

    def planes(self):
        """Activation-plane buffers of the q8 GEMMs (fp16 [R][2k] + int8 exponents [k/64][lde]):
        zp/ze for the normalised rows and the attention output, fp/fe for the GELU output."""
        if self.zp is None:
            R = self.R
            self.lde = (R + 15) // 16 * 16
            self.zp = torch.empty((R, 2 * self.dim), dtype=torch.float16, device="cuda")
            self.ze = torch.empty((self.dim // 64, self.lde), dtype=torch.int8, device="cuda")
            self.fp = torch.empty((R, 2 * self.ff), dtype=torch.float16, device="cuda")
            self.fe = torch.empty((self.ff // 64, self.lde), dtype=torch.int8, device="cuda")
        return self


class DiT:
    """``cosyvoice.flow.DiT.dit.DiT`` (dim 1024, depth 22, heads 16) on the device."""

    def __init__(self, weights, prefix: str = "flow.decoder.estimator."):
        self.w = weights
        self.p = prefix
        m = weights.meta.get("dit", {})
        self.dim = int(m.get("dim", 1024))
        self.depth = int(m.get("depth", 22))
        self.heads = int(m.get("heads", 16))
        self.dim_head = int(m.get("dim_head", 64))
        self.static_chunk_size = int(m.get("static_chunk_size", 50))
        self.num_decoding_left_chunks = int(m.get("num_decoding_left_chunks", -1))
        self.conv_pos_kernel = int(m.get("conv_pos_kernel", 31))
        self.conv_pos_groups = int(m.get("conv_pos_groups", 16))
        self._ready = False
        self._rope = {}
        self._ws = {}
        # q8 block matrices (balanced profile) run cv3_tc_gemm_q8 on the stored int8 weights;
        # False dequantises them to fp32 for the 3xTF32 GEMM instead (the same results
        # within fp32 rounding; kept for comparisons)
        self.q8_gemm = True
        # with q8_gemm: the GEMM operands as activation planes made by the producing kernels
        # (False splits fp32 rows inside each GEMM instead)
        self.q8_planes = True

    def _q8_ok(self, name) -> bool:
        t = self.w.host_tensor(self.p + name) if hasattr(self.w, "host_tensor") else None
        return (isinstance(t, QTensor) and t.kind == "q8" and t.padded_k == t.shape[1] and t.shape[1] % 64 == 0
                and t.shape[0] % 128 == 0)

    # -- weights -------------------------------------------------------------------
    def _wt(self, name):
        return self.w.weight(self.p + name)

    def _f32(self, name):
        return self.w.f32(self.p + name)

    def _dense(self, names):
        """fp32 device matrix (rows stacked) for the dense GEMMs."""
        key = (self.p + "+".join(names) + ":dense",)
        return self.w.cache(key, lambda: torch.cat([f32_of(self._wt(n)) for n in names], 0).contiguous())

    def prepare(self):
        if self._ready:
            return
        d = self.dim
        self.time1 = Lin(f32_of(self._wt("time_embed.time_mlp.0.weight")), self._f32("time_embed.time_mlp.0.bias"))
        self.time2 = Lin(f32_of(self._wt("time_embed.time_mlp.2.weight")), self._f32("time_embed.time_mlp.2.bias"))
        self.proj_in = Lin(self._dense(["input_embed.proj.weight"]), self._f32("input_embed.proj.bias"))
        self.conv = [(self._f32(f"input_embed.conv_pos_embed.{c}.0.weight"),
                      self._f32(f"input_embed.conv_pos_embed.{c}.0.bias")) for c in ("conv1", "conv2")]
        self.conv_tc = [ConvTC(w, b, groups=self.conv_pos_groups) for w, b in self.conv]
        # all AdaLN projections read silu(temb): one stacked matrix, one GEMV per step
        names = [f"transformer_blocks.{i}.attn_norm.linear.weight" for i in range(self.depth)] + \
                ["norm_out.linear.weight"]
        ada = self.w.cache((self.p + "adaln_stack",), lambda: cat_rows([self._wt(n) for n in names]))
        ada_b = self.w.cache((self.p + "adaln_stack_bias",), lambda: torch.cat(
            [self._f32(n[:-len("weight")] + "bias") for n in names]).contiguous())
        self.ada = Lin(ada, ada_b)
        self.mod_width = self.ada.n
        self.blocks = []
        for i in range(self.depth):
            b = f"transformer_blocks.{i}."
            B = _Block()
            qkv_names = [b + "attn.to_q.weight", b + "attn.to_k.weight", b + "attn.to_v.weight"]
            qkv_bias = self.w.cache((self.p + b + "qkv_bias",), lambda b=b: torch.cat(
                [self._f32(b + f"attn.to_{n}.bias") for n in "qkv"]).contiguous())
            if self.q8_gemm and all(self._q8_ok(n) for n in qkv_names + [b + "attn.to_out.0.weight",
                                                                       b + "ff.ff.0.0.weight", b + "ff.ff.2.weight"]):
                # balanced profile: the int8 weights as stored, on the tensor cores
                qkv = self.w.cache((self.p + b + "qkv:q8",), lambda: cat_rows([self._wt(n) for n in qkv_names]))
                B.qkv = LinQ8(qkv, qkv_bias)
                B.out = LinQ8(self._wt(b + "attn.to_out.0.weight"), self._f32(b + "attn.to_out.0.bias"))
                B.ff1 = LinQ8(self._wt(b + "ff.ff.0.0.weight"), self._f32(b + "ff.ff.0.0.bias"))
                B.ff2 = LinQ8(self._wt(b + "ff.ff.2.weight"), self._f32(b + "ff.ff.2.bias"))
            else:
                B.qkv = Lin(self._dense(qkv_names), qkv_bias)
                B.out = Lin(self._dense([b + "attn.to_out.0.weight"]), self._f32(b + "attn.to_out.0.bias"))
                B.ff1 = Lin(self._dense([b + "ff.ff.0.0.weight"]), self._f32(b + "ff.ff.0.0.bias"))
                B.ff2 = Lin(self._dense([b + "ff.ff.2.weight"]), self._f32(b + "ff.ff.2.bias"))
            self.blocks.append(B)
        self.proj_out = Lin(f32_of(self._wt("proj_out.weight")), self._f32("proj_out.bias"))
        # the tf32 remainders of the tensor-core weights exist before any graph capture
        for lin in [self.proj_in, self.proj_out] + [l for B in self.blocks for l in (B.qkv, B.out, B.ff1, B.ff2)]:
            if isinstance(lin, Lin):
                lin.lo()
        self.ff = self.blocks[0].ff1.n
        self._ready = True

    def rope(self, n: int):
        if n not in self._rope:
            c, s = rope_angle_tables(n, self.dim_head)
            self._rope[n] = (torch.from_numpy(c).cuda(), torch.from_numpy(s).cuda())
        return self._rope[n]

    def workspace(self, B: int, N: int) -> Workspace:
        key = (B, N)
        if key not in self._ws:
            self.prepare()
            ws = Workspace(B, N, self.dim, self.ff)
            if self.q8_planes and isinstance(self.blocks[0].qkv, LinQ8) and ws.R >= TC_MIN_ROWS:
                ws.planes()  # before any graph capture reuses the workspace
            self._ws[key] = ws
        return self._ws[key]

    # -- pieces ------------------------------------------------------------------
    def modulation(self, tfeat, mods, temb, st):
        """tfeat [rows, 256] -> mods [rows, mod_width] = adaln_stack(silu(time_mlp(tfeat)))."""
        rows = int(tfeat.shape[0])
        self.time1(tfeat.data_ptr(), rows, temb[0].data_ptr(), stream=st)
        call("cv3_unary", 0, 0.0, temb[0].data_ptr(), temb[0].numel(), temb[0].data_ptr(), st)
        self.time2(temb[0].data_ptr(), rows, temb[1].data_ptr(), stream=st)
        call("cv3_unary", 0, 0.0, temb[1].data_ptr(), temb[1].numel(), temb[1].data_ptr(), st)
        self.ada(temb[1].data_ptr(), rows, mods.data_ptr(), stream=st)

    def body(self, ws: Workspace, mods, rows_per_group: int, st, streaming: bool = False):
        """ws.cat (input rows) -> ws.out (velocity rows); mods [groups, mod_width]."""
        d, R, B, N = self.dim, ws.R, ws.B, ws.N
        mw = self.mod_width
        mp = mods.data_ptr()
        F = 4
        # input embedding + grouped causal conv position embedding (dit.py:92-112)
        self.proj_in(ws.cat.data_ptr(), R, ws.h.data_ptr(), stream=st)
        # h += mish(conv2(mish(conv1(h)))): token-major in and out, mish and the residual in
        # the conv epilogues (no transposes)
        k = self.conv_pos_kernel
        tm = (N * d, 1, d)
        c1, c2 = self.conv_tc
        c1(ws.h.data_ptr(), ws.c2.data_ptr(), B, N, N, pad_left=k - 1, xs=tm, ys=tm, act=4, stream=st)
        c2(ws.c2.data_ptr(), ws.h.data_ptr(), B, N, N, pad_left=k - 1, xs=tm, ys=tm, act=4,
           residual=ws.h.data_ptr(), stream=st)
        cos, sin = self.rope(N)
        scale = float(np.float32(1.0 / math.sqrt(self.dim_head)))
        mk, ma, mb = (2, self.static_chunk_size, self.num_decoding_left_chunks) if streaming else (0, 0, 0)
        H, hd = self.heads, self.dim_head
        for i, blk in enumerate(self.blocks):
            base = mp + i * 6 * d * F
            sh_a, sc_a, g_a, sh_f, sc_f, g_f = (base + j * d * F for j in range(6))
            if R >= TC_MIN_ROWS and isinstance(blk.qkv, LinQ8) and self.q8_planes:
                self._block_planes(ws.planes(), blk, rows_per_group, (sh_a, sc_a, g_a, sh_f, sc_f, g_f),
                                   cos, sin, scale, (mk, ma, mb), st)
                continue
            call("cv3_ln_modulate", ws.h.data_ptr(), R, d, 1e-6, sc_a, sh_a, rows_per_group, mw, ws.z.data_ptr(), st)
            blk.qkv(ws.z.data_ptr(), R, ws.qkv.data_ptr(), stream=st)
            call("cv3_partial_rope", ws.qkv.data_ptr(), R, 3 * d, d, N, hd, cos.data_ptr(), sin.data_ptr(), st)
            q = ws.qkv.data_ptr()
            call("cv3_attention", q, N * 3 * d, hd, 3 * d, q + d * F, N * 3 * d, hd, 3 * d,
                 q + 2 * d * F, N * 3 * d, hd, 3 * d, ws.a.data_ptr(), N * d, hd, d,
                 B, H, H, N, N, hd, scale, mk, ma, mb, st)
            if R >= TC_MIN_ROWS:
                # tensor-core GEMMs with the gated residual / GELU fused in the epilogue
                blk.out.tc(ws.a.data_ptr(), R, ws.h.data_ptr(), 2, g_a, rows_per_group, mw, st)
                call("cv3_ln_modulate", ws.h.data_ptr(), R, d, 1e-6, sc_f, sh_f, rows_per_group, mw,
                     ws.z.data_ptr(), st)
                blk.ff1.tc(ws.z.data_ptr(), R, ws.f1.data_ptr(), 1, stream=st)
                blk.ff2.tc(ws.f1.data_ptr(), R, ws.h.data_ptr(), 2, g_f, rows_per_group, mw, st)
                continue
            blk.out(ws.a.data_ptr(), R, ws.y.data_ptr(), stream=st)
            call("cv3_gate_residual", ws.h.data_ptr(), ws.y.data_ptr(), g_a, R, d, rows_per_group, mw, st)
            call("cv3_ln_modulate", ws.h.data_ptr(), R, d, 1e-6, sc_f, sh_f, rows_per_group, mw, ws.z.data_ptr(), st)
            blk.ff1(ws.z.data_ptr(), R, ws.f1.data_ptr(), stream=st)
            call("cv3_unary", 2, 0.0, ws.f1.data_ptr(), ws.f1.numel(), ws.f1.data_ptr(), st)
            blk.ff2(ws.f1.data_ptr(), R, ws.y.data_ptr(), stream=st)
            call("cv3_gate_residual", ws.h.data_ptr(), ws.y.data_ptr(), g_f, R, d, rows_per_group, mw, st)
        base = mp + self.depth * 6 * d * F
        call("cv3_ln_modulate", ws.h.data_ptr(), R, d, 1e-6, base, base + d * F, rows_per_group, mw,
             ws.z.data_ptr(), st)
        self.proj_out(ws.z.data_ptr(), R, ws.out.data_ptr(), stream=st)

    def _block_planes(self, ws: Workspace, blk, rows_per_group: int, mod, cos, sin, scale, mask, st):
        """One transformer block (dit.py:171-185 DiTBlock) with every GEMM reading activation
        planes: AdaLN and the attention output are split once into fp16 hi/lo planes, the
        first feed-forward linear writes GELU(x) as planes for the second."""
        d, R, N = self.dim, ws.R, ws.N
        mw = self.mod_width
        sh_a, sc_a, g_a, sh_f, sc_f, g_f = mod
        H, hd = self.heads, self.dim_head
        zp, ze, lde = ws.zp.data_ptr(), ws.ze.data_ptr(), ws.lde
        call("cv3_ln_modulate_planes", ws.h.data_ptr(), R, d, 1e-6, sc_a, sh_a, rows_per_group, mw, zp, ze, lde, st)
        blk.qkv.tc_planes(zp, ze, lde, R, ws.qkv.data_ptr(), 0, stream=st)
        call("cv3_partial_rope", ws.qkv.data_ptr(), R, 3 * d, d, N, hd, cos.data_ptr(), sin.data_ptr(), st)
        q = ws.qkv.data_ptr()
        F = 4
        call("cv3_attention", q, N * 3 * d, hd, 3 * d, q + d * F, N * 3 * d, hd, 3 * d,
             q + 2 * d * F, N * 3 * d, hd, 3 * d, ws.a.data_ptr(), N * d, hd, d,
             ws.B, H, H, N, N, hd, scale, mask[0], mask[1], mask[2], st)
        call("cv3_q8_split_rows", ws.a.data_ptr(), d, R, d, zp, ze, lde, st)
        blk.out.tc_planes(zp, ze, lde, R, ws.h.data_ptr(), 2, g_a, rows_per_group, mw, st)
        call("cv3_ln_modulate_planes", ws.h.data_ptr(), R, d, 1e-6, sc_f, sh_f, rows_per_group, mw, zp, ze, lde, st)
        fp, fe = ws.fp.data_ptr(), ws.fe.data_ptr()
        blk.ff1.tc_planes(zp, ze, lde, R, None, 4, stream=st, out_planes=fp, out_exps=fe, out_lde=lde)
        blk.ff2.tc_planes(fp, fe, lde, R, ws.h.data_ptr(), 2, g_f, rows_per_group, mw, st)

    # -- reference-compatible forward ----------------------------------------------
    def forward(self, x, mu, t, spks, cond, streaming: bool = False, seq_chunk: int = 512):
        """``x``/``mu``/``cond`` ``(B, 80, N)``, ``t`` ``(B,)``, ``spks`` ``(B, 80)`` -> ``(B, 80, N)``
        (dit.py:144-180).  Rows are general batch entries (not a CFG pair)."""
        host = D.is_host(x)
        self.prepare()
        xd, md, cd, sd = D.dev(x), D.dev(mu), D.dev(cond), D.dev(spks)
        B, mel, N = (int(s) for s in xd.shape)
        ws = self.workspace(B, N)
        st = D.stream()
        # concat rows [x, cond, mu, spk] per batch entry: the CFG kernel with the
        # "unconditioned" half dropped (every entry is a conditioned row here)
        tmp = D.empty((2 * B, N, ws.cat.shape[1]))
        call("cv3_dit_input_cat", xd.data_ptr(), cd.data_ptr(), md.data_ptr(), sd.data_ptr(), B, N, mel,
             int(sd.shape[1]), tmp.data_ptr(), st)
        ws.cat.copy_(tmp[0::2].reshape(B * N, -1))
        t_host = t.detach().cpu().numpy() if isinstance(t, torch.Tensor) else np.asarray(t)
        tfeat = torch.from_numpy(time_features(t_host.astype(np.float32))).cuda()
        temb = (D.empty((B, self.dim)), D.empty((B, self.dim)))
        mods = D.empty((B, self.mod_width))
        self.modulation(tfeat, mods, temb, st)
        self.body(ws, mods, N, st, streaming)
        out = D.empty((B, mel, N))
        call("cv3_transpose", ws.out.data_ptr(), B, N, mel, out.data_ptr(), 0, st)
        return D.out(out, host)
