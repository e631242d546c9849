"""CausalMaskedDiffWithDiT on the GPU (mirror of ``cv3cpu/models/flow.py``).

``Flow.inference`` keeps the reference's contract (speech tokens + prompt mel
+ speaker vector -> generated mel ``(80, T)``).  :meth:`Flow.solve_batch`
solves several utterances of the same length together: the CFG batch holds
``2 * U`` rows (each utterance conditioned and unconditioned), the ten Euler
steps -- time MLP and AdaLN projection, 22 DiT blocks, the guidance combine and
the update -- are captured once into one CUDA graph per shape and replayed.

The ODE start is the reference's fixed ``torch.randn((1, 80, 15000))`` draw
after ``manual_seed(0)``, generated on the device bit-exactly
(``cv3_torch_randn``) once per process; an utterance of N frames starts from
its first N columns (per-row prefix, as the reference slices it).
"""

from __future__ import annotations

import numpy as np

from .. import _dev as D
from .. import ops
from .._lib import call
from ._common import Graph
from .dit import DiT, time_features

torch = D.torch

NOISE_SHAPE = (1, 80, 50 * 300)
NOISE_SEED = 0


class Flow:
    def __init__(self, weights, prefix: str = "flow."):
        self.w = weights
        self.p = prefix
        m = weights.meta.get("flow", {})
        self.token_mel_ratio = int(m.get("token_mel_ratio", 2))
        self.pre_lookahead_len = int(m.get("pre_lookahead_len", 3))
        self.output_size = int(m.get("output_size", 80))
        self.inference_cfg_rate = float(m.get("inference_cfg_rate", 0.7))
        self.n_timesteps = int(m.get("n_timesteps", 10))
        self.estimator = DiT(weights, prefix + "decoder.estimator.")
        self._noise = None
        self._graphs = {}

    def _t(self, name):
        return self.w.weight(self.p + name)

    def _f32(self, name):
        return self.w.f32(self.p + name)

    # -- fixed ODE start (flow.py:36-43) -------------------------------------------
    def noise(self):
        if self._noise is None:
            n = int(np.prod(NOISE_SHAPE))
            buf = D.empty((n,))
            scratch = D.empty((32,))
            call("cv3_torch_randn", NOISE_SEED, 0, n, buf.data_ptr(), scratch.data_ptr(), D.stream())
            self._noise = buf.reshape(NOISE_SHAPE[1:])
        return self._noise

    def rand_noise(self, n: int):
        if n > NOISE_SHAPE[2]:
            raise ValueError(f"utterance needs {n} mel frames but the fixed CFM noise only has "
                             f"{NOISE_SHAPE[2]}; split the text into shorter segments")
        return self.noise()[:, :n].unsqueeze(0)

    # -- conditioning (flow.py:46-56, :96-125) -----------------------------------------
    def pre_lookahead(self, tokens_emb):
        """``(T, 80)`` device rows -> ``(T, 80)``."""
        x = tokens_emb.t().contiguous()
        h = ops.conv1d(x, self._t("pre_lookahead_layer.conv1.weight"), self._f32("pre_lookahead_layer.conv1.bias"),
                       pad=(0, self.pre_lookahead_len))
        h = ops.leaky_relu(h, 0.01)
        k2 = int(self.w.entry(self.p + "pre_lookahead_layer.conv2.weight")["shape"][-1])
        h = ops.conv1d(h, self._t("pre_lookahead_layer.conv2.weight"), self._f32("pre_lookahead_layer.conv2.bias"),
                       pad=(k2 - 1, 0))
        out = tokens_emb.clone()
        # out = h^T + tokens_emb (flow.py:56): the transpose kernel accumulates
        call("cv3_transpose", h.data_ptr(), 1, int(h.shape[0]), int(h.shape[1]), out.data_ptr(), 1, D.stream())
        return out

    def conditioning(self, token, prompt_token, prompt_feat, embedding):
        """Device ``(mu (80, N), spk (80,), cond (80, N), prompt_frames)`` for one utterance
        from host inputs (ids range-checked here, IndexError as the reference)."""
        ids = np.maximum(np.concatenate([np.asarray(prompt_token, np.int64), np.asarray(token, np.int64)]), 0)
        rows = int(self.w.entry(self.p + "input_embedding")["shape"][0])
        if ids.size and int(ids.max()) >= rows:
            raise IndexError(f"token id {int(ids.max())} is outside the {rows}-row embedding table")
        prompt_feat = np.asarray(prompt_feat, np.float32)
        n_prompt = len(np.asarray(prompt_token))
        dev_ids = torch.from_numpy(ids).cuda()
        return self.conditioning_device(dev_ids[n_prompt:], dev_ids[:n_prompt], D.dev(prompt_feat),
                                        D.dev(np.asarray(embedding, np.float32).reshape(1, -1)))

    def conditioning_device(self, token, prompt_token, prompt_feat, embedding):
        """Same as :meth:`conditioning` from device tensors (no host round trip):
        ``token``/``prompt_token`` int64 ids (non-negative, inside the table),
        ``prompt_feat`` ``(P, 80)``, ``embedding`` ``(1, 192)``."""
        nrm = torch.empty_like(embedding)
        call("cv3_l2_normalize", embedding.data_ptr(), 1, int(embedding.shape[1]), nrm.data_ptr(), D.stream())
        spk = ops.linear(nrm, self._t("spk_embed_affine_layer.weight"), self._f32("spk_embed_affine_layer.bias"))
        ids = torch.cat([prompt_token.reshape(-1), token.reshape(-1)])
        e = ops.embedding(self._t("input_embedding"), ids)
        h = self.pre_lookahead(e)                                                # (T, 80)
        mu = ops.interpolate_nearest(h.t().contiguous(), self.token_mel_ratio)   # (80, 2T)
        p, total = int(prompt_feat.shape[0]), int(mu.shape[1])
        if p > total:
            raise ValueError("prompt mel is longer than the token grid")
        cond = D.zeros((self.output_size, total))
        if p:
            cond[:, :p].copy_(prompt_feat.t())
        return mu, spk.reshape(-1), cond, p

    # -- the solve ---------------------------------------------------------------------
    def schedule(self):
        ts = 1.0 - np.cos(np.linspace(0.0, 1.0, self.n_timesteps + 1, dtype=np.float64) * 0.5 * np.pi)
        return ts.astype(np.float32)

    def _solver(self, U: int, N: int):
        key = (U, N)
        if key in self._graphs:
            return self._graphs[key]
        dit = self.estimator
        dit.prepare()
        dit.rope(N)                      # constant tables exist before any graph capture
        ws = dit.workspace(2 * U, N)
        ts = self.schedule()
        steps = len(ts) - 1
        # t and dt exactly as the reference accumulates them in float32
        # (flow.py:79-90): t_s = t_{s-1} + dt_{s-1}, dt_s = ts[s+1] - t_s
        t_used, dts = [], []
        t, dt = ts[0], ts[1] - ts[0]
        for s in range(1, len(ts)):
            t_used.append(t)
            dts.append(np.float32(dt))
            t = t + dt
            if s < len(ts) - 1:
                dt = ts[s + 1] - t
        state = {
            "x": D.empty((U, 80, N)), "mu": D.empty((U, 80, N)), "cond": D.empty((U, 80, N)),
            "spk": D.empty((U, 80)),
            "tfeat": torch.from_numpy(time_features(np.array(t_used, np.float32))).cuda(),   # one row per step
            "temb": (D.empty((1, dit.dim)), D.empty((1, dit.dim))),
            "mods": D.empty((1, dit.mod_width)),
            "ws": ws, "graph": None,
        }
        state["dts"] = dts
        state["steps"] = steps
        self._graphs[key] = state
        return state

    def _launch_solve(self, S, U: int, N: int, st, streaming: bool = False):
        dit, ws = self.estimator, S["ws"]
        for s in range(S["steps"]):
            call("cv3_dit_input_cat", S["x"].data_ptr(), S["cond"].data_ptr(), S["mu"].data_ptr(),
                 S["spk"].data_ptr(), U, N, 80, 80, ws.cat.data_ptr(), st)
            dit.modulation(S["tfeat"][s:s + 1], S["mods"], S["temb"], st)
            dit.body(ws, S["mods"], 0, st, streaming)
            call("cv3_cfg_euler", S["x"].data_ptr(), ws.out.data_ptr(), U, 80, N, self.inference_cfg_rate,
                 float(S["dts"][s]), st)

    def solve_batch(self, mus, spks, conds, use_graph: bool = True, streaming: bool = False):
        """Euler/CFG solve of U same-length utterances; returns device ``x`` ``(U, 80, N)``."""
        U = len(mus)
        N = int(mus[0].shape[-1])
        if any(int(m.shape[-1]) != N for m in mus):
            raise ValueError("solve_batch needs utterances of equal length")
        S = self._solver(U, N)
        S["x"].copy_(self.rand_noise(N).expand(U, 80, N))
        for u in range(U):
            S["mu"][u].copy_(D.dev(mus[u]).reshape(80, N))
            S["cond"][u].copy_(D.dev(conds[u]).reshape(80, N))
            S["spk"][u].copy_(D.dev(spks[u]).reshape(80))
        if use_graph and not streaming:
            if S["graph"] is None:
                g = Graph()
                # capture records without executing; x was seeded above and is replayed next
                g.capture(lambda st: self._launch_solve(S, U, N, st))
                S["graph"] = g
            S["graph"].replay()
        else:
            self._launch_solve(S, U, N, D.stream(), streaming)
        return S["x"]

    def solve_euler(self, mu, spks, cond, streaming: bool = False, temperature: float = 1.0,
                    seq_chunk: int = 512, progress=None):
        """Reference-compatible single-utterance solve: ``mu``/``cond`` ``(1, 80, N)``, ``spks`` ``(1, 80)``."""
        if temperature != 1.0:
            raise ValueError("the device solve is built for temperature 1.0 (the pipeline's value)")
        host = D.is_host(mu)
        x = self.solve_batch([D.dev(mu)[0]], [D.dev(spks)[0]], [D.dev(cond)[0]], streaming=streaming)
        return D.out(x.clone(), host)

    def inference(self, token, prompt_token, prompt_feat, embedding, streaming: bool = False,
                  seq_chunk: int = 512, progress=None):
        """Generated mel ``(80, T_mel)`` with the prompt frames stripped (flow.py:96-128)."""
        mu, spk, cond, p = self.conditioning(token, prompt_token, prompt_feat, embedding)
        x = self.solve_batch([mu], [spk], [cond], streaming=streaming)
        return x[0, :, p:].cpu().numpy()
