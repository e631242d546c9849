"""CosyVoice3LM on the GPU (mirror of ``cv3cpu/models/llm.py``).

``generate`` keeps the reference's streaming, sampling contract: the forward
pass, head and log-softmax run on the device; the nucleus / repetition-aware
sampler stays on the host with NumPy's PCG64 generator, exactly as the
reference's (llm.py:37-49, :125-149), so sampled tokens match it for a seed.

``generate_greedy`` is the benchmark path: batched greedy decoding (argmax of
the same log-probabilities over the speech tokens, stop ids masked, lowest id
on ties) where a whole step is one CUDA graph replay (:class:`DecodeEngine`).
"""

from __future__ import annotations

from typing import Iterator, List, Optional, Sequence

import numpy as np

from .. import _dev as D
from .. import ops
from .qwen2 import DecodeEngine, Qwen2Config, Qwen2Model

torch = D.torch

SPEECH_TOKEN_SIZE = 6561
SAMPLER_MAX_TOP_K = 32  # cv3_sample_select's largest top_k (larger ones use the host sampler)
MAX_DECODE_BATCH = 32   # sequences one decode engine advances together (the decode GEMV's row limit)
ENDOFPROMPT_ID = 151646


class SamplingConfig:
    """Sampling knobs of cv3cpu/models/llm.py:19-34 (host-side sampler)."""

    def __init__(self, top_p: float = 0.8, top_k: int = 25, win_size: int = 10, tau_r: float = 0.1,
                 seed: Optional[int] = None, max_token_text_ratio: float = 20.0,
                 min_token_text_ratio: float = 2.0, strict_min_len: bool = False):
        self.top_p, self.top_k, self.win_size, self.tau_r = top_p, top_k, win_size, tau_r
        self.max_token_text_ratio = max_token_text_ratio
        self.min_token_text_ratio = min_token_text_ratio
        self.strict_min_len = strict_min_len
        self.rng = np.random.default_rng(seed)


def nucleus_sampling(probs_sorted, idx_sorted, rng, top_p: float, top_k: int) -> int:
    """Take entries until the cumulative probability reaches top_p, at most top_k (llm.py:37-49)."""
    cum, n = 0.0, 0
    for i in range(min(top_k, idx_sorted.shape[0])):
        if cum >= top_p:
            break
        cum += float(probs_sorted[i])
        n += 1
    p = probs_sorted[:n].astype(np.float64)
    p = p / p.sum()
    return int(idx_sorted[rng.choice(n, p=p)])


def _softmax_host(x):
    e = np.exp(x - np.max(x))
    return e / np.sum(e)


class CosyVoice3LM:
    def __init__(self, weights, prefix: str = "llm."):
        self.w = weights
        self.prefix = prefix
        self.cfg = Qwen2Config.from_meta(weights.meta)
        self.body = Qwen2Model(weights, self.cfg, prefix=prefix + "model.")
        self.speech_token_size = int(weights.meta.get("speech_token_size", SPEECH_TOKEN_SIZE))
        self.sos = self.speech_token_size
        self.eos_token = self.speech_token_size + 1
        self.task_id = self.speech_token_size + 2
        self.fill_token = self.speech_token_size + 3
        self.stop_token_ids = set(range(self.speech_token_size, self.speech_token_size + 200))
        self.endofprompt_id = int(weights.meta.get("endofprompt_id", ENDOFPROMPT_ID))
        self._engines = {}
        self._sampling_engines = {}

    # -- pieces (llm.py:68-78) -------------------------------------------------
    def _speech_emb(self, ids):
        return ops.embedding(self.w.weight(self.prefix + "speech_embedding"), ids)

    def _text_emb(self, ids):
        return self.body.embed(ids)

    def _head(self, h):
        name = self.prefix + "llm_decoder.bias"
        bias = self.w.f32(name) if name in self.w else None
        return ops.linear(h, self.w.weight(self.prefix + "llm_decoder.weight"), bias)

    def prompt_embedding(self, text_tokens, prompt_text_tokens=(), prompt_speech_tokens=()):
        """``[sos, text, task, prompt speech]`` rows on the device (llm.py:91-104)."""
        text = list(prompt_text_tokens) + list(text_tokens)
        if self.endofprompt_id not in text:
            raise ValueError(
                f"CosyVoice 3 expects '<|endofprompt|>' (id {self.endofprompt_id}) somewhere in the "
                f"prompt text; prepend e.g. 'You are a helpful assistant.<|endofprompt|>'")
        # host ids: range-checked (IndexError) before the device gather
        parts = [self._speech_emb(np.array([self.sos])), self._text_emb(np.asarray(text)),
                 self._speech_emb(np.array([self.task_id]))]
        if len(prompt_speech_tokens):
            parts.append(self._speech_emb(np.asarray(list(prompt_speech_tokens))))
        return torch.cat([D.dev(p) for p in parts], 0)

    # -- sampling generation (llm.py:80-123) --------------------------------------
    def generate(self, text_tokens: Sequence[int], prompt_text_tokens: Sequence[int] = (),
                 prompt_speech_tokens: Sequence[int] = (), sampling: Optional[SamplingConfig] = None,
                 strict_min_len: Optional[bool] = None, progress=None,
                 device_sampler: bool = True) -> Iterator[int]:
        """Speech tokens for ``text_tokens`` with the reference's sampling (llm.py:80-123).

        ``device_sampler`` (top_k <= 32): the decode steps replay a CUDA graph and the token
        choice runs on the device (cv3_sample_select); the tokens are produced before the
        first is yielded.  Otherwise each step is a device forward followed by the host
        sampler.  Both draw the same random stream from ``sampling.rng``."""
        sampling = sampling or SamplingConfig()
        if strict_min_len is None:
            strict_min_len = sampling.strict_min_len
        x = self.prompt_embedding(text_tokens, prompt_text_tokens, prompt_speech_tokens)
        n_new = len(text_tokens)
        min_len = int(n_new * sampling.min_token_text_ratio)
        max_len = int(n_new * sampling.max_token_text_ratio)
        if max_len <= 0:
            return
        if device_sampler and 1 <= int(sampling.top_k) <= SAMPLER_MAX_TOP_K and sampling.top_p > 0:
            # graph-replayed decode steps with the device sampler: the same tokens and the
            # same random stream as the host sampler (the state is handed back to sampling.rng)
            toks = self.generate_sampled([x], sampling, [min_len], [max_len], strict_min_len)[0]
            for i, t in enumerate(toks):
                yield t
                if progress is not None:
                    progress(i, t)
            return
        cache = self.body.new_cache(1, int(x.shape[0]) + max_len + 1)
        out: List[int] = []
        for i in range(max_len):
            h = self.body.forward(x, cache)
            logp = ops.log_softmax(self._head(h[-1:]))[0].cpu().numpy()
            top = self._sample(logp, out, sampling, i < min_len, strict_min_len)
            if top in self.stop_token_ids:
                break
            yield top
            out.append(top)
            x = D.dev(self._speech_emb(np.array([top])))
            if progress is not None:
                progress(i, top)

    def _sample(self, logp, decoded, cfg: SamplingConfig, ignore_eos: bool, strict_min_len: bool) -> int:
        """Host sampler of llm.py:125-149 (PCG64 draws must match the reference's)."""
        scores = logp.copy()
        if ignore_eos:
            if strict_min_len:
                for t in self.stop_token_ids:
                    scores[t] = -np.inf
            else:
                scores[self.speech_token_size] = -np.inf
        probs = _softmax_host(scores)
        order = np.argsort(-probs, kind="stable")
        top = nucleus_sampling(probs[order], order, cfg.rng, cfg.top_p, cfg.top_k)
        window = decoded[-cfg.win_size:]
        if sum(1 for t in window if t == top) >= cfg.win_size * cfg.tau_r:
            scores[top] = -np.inf
            p = _softmax_host(scores).astype(np.float64)
            p /= p.sum()
            top = int(cfg.rng.choice(p.shape[0], p=p))
        return top

    def sampling_engine(self, batch: int, cap: int, max_steps: int, cfg: SamplingConfig,
                        strict: bool) -> DecodeEngine:
        key = (batch, cap, max_steps, float(cfg.top_p), int(cfg.top_k), int(cfg.win_size), float(cfg.tau_r),
               bool(strict))
        if key not in self._sampling_engines:
            eng = DecodeEngine(self.body, self.w.weight(self.prefix + "llm_decoder.weight"),
                               self.w.weight(self.prefix + "speech_embedding"), self.speech_token_size, batch, cap,
                               max_steps)
            eng.enable_sampling(cfg.top_p, cfg.top_k, cfg.win_size, cfg.tau_r, strict)
            self._sampling_engines[key] = eng
        return self._sampling_engines[key]

    def generate_sampled(self, prompts, sampling: SamplingConfig, min_lens, max_lens, strict_min_len: bool):
        """Sampled decode of every prompt embedding ``(T_b, H)`` with the device sampler.

        Sequence b draws from its own copy of ``sampling.rng``'s stream in turn: b = 0 starts
        from the generator's state, b + 1 from where b ended, as consecutive host calls of
        ``generate`` would; the generator is left where the last one ended.  Returns the
        token lists (stop ids excluded)."""
        st = sampling.rng.bit_generator.state
        if st.get("bit_generator") != "PCG64":
            raise ValueError("the device sampler replays numpy's PCG64 stream")
        B = len(prompts)
        need = max(int(np.shape(p)[0]) for p in prompts) + max(max_lens) + 1
        cap = max(256, -(-need // 256) * 256)
        steps = max(256, -(-max(max_lens) // 256) * 256)
        out = []
        state = (st["state"]["state"], st["state"]["inc"])
        for b in range(B):   # sequential draws share one stream: one sequence per run
            eng = self.sampling_engine(1, cap, steps, sampling, strict_min_len)
            toks, states = eng.run_sampled([prompts[b]], [state], [min_lens[b]], [max_lens[b]])
            out.append(toks[0])
            state = states[0]
        sampling.rng.bit_generator.state = {"bit_generator": "PCG64",
                                             "state": {"state": state[0], "inc": state[1]},
                                             "has_uint32": st["has_uint32"], "uinteger": st["uinteger"]}
        return out

    # -- batched greedy decode ------------------------------------------------
    def engine(self, batch: int, cap: int, max_steps: int) -> DecodeEngine:
        key = (batch, cap, max_steps)
        if key not in self._engines:
            self._engines[key] = DecodeEngine(
                self.body, self.w.weight(self.prefix + "llm_decoder.weight"),
                self.w.weight(self.prefix + "speech_embedding"), self.speech_token_size, batch, cap, max_steps)
        return self._engines[key]

    def generate_greedy(self, prompts, n_tokens: int, cap: Optional[int] = None, use_graph: bool = True,
                        keep_logp: bool = False, persistent: bool = False):
        """Greedy-decode ``n_tokens`` speech tokens for each prompt embedding ``(T_b, H)``.

        Returns the ``[B, n_tokens]`` device tensor of token ids.  The decode steps run as one
        CUDA graph per step (``use_graph``), eager launches, or one persistent cooperative
        launch (``persistent``, where the model allows it).  More than ``MAX_DECODE_BATCH``
        sequences run as consecutive groups of at most that many (each sequence's tokens do
        not depend on the others in its batch).
        """
        B = len(prompts)
        if B > MAX_DECODE_BATCH:
            groups = [prompts[i:i + MAX_DECODE_BATCH] for i in range(0, B, MAX_DECODE_BATCH)]
            need = max(int(np.shape(p)[0]) for p in prompts) + n_tokens
            cap = cap or max(256, -(-need // 256) * 256)
            return torch.cat([self.generate_greedy(g, n_tokens, cap, use_graph, keep_logp, persistent)
                              for g in groups], 0)
        need = max(int(np.shape(p)[0]) for p in prompts) + n_tokens
        cap = cap or max(256, -(-need // 256) * 256)
        eng = self.engine(B, cap, max(n_tokens, 1))
        self.last_engine = eng
        eng.keep_logp = keep_logp
        if keep_logp and eng.graph is not None:
            eng.graph = None
        return eng.run(prompts, n_tokens, use_graph=use_graph and not keep_logp, persistent=persistent)
