"""End-to-end CosyVoice 3 synthesis on the GPU (mirror of ``cv3cpu/pipeline.py``).

``CosyVoice3CUDA`` (aliased ``CosyVoice3CPU`` for drop-in use) keeps the
reference's surface: ``synthesize(text, voice)``, ``synthesize_ids(...)`` with
the reference's sampling semantics, ``save``/``close``.  Weights come from a
cv3cpu ``.safetensors`` file (or an in-memory mapping with ``.meta``) and are
uploaded to HBM on first use; by default every stage stays resident (HBM is
not the constraint the reference's staged eviction works around), and
``release_stages=True`` frees a stage's device weights after it runs, like the
reference's ``MADV_DONTNEED`` release.

``synthesize_greedy_batch`` is the throughput path: a batch of utterances is
decoded together (batched greedy LM steps, one CFG solve for all utterances of
equal length, one batched vocoder pass).
"""

from __future__ import annotations

import struct
from dataclasses import dataclass, field
from typing import Callable, List, Optional, Sequence

import numpy as np

from . import _dev as D
from .models.flow import Flow
from .models.hift import HiFTGenerator
from .models.llm import CosyVoice3LM, SamplingConfig
from .weights import DeviceWeights, WeightFile

torch = D.torch

DEFAULT_SYSTEM_PROMPT = "You are a helpful assistant.<|endofprompt|>"


@dataclass
class SynthesisResult:
    audio: np.ndarray
    sample_rate: int
    speech_tokens: List[List[int]] = field(default_factory=list)
    segments: List[str] = field(default_factory=list)
    memory_report: str = ""

    @property
    def duration(self) -> float:
        return len(self.audio) / self.sample_rate


@dataclass
class Request:
    """One utterance for the batched path: text ids, prompt-text ids, voice."""
    text_ids: Sequence[int]
    prompt_ids: Sequence[int]
    voice: object


class CosyVoice3CUDA:
    """CosyVoice 3 inference with every stage on the GPU."""

    def __init__(self, weights, tokenizer_dir: Optional[str] = None, seed: Optional[int] = None,
                 release_stages: bool = False, track_memory: bool = False, seq_chunk: int = 512,
                 hift_chunk: Optional[int] = 250, tokenizer=None):
        D.require_cuda()
        self._file = WeightFile(weights) if isinstance(weights, str) else None
        host = self._file if self._file is not None else weights
        self.w = DeviceWeights(host)
        self.sample_rate = int(self.w.meta.get("sample_rate", 24000))
        self.release_stages = release_stages
        self.seq_chunk = seq_chunk
        self.hift_chunk = hift_chunk
        self.seed = seed
        self.tokenizer = tokenizer
        if tokenizer_dir and tokenizer is None:
            raise RuntimeError("the device build does not bundle the Qwen BPE tokenizer; pass an object with "
                               "an encode(str) -> ids method as tokenizer=, or use synthesize_ids")
        self._llm = self._flow = self._hift = None

    # -- lazily built stages --------------------------------------------------------
    @property
    def llm(self) -> CosyVoice3LM:
        if self._llm is None:
            self._llm = CosyVoice3LM(self.w, prefix="llm.")
        return self._llm

    @property
    def flow(self) -> Flow:
        if self._flow is None:
            self._flow = Flow(self.w, prefix="flow.")
        return self._flow

    @property
    def hift(self) -> HiFTGenerator:
        if self._hift is None:
            self._hift = HiFTGenerator(self.w, prefix="hift.")
        return self._hift

    def _drop(self, stage: str) -> None:
        if not self.release_stages:
            return
        setattr(self, f"_{stage}", None)
        self.w.evict(f"{stage}.")

    # -- text ------------------------------------------------------------------------
    def encode_text(self, s: str) -> List[int]:
        if self.tokenizer is None:
            raise RuntimeError("no tokenizer loaded; pass tokenizer= (an object with encode(str)) "
                               "or pre-tokenised ids to synthesize_ids")
        return list(self.tokenizer.encode(s))

    def synthesize(self, text: str, voice, split: bool = True, system_prompt: str = DEFAULT_SYSTEM_PROMPT,
                   sampling: Optional[SamplingConfig] = None,
                   on_progress: Optional[Callable[[str, int, int], None]] = None) -> SynthesisResult:
        """Zero-shot synthesis of ``text`` in the voice of ``voice`` (pipeline.py:100-114)."""
        splitter = getattr(self.tokenizer, "split", None)
        segments = splitter(text) if (split and splitter) else ([text] if text.strip() else [])
        if not segments:
            return SynthesisResult(np.zeros(0, np.float32), self.sample_rate)
        prompt_ids = self.encode_text(system_prompt + (voice.prompt_text or ""))
        res = self.synthesize_ids([self.encode_text(s) for s in segments], prompt_ids, voice,
                                  sampling=sampling, on_progress=on_progress)
        res.segments = segments
        return res

    def synthesize_ids(self, segment_ids: Sequence[Sequence[int]], prompt_ids: Sequence[int], voice,
                       sampling: Optional[SamplingConfig] = None,
                       on_progress: Optional[Callable[[str, int, int], None]] = None) -> SynthesisResult:
        """Sampled synthesis with the reference's semantics (pipeline.py:116-173)."""
        sampling = sampling or SamplingConfig(seed=self.seed)
        segments = list(segment_ids)
        if not segments:
            return SynthesisResult(np.zeros(0, np.float32), self.sample_rate)
        token_lists: List[List[int]] = []
        for i, ids in enumerate(segments):
            token_lists.append(list(self.llm.generate(list(ids), prompt_text_tokens=list(prompt_ids),
                                                      prompt_speech_tokens=voice.speech_token.tolist(),
                                                      sampling=sampling)))
            if on_progress:
                on_progress("llm", i + 1, len(segments))
        self._drop("llm")
        mels = []
        for i, toks in enumerate(token_lists):
            if not toks:
                mels.append(None)
                continue
            mels.append(self.flow.inference(toks, voice.speech_token, voice.mel, voice.embedding))
            if on_progress:
                on_progress("flow", i + 1, len(token_lists))
        self._drop("flow")
        waves = []
        for i, mel in enumerate(mels):
            if mel is None or mel.shape[1] == 0:
                continue
            waves.append(self.hift.inference(mel, chunk=self.hift_chunk))
            if on_progress:
                on_progress("hift", i + 1, len(mels))
        self._drop("hift")
        audio = np.concatenate(waves) if waves else np.zeros(0, np.float32)
        return SynthesisResult(audio.astype(np.float32), self.sample_rate, speech_tokens=token_lists)

    # -- batched greedy path -------------------------------------------------------------
    def prepare(self, requests: Sequence[Request]):
        """Upload a batch's inputs (ids, prompt mel, speaker vector) to the device."""
        lm = self.llm
        out = []
        for r in requests:
            v = r.voice
            out.append({
                "prompt": lm.prompt_embedding(list(r.text_ids), list(r.prompt_ids), v.speech_token.tolist()),
                "prompt_token": torch.from_numpy(np.maximum(np.asarray(v.speech_token, np.int64), 0)).cuda(),
                "prompt_mel": D.dev(v.mel),
                "embedding": D.dev(v.embedding.reshape(1, -1)),
            })
        return out

    def run_prepared(self, prepared, n_tokens: int):
        """Batched greedy synthesis of prepared requests -> device waveforms ``[U, 480 * 2 n]``."""
        lm, flow, hift = self.llm, self.flow, self.hift
        toks = lm.generate_greedy([p["prompt"] for p in prepared], n_tokens)        # [U, n] device
        plens = {int(p["prompt_token"].shape[0]) for p in prepared}
        if len(plens) != 1:
            raise ValueError("the batched path needs equal prompt lengths (one CFG solve per shape)")
        mus, spks, conds = [], [], []
        for u, p in enumerate(prepared):
            mu, spk, cond, pf = flow.conditioning_device(toks[u], p["prompt_token"], p["prompt_mel"], p["embedding"])
            mus.append(mu)
            spks.append(spk)
            conds.append(cond)
        x = flow.solve_batch(mus, spks, conds)                                        # [U, 80, N]
        mel = x[:, :, pf:].contiguous()
        return hift.inference_batch(mel, use_graph=True), toks

    def synthesize_greedy_batch(self, requests: Sequence[Request], n_tokens: int = 250, to_host: bool = True):
        """Greedy synthesis of a batch of utterances, each producing ``n_tokens`` speech tokens."""
        wav, toks = self.run_prepared(self.prepare(requests), n_tokens)
        if to_host:
            return wav.cpu().numpy(), toks.cpu().numpy()
        return wav, toks

    # -- misc ---------------------------------------------------------------------------------
    def save(self, result: SynthesisResult, path: str) -> None:
        write_wav(path, result.audio, result.sample_rate)

    def close(self) -> None:
        self._llm = self._flow = self._hift = None
        self.w.evict("")
        if self._file is not None:
            self._file.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


CosyVoice3CPU = CosyVoice3CUDA


def write_wav(path: str, audio: np.ndarray, sr: int) -> None:
    """16-bit PCM mono WAV."""
    pcm = (np.clip(np.asarray(audio, np.float32), -1.0, 1.0) * 32767.0).astype("<i2").tobytes()
    with open(path, "wb") as fh:
        fh.write(b"RIFF" + struct.pack("<I", 36 + len(pcm)) + b"WAVE")
        fh.write(b"fmt " + struct.pack("<IHHIIHH", 16, 1, 1, sr, sr * 2, 2, 16))
        fh.write(b"data" + struct.pack("<I", len(pcm)) + pcm)
