"""Voice packs: the reference speaker's prompt tokens, prompt mel and speaker vector.

Same fields, normalisation and ``.npz`` format as ``cv3cpu/voice.py:16-52``:
the flow consumes exactly two mel frames per prompt speech token, so the
longer of the two is cut to match.
"""

from __future__ import annotations

import os
from dataclasses import dataclass

import numpy as np


@dataclass
class VoicePack:
    speech_token: np.ndarray      # (T,) int32
    mel: np.ndarray               # (2T, 80) float32
    embedding: np.ndarray         # (192,) float32
    prompt_text: str = ""
    sample_rate: int = 24000
    name: str = ""

    def __post_init__(self):
        self.speech_token = np.asarray(self.speech_token, dtype=np.int32).reshape(-1)
        self.mel = np.asarray(self.mel, dtype=np.float32)
        self.embedding = np.asarray(self.embedding, dtype=np.float32).reshape(-1)
        n = min(self.mel.shape[0] // 2, self.speech_token.shape[0])
        self.speech_token = self.speech_token[:n]
        self.mel = self.mel[: 2 * n]

    def save(self, path: str) -> None:
        np.savez_compressed(path, speech_token=self.speech_token, mel=self.mel.astype(np.float32),
                            embedding=self.embedding, prompt_text=np.array(self.prompt_text),
                            sample_rate=np.array(self.sample_rate), name=np.array(self.name))

    @classmethod
    def load(cls, path: str) -> "VoicePack":
        with np.load(path, allow_pickle=False) as z:
            return cls(speech_token=z["speech_token"], mel=z["mel"], embedding=z["embedding"],
                       prompt_text=str(z["prompt_text"]), sample_rate=int(z["sample_rate"]),
                       name=str(z["name"]) if "name" in z else os.path.splitext(os.path.basename(path))[0])

    def __repr__(self) -> str:
        return (f"VoicePack(name={self.name!r}, tokens={len(self.speech_token)}, "
                f"mel={self.mel.shape}, text={self.prompt_text[:40]!r})")
