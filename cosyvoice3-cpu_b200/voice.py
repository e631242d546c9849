"""Voice packs: what synthesis needs to know about one reference speaker.

A pack holds the prompt's speech tokens, its mel frames, the 192-d speaker
vector, the prompt's transcript, the sample rate and a display name.  The
on-disk form is the reference's ``.npz`` (``cv3cpu/voice.py:16-52``): one array
per field under the keys ``speech_token``, ``mel``, ``embedding``,
``prompt_text``, ``sample_rate`` and ``name`` (a pack saved without ``name``
takes the file's stem).  The flow stage conditions on exactly
:data:`FRAMES_PER_TOKEN` mel frames per prompt token, so a pack keeps only the
longest prefix of tokens and frames that pairs up.
"""

from __future__ import annotations

import os
from dataclasses import dataclass

import numpy as np

FRAMES_PER_TOKEN = 2          # 50 Hz speech tokens against 100 Hz mel frames (24 kHz, hop 480 / 2)
NPZ_KEYS = ("speech_token", "mel", "embedding", "prompt_text", "sample_rate", "name")


def _paired(tokens: np.ndarray, mel: np.ndarray):
    """Cut tokens and frames to the longest prefix with FRAMES_PER_TOKEN frames per token."""
    usable = min(tokens.size, mel.shape[0] // FRAMES_PER_TOKEN)
    return tokens[:usable], mel[: usable * FRAMES_PER_TOKEN]


@dataclass
class VoicePack:
    speech_token: np.ndarray      # (T,) int32 prompt speech tokens
    mel: np.ndarray               # (2T, 80) float32 prompt mel frames
    embedding: np.ndarray         # (192,) float32 speaker vector
    prompt_text: str = ""
    sample_rate: int = 24000
    name: str = ""

    def __post_init__(self):
        tokens = np.ravel(np.asarray(self.speech_token)).astype(np.int32)
        mel = np.asarray(self.mel).astype(np.float32, copy=False)
        self.speech_token, self.mel = _paired(tokens, mel)
        self.embedding = np.ravel(np.asarray(self.embedding)).astype(np.float32)

    @property
    def n_tokens(self) -> int:
        return int(self.speech_token.size)

    def to_arrays(self) -> dict:
        """The pack as the ``.npz`` arrays, one per key of :data:`NPZ_KEYS`."""
        return {"speech_token": self.speech_token, "mel": self.mel, "embedding": self.embedding,
                "prompt_text": np.array(self.prompt_text), "sample_rate": np.array(self.sample_rate),
                "name": np.array(self.name)}

    def save(self, path: str) -> None:
        np.savez_compressed(path, **self.to_arrays())

    @classmethod
    def load(cls, path: str) -> "VoicePack":
        with np.load(path, allow_pickle=False) as z:
            arrays = {key: z[key] for key in NPZ_KEYS if key in z.files}
        stem = os.path.splitext(os.path.basename(path))[0]
        return cls(speech_token=arrays["speech_token"], mel=arrays["mel"], embedding=arrays["embedding"],
                   prompt_text=str(arrays["prompt_text"]), sample_rate=int(arrays["sample_rate"]),
                   name=str(arrays["name"]) if "name" in arrays else stem)

    def __repr__(self) -> str:
        text = self.prompt_text if len(self.prompt_text) <= 40 else self.prompt_text[:40] + "..."
        return (f"VoicePack({self.name or 'unnamed'}: {self.n_tokens} prompt tokens, "
                f"{self.mel.shape[0]} mel frames, {self.sample_rate} Hz, prompt text {text!r})")
