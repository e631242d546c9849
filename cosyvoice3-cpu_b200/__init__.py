"""cv3 on B200: the cosyvoice3-cpu (cv3cpu) kernel layer as sm_100a CUDA.

The package mirrors the reference's public surface:

* :mod:`.ops`, :mod:`.quant`, :mod:`.torch_rng` -- ``cv3cpu.ops`` /
  ``cv3cpu.quant`` / ``cv3cpu.torch_rng`` with the same function names and
  signatures, executed by the C-ABI library ``libcv3cuda.so``
  (``include/cv3cuda.h``);
* :mod:`.models` -- the Qwen2 LM, DiT flow and HiFT vocoder stages, device
  resident (weights uploaded once into HBM, activations never leave the GPU);
* :mod:`.pipeline` -- ``CosyVoice3CPU``-compatible synthesis, and
  :mod:`.weights` -- the ``.safetensors`` int8 "balanced" layout.

Import it with ``importlib.import_module("cosyvoice3-cpu_b200")`` (the
directory name is not a Python identifier).  There is no CPU fallback: the
operations raise if the library or a CUDA device is missing.
"""

__version__ = "0.1.0"

__all__ = ["CosyVoice3CPU", "CosyVoice3CUDA", "VoicePack", "SynthesisResult", "SamplingConfig"]


def __getattr__(name):
    if name in ("CosyVoice3CPU", "CosyVoice3CUDA", "SynthesisResult"):
        from . import pipeline
        return getattr(pipeline, name)
    if name == "VoicePack":
        from .voice import VoicePack
        return VoicePack
    if name == "SamplingConfig":
        from .models.llm import SamplingConfig
        return SamplingConfig
    raise AttributeError(name)
