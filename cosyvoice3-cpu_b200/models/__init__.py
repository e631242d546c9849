"""Device-resident CosyVoice 3 stages, mirroring ``cv3cpu/models/*.py``."""
