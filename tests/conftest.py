"""Shared test helpers.

Markers: ``gpu`` -- needs a CUDA device (run with ``-m gpu``); everything else
runs on the CPU.  The package directory ``cosyvoice3-cpu_b200`` is imported
through :func:`pkg` (its name is not a Python identifier).
"""

import importlib
import json
import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(REPO, "tests", "golden")
# The reference checkout: $CV3_REFERENCE, else a checkout named "reference" beside
# this repository.  Tests that need it skip when neither exists (the GPU box).
REFERENCE = os.environ.get("CV3_REFERENCE") or os.path.join(os.path.dirname(REPO), "reference")

if REPO not in sys.path:
    sys.path.insert(0, REPO)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")


def pkg(name: str = ""):
    base = "cosyvoice3-cpu_b200"
    return importlib.import_module(base + ("." + name if name else ""))


def rel_err(got, ref) -> float:
    """max |got - ref| / max |ref| (the reference suite's metric, tests/conftest.py:13-16)."""
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    return float(np.abs(got - ref).max() / max(float(np.abs(ref).max()), 1e-9))


def have_reference() -> bool:
    return os.path.isdir(os.path.join(REFERENCE, "cv3cpu"))


@pytest.fixture(scope="session")
def golden():
    with np.load(os.path.join(GOLDEN, "stages_small.npz")) as z:
        return {k: z[k] for k in z.files}


@pytest.fixture(scope="session")
def rng_golden():
    with open(os.path.join(GOLDEN, "torch_rng.json")) as fh:
        return json.load(fh)


@pytest.fixture(scope="session")
def small_weights():
    """The small synthetic model in both profiles (host tensors)."""
    synth = pkg("synth")
    return {p: synth.synthetic_weights(p, small=True) for p in ("balanced", "f32")}
