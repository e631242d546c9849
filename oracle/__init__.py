"""CPU oracle for the cv3cpu kernel layer -- TEST INFRASTRUCTURE ONLY.

This package restates, in plain NumPy, the arithmetic of the reference
project's kernel layer (``cv3cpu/ops.py``, ``cv3cpu/quant.py``,
``cv3cpu/torch_rng.py``) and of the three model stages that drive it
(``cv3cpu/models/{qwen2,llm,dit,flow,hift}.py``).  Every function names the
reference file and line range whose behaviour it reproduces.

Who may use it: the test suite (``tests/``), ``__graft_entry__.smoke()`` and
the CPU-baseline / reference arm of ``bench.py``.  In all three it is the
*checker* (or the timed CPU baseline), never the thing under test.  The
product package calls CUDA only and fails loudly when its shared library is
missing; nothing in it imports this package.

How it is pinned: ``tests/test_oracle_pins.py`` checks it against the
reference's frozen goldens (the torch RNG samples of
``tests/reference_values.json`` and the upstream outputs of
``tests/fixtures/reference_io.npz``) and against golden vectors produced by
running the reference itself (``tests/golden/make_golden.py``).
"""

from . import numerics, stages  # noqa: F401
