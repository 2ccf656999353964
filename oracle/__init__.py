"""CPU oracle for the exact integer forward pass (TEST INFRASTRUCTURE ONLY).

This package restates, in numpy, the integer program of the reference project
novain-shibu/exact-llm (``exact_llm.py`` and the group-128 / MoE / Freivalds code in
``experiments/``).  It exists to check the CUDA engine: only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` leg of ``bench.py`` may import it.
The product path (``exact_llm_b200``) never imports, links or executes anything here.

Parity of this restatement is pinned against fixtures produced by the reference's own
code (``tests/golden/make_golden.py`` imports the reference and records its outputs).
"""
from .exact_oracle import *  # noqa: F401,F403
from . import synth  # noqa: F401
