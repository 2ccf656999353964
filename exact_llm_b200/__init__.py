"""exact_llm_b200 -- B200-native (sm_100a) engine for exact-llm's exact integer forward pass.

Python is the host: it loads ``libexactb200.so`` through ctypes (``_lib``) and mirrors the
reference's model/engine API (``model.ExactModel``) and its operator API (``import
exact_llm_b200.ops`` registers ``torch.ops.exact.gemv``).  All arithmetic runs in the CUDA library;
there is no CPU fallback.
"""
from . import configs, tables  # noqa: F401
from ._lib import ExbError, lib  # noqa: F401
from .model import Cache, ExactModel  # noqa: F401

__all__ = ["ExactModel", "Cache", "ExbError", "configs", "tables", "lib"]
