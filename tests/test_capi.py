"""The C ABI library loads without a GPU and exports every entry point of include/exactb200.h."""
import os
import re

from tests.conftest import ROOT


def declared_functions():
    src = open(os.path.join(ROOT, "include", "exactb200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(exb_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    from exact_llm_b200 import _lib
    names = declared_functions()
    assert len(names) >= 20
    for n in names:
        assert hasattr(_lib.lib, n), n
        assert n in _lib.SIGNATURES, f"{n} has no ctypes signature"
    assert set(_lib.SIGNATURES) == set(names)


def test_error_path_without_gpu():
    """Argument validation happens on the host and reports through exb_last_error."""
    import ctypes
    from exact_llm_b200 import _lib
    rc = _lib.lib.exb_gemv(None, None, None, 100, 10, None, None)
    assert rc == 1 and b"K % 128" in _lib.lib.exb_last_error()
    cfg = _lib.Config(D=64, H=3, KV=2, hd=16, I=64, V=10, NL=1, max_batch=1, max_seq=8, rope_len=8)
    h = ctypes.c_void_p()
    assert _lib.lib.exb_model_create(ctypes.byref(cfg), ctypes.byref(h)) == 1
    assert b"multiple of KV" in _lib.lib.exb_last_error()
