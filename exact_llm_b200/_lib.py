"""ctypes binding of libexactb200.so (the C ABI declared in include/exactb200.h).

The library is built in-tree (``exact_llm_b200/build.py``).  There is no CPU fallback: if the
shared library is missing or fails to load, importing this module raises.
"""
import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
# EXB_LIB selects another build of the same library (e.g. one compiled with different tuning macros)
LIB_PATH = os.environ.get("EXB_LIB") or os.path.join(HERE, "libexactb200.so")

c_i32p = ctypes.POINTER(ctypes.c_int32)
c_i64p = ctypes.POINTER(ctypes.c_int64)


class Config(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in ("D", "H", "KV", "hd", "I", "V", "NL", "tie", "lin_kind", "n_experts",
                                            "topk", "moe_I", "shared_I", "max_batch", "max_seq", "rope_len",
                                            "emb_shift")]


# name -> (restype, argtypes); must list every entry point of include/exactb200.h
SIGNATURES = {
    "exb_last_error": (ctypes.c_char_p, []),
    "exb_version": (ctypes.c_int, []),
    "exb_gemv": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                                ctypes.c_void_p, ctypes.c_void_p]),
    "exb_linear_g128_scratch_bytes": (ctypes.c_size_t, [ctypes.c_int, ctypes.c_int, ctypes.c_int]),
    "exb_linear_g128": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
                                       ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
                                       ctypes.c_void_p, ctypes.c_void_p]),
    "exb_linear_g128_noalloc": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                                               ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p,
                                               ctypes.c_void_p, ctypes.c_void_p]),
    "exb_linear_channel": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                                          ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p,
                                          ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]),
    "exb_model_create": (ctypes.c_int, [ctypes.POINTER(Config), ctypes.POINTER(ctypes.c_void_p)]),
    "exb_model_destroy": (None, [ctypes.c_void_p]),
    "exb_model_set_tables": (ctypes.c_int, [ctypes.c_void_p, c_i64p, c_i64p, c_i64p, c_i64p, c_i64p]),
    "exb_model_set_tensor": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_void_p, ctypes.c_size_t]),
    "exb_model_generate": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_uint64]),
    "exb_model_finalize": (ctypes.c_int, [ctypes.c_void_p]),
    "exb_seq_reset": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int]),
    "exb_seq_len": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int]),
    "exb_forward": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, c_i32p, c_i32p, c_i64p, c_i32p]),
    "exb_generate": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, c_i32p, ctypes.c_int, c_i32p, c_i64p]),
    "exb_generate_device": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int,
                                           ctypes.c_void_p]),
    "exb_kv_export": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                                     ctypes.c_void_p, ctypes.c_void_p]),
    "exb_trace_enable": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int]),
    "exb_trace_row_len": (ctypes.c_int64, [ctypes.c_void_p]),
    "exb_trace_read": (ctypes.c_int, [ctypes.c_void_p, c_i64p, ctypes.c_int64]),
    "exb_commit_begin": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int]),
    "exb_commit_root": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
                                       ctypes.c_int64]),
    "exb_commit_end": (ctypes.c_int, [ctypes.c_void_p]),
    "exb_sample": (ctypes.c_int, [ctypes.c_void_p, c_i64p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                                  ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p]),
    "exb_sampling": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
                                    ctypes.c_int64]),
    "exb_sampling_positions": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]),
    "exb_verifier_emb_keys": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p]),
    "exb_step_launches": (ctypes.c_int, [ctypes.c_void_p]),
    "exb_verify_cells": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p,
                                        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p,
                                        ctypes.c_int64, ctypes.c_void_p]),
    "exb_freivalds_set_keys": (ctypes.c_int, [ctypes.c_void_p, c_i32p, ctypes.c_int64]),
    "exb_freivalds_read_keys": (ctypes.c_int, [ctypes.c_void_p, c_i32p, ctypes.c_int64]),
    "exb_freivalds_enable": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int]),
    "exb_freivalds_status": (ctypes.c_int, [ctypes.c_void_p, c_i64p, c_i64p]),
    "exb_set_option": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_int64]),
    "exb_moe_selections": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, c_i32p, ctypes.c_int64]),
    "exb_tp_plan": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, c_i32p]),
    "exb_tp_unique_id": (ctypes.c_int, [ctypes.c_char_p]),
    "exb_model_create_tp": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_char_p,
                                           ctypes.POINTER(ctypes.c_void_p)]),
    "exb_device_errors": (ctypes.c_int, [ctypes.c_void_p, c_i32p]),
    "exb_bench_linear": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                        ctypes.POINTER(ctypes.c_float), ctypes.POINTER(ctypes.c_double)]),
    "exb_profile_step": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.POINTER(ctypes.c_float), ctypes.c_int,
                                        ctypes.POINTER(ctypes.c_int)]),
    "exb_model_stream": (ctypes.c_void_p, [ctypes.c_void_p]),
    "exb_model_weight_bytes": (ctypes.c_size_t, [ctypes.c_void_p]),
    "exb_gen_tensor": (ctypes.c_int, [ctypes.c_int, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_int64,
                                      ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p]),
}


class ExbError(RuntimeError):
    pass


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing: build it with `python exact_llm_b200/build.py` "
                          "(there is no CPU fallback)")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


def check(rc):
    if rc != 0:
        raise ExbError(f"exb error {rc}: {lib.exb_last_error().decode(errors='replace')}")
    return rc


def ptr(a, ctype=None):
    """data pointer of a numpy array (contiguous) or a torch tensor as ctypes."""
    if a is None:
        return None
    if hasattr(a, "data_ptr"):
        p = a.data_ptr()
        return ctypes.cast(p, ctypes.POINTER(ctype)) if ctype else ctypes.c_void_p(p)
    if ctype is not None:
        return a.ctypes.data_as(ctypes.POINTER(ctype))
    return ctypes.c_void_p(a.ctypes.data)
