"""Exact model release artifact: float64 conversion, writer and verifying loader.

The reference specifies the release as four files -- ``weights.int8``, ``scales.int``,
``tables.int`` and ``manifest.json`` with the architecture, the Q16 format, the table ids, the spec
version and the SHA-256 of every file (SPEC.md:7-12) -- and converts float checkpoints with float64
arithmetic (exact_llm.py:83-88, 133-139 per channel; experiments/group128_quality_kaggle.py:406-414
per 128-row group).  This module gives that format a concrete layout:

* ``weights.int8``  every int8 matrix, (N, K) row-major (one K-byte row per output), 64-byte aligned
* ``scales.int``    every integer tensor as little-endian int64: scales, biases, norm gains, the Q16
                    embedding rows
* ``tables.int``    the shipped integer tables as little-endian int64: exp (Q24), SiLU and sigmoid
                    (Q16), RoPE cos and sin (Q16, rope_len x hd/2)
* ``manifest.json`` {"spec", "format", "arch", "tables", "tensors", "files"}: per tensor its file,
                    byte offset, shape and dtype; per file its size and SHA-256

``load_artifact`` refuses a release whose file sizes or SHA-256 digests differ from the manifest,
and the engine then runs on the shipped tables, never on recomputed ones.
"""
import hashlib
import json
import os

import numpy as np

from . import tables

SPEC = "exact-model-release 0.4"
FILES = ("weights.int8", "scales.int", "tables.int")
LIN_NAMES = ("q", "k", "v", "o", "gate", "up", "down")
ONE = 1 << 16
GROUP = 128


# ----------------------------------------------------------------------------- float64 conversion
def quantize_channel(w_out_in, bias=None, chunk=16384):
    """Per-output-channel int8 linear from an (out, in) float matrix: scale = max|w| / 127 per
    output (1e-12 where the column is zero), w = clip(rint(w / scale), -127, 127),
    M = rint(scale * 2^28), bias = rint(b * 2^16).  Row blocks of ``chunk`` outputs as the
    reference's ``qlin_chunked`` (exact_llm.py:83-88, 133-139; per-output scales make the blocks
    independent).  Returns w (N, K) int8, M (N,) int64, b (N,) int64 or None."""
    w_out_in = np.asarray(w_out_in)
    ws, Ms = [], []
    for j in range(0, w_out_in.shape[0], chunk):
        w = np.asarray(w_out_in[j:j + chunk], dtype=np.float64).T          # (in, out)
        sc = np.abs(w).max(0)
        sc = np.where(sc == 0, 1e-12, sc) / 127.0
        ws.append(np.clip(np.rint(w / sc), -127, 127).astype(np.int8).T)
        Ms.append(np.rint(sc * (1 << 28)).astype(np.int64))
    b = None if bias is None else np.rint(np.asarray(bias, dtype=np.float64) * ONE).astype(np.int64)
    return np.ascontiguousarray(np.concatenate(ws, 0)), np.concatenate(Ms), b


def quantize_group(w_out_in, bias=None):
    """Group-128 int8 linear from an (out, in) float matrix: per 128 input rows and output column,
    scale = max|w| / 127 (1e-12 where zero), w = clip(rint(w / scale), -127, 127),
    M = rint(scale * 2^28) (experiments/group128_quality_kaggle.py:406-414).  Returns w (N, K) int8,
    M (N, K/128) int64, b (N,) int64 or None."""
    w = np.asarray(w_out_in, dtype=np.float64).T                             # (K, N)
    K, N = w.shape
    if K % GROUP:
        raise ValueError(f"group-128 conversion needs K % 128 == 0 (K = {K})")
    wq = np.empty((K, N), np.int8)
    M = np.empty((K // GROUP, N), np.int64)
    for gi, a in enumerate(range(0, K, GROUP)):
        sc = np.abs(w[a:a + GROUP]).max(0)
        sc = np.where(sc == 0, 1e-12, sc) / 127.0
        wq[a:a + GROUP] = np.clip(np.rint(w[a:a + GROUP] / sc), -127, 127).astype(np.int8)
        M[gi] = np.rint(sc * (1 << 28)).astype(np.int64)
    b = None if bias is None else np.rint(np.asarray(bias, dtype=np.float64) * ONE).astype(np.int64)
    return np.ascontiguousarray(wq.T), np.ascontiguousarray(M.T), b


def convert_checkpoint(get, c, lin="group"):
    """Integer tensors of a Qwen2-family float checkpoint (``get(name)`` returns a float array in
    the Hugging Face naming), as the reference's ``IntModel.__init__`` builds them
    (exact_llm.py:141-157): Q16 norm gains and embedding rows, linears per channel or per 128-row
    group, the head per channel (tied to the embedding when ``c["tie"]``)."""
    q16 = lambda k: np.rint(np.asarray(get(k), dtype=np.float64) * ONE).astype(np.int64)   # noqa: E731
    quant = quantize_group if lin == "group" else quantize_channel
    pfx = "model.layers.{}."
    keys = {"q": ("self_attn.q_proj", True), "k": ("self_attn.k_proj", True), "v": ("self_attn.v_proj", True),
            "o": ("self_attn.o_proj", False), "gate": ("mlp.gate_proj", False), "up": ("mlp.up_proj", False),
            "down": ("mlp.down_proj", False)}
    t = {}
    for i in range(c["NL"]):
        p = pfx.format(i)
        t[f"L{i}.g1"] = q16(p + "input_layernorm.weight")
        t[f"L{i}.g2"] = q16(p + "post_attention_layernorm.weight")
        for nm, (hf, has_bias) in keys.items():
            w, M, b = quant(get(p + hf + ".weight"), get(p + hf + ".bias") if has_bias else None)
            t[f"L{i}.{nm}.w"], t[f"L{i}.{nm}.M"] = w, M
            if b is not None:
                t[f"L{i}.{nm}.b"] = b
    t["gf"] = q16("model.norm.weight")
    emb = np.asarray(get("model.embed_tokens.weight"), dtype=np.float64)
    t["emb_q16"] = np.rint(emb * ONE).astype(np.int64)
    hw, hM, _ = quantize_channel(emb if c.get("tie") else get("lm_head.weight"))
    t["head.w"], t["head.M"] = hw, hM
    return t


# ----------------------------------------------------------------------------- writer / loader
def _sha256_file(path, bufsize=1 << 24):
    h = hashlib.sha256()
    with open(path, "rb") as f:
        while True:
            b = f.read(bufsize)
            if not b:
                break
            h.update(b)
    return h.hexdigest()


def write_artifact(path, c, tensors, rope_len, lin="group"):
    """Write a release of integer ``tensors`` (names as include/exactb200.h; ``emb_q16`` for the
    Q16 embedding rows) for architecture ``c`` with tables for ``rope_len`` positions."""
    os.makedirs(path, exist_ok=True)
    index = {}
    with open(os.path.join(path, "weights.int8"), "wb") as fw, open(os.path.join(path, "scales.int"), "wb") as fs:
        for name in sorted(tensors):
            a = np.asarray(tensors[name])
            if a.dtype == np.int8:
                f, fn, out = fw, "weights.int8", np.ascontiguousarray(a)
                pad = (-f.tell()) % 64
                f.write(b"\0" * pad)
            elif np.issubdtype(a.dtype, np.integer):
                f, fn, out = fs, "scales.int", np.ascontiguousarray(a, dtype="<i8")
            else:
                raise TypeError(f"{name}: integer tensors only (got {a.dtype})")
            index[name] = {"file": fn, "offset": f.tell(), "shape": list(a.shape),
                           "dtype": "int8" if fn == "weights.int8" else "int64"}
            f.write(out.tobytes())
    cos, sin = tables.rope_tables(int(rope_len), c["hd"], c["theta"])
    half = c["hd"] // 2
    tabs = {"exp": tables.exp_table(), "silu": tables.silu_table(), "sig": tables.sig_table(),
            "cos": np.ascontiguousarray(cos[:, :half]), "sin": np.ascontiguousarray(sin[:, :half])}
    tindex = {}
    with open(os.path.join(path, "tables.int"), "wb") as ft:
        for name, a in tabs.items():
            tindex[name] = {"offset": ft.tell(), "shape": list(a.shape)}
            ft.write(np.ascontiguousarray(a, dtype="<i8").tobytes())
    arch = {k: c[k] for k in ("D", "H", "KV", "hd", "I", "V", "NL", "theta") if k in c}
    arch.update(tie=bool(c.get("tie", False)), lin=lin, rope_len=int(rope_len))
    files = {fn: {"bytes": os.path.getsize(os.path.join(path, fn)), "sha256": _sha256_file(os.path.join(path, fn))}
             for fn in FILES}
    manifest = {"spec": SPEC, "format": "Q16",
                "tables": {"exp": "Q24, 1/256 steps on [0, 40)", "silu": "Q16 on [-16, 16) at 1/256",
                           "sig": "Q16 on [-16, 16) at 1/256", "rope": f"Q16 cos/sin, theta {c['theta']}",
                           "index": tindex},
                "arch": arch, "tensors": index, "files": files}
    with open(os.path.join(path, "manifest.json"), "w") as f:
        json.dump(manifest, f, indent=1, sort_keys=True)
    return manifest


def load_artifact(path):
    """(arch, tensors, tables) of a release after checking every file's size and SHA-256 against
    the manifest; arrays are read-only memory maps of the files."""
    with open(os.path.join(path, "manifest.json")) as f:
        man = json.load(f)
    if man.get("spec") != SPEC or man.get("format") != "Q16":
        raise ValueError(f"{path}: not an {SPEC} Q16 release")
    for fn in FILES:
        p = os.path.join(path, fn)
        want = man["files"][fn]
        if os.path.getsize(p) != want["bytes"]:
            raise ValueError(f"{fn}: size {os.path.getsize(p)} != manifest {want['bytes']}")
        got = _sha256_file(p)
        if got != want["sha256"]:
            raise ValueError(f"{fn}: SHA-256 {got} != manifest {want['sha256']}")
    tensors = {}
    for name, e in man["tensors"].items():
        dt = np.int8 if e["dtype"] == "int8" else np.dtype("<i8")
        count = int(np.prod(e["shape"])) if e["shape"] else 1
        tensors[name] = np.memmap(os.path.join(path, e["file"]), dtype=dt, mode="r", offset=e["offset"],
                                  shape=tuple(e["shape"]) if e["shape"] else (count,))
    tabs = {}
    for name, e in man["tables"]["index"].items():
        tabs[name] = np.memmap(os.path.join(path, "tables.int"), dtype=np.dtype("<i8"), mode="r",
                               offset=e["offset"], shape=tuple(e["shape"]))
    return man["arch"], tensors, tabs
