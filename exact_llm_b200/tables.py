"""Integer tables of the exact program, built once on the host (SPEC.md section 1 of the reference:
tables ship as integers and are never recomputed with device math).

The float64 expressions are those of the reference (exact_llm.py:108 exp, :117 SiLU, :127-130 and
:157-158 RoPE; experiments/moe_exact_kaggle.py:419 sigmoid); the integer results are pinned by
the golden fixtures recorded from the reference itself.
"""
import math

import numpy as np

ONE = 1 << 16


def exp_table():
    """Q24 exp(-i/256), i < 10242 (exact_llm.py:108)."""
    return np.array([round(math.exp(-i / 256) * (1 << 24)) for i in range(256 * 40 + 2)], np.int64)


def silu_table():
    """Q16 SiLU on [-16, 16) at 1/256 steps, 8194 entries (exact_llm.py:117)."""
    vals = []
    for i in range(32 * 256 + 2):
        v = (i - 16 * 256) / 256
        vals.append(round(v / (1 + math.exp(-v)) * ONE))
    return np.array(vals, np.int64)


def sig_table():
    """Q16 sigmoid on [-16, 16) at 1/256 steps (experiments/moe_exact_kaggle.py:419)."""
    return np.array([round(1.0 / (1.0 + math.exp(-((i - 16 * 256) / 256))) * ONE) for i in range(32 * 256 + 2)],
                    np.int64)


def rope_tables(T, hd, theta):
    """Q16 cos/sin (T, hd) of angle t * theta^(-2i/hd), halves repeated (exact_llm.py:127-130)."""
    inv = 1.0 / (theta ** (np.arange(0, hd, 2, dtype=np.float64) / hd))
    ang = np.outer(np.arange(T, dtype=np.float64), inv)
    ang = np.concatenate([ang, ang], -1)
    return np.rint(np.cos(ang) * ONE).astype(np.int64), np.rint(np.sin(ang) * ONE).astype(np.int64)


def inv_scale(hd):
    """INV = round(2^16 / sqrt(hd)) (exact_llm.py:164)."""
    return int(round((1 << 16) / math.sqrt(hd)))
