"""numpy restatement of exact-llm's integer forward pass -- TEST ORACLE, not product code.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s ``cpu_baseline`` leg use
this module.  Every function names the reference file:line whose behaviour it restates
(paths are relative to the reference project root).  Parity of this restatement with the
reference itself is pinned by ``tests/test_oracle_golden.py`` against fixtures that
``tests/golden/make_golden.py`` produced by importing and running the reference code.

Conventions: activations are int64 Q16 (``ONE = 2**16``); all arithmetic is numpy int64,
which wraps modulo 2**64 exactly like the reference's numpy arithmetic.
"""
import hashlib
import math

import numpy as np

F = 16
ONE = 1 << F
GROUP = 128
P1, P2 = 2147483647, 2147483629          # experiments/gpu_engine_trace_verify_kaggle.py:782
_POW2 = np.int64(1) << np.arange(63, dtype=np.int64)


def h16(a):
    """Conformance hash: first 16 hex chars of SHA-256 of the int64 bytes (exact_llm.py:22)."""
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()[:16]


# ----------------------------------------------------------------------------- primitives
def shr(a, n):
    """Round-half-up arithmetic shift right; n <= 0 shifts left (exact_llm.py:25-34)."""
    a = np.asarray(a, dtype=np.int64)
    n = np.asarray(n, dtype=np.int64)
    if n.ndim == 0:
        k = int(n)
        return (a << -k) if k <= 0 else ((a + (1 << (k - 1))) >> k)
    right = np.maximum(n, 0)
    bias = np.where(right > 0, np.int64(1) << np.maximum(right - 1, 0), 0)
    return ((a + bias) >> right) << np.maximum(-n, 0)


def bitlen(m):
    """Bit length of non-negative int64 values (exact_llm.py:35-40): #powers of two <= m."""
    m = np.asarray(m, dtype=np.int64)
    return (m[..., None] >= _POW2).sum(-1).astype(np.int64)


def qrow(x, bits=15):
    """Per-row int16 quantisation: s = max(bitlen(max|x|)-15, 0), xq = clip(shr(x, s)) (exact_llm.py:41-46)."""
    lim = (1 << bits) - 1
    s = np.maximum(bitlen(np.abs(x).max(-1, keepdims=True)) - bits, 0)
    return np.clip(shr(x, s), -lim, lim), s


def isqrt(n):
    """floor(sqrt(double(n))) with one correction step each way (exact_llm.py:97-99)."""
    r = np.floor(np.sqrt(n.astype(np.float64))).astype(np.int64)
    r = np.where(r * r > n, r - 1, r)
    return np.where((r + 1) * (r + 1) <= n, r + 1, r)


def irms(x, g):
    """Integer RMSNorm (exact_llm.py:100-106; SPEC.md:20)."""
    k = np.maximum(bitlen(np.abs(x).max(-1, keepdims=True)) - 24, 0)
    xs = shr(x, k)
    ms = (xs * xs).sum(-1, keepdims=True) // x.shape[-1] + 1
    r = np.maximum(isqrt(ms), 1)
    return shr(((x << F) // (r << k)) * g, F)


# Tables are data built once on the host with the same float64 expressions as the reference
# (exact_llm.py:108, :117; experiments/moe_exact_kaggle.py:419) -- never device math.
def exp_table():
    return np.array([round(math.exp(-i / 256) * (1 << 24)) for i in range(256 * 40 + 2)], np.int64)


def silu_table():
    out = []
    for i in range(32 * 256 + 2):
        v = (i - 16 * 256) / 256
        out.append(round(v / (1 + math.exp(-v)) * ONE))
    return np.array(out, np.int64)


def sig_table():
    return np.array([round(1.0 / (1.0 + math.exp(-((i - 16 * 256) / 256))) * ONE) for i in range(32 * 256 + 2)],
                    np.int64)


EXP_T = exp_table()
SILU_T = silu_table()
SIG_T = sig_table()


def isoftmax(sc, valid):
    """Q20 probabilities from Q16 scores via the Q24 exp table (exact_llm.py:109-115; SPEC.md:23)."""
    mx = np.where(valid, sc, np.iinfo(np.int64).min // 4).max(-1, keepdims=True)
    d = np.where(valid, mx - sc, 0)
    i = np.minimum(d >> 8, len(EXP_T) - 2)
    fr = d & 255
    e = EXP_T[i] - shr((EXP_T[i] - EXP_T[i + 1]) * fr, 8)
    e = np.where(valid & (d < (40 << F)), e, 0)
    return (e << 20) // e.sum(-1, keepdims=True)


def _table_interp(x, T, hi_value):
    t = np.clip(x, -16 * ONE, 16 * ONE - 1) + 16 * ONE
    i, fr = t >> 8, t & 255
    y = T[i] + shr((T[i + 1] - T[i]) * fr, 8)
    return np.where(x >= 16 * ONE, hi_value, np.where(x < -16 * ONE, 0, y))


def isilu(x):
    """Q16 SiLU table on [-16,16), identity above, 0 below (exact_llm.py:118-124)."""
    return _table_interp(x, SILU_T, x)


def isig(x):
    """Q16 sigmoid table, ONE above 16, 0 below -16 (experiments/moe_exact_kaggle.py:420-424)."""
    return _table_interp(x, SIG_T, ONE)


def rope_tables(T, hd, theta):
    """Q16 cos/sin tables, float64 on the host, rounded half-to-even (exact_llm.py:127-130, 157-158)."""
    inv = 1.0 / (theta ** (np.arange(0, hd, 2, dtype=np.float64) / hd))
    ang = np.outer(np.arange(T, dtype=np.float64), inv)
    ang = np.concatenate([ang, ang], -1)
    return np.rint(np.cos(ang) * ONE).astype(np.int64), np.rint(np.sin(ang) * ONE).astype(np.int64)


def rot_half(x):
    h = x.shape[-1] // 2
    return np.concatenate([-x[..., h:], x[..., :h]], -1)                      # exact_llm.py:131-132


def rope(x, cos, sin):
    """shr(x*cos + rot_half(x)*sin, 16); x (..., T, hd), cos/sin (T, hd) (exact_llm.py:159-160)."""
    return shr(x * cos + rot_half(x) * sin, F)


def mm_exact(a, b):
    """Exact int64 a @ b through float64 BLAS; valid while every partial sum < 2^53 (SPEC.md:30-32)."""
    return np.rint(np.matmul(a.astype(np.float64), b.astype(np.float64))).astype(np.int64)


# ----------------------------------------------------------------------------- linears
class GroupLinear:
    """Group-128 linear: tot = sum_g M_g * (xq_g . W_g), y = shr(tot, 28 - s) + b.

    Restates ``GQLin.__call__`` (experiments/speed_fair_kaggle.py:722-725; SPEC.md:18).
    Layout: w (N, K) int8 (out, in), M (N, K/128) integer scales, b (N,) Q16 or None.
    """
    kind = "group"

    def __init__(self, w, M, b=None):
        self.w = np.ascontiguousarray(w, dtype=np.int8)
        self.M = np.ascontiguousarray(M, dtype=np.int64)
        self.b = None if b is None else np.asarray(b, np.int64)
        self.N, self.K = self.w.shape
        assert self.K % GROUP == 0 and self.M.shape == (self.N, self.K // GROUP)

    def raw(self, xq):
        tot = np.zeros((xq.shape[0], self.N), np.int64)
        for g in range(self.K // GROUP):
            ks = slice(g * GROUP, (g + 1) * GROUP)
            tot += mm_exact(xq[:, ks], self.w[:, ks].T) * self.M[:, g]
        return tot

    def requant(self, raw, s):
        y = shr(raw, 28 - s)
        return y if self.b is None else y + self.b

    def __call__(self, x, trace=None, name=None):
        xq, s = qrow(x, 15)
        raw = self.raw(xq)
        if trace is not None:
            trace.append((name, raw, xq))
        return self.requant(raw, s)


class ChannelLinear:
    """Per-output-channel linear with the per-row overflow drop rule.

    Restates ``QLin.__call__`` (exact_llm.py:89-96; SPEC.md:18, :28):
    acc = xq . W, drop = max(bitlen(max_row|acc|) + bitlen(max M) - 62, 0),
    y = shr(shr(acc, drop) * M, 28 - s - drop) + b.
    """
    kind = "channel"

    def __init__(self, w, M, b=None):
        self.w = np.ascontiguousarray(w, dtype=np.int8)
        self.M = np.asarray(M, dtype=np.int64)
        self.b = None if b is None else np.asarray(b, np.int64)
        self.N, self.K = self.w.shape
        self.Mbits = int(bitlen(np.array(self.M.max())))

    def raw(self, xq):
        # column chunks of 32768 bound the float64 temporaries, as the reference does (exact_llm.py:92)
        return np.concatenate([mm_exact(xq, self.w[j:j + 32768].T) for j in range(0, self.N, 32768)], -1)

    def requant(self, acc, s):
        drop = np.maximum(bitlen(np.abs(acc).max(-1, keepdims=True)) + self.Mbits - 62, 0)
        y = shr(shr(acc, drop) * self.M, 28 - s - drop)
        return y if self.b is None else y + self.b

    def __call__(self, x, trace=None, name=None):
        xq, s = qrow(x, 15)
        acc = self.raw(xq)
        if trace is not None:
            trace.append((name, acc, xq))
        return self.requant(acc, s)


def quantize_channel(w_out_in, bias=None):
    """float64 per-channel conversion of an (out, in) float matrix (exact_llm.py:83-88, 133-139)."""
    w = np.asarray(w_out_in, dtype=np.float64)
    sc = np.abs(w).max(1)
    sc = np.where(sc == 0, 1e-12, sc) / 127.0
    wi = np.clip(np.rint(w / sc[:, None]), -127, 127).astype(np.int8)
    M = np.rint(sc * (1 << 28)).astype(np.int64)
    b = None if bias is None else np.rint(np.asarray(bias, dtype=np.float64) * ONE).astype(np.int64)
    return ChannelLinear(wi, M, b)


# ----------------------------------------------------------------------------- models
LIN_NAMES = ("q", "k", "v", "o", "gate", "up", "down")


class OracleModel:
    """Dense Qwen2-family integer model with an optional KV cache.

    ``__call__(ids)`` restates ``IntModel.__call__`` (exact_llm.py:161-180): full causal
    recompute.  ``forward(ids, cache)`` is the same program fed incrementally; spec v0.3
    made the model causal, so both give identical bits (exact_torch.py:171-193).

    ``layers``: list of dicts with g1, g2 (D,) Q16 gains and linears q,k,v,o,gate,up,down.
    ``emb_q16``: callable ids -> int64 (T, D) Q16 rows.  ``head``: ChannelLinear.
    """

    def __init__(self, c, layers, gf, head, emb_q16, cos, sin, moe=None):
        self.c, self.layers, self.gf, self.head = c, layers, gf, head
        self.emb_q16, self.cos, self.sin, self.moe = emb_q16, cos, sin, moe
        self.INV = int(round((1 << 16) / math.sqrt(c["hd"])))                  # exact_llm.py:164

    def new_cache(self):
        return {"n": 0, "layers": [None] * len(self.layers)}

    def _attention(self, li, q, k, v, cache, p0):
        H, KV, hd = self.c["H"], self.c["KV"], self.c["hd"]
        T = q.shape[1]
        kq, sk = qrow(k)                                         # per (head, position) row
        if cache is not None:
            prev = cache["layers"][li]
            if prev is not None:
                kq = np.concatenate([prev[0], kq], 1)
                sk = np.concatenate([prev[1], sk], 1)
                v = np.concatenate([prev[2], v], 1)
            cache["layers"][li] = (kq, sk, v)
        S = kq.shape[1]
        valid = np.arange(S)[None, :] <= (p0 + np.arange(T))[:, None]
        out = np.empty((H, T, hd), np.int64)
        for hh in range(H):
            kh = hh // (H // KV)
            qq, sq = qrow(q[hh])
            sc = shr(mm_exact(qq, kq[kh].T) * self.INV, (F - sq - sk[kh].T) + 16)
            p = isoftmax(sc, valid)
            out[hh] = shr(np.matmul(p, v[kh]), 20)               # exact int64, no length cap
        return out

    def _mlp(self, L, m, trace, li, stats):
        if self.moe is not None:
            return self.moe.forward(L, m, trace, li, stats)
        g = L["gate"](m, trace, f"L{li}.gate")
        u = L["up"](m, trace, f"L{li}.up")
        return L["down"](shr(isilu(g) * u, F), trace, f"L{li}.down")

    def forward(self, ids, cache=None, trace=None, stats=None, last_only=False):
        c = self.c
        H, KV, hd = c["H"], c["KV"], c["hd"]
        T = len(ids)
        p0 = cache["n"] if cache is not None else 0
        x = self.emb_q16(np.asarray(ids))
        cos, sin = self.cos[p0:p0 + T], self.sin[p0:p0 + T]
        for li, L in enumerate(self.layers):
            a = irms(x, L["g1"])
            q = rope(L["q"](a, trace, f"L{li}.q").reshape(T, H, hd).transpose(1, 0, 2), cos, sin)
            k = rope(L["k"](a, trace, f"L{li}.k").reshape(T, KV, hd).transpose(1, 0, 2), cos, sin)
            v = L["v"](a, trace, f"L{li}.v").reshape(T, KV, hd).transpose(1, 0, 2)
            out = self._attention(li, q, k, v, cache, p0)
            x = x + L["o"](out.transpose(1, 0, 2).reshape(T, H * hd), trace, f"L{li}.o")
            x = x + self._mlp(L, irms(x, L["g2"]), trace, li, stats)
        if cache is not None:
            cache["n"] = p0 + T
        if last_only:
            x = x[-1:]
        return self.head(irms(x, self.gf), trace, "head")

    def __call__(self, ids, trace=None, stats=None):
        return self.forward(ids, None, trace, stats)


class OracleMoE:
    """Integer MoE block (experiments/moe_exact_kaggle.py:454-467).

    Router = per-channel linear -> isoftmax (Q20) -> top-k by probability, ties to the
    lower expert index (stable sort); expert SwiGLU MLPs weighted by shr(p * y, 20);
    shared expert scaled by shr(isig(sgate(m)) * ys, 16).
    """

    def __init__(self, n_experts, topk):
        self.NE, self.TOPK = n_experts, topk

    def route(self, L, m, trace=None, li=0):
        T = m.shape[0]
        logits = L["router"](m, trace, f"L{li}.router")
        p = isoftmax(logits, np.ones((T, self.NE), bool))
        sel = np.argsort(-p, axis=-1, kind="stable")[:, :self.TOPK]
        return p, sel

    def forward(self, L, m, trace=None, li=0, stats=None):
        p, sel = self.route(L, m, trace, li)
        if stats is not None:
            stats.setdefault(li, []).append(sel.copy())
        out = np.zeros_like(m)
        for e in range(self.NE):
            rows, _ = np.nonzero(sel == e)
            if len(rows) == 0:
                continue
            gp, up, dn = L["ex"][e]
            me = m[rows]
            ye = dn(shr(isilu(gp(me, trace, f"L{li}.e{e}.g")) * up(me, trace, f"L{li}.e{e}.u"), F),
                    trace, f"L{li}.e{e}.d")
            out[rows] += shr(p[rows, e][:, None] * ye, 20)
        ys = L["sd"](shr(isilu(L["sg"](m, trace, f"L{li}.sg")) * L["su"](m, trace, f"L{li}.su"), F),
                     trace, f"L{li}.sd")
        return out + shr(isig(L["sgate"](m, trace, f"L{li}.sgate")) * ys, F)


# ----------------------------------------------------------------------------- greedy decode
def greedy_generate(model, prompt, n_steps):
    """Greedy decode with a KV cache; argmax ties go to the lowest index (exact_llm.py:262-268).

    Returns (prefill logits (T,V), [step logits rows], tokens)."""
    cache = model.new_cache()
    lg = model.forward(list(prompt), cache)
    rows, toks = [], []
    nxt = int(lg[-1].argmax())
    for _ in range(n_steps):
        toks.append(nxt)
        row = model.forward([nxt], cache)[0]
        rows.append(row)
        nxt = int(row.argmax())
    return lg, rows, toks


# ----------------------------------------------------------------------------- Freivalds
def freivalds_key(lin, r_list):
    """Key d_p = (W*M)^T r mod p for each prime (gpu_engine_trace_verify_kaggle.py:803-819).

    ``r_list`` = [(p, r)] with r (N,) in [0, p).  Returns [(p, r, d)] with d (K,) in [0, p).
    Exact: every partial sum below stays < 2^63."""
    out = []
    K = lin.K
    for p, r in r_list:
        if lin.kind == "group":
            Wm = (lin.w.astype(np.int64) * np.repeat(lin.M, GROUP, axis=1)) % p      # (N, K) < 2^31
        else:
            Wm = lin.w.astype(np.int64) % p
        d = np.zeros(K, np.int64)
        for j in range(0, lin.N, 2048):                                          # 2048*2^62 would overflow:
            part = (Wm[j:j + 2048] * r[j:j + 2048, None]) % p                    # each product < 2^62 -> mod p
            d = (d + part.sum(0) % p) % p                                        # sum of 2048 values < 2^42
        out.append((p, r, d))
    return out


def draw_keys(lins, seed=2026):
    """r vectors drawn in the reference's order: per linear, per prime, rng.integers(0, p, N)
    (gpu_engine_trace_verify_kaggle.py:802-828)."""
    rng = np.random.default_rng(seed)
    return [[(p, rng.integers(0, p, lin.N, dtype=np.int64)) for p in (P1, P2)] for lin in lins]


def freivalds_check(keys, xq, acc):
    """Sum_n r_n (acc_n mod p) == Sum_k d_k (xq_k mod p) (mod p) for every row and prime
    (gpu_engine_trace_verify_kaggle.py:830-834; Python % is non-negative)."""
    if acc.shape[1] != keys[0][1].shape[0]:
        return False
    for p, r, d in keys:
        lhs = (((acc % p) * r) % p).sum(-1) % p
        rhs = (((xq % p) * d) % p).sum(-1) % p
        if not bool((lhs == rhs).all()):
            return False
    return True


def freivalds_sides(keys, xq, acc):
    """(lhs, rhs) arrays of shape (rows, 2) for the two primes."""
    lhs = np.stack([(((acc % p) * r) % p).sum(-1) % p for p, r, _ in keys], -1)
    rhs = np.stack([(((xq % p) * d) % p).sum(-1) % p for p, _, d in keys], -1)
    return lhs, rhs


# ----------------------------------------------------------------------------- trace commitment
def step_digest(flat):
    """Per-step trace commitment: SHA-256 over 4 equal chunks of the flat int64 trace, then
    SHA-256 of the 4 digests (experiments/prover_commit_cost_gpu_kaggle.py:811-817)."""
    arr = np.ascontiguousarray(flat, dtype=np.int64)
    step = (len(arr) + 3) // 4
    parts = [hashlib.sha256(arr[i * step:(i + 1) * step].tobytes()).digest() for i in range(4)]
    return hashlib.sha256(b"".join(parts)).digest()


# ----------------------------------------------------------------------------- Merkle trace commitment
def commit_trace(model, ids, fake=None, cheat_layer=None, cheat_down=None):
    """One full forward of ``ids`` recording what the trace commitment covers: the residual
    stream X entering every layer (and the final one), every linear's integer accumulator, the
    roped K and the V rows of every layer, and the head accumulator.  Restates ``prover_trace``
    (experiments/commit_audit_kaggle.py:587-613); a group-128 linear's accumulator is its ``tot``,
    as in the reference's trace capture.  Attack hooks as the reference's: ``fake = (layer, fn)``
    replaces that layer's attention probabilities by ``fn(p)`` (every head), ``cheat_down`` is
    used as layer ``cheat_layer``'s down projection."""
    c = model.c
    H, KV, hd = c["H"], c["KV"], c["hd"]
    T = len(ids)
    x = model.emb_q16(np.asarray(ids))
    cos, sin = model.cos[:T], model.sin[:T]
    X, A, KR = [], [], []
    for li, L in enumerate(model.layers):
        X.append(x.copy())
        tr = []
        a = irms(x, L["g1"])
        q = rope(L["q"](a, tr, "q").reshape(T, H, hd).transpose(1, 0, 2), cos, sin)
        k = rope(L["k"](a, tr, "k").reshape(T, KV, hd).transpose(1, 0, 2), cos, sin)
        v = L["v"](a, tr, "v").reshape(T, KV, hd).transpose(1, 0, 2)
        KR.append((k.copy(), v.copy()))
        if fake is not None and fake[0] == li:
            valid = np.tril(np.ones((T, T), bool))
            out = np.empty((H, T, hd), np.int64)
            for hh in range(H):
                kh = hh // (H // KV)
                qq, sq = qrow(q[hh])
                kk, sk = qrow(k[kh])
                sc = shr(mm_exact(qq, kk.T) * model.INV, (F - sq - sk.T) + 16)
                out[hh] = shr(np.matmul(fake[1](isoftmax(sc, valid)), v[kh]), 20)
        else:
            out = model._attention(li, q, k, v, None, 0)
        x = x + L["o"](out.transpose(1, 0, 2).reshape(T, H * hd), tr, "o")
        m_ = irms(x, L["g2"])
        g = L["gate"](m_, tr, "gate")
        u = L["up"](m_, tr, "up")
        dn = cheat_down if (cheat_down is not None and cheat_layer == li) else L["down"]
        x = x + dn(shr(isilu(g) * u, F), tr, "down")
        A.append({nm: raw for nm, raw, _ in tr})
    X.append(x.copy())
    htr = []
    model.head(irms(x, model.gf), htr, "head")
    return {"X": X, "A": A, "KR": KR, "head": htr[0][1], "T": T}


def hb(*arrs):
    """Leaf digest: SHA-256 over each array's int64 bytes, each followed by b"|"
    (experiments/commit_audit_kaggle.py:567-570)."""
    hh = hashlib.sha256()
    for a in arrs:
        hh.update(np.ascontiguousarray(a, dtype=np.int64).tobytes())
        hh.update(b"|")
    return hh.digest()


def commit_leaves(tr, NL):
    """Leaf digests in the reference order (experiments/commit_audit_kaggle.py:614-628): X of
    every (layer 0..NL, position), then per (layer, position) the k|v accumulators, the roped
    K|V rows, the q accumulator and the o|gate|up|down accumulators, then the head per position."""
    T = tr["T"]
    leaves = [hb(tr["X"][L][t]) for L in range(NL + 1) for t in range(T)]
    for L in range(NL):
        a = tr["A"][L]
        for t in range(T):
            leaves.append(hb(a["k"][t], a["v"][t]))
            leaves.append(hb(tr["KR"][L][0][:, t, :], tr["KR"][L][1][:, t, :]))
            leaves.append(hb(a["q"][t]))
            leaves.append(hb(a["o"][t], a["gate"][t], a["up"][t], a["down"][t]))
    leaves += [hb(tr["head"][t]) for t in range(T)]
    return leaves


def merkle_root(leaves):
    """Merkle root: leaf nodes SHA-256(b"L" + leaf), parents SHA-256(b"N" + left + right), an odd
    last node paired with itself (experiments/commit_audit_kaggle.py:571-575)."""
    lv = [hashlib.sha256(b"L" + leaf).digest() for leaf in leaves]
    while len(lv) > 1:
        lv = [hashlib.sha256(b"N" + lv[i] + (lv[i + 1] if i + 1 < len(lv) else lv[i])).digest()
              for i in range(0, len(lv), 2)]
    return lv[0]


# ----------------------------------------------------------------------------- integer sampler + receipts
MASK64 = (1 << 64) - 1


def splitmix64(seed, pos):
    """exact_llm.py:243-247 (Python integers, modulo 2^64)."""
    z = (seed + (pos + 1) * 0x9E3779B97F4A7C15) & MASK64
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & MASK64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & MASK64
    return z ^ (z >> 31)


def u20(seed, pos):
    """Uniform integer in [0, 2^20) (exact_llm.py:248)."""
    return splitmix64(seed, pos) >> 44


def temp_num(t):
    """Temperature as an integer multiplier (exact_llm.py:249)."""
    return int(round((1 << 16) / t))


def isoftmax_row(lg):
    """Q20 probabilities of one Q16 logits row through the exp table (exact_llm.py:250-255)."""
    T = exp_table()
    d = lg.max() - lg
    i = np.minimum(d >> 8, len(T) - 2)
    fr = d & 255
    e = T[i] - shr((T[i] - T[i + 1]) * fr, 8)
    e = np.where(d < (40 << 16), e, 0)
    return (e << 20) // e.sum()


def sample_int(lg_row, seed, pos, tnum):
    """Token = first index whose cumulative probability exceeds (u20 * total) >> 20
    (exact_llm.py:256-259)."""
    p = isoftmax_row(shr(np.asarray(lg_row, np.int64) * tnum, 16))
    cum = np.cumsum(p)
    target = (u20(seed, pos) * int(cum[-1])) >> 20
    return int(np.searchsorted(cum, target, side="right")), p


def step_hash(prev, lg_row):
    """Receipt chain link: SHA-256 over the previous link's ASCII and the logits row's int64 bytes,
    first 16 hex characters (exact_llm.py:260-261)."""
    return hashlib.sha256(prev.encode() + np.ascontiguousarray(lg_row, dtype=np.int64).tobytes()).hexdigest()[:16]


def sampled_generate(model, prompt_ids, n, seed, temp):
    """Seeded integer sampling with the receipt hash chain, full recompute per token
    (exact_llm.py:262-268)."""
    ids, chain, toks, greedy, tnum = list(prompt_ids), "start", [], [], temp_num(temp)
    for t in range(n):
        lg = model(ids)[-1]
        tok, _ = sample_int(lg, seed, t, tnum)
        chain = step_hash(chain, lg)
        toks.append(tok)
        greedy.append(int(lg.argmax()))
        ids.append(tok)
    return dict(prompt=list(prompt_ids), seed=seed, temp=temp, tokens=toks, chain=chain), greedy


# ----------------------------------------------------------------------------- weightless cell verifier
def leaf_index(kind, L, t, T, NL):
    """Position of a named leaf in the leaves_of order (experiments/commit_audit_kaggle.py:614-628)."""
    if kind == "X":
        return L * T + t
    if kind == "HEAD":
        return (NL + 1) * T + 4 * NL * T + t
    return (NL + 1) * T + (L * T + t) * 4 + ("KV", "KR", "Q", "R").index(kind)


def leaf_values(tr, name):
    """Opened values of a named leaf (experiments/commit_audit_kaggle.py:632-639)."""
    kind, L, t = name
    if kind == "X":
        return [tr["X"][L][t]]
    if kind == "HEAD":
        return [tr["head"][t]]
    if kind == "KR":
        return [tr["KR"][L][0][:, t, :], tr["KR"][L][1][:, t, :]]
    a = tr["A"][L]
    if kind == "KV":
        return [a["k"][t], a["v"][t]]
    if kind == "Q":
        return [a["q"][t]]
    return [a["o"][t], a["gate"][t], a["up"][t], a["down"][t]]


def merkle_levels(leaves):
    lv = [hashlib.sha256(b"L" + leaf).digest() for leaf in leaves]
    levels = [lv]
    while len(lv) > 1:
        lv = [hashlib.sha256(b"N" + lv[i] + (lv[i + 1] if i + 1 < len(lv) else lv[i])).digest()
              for i in range(0, len(lv), 2)]
        levels.append(lv)
    return levels


def merkle_proof(levels, idx):
    """Sibling path, the node itself where it has no sibling (experiments/commit_audit_kaggle.py:576-580)."""
    pr = []
    for lv in levels[:-1]:
        sib = idx ^ 1
        pr.append(lv[sib] if sib < len(lv) else lv[idx])
        idx >>= 1
    return pr


def merkle_verify(root, leaf, idx, pr):
    """experiments/commit_audit_kaggle.py:581-585."""
    h = hashlib.sha256(b"L" + leaf).digest()
    for sib in pr:
        h = hashlib.sha256(b"N" + (h + sib if idx % 2 == 0 else sib + h)).digest()
        idx >>= 1
    return h == root


def needed(cell, NL):
    """Leaves a cell verification opens (experiments/commit_audit_kaggle.py:647-651)."""
    L, t = cell
    if L == NL:
        return [("X", NL, t), ("HEAD", NL, t)]
    return [("X", L, t), ("KV", L, t)] + [("KR", L, s) for s in range(t + 1)] + \
           [("Q", L, t), ("R", L, t), ("X", L + 1, t)]


def open_cell(tr, NL, levels, cell, lie=None):
    """{name: (values, proof)} for a cell; ``lie`` = a name whose first value is altered by one
    (experiments/commit_audit_kaggle.py:640-646)."""
    out = {}
    for n in needed(cell, NL):
        vals = [np.array(v, np.int64, copy=True) for v in leaf_values(tr, n)]
        if lie is not None and n == lie:
            vals[0].reshape(-1)[0] += 1
        out[n] = (vals, merkle_proof(levels, leaf_index(*n, tr["T"], NL)))
    return out


def verifier_keys(model, seed=2026):
    """The weightless verifier's secrets in the reference's draw order (make_verifier,
    experiments/commit_audit_kaggle.py:461-512): per linear (layers' q,k,v,o,gate,up,down, then the
    head) and prime, r ~ U[0, p) of length N and d = W r mod p (W r over the fused W * M for a
    group-128 linear, whose accumulator is tot); for the embedding, r of length D and the digest
    de of every Q16 row."""
    rng = np.random.default_rng(seed)

    def vlin(lin):
        keys = []
        for p in (P1, P2):
            r = rng.integers(0, p, lin.N, dtype=np.int64)
            d = np.zeros(lin.K, np.int64)
            if lin.kind == "group":
                for g in range(lin.K // GROUP):
                    ks = slice(g * GROUP, (g + 1) * GROUP)
                    wm = (lin.w[:, ks].astype(np.int64) * (lin.M[:, g:g + 1] % p)) % p          # (N, 128)
                    for j in range(0, lin.N, 4096):
                        d[ks] = (d[ks] + ((wm[j:j + 4096].T % p) * r[j:j + 4096] % p).sum(-1)) % p
            else:
                for j in range(0, lin.N, 8192):
                    d = (d + lin.w[j:j + 8192].astype(np.int64).T @ r[j:j + 8192]) % p
            keys.append((p, r, d))
        return keys

    keys = {"layers": [{nm: vlin(L[nm]) for nm in ("q", "k", "v", "o", "gate", "up", "down")} for L in model.layers]}
    keys["head"] = vlin(model.head)
    D = model.c["D"]
    X = model.emb_q16(np.arange(model.c["V"]))
    keys["emb"] = []
    for p in (P1, P2):
        r = rng.integers(0, p, D, dtype=np.int64)
        keys["emb"].append((p, r, (((X % p) * r) % p).sum(-1) % p))
    return keys


def fr_row(lin, keys, xq_row, acc_row):
    """Freivalds check of one accumulator row (experiments/commit_audit_kaggle.py:652-656); the
    size bound applies to per-channel accumulators."""
    if acc_row.shape != (lin.N,):
        return False
    if lin.kind != "group" and int(np.abs(acc_row).max()) > 127 * 32767 * lin.K:
        return False
    for p, r, d in keys:
        if int((((acc_row % p) * r) % p).sum() % p) != int((((xq_row % p) * d) % p).sum() % p):
            return False
    return True


def _rq(lin, acc_row, s):
    """experiments/commit_audit_kaggle.py:657-658."""
    return lin.requant(acc_row[None, :], np.array([[s]], np.int64))[0]


def verify_cell(model, keys, root, T, cell, opened, ids):
    """(ok, reason) of one cell from its opened leaves, without the weights (verify_cell,
    experiments/commit_audit_kaggle.py:659-705)."""
    NL = len(model.layers)
    c = model.c
    for n in needed(cell, NL):
        if n not in opened:
            return False, f"missing {n}"
        vals, pr = opened[n]
        if not merkle_verify(root, hb(*vals), leaf_index(*n, T, NL), pr):
            return False, f"merkle {n}"
    L, t = cell
    H, KV, hd = c["H"], c["KV"], c["hd"]
    if L == NL:
        x = opened[("X", NL, t)][0][0]
        hacc = opened[("HEAD", NL, t)][0][0]
        xq, s = qrow(irms(x[None, :], model.gf), 15)
        if not fr_row(model.head, keys["head"], xq[0], hacc):
            return False, "head"
        return True, None
    Lw = model.layers[L]
    K = keys["layers"][L]
    if L == 0:
        xr = opened[("X", 0, t)][0][0]
        for p, r, de in keys["emb"]:
            if int((((xr % p) * r) % p).sum() % p) != int(de[ids[t]]):
                return False, f"embedding@{t}"
    x = opened[("X", L, t)][0][0]
    kacc, vacc = opened[("KV", L, t)][0]
    xq, sh = qrow(irms(x[None, :], Lw["g1"]), 15)
    if not (fr_row(Lw["k"], K["k"], xq[0], kacc) and fr_row(Lw["v"], K["v"], xq[0], vacc)):
        return False, f"kv@{t}"
    ko = _rq(Lw["k"], kacc, sh[0, 0]).reshape(KV, hd)
    vo = _rq(Lw["v"], vacc, sh[0, 0]).reshape(KV, hd)
    kt = shr(ko * model.cos[t] + rot_half(ko) * model.sin[t], F)
    krk, krv = opened[("KR", L, t)][0]
    if not (np.array_equal(krk, kt) and np.array_equal(krv, vo)):
        return False, f"kr@{t}"
    Kc = np.stack([opened[("KR", L, s_)][0][0] for s_ in range(t + 1)], 1)
    Vc = np.stack([opened[("KR", L, s_)][0][1] for s_ in range(t + 1)], 1)
    qacc = opened[("Q", L, t)][0][0]
    oacc, gacc, uacc, dacc = opened[("R", L, t)][0]
    if not fr_row(Lw["q"], K["q"], xq[0], qacc):
        return False, "q"
    qo = _rq(Lw["q"], qacc, sh[0, 0]).reshape(H, hd)
    qo = shr(qo * model.cos[t] + rot_half(qo) * model.sin[t], F)
    out = np.empty((H, hd), np.int64)
    valid = np.ones((1, t + 1), bool)
    for hh in range(H):
        kh = hh // (H // KV)
        qq, sq = qrow(qo[hh][None, :])
        kk, sk = qrow(Kc[kh])
        sc = shr(mm_exact(qq, kk.T) * model.INV, (F - sq - sk.T) + 16)
        out[hh] = shr(np.matmul(isoftmax(sc, valid), Vc[kh]), 20)[0]
    oq, so = qrow(out.reshape(1, H * hd), 15)
    if not fr_row(Lw["o"], K["o"], oq[0], oacc):
        return False, "o"
    x2 = x + _rq(Lw["o"], oacc, so[0, 0])
    mq, sm = qrow(irms(x2[None, :], Lw["g2"]), 15)
    if not (fr_row(Lw["gate"], K["gate"], mq[0], gacc) and fr_row(Lw["up"], K["up"], mq[0], uacc)):
        return False, "gate/up"
    act = shr(isilu(_rq(Lw["gate"], gacc, sm[0, 0])) * _rq(Lw["up"], uacc, sm[0, 0]), F)
    dq, sd = qrow(act[None, :], 15)
    if not fr_row(Lw["down"], K["down"], dq[0], dacc):
        return False, "down"
    if not np.array_equal(x2 + _rq(Lw["down"], dacc, sd[0, 0]), opened[("X", L + 1, t)][0][0]):
        return False, "residual"
    return True, None
