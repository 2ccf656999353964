"""Generate the golden fixtures under tests/golden/ by RUNNING THE REFERENCE's own code.

Usage:  python tests/golden/make_golden.py --ref <path to the exact-llm checkout> [--only NAME ...]

The reference (novain-shibu/exact-llm) is a Python project; this script imports its
``exact_llm.py`` and executes, from its experiment scripts, only the class/function
definitions the hot path needs (the scripts' top-level code downloads checkpoints):

  * ``GQLin``                         experiments/speed_fair_kaggle.py:713-725
  * ``SIG_T``/``isig``                 experiments/moe_exact_kaggle.py:419-424
  * ``MoEInt``                         experiments/moe_exact_kaggle.py:433-482
  * ``P1, P2``                         experiments/gpu_engine_trace_verify_kaggle.py:782
  * ``keys_group/keys_channel/fr``     experiments/gpu_engine_trace_verify_kaggle.py:802-819, 830-834
  * the tiny preflight model           experiments/_pre_tiny.py:1-15
  * the G1 GEMV known-answer inputs    experiments/speed_fair_kaggle.py:704-708
  * ``splitmix64/u20/temp_num/isoftmax_row/sample_int/step_hash/generate``  exact_llm.py:243-263
  * ``GQLin`` constructor (float64 group-128 conversion)  experiments/group128_quality_kaggle.py:406-414
  * ``requant/Hb/merkle/prover_trace/leaves_of``  experiments/commit_audit_kaggle.py:442-445,
                                      567-575, 587-628 (the Merkle trace commitment)
  * ``VLin/VEmb/make_verifier/Prover/needed/verify_cell``  experiments/commit_audit_kaggle.py:460-512,
                                      629-705 (the weightless cell verifier)

Synthetic integer weights come from ``oracle.synth`` and are handed to the reference's
classes through ``__new__`` (no float checkpoint is involved).  Nothing here is imported
by the product or by the GPU tests at run time: they read only the committed outputs.
"""
import argparse
import hashlib
import json
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
from oracle import synth  # noqa: E402
from oracle.exact_oracle import h16  # noqa: E402

OUT_JSON = os.path.join(HERE, "golden.json")


def load_reference(ref):
    sys.path.insert(0, ref)
    import exact_llm as ex

    def exec_lines(rel, a, b, ns):
        with open(os.path.join(ref, rel)) as f:
            lines = f.readlines()
        exec(compile("".join(lines[a - 1:b]), f"{rel}:{a}-{b}", "exec"), ns)

    exec_lines("experiments/speed_fair_kaggle.py", 713, 725, ex.__dict__)           # G_, GQLin
    exec_lines("experiments/moe_exact_kaggle.py", 419, 424, ex.__dict__)            # SIG_T, isig
    fr_ns = dict(ex.__dict__)
    exec_lines("experiments/gpu_engine_trace_verify_kaggle.py", 782, 782, fr_ns)    # P1, P2
    exec_lines("experiments/gpu_engine_trace_verify_kaggle.py", 802, 819, fr_ns)    # rng, keys_group/channel
    exec_lines("experiments/gpu_engine_trace_verify_kaggle.py", 830, 834, fr_ns)    # fr
    ex._fr_ns = fr_ns
    ex._exec_lines = exec_lines
    return ex


# ----------------------------------------------------------------------------- reference objects
def ref_gqlin(ex, lin):
    g = ex.GQLin.__new__(ex.GQLin)
    g.w = np.ascontiguousarray(lin.w.T)                    # reference layout (K, N)
    g.M = np.ascontiguousarray(lin.M.T)                    # (G, N)
    g.groups = [(a, a + 128) for a in range(0, lin.K, 128)]
    g.b = lin.b
    return g


def ref_qlin(ex, lin):
    q = ex.QLin.__new__(ex.QLin)
    q.w = np.ascontiguousarray(lin.w.T)
    q.M = lin.M
    q.Mbits = int(ex.bitlen(np.array([q.M.max()]))[0])
    q.b = lin.b
    return q


def ref_lin(ex, lin):
    return ref_gqlin(ex, lin) if lin.kind == "group" else ref_qlin(ex, lin)


class Recorder:
    """Wraps a reference linear and records its integer accumulator (tot / acc) per call,
    the way the reference's trace capture does (gpu_engine_trace_verify_kaggle.py:746)."""

    def __init__(self, ex, inner, name, log):
        self.ex, self.inner, self.name, self.log = ex, inner, name, log

    def __call__(self, x):
        ex = self.ex
        y = self.inner(x)
        xq, s = ex.qrow(x, 15)
        if isinstance(self.inner, ex.GQLin):
            raw = np.zeros((x.shape[0], self.inner.w.shape[1]), np.int64)
            for gi, (a, b) in enumerate(self.inner.groups):
                raw += ex.exact_mm(xq[:, a:b], self.inner.w[a:b]) * self.inner.M[gi]
            chk = ex.shr(raw, 28 - s)
        else:
            raw = ex.exact_mm(xq, self.inner.w)
            q = self.inner
            drop = np.maximum(ex.bitlen(np.abs(raw).max(-1, keepdims=True)) + q.Mbits - 62, 0)
            chk = ex.shr(ex.shr(raw, drop) * q.M, 28 - s - drop)
        if self.inner.b is not None:
            chk = chk + self.inner.b
        assert np.array_equal(chk, y), "recorded accumulator does not reproduce the reference output"
        if self.log is not None:
            self.log.append((self.name, raw))
        return y


class OutRecorder:
    """Wraps a reference linear and keeps the output of its latest call.  On the K and V
    projections this gives the reference's KV cache: K = qrow(rope(k)) per (head, position) row
    with its shift, V = the Q16 projection (exact_torch.py:146-149)."""

    def __init__(self, inner):
        self.inner, self.last = inner, None

    def __call__(self, x):
        self.last = self.inner(x)
        return self.last


class RowsHead:
    """The reference head applied to selected rows only.  Every output row of QLin.__call__
    depends on its own input row alone (qrow, the product and the drop rule are per row,
    exact_llm.py:89-96), so these rows equal the same rows of the head over all positions."""

    def __init__(self, inner, rows):
        self.inner, self.rows = inner, rows

    def __call__(self, x):
        idx = [r if r >= 0 else x.shape[0] + r for r in self.rows]
        return self.inner(x[idx])


def ref_int_model(ex, om, record=None):
    c = dict(om.c)
    m = ex.IntModel.__new__(ex.IntModel)
    m.c = c
    m.emb = om.emb_i8.astype(np.float64) / 128.0          # rint(emb * 2^16) == emb_i8 << 9 exactly
    m.layers = []
    for li, L in enumerate(om.layers):
        d = dict(g1=L["g1"], g2=L["g2"])
        for nm in ("q", "k", "v", "o", "gate", "up", "down"):
            inner = ref_lin(ex, L[nm])
            d[nm] = Recorder(ex, inner, f"L{li}.{nm}", record) if record is not None else inner
        m.layers.append(d)
    m.gf = om.gf
    head = ref_qlin(ex, om.head)
    m.head = Recorder(ex, head, "head", record) if record is not None else head
    cos, sin = ex.rope_tables(c["T"], c["hd"], c["theta"])
    m.cos = np.rint(cos * ex.ONE).astype(np.int64)
    m.sin = np.rint(sin * ex.ONE).astype(np.int64)
    return m


def ref_moe_model(ex, om):
    c = dict(om.c)
    ns = dict(ex.__dict__)
    ns.update(c=c, NE=c["NE"], TOPK=c["TOPK"])
    ex._exec_lines("experiments/moe_exact_kaggle.py", 433, 482, ns)                # class MoEInt
    MoEInt = ns["MoEInt"]
    m = MoEInt.__new__(MoEInt)
    m.c = c
    m.emb = om.emb_i8.astype(np.float64) / 128.0
    m.layers = []
    for L in om.layers:
        d = dict(g1=L["g1"], g2=L["g2"])
        for nm in ("q", "k", "v", "o", "router", "sgate", "sg", "su", "sd"):
            d[nm] = ref_qlin(ex, L[nm])
        d["ex"] = [tuple(ref_qlin(ex, t) for t in e) for e in L["ex"]]
        m.layers.append(d)
    m.gf = om.gf
    m.head = ref_qlin(ex, om.head)
    cos, sin = ex.rope_tables(c["T"], c["hd"], c["theta"])
    m.cos = np.rint(cos * ex.ONE).astype(np.int64)
    m.sin = np.rint(sin * ex.ONE).astype(np.int64)
    return m


def step_digest_hex(flat):
    arr = np.ascontiguousarray(flat, dtype=np.int64)
    step = (len(arr) + 3) // 4
    parts = [hashlib.sha256(arr[i * step:(i + 1) * step].tobytes()).digest() for i in range(4)]
    return hashlib.sha256(b"".join(parts)).hexdigest()


# ----------------------------------------------------------------------------- fixture builders
def g_tables(ex, G):
    out = dict(EXP_T=h16(ex.EXP_T), SILU_T=h16(ex.SILU_T), SIG_T=h16(ex.SIG_T), rope={})
    for T, hd, th in ((4352, 64, 1e6), (4352, 128, 1e6), (4352, 64, 1e4), (64, 16, 1e4)):
        cos, sin = ex.rope_tables(T, hd, th)
        out["rope"][f"{T}_{hd}_{th:g}"] = [h16(np.rint(cos * ex.ONE).astype(np.int64)),
                                           h16(np.rint(sin * ex.ONE).astype(np.int64))]
    G["tables"] = out


def g_gemv_kat(ex, G):
    """The reference's G1 kernel known-answer test (speed_fair_kaggle.py:704-711): same seeded
    torch inputs, expected output from its own int64 expression."""
    import torch
    g = torch.Generator().manual_seed(0)
    res = []
    for K_, N_ in ((896, 896), (896, 4864), (4864, 896), (1536, 8960), (8960, 1536), (896, 151936)):
        x = torch.randint(-32767, 32768, (K_,), generator=g, dtype=torch.int64)
        w = torch.randint(-127, 128, (K_, N_), generator=g, dtype=torch.int64)
        Mg = torch.randint(1, 1 << 27, (N_, K_ // 128), generator=g, dtype=torch.int64)
        ref = ((x.view(K_ // 128, 128, 1) * w.view(K_ // 128, 128, N_)).sum(1) * Mg.T).sum(0)
        res.append(dict(K=K_, N=N_, out=h16(ref.numpy()), x=h16(x.numpy()), w=h16(w.numpy()), Mg=h16(Mg.numpy())))
    G["gemv_kat"] = res


LINEAR_SHAPES = ((3584, 4608), (3584, 3584), (3584, 37888), (18944, 3584))
LINEAR_ROWS = (1, 16, 256, 2048)


def g_linear(ex, G):
    """BASELINE config 2 through the reference GQLin at every (K, N, M)."""
    res = []
    for K, N in LINEAR_SHAPES:
        for R in LINEAR_ROWS:
            t0 = time.time()
            x, lin = synth.linear_case(1000 + K + N, K, N, R)
            rec = []
            y = Recorder(ex, ref_gqlin(ex, lin), "lin", rec)(x)
            res.append(dict(K=K, N=N, R=R, seed=1000 + K + N, y=h16(y), tot=h16(rec[0][1]),
                            y_row0=[int(v) for v in y[0, :8]], ref_s=round(time.time() - t0, 3)))
            print("linear", K, N, R, res[-1]["ref_s"], flush=True)
    G["linear"] = res


def _dense_case(ex, G, key, cfg, seed, T, steps, prompt_seed, save_npz=False):
    om = synth.build_model(cfg, seed)
    ids = [int(t) for t in synth.prompt_ids(prompt_seed, 1, T, cfg["V"])[0]]
    rec = []
    rm = ref_int_model(ex, om, rec)
    t0 = time.time()
    lg = rm(ids)
    pre_s = time.time() - t0
    n_lin = len(rec)
    prefill_trace = [(nm, raw) for nm, raw in rec]
    toks, rows_h, digests = [], [], []
    cur = list(ids)
    nxt = int(lg[-1].argmax())
    rows = []
    for t in range(steps):                                  # the reference's decode: full recompute
        toks.append(nxt)
        cur.append(nxt)
        rec.clear()
        full = rm(cur)
        row = full[-1]
        rows.append(row)
        rows_h.append(h16(row))
        # per-step flat trace = last row of every accumulator, in call order
        digests.append(step_digest_hex(np.concatenate([raw[-1] for _, raw in rec])))
        nxt = int(row.argmax())
    ent = dict(config=cfg, seed=seed, prompt=ids, prefill=h16(lg), prefill_last=h16(lg[-1]),
               tokens=toks, rows=rows_h, trace_digests=digests, n_linears=n_lin,
               prefill_trace={nm: h16(raw) for nm, raw in prefill_trace}, prefill_s=round(pre_s, 2))
    if save_npz:
        np.savez_compressed(os.path.join(HERE, f"{key}.npz"), prefill=lg, rows=np.array(rows),
                            **{f"tr_{nm}": raw for nm, raw in prefill_trace})
    G.setdefault("models", {})[key] = ent
    print(key, "prefill", h16(lg), "tokens", toks[:8], round(pre_s, 2), flush=True)
    return om, rm, ids, prefill_trace


def g_models(ex, G):
    _dense_case(ex, G, "tiny-g128", synth.config("tiny-g128"), 1, 12, 8, 3, save_npz=True)
    _dense_case(ex, G, "tiny-ch", synth.config("tiny-ch"), 2, 10, 6, 4, save_npz=True)


def g_commit(ex, G):
    """Merkle trace commitment of one full forward, computed by the reference's own prover_trace,
    leaves_of, Hb and merkle (experiments/commit_audit_kaggle.py:442-445, 567-575, 587-628) on the
    per-channel tiny model over its prompt plus its greedy tokens."""
    ns = dict(ex.__dict__)
    ex._exec_lines("experiments/commit_audit_kaggle.py", 442, 445, ns)              # requant
    ex._exec_lines("experiments/commit_audit_kaggle.py", 567, 575, ns)              # Hb, merkle
    ex._exec_lines("experiments/commit_audit_kaggle.py", 587, 628, ns)              # prover_trace, leaves_of
    cfg = synth.config("tiny-ch")
    om = synth.build_model(cfg, 2)
    g = G["models"]["tiny-ch"]
    ids = [int(t) for t in g["prompt"]] + [int(t) for t in g["tokens"]]
    rm = ref_int_model(ex, om)
    tr = ns["prover_trace"](rm, ids)
    index, leaves = ns["leaves_of"](tr, cfg["NL"])
    levels = ns["merkle"](leaves)
    G["commit"] = dict(model="tiny-ch", seed=2, ids=ids, n_leaves=len(leaves),
                       root=levels[-1][0].hex(), leaf0=leaves[0].hex(), leaf_last=leaves[-1].hex(),
                       leaf_sample={str(i): leaves[i].hex() for i in range(0, len(leaves), max(1, len(leaves) // 9))})
    print("commit root", levels[-1][0].hex(), len(leaves), flush=True)


def g_sampler(ex, G):
    """The reference's integer sampler (exact_llm.py:243-263): sample_int on seeded synthetic
    logits rows, and generate() -- seeded, temperature-scaled decode with the receipt hash chain --
    on the group-128 tiny model."""
    rng = np.random.default_rng(31)
    rows = []
    for i, (V, scale, temp, seed, pos) in enumerate([(1000, 4 << 16, 0.8, 12345, 0), (1000, 1 << 16, 1.0, 7, 3),
                                                     (4099, 12 << 16, 0.6, 2**63 + 5, 17),
                                                     (151936, 6 << 16, 0.8, 12345, 1), (50, 40 << 16, 1.7, 0, 9)]):
        lg = rng.integers(-scale, scale, V).astype(np.int64)
        tnum = ex.temp_num(temp)
        tok, p = ex.sample_int(lg, seed, pos, tnum)
        rows.append(dict(V=V, scale=scale, temp=temp, tnum=tnum, seed=seed, pos=pos, rng_index=i,
                         token=tok, p=h16(p), u20=int(ex.u20(seed, pos))))
    g = G["models"]["tiny-g128"]
    om = synth.build_model(synth.config("tiny-g128"), g["seed"])
    rm = ref_int_model(ex, om)
    receipt, greedy = ex.generate(rm, g["prompt"], 8, 12345, 0.8)
    G["sampler"] = dict(rows=rows, rows_seed=31, receipt=receipt, greedy=greedy, model="tiny-g128",
                        model_seed=g["seed"])
    print("sampler", receipt["tokens"], receipt["chain"], greedy, flush=True)


def g_convert(ex, G):
    """float64 checkpoint -> integer release, by the reference's own QLin / qlin_chunked / GQLin and
    IntModel (exact_llm.py:83-88, 133-157; experiments/group128_quality_kaggle.py:406-414), on a
    seeded float stand-in; logits of the converted per-channel model on 16 ids."""
    c = dict(synth.CONVERT_CFG)
    f = synth.float_checkpoint(c, 41)
    ns = dict(ex.__dict__)
    ns["G"] = 128                                    # group size set at experiments/group128_quality_kaggle.py:405
    ex._exec_lines("experiments/group128_quality_kaggle.py", 406, 414, ns)           # GQLin constructor
    GQ = ns["GQLin"]
    mats = {}
    for nm in ("model.layers.0.self_attn.q_proj", "model.layers.1.mlp.down_proj", "model.layers.0.mlp.gate_proj"):
        w = f[nm + ".weight"]
        b = f.get(nm + ".bias")
        q = ex.qlin_chunked(w, b, chunk=100)                  # row blocks: identical to one shot
        g = GQ(w, b)
        mats[nm] = dict(ch_w=h16(np.ascontiguousarray(q.w.T)), ch_M=h16(q.M), b=None if b is None else h16(q.b),
                        g_w=h16(np.ascontiguousarray(g.w.T)), g_M=h16(np.ascontiguousarray(g.M.T)))
    m = ex.IntModel(f.__getitem__, c)
    ids = [int(t) for t in synth.prompt_ids(5, 1, 16, c["V"])[0]]
    lg = m(ids)
    G["convert"] = dict(config=c, seed=41, mats=mats, ids=ids, logits=h16(lg), emb_q16=h16(np.rint(m.emb * ex.ONE)
                                                                                       .astype(np.int64)))
    print("convert", h16(lg), flush=True)


def g_verify(ex, G):
    """Weightless cell verification, by the reference's own make_verifier, prover_trace, Prover,
    needed and verify_cell (experiments/commit_audit_kaggle.py:440-445, 460-512, 567-705) on the
    per-channel tiny model: every honest cell, lying openings, a cheating down projection at one
    layer and consistent fake attention at one layer (the reference's audit gates A1, A5, A2, A3)."""
    ns = dict(ex.__dict__)
    ns["P1"], ns["P2"] = 2147483647, 2147483629
    ex._exec_lines("experiments/commit_audit_kaggle.py", 442, 445, ns)              # requant
    ex._exec_lines("experiments/commit_audit_kaggle.py", 460, 512, ns)              # VER, VLin, VEmb, make_verifier
    ex._exec_lines("experiments/commit_audit_kaggle.py", 567, 705, ns)              # Hb .. verify_cell
    cfg = synth.config("tiny-ch")
    om = synth.build_model(cfg, 2)
    rm = ref_int_model(ex, om)
    ids = [int(t) for t in G["commit"]["ids"]]
    NL, T = cfg["NL"], len(ids)
    vm, _, _ = ns["make_verifier"](rm)
    keys = {"head_d": [h16(d) for _, _, d in vm.head.keys], "emb_de": [h16(de) for _, _, de in vm.emb.keys],
            "L1.down_d": [h16(d) for _, _, d in vm.layers[1]["down"].keys]}
    out = []
    pv = ns["Prover"](ns["prover_trace"](rm, ids), NL)
    for L in range(NL + 1):
        for t in range(T):
            ok, why = ns["verify_cell"](vm, cfg, pv.root, pv.index, (L, t), pv.open(ns["needed"]((L, t), NL)), ids)
            out.append(dict(scenario="honest", cell=[L, t], ok=bool(ok), why=why))
    rng = np.random.default_rng(11)
    for _ in range(8):
        cell = (int(rng.integers(NL + 1)), int(rng.integers(T)))
        names = ns["needed"](cell, NL)
        lie = names[int(rng.integers(len(names)))]
        ok, why = ns["verify_cell"](vm, cfg, pv.root, pv.index, cell, pv.open(names, lie=lie), ids)
        out.append(dict(scenario="lie", cell=list(cell), lie=[lie[0], lie[1], lie[2]], ok=bool(ok), why=why))
    dn = rm.layers[1]["down"]                           # cheating down projection: 7-bit weights
    cheat = ex.QLin.__new__(ex.QLin)
    cheat.w = np.clip(np.rint(dn.w / 2.0), -63, 63).astype(np.int8)
    cheat.M = dn.M * 2
    cheat.Mbits = int(ex.bitlen(np.array([cheat.M.max()]))[0])
    cheat.b = None
    ns["CHEAT_DOWN"] = cheat
    pc = ns["Prover"](ns["prover_trace"](rm, ids, cheat_layer=1), NL)
    for L in range(NL + 1):
        for t in (0, 5, 15):
            ok, why = ns["verify_cell"](vm, cfg, pc.root, pc.index, (L, t), pc.open(ns["needed"]((L, t), NL)), ids)
            out.append(dict(scenario="cheat", cell=[L, t], ok=bool(ok), why=why))

    def fakefn(p):
        p = p.copy()
        for row in range(max(1, p.shape[0] // 2), p.shape[0]):
            a0, a1 = int(p[row, 0]), int(p[row, row])
            p[row, 0], p[row, row] = a1, a0
        return p
    pf = ns["Prover"](ns["prover_trace"](rm, ids, fake=(1, fakefn)), NL)
    for t in (2, 7, 8, 12, 15):
        ok, why = ns["verify_cell"](vm, cfg, pf.root, pf.index, (1, t), pf.open(ns["needed"]((1, t), NL)), ids)
        out.append(dict(scenario="fake", cell=[1, t], ok=bool(ok), why=why))
    G["verify"] = dict(model="tiny-ch", seed=2, ids=ids, keys=keys, cells=out,
                       cheat=dict(layer=1, rule="w = clip(rint(w / 2), -63, 63), M = 2 M"),
                       fake=dict(layer=1, rule="rows >= T/2 swap p[row, 0] and p[row, row]"))
    bad = [(o["scenario"], o["cell"], o["why"]) for o in out if not o["ok"]]
    print("verify", len(out), "cells;", len(bad), "rejected:", bad[:12], flush=True)


def g_config1(ex, G):
    """0.5B architecture, 32 prompt ids, 64 greedy steps (reference full recompute)."""
    _dense_case(ex, G, "qwen2.5-0.5b", synth.config("qwen2.5-0.5b"), 5, 32, 64, 5)


def g_big_layers(ex, G):
    """7B / 14B shapes with reduced depth (every kernel shape of configs 3 and 5)."""
    _dense_case(ex, G, "qwen2.5-7b-L2", synth.config("qwen2.5-7b", NL=2), 7, 8, 3, 7)
    _dense_case(ex, G, "qwen2.5-14b-L1", synth.config("qwen2.5-14b", NL=1), 14, 6, 2, 14)


def g_freivalds(ex, G):
    """Reference keys (rng seeded 2026, in layer/linear order) for tiny-g128; honest trace passes,
    a +-1 or +p tamper fails (gpu_engine_trace_verify_kaggle.py:802-872)."""
    cfg = synth.config("tiny-g128")
    om = synth.build_model(cfg, 1)
    rec = []
    rm = ref_int_model(ex, om, rec)
    ids = [int(t) for t in synth.prompt_ids(3, 1, 12, cfg["V"])[0]]
    rm(ids)
    fr_ns = dict(ex._fr_ns)
    fr_ns["rng"] = np.random.default_rng(2026)
    keys = {}
    for li, L in enumerate(rm.layers):
        for nm in ("q", "k", "v", "o", "gate", "up", "down"):
            keys[f"L{li}.{nm}"] = fr_ns["keys_group"](L[nm].inner)
    keys["head"] = fr_ns["keys_channel"](rm.head.inner)
    ent = {}
    for nm, ks in keys.items():
        ent[nm] = [dict(p=int(p), r=h16(r), d=h16(d)) for p, r, d in ks]
    G["freivalds"] = dict(keys=ent, model="tiny-g128", seed=1, prompt=ids)
    np.savez_compressed(os.path.join(HERE, "freivalds_tiny.npz"),
                        **{f"{nm}|{i}|r": k[1] for nm, ks in keys.items() for i, k in enumerate(ks)},
                        **{f"{nm}|{i}|d": k[2] for nm, ks in keys.items() for i, k in enumerate(ks)})


def g_pre_tiny(ex, G):
    """The reference's own tiny fixture (experiments/_pre_tiny.py), float -> int conversion by
    the reference's QLin; its hash for windows[0][:32] pins conversion + forward."""
    ns = dict(ex.__dict__)
    ex._exec_lines("experiments/_pre_tiny.py", 1, 15, ns)
    get, c, windows = ns["get"], ns["c"], ns["windows"]
    m = ex.IntModel(get, c)
    ids = windows[0][:32]
    lg = m(ids)
    arrs = dict(emb=np.asarray(get("model.embed_tokens.weight"), np.float64), gf=m.gf, head_w=m.head.w,
                head_M=m.head.M, ids=np.array(ids), logits=lg)
    for li, L in enumerate(m.layers):
        arrs[f"L{li}.g1"], arrs[f"L{li}.g2"] = L["g1"], L["g2"]
        for nm in ("q", "k", "v", "o", "gate", "up", "down"):
            arrs[f"L{li}.{nm}.w"] = L[nm].w
            arrs[f"L{li}.{nm}.M"] = L[nm].M
            if L[nm].b is not None:
                arrs[f"L{li}.{nm}.b"] = L[nm].b
    np.savez_compressed(os.path.join(HERE, "pre_tiny.npz"), **arrs)
    G["pre_tiny"] = dict(config=c, logits=h16(lg), ids=[int(t) for t in ids])
    print("pre_tiny", h16(lg), flush=True)


def g_moe(ex, G):
    for key, cfg, seed, T, steps in (("tiny-moe", synth.config("tiny-moe"), 3, 10, 4, ),
                                     ("qwen1.5-moe-L1", synth.config("qwen1.5-moe-a2.7b", NL=1), 4, 8, 2)):
        om = synth.build_model(cfg, seed)
        rm = ref_moe_model(ex, om)
        ids = [int(t) for t in synth.prompt_ids(seed, 1, T, cfg["V"])[0]]
        st = {}
        lg = rm(ids, st)
        sels = {str(k): np.concatenate(v).tolist() for k, v in st.items()}
        cur = list(ids)
        toks, rows_h = [], []
        nxt = int(lg[-1].argmax())
        for _ in range(steps):
            toks.append(nxt)
            cur.append(nxt)
            row = rm(cur)[-1]
            rows_h.append(h16(row))
            nxt = int(row.argmax())
        G.setdefault("moe", {})[key] = dict(config=cfg, seed=seed, prompt=ids, prefill=h16(lg), sel=sels,
                                            tokens=toks, rows=rows_h)
        print(key, h16(lg), toks, flush=True)


def _kv_hashes(ex, rm, li, T):
    """Hashes of the reference KV cache of layer li over T positions, from the K and V
    projection outputs of the latest call that covered all T rows (block_row projects k and v
    for every position of its input, exact_llm.py:339-348): kq, sk = qrow(rope(k)) per (KV head,
    position) row, v as it is (exact_torch.py:146-149)."""
    c = rm.c
    KV, hd = c["KV"], c["hd"]
    k = rm.layers[li]["k"].last
    v = rm.layers[li]["v"].last
    assert k.shape[0] == T and v.shape[0] == T
    kr = rm.rope(k.reshape(T, KV, hd).transpose(1, 0, 2))
    kq = np.empty_like(kr)
    sk = np.empty((KV, T, 1), np.int64)
    for kh in range(KV):
        kq[kh], sk[kh] = ex.qrow(kr[kh])
    return dict(k=h16(kq), sk=h16(sk), v=h16(np.ascontiguousarray(v.reshape(T, KV, hd).transpose(1, 0, 2))),
                k_row0=[int(t) for t in kq[0, 0, :8]], sk_head0=[int(t) for t in sk[0, :8, 0]])


def _long_case(ex, G, key, cfg, seed, T, steps, prompt_seed, rows):
    """Long-prompt parity by the reference's own per-layer machinery: forward_record over the
    prompt (exact_llm.py:359-363, every layer input x_l of every position), the head on the
    selected rows, then greedy decode where each new position runs block_row through every layer
    (exact_llm.py:339-358) on the layer inputs of all earlier positions -- the same rows a full
    recompute of the extended prompt gives, since every layer is causal.  Records hashes of the
    selected prefill rows, the tokens, every decode row and the KV cache of every layer."""
    om = synth.build_model(cfg, seed)
    rm = ref_int_model(ex, om)
    for L in rm.layers:
        L["k"], L["v"] = OutRecorder(L["k"]), OutRecorder(L["v"])
    head = rm.head
    rm.head = RowsHead(head, rows)
    ids = [int(t) for t in synth.prompt_ids(prompt_seed, 1, T, cfg["V"])[0]]
    t0 = time.time()
    xs, lg = ex.forward_record(rm, ids)
    pre_s = time.time() - t0
    print(key, "prefill", round(pre_s, 1), "s", flush=True)
    xs = [np.array(x) for x in xs]
    toks, rows_h, row8 = [], [], []
    nxt = int(lg[-1].argmax()) if rows[-1] == -1 else None
    assert nxt is not None, "the last selected row must be the prompt's last row (the greedy token)"
    cur = list(ids)
    for s in range(steps):
        toks.append(nxt)
        cur.append(nxt)
        t = len(cur) - 1
        x = np.rint(np.asarray(rm.emb[[nxt]], dtype=np.float64) * ex.ONE).astype(np.int64)
        xs[0] = np.concatenate([xs[0], x])
        for li, L in enumerate(rm.layers):
            xn = ex.block_row(rm, L, xs[li], t)
            xs[li + 1] = np.concatenate([xs[li + 1], xn[None]])
        row = head(ex.irms(xs[-1][t:t + 1], rm.gf))[0]
        rows_h.append(h16(row))
        row8.append([int(v) for v in row[:8]])
        nxt = int(row.argmax())
        print(key, "step", s, nxt, round(time.time() - t0, 1), flush=True)
    S = len(cur)
    kv = [_kv_hashes(ex, rm, li, S) for li in range(cfg["NL"])]
    ent = dict(config=cfg, seed=seed, prompt_seed=prompt_seed, T=T, prompt=ids, rows=rows, prefill_all=h16(lg),
               prefill_rows=[h16(r) for r in lg] if len(rows) <= 16 else None, prefill_last8=[int(v) for v in lg[-1][:8]],
               tokens=toks, step_rows=rows_h, step_row8=row8, kv=kv, S=S, prefill_s=round(pre_s, 1),
               x_last=[h16(x[-1]) for x in xs])
    G.setdefault("long", {})[key] = ent
    print(key, "tokens", toks, "kv0", kv[0]["k"], flush=True)


def g_long(ex, G):
    """BASELINE configs 3 and 5 at their real prompt lengths: the 7B architecture (2 layers) after a
    512-token prompt (every prefill row, 4 decode steps) and the 14B architecture (1 layer) after a
    4096-token prompt (rows 999, 2047, 3000 and the last 8; 3 decode steps)."""
    _long_case(ex, G, "qwen2.5-7b-L2-p512", synth.config("qwen2.5-7b", NL=2), 71, 512, 4, 72,
               list(range(-512, 0)))
    _long_case(ex, G, "qwen2.5-14b-L1-p4096", synth.config("qwen2.5-14b", NL=1), 141, 4096, 3, 142,
               [999, 2047, 3000] + list(range(-8, 0)))


def g_moe_wide(ex, G):
    """BASELINE config 4's workload shape on one Qwen1.5-MoE layer: 32 sequences of 256 uniform
    prompt tokens, the router's top-4 experts of every token (MoEInt.moe, experiments/
    moe_exact_kaggle.py:454-467), the last prompt row's logits and 3 greedy steps per sequence
    (the reference's full recompute per step)."""
    cfg = synth.config("qwen1.5-moe-a2.7b", NL=1)
    seed, B, T, steps = 43, 32, 256, 3
    om = synth.build_model(cfg, seed)
    rm = ref_moe_model(ex, om)
    head = rm.head
    rm.head = RowsHead(head, [-1])
    prompts = synth.prompt_ids(44, B, T, cfg["V"])
    seqs = []
    t0 = time.time()
    for b in range(B):
        ids = [int(t) for t in prompts[b]]
        st = {}
        lg = rm(ids, st)
        sel = np.concatenate(st[0]).astype(np.int64)
        cur = list(ids)
        toks, rows_h = [], []
        nxt = int(lg[-1].argmax())
        for _ in range(steps):
            toks.append(nxt)
            cur.append(nxt)
            row = rm(cur)[-1]
            rows_h.append(h16(row))
            nxt = int(row.argmax())
        seqs.append(dict(last=h16(lg[-1]), sel=h16(sel), sel_head=sel[:4].tolist(), tokens=toks, rows=rows_h))
        print("moe-wide", b, toks, round(time.time() - t0, 1), flush=True)
    G["moe_wide"] = dict(config=cfg, seed=seed, prompt_seed=44, B=B, T=T, steps=steps, seqs=seqs)


def g_freivalds_7b(ex, G):
    """Freivalds keys at the 7B architecture's shapes (2 layers): the reference's keys_group /
    keys_channel (experiments/gpu_engine_trace_verify_kaggle.py:802-819, rng seeded 2026, drawn
    in layer / linear order, then the head), hashed per linear and prime."""
    cfg = synth.config("qwen2.5-7b", NL=2)
    om = synth.build_model(cfg, 7)
    rm = ref_int_model(ex, om)
    fr_ns = dict(ex._fr_ns)
    fr_ns["rng"] = np.random.default_rng(2026)
    ent = {}
    t0 = time.time()
    for li, L in enumerate(rm.layers):
        for nm in ("q", "k", "v", "o", "gate", "up", "down"):
            ent[f"L{li}.{nm}"] = [h16(d) for _, _, d in fr_ns["keys_group"](L[nm])]
            print("fr7b", li, nm, round(time.time() - t0, 1), flush=True)
    ent["head"] = [h16(d) for _, _, d in fr_ns["keys_channel"](rm.head)]
    G["freivalds_7b"] = dict(model="qwen2.5-7b-L2", seed=7, d=ent)


BUILDERS = dict(tables=g_tables, gemv_kat=g_gemv_kat, models=g_models, freivalds=g_freivalds,
                pre_tiny=g_pre_tiny, moe=g_moe, linear=g_linear, config1=g_config1, big=g_big_layers,
                commit=g_commit, sampler=g_sampler, convert=g_convert, verify=g_verify, long=g_long,
                moe_wide=g_moe_wide, freivalds_7b=g_freivalds_7b)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="path of the exact-llm reference checkout")
    ap.add_argument("--only", nargs="*", default=None)
    a = ap.parse_args()
    ex = load_reference(a.ref)
    G = json.load(open(OUT_JSON)) if os.path.exists(OUT_JSON) else {}
    for name, fn in BUILDERS.items():
        if a.only and name not in a.only:
            continue
        t0 = time.time()
        fn(ex, G)
        print(f"[{name}] {time.time() - t0:.1f}s", flush=True)
        with open(OUT_JSON, "w") as f:
            json.dump(G, f, indent=1, sort_keys=True)


if __name__ == "__main__":
    main()
