"""Pin the numpy oracle to fixtures recorded by running the reference's own code
(tests/golden/make_golden.py).  CPU only."""
import os

import numpy as np
import pytest

from oracle import exact_oracle as eo
from oracle import synth
from tests.conftest import GOLDEN_DIR


def test_tables_match_reference(golden):
    g = golden["tables"]
    assert eo.h16(eo.EXP_T) == g["EXP_T"]
    assert eo.h16(eo.SILU_T) == g["SILU_T"]
    assert eo.h16(eo.SIG_T) == g["SIG_T"]
    for key, (hc, hs) in g["rope"].items():
        T, hd, th = key.split("_")
        cos, sin = eo.rope_tables(int(T), int(hd), float(th))
        assert eo.h16(cos) == hc and eo.h16(sin) == hs, key


def test_package_tables_match_reference(golden):
    """The product's host-side tables are the reference's tables, bit for bit."""
    from exact_llm_b200 import tables
    g = golden["tables"]
    assert eo.h16(tables.exp_table()) == g["EXP_T"]
    assert eo.h16(tables.silu_table()) == g["SILU_T"]
    assert eo.h16(tables.sig_table()) == g["SIG_T"]
    for key, (hc, hs) in g["rope"].items():
        T, hd, th = key.split("_")
        cos, sin = tables.rope_tables(int(T), int(hd), float(th))
        assert eo.h16(cos) == hc and eo.h16(sin) == hs, key
    assert tables.inv_scale(64) == 8192 and tables.inv_scale(128) == 5793 and tables.inv_scale(16) == 16384


def test_gemv_known_answer(golden):
    """The reference's G1 kernel test vectors (speed_fair_kaggle.py:704-711) through the oracle."""
    import torch
    g = torch.Generator().manual_seed(0)
    for case in golden["gemv_kat"]:
        K, N = case["K"], case["N"]
        x = torch.randint(-32767, 32768, (K,), generator=g, dtype=torch.int64).numpy()
        w = torch.randint(-127, 128, (K, N), generator=g, dtype=torch.int64).numpy()
        Mg = torch.randint(1, 1 << 27, (N, K // 128), generator=g, dtype=torch.int64).numpy()
        assert eo.h16(x) == case["x"] and eo.h16(Mg) == case["Mg"]
        if N > 20000:
            continue                                    # the 896 x 151936 case is checked on the GPU only
        lin = eo.GroupLinear(w.T.astype(np.int8), Mg)
        assert eo.h16(lin.raw(x[None])[0]) == case["out"], (K, N)


@pytest.mark.parametrize("R", [1, 16])
def test_linear_config2_small_rows(golden, R):
    for case in golden["linear"]:
        if case["R"] != R or case["N"] > 4608:          # larger shapes: GPU tests and the slow CPU test
            continue
        x, lin = synth.linear_case(case["seed"], case["K"], case["N"], R)
        tot = lin.raw(eo.qrow(x)[0])
        y = lin(x)
        assert eo.h16(tot) == case["tot"] and eo.h16(y) == case["y"], (case["K"], case["N"], R)


def _dense(golden, key):
    g = golden["models"][key]
    c = dict(g["config"])
    om = synth.build_model(c, g["seed"])
    return g, om


@pytest.mark.parametrize("key", ["tiny-g128", "tiny-ch"])
def test_tiny_models(golden, key):
    g, om = _dense(golden, key)
    ref = np.load(os.path.join(GOLDEN_DIR, f"{key}.npz"))
    trace = []
    lg = om(g["prompt"], trace=trace)
    assert np.array_equal(lg, ref["prefill"])
    assert eo.h16(lg) == g["prefill"]
    for name, raw, _ in trace:
        assert eo.h16(raw) == g["prefill_trace"][name], name
    pre, rows, toks = eo.greedy_generate(om, g["prompt"], len(g["tokens"]))
    assert toks == g["tokens"]
    assert [eo.h16(r) for r in rows] == g["rows"]
    assert np.array_equal(np.array(rows), ref["rows"])


def test_tiny_decode_trace_digests(golden):
    """Per-step flat trace (all accumulators of the new row, call order) -> 4-way SHA-256 digest
    (prover_commit_cost_gpu_kaggle.py:811-817)."""
    g, om = _dense(golden, "tiny-g128")
    cache = om.new_cache()
    lg = om.forward(g["prompt"], cache)
    nxt = int(lg[-1].argmax())
    for step, want in enumerate(g["trace_digests"]):
        tr = []
        row = om.forward([nxt], cache, trace=tr)[0]
        flat = np.concatenate([raw[-1] for _, raw, _ in tr])
        assert eo.step_digest(flat).hex() == want, step
        nxt = int(row.argmax())


def test_pre_tiny_reference_fixture(golden):
    """The reference's own tiny model (experiments/_pre_tiny.py), converted by its QLin."""
    z = np.load(os.path.join(GOLDEN_DIR, "pre_tiny.npz"))
    c = dict(golden["pre_tiny"]["config"])
    layers = []
    for i in range(c["NL"]):
        L = dict(g1=z[f"L{i}.g1"], g2=z[f"L{i}.g2"])
        for nm in eo.LIN_NAMES:
            b = z[f"L{i}.{nm}.b"] if f"L{i}.{nm}.b" in z else None
            L[nm] = eo.ChannelLinear(z[f"L{i}.{nm}.w"].T, z[f"L{i}.{nm}.M"], b)
        layers.append(L)
    head = eo.ChannelLinear(z["head_w"].T, z["head_M"])
    emb = z["emb"]
    cos, sin = eo.rope_tables(c["T"], c["hd"], c["theta"])
    om = eo.OracleModel(c, layers, z["gf"], head, lambda ids: np.rint(emb[ids] * eo.ONE).astype(np.int64), cos, sin)
    lg = om(golden["pre_tiny"]["ids"])
    assert eo.h16(lg) == golden["pre_tiny"]["logits"] == "eb3c5426052399f8"
    # the oracle's float -> int conversion reproduces the reference's QLin (head = tied embedding)
    q = eo.quantize_channel(emb)
    assert np.array_equal(q.w, z["head_w"].T) and np.array_equal(q.M, z["head_M"])


def test_freivalds_keys_match_reference(golden):
    g = golden["freivalds"]
    _, om = _dense(golden, "tiny-g128")
    lins = [L[nm] for L in om.layers for nm in eo.LIN_NAMES] + [om.head]
    names = [f"L{i}.{nm}" for i in range(len(om.layers)) for nm in eo.LIN_NAMES] + ["head"]
    rs = eo.draw_keys(lins, 2026)
    trace = []
    om(g["prompt"], trace=trace)
    by_name = {nm: (raw, xq) for nm, raw, xq in trace}
    for nm, lin, r in zip(names, lins, rs):
        keys = eo.freivalds_key(lin, r)
        for (p, rr, d), want in zip(keys, g["keys"][nm]):
            assert p == want["p"] and eo.h16(rr) == want["r"] and eo.h16(d) == want["d"], nm
        raw, xq = by_name[nm]
        assert eo.freivalds_check(keys, xq, raw), nm
        bad = raw.copy()
        bad[0, 0] += 1
        assert not eo.freivalds_check(keys, xq, bad), nm
        bad = raw.copy()
        bad[-1, -1] += eo.P1
        assert not eo.freivalds_check(keys, xq, bad), nm


@pytest.mark.slow
def test_linear_config2_all_shapes(golden):
    for case in golden["linear"]:
        if case["R"] > 256:
            continue
        x, lin = synth.linear_case(case["seed"], case["K"], case["N"], case["R"])
        assert eo.h16(lin(x)) == case["y"], (case["K"], case["N"], case["R"])


@pytest.mark.parametrize("key", ["tiny-moe", pytest.param("qwen1.5-moe-L1", marks=pytest.mark.slow)])
def test_moe_models(golden, key):
    g = golden["moe"][key]
    c = dict(g["config"])
    om = synth.build_model(c, g["seed"])
    stats = {}
    lg = om(g["prompt"], stats=stats)
    assert eo.h16(lg) == g["prefill"]
    for li, sel in g["sel"].items():
        assert np.array_equal(np.concatenate(stats[int(li)]), np.array(sel)), li
    pre, rows, toks = eo.greedy_generate(om, g["prompt"], len(g["tokens"]))
    assert toks == g["tokens"] and [eo.h16(r) for r in rows] == g["rows"]


def test_commit_root_matches_reference(golden):
    """The Merkle trace commitment restated in the oracle (X, accumulators, roped K/V and head
    leaves, L/N-prefixed SHA-256 tree) reproduces the root the reference's own prover_trace,
    leaves_of and merkle computed on the same integers."""
    g = golden["commit"]
    cfg = synth.config(g["model"])
    om = synth.build_model(cfg, g["seed"])
    tr = eo.commit_trace(om, g["ids"])
    leaves = eo.commit_leaves(tr, cfg["NL"])
    assert len(leaves) == g["n_leaves"] == (5 * cfg["NL"] + 2) * len(g["ids"])
    assert leaves[0].hex() == g["leaf0"] and leaves[-1].hex() == g["leaf_last"]
    for i, h in g["leaf_sample"].items():
        assert leaves[int(i)].hex() == h
    assert eo.merkle_root(leaves).hex() == g["root"]


def test_sampler_matches_reference(golden):
    """Integer sampler (splitmix64 / u20 / isoftmax_row / sample_int) and the seeded decode with
    its receipt chain reproduce the reference's own outputs."""
    g = golden["sampler"]
    rng = np.random.default_rng(g["rows_seed"])
    for row in g["rows"]:
        lg = rng.integers(-row["scale"], row["scale"], row["V"]).astype(np.int64)
        assert eo.temp_num(row["temp"]) == row["tnum"]
        assert eo.u20(row["seed"], row["pos"]) == row["u20"]
        tok, p = eo.sample_int(lg, row["seed"], row["pos"], row["tnum"])
        assert tok == row["token"] and eo.h16(p) == row["p"]
    om = synth.build_model(synth.config(g["model"]), g["model_seed"])
    r = g["receipt"]
    receipt, greedy = eo.sampled_generate(om, r["prompt"], len(r["tokens"]), r["seed"], r["temp"])
    assert receipt == r and greedy == g["greedy"]


def _verify_scenarios(g):
    """(model, ids, NL, traces by scenario) for the weightless-verifier fixture."""
    cfg = synth.config(g["model"])
    om = synth.build_model(cfg, g["seed"])
    ids = g["ids"]
    dn = om.layers[g["cheat"]["layer"]]["down"]
    cheat = eo.ChannelLinear(np.clip(np.rint(dn.w / 2.0), -63, 63).astype(np.int8), dn.M * 2)

    def fakefn(p):
        p = p.copy()
        for row in range(max(1, p.shape[0] // 2), p.shape[0]):
            a0, a1 = int(p[row, 0]), int(p[row, row])
            p[row, 0], p[row, row] = a1, a0
        return p
    trs = {"honest": eo.commit_trace(om, ids),
           "cheat": eo.commit_trace(om, ids, cheat_layer=g["cheat"]["layer"], cheat_down=cheat),
           "fake": eo.commit_trace(om, ids, fake=(g["fake"]["layer"], fakefn))}
    trs["lie"] = trs["honest"]
    return om, ids, cfg["NL"], trs


def test_weightless_verifier_matches_reference(golden):
    """The verifier restatement (keys, Merkle openings, Freivalds rows, recomputed cell) gives the
    reference's verdict and reason on every honest, lying, cheating and fake-attention cell."""
    g = golden["verify"]
    om, ids, NL, trs = _verify_scenarios(g)
    keys = eo.verifier_keys(om)
    assert [eo.h16(d) for _, _, d in keys["head"]] == g["keys"]["head_d"]
    assert [eo.h16(de) for _, _, de in keys["emb"]] == g["keys"]["emb_de"]
    assert [eo.h16(d) for _, _, d in keys["layers"][1]["down"]] == g["keys"]["L1.down_d"]
    T = len(ids)
    levels = {k: eo.merkle_levels(eo.commit_leaves(tr, NL)) for k, tr in trs.items()}
    for case in g["cells"]:
        sc = case["scenario"]
        cell = tuple(case["cell"])
        lie = tuple(case["lie"]) if "lie" in case else None
        opened = eo.open_cell(trs[sc], NL, levels[sc], cell, lie=lie)
        ok, why = eo.verify_cell(om, keys, levels[sc][-1][0], T, cell, opened, ids)
        assert (ok, why) == (case["ok"], case["why"]), case


@pytest.mark.slow
@pytest.mark.parametrize("key", ["qwen2.5-7b-L2-p512", "qwen2.5-14b-L1-p4096"])
def test_long_prompt_fixtures(golden, key):
    """The oracle's KV-cache path (prefill, then one row per decode step) against the long-prompt
    fixtures the reference recorded with forward_record + block_row: the selected prefill rows,
    the tokens, every decode row and the layer-0 KV cache.  About 1 min (7B) / 15 min (14B)."""
    g = golden["long"][key]
    om = synth.build_model(dict(g["config"]), g["seed"])
    cache = om.new_cache()
    T = g["T"]
    rows = g["rows"]
    lg = om.forward(g["prompt"], cache)
    if g["prefill_rows"] is not None:
        assert [eo.h16(lg[r]) for r in rows] == g["prefill_rows"]
    else:
        assert eo.h16(lg) == g["prefill_all"]
    nxt = int(lg[-1].argmax())
    for s, tok in enumerate(g["tokens"]):
        assert tok == nxt, s
        row = om.forward([tok], cache)[0]
        assert eo.h16(row) == g["step_rows"][s], s
        nxt = int(row.argmax())
    kq, sk, v = cache["layers"][0]
    assert cache["n"] == g["S"] == T + len(g["tokens"])
    assert [eo.h16(kq), eo.h16(sk), eo.h16(v)] == [g["kv"][0]["k"], g["kv"][0]["sk"], g["kv"][0]["v"]]
