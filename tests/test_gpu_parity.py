"""CUDA path vs the reference: bit-exact parity through the C ABI (needs a B200).

Every expected value here was recorded from the reference's own code (tests/golden) or is
computed by the numpy oracle, which those fixtures pin."""
import ctypes
import os

import numpy as np
import pytest

from oracle import exact_oracle as eo
from oracle import synth
from tests.conftest import GOLDEN_DIR
from tests.helpers import oracle_tensors

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch_cuda(cuda_ok):
    import torch
    return torch


def _lib():
    from exact_llm_b200 import _lib
    return _lib


def _stream(torch):
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


# ------------------------------------------------------------------ operator level
def test_gemv_known_answer(golden, torch_cuda):
    """The reference's own G1 kernel test (experiments/speed_fair_kaggle.py:704-711), all six shapes."""
    torch = torch_cuda
    L = _lib()
    g = torch.Generator().manual_seed(0)
    for case in golden["gemv_kat"]:
        K, N = case["K"], case["N"]
        x = torch.randint(-32767, 32768, (K,), generator=g, dtype=torch.int64)
        w = torch.randint(-127, 128, (K, N), generator=g, dtype=torch.int64)
        Mg = torch.randint(1, 1 << 27, (N, K // 128), generator=g, dtype=torch.int64)
        ref = ((x.view(K // 128, 128, 1) * w.view(K // 128, 128, N)).sum(1) * Mg.T).sum(0)
        xd = x.to(torch.int16).cuda()
        wd = w.to(torch.int8).T.contiguous().cuda()
        Md = Mg.cuda()
        out = torch.empty(N, dtype=torch.int64, device="cuda")
        L.check(L.lib.exb_gemv(L.ptr(xd), L.ptr(wd), L.ptr(Md), K, N, L.ptr(out), _stream(torch)))
        got = out.cpu()
        assert torch.equal(got, ref), (K, N)
        assert eo.h16(got.numpy()) == case["out"]


def _gen(torch, kind, seed, stream, n, K, dtype):
    L = _lib()
    out = torch.empty(n, dtype=dtype, device="cuda")
    L.check(L.lib.exb_gen_tensor(kind, seed, stream, n, K, L.ptr(out), _stream(torch)))
    return out


def test_device_generator_matches_oracle(torch_cuda):
    torch = torch_cuda
    for kind, fn, dt, K in ((0, lambda: synth.gen_weight(5, 77, 300, 256).reshape(-1), torch.int8, 256),
                            (1, lambda: synth.gen_scale(5, 78, 999, 3584), torch.int32, 3584),
                            (2, lambda: synth.gen_scale(5, 79, 999, 896), torch.int64, 896),
                            (3, lambda: synth.gen_bias(5, 80, 777), torch.int64, 0),
                            (4, lambda: synth.gen_gain(5, 81, 777), torch.int64, 0)):
        want = fn()
        got = _gen(torch, kind, 5, 77 + kind, want.size, K, dt).cpu().numpy()
        assert np.array_equal(got.astype(np.int64), want.astype(np.int64)), kind


@pytest.mark.parametrize("K,N", [(3584, 4608), (3584, 3584), (3584, 37888), (18944, 3584)])
def test_linear_config2(golden, torch_cuda, K, N):
    """exact int8 x int8 linear with group-128 requant at M in {1, 16, 256, 2048},
    against hashes of the reference GQLin's outputs."""
    torch = torch_cuda
    L = _lib()
    cases = [c for c in golden["linear"] if c["K"] == K and c["N"] == N]
    assert len(cases) == 4
    seed = cases[0]["seed"]
    w = _gen(torch, 0, seed, 7, N * K, K, torch.int8)
    M = _gen(torch, 1, seed, 8, N * (K // 128), K, torch.int32)
    for case in cases:
        R = case["R"]
        x = torch.from_numpy(np.random.default_rng(seed).integers(-128, 128, (R, K)).astype(np.int64)).cuda()
        y = torch.empty((R, N), dtype=torch.int64, device="cuda")
        tot = torch.empty((R, N), dtype=torch.int64, device="cuda")
        scratch = torch.empty(L.lib.exb_linear_g128_scratch_bytes(R, K, N), dtype=torch.uint8, device="cuda")
        L.check(L.lib.exb_linear_g128(L.ptr(x), R, K, L.ptr(w), L.ptr(M), None, N, L.ptr(y), L.ptr(tot),
                                      L.ptr(scratch), _stream(torch)))
        yh, th = y.cpu().numpy(), tot.cpu().numpy()
        assert eo.h16(th) == case["tot"], (K, N, R)
        assert eo.h16(yh) == case["y"], (K, N, R)
        assert [int(v) for v in yh[0, :8]] == case["y_row0"]


@pytest.mark.parametrize("scale_bits", [18, 40])
def test_linear_channel_drop_rule(torch_cuda, scale_bits):
    """Per-channel linear incl. the per-row overflow drop rule (exact_llm.py:89-96); 40-bit scales
    force drop > 0 on every row."""
    torch = torch_cuda
    L = _lib()
    rng = np.random.default_rng(scale_bits)
    R, K, N = 5, 896, 1000
    x = rng.integers(-(1 << 40), 1 << 40, (R, K)).astype(np.int64)
    w = rng.integers(-127, 128, (N, K)).astype(np.int8)
    M = rng.integers(1 << (scale_bits - 1), 1 << scale_bits, N).astype(np.int64)
    b = rng.integers(-(1 << 14), 1 << 14, N).astype(np.int64)
    lin = eo.ChannelLinear(w, M, b)
    want = lin(x)
    acc_want = lin.raw(eo.qrow(x)[0])
    if scale_bits == 40:
        assert (eo.bitlen(np.abs(acc_want).max(-1)) + lin.Mbits - 62).min() > 0
    xd, wd, Md, bd = (torch.from_numpy(a).cuda() for a in (x, w, M, b))
    y = torch.empty((R, N), dtype=torch.int64, device="cuda")
    acc = torch.empty((R, N), dtype=torch.int64, device="cuda")
    scratch = torch.empty(L.lib.exb_linear_g128_scratch_bytes(R, K, 0), dtype=torch.uint8, device="cuda")
    L.check(L.lib.exb_linear_channel(L.ptr(xd), R, K, L.ptr(wd), L.ptr(Md), L.ptr(bd), N, L.ptr(y), L.ptr(acc),
                                     L.ptr(scratch), _stream(torch)))
    assert np.array_equal(acc.cpu().numpy(), acc_want)
    assert np.array_equal(y.cpu().numpy(), want)


# ------------------------------------------------------------------ model level
def _engine_from_oracle(om, **kw):
    from exact_llm_b200 import ExactModel
    return ExactModel.from_tensors(om.c, oracle_tensors(om), **kw)


@pytest.mark.parametrize("key", ["tiny-g128", "tiny-ch"])
def test_tiny_model_prefill_decode_trace(golden, cuda_ok, key):
    g = golden["models"][key]
    om = synth.build_model(dict(g["config"]), g["seed"])
    ref = np.load(os.path.join(GOLDEN_DIR, f"{key}.npz"))
    m = _engine_from_oracle(om, max_batch=2, max_seq=64)
    m.trace_enable(True)
    lg = m(g["prompt"])
    assert np.array_equal(lg, ref["prefill"])
    tr = m.trace()
    sizes = m.linear_sizes()
    off = 0
    for name, N, _ in sizes:
        assert eo.h16(np.ascontiguousarray(tr[:, off:off + N])) == g["prefill_trace"][name], name
        off += N
    m.trace_enable(False)
    pre, rows, toks = m.greedy(g["prompt"], len(g["tokens"]))
    assert toks == g["tokens"]
    assert np.array_equal(np.array(rows), ref["rows"])


def test_tiny_decode_trace_digests(golden, cuda_ok):
    g = golden["models"]["tiny-g128"]
    om = synth.build_model(dict(g["config"]), g["seed"])
    m = _engine_from_oracle(om, max_batch=1, max_seq=64)
    lg = m(g["prompt"])
    first = int(lg[-1].argmax())
    m.trace_enable(True)
    m.generate([first], len(g["trace_digests"]))
    tr = m.trace()
    for step, want in enumerate(g["trace_digests"]):
        assert eo.step_digest(tr[step]).hex() == want, step


def test_pre_tiny_reference_fixture(golden, cuda_ok):
    """The reference's own tiny model (float -> int by its QLin; hd = 16): hash eb3c5426052399f8."""
    from exact_llm_b200 import ExactModel
    z = np.load(os.path.join(GOLDEN_DIR, "pre_tiny.npz"))
    c = dict(golden["pre_tiny"]["config"])
    c["lin"] = "channel"
    t = {"emb_q16": np.rint(z["emb"] * eo.ONE).astype(np.int64), "gf": z["gf"], "head.w": z["head_w"].T,
         "head.M": z["head_M"], "emb": np.zeros((c["V"], c["D"]), np.int8)}
    for i in range(c["NL"]):
        t[f"L{i}.g1"], t[f"L{i}.g2"] = z[f"L{i}.g1"], z[f"L{i}.g2"]
        for nm in eo.LIN_NAMES:
            t[f"L{i}.{nm}.w"] = np.ascontiguousarray(z[f"L{i}.{nm}.w"].T)
            t[f"L{i}.{nm}.M"] = z[f"L{i}.{nm}.M"]
            if f"L{i}.{nm}.b" in z:
                t[f"L{i}.{nm}.b"] = z[f"L{i}.{nm}.b"]
    m = ExactModel.from_tensors(c, t, max_batch=1, max_seq=64, tie=False)
    lg = m(golden["pre_tiny"]["ids"])
    assert eo.h16(lg) == "eb3c5426052399f8"


@pytest.mark.parametrize("key", ["qwen2.5-0.5b", "qwen2.5-7b-L2", "qwen2.5-14b-L1"])
def test_synthetic_models_vs_reference(golden, cuda_ok, key):
    """BASELINE config 1 (0.5B: 32 prompt ids + 64 greedy steps) and the 7B / 14B layer shapes,
    weights generated in HBM, against the reference IntModel run on the same integers."""
    from exact_llm_b200 import ExactModel
    if key not in golden["models"]:
        pytest.skip(f"fixture {key} not recorded")
    g = golden["models"][key]
    c = dict(g["config"])
    m = ExactModel.synthetic(c, g["seed"], max_batch=1, max_seq=len(g["prompt"]) + len(g["tokens"]) + 8)
    pre, rows, toks = m.greedy(g["prompt"], len(g["tokens"]))
    assert eo.h16(pre) == g["prefill"]
    assert toks == g["tokens"]
    assert [eo.h16(r) for r in rows] == g["rows"]


@pytest.mark.parametrize("emb_shift", [9, 20])
def test_fused_gemv_inputs_match_separate_kernels(cuda_ok, emb_shift):
    """GEMVs that build their int16 input rows in their prologue (qrow from the producer's published
    max; the norm computed whole by every CTA; the norm finished from the row statistics the
    producers publish), and norms run as the last-CTA tails of the o and down GEMVs, give the
    logits and tokens of the separate row kernels.  emb_shift 20 makes
    max |x| >= 2^24, where irms shifts the row and the statistics prologue takes the full routine."""
    from exact_llm_b200 import ExactModel, configs
    c = configs.arch("qwen2.5-7b", NL=2)
    m = ExactModel.synthetic(c, 55, max_batch=1, max_seq=64, emb_shift=emb_shift)
    prompt = np.random.default_rng(9).integers(0, c["V"], 7).astype(np.int32)
    out = {}
    variants = ((3, 0), (2, 0), (1, 1), (1, 0), (0, 0))
    for key in variants:            # fuse level, norm tails
        for name, v in zip(("fuse", "tail"), key):
            m.set_option(name, v)
        out[key] = m.greedy(prompt, 6)
    ref = out[0, 0]
    for key in variants[:-1]:
        assert np.array_equal(out[key][0], ref[0]), key
        assert out[key][2] == ref[2], key
        assert all(np.array_equal(a, b) for a, b in zip(out[key][1], ref[1])), key


@pytest.mark.parametrize("B", [1, 3])
def test_tensor_core_decode_matches_gemv(cuda_ok, B):
    """Decode steps with the tcgen05 GEMM (8-row tiles, split over the 128-groups, digit planes
    written by the row kernels) give the logits and tokens of the CUDA-core GEMV path."""
    from exact_llm_b200 import ExactModel, configs
    c = configs.arch("qwen2.5-7b", NL=2)
    m = ExactModel.synthetic(c, 63, max_batch=B, max_seq=48)
    prompts = np.random.default_rng(B).integers(0, c["V"], (B, 9)).astype(np.int32)
    out = {}
    for tcd in (1, 0):
        m.set_option("tcd", tcd)
        for b in range(B):
            m.new_cache(b)
        _, nxt = m.forward_rows(prompts.T.reshape(-1), np.tile(np.arange(B, dtype=np.int32), 9), want_logits=False)
        out[tcd] = m.generate(nxt[-B:], 6, want_logits=True)
    assert np.array_equal(out[1][0], out[0][0])
    assert np.array_equal(out[1][1], out[0][1])


@pytest.mark.parametrize("T", [16, 75, 300])
def test_tensor_core_prefill_matches_gemv_path(cuda_ok, T):
    """Prefill of T rows on the tcgen05 GEMM (chunks of up to 256 rows, ragged tails, rows of two
    sequences interleaved) gives the same logits and next tokens as the 4-row CUDA-core GEMV path."""
    from exact_llm_b200 import ExactModel, configs
    c = configs.arch("qwen2.5-7b", NL=2)
    m = ExactModel.synthetic(c, 91, max_batch=2, max_seq=T + 8)
    rng = np.random.default_rng(T)
    ids = rng.integers(0, c["V"], T).astype(np.int32)
    seqs = (np.arange(T) % 2).astype(np.int32)
    out = {}
    for tc in (1, 0):
        m.set_option("tc", tc)
        m.new_cache(0); m.new_cache(1)
        out[tc] = m.forward_rows(ids, seqs, want_logits=True)
    assert np.array_equal(out[1][1], out[0][1])
    assert np.array_equal(out[1][0], out[0][0])


@pytest.mark.parametrize("key", ["tiny-moe", "qwen1.5-moe-L1"])
def test_moe_models_vs_reference(golden, cuda_ok, key):
    """BASELINE config 4 layer shape (Qwen1.5-MoE: 60 experts, top-4, shared expert) and a tiny MoE:
    prefill logits, router selections per layer and token, greedy steps, against the reference
    MoEInt run on the same integers (experiments/moe_exact_kaggle.py:419-482)."""
    from exact_llm_b200 import ExactModel
    g = golden["moe"][key]
    c = dict(g["config"])
    m = ExactModel.synthetic(c, g["seed"], max_batch=1, max_seq=len(g["prompt"]) + len(g["tokens"]) + 8)
    lg = m(g["prompt"])
    assert eo.h16(lg) == g["prefill"]
    for layer, want in g["sel"].items():
        assert m.moe_selections(int(layer)).tolist() == want, layer
    pre, rows, toks = m.greedy(g["prompt"], len(g["tokens"]))
    assert toks == g["tokens"]
    assert [eo.h16(r) for r in rows] == g["rows"]


def test_moe_tensor_core_prefill_matches_gemv_path(golden, cuda_ok):
    """MoE prefill of 40 rows on the tcgen05 GEMM (per-channel raw sums + QLin requant) equals the
    4-row GEMV path: logits, next tokens and the router selections."""
    from exact_llm_b200 import ExactModel
    c = dict(golden["moe"]["qwen1.5-moe-L1"]["config"])
    m = ExactModel.synthetic(c, 17, max_batch=1, max_seq=64)
    ids = np.random.default_rng(4).integers(0, c["V"], 40).astype(np.int32)
    out = {}
    for tc in (1, 0):
        m.set_option("tc", tc)
        lg = m(ids)
        out[tc] = (lg, m.moe_selections(0))
    assert np.array_equal(out[1][1], out[0][1])
    assert np.array_equal(out[1][0], out[0][0])


def test_wide_batch_generate_matches_single_sequences(golden, cuda_ok):
    """Batch-16 greedy decode (every step one tensor-core chunk of 16 rows, BASELINE config 3's bs16)
    produces, for every sequence, the tokens and logits of decoding that sequence alone."""
    from exact_llm_b200 import ExactModel, configs
    c = configs.arch("qwen2.5-7b", NL=1)
    B, P, S = 16, 12, 5
    m = ExactModel.synthetic(c, 23, max_batch=B, max_seq=P + S + 4)
    prompts = np.random.default_rng(8).integers(0, c["V"], (B, P)).astype(np.int32)
    ids = prompts.T.reshape(-1)
    seqs = np.tile(np.arange(B, dtype=np.int32), P)
    for b in range(B):
        m.new_cache(b)
    _, nxt = m.forward_rows(ids, seqs, want_logits=False)
    toks, rows = m.generate(nxt[-B:], S, want_logits=True)
    for b in (0, 7, 15):
        m1 = ExactModel.synthetic(c, 23, max_batch=1, max_seq=P + S + 4)
        pre, rows1, toks1 = m1.greedy(prompts[b], S)
        assert [int(nxt[-B + b])] + list(toks[b, :-1]) == toks1, b
        for s in range(S):
            assert np.array_equal(rows[s, b], rows1[s]), (b, s)


def test_freivalds_keys_and_self_check(golden, cuda_ok):
    """Device keys equal the reference keys (rng seeded 2026); honest steps pass every check;
    a corrupted weight is caught (experiments/gpu_engine_trace_verify_kaggle.py:803-872)."""
    g = golden["models"]["tiny-g128"]
    om = synth.build_model(dict(g["config"]), g["seed"])
    m = _engine_from_oracle(om, max_batch=1, max_seq=64)
    lins = [L[nm] for L in om.layers for nm in eo.LIN_NAMES] + [om.head]
    rs = eo.draw_keys(lins, 2026)
    m.freivalds_set_keys([np.stack([r for _, r in pr]) for pr in rs])
    d_dev = m.freivalds_keys()
    names = [n for n, _, _ in m.linear_sizes()]
    for nm, d, pr in zip(names, d_dev, rs):
        want = golden["freivalds"]["keys"][nm]
        assert eo.h16(d[0]) == want[0]["d"] and eo.h16(d[1]) == want[1]["d"], nm
    m.freivalds_enable(True)
    m(g["prompt"])
    checks, fails = m.freivalds_status()
    assert checks == len(g["prompt"]) * len(names) and fails == 0
    # corrupt one weight of L1.down after the keys were built: the self-check must fail
    w = om.layers[1]["down"].w.copy()
    w[3, 5] = np.int8(w[3, 5] + (1 if w[3, 5] < 127 else -1))
    m.set_tensor("L1.down.w", w)
    m(g["prompt"])
    _, fails = m.freivalds_status()
    assert fails > 0


def test_commit_root_matches_reference(golden, cuda_ok):
    """Merkle trace commitment hashed on the GPU: the root of a 16-token forward of the per-channel
    tiny model equals the root the reference's own prover_trace / leaves_of / merkle computed."""
    g = golden["commit"]
    om = synth.build_model(synth.config(g["model"]), g["seed"])
    m = _engine_from_oracle(om, max_batch=1, max_seq=64)
    m.new_cache(0)
    m.commit_begin(0, 32)
    m.forward(g["ids"], m.new_cache(0))
    root, leaves = m.commit_root(len(g["ids"]), leaves=True)
    assert leaves.shape[0] == g["n_leaves"]
    assert leaves[0].tobytes().hex() == g["leaf0"] and leaves[-1].tobytes().hex() == g["leaf_last"]
    for i, h in g["leaf_sample"].items():
        assert leaves[int(i)].tobytes().hex() == h, i
    assert root.hex() == g["root"]
    m.commit_end()


def test_commit_root_prefill_and_decode_match_oracle(cuda_ok):
    """Group-128 model: positions logged by a prefill and by greedy decode steps give the root of
    one full forward over the same tokens (the oracle restatement of the reference's commitment)."""
    cfg = synth.config("tiny-g128")
    om = synth.build_model(cfg, 5)
    m = _engine_from_oracle(om, max_batch=1, max_seq=64)
    prompt = [int(t) for t in synth.prompt_ids(11, 1, 9, cfg["V"])[0]]
    m.commit_begin(0, 40)
    _, _, toks = m.greedy(prompt, 6)
    ids = prompt + toks
    root = m.commit_root(len(ids))
    tr = eo.commit_trace(om, ids)
    assert root == eo.merkle_root(eo.commit_leaves(tr, cfg["NL"]))
    # a shorter prefix commits to a different root, and positions never logged are refused
    assert m.commit_root(len(ids) - 1) == eo.merkle_root(eo.commit_leaves(eo.commit_trace(om, ids[:-1]), cfg["NL"]))
    with pytest.raises(RuntimeError):
        m.commit_root(len(ids) + 1)
    m.commit_end()


def test_sampler_rows_match_reference(golden, cuda_ok):
    """The GPU integer sampler picks the reference's token for seeded synthetic logits rows
    (vocabularies up to 151,936, temperatures 0.6-1.7, 64-bit seeds)."""
    g = golden["sampler"]
    om = synth.build_model(synth.config(g["model"]), g["model_seed"])
    m = _engine_from_oracle(om, max_batch=1, max_seq=32)
    rng = np.random.default_rng(g["rows_seed"])
    for row in g["rows"]:
        lg = rng.integers(-row["scale"], row["scale"], row["V"]).astype(np.int64)
        tok = m.sample(lg, [row["seed"]], [row["pos"]], row["tnum"])
        assert int(tok[0]) == row["token"], row
    # several rows in one call: each row draws with its own seed and position
    rows = rng.integers(-(8 << 16), 8 << 16, (3, 777)).astype(np.int64)
    got = m.sample(rows, [1, 2, 3], [0, 5, 9], 81920)
    want = [eo.sample_int(rows[i], s, p, 81920)[0] for i, (s, p) in enumerate([(1, 0), (2, 5), (3, 9)])]
    assert [int(t) for t in got] == want


def test_sampled_generate_matches_reference_receipt(golden, cuda_ok):
    """Seeded temperature sampling through the decode graph (device sampler) reproduces the
    reference's generate() receipt -- tokens and hash chain -- and the batched verifier accepts it
    and rejects a changed token or chain."""
    g = golden["sampler"]
    om = synth.build_model(synth.config(g["model"]), g["model_seed"])
    m = _engine_from_oracle(om, max_batch=1, max_seq=64)
    r = g["receipt"]
    receipt, greedy = m.generate_sampled(r["prompt"], len(r["tokens"]), r["seed"], r["temp"])
    assert receipt == r
    assert greedy == g["greedy"]
    assert m.verify_receipt(r) == (True, None)
    bad = dict(r, tokens=list(r["tokens"]))
    bad["tokens"][3] = (bad["tokens"][3] + 1) % om.c["V"]
    assert m.verify_receipt(bad) == (False, 3)
    assert m.verify_receipt(dict(r, chain="0" * 16)) == (False, "chain")


def test_weightless_verifier_gpu_matches_reference(golden, cuda_ok):
    """Batch cell verification on the GPU (no weights used: Freivalds keys, scales, gains, tables,
    embedding digests) gives the reference's verdict and reason on every honest, lying, cheating
    and fake-attention cell of the fixture."""
    from tests.test_oracle_golden import _verify_scenarios
    g = golden["verify"]
    om, ids, NL, trs = _verify_scenarios(g)
    m = _engine_from_oracle(om, max_batch=1, max_seq=64)
    m.verifier_keys(2026)
    keys = eo.verifier_keys(om)
    for li, d in enumerate(m.freivalds_keys()):     # device digests equal the reference-pinned keys
        kk = keys["head"] if li == 7 * NL else keys["layers"][li // 7][eo.LIN_NAMES[li % 7]]
        assert np.array_equal(d, np.stack([x for _, _, x in kk])), li
    T = len(ids)
    levels = {k: eo.merkle_levels(eo.commit_leaves(tr, NL)) for k, tr in trs.items()}
    for sc in ("honest", "cheat", "fake"):
        cases = [c for c in g["cells"] if c["scenario"] == sc]
        cells = [tuple(c["cell"]) for c in cases]
        opened = {cell: eo.open_cell(trs[sc], NL, levels[sc], cell) for cell in cells}
        got = m.verify_cells(T, levels[sc][-1][0], cells, opened, ids)
        assert got == [(c["ok"], c["why"]) for c in cases], sc
    for c in (c for c in g["cells"] if c["scenario"] == "lie"):
        cell = tuple(c["cell"])
        op = {cell: eo.open_cell(trs["lie"], NL, levels["lie"], cell, lie=tuple(c["lie"]))}
        assert m.verify_cells(T, levels["lie"][-1][0], [cell], op, ids) == [(c["ok"], c["why"])], c


def test_weightless_verifier_gpu_group_model(cuda_ok):
    """Group-128 model (accumulators are the scaled group sums): the GPU verifier accepts every
    honest cell and rejects tampered openings and a forged next residual row, as the oracle does."""
    cfg = synth.config("tiny-g128")
    om = synth.build_model(cfg, 3)
    ids = [int(t) for t in synth.prompt_ids(4, 1, 12, cfg["V"])[0]]
    NL, T = cfg["NL"], len(ids)
    tr = eo.commit_trace(om, ids)
    levels = eo.merkle_levels(eo.commit_leaves(tr, NL))
    root = levels[-1][0]
    m = _engine_from_oracle(om, max_batch=1, max_seq=64)
    m.verifier_keys(7)
    cells = [(L, t) for L in range(NL + 1) for t in range(T)]
    opened = {cell: eo.open_cell(tr, NL, levels, cell) for cell in cells}
    assert all(ok for ok, _ in m.verify_cells(T, root, cells, opened, ids))
    # a changed accumulator with its leaf re-committed elsewhere still fails its Merkle proof
    bad = {(1, 5): eo.open_cell(tr, NL, levels, (1, 5), lie=("R", 1, 5))}
    assert m.verify_cells(T, root, [(1, 5)], bad, ids) == [(False, "merkle ('R', 1, 5)")]
    # a prover whose whole commitment carries a wrong down accumulator is caught by Freivalds
    tr2 = eo.commit_trace(om, ids)
    tr2["A"][0]["down"] = tr2["A"][0]["down"].copy()
    tr2["A"][0]["down"][7, 3] += 1
    lv2 = eo.merkle_levels(eo.commit_leaves(tr2, NL))
    got = m.verify_cells(T, lv2[-1][0], [(0, 7), (0, 6)], {c: eo.open_cell(tr2, NL, lv2, c) for c in [(0, 7), (0, 6)]}, ids)
    assert got == [(False, "down"), (True, None)]


@pytest.mark.parametrize("T", [37, 300])
def test_prefill_attention_kernels_agree(cuda_ok, T):
    """Prefill chunks of one sequence through the query-tile attention kernel give the logits of
    the per-row kernel bit for bit (7B layer shapes, chunks of 256 rows, a ragged last tile)."""
    from exact_llm_b200 import ExactModel, configs
    c = configs.arch("qwen2.5-7b", NL=2)
    m = ExactModel.synthetic(c, 91, max_batch=1, max_seq=T + 8)
    ids = np.random.default_rng(T).integers(0, c["V"], T).astype(np.int32)
    out = {}
    for pa in (0, 1):
        m.set_option("pattn", pa)
        out[pa] = m.forward(ids, m.new_cache(0))
    assert np.array_equal(out[0], out[1])


@pytest.mark.parametrize("max_seq", [1120, 2304])
def test_long_context_attention_kernels_agree(cuda_ok, max_seq):
    """1100-token context (every decode-attention CTA walks several key tiles -- 128 keys while the
    cache holds at most 2048 positions, 64 beyond -- and the prefill runs five 256-row chunks): the
    fused decode attention and the query-tile prefill attention give the per-row kernels' logits
    bit for bit."""
    from exact_llm_b200 import ExactModel, configs
    c = configs.arch("qwen2.5-7b", NL=1)
    T, steps = 1100, 12                # every step's new row lies past the first key tile of its CTA
    m = ExactModel.synthetic(c, 17, max_batch=1, max_seq=max_seq)
    ids = np.random.default_rng(5).integers(0, c["V"], T).astype(np.int32)
    out = {}
    for fused in (0, 1):
        m.set_option("pattn", fused)
        m.set_option("attn", fused)
        pre = m.forward(ids, m.new_cache(0))
        toks, rows = m.generate([int(pre[-1].argmax())], steps, want_logits=True)
        out[fused] = (pre, np.array(toks), np.array(rows))
    for a, b in zip(out[0], out[1]):
        assert np.array_equal(a, b)
