"""Parity at the BASELINE configurations' real sizes, through the C ABI (needs a B200).

Every expected value was recorded from the reference's own code by tests/golden/make_golden.py:
  * long["qwen2.5-7b-L2-p512"]    config 3's 512-token prompt (7B architecture, 2 layers): every
                                  prefill row, 4 greedy steps, the KV cache of both layers
  * long["qwen2.5-14b-L1-p4096"]  config 5's 4096-token prompt (14B architecture, 1 layer): rows
                                  999, 2047, 3000 and the last 8, 3 greedy steps, the KV cache
  * moe_wide                      config 4's workload shape (32 sequences x 256 prompt tokens, one
                                  Qwen1.5-MoE layer): the router's top-4 experts of every token,
                                  each sequence's last prompt row and 3 greedy steps decoded as one
                                  32-row batch
  * freivalds_7b                  the reference's Freivalds keys at the 7B shapes
The long prompts were recorded with the reference's per-layer machinery (forward_record, then
block_row per new position, exact_llm.py:322-363), which equals its full recompute."""
import numpy as np
import pytest

from oracle import exact_oracle as eo
from oracle import synth

pytestmark = pytest.mark.gpu


def _kv_equal(m, want, slot=0):
    """The exported KV cache of every layer (K int16 + shift, V) against the reference's cache."""
    from exact_llm_b200.model import Cache
    for li, kv in enumerate(want):
        got = m.kv_cache(li, Cache(m, slot))
        assert [int(t) for t in got["kq"][0, 0, :8]] == kv["k_row0"], li
        assert eo.h16(got["kq"]) == kv["k"], li
        assert eo.h16(got["sk"]) == kv["sk"], li
        assert eo.h16(got["v"]) == kv["v"], li


def test_7b_512_token_prompt_vs_reference(golden, cuda_ok):
    """Config 3's prompt length: the prefill's 512 logits rows (tensor-core chunks, query-tile
    attention over up to 512 cached positions), 4 greedy decode steps (fused decode attention) and
    the exported KV cache of both layers equal the reference's."""
    from exact_llm_b200 import ExactModel
    g = golden["long"]["qwen2.5-7b-L2-p512"]
    c = dict(g["config"])
    steps = len(g["tokens"])
    m = ExactModel.synthetic(c, g["seed"], max_batch=1, max_seq=g["T"] + steps + 8)
    pre, rows, toks = m.greedy(g["prompt"], steps)
    assert [int(v) for v in pre[-1, :8]] == g["prefill_last8"]
    assert eo.h16(pre) == g["prefill_all"]
    assert toks == g["tokens"]
    assert [eo.h16(r) for r in rows] == g["step_rows"]
    _kv_equal(m, g["kv"])


def test_14b_4096_token_prompt_vs_reference(golden, cuda_ok):
    """Config 5's prompt length on one GPU: one prefill of 4088 rows then the last 8 (logits
    compared), 3 greedy decode steps at 4096-4098 cached positions (64-key decode tiles), the KV
    cache; then the same prompt prefilled in pieces ending at rows 999, 2047 and 3000 (single-row
    calls on the GEMV path) gives those rows' logits."""
    from exact_llm_b200 import ExactModel
    g = golden["long"]["qwen2.5-14b-L1-p4096"]
    c = dict(g["config"])
    steps = len(g["tokens"])
    T = g["T"]
    ids = np.asarray(g["prompt"], np.int32)
    m = ExactModel.synthetic(c, g["seed"], max_batch=1, max_seq=T + steps + 8)
    cache = m.new_cache(0)
    m.forward(ids[:T - 8], cache, want_logits=False)
    last = m.forward(ids[T - 8:], cache)
    want_rows = dict(zip(g["rows"], g["prefill_rows"]))
    for i in range(8):
        assert eo.h16(last[i]) == want_rows[i - 8], i - 8
    assert [int(v) for v in last[-1, :8]] == g["prefill_last8"]
    first = int(m.last_next[-1])
    toks, lg = m.generate([first], steps, want_logits=True)
    assert [first] + [int(t) for t in toks[0, :-1]] == g["tokens"]
    assert [eo.h16(lg[s, 0]) for s in range(steps)] == g["step_rows"]
    _kv_equal(m, g["kv"])
    cache = m.new_cache(0)
    start = 0
    for r in (999, 2047, 3000):
        if r > start:
            m.forward(ids[start:r], cache, want_logits=False)
        row = m.forward(ids[r:r + 1], cache)[0]
        assert eo.h16(row) == want_rows[r], r
        start = r + 1


def test_moe_32_sequences_256_tokens_vs_reference(golden, cuda_ok):
    """Config 4's workload shape: 32 sequences of 256 prompt tokens prefilled position-major (rows of
    all 32 sequences in each tensor-core chunk), the router's top-4 experts of every token, each
    sequence's last prompt row, and 3 greedy steps of all 32 sequences as one wide batch."""
    from exact_llm_b200 import ExactModel
    g = golden["moe_wide"]
    c = dict(g["config"])
    B, T, steps = g["B"], g["T"], g["steps"]
    prompts = synth.prompt_ids(g["prompt_seed"], B, T, c["V"]).astype(np.int32)
    m = ExactModel.synthetic(c, g["seed"], max_batch=B, max_seq=T + steps + 8)
    for b in range(B):
        m.new_cache(b)
    sel = np.zeros((B, T, c["TOPK"]), np.int64)
    seqs = np.arange(B, dtype=np.int32)
    for p0, p1 in ((0, 128), (128, T - 1), (T - 1, T)):
        ids = prompts[:, p0:p1].T.reshape(-1)
        lg, nxt = m.forward_rows(ids, np.tile(seqs, p1 - p0), want_logits=(p1 == T))
        sel[:, p0:p1] = m.moe_selections(0).reshape(p1 - p0, B, -1).transpose(1, 0, 2)
    for b, want in enumerate(g["seqs"]):
        assert sel[b, :4].tolist() == want["sel_head"], b
        assert eo.h16(np.ascontiguousarray(sel[b])) == want["sel"], b
        assert eo.h16(lg[b]) == want["last"], b
    first = nxt[-B:].astype(np.int32)
    toks, rows = m.generate(first, steps, want_logits=True)
    for b, want in enumerate(g["seqs"]):
        assert [int(first[b])] + [int(t) for t in toks[b, :-1]] == want["tokens"], b
        assert [eo.h16(rows[s, b]) for s in range(steps)] == want["rows"], b


def test_freivalds_and_trace_at_7b_shapes(golden, cuda_ok):
    """Freivalds at the 7B architecture's shapes (accumulators near 2^55, so the mod-p reduction of
    large signed values matters): device keys equal the reference's keys_group / keys_channel; the
    trace of an honest prefill equals the reference's accumulators and passes every check; a
    corrupted weight is caught."""
    from exact_llm_b200 import ExactModel
    g = golden["models"]["qwen2.5-7b-L2"]
    fz = golden["freivalds_7b"]
    c = dict(g["config"])
    assert fz["seed"] == g["seed"]
    m = ExactModel.synthetic(c, g["seed"], max_batch=1, max_seq=64)
    sizes = m.linear_sizes()

    class _Lin:
        def __init__(self, N):
            self.N = N
    rs = eo.draw_keys([_Lin(N) for _, N, _ in sizes], 2026)
    m.freivalds_set_keys([np.stack([r for _, r in pr]) for pr in rs])
    for (nm, _, _), d in zip(sizes, m.freivalds_keys()):
        assert [eo.h16(d[0]), eo.h16(d[1])] == fz["d"][nm], nm
    m.trace_enable(True)
    m.freivalds_enable(True)
    m(g["prompt"])
    checks, fails = m.freivalds_status()
    assert checks == len(g["prompt"]) * len(sizes) and fails == 0
    tr = m.trace()
    off = 0
    for nm, N, _ in sizes:
        assert eo.h16(np.ascontiguousarray(tr[:, off:off + N])) == g["prefill_trace"][nm], nm
        off += N
    assert int(np.abs(tr).max()).bit_length() > 40          # large accumulators really were reduced
    m.trace_enable(False)
    w = synth.gen_weight(fz["seed"], synth.layer_stream(1, synth.LIN_STREAM["down"]), c["D"], c["I"])
    w[100, 7] = np.int8(w[100, 7] + (1 if w[100, 7] < 127 else -1))
    m.set_tensor("L1.down.w", w)
    m(g["prompt"])
    _, fails = m.freivalds_status()
    assert fails > 0
