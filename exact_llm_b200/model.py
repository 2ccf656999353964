"""Host-side model API mirroring the reference's model/engine interface.

Reference interfaces (novain-shibu/exact-llm) and their counterparts here:

  IntModel(get, c); model(ids) -> int64 (T, V)          exact_llm.py:141-180      ExactModel.__call__
  TModel.forward(ids, cache, last_only); new_cache()     exact_torch.py:140,171-193 ExactModel.forward / new_cache
  GraphDecoder.step(token) (CUDA graph, static cache)    speed_fair_kaggle.py:590-645 ExactModel.step / generate
  TRACE['rec'][name] / flat per-step buffer              gpu_engine_trace_verify_kaggle.py:746,
                                                         prover_commit_cost_gpu_kaggle.py:741-742  ExactModel.trace
  keys_group / keys_channel / fr                         gpu_engine_trace_verify_kaggle.py:803-834 freivalds_*

All compute runs in libexactb200.so (sm_100a CUDA kernels); this module only moves host
arrays and calls the C ABI.  Outputs are numpy int64 Q16 logits exactly as the reference returns.
"""
import ctypes
import hashlib

import numpy as np

from . import tables
from ._lib import Config, check, lib, ptr

LIN_NAMES = ("q", "k", "v", "o", "gate", "up", "down")


class Cache:
    """A KV-cache sequence slot (TModel.new_cache equivalent, exact_torch.py:140)."""

    def __init__(self, model, slot):
        self.model, self.slot = model, slot

    @property
    def n(self):
        return lib.exb_seq_len(self.model.h, self.slot)


class ExactModel:
    """Exact integer Qwen2-family model on one B200.

    ``c`` uses the reference's config keys (D, H, KV, hd, I, V, NL, theta, tie) plus
    ``lin`` ("group" for group-128 GQLin layers, "channel" for per-channel QLin layers).
    """

    def __init__(self, c, max_batch=1, max_seq=None, rope_len=None, emb_shift=9, tie=None, tp=None, tabs=None):
        """``tp`` = (rank, size, unique_id) builds this rank's tensor-parallel slice (one process per
        GPU; every rank constructs its model at the same time; ``unique_id`` = the 128 bytes of
        ``ExactModel.tp_unique_id()`` made on rank 0 and shared by the caller)."""
        self.c = dict(c)
        self.max_batch = int(max_batch)
        self.max_seq = int(max_seq or c.get("T", 4096))
        self.rope_len = int(rope_len or max(self.max_seq, c.get("T", 0)))
        cfg = Config(D=c["D"], H=c["H"], KV=c["KV"], hd=c["hd"], I=c["I"], V=c["V"], NL=c["NL"],
                     tie=int(c.get("tie", False) if tie is None else tie),
                     lin_kind=0 if c.get("lin", "group") == "group" else 1, n_experts=int(c.get("NE", 0)),
                     topk=int(c.get("TOPK", 0)), moe_I=int(c.get("MI", 0)), shared_I=int(c.get("SI", 0)),
                     max_batch=self.max_batch, max_seq=self.max_seq, rope_len=self.rope_len, emb_shift=emb_shift)
        h = ctypes.c_void_p()
        self.tp = tp
        if tp is not None and int(tp[1]) > 1:
            import torch  # noqa: F401  (torch's NCCL, see tp_unique_id)
            rank, size, uid = int(tp[0]), int(tp[1]), bytes(tp[2])
            check(lib.exb_model_create_tp(ctypes.byref(cfg), rank, size, uid, ctypes.byref(h)))
        else:
            check(lib.exb_model_create(ctypes.byref(cfg), ctypes.byref(h)))
        self.h = h
        half = c["hd"] // 2
        if tabs is not None:            # shipped tables of a release (never recomputed)
            if tabs["cos"].shape[0] < self.rope_len:
                raise ValueError(f"the release's RoPE tables cover {tabs['cos'].shape[0]} positions < {self.rope_len}")
            self._tab = [np.ascontiguousarray(tabs[k][:self.rope_len] if k in ("cos", "sin") else tabs[k], dtype=np.int64)
                         for k in ("exp", "silu", "sig", "cos", "sin")]
        else:
            cos, sin = tables.rope_tables(self.rope_len, c["hd"], c["theta"])
            self._tab = [np.ascontiguousarray(t) for t in (tables.exp_table(), tables.silu_table(), tables.sig_table(),
                                                           cos[:, :half], sin[:, :half])]
        check(lib.exb_model_set_tables(self.h, *[ptr(t, ctypes.c_int64) for t in self._tab]))
        self._finalized = False

    @staticmethod
    def tp_unique_id():
        """NCCL unique id (128 bytes) for a tensor-parallel group; make it on rank 0."""
        import torch  # noqa: F401  (loads torch's NCCL first; the library then uses that copy)
        buf = ctypes.create_string_buffer(128)
        check(lib.exb_tp_unique_id(buf))
        return buf.raw

    @staticmethod
    def tp_plan(c, rank, size):
        """This rank's slice: dict(qh0, qh1, kh0, kh1, ig0, ig1, v0, v1, vmax) (host computation)."""
        cfg = Config(D=c["D"], H=c["H"], KV=c["KV"], hd=c["hd"], I=c["I"], V=c["V"], NL=c["NL"],
                     tie=int(c.get("tie", False)), lin_kind=0 if c.get("lin", "group") == "group" else 1,
                     n_experts=int(c.get("NE", 0)), topk=int(c.get("TOPK", 0)), moe_I=int(c.get("MI", 0)),
                     shared_I=int(c.get("SI", 0)), max_batch=1, max_seq=1, rope_len=1, emb_shift=9)
        out = (ctypes.c_int32 * 9)()
        check(lib.exb_tp_plan(ctypes.byref(cfg), int(rank), int(size), out))
        return dict(zip(("qh0", "qh1", "kh0", "kh1", "ig0", "ig1", "v0", "v1", "vmax"), list(out)))

    # ------------------------------------------------------------------ construction
    @classmethod
    def synthetic(cls, c, seed, **kw):
        """Seeded synthetic integer model generated directly in HBM."""
        m = cls(c, **kw)
        check(lib.exb_model_generate(m.h, int(seed)))
        m.finalize()
        return m

    @classmethod
    def from_tensors(cls, c, tensors, **kw):
        """Integer artifact given as {name: array} (names as in include/exactb200.h)."""
        m = cls(c, **kw)
        for name, arr in tensors.items():
            m.set_tensor(name, arr)
        m.finalize()
        return m

    @classmethod
    def from_artifact(cls, path, **kw):
        """Load an exact release (``artifact.write_artifact`` layout): every file's SHA-256 is checked
        against the manifest, the shipped tables are used as they are."""
        from .artifact import load_artifact
        arch, tensors, tabs = load_artifact(path)
        c = dict(arch)
        kw.setdefault("rope_len", int(arch["rope_len"]))
        kw.setdefault("max_seq", int(arch["rope_len"]))
        kw.setdefault("tie", "head.w" not in tensors and bool(arch.get("tie")))   # a shipped head is used as is
        m = cls(c, tabs=tabs, **kw)
        for name, a in tensors.items():
            if name.endswith(".M") and a.ndim == 2:          # group-128 scales ship as int64, run as int32
                if a.size and (int(a.max()) >= 1 << 31 or int(a.min()) < -(1 << 31)):
                    raise ValueError(f"{name}: group scale outside int32")
                a = np.asarray(a, dtype=np.int32)
            m.set_tensor(name, a)
        m.finalize()
        return m

    def set_tensor(self, name, arr):
        a = np.ascontiguousarray(arr)
        check(lib.exb_model_set_tensor(self.h, name.encode(), ptr(a), a.nbytes))

    def finalize(self):
        check(lib.exb_model_finalize(self.h))
        self._finalized = True

    def close(self):
        if getattr(self, "h", None):
            lib.exb_model_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def weight_bytes(self):
        return lib.exb_model_weight_bytes(self.h)

    @property
    def stream(self):
        return lib.exb_model_stream(self.h)

    # ------------------------------------------------------------------ reference-style API
    def new_cache(self, slot=0):
        check(lib.exb_seq_reset(self.h, slot))
        return Cache(self, slot)

    def forward(self, ids, cache=None, last_only=False, want_logits=True):
        """TModel.forward: logits (T, V) of the new tokens (or (1, V) with last_only)."""
        if cache is None:
            cache = self.new_cache(0)
        ids = np.ascontiguousarray(np.asarray(ids, dtype=np.int32).reshape(-1))
        T = len(ids)
        self._rows = T
        seqs = np.full(T, cache.slot, np.int32)
        logits = np.empty((T, self.c["V"]), np.int64) if want_logits else None
        nxt = np.empty(T, np.int32)
        check(lib.exb_forward(self.h, T, ptr(ids, ctypes.c_int32), ptr(seqs, ctypes.c_int32),
                              ptr(logits, ctypes.c_int64), ptr(nxt, ctypes.c_int32)))
        self.last_next = nxt
        if logits is None:
            return None
        return logits[-1:] if last_only else logits

    def __call__(self, ids):
        """IntModel.__call__: full causal forward of a fresh sequence -> int64 (T, V) Q16 logits."""
        return self.forward(ids, self.new_cache(0))

    def forward_rows(self, ids, seqs, want_logits=True):
        """Rows of several sequences in one call (row i appends ids[i] to sequence seqs[i])."""
        ids = np.ascontiguousarray(np.asarray(ids, np.int32).reshape(-1))
        seqs = np.ascontiguousarray(np.asarray(seqs, np.int32).reshape(-1))
        self._rows = len(ids)
        logits = np.empty((len(ids), self.c["V"]), np.int64) if want_logits else None
        nxt = np.empty(len(ids), np.int32)
        check(lib.exb_forward(self.h, len(ids), ptr(ids, ctypes.c_int32), ptr(seqs, ctypes.c_int32),
                              ptr(logits, ctypes.c_int64), ptr(nxt, ctypes.c_int32)))
        return logits, nxt

    def generate(self, first_ids, steps, want_logits=False):
        """Greedy decode of sequences 0..B-1 with on-device token feedback (GraphDecoder loop).
        Returns tokens (B, steps) and, if asked, logits (steps, B, V)."""
        first = np.ascontiguousarray(np.asarray(first_ids, np.int32).reshape(-1))
        B = len(first)
        self._rows = B * int(steps)
        toks = np.empty((steps, B), np.int32)
        logits = np.empty((steps, B, self.c["V"]), np.int64) if want_logits else None
        check(lib.exb_generate(self.h, B, ptr(first, ctypes.c_int32), int(steps), ptr(toks, ctypes.c_int32),
                               ptr(logits, ctypes.c_int64)))
        return (toks.T.copy(), logits) if want_logits else toks.T.copy()

    def greedy(self, prompt, steps, want_logits=True):
        """Prefill ``prompt`` in slot 0, then ``steps`` greedy tokens: (prefill logits, step logits, tokens),
        the first generated token being argmax of the prompt's last row (exact_llm.py:262-268)."""
        lg = self.forward(prompt, self.new_cache(0))
        first = int(self.last_next[-1])
        if steps <= 0:
            return lg, [], []
        toks, rows = self.generate([first], steps, want_logits=True)
        # generate() feeds token t and returns the argmax of its logits as token t+1
        tokens = [first] + [int(t) for t in toks[0, :-1]]
        return lg, [rows[s, 0] for s in range(steps)], tokens

    def step(self, token, cache=None):
        """GraphDecoder.step(token) (experiments/speed_fair_kaggle.py:639-645): append one token to
        the sequence of ``cache`` (slot 0 by default), run one decode step (a captured CUDA graph),
        and return its int64 Q16 logits, shape (1, V).  The row lands in a pinned host buffer that
        the next call reuses: copy it to keep it.  ``last_next`` holds the greedy token (the
        lowest index of the row's maximum)."""
        slot = 0 if cache is None else cache.slot
        if getattr(self, "_step_buf", None) is None:
            import torch
            self._step_t = torch.empty((1, self.c["V"]), dtype=torch.int64, pin_memory=True)
            self._step_buf = self._step_t.numpy()
            self._step_ids = np.empty(1, np.int32)
            self._step_seq = np.empty(1, np.int32)
            self._step_next = np.empty(1, np.int32)
        self._step_ids[0] = int(token)
        self._step_seq[0] = slot
        self._rows = 1
        check(lib.exb_forward(self.h, 1, ptr(self._step_ids, ctypes.c_int32), ptr(self._step_seq, ctypes.c_int32),
                              ptr(self._step_buf, ctypes.c_int64), ptr(self._step_next, ctypes.c_int32)))
        self.last_next = self._step_next
        return self._step_buf

    def kv_cache(self, layer, cache=None):
        """The KV cache of one layer as the reference's TModel keeps it (exact_torch.py:140,
        146-149): dict(kq=int64 (KV, n, hd), sk=int64 (KV, n, 1), v=int64 (KV, n, hd)) over the n
        positions of the sequence (slot 0 by default; tensor parallel: this rank's KV heads)."""
        slot = 0 if cache is None else cache.slot
        n = lib.exb_seq_len(self.h, slot)
        KV = self.c["KV"]
        if self.tp is not None and int(self.tp[1]) > 1:
            p = self.tp_plan(self.c, int(self.tp[0]), int(self.tp[1]))
            KV = p["kh1"] - p["kh0"]
        hd = self.c["hd"]
        k = np.empty((KV, n, hd), np.int16)
        ks = np.empty((KV, n), np.int8)
        v = np.empty((KV, n, hd), np.int32)
        check(lib.exb_kv_export(self.h, int(layer), slot, n, k.ctypes.data, ks.ctypes.data, v.ctypes.data))
        return dict(kq=k.astype(np.int64), sk=ks.astype(np.int64)[..., None], v=v.astype(np.int64))

    def moe_selections(self, layer):
        """Router top-k experts of every row of the last forward call at `layer`: int32 (rows, topk)."""
        k = int(self.c["TOPK"])
        n = min(int(self._rows), 4096)                   # rows of the last forward call
        buf = np.empty((n, k), np.int32)
        check(lib.exb_moe_selections(self.h, int(layer), ptr(buf, ctypes.c_int32), n * k))
        return buf

    def set_option(self, name, value):
        """Engine option (results never change; names and values in include/exactb200.h): "tc", "fuse",
        "attn", "pattn", "tcd", "tpar", "tpx", "tail"."""
        check(lib.exb_set_option(self.h, name.encode(), int(value)))

    # ------------------------------------------------------------------ trace + Freivalds
    def trace_enable(self, on=True):
        check(lib.exb_trace_enable(self.h, int(on)))

    @property
    def trace_row_len(self):
        return int(lib.exb_trace_row_len(self.h))

    def trace(self):
        """Raw accumulators of the last call's rows: int64 (rows, trace_row_len) in the order
        L0.q, L0.k, L0.v, L0.o, L0.gate, L0.up, L0.down, L1.q, ..., head."""
        n = self._rows
        out = np.empty(n * self.trace_row_len, np.int64)
        check(lib.exb_trace_read(self.h, ptr(out, ctypes.c_int64), out.size))
        return out.reshape(n, self.trace_row_len)

    def commit_begin(self, seq=0, capacity=None):
        """Start logging sequence slot ``seq`` for the Merkle trace commitment (turns trace capture on)."""
        check(lib.exb_commit_begin(self.h, int(seq), int(capacity or self.max_seq)))

    def commit_root(self, T, leaves=False):
        """Merkle root (32 bytes) over positions 0..T-1 of the committed sequence, computed on the
        GPU with the reference's leaves and tree (experiments/commit_audit_kaggle.py:567-628); with
        ``leaves=True`` also the leaf digests, shape ((5 NL + 2) T, 32) uint8."""
        root = (ctypes.c_uint8 * 32)()
        n = (5 * self.c["NL"] + 2) * int(T)
        lv = np.empty((n, 32), np.uint8) if leaves else None
        check(lib.exb_commit_root(self.h, int(T), root, lv.ctypes.data if leaves else None, n * 32 if leaves else 0))
        return (bytes(root), lv) if leaves else bytes(root)

    def commit_end(self):
        check(lib.exb_commit_end(self.h))

    # ------------------------------------------------------------------ integer sampler
    @staticmethod
    def temp_num(temp):
        """Temperature as the integer multiplier the sampler uses (exact_llm.py:249)."""
        return int(round((1 << 16) / temp))

    def sample(self, logits, seeds, positions, tnum):
        """Tokens of int64 logits rows (R, V) drawn on the GPU with per-row seeds and positions
        (exact_llm.py:256-259)."""
        lg = np.ascontiguousarray(np.atleast_2d(logits), dtype=np.int64)
        R, V = lg.shape
        sd = np.ascontiguousarray(np.broadcast_to(np.asarray(seeds, np.uint64), (R,)))
        ps = np.ascontiguousarray(np.broadcast_to(np.asarray(positions, np.int32), (R,)))
        out = np.empty(R, np.int32)
        check(lib.exb_sample(self.h, ptr(lg, ctypes.c_int64), R, V, sd.ctypes.data, ps.ctypes.data, int(tnum),
                             out.ctypes.data))
        return out

    def sampling(self, on, seeds=(), positions=(), tnum=1 << 16):
        """Make the decode steps of generate() sample (row b: seeds[b], from positions[b] on)."""
        sd = np.ascontiguousarray(np.asarray(seeds, np.uint64))
        ps = np.ascontiguousarray(np.asarray(positions, np.int32))
        check(lib.exb_sampling(self.h, int(bool(on)), len(sd), sd.ctypes.data if on else None,
                               ps.ctypes.data if on else None, int(tnum)))

    @staticmethod
    def _step_hash(prev, row):
        # receipt chain link (exact_llm.py:260-261): host SHA-256, sequential per step
        return hashlib.sha256(prev.encode() + np.ascontiguousarray(row, dtype=np.int64).tobytes()).hexdigest()[:16]

    def generate_sampled(self, prompt, n, seed, temp, slot=0):
        """Seeded integer sampling of ``n`` tokens after ``prompt`` with the receipt the
        reference's generate() returns (exact_llm.py:262-268): (receipt, greedy argmax per step)."""
        tnum = self.temp_num(temp)
        lg = self.forward(prompt, self.new_cache(slot))
        rows = [lg[-1]]
        toks = [int(self.sample(lg[-1:], [seed], [0], tnum)[0])]
        if n > 1:
            if slot != 0:
                raise ValueError("generate_sampled decodes slot 0")
            self.sampling(True, [seed], [1], tnum)
            try:
                produced, lrows = self.generate([toks[0]], n - 1, want_logits=True)
            finally:
                self.sampling(False)
            toks += [int(t) for t in produced[0]]
            rows += [lrows[s, 0] for s in range(n - 1)]
        chain = "start"
        for r in rows:
            chain = self._step_hash(chain, r)
        receipt = dict(prompt=[int(t) for t in prompt], seed=seed, temp=temp, tokens=toks, chain=chain)
        return receipt, [int(np.argmax(r)) for r in rows]

    def verify_receipt(self, receipt, slot=0):
        """Recompute a receipt with one forward over prompt + tokens: (ok, first bad position or
        "chain" or None), as the reference's verify() (exact_llm.py:269-276)."""
        prompt, toks = list(receipt["prompt"]), list(receipt["tokens"])
        n = len(toks)
        lg = self.forward(prompt + toks[:-1], self.new_cache(slot))[len(prompt) - 1:]
        got = self.sample(lg, [receipt["seed"]] * n, np.arange(n), self.temp_num(receipt["temp"]))
        for t in range(n):
            if int(got[t]) != toks[t]:
                return False, t
        chain = "start"
        for r in lg:
            chain = self._step_hash(chain, r)
        return (True, None) if chain == receipt["chain"] else (False, "chain")

    # ------------------------------------------------------------------ weightless cell verifier
    def verifier_keys(self, seed=2026):
        """Draw the verifier's secrets in the reference's make_verifier order
        (experiments/commit_audit_kaggle.py:461-512): per linear (trace order) r ~ U[0, p) of
        length N for p = 2^31 - 1 then 2147483629, then the embedding's r of length D per prime;
        builds the digests on the device."""
        rng = np.random.default_rng(seed)
        P = (2147483647, 2147483629)
        rs = [np.stack([rng.integers(0, p, N, dtype=np.int64) for p in P]) for _, N, _ in self.linear_sizes()]
        er = np.stack([rng.integers(0, p, self.c["D"], dtype=np.int64) for p in P])
        self.freivalds_set_keys(rs)
        e = np.ascontiguousarray(er.astype(np.int32))
        check(lib.exb_verifier_emb_keys(self.h, e.ctypes.data))

    @staticmethod
    def cell_leaves(cell, NL):
        """Names of the leaves a cell opens, in the reference's needed() order."""
        L, t = cell
        if L == NL:
            return [("X", NL, t), ("HEAD", NL, t)]
        return [("X", L, t), ("KV", L, t)] + [("KR", L, s) for s in range(t + 1)] + \
               [("Q", L, t), ("R", L, t), ("X", L + 1, t)]

    def verify_cells(self, T, root, cells, opened, ids):
        """Verify cells of a committed forward on the GPU without the weights: ``opened[cell]`` maps
        each leaf name of ``cell_leaves(cell)`` to (list of int64 arrays, list of 32-byte Merkle
        siblings), as the reference's Prover.open returns.  Returns [(ok, reason)] with the
        reference's reasons (experiments/commit_audit_kaggle.py:659-705)."""
        NL = self.c["NL"]
        vals, prfs, names = [], [], []
        for cell in cells:
            nm = self.cell_leaves(cell, NL)
            names.append(nm)
            for n in nm:
                v, pr = opened[cell][n]
                vals += [np.asarray(a, np.int64).reshape(-1) for a in v]
                prfs += [bytes(b) for b in pr]
        values = np.ascontiguousarray(np.concatenate(vals))
        proofs = np.frombuffer(b"".join(prfs), np.uint8).copy()
        cl = np.ascontiguousarray(np.asarray(cells, np.int32).reshape(-1, 2))
        idv = np.ascontiguousarray(np.asarray(ids, np.int32))
        rt = np.frombuffer(bytes(root), np.uint8).copy()
        out = np.empty(len(cells), np.int32)
        check(lib.exb_verify_cells(self.h, int(T), rt.ctypes.data, len(cells), cl.ctypes.data, idv.ctypes.data,
                                   values.ctypes.data, values.size, proofs.ctypes.data, proofs.size, out.ctypes.data))
        reasons = {2: "embedding@{t}", 3: "kv@{t}", 4: "kr@{t}", 5: "q", 6: "o", 7: "gate/up", 8: "down",
                   9: "residual", 10: "head"}
        res = []
        for (L, t), v, nm in zip(cells, out, names):
            v = int(v)
            if v == 0:
                res.append((True, None))
            elif v >= 1000:
                res.append((False, f"merkle {nm[v - 1000]}"))
            else:
                res.append((False, reasons[v].format(t=t)))
        return res

    def linear_sizes(self):
        c = self.c
        out = []
        for i in range(c["NL"]):
            out += [(f"L{i}.q", c["H"] * c["hd"], c["D"]), (f"L{i}.k", c["KV"] * c["hd"], c["D"]),
                    (f"L{i}.v", c["KV"] * c["hd"], c["D"]), (f"L{i}.o", c["D"], c["H"] * c["hd"]),
                    (f"L{i}.gate", c["I"], c["D"]), (f"L{i}.up", c["I"], c["D"]), (f"L{i}.down", c["D"], c["I"])]
        out.append(("head", c["V"], c["D"]))
        return out

    def freivalds_set_keys(self, r_list):
        """r_list: per linear (trace order) an int array (2, N) of r values in [0, p)."""
        flat = np.ascontiguousarray(np.concatenate([np.asarray(r, np.int64).reshape(-1) for r in r_list]).astype(np.int32))
        check(lib.exb_freivalds_set_keys(self.h, ptr(flat, ctypes.c_int32), flat.size))

    def freivalds_keys(self):
        sizes = self.linear_sizes()
        n = sum(2 * K for _, _, K in sizes)
        out = np.empty(n, np.int32)
        check(lib.exb_freivalds_read_keys(self.h, ptr(out, ctypes.c_int32), n))
        res, pos = [], 0
        for _, _, K in sizes:
            res.append(out[pos:pos + 2 * K].reshape(2, K).astype(np.int64))
            pos += 2 * K
        return res

    def freivalds_enable(self, on=True):
        check(lib.exb_freivalds_enable(self.h, int(on)))

    def freivalds_status(self):
        a, b = ctypes.c_int64(), ctypes.c_int64()
        check(lib.exb_freivalds_status(self.h, ctypes.byref(a), ctypes.byref(b)))
        return a.value, b.value

