#!/usr/bin/env python
"""Benchmark: exact integer decode on the Qwen2.5-7B architecture, batch 1.

One "step" = one greedy decode token for every sequence of the batch (the reference's
GraphDecoder.step, experiments/speed_fair_kaggle.py:639-645), after a 512-token prefill.
Weights are a seeded random-init integer model of the 7B architecture generated in HBM
(7.3 GB of int8 weights + int32 group scales, far larger than the 126 MB L2, so no flush is
needed between steps).  Multi-GPU (torchrun, N ranks): one model tensor-parallel over the N GPUs
(the north star's scaling for 7B+; strong scaling, integer all-reduces inside the step graph);
``--replicas`` runs N independent replicas instead (weak scaling, no collective).

--impl reference times the reference's CPU algorithm (exact_llm.IntModel decode = full-prefix
recompute per generated token, exact_llm.py:262-268) through the numpy port under oracle/, on
the same config: every timed step is one whole decoder layer of that recompute, the per-token
rate follows from NL layers + the head (stated in the line).  It never loads the CUDA library.
"""
import argparse
import ctypes
import json
import os
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode tok/s (7B-arch, bs1) as % HBM roofline; prefill int8 TOPS; bit-exact"
PROMPT = 512
GU_TRAFFIC = 140.154624e6 + 6.384128e6      # bytes per launch of the 7B gate|up GEMV (one ncu capture)


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


def int8_peak_tops():
    """Dense int8 tensor-core throughput of this GPU measured with the library GEMM (torch._int_mm,
    cuBLASLt, 8192^3, best of 10 after warm-up): the denominator of the prefill utilisation."""
    import torch
    a = torch.randint(-127, 127, (8192, 8192), dtype=torch.int8, device="cuda")
    b = torch.randint(-127, 127, (8192, 8192), dtype=torch.int8, device="cuda")
    for _ in range(3):
        torch._int_mm(a, b)
    best = None
    for _ in range(10):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        torch._int_mm(a, b)
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        best = ms if best is None or ms < best else best
    del a, b
    return 2 * 8192 ** 3 / (best * 1e-3) / 1e12


def gemm_tc_tops(K, N, T, reps=10):
    """The exact linear operator at T rows (qrow + digit planes + tcgen05 GEMM + epilogue) on one
    7B gate|up-shaped layer: effective int16 x int8 TOPS (2 T N K per call) and milliseconds."""
    import ctypes
    import torch
    from exact_llm_b200 import _lib as L
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    w = torch.empty(N * K, dtype=torch.int8, device="cuda")
    M = torch.empty(N * (K // 128), dtype=torch.int32, device="cuda")
    L.check(L.lib.exb_gen_tensor(0, 5, 11, N * K, K, L.ptr(w), st))
    L.check(L.lib.exb_gen_tensor(1, 5, 12, N * (K // 128), K, L.ptr(M), st))
    x = torch.randint(-(1 << 22), 1 << 22, (T, K), dtype=torch.int64, device="cuda")
    y = torch.empty((T, N), dtype=torch.int64, device="cuda")
    sc = torch.empty(L.lib.exb_linear_g128_scratch_bytes(T, K, N), dtype=torch.uint8, device="cuda")

    def f():
        L.check(L.lib.exb_linear_g128(L.ptr(x), T, K, L.ptr(w), L.ptr(M), None, N, L.ptr(y), None, L.ptr(sc), st))
    for _ in range(3):
        f()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record()
    for _ in range(reps):
        f()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    return 2.0 * T * N * K / (ms * 1e-3) / 1e12, ms


def commit_bench(model, T, layers=0):
    """Merkle trace commitment over T logged positions of the named architecture: the GPU root
    (leaf SHA-256 + tree, exb_commit_root) timed against hashlib on one host core over leaves of
    the same byte layout (the reference hashes its trace on the host)."""
    import hashlib
    import torch
    from exact_llm_b200 import ExactModel, configs
    c = configs.arch(model, **({"NL": layers} if layers else {}))  # noqa: F811
    m = ExactModel.synthetic(c, 1234, max_batch=1, max_seq=T + 8)
    ids = np.random.default_rng(7).integers(0, c["V"], T).astype(np.int32)
    m.commit_begin(0, T)
    t0 = time.perf_counter()
    m.forward(ids, m.new_cache(0), want_logits=False)
    torch.cuda.synchronize()
    fwd_s = time.perf_counter() - t0
    m.commit_root(T)                                         # warm-up (module load)
    t0 = time.perf_counter()
    root = m.commit_root(T)
    gpu_s = time.perf_counter() - t0
    NL, D, I, V, kv, q = c["NL"], c["D"], c["I"], c["V"], c["KV"] * c["hd"], c["H"] * c["hd"]
    sizes = [[D]] * ((NL + 1) * T) + [[kv, kv], [kv, kv], [q], [D, I, I, D]] * (NL * T) + [[V]] * T
    buf = np.random.default_rng(0).integers(-2**40, 2**40, max(V, 2 * I + 2 * D), dtype=np.int64).tobytes()
    t0 = time.perf_counter()
    leaves = []
    for segs in sizes:
        hh = hashlib.sha256()
        for n in segs:
            hh.update(buf[:8 * n])
            hh.update(b"|")
        leaves.append(hh.digest())
    lv = [hashlib.sha256(b"L" + x).digest() for x in leaves]
    while len(lv) > 1:
        lv = [hashlib.sha256(b"N" + lv[i] + (lv[i + 1] if i + 1 < len(lv) else lv[i])).digest()
              for i in range(0, len(lv), 2)]
    host_s = time.perf_counter() - t0
    nbytes = sum(8 * n + 1 for segs in sizes for n in segs)
    m.commit_end()
    m.close()
    return {"model": model, "positions": T, "leaves": len(sizes), "hashed_bytes": nbytes,
            "gpu_ms": round(gpu_s * 1e3, 2), "gpu_gbs": round(nbytes / gpu_s / 1e9, 2),
            "host_1core_ms": round(host_s * 1e3, 1), "host_1core_gbs": round(nbytes / host_s / 1e9, 2),
            "speedup": round(host_s / gpu_s, 1), "prefill_with_capture_s": round(fwd_s, 3),
            "root": root.hex()}


# ------------------------------------------------------------------ clocks
class Clocks:
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu):
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.gpu = gpu
        self.p = None

    def __enter__(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                       "-lms", "50"], stdout=self.f, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except (OSError, FileNotFoundError):
            self.p = None
        return self

    def __exit__(self, *a):
        if self.p:
            self.p.terminate()
            self.p.wait()

    def summary(self):
        self.f.flush()
        rows = [r.split(",") for r in open(self.f.name).read().strip().splitlines() if r.count(",") >= 8]
        os.unlink(self.f.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}
        sm = [float(r[1]) for r in rows]
        reasons = set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for r in rows:
            for nm, v in zip(names, r[5:9]):
                if v.strip() == "Active":
                    reasons.add(nm)
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": float(rows[0][2]), "samples": len(rows),
                "power_w_max": max(float(r[3]) for r in rows if r[3].strip().replace(".", "").isdigit()) if rows else None,
                "reasons": sorted(reasons)}


# ------------------------------------------------------------------ CPU baseline (numpy port of the reference)
class CpuDecodeSample:
    """The reference's per-token decode work on the host: exact_llm.generate re-runs IntModel over
    the whole prefix (no KV cache), i.e. NL decoder layers + the head over `prefix` rows.  One
    sample = one decoder layer over the prefix (every op); the head is timed once on 64 of the
    rows and scaled (its cost is linear in rows)."""

    def __init__(self, c, prefix):
        from oracle import exact_oracle as eo
        self.eo, self.c, self.prefix = eo, c, prefix
        rng = np.random.default_rng(0)
        D, H, KV, hd, I, V = (c[k] for k in ("D", "H", "KV", "hd", "I", "V"))

        def glin(N, K, bias):
            return eo.GroupLinear(rng.integers(-127, 128, (N, K), dtype=np.int8),
                                  rng.integers(1 << 16, 1 << 17, (N, K // 128)),
                                  rng.integers(-16384, 16384, N) if bias else None)

        self.L = dict(g1=np.full(D, 65536, np.int64), g2=np.full(D, 65536, np.int64), q=glin(H * hd, D, True),
                      k=glin(KV * hd, D, True), v=glin(KV * hd, D, True), o=glin(D, H * hd, False),
                      gate=glin(I, D, False), up=glin(I, D, False), down=glin(D, I, False))
        self.head = eo.ChannelLinear(rng.integers(-127, 128, (V, D), dtype=np.int8), rng.integers(1 << 16, 1 << 17, V))
        self.cos, self.sin = eo.rope_tables(prefix, hd, c["theta"])
        self.om = eo.OracleModel(dict(c, NL=1), [self.L], np.full(D, 65536, np.int64), self.head,
                                 lambda ids: (rng.integers(-127, 128, (len(ids), D)) << 9), self.cos, self.sin)
        self.x = rng.integers(-(1 << 17), 1 << 17, (prefix, D))
        self.head_rows = min(prefix, 64)
        self.t_head = None

    def layer(self):
        eo, L, c, T = self.eo, self.L, self.c, self.prefix
        H, KV, hd = c["H"], c["KV"], c["hd"]
        t0 = time.perf_counter()
        a = eo.irms(self.x, L["g1"])
        q = eo.rope(L["q"](a).reshape(T, H, hd).transpose(1, 0, 2), self.cos, self.sin)
        k = eo.rope(L["k"](a).reshape(T, KV, hd).transpose(1, 0, 2), self.cos, self.sin)
        v = L["v"](a).reshape(T, KV, hd).transpose(1, 0, 2)
        out = self.om._attention(0, q, k, v, None, 0)
        x = self.x + L["o"](out.transpose(1, 0, 2).reshape(T, H * hd))
        m = eo.irms(x, L["g2"])
        x = x + L["down"](eo.shr(eo.isilu(L["gate"](m)) * L["up"](m), 16))
        self.x_out = x
        return time.perf_counter() - t0

    def head_time(self):
        x = getattr(self, "x_out", self.x)
        t0 = time.perf_counter()
        self.head(self.eo.irms(x[:self.head_rows], self.om.gf))
        self.t_head = (time.perf_counter() - t0) * self.prefix / self.head_rows
        return self.t_head

    def describe(self, t_layer):
        return (f"one of {self.c['NL']} decoder layers over a {self.prefix}-token prefix per timed step (full-prefix "
                f"recompute per generated token, as exact_llm.generate does) + the head timed over {self.head_rows} "
                f"of {self.prefix} rows and scaled; per token = {self.c['NL']} x layer {t_layer:.2f} s + head "
                f"{self.t_head:.2f} s")


def cpu_cores():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count()


def arch_config(a):
    """The architecture dict of --model (the oracle's copy: the reference arm never loads the CUDA
    library, and both arms describe the same workload)."""
    from oracle import synth
    c = synth.config(a.model, **({"NL": a.layers} if a.layers else {}))
    c.pop("T", None)
    return c


def workload_config(a, c, world, tp):
    return {"workload": f"{a.model}-arch greedy decode, batch {a.batch}, after a {PROMPT}-token uniform prompt",
            "batch": a.batch, "prompt": PROMPT, "decode_steps": a.steps, "layers": c["NL"],
            "parallelism": (f"tensor parallel x{world}" if tp else f"replicas x{world}" if world > 1 else "single GPU"),
            "l2": "no flush: the weights stream from HBM every step (7.3 GB at 7B, L2 126 MB)"}


# ------------------------------------------------------------------ reference arm
def run_reference(a, rank, world):
    if rank != 0:
        return
    c = arch_config(a)
    tp = world > 1 and not a.replicas
    smp = CpuDecodeSample(c, PROMPT + 1)
    # bounded so the whole arm ends within a few minutes whatever --steps / --warmup say: at most 2
    # untimed warm-up samples, then timed samples until --steps or about 90 s of sampling (at least
    # 3); the line reports the samples actually timed
    for _ in range(min(2, max(1, a.warmup))):                 # untimed warm-up samples
        smp.layer()
    smp.head_time()
    times = []
    while len(times) < max(1, a.steps) and (len(times) < 3 or sum(times) < 90.0):
        times.append(smp.layer())                             # each timed step: one whole decoder layer
    t_layer = float(np.median(times))
    per_tok = c["NL"] * t_layer + smp.t_head
    val = 1.0 / per_tok                                       # IntModel decodes one sequence at a time
    line = {"impl": "reference", "metric": METRIC, "value": val, "unit": "tok/s", "n_gpus": world,
            "steps": len(times), "warmup": min(2, max(1, a.warmup)), "ms_per_step": t_layer * 1e3,
            "higher_is_better": True,
            "scaling": "strong" if tp else "weak", "vs_baseline": None,
            "dtype": "int64 (float64 BLAS, exact < 2^53)", "data": "synthetic",
            "config": workload_config(a, c, world, tp),
            "timed_step": {"unit": f"one decoder layer of the {PROMPT + 1}-token full-prefix recompute",
                           "seconds": times, "per_token_layers": c["NL"], "head_s": smp.t_head,
                           "value_is": f"1 / ({c['NL']} x median step + head)"},
            "cpu_baseline": {"value": val, "unit": "tok/s", "cores": cpu_cores(), "kind": "port",
                             "sample": smp.describe(t_layer)},
            "e2e": {"value": val, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ our arm
def lin_flops_fn(c):
    """2 x MACs of every linear and the head for one token (int16 x int8 products)."""
    return 2 * (c["NL"] * ((c["H"] + 2 * c["KV"]) * c["hd"] * c["D"] + c["D"] * c["H"] * c["hd"] + 3 * c["I"] * c["D"])
                + c["V"] * c["D"])


def step_bytes(c, B, S):
    """Algorithmic HBM bytes of one decode step (all B rows): int8 weights + group scales + head
    (int8 + int64 per-channel scales) + KV cache read (K int16 + shift, V int32) at S positions."""
    D, H, KV, hd, I, V, NL = (c[k] for k in ("D", "H", "KV", "hd", "I", "V", "NL"))
    lin = (H + 2 * KV) * hd * D + D * H * hd + 2 * I * D + D * I
    w = NL * (lin + lin // 128 * 4 + (H + 2 * KV) * hd * 8 + 2 * D * 8) + V * D + V * 8 + D * 8
    kv = B * NL * KV * S * (hd * 2 + 1 + hd * 4)
    return w + kv


def run_ours(a, rank, world, local_rank):
    import torch
    torch.cuda.set_device(local_rank)
    from exact_llm_b200 import ExactModel
    from exact_llm_b200._lib import check, lib, ptr
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))

    def barrier():
        if dist:
            dist.barrier()
        torch.cuda.synchronize()

    c = arch_config(a)
    B, K, W = a.batch, a.steps, a.warmup
    max_seq = PROMPT + W + 3 * K + 16          # warm-up, timed steps, the two e2e loops
    tp = world > 1 and not a.replicas
    if tp:
        # one model split over the ranks (tensor parallel): NCCL id from rank 0
        uid = [ExactModel.tp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        m = ExactModel(c, max_batch=B, max_seq=max_seq, tp=(rank, world, uid[0]))
        check(lib.exb_model_generate(m.h, 1234))
        m.finalize()
    else:
        m = ExactModel.synthetic(c, 1234, max_batch=B, max_seq=max_seq)
    for opt in a.option:
        name, val = opt.split("=")
        m.set_option(name, int(val))
    stream = torch.cuda.ExternalStream(m.stream)
    rng = np.random.default_rng(100 + rank)
    prompts = rng.integers(0, c["V"], (B, PROMPT)).astype(np.int32)
    # prefill (outside the decode timing): rows of all sequences, position-major so every chunk
    # holds B sequences; CUDA events on the model stream around the whole forward call, after one
    # untimed prefill of the same prompts (first-launch module loading stays out of the number)
    barrier()
    ids = prompts.T.reshape(-1)
    seqs = np.tile(np.arange(B, dtype=np.int32), PROMPT)
    for b in range(B):
        m.new_cache(b)
    m.forward_rows(ids, seqs, want_logits=False)
    torch.cuda.synchronize()
    for b in range(B):
        m.new_cache(b)
    p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    p0.record(stream)
    _, nxt = m.forward_rows(ids, seqs, want_logits=False)
    p1.record(stream)
    torch.cuda.synchronize()
    prefill_s = p0.elapsed_time(p1) / 1e3
    first = nxt[-B:].astype(np.int32)
    ids_dev = torch.from_numpy(first).cuda()
    tok_dev = torch.empty((max(W, K), B), dtype=torch.int32, device="cuda")
    check(lib.exb_generate_device(m.h, B, ptr(ids_dev), W, ptr(tok_dev)))       # warm-up (captures graphs)
    torch.cuda.synchronize()
    step_kernels = lib.exb_step_launches(m.h)       # kernel nodes of the step graph the timed loop replays
    ids_dev = tok_dev[W - 1].clone() if W > 0 else ids_dev
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    with Clocks(local_rank) as clk:
        e0.record(stream)
        check(lib.exb_generate_device(m.h, B, ptr(ids_dev), K, ptr(tok_dev)))
        e1.record(stream)
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    barrier()
    if dist:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    # e2e through the public API with HOST buffers, as GraphDecoder.step does: host token in
    # (pinned staging), the step's int64 logits row out to pinned host memory, every step
    # (sequence 0; batch > 1 rows go through forward_rows with all B logits rows)
    last = tok_dev[K - 1].cpu().numpy().astype(np.int32)
    seqs_b = np.arange(B, dtype=np.int32)
    Vg = c["V"]
    if B > 1:
        lg_host = torch.empty((B, Vg), dtype=torch.int64, pin_memory=True).numpy()
        nxt_b = np.empty(B, np.int32)
    barrier()
    t0 = time.perf_counter()
    cur = last
    for _ in range(K):
        if B == 1:
            m.step(int(cur[0]))
            cur = m.last_next
        else:
            check(lib.exb_forward(m.h, B, ptr(np.ascontiguousarray(cur, np.int32), ctypes.c_int32),
                                  ptr(seqs_b, ctypes.c_int32), ptr(lg_host, ctypes.c_int64), ptr(nxt_b, ctypes.c_int32)))
            cur = nxt_b
    e2e_s = time.perf_counter() - t0
    # the same loop returning only the next token (4 bytes per row) for comparison
    barrier()
    t0 = time.perf_counter()
    for _ in range(K):
        _, cur = m.forward_rows(cur, seqs_b, want_logits=False)
    e2e_tok_s = time.perf_counter() - t0
    if dist:
        t = torch.tensor([e2e_s, e2e_tok_s], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s, e2e_tok_s = float(t[0].item()), float(t[1].item())
    # dominant kernel: the fused gate|up GEMV of one layer, timed alone with CUDA events
    avg = ctypes.c_float()
    nbytes = ctypes.c_double()
    if B <= 4:
        check(lib.exb_bench_linear(m.h, 0, 2, B, 50, ctypes.byref(avg), ctypes.byref(nbytes)))
        kern_name = "k_gemv<R,2,group> (fused gate|up, SwiGLU epilogue), layer 0"
    else:
        # wider batches run every linear on the tcgen05 GEMM: time the gate|up-shaped linear at B rows
        _, gms = gemm_tc_tops(c["D"], 2 * c["I"], B)
        avg.value = gms
        nbytes.value = 2 * c["I"] * c["D"] * (1 + 4 / 128) + B * c["D"] * 8 + B * 2 * c["I"] * 8
        kern_name = f"tcgen05 group-128 GEMM, gate|up shape, {B} rows (qrow + digits + GEMM)"
    hbm, _, src = peaks()
    kern_gbs = nbytes.value / (avg.value * 1e-3) / 1e9
    S_mid = PROMPT + W + K // 2
    sb = step_bytes(c, B, S_mid)
    step_ms = ms / K
    step_gbs = sb / (step_ms * 1e-3) / 1e9
    gpu_gbs = step_gbs / world if tp else step_gbs        # tensor parallel: each GPU streams its 1/N slice
    if rank != 0:
        m.close()                      # step graphs (NCCL inside under --tp) go before the process group
        if dist:
            dist.destroy_process_group()
        return
    value = (1 if tp else world) * B * K / (ms * 1e-3)
    units = 1 if tp else world
    # prefill: the whole forward (every op) and the tcgen05 linear alone at the 7B gate|up shape
    prefill = {"tokens": PROMPT * B, "seconds": prefill_s, "tok_s": PROMPT * B / prefill_s,
               "effective_tops": lin_flops_fn(c) * PROMPT * B / prefill_s / 1e12,
               "path": "linears on the tcgen05 int8 GEMM (int16 activations as 2 int8 digits), 512-row chunks"}
    if PROMPT * B >= 16 and not a.no_gemm:
        tops, gms = gemm_tc_tops(c["D"], 2 * c["I"], 2048)
        peak8 = int8_peak_tops()
        prefill["gemm"] = {"shape": f"T=2048 K={c['D']} N={2 * c['I']} (gate|up)", "ms": gms, "effective_tops": tops,
                           "tensor_pipe_tops": 2 * tops, "int8_peak_tops": peak8,
                           "peak_source": "measured: torch._int_mm (cuBLASLt) 8192^3 int8, best of 10",
                           "frac": 2 * tops / peak8}

    line = {
        "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": step_ms, "higher_is_better": True, "scaling": "strong" if tp else "weak", "vs_baseline": None,
        "dtype": "int8 x int16 -> int64", "data": "synthetic",
        "config": workload_config(a, c, world, tp),
        "decode_hbm": {"bytes_per_step": sb, "achieved_gbs": step_gbs, "per_gpu_gbs": gpu_gbs, "peak_gbs": hbm,
                       "frac": gpu_gbs / hbm, "peak_source": src},
        "roofline": {"bound": "hbm", "kernel": kern_name,
                     "achieved": kern_gbs, "peak": hbm, "unit": "GB/s", "frac": kern_gbs / hbm,
                     "traffic": GU_TRAFFIC if a.model == "qwen2.5-7b" and B == 1 else None,   # R=1 capture
                     "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of this kernel, "
                                       "profiles/gemv_gate_up_7b_bs1.md",
                     "avg_launch_ms": avg.value, "algorithmic_bytes": nbytes.value,
                     "peak_source": src},
        "prefill": prefill,
        "e2e": {"value": units * B * K / e2e_s, "unit": "tok/s", "h2d_bytes_per_step": 4 * 3 * 4,
                "d2h_bytes_per_step": 8 * Vg * B + 4 * B,
                "path": "ExactModel.step(token) (GraphDecoder.step): host token in, the int64 logits row out to "
                        "pinned host memory, one call per step",
                "tokens_only": {"value": units * B * K / e2e_tok_s, "d2h_bytes_per_step": 4 * B,
                                "path": "forward_rows(host ids) -> host next-token"}},
        # B <= 4: every step is one CUDA graph whose kernel nodes the engine counts at capture (embed,
        # 7 per layer, final norm, head, token feedback); wider batches launch one tensor-core chunk
        # per step (embed, 14 per layer: norms, digit planes, GEMMs, rope, attention, qrow; final
        # norm, digits, head GEMM, head rows)
        "gpu_launches": K * step_kernels if B <= 4 else K * (1 + 14 * c["NL"] + 4),
        "clocks": clk.summary(),
    }
    if world == 1 and not a.no_cpu:
        smp = CpuDecodeSample(c, PROMPT + 1)
        t_layer = smp.layer()
        smp.head_time()
        line["cpu_baseline"] = {"value": 1.0 / (c["NL"] * t_layer + smp.t_head), "unit": "tok/s", "cores": cpu_cores(),
                                "kind": "port", "sample": smp.describe(t_layer)}
    print(json.dumps(line), flush=True)
    m.close()
    if dist:
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=16)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--model", default="qwen2.5-7b")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-gemm", action="store_true", help="skip the tensor-core GEMM / int8 peak measurement")
    ap.add_argument("--replicas", action="store_true",
                    help="with --gpus N under torchrun: N independent replicas instead of one tensor-parallel model")
    ap.add_argument("--prompt", type=int, default=PROMPT, help="prompt tokens before decode (profiling uses a short one)")
    ap.add_argument("--layers", type=int, default=0, help="override the layer count (small ncu captures only)")
    ap.add_argument("--option", action="append", default=[], metavar="NAME=VALUE",
                    help="engine option for the timed model (exb_set_option; results never change)")
    ap.add_argument("--commit", type=int, default=0, metavar="T",
                    help="only the Merkle trace commitment of T logged 7B positions: GPU vs host hashlib")
    ap.add_argument("--linear", type=int, default=0, metavar="T",
                    help="only the exact linear op at T rows on the 7B gate|up shape (profiling)")
    a = ap.parse_args()
    globals()["PROMPT"] = a.prompt
    if a.commit:
        print(json.dumps({"commit": commit_bench(a.model, a.commit, a.layers)}))
        return
    if a.linear:
        import torch
        torch.cuda.set_device(0)
        tops, ms = gemm_tc_tops(3584, 37888, a.linear, reps=max(1, a.steps))
        print(json.dumps({"linear": {"T": a.linear, "K": 3584, "N": 37888, "ms": round(ms, 4),
                                     "effective_tops": round(tops, 1)}}))
        return
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    if a.warmup < 3 and a.impl == "ours":
        ap.error("--warmup must be >= 3")
    if a.impl == "reference":
        run_reference(a, rank, world)
    else:
        run_ours(a, rank, world, local_rank)


if __name__ == "__main__":
    main()
