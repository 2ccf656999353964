"""One rank of a tensor-parallel parity run (launched by tests/test_tp_multigpu.py through
torch.distributed.run, one process per GPU).  Rank 0 makes the NCCL unique id; the id travels
over a gloo process group (127.0.0.1).  Every rank builds its slice of the synthetic model of a
golden fixture (weights generated globally on the device and cut per rank), runs the reference's
greedy loop, and rank 0 compares the prefill logits, the step logits and the tokens with the
fixture recorded from the reference IntModel.

Mode "trace" (BASELINE config 5's capture under tensor parallelism): the global trace of the
prefill (every linear's accumulator, gathered from the ranks' shards) and of the decode steps
against the reference's recorded per-linear hashes and per-step digests; the Freivalds keys
reassembled from the shards against the reference keys (the 7B fixture), every shard's
self-check passing on an honest run and a tampered weight of one shard caught."""
import json
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
from exact_llm_b200 import ExactModel  # noqa: E402
from oracle import exact_oracle as eo  # noqa: E402


class _Lin:
    def __init__(self, N):
        self.N = N


def trace_mode(m, g, G, key, rank, world):
    parts = {}
    m.trace_enable(True)
    m(g["prompt"])
    tr = m.trace()                                      # collective: global rows from every rank's shard
    off = 0
    bad = []
    for name, N, _ in m.linear_sizes():
        if eo.h16(np.ascontiguousarray(tr[:, off:off + N])) != g["prefill_trace"][name]:
            bad.append(name)
        off += N
    parts["prefill_trace"] = not bad and off == tr.shape[1]
    parts["prefill_trace_bad"] = bad[:6]
    first = int(m.last_next[-1])
    steps = len(g["trace_digests"])
    m.generate([first], steps)
    tr = m.trace()
    parts["step_digests"] = [eo.step_digest(tr[s]).hex() for s in range(steps)] == g["trace_digests"]
    m.trace_enable(False)
    lins = [_Lin(N) for _, N, _ in m.linear_sizes()]
    rs = eo.draw_keys(lins, 2026)
    m.freivalds_set_keys([np.stack([r for _, r in pr]) for pr in rs])
    d = m.freivalds_keys()                              # collective: the global d of every linear
    if key == "qwen2.5-7b-L2":
        want = G["freivalds_7b"]["d"]
        parts["keys"] = all([eo.h16(x[0]), eo.h16(x[1])] == want[nm] for (nm, _, _), x in zip(m.linear_sizes(), d))
    m.freivalds_enable(True)
    m(g["prompt"])
    checks, fails = m.freivalds_status()                # collective: totals over the ranks
    parts["honest"] = fails == 0 and checks == world * len(g["prompt"]) * len(lins)
    c = m.c
    from oracle import synth
    li = c["NL"] - 1
    w = synth.gen_weight(g["seed"], synth.layer_stream(li, synth.LIN_STREAM["k"]), c["KV"] * c["hd"], c["D"])
    w[3, 5] = np.int8(w[3, 5] + (1 if w[3, 5] < 127 else -1))
    m.set_tensor(f"L{li}.k.w", w)                       # lands in the shard holding KV head 0
    m(g["prompt"])
    _, fails = m.freivalds_status()
    parts["tamper_caught"] = fails > 0
    m.freivalds_enable(False)
    return parts


def main():
    key = sys.argv[1]
    mode = sys.argv[2] if len(sys.argv) > 2 else "greedy"
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
    dist.init_process_group("gloo")
    uid = [ExactModel.tp_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(uid, src=0)
    G = json.load(open(os.path.join(ROOT, "tests", "golden", "golden.json")))
    g = G["models"][key]
    c = dict(g["config"])
    m = ExactModel(c, max_batch=1, max_seq=len(g["prompt"]) + len(g["tokens"]) + 8, tp=(rank, world, uid[0]))
    from exact_llm_b200._lib import check, lib
    check(lib.exb_model_generate(m.h, int(g["seed"])))
    m.finalize()
    # the decode step's exchanges: fused into the producing / consuming kernels (default), the
    # one-shot all-reduce kernels ("allreduce"), or NCCL ("nccl")
    if mode == "allreduce":
        m.set_option("tpx", 0)
    elif mode == "nccl":
        m.set_option("tpar", 0)
    if mode == "trace":
        parts = trace_mode(m, g, G, key, rank, world)
        ok = all(v for k, v in parts.items() if not k.endswith("_bad"))
    else:
        pre, rows, toks = m.greedy(g["prompt"], len(g["tokens"]))
        parts = {"prefill": eo.h16(pre) == g["prefill"], "tokens": toks == g["tokens"],
                 "rows": [eo.h16(r) for r in rows] == g["rows"]}
        ok = all(parts.values())
    flags = [None] * world
    dist.all_gather_object(flags, bool(ok))
    if rank == 0:
        print(json.dumps({"key": key, "mode": mode, "world": world, "ranks_ok": flags, "rank0_parts": parts}),
              flush=True)
    m.close()
    dist.destroy_process_group()
    sys.exit(0 if all(flags) else 1)


if __name__ == "__main__":
    main()
