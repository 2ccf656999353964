"""One rank of a tensor-parallel parity run (launched by tests/test_tp_multigpu.py through
torch.distributed.run, one process per GPU).  Rank 0 makes the NCCL unique id; the id travels
over a gloo process group (127.0.0.1).  Every rank builds its slice of the synthetic model of a
golden fixture (weights generated globally on the device and cut per rank), runs the reference's
greedy loop, and rank 0 compares the prefill logits, the step logits and the tokens with the
fixture recorded from the reference IntModel."""
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


def main():
    key = sys.argv[1]
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
    dist.init_process_group("gloo")
    uid = [ExactModel.tp_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(uid, src=0)
    g = json.load(open(os.path.join(ROOT, "tests", "golden", "golden.json")))["models"][key]
    c = dict(g["config"])
    m = ExactModel(c, max_batch=1, max_seq=len(g["prompt"]) + len(g["tokens"]) + 8, tp=(rank, world, uid[0]))
    from exact_llm_b200._lib import check, lib
    check(lib.exb_model_generate(m.h, int(g["seed"])))
    m.finalize()
    pre, rows, toks = m.greedy(g["prompt"], len(g["tokens"]))
    parts = {"prefill": eo.h16(pre) == g["prefill"], "tokens": toks == g["tokens"],
             "rows": [eo.h16(r) for r in rows] == g["rows"]}
    ok = all(parts.values())
    flags = [None] * world
    dist.all_gather_object(flags, bool(ok))
    if rank == 0:
        print(json.dumps({"key": key, "world": world, "ranks_ok": flags, "rank0_parts": parts}), flush=True)
    m.close()
    dist.destroy_process_group()
    sys.exit(0 if all(flags) else 1)


if __name__ == "__main__":
    main()
