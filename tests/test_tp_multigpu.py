"""Tensor parallelism: the shard plan (host logic, CPU), its agreement across ranks (gloo, 2
processes on CPU), and bit-exact parity of a 2-GPU NCCL run with the reference fixtures (skipped
when fewer than 2 GPUs are visible)."""
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _plans(name, size):
    from exact_llm_b200 import ExactModel, configs
    c = configs.arch(name)
    return c, [ExactModel.tp_plan(c, r, size) for r in range(size)]


@pytest.mark.parametrize("name,size", [("qwen2.5-7b", 2), ("qwen2.5-7b", 4), ("qwen2.5-7b", 8), ("qwen2.5-14b", 8)])
def test_tp_plan_tiles_the_model(name, size):
    """Heads, KV heads, I groups and the vocabulary are covered exactly once (KV heads may repeat
    across the ranks of one group); each rank's query heads use only its own KV heads."""
    c, plans = _plans(name, size)
    rep = c["H"] // c["KV"]
    q = [h for p in plans for h in range(p["qh0"], p["qh1"])]
    assert q == list(range(c["H"]))
    g = [x for p in plans for x in range(p["ig0"], p["ig1"])]
    assert g == list(range(c["I"] // 128))
    v = [x for p in plans for x in range(p["v0"], p["v1"])]
    assert v == list(range(c["V"]))
    for p in plans:
        assert all(p["kh0"] <= h // rep < p["kh1"] for h in range(p["qh0"], p["qh1"]))
        assert ((p["qh1"] - p["qh0"]) * c["hd"]) % 128 == 0


def test_tp_plan_matches_reference_partition():
    """7B TP8: 4/3 query heads per rank pair, one KV head each; I = 148 groups as 19x4 + 18x4
    (the partition the reference survey gives for the 7B layer)."""
    _, plans = _plans("qwen2.5-7b", 8)
    assert [p["qh1"] - p["qh0"] for p in plans] == [4, 3] * 4
    assert all(p["kh1"] - p["kh0"] == 1 for p in plans)
    assert [p["ig1"] - p["ig0"] for p in plans] == [19] * 4 + [18] * 4
    _, plans = _plans("qwen2.5-14b", 8)
    assert [p["qh1"] - p["qh0"] for p in plans] == [5] * 8
    assert [p["ig1"] - p["ig0"] for p in plans] == [14] * 4 + [13] * 4


def _gloo_rank(rank, world, port, q):
    import torch.distributed as dist
    sys.path.insert(0, ROOT)
    from exact_llm_b200 import ExactModel, configs
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    c = configs.arch("qwen2.5-7b")
    mine = ExactModel.tp_plan(c, rank, world)
    allp = [None] * world
    dist.all_gather_object(allp, mine)
    q.put((rank, allp))
    dist.destroy_process_group()


def test_tp_plan_agrees_across_gloo_ranks():
    """Two CPU processes (gloo) each compute their own slice; the gathered slices are the same on
    both ranks and tile the model, as the NCCL ranks rely on."""
    import multiprocessing as mp
    import socket
    ctx = mp.get_context("spawn")
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    q = ctx.Queue()
    procs = [ctx.Process(target=_gloo_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert res[0] == res[1]
    assert res[0][0]["qh1"] == res[0][1]["qh0"] and res[0][0]["ig1"] == res[0][1]["ig0"]


def _run_tp(key, mode, port, n=2):
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(["timeout", "-k", "30", "900", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
                        f"--nproc-per-node={n}", "--master-addr", "127.0.0.1", "--master-port", str(port),
                        os.path.join(ROOT, "tests", "tp_worker.py"), key, mode],
                       capture_output=True, text=True, timeout=1000, env=env)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]


@pytest.mark.gpu
@pytest.mark.parametrize("key", ["qwen2.5-7b-L2", "qwen2.5-14b-L1"])
def test_tp2_matches_reference_fixture(golden, key):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    _run_tp(key, "greedy", 29731)


@pytest.mark.gpu
@pytest.mark.parametrize("mode", ["allreduce", "nccl"])
def test_tp2_exchange_variants_match_reference_fixture(golden, mode):
    """The same decode with the step's exchanges as separate one-shot all-reduce kernels, or NCCL,
    instead of fused into the producing and consuming kernels: the same bits."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    _run_tp("qwen2.5-7b-L2", mode, 29735)


@pytest.mark.gpu
@pytest.mark.parametrize("key", ["qwen2.5-7b-L2", "qwen2.5-14b-L1"])
def test_tp2_trace_and_freivalds_match_reference(golden, key):
    """BASELINE config 5's capture under tensor parallelism: global trace hashes, step digests and
    Freivalds keys equal the reference's; every shard's self-check passes honestly and a tampered
    shard is caught."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    _run_tp(key, "trace", 29733)
