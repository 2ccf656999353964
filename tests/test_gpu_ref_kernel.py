"""The reference's own CUDA kernel, gemv_g128_v2 (experiments/speed_fair_kaggle.py:662-693), built
for sm_100a by oracle/build_ref.py, run on the B200 beside this library's GEMVs (needs a B200).

Parity: ``torch.ops.exact.gemv`` (exb_gemv) and the engine's decode GEMV (exb_linear_g128 at one
row, whose tot output is the same sum) give the reference kernel's int64 outputs bit for bit on
the reference's six G1 shapes and on the 7B projection shapes.  Timing (CUDA events, inputs
generated on the device, 7B shapes larger than L2 are streamed from HBM every launch) is printed
and, when EXB_TIMING_OUT names a file, written there as JSON."""
import ctypes
import json
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SHAPES = [(896, 896), (896, 4864), (4864, 896), (1536, 8960), (8960, 1536), (896, 151936),   # G1 (:705)
          (3584, 4608), (3584, 3584), (3584, 37888), (18944, 3584), (3584, 152064)]          # 7B layer + head


def _ref():
    from oracle.build_ref import load
    mod = load()
    if mod is None:
        pytest.skip("oracle/_ref/exact_gemv_ref.so not built (needs the reference checkout at build time)")
    return mod


def _time(torch, fn, reps=50):
    for _ in range(5):
        fn()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record()
    for _ in range(reps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps


def test_reference_gemv_kernel_vs_ours(cuda_ok):
    import torch
    import exact_llm_b200.ops  # noqa: F401  (registers torch.ops.exact.gemv)
    from exact_llm_b200 import _lib as L
    ref = _ref()
    g = torch.Generator(device="cuda").manual_seed(0)
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rows = []
    for K, N in SHAPES:
        x = torch.randint(-32767, 32768, (K,), generator=g, device="cuda", dtype=torch.int16)
        wT = torch.randint(-127, 128, (N, K), generator=g, device="cuda", dtype=torch.int8)
        Mg = torch.randint(1, 1 << 27, (N, K // 128), generator=g, device="cuda", dtype=torch.int64)
        want = ref.gemv(x, wT, Mg)
        got = torch.ops.exact.gemv(x, wT, Mg)
        assert torch.equal(got, want), (K, N)
        # the engine's decode GEMV: same sum as tot, from int32 scales and an int64 row whose qrow is x
        M32 = Mg.to(torch.int32).contiguous()
        x64 = x.to(torch.int64).view(1, K).contiguous()
        x64[0, 0] = 32767                      # pin the row max so qrow keeps the values (shift 0)
        want1 = ref.gemv(x64[0].to(torch.int16), wT, Mg)
        y = torch.empty((1, N), dtype=torch.int64, device="cuda")
        tot = torch.empty((1, N), dtype=torch.int64, device="cuda")
        scratch = torch.empty(L.lib.exb_linear_g128_scratch_bytes(1, K, N), dtype=torch.uint8, device="cuda")

        def k1():
            L.check(L.lib.exb_linear_g128(L.ptr(x64), 1, K, L.ptr(wT), L.ptr(M32), None, N, L.ptr(y), L.ptr(tot),
                                          L.ptr(scratch), st))
        k1()
        torch.cuda.synchronize()
        assert torch.equal(tot[0], want1), (K, N)
        t_ref = _time(torch, lambda: ref.gemv(x, wT, Mg))
        t_op = _time(torch, lambda: torch.ops.exact.gemv(x, wT, Mg))
        t_k1 = _time(torch, k1)
        mb_ref = (N * K + N * (K // 128) * 8 + 2 * K + 8 * N) / 1e6     # int8 W, int64 scales
        mb_k1 = (N * K + N * (K // 128) * 4 + 8 * K + 16 * N) / 1e6     # int8 W, int32 scales
        rows.append(dict(K=K, N=N, ref_us=round(t_ref * 1e3, 2), op_us=round(t_op * 1e3, 2), k1_us=round(t_k1 * 1e3, 2),
                         ref_gbs=round(mb_ref / t_ref, 1), op_gbs=round(mb_ref / t_op, 1), k1_gbs=round(mb_k1 / t_k1, 1)))
        print(rows[-1], flush=True)
    out = os.environ.get("EXB_TIMING_OUT")
    if out:
        with open(out, "w") as f:
            json.dump(rows, f, indent=1)
