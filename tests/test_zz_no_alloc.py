"""exb_linear_g128_noalloc: the exact group-128 linear for callers that cannot allocate device memory
(hosts with a device-memory budget fixed at start-up, plugin hosts that own the allocator).  Its
scratch lives in a fixed array inside the library instead of a caller buffer.  Checked through the
C ABI against exb_linear_g128 (bit-exact, the tolerance of every integer test here) on two calls in
a row with different shapes, so the second call runs on the first call's leftovers in that array.

The file name makes pytest collect it last; it passes alone in a fresh process as well."""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _setup():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test collected without a CUDA device")
    from exact_llm_b200 import _lib
    return torch, _lib


def _linear_pair(torch, L, seed, R, K, N):
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    w = torch.empty(N * K, dtype=torch.int8, device="cuda")
    M = torch.empty(N * (K // 128), dtype=torch.int32, device="cuda")
    L.check(L.lib.exb_gen_tensor(0, seed, 11, N * K, K, L.ptr(w), stream))
    L.check(L.lib.exb_gen_tensor(1, seed, 12, N * (K // 128), K, L.ptr(M), stream))
    b = torch.from_numpy(np.random.default_rng(seed).integers(-16384, 16384, N).astype(np.int64)).cuda()
    x = torch.from_numpy(np.random.default_rng(seed + 1).integers(-(1 << 22), 1 << 22, (R, K)).astype(np.int64)).cuda()
    # reference path: caller-provided scratch
    y_ref = torch.empty((R, N), dtype=torch.int64, device="cuda")
    t_ref = torch.empty((R, N), dtype=torch.int64, device="cuda")
    scratch = torch.empty(L.lib.exb_linear_g128_scratch_bytes(R, K, N), dtype=torch.uint8, device="cuda")
    L.check(L.lib.exb_linear_g128(L.ptr(x), R, K, L.ptr(w), L.ptr(M), L.ptr(b), N, L.ptr(y_ref), L.ptr(t_ref),
                                  L.ptr(scratch), stream))
    # no-allocation path
    y = torch.full((R, N), -7, dtype=torch.int64, device="cuda")
    t = torch.full((R, N), -7, dtype=torch.int64, device="cuda")
    L.check(L.lib.exb_linear_g128_noalloc(L.ptr(x), R, K, L.ptr(w), L.ptr(M), L.ptr(b), N, L.ptr(y), L.ptr(t), stream))
    torch.cuda.synchronize()
    return y.cpu().numpy(), t.cpu().numpy(), y_ref.cpu().numpy(), t_ref.cpu().numpy()


def test_noalloc_linear_matches_scratch_linear_twice():
    torch, L = _setup()
    # calls in a row with different shapes, so each call runs on the previous call's leftovers in
    # the fixed array: the tensor-core path (16 rows), the GEMV (3 rows), then scale rows of 3 and
    # 5 int32 (K = 384, 640: not a multiple of 4 groups) on both paths
    for seed, R, K, N in ((21, 16, 3584, 4608), (22, 3, 18944, 3584), (23, 5, 384, 1000), (24, 40, 640, 256),
                          (25, 2, 640, 384)):
        y, t, y_ref, t_ref = _linear_pair(torch, L, seed, R, K, N)
        assert np.array_equal(t, t_ref), (R, K, N)
        assert np.array_equal(y, y_ref), (R, K, N)


def test_noalloc_linear_on_a_second_device():
    """Per-device state (the array's address, the kernels' shared-memory attributes) is set up for
    each device it is used on: the same calls on GPU 1 after GPU 0 in one process."""
    torch, L = _setup()
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    for dev in (0, 1):
        with torch.cuda.device(dev):
            for seed, R, K, N in ((31, 4, 18944, 3584), (32, 16, 3584, 4608)):
                y, t, y_ref, t_ref = _linear_pair(torch, L, seed, R, K, N)
                assert np.array_equal(t, t_ref) and np.array_equal(y, y_ref), (dev, R, K, N)


def test_noalloc_rejects_oversize_requests():
    torch, L = _setup()
    big_r = 4096
    K = 3584                                              # 4096 * 3584 > the fixed array
    rc = L.lib.exb_linear_g128_noalloc(ctypes.c_void_p(16), big_r, K, ctypes.c_void_p(16), ctypes.c_void_p(16), None,
                                       128, ctypes.c_void_p(16), None, None)
    assert rc == 1
    assert b"exceeds the fixed scratch" in L.lib.exb_last_error()
    rc = L.lib.exb_linear_g128_noalloc(ctypes.c_void_p(16), 1, 25728, ctypes.c_void_p(16), ctypes.c_void_p(16), None,
                                       128, ctypes.c_void_p(16), None, None)
    assert rc == 1
    assert b"exceeds 25600" in L.lib.exb_last_error()
