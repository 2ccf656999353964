"""The reference's operator API for the hot path, backed by libexactb200.so.

``torch.ops.exact.gemv(x16, wT, Mg)`` is the operator the reference's engine calls for every
batch-1 group-128 linear (experiments/speed_fair_kaggle.py:698-702, caller TLinG.__call__ at
:737-738):

    x16  int16 (K,)      the quantised activation row
    wT   int8  (N, K)    weights, one contiguous K-byte row per output
    Mg   int64 (N, K/128) group scales
    ->   int64 (N,)      out[n] = sum_g Mg[n, g] * sum_{k in g} x16[k] * wT[n, k]   (exact)

As in the reference, the output is allocated by the op, the kernel runs on the current CUDA
stream, there is no host synchronisation (the op can be captured in a CUDA graph) and the fake
(meta) implementation gives the output shape for tracing.  Unlike the reference, shapes, dtypes,
devices and alignment are checked and a failing launch raises.  Importing this module registers
the op; it needs torch.
"""
import torch

from ._lib import check, lib


def _check_args(x16, wT, Mg):
    if x16.dtype != torch.int16 or wT.dtype != torch.int8 or Mg.dtype != torch.int64:
        raise TypeError("exact::gemv wants x16 int16, wT int8, Mg int64")
    if x16.dim() != 1 or wT.dim() != 2 or Mg.dim() != 2:
        raise ValueError("exact::gemv wants x16 (K,), wT (N, K), Mg (N, K/128)")
    N, K = wT.shape
    if K % 128 or x16.shape[0] != K or tuple(Mg.shape) != (N, K // 128):
        raise ValueError(f"exact::gemv shapes: x16 {tuple(x16.shape)}, wT {tuple(wT.shape)}, Mg {tuple(Mg.shape)}"
                         " (K a multiple of 128)")
    return N, K


@torch.library.custom_op("exact::gemv", mutates_args=())
def gemv(x16: torch.Tensor, wT: torch.Tensor, Mg: torch.Tensor) -> torch.Tensor:
    N, K = _check_args(x16, wT, Mg)
    if not (x16.is_cuda and wT.device == x16.device and Mg.device == x16.device):
        raise ValueError("exact::gemv runs on one CUDA device (all three tensors on it)")
    x16, wT, Mg = x16.contiguous(), wT.contiguous(), Mg.contiguous()
    out = torch.empty((N,), dtype=torch.int64, device=x16.device)
    stream = torch.cuda.current_stream(x16.device).cuda_stream
    with torch.cuda.device(x16.device):
        check(lib.exb_gemv(x16.data_ptr(), wT.data_ptr(), Mg.data_ptr(), K, N, out.data_ptr(), stream))
    return out


@gemv.register_fake
def _gemv_fake(x16, wT, Mg):
    return torch.empty((wT.shape[0],), dtype=torch.int64, device=x16.device)
