// One-shot all-reduce over NVLink peer memory for the tensor-parallel decode step.
//
// Each rank owns one device buffer, mapped into every other rank's address space with CUDA IPC.
// A call reduces n values (uint64 MAX, int64 SUM or int32 MIN) over the ranks: every CTA of the
// kernel takes a fixed slice of CH elements, stores its slice of the local vector into its slot
// of every peer's buffer (plain stores through the peer mapping), fences at system scope and
// raises its flag in every peer's buffer; then it waits until every peer's flag for this slice
// has arrived in its own buffer and reduces the slots locally.  Integer MAX / SUM / MIN are
// order-independent, so the result is bit-identical to NCCL's (and to one GPU's).
//
// Flags carry an epoch: each CTA slice keeps its own call counter in local memory, every rank
// makes the same calls in the same order, so the epochs agree.  Two buffer sets alternate by
// epoch parity: a rank can run at most one call ahead of a peer on a slice (it needs the peer's
// contribution to finish a call), so the set it writes is never the one the peer still reads.
// Every wait is bounded: on timeout the CTA records ERR_WAIT_TIMEOUT in the error word and
// returns (the step's result is then invalid and the host reports the error).
#include "common.cuh"
#include "exb_internal.h"
#include "tpx.cuh"

namespace exb {

constexpr int TPC_THREADS = 256;
constexpr unsigned TPC_SPIN_LIMIT = 1u << 21;      // flag polls (back-off to 1 us): about 2 s

// buffer layout of one rank: data[2][nblk][size][CH] (8-byte words), then flags[2][nblk][size]
EXB_DEV unsigned long long* tpc_data(const TpComm& c, int q, int set, int blk, int slot) {
  return reinterpret_cast<unsigned long long*>(c.base[q]) + (((size_t)set * c.nblk + blk) * c.size + slot) * TPC_CH;
}
EXB_DEV unsigned long long* tpc_flag(const TpComm& c, int q, int set, int blk, int slot) {
  return reinterpret_cast<unsigned long long*>(c.base[q]) + (size_t)2 * c.nblk * c.size * TPC_CH +
         ((size_t)set * c.nblk + blk) * c.size + slot;
}

// op: 0 uint64 max, 1 int64 sum, 2 int32 min (values widened to 8-byte words), 3 int64 max.  With `resid`
// (int64 sum): x[r, j] += shr(sum, 28 - xs[r]) (+ b[j]) for element i = r * N + j, the residual
// update of a row-split linear, instead of writing dst.
__global__ void __launch_bounds__(TPC_THREADS) k_tp_allreduce(TpComm c, const void* src, void* dst, int n, int op,
                                                             TpResid rz) {
  const int blk = blockIdx.x, tid = threadIdx.x;
  const int i0 = blk * TPC_CH, i1 = min(n, i0 + TPC_CH);
  __shared__ unsigned long long e_s;
  __shared__ int timeout_s;
  // launched as a programmatic dependent: wait for the producer of `src`, then let the next kernel
  // launch at once (its CTAs stage their weights while this exchange crosses NVLink)
  pdl_wait();
  pdl_launch_dependents();
  if (tid == 0) {
    e_s = c.epoch[blk] + 1;
    timeout_s = 0;
  }
  __syncthreads();
  const unsigned long long e = e_s;
  const int set = (int)(e & 1);
  auto word = [&](int i) -> unsigned long long {
    if (op == 2) return (unsigned long long)(long long)reinterpret_cast<const int32_t*>(src)[i];
    return reinterpret_cast<const unsigned long long*>(src)[i];
  };
  // 1. this slice of the local vector into this rank's slot of every peer's buffer
  for (int q = 0; q < c.size; ++q) {
    if (q == c.rank) continue;
    unsigned long long* d = tpc_data(c, q, set, blk, c.rank);
    for (int i = i0 + tid; i < i1; i += TPC_THREADS) d[i - i0] = word(i);
  }
  // the CTA barrier orders every thread's stores before the signalling threads' system-scope fence
  // and release store (one fence per peer flag, not one per thread)
  __syncthreads();
  if (tid < c.size && tid != c.rank) {
    __threadfence_system();
    st_release_sys_u64(tpc_flag(c, tid, set, blk, c.rank), e);
  }
  // 2. wait for every peer's slice of this call (bounded)
  if (tid < c.size && tid != c.rank) {
    const unsigned long long* f = tpc_flag(c, c.rank, set, blk, tid);
    unsigned spins = 0;
    while (ld_acquire_sys_u64(f) < e) {
      if (++spins > TPC_SPIN_LIMIT) {
        timeout_s = 1;
        break;
      }
      if (spins > 64) __nanosleep(spins > 4096 ? 1024 : 64);
    }
  }
  __syncthreads();
  if (timeout_s) {
    if (tid == 0) {
      set_err(c.err, ERR_WAIT_TIMEOUT);
      c.epoch[blk] = e;
    }
    tl_exit();
    return;
  }
  // 3. reduce the slots locally
  for (int i = i0 + tid; i < i1; i += TPC_THREADS) {
    unsigned long long v = word(i);
    for (int q = 0; q < c.size; ++q) {
      if (q == c.rank) continue;
      const unsigned long long w = __ldcg(tpc_data(c, c.rank, set, blk, q) + (i - i0));
      if (op == 0) v = w > v ? w : v;
      else if (op == 1) v += w;
      else if (op == 2) v = (long long)w < (long long)v ? w : v;
      else v = (long long)w > (long long)v ? w : v;
    }
    if (rz.x) {
      const int r = i / rz.N, j = i - r * rz.N;
      const int sh = rz.amax ? qrow_shift(__ldcg(rz.amax + r)) : rz.xs[r];
      int64_t y = shr64((int64_t)v, 28 - sh);
      if (rz.b) y = (int64_t)((uint64_t)y + (uint64_t)rz.b[j]);
      int64_t* o = rz.x + (size_t)r * rz.ldx + j;
      *o = (int64_t)((uint64_t)*o + (uint64_t)y);
      if (rz.tot) rz.tot[(size_t)r * rz.ldt + j] = (int64_t)v;        // the trace records the full sum
    } else if (op == 2) {
      reinterpret_cast<int32_t*>(dst)[i] = (int32_t)(long long)v;
    } else {
      reinterpret_cast<unsigned long long*>(dst)[i] = v;
    }
  }
  __syncthreads();
  if (tid == 0) c.epoch[blk] = e;
  tl_exit();
}

cudaError_t launch_tp_allreduce(const TpComm& c, const void* src, void* dst, int n, int op, const TpResid& rz,
                                cudaStream_t st, bool pdl) {
  if (n <= 0) return cudaSuccess;
  const int nb = (n + TPC_CH - 1) / TPC_CH;
  if (nb > c.nblk || c.size > TPC_MAX_RANKS) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(nb);
  cfg.blockDim = dim3(TPC_THREADS);
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, k_tp_allreduce, c, src, dst, n, op, rz);
}

size_t tp_comm_bytes(int size, int nblk) {
  return ((size_t)2 * nblk * size * TPC_CH + (size_t)2 * nblk * size) * 8;
}

size_t tpx_bytes(int size, int D) {
  return ((size_t)2 * size * TPX_ROWS + (size_t)2 * size * TPX_ROWS * D + (size_t)4 * size) * 8;
}

}  // namespace exb
