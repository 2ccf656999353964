// Fused tensor-parallel exchanges of the decode step.
//
// Every rank owns one exchange area (inside its one-shot all-reduce buffer), mapped into every other
// rank's address space with CUDA IPC:
//   max words  [2: amax_o, amax_h][size: source rank][TPX_ROWS]            uint64 = epoch << 8 | bitlen
//   sum slots  [2: o, down][size: source rank][TPX_ROWS * D]               int64
//   flags      [4: exchange type][size: source rank]                        uint64 (epoch)
// MAX exchanges (a row's max |x|, needed only for the qrow shift max(bitlen - 15, 0), and the
// bit length of a max is the max of the bit lengths): the producing kernel's last CTA stores one
// 64-bit word per row, epoch and bit length together, into every rank's area; the word is its own
// flag, so no fence is needed.  SUM exchanges (a row-split linear's partial sums): the producing
// kernel's epilogue stores its values into slot [source = its rank] of every rank's area (plain
// stores through the peer mappings), and its last CTA, elected with an atomic ticket after every
// CTA's device-scope fence, raises flag [type][its rank] in every peer's area with the exchange's
// epoch (a system-scope fence, then a release store).  The consuming kernel waits (bounded) until
// every peer's word / flag has reached the epoch, then reduces its own area's slots: integer MAX
// and SUM, order-independent, so the result is bit-identical to NCCL's and to one GPU's.
//
// Epochs: each rank counts its exchanges per type in local memory (the producer's last CTA
// increments; the consumer, launched after the producer on the same stream, reads the count) and
// every rank makes the same exchanges in the same order, so the counts agree.  One slot set per
// type suffices: a rank writes exchange k + 1 of a type only after it consumed another exchange that
// a peer produced after that peer had consumed exchange k (decode layer order norm1 -> q|k|v ->
// attention -> o -> norm2 -> gate|up -> down).
#pragma once
#include "common.cuh"
#include "exb_internal.h"

namespace exb {

constexpr unsigned TPX_SPIN_LIMIT = 1u << 21;      // flag polls (back-off to 1 us): about 2 s

EXB_DEV unsigned long long ld_acquire_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
EXB_DEV void st_release_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

EXB_DEV void st_relaxed_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// `which`: 0 = amax_o / o, 1 = amax_h / down
EXB_DEV unsigned long long* tpx_max_slot(const TpX& x, int q, int which, int src) {
  return reinterpret_cast<unsigned long long*>(x.base[q]) + ((size_t)which * x.size + src) * TPX_ROWS;
}
EXB_DEV int64_t* tpx_sum_slot(const TpX& x, int q, int which, int src) {
  return reinterpret_cast<int64_t*>(x.base[q]) + (size_t)2 * x.size * TPX_ROWS +
         ((size_t)which * x.size + src) * TPX_ROWS * x.D;
}
EXB_DEV unsigned long long* tpx_flag(const TpX& x, int q, int type, int src) {
  return reinterpret_cast<unsigned long long*>(x.base[q]) + (size_t)2 * x.size * TPX_ROWS +
         (size_t)2 * x.size * TPX_ROWS * x.D + (size_t)type * x.size + src;
}

// Producer, last CTA, every thread: count the exchange and raise this rank's flag of `type` in every
// peer's area.  The CTA barrier orders the slot stores of this CTA's threads (and, through the
// ticket, those of every other CTA) before each signalling thread's system-scope fence.
EXB_DEV void tpx_signal(const TpX& x, int type) {
  __shared__ unsigned long long e_s;
  if (threadIdx.x == 0) {
    e_s = x.ep[type] + 1;
    x.ep[type] = e_s;
  }
  __syncthreads();
  if ((int)threadIdx.x < x.size && (int)threadIdx.x != x.rank) {
    __threadfence_system();
    st_release_sys_u64(tpx_flag(x, threadIdx.x, type, x.rank), e_s);
  }
}

// Producer, last CTA, every thread: the final rows of a MAX exchange (epoch and bit length in one
// word per row) into every rank's area.
EXB_DEV void tpx_publish_max(const TpX& x, int type, const unsigned long long* amax, int R) {
  __shared__ unsigned long long e_s;
  if (threadIdx.x == 0) {
    e_s = x.ep[type] + 1;
    x.ep[type] = e_s;
  }
  __syncthreads();
  const int which = type == TPX_AMAX_O ? 0 : 1;
  if ((int)threadIdx.x < R) {
    const unsigned long long w = e_s << 8 | (unsigned long long)bitlen64(__ldcg(amax + threadIdx.x));
    for (int q = 0; q < x.size; ++q) st_relaxed_sys_u64(tpx_max_slot(x, q, which, x.rank) + threadIdx.x, w);
  }
}

// Consumer, every thread of the CTA: wait until every peer's contribution to the exchange of `type`
// this rank counted last has arrived (the flag of a SUM exchange, the R row words of a MAX exchange).
// Bounded: on timeout the error word gets ERR_WAIT_TIMEOUT and the caller goes on with whatever the
// slots hold (the step's result is then invalid and the host reports the error).
EXB_DEV void tpx_wait(const TpX& x, int type, int R) {
  __shared__ int timeout_s;
  if (threadIdx.x == 0) timeout_s = 0;
  __syncthreads();
  const bool is_max = type == TPX_AMAX_O || type == TPX_AMAX_H;
  const int per = is_max ? R : 1;                       // words to watch per peer
  const int q = threadIdx.x / per, r = threadIdx.x - q * per;
  if (q < x.size && q != x.rank) {
    const unsigned long long e = __ldcg(x.ep + type);
    const unsigned long long* f = is_max ? tpx_max_slot(x, x.rank, type == TPX_AMAX_O ? 0 : 1, q) + r
                                         : tpx_flag(x, x.rank, type, q);
    unsigned spins = 0;
    while ((is_max ? ld_acquire_sys_u64(f) >> 8 : ld_acquire_sys_u64(f)) < e) {
      if (++spins > TPX_SPIN_LIMIT) {
        timeout_s = 1;
        break;
      }
      if (spins > 64) __nanosleep(spins > 4096 ? 1024 : 64);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0 && timeout_s) set_err(x.err, ERR_WAIT_TIMEOUT);
}

// Consumer: row r's qrow shift from a MAX exchange (after tpx_wait): max(bitlen(max over ranks) - 15, 0)
EXB_DEV int tpx_shift(const TpX& x, int which, int r) {
  int b = 0;
  for (int q = 0; q < x.size; ++q) {
    const int v = (int)(__ldcg(tpx_max_slot(x, x.rank, which, q) + r) & 255);
    b = v > b ? v : b;
  }
  return b > 15 ? b - 15 : 0;
}

}  // namespace exb
