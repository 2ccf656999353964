// Shared device helpers for the exact integer engine (sm_100a).
//
// Integer semantics follow the reference program exactly (exact_llm.py:25-46, :97-124 of
// novain-shibu/exact-llm; SPEC.md:18-28).  All int64 arithmetic wraps modulo 2^64, like
// numpy's, so every result is bit-identical to the reference's numpy int64 result.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#define EXB_DEV __device__ __forceinline__

namespace exb {

// error bits reported through the engine's device error word
enum : int {
  ERR_V_RANGE = 1,        // |V| >= 2^31: the int32 V cache cannot hold the value exactly
  ERR_WAIT_TIMEOUT = 2,   // a bounded device wait gave up
  ERR_FREIVALDS = 4,      // a Freivalds self-check failed
  ERR_BOUNDS = 8,         // an index/size check failed inside a kernel
  ERR_SHIFT_RANGE = 16,   // a shift count outside [-63, 63] (numpy semantics not representable)
};

// round-half-up arithmetic shift right (n > 0); n <= 0 is a left shift (exact_llm.py:25-34).
// Sum and left shift are done in uint64 so overflow wraps exactly like numpy int64.
EXB_DEV int64_t shr64(int64_t a, int n) {
  if (n <= 0) {
    int m = -n;
    return m >= 64 ? 0 : (int64_t)((uint64_t)a << m);
  }
  if (n >= 64) return a < 0 ? -1 : 0;                 // only reachable for pathological inputs
  uint64_t s = (uint64_t)a + (1ull << (n - 1));
  return ((int64_t)s) >> n;
}

// shr64 for a shift count known to lie in [0, 63]: branch-free (same result as shr64 there)
EXB_DEV int64_t shr_nn(int64_t a, int n) {
  const uint64_t bias = n > 0 ? (1ull << ((n - 1) & 63)) : 0ull;
  return ((int64_t)((uint64_t)a + bias)) >> n;
}

// bit length of a non-negative value (exact_llm.py:35-40)
EXB_DEV int bitlen64(uint64_t m) { return m ? 64 - __clzll((long long)m) : 0; }

EXB_DEV uint64_t uabs64(int64_t a) { return a < 0 ? (uint64_t)0 - (uint64_t)a : (uint64_t)a; }

// floor division by a positive divisor (numpy // on int64)
EXB_DEV int64_t floordiv64(int64_t a, int64_t b) {
  int64_t q = a / b;
  int64_t r = a - q * b;
  return (r != 0 && a < 0) ? q - 1 : q;
}

// floor(a / b) for b > 0, exact for every int64 a: a double-precision estimate, a second
// estimate on the (small) remainder, then integer corrections until 0 <= a - q*b < b.  About 30
// instructions instead of the ~hundreds of a software 64-bit division.
EXB_DEV int64_t floordiv_fast(int64_t a, int64_t b) {
  const double db = (double)b;
  int64_t q = (int64_t)floor(__ll2double_rn(a) / db);
  int64_t r = (int64_t)((uint64_t)a - (uint64_t)q * (uint64_t)b);
  q += (int64_t)floor(__ll2double_rn(r) / db);
  r = (int64_t)((uint64_t)a - (uint64_t)q * (uint64_t)b);
  for (int i = 0; i < 4 && r < 0; ++i) { q -= 1; r += b; }
  for (int i = 0; i < 4 && r >= b; ++i) { q += 1; r -= b; }
  return q;
}

// floor(a / b) for b > 0 with a precomputed inv = 1.0 / b: the same estimate + exact integer
// correction as floordiv_fast, with multiplications instead of double divisions.
EXB_DEV int64_t floordiv_recip(int64_t a, int64_t b, double inv) {
  int64_t q = (int64_t)floor(__ll2double_rn(a) * inv);
  int64_t r = (int64_t)((uint64_t)a - (uint64_t)q * (uint64_t)b);
  q += (int64_t)floor(__ll2double_rn(r) * inv);
  r = (int64_t)((uint64_t)a - (uint64_t)q * (uint64_t)b);
  for (int i = 0; i < 4 && r < 0; ++i) { q -= 1; r += b; }
  for (int i = 0; i < 4 && r >= b; ++i) { q += 1; r -= b; }
  return q;
}

// floor(sqrt(double(n))) with one correction step each way (exact_llm.py:97-99)
EXB_DEV int64_t isqrt_ref(int64_t n) {
  int64_t r = (int64_t)floor(sqrt(__ll2double_rn(n)));
  if (r * r > n) r -= 1;
  if ((r + 1) * (r + 1) <= n) r += 1;
  return r;
}

// qrow clip bound (exact_llm.py:41-46)
constexpr int64_t QLIM = 32767;
EXB_DEV int qrow_shift(uint64_t amax) { int s = bitlen64(amax) - 15; return s > 0 ? s : 0; }
EXB_DEV int16_t qrow_value(int64_t x, int s) {
  int64_t v = shr_nn(x, s);                        // 0 <= s <= 49 (qrow_shift of a 64-bit max)
  v = v > QLIM ? QLIM : (v < -QLIM ? -QLIM : v);
  return (int16_t)v;
}

// exp table lookup for the integer softmax (exact_llm.py:109-115); d >= 0
constexpr int EXP_LEN = 256 * 40 + 2;
EXB_DEV int64_t exp_lookup(const int32_t* __restrict__ T, int64_t d) {
  if (d >= (40ll << 16)) return 0;
  int64_t i = d >> 8;
  if (i > EXP_LEN - 2) i = EXP_LEN - 2;
  int64_t fr = d & 255;
  int64_t a = T[i], b = T[i + 1];
  return a - shr64((a - b) * fr, 8);
}

// SiLU / sigmoid tables on [-16, 16) at 1/256 steps (exact_llm.py:118-124; moe_exact_kaggle.py:420-424)
constexpr int SILU_LEN = 32 * 256 + 2;
EXB_DEV int64_t table_interp(const int32_t* __restrict__ T, int64_t x, int64_t hi_value) {
  const int64_t lo = -(16ll << 16), hi = (16ll << 16);
  if (x >= hi) return hi_value;
  if (x < lo) return 0;
  int64_t t = x + hi;                       // clip is a no-op inside the range
  int64_t i = t >> 8, fr = t & 255;
  int64_t a = T[i], b = T[i + 1];
  return a + shr64((b - a) * fr, 8);
}
EXB_DEV int64_t isilu_dev(const int32_t* T, int64_t x) { return table_interp(T, x, x); }
EXB_DEV int64_t isig_dev(const int32_t* T, int64_t x) { return table_interp(T, x, 1ll << 16); }

// ---------------------------------------------------------------- warp / block reductions
// 64-bit warp max and sum from 32-bit single-instruction warp reductions (redux.sync)
EXB_DEV uint64_t warp_max_u64(uint64_t v) {
  const unsigned hi = __reduce_max_sync(0xffffffffu, (unsigned)(v >> 32));
  const unsigned lo = __reduce_max_sync(0xffffffffu, (unsigned)(v >> 32) == hi ? (unsigned)v : 0u);
  return ((uint64_t)hi << 32) | lo;
}
EXB_DEV uint64_t warp_sum_u64(uint64_t v) {
  // three 22-bit digits: a warp sum of each fits in 27 bits; recombined modulo 2^64
  const unsigned d0 = __reduce_add_sync(0xffffffffu, (unsigned)(v & 0x3fffffu));
  const unsigned d1 = __reduce_add_sync(0xffffffffu, (unsigned)((v >> 22) & 0x3fffffu));
  const unsigned d2 = __reduce_add_sync(0xffffffffu, (unsigned)(v >> 44));
  return (uint64_t)d0 + ((uint64_t)d1 << 22) + ((uint64_t)d2 << 44);
}
// ---------------------------------------------------------------- block reductions
template <int NT>
EXB_DEV uint64_t block_max_u64(uint64_t v, uint64_t* red) {
  for (int o = 16; o > 0; o >>= 1) { uint64_t w = __shfl_xor_sync(0xffffffffu, v, o); v = w > v ? w : v; }
  const int wid = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[wid] = v;
  __syncthreads();
  if (wid == 0) {
    v = lane < NT / 32 ? red[lane] : 0;
    for (int o = 16; o > 0; o >>= 1) { uint64_t w = __shfl_xor_sync(0xffffffffu, v, o); v = w > v ? w : v; }
    if (lane == 0) red[32] = v;
  }
  __syncthreads();
  return red[32];
}

template <int NT>
EXB_DEV int64_t block_sum_i64(int64_t v, uint64_t* red) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int wid = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[wid] = (uint64_t)v;
  __syncthreads();
  if (wid == 0) {
    v = lane < NT / 32 ? (int64_t)red[lane] : 0;
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) red[32] = (uint64_t)v;
  }
  __syncthreads();
  return (int64_t)red[32];
}

// ---------------------------------------------------------------- programmatic dependent launch
// Kernels launched with the PDL attribute may start while the previous kernel drains; they
// must call pdl_wait() before touching data the previous kernel produced.
#ifndef EXB_TIMELINE
EXB_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
EXB_DEV void tl_exit() {}
EXB_DEV void tl_start() {}
EXB_DEV void tl_point(int) {}
#else
// Timeline build (compiled with -DEXB_TIMELINE; never the shipped library): each kernel of a
// step stamps %globaltimer into slot `seq` of a device buffer -- earliest CTA arrival at the
// dependency wait, earliest CTA past it, latest CTA exit -- and the last CTA to exit advances
// `seq`.  A kernel's successors wait for its completion, so slot n is the n-th kernel.
constexpr int TL_SLOTS = 4096;
struct TlBuf {
  unsigned long long seq, cnt, pad[2];
  unsigned long long t[TL_SLOTS][8];      // enter (min), waited (min), exit (max), CTAs, enter (max),
                                          // waited (max), exit (min), spare
  unsigned long long pt[TL_SLOTS][16];    // in-kernel points: 0-7 min over CTAs, 8-15 max
};
static __device__ TlBuf* g_tlb = nullptr;
static __shared__ unsigned long long tl_slot;    // this kernel's slot, read once at the wait
static __shared__ TlBuf* tl_buf;                 // g_tlb, read once at the wait
EXB_DEV unsigned long long tl_now() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
EXB_DEV unsigned long long tl_seq() {
  return *reinterpret_cast<volatile unsigned long long*>(&g_tlb->seq) % TL_SLOTS;
}
EXB_DEV void tl_mark(unsigned long long t0) {
  if (threadIdx.x == 0 && threadIdx.y == 0) tl_buf = g_tlb;
  if (g_tlb && threadIdx.x == 0 && threadIdx.y == 0) {
    const unsigned long long q = tl_seq();
    tl_slot = q;
    const unsigned long long t1 = tl_now();
    atomicMin(&g_tlb->t[q][0], t0);
    atomicMin(&g_tlb->t[q][1], t1);
    atomicMax(&g_tlb->t[q][4], t0);
    atomicMax(&g_tlb->t[q][5], t1);
  }
}
EXB_DEV void pdl_wait() {
  const unsigned long long t0 = tl_now();
  asm volatile("griddepcontrol.wait;" ::: "memory");
  tl_mark(t0);
}
EXB_DEV void tl_start() { tl_mark(tl_now()); }     // kernels launched without a dependency wait
EXB_DEV void tl_point(int i) {                       // thread 0 of each CTA passed point i (0..7)
  if (threadIdx.x == 0 && threadIdx.y == 0) {
    const unsigned long long t = tl_now();
    TlBuf* b = tl_buf;
    if (!b) return;
    const unsigned long long q = tl_slot % TL_SLOTS;
    atomicMin(&b->pt[q][i], t);
    atomicMax(&b->pt[q][8 + i], t);
  }
}
EXB_DEV void tl_exit() {
  __syncthreads();
  if (g_tlb && threadIdx.x == 0 && threadIdx.y == 0) {
    const unsigned long long te = tl_now();      // stamp first: the slot read below has latency
    const unsigned long long q = tl_seq();
    atomicMax(&g_tlb->t[q][2], te);
    atomicMin(&g_tlb->t[q][6], te);
    atomicAdd(&g_tlb->t[q][3], 1ull);
    __threadfence();
    const unsigned long long nb = (unsigned long long)gridDim.x * gridDim.y * gridDim.z;
    if (atomicAdd(&g_tlb->cnt, 1ull) + 1 == nb) {
      atomicExch(&g_tlb->cnt, 0ull);
      __threadfence();
      atomicAdd(&g_tlb->seq, 1ull);
    }
  }
}
int tl_register(int (*install)(void*));
static int tl_install(void* p) { return cudaMemcpyToSymbol(g_tlb, &p, sizeof(p)) == cudaSuccess ? 0 : -1; }
static const int tl_registered = tl_register(&tl_install);
#endif
EXB_DEV void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
EXB_DEV void prefetch_l2_bulk(const void* p, uint32_t bytes) {
  // fire-and-forget L2 prefetch of a 16-byte aligned range (no completion to wait for)
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

EXB_DEV void set_err(int* err, int bit) { if (err) atomicOr(err, bit); }

// Freivalds primes p1 = 2^31 - 1, p2 = 2147483629 (experiments/gpu_engine_trace_verify_kaggle.py:782)
EXB_DEV unsigned long long fr_prime(int i) { return i ? 2147483629ull : 2147483647ull; }

}  // namespace exb

// ---------------------------------------------------------------- mbarrier + bulk async copy (sm_90+)
namespace exb {
EXB_DEV uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
EXB_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
EXB_DEV void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
EXB_DEV void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
EXB_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
EXB_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: gives up after ~`limit` polls (each try_wait may itself suspend for a while).
// Returns false on timeout; the caller records ERR_WAIT_TIMEOUT and stops.
EXB_DEV bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t limit = (1u << 24)) {
  for (uint32_t i = 0; i < limit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}
// global -> shared bulk copy (16-byte aligned addresses, size multiple of 16), completion counted
// in bytes on `bar`
EXB_DEV void bulk_g2s(void* dst_smem, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst_smem)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
// lane-private asynchronous copies global -> shared (completion tracked per thread in groups)
EXB_DEV void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
EXB_DEV void cp_async4(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
EXB_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
EXB_DEV void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }
EXB_DEV void named_sync(int id, int nthreads) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory"); }
}  // namespace exb
