// K3: exact group-128 linear on tcgen05 tensor cores, for many activation rows (prefill chunks,
// batched decode, the reference linear operator at M >= 16).
//
//   tot[t, n] = sum_g M[n, g] * sum_{k in g} xq[t, k] * W[n, k]        (int64, exact)
//   (experiments/speed_fair_kaggle.py:722-725 of novain-shibu/exact-llm; SPEC.md:18)
//
// int16 activations do not fit an int8 MMA, so each row is split into two int8 digit planes,
// xq = 256 * hi + lo with lo = xq & 255 (unsigned) and hi = xq >> 8 (signed).  Per 128-wide group
// the tensor core accumulates two int32 sums (kind::i8, A = W signed, B = lo unsigned / hi
// signed); |sum| <= 128 * 255 * 127 < 2^31, so both are exact, and acc_g = 256 * hi + lo is the
// reference's exact group sum (it fits int32: 128 * 32767 * 127 < 2^31).  The epilogue warps then
// form tot += acc_g * M[n, g] in int64 registers, one TMEM lane (= one output row n) per thread.
//
// Roles ("swap AB": the weights are the MMA's M side, the activation rows its N side):
//   warp 0  TMA producer: per group a 128 x 128-byte weight tile and two 64 x 128-byte digit
//           tiles (128-byte swizzle) into a 4-stage shared-memory ring
//   warp 1  TMEM allocation and the MMA issuer (one elected thread): 8 MMAs per group (2 digits
//           x 4 K-steps of 32) into a double-buffered TMEM accumulator
//   warps 2-5  epilogue: tcgen05.ld of both digit accumulators, int64 fold with the group scale,
//           and at the end requant / bias / residual / SwiGLU (exact_llm.py:41-46, 176-179)
// Every wait is bounded: a stuck barrier sets the error word, the roles stop, TMEM is freed.
#include <cuda.h>

#include "common.cuh"
#include "exb_internal.h"
#include "gemvdev.cuh"

namespace exb {

constexpr int TC_BM = 128;                              // output rows per tile (MMA M)
constexpr int TC_PAD = TC_PAD_ROWS;                     // activation rows are padded to this
constexpr int TC_STAGES = 4;
constexpr int TC_A_BYTES = TC_BM * 128;                 // one group of 128 weight rows
constexpr uint32_t TC_WAIT_LIMIT = 1u << 24;

// Tile geometry for BN activation rows per tile (MMA N = 8, 64 or 128).  Every epilogue thread owns
// one output row (TMEM lane) and CW activation columns; BN = 128 takes 16 epilogue warps (four per
// TMEM lane quarter, 32 columns each), so each scheduler has four folding warps to hide the TMEM
// load latency behind.
#ifndef EXB_TC_EPI16
#define EXB_TC_EPI16 1
#endif
template <int BN>
struct TcGeo {
  static constexpr int B_BYTES = BN * 128;              // one group of BN activation rows, one digit
  static constexpr int STAGE_BYTES = TC_A_BYTES + 2 * B_BYTES;
  static constexpr int EPI_WARPS = (BN == 128 && EXB_TC_EPI16) ? 16 : BN >= 64 ? 4 * (BN / 64) : 4;
  static constexpr int CW = BN * 4 / EPI_WARPS;         // columns per epilogue thread
  static constexpr int THREADS = 64 + 32 * EPI_WARPS;
  static constexpr int TMEM_COLS = 4 * BN < 32 ? 32 : 4 * BN;   // 2 buffers x 2 digits x BN
  static constexpr int SMEM = TC_STAGES * STAGE_BYTES + 1024;   // + alignment slack
};

struct TcArgs {
  int N = 0, K = 0, T = 0;
  int ldm = 0;
  const int32_t* Mg = nullptr;        // (N, ldm) group scales; nullptr: unscaled sums (per-channel linear)
  const int32_t* xs = nullptr;        // (T) activation row shifts
  const int64_t* bias = nullptr;
  int epi = EPI_RAW;                  // EPI_RAW, EPI_STORE, EPI_RESID, EPI_SWIGLU
  int64_t* out = nullptr; int ldo = 0;
  int64_t* raw = nullptr; int ldr = 0;
  int64_t* raw2 = nullptr;            // SwiGLU: raw sums of the up rows
  const int32_t* silu_t = nullptr;
  int* err = nullptr;
  // decode extras
  int act_fast = 0;                   // grid.x indexes activation tiles (CTAs resident together
                                      // share a weight tile, read from HBM once), grid.y weight tiles
  int persist = 0;                    // persistent grid: CTA c takes tiles c, c + gridDim.x, ... of the
  int ntn = 0, ntiles = 0;            // ntiles tiles (activation tiles fastest, ntn per weight tile)
  int ksplit = 1;                     // CTAs sharing one 128-row tile over the 128-groups
  int64_t* tot_buf = nullptr;         // (T, N) int64 partial sums (zero between uses)
  unsigned int* tickets = nullptr;    // (N / 128) last-CTA counters (zero between uses)
  unsigned long long* amax_out = nullptr;   // SwiGLU: per-row max |h| (atomicMax)
  unsigned long long* zero = nullptr; int nzero = 0;   // cleared by CTA (0, 0) for a later producer
};

// ---------------------------------------------------------------- PTX wrappers
EXB_DEV bool tc_wait(uint64_t* bar, uint32_t parity) {
  for (uint32_t i = 0; i < TC_WAIT_LIMIT; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}
EXB_DEV void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
EXB_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
EXB_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
EXB_DEV void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
EXB_DEV void tc_mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, bool accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}\n"
      ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"((uint32_t)accumulate)
      : "memory");
}
// 8 consecutive 32-bit TMEM columns of this thread's lane
EXB_DEV void tmem_ld8(uint32_t taddr, int32_t* v) {
  uint32_t r[8];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = (int32_t)r[i];
}
// 16 consecutive 32-bit TMEM columns of this thread's lane
EXB_DEV void tmem_ld16(uint32_t taddr, int32_t* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = (int32_t)r[i];
}
EXB_DEV void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// t + a * b with a 32 x 32 -> 64-bit product (one multiply-add; wraps modulo 2^64 like numpy)
EXB_DEV int64_t mad_wide(int32_t a, int32_t b, int64_t t) {
  int64_t d;
  asm("mad.wide.s32 %0, %1, %2, %3;" : "=l"(d) : "r"(a), "r"(b), "l"(t));
  return d;
}

// Shared-memory matrix descriptor: K-major operand in the 128-byte swizzled layout written by
// TMA (rows of 128 bytes, 8-row core groups 1024 bytes apart), advanced by 32 bytes per K-step.
EXB_DEV uint64_t tc_desc(const void* tile, int kstep) {
  const uint32_t addr = smem_u32(tile) + 32u * (uint32_t)kstep;
  return (uint64_t)((addr >> 4) & 0x3FFF) | (1ull << 16) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) |
         (2ull << 61);
}
// Instruction descriptor: int32 accumulate, A = signed int8 (weights), B = unsigned (low digit)
// or signed (high digit) int8, both K-major, M = 128, N = BN.
template <int BN>
__host__ __device__ constexpr uint32_t tc_idesc(bool b_signed) {
  return (2u << 4) | (1u << 7) | ((b_signed ? 1u : 0u) << 10) | ((uint32_t)(BN >> 3) << 17) |
         ((uint32_t)(TC_BM >> 4) << 24);
}

// final epilogue of one (activation row t, output row n) total; SwiGLU pairs sit in adjacent lanes
// (every lane of the warp calls this with the same t)
EXB_DEV void tc_finish(const TcArgs& a, int t, int n, int64_t v, bool live, uint64_t& hmax) {
  if (a.epi == EPI_SWIGLU) {
    const int sh = live ? a.xs[t] : 0;
    const int64_t y = shr64(v, 28 - sh);
    const int64_t other = __shfl_xor_sync(0xffffffffu, y, 1);
    const int64_t vother = __shfl_xor_sync(0xffffffffu, v, 1);
    if (live && !(n & 1)) {
      const int u = n >> 1;
      const int64_t hv = shr64((int64_t)((uint64_t)isilu_dev(a.silu_t, y) * (uint64_t)other), 16);
      a.out[(size_t)t * a.ldo + u] = hv;
      const uint64_t ah = uabs64(hv);
      hmax = ah > hmax ? ah : hmax;
      if (a.raw) a.raw[(size_t)t * a.ldr + u] = v;
      if (a.raw2) a.raw2[(size_t)t * a.ldr + u] = vother;
    }
    return;
  }
  if (!live) return;
  if (a.raw) a.raw[(size_t)t * a.ldr + n] = v;
  if (a.epi == EPI_RAW) return;
  int64_t y = shr64(v, 28 - a.xs[t]);
  if (a.bias) y = (int64_t)((uint64_t)y + (uint64_t)a.bias[n]);
  int64_t* o = a.out + (size_t)t * a.ldo + n;
  if (a.epi == EPI_RESID) *o = (int64_t)((uint64_t)__ldcg(reinterpret_cast<const long long*>(o)) + (uint64_t)y);
  else *o = y;
}

// per-row max |h| of a SwiGLU tile column: warp maximum, one atomic per warp
EXB_DEV void tc_publish_hmax(const TcArgs& a, int t, uint64_t v) {
  v = warp_max_u64(v);
  if ((threadIdx.x & 31) == 0 && v && t < a.T) atomicMax(a.amax_out + t, (unsigned long long)v);
}

// ---------------------------------------------------------------- the kernel
template <int BN>
__global__ void __launch_bounds__(TcGeo<BN>::THREADS, 1)
    k_gemm_tc(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmLo,
              const __grid_constant__ CUtensorMap tmHi, const TcArgs a) {
  using Geo = TcGeo<BN>;
  constexpr int B_BYTES = Geo::B_BYTES;
  constexpr int STAGE_BYTES = Geo::STAGE_BYTES;
  constexpr int TMEM_COLS = Geo::TMEM_COLS;
  constexpr int NEPI = 32 * Geo::EPI_WARPS;               // epilogue threads
  constexpr int CW = Geo::CW;
  extern __shared__ unsigned char smem_raw[];
  __shared__ uint64_t full[TC_STAGES], empty[TC_STAGES], accf[2], acce[2];
  __shared__ uint32_t tmem_base_sh;
  __shared__ int abort_sh, issued_sh, consumed_sh, last_sh;
  unsigned char* smem = reinterpret_cast<unsigned char*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool af = a.act_fast && a.ksplit <= 1;
  const int G = a.K >> 7;
  // Tiles of this CTA: one (from the grid position) or, with a persistent grid, tiles w0, w0 +
  // wstep, ... of the activation-fastest order.  Every role walks the same sequence; `it` counts
  // the CTA's (tile, 128-group) iterations, which index the stage ring and the TMEM buffers.
  const int w0 = a.persist ? (int)blockIdx.x : 0;
  const int wend = a.persist ? a.ntiles : 1;
  const int wstep = a.persist ? (int)gridDim.x : 1;
  auto tile_of = [&](int w, int& tm, int& tn, int& g0, int& ng) {
    int ks = 0;
    if (a.persist) {
      tn = w % a.ntn;
      tm = w / a.ntn;
    } else {
      tm = af ? (int)blockIdx.y : (int)blockIdx.x;
      tn = a.ksplit > 1 ? 0 : (af ? (int)blockIdx.x : (int)blockIdx.y);   // split-K: grid.y = K ranges
      ks = a.ksplit > 1 ? (int)blockIdx.y : 0;
    }
    g0 = (int)((long long)G * ks / a.ksplit);
    ng = (int)((long long)G * (ks + 1) / a.ksplit) - g0;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < TC_STAGES; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
    for (int b = 0; b < 2; ++b) { mbar_init(&accf[b], 1); mbar_init(&acce[b], NEPI); }
    abort_sh = 0; issued_sh = 0; consumed_sh = 0; last_sh = 0;
    mbar_fence_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_sh)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_sh;

  if (warp == 0) {
    // ---- TMA producer: the weight tiles of the first stages do not depend on the previous
    // kernel and go out before the programmatic-dependent-launch wait; activation digits after it
    if (lane == 0) {
      int tm, tn, g0, ng;
      tile_of(w0, tm, tn, g0, ng);
      const int pre = ng < TC_STAGES ? ng : TC_STAGES;
      for (int i = 0; i < pre; ++i) {
        unsigned char* st = smem + (size_t)i * STAGE_BYTES;
        mbar_expect_tx(&full[i], STAGE_BYTES);
        tma_load_2d(st, &tmA, (g0 + i) * 128, tm * TC_BM, &full[i]);
      }
      pdl_wait();
      for (int i = 0; i < pre; ++i) {
        unsigned char* st = smem + (size_t)i * STAGE_BYTES;
        tma_load_2d(st + TC_A_BYTES, &tmLo, (g0 + i) * 128, tn * BN, &full[i]);
        tma_load_2d(st + TC_A_BYTES + B_BYTES, &tmHi, (g0 + i) * 128, tn * BN, &full[i]);
      }
      *(volatile int*)&issued_sh = pre;
      // the ring runs on across tile boundaries: the next tile's first groups load while the
      // epilogue finishes the current one (on a fresh barrier the parity-1 wait returns at once)
      int it = pre, i = pre;
      for (int w = w0;;) {
        for (; i < ng; ++i, ++it) {
          const int s = it % TC_STAGES;
          if (!tc_wait(&empty[s], ((it / TC_STAGES) - 1) & 1)) {
            abort_sh = 1;
            set_err(a.err, ERR_WAIT_TIMEOUT);
            break;
          }
          if (*(volatile int*)&abort_sh) break;
          unsigned char* st = smem + (size_t)s * STAGE_BYTES;
          mbar_expect_tx(&full[s], STAGE_BYTES);
          tma_load_2d(st, &tmA, (g0 + i) * 128, tm * TC_BM, &full[s]);
          tma_load_2d(st + TC_A_BYTES, &tmLo, (g0 + i) * 128, tn * BN, &full[s]);
          tma_load_2d(st + TC_A_BYTES + B_BYTES, &tmHi, (g0 + i) * 128, tn * BN, &full[s]);
          *(volatile int*)&issued_sh = it + 1;
        }
        if (*(volatile int*)&abort_sh) break;
        w += wstep;
        if (w >= wend) break;
        tile_of(w, tm, tn, g0, ng);
        i = 0;
      }
    }
  } else if (warp == 1) {
    // ---- MMA issuer
    if (lane == 0) {
      const uint32_t id_lo = tc_idesc<BN>(false), id_hi = tc_idesc<BN>(true);
      int ntot = 0;                     // this CTA's (tile, group) iterations
      for (int w = w0; w < wend; w += wstep) {
        int tm, tn, g0, ng;
        tile_of(w, tm, tn, g0, ng);
        ntot += ng;
      }
      for (int i = 0; i < ntot; ++i) {
        const int s = i % TC_STAGES, b = i & 1;
        if (!tc_wait(&full[s], (i / TC_STAGES) & 1) || !tc_wait(&acce[b], ((i >> 1) & 1) ^ 1)) {
          abort_sh = 1;
          set_err(a.err, ERR_WAIT_TIMEOUT);
          break;
        }
        tc_fence_after();
        const unsigned char* st = smem + (size_t)s * STAGE_BYTES;
        const uint32_t d_lo = tmem + (uint32_t)(b * 2 * BN), d_hi = d_lo + BN;
#pragma unroll
        for (int k = 0; k < 4; ++k) tc_mma_i8(d_lo, tc_desc(st, k), tc_desc(st + TC_A_BYTES, k), id_lo, k > 0);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          tc_mma_i8(d_hi, tc_desc(st, k), tc_desc(st + TC_A_BYTES + B_BYTES, k), id_hi, k > 0);
        tc_commit(&empty[s]);           // the stage is free once these MMAs have read it
        tc_commit(&accf[b]);            // the group's accumulators are complete
        *(volatile int*)&consumed_sh = i + 1;
      }
    }
  } else {
    // ---- epilogue: warp w reads TMEM lanes 32 (w % 4) .. + 31 (thread = output row n) and the
    // CW accumulator columns [hc * CW, hc * CW + CW) of each digit
    pdl_wait();
    if (a.zero && blockIdx.x == 0 && blockIdx.y == 0)
      for (int i = (int)threadIdx.x - 64; i < a.nzero; i += NEPI) a.zero[i] = 0;
    const int q = warp & 3;
    const int hc = (warp - 2) >> 2;
    const int row = q * 32 + lane;
    bool ok = true;
    int it = 0;                         // this CTA's (tile, group) iterations so far
    for (int w = w0; w < wend && ok; w += wstep) {
      int tm, tn, g0, ng;
      tile_of(w, tm, tn, g0, ng);
      const int n = tm * TC_BM + row;
      int64_t tot[CW];
#pragma unroll
      for (int j = 0; j < CW; ++j) tot[j] = 0;
      const int32_t* mrow = a.Mg ? a.Mg + (size_t)n * a.ldm : nullptr;
      int32_t mnext = (mrow && ng > 0) ? __ldg(mrow + g0) : 1;
      for (int i = 0; i < ng; ++i, ++it) {
        const int b = it & 1;
        const int32_t mv = mnext;
        if (mrow && i + 1 < ng) mnext = __ldg(mrow + g0 + i + 1);
        // warp-uniform outcome: the TMEM loads below are .sync.aligned over the whole warp
        if (!__all_sync(0xffffffffu, tc_wait(&accf[b], (it >> 1) & 1))) {
          ok = false;
          set_err(a.err, ERR_WAIT_TIMEOUT);
          abort_sh = 1;
          break;
        }
        tc_fence_after();
        const uint32_t t_lo = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * 2 * BN + hc * CW);
        // TMEM columns per load: 16 where the registers allow (BN = 64), else 8 (the 16-warp epilogue
        // of BN = 128 runs at 96 registers per thread and would spill)
        constexpr int CH = (CW >= 16 && BN < 128) ? 16 : 8;
#pragma unroll
        for (int c = 0; c < CW / CH; ++c) {
          int32_t lo[CH], hi[CH];
          if constexpr (CH == 16) {
            tmem_ld16(t_lo + c * CH, lo);
            tmem_ld16(t_lo + BN + c * CH, hi);
          } else {
            tmem_ld8(t_lo + c * CH, lo);
            tmem_ld8(t_lo + BN + c * CH, hi);
          }
          tmem_wait_ld();
          if (c == CW / CH - 1) {
            tc_fence_before();
            mbar_arrive(&acce[b]);        // buffer b may be overwritten by the next-but-one group
          }
#pragma unroll
          for (int e = 0; e < CH; ++e)    // exact group sum 256 hi + lo (|.| < 2^30), times the scale
            tot[c * CH + e] = mad_wide(hi[e] * 256 + lo[e], mv, tot[c * CH + e]);
        }
      }
      if (w == w0) pdl_launch_dependents();
      // every epilogue thread reaches this point (finished or timed out): one decision for all
      named_sync(1, NEPI);
      ok = ok && !*(volatile int*)&abort_sh;
      ok = __all_sync(0xffffffffu, ok);
      named_sync(1, NEPI);
      if (ok && a.ksplit == 1) {
#pragma unroll
        for (int j = 0; j < CW; ++j) {
          const int t = tn * BN + hc * CW + j;
          uint64_t hm = 0;
          tc_finish(a, t, n, tot[j], t < a.T, hm);
          if (a.amax_out) tc_publish_hmax(a, t, hm);
        }
      } else if (ok) {
        // split-K: add this CTA's partial sums, the last CTA of the tile finishes it
#pragma unroll
        for (int j = 0; j < CW; ++j) {
          const int t = hc * CW + j;
          if (t < a.T) atomicAdd(reinterpret_cast<unsigned long long*>(a.tot_buf + (size_t)t * a.N + n),
                                 (unsigned long long)tot[j]);
        }
        __threadfence();
        named_sync(1, NEPI);
        if (threadIdx.x == 64) {
          const unsigned prev = atomicAdd(a.tickets + tm, 1u);
          last_sh = prev == (unsigned)(a.ksplit - 1);
          if (last_sh) a.tickets[tm] = 0;
        }
        named_sync(1, NEPI);
        if (last_sh) {
          __threadfence();
#pragma unroll
          for (int j = 0; j < CW; ++j) {
            const int t = hc * CW + j;
            int64_t v = 0;
            if (t < a.T) {
              int64_t* p = a.tot_buf + (size_t)t * a.N + n;
              v = (int64_t)__ldcg(reinterpret_cast<const long long*>(p));
              *p = 0;                     // ready for the next use
            }
            uint64_t hm = 0;
            tc_finish(a, t, n, v, t < a.T, hm);
            if (a.amax_out) tc_publish_hmax(a, t, hm);
          }
        }
      }
    }
  }
  // drain: on an aborted run wait (bounded) for the weight/digit copies that were issued but never
  // consumed and for the last MMA group, so nothing writes shared memory or TMEM after the exit
  __syncthreads();
  if (abort_sh && threadIdx.x == 32) {
    for (int g = consumed_sh; g < issued_sh; ++g) (void)tc_wait(&full[g % TC_STAGES], (g / TC_STAGES) & 1);
    if (consumed_sh > 0) {
      const int g = consumed_sh - 1;
      (void)tc_wait(&accf[g & 1], (g >> 1) & 1);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
  tl_exit();
}

// ---------------------------------------------------------------- digit planes
// lo = xq & 255 (as uint8), hi = xq >> 8 (int8); rows t >= T are zero (padding to a tile)
__global__ void k_digits(const int16_t* __restrict__ xq, int ldx, int T, int K, int Tpad, uint8_t* __restrict__ lo,
                         int8_t* __restrict__ hi) {
  const long long n = (long long)Tpad * K / 2;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const long long e = 2 * i;
    const int t = (int)(e / K), k = (int)(e - (long long)t * K);
    short2 v = make_short2(0, 0);
    if (t < T) v = *reinterpret_cast<const short2*>(xq + (size_t)t * ldx + k);
    reinterpret_cast<uchar2*>(lo)[i] = make_uchar2((uint8_t)(v.x & 255), (uint8_t)(v.y & 255));
    reinterpret_cast<char2*>(hi)[i] = make_char2((int8_t)(v.x >> 8), (int8_t)(v.y >> 8));
  }
  tl_exit();
}

// ---------------------------------------------------------------- host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// rows x cols bytes, row pitch `pitch` bytes, box of box_rows x 128 bytes, 128-byte swizzle
static bool make_map(CUtensorMap* m, const void* base, int rows, int cols, size_t pitch, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)pitch};
  const cuuint32_t box[2] = {128, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

size_t gemm_tc_digit_bytes(int T, int K) {
  const size_t Tpad = (size_t)(T + TC_PAD - 1) / TC_PAD * TC_PAD;
  return 2 * Tpad * (size_t)K;
}

cudaError_t launch_digits(const int16_t* xq, int ldx, int T, int K, void* digits, cudaStream_t st) {
  const int Tpad = (T + TC_PAD - 1) / TC_PAD * TC_PAD;
  uint8_t* lo = static_cast<uint8_t*>(digits);
  int8_t* hi = reinterpret_cast<int8_t*>(lo + (size_t)Tpad * K);
  const long long n = (long long)Tpad * K / 2;
  const int blocks = (int)((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096);
  k_digits<<<blocks, 256, 0, st>>>(xq, ldx, T, K, Tpad, lo, hi);
  return cudaGetLastError();
}

bool gemm_tc_supported(const LinW& L, int epi) {
  if (!L.Mg && epi != EPI_RAW) return false;      // per-channel linears: raw sums, requant elsewhere
  return L.w && L.K % 128 == 0 && L.N % TC_BM == 0 && ((uintptr_t)L.w & 15) == 0 &&
         (epi == EPI_RAW || epi == EPI_STORE || epi == EPI_RESID || epi == EPI_SWIGLU) && encode_fn() != nullptr;
}

template <int BN>
static cudaError_t tc_launch(dim3 grid, const CUtensorMap& mA, const CUtensorMap& mLo, const CUtensorMap& mHi,
                             const TcArgs& a, bool pdl, cudaStream_t st) {
  static DevOnce attr;                 // raised once to the full budget, never lowered
  if (!attr.done()) {
    cudaError_t e = cudaFuncSetAttribute(k_gemm_tc<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, TcGeo<BN>::SMEM);
    if (e != cudaSuccess) return e;
    attr.set();
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(TcGeo<BN>::THREADS);
  cfg.dynamicSmemBytes = TcGeo<BN>::SMEM;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, k_gemm_tc<BN>, mA, mLo, mHi, a);
}

// process-wide choice of the persistent grid for the multi-row GEMM (engine option "tcp")
#ifndef EXB_TC_PERSIST
#define EXB_TC_PERSIST 1
#endif
static int g_tc_persist = EXB_TC_PERSIST;
void gemm_tc_set_persist(int on) { g_tc_persist = on; }
static int tc_sm_count() {
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

cudaError_t launch_gemm_tc(const void* digits, int T, const LinW& L, const int32_t* xs, int epi, int64_t* out, int ldo,
                           int64_t* raw, int64_t* raw2, int ldr, const int32_t* silu_t, int* err, cudaStream_t st,
                           const TcDecode* dec, unsigned long long* amax_out) {
  if (!gemm_tc_supported(L, epi) || T <= 0) return cudaErrorInvalidValue;
  // activation-row tile: 8 for decode steps (digit planes of TC_DECODE_ROWS rows), else 64 / 128
  const int BN = dec ? 8 : (T > 64 ? 128 : 64);
  const int Tpad = dec ? TC_DECODE_ROWS : (T + TC_PAD - 1) / TC_PAD * TC_PAD;
  if (dec && (T > TC_DECODE_ROWS || dec->ksplit < 1 || (dec->ksplit > 1 && (!dec->tot_buf || !dec->tickets))))
    return cudaErrorInvalidValue;
  const uint8_t* lo = static_cast<const uint8_t*>(digits);
  const uint8_t* hi = lo + (size_t)Tpad * L.K;
  CUtensorMap mA, mLo, mHi;
  if (!make_map(&mA, L.w, L.N, L.K, (size_t)L.K, TC_BM) || !make_map(&mLo, lo, Tpad, L.K, (size_t)L.K, BN) ||
      !make_map(&mHi, hi, Tpad, L.K, (size_t)L.K, BN))
    return cudaErrorInvalidValue;
  TcArgs a;
  a.N = L.N; a.K = L.K; a.T = T; a.ldm = L.ldm; a.Mg = L.Mg; a.xs = xs; a.bias = L.b; a.epi = epi;
  a.out = out; a.ldo = ldo; a.raw = raw; a.ldr = ldr; a.raw2 = raw2; a.silu_t = silu_t; a.err = err;
  if (dec) {
    const int G = L.K / 128;
    a.ksplit = dec->ksplit < G ? dec->ksplit : G;
    a.tot_buf = dec->tot_buf; a.tickets = dec->tickets; a.amax_out = dec->amax_out;
    a.zero = dec->zero; a.nzero = dec->nzero;
    return tc_launch<8>(dim3(L.N / TC_BM, a.ksplit), mA, mLo, mHi, a, dec->pdl, st);
  }
  // activation tiles fastest: the CTAs resident together cover a few weight tiles x every
  // activation tile, so each weight byte comes from HBM once and the activations stay in L2
  a.act_fast = 1;
  a.amax_out = amax_out;                // SwiGLU: per-row max |h| (zero before the launch)
  const int ntn = BN == 128 ? Tpad / 128 : (T + 63) / 64, ntm = L.N / TC_BM;
  if (g_tc_persist) {
    // persistent grid: one CTA per SM walks the tiles in the same activation-fastest order, so
    // the TMA ring and the TMEM allocation carry over from tile to tile
    a.persist = 1; a.ntn = ntn; a.ntiles = ntn * ntm;
    const int grid = a.ntiles < tc_sm_count() ? a.ntiles : tc_sm_count();
    if (BN == 128) return tc_launch<128>(dim3(grid, 1), mA, mLo, mHi, a, false, st);
    return tc_launch<64>(dim3(grid, 1), mA, mLo, mHi, a, false, st);
  }
  if (BN == 128) return tc_launch<128>(dim3(ntn, ntm), mA, mLo, mHi, a, false, st);
  return tc_launch<64>(dim3(ntn, ntm), mA, mLo, mHi, a, false, st);
}

}  // namespace exb
