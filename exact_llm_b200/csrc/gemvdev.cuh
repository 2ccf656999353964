// Device pieces of the exact GEMV shared by the standalone GEMV kernels (gemv.cu) and the
// persistent decode-step kernel (step.cu): the streaming weight load, the 16-MAC int16 x int8
// dot product, the requantisation, the per-column epilogues and the warp reduction.
#pragma once
#include "common.cuh"
#include "exb_internal.h"

namespace exb {

EXB_DEV int4 ldg_stream(const int4* p) {
  int4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.s32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// 16 int16 activations (xa: 0..7, xb: 8..15, packed in pairs) times 16 int8 weights; two
// independent dp2a chains halve the dependent latency
EXB_DEV int dot16(const int4 w, const int4 xa, const int4 xb) {
  int s = 0, t = 0;
  s = __dp2a_lo(xa.x, w.x, s); t = __dp2a_lo(xb.x, w.z, t);
  s = __dp2a_hi(xa.y, w.x, s); t = __dp2a_hi(xb.y, w.z, t);
  s = __dp2a_lo(xa.z, w.y, s); t = __dp2a_lo(xb.z, w.w, t);
  s = __dp2a_hi(xa.w, w.y, s); t = __dp2a_hi(xb.w, w.w, t);
  return s + t;
}

EXB_DEV unsigned long long mod_p(int64_t v, unsigned long long P) {
  int64_t m = v % (int64_t)P;
  return (unsigned long long)(m < 0 ? m + (int64_t)P : m);
}

// requant of one accumulator (group: shr(tot, 28-s); per-channel with the drop rule proven
// inactive for every input: shr(acc * M, 28 - s))
EXB_DEV int64_t requant1(const LinW& L, int n, int64_t tot, int s) {
  int64_t y;
  if (L.Mg) y = shr64(tot, 28 - s);
  else y = shr64((int64_t)((uint64_t)tot * (uint64_t)L.Mc[n]), 28 - s);
  if (L.b) y = (int64_t)((uint64_t)y + (uint64_t)L.b[n]);
  return y;
}

// Per-(epilogue lane, activation row) accumulators, kept in shared memory to spare registers.
struct EpiState {
  unsigned long long frl[3][2];   // Freivalds left-hand side residue sums (segment, prime)
  uint64_t omax;                  // max |output| (SwiGLU), max |x_new| (residual statistics)
  uint64_t ssq;                   // sum of x_new^2 (residual statistics; exact while max |x_new| < 2^24)
  int64_t best_v;                 // greedy argmax value / index
  int best_n;
};

// Epilogue of one output unit (1 column, or a gate/up pair) for activation row r.
// LEAN: no Freivalds or residual row statistics; HEADA: the greedy argmax (the launch guarantees
// nothing compiled out is asked for)
template <int RPU, bool LEAN = false, bool HEADA = !LEAN>
EXB_DEV void unit_epilogue(const GemvArgs& a, int ug, int r, const int64_t* t2, int sh, EpiState& E) {
  uint64_t& omax = E.omax;
  unsigned long long (&frl)[3][2] = E.frl;
  int64_t& best_v = E.best_v;
  int& best_n = E.best_n;
  if (RPU == 2) {
    // SwiGLU pair: fused row 2u = gate u, 2u + 1 = up u (exact_llm.py:179)
    const int64_t yg = requant1(a.L, 2 * ug, t2[0], sh);
    const int64_t yu = requant1(a.L, 2 * ug + 1, t2[RPU - 1], sh);
    const int64_t hv = shr64((int64_t)((uint64_t)isilu_dev(a.silu_t, yg) * (uint64_t)yu), 16);
    a.out[(size_t)r * a.ldo + ug] = hv;
    const uint64_t ah = uabs64(hv);
    omax = ah > omax ? ah : omax;
    if (a.raw) a.raw[(size_t)r * a.ldr + ug] = t2[0];
    if (a.raw2) a.raw2[(size_t)r * a.ldr + ug] = t2[RPU - 1];
    if (!LEAN && a.fr_nseg) {
      const int I = a.L.N / 2;
#pragma unroll
      for (int pi = 0; pi < 2; ++pi) {
        frl[0][pi] += mod_p(t2[0], fr_prime(pi)) * (unsigned long long)a.fr_r[0][pi * I + ug] % fr_prime(pi);
        frl[1][pi] += mod_p(t2[RPU - 1], fr_prime(pi)) * (unsigned long long)a.fr_r[1][pi * I + ug] % fr_prime(pi);
      }
    }
    return;
  }
  const int n = ug;
  const int64_t t = t2[0];
  if (a.raw) a.raw[(size_t)r * a.ldr + n] = t;
  if (!LEAN && a.fr_nseg) {
    const int sg = (a.fr_nseg > 2 && n >= a.fr_seg_start[2]) ? 2 : (a.fr_nseg > 1 && n >= a.fr_seg_start[1]) ? 1 : 0;
    const int ncols = (sg + 1 < a.fr_nseg ? a.fr_seg_start[sg + 1] : a.L.N) - a.fr_seg_start[sg];
    const int loc = n - a.fr_seg_start[sg];
#pragma unroll
    for (int pi = 0; pi < 2; ++pi) {
      const unsigned long long v = mod_p(t, fr_prime(pi)) * (unsigned long long)a.fr_r[sg][pi * ncols + loc] % fr_prime(pi);
      if (sg == 0) frl[0][pi] += v; else if (sg == 1) frl[1][pi] += v; else frl[2][pi] += v;
    }
  }
  if (a.epi == EPI_RAW) return;
  const int64_t y = requant1(a.L, n, t, sh);
  if (a.epi == EPI_RESID) {
    // the residual row may have been written by another CTA of a persistent kernel: read it from L2
    int64_t* o = a.out + (size_t)r * a.ldo + n;
    const int64_t xn = (int64_t)((uint64_t)__ldcg(reinterpret_cast<const long long*>(o)) + (uint64_t)y);
    *o = xn;
    if (!LEAN && a.nstat_out) {
      const uint64_t ax = uabs64(xn);
      omax = ax > omax ? ax : omax;
      E.ssq += (uint64_t)xn * (uint64_t)xn;          // wraps harmlessly when max |x_new| >= 2^24 (unused then)
    }
  } else if (a.out) {
    a.out[(size_t)r * a.ldo + n] = y;
  }
  if (HEADA && a.epi == EPI_HEAD && (y > best_v || (y == best_v && n < best_n))) {
    best_v = y;
    best_n = n;
  }
}

// Sum V int64 values over the warp by recursive halving; payload of P int64 per value.
// On return lane l holds the totals of value (l / (32 / V)).
template <int V, int P>
EXB_DEV void warp_reduce_halving(int64_t (&v)[V][P]) {
  const int lane = threadIdx.x & 31;
  int cnt = V;
#pragma unroll
  for (int step = 16; step >= 1; step >>= 1) {
    if (cnt > 1) {
      const int half = cnt >> 1;
      const bool upper = (lane & step) != 0;
#pragma unroll
      for (int i = 0; i < V / 2; ++i) {
        if (i < half) {
#pragma unroll
          for (int p = 0; p < P; ++p) {
            const int64_t send = upper ? v[i][p] : v[i + half][p];
            const int64_t keep = upper ? v[i + half][p] : v[i][p];
            v[i][p] = (int64_t)((uint64_t)keep + (uint64_t)__shfl_xor_sync(0xffffffffu, send, step));
          }
        }
      }
      cnt = half;
    } else {
#pragma unroll
      for (int p = 0; p < P; ++p)
        v[0][p] = (int64_t)((uint64_t)v[0][p] + (uint64_t)__shfl_xor_sync(0xffffffffu, v[0][p], step));
    }
  }
}

}  // namespace exb
