// Per-row integer operations as block-level device functions, shared by the standalone row
// kernels and by the "last CTA" tails of the GEMV and attention kernels.
//
//   norm_q   a = irms(x, g) (exact_llm.py:100-106), then xq, s = qrow(a) (:41-46)
//   quant    xq, s = qrow(x)
//   rope     RoPE of q and k (exact_llm.py:159-160), K-cache row quantisation + V cache write
//            (exact_torch.py:146-149), q row quantisation for the scores (exact_llm.py:173)
//
// Inputs written by other CTAs of the same kernel are read with ld.global.cg (L2), never
// through a possibly stale L1 line.
#pragma once
#include "common.cuh"
#include "exb_internal.h"

namespace exb {

EXB_DEV int64_t ld_cg(const int64_t* p) { return (int64_t)__ldcg(reinterpret_cast<const long long*>(p)); }

// Two-barrier block reductions for the latency-bound row operations: warp shuffles, one slot per
// warp in `buf` (NT/32 entries), one barrier, then every thread folds the slots itself.  A caller
// alternates two buffers between consecutive reductions (the barrier of reduction i+1 orders
// every read of reduction i's buffer before reduction i+2 writes it).
template <int NT>
EXB_DEV uint64_t block_max_fast(uint64_t v, uint64_t* buf) {
  v = warp_max_u64(v);
  if ((threadIdx.x & 31) == 0) buf[threadIdx.x >> 5] = v;
  __syncthreads();
  const int lane = threadIdx.x & 31;
  return warp_max_u64(lane < NT / 32 ? buf[lane] : 0);
}
template <int NT>
EXB_DEV uint64_t block_sum_fast(uint64_t v, uint64_t* buf) {
  v = warp_sum_u64(v);
  if ((threadIdx.x & 31) == 0) buf[threadIdx.x >> 5] = v;
  __syncthreads();
  const int lane = threadIdx.x & 31;
  return warp_sum_u64(lane < NT / 32 ? buf[lane] : 0);
}

// floor(a / b) for b > 0 when the quotient is known to be far below 2^50: one estimate with a
// precomputed reciprocal, then at most two exact integer corrections each way; any other case
// (never met for the operands below) takes the general exact routine.
EXB_DEV int64_t floordiv_small_q(int64_t a, int64_t b, double inv) {
  int64_t q = __double2ll_rz(__ll2double_rn(a) * inv);
  int64_t r = (int64_t)((uint64_t)a - (uint64_t)q * (uint64_t)b);
  if (r < 0) { q -= 1; r += b; }
  if (r < 0) { q -= 1; r += b; }
  if (r >= b) { q += 1; r -= b; }
  if (r >= b) { q += 1; r -= b; }
  if (r < 0 || r >= b) q = floordiv_recip(a, b, inv);
  return q;
}

// Row-constant divisor of irms: den = rt << k (exact_llm.py:105).  y = (x << 16) // den with
// numpy int64 semantics.  Fast path (|x| < 2^47, so x << 16 does not wrap, and rt << k < 2^62):
// floor division nests, y = ((x << 16) >> k) // rt with |(x << 16) >> k| < 2^41 and rt < 2^25,
// computed with a 64-bit reciprocal (high half of a 64 x 64 product) and one exact correction.
struct NormDiv {
  int64_t den, rt;
  uint64_t m;            // ~2^64 / rt, within 2^12 below the exact value
  double inv;            // 1 / den for the general path
  int k;
  bool fast;
};
EXB_DEV NormDiv make_norm_div(int64_t rt, int k) {
  NormDiv d;
  d.rt = rt; d.k = k;
  d.den = (int64_t)((uint64_t)rt << k);
  d.inv = __drcp_rn((double)d.den);
  d.fast = (bitlen64((uint64_t)rt) + k) <= 62;
  const double e = 18446744073709551616.0 / (double)rt;             // 2^64 / rt
  d.m = e >= 18446744073709549568.0 ? ~0ull : (uint64_t)e;           // rt = 1: saturate
  d.m = d.m > 4096 ? d.m - 4096 : 0;                                 // never above the exact value
  return d;
}
EXB_DEV int64_t norm_div(int64_t x, const NormDiv& d) {
  const uint64_t ax = uabs64(x);
  if (d.fast && ax < (1ull << 47)) {
    const int64_t n = ((int64_t)((uint64_t)x << 16)) >> d.k;         // floor((x << 16) / 2^k)
    const uint64_t an = uabs64(n);
    uint64_t q = __umul64hi(an, d.m);                                // floor(an / rt) - {0, 1, 2}
    uint64_t r = an - q * (uint64_t)d.rt;
    if (r >= (uint64_t)d.rt) { q += 1; r -= (uint64_t)d.rt; }
    if (r >= (uint64_t)d.rt) { q += 1; r -= (uint64_t)d.rt; }
    if (r >= (uint64_t)d.rt) { q += 1; r -= (uint64_t)d.rt; }
    return n >= 0 ? (int64_t)q : -(int64_t)q - (r != 0 ? 1 : 0);
  }
  return floordiv_recip((int64_t)((uint64_t)x << 16), d.den, d.inv);
}

// One row already staged in shared memory (`ys`, D int64; overwritten): irms + qrow
// (exact_llm.py:100-106 then :41-46).  `m` is this thread's partial max |x| over the elements
// it staged; `gs` holds the gains (D int64) when the caller staged them too, else nullptr (gains
// are then read from global memory).  `red` holds 2 * NT/32 uint64.
//   k   = max(bitlen(max|x|) - 24, 0);  ms = sum(shr(x, k)^2) // D + 1;  r = max(isqrt(ms), 1)
//   y_i = (x_i << 16) // (r << k);      a_i = shr(y_i * g_i, 16);        xq, s = qrow(a)
// |y_i| <= 2^16 sqrt(D) (2^(k+24) * 2^16 at k = 0), so every quotient is far below 2^50.
template <int NT>
EXB_DEV void row_norm_q_staged(const int64_t* __restrict__ g, int D, int16_t* __restrict__ xq,
                               int32_t* __restrict__ xs_out, int64_t* ys, uint64_t* red, uint64_t m,
                               const int64_t* gs = nullptr) {
  uint64_t* rA = red;
  uint64_t* rB = red + NT / 32;
  m = block_max_fast<NT>(m, rA);
  int k = bitlen64(m) - 24;
  k = k > 0 ? k : 0;
  uint64_t ss = 0;
#pragma unroll 4
  for (int i = threadIdx.x; i < D; i += NT) {
    const int64_t v = shr64(ys[i], k);
    ss += (uint64_t)v * (uint64_t)v;
  }
  const uint64_t sum = block_sum_fast<NT>(ss, rB);      // < D * 2^48: non-negative as int64
  // ms = sum // D + 1 with a double estimate and exact corrections
  const double invD = 1.0 / (double)D;
  int64_t q = __double2ll_rz(__ll2double_rn((int64_t)sum) * invD);
  int64_t rem = (int64_t)sum - q * (int64_t)D;
  while (rem < 0) { q -= 1; rem += D; }
  while (rem >= D) { q += 1; rem -= D; }
  const int64_t ms = q + 1;
  int64_t rt = isqrt_ref(ms);
  rt = rt > 1 ? rt : 1;
  const int64_t den = (int64_t)((uint64_t)rt << k);
  const double inv = __drcp_rn((double)den);
  uint64_t m2 = 0;
#pragma unroll 4
  for (int i = threadIdx.x; i < D; i += NT) {
    const int64_t y = floordiv_small_q((int64_t)((uint64_t)ys[i] << 16), den, inv);
    const int64_t gi = gs ? gs[i] : __ldg(g + i);
    const int64_t a = shr64((int64_t)((uint64_t)y * (uint64_t)gi), 16);
    ys[i] = a;
    const uint64_t u = uabs64(a);
    m2 = u > m2 ? u : m2;
  }
  m2 = block_max_fast<NT>(m2, rA);
  const int s = qrow_shift(m2);
#pragma unroll 4
  for (int i = threadIdx.x; i < D; i += NT) xq[i] = qrow_value(ys[i], s);
  if (threadIdx.x == 0) *xs_out = s;
  __syncthreads();
}

// One row: irms + qrow with the row held in registers: EPT elements per thread (D <= NT * EPT),
// element i = threadIdx.x + j * NT in slot j.  Every per-element step is an independent chain the
// compiler interleaves across the EPT slots; nothing is staged in shared memory.  `red` holds
// 2 * NT/32 uint64.  Same arithmetic as row_norm_q_staged (exact_llm.py:100-106 then :41-46).
template <int NT, int EPT>
EXB_DEV void row_norm_q_regs(const int64_t* __restrict__ xr, const int64_t* __restrict__ g, int D,
                             int16_t* __restrict__ xq, int32_t* __restrict__ xs_out, uint64_t* red) {
  uint64_t* rA = red;
  uint64_t* rB = red + NT / 32;
  int64_t v[EPT], gv[EPT];
  uint64_t m = 0;
#pragma unroll
  for (int j = 0; j < EPT; ++j) {
    const int i = threadIdx.x + j * NT;
    v[j] = i < D ? ld_cg(xr + i) : 0;
    gv[j] = i < D ? __ldg(g + i) : 0;
  }
#pragma unroll
  for (int j = 0; j < EPT; ++j) { const uint64_t u = uabs64(v[j]); m = u > m ? u : m; }
  m = block_max_fast<NT>(m, rA);
  int k = bitlen64(m) - 24;
  k = k > 0 ? k : 0;
  uint64_t ss = 0;
#pragma unroll
  for (int j = 0; j < EPT; ++j) {
    const int64_t t = shr_nn(v[j], k);                 // 0 for the padding slots; 0 <= k <= 39
    ss += (uint64_t)t * (uint64_t)t;
  }
  const uint64_t sum = block_sum_fast<NT>(ss, rB);
  const double invD = 1.0 / (double)D;
  int64_t q = __double2ll_rz(__ll2double_rn((int64_t)sum) * invD);
  int64_t rem = (int64_t)sum - q * (int64_t)D;
  while (rem < 0) { q -= 1; rem += D; }
  while (rem >= D) { q += 1; rem -= D; }
  int64_t rt = isqrt_ref(q + 1);
  rt = rt > 1 ? rt : 1;
  const NormDiv nd = make_norm_div(rt, k);
  uint64_t m2 = 0;
#pragma unroll
  for (int j = 0; j < EPT; ++j) {
    const int64_t y = norm_div(v[j], nd);
    v[j] = shr_nn((int64_t)((uint64_t)y * (uint64_t)gv[j]), 16);
    const uint64_t u = uabs64(v[j]);
    m2 = u > m2 ? u : m2;
  }
  m2 = block_max_fast<NT>(m2, rA);
  const int s = qrow_shift(m2);
#pragma unroll
  for (int j = 0; j < EPT; ++j) {
    const int i = threadIdx.x + j * NT;
    if (i < D) xq[i] = qrow_value(v[j], s);
  }
  if (threadIdx.x == 0) *xs_out = s;
  __syncthreads();
}

// irms + qrow of one row from its published statistics m = max |x| and ss = sum x^2 (summed by the
// CTAs that produced the row).  When m < 2^24 the shift k of irms is 0, so ss is exactly
// sum(shr(x, k)^2) and only the qrow maximum is left to reduce; otherwise (k > 0) returns false
// and the caller runs the full routine.  Row in registers (D <= EPT * NT).
template <int NT, int EPT>
EXB_DEV bool row_norm_q_stats_regs(const int64_t* __restrict__ xr, const int64_t* __restrict__ g, int D, uint64_t m,
                                   uint64_t ss, int16_t* __restrict__ xq, int32_t* __restrict__ xs_out, uint64_t* red) {
  if (bitlen64(m) > 24) return false;
  int64_t v[EPT], gv[EPT];
#pragma unroll
  for (int j = 0; j < EPT; ++j) {
    const int i = threadIdx.x + j * NT;
    v[j] = i < D ? ld_cg(xr + i) : 0;
    gv[j] = i < D ? __ldg(g + i) : 0;
  }
  // ms = ss // D + 1, r = max(isqrt(ms), 1)   (exact_llm.py:103-104)
  const double invD = 1.0 / (double)D;
  int64_t q = __double2ll_rz(__ll2double_rn((int64_t)ss) * invD);
  int64_t rem = (int64_t)ss - q * (int64_t)D;
  while (rem < 0) { q -= 1; rem += D; }
  while (rem >= D) { q += 1; rem -= D; }
  int64_t rt = isqrt_ref(q + 1);
  rt = rt > 1 ? rt : 1;
  const NormDiv nd = make_norm_div(rt, 0);
  uint64_t m2 = 0;
#pragma unroll
  for (int j = 0; j < EPT; ++j) {
    const int64_t y = norm_div(v[j], nd);
    v[j] = shr_nn((int64_t)((uint64_t)y * (uint64_t)gv[j]), 16);
    const uint64_t u = uabs64(v[j]);
    m2 = u > m2 ? u : m2;
  }
  m2 = block_max_fast<NT>(m2, red);
  const int s = qrow_shift(m2);
#pragma unroll
  for (int j = 0; j < EPT; ++j) {
    const int i = threadIdx.x + j * NT;
    if (i < D) xq[i] = qrow_value(v[j], s);
  }
  if (threadIdx.x == 0) *xs_out = s;
  __syncthreads();
  return true;
}

template <int NT>
EXB_DEV bool row_norm_q_stats(const int64_t* __restrict__ xr, const int64_t* __restrict__ g, int D, uint64_t m,
                              uint64_t ss, int16_t* __restrict__ xq, int32_t* __restrict__ xs_out, uint64_t* red) {
  if (D <= 4 * NT) return row_norm_q_stats_regs<NT, 4>(xr, g, D, m, ss, xq, xs_out, red);
  if (D <= 8 * NT) return row_norm_q_stats_regs<NT, 8>(xr, g, D, m, ss, xq, xs_out, red);
  if (D <= 12 * NT) return row_norm_q_stats_regs<NT, 12>(xr, g, D, m, ss, xq, xs_out, red);
  return false;
}

// irms + qrow of one row: registers when D <= 12 NT, else staged in shared memory (`ys`, 2*D int64)
template <int NT>
EXB_DEV void row_norm_q_any(const int64_t* __restrict__ xr, const int64_t* __restrict__ g, int D,
                            int16_t* __restrict__ xq, int32_t* __restrict__ xs_out, int64_t* ys, uint64_t* red);

// One row: irms + qrow.  `ys` = 2*D int64 of shared memory (row, then gains), loaded with all
// requests in flight (16-byte loads); `red` = 33 uint64 of shared memory.  D is even.
template <int NT>
EXB_DEV void row_norm_q(const int64_t* __restrict__ xr, const int64_t* __restrict__ g, int D, int16_t* __restrict__ xq,
                        int32_t* __restrict__ xs_out, int64_t* ys, uint64_t* red) {
  int64_t* gs = ys + D;
  const longlong2* x2 = reinterpret_cast<const longlong2*>(xr);
  const longlong2* g2 = reinterpret_cast<const longlong2*>(g);
  uint64_t m = 0;
#pragma unroll 4
  for (int i = threadIdx.x; i < (D >> 1); i += NT) {
    const longlong2 v = __ldcg(x2 + i);
    const longlong2 w = __ldg(g2 + i);
    reinterpret_cast<longlong2*>(ys)[i] = v;
    reinterpret_cast<longlong2*>(gs)[i] = w;
    const uint64_t a = uabs64(v.x), b = uabs64(v.y);
    m = a > m ? a : m;
    m = b > m ? b : m;
  }
  __syncthreads();
  row_norm_q_staged<NT>(g, D, xq, xs_out, ys, red, m, gs);
}

template <int NT>
EXB_DEV void row_norm_q_any(const int64_t* __restrict__ xr, const int64_t* __restrict__ g, int D,
                            int16_t* __restrict__ xq, int32_t* __restrict__ xs_out, int64_t* ys, uint64_t* red) {
  if (D <= 4 * NT) row_norm_q_regs<NT, 4>(xr, g, D, xq, xs_out, red);
  else if (D <= 8 * NT) row_norm_q_regs<NT, 8>(xr, g, D, xq, xs_out, red);
  else if (D <= 12 * NT) row_norm_q_regs<NT, 12>(xr, g, D, xq, xs_out, red);
  else row_norm_q<NT>(xr, g, D, xq, xs_out, ys, red);
}

// One row: qrow.  Values are staged in shared memory (`ys`, K int64) so the row is read once.
template <int NT>
EXB_DEV void row_quant(const int64_t* __restrict__ xr, int K, int16_t* __restrict__ xq, int32_t* __restrict__ xs_out,
                       int64_t* ys, uint64_t* red) {
  uint64_t m = 0;
#pragma unroll 8
  for (int i = threadIdx.x; i < K; i += NT) {
    const int64_t v = ld_cg(xr + i);
    ys[i] = v;
    const uint64_t a = uabs64(v);
    m = a > m ? a : m;
  }
  m = block_max_u64<NT>(m, red);
  const int s = qrow_shift(m);
  for (int i = threadIdx.x; i < K; i += NT) xq[i] = qrow_value(ys[i], s);
  if (threadIdx.x == 0) *xs_out = s;
  __syncthreads();
}

// One row: xq = clip(shr(x, s)) with s already known (from a published row max); no staging.
template <int NT>
EXB_DEV void row_quant_known(const int64_t* __restrict__ xr, int K, int s, int16_t* __restrict__ xq) {
  const longlong2* x2 = reinterpret_cast<const longlong2*>(xr);
  const int K2 = K >> 1;
#pragma unroll 8
  for (int i = threadIdx.x; i < K2; i += NT) {
    const longlong2 v = __ldcg(x2 + i);
    const short2 q = make_short2(qrow_value(v.x, s), qrow_value(v.y, s));
    reinterpret_cast<short2*>(xq)[i] = q;
  }
  if ((K & 1) && threadIdx.x == 0) xq[K - 1] = qrow_value(ld_cg(xr + K - 1), s);
}

// RoPE + cache write for rows 0..R-1; one warp per (row, head) task.  Heads 0..KV-1 are the
// key heads (RoPE, per-row quantisation, K and V cache write), heads KV..KV+H-1 the query heads
// (RoPE + per-row quantisation into qq/qs).
// Tasks are split over the grid: this CTA's warps take tasks first_task + warp, + stride, ...
template <int NT>
EXB_DEV void rope_cache_rows(const AttnArgs& a, int first_task = 0, int stride = NT / 32) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hd = a.hd, half = hd >> 1;
  const int tasks = a.R * (a.KV + a.H);
  for (int t = first_task + warp; t < tasks; t += stride) {
    const int r = t / (a.KV + a.H), h = t - r * (a.KV + a.H);
    const int pos = a.row_pos[r], seq = a.row_seq[r];
    if (pos < 0 || pos >= a.Smax || pos >= a.Tmax) {
      if (lane == 0) set_err(a.err, ERR_BOUNDS);
      continue;
    }
    const bool is_k = h < a.KV;
    const int64_t* row = a.qkv + (size_t)r * a.ldqkv + (size_t)(is_k ? a.H + h : h - a.KV) * hd;
    int64_t out[4];                           // hd <= 128 -> at most 4 values per lane
    uint64_t m = 0;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int d = lane + 32 * q;
      out[q] = 0;
      if (d < hd) {
        const int64_t c = a.cos_t[(size_t)pos * half + (d % half)], s = a.sin_t[(size_t)pos * half + (d % half)];
        const int64_t x = ld_cg(row + d);
        const int64_t rot = d < half ? (int64_t)(0ull - (uint64_t)ld_cg(row + d + half)) : ld_cg(row + d - half);
        out[q] = shr64((int64_t)((uint64_t)x * (uint64_t)c + (uint64_t)rot * (uint64_t)s), 16);
        const uint64_t u = uabs64(out[q]);
        m = u > m ? u : m;
      }
    }
    for (int o = 16; o > 0; o >>= 1) { const uint64_t w = __shfl_xor_sync(0xffffffffu, m, o); m = w > m ? w : m; }
    const int sh = qrow_shift(m);
    if (is_k) {
      const size_t cidx = ((size_t)seq * a.KV + h) * a.Smax + pos;
      const int64_t* vrow = a.qkv + (size_t)r * a.ldqkv + (size_t)(a.H + a.KV + h) * hd;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int d = lane + 32 * q;
        if (d < hd) {
          a.kc[cidx * hd + d] = qrow_value(out[q], sh);
          const int64_t v = ld_cg(vrow + d);
          if (v > INT32_MAX || v < INT32_MIN) set_err(a.err, ERR_V_RANGE);
          a.vc[cidx * hd + d] = (int32_t)v;
        }
      }
      if (lane == 0) a.ks[cidx] = (int8_t)sh;
    } else {
      const int hq = h - a.KV;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int d = lane + 32 * q;
        if (d < hd) a.qq[((size_t)r * a.H + hq) * hd + d] = qrow_value(out[q], sh);
      }
      if (lane == 0) a.qs[(size_t)r * a.H + hq] = sh;
    }
  }
}

// "Last CTA" election: every CTA calls this after its global writes; returns true in exactly one
// CTA (the last to arrive), which then sees all other CTAs' writes.  The counter is reset by the
// elected CTA, so the kernel can be replayed (CUDA graphs).  No spinning.
EXB_DEV bool last_cta(unsigned int* ticket, unsigned int n_ctas) {
  __shared__ bool is_last;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned t = atomicAdd(ticket, 1u);
    is_last = (t == n_ctas - 1);
    if (is_last) *ticket = 0;
  }
  __syncthreads();
  if (is_last) __threadfence();
  return is_last;
}

}  // namespace exb
