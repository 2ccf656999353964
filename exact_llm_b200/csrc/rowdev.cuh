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

// One row already staged in shared memory (`ys`, D int64; overwritten): irms + qrow.
// `m` is this thread's partial max |x| over the elements it staged; `gs` holds the gains (D int64)
// when the caller staged them too, else nullptr (gains are then read from global memory).
template <int NT>
EXB_DEV void row_norm_q_staged(const int64_t* __restrict__ g, int D, int16_t* __restrict__ xq,
                               int32_t* __restrict__ xs_out, int64_t* ys, uint64_t* red, uint64_t m,
                               const int64_t* gs = nullptr) {
  m = block_max_u64<NT>(m, red);
  int k = bitlen64(m) - 24;
  k = k > 0 ? k : 0;
  uint64_t ss = 0;
  for (int i = threadIdx.x; i < D; i += NT) {
    const int64_t v = shr64(ys[i], k);
    ss += (uint64_t)v * (uint64_t)v;
  }
  const int64_t sum = block_sum_i64<NT>((int64_t)ss, red);
  const int64_t ms = floordiv64(sum, D) + 1;
  int64_t rt = isqrt_ref(ms);
  rt = rt > 1 ? rt : 1;
  const int64_t den = (int64_t)((uint64_t)rt << k);
  const double inv = 1.0 / (double)den;
  uint64_t m2 = 0;
  for (int i = threadIdx.x; i < D; i += NT) {
    const int64_t y = floordiv_recip((int64_t)((uint64_t)ys[i] << 16), den, inv);
    const int64_t gi = gs ? gs[i] : __ldg(g + i);
    const int64_t a = shr64((int64_t)((uint64_t)y * (uint64_t)gi), 16);
    ys[i] = a;
    const uint64_t u = uabs64(a);
    m2 = u > m2 ? u : m2;
  }
  m2 = block_max_u64<NT>(m2, red);
  const int s = qrow_shift(m2);
  for (int i = threadIdx.x; i < D; i += NT) xq[i] = qrow_value(ys[i], s);
  if (threadIdx.x == 0) *xs_out = s;
  __syncthreads();
}

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
