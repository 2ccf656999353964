// Persistent decode step (opt-in engine option "step"): the complete exact forward pass of R <= 2
// decode rows (embedding, every layer, final norm, head and greedy argmax) as ONE cooperative
// kernel, one CTA of 1024 threads per SM, phases separated by bounded grid barriers.
//
// The reference decode step (GraphDecoder.step, experiments/speed_fair_kaggle.py:639-645; the
// layer math of exact_llm.py:157-180) is a chain of small dependent operations:
//
//   embed + clear          x = emb[id] << shift; per-layer accumulators cleared
//   per layer l:
//     q|k|v                every CTA: xq = qrow(irms(x, g1)) (redundantly, from L2), then its
//                          slice of the fused q|k|v GEMV
//     attention A          CTA per (row, KV head, key chunk): RoPE of its query heads and of the
//                          new key rows, K/V cache write, scores, atomic max per head
//     attention B          e = EXP_T(max - score), atomic sum per head
//     attention C          p = (e << 20) // sum, partial sum_t p_t v_t -> atomic int64 add
//     o                    xq = qrow(shr(att, 20)); x += o(xq)
//     gate|up              xq = qrow(irms(x, g2)); h = shr(isilu(g) u, 16), atomic max |h|
//     qrow(h)              split over the grid
//     down                 x += down(hq)
//   head                   xq = qrow(irms(x, gf)); logits, argmax (last-CTA election)
//
// Weight bytes stream through lane-private cp.async rings; where HBM would otherwise idle
// (attention, the qrow(h) split) one thread per CTA prefetches the next weight slices into L2.
// Measured on B200 (7B, batch 1) this path is slower than one kernel per operation with
// programmatic dependent launch (4.4 vs 3.0 ms per step): the redundant per-CTA norm prologues
// and the three attention phases are latency chains that the barriers cannot overlap.  It stays
// as a tested alternative (bit-identical results; parity test against the per-kernel path).
//
// Every integer result is the reference's: the phases run the same device arithmetic as the
// standalone kernels, and every cross-CTA sum is an integer sum.  Barriers are bounded: a CTA
// that waits too long raises the abort flag and the error word, and every CTA then returns.
#include <algorithm>
#include <climits>
#include <cstdlib>

#include "common.cuh"
#include "exb_internal.h"
#include "gemvdev.cuh"
#include "rowdev.cuh"

namespace exb {

constexpr int SNCW = 32;                       // warps per CTA (one CTA per SM)
constexpr int STEP_THREADS = 32 * SNCW;
constexpr int STEP_MIN_BLOCKS = 1;
constexpr int STEP_RMAX = 2;
constexpr int STEP_REP_MAX = 8;                // query heads per KV head
constexpr unsigned SPIN_LIMIT = 1u << 22;      // barrier polls (with back-off) before giving up
constexpr int STEP_SMEM_MAX = 200 * 1024;      // dynamic shared memory ceiling
constexpr int ATT_TT = 32;                     // key/value positions staged per attention tile
#ifndef EXB_STEP_RING
#define EXB_STEP_RING 6
#endif
constexpr int STEP_RING = EXB_STEP_RING;       // cp.async ring depth per lane (16-byte chunks in flight)

EXB_DEV unsigned ld_acquire_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

EXB_DEV unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Grid-wide barrier over a monotonically increasing arrival counter (zeroed before the launch).
// Returns false in every thread of the CTA when the step was aborted (timeout here or elsewhere).
EXB_DEV bool grid_sync(const StepArgs& a, unsigned& target, int* ok_s) {
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned k = target / gridDim.x;          // barrier index
    target += gridDim.x;
    int ok = 1;
    if (a.prof) a.prof[(size_t)(2 * k) * gridDim.x + blockIdx.x] = globaltimer_ns();
    __threadfence();
    atomicAdd(a.bar, 1u);
    for (unsigned it = 0;; ++it) {
      if ((int)(ld_acquire_u32(a.bar) - target) >= 0) break;
      if (ld_acquire_u32(a.bar + 1) != 0u) { ok = 0; break; }
      if (it > SPIN_LIMIT) {
        ok = 0;
        atomicExch(a.bar + 1, 1u);
        set_err(a.err, ERR_WAIT_TIMEOUT);
        break;
      }
      __nanosleep(64);
    }
    if (a.prof) a.prof[(size_t)(2 * k + 1) * gridDim.x + blockIdx.x] = globaltimer_ns();
    *ok_s = ok;
  }
  __syncthreads();
  return *ok_s != 0;
}

// profiling: time stamp of thread 0 right after a phase's prologue (index = barriers passed)
EXB_DEV void prof_mid(const StepArgs& a, unsigned target) {
  if (a.prof && threadIdx.x == 0) {
    const unsigned nb = 1 + 8 * a.NL;
    a.prof[(size_t)(2 * nb + target / gridDim.x) * gridDim.x + blockIdx.x] = globaltimer_ns();
  }
}

// ------------------------------------------------------------------ weight phases and prefetch
// p = 4 l + {0: q|k|v, 1: o, 2: gate|up, 3: down}; p = 4 NL: head
EXB_DEV int step_rb(int, int, int) { return 1; }

EXB_DEV const LinW* phase_lin(const StepArgs& a, int p, int& rpu) {
  rpu = 1;
  if (p >= 4 * a.NL) return &a.head;
  const StepLayer* Ly = a.layers + (p >> 2);
  switch (p & 3) {
    case 0: return &Ly->qkv;
    case 1: return &Ly->o;
    case 2: rpu = 2; return &Ly->gu;
    default: return &Ly->down;
  }
}

struct PhaseGeom {
  const int8_t* w;
  const int32_t* Mg;
  int K, ldm, rpu, rb, ulo, uhi;
};

EXB_DEV void phase_geom(const StepArgs& a, int p, PhaseGeom& g) {
  int rpu;
  const LinW* L = phase_lin(a, p, rpu);
  g.w = L->w; g.Mg = L->Mg; g.K = L->K; g.ldm = L->ldm; g.rpu = rpu;
  const int units = L->N / rpu;
  g.ulo = (int)((long long)units * blockIdx.x / gridDim.x);
  g.uhi = (int)((long long)units * (blockIdx.x + 1) / gridDim.x);
  g.rb = step_rb(a.R, units, gridDim.x);
}

// thread 0: pull the first `bytes` of this CTA's weight slice of phase p into L2 (the slice of a
// phase is one contiguous row range; fire-and-forget bulk prefetches).  Issued where HBM would
// otherwise idle: during the attention phases, the q(h) split and the embedding.
EXB_DEV void pf_slice(const StepArgs& a, int p, size_t bytes) {
  if (threadIdx.x != 0 || p > 4 * a.NL || bytes == 0) return;
  PhaseGeom g;
  phase_geom(a, p, g);
  const size_t row0 = (size_t)g.ulo * g.rpu, nrows = (size_t)(g.uhi - g.ulo) * g.rpu;
  const char* w = reinterpret_cast<const char*>(g.w) + row0 * g.K;
  size_t nb = nrows * g.K;
  nb = nb < bytes ? nb : bytes;
  for (size_t off = 0; off < nb; off += 32768)
    prefetch_l2_bulk(w + off, (uint32_t)(nb - off < 32768 ? nb - off : 32768));
  if (g.Mg) {
    size_t mb = (nb / g.K + 1) * g.ldm * 4;
    const size_t mall = nrows * g.ldm * 4;
    mb = mb < mall ? mb : mall;
    if (mb) prefetch_l2_bulk(g.Mg + row0 * g.ldm, (uint32_t)mb);
  }
}

// ------------------------------------------------------------------ GEMV phase
struct StepEpi {
  const LinW* L;
  int epi;                      // EPI_STORE, EPI_RESID, EPI_SWIGLU or EPI_HEAD
  int64_t* out; int ldo;
  const int32_t* silu_t;
  unsigned long long* amax_out; // SwiGLU: per-row max |h|
};

// epilogue of unit ug (one column, or a gate/up pair) for activation row r; per-lane running
// max |h| (SwiGLU) and best (value, index) (head) in omax / bv / bn
template <int RPU>
EXB_DEV void step_epilogue(const StepEpi& e, int ug, int r, const int64_t* t2, int sh, uint64_t& omax, int64_t& bv,
                           int& bn) {
  const LinW& L = *e.L;
  if (RPU == 2) {
    // SwiGLU pair: fused row 2u = gate u, 2u + 1 = up u (exact_llm.py:179)
    const int64_t yg = requant1(L, 2 * ug, t2[0], sh);
    const int64_t yu = requant1(L, 2 * ug + 1, t2[RPU - 1], sh);
    const int64_t hv = shr64((int64_t)((uint64_t)isilu_dev(e.silu_t, yg) * (uint64_t)yu), 16);
    e.out[(size_t)r * e.ldo + ug] = hv;
    const uint64_t ah = uabs64(hv);
    omax = ah > omax ? ah : omax;
    return;
  }
  const int n = ug;
  const int64_t y = requant1(L, n, t2[0], sh);
  if (e.epi == EPI_RESID) {
    int64_t* o = e.out + (size_t)r * e.ldo + n;
    *o = (int64_t)((uint64_t)__ldcg(reinterpret_cast<const long long*>(o)) + (uint64_t)y);
  } else if (e.out) {
    e.out[(size_t)r * e.ldo + n] = y;
  }
  if (e.epi == EPI_HEAD && (y > bv || (y == bv && n < bn))) {
    bv = y;
    bn = n;
  }
}

struct StepShared {
  unsigned long long head_best[SNCW][STEP_RMAX][2];
  uint64_t rred[2 * SNCW + 1];
  int sh[STEP_RMAX];
  int qsh[STEP_REP_MAX];
  int ksh[STEP_RMAX];
  int ok;
};

// This CTA's columns of one linear.  Activations xs: R rows of K int16 in shared memory (shifts
// in ss.sh).  The CTA's weight rows [ulo*RPU, uhi*RPU) are one contiguous byte range; it is
// split evenly over the 16 warps as runs of 16-byte chunks, so every warp streams one contiguous
// run whatever the row count (lane l: chunks l, l + 32, ... of the warp's run).  Chunks travel
// through a lane-private cp.async ring of STEP_RING slots (loads in flight without registers).
// Per chunk: 8 dp2a (16 MACs) per activation row, times the chunk's group scale, into an int64
// lane partial of the current row; a lane adds its partial to the row's shared-memory sum when
// its chunks move to the next row.  Integer addition is associative, so the sums are the
// reference's (modulo 2^64, like numpy int64).  Then one thread per unit runs the epilogue.
template <int R, int RPU, bool GROUP>
__device__ __noinline__ void gemv_phase(const StepArgs& a, const StepEpi& e, const int16_t* xs, unsigned char* ring,
                                        int64_t* rowsum, StepShared& ss) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const LinW& L = *e.L;
  const int K = L.K, C = K >> 4, ldm = L.ldm;
  const int units = L.N / RPU;
  const int ulo = (int)((long long)units * blockIdx.x / gridDim.x);
  const int uhi = (int)((long long)units * (blockIdx.x + 1) / gridDim.x);
  const int nrow = (uhi - ulo) * RPU;
  const long long T = (long long)nrow * C;
  const long long c0 = T * warp / SNCW, c1 = T * (warp + 1) / SNCW;
  const int8_t* Wt = L.w + (size_t)ulo * RPU * K;
  const int32_t* Mg = GROUP ? L.Mg + (size_t)ulo * RPU * ldm : nullptr;
  for (int i = tid; i < nrow * R; i += STEP_THREADS) rowsum[i] = 0;
  int sh[R];
#pragma unroll
  for (int r = 0; r < R; ++r) sh[r] = ss.sh[r];
  int4* wring = reinterpret_cast<int4*>(ring) + (size_t)warp * STEP_RING * 32;
  __syncthreads();

  // issue cursor (chunk ci = row irow, chunk icol of the row)
  long long ci = c0 + lane;
  int irow = (int)(ci / C), icol = (int)(ci - (long long)irow * C);
  auto issue = [&](int slot) {
    if (ci < c1) {
      cp_async16(wring + slot * 32 + lane, Wt + (size_t)ci * 16);
    }
    cp_async_commit();
    ci += 32; icol += 32;
    while (icol >= C) { icol -= C; ++irow; }
  };
#pragma unroll
  for (int s0 = 0; s0 < STEP_RING; ++s0) issue(s0);
  int slot = 0;
  long long cc = c0 + lane;
  int crow = (int)(cc / C), ccol = (int)(cc - (long long)crow * C);
  int arow = crow;
  int64_t acc[R];
#pragma unroll
  for (int r = 0; r < R; ++r) acc[r] = 0;
  for (; cc < c1; cc += 32) {
    cp_async_wait<STEP_RING - 1>();
    const int4 wv = wring[slot * 32 + lane];
    const int32_t mv = GROUP ? __ldg(Mg + (size_t)crow * ldm + (ccol >> 3)) : 1;   // group scale (L1)
    issue(slot);                                                 // refill: the chunk STEP_RING ahead
    slot = slot + 1 == STEP_RING ? 0 : slot + 1;
    if (crow != arow) {
#pragma unroll
      for (int r = 0; r < R; ++r) {
        atomicAdd(reinterpret_cast<unsigned long long*>(rowsum + (size_t)arow * R + r), (unsigned long long)acc[r]);
        acc[r] = 0;
      }
      arow = crow;
    }
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int4* xp = reinterpret_cast<const int4*>(xs + (size_t)r * K + 16 * ccol);
      const int p = dot16(wv, xp[0], xp[1]);
      acc[r] = (int64_t)((uint64_t)acc[r] + (uint64_t)(GROUP ? (int64_t)p * mv : (int64_t)p));
    }
    ccol += 32;
    while (ccol >= C) { ccol -= C; ++crow; }
  }
  if (c0 + lane < c1) {
#pragma unroll
    for (int r = 0; r < R; ++r)
      atomicAdd(reinterpret_cast<unsigned long long*>(rowsum + (size_t)arow * R + r), (unsigned long long)acc[r]);
  }
  cp_async_wait<0>();
  __syncthreads();

  // epilogues: one thread per unit
  uint64_t omax[R];
  int64_t best_v[R];
  int best_n[R];
#pragma unroll
  for (int r = 0; r < R; ++r) { omax[r] = 0; best_v[r] = INT64_MIN; best_n[r] = 0x7fffffff; }
  for (int ul = tid; ul < uhi - ulo; ul += STEP_THREADS) {
#pragma unroll
    for (int r = 0; r < R; ++r) {
      int64_t t2[RPU];
#pragma unroll
      for (int q = 0; q < RPU; ++q) t2[q] = rowsum[(size_t)(ul * RPU + q) * R + r];
      step_epilogue<RPU>(e, ulo + ul, r, t2, sh[r], omax[r], best_v[r], best_n[r]);
    }
  }
  if (e.epi != EPI_SWIGLU && e.epi != EPI_HEAD) return;     // no cross-thread state to fold
  if (e.epi == EPI_SWIGLU) {
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const uint64_t v = block_max_fast<STEP_THREADS>(omax[r], ss.rred + (r & 1) * (STEP_THREADS / 32));
      if (tid == 0 && v) atomicMax(e.amax_out + r, (unsigned long long)v);
    }
    return;
  }
  // greedy argmax (first index on ties, exact_llm.py:267): per-warp, per-CTA, then the last CTA
#pragma unroll
  for (int r = 0; r < R; ++r)
    for (int o = 16; o > 0; o >>= 1) {
      const int64_t ov = __shfl_xor_sync(0xffffffffu, best_v[r], o);
      const int on = __shfl_xor_sync(0xffffffffu, best_n[r], o);
      if (ov > best_v[r] || (ov == best_v[r] && on < best_n[r])) { best_v[r] = ov; best_n[r] = on; }
    }
  if (lane == 0) {
#pragma unroll
    for (int r = 0; r < R; ++r) {
      ss.head_best[warp][r][0] = (unsigned long long)best_v[r];
      ss.head_best[warp][r][1] = (unsigned long long)(unsigned)best_n[r];
    }
  }
  __syncthreads();
  if (tid < R) {
    const int r = tid;
    int64_t bv = INT64_MIN;
    int bn = 0x7fffffff;
    for (int w = 0; w < SNCW; ++w) {
      const int64_t v = (int64_t)ss.head_best[w][r][0];
      const int n = (int)ss.head_best[w][r][1];
      if (v > bv || (v == bv && n < bn)) { bv = v; bn = n; }
    }
    a.head_part[((size_t)blockIdx.x * R + r) * 2 + 0] = (unsigned long long)bv;
    a.head_part[((size_t)blockIdx.x * R + r) * 2 + 1] = (unsigned long long)(unsigned)bn;
  }
  if (last_cta(a.head_ticket, gridDim.x) && tid < R) {
    const int r = tid;
    int64_t bv = INT64_MIN;
    int bn = 0x7fffffff;
    for (unsigned c = 0; c < gridDim.x; ++c) {
      const int64_t v = (int64_t)__ldcg(a.head_part + ((size_t)c * R + r) * 2);
      const int n = (int)__ldcg(a.head_part + ((size_t)c * R + r) * 2 + 1);
      if (v > bv || (v == bv && n < bn)) { bv = v; bn = n; }
    }
    a.next_tok[r] = bn;
  }
}

template <int R, int RPU, bool GROUP>
EXB_DEV void gemv_phase_rb(const StepArgs& a, const StepEpi& e, const int16_t* xs, unsigned char* ring, StepShared& ss) {
  int64_t* rowsum = reinterpret_cast<int64_t*>(ring + (size_t)SNCW * STEP_RING * 32 * 16);
  gemv_phase<R, RPU, GROUP>(a, e, xs, ring, rowsum, ss);
}

// ------------------------------------------------------------------ activation prologues
// xq, s = qrow(irms(x, g)) for every row (exact_llm.py:100-106, 41-46); each CTA computes it
template <int R>
__device__ __noinline__ void stage_norm(const StepArgs& a, const int64_t* g, int16_t* xs, int64_t* ys, StepShared& ss) {
  for (int r = 0; r < R; ++r)
    row_norm_q_any<STEP_THREADS>(a.x + (size_t)r * a.D, g, a.D, xs + (size_t)r * a.D, &ss.sh[r], ys, ss.rred);
}

// xq, s = qrow(shr(att, 20)) (exact_llm.py:176, 41-46)
template <int R>
EXB_DEV void stage_attn_out(const StepArgs& a, int l, int16_t* xs, int64_t* ys, StepShared& ss) {
  const int Hd = a.H * a.hd;
  for (int r = 0; r < R; ++r) {
    const longlong2* src = reinterpret_cast<const longlong2*>(a.att + ((size_t)l * a.R + r) * Hd);
    uint64_t m = 0;
    for (int i = threadIdx.x; i < (Hd >> 1); i += STEP_THREADS) {
      const longlong2 v = __ldcg(src + i);
      const int64_t o0 = shr64(v.x, 20), o1 = shr64(v.y, 20);
      ys[2 * i] = o0;
      ys[2 * i + 1] = o1;
      const uint64_t u0 = uabs64(o0), u1 = uabs64(o1);
      m = u0 > m ? u0 : m;
      m = u1 > m ? u1 : m;
    }
    m = block_max_u64<STEP_THREADS>(m, ss.rred);
    const int s = qrow_shift(m);
    for (int i = threadIdx.x; i < Hd; i += STEP_THREADS) xs[(size_t)r * Hd + i] = qrow_value(ys[i], s);
    if (threadIdx.x == 0) ss.sh[r] = s;
    __syncthreads();
  }
}

// the grid's share of hq = qrow(h) with the published row max (exact_llm.py:41-46)
template <int R>
EXB_DEV void quant_h_split(const StepArgs& a, int l) {
  const int I = a.I;
  const long long total = (long long)R * I;
  const long long lo = total * blockIdx.x / gridDim.x, hi = total * (blockIdx.x + 1) / gridDim.x;
  int s[R];
#pragma unroll
  for (int r = 0; r < R; ++r) s[r] = qrow_shift(__ldcg(a.amax_h + (size_t)l * a.R + r));
  for (long long i = lo + threadIdx.x; i < hi; i += STEP_THREADS) {
    const int r = (int)(i / I);
    a.hq[i] = qrow_value((int64_t)__ldcg(reinterpret_cast<const long long*>(a.hb + i)), s[r]);
  }
}

template <int R>
EXB_DEV void stage_hq(const StepArgs& a, int l, int16_t* xs, StepShared& ss) {
  const int n8 = a.I >> 3;
  for (int i = threadIdx.x; i < R * n8; i += STEP_THREADS) {
    const int r = i / n8, c = i - r * n8;
    reinterpret_cast<int4*>(xs + (size_t)r * a.I)[c] = __ldcg(reinterpret_cast<const int4*>(a.hq + (size_t)r * a.I) + c);
  }
  if (threadIdx.x < R) ss.sh[threadIdx.x] = qrow_shift(__ldcg(a.amax_h + (size_t)l * a.R + threadIdx.x));
  __syncthreads();
}

// ------------------------------------------------------------------ attention phases
// RoPE of one head row at position pos (exact_llm.py:159-160), then qrow of the row; a warp per
// row, lane l holds dims l, l+32, ...  Returns the row's shift (all lanes).
EXB_DEV int rope_quant_head(const StepArgs& a, const int64_t* row, int pos, int16_t* out) {
  const int lane = threadIdx.x & 31, hd = a.hd, half = hd >> 1;
  int64_t v[4];
  uint64_t m = 0;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int d = lane + 32 * q;
    v[q] = 0;
    if (d < hd) {
      const int64_t c = a.cos_t[(size_t)pos * half + (d % half)], s = a.sin_t[(size_t)pos * half + (d % half)];
      const int64_t x = ld_cg(row + d);
      const int64_t rot = d < half ? (int64_t)(0ull - (uint64_t)ld_cg(row + d + half)) : ld_cg(row + d - half);
      v[q] = shr64((int64_t)((uint64_t)x * (uint64_t)c + (uint64_t)rot * (uint64_t)s), 16);
      const uint64_t u = uabs64(v[q]);
      m = u > m ? u : m;
    }
  }
  for (int o = 16; o > 0; o >>= 1) { const uint64_t w = __shfl_xor_sync(0xffffffffu, m, o); m = w > m ? w : m; }
  const int sh = qrow_shift(m);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int d = lane + 32 * q;
    if (d < hd) out[d] = qrow_value(v[q], sh);
  }
  return sh;
}

EXB_DEV int64_t dot_row_i16(const int16_t* __restrict__ q, const int16_t* __restrict__ k, int hd) {
  int64_t acc = 0;
  for (int d = 0; d < hd; d += 8) {
    const int4 x = *reinterpret_cast<const int4*>(q + d);
    const int4 y = *reinterpret_cast<const int4*>(k + d);
    const int xs[4] = {x.x, x.y, x.z, x.w}, ys[4] = {y.x, y.y, y.z, y.w};
#pragma unroll
    for (int t = 0; t < 4; ++t)
      acc += (int)(short)(xs[t] & 0xffff) * (int)(short)(ys[t] & 0xffff) + (xs[t] >> 16) * (ys[t] >> 16);
  }
  return acc;
}

// Stage 0: RoPE + cache write + scores + atomic max; 1: e + atomic sum; 2: p, partial p.v.
// CTA `task` < R * KV * att_split owns key positions [t0, t1) of (row r, KV head kv); its
// scores stay in shared memory across the three stages (exact_llm.py:170-176).
template <int R>
__device__ __noinline__ void attn_stage(const StepArgs& a, int l, int stage, unsigned char* smem, StepShared& ss) {
  const int split = a.att_split;
  const int task = blockIdx.x;
  if (task >= R * a.KV * split) return;                      // uniform over the CTA
  const int r = task / (a.KV * split);
  const int kv = (task / split) % a.KV;
  const int c = task % split;
  const int hd = a.hd, rep = a.H / a.KV;
  const int pos = a.pos[r], seq = a.seq[r];
  if (pos < 0 || pos >= a.Smax || pos >= a.Tmax || seq < 0 || seq >= a.max_batch) {
    if (threadIdx.x == 0 && stage == 0) set_err(a.err, ERR_BOUNDS);
    return;
  }
  const int S = pos + 1;
  const int chunk = (S + split - 1) / split;
  const int t0 = c * chunk;
  const int t1 = min(S, t0 + chunk);
  const int n = t1 > t0 ? t1 - t0 : 0;
  if (n > a.att_chunk_max) {
    if (threadIdx.x == 0 && stage == 0) set_err(a.err, ERR_BOUNDS);
    return;
  }
  const int cm = a.att_chunk_max;
  int16_t* qsm = reinterpret_cast<int16_t*>(smem);                        // rep x hd
  int16_t* knew = qsm + STEP_REP_MAX * 128;                               // STEP_RMAX x hd
  int32_t* vnew = reinterpret_cast<int32_t*>(knew + STEP_RMAX * 128);     // STEP_RMAX x hd
  int64_t* sc = reinterpret_cast<int64_t*>(vnew + STEP_RMAX * 128);       // rep x cm
  int16_t* ktile = reinterpret_cast<int16_t*>(sc + (size_t)STEP_REP_MAX * cm);   // ATT_TT x (hd + 8)
  int32_t* vtile = reinterpret_cast<int32_t*>(ktile + ATT_TT * (128 + 8));        // ATT_TT x hd
  int* kshift = reinterpret_cast<int*>(vtile + ATT_TT * 128);                     // ATT_TT
  const size_t cbase = ((size_t)seq * a.KV + kv) * a.Smax;
  int16_t* kc = a.kc + a.kv_layer_elems * l;
  int32_t* vc = a.vc + a.kv_layer_elems * l;
  int8_t* ks = a.ks + a.ks_layer_elems * l;
  const size_t hoff = ((size_t)l * a.R + r) * a.H + (size_t)kv * rep;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // Key positions written in THIS step (rows of the same sequence, e.g. consecutive prompt
  // tokens in one chunk) are never read back from the cache, which another CTA may still be
  // writing: the CTA whose chunk holds such a position computes that row itself.
  int fpos[STEP_RMAX];
#pragma unroll
  for (int q = 0; q < STEP_RMAX; ++q) {
    fpos[q] = -1;
    if (q < R && a.seq[q] == seq) {
      const int pq = a.pos[q];
      if (pq >= t0 && pq < t1 && pq < a.Tmax) fpos[q] = pq;
    }
  }

  if (stage == 0) {
    if (warp < rep) {
      const int64_t* row = a.qkv + (size_t)r * a.Nqkv;
      const int s = rope_quant_head(a, row + (size_t)(kv * rep + warp) * hd, pos, qsm + warp * hd);
      if (lane == 0) ss.qsh[warp] = s;
    }
    const int q = SNCW - 1 - warp;                                        // warps 15, 14: fresh rows
    if (q >= 0 && q < STEP_RMAX && fpos[q] >= 0) {
      // RoPE + qrow of the new key row, K cache row + shift, V row (exact_torch.py:146-149);
      // every CTA that owns the position writes the same values
      const int64_t* row = a.qkv + (size_t)q * a.Nqkv;
      const int pq = fpos[q];
      int16_t* kn = knew + q * 128;
      const int s = rope_quant_head(a, row + (size_t)(a.H + kv) * hd, pq, kn);
      if (lane == 0) { ss.ksh[q] = s; ks[cbase + pq] = (int8_t)s; }
      const int64_t* vrow = row + (size_t)(a.H + a.KV + kv) * hd;
      for (int d = lane; d < hd; d += 32) {
        const int64_t v = ld_cg(vrow + d);
        if (v > INT32_MAX || v < INT32_MIN) set_err(a.err, ERR_V_RANGE);
        vnew[q * 128 + d] = (int32_t)v;
        vc[(cbase + pq) * hd + d] = (int32_t)v;
        kc[(cbase + pq) * hd + d] = kn[d];
      }
    }
    __syncthreads();
    // key rows staged one tile at a time (all loads in flight together; rows padded by 16 bytes)
    const int per_row = hd >> 3;                                          // int4 per key row
    for (int tt = 0; tt < n; tt += ATT_TT) {
      const int nt = min(ATT_TT, n - tt);
      for (int e = tid; e < nt * per_row; e += STEP_THREADS) {
        const int t = e / per_row, c4 = e - t * per_row, pt = t0 + tt + t;
        int fr = -1;
#pragma unroll
        for (int q2 = 0; q2 < STEP_RMAX; ++q2) fr = fpos[q2] == pt ? q2 : fr;
        const int4* src = fr >= 0 ? reinterpret_cast<const int4*>(knew + fr * 128)
                                  : reinterpret_cast<const int4*>(kc + (cbase + pt) * hd);
        *reinterpret_cast<int4*>(ktile + t * (128 + 8) + c4 * 8) = src[c4];
        if (c4 == 0) kshift[t] = fr >= 0 ? ss.ksh[fr] : (int)ks[cbase + pt];
      }
      __syncthreads();
      for (int e = tid; e < rep * nt; e += STEP_THREADS) {
        const int i = e / nt, t = e - i * nt;
        const int64_t acc = dot_row_i16(qsm + i * hd, ktile + t * (128 + 8), hd);
        sc[(size_t)i * cm + tt + t] = shr64((int64_t)((uint64_t)acc * (uint64_t)a.inv), 32 - ss.qsh[i] - kshift[t]);
      }
      __syncthreads();
    }
    if (warp < rep && n > 0) {
      int64_t m = INT64_MIN;
      for (int t = lane; t < n; t += 32) { const int64_t v = sc[(size_t)warp * cm + t]; m = v > m ? v : m; }
      for (int o = 16; o > 0; o >>= 1) { const int64_t w = __shfl_xor_sync(0xffffffffu, m, o); m = w > m ? w : m; }
      if (lane == 0) atomicMax(a.gmax + hoff + warp, (long long)m);
    }
  } else if (stage == 1) {
    for (int e = tid; e < rep * n; e += STEP_THREADS) {
      const int i = e / n, t = e - i * n;
      int64_t* p = sc + (size_t)i * cm + t;
      *p = exp_lookup(a.exp_t, (int64_t)__ldcg(a.gmax + hoff + i) - *p);
    }
    __syncthreads();
    if (warp < rep && n > 0) {
      int64_t s = 0;
      for (int t = lane; t < n; t += 32) s += sc[(size_t)warp * cm + t];
      for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      if (lane == 0 && s) atomicAdd(a.gsum + hoff + warp, (unsigned long long)s);
    }
  } else {
    for (int e = tid; e < rep * n; e += STEP_THREADS) {
      const int i = e / n, t = e - i * n;
      int64_t* p = sc + (size_t)i * cm + t;
      *p = (int64_t)(((uint64_t)*p << 20) / __ldcg(a.gsum + hoff + i));
    }
    __syncthreads();
    // partial sum_t p_t v_t over this chunk, value rows staged one tile at a time
    int64_t* att = a.att + hoff * hd;
    int64_t acc[2] = {0, 0};                       // (i, d) pairs e = tid, tid + 512 (rep * hd <= 1024)
    const int per_row = hd >> 2;                   // int4 per value row
    for (int tt = 0; tt < n; tt += ATT_TT) {
      const int nt = min(ATT_TT, n - tt);
      for (int e = tid; e < nt * per_row; e += STEP_THREADS) {
        const int t = e / per_row, c4 = e - t * per_row, pt = t0 + tt + t;
        int fr = -1;
#pragma unroll
        for (int q2 = 0; q2 < STEP_RMAX; ++q2) fr = fpos[q2] == pt ? q2 : fr;
        const int4* src = fr >= 0 ? reinterpret_cast<const int4*>(vnew + fr * 128)
                                  : reinterpret_cast<const int4*>(vc + (cbase + pt) * hd);
        reinterpret_cast<int4*>(vtile)[t * per_row + c4] = src[c4];
      }
      __syncthreads();
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
        const int e = tid + h2 * STEP_THREADS;
        if (e < rep * hd) {
          const int i = e / hd, d = e - i * hd;
          const int64_t* pr = sc + (size_t)i * cm + tt;
          int64_t s2 = acc[h2];
          for (int t = 0; t < nt; ++t)
            s2 = (int64_t)((uint64_t)s2 + (uint64_t)pr[t] * (uint64_t)(int64_t)vtile[t * hd + d]);
          acc[h2] = s2;
        }
      }
      __syncthreads();
    }
    if (n > 0) {
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
        const int e = tid + h2 * STEP_THREADS;
        if (e < rep * hd) atomicAdd(reinterpret_cast<unsigned long long*>(att + e), (unsigned long long)acc[h2]);
      }
    }
  }
}

// ------------------------------------------------------------------ the kernel
template <int R>
__global__ void __launch_bounds__(STEP_THREADS, STEP_MIN_BLOCKS) k_step(const __grid_constant__ StepArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ StepShared ss;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // xq rows at the start of dynamic shared memory; staging rows (int64) behind the norm's R x D rows
  int16_t* xs = reinterpret_cast<int16_t*>(smem);
  int64_t* ys = reinterpret_cast<int64_t*>(smem + (((size_t)R * a.D * 2 + 127) & ~(size_t)127));
  // the GEMV rings behind the R x KMAX activation rows (the norm staging area may overlap them)
  unsigned char* ring = smem + (((size_t)R * a.KMAX * 2 + 127) & ~(size_t)127);
  const size_t pfb = (size_t)a.pf_bytes;
  unsigned target = 0;
  (void)warp; (void)lane;
  pf_slice(a, 0, pfb);
  // ---- embed + clear the per-layer accumulators
  {
    const long long gt = (long long)blockIdx.x * STEP_THREADS + threadIdx.x, gs = (long long)gridDim.x * STEP_THREADS;
    for (long long i = gt; i < (long long)R * a.D; i += gs) {
      const int r = (int)(i / a.D), d = (int)(i - (long long)r * a.D);
      int id = a.ids[r];
      if (id < 0 || id >= a.V) { set_err(a.err, ERR_BOUNDS); id = 0; }
      a.x[i] = (int64_t)a.emb[(size_t)id * a.D + d] << a.emb_shift;
    }
    const long long natt = (long long)a.NL * a.R * a.H * a.hd;
    for (long long i = gt; i < natt; i += gs) a.att[i] = 0;
    const long long nh = (long long)a.NL * a.R * a.H;
    for (long long i = gt; i < nh; i += gs) { a.gmax[i] = LLONG_MIN; a.gsum[i] = 0; }
    for (long long i = gt; i < (long long)a.NL * a.R; i += gs) a.amax_h[i] = 0;
  }
  if (!grid_sync(a, target, &ss.ok)) return;

  for (int l = 0; l < a.NL; ++l) {
    const StepLayer* Ly = a.layers + l;
    StepEpi e;
    e.silu_t = a.silu_t; e.amax_out = nullptr;
    // ---- q|k|v
    stage_norm<R>(a, Ly->g1, xs, ys, ss);
    prof_mid(a, target);
    e.L = &Ly->qkv; e.epi = EPI_STORE; e.out = a.qkv; e.ldo = a.Nqkv;
    gemv_phase_rb<R, 1, true>(a, e, xs, ring, ss);
    if (!grid_sync(a, target, &ss.ok)) return;
    // ---- attention
    pf_slice(a, 4 * l + 1, pfb);                 // HBM is idle during attention: o and gate|up heads
    pf_slice(a, 4 * l + 2, pfb);
    for (int stage = 0; stage < 3; ++stage) {
      attn_stage<R>(a, l, stage, smem, ss);
      if (!grid_sync(a, target, &ss.ok)) return;
    }
    // ---- o (+ residual)
    stage_attn_out<R>(a, l, xs, ys, ss);
    prof_mid(a, target);
    e.L = &Ly->o; e.epi = EPI_RESID; e.out = a.x; e.ldo = a.D;
    gemv_phase_rb<R, 1, true>(a, e, xs, ring, ss);
    if (!grid_sync(a, target, &ss.ok)) return;
    // ---- gate|up (SwiGLU)
    stage_norm<R>(a, Ly->g2, xs, ys, ss);
    prof_mid(a, target);
    e.L = &Ly->gu; e.epi = EPI_SWIGLU; e.out = a.hb; e.ldo = a.I; e.amax_out = a.amax_h + (size_t)l * a.R;
    gemv_phase_rb<R, 2, true>(a, e, xs, ring, ss);
    if (!grid_sync(a, target, &ss.ok)) return;
    pf_slice(a, 4 * l + 3, pfb);
    quant_h_split<R>(a, l);
    if (!grid_sync(a, target, &ss.ok)) return;
    // ---- down (+ residual)
    stage_hq<R>(a, l, xs, ss);
    prof_mid(a, target);
    e.L = &Ly->down; e.epi = EPI_RESID; e.out = a.x; e.ldo = a.D; e.amax_out = nullptr;
    pf_slice(a, 4 * l + 4, pfb);                 // next layer's q|k|v (or the head)
    gemv_phase_rb<R, 1, true>(a, e, xs, ring, ss);
    if (!grid_sync(a, target, &ss.ok)) return;
  }
  // ---- head: logits (optional) and greedy argmax
  stage_norm<R>(a, a.gf, xs, ys, ss);
  StepEpi e;
  e.L = &a.head; e.epi = EPI_HEAD; e.out = a.logits; e.ldo = a.V; e.silu_t = a.silu_t; e.amax_out = nullptr;
  gemv_phase_rb<R, 1, false>(a, e, xs, ring, ss);
}

// ------------------------------------------------------------------ host side
static int step_sm_count() {
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

template <int R>
static cudaError_t step_attr() {
  static DevOnce done;                    // raised once to the ceiling, never lowered
  if (done.done()) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(k_step<R>, cudaFuncAttributeMaxDynamicSharedMemorySize, STEP_SMEM_MAX);
  if (e == cudaSuccess) done.set();
  return e;
}

static size_t step_smem(const StepArgs& a) {
  // activation rows, the GEMV rings, per-row partial sums (rows per CTA bounded with one CTA per SM)
  const int sms = step_sm_count();
  int rows = (a.V + sms - 1) / sms;
  rows = std::max(rows, 2 * ((a.I + sms - 1) / sms));
  rows = std::max(rows, (a.Nqkv + sms - 1) / sms);
  const size_t A = (((size_t)a.R * a.KMAX * 2 + 127) & ~(size_t)127) + (size_t)SNCW * STEP_RING * 32 * 16 +
                   (size_t)(rows + 2) * a.R * 8;
  const int Hd = a.H * a.hd;
  const size_t B = (((size_t)a.R * a.D * 2 + 127) & ~(size_t)127) + (size_t)2 * (a.D > Hd ? a.D : Hd) * 8;
  const size_t C = (size_t)STEP_REP_MAX * 128 * 2 + STEP_RMAX * 128 * (2 + 4) + (size_t)STEP_REP_MAX * a.att_chunk_max * 8 +
                   (size_t)ATT_TT * (128 + 8) * 2 + (size_t)ATT_TT * 128 * 4 + ATT_TT * 4;
  size_t s = A > B ? A : B;
  return s > C ? s : C;
}

int step_grid(const StepArgs& a, size_t* smem) {
  if (a.R < 1 || a.R > STEP_RMAX || a.KV <= 0 || a.H % a.KV || a.H / a.KV > STEP_REP_MAX || a.hd > 128 ||
      a.hd % 16 || a.D % 2 || a.I % 8 || a.KMAX < a.I || a.H * a.hd != a.D)
    return 0;
  if ((a.R == 1 ? step_attr<1>() : step_attr<2>()) != cudaSuccess) return 0;
  const size_t s = step_smem(a);
  if (s > STEP_SMEM_MAX) return 0;
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, a.R == 1 ? (const void*)k_step<1> : (const void*)k_step<2>,
                                                    STEP_THREADS, s) != cudaSuccess || per_sm < 1)
    return 0;
  if (smem) *smem = s;
  return step_sm_count();                  // one CTA per SM
}

cudaError_t launch_step(const StepArgs& a, cudaStream_t st) {
  size_t smem = 0;
  const int grid = step_grid(a, &smem);
  if (grid <= 0 || a.R * a.KV * a.att_split > grid) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(STEP_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeCooperative;
  at[0].val.cooperative = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return a.R == 1 ? cudaLaunchKernelEx(&cfg, k_step<1>, a) : cudaLaunchKernelEx(&cfg, k_step<2>, a);
}

}  // namespace exb
