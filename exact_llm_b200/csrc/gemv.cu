// K1: HBM-streaming exact GEMV for batch-1 / small-batch decode (CUDA cores, no tensor cores).
//
// For each activation row r and output column n of a group-128 linear
// (experiments/speed_fair_kaggle.py:722-725 of novain-shibu/exact-llm; SPEC.md:18)
//     tot[r, n] = sum_g M[n, g] * sum_{k in g} xq[r, k] * W[n, k]          (int64, exact)
// or, for a per-channel linear (exact_llm.py:89-96), acc[r, n] = sum_k xq[r, k] * W[n, k],
// followed by a fused epilogue (requant + bias, residual add, SwiGLU, greedy argmax, trace
// capture, Freivalds left/right-hand sides) and an optional last-CTA tail that builds the next
// GEMV's int16 input rows (RMSNorm + qrow, qrow, or RoPE + KV-cache write).
//
// B200 design: one CTA per SM.  Every CTA owns a contiguous range of output columns, i.e. one
// contiguous range of weight bytes (weights are (N, K) row-major, one K-byte row per column),
// cut into stages of a few columns.  Each of the 8 warps owns every 8th stage and its own slots of
// a shared-memory ring: it streams its stages with bulk asynchronous copies (cp.async.bulk,
// completion counted on an mbarrier per slot) -- weight rows and their group scales in one
// transaction -- so HBM traffic needs no registers, warps never wait on each other, and the
// first stages are requested before the programmatic-dependent-launch wait (weights never depend
// on the previous kernel).  Lane l handles the 16-byte chunks l, l+32, ... of a column: 16 MACs =
// 8 dp2a (int16 x int8 -> int32, exact since 16 * 32767 * 127 < 2^31), each chunk's int32 times
// its group scale into an int64 lane total, lanes combined by 64-bit shuffles; then lane u runs
// the epilogue of the stage's column u, so epilogue latencies overlap.  Integer addition is
// associative, so this order gives the reference's modulo-2^64 int64 result bit for bit.  Every
// mbarrier wait is bounded.
#include "common.cuh"
#include "exb_internal.h"
#include "rowdev.cuh"

namespace exb {

constexpr int NCW = 8;                          // warps; each streams and consumes its own stages
constexpr int XREG_CHUNKS = 8;                  // K <= 32 * 16 * 8 = 4096: activations live in registers
constexpr int L2_AHEAD = 2;                     // ring generations prefetched into L2 ahead of the copies
constexpr int GEMV_THREADS = 32 * NCW;
constexpr int STAGE_BYTES = 24 * 1024;          // target weight bytes per stage
constexpr int MAX_STAGES = 32;
constexpr int BAR_BYTES = MAX_STAGES * 8;       // full[] mbarriers at the start of shared memory

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

struct GemvPlan {        // host-computed stage geometry (passed by value)
  int SR;                // weight rows per stage (multiple of RPU)
  int NS;                // stages in the ring
  int stage_bytes;       // bytes per ring slot (weights + scales, 128-aligned)
  int xs_bytes;          // bytes of the staged int16 activations (128-aligned)
};

// Epilogue of one output unit (1 column, or a gate/up pair) for activation row r.
template <int RPU>
EXB_DEV void unit_epilogue(const GemvArgs& a, int ug, int r, const int64_t* t2, int sh, uint64_t& omax,
                           unsigned long long (&frl)[3][2], int64_t& best_v, int& best_n) {
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
    if (a.fr_nseg) {
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
  if (a.fr_nseg) {
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
    int64_t* o = a.out + (size_t)r * a.ldo + n;
    *o = (int64_t)((uint64_t)*o + (uint64_t)y);
  } else if (a.out) {
    a.out[(size_t)r * a.ldo + n] = y;
  }
  if (a.epi == EPI_HEAD && (y > best_v || (y == best_v && n < best_n))) {
    best_v = y;
    best_n = n;
  }
}

template <int R, int RPU, bool GROUP, bool XREG>
__global__ void __launch_bounds__(GEMV_THREADS, 1) k_gemv(const GemvArgs a, const GemvPlan P) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem_raw);                 // [MAX_STAGES]
  int16_t* xs = reinterpret_cast<int16_t*>(smem_raw + BAR_BYTES);         // R x K int16
  unsigned char* ring = smem_raw + BAR_BYTES + P.xs_bytes;                // NS x stage_bytes
  __shared__ unsigned long long red[NCW][R][6];
  __shared__ unsigned long long head_best[NCW][R][2];
  __shared__ uint64_t rred[33];
  __shared__ int sh_s[R];
  __shared__ int abort_flag;

  const int K = a.L.K, C = K >> 4, ldm = a.L.ldm;
  const int units = a.L.N / RPU;
  const int ulo = (int)((int64_t)units * blockIdx.x / gridDim.x);
  const int uhi = (int)((int64_t)units * (blockIdx.x + 1) / gridDim.x);
  const int row0 = ulo * RPU, nrows = (uhi - ulo) * RPU;
  const int nst = (nrows + P.SR - 1) / P.SR;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nact = P.NS < NCW ? P.NS : NCW;         // warps that stream (all, unless the ring is tiny)
  const int NSW = P.NS / nact;                      // ring slots owned by each streaming warp
  const int SU = P.SR / RPU;                        // units per full stage

  if (threadIdx.x == 0) {
    for (int i = 0; i < P.NS; ++i) mbar_init(&full[i], 1);
    abort_flag = 0;
    mbar_fence_init();
  }
  __syncthreads();

  // stage s belongs to warp s % nact; that warp's j-th stage (j = s / nact) lives in slot
  // warp * NSW + j % NSW and completes phase (j / NSW) of that slot's mbarrier
  auto issue = [&](int s) {
    const int j = s / nact, slot = warp * NSW + j % NSW;
    const int r0 = row0 + s * P.SR;
    const int rows = min(P.SR, nrows - s * P.SR);
    const uint32_t wb = (uint32_t)rows * K, mb = GROUP ? (uint32_t)rows * ldm * 4 : 0;
    unsigned char* dst = ring + (size_t)slot * P.stage_bytes;
    mbar_expect_tx(&full[slot], wb + mb);
    bulk_g2s(dst, a.L.w + (size_t)r0 * K, wb, &full[slot]);
    if (GROUP) bulk_g2s(dst + (size_t)P.SR * K, a.L.Mg + (size_t)r0 * ldm, mb, &full[slot]);
  };
  // HBM latency under full load is several microseconds -- more than the shared-memory ring can
  // cover -- so each warp also asks L2 for its stages L2_AHEAD ring generations ahead; the
  // bulk copies into shared memory then mostly hit L2.
  auto prefetch = [&](int s) {
    if (s >= nst) return;
    const int r0 = row0 + s * P.SR;
    const int rows = min(P.SR, nrows - s * P.SR);
    prefetch_l2_bulk(a.L.w + (size_t)r0 * K, (uint32_t)rows * K);
    if (GROUP) prefetch_l2_bulk(a.L.Mg + (size_t)r0 * ldm, (uint32_t)rows * ldm * 4);
  };
  // Weights never depend on the previous kernel: fill every warp's ring before the PDL wait.
  int issued = 0;                                   // stages issued by this warp (lane 0)
  if (lane == 0 && warp < nact) {
    for (int j = 0; j < NSW && warp + j * nact < nst; ++j) { issue(warp + j * nact); issued = j + 1; }
    for (int j = NSW; j < NSW * (1 + L2_AHEAD); ++j) prefetch(warp + j * nact);
  }

  int64_t best_v[R];
  int best_n[R];
  uint64_t omax[R];
  unsigned long long frl[R][3][2];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    best_v[r] = INT64_MIN;
    best_n[r] = 0x7fffffff;
    omax[r] = 0;
#pragma unroll
    for (int q = 0; q < 3; ++q) frl[r][q][0] = frl[r][q][1] = 0;
  }

  pdl_wait();
  if (blockIdx.x == 0 && a.zero)
    for (int i = threadIdx.x; i < a.nzero; i += GEMV_THREADS) a.zero[i] = 0;
  {
    const int n16 = K >> 3;                                   // int4 per activation row
    for (int i = threadIdx.x; i < R * n16; i += GEMV_THREADS) {
      const int r = i / n16, c = i - r * n16;
      reinterpret_cast<int4*>(xs + (size_t)r * K)[c] = reinterpret_cast<const int4*>(a.xq + (size_t)r * a.ldx)[c];
    }
    if (threadIdx.x < R) sh_s[threadIdx.x] = a.xs[threadIdx.x];
  }
  __syncthreads();
  int sh[R];
#pragma unroll
  for (int r = 0; r < R; ++r) sh[r] = sh_s[r];
  // XREG (R == 1, K <= 4096): a lane always multiplies the same activation chunks
  // lane + 32 i, so they are loaded once into registers instead of from shared memory per column
  int4 xr_a[XREG ? XREG_CHUNKS : 1], xr_b[XREG ? XREG_CHUNKS : 1];
  if (XREG) {
#pragma unroll
    for (int i = 0; i < XREG_CHUNKS; ++i) {
      const int ch = lane + 32 * i;
      if (ch < C) {
        const int4* xp = reinterpret_cast<const int4*>(xs + 16 * ch);
        xr_a[i] = xp[0];
        xr_b[i] = xp[1];
      } else {
        xr_a[i] = xr_b[i] = make_int4(0, 0, 0, 0);
      }
    }
  }

  for (int j = 0; warp < nact; ++j) {
    const int s = warp + j * nact;
    if (s >= nst) break;
    const int slot = warp * NSW + j % NSW;
    if (!mbar_wait(&full[slot], (j / NSW) & 1)) { abort_flag = 1; break; }
    const unsigned char* st = ring + (size_t)slot * P.stage_bytes;
    const int su = min(P.SR, nrows - s * P.SR) / RPU;
    int64_t mine[R][RPU];                           // lane u keeps unit u's totals
    for (int u = 0; u < su; ++u) {
      int64_t tot[R][RPU];
#pragma unroll
      for (int r = 0; r < R; ++r)
#pragma unroll
        for (int q = 0; q < RPU; ++q) tot[r][q] = 0;
      if (XREG) {
        // R == 1: activations in registers; chunk i of this lane is lane + 32 i
        int64_t tot2[RPU];
#pragma unroll
        for (int q = 0; q < RPU; ++q) tot2[q] = 0;
#pragma unroll
        for (int i = 0; i < XREG_CHUNKS; ++i) {
          const int ch = lane + 32 * i;
          if (ch < C) {
#pragma unroll
            for (int q = 0; q < RPU; ++q) {
              const int lr = u * RPU + q;
              const int4 wv = reinterpret_cast<const int4*>(st + (size_t)lr * K)[ch];
              const int32_t mv = GROUP ? reinterpret_cast<const int32_t*>(st + (size_t)P.SR * K)[lr * ldm + (ch >> 3)] : 1;
              const int p = dot16(wv, xr_a[i], xr_b[i]);
              const uint64_t term = (uint64_t)(GROUP ? (int64_t)p * mv : (int64_t)p);
              // two independent accumulators (even / odd chunks); uint64 wraps like numpy int64
              if (i & 1) tot2[q] = (int64_t)((uint64_t)tot2[q] + term);
              else tot[0][q] = (int64_t)((uint64_t)tot[0][q] + term);
            }
          }
        }
#pragma unroll
        for (int q = 0; q < RPU; ++q) tot[0][q] = (int64_t)((uint64_t)tot[0][q] + (uint64_t)tot2[q]);
      } else {
#pragma unroll 4
      for (int ch = lane; ch < C; ch += 32) {
        int4 wv[RPU];
        int32_t mv[RPU];
#pragma unroll
        for (int q = 0; q < RPU; ++q) {
          const int lr = u * RPU + q;                           // row within the stage
          wv[q] = reinterpret_cast<const int4*>(st + (size_t)lr * K)[ch];
          mv[q] = GROUP ? reinterpret_cast<const int32_t*>(st + (size_t)P.SR * K)[lr * ldm + (ch >> 3)] : 1;
        }
#pragma unroll
        for (int r = 0; r < R; ++r) {
          const int4* xp = reinterpret_cast<const int4*>(xs + (size_t)r * K + 16 * ch);
          const int4 xa = xp[0], xb = xp[1];
#pragma unroll
          for (int q = 0; q < RPU; ++q) {
            const int p = dot16(wv[q], xa, xb);
            // uint64 accumulation: any overflow wraps like numpy int64
            tot[r][q] = (int64_t)((uint64_t)tot[r][q] + (uint64_t)(GROUP ? (int64_t)p * mv[q] : (int64_t)p));
          }
        }
      }
      }
#pragma unroll
      for (int r = 0; r < R; ++r)
#pragma unroll
        for (int q = 0; q < RPU; ++q) {
#pragma unroll
          for (int o = 16; o > 0; o >>= 1)
            tot[r][q] = (int64_t)((uint64_t)tot[r][q] + (uint64_t)__shfl_xor_sync(0xffffffffu, tot[r][q], o));
          if (lane == u) mine[r][q] = tot[r][q];    // every lane holds the sum after the butterfly
        }
    }
    // slot fully read: hand it back to the bulk-copy engine for this warp's stage j + NSW
    __syncwarp();
    if (lane == 0 && s + NSW * nact < nst) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      issue(s + NSW * nact);
      issued = j + NSW + 1;
      prefetch(s + NSW * nact * (1 + L2_AHEAD));
    }
    // epilogues of this stage's units in parallel: lane u finishes unit u
    if (lane < su) {
      const int ug = ulo + s * SU + lane;
#pragma unroll
      for (int r = 0; r < R; ++r) unit_epilogue<RPU>(a, ug, r, mine[r], sh[r], omax[r], frl[r], best_v[r], best_n[r]);
    }
    if (*(volatile int*)&abort_flag) break;
  }
  __syncthreads();
  if (abort_flag) {
    // a bounded wait gave up: record it, let every copy this warp issued land (bounded), stop
    if (lane == 0) {
      set_err(a.err, ERR_WAIT_TIMEOUT);
      for (int j = 0; j < issued; ++j) mbar_wait(&full[warp * NSW + j % NSW], (j / NSW) & 1, 1u << 20);
    }
    __syncthreads();
    return;
  }
  // fold the per-lane epilogue state into lane 0 of each warp
#pragma unroll
  for (int r = 0; r < R; ++r) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const uint64_t om = __shfl_xor_sync(0xffffffffu, omax[r], o);
      omax[r] = om > omax[r] ? om : omax[r];
      const int64_t bv = __shfl_xor_sync(0xffffffffu, best_v[r], o);
      const int bn = __shfl_xor_sync(0xffffffffu, best_n[r], o);
      if (bv > best_v[r] || (bv == best_v[r] && bn < best_n[r])) { best_v[r] = bv; best_n[r] = bn; }
#pragma unroll
      for (int q = 0; q < 3; ++q) {
        frl[r][q][0] += __shfl_xor_sync(0xffffffffu, frl[r][q][0], o);
        frl[r][q][1] += __shfl_xor_sync(0xffffffffu, frl[r][q][1], o);
      }
    }
  }
  pdl_launch_dependents();

  // ---- per-row max |output| for the consumer's qrow (SwiGLU output)
  if (a.amax_out) {
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const uint64_t v = block_max_u64<GEMV_THREADS>(omax[r], rred);
      if (threadIdx.x == 0 && v) atomicMax(a.amax_out + r, (unsigned long long)v);
    }
  }
  // ---- Freivalds: per-CTA partial sums -> one atomic per (segment, row, prime)
  if (a.fr_nseg) {
    if (lane == 0) {
#pragma unroll
      for (int r = 0; r < R; ++r)
#pragma unroll
        for (int q = 0; q < 3; ++q) {
          red[warp][r][2 * q] = frl[r][q][0];
          red[warp][r][2 * q + 1] = frl[r][q][1];
        }
    }
    __syncthreads();
    if (threadIdx.x < R * 2 * a.fr_nseg) {
      const int r = threadIdx.x / (2 * a.fr_nseg), q = threadIdx.x % (2 * a.fr_nseg);
      unsigned long long s = 0;
      for (int w = 0; w < NCW; ++w) s += red[w][r][q];
      if (s) atomicAdd(a.fr_acc[q >> 1] + r * 4 + (q & 1), s);
    }
    // right-hand side: sum_k d_k (xq_k mod p), k range split over the grid
    const int k0 = (int)((int64_t)K * blockIdx.x / gridDim.x), k1 = (int)((int64_t)K * (blockIdx.x + 1) / gridDim.x);
    for (int sg = 0; sg < a.fr_nseg; ++sg) {
      for (int r = 0; r < R; ++r) {
#pragma unroll
        for (int pi = 0; pi < 2; ++pi) {
          unsigned long long s = 0;
          for (int k = k0 + (int)threadIdx.x; k < k1; k += GEMV_THREADS)
            s += mod_p(xs[(size_t)r * K + k], fr_prime(pi)) * (unsigned long long)a.fr_d[sg][pi * K + k] % fr_prime(pi);
          for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
          if (lane == 0 && s) atomicAdd(a.fr_acc[sg] + r * 4 + 2 + pi, s);
        }
      }
    }
  }
  // ---- greedy argmax (first index on ties, exact_llm.py:267): last-CTA reduction
  if (a.epi == EPI_HEAD && a.next_tok) {
    if (lane == 0) {
#pragma unroll
      for (int r = 0; r < R; ++r) {
        head_best[warp][r][0] = (unsigned long long)best_v[r];
        head_best[warp][r][1] = (unsigned long long)(unsigned)best_n[r];
      }
    }
    __syncthreads();
    if (threadIdx.x < R) {
      const int r = threadIdx.x;
      int64_t bv = INT64_MIN;
      int bn = 0x7fffffff;
      for (int w = 0; w < NCW; ++w) {
        const int64_t v = (int64_t)head_best[w][r][0];
        const int n = (int)head_best[w][r][1];
        if (v > bv || (v == bv && n < bn)) { bv = v; bn = n; }
      }
      a.head_part[((size_t)blockIdx.x * R + r) * 2 + 0] = (unsigned long long)bv;
      a.head_part[((size_t)blockIdx.x * R + r) * 2 + 1] = (unsigned long long)(unsigned)bn;
    }
    if (last_cta(a.head_ticket, gridDim.x) && threadIdx.x < R) {
      const int r = threadIdx.x;
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
  // ---- last CTA: build the next GEMV's int16 input rows from this kernel's complete output;
  // the activation staging area and the ring (contiguous) are free now and stage the row.
  if (a.tail != TAIL_NONE && last_cta(a.ticket, gridDim.x)) {
    int64_t* ys = reinterpret_cast<int64_t*>(smem_raw + BAR_BYTES);
    if (a.tail == TAIL_ROPE) {
      rope_cache_rows<GEMV_THREADS>(a.rope);
    } else if (a.tail == TAIL_NORM) {
      for (int r = 0; r < R; ++r)
        row_norm_q<GEMV_THREADS>(a.tail_x + (size_t)r * a.tail_ldx, a.tail_gain, a.tail_K,
                                 a.tail_xq + (size_t)r * a.tail_ldq, a.tail_xs + r, ys, rred);
    } else {
      for (int r = 0; r < R; ++r) {
        const int s = qrow_shift(__ldcg(a.tail_amax + r));
        row_quant_known<GEMV_THREADS>(a.tail_x + (size_t)r * a.tail_ldx, a.tail_K, s,
                                      a.tail_xq + (size_t)r * a.tail_ldq);
        if (threadIdx.x == 0) a.tail_xs[r] = s;
      }
    }
  }
}

template <int R, int RPU, bool GROUP, bool XREG>
static cudaError_t launch_t(const GemvArgs& a, const GemvPlan& P, size_t smem, cudaStream_t st, bool pdl) {
  auto kern = k_gemv<R, RPU, GROUP, XREG>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.grid);
  cfg.blockDim = dim3(GEMV_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, a, P);
}

template <int RPU, bool GROUP>
static cudaError_t launch_r(const GemvArgs& a, const GemvPlan& P, size_t smem, cudaStream_t st, bool pdl) {
  switch (a.R) {
    case 1:
      return a.L.K <= 32 * 16 * XREG_CHUNKS ? launch_t<1, RPU, GROUP, true>(a, P, smem, st, pdl)
                                            : launch_t<1, RPU, GROUP, false>(a, P, smem, st, pdl);
    case 2: return launch_t<2, RPU, GROUP, false>(a, P, smem, st, pdl);
    case 3: return launch_t<3, RPU, GROUP, false>(a, P, smem, st, pdl);
    case 4: return launch_t<4, RPU, GROUP, false>(a, P, smem, st, pdl);
    default: return cudaErrorInvalidValue;
  }
}

static int sm_count() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

int gemv_grid(int N, bool swiglu) {
  const int units = swiglu ? N / 2 : N;
  const int sms = sm_count();
  return units < sms ? units : sms;
}

cudaError_t launch_gemv(const GemvArgs& a0, cudaStream_t st, bool pdl) {
  GemvArgs a = a0;
  const bool group = a.L.Mg != nullptr;
  const int RPU = a.epi == EPI_SWIGLU ? 2 : 1;
  if ((group ? a.L.K % 128 : a.L.K % 16) != 0 || a.L.N <= 0 || a.R < 1 || a.R > 4) return cudaErrorInvalidValue;
  if (group && (a.L.ldm < a.L.K / 128 || a.L.ldm % 4 || ((uintptr_t)a.L.Mg & 15))) return cudaErrorInvalidValue;
  if (((uintptr_t)a.L.w & 15) || ((uintptr_t)a.xq & 15) || (a.ldx % 8)) return cudaErrorInvalidValue;
  if (RPU == 2 && (a.L.N & 1)) return cudaErrorInvalidValue;
  if (a.grid <= 0) a.grid = gemv_grid(a.L.N, RPU == 2);
  GemvPlan P;
  const int K = a.L.K;
  const size_t budget = 200 * 1024;
  P.xs_bytes = ((a.R * K * 2) + 127) & ~127;
  if ((size_t)P.xs_bytes + BAR_BYTES >= budget) return cudaErrorInvalidValue;
  const size_t avail = budget - BAR_BYTES - P.xs_bytes;
  const int row_bytes = K + (group ? a.L.ldm * 4 : 0);
  // stage size: two slots per consumer warp when that leaves at least one unit per stage
  size_t target = avail / (2 * NCW);
  if (target < (size_t)RPU * row_bytes) target = avail / NCW;
  P.SR = (int)(target / row_bytes);
  if (P.SR > STAGE_BYTES / K) P.SR = STAGE_BYTES / K;
  {  // spread a CTA's columns over all consumer warps
    const int units = a.L.N / RPU;
    const int rows_cta = ((units + a.grid - 1) / a.grid) * RPU;
    const int per_warp = ((rows_cta + NCW - 1) / NCW + RPU - 1) / RPU * RPU;
    if (P.SR > per_warp) P.SR = per_warp;
  }
  if (P.SR > 32 * RPU) P.SR = 32 * RPU;            // lane u finishes unit u of a stage
  if (P.SR < RPU) P.SR = RPU;
  P.SR -= P.SR % RPU;
  P.stage_bytes = (P.SR * row_bytes + 127) & ~127;
  int NS = (int)(avail / P.stage_bytes);
  if (NS > MAX_STAGES) NS = MAX_STAGES;
  if (NS >= NCW) NS -= NS % NCW;                   // every streaming warp owns NS / min(NS, 8) slots
  const size_t need_tail = a.tail == TAIL_NORM ? (size_t)a.tail_K * 16 : 0;
  if (NS < 1) return cudaErrorInvalidValue;
  if ((size_t)P.xs_bytes + (size_t)NS * P.stage_bytes < need_tail) return cudaErrorInvalidValue;
  P.NS = NS;
  const size_t smem = BAR_BYTES + P.xs_bytes + (size_t)NS * P.stage_bytes;
  if (RPU == 2) return group ? launch_r<2, true>(a, P, smem, st, pdl) : launch_r<2, false>(a, P, smem, st, pdl);
  return group ? launch_r<1, true>(a, P, smem, st, pdl) : launch_r<1, false>(a, P, smem, st, pdl);
}

// ---------------------------------------------------------------------------------------------
// Drop-in for the reference operator exact::gemv(x16 int16[K], wT int8[N,K], Mg int64[N,G]) ->
// int64[N] (experiments/speed_fair_kaggle.py:662-702): raw tot, int64 scales read as given.
__global__ void __launch_bounds__(256) k_gemv_op(const int16_t* __restrict__ x, const int8_t* __restrict__ wT,
                                                 const int64_t* __restrict__ Mg, int K, int N, int64_t* __restrict__ out) {
  extern __shared__ __align__(16) unsigned char smem_op[];
  int16_t* xs = reinterpret_cast<int16_t*>(smem_op);
  for (int i = threadIdx.x; i < (K >> 3); i += 256) reinterpret_cast<int4*>(xs)[i] = reinterpret_cast<const int4*>(x)[i];
  __syncthreads();
  const int C = K >> 4, G = K >> 7;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int n = blockIdx.x * 8 + warp; n < N; n += gridDim.x * 8) {
    const int4* wr = reinterpret_cast<const int4*>(wT + (size_t)n * K);
    int64_t tot = 0;
    for (int ch = lane; ch < C; ch += 32) {
      const int4 w = ldg_stream(wr + ch);
      const int4* xp = reinterpret_cast<const int4*>(xs + 16 * ch);
      const int p = dot16(w, xp[0], xp[1]);
      tot = (int64_t)((uint64_t)tot + (uint64_t)p * (uint64_t)Mg[(size_t)n * G + (ch >> 3)]);
    }
    for (int o = 16; o > 0; o >>= 1) tot = (int64_t)((uint64_t)tot + (uint64_t)__shfl_xor_sync(0xffffffffu, tot, o));
    if (lane == 0) out[n] = tot;
  }
}

cudaError_t launch_gemv_op(const int16_t* x16, const int8_t* wT, const int64_t* Mg, int K, int N, int64_t* out,
                           cudaStream_t st) {
  if (K % 128 != 0 || N <= 0) return cudaErrorInvalidValue;
  const size_t smem = (size_t)K * 2;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(k_gemv_op, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  int blocks = (N + 7) / 8;
  if (blocks > 148 * 8) blocks = 148 * 8;
  k_gemv_op<<<blocks, 256, smem, st>>>(x16, wT, Mg, K, N, out);
  return cudaGetLastError();
}

}  // namespace exb
