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
// B200 design (from a read-bandwidth calibration on this pool: plain 128-bit loads from 2 CTAs x
// 512 threads per SM stream HBM at ~98% of the measured copy peak, bulk-copy rings at ~85%):
// every CTA owns a contiguous range of output columns = one contiguous range of weight bytes
// (weights are (N, K) row-major, one K-byte row per column).  Each warp takes blocks of RB
// columns; lane l loads the 16-byte chunks l, l+32, ... of a column in batches of up to 8
// independent 128-bit non-allocating loads (their group scales alongside), computes 16 MACs per
// chunk as 8 dp2a (int16 x int8 -> int32, exact since 16 * 32767 * 127 < 2^31) against the int16
// activations in shared memory, and multiplies each chunk's int32 by its group scale into an int64
// lane partial.  The RB columns' partials are combined across the warp by recursive halving
// (RB - 1 + 5 - log2 RB 64-bit shuffles instead of 5 RB), which leaves column b's total in lane
// b * 32/RB, and those RB lanes run the epilogues in parallel.  The CTA's first weight bytes are
// prefetched into L2 before the programmatic-dependent-launch wait.  Integer addition is
// associative, so this order gives the reference's modulo-2^64 int64 result bit for bit.
#include "common.cuh"
#include "exb_internal.h"
#include "rowdev.cuh"
#include "tpx.cuh"
#include "gemvdev.cuh"

namespace exb {

constexpr int NCW = 16;                         // warps per CTA
constexpr int GEMV_THREADS = 32 * NCW;          // 2 CTAs per SM (64 registers per thread)
constexpr int PREFETCH_BYTES = 64 * 1024;       // per-CTA L2 prefetch before the PDL wait
constexpr int DYN_SMEM_MAX = 200 * 1024;        // dynamic shared memory budget of one CTA
constexpr int PRE_SMEM_MAX = 104 * 1024;        // with the pre-wait area: two CTAs still fit one SM

// MODE: 0 lean (the decode hot path: int16 or qrow inputs, store / residual / SwiGLU / raw
// epilogues, no Freivalds, tails, norm prologues, row statistics or argmax), 1 full, 2 lean with the
// tensor-parallel exchanges, 3 lean with the norm prologue (row staged in shared memory), 4 lean with
// the greedy argmax (the decode head).  Each is its own instantiation: code a launch never runs still costs
// registers (spills) in the streaming loop.
template <int R, int RPU, bool GROUP, int RB, int MODE>
__global__ void __launch_bounds__(GEMV_THREADS, 2) k_gemv(const GemvArgs a) {
  constexpr bool LEAN = MODE != 1, TPX = MODE == 2, NORMP = MODE == 1 || MODE == 3, HEADA = MODE == 1 || MODE == 4;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  int16_t* xs = reinterpret_cast<int16_t*>(smem_raw);                    // R x K int16 (tail: D int64 x 2)
  __shared__ unsigned long long red[NCW][R][6];
  __shared__ unsigned long long head_best[NCW][R][2];
  __shared__ uint64_t rred[33];
  __shared__ int sh_s[R];
  __shared__ EpiState est[NCW][RB][R];
  constexpr int CPL = RB == 1 ? 8 : 4;              // chunks per lane per load batch
  constexpr int PAY = R * RPU;                      // int64 totals per column block entry

  const int K = a.L.K, C = K >> 4, ldm = a.L.ldm;
  const int units = a.L.N / RPU;
  const int ulo = (int)((int64_t)units * blockIdx.x / gridDim.x);
  const int uhi = (int)((int64_t)units * (blockIdx.x + 1) / gridDim.x);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // Weights never depend on the previous kernel: pull this CTA's first bytes into L2 before the
  // PDL wait (fire-and-forget; no completion to wait for).
  if (threadIdx.x == 0 && uhi > ulo) {
    const char* w0 = reinterpret_cast<const char*>(a.L.w) + (size_t)ulo * RPU * K;
    size_t bytes = (size_t)(uhi - ulo) * RPU * K;
    bytes = bytes > PREFETCH_BYTES ? PREFETCH_BYTES : bytes;
    for (size_t off = 0; off < bytes; off += 16384)
      prefetch_l2_bulk(w0 + off, (uint32_t)(bytes - off < 16384 ? bytes - off : 16384));
  }

  // The group scales, per-channel multipliers and biases of this CTA's columns are weights too:
  // one 128-byte line per thread into L2 before the wait, so the epilogue never waits on HBM.
  if (uhi > ulo) {
    const int n0 = ulo * RPU, n1 = uhi * RPU;
    int t = threadIdx.x;
    auto pf_lines = [&](const void* p0, const void* p1) {
      const uintptr_t a0 = reinterpret_cast<uintptr_t>(p0) & ~(uintptr_t)127;
      const int nl = (int)((reinterpret_cast<uintptr_t>(p1) - a0 + 127) >> 7);
      if (t >= 0 && t < nl) asm volatile("prefetch.global.L2 [%0];" ::"l"(a0 + ((uintptr_t)t << 7)));
      t -= nl;
    };
    if (GROUP) pf_lines(a.L.Mg + (size_t)n0 * ldm, a.L.Mg + (size_t)n1 * ldm);
    if (a.L.Mc) pf_lines(a.L.Mc + n0, a.L.Mc + n1);
    if (a.L.b) pf_lines(a.L.b + n0, a.L.b + n1);
  }

  // Weights never depend on the previous kernel either: each warp's first load batch (its first
  // column's first CPL chunks per lane) is copied to a lane-private shared-memory area before the
  // wait, its group scales held in registers, so the first round of HBM latency overlaps the
  // previous kernel instead of following it.
  const int nblk = (uhi - ulo + RB - 1) / RB;
  const bool pre = a.pre_off > 0 && warp < nblk;
  int4* pre_s = reinterpret_cast<int4*>(smem_raw + a.pre_off) + (size_t)warp * CPL * 32;
  int32_t* pre_m = reinterpret_cast<int32_t*>(reinterpret_cast<int4*>(smem_raw + a.pre_off) + (size_t)NCW * CPL * 32) +
                   (size_t)warp * CPL * 32;
  if (pre) {
    const int n = (ulo + warp * RB) * RPU;
    const int4* wrow = reinterpret_cast<const int4*>(a.L.w + (size_t)n * K);
    const int32_t* mrow = GROUP ? a.L.Mg + (size_t)n * ldm : nullptr;
#pragma unroll
    for (int i = 0; i < CPL; ++i) {
      const int ch = lane + 32 * i;
      if (ch < C) {
        cp_async16(pre_s + i * 32 + lane, wrow + ch);
        if (GROUP) cp_async4(pre_m + i * 32 + lane, mrow + (ch >> 3));
      }
    }
    cp_async_commit();
  }

  if (lane < RB)
    for (int r = 0; r < R; ++r) {
      EpiState& E = est[warp][lane][r];
      for (int q = 0; q < 3; ++q) E.frl[q][0] = E.frl[q][1] = 0;
      E.omax = 0;
      E.ssq = 0;
      E.best_v = INT64_MIN;
      E.best_n = 0x7fffffff;
    }

  pdl_wait();
  if (blockIdx.x == 0 && a.zero)
    for (int i = threadIdx.x; i < a.nzero; i += GEMV_THREADS) a.zero[i] = 0;
  if (blockIdx.x == 0 && a.zero2)
    for (int i = threadIdx.x; i < a.nzero2; i += GEMV_THREADS) a.zero2[i] = 0;
  if (a.xin == XIN_Q16) {
    const int n16 = K >> 3;                                   // int4 per activation row
    for (int i = threadIdx.x; i < R * n16; i += GEMV_THREADS) {
      const int r = i / n16, c = i - r * n16;
      reinterpret_cast<int4*>(xs + (size_t)r * K)[c] = reinterpret_cast<const int4*>(a.xq + (size_t)r * a.ldx)[c];
    }
    if (threadIdx.x < R) sh_s[threadIdx.x] = a.xs[threadIdx.x];
  } else if (!LEAN && a.xin == XIN_NORMST) {
    // the norm from the row statistics the producers published (max |x|, sum x^2); the full
    // routine when irms would shift the row (max |x| >= 2^24) or the row is too long for registers
    int64_t* ys = reinterpret_cast<int64_t*>(smem_raw + (((size_t)R * K * 2 + 127) & ~(size_t)127));
    for (int r = 0; r < R; ++r) {
      const uint64_t mx = __ldcg(a.nstat_in + 2 * r), ss = __ldcg(a.nstat_in + 2 * r + 1);
      if (!row_norm_q_stats<GEMV_THREADS>(a.x64 + (size_t)r * a.ldx64, a.gain, K, mx, ss, xs + (size_t)r * K, &sh_s[r],
                                          rred))
        row_norm_q_any<GEMV_THREADS>(a.x64 + (size_t)r * a.ldx64, a.gain, K, xs + (size_t)r * K, &sh_s[r], ys, rred);
    }
  } else if (NORMP && a.xin == XIN_NORM) {
    // xq, s = qrow(irms(x, g)) for every row, computed by this CTA (exact_llm.py:100-106, 41-46)
    int64_t* ys = reinterpret_cast<int64_t*>(smem_raw + (((size_t)R * K * 2 + 127) & ~(size_t)127));
    for (int r = 0; r < R; ++r) {
      if constexpr (LEAN)     // one routine only: the row and gains staged in shared memory
        row_norm_q<GEMV_THREADS>(a.x64 + (size_t)r * a.ldx64, a.gain, K, xs + (size_t)r * K, &sh_s[r], ys, rred);
      else
        row_norm_q_any<GEMV_THREADS>(a.x64 + (size_t)r * a.ldx64, a.gain, K, xs + (size_t)r * K, &sh_s[r], ys, rred);
    }
  } else {
    // xq = clip(shr(x, s)) with s from the producer's published row max (exact_llm.py:41-46); under
    // tensor parallelism the max over every rank's rows, from the fused exchange
    if (TPX && a.tpx_in >= 0) tpx_wait(*a.tpx, a.tpx_in, R);
    for (int r = 0; r < R; ++r) {
      const int s = TPX && a.tpx_in >= 0 ? tpx_shift(*a.tpx, a.tpx_in == TPX_AMAX_O ? 0 : 1, r)
                                         : qrow_shift(__ldcg(a.amax_in + r));
      row_quant_known<GEMV_THREADS>(a.x64 + (size_t)r * a.ldx64, K, s, xs + (size_t)r * K);
      if (threadIdx.x == 0) sh_s[r] = s;
    }
  }
  __syncthreads();
  tl_point(0);
  pdl_launch_dependents();
  int sh[R];
#pragma unroll
  for (int r = 0; r < R; ++r) sh[r] = sh_s[r];

  for (int blk = warp; blk < nblk; blk += NCW) {
    const int u0 = ulo + blk * RB;
    int64_t acc[RB][PAY];
#pragma unroll
    for (int b = 0; b < RB; ++b)
#pragma unroll
      for (int p = 0; p < PAY; ++p) acc[b][p] = 0;
#pragma unroll
    for (int b = 0; b < RB; ++b) {
      const int u = u0 + b;
      if (u < uhi) {
#pragma unroll
        for (int q = 0; q < RPU; ++q) {
          const int n = u * RPU + q;
          const int4* wrow = reinterpret_cast<const int4*>(a.L.w + (size_t)n * K);
          const int32_t* mrow = GROUP ? a.L.Mg + (size_t)n * ldm : nullptr;
          for (int c0 = 0; c0 < C; c0 += 32 * CPL) {
            int4 wv[CPL];
            int32_t mv[CPL];
            if (b == 0 && q == 0 && pre && c0 == 0 && blk == warp) {
              cp_async_wait<0>();                      // this lane's own copies
              tl_point(3);
#pragma unroll
              for (int i = 0; i < CPL; ++i) {
                const int ch = lane + 32 * i;
                wv[i] = ch < C ? pre_s[i * 32 + lane] : make_int4(0, 0, 0, 0);
                mv[i] = ch < C ? (GROUP ? pre_m[i * 32 + lane] : 1) : 0;
              }
            } else {
#pragma unroll
              for (int i = 0; i < CPL; ++i) {
                const int ch = c0 + lane + 32 * i;
                if (ch < C) {
                  wv[i] = ldg_stream(wrow + ch);
                  mv[i] = GROUP ? __ldg(mrow + (ch >> 3)) : 1;
                } else {
                  wv[i] = make_int4(0, 0, 0, 0);
                  mv[i] = 0;
                }
              }
            }
#pragma unroll
            for (int i = 0; i < CPL; ++i) {
              const int ch = c0 + lane + 32 * i;
              if (ch < C) {
#pragma unroll
                for (int r = 0; r < R; ++r) {
                  const int4* xp = reinterpret_cast<const int4*>(xs + (size_t)r * K + 16 * ch);
                  const int p = dot16(wv[i], xp[0], xp[1]);
                  // uint64 accumulation: any overflow wraps like numpy int64
                  acc[b][r * RPU + q] = (int64_t)((uint64_t)acc[b][r * RPU + q] +
                                                  (uint64_t)(GROUP ? (int64_t)p * mv[i] : (int64_t)p));
                }
              }
            }
          }
        }
      }
    }
    if (blk == warp) tl_point(4);
    warp_reduce_halving<RB, PAY>(acc);
    if (blk == warp) tl_point(5);
    // lane b * (32 / RB) holds the totals of column block entry b: run its epilogue
    if ((lane & (32 / RB - 1)) == 0) {
      const int b = lane / (32 / RB);
      const int ug = u0 + b;
      if (ug < uhi) {
#pragma unroll
        for (int r = 0; r < R; ++r) {
          int64_t t2[RPU];
#pragma unroll
          for (int q = 0; q < RPU; ++q) t2[q] = acc[0][r * RPU + q];
          unit_epilogue<RPU, LEAN, HEADA>(a, ug, r, t2, sh[r], est[warp][b][r]);
          if constexpr (TPX && RPU == 1)
            if (a.tpx_out == TPX_SUM_O || a.tpx_out == TPX_SUM_D) {   // partial sums into every peer's slot
              const TpX& x = *a.tpx;
              const int which = a.tpx_out == TPX_SUM_O ? 0 : 1;
              for (int q = 0; q < x.size; ++q)
                if (q != x.rank) tpx_sum_slot(x, q, which, x.rank)[(size_t)r * x.D + ug] = t2[0];
            }
        }
      }
    }
    if (blk == warp) tl_point(6);
  }
  __syncwarp();
  tl_point(1);
  // fold this warp's epilogue states (one per column-block entry) into lane-0 values
  uint64_t omax[R], ssq[R];
  int64_t best_v[R];
  int best_n[R];
  unsigned long long frl[R][3][2];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    omax[r] = 0;
    ssq[r] = 0;
    best_v[r] = INT64_MIN;
    best_n[r] = 0x7fffffff;
#pragma unroll
    for (int q = 0; q < 3; ++q) frl[r][q][0] = frl[r][q][1] = 0;
    for (int b = 0; b < RB; ++b) {
      const EpiState& E = est[warp][b][r];
      omax[r] = E.omax > omax[r] ? E.omax : omax[r];
      ssq[r] += E.ssq;
      if (E.best_v > best_v[r] || (E.best_v == best_v[r] && E.best_n < best_n[r])) { best_v[r] = E.best_v; best_n[r] = E.best_n; }
#pragma unroll
      for (int q = 0; q < 3; ++q) { frl[r][q][0] += E.frl[q][0]; frl[r][q][1] += E.frl[q][1]; }
    }
  }
  __syncthreads();
  tl_point(2);

  // ---- per-row max |output| for the consumer's qrow (SwiGLU output)
  if (a.amax_out) {
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const uint64_t v = block_max_u64<GEMV_THREADS>(lane == 0 ? omax[r] : 0, rred);
      if (threadIdx.x == 0 && v) atomicMax(a.amax_out + r, (unsigned long long)v);
    }
  }
  // ---- residual row statistics for the next norm (max |x_new|, sum x_new^2), one atomic each per CTA
  if (!LEAN && a.nstat_out) {
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const uint64_t v = block_max_u64<GEMV_THREADS>(lane == 0 ? omax[r] : 0, rred);
      if (threadIdx.x == 0 && v) atomicMax(a.nstat_out + 2 * r, (unsigned long long)v);
      const uint64_t sq = (uint64_t)block_sum_i64<GEMV_THREADS>(lane == 0 ? (int64_t)ssq[r] : 0, rred);
      if (threadIdx.x == 0 && sq) atomicAdd(a.nstat_out + 2 * r + 1, (unsigned long long)sq);
    }
  }
  // ---- Freivalds: per-CTA partial sums -> one atomic per (segment, row, prime)
  if (!LEAN && a.fr_nseg) {
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
  if (HEADA && a.epi == EPI_HEAD && a.next_tok) {
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
      if (a.head_val) a.head_val[r] = bv;                  // tensor parallel: the shard's best value
    }
  }
  // ---- tensor parallel: the last CTA publishes this kernel's exchange (every CTA's peer stores
  // are ordered before its ticket by the election's fence and barrier)
  if (TPX && a.tpx_out >= 0) {
    if (last_cta(a.tpx_ticket, gridDim.x)) {
      if (a.tpx_out == TPX_AMAX_H) tpx_publish_max(*a.tpx, TPX_AMAX_H, a.amax_out, R);
      else tpx_signal(*a.tpx, a.tpx_out);
    }
  }
  // ---- last CTA: build the next GEMV's int16 input rows from this kernel's complete output;
  // the activation staging area and the ring (contiguous) are free now and stage the row.
  if (!LEAN && a.tail != TAIL_NONE && last_cta(a.ticket, gridDim.x)) {
    int64_t* ys = reinterpret_cast<int64_t*>(smem_raw);
    if (a.tail == TAIL_ROPE) {
      rope_cache_rows<GEMV_THREADS>(a.rope);
    } else if (a.tail == TAIL_NORM) {
      for (int r = 0; r < R; ++r) {
        bool done = false;
        if (a.tail_nstat)     // the statistics every CTA published before the election
          done = row_norm_q_stats<GEMV_THREADS>(a.tail_x + (size_t)r * a.tail_ldx, a.tail_gain, a.tail_K,
                                                __ldcg(a.tail_nstat + 2 * r), __ldcg(a.tail_nstat + 2 * r + 1),
                                                a.tail_xq + (size_t)r * a.tail_ldq, a.tail_xs + r, rred);
        if (!done)
          row_norm_q_any<GEMV_THREADS>(a.tail_x + (size_t)r * a.tail_ldx, a.tail_gain, a.tail_K,
                                       a.tail_xq + (size_t)r * a.tail_ldq, a.tail_xs + r, ys, rred);
      }
    } else {
      for (int r = 0; r < R; ++r) {
        const int s = qrow_shift(__ldcg(a.tail_amax + r));
        row_quant_known<GEMV_THREADS>(a.tail_x + (size_t)r * a.tail_ldx, a.tail_K, s,
                                      a.tail_xq + (size_t)r * a.tail_ldq);
        if (threadIdx.x == 0) a.tail_xs[r] = s;
      }
    }
  }
  tl_exit();
}

template <int R, int RPU, bool GROUP, int RB, int MODE>
static cudaError_t launch_t(const GemvArgs& a, size_t smem, cudaStream_t st, bool pdl) {
  auto kern = k_gemv<R, RPU, GROUP, RB, MODE>;
  // The max-dynamic-shared-memory attribute is raised once to the full budget and never lowered:
  // launches of one instantiation use different sizes, and a captured graph node (or a profiler
  // replay) must never find a smaller maximum than it was launched with.
  static DevOnce attr_set;
  if (!attr_set.done()) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, DYN_SMEM_MAX);
    if (e != cudaSuccess) return e;
    attr_set.set();
  }
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
  return cudaLaunchKernelEx(&cfg, kern, a);
}

template <int RPU, bool GROUP, int MODE>
static cudaError_t launch_m(const GemvArgs& a, size_t smem, cudaStream_t st, bool pdl) {
  switch (a.R) {
    case 1: return a.rb == 1 ? launch_t<1, RPU, GROUP, 1, MODE>(a, smem, st, pdl)
                             : launch_t<1, RPU, GROUP, 4, MODE>(a, smem, st, pdl);
    case 2: return launch_t<2, RPU, GROUP, 2, MODE>(a, smem, st, pdl);
    case 3: return launch_t<3, RPU, GROUP, 1, MODE>(a, smem, st, pdl);
    case 4: return launch_t<4, RPU, GROUP, 1, MODE>(a, smem, st, pdl);
    default: return cudaErrorInvalidValue;
  }
}

template <int RPU, bool GROUP>
static cudaError_t launch_r(const GemvArgs& a, size_t smem, cudaStream_t st, bool pdl) {
  const bool lean = a.fr_nseg == 0 && a.tail == TAIL_NONE && (a.xin == XIN_Q16 || a.xin == XIN_QUANT) &&
                    !a.nstat_out && a.epi != EPI_HEAD;
  if (a.tpx) {                       // tensor-parallel decode exchanges (group-128 models, lean launches)
    if constexpr (GROUP) {
      if (lean) return launch_m<RPU, GROUP, 2>(a, smem, st, pdl);
    }
    return cudaErrorInvalidValue;
  }
  if (lean) return launch_m<RPU, GROUP, 0>(a, smem, st, pdl);
  const bool head_lean = a.fr_nseg == 0 && a.tail == TAIL_NONE && (a.xin == XIN_Q16 || a.xin == XIN_QUANT) &&
                         !a.nstat_out && a.epi == EPI_HEAD;
  if (head_lean) return launch_m<RPU, GROUP, 4>(a, smem, st, pdl);
  const bool norm_lean = a.fr_nseg == 0 && a.tail == TAIL_NONE && a.xin == XIN_NORM && !a.nstat_out &&
                         a.epi != EPI_HEAD;
  return norm_lean ? launch_m<RPU, GROUP, 3>(a, smem, st, pdl) : launch_m<RPU, GROUP, 1>(a, smem, st, pdl);
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
  const int ctas = 2 * sm_count();                 // 2 CTAs of 512 threads per SM
  const int g = (units + 3) / 4;                   // at least 4 columns per CTA
  return g < ctas ? (g > 0 ? g : 1) : ctas;
}

cudaError_t launch_gemv(const GemvArgs& a0, cudaStream_t st, bool pdl) {
  GemvArgs a = a0;
  const bool group = a.L.Mg != nullptr;
  const int RPU = a.epi == EPI_SWIGLU ? 2 : 1;
  if ((group ? a.L.K % 128 : a.L.K % 16) != 0 || a.L.N <= 0 || a.R < 1 || a.R > 4) return cudaErrorInvalidValue;
  if (group && (a.L.ldm < a.L.K / 128)) return cudaErrorInvalidValue;
  if (a.xin == XIN_Q16 && (((uintptr_t)a.xq & 15) || (a.ldx % 8))) return cudaErrorInvalidValue;
  if (a.xin != XIN_Q16 && (((uintptr_t)a.x64 & 15) || (a.ldx64 & 1) || (a.L.K & 1))) return cudaErrorInvalidValue;
  if ((uintptr_t)a.L.w & 15) return cudaErrorInvalidValue;
  if (RPU == 2 && (a.L.N & 1)) return cudaErrorInvalidValue;
  if (a.grid <= 0) a.grid = gemv_grid(a.L.N, RPU == 2);
  if (a.rb <= 0) {
    // one column per warp when the grid has a warp for (nearly) every column: every load of the
    // kernel is then issued in one round; otherwise blocks of 4 columns amortise the reduction
    const int units = a.L.N / RPU;
    a.rb = units <= a.grid * NCW * 2 ? 1 : 4;
  }
  size_t smem = (((size_t)a.R * a.L.K * 2 + 127) & ~(size_t)127);
  if (a.xin == XIN_NORM || (a.xin == XIN_NORMST && a.L.K > 12 * GEMV_THREADS))
    smem += (size_t)a.L.K * 16;                                                              // row + gains
  if (a.xin == XIN_NORMST && !a.nstat_in) return cudaErrorInvalidValue;
  if (a.tail == TAIL_NORM && smem < (size_t)a.tail_K * 16) smem = (size_t)a.tail_K * 16;   // tail stages row + gains
  if (smem > DYN_SMEM_MAX) return cudaErrorInvalidValue;
  a.pre_off = 0;
  if (a.pre != 0) {
    // the pre-wait area: NCW warps x CPL chunks x 32 lanes x 16 bytes, when two CTAs per SM fit
    const size_t off = (smem + 127) & ~(size_t)127;
    const int rb_eff = a.R == 1 ? a.rb : (a.R == 2 ? 2 : 1);     // the RB launch_r instantiates
    const size_t bytes = (size_t)NCW * (rb_eff == 1 ? 8 : 4) * 32 * 20;   // 16-byte chunk + its scale
    if (off + bytes <= PRE_SMEM_MAX) {
      a.pre_off = (int)off;
      smem = off + bytes;
    }
  }
  if (RPU == 2) return group ? launch_r<2, true>(a, smem, st, pdl) : launch_r<2, false>(a, smem, st, pdl);
  return group ? launch_r<1, true>(a, smem, st, pdl) : launch_r<1, false>(a, smem, st, pdl);
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
  if (smem > DYN_SMEM_MAX) return cudaErrorInvalidValue;
  static DevOnce attr_set;
  if (!attr_set.done()) {
    cudaError_t e = cudaFuncSetAttribute(k_gemv_op, cudaFuncAttributeMaxDynamicSharedMemorySize, DYN_SMEM_MAX);
    if (e != cudaSuccess) return e;
    attr_set.set();
  }
  int blocks = (N + 7) / 8;
  if (blocks > 148 * 8) blocks = 148 * 8;
  k_gemv_op<<<blocks, 256, smem, st>>>(x16, wT, Mg, K, N, out);
  return cudaGetLastError();
}

}  // namespace exb
