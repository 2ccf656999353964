// K1: HBM-streaming exact GEMV for batch-1 / small-batch decode (no tensor cores).
//
// Computes, for each activation row r and output column n of a group-128 linear
// (experiments/speed_fair_kaggle.py:722-725 of novain-shibu/exact-llm; SPEC.md:18),
//     tot[r, n] = sum_g M[n, g] * sum_{k in g} xq[r, k] * W[n, k]          (int64, exact)
// or, for a per-channel linear (exact_llm.py:89-96), acc[r, n] = sum_k xq[r, k] * W[n, k],
// followed by a fused epilogue (requant + bias, residual add, SwiGLU, greedy head argmax,
// trace capture and the Freivalds left-hand side).
//
// Design (B200): one CTA per slice of output columns, rows split evenly by bytes over the
// whole grid.  Each warp owns whole output columns; lane l streams the 16-byte chunks
// l, l+32, ... of the column's K int8 weights with 128-bit non-allocating loads (4 chunks in
// flight per lane per column), so a warp reads 512 contiguous bytes per step.  The int16
// activations of all R rows sit in shared memory and are read as two 128-bit words per chunk.
// A chunk is 16 MACs = 8 dp2a (int16 x int8 -> int32), exact because |16 * 32767 * 127| < 2^31;
// each chunk's int32 partial is multiplied by its group scale into an int64 lane total (a lane's
// chunks never share a group, so no int32 group sum is needed), and lane totals are combined with
// a butterfly of 64-bit shuffles.  Integer addition is associative, so the result does not depend
// on this order: it equals the reference's modulo-2^64 int64 result bit for bit.
#include "common.cuh"
#include "exb_internal.h"

namespace exb {

constexpr int GEMV_THREADS = 256;
constexpr int GEMV_U = 4;

EXB_DEV int4 ldg_stream(const int4* p) {
  int4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.s32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// 16 int16 activations (xa: 0..7, xb: 8..15, packed in pairs) times 16 int8 weights
EXB_DEV int dot16(const int4 w, const int4 xa, const int4 xb) {
  int s = 0;
  s = __dp2a_lo(xa.x, w.x, s); s = __dp2a_hi(xa.y, w.x, s);
  s = __dp2a_lo(xa.z, w.y, s); s = __dp2a_hi(xa.w, w.y, s);
  s = __dp2a_lo(xb.x, w.z, s); s = __dp2a_hi(xb.y, w.z, s);
  s = __dp2a_lo(xb.z, w.w, s); s = __dp2a_hi(xb.w, w.w, s);
  return s;
}

EXB_DEV unsigned long long mod_p(int64_t v, unsigned long long P) {
  int64_t m = v % (int64_t)P;
  return (unsigned long long)(m < 0 ? m + (int64_t)P : m);
}

// requant of one accumulator (group: shr(tot, 28-s); channel, drop rule proven inactive: shr(acc*M, 28-s))
EXB_DEV int64_t requant1(const LinW& L, int n, int64_t tot, int s) {
  int64_t y;
  if (L.Mg) y = shr64(tot, 28 - s);
  else y = shr64((int64_t)((uint64_t)tot * (uint64_t)L.Mc[n]), 28 - s);
  if (L.b) y = (int64_t)((uint64_t)y + (uint64_t)L.b[n]);
  return y;
}

template <int R, int RPU, bool GROUP>
__global__ void __launch_bounds__(GEMV_THREADS) k_gemv(const GemvArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  int16_t* xs = reinterpret_cast<int16_t*>(smem_raw);                 // R x K
  __shared__ unsigned long long red[GEMV_THREADS / 32][R][6];
  __shared__ unsigned long long head_best[GEMV_THREADS / 32][R][2];

  const int K = a.L.K, C = K >> 4, G = K >> 7;
  const int units = a.L.N / RPU;
  const int lo = (int)((int64_t)units * blockIdx.x / gridDim.x);
  const int hi = (int)((int64_t)units * (blockIdx.x + 1) / gridDim.x);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int NW = GEMV_THREADS / 32;

  pdl_wait();
  // stage the R activation rows (int16) into shared memory
  {
    const int n16 = K >> 3;                                   // int4 per row
    for (int i = threadIdx.x; i < R * n16; i += GEMV_THREADS) {
      int r = i / n16, c = i - r * n16;
      reinterpret_cast<int4*>(xs + (size_t)r * K)[c] = reinterpret_cast<const int4*>(a.xq + (size_t)r * a.ldx)[c];
    }
  }
  __syncthreads();

  int sh[R];
#pragma unroll
  for (int r = 0; r < R; ++r) sh[r] = a.xs[r];

  unsigned long long frl[R][3][2];
  int64_t best_v[R];
  int best_n[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
#pragma unroll
    for (int q = 0; q < 3; ++q) frl[r][q][0] = frl[r][q][1] = 0;
    best_v[r] = INT64_MIN;
    best_n[r] = 0x7fffffff;
  }

  for (int u = lo + warp; u < hi; u += NW) {
    int64_t tot[R][RPU];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int j = 0; j < RPU; ++j) tot[r][j] = 0;
    const int4* wrow[RPU];
    const int32_t* mrow[RPU];
#pragma unroll
    for (int j = 0; j < RPU; ++j) {
      const int n = u * RPU + j;
      wrow[j] = reinterpret_cast<const int4*>(a.L.w + (size_t)n * K);
      mrow[j] = GROUP ? a.L.Mg + (size_t)n * G : nullptr;
    }
    for (int i0 = 0; i0 < C; i0 += 32 * GEMV_U) {
      int4 wv[GEMV_U][RPU];
      int32_t mv[GEMV_U][RPU];
#pragma unroll
      for (int q = 0; q < GEMV_U; ++q) {
        const int ch = i0 + q * 32 + lane;
#pragma unroll
        for (int j = 0; j < RPU; ++j) {
          if (ch < C) {
            wv[q][j] = ldg_stream(wrow[j] + ch);
            mv[q][j] = GROUP ? __ldg(mrow[j] + (ch >> 3)) : 1;
          } else {
            wv[q][j] = make_int4(0, 0, 0, 0);
            mv[q][j] = 0;
          }
        }
      }
#pragma unroll
      for (int q = 0; q < GEMV_U; ++q) {
        const int ch = i0 + q * 32 + lane;
        if (ch < C) {
#pragma unroll
          for (int r = 0; r < R; ++r) {
            const int4* xp = reinterpret_cast<const int4*>(xs + (size_t)r * K + 16 * ch);
            const int4 xa = xp[0], xb = xp[1];
#pragma unroll
            for (int j = 0; j < RPU; ++j) {
              const int p = dot16(wv[q][j], xa, xb);
              // accumulate in uint64 so any overflow wraps like numpy int64
              if (GROUP) tot[r][j] = (int64_t)((uint64_t)tot[r][j] + (uint64_t)((int64_t)p * mv[q][j]));
              else tot[r][j] = (int64_t)((uint64_t)tot[r][j] + (uint64_t)(int64_t)p);
            }
          }
        }
      }
    }
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int j = 0; j < RPU; ++j)
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
          tot[r][j] = (int64_t)((uint64_t)tot[r][j] + (uint64_t)__shfl_xor_sync(0xffffffffu, tot[r][j], o));

    if (lane == 0) {
#pragma unroll
      for (int r = 0; r < R; ++r) {
        if (RPU == 2) {
          // SwiGLU pair: row 2u = gate u, row 2u+1 = up u (exact_llm.py:179)
          const int ng = 2 * u, nu = 2 * u + 1;
          const int64_t yg = requant1(a.L, ng, tot[r][0], sh[r]);
          const int64_t yu = requant1(a.L, nu, tot[r][RPU - 1], sh[r]);
          const int64_t act = isilu_dev(a.silu_t, yg);
          a.out[(size_t)r * a.ldo + u] = shr64((int64_t)((uint64_t)act * (uint64_t)yu), 16);
          if (a.raw) a.raw[(size_t)r * a.ldr + u] = tot[r][0];
          if (a.raw2) a.raw2[(size_t)r * a.ldr + u] = tot[r][RPU - 1];
          if (a.fr_nseg) {
            const int I = a.L.N / 2;
#pragma unroll
            for (int pi = 0; pi < 2; ++pi) {
              frl[r][0][pi] += mod_p(tot[r][0], fr_prime(pi)) * (unsigned long long)a.fr_r[0][pi * I + u] % fr_prime(pi);
              frl[r][1][pi] += mod_p(tot[r][RPU - 1], fr_prime(pi)) * (unsigned long long)a.fr_r[1][pi * I + u] % fr_prime(pi);
            }
          }
        } else {
          const int n = u;
          const int64_t t = tot[r][0];
          if (a.raw) a.raw[(size_t)r * a.ldr + n] = t;
          if (a.fr_nseg) {
            const int sg = (a.fr_nseg > 2 && n >= a.fr_seg_start[2]) ? 2 : (a.fr_nseg > 1 && n >= a.fr_seg_start[1]) ? 1 : 0;
            const int nseg_cols = (sg + 1 < a.fr_nseg ? a.fr_seg_start[sg + 1] : a.L.N) - a.fr_seg_start[sg];
            const int loc = n - a.fr_seg_start[sg];
#pragma unroll
            for (int pi = 0; pi < 2; ++pi)
              frl[r][sg][pi] += mod_p(t, fr_prime(pi)) * (unsigned long long)a.fr_r[sg][pi * nseg_cols + loc] % fr_prime(pi);
          }
          if (a.epi != EPI_RAW) {
            const int64_t y = requant1(a.L, n, t, sh[r]);
            if (a.epi == EPI_RESID) {
              int64_t* o = a.out + (size_t)r * a.ldo + n;
              *o = (int64_t)((uint64_t)*o + (uint64_t)y);
            } else if (a.out) {
              a.out[(size_t)r * a.ldo + n] = y;
            }
            if (a.epi == EPI_HEAD && (y > best_v[r] || (y == best_v[r] && n < best_n[r]))) {
              best_v[r] = y;
              best_n[r] = n;
            }
          }
        }
      }
    }
  }

  // ---- Freivalds left-hand side: per-CTA partial sums -> one atomic per (segment, row, prime)
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
      for (int w = 0; w < NW; ++w) s += red[w][r][q];
      if (s) atomicAdd(a.fr_acc[q >> 1] + r * 4 + (q & 1), s);
    }
    // ---- right-hand side: sum_k d_k (xq_k mod p), k range split over the grid
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
    __shared__ bool last;
    if (threadIdx.x < R) {
      const int r = threadIdx.x;
      int64_t bv = INT64_MIN;
      int bn = 0x7fffffff;
      for (int w = 0; w < NW; ++w) {
        const int64_t v = (int64_t)head_best[w][r][0];
        const int n = (int)head_best[w][r][1];
        if (v > bv || (v == bv && n < bn)) { bv = v; bn = n; }
      }
      a.head_part[((size_t)blockIdx.x * R + r) * 2 + 0] = (unsigned long long)bv;
      a.head_part[((size_t)blockIdx.x * R + r) * 2 + 1] = (unsigned long long)(unsigned)bn;
      __threadfence();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      const unsigned t = atomicAdd(a.head_ticket, 1u);
      last = (t == gridDim.x - 1);
    }
    __syncthreads();
    if (last) {
      __threadfence();
      if (threadIdx.x < R) {
        const int r = threadIdx.x;
        int64_t bv = INT64_MIN;
        int bn = 0x7fffffff;
        for (unsigned c = 0; c < gridDim.x; ++c) {
          const volatile unsigned long long* hp = a.head_part + ((size_t)c * R + r) * 2;
          const int64_t v = (int64_t)hp[0];
          const int n = (int)hp[1];
          if (v > bv || (v == bv && n < bn)) { bv = v; bn = n; }
        }
        a.next_tok[r] = bn;
      }
      if (threadIdx.x == 0) *a.head_ticket = 0;
    }
  }
  pdl_launch_dependents();
}

template <int R, int RPU, bool GROUP>
static cudaError_t launch_t(const GemvArgs& a, cudaStream_t st, bool pdl) {
  const size_t smem = (size_t)R * a.L.K * sizeof(int16_t);
  auto kern = k_gemv<R, RPU, GROUP>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
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

template <int RPU, bool GROUP>
static cudaError_t launch_r(const GemvArgs& a, cudaStream_t st, bool pdl) {
  switch (a.R) {
    case 1: return launch_t<1, RPU, GROUP>(a, st, pdl);
    case 2: return launch_t<2, RPU, GROUP>(a, st, pdl);
    case 3: return launch_t<3, RPU, GROUP>(a, st, pdl);
    case 4: return launch_t<4, RPU, GROUP>(a, st, pdl);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_gemv(const GemvArgs& a0, cudaStream_t st, bool pdl) {
  GemvArgs a = a0;
  if ((a.L.Mg ? a.L.K % 128 : a.L.K % 16) != 0 || a.L.N <= 0 || a.R < 1 || a.R > 4) return cudaErrorInvalidValue;
  if (a.epi == EPI_SWIGLU && (a.L.N & 1)) return cudaErrorInvalidValue;
  if (a.grid <= 0) {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int units = a.epi == EPI_SWIGLU ? a.L.N / 2 : a.L.N;
    a.grid = units < 4 * sms ? (units + 3) / 4 : 4 * sms;   // >= 4 columns per CTA, <= 4 CTAs per SM
    if (a.grid < 1) a.grid = 1;
  }
  const bool group = a.L.Mg != nullptr;
  if (a.epi == EPI_SWIGLU) return group ? launch_r<2, true>(a, st, pdl) : launch_r<2, false>(a, st, pdl);
  return group ? launch_r<1, true>(a, st, pdl) : launch_r<1, false>(a, st, pdl);
}

// ---------------------------------------------------------------------------------------------
// Drop-in for the reference operator exact::gemv(x16 int16[K], wT int8[N,K], Mg int64[N,G]) ->
// int64[N] (experiments/speed_fair_kaggle.py:662-702): raw tot, int64 scales read as given.
__global__ void __launch_bounds__(GEMV_THREADS) k_gemv_op(const int16_t* __restrict__ x, const int8_t* __restrict__ wT,
                                                          const int64_t* __restrict__ Mg, int K, int N,
                                                          int64_t* __restrict__ out) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  int16_t* xs = reinterpret_cast<int16_t*>(smem_raw);
  for (int i = threadIdx.x; i < (K >> 3); i += GEMV_THREADS)
    reinterpret_cast<int4*>(xs)[i] = reinterpret_cast<const int4*>(x)[i];
  __syncthreads();
  const int C = K >> 4, G = K >> 7;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int n = blockIdx.x * (GEMV_THREADS / 32) + warp; n < N; n += gridDim.x * (GEMV_THREADS / 32)) {
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
  k_gemv_op<<<blocks, GEMV_THREADS, smem, st>>>(x16, wT, Mg, K, N, out);
  return cudaGetLastError();
}

}  // namespace exb
