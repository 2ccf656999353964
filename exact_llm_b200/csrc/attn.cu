// K6/K7: RoPE + KV-cache write, and exact integer attention for decode rows.
//
// Reference semantics (novain-shibu/exact-llm):
//   RoPE            shr(x*cos + rot_half(x)*sin, 16)                    exact_llm.py:159-160
//   K cache         qrow(k) per (head, position) row, V kept as Q16      exact_torch.py:146-149
//   scores          shr((qq . kq) * INV, 32 - sq - sk), INV=round(2^16/sqrt(hd))   exact_llm.py:164,174
//   softmax         Q24 exp table, p = (e << 20) // sum(e)               exact_llm.py:109-115
//   output          shr(sum_t p_t * v_t, 20) in int64                    exact_llm.py:176 (SPEC v0.4)
//
// The softmax needs the global row max and the global sum of e before any p*v term, so an
// online (rescaling) softmax cannot be used.  On B200 each (row, KV head) pair is handled by a
// thread-block CLUSTER of 8 CTAs that split the key positions; the three exact phases (scores +
// local max -> global max -> e + local sum -> global sum -> p and partial p.v) exchange their
// per-CTA maxima, sums and partial outputs through distributed shared memory between hardware
// cluster barriers.  Every sum is an integer sum, so the split does not change any bit.
#include <cooperative_groups.h>

#include "common.cuh"
#include "exb_internal.h"
#include "rowdev.cuh"
#include "tpx.cuh"

namespace cg = cooperative_groups;

namespace exb {

constexpr int CL = 8;               // CTAs per cluster (portable cluster size)
constexpr int ATT_THREADS = 256;
constexpr int REP_MAX = 8;          // query heads per KV head handled by one cluster
constexpr int ATT_TILE = 64;        // key/value positions staged in shared memory at a time

// ---------------------------------------------------------------- RoPE + cache write + q quantisation
// Standalone form of rope_cache_rows (the decode path runs it as the q|k|v GEMV's last-CTA tail).
__global__ void __launch_bounds__(256) k_rope_cache(const AttnArgs a) {
  pdl_wait();
  pdl_launch_dependents();
  rope_cache_rows<256>(a, blockIdx.x * 8, gridDim.x * 8);
  tl_exit();
}

cudaError_t launch_rope_cache(const AttnArgs& a, cudaStream_t st, bool pdl) {
  if (a.hd > 128 || (a.hd & 1) || a.H % a.KV) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((a.R * (a.KV + a.H) + 7) / 8);      // one warp per (row, head) task
  cfg.blockDim = dim3(256);
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, k_rope_cache, a);
}

// ---------------------------------------------------------------- decode attention (one cluster per row x KV head)
template <int HD>
EXB_DEV int64_t dot_i16(const int16_t* __restrict__ a, const int16_t* __restrict__ b) {
  int64_t acc = 0;
#pragma unroll
  for (int d = 0; d < HD; d += 8) {
    const int4 x = *reinterpret_cast<const int4*>(a + d);
    const int4 y = *reinterpret_cast<const int4*>(b + d);
    const int xs[4] = {x.x, x.y, x.z, x.w}, ys[4] = {y.x, y.y, y.z, y.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      // a pair of int16 products is < 2 * 32767^2 < 2^31: exact in int32
      const int p = (int)(short)(xs[q] & 0xffff) * (int)(short)(ys[q] & 0xffff) + (xs[q] >> 16) * (ys[q] >> 16);
      acc += p;
    }
  }
  return acc;
}

template <int HD>
__global__ void __cluster_dims__(CL, 1, 1) __launch_bounds__(ATT_THREADS) k_attn_decode(const AttnArgs a, int SCmax) {
  extern __shared__ __align__(16) unsigned char sm[];
  __shared__ int64_t lmax[REP_MAX], lsum[REP_MAX], gmax[REP_MAX], gsum[REP_MAX];
  __shared__ int qsh[REP_MAX];
  cg::cluster_group cluster = cg::this_cluster();
  const int c = (int)cluster.block_rank();
  const int j = blockIdx.y, r = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  constexpr int hd = HD;
  const int rep = a.H / a.KV;

  int16_t* qs_sm = reinterpret_cast<int16_t*>(sm);                                  // rep*hd
  int64_t* sc = reinterpret_cast<int64_t*>(sm + ((rep * hd * 2 + 15) & ~15));      // rep*SCmax
  int64_t* pout = sc + (size_t)rep * SCmax;                                          // rep*hd
  int64_t* pv = pout + (size_t)rep * hd;                                             // ATT_THREADS*REP_MAX
  int16_t* ktile = reinterpret_cast<int16_t*>(pv + (size_t)ATT_THREADS * REP_MAX);   // ATT_TILE x (hd + 8)
  int32_t* vtile = reinterpret_cast<int32_t*>(ktile + (size_t)ATT_TILE * (hd + 8));   // ATT_TILE x hd

  pdl_wait();
  pdl_launch_dependents();
  const int pos = a.row_pos[r], seq = a.row_seq[r];
  const int S = pos + 1;
  const int chunk = (S + CL - 1) / CL;
  const int t0 = c * chunk;
  const int t1 = min(S, t0 + chunk);
  const int n = t1 > t0 ? t1 - t0 : 0;
  const size_t cbase = ((size_t)seq * a.KV + j) * a.Smax;

  for (int e = tid; e < rep * hd; e += ATT_THREADS) qs_sm[e] = a.qq[((size_t)r * a.H + j * rep) * hd + e];
  if (tid < rep) qsh[tid] = a.qs[(size_t)r * a.H + j * rep + tid];
  __syncthreads();

  // phase 1: scores of this CTA's positions, local max per head.  Key rows are staged in shared
  // memory one tile at a time (all loads in flight together; rows padded by 16 bytes so the
  // 128-bit reads of 8 consecutive rows hit distinct banks).
  for (int tt = 0; tt < n; tt += ATT_TILE) {
    const int nt = min(ATT_TILE, n - tt);
    const int per_row = hd / 8;                                         // int4 per key row
    for (int e = tid; e < nt * per_row; e += ATT_THREADS) {
      const int t = e / per_row, c4 = e - t * per_row;
      *reinterpret_cast<int4*>(ktile + (size_t)t * (hd + 8) + c4 * 8) =
          reinterpret_cast<const int4*>(a.kc + (cbase + t0 + tt + t) * hd)[c4];
    }
    __syncthreads();
    for (int e = tid; e < rep * nt; e += ATT_THREADS) {
      const int i = e / nt, t = e - i * nt;
      const int64_t acc = dot_i16<HD>(qs_sm + i * hd, ktile + (size_t)t * (hd + 8));
      sc[(size_t)i * SCmax + tt + t] =
          shr64((int64_t)((uint64_t)acc * (uint64_t)a.inv), 32 - qsh[i] - (int)a.ks[cbase + t0 + tt + t]);
    }
    __syncthreads();
  }
  __syncthreads();
  if (warp < rep) {
    int64_t m = INT64_MIN;
    for (int t = lane; t < n; t += 32) { const int64_t v = sc[(size_t)warp * SCmax + t]; m = v > m ? v : m; }
    for (int o = 16; o > 0; o >>= 1) { const int64_t w = __shfl_xor_sync(0xffffffffu, m, o); m = w > m ? w : m; }
    if (lane == 0) lmax[warp] = m;
  }
  cluster.sync();
  if (tid < rep) {
    int64_t g = INT64_MIN;
    for (int cc = 0; cc < CL; ++cc) { const int64_t v = cluster.map_shared_rank(lmax, cc)[tid]; g = v > g ? v : g; }
    gmax[tid] = g;
  }
  __syncthreads();
  // phase 2: e = exp table at (max - score), local sums
  for (int e = tid; e < rep * n; e += ATT_THREADS) {
    const int i = e / n, t = e - i * n;
    int64_t* p = sc + (size_t)i * SCmax + t;
    *p = exp_lookup(a.exp_t, gmax[i] - *p);
  }
  __syncthreads();
  if (warp < rep) {
    int64_t s = 0;
    for (int t = lane; t < n; t += 32) s += sc[(size_t)warp * SCmax + t];
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) lsum[warp] = s;
  }
  cluster.sync();
  if (tid < rep) {
    int64_t g = 0;
    for (int cc = 0; cc < CL; ++cc) g += cluster.map_shared_rank(lsum, cc)[tid];
    gsum[tid] = g;
  }
  __syncthreads();
  // phase 3: p = (e << 20) // sum(e) (non-negative), then partial p . v
  for (int e = tid; e < rep * n; e += ATT_THREADS) {
    const int i = e / n, t = e - i * n;
    int64_t* p = sc + (size_t)i * SCmax + t;
    *p = (int64_t)(((uint64_t)*p << 20) / (uint64_t)gsum[i]);
  }
  __syncthreads();
  {
    const int nparts = ATT_THREADS / hd;                  // hd divides ATT_THREADS (16, 32, 64, 128)
    const int d = tid % hd, part = tid / hd;
    int64_t acc[REP_MAX];
#pragma unroll
    for (int i = 0; i < REP_MAX; ++i) acc[i] = 0;
    // value rows staged in shared memory one tile at a time
    for (int tt = 0; tt < n; tt += ATT_TILE) {
      const int nt = min(ATT_TILE, n - tt);
      const int per_row = hd / 4;                                       // int4 per value row
      for (int e = tid; e < nt * per_row; e += ATT_THREADS) {
        const int t = e / per_row, c4 = e - t * per_row;
        reinterpret_cast<int4*>(vtile)[(size_t)t * per_row + c4] =
            reinterpret_cast<const int4*>(a.vc + (cbase + t0 + tt + t) * hd)[c4];
      }
      __syncthreads();
#pragma unroll 4
      for (int t = part; t < nt; t += nparts) {
        const int64_t v = vtile[(size_t)t * hd + d];
#pragma unroll
        for (int i = 0; i < REP_MAX; ++i)
          if (i < rep) acc[i] += sc[(size_t)i * SCmax + tt + t] * v;
      }
      __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < REP_MAX; ++i) pv[(size_t)tid * REP_MAX + i] = acc[i];
    __syncthreads();
    for (int e = tid; e < rep * hd; e += ATT_THREADS) {
      const int i = e / hd, dd = e - i * hd;
      int64_t s = 0;
      for (int q = 0; q < nparts; ++q) s += pv[(size_t)(q * hd + dd) * REP_MAX + i];
      pout[e] = s;
    }
  }
  cluster.sync();
  // combine the cluster's partial outputs: CTA c finalises a slice of the rep*hd outputs
  {
    const int tot = rep * hd, per = (tot + CL - 1) / CL;
    const int e0 = c * per, e1 = min(tot, e0 + per);
    uint64_t om = 0;
    for (int e = e0 + tid; e < e1; e += ATT_THREADS) {
      int64_t s = 0;
      for (int cc = 0; cc < CL; ++cc) s += cluster.map_shared_rank(pout, cc)[e];
      const int64_t o = shr64(s, 20);
      a.out[(size_t)r * a.ldo + (size_t)j * rep * hd + e] = o;
      const uint64_t u = uabs64(o);
      om = u > om ? u : om;
    }
    if (a.amax_out) {
      // per-row max |out| for the o-projection's row quantisation (exact_llm.py:41-46)
      for (int o = 16; o > 0; o >>= 1) { const uint64_t w = __shfl_xor_sync(0xffffffffu, om, o); om = w > om ? w : om; }
      if (lane == 0 && om) atomicMax(a.amax_out + r, (unsigned long long)om);
    }
  }
  cluster.sync();                                        // peers' shared memory stays alive until read
  // last CTA of the grid: qrow of the complete output rows for the o projection
  if (a.xq_out && last_cta(a.ticket, gridDim.x * gridDim.y * gridDim.z)) {
    for (int rr = 0; rr < a.R; ++rr) {
      const int s = qrow_shift(__ldcg(a.amax_out + rr));
      row_quant_known<ATT_THREADS>(a.out + (size_t)rr * a.ldo, a.H * hd, s, a.xq_out + (size_t)rr * a.ldq);
      if (tid == 0) a.xs_out[rr] = s;
    }
  }
  tl_exit();
}

cudaError_t launch_attn_decode(const AttnArgs& a, cudaStream_t st, bool pdl) {
  const int rep = a.H / a.KV;
  if (rep > REP_MAX || a.H % a.KV || ATT_THREADS % a.hd || a.hd % 8) return cudaErrorInvalidValue;
  const int SCmax = (((a.Smax + CL - 1) / CL) + 1) & ~1;   // even: keeps the tiles after sc 16-byte aligned
  const size_t smem = (size_t)((rep * a.hd * 2 + 15) & ~15) + (size_t)rep * SCmax * 8 + (size_t)rep * a.hd * 8 +
                      (size_t)ATT_THREADS * REP_MAX * 8 + (size_t)ATT_TILE * (a.hd + 8) * 2 + (size_t)ATT_TILE * a.hd * 4;
  if (smem > 200 * 1024) return cudaErrorInvalidValue;
  void (*kern)(const AttnArgs, int) = a.hd == 128 ? k_attn_decode<128> : a.hd == 64 ? k_attn_decode<64>
                                    : a.hd == 32 ? k_attn_decode<32> : k_attn_decode<16>;
  if (a.hd != 128 && a.hd != 64 && a.hd != 32 && a.hd != 16) return cudaErrorInvalidValue;
  // raised once to the full budget and never lowered (see the GEMV launcher)
  static DevOnce attr_set[4];
  const int ti = a.hd == 128 ? 0 : a.hd == 64 ? 1 : a.hd == 32 ? 2 : 3;
  if (!attr_set[ti].done()) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e != cudaSuccess) return e;
    attr_set[ti].set();
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(CL, a.KV, a.R);
  cfg.blockDim = dim3(ATT_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, a, SCmax);
}


// ---------------------------------------------------------------- fused RoPE + cache write + decode attention
// One 8-CTA cluster per (row, query head); CTA c of the cluster takes a contiguous slice of the
// key positions.  The rows cached by earlier steps never depend on the kernel before this one, so
// each CTA stages its first tile of K/V rows (and the row's cos/sin) in shared memory BEFORE the
// dependent-launch wait; after it, the CTA ropes and quantises its query head (exact_llm.py:157-160,
// 41-46) and computes the rows of this step (positions of the chunk's rows of the same sequence)
// directly from q|k|v, never reading them back from the cache.  The cluster of the first query
// head of a KV group writes the row of its own position to the cache (one writer per KV row).
// The three exact softmax phases exchange maxima, sums and partial p.v through distributed shared
// memory (every peer value loaded at once); all sums are integer sums, so the split changes no bit.
// key/value positions staged in shared memory at a time: 128, or 64 where the cache holds more than
// 2048 positions, so the score array and the tiles stay small enough for every CTA of a 40-head
// model to be resident at once (one wave)

EXB_DEV int64_t rope_value(const int64_t* row, int d, int half, int64_t c, int64_t s) {
  const int64_t x = ld_cg(row + d);
  const int64_t rot = d < half ? (int64_t)(0ull - (uint64_t)ld_cg(row + d + half)) : ld_cg(row + d - half);
  return shr64((int64_t)((uint64_t)x * (uint64_t)c + (uint64_t)rot * (uint64_t)s), 16);
}

// EXTRA: the trace-commitment capture of the roped K / V rows and the tensor-parallel publication of
// the row maxima (a separate instantiation keeps them out of the single-GPU decode kernel)
template <int HD, int TILE, bool EXTRA>
__global__ void __cluster_dims__(CL, 1, 1) __launch_bounds__(ATT_THREADS) k_attn_rope(const AttnArgs a, int SCmax) {
  extern __shared__ __align__(16) unsigned char sm[];
  constexpr int TP = HD + 8;                 // padded K row (int16): 8 consecutive rows hit distinct banks
  constexpr int HALF = HD / 2;
  constexpr int NW = ATT_THREADS / 32;
  __shared__ uint64_t red[NW];
  __shared__ int64_t lmax_s, lsum_s, gmax_s, gsum_s;
  __shared__ int qs_s;
  __shared__ int64_t gath[HD];
  cg::cluster_group cluster = cg::this_cluster();
  const int c = (int)cluster.block_rank();
  const int h = blockIdx.y, r = blockIdx.z;
  const int rep = a.H / a.KV, j = h / rep;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  int16_t* qq_s = reinterpret_cast<int16_t*>(sm);                            // HD
  int32_t* cs_s = reinterpret_cast<int32_t*>(sm + 256);                      // HALF cos | HALF sin
  int64_t* sc = reinterpret_cast<int64_t*>(sm + 768);                        // SCmax
  int64_t* pout = sc + SCmax;                                                 // HD
  int64_t* pv = pout + HD;                                                    // ATT_THREADS
  int* ksh = reinterpret_cast<int*>(pv + ATT_THREADS);                        // TILE
  int16_t* ktile = reinterpret_cast<int16_t*>(ksh + TILE);                // TILE x TP
  int32_t* vtile = reinterpret_cast<int32_t*>(ktile + (size_t)TILE * TP); // TILE x HD

  // ---- before the wait: positions, this row's cos/sin, the first tile of cached rows
  const int pos = a.row_pos[r], seq = a.row_seq[r];
  const bool ok = pos >= 0 && pos < a.Smax && pos < a.Tmax;
  const int S = ok ? pos + 1 : 0;
  const int chunk = (S + CL - 1) / CL;
  const int t0 = min(S, c * chunk);
  const int t1 = min(S, t0 + chunk);
  const int n = t1 - t0;
  const size_t cbase = ((size_t)seq * a.KV + j) * a.Smax;
  if (ok)
    for (int i = tid; i < HALF; i += ATT_THREADS) {
      cs_s[i] = a.cos_t[(size_t)pos * HALF + i];
      cs_s[HALF + i] = a.sin_t[(size_t)pos * HALF + i];
    }
  auto stage_k = [&](int tb, int nt) {
    for (int e = tid; e < nt * (HD / 8); e += ATT_THREADS) {
      const int t = e / (HD / 8), c4 = e - t * (HD / 8);
      *reinterpret_cast<int4*>(ktile + (size_t)t * TP + c4 * 8) =
          reinterpret_cast<const int4*>(a.kc + (cbase + t0 + tb + t) * HD)[c4];
    }
    for (int t = tid; t < nt; t += ATT_THREADS) ksh[t] = a.ks[cbase + t0 + tb + t];
  };
  auto stage_v = [&](int tb, int nt) {
    for (int e = tid; e < nt * (HD / 4); e += ATT_THREADS)
      reinterpret_cast<int4*>(vtile)[e] = reinterpret_cast<const int4*>(a.vc + (cbase + t0 + tb) * HD)[e];
  };
  const int nt0 = min(TILE, n);
  stage_k(0, nt0);
  stage_v(0, nt0);

  pdl_wait();
  pdl_launch_dependents();
  if (!ok && c == 0 && tid == 0) set_err(a.err, ERR_BOUNDS);
  __syncthreads();                                       // cos/sin staged by other threads

  // ---- this head's query row: RoPE, then qrow over the head (one shift per (row, head))
  int64_t qv = 0;
  if (ok && tid < HD)
    qv = rope_value(a.qkv + (size_t)r * a.ldqkv + (size_t)h * HD, tid, HALF, cs_s[tid % HALF], cs_s[HALF + tid % HALF]);
  {
    const uint64_t m = warp_max_u64(uabs64(qv));
    if (lane == 0) red[warp] = m;
    __syncthreads();
    uint64_t mm = 0;
#pragma unroll
    for (int w = 0; w < NW; ++w) mm = red[w] > mm ? red[w] : mm;
    const int s = qrow_shift(mm);
    if (tid < HD) qq_s[tid] = qrow_value(qv, s);
    if (tid == 0) qs_s = s;
  }

  // ---- rows of this step that fall in [t0 + tb, t0 + tb + nt): computed from q|k|v (one warp
  // per row of the chunk); the (first head of the group, own row) cluster writes them to the cache
  auto patch = [&](int tb, int nt, bool do_k, bool do_v) {
    if (warp < a.R) {
      const int r2 = warp;
      const int p2 = a.row_pos[r2];
      if (ok && a.row_seq[r2] == seq && p2 >= t0 + tb && p2 < t0 + tb + nt && p2 < a.Tmax) {
        const int t = p2 - t0 - tb;
        const bool writer = (h == j * rep) && r2 == r;
        const size_t cidx = cbase + p2;
        if (do_k) {
          const int64_t* krow = a.qkv + (size_t)r2 * a.ldqkv + (size_t)(a.H + j) * HD;
          int64_t kv[4];
          uint64_t m = 0;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int d = lane + 32 * q;
            kv[q] = 0;
            if (d < HD) {
              kv[q] = rope_value(krow, d, HALF, a.cos_t[(size_t)p2 * HALF + d % HALF], a.sin_t[(size_t)p2 * HALF + d % HALF]);
              const uint64_t u = uabs64(kv[q]);
              m = u > m ? u : m;
            }
          }
          for (int o = 16; o > 0; o >>= 1) { const uint64_t w = __shfl_xor_sync(0xffffffffu, m, o); m = w > m ? w : m; }
          const int sh = qrow_shift(m);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int d = lane + 32 * q;
            if (d < HD) {
              const int16_t v16 = qrow_value(kv[q], sh);
              ktile[(size_t)t * TP + d] = v16;
              if (writer) a.kc[cidx * HD + d] = v16;
              if (EXTRA && writer && a.kr_out) a.kr_out[(size_t)r2 * a.ldkr + (size_t)j * HD + d] = kv[q];   // roped K
            }
          }
          if (lane == 0) {
            ksh[t] = sh;
            if (writer) a.ks[cidx] = (int8_t)sh;
          }
        }
        if (do_v) {
          const int64_t* vrow = a.qkv + (size_t)r2 * a.ldqkv + (size_t)(a.H + a.KV + j) * HD;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int d = lane + 32 * q;
            if (d < HD) {
              const int64_t v = ld_cg(vrow + d);
              if (v > INT32_MAX || v < INT32_MIN) set_err(a.err, ERR_V_RANGE);
              vtile[(size_t)t * HD + d] = (int32_t)v;
              if (writer) a.vc[cidx * HD + d] = (int32_t)v;
              if (EXTRA && writer && a.kr_out) a.kr_out[(size_t)r2 * a.ldkr + (size_t)(a.KV + j) * HD + d] = v;
            }
          }
        }
      }
    }
  };
  patch(0, nt0, true, true);
  __syncthreads();

  // ---- phase 1: scores (two threads per key row, half a head each), local max
  const int qs = qs_s;
  for (int tb = 0; tb < n; tb += TILE) {
    const int nt = min(TILE, n - tb);
    if (tb > 0) {
      __syncthreads();
      stage_k(tb, nt);
      __syncthreads();                                   // the staged tile before this step's rows overwrite
      patch(tb, nt, true, false);                        // theirs (else a stale cache row can win the race)
      __syncthreads();
    }
    for (int p0 = 0; p0 < 2 * TILE; p0 += ATT_THREADS) {
      const int p = p0 + tid, t = p >> 1, hf = p & 1;
      int64_t acc = 0;
      if (t < nt) {
        const int16_t* kr = ktile + (size_t)t * TP + hf * HALF;
        const int16_t* qr = qq_s + hf * HALF;
#pragma unroll
        for (int d = 0; d < HALF; d += 8) {
          const int4 x = *reinterpret_cast<const int4*>(qr + d);
          const int4 y = *reinterpret_cast<const int4*>(kr + d);
          const int xs[4] = {x.x, x.y, x.z, x.w}, ys[4] = {y.x, y.y, y.z, y.w};
#pragma unroll
          for (int q = 0; q < 4; ++q)
            acc += (int)(short)(xs[q] & 0xffff) * (int)(short)(ys[q] & 0xffff) + (xs[q] >> 16) * (ys[q] >> 16);
        }
      }
      acc += __shfl_xor_sync(0xffffffffu, acc, 1);
      if (t < nt && hf == 0)
        sc[tb + t] = shr64((int64_t)((uint64_t)acc * (uint64_t)a.inv), 32 - qs - ksh[t]);
    }
  }
  __syncthreads();
  {
    int64_t m = INT64_MIN;
    for (int t = tid; t < n; t += ATT_THREADS) m = sc[t] > m ? sc[t] : m;
    for (int o = 16; o > 0; o >>= 1) { const int64_t w = __shfl_xor_sync(0xffffffffu, m, o); m = w > m ? w : m; }
    if (lane == 0) red[warp] = (uint64_t)m;
    __syncthreads();
    if (tid == 0) {
      int64_t mm = INT64_MIN;
      for (int w = 0; w < NW; ++w) mm = (int64_t)red[w] > mm ? (int64_t)red[w] : mm;
      lmax_s = mm;
    }
  }
  cluster.sync();
  if (warp == 0) {
    int64_t g = lane < CL ? *cluster.map_shared_rank(&lmax_s, lane) : INT64_MIN;
    for (int o = 16; o > 0; o >>= 1) { const int64_t w = __shfl_xor_sync(0xffffffffu, g, o); g = w > g ? w : g; }
    if (lane == 0) gmax_s = g;
  }
  __syncthreads();
  // ---- phase 2: e = exp table at (max - score), local sum
  {
    const int64_t g = gmax_s;
    int64_t s = 0;
    for (int t = tid; t < n; t += ATT_THREADS) {
      const int64_t e = exp_lookup(a.exp_t, g - sc[t]);
      sc[t] = e;
      s += e;
    }
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) red[warp] = (uint64_t)s;
    __syncthreads();
    if (tid == 0) {
      int64_t ss = 0;
      for (int w = 0; w < NW; ++w) ss += (int64_t)red[w];
      lsum_s = ss;
    }
  }
  cluster.sync();
  if (warp == 0) {
    int64_t g = lane < CL ? *cluster.map_shared_rank(&lsum_s, lane) : 0;
    for (int o = 16; o > 0; o >>= 1) g += __shfl_xor_sync(0xffffffffu, g, o);
    if (lane == 0) gsum_s = g;
  }
  __syncthreads();
  // ---- phase 3: p = (e << 20) // sum(e), partial p.v over this CTA's positions
  {
    const uint64_t g = (uint64_t)gsum_s;
    for (int t = tid; t < n; t += ATT_THREADS) sc[t] = (int64_t)(((uint64_t)sc[t] << 20) / g);
  }
  {
    constexpr int NP = ATT_THREADS / HD;
    const int d = tid % HD, part = tid / HD;
    int64_t acc = 0;
    for (int tb = 0; tb < n; tb += TILE) {
      const int nt = min(TILE, n - tb);
      __syncthreads();
      if (tb > 0) {
        stage_v(tb, nt);
        __syncthreads();                                 // as for the K tiles
        patch(tb, nt, false, true);
        __syncthreads();
      }
#pragma unroll 4
      for (int t = part; t < nt; t += NP) acc += sc[tb + t] * (int64_t)vtile[(size_t)t * HD + d];
    }
    pv[tid] = acc;
    __syncthreads();
    if (tid < HD) {
      int64_t s = 0;
#pragma unroll
      for (int q = 0; q < NP; ++q) s += pv[q * HD + tid];
      pout[tid] = s;
    }
  }
  cluster.sync();
  // ---- combine: CTA c finalises HD / CL output dims, each from the CL partials loaded at once
  {
    constexpr int PER = HD / CL;
    if (tid < HD) {
      const int dd = c * PER + tid / CL, peer = tid % CL;
      gath[tid] = cluster.map_shared_rank(pout, peer)[dd];
    }
    __syncthreads();
    uint64_t om = 0;
    if (tid < PER) {
      int64_t s = 0;
#pragma unroll
      for (int q = 0; q < CL; ++q) s += gath[tid * CL + q];
      const int64_t o = shr64(s, 20);
      if (ok) a.out[(size_t)r * a.ldo + (size_t)h * HD + c * PER + tid] = o;
      om = uabs64(o);
    }
    if (warp == 0 && a.amax_out) {
      om = warp_max_u64(om);
      if (lane == 0 && om && ok) atomicMax(a.amax_out + r, (unsigned long long)om);
    }
  }
  cluster.sync();                                        // peers' shared memory stays alive until read
  // tensor parallel: the last CTA publishes the complete row maxima to every rank (TPX_AMAX_O)
  if (EXTRA && a.tpx && last_cta(a.tpx_ticket, gridDim.x * gridDim.y * gridDim.z))
    tpx_publish_max(*a.tpx, TPX_AMAX_O, a.amax_out, a.R);
  tl_exit();
}

cudaError_t launch_attn_rope(const AttnArgs& a, cudaStream_t st, bool pdl) {
  const int rep = a.KV > 0 ? a.H / a.KV : 0;
  if (rep < 1 || a.H % a.KV || a.R < 1 || a.R > ATT_THREADS / 32) return cudaErrorInvalidValue;
  if (a.hd != 128 && a.hd != 64 && a.hd != 32 && a.hd != 16) return cudaErrorInvalidValue;
  const int SCmax = (((a.Smax + CL - 1) / CL) + 1) & ~1;   // even: keeps the arrays after sc 16-byte aligned
  const bool longc = a.Smax > 2048;
  const size_t tile = longc ? 64 : 128;
  const size_t smem = 768 + (size_t)SCmax * 8 + (size_t)a.hd * 8 + (size_t)ATT_THREADS * 8 + tile * 4 +
                      tile * (a.hd + 8) * 2 + tile * a.hd * 4;
  if (smem > 200 * 1024) return cudaErrorInvalidValue;
  void (*kern)(const AttnArgs, int) =
      !(a.kr_out || a.tpx)
          ? (longc ? (a.hd == 128 ? k_attn_rope<128, 64, false> : a.hd == 64 ? k_attn_rope<64, 64, false>
                      : a.hd == 32 ? k_attn_rope<32, 64, false> : k_attn_rope<16, 64, false>)
                   : (a.hd == 128 ? k_attn_rope<128, 128, false> : a.hd == 64 ? k_attn_rope<64, 128, false>
                      : a.hd == 32 ? k_attn_rope<32, 128, false> : k_attn_rope<16, 128, false>))
          : (longc ? (a.hd == 128 ? k_attn_rope<128, 64, true> : a.hd == 64 ? k_attn_rope<64, 64, true>
                      : a.hd == 32 ? k_attn_rope<32, 64, true> : k_attn_rope<16, 64, true>)
                   : (a.hd == 128 ? k_attn_rope<128, 128, true> : a.hd == 64 ? k_attn_rope<64, 128, true>
                      : a.hd == 32 ? k_attn_rope<32, 128, true> : k_attn_rope<16, 128, true>));
  static DevOnce attr_set[16];
  const int ti = (a.hd == 128 ? 0 : a.hd == 64 ? 1 : a.hd == 32 ? 2 : 3) + (longc ? 4 : 0) + (a.kr_out || a.tpx ? 8 : 0);
  if (!attr_set[ti].done()) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e != cudaSuccess) return e;
    attr_set[ti].set();
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(CL, a.H, a.R);
  cfg.blockDim = dim3(ATT_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, a, SCmax);
}


// ---------------------------------------------------------------- prefill attention (query tiles)
// A chunk of consecutive positions of ONE sequence: each CTA takes PRT query rows of one head and
// streams that KV head's cached rows 0..(its last position) in tiles of PKT keys, three times --
// the row maxima, then the sums of the exp table at (max - score), then p = (e << 20) // sum and
// p.v -- recomputing the scores each time, so the exact softmax needs no rescaling and every
// cached K/V byte a CTA reads serves PRT query rows (the per-row kernel reads the whole prefix
// once per row).  Queries and keys are staged as two byte planes each (x = 256 hi + lo, lo
// unsigned, hi signed) and a 32 x 64 score tile is int8 tensor-core MMAs (mma.sync m16n8k32, int32
// accumulators): q.k = 65536 (qh.kh) + 256 (qh.kl + ql.kh) + ql.kl, each plane product over 128
// dims below 128 * 255 * 255 < 2^31, combined exactly in int64.  Scores, table and shifts are the
// decode kernel's (exact_llm.py:170-176).
constexpr int PRT = 32;             // query rows per CTA
constexpr int PKT = 64;             // keys per tile
constexpr int PA_THREADS = 256;

// 8 int16 -> their 8 low bytes (unsigned digits) and 8 high bytes (signed digits), element order kept
EXB_DEV void split_planes(const int4 v, uint2& lo, uint2& hi) {
  lo = make_uint2(__byte_perm((uint32_t)v.x, (uint32_t)v.y, 0x6420), __byte_perm((uint32_t)v.z, (uint32_t)v.w, 0x6420));
  hi = make_uint2(__byte_perm((uint32_t)v.x, (uint32_t)v.y, 0x7531), __byte_perm((uint32_t)v.z, (uint32_t)v.w, 0x7531));
}

EXB_DEV uint32_t ld_s32(const uint8_t* p) { return *reinterpret_cast<const uint32_t*>(p); }

// D += A (16 x 32) . B (32 x 8), int8 digits (signed or unsigned per operand), int32 accumulators
template <bool AS, bool BS>
EXB_DEV void mma_i8(int (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  if constexpr (!AS && !BS)
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3]) : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  else if constexpr (!AS && BS)
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3]) : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  else if constexpr (AS && !BS)
    asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3]) : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  else
    asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3]) : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <int HD>
__global__ void __launch_bounds__(PA_THREADS, 3) k_attn_prefill(const AttnArgs a) {
  extern __shared__ __align__(16) unsigned char sm[];
  constexpr int PW = HD < 32 ? 32 : HD;               // plane row: whole 32-dim MMA steps (zero tail)
  constexpr int TB = PW + 16;                          // padded plane row: fragment loads hit 32 banks
  constexpr int KS = PW / 32;                          // MMA k-steps per score
  uint8_t* qlo = sm;                                                              // PRT x TB
  uint8_t* qhi = qlo + PRT * TB;                                                  // PRT x TB
  uint8_t* klo = qhi + PRT * TB;                                                  // PKT x TB
  uint8_t* khi = klo + PKT * TB;                                                  // PKT x TB
  int32_t* vt = reinterpret_cast<int32_t*>(khi + PKT * TB);                       // PKT x HD
  int32_t* pt = vt + PKT * HD;                                                    // PRT x PKT (p <= 2^20)
  __shared__ int64_t mx[PRT], ssum[PRT];
  __shared__ double sinv[PRT];
  __shared__ int rpos[PRT], rqs[PRT], kshift[PKT];
  const int tid = threadIdx.x, h = blockIdx.y;
  const int r0 = blockIdx.x * PRT;
  const int nr = min(PRT, a.R - r0);
  const int rep = a.H / a.KV, j = h / rep;
  const int seq = a.row_seq[r0];
  const size_t cbase = ((size_t)seq * a.KV + j) * a.Smax;
  for (int e = tid; e < PRT * (PW / 8); e += PA_THREADS) {
    const int r = e / (PW / 8), c8 = e - r * (PW / 8);
    int4 v = make_int4(0, 0, 0, 0);
    if (r < nr && c8 < HD / 8) v = reinterpret_cast<const int4*>(a.qq + ((size_t)(r0 + r) * a.H + h) * HD)[c8];
    uint2 lo, hi;
    split_planes(v, lo, hi);
    *reinterpret_cast<uint2*>(qlo + r * TB + c8 * 8) = lo;
    *reinterpret_cast<uint2*>(qhi + r * TB + c8 * 8) = hi;
  }
  if (tid < PRT) {
    rpos[tid] = tid < nr ? a.row_pos[r0 + tid] : -1;
    rqs[tid] = tid < nr ? a.qs[(size_t)(r0 + tid) * a.H + h] : 0;
    mx[tid] = INT64_MIN;
    ssum[tid] = 0;
  }
  __syncthreads();
  int pend = 0;
  for (int r = 0; r < nr; ++r) pend = max(pend, rpos[r] + 1);
  // warp tile: rows 16 mt .. +15, keys 16 nq .. +15 (two n8 MMA tiles); this thread's scores are
  // the accumulator fragment: rows 16 mt + g (+ 8), keys 16 nq + 8 n + 2 tq (+ 1)
  const int warp = tid >> 5, lane = tid & 31, g = lane >> 2, tq = lane & 3;
  const int mt = warp & 1, nq = warp >> 1;
  auto srow = [&](int i) { return mt * 16 + g + 8 * i; };
  auto skey = [&](int k) { return nq * 16 + (k >> 1) * 8 + 2 * tq + (k & 1); };
  auto scores = [&](int t0, int64_t sc[2][4], bool valid[2][4]) {
    int acc[4][2][4];                                  // plane product (ll, lh, hl, hh) x n tile x fragment
#pragma unroll
    for (int p = 0; p < 4; ++p)
#pragma unroll
      for (int n = 0; n < 2; ++n)
#pragma unroll
        for (int f = 0; f < 4; ++f) acc[p][n][f] = 0;
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
      const int d0 = ks * 32 + 4 * tq;
      const int ra = (mt * 16 + g) * TB + d0, rb = ra + 8 * TB;
      const uint32_t al[4] = {ld_s32(qlo + ra), ld_s32(qlo + rb), ld_s32(qlo + ra + 16), ld_s32(qlo + rb + 16)};
      const uint32_t ah[4] = {ld_s32(qhi + ra), ld_s32(qhi + rb), ld_s32(qhi + ra + 16), ld_s32(qhi + rb + 16)};
#pragma unroll
      for (int n = 0; n < 2; ++n) {
        const int kb = (nq * 16 + n * 8 + g) * TB + d0;
        const uint32_t bl0 = ld_s32(klo + kb), bl1 = ld_s32(klo + kb + 16);
        const uint32_t bh0 = ld_s32(khi + kb), bh1 = ld_s32(khi + kb + 16);
        mma_i8<false, false>(acc[0][n], al, bl0, bl1);
        mma_i8<false, true>(acc[1][n], al, bh0, bh1);
        mma_i8<true, false>(acc[2][n], ah, bl0, bl1);
        mma_i8<true, true>(acc[3][n], ah, bh0, bh1);
      }
    }
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int n = k >> 1, f = 2 * i + (k & 1);
        const int row = srow(i), key = skey(k);
        const int64_t qk = (int64_t)acc[3][n][f] * 65536 + ((int64_t)acc[1][n][f] + (int64_t)acc[2][n][f]) * 256 +
                           (int64_t)acc[0][n][f];
        valid[i][k] = row < nr && t0 + key <= rpos[row];
        sc[i][k] = valid[i][k] ? shr64((int64_t)((uint64_t)qk * (uint64_t)a.inv), 32 - rqs[row] - kshift[key]) : 0;
      }
  };
  auto load_k = [&](int t0) {
    const int nk = min(PKT, pend - t0);
    for (int e = tid; e < PKT * (PW / 8); e += PA_THREADS) {
      const int t = e / (PW / 8), c8 = e - t * (PW / 8);
      int4 v = make_int4(0, 0, 0, 0);
      if (t < nk && c8 < HD / 8) v = reinterpret_cast<const int4*>(a.kc + (cbase + t0 + t) * HD)[c8];
      uint2 lo, hi;
      split_planes(v, lo, hi);
      *reinterpret_cast<uint2*>(klo + t * TB + c8 * 8) = lo;
      *reinterpret_cast<uint2*>(khi + t * TB + c8 * 8) = hi;
    }
    for (int t = tid; t < PKT; t += PA_THREADS) kshift[t] = t < nk ? a.ks[cbase + t0 + t] : 0;
  };
  // pass 1: row maxima (the four lanes of a row in the warp by shuffles, the four warps of a row
  // by shared-memory atomics)
  for (int t0 = 0; t0 < pend; t0 += PKT) {
    __syncthreads();
    load_k(t0);
    __syncthreads();
    int64_t sc[2][4];
    bool valid[2][4];
    scores(t0, sc, valid);
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      int64_t m = INT64_MIN;
#pragma unroll
      for (int k = 0; k < 4; ++k) m = valid[i][k] && sc[i][k] > m ? sc[i][k] : m;
#pragma unroll
      for (int o = 1; o < 4; o <<= 1) { const int64_t w = __shfl_xor_sync(0xffffffffu, m, o); m = w > m ? w : m; }
      if (tq == 0 && m != INT64_MIN) atomicMax(reinterpret_cast<long long*>(&mx[srow(i)]), (long long)m);
    }
  }
  // pass 2: sums of e
  for (int t0 = 0; t0 < pend; t0 += PKT) {
    __syncthreads();
    load_k(t0);
    __syncthreads();
    int64_t sc[2][4];
    bool valid[2][4];
    scores(t0, sc, valid);
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      int64_t sacc = 0;
#pragma unroll
      for (int k = 0; k < 4; ++k) sacc += valid[i][k] ? exp_lookup(a.exp_t, mx[srow(i)] - sc[i][k]) : 0;
#pragma unroll
      for (int o = 1; o < 4; o <<= 1) sacc += __shfl_xor_sync(0xffffffffu, sacc, o);
      if (tq == 0 && sacc) atomicAdd(reinterpret_cast<unsigned long long*>(&ssum[srow(i)]), (unsigned long long)sacc);
    }
  }
  if constexpr (HD >= 32) {
    // pass 3 on the tensor cores: p = (e << 20) // sum (exact floor division through a per-row
    // reciprocal and integer corrections; 0 <= p <= 2^20) as three unsigned byte digits, V (int32) as
    // three unsigned bytes and a signed top byte; out = sum over the 12 digit products of
    // (p_i . v_j) << 8 (i + j), each an int8 MMA over the 64 keys of a tile (|.| < 2^23), the products
    // of one weight 8 s summed in int32 (< 2^25) and shifted into int64 per tile.  Warp w: rows
    // 16 (w % 2) .. + 15, dims (w / 2) HD/4 .. + HD/4 - 1 (HD/32 tiles of 8 dims).
    constexpr int TBV = PKT + 16;                      // plane row of 64 keys: 20 words, conflict-free
    constexpr int NTW = HD / 32;
    uint8_t* vpl = reinterpret_cast<uint8_t*>(vt);     // 4 planes x HD dims x TBV (over V and P tiles)
    uint8_t* ppl = klo;                                // 3 planes x PRT rows x TBV (over the key planes)
    __syncthreads();
    if (tid < PRT) sinv[tid] = ssum[tid] > 0 ? __drcp_rn((double)ssum[tid]) : 0.0;
    const int mtw = warp & 1, dq = warp >> 1;
    int64_t o64[NTW][4];
#pragma unroll
    for (int nt = 0; nt < NTW; ++nt)
#pragma unroll
      for (int f = 0; f < 4; ++f) o64[nt][f] = 0;
    for (int t0 = 0; t0 < pend; t0 += PKT) {
      __syncthreads();
      const int nk = min(PKT, pend - t0);
      // V tile -> byte planes, keys contiguous per dim (dims fastest over the threads: every warp
      // reads 128 contiguous bytes of a cached row); keys t >= nk are zero
      for (int e = tid; e < (PKT / 4) * HD; e += PA_THREADS) {
        const int d = e % HD, kg = e / HD;
        uint32_t v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int t = 4 * kg + u;
          v[u] = t < nk ? (uint32_t)a.vc[(cbase + t0 + t) * HD + d] : 0u;
        }
        const uint32_t lo01 = __byte_perm(v[0], v[1], 0x5140), lo23 = __byte_perm(v[2], v[3], 0x5140);
        const uint32_t hi01 = __byte_perm(v[0], v[1], 0x7362), hi23 = __byte_perm(v[2], v[3], 0x7362);
        *reinterpret_cast<uint32_t*>(vpl + (0 * HD + d) * TBV + 4 * kg) = __byte_perm(lo01, lo23, 0x5410);
        *reinterpret_cast<uint32_t*>(vpl + (1 * HD + d) * TBV + 4 * kg) = __byte_perm(lo01, lo23, 0x7632);
        *reinterpret_cast<uint32_t*>(vpl + (2 * HD + d) * TBV + 4 * kg) = __byte_perm(hi01, hi23, 0x5410);
        *reinterpret_cast<uint32_t*>(vpl + (3 * HD + d) * TBV + 4 * kg) = __byte_perm(hi01, hi23, 0x7632);
      }
      load_k(t0);
      __syncthreads();
      int64_t sc[2][4];
      bool valid[2][4];
      scores(t0, sc, valid);
      uint32_t pv[2][4];
#pragma unroll
      for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int row = srow(i);
          pv[i][k] = valid[i][k]
                         ? (uint32_t)floordiv_small_q(exp_lookup(a.exp_t, mx[row] - sc[i][k]) << 20, ssum[row], sinv[row])
                         : 0u;
        }
      __syncthreads();                                 // every warp's scores have read the key planes
#pragma unroll
      for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int n = 0; n < 2; ++n) {
          const int row = srow(i), key = nq * 16 + n * 8 + 2 * tq;
          const uint32_t pa = pv[i][2 * n], pb = pv[i][2 * n + 1];
#pragma unroll
          for (int d = 0; d < 3; ++d)                  // digit d of the two keys, little-endian
            *reinterpret_cast<uint16_t*>(ppl + (d * PRT + row) * TBV + key) =
                (uint16_t)(((pa >> (8 * d)) & 255u) | (((pb >> (8 * d)) & 255u) << 8));
        }
      __syncthreads();
#pragma unroll 1
      for (int sft = 0; sft < 6; ++sft) {
        int acc[NTW][4];
#pragma unroll
        for (int nt = 0; nt < NTW; ++nt)
#pragma unroll
          for (int f = 0; f < 4; ++f) acc[nt][f] = 0;
#pragma unroll 1
        for (int pi = 0; pi < 3; ++pi) {
          const int vj = sft - pi;
          if (vj < 0 || vj > 3) continue;
#pragma unroll
          for (int ks = 0; ks < PKT / 32; ++ks) {
            const int ra = (pi * PRT + mtw * 16 + g) * TBV + ks * 32 + 4 * tq, rb = ra + 8 * TBV;
            const uint32_t af[4] = {ld_s32(ppl + ra), ld_s32(ppl + rb), ld_s32(ppl + ra + 16), ld_s32(ppl + rb + 16)};
#pragma unroll
            for (int nt = 0; nt < NTW; ++nt) {
              const int kb = (vj * HD + dq * (HD / 4) + nt * 8 + g) * TBV + ks * 32 + 4 * tq;
              const uint32_t b0 = ld_s32(vpl + kb), b1 = ld_s32(vpl + kb + 16);
              if (vj == 3) mma_i8<false, true>(acc[nt], af, b0, b1);
              else mma_i8<false, false>(acc[nt], af, b0, b1);
            }
          }
        }
#pragma unroll
        for (int nt = 0; nt < NTW; ++nt)
#pragma unroll
          for (int f = 0; f < 4; ++f)
            o64[nt][f] = (int64_t)((uint64_t)o64[nt][f] + ((uint64_t)(int64_t)acc[nt][f] << (8 * sft)));
      }
    }
#pragma unroll
    for (int nt = 0; nt < NTW; ++nt)
#pragma unroll
      for (int f = 0; f < 4; ++f) {
        const int row = mtw * 16 + g + 8 * (f >> 1), dim = dq * (HD / 4) + nt * 8 + 2 * tq + (f & 1);
        if (row < nr) a.out[(size_t)(r0 + row) * a.ldo + (size_t)h * HD + dim] = shr64(o64[nt][f], 20);
      }
  } else {
    // pass 3: p = (e << 20) // sum (exact floor division through a per-row reciprocal and integer
    // corrections; p <= 2^20), then out += p . v as 32 x 32 -> 64-bit products (thread: row tid / 8,
    // dims 32 i + 4 (tid % 8) + (0..3): int4 reads of V, the 8 threads of a row on 32 distinct banks;
    // head dim 16: dims tid % 8 + 8 i)
    __syncthreads();
    if (tid < PRT) sinv[tid] = ssum[tid] > 0 ? __drcp_rn((double)ssum[tid]) : 0.0;
    constexpr int DPT = HD / 8;
    constexpr bool VEC = DPT % 4 == 0;                   // int4 runs of V (head dims >= 32)
    const int orow = tid >> 3, od = tid & 7;
    auto dim_of = [&](int jd) { return VEC ? (jd >> 2) * 32 + od * 4 + (jd & 3) : od + 8 * jd; };
    int64_t oacc[DPT];
  #pragma unroll
    for (int i = 0; i < DPT; ++i) oacc[i] = 0;
    for (int t0 = 0; t0 < pend; t0 += PKT) {
      __syncthreads();
      const int nk = min(PKT, pend - t0);
      for (int e = tid; e < PKT * (HD / 4); e += PA_THREADS) {     // V tile lands during the scores
        const int t = e / (HD / 4), c4 = e - t * (HD / 4);
        if (t < nk) cp_async16(reinterpret_cast<int4*>(vt) + e, reinterpret_cast<const int4*>(a.vc + (cbase + t0 + t) * HD) + c4);
        else reinterpret_cast<int4*>(vt)[e] = make_int4(0, 0, 0, 0);
      }
      cp_async_commit();
      load_k(t0);
      __syncthreads();
      int64_t sc[2][4];
      bool valid[2][4];
      scores(t0, sc, valid);
  #pragma unroll
      for (int i = 0; i < 2; ++i)
  #pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int row = srow(i);
          int32_t p = 0;
          if (valid[i][k])
            p = (int32_t)floordiv_small_q(exp_lookup(a.exp_t, mx[row] - sc[i][k]) << 20, ssum[row], sinv[row]);
          pt[row * PKT + skey(k)] = p;
        }
      cp_async_wait<0>();
      __syncthreads();
  #pragma unroll 2
      for (int t = 0; t < nk; ++t) {
        const int64_t p = pt[orow * PKT + t];
        if constexpr (VEC) {
  #pragma unroll
          for (int i = 0; i < DPT / 4; ++i) {
            const int4 v = *reinterpret_cast<const int4*>(vt + t * HD + dim_of(4 * i));
            oacc[4 * i] += p * v.x;
            oacc[4 * i + 1] += p * v.y;
            oacc[4 * i + 2] += p * v.z;
            oacc[4 * i + 3] += p * v.w;
          }
        } else {
  #pragma unroll
          for (int i = 0; i < DPT; ++i) oacc[i] += p * (int64_t)vt[t * HD + dim_of(i)];
        }
      }
    }
    if (orow < nr)
  #pragma unroll
      for (int i = 0; i < DPT; ++i) a.out[(size_t)(r0 + orow) * a.ldo + (size_t)h * HD + dim_of(i)] = shr64(oacc[i], 20);
  }
  tl_exit();
}

cudaError_t launch_attn_prefill(const AttnArgs& a, cudaStream_t st) {
  const int rep = a.KV > 0 ? a.H / a.KV : 0;
  if (rep < 1 || a.H % a.KV || a.R < 1) return cudaErrorInvalidValue;
  if (a.hd != 128 && a.hd != 64 && a.hd != 32 && a.hd != 16) return cudaErrorInvalidValue;
  const size_t tb = (size_t)(a.hd < 32 ? 32 : a.hd) + 16;
  const size_t smem = 2 * (size_t)PRT * tb + 2 * (size_t)PKT * tb + (size_t)PKT * a.hd * 4 + (size_t)PRT * PKT * 4;
  void (*kern)(const AttnArgs) = a.hd == 128 ? k_attn_prefill<128> : a.hd == 64 ? k_attn_prefill<64>
                               : a.hd == 32 ? k_attn_prefill<32> : k_attn_prefill<16>;
  static DevOnce attr_set[4];
  const int ti = a.hd == 128 ? 0 : a.hd == 64 ? 1 : a.hd == 32 ? 2 : 3;
  if (!attr_set[ti].done()) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e != cudaSuccess) return e;
    attr_set[ti].set();
  }
  kern<<<dim3((a.R + PRT - 1) / PRT, a.H), PA_THREADS, smem, st>>>(a);
  return cudaGetLastError();
}

}  // namespace exb
