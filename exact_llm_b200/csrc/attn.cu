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
  static bool attr_set[4] = {false, false, false, false};
  const int ti = a.hd == 128 ? 0 : a.hd == 64 ? 1 : a.hd == 32 ? 2 : 3;
  if (!attr_set[ti]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e != cudaSuccess) return e;
    attr_set[ti] = true;
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

}  // namespace exb
