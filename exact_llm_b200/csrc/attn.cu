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

namespace cg = cooperative_groups;

namespace exb {

constexpr int CL = 8;               // CTAs per cluster (portable cluster size)
constexpr int ATT_THREADS = 256;
constexpr int REP_MAX = 8;          // query heads per KV head handled by one cluster

// ---------------------------------------------------------------- RoPE + cache write + q quantisation
__global__ void __launch_bounds__(128) k_rope_cache(const AttnArgs a) {
  __shared__ uint64_t red[33];
  pdl_wait();
  const int r = blockIdx.x, j = blockIdx.y, d = threadIdx.x;
  const int hd = a.hd, half = hd >> 1, rep = a.H / a.KV;
  const int pos = a.row_pos[r], seq = a.row_seq[r];
  if (pos < 0 || pos >= a.Smax || pos >= a.Tmax) {
    if (d == 0) set_err(a.err, ERR_BOUNDS);
    return;
  }
  const int64_t* row = a.qkv + (size_t)r * a.ldqkv;
  int64_t c = 0, s = 0;
  if (d < hd) {
    c = a.cos_t[(size_t)pos * half + (d % half)];
    s = a.sin_t[(size_t)pos * half + (d % half)];
  }
  auto rope1 = [&](const int64_t* x) -> int64_t {
    if (d >= hd) return 0;
    const int64_t rot = d < half ? (int64_t)(0ull - (uint64_t)x[d + half]) : x[d - half];
    return shr64((int64_t)((uint64_t)x[d] * (uint64_t)c + (uint64_t)rot * (uint64_t)s), 16);
  };
  // key head j: RoPE, per-row quantisation, cache write; value head j: cache write
  const int64_t kr = rope1(row + (size_t)(a.H + j) * hd);
  const int sk = qrow_shift(block_max_u64<128>(d < hd ? uabs64(kr) : 0, red));
  const size_t cidx = ((size_t)seq * a.KV + j) * a.Smax + pos;
  if (d < hd) {
    a.kc[cidx * hd + d] = qrow_value(kr, sk);
    const int64_t v = row[(size_t)(a.H + a.KV + j) * hd + d];
    if (v > INT32_MAX || v < INT32_MIN) set_err(a.err, ERR_V_RANGE);
    a.vc[cidx * hd + d] = (int32_t)v;
  }
  if (d == 0) a.ks[cidx] = (int8_t)sk;
  // query heads of this KV group: RoPE + per-row quantisation
  for (int i = 0; i < rep; ++i) {
    const int h = j * rep + i;
    const int64_t qr = rope1(row + (size_t)h * hd);
    const int sq = qrow_shift(block_max_u64<128>(d < hd ? uabs64(qr) : 0, red));
    if (d < hd) a.qq[((size_t)r * a.H + h) * hd + d] = qrow_value(qr, sq);
    if (d == 0) a.qs[(size_t)r * a.H + h] = sq;
  }
  pdl_launch_dependents();
}

cudaError_t launch_rope_cache(const AttnArgs& a, cudaStream_t st, bool pdl) {
  if (a.hd > 128 || (a.hd & 1) || a.H % a.KV) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.R, a.KV);
  cfg.blockDim = dim3(128);
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, k_rope_cache, a);
}

// ---------------------------------------------------------------- decode attention (one cluster per row x KV head)
EXB_DEV int64_t dot_i16(const int16_t* __restrict__ a, const int16_t* __restrict__ b, int hd) {
  int64_t acc = 0;
  for (int d = 0; d < hd; d += 8) {
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

__global__ void __cluster_dims__(CL, 1, 1) __launch_bounds__(ATT_THREADS) k_attn_decode(const AttnArgs a, int SCmax) {
  extern __shared__ __align__(16) unsigned char sm[];
  __shared__ int64_t lmax[REP_MAX], lsum[REP_MAX], gmax[REP_MAX], gsum[REP_MAX];
  __shared__ int qsh[REP_MAX];
  cg::cluster_group cluster = cg::this_cluster();
  const int c = (int)cluster.block_rank();
  const int j = blockIdx.y, r = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int hd = a.hd, rep = a.H / a.KV;

  int16_t* qs_sm = reinterpret_cast<int16_t*>(sm);                                  // rep*hd
  int64_t* sc = reinterpret_cast<int64_t*>(sm + ((rep * hd * 2 + 15) & ~15));      // rep*SCmax
  int64_t* pout = sc + (size_t)rep * SCmax;                                          // rep*hd
  int64_t* pv = pout + (size_t)rep * hd;                                             // ATT_THREADS*REP_MAX

  pdl_wait();
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

  // phase 1: scores of this CTA's positions, local max per head
  for (int e = tid; e < rep * n; e += ATT_THREADS) {
    const int i = e / n, t = t0 + (e - i * n);
    const int64_t acc = dot_i16(qs_sm + i * hd, a.kc + (cbase + t) * hd, hd);
    sc[(size_t)i * SCmax + (t - t0)] =
        shr64((int64_t)((uint64_t)acc * (uint64_t)a.inv), 32 - qsh[i] - (int)a.ks[cbase + t]);
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
    for (int t = part; t < n; t += nparts) {
      const int64_t v = a.vc[(cbase + t0 + t) * hd + d];
#pragma unroll
      for (int i = 0; i < REP_MAX; ++i)
        if (i < rep) acc[i] += sc[(size_t)i * SCmax + t] * v;
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
    for (int e = e0 + tid; e < e1; e += ATT_THREADS) {
      int64_t s = 0;
      for (int cc = 0; cc < CL; ++cc) s += cluster.map_shared_rank(pout, cc)[e];
      a.out[(size_t)r * a.ldo + (size_t)j * rep * hd + e] = shr64(s, 20);
    }
  }
  cluster.sync();                                        // peers' shared memory stays alive until read
  pdl_launch_dependents();
}

cudaError_t launch_attn_decode(const AttnArgs& a, cudaStream_t st, bool pdl) {
  const int rep = a.H / a.KV;
  if (rep > REP_MAX || a.H % a.KV || ATT_THREADS % a.hd || a.hd % 8) return cudaErrorInvalidValue;
  const int SCmax = (a.Smax + CL - 1) / CL;
  const size_t smem = (size_t)((rep * a.hd * 2 + 15) & ~15) + (size_t)rep * SCmax * 8 + (size_t)rep * a.hd * 8 +
                      (size_t)ATT_THREADS * REP_MAX * 8;
  if (smem > 200 * 1024) return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(k_attn_decode, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
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
  return cudaLaunchKernelEx(&cfg, k_attn_decode, a, SCmax);
}

}  // namespace exb
