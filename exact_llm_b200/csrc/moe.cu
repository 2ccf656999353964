// Mixture-of-experts MLP block (Qwen1.5-MoE shape): the exact integer MoE of
// experiments/moe_exact_kaggle.py:419-482 of novain-shibu/exact-llm.  Every linear is per-channel
// (QLin, exact_llm.py:89-96, with its per-row overflow drop rule); the MLP input m = irms(x, g2) is
// quantised once per row (xq, s) and shared by the router, the experts and the shared expert.
//
//   router        r = QLin_router(m)                      (NE logits, Q16)
//   p             isoftmax(r) in Q20 over all NE experts   (exact_llm.py:109-115)
//   sel           top-k experts by p, ties to the lower index (stable sort)
//   expert e      y_e = down_e(qrow(shr(isilu(gate_e(m)) * up_e(m), 16)))
//   shared        y_s = sd(qrow(shr(isilu(sg(m)) * su(m), 16)))
//   out           x += sum_k shr(p_k * y_{sel_k}, 20) + shr(isig(sgate(m)) * y_s, 16)
//
// B200 layout of the work: routing is one CTA per row (NE + 1 dot products: the router and the
// shared-expert gate); a one-CTA plan kernel lists, for every expert, the (row, k) "slots" routed
// to it (the shared expert is expert NE and takes every row); the expert MLPs are grouped GEMVs
// with one grid row per expert, so each active expert's weights stream from HBM once for all of
// its slots; activations and the final weighted combine are per-slot / per-row kernels.  Integer
// addition is associative, so the grouping never changes a bit.
#include "common.cuh"
#include "exb_internal.h"
#include "gemvdev.cuh"
#include "rowdev.cuh"

namespace exb {

constexpr int MOE_THREADS = 256;
constexpr int MOE_CH = 32;                  // output channels per CTA of the grouped GEMV
constexpr int MOE_RB = 4;                   // slots per pass of the grouped GEMV

// ---------------------------------------------------------------- routing (one CTA per row)
// Per-channel requant with the drop rule for one row of n raw sums (exact_llm.py:89-96).
EXB_DEV int ch_drop(uint64_t amax, int mbits) {
  const int d = bitlen64(amax) + mbits - 62;
  return d > 0 ? d : 0;
}
EXB_DEV int64_t ch_requant(int64_t acc, int64_t M, int s, int drop) {
  return shr64((int64_t)((uint64_t)shr64(acc, drop) * (uint64_t)M), 28 - s - drop);
}

__global__ void __launch_bounds__(MOE_THREADS) k_moe_route(MoeArgs a) {
  extern __shared__ __align__(16) unsigned char sm[];
  int16_t* xr = reinterpret_cast<int16_t*>(sm);                          // D
  int64_t* acc = reinterpret_cast<int64_t*>(sm + (((size_t)a.D * 2 + 15) & ~(size_t)15));   // NE + 1
  int64_t* pr = acc + a.NE + 1;                                           // NE
  const int r = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  for (int i = tid; i < (a.D >> 3); i += MOE_THREADS)
    reinterpret_cast<int4*>(xr)[i] = reinterpret_cast<const int4*>(a.xq + (size_t)r * a.ldq)[i];
  __syncthreads();
  // NE router channels and the shared-expert gate (channel NE)
  for (int ch = warp; ch <= a.NE; ch += MOE_THREADS / 32) {
    const int8_t* wrow = ch < a.NE ? a.w_router + (size_t)ch * a.D : a.w_sgate;
    int64_t s = 0;
    for (int c = lane; c < (a.D >> 4); c += 32) {
      const int4 w = __ldg(reinterpret_cast<const int4*>(wrow) + c);
      const int4* xp = reinterpret_cast<const int4*>(xr + 16 * c);
      s += dot16(w, xp[0], xp[1]);
    }
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) acc[ch] = s;
  }
  __syncthreads();
  if (tid == 0) {
    const int sh = a.xs[r];
    uint64_t mx = 0;
    for (int e = 0; e < a.NE; ++e) { const uint64_t u = uabs64(acc[e]); mx = u > mx ? u : mx; }
    const int drop = ch_drop(mx, a.mbits_router);
    int64_t best = INT64_MIN;
    for (int e = 0; e < a.NE; ++e) {
      pr[e] = ch_requant(acc[e], a.M_router[e], sh, drop);
      best = pr[e] > best ? pr[e] : best;
    }
    // isoftmax over all experts: e = EXP_T(max - r) (Q24), p = (e << 20) // sum e
    int64_t tot = 0;
    for (int e = 0; e < a.NE; ++e) { pr[e] = exp_lookup(a.exp_t, best - pr[e]); tot += pr[e]; }
    for (int e = 0; e < a.NE; ++e) pr[e] = (int64_t)(((uint64_t)pr[e] << 20) / (uint64_t)tot);
    // top-k, ties to the lower expert index
    uint64_t taken[2] = {0, 0};
    for (int k = 0; k < a.TOPK; ++k) {
      int be = -1;
      for (int e = 0; e < a.NE; ++e) {
        if ((taken[e >> 6] >> (e & 63)) & 1) continue;
        if (be < 0 || pr[e] > pr[be]) be = e;
      }
      taken[be >> 6] |= 1ull << (be & 63);
      a.sel[(size_t)r * a.TOPK + k] = be;
      a.prob[(size_t)r * a.TOPK + k] = pr[be];
      if (a.sel_hist) a.sel_hist[(size_t)r * a.TOPK + k] = be;
    }
    // shared-expert gate: isig(QLin_sgate(m)) (moe_exact_kaggle.py:420-424, 467)
    const int dg = ch_drop(uabs64(acc[a.NE]), a.mbits_sgate);
    a.sgv[r] = isig_dev(a.sig_t, ch_requant(acc[a.NE], a.M_sgate[0], sh, dg));
  }
}

// ---------------------------------------------------------------- plan (one CTA)
// slots of expert e: off[e] .. off[e+1]-1, rows ascending; the shared expert (index NE) takes
// every row.  slot_row / slot_exp describe a slot; slot_of[r * TOPK + k] names the slot of (r, k).
__global__ void k_moe_plan(MoeArgs a) {
  __shared__ int cnt[MOE_MAX_EXPERTS + 2];
  const int tid = threadIdx.x;
  for (int e = tid; e <= a.NE; e += blockDim.x) cnt[e] = 0;
  __syncthreads();
  for (int i = tid; i < a.R * a.TOPK; i += blockDim.x) atomicAdd(&cnt[a.sel[i]], 1);
  if (tid == 0) cnt[a.NE] = a.R;
  __syncthreads();
  if (tid == 0) {
    int o = 0;
    for (int e = 0; e <= a.NE; ++e) { a.off[e] = o; o += cnt[e]; }
    a.off[a.NE + 1] = o;
  }
  __syncthreads();
  for (int e = tid; e <= a.NE; e += blockDim.x) {
    int o = a.off[e];
    for (int r = 0; r < a.R; ++r) {
      if (e == a.NE) {
        a.slot_row[o] = r; a.slot_exp[o] = e; ++o;
        continue;
      }
      for (int k = 0; k < a.TOPK; ++k)
        if (a.sel[(size_t)r * a.TOPK + k] == e) {
          a.slot_row[o] = r; a.slot_exp[o] = e; a.slot_of[(size_t)r * a.TOPK + k] = o; ++o;
        }
    }
  }
}

// ---------------------------------------------------------------- grouped GEMV (per-channel raw sums)
// grid (ceil(max N / MOE_CH), NE + 1): CTA (bx, e) computes channels [bx*MOE_CH, +MOE_CH) of expert
// e's matrix for all of e's slots, in passes of MOE_RB slots whose int16 rows are staged in shared
// memory.  stage 0: gate|up (input = the slot row's xq), stage 1: down (input = the slot's hq).
__global__ void __launch_bounds__(MOE_THREADS) k_moe_gemv(MoeArgs a, int stage) {
  extern __shared__ __align__(16) unsigned char sm[];
  const int e = blockIdx.y;
  const int s0 = a.off[e], s1 = a.off[e + 1];
  if (s1 <= s0) return;                                       // expert not routed to this step
  const ExpertW& X = a.ex[e];
  const int N = stage == 0 ? 2 * X.I : a.D;
  const int K = stage == 0 ? a.D : X.I;
  const int8_t* W = stage == 0 ? X.w_gu : X.w_d;
  const int c0 = blockIdx.x * MOE_CH;
  if (c0 >= N) return;
  const int c1 = min(N, c0 + MOE_CH);
  int16_t* xs = reinterpret_cast<int16_t*>(sm);               // MOE_RB x K
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, C = K >> 4;
  int64_t* raw = stage == 0 ? a.raw_gu : a.raw_d;
  const int ldraw = stage == 0 ? a.ld_gu : a.D;
  for (int sb = s0; sb < s1; sb += MOE_RB) {
    const int nb = min(MOE_RB, s1 - sb);
    __syncthreads();
    for (int i = tid; i < nb * (K >> 3); i += MOE_THREADS) {
      const int j = i / (K >> 3), c = i - j * (K >> 3);
      const int16_t* src = stage == 0 ? a.xq + (size_t)a.slot_row[sb + j] * a.ldq : a.hq + (size_t)(sb + j) * a.ld_h;
      reinterpret_cast<int4*>(xs + (size_t)j * K)[c] = reinterpret_cast<const int4*>(src)[c];
    }
    __syncthreads();
    for (int ch = c0 + warp; ch < c1; ch += MOE_THREADS / 32) {
      const int4* wrow = reinterpret_cast<const int4*>(W + (size_t)ch * K);
      int64_t acc[MOE_RB] = {0, 0, 0, 0};
      for (int c = lane; c < C; c += 32) {
        const int4 w = __ldg(wrow + c);
#pragma unroll
        for (int j = 0; j < MOE_RB; ++j)
          if (j < nb) {
            const int4* xp = reinterpret_cast<const int4*>(xs + (size_t)j * K + 16 * c);
            acc[j] += dot16(w, xp[0], xp[1]);
          }
      }
#pragma unroll
      for (int j = 0; j < MOE_RB; ++j) {
        int64_t v = acc[j];
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0 && j < nb) raw[(size_t)(sb + j) * ldraw + ch] = v;
      }
    }
  }
}

// ---------------------------------------------------------------- per-slot activation
// gate|up raw sums (interleaved: channel 2j gate j, 2j+1 up j) -> per-channel requant of gate and
// up as two QLins (each its own drop) -> h = shr(isilu(g) * u, 16) -> xq, s = qrow(h)
__global__ void __launch_bounds__(MOE_THREADS) k_moe_act(MoeArgs a) {
  extern __shared__ __align__(16) unsigned char sm[];
  int64_t* hv = reinterpret_cast<int64_t*>(sm);                      // I
  __shared__ uint64_t red[33];
  const int slot = blockIdx.x;
  if (slot >= a.off[a.NE + 1]) return;
  const int e = a.slot_exp[slot], r = a.slot_row[slot];
  const ExpertW& X = a.ex[e];
  const int I = X.I, sh = a.xs[r];
  const int64_t* rw = a.raw_gu + (size_t)slot * a.ld_gu;
  uint64_t mg = 0, mu = 0;
  for (int j = threadIdx.x; j < I; j += MOE_THREADS) {
    const uint64_t g = uabs64(rw[2 * j]), u = uabs64(rw[2 * j + 1]);
    mg = g > mg ? g : mg;
    mu = u > mu ? u : mu;
  }
  mg = block_max_u64<MOE_THREADS>(mg, red);
  mu = block_max_u64<MOE_THREADS>(mu, red);
  const int dg = ch_drop(mg, X.mb_g), du = ch_drop(mu, X.mb_u);
  uint64_t mh = 0;
  for (int j = threadIdx.x; j < I; j += MOE_THREADS) {
    const int64_t yg = ch_requant(rw[2 * j], X.M_gu[2 * j], sh, dg);
    const int64_t yu = ch_requant(rw[2 * j + 1], X.M_gu[2 * j + 1], sh, du);
    const int64_t h = shr64((int64_t)((uint64_t)isilu_dev(a.silu_t, yg) * (uint64_t)yu), 16);
    hv[j] = h;
    const uint64_t ah = uabs64(h);
    mh = ah > mh ? ah : mh;
  }
  mh = block_max_u64<MOE_THREADS>(mh, red);
  const int s = qrow_shift(mh);
  for (int j = threadIdx.x; j < I; j += MOE_THREADS) a.hq[(size_t)slot * a.ld_h + j] = qrow_value(hv[j], s);
  if (threadIdx.x == 0) a.hs[slot] = s;
}

// ---------------------------------------------------------------- combine (one CTA per row)
// x[r] += sum_k shr(p_k * y_k, 20) + shr(isig(sgate) * y_shared, 16); y = QLin_down requant of the
// slot's raw sums (its own drop over the D channels)
__global__ void __launch_bounds__(MOE_THREADS) k_moe_combine(MoeArgs a, int64_t* x, int ldx) {
  __shared__ uint64_t red[33];
  __shared__ int dr[MOE_MAX_TOPK + 1];
  const int r = blockIdx.x;
  const int K1 = a.TOPK + 1;
  for (int k = 0; k < K1; ++k) {
    const int slot = k < a.TOPK ? a.slot_of[(size_t)r * a.TOPK + k] : a.off[a.NE] + r;
    const int64_t* rw = a.raw_d + (size_t)slot * a.D;
    uint64_t m = 0;
    for (int i = threadIdx.x; i < a.D; i += MOE_THREADS) { const uint64_t u = uabs64(rw[i]); m = u > m ? u : m; }
    m = block_max_u64<MOE_THREADS>(m, red);
    if (threadIdx.x == 0) dr[k] = ch_drop(m, a.ex[a.slot_exp[slot]].mb_d);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < a.D; i += MOE_THREADS) {
    int64_t add = 0;
    for (int k = 0; k < K1; ++k) {
      const int slot = k < a.TOPK ? a.slot_of[(size_t)r * a.TOPK + k] : a.off[a.NE] + r;
      const ExpertW& X = a.ex[a.slot_exp[slot]];
      const int64_t y = ch_requant(a.raw_d[(size_t)slot * a.D + i], X.M_d[i], a.hs[slot], dr[k]);
      if (k < a.TOPK) add = (int64_t)((uint64_t)add + (uint64_t)shr64((int64_t)((uint64_t)a.prob[(size_t)r * a.TOPK + k] * (uint64_t)y), 20));
      else add = (int64_t)((uint64_t)add + (uint64_t)shr64((int64_t)((uint64_t)a.sgv[r] * (uint64_t)y), 16));
    }
    int64_t* o = x + (size_t)r * ldx + i;
    *o = (int64_t)((uint64_t)*o + (uint64_t)add);
  }
}

// ---------------------------------------------------------------- host
cudaError_t launch_moe(const MoeArgs& a, int64_t* x, int ldx, cudaStream_t st) {
  if (a.NE > MOE_MAX_EXPERTS || a.TOPK > MOE_MAX_TOPK || a.D % 16 || a.R <= 0) return cudaErrorInvalidValue;
  const size_t smem_route = ((size_t)a.D * 2 + 15) / 16 * 16 + (size_t)(2 * a.NE + 1) * 8;
  k_moe_route<<<a.R, MOE_THREADS, smem_route, st>>>(a);
  k_moe_plan<<<1, 256, 0, st>>>(a);
  int nmax = 2 * a.IMAX > a.D ? 2 * a.IMAX : a.D;
  const size_t smem_g = (size_t)MOE_RB * (a.D > a.IMAX ? a.D : a.IMAX) * 2;
  static DevOnce attr;
  if (!attr.done()) {
    cudaError_t e = cudaFuncSetAttribute(k_moe_gemv, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(k_moe_act, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024);
    if (e != cudaSuccess) return e;
    attr.set();
  }
  k_moe_gemv<<<dim3((nmax + MOE_CH - 1) / MOE_CH, a.NE + 1), MOE_THREADS, smem_g, st>>>(a, 0);
  k_moe_act<<<a.R * (a.TOPK + 1), MOE_THREADS, (size_t)a.IMAX * 8, st>>>(a);
  k_moe_gemv<<<dim3((nmax + MOE_CH - 1) / MOE_CH, a.NE + 1), MOE_THREADS, smem_g, st>>>(a, 1);
  k_moe_combine<<<a.R, MOE_THREADS, 0, st>>>(a, x, ldx);
  return cudaGetLastError();
}

}  // namespace exb
