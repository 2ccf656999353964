// Per-row integer kernels: embedding gather, integer RMSNorm + row quantisation, row
// quantisation, per-channel requant with the drop rule, and the Freivalds comparison.
//
// Reference semantics (novain-shibu/exact-llm): irms exact_llm.py:100-106, qrow :41-46,
// QLin requant + per-row drop rule :89-96 (SPEC.md:28), embedding rows :163.
#include "common.cuh"
#include "exb_internal.h"

namespace exb {

constexpr int ROW_THREADS = 512;

static cudaError_t launch_simple(const void* fn, dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl,
                                 void** args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelExC(&cfg, fn, args);
}

// ---------------------------------------------------------------- embedding: x = emb[id] << shift
__global__ void k_embed(const int8_t* __restrict__ emb, int shift, const int32_t* __restrict__ ids, int D,
                        int64_t* __restrict__ x) {
  pdl_wait();
  const int r = blockIdx.x;
  const int8_t* e = emb + (size_t)ids[r] * D;
  for (int i = threadIdx.x; i < D; i += blockDim.x) x[(size_t)r * D + i] = (int64_t)e[i] << shift;
  pdl_launch_dependents();
}

cudaError_t launch_embed(const int8_t* emb, int emb_shift, const int32_t* ids, int R, int D, int64_t* x,
                         cudaStream_t st, bool pdl) {
  void* args[] = {(void*)&emb, (void*)&emb_shift, (void*)&ids, (void*)&D, (void*)&x};
  return launch_simple((const void*)k_embed, dim3(R), dim3(256), 0, st, pdl, args);
}

__global__ void k_embed64(const int64_t* __restrict__ emb, const int32_t* __restrict__ ids, int D,
                          int64_t* __restrict__ x) {
  pdl_wait();
  const int r = blockIdx.x;
  const int64_t* e = emb + (size_t)ids[r] * D;
  for (int i = threadIdx.x; i < D; i += blockDim.x) x[(size_t)r * D + i] = e[i];
  pdl_launch_dependents();
}

cudaError_t launch_embed64(const int64_t* emb, const int32_t* ids, int R, int D, int64_t* x, cudaStream_t st,
                           bool pdl) {
  void* args[] = {(void*)&emb, (void*)&ids, (void*)&D, (void*)&x};
  return launch_simple((const void*)k_embed64, dim3(R), dim3(256), 0, st, pdl, args);
}

// ---------------------------------------------------------------- irms + qrow
// a = irms(x, g) (exact_llm.py:100-106), then xq, s = qrow(a) (:41-46).
__global__ void __launch_bounds__(ROW_THREADS) k_norm_q(const int64_t* __restrict__ x, int ldx,
                                                        const int64_t* __restrict__ g, int D,
                                                        int16_t* __restrict__ xq, int ldq, int32_t* __restrict__ xs) {
  extern __shared__ int64_t ys[];
  __shared__ uint64_t red[33];
  pdl_wait();
  const int r = blockIdx.x;
  const int64_t* xr = x + (size_t)r * ldx;
  uint64_t m = 0;
  for (int i = threadIdx.x; i < D; i += ROW_THREADS) { uint64_t v = uabs64(xr[i]); m = v > m ? v : m; }
  m = block_max_u64<ROW_THREADS>(m, red);
  int k = bitlen64(m) - 24;
  k = k > 0 ? k : 0;
  uint64_t ss = 0;
  for (int i = threadIdx.x; i < D; i += ROW_THREADS) {
    const int64_t v = shr64(xr[i], k);
    ss += (uint64_t)v * (uint64_t)v;
  }
  const int64_t sum = block_sum_i64<ROW_THREADS>((int64_t)ss, red);
  const int64_t ms = floordiv64(sum, D) + 1;
  int64_t rt = isqrt_ref(ms);
  rt = rt > 1 ? rt : 1;
  const int64_t den = (int64_t)((uint64_t)rt << k);
  uint64_t m2 = 0;
  for (int i = threadIdx.x; i < D; i += ROW_THREADS) {
    const int64_t y = floordiv64((int64_t)((uint64_t)xr[i] << 16), den);
    const int64_t a = shr64((int64_t)((uint64_t)y * (uint64_t)g[i]), 16);
    ys[i] = a;
    const uint64_t v = uabs64(a);
    m2 = v > m2 ? v : m2;
  }
  m2 = block_max_u64<ROW_THREADS>(m2, red);
  const int s = qrow_shift(m2);
  for (int i = threadIdx.x; i < D; i += ROW_THREADS) xq[(size_t)r * ldq + i] = qrow_value(ys[i], s);
  if (threadIdx.x == 0) xs[r] = s;
  pdl_launch_dependents();
}

cudaError_t launch_norm_q(const int64_t* x, int ldx, const int64_t* g, int R, int D, int16_t* xq, int ldq,
                          int32_t* xs, cudaStream_t st, bool pdl) {
  const size_t smem = (size_t)D * 8;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(k_norm_q, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  void* args[] = {(void*)&x, (void*)&ldx, (void*)&g, (void*)&D, (void*)&xq, (void*)&ldq, (void*)&xs};
  return launch_simple((const void*)k_norm_q, dim3(R), dim3(ROW_THREADS), smem, st, pdl, args);
}

// ---------------------------------------------------------------- qrow only
__global__ void __launch_bounds__(ROW_THREADS) k_quant(const int64_t* __restrict__ x, int ldx, int K,
                                                       int16_t* __restrict__ xq, int ldq, int32_t* __restrict__ xs) {
  __shared__ uint64_t red[33];
  pdl_wait();
  const int r = blockIdx.x;
  const int64_t* xr = x + (size_t)r * ldx;
  uint64_t m = 0;
  for (int i = threadIdx.x; i < K; i += ROW_THREADS) { uint64_t v = uabs64(xr[i]); m = v > m ? v : m; }
  m = block_max_u64<ROW_THREADS>(m, red);
  const int s = qrow_shift(m);
  for (int i = threadIdx.x; i < K; i += ROW_THREADS) xq[(size_t)r * ldq + i] = qrow_value(xr[i], s);
  if (threadIdx.x == 0) xs[r] = s;
  pdl_launch_dependents();
}

cudaError_t launch_quant(const int64_t* x, int ldx, int R, int K, int16_t* xq, int ldq, int32_t* xs,
                         cudaStream_t st, bool pdl) {
  void* args[] = {(void*)&x, (void*)&ldx, (void*)&K, (void*)&xq, (void*)&ldq, (void*)&xs};
  return launch_simple((const void*)k_quant, dim3(R), dim3(ROW_THREADS), 0, st, pdl, args);
}

// ---------------------------------------------------------------- per-channel requant, general drop rule
// drop = max(bitlen(max_row |acc|) + Mbits - 62, 0); y = shr(shr(acc, drop) * M, 28 - s - drop) + b
// (exact_llm.py:93-96).  Used when the host cannot prove drop == 0 for every input.
__global__ void __launch_bounds__(ROW_THREADS) k_requant_ch(const int64_t* __restrict__ acc, int ld, int N,
                                                            const int64_t* __restrict__ M, int mbits,
                                                            const int64_t* __restrict__ b, const int32_t* __restrict__ xs,
                                                            int64_t* __restrict__ out, int ldo, int resid) {
  __shared__ uint64_t red[33];
  pdl_wait();
  const int r = blockIdx.x;
  const int64_t* ar = acc + (size_t)r * ld;
  uint64_t m = 0;
  for (int i = threadIdx.x; i < N; i += ROW_THREADS) { uint64_t v = uabs64(ar[i]); m = v > m ? v : m; }
  m = block_max_u64<ROW_THREADS>(m, red);
  int drop = bitlen64(m) + mbits - 62;
  drop = drop > 0 ? drop : 0;
  const int s = xs[r];
  for (int i = threadIdx.x; i < N; i += ROW_THREADS) {
    int64_t y = shr64((int64_t)((uint64_t)shr64(ar[i], drop) * (uint64_t)M[i]), 28 - s - drop);
    if (b) y = (int64_t)((uint64_t)y + (uint64_t)b[i]);
    int64_t* o = out + (size_t)r * ldo + i;
    *o = resid ? (int64_t)((uint64_t)*o + (uint64_t)y) : y;
  }
  pdl_launch_dependents();
}

cudaError_t launch_requant_channel(const int64_t* acc, int ld, int R, const LinW& L, int64_t* out, int ldo,
                                   const int32_t* xs, int epi, cudaStream_t st, bool pdl) {
  int N = L.N, mbits = L.mbits, resid = epi == EPI_RESID ? 1 : 0;
  const int64_t* M = L.Mc;
  const int64_t* b = L.b;
  void* args[] = {(void*)&acc, (void*)&ld, (void*)&N, (void*)&M, (void*)&mbits, (void*)&b, (void*)&xs,
                  (void*)&out, (void*)&ldo, (void*)&resid};
  return launch_simple((const void*)k_requant_ch, dim3(R), dim3(ROW_THREADS), 0, st, pdl, args);
}

// ---------------------------------------------------------------- Freivalds comparison
// acc layout: (nchecks, 4) = lhs_p1, lhs_p2, rhs_p1, rhs_p2 (each an unreduced sum of residues)
__global__ void k_fr_check(const unsigned long long* __restrict__ acc, int n, int* fail, int* err) {
  pdl_wait();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    bool ok = true;
    for (int p = 0; p < 2; ++p) ok &= (acc[(size_t)i * 4 + p] % fr_prime(p)) == (acc[(size_t)i * 4 + 2 + p] % fr_prime(p));
    if (!ok) {
      atomicAdd(fail, 1);
      set_err(err, ERR_FREIVALDS);
    }
  }
  pdl_launch_dependents();
}

cudaError_t launch_fr_check(const unsigned long long* acc, int nchecks, int* fail_count, int* err,
                            cudaStream_t st, bool pdl) {
  if (nchecks <= 0) return cudaSuccess;
  void* args[] = {(void*)&acc, (void*)&nchecks, (void*)&fail_count, (void*)&err};
  int blocks = (nchecks + 255) / 256;
  return launch_simple((const void*)k_fr_check, dim3(blocks), dim3(256), 0, st, pdl, args);
}

}  // namespace exb
