// Per-row integer kernels: embedding gather, integer RMSNorm + row quantisation, row
// quantisation, per-channel requant with the drop rule, and the Freivalds comparison.
//
// Reference semantics (novain-shibu/exact-llm): irms exact_llm.py:100-106, qrow :41-46,
// QLin requant + per-row drop rule :89-96 (SPEC.md:28), embedding rows :163.
#include "common.cuh"
#include "exb_internal.h"
#include "rowdev.cuh"
#include "tpx.cuh"

namespace exb {

constexpr int ROW_THREADS = 512;

// The norm gains are weights: pull them into L2 before the dependent-launch wait, so the norm reads
// them from L2 instead of HBM once the row is ready.
EXB_DEV void prefetch_gains(const int64_t* g, int D) {
  if (threadIdx.x == 0 && !((uintptr_t)g & 15) && !(D & 1)) prefetch_l2_bulk(g, (uint32_t)D * 8);
}

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
// With `nstat`, the row's (max |x|, sum x^2) for a consumer that finishes the norm from them.
EXB_DEV void embed_stats(uint64_t m, uint64_t ss, unsigned long long* nstat) {
  __shared__ uint64_t red[33];
  m = block_max_u64<256>(m, red);
  ss = (uint64_t)block_sum_i64<256>((int64_t)ss, red);
  if (threadIdx.x == 0) { nstat[0] = m; nstat[1] = ss; }
}

__global__ void __launch_bounds__(256) k_embed(const int8_t* __restrict__ emb, int shift, const int32_t* __restrict__ ids,
                                               int D, int64_t* __restrict__ x, unsigned long long* __restrict__ nstat) {
  pdl_wait();
  const int r = blockIdx.x;
  const int8_t* e = emb + (size_t)ids[r] * D;
  uint64_t m = 0, ss = 0;
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    const int64_t v = (int64_t)e[i] << shift;
    x[(size_t)r * D + i] = v;
    const uint64_t a = uabs64(v);
    m = a > m ? a : m;
    ss += (uint64_t)v * (uint64_t)v;
  }
  if (nstat) embed_stats(m, ss, nstat + 2 * r);
  pdl_launch_dependents();
  tl_exit();
}

cudaError_t launch_embed(const int8_t* emb, int emb_shift, const int32_t* ids, int R, int D, int64_t* x,
                         cudaStream_t st, bool pdl, unsigned long long* nstat) {
  void* args[] = {(void*)&emb, (void*)&emb_shift, (void*)&ids, (void*)&D, (void*)&x, (void*)&nstat};
  return launch_simple((const void*)k_embed, dim3(R), dim3(256), 0, st, pdl, args);
}

__global__ void k_embed64(const int64_t* __restrict__ emb, const int32_t* __restrict__ ids, int D,
                          int64_t* __restrict__ x) {
  pdl_wait();
  const int r = blockIdx.x;
  const int64_t* e = emb + (size_t)ids[r] * D;
  for (int i = threadIdx.x; i < D; i += blockDim.x) x[(size_t)r * D + i] = e[i];
  pdl_launch_dependents();
  tl_exit();
}

cudaError_t launch_embed64(const int64_t* emb, const int32_t* ids, int R, int D, int64_t* x, cudaStream_t st,
                           bool pdl) {
  void* args[] = {(void*)&emb, (void*)&ids, (void*)&D, (void*)&x};
  return launch_simple((const void*)k_embed64, dim3(R), dim3(256), 0, st, pdl, args);
}

// ---------------------------------------------------------------- embedding + first irms/qrow
// x = emb[id] (int8 << shift, or general int64 Q16 rows); xq, s = qrow(irms(x, g)).
__global__ void __launch_bounds__(ROW_THREADS) k_embed_norm(const int8_t* __restrict__ emb,
                                                            const int64_t* __restrict__ emb_q16, int shift,
                                                            const int32_t* __restrict__ ids, int D,
                                                            const int64_t* __restrict__ g, int64_t* __restrict__ x,
                                                            int16_t* __restrict__ xq, int ldq, int32_t* __restrict__ xs) {
  extern __shared__ int64_t ys[];
  __shared__ uint64_t red[33];
  pdl_wait();
  pdl_launch_dependents();
  const int r = blockIdx.x;
  const size_t row = (size_t)ids[r] * D;
  uint64_t m = 0;
  for (int i = threadIdx.x; i < D; i += ROW_THREADS) {
    const int64_t v = emb_q16 ? emb_q16[row + i] : (int64_t)emb[row + i] << shift;
    ys[i] = v;
    x[(size_t)r * D + i] = v;
    const uint64_t a = uabs64(v);
    m = a > m ? a : m;
  }
  row_norm_q_staged<ROW_THREADS>(g, D, xq + (size_t)r * ldq, xs + r, ys, red, m);
  tl_exit();
}

cudaError_t launch_embed_norm(const int8_t* emb, const int64_t* emb_q16, int emb_shift, const int32_t* ids, int R,
                              int D, const int64_t* g, int64_t* x, int16_t* xq, int ldq, int32_t* xs,
                              cudaStream_t st, bool pdl) {
  const size_t smem = (size_t)D * 8;
  static DevOnce attr_set;   // raised once to the full budget, never lowered
  if (!attr_set.done()) {
    cudaError_t e = cudaFuncSetAttribute(k_embed_norm, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e != cudaSuccess) return e;
    attr_set.set();
  }
  void* args[] = {(void*)&emb, (void*)&emb_q16, (void*)&emb_shift, (void*)&ids, (void*)&D, (void*)&g, (void*)&x,
                  (void*)&xq, (void*)&ldq, (void*)&xs};
  return launch_simple((const void*)k_embed_norm, dim3(R), dim3(ROW_THREADS), smem, st, pdl, args);
}

// ---------------------------------------------------------------- irms + qrow, qrow (one CTA per row)
// int8 digit planes (lo = xq & 255, hi = xq >> 8) of row r for the tensor-core GEMM: planes of
// prow rows of K bytes (TC_DECODE_ROWS for decode steps, the padded chunk for prefill), the hi plane
// right after the lo plane
EXB_DEV void put_digits(uint8_t* dig, int prow, int K, int r, int i, int16_t v) {
  dig[(size_t)r * K + i] = (uint8_t)(v & 255);
  dig[(size_t)(prow + r) * K + i] = (uint8_t)(int8_t)(v >> 8);
}

// EPT: elements per thread of the register variant (D <= EPT * ROW_THREADS), 0 = the row staged in
// shared memory; one instantiation per variant keeps the others' registers out of it
template <int EPT>
__global__ void __launch_bounds__(ROW_THREADS) k_norm_q(const int64_t* __restrict__ x, int ldx,
                                                        const int64_t* __restrict__ g, int D,
                                                        int16_t* __restrict__ xq, int ldq, int32_t* __restrict__ xs,
                                                        uint8_t* __restrict__ dig, int64_t* __restrict__ xcap,
                                                        int64_t ldcap, int dig_rows) {
  extern __shared__ int64_t ys[];
  __shared__ uint64_t red[33];
  prefetch_gains(g, D);
  pdl_wait();
  pdl_launch_dependents();
  const int r = blockIdx.x;
  if constexpr (EPT > 0) row_norm_q_regs<ROW_THREADS, EPT>(x + (size_t)r * ldx, g, D, xq + (size_t)r * ldq, xs + r, red);
  else row_norm_q<ROW_THREADS>(x + (size_t)r * ldx, g, D, xq + (size_t)r * ldq, xs + r, ys, red);
  if (dig)   // the row was written by this CTA (visible after the function's final barrier)
    for (int i = threadIdx.x; i < D; i += ROW_THREADS) put_digits(dig, dig_rows, D, r, i, xq[(size_t)r * ldq + i]);
  if (xcap)
    for (int i = threadIdx.x; i < D; i += ROW_THREADS) xcap[(size_t)r * ldcap + i] = ld_cg(x + (size_t)r * ldx + i);
  tl_exit();
}

cudaError_t launch_norm_q(const int64_t* x, int ldx, const int64_t* g, int R, int D, int16_t* xq, int ldq,
                          int32_t* xs, cudaStream_t st, bool pdl, uint8_t* dig, int64_t* xcap, int64_t ldcap,
                          int dig_rows) {
  const int v = D <= 4 * ROW_THREADS ? 0 : D <= 8 * ROW_THREADS ? 1 : D <= 12 * ROW_THREADS ? 2 : 3;
  const void* fn = v == 0 ? (const void*)k_norm_q<4> : v == 1 ? (const void*)k_norm_q<8>
                 : v == 2 ? (const void*)k_norm_q<12> : (const void*)k_norm_q<0>;
  const size_t smem = v == 3 ? (size_t)D * 16 : 0;
  if (smem > 200 * 1024) return cudaErrorInvalidValue;
  static DevOnce attr_set;   // raised once to the full budget, never lowered
  if (v == 3 && !attr_set.done()) {
    cudaError_t e = cudaFuncSetAttribute(k_norm_q<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e != cudaSuccess) return e;
    attr_set.set();
  }
  void* args[] = {(void*)&x,   (void*)&ldx, (void*)&g,   (void*)&D,     (void*)&xq,      (void*)&ldq,
                  (void*)&xs,  (void*)&dig, (void*)&xcap, (void*)&ldcap, (void*)&dig_rows};
  return launch_simple(fn, dim3(R), dim3(ROW_THREADS), smem, st, pdl, args);
}

__global__ void __launch_bounds__(ROW_THREADS) k_quant(const int64_t* __restrict__ x, int ldx, int K,
                                                       int16_t* __restrict__ xq, int ldq, int32_t* __restrict__ xs,
                                                       uint8_t* __restrict__ dig, int dig_rows) {
  extern __shared__ int64_t ys[];
  __shared__ uint64_t red[33];
  pdl_wait();
  pdl_launch_dependents();
  const int r = blockIdx.x;
  row_quant<ROW_THREADS>(x + (size_t)r * ldx, K, xq + (size_t)r * ldq, xs + r, ys, red);
  if (dig)   // the row was written by this CTA (visible after the function's final barrier)
    for (int i = threadIdx.x; i < K; i += ROW_THREADS) put_digits(dig, dig_rows, K, r, i, xq[(size_t)r * ldq + i]);
  tl_exit();
}

cudaError_t launch_quant(const int64_t* x, int ldx, int R, int K, int16_t* xq, int ldq, int32_t* xs,
                         cudaStream_t st, bool pdl, uint8_t* dig, int dig_rows) {
  const size_t smem = (size_t)K * 8;
  if (smem > 200 * 1024) return cudaErrorInvalidValue;   // one row staged in shared memory
  static DevOnce attr_set;   // raised once to the full budget, never lowered
  if (!attr_set.done()) {
    cudaError_t e = cudaFuncSetAttribute(k_quant, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e != cudaSuccess) return e;
    attr_set.set();
  }
  void* args[] = {(void*)&x, (void*)&ldx, (void*)&K, (void*)&xq, (void*)&ldq, (void*)&xs, (void*)&dig, (void*)&dig_rows};
  return launch_simple((const void*)k_quant, dim3(R), dim3(ROW_THREADS), smem, st, pdl, args);
}

// ---------------------------------------------------------------- tensor parallel: exchange + norm
// Consumer of a row-split linear's fused exchange (TPX_SUM_O after o, TPX_SUM_D after down) and the
// norm that follows it, one CTA per row: x[r, j] += shr(sum over ranks, 28 - s) + b[j]
// (exact_llm.py:89-96 on the full accumulator), s = qrow_shift of the max over ranks of the linear's
// input row max, then xq, s' = qrow(irms(x[r], g)) (exact_llm.py:100-106, 41-46).
__global__ void __launch_bounds__(ROW_THREADS) k_tpx_norm(const TpX x, int sum_type, const int64_t* __restrict__ bias,
                                                          int64_t* __restrict__ xr, int ldx,
                                                          const int64_t* __restrict__ g, int D,
                                                          int16_t* __restrict__ xq, int ldq, int32_t* __restrict__ xs) {
  extern __shared__ int64_t ys[];
  __shared__ uint64_t red[33];
  prefetch_gains(g, D);
  if (bias && threadIdx.x == 32 && !((uintptr_t)bias & 15)) prefetch_l2_bulk(bias, (uint32_t)D * 8);
  pdl_wait();
  pdl_launch_dependents();
  tpx_wait(x, sum_type, 1);
  const int r = blockIdx.x;
  const int which = sum_type == TPX_SUM_O ? 0 : 1;
  const int sh = tpx_shift(x, which, r);
  int64_t* row = xr + (size_t)r * ldx;
  for (int j = threadIdx.x; j < D; j += ROW_THREADS) {
    uint64_t tot = 0;
    for (int q = 0; q < x.size; ++q) tot += (uint64_t)ld_cg(tpx_sum_slot(x, x.rank, which, q) + (size_t)r * x.D + j);
    int64_t y = shr64((int64_t)tot, 28 - sh);
    if (bias) y = (int64_t)((uint64_t)y + (uint64_t)bias[j]);
    row[j] = (int64_t)((uint64_t)row[j] + (uint64_t)y);
  }
  __syncthreads();
  row_norm_q_any<ROW_THREADS>(row, g, D, xq + (size_t)r * ldq, xs + r, ys, red);
  tl_exit();
}

cudaError_t launch_tpx_norm(const TpX& x, int sum_type, const int64_t* bias, int64_t* xr, int ldx, const int64_t* g,
                            int R, int D, int16_t* xq, int ldq, int32_t* xs, cudaStream_t st, bool pdl) {
  if (R < 1 || R > TPX_ROWS || D != x.D || x.size < 2 || (sum_type != TPX_SUM_O && sum_type != TPX_SUM_D))
    return cudaErrorInvalidValue;
  const size_t smem = (size_t)D * 16;
  static DevOnce attr_set;   // raised once to the full budget, never lowered
  if (!attr_set.done()) {
    cudaError_t e = cudaFuncSetAttribute(k_tpx_norm, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e != cudaSuccess) return e;
    attr_set.set();
  }
  if (smem > 200 * 1024) return cudaErrorInvalidValue;
  void* args[] = {(void*)&x, (void*)&sum_type, (void*)&bias, (void*)&xr, (void*)&ldx, (void*)&g,
                  (void*)&D, (void*)&xq, (void*)&ldq, (void*)&xs};
  return launch_simple((const void*)k_tpx_norm, dim3(R), dim3(ROW_THREADS), smem, st, pdl, args);
}

// ---------------------------------------------------------------- qrow with a published row max
// xq = clip(shr(x, s)), s = max(bitlen(amax[r]) - 15, 0); grid (slices, R): every CTA converts a
// slice of a row, so a long row (e.g. the 18944-wide MLP activation) is converted in parallel.
__global__ void __launch_bounds__(256) k_quant_known(const int64_t* __restrict__ x, int ldx, int K,
                                                     const unsigned long long* __restrict__ amax,
                                                     int16_t* __restrict__ xq, int ldq, int32_t* __restrict__ xs,
                                                     uint8_t* __restrict__ dig, int dig_rows) {
  pdl_wait();
  pdl_launch_dependents();
  const int r = blockIdx.y;
  const int s = qrow_shift(__ldcg(amax + r));
  const int per = ((K + gridDim.x - 1) / gridDim.x + 1) & ~1;      // even slice length
  const int k0 = blockIdx.x * per, k1 = min(K, k0 + per);
  const longlong2* x2 = reinterpret_cast<const longlong2*>(x + (size_t)r * ldx);
  short2* q2 = reinterpret_cast<short2*>(xq + (size_t)r * ldq);
  for (int i = (k0 >> 1) + threadIdx.x; i < (k1 >> 1); i += 256) {
    const longlong2 v = __ldcg(x2 + i);
    const short2 q = make_short2(qrow_value(v.x, s), qrow_value(v.y, s));
    q2[i] = q;
    if (dig) { put_digits(dig, dig_rows, K, r, 2 * i, q.x); put_digits(dig, dig_rows, K, r, 2 * i + 1, q.y); }
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) xs[r] = s;
  tl_exit();
}

cudaError_t launch_quant_known(const int64_t* x, int ldx, int R, int K, const unsigned long long* amax, int16_t* xq,
                               int ldq, int32_t* xs, cudaStream_t st, bool pdl, uint8_t* dig, int dig_rows) {
  if ((K & 1) || (ldx & 1) || (ldq & 1)) return cudaErrorInvalidValue;
  int slices = (K + 2047) / 2048;
  void* args[] = {(void*)&x,   (void*)&ldx, (void*)&K,   (void*)&amax,    (void*)&xq,
                  (void*)&ldq, (void*)&xs,  (void*)&dig, (void*)&dig_rows};
  return launch_simple((const void*)k_quant_known, dim3(slices, R), dim3(256), 0, st, pdl, args);
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
  tl_exit();
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

// ---------------------------------------------------------------- head rows: requant + greedy argmax
// One CTA per activation row: y = QLin requant of the raw per-channel sums (drop rule of
// exact_llm.py:89-96), optional logits, next token = first index of the maximum (exact_llm.py:267).
__global__ void __launch_bounds__(ROW_THREADS) k_head_rows(const int64_t* __restrict__ acc, int ld, int N,
                                                           const int64_t* __restrict__ M, int mbits,
                                                           const int32_t* __restrict__ xs, int64_t* __restrict__ logits,
                                                           int ldl, int32_t* __restrict__ next) {
  __shared__ uint64_t red[33];
  __shared__ int64_t bv_s[ROW_THREADS / 32];
  __shared__ int bn_s[ROW_THREADS / 32];
  const int r = blockIdx.x;
  const int64_t* ar = acc + (size_t)r * ld;
  uint64_t m = 0;
  for (int i = threadIdx.x; i < N; i += ROW_THREADS) { const uint64_t v = uabs64(ar[i]); m = v > m ? v : m; }
  m = block_max_u64<ROW_THREADS>(m, red);
  int drop = bitlen64(m) + mbits - 62;
  drop = drop > 0 ? drop : 0;
  const int s = xs[r];
  int64_t bv = INT64_MIN;
  int bn = 0x7fffffff;
  for (int i = threadIdx.x; i < N; i += ROW_THREADS) {
    const int64_t y = shr64((int64_t)((uint64_t)shr64(ar[i], drop) * (uint64_t)M[i]), 28 - s - drop);
    if (logits) logits[(size_t)r * ldl + i] = y;
    if (y > bv) { bv = y; bn = i; }              // i increases: the first maximum is kept
  }
  for (int o = 16; o > 0; o >>= 1) {
    const int64_t ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int on = __shfl_xor_sync(0xffffffffu, bn, o);
    if (ov > bv || (ov == bv && on < bn)) { bv = ov; bn = on; }
  }
  if ((threadIdx.x & 31) == 0) { bv_s[threadIdx.x >> 5] = bv; bn_s[threadIdx.x >> 5] = bn; }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < ROW_THREADS / 32; ++w)
      if (bv_s[w] > bv || (bv_s[w] == bv && bn_s[w] < bn)) { bv = bv_s[w]; bn = bn_s[w]; }
    next[r] = bn;
  }
  tl_exit();
}

cudaError_t launch_head_rows(const int64_t* acc, int ld, int R, const LinW& L, const int32_t* xs, int64_t* logits,
                             int ldl, int32_t* next, cudaStream_t st) {
  k_head_rows<<<R, ROW_THREADS, 0, st>>>(acc, ld, L.N, L.Mc, L.mbits, xs, logits, ldl, next);
  return cudaGetLastError();
}

// ---------------------------------------------------------------- tensor parallel helpers
__global__ void k_tp_resid(const int64_t* __restrict__ tot, int N, const int32_t* __restrict__ xs,
                           const int64_t* __restrict__ b, int64_t* __restrict__ x, int ldx,
                           const unsigned long long* __restrict__ amax) {
  const int r = blockIdx.y;
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  if (n >= N) return;
  const int sh = amax ? qrow_shift(__ldcg(amax + r)) : xs[r];
  int64_t y = shr64(tot[(size_t)r * N + n], 28 - sh);
  if (b) y = (int64_t)((uint64_t)y + (uint64_t)b[n]);
  int64_t* o = x + (size_t)r * ldx + n;
  *o = (int64_t)((uint64_t)*o + (uint64_t)y);
}

cudaError_t launch_tp_resid(const int64_t* tot, int R, int N, const int32_t* xs, const int64_t* b, int64_t* x, int ldx,
                            cudaStream_t st, const unsigned long long* amax) {
  k_tp_resid<<<dim3((N + 255) / 256, R), 256, 0, st>>>(tot, N, xs, b, x, ldx, amax);
  return cudaGetLastError();
}

__global__ void k_tp_pick(const int64_t* val, const int64_t* gmax, int32_t* idx, int v0, int R) {
  const int r = threadIdx.x;
  if (r < R) idx[r] = val[r] == gmax[r] ? v0 + idx[r] : 0x7fffffff;
}

cudaError_t launch_tp_pick(const int64_t* val, const int64_t* gmax, int32_t* idx, int v0, int R, cudaStream_t st) {
  k_tp_pick<<<1, 32, 0, st>>>(val, gmax, idx, v0, R);
  return cudaGetLastError();
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
