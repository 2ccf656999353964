// Integer sampler on the GPU: seeded, temperature-scaled token choice from a Q16 logits row.
//
// Reference semantics (novain-shibu/exact-llm, exact_llm.py):
//   splitmix64(seed, pos), u20 = splitmix64 >> 44                       :243-248
//   y = shr(lg * tnum, 16), tnum = round(2^16 / temperature)            :249, 257
//   isoftmax_row: d = max(y) - y, e = exp table at d (0 from 40 on),
//                 p = (e << 20) // sum(e)                               :250-255
//   token = searchsorted(cumsum(p), (u20 * sum(p)) >> 20, "right")      :256-259
// One CTA per row: the row's max and exp-sum by block reductions, then per-thread sums of p over
// contiguous slices, an exclusive block scan of those sums, and the one thread whose slice holds
// the target finds the first index whose running sum exceeds it.  Every quantity is an integer,
// so the order of the sums changes no bit.
#include "common.cuh"
#include "exb_internal.h"

namespace exb {

constexpr int SMP_THREADS = 1024;

EXB_DEV uint64_t splitmix64_dev(uint64_t seed, uint64_t pos) {
  uint64_t z = seed + (pos + 1) * 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

EXB_DEV int64_t block_max_i64(int64_t v, int64_t* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const int64_t w = __shfl_xor_sync(0xffffffffu, v, o);
    v = w > v ? w : v;
  }
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  int64_t m = red[0];
  for (int i = 1; i < SMP_THREADS / 32; ++i) m = red[i] > m ? red[i] : m;
  return m;
}

EXB_DEV int64_t block_sum_i64(int64_t v, int64_t* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  int64_t s = 0;
  for (int i = 0; i < SMP_THREADS / 32; ++i) s += red[i];
  return s;
}

__global__ void __launch_bounds__(SMP_THREADS) k_sample(const int64_t* __restrict__ lg, int V, int64_t ld,
                                                        const unsigned long long* __restrict__ seeds,
                                                        int32_t* __restrict__ pos, int pos_inc, int64_t tnum,
                                                        const int32_t* __restrict__ exp_t, int32_t* __restrict__ tokens) {
  __shared__ int64_t red[SMP_THREADS / 32];
  __shared__ int64_t scan[SMP_THREADS];
  __shared__ int tok_sh;
  pdl_wait();
  const int r = blockIdx.x, tid = threadIdx.x;
  const int64_t* row = lg + (int64_t)r * ld;
  const int c0 = (int)((int64_t)V * tid / SMP_THREADS), c1 = (int)((int64_t)V * (tid + 1) / SMP_THREADS);
  auto y_at = [&](int i) { return shr64((int64_t)((uint64_t)__ldcg(reinterpret_cast<const long long*>(row + i)) *
                                                  (uint64_t)tnum), 16); };
  int64_t m = INT64_MIN;
  for (int i = c0; i < c1; ++i) { const int64_t y = y_at(i); m = y > m ? y : m; }
  m = block_max_i64(m, red);
  int64_t s = 0;
  for (int i = c0; i < c1; ++i) s += exp_lookup(exp_t, m - y_at(i));
  const uint64_t S = (uint64_t)block_sum_i64(s, red);        // >= 2^24 (the maximum's own term)
  int64_t ps = 0;
  for (int i = c0; i < c1; ++i) ps += (int64_t)(((uint64_t)exp_lookup(exp_t, m - y_at(i)) << 20) / S);
  // exclusive scan of the per-thread sums (Hillis-Steele over the block)
  scan[tid] = ps;
  __syncthreads();
  for (int o = 1; o < SMP_THREADS; o <<= 1) {
    const int64_t add = tid >= o ? scan[tid - o] : 0;
    __syncthreads();
    scan[tid] += add;
    __syncthreads();
  }
  const int64_t total = scan[SMP_THREADS - 1];
  const int64_t before = scan[tid] - ps;
  const int p0 = pos[r];
  const uint64_t u = splitmix64_dev(seeds[r], (uint64_t)(int64_t)p0) >> 44;
  const int64_t target = (int64_t)((u * (uint64_t)total) >> 20);
  if (tid == 0) tok_sh = V - 1;
  __syncthreads();
  if (before <= target && target < before + ps) {
    int64_t cum = before;
    for (int i = c0; i < c1; ++i) {
      cum += (int64_t)(((uint64_t)exp_lookup(exp_t, m - y_at(i)) << 20) / S);
      if (cum > target) { tok_sh = i; break; }
    }
  }
  __syncthreads();
  pdl_launch_dependents();
  if (tid == 0) {
    tokens[r] = tok_sh;
    if (pos_inc) pos[r] = p0 + 1;
  }
}

cudaError_t launch_sample(int R, const int64_t* logits, int V, int64_t ld, const unsigned long long* seeds, int32_t* pos,
                          bool pos_inc, int64_t tnum, const int32_t* exp_t, int32_t* tokens, cudaStream_t st, bool pdl) {
  if (R < 1 || V < 1 || ld < V || !logits || !seeds || !pos || !exp_t || !tokens) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(R);
  cfg.blockDim = dim3(SMP_THREADS);
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, k_sample, logits, V, ld, seeds, pos, pos_inc ? 1 : 0, tnum, exp_t, tokens);
}

}  // namespace exb
