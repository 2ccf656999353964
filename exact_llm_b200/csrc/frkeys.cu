// K12: Freivalds key build on the device.
//
// For a linear with integer weights W (N, K) and group-128 scales M (N, K/128), the verifier key
// of the reference (experiments/gpu_engine_trace_verify_kaggle.py:803-819) is
//     d_p[k] = sum_n r_p[n] * (W[n, k] * M[n, k/128] mod p)  mod p,   p in {2^31-1, 2147483629},
// (per-channel linears: M = 1, keys_channel).  One pass over the weights in HBM: threads own
// columns k (coalesced along a weight row), the row range is split over grid.y, partial sums of
// residues (< 2^31 each) are added into a 64-bit accumulator and reduced mod p at the end.
#include "common.cuh"
#include "exb_internal.h"

namespace exb {

__global__ void k_fr_keys_acc(const int8_t* __restrict__ w, const int32_t* __restrict__ Mg, int ldm, int N, int K, int row0,
                              int row_step, const int32_t* __restrict__ r, unsigned long long* __restrict__ acc) {
  const int k = blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= K) return;
  const int i0 = (int)((int64_t)N * blockIdx.y / gridDim.y), i1 = (int)((int64_t)N * (blockIdx.y + 1) / gridDim.y);
  unsigned long long s0 = 0, s1 = 0;
  for (int i = i0; i < i1; ++i) {
    const size_t row = (size_t)row0 + (size_t)i * row_step;
    int64_t wm = w[row * K + k];
    if (Mg) wm *= Mg[row * ldm + (k >> 7)];
    int64_t m0 = wm % (int64_t)fr_prime(0); if (m0 < 0) m0 += fr_prime(0);
    int64_t m1 = wm % (int64_t)fr_prime(1); if (m1 < 0) m1 += fr_prime(1);
    s0 += (unsigned long long)m0 * (unsigned long long)r[i] % fr_prime(0);
    s1 += (unsigned long long)m1 * (unsigned long long)r[N + i] % fr_prime(1);
  }
  atomicAdd(acc + k, s0);
  atomicAdd(acc + K + k, s1);
}

__global__ void k_fr_keys_fin(const unsigned long long* __restrict__ acc, int K, int32_t* __restrict__ d) {
  const int k = blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= K) return;
  d[k] = (int32_t)(acc[k] % fr_prime(0));
  d[K + k] = (int32_t)(acc[K + k] % fr_prime(1));
}

// r: (2, N) int32 in [0, p); d: (2, K) int32 out.  Rows of the logical linear are fused rows
// row0 + i*row_step of the (fused) weight matrix w with K columns.
cudaError_t launch_fr_keys(const int8_t* w, const int32_t* Mg, int ldm, int N, int K, int row0, int row_step,
                           const int32_t* r, int32_t* d, cudaStream_t st) {
  unsigned long long* acc = nullptr;
  cudaError_t e = cudaMallocAsync(&acc, sizeof(unsigned long long) * 2 * K, st);
  if (e != cudaSuccess) return e;
  cudaMemsetAsync(acc, 0, sizeof(unsigned long long) * 2 * K, st);
  int ysplit = N / 256;
  ysplit = ysplit < 1 ? 1 : (ysplit > 64 ? 64 : ysplit);
  dim3 grid((K + 255) / 256, ysplit);
  k_fr_keys_acc<<<grid, 256, 0, st>>>(w, Mg, ldm, N, K, row0, row_step, r, acc);
  k_fr_keys_fin<<<(K + 255) / 256, 256, 0, st>>>(acc, K, d);
  e = cudaGetLastError();
  cudaFreeAsync(acc, st);
  return e;
}

}  // namespace exb
