// Seeded synthetic integer tensors generated on the device.
//
// Each element is a pure function of (seed, stream, index):
//   h = mix64(mix64(seed*G + stream) + (i+1)*G),  G = 0x9E3779B97F4A7C15,
//   mix64 = the splitmix64 finaliser (Steele, Lea & Flood, 2014).
// int8 weight  = clip(shr(a+b+c-98302, 10), -127, 127)   (a,b,c: low three 16-bit fields of h)
// scale        = (2^23 // isqrt(K)) + (h & 1023)
// bias (Q16)   = (h & 0x7FFF) - 16384
// gain (Q16)   = 65536 + shr(a+b+c-98302, 2)
// The host-side numpy twin in the test oracle produces the same integers, so models of any
// size can be built directly in HBM and checked against the oracle on a slice.
#include "common.cuh"
#include "exb_internal.h"

namespace exb {

static constexpr uint64_t G64 = 0x9E3779B97F4A7C15ull;

EXB_DEV uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
EXB_DEV int64_t tri16(uint64_t h) {
  return (int64_t)(h & 0xFFFF) + (int64_t)((h >> 16) & 0xFFFF) + (int64_t)((h >> 32) & 0xFFFF) - 98302;
}

__global__ void k_gen(int kind, uint64_t seed, uint64_t stream, int64_t n, int64_t base_scale, void* out) {
  const uint64_t base = mix64(seed * G64 + stream);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    uint64_t h = mix64(base + (uint64_t)(i + 1) * G64);
    switch (kind) {
      case GEN_WEIGHT: {
        int64_t v = (tri16(h) + 512) >> 10;
        v = v > 127 ? 127 : (v < -127 ? -127 : v);
        static_cast<int8_t*>(out)[i] = (int8_t)v;
        break;
      }
      case GEN_SCALE32: static_cast<int32_t*>(out)[i] = (int32_t)(base_scale + (int64_t)(h & 1023)); break;
      case GEN_SCALE64: static_cast<int64_t*>(out)[i] = base_scale + (int64_t)(h & 1023); break;
      case GEN_BIAS: static_cast<int64_t*>(out)[i] = (int64_t)(h & 0x7FFF) - 16384; break;
      case GEN_GAIN: static_cast<int64_t*>(out)[i] = 65536 + ((tri16(h) + 2) >> 2); break;
      default: break;
    }
  }
}

int64_t isqrt_host(int64_t n) {
  int64_t r = 0;
  while ((r + 1) * (r + 1) <= n) ++r;
  return r;
}

cudaError_t gen_tensor(int kind, uint64_t seed, uint64_t stream, int64_t n, int64_t K, void* out, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  int64_t base = K > 0 ? (int64_t(1) << 23) / isqrt_host(K) : 0;
  int64_t blocks = (n + 255) / 256;
  if (blocks > 148 * 32) blocks = 148 * 32;
  k_gen<<<(int)blocks, 256, 0, st>>>(kind, seed, stream, n, base, out);
  return cudaGetLastError();
}

}  // namespace exb
