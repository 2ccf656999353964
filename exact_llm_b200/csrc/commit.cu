// Merkle trace commitment on the GPU (the reference hashes its traces on the host).
//
// Reference semantics (novain-shibu/exact-llm, experiments/commit_audit_kaggle.py):
//   Hb(*arrs)      SHA-256 over each int64 array's little-endian bytes, each followed by "|"  :567-570
//   merkle(leaves) leaf node SHA-256("L" + leaf), parent SHA-256("N" + left + right), an odd
//                  last node paired with itself                                               :571-575
//   leaves_of      X of every (layer 0..NL, position); per (layer, position) the k|v
//                  accumulators, the roped K|V rows, the q accumulator, the o|gate|up|down
//                  accumulators; the head accumulator per position                            :614-628
//
// Layout on the device: every committed position owns one row of the commitment log = the
// step's trace row (every linear's accumulator, in the order L0.q, L0.k, ..., head) followed by
// the captured residual rows X[0..NL] (D each) and the roped K|V rows of every layer (2 KV hd).
// One thread hashes one leaf (SHA-256 is sequential within a message; leaves are independent),
// then one thread per node builds each Merkle level.  SHA-256 follows FIPS 180-4.
#include "common.cuh"
#include "exb_internal.h"

namespace exb {

__constant__ uint32_t SHA_K[64] = {
    0x428a2f98u, 0x71374491u, 0xb5c0fbcfu, 0xe9b5dba5u, 0x3956c25bu, 0x59f111f1u, 0x923f82a4u, 0xab1c5ed5u,
    0xd807aa98u, 0x12835b01u, 0x243185beu, 0x550c7dc3u, 0x72be5d74u, 0x80deb1feu, 0x9bdc06a7u, 0xc19bf174u,
    0xe49b69c1u, 0xefbe4786u, 0x0fc19dc6u, 0x240ca1ccu, 0x2de92c6fu, 0x4a7484aau, 0x5cb0a9dcu, 0x76f988dau,
    0x983e5152u, 0xa831c66du, 0xb00327c8u, 0xbf597fc7u, 0xc6e00bf3u, 0xd5a79147u, 0x06ca6351u, 0x14292967u,
    0x27b70a85u, 0x2e1b2138u, 0x4d2c6dfcu, 0x53380d13u, 0x650a7354u, 0x766a0abbu, 0x81c2c92eu, 0x92722c85u,
    0xa2bfe8a1u, 0xa81a664bu, 0xc24b8b70u, 0xc76c51a3u, 0xd192e819u, 0xd6990624u, 0xf40e3585u, 0x106aa070u,
    0x19a4c116u, 0x1e376c08u, 0x2748774cu, 0x34b0bcb5u, 0x391c0cb3u, 0x4ed8aa4au, 0x5b9cca4fu, 0x682e6ff3u,
    0x748f82eeu, 0x78a5636fu, 0x84c87814u, 0x8cc70208u, 0x90befffau, 0xa4506cebu, 0xbef9a3f7u, 0xc67178f2u};

EXB_DEV uint32_t rotr(uint32_t x, int n) { return __funnelshift_r(x, x, n); }

struct Sha256 {
  uint32_t h[8];
  uint32_t w[16];       // the block being filled, big-endian words
  uint32_t nb;          // bytes in the block
  uint64_t total;       // message bytes so far
};

EXB_DEV void sha_init(Sha256& s) {
  const uint32_t iv[8] = {0x6a09e667u, 0xbb67ae85u, 0x3c6ef372u, 0xa54ff53au,
                          0x510e527fu, 0x9b05688cu, 0x1f83d9abu, 0x5be0cd19u};
#pragma unroll
  for (int i = 0; i < 8; ++i) s.h[i] = iv[i];
#pragma unroll
  for (int i = 0; i < 16; ++i) s.w[i] = 0;
  s.nb = 0;
  s.total = 0;
}

EXB_DEV void sha_compress(uint32_t h[8], uint32_t w[16]) {
  uint32_t a = h[0], b = h[1], c = h[2], d = h[3], e = h[4], f = h[5], g = h[6], hh = h[7];
#pragma unroll
  for (int t = 0; t < 64; ++t) {
    uint32_t wt;
    if (t < 16) {
      wt = w[t];
    } else {   // message schedule kept in the 16-word circular window
      const uint32_t w15 = w[(t - 15) & 15], w2 = w[(t - 2) & 15];
      const uint32_t s0 = rotr(w15, 7) ^ rotr(w15, 18) ^ (w15 >> 3);
      const uint32_t s1 = rotr(w2, 17) ^ rotr(w2, 19) ^ (w2 >> 10);
      wt = w[t & 15] + s0 + w[(t - 7) & 15] + s1;
      w[t & 15] = wt;
    }
    const uint32_t S1 = rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25);
    const uint32_t ch = (e & f) ^ (~e & g);
    const uint32_t t1 = hh + S1 + ch + SHA_K[t] + wt;
    const uint32_t S0 = rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22);
    const uint32_t mj = (a & b) ^ (a & c) ^ (b & c);
    const uint32_t t2 = S0 + mj;
    hh = g; g = f; f = e; e = d + t1; d = c; c = b; b = a; a = t1 + t2;
  }
  h[0] += a; h[1] += b; h[2] += c; h[3] += d; h[4] += e; h[5] += f; h[6] += g; h[7] += hh;
}

EXB_DEV void sha_block_done(Sha256& s) {
  sha_compress(s.h, s.w);
#pragma unroll
  for (int i = 0; i < 16; ++i) s.w[i] = 0;
  s.nb = 0;
}

EXB_DEV void sha_byte(Sha256& s, uint32_t byte) {
  s.w[s.nb >> 2] |= (byte & 0xffu) << (24 - 8 * (s.nb & 3));
  s.total += 1;
  if (++s.nb == 64) sha_block_done(s);
}

// eight bytes of an int64 in little-endian order (numpy's tobytes())
EXB_DEV void sha_i64(Sha256& s, uint64_t v) {
  if (s.nb + 8 <= 64) {
    const uint64_t be = ((uint64_t)__byte_perm((uint32_t)v, 0, 0x0123) << 32) | __byte_perm((uint32_t)(v >> 32), 0, 0x0123);
    const uint32_t hi = (uint32_t)(be >> 32), lo = (uint32_t)be;
    const int o = (int)(s.nb & 3), wi = (int)(s.nb >> 2);
    if (o == 0) {
      s.w[wi] = hi;
      s.w[wi + 1] = lo;
    } else {
      s.w[wi] |= hi >> (8 * o);
      s.w[wi + 1] = __funnelshift_r(lo, hi, 8 * o);
      s.w[wi + 2] = lo << (32 - 8 * o);
    }
    s.total += 8;
    s.nb += 8;
    if (s.nb == 64) sha_block_done(s);
  } else {
    for (int i = 0; i < 8; ++i) sha_byte(s, (uint32_t)(v >> (8 * i)));
  }
}

EXB_DEV void sha_final(Sha256& s, uint8_t* out) {
  const uint64_t bits = s.total * 8;
  sha_byte(s, 0x80u);
  s.total -= 1;                                   // padding is not message
  while (s.nb != 56) { sha_byte(s, 0u); s.total -= 1; }
  s.w[14] = (uint32_t)(bits >> 32);
  s.w[15] = (uint32_t)bits;
  sha_compress(s.h, s.w);
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) out[4 * i + j] = (uint8_t)(s.h[i] >> (24 - 8 * j));
}

// ---------------------------------------------------------------- step capture -> commitment log
__global__ void __launch_bounds__(256) k_commit_log(int R, const int32_t* __restrict__ row_seq,
                                                    const int32_t* __restrict__ row_pos, int seq,
                                                    const int64_t* __restrict__ trace, int64_t trace_row,
                                                    const int64_t* __restrict__ cap, int64_t cap_row,
                                                    int64_t* __restrict__ log, int npos_cap, int* npos, int* err) {
  const int r = blockIdx.y;
  if (r >= R || row_seq[r] != seq) return;
  const int pos = row_pos[r];
  if (pos < 0 || pos >= npos_cap) {
    if (blockIdx.x == 0 && threadIdx.x == 0) set_err(err, ERR_BOUNDS);
    return;
  }
  const int64_t row = trace_row + cap_row;
  int64_t* dst = log + (int64_t)pos * row;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < trace_row; i += stride)
    dst[i] = trace[(int64_t)r * trace_row + i];
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < cap_row; i += stride)
    dst[trace_row + i] = cap[(int64_t)r * cap_row + i];
  if (blockIdx.x == 0 && threadIdx.x == 0) atomicMax(npos, pos + 1);
}

cudaError_t launch_commit_log(int R, const int32_t* row_seq, const int32_t* row_pos, int seq, const int64_t* trace,
                              int64_t trace_row, const int64_t* cap, int64_t cap_row, int64_t* log, int npos_cap,
                              int* npos, int* err, cudaStream_t st) {
  const int64_t row = trace_row + cap_row;
  int blocks = (int)std::min<int64_t>(256, (row + 1023) / 1024);
  if (blocks < 1) blocks = 1;
  k_commit_log<<<dim3(blocks, R), 256, 0, st>>>(R, row_seq, row_pos, seq, trace, trace_row, cap, cap_row, log,
                                                npos_cap, npos, err);
  return cudaGetLastError();
}

// ---------------------------------------------------------------- leaves in the reference order
// leaf -> up to four (offset within the log row, length) int64 segments
EXB_DEV int leaf_segments(const CommitLayout& c, int64_t idx, int T, int& t, int64_t off[4], int64_t len[4]) {
  const int NL = c.NL;
  const int64_t nx = (int64_t)(NL + 1) * T;
  if (idx < nx) {                                               // X (layer L, position t)
    const int L = (int)(idx / T);
    t = (int)(idx % T);
    off[0] = c.x_off + (int64_t)L * c.D; len[0] = c.D;
    return 1;
  }
  idx -= nx;
  if (idx < (int64_t)4 * NL * T) {
    const int L = (int)(idx / (4 * (int64_t)T));
    const int64_t rem = idx % (4 * (int64_t)T);
    t = (int)(rem / 4);
    const int kind = (int)(rem % 4);
    const int b = 7 * L;
    if (kind == 0) {                                            // k | v accumulators
      off[0] = c.lin_off[b + 1]; len[0] = c.lin_len[b + 1];
      off[1] = c.lin_off[b + 2]; len[1] = c.lin_len[b + 2];
      return 2;
    }
    if (kind == 1) {                                            // roped K | V rows
      const int64_t kv = (int64_t)c.KV * c.hd;
      off[0] = c.kr_off + (int64_t)L * 2 * kv; len[0] = kv;
      off[1] = off[0] + kv; len[1] = kv;
      return 2;
    }
    if (kind == 2) {                                            // q accumulator
      off[0] = c.lin_off[b]; len[0] = c.lin_len[b];
      return 1;
    }
    for (int j = 0; j < 4; ++j) { off[j] = c.lin_off[b + 3 + j]; len[j] = c.lin_len[b + 3 + j]; }   // o gate up down
    return 4;
  }
  t = (int)(idx - (int64_t)4 * NL * T);                         // head
  off[0] = c.lin_off[7 * NL]; len[0] = c.lin_len[7 * NL];
  return 1;
}

__global__ void __launch_bounds__(128) k_commit_leaves(const int64_t* __restrict__ log, int64_t row, int T,
                                                       const CommitLayout c, int64_t n, uint8_t* __restrict__ out) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= n) return;
  int t = 0;
  int64_t off[4], len[4];
  const int ns = leaf_segments(c, idx, T, t, off, len);
  const int64_t* base = log + (int64_t)t * row;
  Sha256 s;
  sha_init(s);
  for (int j = 0; j < ns; ++j) {
    const int64_t* p = base + off[j];
    for (int64_t i = 0; i < len[j]; ++i) sha_i64(s, (uint64_t)__ldg(reinterpret_cast<const long long*>(p + i)));
    sha_byte(s, '|');
  }
  sha_final(s, out + idx * 32);
}

// level 0: SHA-256("L" + leaf); level k: SHA-256("N" + left + right), the odd last node twice
__global__ void __launch_bounds__(128) k_merkle_level(const uint8_t* __restrict__ in, int64_t n, int leaf_level,
                                                      uint8_t* __restrict__ out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t nout = leaf_level ? n : (n + 1) / 2;
  if (i >= nout) return;
  Sha256 s;
  sha_init(s);
  if (leaf_level) {
    sha_byte(s, 'L');
    for (int j = 0; j < 32; ++j) sha_byte(s, in[i * 32 + j]);
  } else {
    const int64_t l = 2 * i, r = 2 * i + 1 < n ? 2 * i + 1 : 2 * i;
    sha_byte(s, 'N');
    for (int j = 0; j < 32; ++j) sha_byte(s, in[l * 32 + j]);
    for (int j = 0; j < 32; ++j) sha_byte(s, in[r * 32 + j]);
  }
  sha_final(s, out + i * 32);
}

cudaError_t commit_root(const int64_t* log, int64_t row, int T, const CommitLayout& c, uint8_t* leaves,
                        uint8_t* lv_a, uint8_t* lv_b, uint8_t** root_dev, cudaStream_t st) {
  const int64_t n = commit_leaf_count(c.NL, T);
  if (n <= 0) return cudaErrorInvalidValue;
  k_commit_leaves<<<(unsigned)((n + 127) / 128), 128, 0, st>>>(log, row, T, c, n, leaves);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  k_merkle_level<<<(unsigned)((n + 127) / 128), 128, 0, st>>>(leaves, n, 1, lv_a);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  int64_t cur = n;
  uint8_t *src = lv_a, *dst = lv_b;
  while (cur > 1) {
    const int64_t nxt = (cur + 1) / 2;
    k_merkle_level<<<(unsigned)((nxt + 127) / 128), 128, 0, st>>>(src, cur, 0, dst);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    cur = nxt;
    uint8_t* tmp = src; src = dst; dst = tmp;
  }
  *root_dev = src;
  return cudaSuccess;
}

}  // namespace exb
