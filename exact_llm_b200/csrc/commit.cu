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
#include "sha256.cuh"

namespace exb {

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
    sha_i64_array(s, base + off[j], len[j]);
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
