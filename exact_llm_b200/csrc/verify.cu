// Weightless cell verifier on the GPU: batch replay of the reference's verify_cell.
//
// Reference semantics (novain-shibu/exact-llm, experiments/commit_audit_kaggle.py:647-705): a
// verifier that holds no weights -- only each linear's Freivalds digests d_p = W r_p mod p (over
// W * M for a group-128 linear), the scales, biases, norm gains, the integer tables and a digest of
// every embedding row -- checks one cell (layer L, position t) of a committed forward from the
// opened leaves: every leaf against the Merkle root, the embedding row digest (L = 0), each
// accumulator by its Freivalds identity, and the cell's own recomputation: k/v requant + RoPE equal
// to the committed K/V row, attention of the roped q over the committed K/V rows 0..t, o, the
// residual, the second norm, gate/up, SiLU, down and the next residual row.
//
// Work split: one thread per opened leaf hashes it (Hb) and walks its Merkle proof; then one CTA
// per cell replays the cell in order, stopping at the first failed check like the reference.
// Vectors of the cell live in an L2-resident scratch row; every reduction is a CTA reduction.
#include "common.cuh"
#include "exb_internal.h"
#include "gemvdev.cuh"
#include "rowdev.cuh"
#include "sha256.cuh"

namespace exb {

constexpr int VT = 512;

// ---------------------------------------------------------------- leaf proofs
__global__ void __launch_bounds__(128) k_verify_leaves(int n, const VLeafRec* __restrict__ recs,
                                                       const int64_t* __restrict__ values,
                                                       const uint8_t* __restrict__ proofs, int depth,
                                                       const uint8_t* __restrict__ root, int* __restrict__ ok) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const VLeafRec r = recs[i];
  Sha256 s;
  sha_init(s);
  int64_t off = r.voff;
  for (int j = 0; j < r.nseg; ++j) {
    sha_i64_array(s, values + off, r.len[j]);
    sha_byte(s, '|');
    off += r.len[j];
  }
  uint8_t h[32];
  sha_final(s, h);
  sha_init(s);                                  // leaf node: SHA-256("L" + leaf)
  sha_byte(s, 'L');
  for (int j = 0; j < 32; ++j) sha_byte(s, h[j]);
  sha_final(s, h);
  int64_t idx = r.leaf;
  const uint8_t* pr = proofs + r.poff;
  for (int lv = 0; lv < depth; ++lv) {          // parent: SHA-256("N" + left + right)
    sha_init(s);
    sha_byte(s, 'N');
    const uint8_t* sib = pr + 32 * lv;
    if ((idx & 1) == 0) {
      for (int j = 0; j < 32; ++j) sha_byte(s, h[j]);
      for (int j = 0; j < 32; ++j) sha_byte(s, sib[j]);
    } else {
      for (int j = 0; j < 32; ++j) sha_byte(s, sib[j]);
      for (int j = 0; j < 32; ++j) sha_byte(s, h[j]);
    }
    sha_final(s, h);
    idx >>= 1;
  }
  int same = 1;
  for (int j = 0; j < 32; ++j) same &= h[j] == root[j];
  ok[i] = same;
}

// ---------------------------------------------------------------- CTA helpers
EXB_DEV uint64_t vmax(uint64_t v, uint64_t* buf) { const uint64_t r = block_max_fast<VT>(v, buf); __syncthreads(); return r; }
EXB_DEV uint64_t vsum(uint64_t v, uint64_t* buf) { const uint64_t r = block_sum_fast<VT>(v, buf); __syncthreads(); return r; }

// Freivalds identity of one accumulator row: sum_n r_n (acc_n mod p) == sum_k d_k (xq_k mod p)
// (mod p) for both primes; a per-channel accumulator must also respect |acc| <= 127 * 32767 * K
EXB_DEV bool v_fr(const VLinDev& L, const int64_t* acc, const int16_t* xq, uint64_t* buf) {
  uint64_t m = 0;
  for (int n = threadIdx.x; n < L.N; n += VT) { const uint64_t u = uabs64(acc[n]); m = u > m ? u : m; }
  m = vmax(m, buf);
  if (!L.group && m > 127ull * 32767ull * (uint64_t)L.K) return false;
#pragma unroll
  for (int pi = 0; pi < 2; ++pi) {
    const unsigned long long p = fr_prime(pi);
    uint64_t a = 0, b = 0;
    for (int n = threadIdx.x; n < L.N; n += VT) a += mod_p(acc[n], p) * (uint64_t)L.r[pi * L.N + n] % p;
    for (int k = threadIdx.x; k < L.K; k += VT) b += mod_p(xq[k], p) * (uint64_t)L.d[pi * L.K + k] % p;
    a = vsum(a % p, buf) % p;        // per-thread sums stay below N * 2^31 < 2^63
    b = vsum(b % p, buf) % p;
    if (a != b) return false;
  }
  return true;
}

// requant of one accumulator row (group: shr(tot, 28 - s); per channel with the per-row drop rule)
EXB_DEV void v_rq(const VLinDev& L, const int64_t* acc, int s, int64_t* y, uint64_t* buf) {
  int drop = 0;
  if (!L.group) {
    uint64_t m = 0;
    for (int n = threadIdx.x; n < L.N; n += VT) { const uint64_t u = uabs64(acc[n]); m = u > m ? u : m; }
    m = vmax(m, buf);
    drop = bitlen64(m) + L.mbits - 62;
    drop = drop > 0 ? drop : 0;
  }
  for (int n = threadIdx.x; n < L.N; n += VT) {
    const int row = L.row0 + n * L.row_step;
    int64_t v = L.group ? shr64(acc[n], 28 - s)
                        : shr64((int64_t)((uint64_t)shr64(acc[n], drop) * (uint64_t)L.Mc[row]), 28 - s - drop);
    if (L.b) v = (int64_t)((uint64_t)v + (uint64_t)L.b[row]);
    y[n] = v;
  }
  __syncthreads();
}

// qrow of an int64 row (no norm): shift from the CTA max, int16 values
EXB_DEV int v_qrow(const int64_t* x, int n, int16_t* xq, uint64_t* buf) {
  uint64_t m = 0;
  for (int i = threadIdx.x; i < n; i += VT) { const uint64_t u = uabs64(x[i]); m = u > m ? u : m; }
  const int s = qrow_shift(vmax(m, buf));
  for (int i = threadIdx.x; i < n; i += VT) xq[i] = qrow_value(x[i], s);
  __syncthreads();
  return s;
}

// RoPE of `heads` rows of hd at position t: shr(x * cos + rot_half(x) * sin, 16) (exact_llm.py:157-160)
EXB_DEV void v_rope(const int64_t* x, int heads, int hd, const int32_t* cos_t, const int32_t* sin_t, int t, int64_t* y) {
  const int half = hd / 2;
  for (int i = threadIdx.x; i < heads * hd; i += VT) {
    const int h = i / hd, d = i - h * hd;
    const int64_t c = cos_t[(size_t)t * half + d % half], sn = sin_t[(size_t)t * half + d % half];
    const int64_t a = x[i];
    const int64_t rot = d < half ? (int64_t)(0ull - (uint64_t)x[h * hd + d + half]) : x[h * hd + d - half];
    y[i] = shr64((int64_t)((uint64_t)a * (uint64_t)c + (uint64_t)rot * (uint64_t)sn), 16);
  }
  __syncthreads();
}

// ---------------------------------------------------------------- one CTA per cell
__global__ void __launch_bounds__(VT) k_verify_cells(const VerifyArgs a) {
  extern __shared__ __align__(16) unsigned char vsm[];
  __shared__ uint64_t buf[2 * VT / 32 + 1];
  __shared__ int32_t sh_s;
  const int c = blockIdx.x, tid = threadIdx.x;
  const int L = a.cells[2 * c], t = a.cells[2 * c + 1];
  const int D = a.D, H = a.H, KV = a.KV, hd = a.hd, I = a.I;
  const int Hd = H * hd, KVd = KV * hd;
  int16_t* xq = reinterpret_cast<int16_t*>(vsm);                                 // max(D, Hd, I) int16
  int64_t* ys = reinterpret_cast<int64_t*>(vsm + (((size_t)a.q16_len * 2 + 15) & ~(size_t)15));   // norm staging
  int64_t* scr = a.scratch + (size_t)c * a.scr_len;
  int64_t* qo = scr;                 // Hd
  int64_t* att = qo + Hd;            // Hd
  int64_t* x2 = att + Hd;            // D
  int64_t* y1 = x2 + D;              // max(I, Hd, 2 KVd): requant output
  int64_t* y2 = y1 + a.ymax;         // max(I, KVd)
  int64_t* sc = y2 + a.ymax;         // H x T scores
  int verdict = 0;
  // ---- 1. every opened leaf against the root (the first failure names it)
  {
    int bad = 0x7fffffff;
    for (int j = a.cell_leaf0[c] + tid; j < a.cell_leaf0[c + 1]; j += VT)
      if (!a.leaf_ok[j]) bad = min(bad, j - a.cell_leaf0[c]);
    const uint64_t m = vmax((uint64_t)(0x7fffffff - bad), buf);
    if (m) { verdict = VERDICT_MERKLE + (int)(0x7fffffff - m); goto done; }
  }
  {
    const int64_t* v = a.values + a.cell_voff[c];
    if (L == a.NL) {                 // head cell: X(NL, t) | head acc
      const int64_t* x = v;
      const int64_t* hacc = x + D;
      row_norm_q_any<VT>(x, a.gf, D, xq, &sh_s, ys, buf);
      __syncthreads();
      if (!v_fr(a.lins[7 * a.NL], hacc, xq, buf)) verdict = VERDICT_HEAD;
      goto done;
    }
    const VLinDev* Ln = a.lins + 7 * L;              // q k v o gate up down
    const int64_t* x = v;
    const int64_t* kacc = x + D;
    const int64_t* vacc = kacc + KVd;
    const int64_t* kr = vacc + KVd;                  // (t + 1) x (K | V rows)
    const int64_t* qacc = kr + (size_t)(t + 1) * 2 * KVd;
    const int64_t* oacc = qacc + Hd;
    const int64_t* gacc = oacc + D;
    const int64_t* uacc = gacc + I;
    const int64_t* dacc = uacc + I;
    const int64_t* xnext = dacc + D;
    // ---- 2. embedding row digest (layer 0)
    if (L == 0) {
      const int tok = a.ids[t];
      for (int pi = 0; pi < 2; ++pi) {
        const unsigned long long p = fr_prime(pi);
        uint64_t s = 0;
        for (int i = tid; i < D; i += VT) s += mod_p(x[i], p) * (uint64_t)a.emb_r[pi * D + i] % p;
        s = vsum(s % p, buf) % p;
        if (s != (uint64_t)a.emb_de[(size_t)pi * a.V + tok]) { verdict = VERDICT_EMB; goto done; }
      }
    }
    // ---- 3. k / v: Freivalds, requant + RoPE against the committed row
    row_norm_q_any<VT>(x, a.g1[L], D, xq, &sh_s, ys, buf);
    __syncthreads();
    const int sh = sh_s;
    if (!v_fr(Ln[1], kacc, xq, buf) || !v_fr(Ln[2], vacc, xq, buf)) { verdict = VERDICT_KV; goto done; }
    v_rq(Ln[1], kacc, sh, y1, buf);
    v_rq(Ln[2], vacc, sh, y2, buf);
    v_rope(y1, KV, hd, a.cos_t, a.sin_t, t, att);
    {
      const int64_t* krt = kr + (size_t)t * 2 * KVd;
      int diff = 0;
      for (int i = tid; i < KVd; i += VT) diff |= (att[i] != krt[i]) | (y2[i] != krt[KVd + i]);
      if (vmax((uint64_t)diff, buf)) { verdict = VERDICT_KR; goto done; }
    }
    // ---- 4. q: Freivalds, requant + RoPE
    if (!v_fr(Ln[0], qacc, xq, buf)) { verdict = VERDICT_Q; goto done; }
    v_rq(Ln[0], qacc, sh, y1, buf);
    v_rope(y1, H, hd, a.cos_t, a.sin_t, t, qo);
    // ---- 5. attention over the committed K/V rows 0..t: one warp per head
    {
      const int warp = tid >> 5, lane = tid & 31, rep = H / KV;
      for (int hh = warp; hh < H; hh += VT / 32) {
        const int kh = hh / rep;
        int64_t* srow = sc + (size_t)hh * a.T;
        uint64_t m = 0;
        for (int d = lane; d < hd; d += 32) { const uint64_t u = uabs64(qo[hh * hd + d]); m = u > m ? u : m; }
        const int sq = qrow_shift(warp_max_u64(m));
        int64_t smax = INT64_MIN;
        for (int s = 0; s <= t; ++s) {
          const int64_t* krow = kr + (size_t)s * 2 * KVd + (size_t)kh * hd;
          uint64_t km = 0;
          for (int d = lane; d < hd; d += 32) { const uint64_t u = uabs64(krow[d]); km = u > km ? u : km; }
          const int sk = qrow_shift(warp_max_u64(km));
          int64_t dot = 0;
          for (int d = lane; d < hd; d += 32)
            dot += (int64_t)qrow_value(qo[hh * hd + d], sq) * (int64_t)qrow_value(krow[d], sk);
          dot = (int64_t)warp_sum_u64((uint64_t)dot);
          const int64_t scv = shr64((int64_t)((uint64_t)dot * (uint64_t)a.inv), 32 - sq - sk);
          if (lane == 0) srow[s] = scv;
          smax = scv > smax ? scv : smax;
        }
        __syncwarp();
        int64_t es = 0;
        for (int s = lane; s <= t; s += 32) { const int64_t e = exp_lookup(a.exp_t, smax - srow[s]); srow[s] = e; es += e; }
        es = (int64_t)warp_sum_u64((uint64_t)es);
        __syncwarp();
        for (int s = lane; s <= t; s += 32) srow[s] = (int64_t)(((uint64_t)srow[s] << 20) / (uint64_t)es);
        __syncwarp();
        for (int d = lane; d < hd; d += 32) {
          int64_t acc = 0;
          for (int s = 0; s <= t; ++s) acc += srow[s] * kr[(size_t)s * 2 * KVd + KVd + (size_t)kh * hd + d];
          att[hh * hd + d] = shr64(acc, 20);
        }
      }
      __syncthreads();
    }
    // ---- 6. o, residual
    {
      const int so = v_qrow(att, Hd, xq, buf);
      if (!v_fr(Ln[3], oacc, xq, buf)) { verdict = VERDICT_O; goto done; }
      v_rq(Ln[3], oacc, so, y1, buf);
      for (int i = tid; i < D; i += VT) x2[i] = (int64_t)((uint64_t)x[i] + (uint64_t)y1[i]);
      __syncthreads();
    }
    // ---- 7. gate / up, SiLU, down, next residual row
    row_norm_q_any<VT>(x2, a.g2[L], D, xq, &sh_s, ys, buf);
    __syncthreads();
    {
      const int sm = sh_s;
      if (!v_fr(Ln[4], gacc, xq, buf) || !v_fr(Ln[5], uacc, xq, buf)) { verdict = VERDICT_GU; goto done; }
      v_rq(Ln[4], gacc, sm, y1, buf);
      v_rq(Ln[5], uacc, sm, y2, buf);
      for (int i = tid; i < I; i += VT)
        y1[i] = shr64((int64_t)((uint64_t)isilu_dev(a.silu_t, y1[i]) * (uint64_t)y2[i]), 16);
      __syncthreads();
      const int sd = v_qrow(y1, I, xq, buf);
      if (!v_fr(Ln[6], dacc, xq, buf)) { verdict = VERDICT_DOWN; goto done; }
      v_rq(Ln[6], dacc, sd, y2, buf);
      int diff = 0;
      for (int i = tid; i < D; i += VT) diff |= (int64_t)((uint64_t)x2[i] + (uint64_t)y2[i]) != xnext[i];
      if (vmax((uint64_t)diff, buf)) verdict = VERDICT_RESID;
    }
  }
done:
  if (tid == 0) a.verdict[c] = verdict;
}

// ---------------------------------------------------------------- embedding digests
__global__ void __launch_bounds__(256) k_emb_digest(const int8_t* __restrict__ emb, int shift,
                                                    const int64_t* __restrict__ emb_q16, int V, int D,
                                                    const int32_t* __restrict__ r, int64_t* __restrict__ de) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= V) return;
  for (int pi = 0; pi < 2; ++pi) {
    const unsigned long long p = fr_prime(pi);
    uint64_t s = 0;
    for (int i = lane; i < D; i += 32) {
      const int64_t x = emb_q16 ? emb_q16[(size_t)warp * D + i] : ((int64_t)emb[(size_t)warp * D + i] << shift);
      s += mod_p(x, p) * (uint64_t)r[pi * D + i] % p;
    }
    s = warp_sum_u64(s % p) % p;
    if (lane == 0) de[(size_t)pi * V + warp] = (int64_t)s;
  }
}

cudaError_t launch_emb_digest(const int8_t* emb, int shift, const int64_t* emb_q16, int V, int D, const int32_t* r,
                              int64_t* de, cudaStream_t st) {
  k_emb_digest<<<(unsigned)(((int64_t)V * 32 + 255) / 256), 256, 0, st>>>(emb, shift, emb_q16, V, D, r, de);
  return cudaGetLastError();
}

cudaError_t launch_verify(const VerifyArgs& a, int n_cells, int n_leaves, const VLeafRec* recs, const uint8_t* proofs,
                          int depth, const uint8_t* root, int* leaf_ok, cudaStream_t st) {
  if (n_leaves > 0) {
    k_verify_leaves<<<(n_leaves + 127) / 128, 128, 0, st>>>(n_leaves, recs, a.values, proofs, depth, root, leaf_ok);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  const size_t smem = (((size_t)a.q16_len * 2 + 15) & ~(size_t)15) + (size_t)a.D * 16;
  static DevOnce attr;
  if (!attr.done()) {
    cudaError_t e = cudaFuncSetAttribute(k_verify_cells, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e != cudaSuccess) return e;
    attr.set();
  }
  if (smem > 200 * 1024) return cudaErrorInvalidValue;
  k_verify_cells<<<n_cells, VT, smem, st>>>(a);
  return cudaGetLastError();
}

}  // namespace exb
