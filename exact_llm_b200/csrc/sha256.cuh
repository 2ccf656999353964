// SHA-256 (FIPS 180-4) for one message per thread: state and block buffer per thread, int64
// little-endian words fed 8 bytes at a time where the block offset allows, bytes otherwise.
// Used by the trace commitment (csrc/commit.cu) and the cell verifier (csrc/verify.cu).
#pragma once
#include "common.cuh"

namespace exb {

static __constant__ uint32_t SHA_K[64] = {
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

// An int64 array's little-endian bytes: bytes up to the next block boundary go through the
// buffer, then whole 64-byte blocks are assembled straight from memory (aligned 32-bit loads,
// shifted by the stream's byte offset, byte-swapped to big-endian words) into a register block,
// then the tail goes through the buffer again.  No load reaches past the array: the extra word of
// a misaligned block is 4-byte aligned and starts inside the array, whose end is 8-byte aligned.
EXB_DEV void sha_i64_array(Sha256& s, const int64_t* p, int64_t n) {
  const uint8_t* src = reinterpret_cast<const uint8_t*>(p);
  const int64_t nbytes = n * 8;
  int64_t pos = 0;
  while (s.nb != 0 && pos < nbytes) {
    if ((pos & 7) == 0 && s.nb + 8 <= 64 && pos + 8 <= nbytes) {
      sha_i64(s, (uint64_t)__ldg(reinterpret_cast<const long long*>(src + pos)));
      pos += 8;
    } else {
      sha_byte(s, src[pos]);
      ++pos;
    }
  }
  if (nbytes - pos >= 64) {
    const uintptr_t a0 = reinterpret_cast<uintptr_t>(src + pos);
    const int sh = (int)(a0 & 3) * 8;
    const uint32_t* wsrc = reinterpret_cast<const uint32_t*>(a0 & ~(uintptr_t)3);
    const int64_t nblk = (nbytes - pos) / 64;
    uint32_t h[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) h[i] = s.h[i];
    for (int64_t b = 0; b < nblk; ++b) {
      uint32_t lw[17];
#pragma unroll
      for (int i = 0; i < 16; ++i) lw[i] = __ldg(wsrc + 16 * b + i);
      lw[16] = sh ? __ldg(wsrc + 16 * b + 16) : 0u;
      uint32_t w[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) w[i] = __byte_perm(__funnelshift_r(lw[i], lw[i + 1], sh), 0, 0x0123);
      sha_compress(h, w);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) s.h[i] = h[i];
    s.total += (uint64_t)nblk * 64;
    pos += nblk * 64;
  }
  for (; pos < nbytes; ++pos) sha_byte(s, src[pos]);
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

}  // namespace exb
