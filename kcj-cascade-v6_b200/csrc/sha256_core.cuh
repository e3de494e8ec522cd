// SHA-256 compression (FIPS 180-4 6.2.2) for one chain held in registers.
//
// Block IDs of cascade_Code/cpp/src/cascade_core.cpp:47-58 are the first 16
// bytes of SHA-256(block); bit-exact IDs forbid tree hashing, so each block is
// one serial Merkle-Damgard chain and the GPU parallelises across blocks only.
// A lane owns one chain: its state and the 16-word message window live in
// registers; every round below is fully unrolled so the window indices and
// the round constants are compile-time (constant-bank operands).
#pragma once

#include <stdint.h>

#include "common.cuh"

// Device-only under nvcc; plain inline functions when the header is compiled by
// a host compiler (used by the host-side self-check of the unrolled schedule).
#if defined(__CUDACC__)
#define CB_SHA_FN __device__ __forceinline__
#else
#define CB_SHA_FN inline
#endif

namespace cb {

// FIPS 180-4 4.2.2 round constants.
#if defined(__CUDACC__)
__constant__
#endif
static const uint32_t kSha256K[64] = {
    0x428a2f98u, 0x71374491u, 0xb5c0fbcfu, 0xe9b5dba5u, 0x3956c25bu, 0x59f111f1u, 0x923f82a4u,
    0xab1c5ed5u, 0xd807aa98u, 0x12835b01u, 0x243185beu, 0x550c7dc3u, 0x72be5d74u, 0x80deb1feu,
    0x9bdc06a7u, 0xc19bf174u, 0xe49b69c1u, 0xefbe4786u, 0x0fc19dc6u, 0x240ca1ccu, 0x2de92c6fu,
    0x4a7484aau, 0x5cb0a9dcu, 0x76f988dau, 0x983e5152u, 0xa831c66du, 0xb00327c8u, 0xbf597fc7u,
    0xc6e00bf3u, 0xd5a79147u, 0x06ca6351u, 0x14292967u, 0x27b70a85u, 0x2e1b2138u, 0x4d2c6dfcu,
    0x53380d13u, 0x650a7354u, 0x766a0abbu, 0x81c2c92eu, 0x92722c85u, 0xa2bfe8a1u, 0xa81a664bu,
    0xc24b8b70u, 0xc76c51a3u, 0xd192e819u, 0xd6990624u, 0xf40e3585u, 0x106aa070u, 0x19a4c116u,
    0x1e376c08u, 0x2748774cu, 0x34b0bcb5u, 0x391c0cb3u, 0x4ed8aa4au, 0x5b9cca4fu, 0x682e6ff3u,
    0x748f82eeu, 0x78a5636fu, 0x84c87814u, 0x8cc70208u, 0x90befffau, 0xa4506cebu, 0xbef9a3f7u,
    0xc67178f2u};

// FIPS 180-4 5.3.3 initial hash value.
#define CB_SHA256_H0 \
  {0x6a09e667u, 0xbb67ae85u, 0x3c6ef372u, 0xa54ff53au, 0x510e527fu, 0x9b05688cu, 0x1f83d9abu, 0x5be0cd19u}

CB_SHA_FN uint32_t rotr32(uint32_t x, int n) {
#if defined(__CUDA_ARCH__)
  return __funnelshift_r(x, x, n);
#else
  return (x >> n) | (x << (32 - n));
#endif
}

CB_SHA_FN uint32_t bswap32(uint32_t x) {
#if defined(__CUDA_ARCH__)
  return __byte_perm(x, 0, 0x0123);
#else
  return (x >> 24) | ((x >> 8) & 0xff00u) | ((x << 8) & 0xff0000u) | (x << 24);
#endif
}

CB_SHA_FN uint32_t big_sigma0(uint32_t a) { return rotr32(a, 2) ^ rotr32(a, 13) ^ rotr32(a, 22); }
CB_SHA_FN uint32_t big_sigma1(uint32_t e) { return rotr32(e, 6) ^ rotr32(e, 11) ^ rotr32(e, 25); }
CB_SHA_FN uint32_t small_sigma0(uint32_t x) { return rotr32(x, 7) ^ rotr32(x, 18) ^ (x >> 3); }
CB_SHA_FN uint32_t small_sigma1(uint32_t x) { return rotr32(x, 17) ^ rotr32(x, 19) ^ (x >> 10); }
CB_SHA_FN uint32_t sha_ch(uint32_t e, uint32_t f, uint32_t g) { return (e & f) ^ (~e & g); }
CB_SHA_FN uint32_t sha_maj(uint32_t a, uint32_t b, uint32_t c) { return (a & b) | (c & (a | b)); }

// One compression: st <- st + rounds(st, w). w holds the 16 big-endian
// message words and is consumed (used as the rolling schedule window).
CB_SHA_FN void sha256_compress(uint32_t st[8], uint32_t w[16]) {
  uint32_t a = st[0], b = st[1], c = st[2], d = st[3];
  uint32_t e = st[4], f = st[5], g = st[6], h = st[7];
#if defined(__CUDA_ARCH__)
#pragma unroll
#endif
  for (int t = 0; t < 64; ++t) {
    uint32_t wt;
    if (t < 16) {
      wt = w[t];
    } else {
      wt = w[t & 15] + small_sigma0(w[(t + 1) & 15]) + w[(t + 9) & 15] +
           small_sigma1(w[(t + 14) & 15]);
      w[t & 15] = wt;
    }
    // h + K + W does not depend on this round's e/a: it is off the critical
    // path, leaving Sigma1/Ch -> add -> e as the loop-carried chain.
    const uint32_t hkw = h + kSha256K[t] + wt;
    const uint32_t t1 = hkw + big_sigma1(e) + sha_ch(e, f, g);
    const uint32_t t2 = big_sigma0(a) + sha_maj(a, b, c);
    h = g;
    g = f;
    f = e;
    e = d + t1;
    d = c;
    c = b;
    b = a;
    a = t1 + t2;
  }
  st[0] += a;
  st[1] += b;
  st[2] += c;
  st[3] += d;
  st[4] += e;
  st[5] += f;
  st[6] += g;
  st[7] += h;
}

}  // namespace cb
