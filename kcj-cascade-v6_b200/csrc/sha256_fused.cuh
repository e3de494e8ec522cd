// Fused SHA-256 kernel for many chains in flight (pipelined puts): one warp
// per 32 blocks, included by sha256.cu (it uses that file's load, padding and
// progress-wait helpers).
//
// Each lane runs its block's whole compression - message schedule and
// rounds - with no shared-memory hand-off, and every addition is issued as
// IMAD on the FMA pipe, so the half-rate integer ALU pipe carries only the
// rotates, shifts and 3-input logic: 10 instructions per round (Sigma0,
// Sigma1: 3 SHF + LOP3 each; Ch, Maj: one LOP3) and 8 per schedule word
// (sigma0, sigma1: 2 SHF + SHR + LOP3 each). The schedule words of each
// 16-round block are expanded together before its rounds: two independent
// recurrences (W[t] on W[t-2]) that issue back to back, where interleaving
// one word per round stalled the in-order issue on each word's latency.
//
// Measured on B200 (917,504-byte blocks, digests equal to the
// producer/consumer kernel's): one warp per sub-partition runs ~46 cycles
// per round (the producer/consumer pair ~31, but it occupies two
// sub-partitions per 32 chains), so with 16,384 chains in flight (16
// concurrent 1024-block launches) this kernel hashes 693 GB/s against 555,
// and 904 against 667 GB/s at 37,888 chains; at 1024 chains alone the pair
// is faster (63.5 against 43.8 GB/s), which is why the synchronous put keeps
// it.
#pragma once

namespace cb {
namespace {

constexpr int kFusedWarps = 4;  // warps (of 32 chains) per CTA

// The next 16 schedule words, in place: w[j] = W[t0 + j] from the previous
// 16 (FIPS 180-4 6.2.2 step 1).
CB_D void expand16(uint32_t w[16], uint32_t one) {
#pragma unroll
  for (int j = 0; j < 16; ++j)
    w[j] = madd(madd(w[j], small_sigma0(w[(j + 1) & 15]), one),
                madd(w[(j + 9) & 15], small_sigma1(w[(j + 14) & 15]), one), one);
}

// 16 rounds with the schedule words w[0..15] and round constants k(0..15).
template <class K>
CB_D void rounds16(uint32_t &a, uint32_t &b, uint32_t &c, uint32_t &d, uint32_t &e, uint32_t &f, uint32_t &g,
                   uint32_t &h, const uint32_t w[16], K k, uint32_t one) {
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    // T1 = h + K + W + Ch(e,f,g) + Sigma1(e); e' = d + T1;
    // a' = T1 + Sigma0(a) + Maj(a,b,c)
    const uint32_t hkw = madd(madd(w[j], k(j), one), h, one);
    const uint32_t t1 = madd(madd(hkw, sha_ch(e, f, g), one), big_sigma1(e), one);
    const uint32_t t2 = madd(big_sigma0(a), sha_maj(a, b, c), one);
    h = g;
    g = f;
    f = e;
    e = madd(t1, d, one);
    d = c;
    c = b;
    b = a;
    a = madd(t1, t2, one);
  }
}

__global__ void __launch_bounds__(32 * kFusedWarps) sha256_fused_kernel(const HashJob *__restrict__ jobs, int n,
                                                                          uint32_t *__restrict__ digests,
                                                                          unsigned *err, uint32_t one,
                                                                          HashProgress pg) {
  // round constants of the runtime-indexed rounds 16..63 (warp-uniform
  // shared-memory reads are broadcasts)
  __shared__ uint32_t kk[64];
  for (int t = threadIdx.x; t < 64; t += blockDim.x) kk[t] = kSha256K[t];
  __syncthreads();
  if ((int64_t)blockIdx.x * blockDim.x + (threadIdx.x & ~31) >= n) return;  // whole warp past the end
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const bool valid = i < n;
  const uint8_t *p = valid ? reinterpret_cast<const uint8_t *>(jobs[i].ptr) : nullptr;
  const uint64_t len = valid ? jobs[i].size : 0;
  const uint64_t nchunks = valid ? (len + 9 + 63) >> 6 : 0;  // padded chunks: ceil((len + 9) / 64)
  uint64_t maxc = nchunks;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const uint64_t other = __shfl_xor_sync(0xffffffffu, maxc, o);
    maxc = other > maxc ? other : maxc;
  }
  const uint64_t nfull = len >> 6;  // chunks made only of block bytes
  const bool aligned = (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
  const uint4 *q = reinterpret_cast<const uint4 *>(p);
  uint4 v0 = make_uint4(0, 0, 0, 0), v1 = v0, v2 = v0, v3 = v0;
  uint32_t seen = 0;
  if (!wait_progress(pg, 1, seen)) {
    if ((threadIdx.x & 31) == 0) atomicOr(err, kErrTimeout);
    return;
  }
  if (aligned && nfull) {
    v0 = ld_stream16(q);
    v1 = ld_stream16(q + 1);
    v2 = ld_stream16(q + 2);
    v3 = ld_stream16(q + 3);
  }
  uint32_t st[8] = CB_SHA256_H0;
  for (uint64_t c = 0; c < maxc; ++c) {
    if (pg.counter) {
      // this iteration reads chunk c (slow path) and prefetches chunk c+1
      const uint64_t last = pg.data_chunks ? pg.data_chunks - 1 : 0;
      const uint64_t need_chunk = c + 1 < last ? c + 1 : last;
      if (!wait_progress(pg, (uint32_t)(need_chunk / pg.seg_chunks) + 1, seen)) {
        if ((threadIdx.x & 31) == 0) atomicOr(err, kErrTimeout);
        return;
      }
    }
    uint32_t w[16];
    if (c < nfull && aligned) {
      unpack_be(v0, v1, v2, v3, w);
      if (c + 1 < nfull) {
        q += 4;
        v0 = ld_stream16(q);
        v1 = ld_stream16(q + 1);
        v2 = ld_stream16(q + 2);
        v3 = ld_stream16(q + 3);
      }
    } else if (c < nchunks) {
      load_chunk_slow(p, len, c, nchunks, w);
    } else {
#pragma unroll
      for (int k = 0; k < 16; ++k) w[k] = 0;
    }
    uint32_t a = st[0], b = st[1], cc = st[2], d = st[3];
    uint32_t e = st[4], f = st[5], g = st[6], h = st[7];
    rounds16(a, b, cc, d, e, f, g, h, w, [](int j) { return kSha256K[j]; }, one);
    // rounds 16..63: one 16-round body (instruction-cache sized) run three
    // times, after the expansion of its schedule words
#pragma unroll 1
    for (int it = 1; it < 4; ++it) {
      expand16(w, one);
      const uint32_t *kb = kk + 16 * it;
      rounds16(a, b, cc, d, e, f, g, h, w, [kb](int j) { return kb[j]; }, one);
    }
    if (c < nchunks) {
      st[0] += a;
      st[1] += b;
      st[2] += cc;
      st[3] += d;
      st[4] += e;
      st[5] += f;
      st[6] += g;
      st[7] += h;
    }
  }
  if (valid) {
    uint4 *out = reinterpret_cast<uint4 *>(digests + 8 * i);
    out[0] = make_uint4(bswap32(st[0]), bswap32(st[1]), bswap32(st[2]), bswap32(st[3]));
    out[1] = make_uint4(bswap32(st[4]), bswap32(st[5]), bswap32(st[6]), bswap32(st[7]));
  }
}

}  // namespace
}  // namespace cb
