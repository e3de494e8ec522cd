// Fused SHA-256 kernel: one warp per 32 blocks, included by sha256.cu (it
// uses that file's load, padding and progress-wait helpers).
//
// Each lane runs its block's message schedule and rounds itself, with no
// shared-memory hand-off, and every addition is issued as IMAD on the FMA
// pipe. The half-rate integer ALU pipe then carries only the rotates,
// shifts and 3-input logic: 10 instructions per round (Sigma0, Sigma1: 3
// SHF + LOP3 each; Ch, Maj: one LOP3) and 8 per schedule word (sigma0,
// sigma1: 2 SHF + SHR + LOP3 each), i.e. 1040 ALU instructions per 64-byte
// chunk with the byte swaps, while 7 + 3 IMAD go to the FMA pipe beside
// them. The independent schedule words fill the gaps of the two round
// recurrences, so one such warp keeps its sub-partition's ALU pipe busy: a
// GPU full of them hashes at the ALU-pipe rate, where the producer/consumer
// pair spends a second sub-partition on the schedule of the same 32 chains.
#pragma once

namespace cb {
namespace {

constexpr int kFusedWarps = 4;  // warps (of 32 chains) per CTA

// Rounds T0..T0+15 of one chunk; for T0 >= 16 the window w is extended by
// the message schedule in place. kk: the 16 round constants of this block
// (shared memory) when T0 >= 16.
template <int T0>
CB_D void rounds16(uint32_t &a, uint32_t &b, uint32_t &c, uint32_t &d, uint32_t &e, uint32_t &f, uint32_t &g,
                   uint32_t &h, uint32_t w[16], const uint32_t *kk, uint32_t one) {
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    uint32_t wt;
    if (T0 == 0) {
      wt = w[j];
    } else {
      const uint32_t x15 = w[(j + 1) & 15], x2 = w[(j + 14) & 15];
      wt = madd(madd(w[j], small_sigma0(x15), one), madd(w[(j + 9) & 15], small_sigma1(x2), one), one);
      w[j] = wt;
    }
    // T1 = h + K + W + Ch(e,f,g) + Sigma1(e); e' = d + T1;
    // a' = T1 + Sigma0(a) + Maj(a,b,c): every add on the FMA pipe
    const uint32_t hkw = madd(madd(wt, T0 == 0 ? kSha256K[j] : kk[j], one), h, one);
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
  // round constants for the runtime-indexed 16-round loop (warp-uniform
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
    rounds16<0>(a, b, cc, d, e, f, g, h, w, kk, one);
    // rounds 16..63: one 16-round body (instruction-cache sized) run three
    // times, the round constants from shared memory
#pragma unroll 1
    for (int it = 1; it < 4; ++it) rounds16<16>(a, b, cc, d, e, f, g, h, w, kk + 16 * it, one);
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
