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
//
// Block bytes reach the lanes through shared memory: the warp copies the
// next two chunks of all its 32 chains with cp.async while it hashes the
// current two, each copy instruction reading 128 contiguous bytes of 4
// blocks. Per-lane loads (16 bytes of each of 32 blocks per instruction)
// were as fast only while the warp's blocks sat next to each other in
// memory: with 65,536 blocks at shuffled places they hashed 550 GB/s against
// 809 in order; the staged copies hash about 800 GB/s in both layouts.
#pragma once

namespace cb {
namespace {

constexpr int kFusedWarps = 4;  // warps (of 32 chains) per CTA
constexpr int kFusedTile = 2;   // chunks of each chain staged per shared-memory tile
constexpr int kTilePieces = 4 * kFusedTile;  // 16-byte pieces of one chain in a tile
static_assert(kTilePieces >= 8 && 32 % kTilePieces == 0, "the bank swizzle needs 8..32 pieces per chain");

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

// Asynchronous 16-byte global -> shared copies (cp.async, L1 bypassed).
CB_D void cp_async16(void *smem, const void *g) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem)), "l"(g) : "memory");
}
CB_D void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
CB_D void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// One 64-round compression of the schedule words w into the state st
// (FIPS 180-4 6.2.2 steps 2-4); w is consumed.
CB_D void compress_chunk(uint32_t st[8], uint32_t w[16], const uint32_t *kk, uint32_t one) {
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
  st[0] += a;
  st[1] += b;
  st[2] += cc;
  st[3] += d;
  st[4] += e;
  st[5] += f;
  st[6] += g;
  st[7] += h;
}

__global__ void __launch_bounds__(32 * kFusedWarps) sha256_fused_kernel(const HashJob *__restrict__ jobs, int n,
                                                                          uint32_t *__restrict__ digests,
                                                                          unsigned *err, uint32_t one,
                                                                          HashProgress pg) {
  // round constants of the runtime-indexed rounds 16..63 (warp-uniform
  // shared-memory reads are broadcasts), and per warp two tiles of
  // kFusedTile chunks of each of its 32 chains
  __shared__ uint32_t kk[64];
  __shared__ uint4 stage[kFusedWarps][2][32 * kTilePieces];
  for (int t = threadIdx.x; t < 64; t += blockDim.x) kk[t] = kSha256K[t];
  __syncthreads();
  if ((int64_t)blockIdx.x * blockDim.x + (threadIdx.x & ~31) >= n) return;  // whole warp past the end
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const bool valid = i < n;
  const uint8_t *p = valid ? reinterpret_cast<const uint8_t *>(jobs[i].ptr) : nullptr;
  const uint64_t len = valid ? jobs[i].size : 0;
  const uint64_t nchunks = valid ? (len + 9 + 63) >> 6 : 0;  // padded chunks: ceil((len + 9) / 64)
  const uint64_t nfull = len >> 6;                           // chunks made only of block bytes
  const bool aligned = (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
  // maxc: the warp's longest chain; staged: chunks every chain of the warp
  // reads through the shared-memory tiles (whole tiles of full chunks; 0
  // when a lane is unaligned or past the end, or the input is still being
  // copied in)
  uint64_t maxc = nchunks, staged = (valid && aligned && !pg.counter) ? nfull : 0;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const uint64_t a = __shfl_xor_sync(0xffffffffu, maxc, o);
    maxc = a > maxc ? a : maxc;
    const uint64_t b = __shfl_xor_sync(0xffffffffu, staged, o);
    staged = b < staged ? b : staged;
  }
  staged -= staged % kFusedTile;
  uint32_t seen = 0;
  if (!wait_progress(pg, 1, seen)) {
    if (lane == 0) atomicOr(err, kErrTimeout);
    return;
  }
  uint32_t st[8] = CB_SHA256_H0;

  // Staged part. Instruction m of a tile copies 16-byte piece (lane % P) of
  // chain m * (32 / P) + lane / P (P = kTilePieces), so one warp-wide copy
  // reads contiguous bytes of 32 / P blocks instead of 16 bytes of each of
  // 32 blocks scattered over memory; piece k of chain ch sits at slot
  // ch * P + (k ^ (ch & 7)), so the 8 lanes of each shared-memory phase hit
  // 8 different bank groups on both the copy and the read.
  const uint64_t ntiles = staged / kFusedTile;
  auto issue_tile = [&](uint64_t t, uint4 *sb) {
#pragma unroll
    for (int m = 0; m < kTilePieces; ++m) {
      const int ch = m * (32 / kTilePieces) + lane / kTilePieces, pc = lane % kTilePieces;
      const uint8_t *src =
          reinterpret_cast<const uint8_t *>(__shfl_sync(0xffffffffu, reinterpret_cast<uintptr_t>(p), ch));
      cp_async16(sb + ch * kTilePieces + (pc ^ (ch & 7)), src + t * (64ull * kFusedTile) + 16ull * pc);
    }
    cp_async_commit();
  };
  if (ntiles) issue_tile(0, stage[warp][0]);
  for (uint64_t t = 0; t < ntiles; ++t) {
    if (t + 1 < ntiles) {  // the next tile streams in while this one is hashed
      issue_tile(t + 1, stage[warp][(t + 1) & 1]);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncwarp();  // every lane's copies of tile t are visible to the warp
    const uint4 *sb = stage[warp][t & 1] + lane * kTilePieces;
    const int x = lane & 7;
#pragma unroll 1
    for (int j = 0; j < kFusedTile; ++j) {
      uint32_t w[16];
      unpack_be(sb[(4 * j) ^ x], sb[(4 * j + 1) ^ x], sb[(4 * j + 2) ^ x], sb[(4 * j + 3) ^ x], w);
      compress_chunk(st, w, kk, one);
    }
    __syncwarp();  // tile t's buffer is read before tile t + 2 is copied into it
  }

  // The rest of each chain (all of it when nothing was staged): per-lane
  // 16-byte loads one chunk ahead, then the padded tail chunks.
  const uint4 *q = reinterpret_cast<const uint4 *>(p) + 4 * staged;
  uint4 v0 = make_uint4(0, 0, 0, 0), v1 = v0, v2 = v0, v3 = v0;
  if (aligned && staged < nfull) {
    v0 = ld_stream16(q);
    v1 = ld_stream16(q + 1);
    v2 = ld_stream16(q + 2);
    v3 = ld_stream16(q + 3);
  }
  for (uint64_t c = staged; c < maxc; ++c) {
    if (pg.counter) {
      // this iteration reads chunk c (slow path) and prefetches chunk c+1
      const uint64_t last = pg.data_chunks ? pg.data_chunks - 1 : 0;
      const uint64_t need_chunk = c + 1 < last ? c + 1 : last;
      if (!wait_progress(pg, (uint32_t)(need_chunk / pg.seg_chunks) + 1, seen)) {
        if (lane == 0) atomicOr(err, kErrTimeout);
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
    // lanes whose chain has ended run the rounds with the warp and drop them
    uint32_t next[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) next[k] = st[k];
    compress_chunk(next, w, kk, one);
    if (c < nchunks) {
#pragma unroll
      for (int k = 0; k < 8; ++k) st[k] = next[k];
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
