// Batched SHA-256 of variable-size blocks: the GPU form of
// compute_block_id (cascade_Code/cpp/src/cascade_core.cpp:47-58).
//
// Bit-exact block IDs make every block one serial Merkle-Damgard chain, so
// the batch size caps the chains in flight and the time of one launch is the
// time of one chain. Measured on B200, a lane that runs the whole
// compression (message schedule + 64 rounds) is bound by its sub-partition's
// integer ALU pipe: ~22 instructions per round at half rate.
//
// The kernel therefore splits each chain across two warps of one CTA, each
// on its own SM sub-partition:
//  * producer warp: streams the 64-byte chunks of its 32 blocks (16-byte
//    loads, one chunk ahead), builds the FIPS 180-4 padding, expands the
//    message schedule and writes W[t] + K[t] for all 64 rounds into a
//    shared-memory ring (kStages chunks deep);
//  * consumer warp: runs the 64 rounds per chunk from the ring. The rotates
//    and 3-input logic (Sigma, Ch, Maj) need the half-rate ALU pipe; the
//    additions that are off the e-recurrence are issued as IMAD so they run
//    on the FMA pipe beside it.
// The ring is handed over with mbarriers (bounded waits; on timeout the
// kernel raises kErrTimeout, sets the ring's abort word, which the other
// warp's waits also watch, and both warps leave).
#include "kernels.cuh"
#include "sha256_core.cuh"

namespace cb {

namespace {

constexpr int kStages = 4;
constexpr uint64_t kWaitLimit = 1ull << 26;

CB_D uint4 ld_stream16(const void *p) {
  uint4 r;
  asm("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
      : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
      : "l"(p));
  return r;
}

CB_D uint32_t ld_byte(const uint8_t *p) { return (uint32_t)__ldg(p); }

// a + b on the FMA pipe: IMAD with a multiplier the compiler cannot fold.
CB_D uint32_t madd(uint32_t a, uint32_t b, uint32_t one) {
  uint32_t r;
  asm("mad.lo.u32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(one), "r"(b));
  return r;
}

CB_D uint32_t smem_u32(const void *p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

CB_D void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
CB_D void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// Bounded wait on an mbarrier phase that also gives up as soon as the other
// warp has set *abort.
CB_D bool mbar_wait(uint64_t *bar, uint32_t parity, const volatile uint32_t *abort) {
  const uint32_t a = smem_u32(bar);
  for (uint64_t it = 0; it < kWaitLimit; ++it) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(a), "r"(parity)
        : "memory");
    if (ok) return true;
    if (*abort) return false;
  }
  return false;
}

// Message words of padded chunk c (FIPS 180-4 5.1.1) for a block of len
// bytes at p: data bytes, then 0x80, zeros, and the 64-bit bit length in the
// last 8 bytes of the final chunk. Used for the last one or two chunks and
// for unaligned blocks.
CB_D void load_chunk_slow(const uint8_t *p, uint64_t len, uint64_t c, uint64_t nchunks, uint32_t w[16]) {
  const uint64_t base = c << 6;
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    uint32_t word = 0;
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const uint64_t idx = base + 4 * k + b;
      const uint32_t byte = idx < len ? ld_byte(p + idx) : (idx == len ? 0x80u : 0u);
      word = (word << 8) | byte;
    }
    w[k] = word;
  }
  if (c + 1 == nchunks) {
    const uint64_t bits = len << 3;
    w[14] = (uint32_t)(bits >> 32);
    w[15] = (uint32_t)bits;
  }
}

CB_D void unpack_be(const uint4 &v0, const uint4 &v1, const uint4 &v2, const uint4 &v3, uint32_t w[16]) {
  w[0] = bswap32(v0.x);
  w[1] = bswap32(v0.y);
  w[2] = bswap32(v0.z);
  w[3] = bswap32(v0.w);
  w[4] = bswap32(v1.x);
  w[5] = bswap32(v1.y);
  w[6] = bswap32(v1.z);
  w[7] = bswap32(v1.w);
  w[8] = bswap32(v2.x);
  w[9] = bswap32(v2.y);
  w[10] = bswap32(v2.z);
  w[11] = bswap32(v2.w);
  w[12] = bswap32(v3.x);
  w[13] = bswap32(v3.y);
  w[14] = bswap32(v3.z);
  w[15] = bswap32(v3.w);
}

struct Ring {
  uint4 kw[kStages][16][32];  // [stage][round/4][lane]: W[t]+K[t] for 4 rounds
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint32_t abort;  // set by a warp that gives up; the other warp's waits watch it
};

// A warp that gives up: record the error once and tell the other warp.
CB_D void give_up(Ring &ring, unsigned *err) {
  if ((threadIdx.x & 31) == 0) {
    atomicOr(err, kErrTimeout);
    *reinterpret_cast<volatile uint32_t *>(&ring.abort) = 1u;
  }
  __syncwarp();
}

// Waits (bounded) until the copy stream has published segment `need - 1`.
// Called by the whole producer warp with a warp-uniform `need`; lane 0
// polls the counter with acquire loads, the result is broadcast.
CB_D bool wait_progress(const HashProgress &pg, uint32_t need, uint32_t &seen) {
  if (!pg.counter || seen >= need) return true;
  const uint64_t limit = pg.wait_iters ? pg.wait_iters : kWaitLimit;
  uint32_t v = 0;
  if ((threadIdx.x & 31) == 0) {
    for (uint64_t it = 0; it < limit; ++it) {
      asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(pg.counter) : "memory");
      if (v >= need) break;
      __nanosleep(128);
    }
  }
  v = __shfl_sync(0xffffffffu, v, 0);
  __syncwarp();
  if (v < need) return false;
  seen = v;
  return true;
}

__global__ void __launch_bounds__(64) sha256_pc_kernel(const HashJob *__restrict__ jobs, int n,
                                                       uint32_t *__restrict__ digests, unsigned *err,
                                                       uint32_t one, HashProgress pg) {
  __shared__ __align__(16) Ring ring;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t i = (int64_t)blockIdx.x * 32 + lane;
  const bool valid = i < n;
  const uint8_t *p = valid ? reinterpret_cast<const uint8_t *>(jobs[i].ptr) : nullptr;
  const uint64_t len = valid ? jobs[i].size : 0;
  // Padded chunk count: ceil((len + 9) / 64).
  const uint64_t nchunks = valid ? (len + 9 + 63) >> 6 : 0;
  uint64_t maxc = nchunks;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const uint64_t other = __shfl_xor_sync(0xffffffffu, maxc, o);
    maxc = other > maxc ? other : maxc;
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&ring.full[s], 32);
      mbar_init(&ring.empty[s], 32);
    }
    ring.abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  const volatile uint32_t *abort = &ring.abort;

  if (warp == 1) {
    // ------------------------------------------------------------ producer
    const uint64_t nfull = len >> 6;  // chunks made only of block bytes
    const bool aligned = (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
    const uint4 *q = reinterpret_cast<const uint4 *>(p);
    uint4 v0 = make_uint4(0, 0, 0, 0), v1 = v0, v2 = v0, v3 = v0;
    // When the blocks are still arriving (host put overlapped with the
    // copy), chunk c may only be read once its segment has landed.
    uint32_t seen = 0;
    if (!wait_progress(pg, 1, seen)) {
      give_up(ring, err);
      return;
    }
    if (aligned && nfull) {
      v0 = ld_stream16(q);
      v1 = ld_stream16(q + 1);
      v2 = ld_stream16(q + 2);
      v3 = ld_stream16(q + 3);
    }
    for (uint64_t c = 0; c < maxc; ++c) {
      const int s = (int)(c % kStages);
      if (c >= kStages && !mbar_wait(&ring.empty[s], (uint32_t)((c / kStages) - 1) & 1u, abort)) {
        give_up(ring, err);
        return;
      }
      if (pg.counter) {
        // this iteration reads chunk c (slow path) and prefetches chunk c+1
        const uint64_t last = pg.data_chunks ? pg.data_chunks - 1 : 0;
        const uint64_t need_chunk = c + 1 < last ? c + 1 : last;
        if (!wait_progress(pg, (uint32_t)(need_chunk / pg.seg_chunks) + 1, seen)) {
          give_up(ring, err);
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
#pragma unroll
      for (int g = 0; g < 16; ++g) {
        uint32_t kw[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int t = 4 * g + j;
          uint32_t wt;
          if (t < 16) {
            wt = w[t];
          } else {
            const uint32_t x15 = w[(t + 1) & 15], x2 = w[(t + 14) & 15];
            const uint32_t s0 = rotr32(x15, 7) ^ rotr32(x15, 18) ^ (x15 >> 3);
            const uint32_t s1 = rotr32(x2, 17) ^ rotr32(x2, 19) ^ (x2 >> 10);
            wt = madd(madd(w[t & 15], s0, one), madd(w[(t + 9) & 15], s1, one), one);
            w[t & 15] = wt;
          }
          kw[j] = madd(wt, kSha256K[t], one);
        }
        ring.kw[s][g][lane] = make_uint4(kw[0], kw[1], kw[2], kw[3]);
      }
      mbar_arrive(&ring.full[s]);
    }
    return;
  }

  // -------------------------------------------------------------- consumer
  uint32_t st[8] = CB_SHA256_H0;
  for (uint64_t c = 0; c < maxc; ++c) {
    const int s = (int)(c % kStages);
    if (!mbar_wait(&ring.full[s], (uint32_t)(c / kStages) & 1u, abort)) {
      give_up(ring, err);
      return;
    }
    uint32_t a = st[0], b = st[1], cc = st[2], d = st[3];
    uint32_t e = st[4], f = st[5], g = st[6], h = st[7];
    // 4 x 16 rounds: the 16-round body keeps the register roles (period 4)
    // and fits the instruction cache; a fully unrolled 64-round body measured
    // ~10% slower from instruction-fetch stalls.
#pragma unroll 1
    for (int it = 0; it < 4; ++it)
#pragma unroll
    for (int gq = 0; gq < 4; ++gq) {
      const int gi = 4 * it + gq;
      const uint4 kv = ring.kw[s][gi][lane];
      const uint32_t kw4[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        // e' = (d + h + W + K) + Ch(e,f,g) + Sigma1(e): the e recurrence stays
        //      on the ALU pipe (rotate -> LOP3 -> IADD3), its off-path sum
        //      d + h + WK on the FMA pipe;
        // a' = e' + (Sigma0(a) + Maj(a,b,c) - d): the last add on the FMA pipe.
        // (Measured on B200: fastest of the pipe splits tried, ~27 cycles per
        // round in isolation against ~31 for the textbook form.)
        const uint32_t p = madd(madd(d, h, one), kw4[j], one);
        const uint32_t ne = p + sha_ch(e, f, g) + big_sigma1(e);
        const uint32_t q = big_sigma0(a) + sha_maj(a, b, cc) - d;
        h = g;
        g = f;
        f = e;
        e = ne;
        d = cc;
        cc = b;
        b = a;
        a = madd(ne, q, one);
      }
    }
    mbar_arrive(&ring.empty[s]);
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

#include "sha256_fused.cuh"

namespace cb {

cudaError_t prepare_sha256_kernel() {
  cudaFuncAttributes a;
  return cudaFuncGetAttributes(&a, sha256_pc_kernel);  // loads this file's module (both kernels)
}

cudaError_t launch_sha256_batch(const HashJob *d_jobs, int n, uint32_t *d_digests, int lanes,
                                unsigned *d_err, cudaStream_t stream, const HashProgress *progress,
                                bool many_chains) {
  (void)lanes;
  if (n <= 0) return cudaSuccess;
  const HashProgress pg = progress ? *progress : HashProgress{nullptr, 1, 0, 0};
  if (many_chains) {
    constexpr int kThreads = 32 * kFusedWarps;
    sha256_fused_kernel<<<(n + kThreads - 1) / kThreads, kThreads, 0, stream>>>(d_jobs, n, d_digests, d_err, 1u,
                                                                               pg);
  } else {
    sha256_pc_kernel<<<(n + 31) / 32, 64, 0, stream>>>(d_jobs, n, d_digests, d_err, 1u, pg);
  }
  return cudaGetLastError();
}

}  // namespace cb
