// Batched SHA-256 of variable-size blocks: the GPU form of
// compute_block_id (cascade_Code/cpp/src/cascade_core.cpp:47-58).
//
// Layout: one lane = one block = one serial compression chain. A CTA is one
// warp carrying up to kLanes chains, so a batch of n blocks occupies
// ceil(n / kLanes) warps, each alone on an SM sub-partition scheduler: the
// round function is latency/issue bound per chain and chains never share a
// scheduler unless the batch exceeds the machine.
//
// Each lane streams its block with 16-byte non-coherent loads that also ask
// L2 to fetch the surrounding 256 B, one chunk (64 B) of register prefetch
// ahead, so the next compression's message words are resident when it starts.
#include "kernels.cuh"
#include "sha256_core.cuh"

namespace cb {

namespace {

CB_D uint4 ld_stream16(const void *p) {
  uint4 r;
  asm("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
      : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
      : "l"(p));
  return r;
}

CB_D uint32_t ld_byte(const uint8_t *p) { return (uint32_t)__ldg(p); }

// Big-endian word at an arbitrary address (slow path for unaligned blocks).
CB_D uint32_t ld_be32_unaligned(const uint8_t *p) {
  return (ld_byte(p) << 24) | (ld_byte(p + 1) << 16) | (ld_byte(p + 2) << 8) | ld_byte(p + 3);
}

__device__ __noinline__ void compress_ni(uint32_t st[8], uint32_t w[16]) { sha256_compress(st, w); }

template <int kLanes>
__global__ void __launch_bounds__(32) sha256_batch_kernel(const HashJob *__restrict__ jobs, int n,
                                                          uint32_t *__restrict__ digests) {
  const int lane = threadIdx.x;
  const int64_t i = (int64_t)blockIdx.x * kLanes + lane;
  if (lane >= kLanes || i >= n) return;
  const uint8_t *p = reinterpret_cast<const uint8_t *>(jobs[i].ptr);
  const uint64_t len = jobs[i].size;
  uint32_t st[8] = CB_SHA256_H0;
  uint32_t w[16];
  const uint64_t nfull = len >> 6;

  if ((reinterpret_cast<uintptr_t>(p) & 15u) == 0) {
    const uint4 *q = reinterpret_cast<const uint4 *>(p);
    uint4 v0 = make_uint4(0, 0, 0, 0), v1 = v0, v2 = v0, v3 = v0;
    if (nfull) {
      v0 = ld_stream16(q);
      v1 = ld_stream16(q + 1);
      v2 = ld_stream16(q + 2);
      v3 = ld_stream16(q + 3);
    }
    for (uint64_t c = 0; c < nfull; ++c) {
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
      if (c + 1 < nfull) {
        q += 4;
        v0 = ld_stream16(q);
        v1 = ld_stream16(q + 1);
        v2 = ld_stream16(q + 2);
        v3 = ld_stream16(q + 3);
      }
      sha256_compress(st, w);
    }
  } else {
    for (uint64_t c = 0; c < nfull; ++c) {
      const uint8_t *b = p + (c << 6);
#pragma unroll
      for (int k = 0; k < 16; ++k) w[k] = ld_be32_unaligned(b + 4 * k);
      compress_ni(st, w);
    }
  }

  // FIPS 180-4 5.1.1 padding: remaining bytes, 0x80, zeros, 64-bit length.
  const uint8_t *tp = p + (nfull << 6);
  const uint32_t rem = (uint32_t)(len & 63);
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    uint32_t word = 0;
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const uint32_t idx = 4 * k + b;
      const uint32_t byte = idx < rem ? ld_byte(tp + idx) : (idx == rem ? 0x80u : 0u);
      word = (word << 8) | byte;
    }
    w[k] = word;
  }
  const uint64_t bits = len << 3;
  if (rem >= 56) {
    compress_ni(st, w);
#pragma unroll
    for (int k = 0; k < 14; ++k) w[k] = 0;
  }
  w[14] = (uint32_t)(bits >> 32);
  w[15] = (uint32_t)bits;
  compress_ni(st, w);

  uint4 *out = reinterpret_cast<uint4 *>(digests + 8 * i);
  out[0] = make_uint4(bswap32(st[0]), bswap32(st[1]), bswap32(st[2]), bswap32(st[3]));
  out[1] = make_uint4(bswap32(st[4]), bswap32(st[5]), bswap32(st[6]), bswap32(st[7]));
}

}  // namespace

cudaError_t launch_sha256_batch(const HashJob *d_jobs, int n, uint32_t *d_digests, int lanes,
                                cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  switch (lanes) {
    case 8:
      sha256_batch_kernel<8><<<(n + 7) / 8, 32, 0, stream>>>(d_jobs, n, d_digests);
      break;
    case 16:
      sha256_batch_kernel<16><<<(n + 15) / 16, 32, 0, stream>>>(d_jobs, n, d_digests);
      break;
    default:
      sha256_batch_kernel<32><<<(n + 31) / 32, 32, 0, stream>>>(d_jobs, n, d_digests);
      break;
  }
  return cudaGetLastError();
}

}  // namespace cb
