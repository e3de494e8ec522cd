// Shared definitions for the Cascade B200 block data path (device + host).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "cascade_b200.h"

#if defined(__CUDACC__)
#define CB_HD __host__ __device__ __forceinline__
#define CB_D __device__ __forceinline__
#else
#define CB_HD inline
#endif

namespace cb {

// A block key is the first 16 bytes of the block's SHA-256 digest (the binary
// form of the 32-hex BlockId of cascade_Code/cpp/src/cascade_core.cpp:47-58).
// lo = bytes 0..7, hi = bytes 8..15, both loaded little-endian.
struct Key {
  uint64_t lo, hi;
};

CB_HD bool key_eq(const Key &a, const Key &b) { return a.lo == b.lo && a.hi == b.hi; }

// Owner shard of a key in an W-GPU DHT: the first 8 digest bytes read as a
// big-endian u64, modulo W.
CB_HD uint64_t bswap64(uint64_t x) {
  x = ((x & 0x00FF00FF00FF00FFull) << 8) | ((x >> 8) & 0x00FF00FF00FF00FFull);
  x = ((x & 0x0000FFFF0000FFFFull) << 16) | ((x >> 16) & 0x0000FFFF0000FFFFull);
  return (x << 32) | (x >> 32);
}
CB_HD int owner_of(const Key &k, int world) {
  return world <= 1 ? 0 : (int)(bswap64(k.lo) % (uint64_t)world);
}

// Index slot hash: bytes 8..15 of the digest (independent of the owner bits).
CB_HD uint64_t slot_hash(const Key &k) { return k.hi ^ (k.lo >> 29) ^ (k.lo << 35); }

// ---------------------------------------------------------------------------
// Device index slot (32 B, one sector). Open addressing, linear probing.
//   meta: bit 63 occupied, bit 62 tombstone, bit 61 claim-in-progress,
//         bit 49 packed (the DRAM copy is INT8-packed, kv_compression),
//         bit 48 prefix flag, bits 0..47 logical block size (for a packed
//         block: its unpacked size).
//   loc : bit 63 tier (0 = HBM pool, 1 = pinned DRAM arena), bits 0..62 byte
//         offset inside that arena.
// ---------------------------------------------------------------------------
struct __align__(16) Slot {
  uint64_t klo, khi;
  uint64_t loc;
  unsigned long long meta;
};

constexpr uint64_t kMetaOccupied = 1ull << 63;
constexpr uint64_t kMetaTomb = 1ull << 62;
constexpr uint64_t kMetaClaim = 1ull << 61;
constexpr uint64_t kMetaPacked = 1ull << 49;
constexpr uint64_t kMetaPrefix = 1ull << 48;
constexpr uint64_t kSizeMask = (1ull << 48) - 1;
constexpr uint64_t kLocDram = 1ull << 63;
constexpr uint64_t kLocOffMask = ~kLocDram;

// Record passed to the index mutation kernels.
struct IndexRec {
  uint64_t klo, khi;
  uint64_t loc;
  uint64_t meta;  // without the occupied bit; the kernel sets it
};

// One copy of `size` bytes from src to dst (either side may be device memory,
// peer device memory, or mapped pinned host memory).
struct CopyDesc {
  uint64_t src;
  uint64_t dst;
  uint64_t size;
  uint64_t flags;  // kCopyHost | kCopyUnpack | kCopyFault
};
constexpr uint64_t kCopyHost = 1;    // either side is host or peer memory (no TMA)
constexpr uint64_t kCopyUnpack = 2;  // src is an INT8-packed block; size = unpacked bytes
constexpr uint64_t kCopyFault = 4;   // self-test: report kErrBounds, touch no memory

// Result of a device lookup for one get request.
struct GetResult {
  uint64_t size;  // block size when found
  uint32_t code;  // CB_FOUND_* | CB_FOUND_NOT_COPIED
  uint32_t pad;
};

// Device-side error bits (written with atomicOr into the store's error word).
constexpr unsigned kErrBounds = 1u;      // arena offset outside the arena
constexpr unsigned kErrTimeout = 2u;     // a bounded wait ran out
constexpr unsigned kErrIndexFull = 4u;   // probe sequence exhausted on insert
constexpr unsigned kErrIndexMiss = 8u;   // update/erase of a key not present

// Bytes of the copy work unit (one CTA iteration). Multiple of 16.
constexpr uint64_t kCopyUnit = 64 * 1024;

}  // namespace cb
