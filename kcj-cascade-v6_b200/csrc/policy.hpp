// Host-side placement policy of the B200 store: extent allocators for the HBM
// slab pool and the pinned DRAM arena, the authoritative block metadata, LRU
// order, sequential dedup, and prefix-protected eviction / promotion planning.
//
// It never touches device memory: it only decides. The store turns its plans
// into batched kernels (scatter, tier moves, index updates). Keeping it free of
// CUDA lets the CPU test-suite drive it directly.
//
// Reference behaviour restated here:
//   * dedup: DistributedStore::put / put_batch (src/distributed_backend.cpp:
//     601-608, 813-841) - a block is a hit iff its key was stored earlier in
//     stream order (including earlier in the same batch);
//   * pool allocation: GPUMemoryPool::alloc/free (src/gpu_backend.cu:81-160)
//     and DistributedDRAMBackend::allocate/deallocate
//     (src/distributed_backend.cpp:88-158) - best fit with coalescing;
//     here O(log n) with ordered maps instead of an O(n) list scan;
//   * eviction: GPUBackend::evict_lru_semantic / evict_for_space
//     (src/gpu_backend.cu:482-537) - never a prefix block while a non-prefix
//     block is evictable, fall back to prefix blocks when nothing else is left;
//     victims go to the DRAM tier (DistributedStore::evict_gpu_to_dram,
//     src/distributed_backend.cpp:876-941);
//   * DRAM eviction: DistributedDRAMBackend::evict_for_space
//     (src/distributed_backend.cpp:240-284) - LRU, prefix blocks skipped, no
//     fallback; with no Lustre tier an evicted DRAM block is dropped.
//   * INT8 KV compression (kv_compression): DistributedStore keeps HBM blocks
//     as they are and stores DRAM-tier copies of blocks >= 64 B in the
//     KVCompressor format (src/distributed_backend.cpp:611-620, :898-903;
//     src/cascade_core.cpp:908-967): 8 + size/2 bytes in DRAM, and a read
//     returns (size/2)*2 bytes. Such a block is "packed": its DRAM footprint
//     is 8 + size/2 and its size from then on is the even unpacked size.
// Victim order is exact LRU (the reference approximates it per shard,
// src/cascade_core.cpp:160-221); order is not a parity target, the
// protection rule is.
#pragma once

#include <stdint.h>

#include <list>
#include <map>
#include <set>
#include <unordered_map>
#include <utility>
#include <vector>

namespace cb {

struct HKey {
  uint64_t lo, hi;
  bool operator==(const HKey &o) const { return lo == o.lo && hi == o.hi; }
};
struct HKeyHash {
  size_t operator()(const HKey &k) const { return (size_t)(k.hi ^ (k.lo * 0x9E3779B97F4A7C15ull)); }
};

// Best-fit extent allocator with coalescing (granule-aligned).
class ExtentAllocator {
 public:
  ExtentAllocator() = default;
  ExtentAllocator(uint64_t capacity, uint64_t granule) { reset(capacity, granule); }
  void reset(uint64_t capacity, uint64_t granule);
  // Returns the offset, or UINT64_MAX when no extent fits.
  uint64_t alloc(uint64_t size);
  void free(uint64_t off, uint64_t size);
  uint64_t rounded(uint64_t size) const { return (size + granule_ - 1) / granule_ * granule_; }
  uint64_t capacity() const { return capacity_; }
  uint64_t free_bytes() const { return free_bytes_; }
  uint64_t largest_free() const;
  size_t num_extents() const { return by_off_.size(); }

 private:
  uint64_t capacity_ = 0, granule_ = 256, free_bytes_ = 0;
  std::map<uint64_t, uint64_t> by_off_;          // offset -> size
  std::set<std::pair<uint64_t, uint64_t>> by_sz_; // (size, offset)
  void insert_extent(uint64_t off, uint64_t size);
  void erase_extent(uint64_t off, uint64_t size);
};

enum : uint8_t { kTierHbm = 0, kTierDram = 1 };

// INT8 packing of DRAM-tier blocks (KVCompressor, include/cascade.hpp:386-418).
constexpr uint64_t kPackHeaderBytes = 8;  // [f32 scale][i8 zero point][3 pad]
constexpr uint64_t kPackMinBytes = 64;    // smaller blocks are stored as they are
// A packed block starts kPackLead bytes into its (256-byte aligned) extent so
// that its int8 payload, after the 8-byte header, is 16-byte aligned.
constexpr uint64_t kPackLead = 8;
inline uint64_t packed_bytes(uint64_t size) { return kPackHeaderBytes + size / 2; }

// Tier moves of blocks of at least this many bytes go through the copy
// engines (packed ones through an HBM staging area of at most
// kPackStagingBytes per direction; the rest use the SM kernels).
constexpr uint64_t kDmaMinBytes = 256 * 1024;
constexpr uint64_t kPackStagingBytes = 1ull << 30;

// How a tier move transforms the bytes it moves.
enum : uint8_t { kMoveCopy = 0, kMovePack = 1, kMoveUnpack = 2 };

struct BlockMeta {
  uint64_t off = 0;
  uint64_t size = 0;
  uint8_t tier = kTierHbm;
  uint8_t prefix = 0;
  uint8_t pending = 0;  // placed by the batch being planned; not evictable yet
  uint8_t packed = 0;   // DRAM copy in the INT8 format (size is then even)
  uint32_t pins = 0;    // outstanding zero-copy views: never a victim, never moved
  uint64_t stamp = 0;   // recency (larger = more recent)
  std::list<HKey>::iterator lru;
};

// A tier move the store executes from (src_tier, src_off) to (dst_tier,
// dst_off); the offsets are those of the block's first byte. Moves of one
// plan run in vector order. size = bytes on the plain side: kMoveCopy copies
// size bytes, kMovePack packs a size-byte block into packed_bytes(size)
// bytes, kMoveUnpack unpacks into size (even) bytes.
struct TierMove {
  HKey key;
  uint8_t src_tier, dst_tier;
  uint64_t src_off, dst_off, size;
  uint8_t op = kMoveCopy;
  // Set by the store: a device address holding the block's (unpacked) bytes
  // to read instead of the source tier (a promotion after a get that has
  // just copied the block into a device buffer). 0 = read the source tier.
  uint64_t src_dev = 0;
};

struct Placement {
  int32_t idx;  // batch index
  HKey key;
  uint64_t off;  // offset of the block's first byte in the tier's arena
  uint64_t size;
  uint8_t prefix;
  uint8_t tier;  // kTierHbm normally; kTierDram when larger than the HBM pool
  uint8_t packed = 0;  // DRAM placement in the INT8 format (size = source bytes)
};

struct PutPlan {
  std::vector<uint8_t> status;      // per item: 0 stored, 1 dedup, 2 failed
  std::vector<Placement> places;    // new blocks to scatter into HBM
  std::vector<TierMove> moves;      // demotions to run BEFORE the scatter
  std::vector<HKey> dropped;        // blocks dropped from the store (index erase)
  void clear() {
    status.clear();
    places.clear();
    moves.clear();
    dropped.clear();
  }
};

struct PolicyCounters {
  uint64_t dedup_hits = 0, dedup_bytes_saved = 0;
  uint64_t gpu_evictions = 0, dram_evictions = 0;
  uint64_t evicted_bytes = 0, promoted_bytes = 0, promotions = 0;
  uint64_t dropped_blocks = 0, prefix_blocks = 0;
  uint64_t compression_savings = 0;  // bytes saved by packing into DRAM
};

class Policy {
 public:
  Policy(uint64_t hbm_capacity, uint64_t dram_capacity, bool semantic_eviction,
         uint64_t granule = 256);

  // Sequential dedup + placement of a batch (see file comment). Placements
  // stay pending until commit(); they are never chosen as victims inside the
  // batch that placed them.
  void plan_put(const HKey *keys, const uint64_t *sizes, const uint8_t *prefix, int n,
                bool dedup_enabled, PutPlan &plan);
  void commit();

  // Bring a DRAM-tier block back to HBM (may demote others first).
  // Appends the promotion move last. Returns false when it cannot fit.
  bool plan_promote(const HKey &k, std::vector<TierMove> &moves, std::vector<HKey> &dropped);

  // Demote HBM blocks until `bytes` of HBM are free (cb_evict).
  uint64_t plan_evict(uint64_t bytes, std::vector<TierMove> &moves, std::vector<HKey> &dropped);

  const BlockMeta *find(const HKey &k) const;
  void touch(const HKey &k);  // mark most recently used
  // find + touch with one lookup (a get's hit)
  const BlockMeta *find_touch(const HKey &k);
  // Keep a block out of every victim choice until commit() (a get is still
  // reading it while this plan's moves run).
  void protect(const HKey &k);
  // Zero-copy views: a pinned block is never chosen as a victim (so it is
  // neither moved nor dropped) until every pin is released.
  bool pin(const HKey &k);
  bool unpin(const HKey &k);
  uint64_t pinned_blocks() const { return pinned_; }
  void clear();

  uint64_t hbm_used() const { return hbm_used_; }
  uint64_t dram_used() const { return dram_used_; }
  uint64_t hbm_capacity() const { return hbm_cap_; }
  uint64_t dram_capacity() const { return dram_cap_; }
  size_t size() const { return map_.size(); }
  const PolicyCounters &counters() const { return ctr_; }
  void reset_counters() { ctr_ = PolicyCounters{}; }
  const ExtentAllocator &hbm_alloc() const { return hbm_; }
  // Bytes of new blocks one plan_put may place straight into the DRAM tier
  // (counted as 256-byte-rounded block sizes); a new block that cannot get
  // HBM beyond that fails. Unlimited on one GPU; on a DHT owner the size of
  // its inbox, through which remote writers hand such blocks over.
  void set_direct_dram_budget(uint64_t bytes) { direct_dram_budget_ = bytes; }
  // INT8 packing of DRAM-tier blocks >= kPackMinBytes (kv_compression).
  void set_compression(bool on) { compress_ = on; }
  bool compression() const { return compress_; }
  // Bytes a block holds in its tier (logical, the reference's used bytes).
  static uint64_t footprint(const BlockMeta &m) { return m.packed ? packed_bytes(m.size) : m.size; }
  // Bytes of its extent in the arena (a packed block starts kPackLead in).
  static uint64_t extent_bytes(const BlockMeta &m) { return m.packed ? kPackLead + packed_bytes(m.size) : m.size; }
  // Byte offset of the block's first byte in its tier's arena.
  static uint64_t data_offset(const BlockMeta &m) { return m.off + (m.packed ? kPackLead : 0); }
  template <class F>
  void for_each(F f) const {
    for (const auto &kv : map_) f(kv.first, kv.second);
  }

 private:
  bool make_hbm_room(uint64_t size, std::vector<TierMove> &moves, std::vector<HKey> &dropped);
  // Room for a block holding `size` bytes in an extent of `extent` bytes.
  bool make_dram_room(uint64_t size, uint64_t extent, std::vector<HKey> &dropped);
  bool demote_one(std::vector<TierMove> &moves, std::vector<HKey> &dropped);
  bool pick_victim(uint8_t tier, bool prefix_fallback, HKey &out) const;
  void drop(const HKey &k, std::vector<HKey> &dropped);

  uint64_t hbm_cap_, dram_cap_;
  bool semantic_;
  uint64_t direct_dram_budget_ = UINT64_MAX;
  bool compress_ = false;
  ExtentAllocator hbm_, dram_;
  uint64_t hbm_used_ = 0, dram_used_ = 0;  // logical bytes (reference used_)
  std::unordered_map<HKey, BlockMeta, HKeyHash> map_;
  // LRU lists, front = most recent: [tier][prefix]
  std::list<HKey> lru_[2][2];
  std::vector<BlockMeta *> pending_;  // marked pending until commit (never erased before it)
  std::vector<std::pair<uint64_t, uint64_t>> deferred_free_;  // DRAM extents freed at commit
  uint64_t clock_ = 0;
  uint64_t pinned_ = 0;  // blocks with pins > 0
  PolicyCounters ctr_;
};

}  // namespace cb
