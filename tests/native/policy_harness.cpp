// Test-only C wrapper around the store's host policy (kcj-cascade-v6_b200/
// csrc/policy.cpp), compiled by tests/test_policy.py with g++ so the CPU
// suite can drive allocation, dedup and eviction decisions without a GPU.
#include <string.h>

#include <vector>

#include "policy.hpp"

using namespace cb;

extern "C" {

void *ph_create(uint64_t hbm, uint64_t dram, int semantic) { return new Policy(hbm, dram, semantic != 0); }
void ph_destroy(void *p) { delete static_cast<Policy *>(p); }
void ph_set_compression(void *p, int on) { static_cast<Policy *>(p)->set_compression(on != 0); }
int ph_pin(void *p, uint64_t lo, uint64_t hi) { return static_cast<Policy *>(p)->pin(HKey{lo, hi}) ? 1 : 0; }
int ph_unpin(void *p, uint64_t lo, uint64_t hi) { return static_cast<Policy *>(p)->unpin(HKey{lo, hi}) ? 1 : 0; }

// keys: n*2 u64; out_status: n; out_moves: up to cap records of 7 u64
// (key.lo, key.hi, src_tier, dst_tier, src_off, dst_off, op); returns #moves,
// *n_dropped receives the dropped count (keys into out_dropped, 2 u64 each).
int ph_put(void *p, const uint64_t *keys, const uint64_t *sizes, const uint8_t *prefix, int n, int dedup,
           uint8_t *out_status, uint64_t *out_moves, int cap, uint64_t *out_dropped, int *n_dropped,
           uint64_t *out_places /* n*4: idx, off, tier, size */, int *n_places) {
  Policy *pol = static_cast<Policy *>(p);
  std::vector<HKey> k(n);
  for (int i = 0; i < n; ++i) k[i] = HKey{keys[2 * i], keys[2 * i + 1]};
  PutPlan plan;
  pol->plan_put(k.data(), sizes, prefix, n, dedup != 0, plan);
  pol->commit();
  memcpy(out_status, plan.status.data(), n);
  int m = 0;
  for (const auto &mv : plan.moves) {
    if (m >= cap) break;
    uint64_t *r = out_moves + 7 * m++;
    r[0] = mv.key.lo;
    r[1] = mv.key.hi;
    r[2] = mv.src_tier;
    r[3] = mv.dst_tier;
    r[4] = mv.src_off;
    r[5] = mv.dst_off;
    r[6] = mv.op;
  }
  *n_dropped = (int)plan.dropped.size();
  for (size_t i = 0; i < plan.dropped.size() && (int)i < cap; ++i) {
    out_dropped[2 * i] = plan.dropped[i].lo;
    out_dropped[2 * i + 1] = plan.dropped[i].hi;
  }
  *n_places = (int)plan.places.size();
  for (size_t i = 0; i < plan.places.size() && (int)i < n; ++i) {
    out_places[4 * i] = (uint64_t)plan.places[i].idx;
    out_places[4 * i + 1] = plan.places[i].off;
    out_places[4 * i + 2] = plan.places[i].tier;
    out_places[4 * i + 3] = plan.places[i].size;
  }
  return m;
}

// Returns tier (0 HBM, 1 DRAM) or -1 when absent; *off receives the offset.
int ph_find(void *p, uint64_t lo, uint64_t hi, uint64_t *off) {
  const BlockMeta *m = static_cast<Policy *>(p)->find(HKey{lo, hi});
  if (!m) return -1;
  *off = m->off;
  return m->tier;
}

void ph_touch(void *p, uint64_t lo, uint64_t hi) { static_cast<Policy *>(p)->touch(HKey{lo, hi}); }

int ph_promote(void *p, uint64_t lo, uint64_t hi) {
  std::vector<TierMove> moves;
  std::vector<HKey> dropped;
  Policy *pol = static_cast<Policy *>(p);
  const bool ok = pol->plan_promote(HKey{lo, hi}, moves, dropped);
  pol->commit();
  return ok ? (int)moves.size() : -1;
}

uint64_t ph_evict(void *p, uint64_t bytes) {
  std::vector<TierMove> moves;
  std::vector<HKey> dropped;
  Policy *pol = static_cast<Policy *>(p);
  const uint64_t r = pol->plan_evict(bytes, moves, dropped);
  pol->commit();
  return r;
}

// counters: hbm_used, dram_used, size, dedup_hits, dedup_bytes, gpu_evictions,
// dram_evictions, dropped, prefix_blocks, promotions, compression_savings
void ph_counters(void *p, uint64_t *out) {
  Policy *pol = static_cast<Policy *>(p);
  const PolicyCounters &c = pol->counters();
  out[0] = pol->hbm_used();
  out[1] = pol->dram_used();
  out[2] = pol->size();
  out[3] = c.dedup_hits;
  out[4] = c.dedup_bytes_saved;
  out[5] = c.gpu_evictions;
  out[6] = c.dram_evictions;
  out[7] = c.dropped_blocks;
  out[8] = c.prefix_blocks;
  out[9] = c.promotions;
  out[10] = c.compression_savings;
}

// Returns the block's size (its unpacked size once packed) and packed flag.
int ph_size(void *p, uint64_t lo, uint64_t hi, uint64_t *size) {
  const BlockMeta *m = static_cast<Policy *>(p)->find(HKey{lo, hi});
  if (!m) return -1;
  *size = m->size;
  return m->packed;
}

// Extent allocator checks.
void *ph_alloc_create(uint64_t cap) { return new ExtentAllocator(cap, 256); }
void ph_alloc_destroy(void *a) { delete static_cast<ExtentAllocator *>(a); }
uint64_t ph_alloc(void *a, uint64_t size) { return static_cast<ExtentAllocator *>(a)->alloc(size); }
void ph_free(void *a, uint64_t off, uint64_t size) { static_cast<ExtentAllocator *>(a)->free(off, size); }
uint64_t ph_alloc_free_bytes(void *a) { return static_cast<ExtentAllocator *>(a)->free_bytes(); }
uint64_t ph_alloc_extents(void *a) { return static_cast<ExtentAllocator *>(a)->num_extents(); }
uint64_t ph_alloc_largest(void *a) { return static_cast<ExtentAllocator *>(a)->largest_free(); }
}
