// Host-side placement policy (see policy.hpp for the reference behaviour).
#include "policy.hpp"

#include <algorithm>
#include <iterator>

namespace cb {

// ---------------------------------------------------------------- allocator

void ExtentAllocator::reset(uint64_t capacity, uint64_t granule) {
  granule_ = granule ? granule : 256;
  capacity_ = capacity / granule_ * granule_;
  by_off_.clear();
  by_sz_.clear();
  free_bytes_ = 0;
  if (capacity_) insert_extent(0, capacity_);
  free_bytes_ = capacity_;
}

void ExtentAllocator::insert_extent(uint64_t off, uint64_t size) {
  by_off_.emplace(off, size);
  by_sz_.emplace(size, off);
}

void ExtentAllocator::erase_extent(uint64_t off, uint64_t size) {
  by_off_.erase(off);
  by_sz_.erase({size, off});
}

uint64_t ExtentAllocator::largest_free() const {
  return by_sz_.empty() ? 0 : by_sz_.rbegin()->first;
}

uint64_t ExtentAllocator::alloc(uint64_t size) {
  const uint64_t r = std::max(rounded(size), granule_);
  auto it = by_sz_.lower_bound({r, 0});  // best fit: smallest extent >= r
  if (it == by_sz_.end()) return UINT64_MAX;
  const uint64_t sz = it->first, off = it->second;
  erase_extent(off, sz);
  if (sz > r) insert_extent(off + r, sz - r);
  free_bytes_ -= r;
  return off;
}

void ExtentAllocator::free(uint64_t off, uint64_t size) {
  uint64_t r = std::max(rounded(size), granule_);
  uint64_t start = off;
  auto next = by_off_.lower_bound(off);
  if (next != by_off_.end() && off + r == next->first) {
    const uint64_t nsz = next->second, noff = next->first;
    erase_extent(noff, nsz);
    r += nsz;
  }
  next = by_off_.lower_bound(off);
  if (next != by_off_.begin()) {
    auto prev = std::prev(next);
    if (prev->first + prev->second == off) {
      const uint64_t poff = prev->first, psz = prev->second;
      erase_extent(poff, psz);
      start = poff;
      r += psz;
    }
  }
  insert_extent(start, r);
  free_bytes_ += std::max(rounded(size), granule_);
}

// ------------------------------------------------------------------- policy

Policy::Policy(uint64_t hbm_capacity, uint64_t dram_capacity, bool semantic_eviction,
               uint64_t granule)
    : hbm_cap_(hbm_capacity), dram_cap_(dram_capacity), semantic_(semantic_eviction),
      hbm_(hbm_capacity, granule), dram_(dram_capacity, granule) {}

const BlockMeta *Policy::find(const HKey &k) const {
  auto it = map_.find(k);
  return it == map_.end() ? nullptr : &it->second;
}

void Policy::touch(const HKey &k) { find_touch(k); }

const BlockMeta *Policy::find_touch(const HKey &k) {
  auto it = map_.find(k);
  if (it == map_.end()) return nullptr;
  BlockMeta &m = it->second;
  auto &lst = lru_[m.tier][m.prefix];
  lst.splice(lst.begin(), lst, m.lru);
  m.stamp = ++clock_;
  return &m;
}

bool Policy::pin(const HKey &k) {
  auto it = map_.find(k);
  if (it == map_.end()) return false;
  if (it->second.pins++ == 0) pinned_++;
  return true;
}

bool Policy::unpin(const HKey &k) {
  auto it = map_.find(k);
  if (it == map_.end() || it->second.pins == 0) return false;
  if (--it->second.pins == 0) pinned_--;
  return true;
}

void Policy::protect(const HKey &k) {
  auto it = map_.find(k);
  if (it == map_.end() || it->second.pending) return;
  it->second.pending = 1;
  pending_.push_back(&it->second);
}

void Policy::clear() {
  map_.clear();
  for (auto &t : lru_)
    for (auto &l : t) l.clear();
  pending_.clear();
  deferred_free_.clear();
  clock_ = 0;
  pinned_ = 0;
  hbm_.reset(hbm_cap_, 256);
  dram_.reset(dram_cap_, 256);
  hbm_used_ = dram_used_ = 0;
  ctr_ = PolicyCounters{};
}

bool Policy::pick_victim(uint8_t tier, bool prefix_fallback, HKey &out) const {
  // Semantic eviction: the least recently used non-prefix block; prefix blocks
  // only when no non-prefix block is evictable and the tier allows it (HBM:
  // gpu_backend.cu:482-492 falls back; DRAM: distributed_backend.cpp:257-261
  // never does). Without it: plain LRU over both lists (older tail wins).
  const HKey *cand[2] = {nullptr, nullptr};
  for (int p = 0; p < 2; ++p) {
    const std::list<HKey> &lst = lru_[tier][p];
    for (auto it = lst.rbegin(); it != lst.rend(); ++it) {
      const BlockMeta &m = map_.at(*it);
      if (!m.pending && !m.pins) {
        cand[p] = &*it;
        break;
      }
    }
  }
  if (semantic_) {
    const HKey *c = cand[0] ? cand[0] : (prefix_fallback ? cand[1] : nullptr);
    if (!c) return false;
    out = *c;
    return true;
  }
  if (!cand[0] || !cand[1]) {
    const HKey *c = cand[0] ? cand[0] : cand[1];
    if (!c) return false;
    out = *c;
    return true;
  }
  out = map_.at(*cand[0]).stamp <= map_.at(*cand[1]).stamp ? *cand[0] : *cand[1];
  return true;
}

void Policy::drop(const HKey &k, std::vector<HKey> &dropped) {
  auto it = map_.find(k);
  if (it == map_.end()) return;
  BlockMeta &m = it->second;
  if (m.tier == kTierHbm) {
    hbm_.free(m.off, m.size);
    hbm_used_ -= m.size;
  } else {
    dram_.free(m.off, extent_bytes(m));
    dram_used_ -= footprint(m);
    ctr_.dram_evictions++;
  }
  lru_[m.tier][m.prefix].erase(m.lru);
  if (m.prefix && ctr_.prefix_blocks) ctr_.prefix_blocks--;
  ctr_.dropped_blocks++;
  dropped.push_back(k);
  map_.erase(it);
}

bool Policy::make_dram_room(uint64_t size, uint64_t extent, std::vector<HKey> &dropped) {
  if (dram_cap_ == 0 || size > dram_cap_ || extent > dram_.capacity()) return false;
  const uint64_t need = std::max(dram_.rounded(extent), (uint64_t)256);
  while (dram_used_ + size > dram_cap_ || dram_.largest_free() < need) {
    // DistributedDRAMBackend::evict_for_space: LRU tail, prefix blocks
    // protected with no fallback (distributed_backend.cpp:240-284).
    HKey v;
    if (!pick_victim(kTierDram, false, v)) return false;
    drop(v, dropped);
  }
  return true;
}

bool Policy::demote_one(std::vector<TierMove> &moves, std::vector<HKey> &dropped) {
  HKey v;
  if (!pick_victim(kTierHbm, true, v)) return false;
  BlockMeta &m = map_.at(v);
  ctr_.gpu_evictions++;
  // evict_gpu_to_dram compresses blocks >= 64 B on their way to DRAM
  // (distributed_backend.cpp:898-903).
  const bool pack = compress_ && m.size >= kPackMinBytes;
  const uint64_t dbytes = pack ? packed_bytes(m.size) : m.size;
  const uint64_t dext = pack ? kPackLead + dbytes : dbytes;
  if (!make_dram_room(dbytes, dext, dropped)) {
    // No DRAM room: the reference sends the victim to Lustre
    // (distributed_backend.cpp:915-918); without that tier it is dropped.
    drop(v, dropped);
    return true;
  }
  BlockMeta &mm = map_.at(v);  // make_dram_room never drops pending/HBM blocks
  const uint64_t doff = dram_.alloc(dext);
  moves.push_back(
      TierMove{v, kTierHbm, kTierDram, mm.off, doff + (pack ? kPackLead : 0), mm.size, pack ? kMovePack : kMoveCopy});
  hbm_.free(mm.off, mm.size);
  hbm_used_ -= mm.size;
  dram_used_ += dbytes;
  ctr_.evicted_bytes += mm.size;
  if (pack) {
    ctr_.compression_savings += mm.size - dbytes;
    mm.size &= ~1ull;  // what a read of the packed block returns
    mm.packed = 1;
  }
  auto &src = lru_[kTierHbm][mm.prefix];
  auto &dst = lru_[kTierDram][mm.prefix];
  dst.splice(dst.begin(), src, mm.lru);
  mm.stamp = ++clock_;
  mm.tier = kTierDram;
  mm.off = doff;
  mm.pending = 1;  // moved by this plan: not a DRAM victim inside it
  pending_.push_back(&mm);
  return true;
}

bool Policy::make_hbm_room(uint64_t size, std::vector<TierMove> &moves,
                           std::vector<HKey> &dropped) {
  if (size > hbm_cap_) return false;
  const uint64_t need = std::max(hbm_.rounded(size), (uint64_t)256);
  while (hbm_used_ + size > hbm_cap_ || hbm_.largest_free() < need) {
    if (!demote_one(moves, dropped)) return false;
  }
  return true;
}

void Policy::plan_put(const HKey *keys, const uint64_t *sizes, const uint8_t *prefix, int n,
                      bool dedup_enabled, PutPlan &plan) {
  plan.clear();
  plan.status.assign(n, 0);
  uint64_t direct_left = direct_dram_budget_;
  for (int i = 0; i < n; ++i) {
    const HKey &k = keys[i];
    const uint64_t size = sizes[i];
    // one hash lookup: a new key's entry is filled below (it is in no LRU
    // list yet, so the demotions that make room never see it) or erased
    const auto ins = map_.try_emplace(k);
    if (!ins.second) {
      // DistributedStore::put: dedup hit (distributed_backend.cpp:604-608).
      // With dedup disabled the GPU tier still refuses a second copy
      // (gpu_backend.cu:302-304) but nothing is counted.
      plan.status[i] = 1;
      if (dedup_enabled) {
        ctr_.dedup_hits++;
        ctr_.dedup_bytes_saved += size;
      }
      continue;
    }
    const uint8_t pf = prefix ? (prefix[i] ? 1 : 0) : 0;
    uint8_t tier = kTierHbm;
    uint64_t off = UINT64_MAX;
    if (make_hbm_room(size, plan.moves, plan.dropped)) {
      off = hbm_.alloc(size);
    }
    bool pack = false;
    const uint64_t staged = (size + 255) / 256 * 256;
    if (off == UINT64_MAX && staged <= direct_left) {
      // Larger than the whole HBM pool (or every HBM block pending): the
      // reference's put still succeeds through its DRAM copy
      // (distributed_backend.cpp:643-652), compressed when kv_compression is
      // on (:615-620).
      pack = compress_ && size >= kPackMinBytes;
      const uint64_t dbytes = pack ? packed_bytes(size) : size;
      const uint64_t dext = pack ? kPackLead + dbytes : dbytes;
      if (make_dram_room(dbytes, dext, plan.dropped)) {
        off = dram_.alloc(dext);
        tier = kTierDram;
        if (direct_left != UINT64_MAX) direct_left -= staged;
      }
    }
    if (off == UINT64_MAX) {
      map_.erase(ins.first);
      plan.status[i] = 2;
      continue;
    }
    if (tier != kTierDram) pack = false;
    BlockMeta &m = ins.first->second;
    m.off = off;
    m.size = pack ? (size & ~1ull) : size;
    m.tier = tier;
    m.prefix = pf;
    m.pending = 1;
    m.packed = pack ? 1 : 0;
    m.stamp = ++clock_;
    auto &lst = lru_[tier][pf];
    lst.push_front(k);
    m.lru = lst.begin();
    pending_.push_back(&m);
    if (tier == kTierHbm) {
      hbm_used_ += size;
    } else {
      dram_used_ += pack ? packed_bytes(size) : size;
      if (pack) ctr_.compression_savings += size - packed_bytes(size);
    }
    if (pf) ctr_.prefix_blocks++;
    plan.places.push_back(Placement{i, k, off + (pack ? kPackLead : 0), size, pf, tier, (uint8_t)(pack ? 1 : 0)});
  }
}

void Policy::commit() {
  for (BlockMeta *m : pending_) m->pending = 0;
  pending_.clear();
  for (const auto &e : deferred_free_) dram_.free(e.first, e.second);
  deferred_free_.clear();
}

bool Policy::plan_promote(const HKey &k, std::vector<TierMove> &moves,
                          std::vector<HKey> &dropped) {
  auto it = map_.find(k);
  if (it == map_.end() || it->second.tier != kTierDram) return false;
  it->second.pending = 1;  // protect the source while making room
  pending_.push_back(&it->second);
  const uint64_t size = it->second.size;
  if (!make_hbm_room(size, moves, dropped)) return false;
  const uint64_t hoff = hbm_.alloc(size);
  if (hoff == UINT64_MAX) return false;
  BlockMeta &m = map_.at(k);
  moves.push_back(TierMove{k, kTierDram, kTierHbm, data_offset(m), hoff, size, m.packed ? kMoveUnpack : kMoveCopy});
  // The DRAM extent is released now; no later move of this plan writes DRAM
  // after promotions read it because the store runs every HBM->DRAM move of a
  // plan before any DRAM->HBM move, and DRAM destinations of those demotions
  // were allocated while this extent was still held.
  deferred_free_.push_back({m.off, extent_bytes(m)});
  dram_used_ -= footprint(m);
  hbm_used_ += size;
  m.packed = 0;
  auto &src = lru_[kTierDram][m.prefix];
  auto &dst = lru_[kTierHbm][m.prefix];
  dst.splice(dst.begin(), src, m.lru);
  m.stamp = ++clock_;
  m.tier = kTierHbm;
  m.off = hoff;
  ctr_.promotions++;
  ctr_.promoted_bytes += size;
  return true;
}

uint64_t Policy::plan_evict(uint64_t bytes, std::vector<TierMove> &moves,
                            std::vector<HKey> &dropped) {
  // GPUBackend::evict_for_space (src/gpu_backend.cu:514-537): demote victims
  // until at least `bytes` have left HBM (or nothing is left to demote).
  const uint64_t before = hbm_used_;
  while (before - hbm_used_ < bytes) {
    if (!demote_one(moves, dropped)) break;
  }
  return before - hbm_used_;
}

}  // namespace cb
