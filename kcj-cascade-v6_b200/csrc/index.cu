// Device-resident block index: open addressing over 32-byte slots (one
// sector each), linear probing from slot_hash(key). It is the GPU form of the
// location index the reference keeps in host hash maps
// (ShardedIndex, src/cascade_core.cpp:71-247; DistributedIndex,
// include/cascade_distributed.hpp:86-156): kernels resolve a batch of keys to
// pool addresses without a host round trip, which the DHT owner side needs.
//
// Mutations come from the host policy, which guarantees that an inserted key
// is absent and that an updated or erased key is present; mutation kernels
// are stream-ordered with lookups, so a slot is never read while written.
#include "kernels.cuh"
#include "kvquant.cuh"

namespace cb {

namespace {

constexpr int kThreads = 256;

CB_D unsigned long long load_meta(const Slot *s) {
  return *reinterpret_cast<const volatile unsigned long long *>(&s->meta);
}

__global__ void index_insert_kernel(Slot *table, uint64_t mask, const IndexRec *__restrict__ recs,
                                    int n, unsigned *err) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const IndexRec r = recs[i];
  const Key k{r.klo, r.khi};
  const uint64_t h = slot_hash(k);
  for (uint64_t probe = 0; probe <= mask; ++probe) {
    Slot *s = &table[(h + probe) & mask];
    const unsigned long long m = load_meta(s);
    if (m & (kMetaOccupied | kMetaClaim)) continue;
    // Empty or tombstone: claim it, fill it, then publish the meta word.
    if (atomicCAS(&s->meta, m, (unsigned long long)kMetaClaim) == m) {
      s->klo = r.klo;
      s->khi = r.khi;
      s->loc = r.loc;
      __threadfence();
      atomicExch(&s->meta, (unsigned long long)(r.meta | kMetaOccupied));
      return;
    }
  }
  atomicOr(err, kErrIndexFull);
}

// Finds the slot of key k; nullptr when absent.
CB_D Slot *find_slot(Slot *table, uint64_t mask, const Key &k) {
  const uint64_t h = slot_hash(k);
  for (uint64_t probe = 0; probe <= mask; ++probe) {
    Slot *s = &table[(h + probe) & mask];
    const unsigned long long m = load_meta(s);
    if (m == 0) return nullptr;  // never-used slot ends the probe sequence
    if ((m & kMetaOccupied) && s->klo == k.lo && s->khi == k.hi) return s;
  }
  return nullptr;
}

__global__ void index_update_kernel(Slot *table, uint64_t mask, const IndexRec *__restrict__ recs,
                                    int n, unsigned *err) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const IndexRec r = recs[i];
  Slot *s = find_slot(table, mask, Key{r.klo, r.khi});
  if (!s) {
    atomicOr(err, kErrIndexMiss);
    return;
  }
  s->loc = r.loc;
  __threadfence();
  atomicExch(&s->meta, (unsigned long long)(r.meta | kMetaOccupied));
}

__global__ void index_erase_kernel(Slot *table, uint64_t mask, const IndexRec *__restrict__ recs,
                                   int n, unsigned *err) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const IndexRec r = recs[i];
  Slot *s = find_slot(table, mask, Key{r.klo, r.khi});
  if (!s) {
    atomicOr(err, kErrIndexMiss);
    return;
  }
  atomicExch(&s->meta, (unsigned long long)kMetaTomb);
}

__global__ void index_lookup_kernel(LookupArgs a) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= a.n) return;
  const Key k = a.keys[i];
  const uint64_t h = slot_hash(k);
  CopyDesc d{0, a.outs[i], 0, 0};
  GetResult res{0, CB_FOUND_MISS, 0};
  for (uint64_t probe = 0; probe <= a.mask; ++probe) {
    const Slot *s = &a.table[(h + probe) & a.mask];
    const uint64_t m = s->meta;
    if (m == 0) break;
    if (!(m & kMetaOccupied) || s->klo != k.lo || s->khi != k.hi) continue;
    const uint64_t loc = s->loc;
    const uint64_t size = m & kSizeMask;
    const bool dram = (loc & kLocDram) != 0;
    const uint64_t off = loc & kLocOffMask;
    const bool packed = dram && (m & kMetaPacked);
    const uint64_t foot = packed ? packed_size(size) : size;  // bytes held in the arena
    const uint64_t base = dram ? a.dram_base : a.pool_base;
    const uint64_t bytes = dram ? a.dram_bytes : a.pool_bytes;
    if (off > bytes || foot > bytes - off) {
      atomicOr(a.err, kErrBounds);
      break;
    }
    res.size = size;
    res.code = dram ? a.code_dram : a.code_hbm;
    const uint64_t reserved = (uint64_t)(a.unit_start[i + 1] - a.unit_start[i]) * kCopyUnit;
    if (size <= a.caps[i] && size > reserved) {
      // Host metadata and device index disagree on the size: copy nothing.
      atomicOr(a.err, kErrBounds);
      res.code |= CB_FOUND_NOT_COPIED;
    } else if (size <= a.caps[i]) {
      d.src = base + off;
      d.size = size;
      d.flags = dram ? (kCopyHost | (packed ? kCopyUnpack : 0)) : 0;
    } else {
      res.code |= CB_FOUND_NOT_COPIED;
    }
    break;
  }
  a.desc[i] = d;
  a.res[i] = res;
}

// Owner side of a DHT lookup: for each received key, its slot's location
// and meta words (meta = 0 when absent). `table` may be a peer's index
// mapped into this process (one-sided probes).
__global__ void index_serve_kernel(const Slot *table, uint64_t mask, const Key *__restrict__ keys, int n,
                                   uint64_t *__restrict__ reps) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const Key k = keys[i];
  const uint64_t h = slot_hash(k);
  uint64_t loc = 0, meta = 0;
  for (uint64_t probe = 0; probe <= mask; ++probe) {
    const Slot *s = &table[(h + probe) & mask];
    const uint64_t m = load_meta(s);
    if (m == 0) break;
    if ((m & kMetaOccupied) && s->klo == k.lo && s->khi == k.hi) {
      loc = s->loc;
      meta = m;
      break;
    }
  }
  reps[2 * i] = loc;
  reps[2 * i + 1] = meta;
}

inline int blocks_for(int n) { return (n + kThreads - 1) / kThreads; }

}  // namespace

cudaError_t launch_index_insert(Slot *table, uint64_t mask, const IndexRec *recs, int n,
                                unsigned *d_err, cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  index_insert_kernel<<<blocks_for(n), kThreads, 0, stream>>>(table, mask, recs, n, d_err);
  return cudaGetLastError();
}

cudaError_t launch_index_update(Slot *table, uint64_t mask, const IndexRec *recs, int n,
                                unsigned *d_err, cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  index_update_kernel<<<blocks_for(n), kThreads, 0, stream>>>(table, mask, recs, n, d_err);
  return cudaGetLastError();
}

cudaError_t launch_index_erase(Slot *table, uint64_t mask, const IndexRec *recs, int n,
                               unsigned *d_err, cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  index_erase_kernel<<<blocks_for(n), kThreads, 0, stream>>>(table, mask, recs, n, d_err);
  return cudaGetLastError();
}

cudaError_t launch_index_serve(const Slot *table, uint64_t mask, const Key *keys, int n, uint64_t *reps,
                               cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  index_serve_kernel<<<blocks_for(n), kThreads, 0, stream>>>(table, mask, keys, n, reps);
  return cudaGetLastError();
}

cudaError_t launch_index_lookup(const LookupArgs &a, cudaStream_t stream) {
  if (a.n <= 0) return cudaSuccess;
  index_lookup_kernel<<<blocks_for(a.n), kThreads, 0, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace cb
