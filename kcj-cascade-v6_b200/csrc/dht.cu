// Multi-GPU hash-sharded DHT: the B200 form of DistributedGPUBackend's
// remote tier (src/distributed_backend.cpp:303-514) and of the replicated
// location index that sync_metadata maintains with MPI_Allgatherv
// (:1323-1382).
//
// One process per GPU, W ranks. Owner(block) = first 8 ID bytes (big-endian)
// mod W. Each rank's HBM slab pool and device index are exported with CUDA
// IPC and mapped into every other rank at attach time, so payloads move by
// direct peer loads/stores over NVLink; only 16-32-byte lookup records travel
// through NCCL (grouped send/recv = all-to-all, preceded by an all-gather of
// the per-peer counts). Every copy whose source or destination is a peer's
// memory (or pinned host memory) runs on the LSU engine: plain 16-byte loads
// and stores. No TMA copy of any kind ever touches peer memory, and no TMA
// multicast is used anywhere.
//
// batch_put : local SHA-256 -> requests to owners -> owners dedup in
//             (source rank, batch index) order, allocate, insert into their
//             index, reply {status, offset} -> writers copy new blocks into
//             the owners' pools -> closing all-reduce (barrier).
// batch_get : keys to owners -> owner index lookup kernel -> replies
//             {location, meta} -> gather kernel reading the owners' pools
//             (the next step's counts all-gather keeps owners from reusing
//             extents before the readers are done).
// Every collective call is made by all ranks in the same order. Waits are
// bounded: a collective that does not finish within the timeout aborts the
// communicator and returns CB_ERR_TIMEOUT.
#include <nccl.h>
#include <string.h>

#include <algorithm>
#include <numeric>
#include <climits>
#include <chrono>
#include <thread>
#include <unordered_set>
#include <vector>

#include "kernels.cuh"
#include "store.hpp"

namespace cb {

namespace {

struct PutReq {
  uint64_t klo, khi, size, flags;  // flags bit 0: prefix
};
struct PutRep {
  uint64_t loc;  // offset | kLocDram
  uint32_t status;
  uint32_t pad;
};
struct Export {
  cudaIpcMemHandle_t pool, table, outbox;
  uint64_t pool_bytes, table_slots, outbox_bytes;
  int32_t device, pad;
};

// A location word with this bit names a byte offset in the owner's outbox:
// HBM through which blocks of the owner's DRAM tier reach peers (peers map
// only each other's HBM, not pinned host memory).
constexpr uint64_t kLocOutbox = 1ull << 62;
constexpr uint64_t kLocOutboxOff = ~(kLocDram | kLocOutbox);

// Index meta word of a block (occupied, packed, prefix, size).
inline uint64_t meta_of(const BlockMeta &m) {
  return kMetaOccupied | (m.size & kSizeMask) | (m.prefix ? kMetaPrefix : 0) | (m.packed ? kMetaPacked : 0);
}

inline uint64_t be_owner(const HKey &k, int world) {
  return (uint64_t)owner_of(Key{k.lo, k.hi}, world);
}

}  // namespace

// Writer side of a DHT batch: the owner rank of every key, the order in
// which the keys are sent (grouped by owner, batch order inside a group) and
// the number of keys per owner. The requests an owner receives are
// therefore in (source rank, batch index) order.
void dht_route(const HKey *keys, int n, int W, int *owner, int *order, uint32_t *scount) {
  for (int r = 0; r < W; ++r) scount[r] = 0;
  for (int i = 0; i < n; ++i) {
    owner[i] = (int)be_owner(keys[i], W);
    scount[owner[i]]++;
  }
  std::vector<uint32_t> pos(W, 0);
  for (int r = 1; r < W; ++r) pos[r] = pos[r - 1] + scount[r - 1];
  for (int i = 0; i < n; ++i) order[pos[owner[i]]++] = i;
}

// Owner side of a DHT put step: the requests of every rank, in (source
// rank, batch index) order, go through the owner's policy with the
// sequential dedup rule of DistributedStore::put (src/distributed_backend.cpp:
// 604-608) - among equal keys of one step the lowest (rank, index) is stored,
// every other one is a dedup hit - and get one reply each {status, location}.
void dht_owner_plan(Policy &policy, const HKey *keys, const uint64_t *sizes, const uint8_t *prefix, uint32_t n,
                    bool dedup, PutPlan &plan, uint32_t *status, uint64_t *loc) {
  policy.plan_put(keys, sizes, prefix, (int)n, dedup, plan);
  for (uint32_t j = 0; j < n; ++j) {
    status[j] = plan.status[j];
    loc[j] = 0;
  }
  for (const Placement &p : plan.places) loc[p.idx] = p.off | (p.tier == kTierDram ? kLocDram : 0);
}

struct DhtState {
  ncclComm_t comm = nullptr;
  int W = 1, me = 0;
  std::vector<uint64_t> pool, pool_bytes, table, slots;
  // Outbox (HBM, exported like the pool): a get stages the DRAM-tier blocks
  // that other ranks requested here, a put receives here the new blocks
  // this owner places straight into its DRAM tier. Reused every step: a
  // put's closing all-reduce, and a get's successor step's opening counts
  // all-gather, keep its contents until every peer is done with them.
  uint8_t *outbox = nullptr;
  uint64_t outbox_bytes = 0;
  std::vector<uint64_t> peer_outbox, peer_outbox_bytes;
  std::vector<int> device;
  std::vector<void *> opened;
  DevBuf d_send, d_recv, d_misc;
  PinnedBuf h_send, h_recv, h_misc;
  double timeout_s = 600.0;

  // Locality-aware placement (DistributedStore::record_access /
  // should_promote_local / promote_to_local_gpu, src/distributed_backend.cpp:
  // 1224-1275; AccessRecord, include/cascade_distributed.hpp:162-180): a
  // block this rank keeps fetching from a peer is copied into a local replica
  // region and served from local HBM afterwards. Blocks are content-addressed
  // and immutable, so a replica never goes stale; evicting one only drops it.
  bool locality = false;
  uint32_t threshold = 3;
  uint8_t *rbase = nullptr;  // replica region (local HBM)
  uint64_t rbytes = 0;
  ExtentAllocator ralloc;
  struct Rep {
    uint64_t off, size;
    std::list<HKey>::iterator lru;  // in rlru unless pinned
    bool pinned;                    // a prefix replica: never dropped for another replica
  };
  std::unordered_map<HKey, Rep, HKeyHash> rmap;
  std::list<HKey> rlru;  // hot-block replicas, front = most recent

  // Prefix registry (DistributedStore::prefix_registry_,
  // include/cascade_distributed.hpp:432): the prefix blocks this rank has
  // stored, and after sync_metadata every prefix block of the cluster.
  std::unordered_set<HKey, HKeyHash> registry;
  bool replicate_prefixes = false;  // DistributedConfig::prefix_replication
  uint64_t prefix_replicas = 0;

  // Frees hot-block replicas, least recently used first, until `size` bytes
  // fit; returns the offset or UINT64_MAX.
  uint64_t alloc_replica(uint64_t size) {
    uint64_t off = ralloc.alloc(size);
    while (off == UINT64_MAX && !rlru.empty()) {
      const HKey v = rlru.back();
      auto it = rmap.find(v);
      ralloc.free(it->second.off, it->second.size);
      rlru.pop_back();
      rmap.erase(it);
      off = ralloc.alloc(size);
    }
    return off;
  }
  struct Access {
    uint32_t total = 0, local = 0, remote = 0, wtotal = 0, wremote = 0;
    float ema = 0.f;
  };
  std::unordered_map<HKey, Access, HKeyHash> access;

  void record_access(const HKey &k, bool remote) {
    Access &a = access[k];
    a.total++;
    a.wtotal++;
    if (remote) {
      a.remote++;
      a.wremote++;
    } else {
      a.local++;
    }
    if (a.wtotal >= 8) {  // AccessRecord::WINDOW_SIZE, EMA_ALPHA = 0.3
      const float cur = static_cast<float>(a.wremote) / a.wtotal;
      a.ema = 0.3f * cur + (1.0f - 0.3f) * a.ema;
      a.wremote = 0;
      a.wtotal = 0;
    }
  }
  bool should_promote(const HKey &k) const {
    auto it = access.find(k);
    return it != access.end() && it->second.total >= threshold && it->second.ema > 0.5f;
  }
  void clear_replicas() {
    rmap.clear();
    rlru.clear();
    access.clear();
    registry.clear();
    prefix_replicas = 0;
    ralloc.reset(rbytes, 256);
  }
};

// ------------------------------------------------------------ plumbing

int Store::dht_nccl(int r, const char *what) {
  if (r == ncclSuccess) return CB_OK;
  if (r == ncclInProgress) {
    const auto t0 = std::chrono::steady_clock::now();
    ncclResult_t st = ncclInProgress;
    while (st == ncclInProgress) {
      if (ncclCommGetAsyncError(dht->comm, &st) != ncclSuccess) break;
      if (st != ncclInProgress) break;
      if (std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() > dht->timeout_s) {
        ncclCommAbort(dht->comm);
        dht->comm = nullptr;
        return fail(CB_ERR_TIMEOUT, "%s: NCCL call did not complete", what);
      }
      std::this_thread::yield();
    }
    if (st == ncclSuccess) return CB_OK;
    r = st;
  }
  return fail(CB_ERR_NCCL, "%s: %s", what, ncclGetErrorString((ncclResult_t)r));
}

// Waits for the stream while watching the communicator (bounded).
int Store::dht_sync(cudaStream_t st) {
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    cudaError_t e = cudaStreamQuery(st);
    if (e == cudaSuccess) break;
    if (e != cudaErrorNotReady) return cuda_fail(e, "DHT stream");
    ncclResult_t ar = ncclSuccess;
    ncclCommGetAsyncError(dht->comm, &ar);
    if (ar != ncclSuccess && ar != ncclInProgress) {
      ncclCommAbort(dht->comm);
      dht->comm = nullptr;
      return fail(CB_ERR_NCCL, "DHT collective failed: %s", ncclGetErrorString(ar));
    }
    if (std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() > dht->timeout_s) {
      ncclCommAbort(dht->comm);
      dht->comm = nullptr;
      return fail(CB_ERR_TIMEOUT, "DHT collective timed out");
    }
    std::this_thread::yield();
  }
  return CB_OK;
}

// End of a collective step: the device error word comes back with the
// stream's last copy, so one bounded wait covers both.
int Store::dht_finish(cudaStream_t st) {
  CB_TRY_CUDA(cudaMemcpyAsync(h_err.ptr, d_err, sizeof(unsigned), cudaMemcpyDeviceToHost, st), "D2H err");
  int rc = dht_sync(st);
  if (rc) return rc;
  resolve_prof();
  if (*static_cast<unsigned *>(h_err.ptr) == 0) return CB_OK;
  return check_device_error(st);  // reads it again, clears it and reports
}

// All-gather of the per-destination counts: on return rcount[r] = number of
// records rank r sends to this rank.
int Store::dht_counts(const uint32_t *scount, uint32_t *rcount, cudaStream_t st) {
  const int W = dht->W;
  CB_TRY_CUDA(dht->h_misc.ensure(4ull * W * (W + 1)), "pinned");
  CB_TRY_CUDA(dht->d_misc.ensure(4ull * W * (W + 1)), "device");
  uint32_t *h = static_cast<uint32_t *>(dht->h_misc.ptr);
  uint32_t *d = static_cast<uint32_t *>(dht->d_misc.ptr);
  memcpy(h, scount, 4ull * W);
  CB_TRY_CUDA(cudaMemcpyAsync(d, h, 4ull * W, cudaMemcpyHostToDevice, st), "H2D counts");
  int rc = timed_coll(4ull * W, st, [&] {
    return dht_nccl(ncclAllGather(d, d + W, (size_t)W, ncclUint32, dht->comm, st), "ncclAllGather(counts)");
  });
  if (rc) return rc;
  CB_TRY_CUDA(cudaMemcpyAsync(h + W, d + W, 4ull * W * W, cudaMemcpyDeviceToHost, st), "D2H counts");
  rc = dht_sync(st);
  if (rc) return rc;
  for (int r = 0; r < W; ++r) rcount[r] = h[W + r * W + dht->me];
  return CB_OK;
}

// Variable all-to-all of fixed-size records (grouped ncclSend/ncclRecv).
int Store::dht_alltoallv(const void *d_send, const uint32_t *scount, void *d_recv, const uint32_t *rcount,
                         size_t rec, cudaStream_t st) {
  uint64_t sent = 0;
  for (int r = 0; r < dht->W; ++r) sent += scount[r] * rec;
  return timed_coll(sent, st, [&] { return dht_alltoallv_group(d_send, scount, d_recv, rcount, rec, st); });
}

int Store::dht_alltoallv_group(const void *d_send, const uint32_t *scount, void *d_recv, const uint32_t *rcount,
                               size_t rec, cudaStream_t st) {
  const int W = dht->W;
  int rc = dht_nccl(ncclGroupStart(), "ncclGroupStart");
  if (rc) return rc;
  // Inside the group the calls only enqueue (completion is checked at
  // ncclGroupEnd); a failed enqueue still closes the group, so no NCCL group
  // stays open on this thread for the caller's next NCCL call.
  auto enqueued = [&](ncclResult_t r, const char *what) -> int {
    if (r == ncclSuccess || r == ncclInProgress) return CB_OK;
    ncclGroupEnd();
    return fail(CB_ERR_NCCL, "%s: %s", what, ncclGetErrorString(r));
  };
  size_t so = 0, ro = 0;
  for (int r = 0; r < W; ++r) {
    if (scount[r]) {
      rc = enqueued(
          ncclSend(static_cast<const uint8_t *>(d_send) + so, scount[r] * rec, ncclUint8, r, dht->comm, st),
          "ncclSend");
      if (rc) return rc;
    }
    if (rcount[r]) {
      rc = enqueued(ncclRecv(static_cast<uint8_t *>(d_recv) + ro, rcount[r] * rec, ncclUint8, r, dht->comm, st),
                    "ncclRecv");
      if (rc) return rc;
    }
    so += scount[r] * rec;
    ro += rcount[r] * rec;
  }
  return dht_nccl(ncclGroupEnd(), "ncclGroupEnd");
}

int Store::dht_barrier() {
  if (!dht || !dht->comm) return fail(CB_ERR_STATE, "DHT not attached (or its communicator was aborted after a failure)");
  CB_TRY_CUDA(dht->d_misc.ensure(256), "device");
  int rc = dht_nccl(ncclAllReduce(dht->d_misc.ptr, dht->d_misc.ptr, 1, ncclInt32, ncclSum, dht->comm, own_stream),
                    "ncclAllReduce(barrier)");
  if (rc) return rc;
  return dht_sync(own_stream);
}

// ------------------------------------------------------------ attach

int Store::dht_attach(int r, int W, const uint8_t *uid) {
  if (world > 1 || dht) return fail(CB_ERR_STATE, "already attached to a DHT");
  if (W < 2 || r < 0 || r >= W) return fail(CB_ERR_ARG, "bad rank/world");
  if (!pool) return fail(CB_ERR_STATE, "a DHT member needs an HBM pool (gpu_capacity_bytes > 0)");
  // The index is mapped by peers: size it once, it is never reallocated.
  const int want_log2 = std::max(cfg.index_log2 > 0 ? cfg.index_log2 : 16, 20);
  if (table_slots < (1ull << want_log2)) {
    int rc = CB_OK;
    if (policy.size() == 0) {
      CB_TRY_CUDA(alloc_table(1ull << want_log2), "index");
    } else {
      rc = reserve_index((1ull << want_log2) / 2, own_stream);
      if (rc) return rc;
    }
  }
  dht = new DhtState;
  dht->W = W;
  dht->me = r;
  if (cfg.collective_timeout_ms) dht->timeout_s = (double)cfg.collective_timeout_ms / 1000.0;
  ncclUniqueId id;
  memcpy(&id, uid, sizeof id);
  ncclConfig_t nc = NCCL_CONFIG_INITIALIZER;
  nc.blocking = 0;
  nc.minCTAs = 1;
  nc.maxCTAs = kDhtNcclCtas;  // every collective fits on the SMs the hash launches leave free
  int rc = dht_nccl(ncclCommInitRankConfig(&dht->comm, W, id, r, &nc), "ncclCommInitRankConfig");
  if (rc) {
    delete dht;
    dht = nullptr;
    return rc;
  }
  Export ex;
  memset(&ex, 0, sizeof ex);
  CB_TRY_CUDA(cudaIpcGetMemHandle(&ex.pool, pool), "cudaIpcGetMemHandle(pool)");
  CB_TRY_CUDA(cudaIpcGetMemHandle(&ex.table, table), "cudaIpcGetMemHandle(index)");
  if (policy.dram_capacity() > 0) {  // a DRAM tier: peers reach it through the outbox
    // an eighth of the pool (at least 64 MiB), at most 2 GiB or the DRAM tier
    const uint64_t want = std::max<uint64_t>(pool_bytes / 8, 64ull << 20);
    const uint64_t ob = std::min<uint64_t>(std::min<uint64_t>(want, 2ull << 30), policy.dram_capacity()) / 256 * 256;
    if (ob) {
      CB_TRY_CUDA(cudaMalloc(&dht->outbox, ob), "outbox");
      dht->outbox_bytes = ob;
      CB_TRY_CUDA(cudaIpcGetMemHandle(&ex.outbox, dht->outbox), "cudaIpcGetMemHandle(outbox)");
      ex.outbox_bytes = ob;
    }
  }
  ex.pool_bytes = pool_bytes;
  ex.table_slots = table_slots;
  ex.device = device;
  CB_TRY_CUDA(dht->h_misc.ensure(sizeof(Export) * (W + 1)), "pinned");
  CB_TRY_CUDA(dht->d_misc.ensure(sizeof(Export) * (W + 1)), "device");
  uint8_t *h = static_cast<uint8_t *>(dht->h_misc.ptr);
  uint8_t *d = static_cast<uint8_t *>(dht->d_misc.ptr);
  memcpy(h, &ex, sizeof ex);
  CB_TRY_CUDA(cudaMemcpyAsync(d, h, sizeof ex, cudaMemcpyHostToDevice, own_stream), "H2D export");
  rc = dht_nccl(ncclAllGather(d, d + sizeof(Export), sizeof(Export), ncclUint8, dht->comm, own_stream),
                "ncclAllGather(exports)");
  if (rc) return rc;
  CB_TRY_CUDA(cudaMemcpyAsync(h + sizeof(Export), d + sizeof(Export), sizeof(Export) * W, cudaMemcpyDeviceToHost,
                              own_stream),
              "D2H exports");
  rc = dht_sync(own_stream);
  if (rc) return rc;
  dht->pool.assign(W, 0);
  dht->pool_bytes.assign(W, 0);
  dht->table.assign(W, 0);
  dht->slots.assign(W, 0);
  dht->device.assign(W, -1);
  dht->peer_outbox.assign(W, 0);
  dht->peer_outbox_bytes.assign(W, 0);
  for (int p = 0; p < W; ++p) {
    Export e;
    memcpy(&e, h + sizeof(Export) * (p + 1), sizeof e);
    dht->pool_bytes[p] = e.pool_bytes;
    dht->slots[p] = e.table_slots;
    dht->device[p] = e.device;
    dht->peer_outbox_bytes[p] = e.outbox_bytes;
    if (p == r) {
      dht->pool[p] = (uint64_t)pool;
      dht->table[p] = (uint64_t)table;
      dht->peer_outbox[p] = (uint64_t)dht->outbox;
      continue;
    }
    if (e.outbox_bytes) {
      void *po = nullptr;
      CB_TRY_CUDA(cudaIpcOpenMemHandle(&po, e.outbox, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle(outbox)");
      dht->opened.push_back(po);
      dht->peer_outbox[p] = (uint64_t)po;
    }
    void *pp = nullptr, *pt = nullptr;
    CB_TRY_CUDA(cudaIpcOpenMemHandle(&pp, e.pool, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle(pool)");
    dht->opened.push_back(pp);
    CB_TRY_CUDA(cudaIpcOpenMemHandle(&pt, e.table, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle(index)");
    dht->opened.push_back(pt);
    dht->pool[p] = (uint64_t)pp;
    dht->table[p] = (uint64_t)pt;
  }
  rank = r;
  world = W;
  // a new block an owner places straight into its DRAM tier arrives through
  // its outbox: at most the outbox's bytes per put step
  policy.set_direct_dram_budget(dht->outbox_bytes);
  if (cfg.locality_aware || cfg.prefix_replication) {
    // one replica region serves hot-block replicas and prefix replicas
    uint64_t rb = cfg.replica_bytes ? cfg.replica_bytes : std::min<uint64_t>(pool_bytes / 32, 4ull << 30);
    rb = rb / 256 * 256;
    if (rb) {
      CB_TRY_CUDA(cudaMalloc(&dht->rbase, rb), "replica region");
      dht->rbytes = rb;
      dht->ralloc.reset(rb, 256);
      dht->locality = cfg.locality_aware != 0;
      dht->replicate_prefixes = cfg.prefix_replication != 0;
      dht->threshold = cfg.promotion_threshold ? cfg.promotion_threshold : 3;
    }
  }
  return CB_OK;
}

void Store::dht_detach() {
  if (!dht) return;
  if (dht->comm) {
    ncclCommAbort(dht->comm);  // no collective on the way out: peers may be gone
    dht->comm = nullptr;
  }
  for (void *p : dht->opened) cudaIpcCloseMemHandle(p);
  if (dht->rbase) cudaFree(dht->rbase);
  if (dht->outbox) cudaFree(dht->outbox);
  dht->d_send.release();
  dht->d_recv.release();
  dht->d_misc.release();
  dht->h_send.release();
  dht->h_recv.release();
  dht->h_misc.release();
  delete dht;
  dht = nullptr;
}

// ------------------------------------------------------------ put

int Store::dht_put(const void *const *ptrs, const uint64_t *sizes, const uint8_t *is_prefix,
                   const uint8_t *keys_in, int n, int mem_kind, uint8_t *keys_out, uint8_t *status_out,
                   cudaStream_t st, const uint16_t *step) {
  Trace tr("cb.dht_put");
  if (!dht || !dht->comm) return fail(CB_ERR_STATE, "DHT not attached (or its communicator was aborted after a failure)");
  const int W = dht->W, me = dht->me;
  // 0. device addresses of the blocks (host blocks: one staging area)
  std::vector<uint64_t> dptr(n);
  // Host blocks at a constant stride are staged segment-major on copy_stream
  // while the hash consumes them (stage_overlapped, as for 1-GPU host puts).
  HashProgress pg;
  bool overlapped = false;
  if (mem_kind == CB_MEM_HOST) {
    uint64_t total = 0;
    for (int i = 0; i < n; ++i) total += align_up(sizes[i], 256);
    CB_TRY_CUDA(d_staging.ensure(std::max<uint64_t>(total, 256)), "device staging");
    overlapped = !keys_in && n && stage_overlapped(ptrs, sizes, n, dptr.data(), pg, st) == CB_OK;
    uint64_t off = 0;
    for (int i = 0; i < n && !overlapped; ++i) {
      dptr[i] = (uint64_t)d_staging.ptr + off;
      if (sizes[i])
        CB_TRY_CUDA(cudaMemcpyAsync(reinterpret_cast<void *>(dptr[i]), ptrs[i], sizes[i], cudaMemcpyHostToDevice, st),
                    "H2D block");
      off += align_up(sizes[i], 256);
    }
  } else {
    for (int i = 0; i < n; ++i) dptr[i] = (uint64_t)ptrs[i];
  }
  // 1. keys
  std::vector<HKey> keys(n);
  if (keys_in) {
    for (int i = 0; i < n; ++i) keys[i] = to_hkey(keys_in + 16 * i);
  } else if (n) {
    // with overlapped staging, st also waits for every copy after the hash
    int rc = hash_device(dptr.data(), sizes, n, st, overlapped ? &pg : nullptr, overlapped ? ev_copies : nullptr);
    if (overlapped) {
      const cudaError_t e = cudaStreamSynchronize(copy_stream);
      if (rc == CB_OK && e != cudaSuccess) return cuda_fail(e, "copy stream");
    }
    if (rc) return rc;
    const uint8_t *dig = static_cast<const uint8_t *>(h_out.ptr);
    for (int i = 0; i < n; ++i) keys[i] = to_hkey(dig + 32 * i);
  }
  // 2. bucket by owner (batch order inside each bucket)
  std::vector<uint32_t> scount(W, 0), rcount(W, 0);
  std::vector<int> order(n), kowner(n);
  dht_route(keys.data(), n, W, kowner.data(), order.data(), scount.data());
  int rc = dht_counts(scount.data(), rcount.data(), st);
  if (rc) return rc;
  uint32_t nrecv = 0;
  for (int r = 0; r < W; ++r) nrecv += rcount[r];
  // 3. requests to owners
  CB_TRY_CUDA(dht->h_send.ensure(sizeof(PutReq) * std::max(n, 1)), "pinned");
  CB_TRY_CUDA(dht->d_send.ensure(sizeof(PutReq) * std::max(n, 1)), "device");
  CB_TRY_CUDA(dht->h_recv.ensure(sizeof(PutReq) * std::max<uint32_t>(nrecv, 1)), "pinned");
  CB_TRY_CUDA(dht->d_recv.ensure(sizeof(PutReq) * std::max<uint32_t>(nrecv, 1)), "device");
  PutReq *sreq = static_cast<PutReq *>(dht->h_send.ptr);
  for (int j = 0; j < n; ++j) {
    const int i = order[j];
    const uint64_t flags = ((is_prefix && is_prefix[i]) ? 1ull : 0ull) | ((step ? (uint64_t)step[i] : 0ull) << 8);
    sreq[j] = PutReq{keys[i].lo, keys[i].hi, sizes[i], flags};
  }
  CB_TRY_CUDA(cudaMemcpyAsync(dht->d_send.ptr, sreq, sizeof(PutReq) * n, cudaMemcpyHostToDevice, st), "H2D req");
  rc = dht_alltoallv(dht->d_send.ptr, scount.data(), dht->d_recv.ptr, rcount.data(), sizeof(PutReq), st);
  if (rc) return rc;
  CB_TRY_CUDA(cudaMemcpyAsync(dht->h_recv.ptr, dht->d_recv.ptr, sizeof(PutReq) * nrecv, cudaMemcpyDeviceToHost, st),
              "D2H req");
  rc = dht_sync(st);
  if (rc) return rc;
  // 4. owner: sequential dedup + placement in (step, source rank, index)
  // order. The requests arrive grouped by source rank, each rank's in batch
  // order; a step tag (bits 8.. of flags) names the batch of a group of
  // pipelined batches placed together, so a stable sort by step restores the
  // order of placing those batches one collective step at a time.
  const PutReq *rreq = static_cast<const PutReq *>(dht->h_recv.ptr);
  std::vector<uint32_t> perm(nrecv);
  for (uint32_t j = 0; j < nrecv; ++j) perm[j] = j;
  if (step)
    std::stable_sort(perm.begin(), perm.end(),
                     [rreq](uint32_t x, uint32_t y) { return (rreq[x].flags >> 8) < (rreq[y].flags >> 8); });
  std::vector<HKey> okeys(nrecv);
  std::vector<uint64_t> osizes(nrecv);
  std::vector<uint8_t> oprefix(nrecv);
  for (uint32_t j = 0; j < nrecv; ++j) {
    const PutReq &q = rreq[perm[j]];
    okeys[j] = HKey{q.klo, q.khi};
    osizes[j] = q.size;
    oprefix[j] = (uint8_t)(q.flags & 1);
  }
  rc = reserve_index(nrecv, st);
  if (rc) return rc;
  PutPlan &plan = put_plan;
  std::vector<uint32_t> ostatus(nrecv);  // in planning order (perm)
  std::vector<uint64_t> oloc(nrecv);
  dht_owner_plan(policy, okeys.data(), osizes.data(), oprefix.data(), nrecv, cfg.dedup_enabled != 0, plan,
                 ostatus.data(), oloc.data());
  plan_flag() = true;
  rc = run_moves(plan.moves, plan.dropped, st);
  if (rc) {
    policy.commit();
    return rc;
  }
  std::vector<PutRep> reps(nrecv);  // in received order
  for (uint32_t j = 0; j < nrecv; ++j) reps[perm[j]] = PutRep{oloc[j], ostatus[j], 0};
  // A new block this owner places straight into its DRAM tier (no HBM room
  // even after demotions) is handed over through the outbox: the writer
  // stores it there, the owner moves it to DRAM once the step's writes are
  // done (below). The index records the final DRAM location.
  std::vector<std::pair<const Placement *, uint64_t>> inbox;  // placement, outbox offset
  uint64_t ib = 0;
  std::vector<IndexRec> ins;
  ins.reserve(plan.places.size());
  for (const Placement &p : plan.places) {
    if (p.tier == kTierDram) {
      inbox.emplace_back(&p, ib);
      reps[perm[p.idx]].loc = ib | kLocOutbox;
      ib += align_up(p.size, 256);
    }
    ins.push_back(IndexRec{p.key.lo, p.key.hi, oloc[p.idx],
                           ((p.packed ? (p.size & ~1ull) : p.size) & kSizeMask) | (p.prefix ? kMetaPrefix : 0) |
                               (p.packed ? kMetaPacked : 0)});
  }
  policy.commit();
  // replies reuse the request buffers (PutRep <= PutReq)
  memcpy(dht->h_recv.ptr, reps.data(), sizeof(PutRep) * nrecv);
  if (!ins.empty()) {
    CB_TRY_CUDA(h_scratch.ensure(sizeof(IndexRec) * ins.size()), "pinned");
    CB_TRY_CUDA(d_scratch.ensure(sizeof(IndexRec) * ins.size()), "device");
    memcpy(h_scratch.ptr, ins.data(), sizeof(IndexRec) * ins.size());
    CB_TRY_CUDA(cudaMemcpyAsync(d_scratch.ptr, h_scratch.ptr, sizeof(IndexRec) * ins.size(), cudaMemcpyHostToDevice,
                                st),
                "H2D index");
    CB_TRY_CUDA(launch_index_insert(table, table_slots - 1, static_cast<const IndexRec *>(d_scratch.ptr),
                                    (int)ins.size(), d_err, st),
                "index insert");
    launches++;
    table_used += ins.size();
  }
  CB_TRY_CUDA(cudaMemcpyAsync(dht->d_recv.ptr, dht->h_recv.ptr, sizeof(PutRep) * nrecv, cudaMemcpyHostToDevice, st),
              "H2D rep");
  // 5. replies back to the writers
  rc = dht_alltoallv(dht->d_recv.ptr, rcount.data(), dht->d_send.ptr, scount.data(), sizeof(PutRep), st);
  if (rc) return rc;
  CB_TRY_CUDA(cudaMemcpyAsync(dht->h_send.ptr, dht->d_send.ptr, sizeof(PutRep) * n, cudaMemcpyDeviceToHost, st),
              "D2H rep");
  rc = dht_sync(st);
  if (rc) return rc;
  // 6. writers copy new blocks into the owners' pools: local destinations
  // through the TMA engine on st (one issuing lane per SM, so it runs beside
  // the hash CTAs), peer destinations through the LSU engine on peer_stream
  // (many warps keep NVLink stores in flight), both at once.
  std::vector<PutRep> mine(static_cast<const PutRep *>(dht->h_send.ptr), static_cast<const PutRep *>(dht->h_send.ptr) + n);
  std::vector<CopyDesc> ldesc, rdesc;
  std::vector<uint32_t> lus, rus;
  uint32_t ltotal = 0, rtotal = 0;
  uint64_t lbytes = 0, rbytes = 0;
  std::vector<uint8_t> status(n, CB_PUT_FAILED);
  for (int j = 0; j < n; ++j) {
    const int i = order[j];
    const int owner = kowner[i];
    status[i] = (uint8_t)mine[j].status;
    if (mine[j].status == CB_PUT_DEDUP) {
      remote_dedup_hits += cfg.dedup_enabled ? 1 : 0;
      remote_dedup_bytes += cfg.dedup_enabled ? sizes[i] : 0;
    }
    if (mine[j].status != CB_PUT_STORED || !sizes[i]) continue;
    uint64_t dst;
    if (mine[j].loc & kLocOutbox) {  // bound for the owner's DRAM tier, through its outbox
      dst = dht->peer_outbox[owner] + (mine[j].loc & kLocOutboxOff);
    } else {
      dst = dht->pool[owner] + (mine[j].loc & kLocOffMask);
    }
    const uint32_t units = (uint32_t)((sizes[i] + kCopyUnit - 1) / kCopyUnit);
    if (owner == me && mem_kind != CB_MEM_HOST) {
      lus.push_back(ltotal);
      ldesc.push_back(CopyDesc{dptr[i], dst, sizes[i], 0u});
      ltotal += units;
      lbytes += sizes[i];
    } else {
      if (owner != me) peer_bytes_written += sizes[i];
      rus.push_back(rtotal);
      rdesc.push_back(CopyDesc{dptr[i], dst, sizes[i], owner == me ? 0u : 1u});
      rtotal += units;
      rbytes += sizes[i];
    }
  }
  if (!ldesc.empty() || !rdesc.empty()) {
    if (!peer_stream) CB_TRY_CUDA(cudaStreamCreateWithFlags(&peer_stream, cudaStreamNonBlocking), "peer stream");
    if (!ev_peer_in) CB_TRY_CUDA(cudaEventCreateWithFlags(&ev_peer_in, cudaEventDisableTiming), "event");
    if (!ev_peer_out) CB_TRY_CUDA(cudaEventCreateWithFlags(&ev_peer_out, cudaEventDisableTiming), "event");
    lus.push_back(ltotal);
    rus.push_back(rtotal);
    Layout L;
    const size_t o_ld = L.add(sizeof(CopyDesc) * ldesc.size());
    const size_t o_lu = L.add(4 * lus.size());
    const size_t o_rd = L.add(sizeof(CopyDesc) * rdesc.size());
    const size_t o_ru = L.add(4 * rus.size());
    CB_TRY_CUDA(h_scratch.ensure(L.off), "pinned");
    CB_TRY_CUDA(d_scratch.ensure(L.off), "device");
    uint8_t *h = static_cast<uint8_t *>(h_scratch.ptr);
    if (!ldesc.empty()) memcpy(h + o_ld, ldesc.data(), sizeof(CopyDesc) * ldesc.size());
    memcpy(h + o_lu, lus.data(), 4 * lus.size());
    if (!rdesc.empty()) memcpy(h + o_rd, rdesc.data(), sizeof(CopyDesc) * rdesc.size());
    memcpy(h + o_ru, rus.data(), 4 * rus.size());
    uint8_t *d = static_cast<uint8_t *>(d_scratch.ptr);
    CB_TRY_CUDA(cudaMemcpyAsync(d, h, L.off, cudaMemcpyHostToDevice, st), "H2D scatter");
    if (!rdesc.empty()) {
      CB_TRY_CUDA(cudaEventRecord(ev_peer_in, st), "event");
      CB_TRY_CUDA(cudaStreamWaitEvent(peer_stream, ev_peer_in, 0), "wait");
      const int nr = (int)rdesc.size();
      CB_TRY_CUDA(timed(1, rbytes, peer_stream,
                        [&] {
                          return launch_batch_copy(reinterpret_cast<const CopyDesc *>(d + o_rd),
                                                   reinterpret_cast<const uint32_t *>(d + o_ru), nr, rtotal, 2,
                                                   d_err, num_sms, peer_stream);
                        }),
                  "peer scatter");
      CB_TRY_CUDA(cudaEventRecord(ev_peer_out, peer_stream), "event");
    }
    if (!ldesc.empty()) {
      const int nl = (int)ldesc.size();
      CB_TRY_CUDA(timed(1, lbytes, st,
                        [&] {
                          return launch_batch_copy(reinterpret_cast<const CopyDesc *>(d + o_ld),
                                                   reinterpret_cast<const uint32_t *>(d + o_lu), nl, ltotal,
                                                   copy_engine, d_err, num_sms, st);
                        }),
                  "local scatter");
    }
    if (!rdesc.empty()) CB_TRY_CUDA(cudaStreamWaitEvent(st, ev_peer_out, 0), "join");
  }
  // 7. closing barrier: every writer's copies precede every later op
  CB_TRY_CUDA(dht->d_misc.ensure(256), "device");
  rc = timed_coll(4, st, [&] {
    return dht_nccl(ncclAllReduce(dht->d_misc.ptr, dht->d_misc.ptr, 1, ncclInt32, ncclSum, dht->comm, st),
                    "ncclAllReduce(put barrier)");
  });
  if (rc) return rc;
  rc = dht_finish(st);
  if (rc) return rc;
  if (!inbox.empty()) {
    rc = dht_drain_inbox(inbox, st);
    if (rc) return rc;
  }
  for (int i = 0; i < n; ++i) {
    if (keys_out) memcpy(keys_out + 16 * i, &keys[i], 16);
    if (status_out) status_out[i] = status[i];
    // DistributedStore::put registers a prefix block it has stored
    // (src/distributed_backend.cpp:680-683)
    if (status[i] == CB_PUT_STORED && is_prefix && is_prefix[i]) dht->registry.insert(keys[i]);
  }
  return CB_OK;
}

// Owner side, after a put step's writes: the blocks writers stored in this
// owner's outbox go to their DRAM-tier extents - plain ones by the D2H copy
// engine, INT8-packed ones (kv_compression) by the pack kernels writing the
// mapped arena.
int Store::dht_drain_inbox(const std::vector<std::pair<const Placement *, uint64_t>> &inbox, cudaStream_t st) {
  CB_TRY_CUDA(ensure_dram(), "pinned DRAM arena cudaHostAlloc");
  std::vector<CopyDesc> desc;
  std::vector<uint32_t> us;
  uint32_t total = 0;
  for (const auto &pe : inbox) {
    const Placement &p = *pe.first;
    const uint8_t *src = dht->outbox + pe.second;
    if (!p.size) continue;
    if (!p.packed) {
      CB_TRY_CUDA(cudaMemcpyAsync(dram_host + p.off, src, p.size, cudaMemcpyDeviceToHost, st), "inbox to DRAM");
      continue;
    }
    us.push_back(total);
    desc.push_back(CopyDesc{(uint64_t)src, (uint64_t)dram_dev + p.off, p.size, kCopyHost});
    total += (uint32_t)((p.size + kCopyUnit - 1) / kCopyUnit);
  }
  if (!desc.empty()) {
    const int nd = (int)desc.size();
    us.push_back(total);
    const size_t o_us = align_up(sizeof(CopyDesc) * nd, 256);
    const size_t o_mm = align_up(o_us + 4 * us.size(), 256);
    const size_t need = o_mm + sizeof(int) * 2 * nd;
    CB_TRY_CUDA(h_scratch.ensure(need), "pinned");
    CB_TRY_CUDA(d_scratch.ensure(need), "device");
    uint8_t *h = static_cast<uint8_t *>(h_scratch.ptr);
    memcpy(h, desc.data(), sizeof(CopyDesc) * nd);
    memcpy(h + o_us, us.data(), 4 * us.size());
    int *mm = reinterpret_cast<int *>(h + o_mm);
    for (int j = 0; j < nd; ++j) {
      mm[2 * j] = INT_MAX;
      mm[2 * j + 1] = INT_MIN;
    }
    uint8_t *d = static_cast<uint8_t *>(d_scratch.ptr);
    CB_TRY_CUDA(cudaMemcpyAsync(d, h, need, cudaMemcpyHostToDevice, st), "H2D pack");
    CB_TRY_CUDA(launch_kv_pack(reinterpret_cast<const CopyDesc *>(d), reinterpret_cast<const uint32_t *>(d + o_us), nd,
                               total, reinterpret_cast<int *>(d + o_mm), num_sms, st),
                "inbox pack");
    launches += 2;
  }
  return check_device_error(st);  // syncs
}

// ------------------------------------------------------------ prefix sync

namespace {
struct PrefixRec {
  uint64_t klo, khi;
  uint64_t loc;   // byte offset of the block in the owner's arena | kLocDram
  uint64_t size;
};
}  // namespace

// sync_prefix_registry + broadcast_prefix_data (src/distributed_backend.cpp:
// 958-1217). The reference all-gathers every rank's prefix IDs (Allgatherv)
// and then has each owner MPI_Bcast its prefix blocks, which every other rank
// stores in its GPU tier. Here every prefix block has one owner that knows
// its location, so: each owner all-gathers one 32-byte record {key,
// location, size} per prefix block it holds (ncclAllGather, padded to the
// largest count); every rank merges the keys into its registry and, with
// prefix_replication, copies the blocks it does not own, and that sit in
// their owner's HBM pool, straight from the owners' pools into its replica
// region with one batched peer-load copy (no staging, no broadcast of
// payload through NCCL). A block in an owner's pinned DRAM tier is
// registered but not copied (peers cannot map that memory). Prefix replicas
// are pinned: hot-block replicas never displace them; they may displace hot
// replicas. A closing all-reduce keeps owners from reusing pool extents
// before every reader is done.
int Store::dht_sync_prefixes(cudaStream_t st) {
  Trace tr("cb.dht_sync_prefixes");
  if (!dht || !dht->comm) return fail(CB_ERR_STATE, "DHT not attached (or its communicator was aborted after a failure)");
  const int W = dht->W, me = dht->me;
  std::vector<PrefixRec> mine;
  policy.for_each([&](const HKey &k, const BlockMeta &m) {
    if (m.prefix)
      mine.push_back(PrefixRec{k.lo, k.hi, Policy::data_offset(m) | (m.tier == kTierDram ? kLocDram : 0), m.size});
  });
  // 1. counts (every rank takes every collective step below in the same order)
  CB_TRY_CUDA(dht->h_misc.ensure(4ull * (W + 1)), "pinned");
  CB_TRY_CUDA(dht->d_misc.ensure(4ull * (W + 1)), "device");
  uint32_t *hc = static_cast<uint32_t *>(dht->h_misc.ptr);
  uint32_t *dc = static_cast<uint32_t *>(dht->d_misc.ptr);
  hc[0] = (uint32_t)mine.size();
  CB_TRY_CUDA(cudaMemcpyAsync(dc, hc, 4, cudaMemcpyHostToDevice, st), "H2D count");
  int rc = dht_nccl(ncclAllGather(dc, dc + 1, 1, ncclUint32, dht->comm, st), "ncclAllGather(prefix counts)");
  if (rc) return rc;
  CB_TRY_CUDA(cudaMemcpyAsync(hc + 1, dc + 1, 4ull * W, cudaMemcpyDeviceToHost, st), "D2H counts");
  rc = dht_sync(st);
  if (rc) return rc;
  std::vector<uint32_t> counts(hc + 1, hc + 1 + W);
  const uint32_t max_n = *std::max_element(counts.begin(), counts.end());
  for (const PrefixRec &r : mine) dht->registry.insert(HKey{r.klo, r.khi});
  std::vector<CopyDesc> desc;
  std::vector<uint32_t> us;
  uint32_t total = 0;
  uint64_t bytes = 0;
  if (max_n) {
    // 2. records, padded to max_n per rank
    const size_t rb = sizeof(PrefixRec) * max_n;
    CB_TRY_CUDA(dht->h_send.ensure(rb), "pinned");
    CB_TRY_CUDA(dht->d_send.ensure(rb), "device");
    CB_TRY_CUDA(dht->h_recv.ensure(rb * W), "pinned");
    CB_TRY_CUDA(dht->d_recv.ensure(rb * W), "device");
    memset(dht->h_send.ptr, 0, rb);
    if (!mine.empty()) memcpy(dht->h_send.ptr, mine.data(), sizeof(PrefixRec) * mine.size());
    CB_TRY_CUDA(cudaMemcpyAsync(dht->d_send.ptr, dht->h_send.ptr, rb, cudaMemcpyHostToDevice, st), "H2D prefixes");
    rc = dht_nccl(ncclAllGather(dht->d_send.ptr, dht->d_recv.ptr, rb, ncclUint8, dht->comm, st),
                  "ncclAllGather(prefixes)");
    if (rc) return rc;
    CB_TRY_CUDA(cudaMemcpyAsync(dht->h_recv.ptr, dht->d_recv.ptr, rb * W, cudaMemcpyDeviceToHost, st),
                "D2H prefixes");
    rc = dht_sync(st);
    if (rc) return rc;
    // 3. merge, and plan the copies of other owners' prefix blocks
    const PrefixRec *all = static_cast<const PrefixRec *>(dht->h_recv.ptr);
    for (int r = 0; r < W; ++r) {
      if (r == me) continue;
      for (uint32_t j = 0; j < counts[r]; ++j) {
        const PrefixRec &rec = all[(size_t)r * max_n + j];
        const HKey k{rec.klo, rec.khi};
        dht->registry.insert(k);
        if (!dht->replicate_prefixes || !dht->rbase || !rec.size || (rec.loc & kLocDram)) continue;
        const uint64_t off = rec.loc & kLocOffMask;
        if (off > dht->pool_bytes[r] || rec.size > dht->pool_bytes[r] - off) continue;  // not a pool extent
        auto it = dht->rmap.find(k);
        if (it != dht->rmap.end()) {  // already a hot replica: keep it, pinned from now on
          if (!it->second.pinned) {
            dht->rlru.erase(it->second.lru);
            it->second.pinned = true;
            dht->prefix_replicas++;
          }
          continue;
        }
        const uint64_t roff = dht->alloc_replica(rec.size);
        if (roff == UINT64_MAX) continue;  // the replica region is full of prefix replicas
        dht->rmap.emplace(k, DhtState::Rep{roff, rec.size, {}, true});
        us.push_back(total);
        desc.push_back(CopyDesc{dht->pool[r] + off, (uint64_t)dht->rbase + roff, rec.size, kCopyHost});
        total += (uint32_t)((rec.size + kCopyUnit - 1) / kCopyUnit);
        bytes += rec.size;
        dht->prefix_replicas++;
      }
    }
  }
  // 4. one batched copy from the owners' pools (peer loads over NVLink)
  if (!desc.empty()) {
    us.push_back(total);
    const size_t o_us = align_up(sizeof(CopyDesc) * desc.size(), 256);
    const size_t need = o_us + 4 * us.size();
    CB_TRY_CUDA(h_scratch.ensure(need), "pinned");
    CB_TRY_CUDA(d_scratch.ensure(need), "device");
    uint8_t *h = static_cast<uint8_t *>(h_scratch.ptr);
    memcpy(h, desc.data(), sizeof(CopyDesc) * desc.size());
    memcpy(h + o_us, us.data(), 4 * us.size());
    uint8_t *d = static_cast<uint8_t *>(d_scratch.ptr);
    CB_TRY_CUDA(cudaMemcpyAsync(d, h, need, cudaMemcpyHostToDevice, st), "H2D prefix copies");
    const int nd = (int)desc.size();
    CB_TRY_CUDA(timed(2, bytes, st,
                      [&] {
                        return launch_batch_copy(reinterpret_cast<const CopyDesc *>(d),
                                                 reinterpret_cast<const uint32_t *>(d + o_us), nd, total, 2, d_err,
                                                 num_sms, st);
                      }),
                "prefix copies");
    peer_bytes_read += bytes;
  }
  // 5. owners keep their extents until every reader is done
  CB_TRY_CUDA(dht->d_misc.ensure(256), "device");
  rc = dht_nccl(ncclAllReduce(dht->d_misc.ptr, dht->d_misc.ptr, 1, ncclInt32, ncclSum, dht->comm, st),
                "ncclAllReduce(prefix sync barrier)");
  if (rc) return rc;
  return dht_finish(st);
}

uint64_t Store::dht_registry_size() const { return dht ? dht->registry.size() : 0; }
uint64_t Store::dht_prefix_replicas() const { return dht ? dht->prefix_replicas : 0; }

// ------------------------------------------------------------ lookup

// Sends keys to their owners, runs the owner lookup kernel, returns for each
// key (in the caller's order) {location, meta} in reps (host) and the owner.
int Store::dht_lookup(const uint8_t *keys, int n, std::vector<uint64_t> &reps, std::vector<int> &owner,
                      cudaStream_t st, bool stage) {
  const int W = dht->W;
  std::vector<uint32_t> scount(W, 0), rcount(W, 0);
  std::vector<int> order(n);
  owner.assign(n, 0);
  {
    std::vector<HKey> hk(n);
    for (int i = 0; i < n; ++i) hk[i] = to_hkey(keys + 16 * i);
    dht_route(hk.data(), n, W, owner.data(), order.data(), scount.data());
  }
  int rc = dht_counts(scount.data(), rcount.data(), st);
  if (rc) return rc;
  uint32_t nrecv = 0;
  for (int r = 0; r < W; ++r) nrecv += rcount[r];
  const size_t smax = std::max<size_t>(n, 1), rmax = std::max<size_t>(nrecv, 1);
  CB_TRY_CUDA(dht->h_send.ensure(16 * smax), "pinned");
  CB_TRY_CUDA(dht->d_send.ensure(16 * smax), "device");
  CB_TRY_CUDA(dht->h_recv.ensure(16 * rmax), "pinned");
  CB_TRY_CUDA(dht->d_recv.ensure(16 * rmax + 16 * rmax), "device");
  uint8_t *hs = static_cast<uint8_t *>(dht->h_send.ptr);
  for (int j = 0; j < n; ++j) memcpy(hs + 16 * j, keys + 16 * order[j], 16);
  CB_TRY_CUDA(cudaMemcpyAsync(dht->d_send.ptr, hs, 16ull * n, cudaMemcpyHostToDevice, st), "H2D keys");
  uint8_t *rk = static_cast<uint8_t *>(dht->d_recv.ptr);  // received keys
  uint64_t *rr = reinterpret_cast<uint64_t *>(rk + 16 * rmax);  // replies
  rc = dht_alltoallv(dht->d_send.ptr, scount.data(), rk, rcount.data(), 16, st);
  if (rc) return rc;
  if (dht->outbox && policy.dram_used() > 0) {
    rc = dht_serve_host(rk, nrecv, rcount.data(), rr, st, stage);
    if (rc) return rc;
  } else {
    CB_TRY_CUDA(launch_index_serve(table, table_slots - 1, reinterpret_cast<const Key *>(rk), (int)nrecv, rr, st),
                "index serve");
    launches++;
  }
  // keys this owner served, for its LRU order (read after the sync below)
  CB_TRY_CUDA(cudaMemcpyAsync(dht->h_recv.ptr, rk, 16ull * nrecv, cudaMemcpyDeviceToHost, st), "D2H served keys");
  rc = dht_alltoallv(rr, rcount.data(), dht->d_send.ptr, scount.data(), 16, st);
  if (rc) return rc;
  CB_TRY_CUDA(cudaMemcpyAsync(hs, dht->d_send.ptr, 16ull * n, cudaMemcpyDeviceToHost, st), "D2H replies");
  rc = dht_sync(st);
  if (rc) return rc;
  const uint8_t *served = static_cast<const uint8_t *>(dht->h_recv.ptr);
  for (uint32_t j = 0; j < nrecv; ++j) policy.touch(to_hkey(served + 16 * j));
  reps.assign(2ull * n, 0);
  const uint64_t *hr = reinterpret_cast<const uint64_t *>(hs);
  for (int j = 0; j < n; ++j) {
    reps[2ull * order[j]] = hr[2ull * j];
    reps[2ull * order[j] + 1] = hr[2ull * j + 1];
  }
  return CB_OK;
}

// Owner side of a lookup with a non-empty DRAM tier. The host metadata is
// authoritative for the blocks this rank owns, so the replies are built from
// it; a DRAM-tier block another rank asked for is copied by the H2D copy
// engine from the pinned arena into the outbox (as it sits there: INT8-packed
// blocks stay packed, the requester's gather unpacks them) and the reply
// names its outbox offset. The reference serves such reads from the owner's
// DRAM shadow through MPI_Get (src/distributed_backend.cpp:729-767,
// :210-219); it leaves the owner's tiers as they are, and so does this.
// Requests of this rank for its own DRAM blocks are read from the mapped
// arena directly. Blocks beyond the outbox's room are reported as found in
// remote DRAM and not copied.
int Store::dht_serve_host(const uint8_t *d_keys, uint32_t nrecv, const uint32_t *rcount, uint64_t *d_reps,
                          cudaStream_t st, bool stage) {
  const int W = dht->W, me = dht->me;
  const size_t o_rep = align_up(16ull * nrecv, 256);
  CB_TRY_CUDA(h_scratch.ensure(o_rep + 16ull * std::max<uint32_t>(nrecv, 1)), "pinned");
  uint8_t *h = static_cast<uint8_t *>(h_scratch.ptr);
  if (nrecv) CB_TRY_CUDA(cudaMemcpyAsync(h, d_keys, 16ull * nrecv, cudaMemcpyDeviceToHost, st), "D2H keys");
  int rc = dht_sync(st);
  if (rc) return rc;
  uint64_t *reps = reinterpret_cast<uint64_t *>(h + o_rep);
  uint64_t ob = 0;
  uint32_t j = 0;
  for (int r = 0; r < W; ++r) {
    for (uint32_t t = 0; t < rcount[r]; ++t, ++j) {
      const BlockMeta *m = policy.find(to_hkey(h + 16ull * j));
      uint64_t loc = 0, meta = 0;
      if (m) {
        meta = meta_of(*m);
        loc = Policy::data_offset(*m);
        if (m->tier == kTierDram) {
          loc |= kLocDram;
          const uint64_t foot = Policy::footprint(*m);
          const uint64_t lead = m->packed ? kPackLead : 0;  // keeps a packed payload 16-byte aligned
          const uint64_t slot = align_up(lead + foot, 256);
          if (stage && r != me && ob + slot <= dht->outbox_bytes) {
            if (foot)
              CB_TRY_CUDA(cudaMemcpyAsync(dht->outbox + ob + lead, dram_host + Policy::data_offset(*m), foot,
                                          cudaMemcpyHostToDevice, st),
                          "DRAM block to outbox");
            loc = (ob + lead) | kLocOutbox;
            ob += slot;
          }
        }
      }
      reps[2ull * j] = loc;
      reps[2ull * j + 1] = meta;
    }
  }
  if (nrecv)
    CB_TRY_CUDA(cudaMemcpyAsync(d_reps, reps, 16ull * nrecv, cudaMemcpyHostToDevice, st), "H2D replies");
  return CB_OK;
}

int Store::dht_get(const uint8_t *keys, int n, void *const *outs, const uint64_t *caps, int mem_kind,
                   uint64_t *sizes_out, uint8_t *found_out, cudaStream_t st) {
  Trace tr("cb.dht_get");
  if (!dht || !dht->comm) return fail(CB_ERR_STATE, "DHT not attached (or its communicator was aborted after a failure)");
  const int me = dht->me;
  // Replica hits are served from local HBM. Other keys repeated inside the
  // batch (hot keys under a skewed access pattern) are looked up and fetched
  // over NVLink once; the other occurrences are filled from the first copy.
  std::vector<int> uidx(n, -1);
  std::vector<int64_t> rep_off(n, -1);
  std::vector<uint8_t> ukeys;
  ukeys.reserve(16ull * n);
  {
    std::unordered_map<HKey, int, HKeyHash> first;
    first.reserve(2ull * n);
    for (int i = 0; i < n; ++i) {
      const HKey k = to_hkey(keys + 16 * i);
      if (dht->rbase) {
        auto r = dht->rmap.find(k);
        if (r != dht->rmap.end()) {
          rep_off[i] = (int64_t)r->second.off;
          if (!r->second.pinned) dht->rlru.splice(dht->rlru.begin(), dht->rlru, r->second.lru);
          continue;
        }
      }
      auto ins = first.emplace(k, (int)(ukeys.size() / 16));
      if (ins.second) ukeys.insert(ukeys.end(), keys + 16 * i, keys + 16 * i + 16);
      uidx[i] = ins.first->second;
    }
  }
  const int m = (int)(ukeys.size() / 16);
  std::vector<uint64_t> ureps;
  std::vector<int> uowner;
  int rc = dht_lookup(ukeys.data(), m, ureps, uowner, st);  // collective, also when m == 0
  if (rc) return rc;
  std::vector<uint64_t> reps(2ull * n, 0);
  std::vector<int> owner(n, me);
  for (int i = 0; i < n; ++i) {
    if (rep_off[i] >= 0) {
      const HKey k = to_hkey(keys + 16 * i);
      reps[2ull * i] = (uint64_t)rep_off[i];
      reps[2ull * i + 1] = kMetaOccupied | (dht->rmap.at(k).size & kSizeMask);
      continue;
    }
    reps[2ull * i] = ureps[2ull * uidx[i]];
    reps[2ull * i + 1] = ureps[2ull * uidx[i] + 1];
    owner[i] = uowner[uidx[i]];
  }
  std::vector<int> leader(m, -1);  // occurrence that fetches the block
  // host outputs: gather into staging, then DMA out
  std::vector<uint64_t> dst(n);
  if (mem_kind == CB_MEM_HOST) {
    uint64_t total = 0;
    for (int i = 0; i < n; ++i) {
      const uint64_t sz = reps[2ull * i + 1] & kSizeMask;
      total += (reps[2ull * i + 1] && sz <= caps[i]) ? align_up(sz, 256) : 0;
    }
    CB_TRY_CUDA(d_staging.ensure(std::max<uint64_t>(total, 256)), "device staging");
    uint64_t off = 0;
    for (int i = 0; i < n; ++i) {
      const uint64_t sz = reps[2ull * i + 1] & kSizeMask;
      dst[i] = (uint64_t)d_staging.ptr + off;
      off += (reps[2ull * i + 1] && sz <= caps[i]) ? align_up(sz, 256) : 0;
    }
  } else {
    for (int i = 0; i < n; ++i) dst[i] = (uint64_t)outs[i];
  }
  std::vector<CopyDesc> desc;
  std::vector<uint32_t> us;
  uint32_t total = 0;
  uint64_t bytes = 0;
  for (int i = 0; i < n; ++i) {
    const uint64_t meta = reps[2ull * i + 1], loc = reps[2ull * i];
    const uint64_t sz = meta & kSizeMask;
    const bool replica = rep_off[i] >= 0;
    const bool staged = !replica && (loc & kLocOutbox) != 0;  // a DRAM-tier block, in the owner's outbox
    const bool dram = !replica && !staged && (loc & kLocDram) != 0;
    const bool in_dram = dram || staged;
    const bool local = owner[i] == me;
    sizes_out[i] = 0;
    if (!(meta & kMetaOccupied)) {
      found_out[i] = CB_FOUND_MISS;
      misses++;
      continue;
    }
    sizes_out[i] = sz;
    found_out[i] = in_dram ? (local ? CB_FOUND_LOCAL_DRAM : CB_FOUND_REMOTE_DRAM)
                           : (local ? CB_FOUND_LOCAL_HBM : CB_FOUND_REMOTE_HBM);
    if (local && !in_dram) local_gpu_hits++;
    if (local && in_dram) local_dram_hits++;
    if (!local && !in_dram) remote_gpu_hits++;
    if (!local && in_dram) remote_dram_hits++;
    if (dht->locality) dht->record_access(to_hkey(keys + 16 * i), !local);
    if (sz > caps[i] || (dram && !local)) {  // too small, or a peer's pinned DRAM (not mapped here)
      found_out[i] |= CB_FOUND_NOT_COPIED;
      continue;
    }
    if (!sz) continue;
    uint64_t src;
    uint64_t flags = 0;
    if (replica) {
      src = (uint64_t)dht->rbase + loc;
    } else {
      if (leader[uidx[i]] >= 0) continue;  // a repeat: filled from the leader below
      leader[uidx[i]] = i;
      const bool packed = in_dram && (meta & kMetaPacked);
      if (!local) peer_bytes_read += packed ? packed_bytes(sz) : sz;
      if (staged) {
        src = dht->peer_outbox[owner[i]] + (loc & kLocOutboxOff);
      } else {
        const uint64_t off = loc & kLocOffMask;
        src = dram ? (uint64_t)dram_dev + off : dht->pool[owner[i]] + off;
      }
      flags = (in_dram || !local) ? kCopyHost : 0;  // peer and pinned-host sources: plain loads
      if (packed) flags |= kCopyUnpack;
    }
    us.push_back(total);
    desc.push_back(CopyDesc{src, dst[i], sz, flags});
    total += (uint32_t)((sz + kCopyUnit - 1) / kCopyUnit);
    bytes += sz;
  }
  // second pass (after the gather): repeats copied from their leader's
  // output, and promotions of hot remote blocks into the replica region
  std::vector<CopyDesc> rdesc;
  std::vector<uint32_t> rus;
  uint32_t rtotal = 0;
  auto add2 = [&](uint64_t s, uint64_t d, uint64_t sz) {
    rus.push_back(rtotal);
    rdesc.push_back(CopyDesc{s, d, sz, 0u});
    rtotal += (uint32_t)((sz + kCopyUnit - 1) / kCopyUnit);
  };
  for (int i = 0; i < n; ++i) {
    if (uidx[i] < 0) continue;
    const int l = leader[uidx[i]];
    if (l < 0 || l == i || (found_out[i] & CB_FOUND_NOT_COPIED) || (found_out[i] & 0x0f) == CB_FOUND_MISS ||
        !sizes_out[i])
      continue;
    add2(dst[l], dst[i], sizes_out[i]);
  }
  if (dht->locality) {
    for (int u = 0; u < m; ++u) {
      const int l = leader[u];
      if (l < 0) continue;
      const uint32_t code = found_out[l];
      if ((code & CB_FOUND_NOT_COPIED) ||
          ((code & 0x0f) != CB_FOUND_REMOTE_HBM && (code & 0x0f) != CB_FOUND_REMOTE_DRAM))
        continue;
      const HKey k = to_hkey(ukeys.data() + 16 * u);
      if (dht->rmap.count(k) || !dht->should_promote(k)) continue;
      const uint64_t sz = sizes_out[l];
      const uint64_t off = dht->alloc_replica(sz);  // drops least recently used hot replicas
      if (off == UINT64_MAX) continue;
      dht->rlru.push_front(k);
      dht->rmap.emplace(k, DhtState::Rep{off, sz, dht->rlru.begin(), false});
      add2(dst[l], (uint64_t)dht->rbase + off, sz);
      replica_promotions++;
    }
  }
  if (!desc.empty()) {
    us.push_back(total);
    const size_t o_us = align_up(sizeof(CopyDesc) * desc.size(), 256);
    const size_t need = o_us + 4 * us.size();
    CB_TRY_CUDA(h_scratch.ensure(need), "pinned");
    CB_TRY_CUDA(d_scratch.ensure(need), "device");
    uint8_t *h = static_cast<uint8_t *>(h_scratch.ptr);
    memcpy(h, desc.data(), sizeof(CopyDesc) * desc.size());
    memcpy(h + o_us, us.data(), 4 * us.size());
    uint8_t *d = static_cast<uint8_t *>(d_scratch.ptr);
    CB_TRY_CUDA(cudaMemcpyAsync(d, h, need, cudaMemcpyHostToDevice, st), "H2D gather");
    const int nd = (int)desc.size();
    CB_TRY_CUDA(timed(2, bytes, st,
                      [&] {
                        // many warps per SM keep enough peer loads in flight
                        return launch_batch_copy(reinterpret_cast<const CopyDesc *>(d),
                                                 reinterpret_cast<const uint32_t *>(d + o_us), nd, total, 2, d_err,
                                                 num_sms, st);
                      }),
                "gather");
  }
  if (!rdesc.empty()) {
    rus.push_back(rtotal);
    const size_t o_us = align_up(sizeof(CopyDesc) * rdesc.size(), 256);
    const size_t need = o_us + 4 * rus.size();
    // the gather above may still read its descriptors from d_scratch
    CB_TRY_CUDA(cudaStreamSynchronize(st), "gather");
    CB_TRY_CUDA(h_scratch.ensure(need), "pinned");
    CB_TRY_CUDA(d_scratch.ensure(need), "device");
    uint8_t *h = static_cast<uint8_t *>(h_scratch.ptr);
    memcpy(h, rdesc.data(), sizeof(CopyDesc) * rdesc.size());
    memcpy(h + o_us, rus.data(), 4 * rus.size());
    uint8_t *d = static_cast<uint8_t *>(d_scratch.ptr);
    CB_TRY_CUDA(cudaMemcpyAsync(d, h, need, cudaMemcpyHostToDevice, st), "H2D repeats");
    const int nr = (int)rdesc.size();
    CB_TRY_CUDA(launch_batch_copy(reinterpret_cast<const CopyDesc *>(d), reinterpret_cast<const uint32_t *>(d + o_us),
                                  nr, rtotal, copy_engine, d_err, num_sms, st),
                "repeat copies");
    launches++;
  }
  // No closing barrier: an owner rewrites its pool or outbox only in a later
  // collective step (a put's scatter into extents it plans then, the staging
  // of a later get), and every step opens with the counts all-gather, which
  // completes on the owner only after every reader enqueued its part of it -
  // behind this gather on the reader's stream (and this call waits for the
  // gather before it returns anyway).
  if (mem_kind == CB_MEM_HOST) {
    // one D2H per run of blocks contiguous both in staging and in the
    // caller's memory (a caller's [n, block] buffer is one copy)
    auto copied = [&](int i) {
      return (found_out[i] & 0x0f) != CB_FOUND_MISS && !(found_out[i] & CB_FOUND_NOT_COPIED) && sizes_out[i];
    };
    int i = 0;
    while (i < n) {
      if (!copied(i)) {
        ++i;
        continue;
      }
      int e = i + 1;
      uint64_t run = sizes_out[i];
      const AddrRange rg = e < n ? alloc_range(outs[i]) : AddrRange{0, 0};
      while (e < n && copied(e) && dst[e] - dst[i] == run && dst[e] - dst[e - 1] == sizes_out[e - 1] &&
             static_cast<uint8_t *>(outs[i]) + run == outs[e] && rg.holds(outs[i], run + sizes_out[e])) {
        run += sizes_out[e];
        ++e;
      }
      CB_TRY_CUDA(cudaMemcpyAsync(outs[i], reinterpret_cast<void *>(dst[i]), run, cudaMemcpyDeviceToHost, st),
                  "D2H blocks");
      i = e;
    }
  }
  return dht_finish(st);
}

int Store::dht_contains(const uint8_t *keys, int n, uint8_t *found_out, cudaStream_t st) {
  if (!dht || !dht->comm) return fail(CB_ERR_STATE, "DHT not attached (or its communicator was aborted after a failure)");
  std::vector<uint64_t> reps;
  std::vector<int> owner;
  int rc = dht_lookup(keys, n, reps, owner, st, false);
  if (rc) return rc;
  for (int i = 0; i < n; ++i) found_out[i] = (reps[2ull * i + 1] & kMetaOccupied) ? 1 : 0;
  return CB_OK;
}

// One-sided probe of the owner's index through its peer mapping (locate is
// not collective in the reference either: it reads local metadata).
int Store::dht_locate(const uint8_t *key, cb_location *out, int32_t *found) {
  if (!dht) return fail(CB_ERR_STATE, "DHT not attached (or its communicator was aborted after a failure)");
  const HKey k = to_hkey(key);
  const int o = (int)be_owner(k, dht->W);
  CB_TRY_CUDA(h_scratch.ensure(64), "pinned");
  CB_TRY_CUDA(d_scratch.ensure(64), "device");
  uint8_t *h = static_cast<uint8_t *>(h_scratch.ptr);
  uint8_t *d = static_cast<uint8_t *>(d_scratch.ptr);
  memcpy(h, key, 16);
  CB_TRY_CUDA(cudaMemcpyAsync(d, h, 16, cudaMemcpyHostToDevice, own_stream), "H2D key");
  CB_TRY_CUDA(launch_index_serve(reinterpret_cast<const Slot *>(dht->table[o]), dht->slots[o] - 1,
                                 reinterpret_cast<const Key *>(d), 1, reinterpret_cast<uint64_t *>(d + 16), own_stream),
              "index probe");
  launches++;
  CB_TRY_CUDA(cudaMemcpyAsync(h + 16, d + 16, 16, cudaMemcpyDeviceToHost, own_stream), "D2H probe");
  CB_TRY_CUDA(cudaStreamSynchronize(own_stream), "probe");
  uint64_t loc, meta;
  memcpy(&loc, h + 16, 8);
  memcpy(&meta, h + 24, 8);
  memset(out, 0, sizeof *out);
  *found = (meta & kMetaOccupied) ? 1 : 0;
  if (!*found) return CB_OK;
  out->node_id = o;
  out->is_gpu = (loc & kLocDram) ? 0 : 1;
  out->gpu_id = out->is_gpu ? dht->device[o] : -1;
  out->offset = loc & kLocOffMask;
  out->size = meta & kSizeMask;
  out->is_prefix = (meta & kMetaPrefix) ? 1 : 0;
  return CB_OK;
}

int Store::dht_cluster_usage(cb_stats *o) {
  if (!dht || !dht->comm) return fail(CB_ERR_STATE, "DHT not attached (or its communicator was aborted after a failure)");
  CB_TRY_CUDA(dht->h_misc.ensure(64), "pinned");
  CB_TRY_CUDA(dht->d_misc.ensure(64), "device");
  uint64_t *h = static_cast<uint64_t *>(dht->h_misc.ptr);
  h[0] = o->local_gpu_used;
  h[1] = o->local_dram_used;
  CB_TRY_CUDA(cudaMemcpyAsync(dht->d_misc.ptr, h, 16, cudaMemcpyHostToDevice, own_stream), "H2D usage");
  int rc = dht_nccl(ncclAllReduce(dht->d_misc.ptr, dht->d_misc.ptr, 2, ncclUint64, ncclSum, dht->comm, own_stream),
                    "ncclAllReduce(usage)");
  if (rc) return rc;
  CB_TRY_CUDA(cudaMemcpyAsync(h, dht->d_misc.ptr, 16, cudaMemcpyDeviceToHost, own_stream), "D2H usage");
  rc = dht_sync(own_stream);
  if (rc) return rc;
  o->cluster_gpu_used = h[0];
  o->cluster_dram_used = h[1];
  return CB_OK;
}

}  // namespace cb

// Host-only planner: the DHT owner's policy without a GPU (cb_planner_*).
struct cb_planner {
  cb::Policy policy;
  bool dedup;
  cb::PutPlan plan;
  cb_planner(uint64_t hbm, uint64_t dram, bool semantic, bool dd) : policy(hbm, dram, semantic), dedup(dd) {
    policy.set_direct_dram_budget(0);  // as a DHT owner without an outbox (cb_dht_attach)
  }
};

extern "C" {

int cb_dht_route(const uint8_t *keys, int32_t n, int32_t world, int32_t *owner_out, int32_t *order_out,
                 uint32_t *counts_out) {
  if (n < 0 || world < 1 || (n > 0 && (!keys || !owner_out || !order_out)) || !counts_out) return CB_ERR_ARG;
  std::vector<cb::HKey> hk(n);
  for (int i = 0; i < n; ++i) hk[i] = cb::to_hkey(keys + 16ull * i);
  std::vector<int> owner(n), order(n);
  cb::dht_route(hk.data(), n, world, owner.data(), order.data(), counts_out);
  for (int i = 0; i < n; ++i) {
    owner_out[i] = owner[i];
    order_out[i] = order[i];
  }
  return CB_OK;
}

int cb_planner_create(uint64_t gpu_capacity_bytes, uint64_t dram_capacity_bytes, int32_t semantic_eviction,
                      int32_t dedup_enabled, cb_planner **out) {
  if (!out) return CB_ERR_ARG;
  try {
    *out = new cb_planner(gpu_capacity_bytes, dram_capacity_bytes, semantic_eviction != 0, dedup_enabled != 0);
  } catch (...) {
    *out = nullptr;
    return CB_ERR_NOSPACE;
  }
  return CB_OK;
}

int cb_planner_destroy(cb_planner *p) {
  delete p;
  return CB_OK;
}

int cb_dht_plan_put(cb_planner *p, const uint8_t *keys, const uint64_t *sizes, const uint8_t *prefix, int32_t n,
                    uint8_t *status_out, uint64_t *loc_out) {
  if (!p || n < 0 || (n > 0 && (!keys || !sizes || !status_out || !loc_out))) return CB_ERR_ARG;
  try {
    std::vector<cb::HKey> hk(n);
    for (int i = 0; i < n; ++i) hk[i] = cb::to_hkey(keys + 16ull * i);
    std::vector<uint32_t> st(n);
    std::vector<uint64_t> loc(n);
    cb::dht_owner_plan(p->policy, hk.data(), sizes, prefix, (uint32_t)n, p->dedup, p->plan, st.data(), loc.data());
    p->policy.commit();
    for (int i = 0; i < n; ++i) {
      status_out[i] = (uint8_t)st[i];
      loc_out[i] = loc[i];
    }
  } catch (...) {
    return CB_ERR_NOSPACE;
  }
  return CB_OK;
}

int cb_dht_unique_id(uint8_t *uid_out) {
  if (!uid_out) return CB_ERR_ARG;
  ncclUniqueId id;
  if (ncclGetUniqueId(&id) != ncclSuccess) return CB_ERR_NCCL;
  memcpy(uid_out, &id, sizeof id);
  return CB_OK;
}

}  // extern "C"

namespace cb {
void Store::dht_clear_replicas() {
  if (dht) dht->clear_replicas();
}
}  // namespace cb
