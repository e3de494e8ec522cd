// Stream-ordered (pipelined) puts and gets of one store.
//
// A synchronous batch_put hashes its batch, plans it and scatters it before
// it returns, so at most `batch` SHA-256 chains run at once: one chain per
// block, 32 per CTA, 32 CTAs for a 1024-block batch on a 148-SM GPU. The
// reference's CPU put_batch keeps every core busy at any batch size with
// OpenMP over the batch (src/cascade_core.cpp:1358-1373); the GPU form of
// that is to keep many batches hashing at once:
//
//  * cb_put_batch_async launches the batch's SHA-256 at submission on one of
//    kHashSlots side streams (small batches queued back to back share one
//    launch of up to kLaunchBlocks blocks) and returns a ticket;
//  * batches are placed - sequential dedup plan, tier moves, scatter into the
//    pool, index insert - strictly in ticket order: while more than
//    `pipeline_blocks` blocks are hashing (the host plans finished batches
//    while the GPU hashes), when a hash slot is needed again, or when
//    cb_put_wait / any other data call needs them. Placement in ticket order keeps the sequential dedup rule of
//    DistributedStore::put_batch (src/distributed_backend.cpp:813-841)
//    exactly: a block is a dedup hit iff its key was stored before it.
//
// On a DHT member the placement of a batch is the collective DHT put with
// the digests as keys, run by the store's placement thread so that the
// caller keeps submitting (and the GPU keeps hashing) while a group's
// exchanges, owner planning and peer stores run. Every rank must make the
// same sequence of collectives, so batches are assigned to that thread by
// counts alone (never by timing or block counts, which differ between
// ranks): once more than kDhtPending batches are unassigned the oldest
// kDhtGroup go as one group - one collective step, owners keep the batch
// order - and a wait assigns the rest in groups. How many blocks hash at
// once is the caller's local business (it waits on its own launches only).
//
// cb_get_batch_async serves the common case of a 1-GPU get without a device
// round trip: when every requested block is in the HBM tier (or missing),
// the host metadata - authoritative on one GPU - already holds each block's
// pool offset and size, so the call builds the gather descriptors from it,
// enqueues the gather on the caller's stream and returns with found/sizes
// final and the bytes landing in stream order. A batch that touches the DRAM
// tier takes the synchronous path. Pool extents a stream-ordered gather may
// still read are protected: every later pool write (scatter, tier move)
// waits for those gathers on the device (fence_reads).
//
// Device-side errors of stream-ordered work surface at the next call that
// settles (cb_put_wait, cb_sync, and every synchronous data call): that call
// returns the error. A failed placement leaves the host metadata ahead of
// the pool, so the store then refuses data calls until cb_clear.
#include <cuda.h>  // green-context types; the functions come from cudaGetDriverEntryPoint
#include <string.h>

#include <algorithm>

#include "kernels.cuh"
#include "store.hpp"

namespace cb {

namespace {

constexpr int kLaunchBlocks = 1024;              // queued small batches share a launch up to this size
// blocks hashing at once by default (device-resident inputs; host blocks are
// placed at submission): 65,536 chains keep ~3.5 warps on every SM
// sub-partition, where the hash kernel reaches its ALU-bound rate
constexpr uint64_t kDefaultPipelineBlocks = 65536;
constexpr size_t kDhtPending = 8;                // DHT: batches submitted and not yet assigned (every rank alike)
constexpr size_t kDhtGroup = 8;                  // DHT: batches placed together in one collective step
constexpr int kScatterLsuCtasPerSm = 4;          // LSU engine (copy_engine = 2): CTAs per SM beside the hashes

inline size_t digest_offset(int cap) { return align_up(sizeof(HashJob) * (size_t)cap, 256); }

}  // namespace

namespace {

template <class F>
F driver_fn(const char *name) {
  void *fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint(name, &fn, cudaEnableDefault, &q) != cudaSuccess || q != cudaDriverEntryPointSuccess)
    return nullptr;
  return reinterpret_cast<F>(fn);
}

}  // namespace

// A green context of at least `sms` SMs for the hash streams. Returns CB_OK
// with green == null when the driver offers no such partition (the hash
// streams then use every SM).
int Store::make_hash_green_context(int sms) {
  using GetDev = CUresult (*)(CUdevice *, int);
  using GetRes = CUresult (*)(CUdevice, CUdevResource *, CUdevResourceType);
  using Split = CUresult (*)(CUdevResource *, unsigned *, const CUdevResource *, CUdevResource *, unsigned, unsigned);
  using Desc = CUresult (*)(CUdevResourceDesc *, CUdevResource *, unsigned);
  using Create = CUresult (*)(CUgreenCtx *, CUdevResourceDesc, CUdevice, unsigned);
  auto get_dev = driver_fn<GetDev>("cuDeviceGet");
  auto get_res = driver_fn<GetRes>("cuDeviceGetDevResource");
  auto split = driver_fn<Split>("cuDevSmResourceSplitByCount");
  auto desc_fn = driver_fn<Desc>("cuDevResourceGenerateDesc");
  auto create = driver_fn<Create>("cuGreenCtxCreate");
  if (!get_dev || !get_res || !split || !desc_fn || !create) return CB_OK;
  CUdevice dev;
  CUdevResource all{}, part{}, rest{};
  unsigned nb = 1;
  CUdevResourceDesc desc;
  CUgreenCtx g = nullptr;
  if (get_dev(&dev, device) != CUDA_SUCCESS || get_res(dev, &all, CU_DEV_RESOURCE_TYPE_SM) != CUDA_SUCCESS ||
      split(&part, &nb, &all, &rest, 0, (unsigned)sms) != CUDA_SUCCESS || nb < 1 ||
      desc_fn(&desc, &part, 1) != CUDA_SUCCESS || create(&g, desc, dev, CU_GREEN_CTX_DEFAULT_STREAM) != CUDA_SUCCESS)
    return CB_OK;
  green = g;
  hash_sm_count = (int)part.sm.smCount;
  return CB_OK;
}

cudaError_t Store::create_hash_stream(cudaStream_t &s) {
  if (green) {
    using StreamCreate = CUresult (*)(CUstream *, CUgreenCtx, unsigned, int);
    auto fn = driver_fn<StreamCreate>("cuGreenCtxStreamCreate");
    CUstream cs = nullptr;
    if (fn && fn(&cs, static_cast<CUgreenCtx>(green), CU_STREAM_NON_BLOCKING, 0) == CUDA_SUCCESS) {
      s = reinterpret_cast<cudaStream_t>(cs);
      return cudaSuccess;
    }
    return cudaErrorInvalidResourceHandle;
  }
  return cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
}

int Store::pipeline_init() {
  if (pipeline_ready) return CB_OK;
  if (!hash_sm_count) {
    hash_sm_count = num_sms;
    const int want = cfg.hash_sms > 0 ? cfg.hash_sms : (dht ? num_sms - kDhtSpareSms : 0);
    if (want > 0 && want < num_sms) {
      const int rc = make_hash_green_context(want);
      if (rc) return rc;
    }
  }
  for (HashSlot &h : hslots) {
    if (!h.stream) CB_TRY_CUDA(create_hash_stream(h.stream), "hash stream");
    h.h.flags = cudaHostAllocPortable | cudaHostAllocMapped;
  }
  for (ScratchSlot &s : sslots)
    if (!s.done) CB_TRY_CUDA(cudaEventCreateWithFlags(&s.done, cudaEventDisableTiming), "event");
  if (!put_stream) CB_TRY_CUDA(cudaStreamCreateWithFlags(&put_stream, cudaStreamNonBlocking), "put stream");
  if (!ev_submit) CB_TRY_CUDA(cudaEventCreateWithFlags(&ev_submit, cudaEventDisableTiming), "event");
  if (!d_err_get) {
    CB_TRY_CUDA(cudaMalloc(&d_err_get, sizeof(unsigned)), "error word");
    CB_TRY_CUDA(cudaMemset(d_err_get, 0, sizeof(unsigned)), "error word");
  }
  pipeline_ready = true;
  return CB_OK;
}

// Waits for everything the pipeline has in flight and forgets the batches
// not placed yet (clear(), destruction).
void Store::drop_pipeline() {
  if (!pipeline_ready) return;
  placer_idle();  // assigned groups run (every rank runs them); a failure is already recorded
  for (HashSlot &h : hslots) {
    cudaStreamSynchronize(h.stream);
    h.users = 0;
    h.n = 0;
    h.launched = false;
    h.finished = false;
  }
  hashing_blocks = 0;
  for (ScratchSlot &s : sslots) {
    if (s.pending) cudaEventSynchronize(s.done);
    s.pending = false;
  }
  cudaStreamSynchronize(put_stream);
  aput.clear();
  open_slot = -1;
  inflight_blocks = 0;
  placed_unsettled = false;
  cudaGetLastError();
}

// Batches still queued are dropped (their outputs are never written).
void Store::pipeline_release() {
  placer_join();
  for (HashSlot &h : hslots) {
    if (h.stream) {
      cudaStreamSynchronize(h.stream);
      cudaStreamDestroy(h.stream);
    }
    h.h.release();
    h.d.release();
    h = HashSlot{};
  }
  for (ScratchSlot &s : sslots) {
    if (s.done) {
      cudaEventSynchronize(s.done);
      cudaEventDestroy(s.done);
    }
    s.h.release();
    s.d.release();
    s = ScratchSlot{};
  }
  if (put_stream) {
    cudaStreamSynchronize(put_stream);
    cudaStreamDestroy(put_stream);
    put_stream = nullptr;
  }
  if (ev_submit) cudaEventDestroy(ev_submit);
  ev_submit = nullptr;
  if (green) {  // after its streams
    using Destroy = CUresult (*)(CUgreenCtx);
    if (auto fn = driver_fn<Destroy>("cuGreenCtxDestroy")) fn(static_cast<CUgreenCtx>(green));
    green = nullptr;
  }
  hash_sm_count = 0;
  if (d_err_get) cudaFree(d_err_get);
  d_err_get = nullptr;
  aput.clear();
  open_slot = -1;
  pipeline_ready = false;
}

Store::ScratchSlot *Store::take_scratch(size_t bytes, int &rc) {
  ScratchSlot &s = sslots[sslot_next];
  sslot_next = (sslot_next + 1) % kScratchSlots;
  rc = CB_OK;
  if (s.pending) {  // its previous kernels must be done reading it
    cudaError_t e = cudaEventSynchronize(s.done);
    if (e != cudaSuccess) {
      rc = cuda_fail(e, "stream-ordered kernel");
      return nullptr;
    }
    s.pending = false;
  }
  cudaError_t e = s.h.ensure(bytes);
  if (e == cudaSuccess) e = s.d.ensure(bytes);
  if (e != cudaSuccess) {
    rc = cuda_fail(e, "scratch");
    return nullptr;
  }
  return &s;
}

bool Store::scratch_free() const {
  const ScratchSlot &s = sslots[sslot_next];
  // an error is reported by the take_scratch that waits for it
  return !s.pending || cudaEventQuery(s.done) != cudaErrorNotReady;
}

int Store::fence_reads(cudaStream_t st) {
  if (!pipeline_ready) return CB_OK;
  for (ScratchSlot &s : sslots)
    if (s.pending) CB_TRY_CUDA(cudaStreamWaitEvent(st, s.done, 0), "fence");
  return CB_OK;
}

// ------------------------------------------------------------------ put

int Store::launch_open_slot() {
  if (open_slot < 0) return CB_OK;
  HashSlot &h = hslots[open_slot];
  open_slot = -1;
  const size_t o_dig = digest_offset(h.cap);
  uint8_t *hp = static_cast<uint8_t *>(h.h.ptr);
  uint8_t *dp = static_cast<uint8_t *>(h.d.ptr);
  uint64_t bytes = 0;
  const HashJob *jobs = reinterpret_cast<const HashJob *>(hp);
  for (int i = 0; i < h.n; ++i) bytes += jobs[i].size;
  CB_TRY_CUDA(cudaMemcpyAsync(dp, hp, sizeof(HashJob) * h.n, cudaMemcpyHostToDevice, h.stream), "H2D jobs");
  // The kernel is the last operation on its stream: it writes the digests
  // straight into the slot's mapped host buffer, and completion is read from
  // the stream itself (cudaStreamQuery / cudaStreamSynchronize). An
  // operation queued after a long kernel (a D2H copy, an event record, the
  // timing events of profiling) blocks the hardware queue it shares with
  // other streams until the kernel ends: with dozens of hash streams that
  // held back the placements' copies and a DHT member's collectives for tens
  // of milliseconds (and, as timing events, halved the hashing throughput).
  // Bytes and launch counts are kept; a caller times the hashing as a whole
  // (the put phase) on its own stream.
  void *hdig = nullptr;
  CB_TRY_CUDA(cudaHostGetDevicePointer(&hdig, hp + o_dig, 0), "mapped digests");
  CB_TRY_CUDA(launch_sha256_batch(reinterpret_cast<const HashJob *>(dp), h.n, static_cast<uint32_t *>(hdig),
                                  hash_lanes, d_err, h.stream, nullptr, /*many_chains=*/true),
              "sha256 launch");
  launches++;
  prof_bytes[0] += bytes;
  prof_launches[0]++;
  h.launched = true;
  h.finished = false;
  hashing_blocks += (uint64_t)h.n;
  return CB_OK;
}

void Store::refresh_hashing() {
  for (HashSlot &h : hslots) {
    if (!h.launched || h.finished) continue;
    if (cudaStreamQuery(h.stream) != cudaSuccess) continue;  // not ready (or an error the wait reports)
    h.finished = true;
    hashing_blocks -= (uint64_t)h.n;
  }
}

bool Store::front_ready() const {
  if (aput.empty()) return false;
  const AsyncPut &f = aput.front();
  return f.slot < 0 || hslots[f.slot].finished;
}

int Store::put_async(const uint64_t *ptrs, const uint64_t *sizes, const uint8_t *is_prefix, const uint8_t *keys_in,
                     int n, uint8_t *keys_out, uint8_t *status_out, uint64_t *ticket, cudaStream_t st) {
  int rc = pipeline_init();
  if (rc) return rc;
  AsyncPut b;
  b.ticket = next_ticket;
  b.ptrs.assign(ptrs, ptrs + n);
  b.sizes.assign(sizes, sizes + n);
  if (is_prefix) b.prefix.assign(is_prefix, is_prefix + n);
  if (keys_in) b.keys_in.assign(keys_in, keys_in + 16ull * n);
  b.keys_out = keys_out;
  b.status_out = status_out;
  if (!keys_in && n > 0) {
    // A DHT member gives every batch its own launch, so that slot reuse
    // (and the placements it may force) happens at the same call on every
    // rank; one GPU queues small batches into a shared launch.
    if (open_slot >= 0 && (dht || hslots[open_slot].n + n > hslots[open_slot].cap)) {
      rc = launch_open_slot();
      if (rc) return rc;
    }
    if (open_slot < 0) {
      const int s = hslot_next;
      if (dht) {  // its batch is long assigned: wait until the placement thread has placed it
        rc = dht_slot_free(s);
        if (rc) return rc;
      } else {
        while (hslots[s].users > 0) {  // its batches are the oldest in flight: place them
          rc = place_oldest();
          if (rc) return rc;
        }
      }
      HashSlot &h = hslots[s];
      if (h.launched && !h.finished) hashing_blocks -= (uint64_t)h.n;  // placed, so hashed
      const int cap = std::max(n, kLaunchBlocks);
      const size_t bytes = digest_offset(cap) + 32ull * cap;
      CB_TRY_CUDA(h.h.ensure(bytes), "pinned hash slot");
      CB_TRY_CUDA(h.d.ensure(bytes), "device hash slot");
      h.cap = cap;
      h.n = 0;
      h.users = 0;
      h.launched = false;
      h.finished = false;
      open_slot = s;
      hslot_next = (s + 1) % kHashSlots;
    }
    HashSlot &h = hslots[open_slot];
    HashJob *jobs = static_cast<HashJob *>(h.h.ptr) + h.n;
    for (int i = 0; i < n; ++i) jobs[i] = HashJob{ptrs[i], sizes[i]};
    b.slot = open_slot;
    b.off = h.n;
    h.n += n;
    h.users++;
    // the hash reads the blocks after the caller's earlier work on st
    CB_TRY_CUDA(cudaEventRecord(ev_submit, st), "event");
    CB_TRY_CUDA(cudaStreamWaitEvent(h.stream, ev_submit, 0), "wait");
    if (dht || h.n >= kLaunchBlocks) {
      rc = launch_open_slot();
      if (rc) return rc;
    }
  }
  next_ticket++;
  *ticket = b.ticket;
  inflight_blocks += (uint64_t)n;
  aput.push_back(std::move(b));
  if (dht) {
    // assignment by counts only: every rank assigns the same groups at the
    // same call
    if (aput.size() > kDhtPending) {
      rc = assign_dht_group(kDhtGroup);
      if (rc) return rc;
    }
    // at most `limit` blocks hash at once: wait for this GPU's own oldest
    // launch (no collective depends on it)
    const uint64_t limit = cfg.pipeline_blocks ? cfg.pipeline_blocks : kDefaultPipelineBlocks;
    for (;;) {
      refresh_hashing();
      if (hashing_blocks <= limit) break;
      HashSlot *oldest = nullptr;
      for (int k = 1; k <= kHashSlots && !oldest; ++k) {  // launch order = slot ring order
        HashSlot &h = hslots[(hslot_next + k - 1) % kHashSlots];
        if (h.launched && !h.finished) oldest = &h;
      }
      if (!oldest) break;
      CB_TRY_CUDA(cudaStreamSynchronize(oldest->stream), "pipelined hash");
    }
    return CB_OK;
  }
  // Batches whose digests are back are placed (host planning; the scatter
  // overlaps the hashes still running) as long as their scatter can be
  // queued without waiting for an earlier one to finish: the scatter runs
  // at a fraction of HBM speed beside dozens of hash launches, and a host
  // blocked on it would delay the caller's next submission - the launch of
  // the next hash. At most `limit` blocks hash at once; beyond that the host
  // waits for the oldest launch.
  const uint64_t limit = cfg.pipeline_blocks ? cfg.pipeline_blocks : kDefaultPipelineBlocks;
  for (;;) {
    refresh_hashing();
    while (front_ready() && scratch_free()) {
      rc = place_oldest();
      if (rc) return rc;
    }
    if (hashing_blocks <= limit) break;
    HashSlot *oldest = nullptr;  // the launch of the oldest batch still hashing
    for (const AsyncPut &b : aput) {
      if (b.slot >= 0 && hslots[b.slot].launched && !hslots[b.slot].finished) {
        oldest = &hslots[b.slot];
        break;
      }
    }
    if (!oldest) break;
    CB_TRY_CUDA(cudaStreamSynchronize(oldest->stream), "pipelined hash");
  }
  return CB_OK;
}

// Placement thread: one group of batches in one collective put. Their
// blocks go out as one request batch, each tagged with its batch's position
// in the group; owners apply them in (batch, source rank, index) order, so
// dedup decisions and statuses equal those of one collective step per batch,
// for a fraction of the exchanges and synchronisations. One difference under
// capacity pressure: the group is one owner plan, and a plan never demotes
// the blocks it places itself, so a new block that finds no HBM room goes to
// the owner's DRAM tier (through the outbox) where a per-batch step could
// have demoted an earlier batch's block of the same group instead.
// The thread only reads the batches' hash slots (their digests and events);
// the caller's fields of those slots are left to the caller.
int Store::place_dht_batches(std::vector<AsyncPut> &g) {
  size_t total = 0;
  for (const AsyncPut &b : g) total += b.sizes.size();
  std::vector<uint64_t> ptrs, sizes;
  std::vector<uint8_t> prefix, keys16;
  std::vector<uint16_t> step;
  ptrs.reserve(total);
  sizes.reserve(total);
  prefix.reserve(total);
  step.reserve(total);
  keys16.reserve(16 * total);
  for (size_t j = 0; j < g.size(); ++j) {
    AsyncPut &b = g[j];
    const size_t n = b.sizes.size();
    const uint8_t *dig = nullptr;
    if (b.slot >= 0) {
      HashSlot &h = hslots[b.slot];
      CB_TRY_CUDA(cudaStreamSynchronize(h.stream), "pipelined hash");
      dig = static_cast<const uint8_t *>(h.h.ptr) + digest_offset(h.cap) + 32ull * b.off;
    }
    for (size_t i = 0; i < n; ++i) {
      ptrs.push_back(b.ptrs[i]);
      sizes.push_back(b.sizes[i]);
      prefix.push_back(b.prefix.empty() ? 0 : b.prefix[i]);
      step.push_back((uint16_t)j);
      const uint8_t *k = dig ? dig + 32 * i : b.keys_in.data() + 16 * i;
      keys16.insert(keys16.end(), k, k + 16);
    }
  }
  std::vector<uint8_t> kout(16 * std::max<size_t>(total, 1)), sout(std::max<size_t>(total, 1));
  const int rc = dht_put(reinterpret_cast<const void *const *>(ptrs.data()), sizes.data(), prefix.data(),
                         keys16.data(), (int)total, CB_MEM_DEVICE, kout.data(), sout.data(), put_stream, step.data());
  if (rc) return rc;
  size_t off = 0;
  for (AsyncPut &b : g) {
    const size_t n = b.sizes.size();
    if (b.keys_out) memcpy(b.keys_out, kout.data() + 16 * off, 16 * n);
    if (b.status_out) memcpy(b.status_out, sout.data() + off, n);
    off += n;
  }
  return CB_OK;
}

// Caller: the `count` oldest unassigned batches go to the placement thread
// as one group (started on first use).
int Store::assign_dht_group(size_t count) {
  count = std::min(count, aput.size());
  if (!count) return CB_OK;
  std::vector<AsyncPut> g;
  g.reserve(count);
  for (size_t j = 0; j < count; ++j) {
    inflight_blocks -= (uint64_t)aput.front().sizes.size();
    g.push_back(std::move(aput.front()));
    aput.pop_front();
  }
  std::lock_guard<std::mutex> lk(pmu);
  if (!placer.joinable()) {
    placer_stop = false;
    placer = std::thread([this] { placer_loop(); });
    placer_id = placer.get_id();  // set under pmu, which the thread takes before any work
  }
  pgroups.push_back(std::move(g));
  pcv.notify_all();
  return CB_OK;
}

void Store::placer_loop() {
  std::unique_lock<std::mutex> lk(pmu);
  cudaSetDevice(device);
  for (;;) {
    pcv.wait(lk, [&] { return placer_stop || !pgroups.empty(); });
    if (pgroups.empty()) return;  // asked to stop with nothing left
    std::vector<AsyncPut> g = std::move(pgroups.front());
    pgroups.pop_front();
    placer_busy = true;
    const bool skip = placer_rc != 0;  // after a failure nothing more is placed
    lk.unlock();
    int rc = CB_OK;
    if (!skip) {
      try {
        rc = place_dht_batches(g);
      } catch (const std::bad_alloc &) {
        rc = fail(CB_ERR_NOSPACE, "host allocation failed");
      } catch (const std::exception &ex) {
        rc = fail(CB_ERR_STATE, "%s", ex.what());
      }
    }
    const std::string err = rc ? last_error_copy() : std::string();
    lk.lock();
    for (AsyncPut &b : g)
      if (b.slot >= 0) hslots[b.slot].users--;
    if (rc) {
      placer_rc = rc;
      placer_err = err;
    } else if (!skip && !g.empty()) {
      placed_ticket = g.back().ticket;
    }
    placer_busy = false;
    pcv.notify_all();
  }
}

// Caller: waits until every assigned group is placed. A failure of the
// placement thread is returned once; the store's state is then lost (its
// metadata may be ahead of its memory and its peers') until clear().
int Store::placer_idle() {
  std::unique_lock<std::mutex> lk(pmu);
  if (!placer.joinable()) return CB_OK;
  pcv.wait(lk, [&] { return pgroups.empty() && !placer_busy; });
  if (!placer_rc) return CB_OK;
  const int rc = placer_rc;
  placer_rc = 0;
  if (lost.empty()) lost = placer_err;
  {
    std::lock_guard<std::mutex> g(err_mu);
    last_error = placer_err;
  }
  return rc;
}

// Caller: hash slot s may be reused once the thread has placed its batch.
int Store::dht_slot_free(int s) {
  for (;;) {
    bool assigned = true;
    for (const AsyncPut &b : aput) assigned &= b.slot != s;
    if (assigned) break;
    const int rc = assign_dht_group(kDhtGroup);
    if (rc) return rc;
  }
  std::unique_lock<std::mutex> lk(pmu);
  pcv.wait(lk, [&] { return hslots[s].users == 0 || placer_rc != 0; });
  if (!placer_rc) return CB_OK;
  lk.unlock();
  return placer_idle();
}

void Store::placer_join() {
  {
    std::lock_guard<std::mutex> lk(pmu);
    if (!placer.joinable()) return;
    placer_stop = true;
    pcv.notify_all();
  }
  placer.join();  // runs what is assigned first
  std::lock_guard<std::mutex> lk(pmu);
  placer = std::thread();
  placer_id = std::thread::id();
  placer_rc = 0;
}

// Places the oldest submitted batch (waiting for its digests if need be).
int Store::place_oldest() {
  if (dht) {
    const int rc = assign_dht_group(1);
    return rc ? rc : placer_idle();
  }
  AsyncPut &b = aput.front();
  const int n = (int)b.sizes.size();
  std::vector<HKey> keys(n);
  int rc = CB_OK;
  if (b.slot >= 0) {
    HashSlot &h = hslots[b.slot];
    if (!h.launched) {
      rc = launch_open_slot();  // b is among the open slot's batches
      if (rc) return rc;
    }
    CB_TRY_CUDA(cudaStreamSynchronize(h.stream), "pipelined hash");
    if (!h.finished) {
      h.finished = true;
      hashing_blocks -= (uint64_t)h.n;
    }
    const uint8_t *dig = static_cast<const uint8_t *>(h.h.ptr) + digest_offset(h.cap) + 32ull * b.off;
    for (int i = 0; i < n; ++i) keys[i] = to_hkey(dig + 32ull * i);
  } else {
    for (int i = 0; i < n; ++i) keys[i] = to_hkey(b.keys_in.data() + 16ull * i);
  }
  rc = n ? place_batch(keys, b) : CB_OK;
  if (rc) return rc;
  if (b.slot >= 0) hslots[b.slot].users--;
  inflight_blocks -= (uint64_t)n;
  placed_ticket = b.ticket;
  aput.pop_front();
  return CB_OK;
}

// 1 GPU: the synchronous put's plan and scatter, stream-ordered on
// put_stream with descriptors in a scratch slot; nothing waits here.
int Store::place_batch(const std::vector<HKey> &keys, AsyncPut &b) {
  Trace tr("cb.place");
  const int n = (int)keys.size();
  int rc = reserve_index((uint64_t)n, put_stream);
  if (rc) return rc;
  PutPlan &plan = put_plan;
  policy.plan_put(keys.data(), b.sizes.data(), b.prefix.empty() ? nullptr : b.prefix.data(), n,
                  cfg.dedup_enabled != 0, plan);
  plan_open = true;
  rc = fence_reads(put_stream);  // extents a stream-ordered gather still reads
  if (rc) return rc;
  rc = run_moves(plan.moves, plan.dropped, put_stream);
  if (rc) return rc;
  if (!plan.places.empty()) {
    ScratchSlot *sl = take_scratch(4096, rc);
    if (!sl) return rc;
    // the TMA engine: one lane per SM issues the bulk copies, so the scatter
    // takes next to no issue slots from the hash warps beside it
    rc = enqueue_places(plan, b.ptrs.data(), put_stream, sl->h, sl->d, copy_engine, kScatterLsuCtasPerSm);
    if (rc) return rc;
    CB_TRY_CUDA(cudaEventRecord(sl->done, put_stream), "event");
    sl->pending = true;
  }
  policy.commit();
  plan_open = false;
  placed_unsettled = true;
  for (int i = 0; i < n; ++i) {
    if (b.keys_out) {
      memcpy(b.keys_out + 16ull * i, &keys[i].lo, 8);
      memcpy(b.keys_out + 16ull * i + 8, &keys[i].hi, 8);
    }
    if (b.status_out) b.status_out[i] = plan.status[i];
  }
  return CB_OK;
}

int Store::place_until(uint64_t ticket) {
  // batches still queued for a launch start hashing now, beside the ones
  // whose placements come first
  if (open_slot >= 0 && !aput.empty() && aput.front().ticket <= ticket) {
    const int rc = launch_open_slot();
    if (rc) return rc;
  }
  while (!aput.empty() && aput.front().ticket <= ticket) {
    int rc;
    if (dht) {  // groups of up to kDhtGroup batches, the same on every rank
      size_t cnt = 0;
      while (cnt < aput.size() && cnt < kDhtGroup && aput[cnt].ticket <= ticket) ++cnt;
      rc = assign_dht_group(cnt);
    } else {
      rc = place_oldest();
    }
    if (rc) return rc;
  }
  return dht ? placer_idle() : CB_OK;
}

// Device work of the placements made so far is complete; a device-side
// error of one of them is returned (and, since the host metadata already
// records those placements, leaves the store refusing data calls).
int Store::finish_placements() {
  if (!placed_unsettled) return CB_OK;
  CB_TRY_CUDA(cudaStreamSynchronize(put_stream), "placements");
  placed_unsettled = false;
  const int rc = read_error_word(d_err, put_stream);
  if (rc) plan_open = true;
  return rc;
}

// Places every batch up to `ticket` (they need not be hashed yet) and
// waits for their device work; later batches keep hashing.
int Store::put_wait(uint64_t ticket) {
  int rc = place_until(ticket);
  if (rc) return rc;
  return finish_placements();
}

int Store::settle() {
  if (!pipeline_ready) return CB_OK;
  if (!lost.empty()) {  // nothing more is placed on a store that lost its state
    drop_pipeline();
    return CB_OK;
  }
  int rc = place_until(UINT64_MAX);
  if (rc) return rc;
  bool gathers = false;
  for (ScratchSlot &s : sslots) {
    if (!s.pending) continue;
    CB_TRY_CUDA(cudaEventSynchronize(s.done), "stream-ordered kernel");
    s.pending = false;
    gathers = true;
  }
  rc = finish_placements();
  if (rc) return rc;
  // an error of a stream-ordered get changed nothing in the store: report it
  return gathers ? read_error_word(d_err_get, put_stream) : CB_OK;
}

// ------------------------------------------------------------------ get

int Store::get_async(const uint8_t *keys, int n, const uint64_t *outs, const uint64_t *caps, uint64_t *sizes_out,
                     uint8_t *found_out, cudaStream_t st) {
  int rc = pipeline_init();
  if (rc) return rc;
  // every put submitted earlier is visible to this get
  if (!aput.empty()) {
    rc = place_until(UINT64_MAX);
    if (rc) return rc;
  }
  // One lookup per key, which also marks the hit most recently used
  // (CascadeStore::get touches on hit, src/cascade_core.cpp:1281). A batch
  // that reads the DRAM tier (and may promote) takes the synchronous path
  // instead, which touches every key in batch order itself; the keys this
  // loop touched before the first DRAM hit are then touched again in the
  // same order, which leaves the LRU order of a single pass.
  std::vector<const BlockMeta *> meta(n);
  for (int i = 0; i < n; ++i) {
    meta[i] = policy.find_touch(to_hkey(keys + 16ull * i));
    if (meta[i] && meta[i]->tier != kTierHbm && meta[i]->size <= caps[i]) {
      rc = settle();
      if (rc) return rc;
      return get_device(keys, n, outs, caps, sizes_out, found_out, st);
    }
  }
  if (placed_unsettled) {  // the gather reads what the pipelined scatters wrote
    CB_TRY_CUDA(cudaEventRecord(ev_submit, put_stream), "event");
    CB_TRY_CUDA(cudaStreamWaitEvent(st, ev_submit, 0), "wait");
  }
  const bool inject = inject_get_error;
  inject_get_error = false;
  const int nd = n + (inject ? 1 : 0);
  const size_t o_us = align_up(sizeof(CopyDesc) * nd, 256);
  const size_t bytes = o_us + 4ull * (nd + 1);
  ScratchSlot *sl = take_scratch(bytes, rc);
  if (!sl) return rc;
  uint8_t *h = static_cast<uint8_t *>(sl->h.ptr);
  CopyDesc *desc = reinterpret_cast<CopyDesc *>(h);
  uint32_t *us = reinterpret_cast<uint32_t *>(h + o_us);
  uint32_t total = 0;
  uint64_t moved = 0;
  for (int i = 0; i < n; ++i) {
    const BlockMeta *m = meta[i];
    us[i] = total;
    if (!m) {
      desc[i] = CopyDesc{0, 0, 0, 0};
      sizes_out[i] = 0;
      found_out[i] = CB_FOUND_MISS;
      misses++;
      continue;
    }
    local_gpu_hits++;
    sizes_out[i] = m->size;
    if (m->size > caps[i]) {
      desc[i] = CopyDesc{0, 0, 0, 0};
      found_out[i] = CB_FOUND_LOCAL_HBM | CB_FOUND_NOT_COPIED;
      continue;
    }
    found_out[i] = CB_FOUND_LOCAL_HBM;
    desc[i] = CopyDesc{(uint64_t)pool + m->off, outs[i], m->size, 0};
    total += (uint32_t)((m->size + kCopyUnit - 1) / kCopyUnit);
    moved += m->size;
  }
  if (inject) {  // self-test: one descriptor whose kernel reports an error
    us[n] = total;
    desc[n] = CopyDesc{0, 0, 16, kCopyFault};
    total += 1;
  }
  us[nd] = total;
  if (total) {
    uint8_t *d = static_cast<uint8_t *>(sl->d.ptr);
    CB_TRY_CUDA(cudaMemcpyAsync(d, h, bytes, cudaMemcpyHostToDevice, st), "H2D gather");
    CB_TRY_CUDA(timed(2, moved, st,
                      [&] {
                        return launch_batch_copy(reinterpret_cast<const CopyDesc *>(d),
                                                 reinterpret_cast<const uint32_t *>(d + o_us), nd, total, copy_engine,
                                                 d_err_get, num_sms, st);
                      }),
                "gather");
    CB_TRY_CUDA(cudaEventRecord(sl->done, st), "event");
    sl->pending = true;
  }
  return CB_OK;
}

}  // namespace cb
