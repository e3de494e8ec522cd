// The B200 store behind the C ABI: one HBM slab pool + device index per GPU,
// an optional pinned DRAM arena, and the host policy. Every batch becomes a
// handful of launches: SHA-256 -> (host dedup/placement plan) -> tier moves ->
// scatter -> index mutations for put; index lookup -> gather for get (with
// the promotions of DRAM hits planned before the lookup, their room-making
// demotions on a second stream). Moves between HBM and the pinned arena of
// blocks >= 256 KiB use the copy engines (INT8-packed ones through an HBM
// staging area); smaller ones use the copy kernels on the mapped arena.
//
// Reference call stacks this replaces:
//   put  : DistributedStore::put (src/distributed_backend.cpp:601-692) ->
//          DistributedGPUBackend::put_local (:412-436) -> GPUBackend::put
//          (src/gpu_backend.cu:300-351, one cudaMemcpyAsync per block)
//   get  : DistributedStore::get (:698-795) -> get_local scans every GPU
//          (:455-464) -> read_block_to_host (src/gpu_backend.cu:390-425)
//   evict: DistributedStore::evict_gpu_to_dram (:876-941) ->
//          GPUBackend::evict_for_space (src/gpu_backend.cu:514-537)
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <climits>
#include <mutex>
#include <new>
#include <string>
#include <vector>

#include <cuda.h>  // CUpointer_attribute (the entry point is fetched at run time)

#include "cascade_b200.h"
#include "kernels.cuh"
#include "policy.hpp"
#include "store.hpp"

namespace cb {

thread_local std::string g_create_error;

namespace {

inline void from_hkey(const HKey &k, uint8_t *p) {
  memcpy(p, &k.lo, 8);
  memcpy(p + 8, &k.hi, 8);
}

inline uint64_t meta_word(uint64_t size, uint8_t prefix) {
  return (size & kSizeMask) | (prefix ? kMetaPrefix : 0);
}

}  // namespace

// ------------------------------------------------------------ allocations

namespace {
using PtrAttrFn = CUresult (*)(void *, CUpointer_attribute, CUdeviceptr);
PtrAttrFn pointer_attribute_fn() {
  static const PtrAttrFn fn = [] {
    void *f = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuPointerGetAttribute", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<PtrAttrFn>(nullptr);
    return reinterpret_cast<PtrAttrFn>(f);
  }();
  return fn;
}
}  // namespace

AddrRange alloc_range(const void *p) {
  const uint64_t a = reinterpret_cast<uint64_t>(p);
  const PtrAttrFn fn = pointer_attribute_fn();
  if (!fn) return AddrRange{a, a};
  CUdeviceptr start = 0;
  size_t size = 0;
  if (fn(&start, CU_POINTER_ATTRIBUTE_RANGE_START_ADDR, static_cast<CUdeviceptr>(a)) != CUDA_SUCCESS) {
    cudaPointerAttributes at;
    const bool known = cudaPointerGetAttributes(&at, p) == cudaSuccess && at.type != cudaMemoryTypeUnregistered;
    cudaGetLastError();
    return known ? AddrRange{a, a} : AddrRange{0, UINT64_MAX};  // pageable host memory: any extent
  }
  if (fn(&size, CU_POINTER_ATTRIBUTE_RANGE_SIZE, static_cast<CUdeviceptr>(a)) != CUDA_SUCCESS) return AddrRange{a, a};
  return AddrRange{static_cast<uint64_t>(start), static_cast<uint64_t>(start) + size};
}

// ------------------------------------------------------------ buffers

cudaError_t PinnedBuf::ensure(size_t bytes) {
  if (bytes <= cap) return cudaSuccess;
  if (ptr) cudaFreeHost(ptr);
  ptr = nullptr;
  cap = 0;
  const size_t want = std::max<size_t>(align_up(bytes + bytes / 2, 4096), 1 << 20);
  cudaError_t e = cudaHostAlloc(&ptr, want, flags);
  if (e == cudaSuccess) cap = want;
  return e;
}
void PinnedBuf::release() {
  if (ptr) cudaFreeHost(ptr);
  ptr = nullptr;
  cap = 0;
}

cudaError_t DevBuf::ensure(size_t bytes) {
  if (bytes <= cap) return cudaSuccess;
  if (ptr) cudaFree(ptr);
  ptr = nullptr;
  cap = 0;
  const size_t want = std::max<size_t>(align_up(bytes + bytes / 2, 4096), 1 << 20);
  cudaError_t e = cudaMalloc(&ptr, want);
  if (e == cudaSuccess) cap = want;
  return e;
}
void DevBuf::release() {
  if (ptr) cudaFree(ptr);
  ptr = nullptr;
  cap = 0;
}

// ------------------------------------------------------------ store

int Store::fail(int code, const char *fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  std::lock_guard<std::mutex> g(err_mu);
  last_error = buf;
  return code;
}

int Store::cuda_fail(cudaError_t e, const char *what) {
  return fail(CB_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

#define CB_TRY(call, what)                     \
  do {                                         \
    cudaError_t _e = (call);                   \
    if (_e != cudaSuccess) return cuda_fail(_e, what); \
  } while (0)

Store::Store(const cb_config &c)
    : cfg(c), policy(c.gpu_capacity_bytes, c.dram_capacity_bytes, c.semantic_eviction != 0) {}

int Store::init() {
  device = cfg.device;
  int ndev = 0;
  CB_TRY(cudaGetDeviceCount(&ndev), "cudaGetDeviceCount");
  if (device < 0 || device >= ndev) return fail(CB_ERR_ARG, "device %d out of range (%d)", device, ndev);
  CB_TRY(cudaSetDevice(device), "cudaSetDevice");
  CB_TRY(cudaDeviceGetAttribute(&num_sms, cudaDevAttrMultiProcessorCount, device), "sm count");
  // A blocking stream: it is ordered with the legacy default stream, so a
  // caller whose current stream is the default one (handle 0, which reaches
  // the C ABI as NULL) sees its earlier writes before the store reads them.
  CB_TRY(cudaStreamCreateWithFlags(&own_stream, cudaStreamDefault), "stream");
  pool_bytes = policy.hbm_capacity() / 256 * 256;
  if (pool_bytes) CB_TRY(cudaMalloc(&pool, pool_bytes), "HBM pool cudaMalloc");
  CB_TRY(cudaMalloc(&d_err, sizeof(unsigned)), "error word");
  CB_TRY(cudaMemset(d_err, 0, sizeof(unsigned)), "error word");
  const int log2 = cfg.index_log2 > 0 ? cfg.index_log2 : 16;
  CB_TRY(alloc_table((uint64_t)1 << log2), "index");
  CB_TRY(h_err.ensure(64), "pinned");
  profile = cfg.profile != 0;
  policy.set_compression(cfg.kv_compression != 0);
  hash_lanes = (cfg.hash_lanes == 8 || cfg.hash_lanes == 16) ? cfg.hash_lanes : 32;
  CB_TRY(cudaStreamCreateWithFlags(&move_stream, cudaStreamNonBlocking), "move stream");
  CB_TRY(cudaEventCreateWithFlags(&ev_move_in, cudaEventDisableTiming), "event");
  CB_TRY(cudaEventCreateWithFlags(&ev_move_done, cudaEventDisableTiming), "event");
  CB_TRY(cudaStreamCreateWithFlags(&copy_stream, cudaStreamNonBlocking), "copy stream");
  CB_TRY(cudaEventCreateWithFlags(&ev_reset, cudaEventDisableTiming), "event");
  CB_TRY(cudaEventCreateWithFlags(&ev_copies, cudaEventDisableTiming), "event");
  CB_TRY(cudaMalloc(&d_progress, 256), "progress word");
  return CB_OK;
}

Store::~Store() {
  if (device >= 0) cudaSetDevice(device);
  if (own_stream) cudaStreamSynchronize(own_stream);
  pipeline_release();
  dht_detach();
  if (pool) cudaFree(pool);
  if (table) cudaFree(table);
  if (d_err) cudaFree(d_err);
  if (dram_host) cudaFreeHost(dram_host);
  d_scratch.release();
  h_scratch.release();
  h_out.release();
  h_err.release();
  d_staging.release();
  d_pack.release();
  d_unpack.release();
  if (move_stream) {
    cudaStreamSynchronize(move_stream);
    cudaStreamDestroy(move_stream);
  }
  if (peer_stream) {
    cudaStreamSynchronize(peer_stream);
    cudaStreamDestroy(peer_stream);
  }
  if (ev_peer_in) cudaEventDestroy(ev_peer_in);
  if (ev_peer_out) cudaEventDestroy(ev_peer_out);
  if (ev_move_in) cudaEventDestroy(ev_move_in);
  if (ev_move_done) cudaEventDestroy(ev_move_done);
  for (cudaEvent_t e : prof_events) cudaEventDestroy(e);
  h_mscratch.release();
  d_mscratch.release();
  if (copy_stream) {
    cudaStreamSynchronize(copy_stream);
    cudaStreamDestroy(copy_stream);
  }
  if (ev_reset) cudaEventDestroy(ev_reset);
  if (ev_copies) cudaEventDestroy(ev_copies);
  if (d_progress) cudaFree(d_progress);
  h_progress.release();
  if (own_stream) cudaStreamDestroy(own_stream);
}

// The new index is allocated and cleared before the old one is released, so
// a growth that fails leaves the store on its previous, still valid index.
cudaError_t Store::alloc_table(uint64_t slots) {
  Slot *t = nullptr;
  cudaError_t e = cudaMalloc(&t, slots * sizeof(Slot));
  if (e != cudaSuccess) return e;
  e = cudaMemset(t, 0, slots * sizeof(Slot));
  if (e != cudaSuccess) {
    cudaFree(t);
    return e;
  }
  if (table) cudaFree(table);
  table = t;
  table_slots = slots;
  table_used = 0;
  table_tombs = 0;
  return cudaSuccess;
}

cudaError_t Store::ensure_dram() {
  if (dram_host || policy.dram_capacity() == 0) return cudaSuccess;
  dram_bytes = policy.dram_capacity() / 256 * 256;
  cudaError_t e = cudaHostAlloc(reinterpret_cast<void **>(&dram_host), dram_bytes,
                                cudaHostAllocMapped | cudaHostAllocPortable);
  if (e != cudaSuccess) {
    dram_host = nullptr;
    return e;
  }
  return cudaHostGetDevicePointer(reinterpret_cast<void **>(&dram_dev), dram_host, 0);
}

// Grows (or compacts) the device index so that `incoming` more keys keep
// the load factor at or below 1/2, rebuilding it from the host metadata.
int Store::reserve_index(uint64_t incoming, cudaStream_t st) {
  const uint64_t live = policy.size();
  if ((table_used + table_tombs + incoming) * 2 <= table_slots) return CB_OK;
  if (dht) {
    // Peers map this index: it is never reallocated while attached.
    if ((live + incoming) <= table_slots - table_slots / 8) return CB_OK;
    return fail(CB_ERR_NOSPACE, "device index full (%llu slots); raise index_log2",
                (unsigned long long)table_slots);
  }
  uint64_t slots = table_slots;
  while ((live + incoming) * 2 > slots) slots *= 2;
  CB_TRY(cudaStreamSynchronize(st), "sync before index rebuild");
  CB_TRY(alloc_table(slots), "index rebuild alloc");
  if (live == 0) return CB_OK;
  std::vector<IndexRec> recs;
  recs.reserve(live);
  policy.for_each([&](const HKey &k, const BlockMeta &m) {
    recs.push_back(IndexRec{k.lo, k.hi, Policy::data_offset(m) | (m.tier == kTierDram ? kLocDram : 0),
                            meta_word(m.size, m.prefix) | (m.packed ? kMetaPacked : 0)});
  });
  const size_t bytes = recs.size() * sizeof(IndexRec);
  CB_TRY(h_scratch.ensure(bytes), "pinned scratch");
  CB_TRY(d_scratch.ensure(bytes), "device scratch");
  memcpy(h_scratch.ptr, recs.data(), bytes);
  CB_TRY(cudaMemcpyAsync(d_scratch.ptr, h_scratch.ptr, bytes, cudaMemcpyHostToDevice, st), "H2D");
  CB_TRY(launch_index_insert(table, table_slots - 1, static_cast<IndexRec *>(d_scratch.ptr),
                             (int)recs.size(), d_err, st),
         "index insert");
  launches++;
  CB_TRY(cudaStreamSynchronize(st), "index rebuild");
  table_used = live;
  return CB_OK;
}

cudaError_t Store::prof_event(cudaEvent_t &e) {
  if (prof_free.empty()) {
    cudaEvent_t ne;
    cudaError_t r = cudaEventCreate(&ne);
    if (r != cudaSuccess) return r;
    prof_events.push_back(ne);
    e = ne;
    return cudaSuccess;
  }
  e = prof_free.back();
  prof_free.pop_back();
  return cudaSuccess;
}

// Launches still running on other streams (pipelined hashes) keep their
// records pending unless `wait` is set.
void Store::resolve_prof(bool wait) {
  size_t keep = 0;
  for (size_t k = 0; k < prof_pending.size(); ++k) {
    const ProfRec r = prof_pending[k];
    if (!wait && cudaEventQuery(r.b) == cudaErrorNotReady) {
      prof_pending[keep++] = r;
      continue;
    }
    float ms = 0.f;
    if (cudaEventSynchronize(r.b) == cudaSuccess && cudaEventElapsedTime(&ms, r.a, r.b) == cudaSuccess) {
      prof_ns[r.kind] += (uint64_t)(ms * 1.0e6);
      prof_bytes[r.kind] += r.bytes;
      prof_launches[r.kind]++;
    }
    prof_free.push_back(r.a);
    prof_free.push_back(r.b);
  }
  prof_pending.resize(keep);
  cudaGetLastError();  // a not-ready query leaves nothing sticky, but be sure
}

// Reads and clears the device error word (after a stream sync).
int Store::check_device_error(cudaStream_t st) { return read_error_word(d_err, st); }

int Store::read_error_word(unsigned *word, cudaStream_t st) {
  CB_TRY(cudaMemcpyAsync(h_err.ptr, word, sizeof(unsigned), cudaMemcpyDeviceToHost, st), "D2H err");
  CB_TRY(cudaStreamSynchronize(st), "stream sync");
  resolve_prof();
  const unsigned e = *static_cast<unsigned *>(h_err.ptr);
  if (!e) return CB_OK;
  CB_TRY(cudaMemsetAsync(word, 0, sizeof(unsigned), st), "clear err");
  CB_TRY(cudaStreamSynchronize(st), "stream sync");
  if (e & kErrTimeout) return fail(CB_ERR_TIMEOUT, "device wait timed out (error bits 0x%x)", e);
  return fail(CB_ERR_DEVICE, "device-side check failed (error bits 0x%x)", e);
}

// ------------------------------------------------------------ packing



// Copy descriptors + unit prefix for a list of (src, dst, size, flags).
static uint32_t units_of(uint64_t size) {
  return (uint32_t)((size + kCopyUnit - 1) / kCopyUnit);
}

// Executes tier moves (HBM->DRAM first, then DRAM->HBM), index updates for
// moved blocks and index erases for dropped blocks, stream-ordered on st.
int Store::run_moves(const std::vector<TierMove> &moves, const std::vector<HKey> &dropped, cudaStream_t st,
                     const std::function<int()> &concurrent) {
  Trace tr("cb.tier_moves");
  if (moves.empty() && dropped.empty()) return concurrent ? concurrent() : CB_OK;
  if (fake_move_failures > 0) {  // before any copy is issued, like a failed arena allocation
    --fake_move_failures;
    return fail(CB_ERR_NOSPACE, "injected tier-move failure (self-test)");
  }
  bool need_dram = false;
  for (const auto &m : moves) need_dram |= (m.src_tier == kTierDram || m.dst_tier == kTierDram);
  if (need_dram) {
    cudaError_t e = ensure_dram();
    if (e != cudaSuccess) return cuda_fail(e, "pinned DRAM arena cudaHostAlloc");
  }
  // Groups: 0 demotions copied by the LSU kernel, 1 demotions packed to INT8
  // straight into the mapped arena (kv_compression), 2 promotions by kernel
  // (copies from a device copy, unpacks, small blocks), 3 demotions and 4
  // promotions of large plain blocks by the copy engines (cudaMemcpyAsync:
  // the DMA engines move each direction at the link rate and overlap each
  // other, which SM-issued host-memory traffic does not), 5 large demotions
  // packed into an HBM staging area and moved by the D2H copy engine. Every
  // promotion runs after every demotion: its HBM destination may be an
  // extent a demotion of the same plan vacated.
  constexpr int kGroups = 6;
  std::vector<const TierMove *> grp[kGroups];
  std::vector<uint64_t> pslot;  // group 5: staging offsets of the packed images
  uint64_t pstage = 0;
  for (const auto &m : moves) {
    const bool big = !m.src_dev && m.size >= kDmaMinBytes;
    int g;
    if (m.dst_tier == kTierDram && m.op == kMovePack) {
      const uint64_t slot = align_up(kPackLead + packed_bytes(m.size), 256);
      g = (big && pstage + slot <= kPackStagingBytes) ? 5 : 1;
      if (g == 5) {
        pslot.push_back(pstage);
        pstage += slot;
      }
    } else if (m.dst_tier == kTierDram) {
      g = (big && m.op == kMoveCopy) ? 3 : 0;
    } else {
      g = (big && m.op == kMoveCopy) ? 4 : 2;
    }
    grp[g].push_back(&m);
  }
  if (pstage) CB_TRY(d_pack.ensure(pstage), "packing staging");  // before any concurrent work
  const int nm = (int)moves.size(), nd = (int)dropped.size();
  Layout L;
  const size_t o_desc = L.add(sizeof(CopyDesc) * nm);
  size_t o_us[kGroups];
  for (int g = 0; g < kGroups; ++g) o_us[g] = L.add(sizeof(uint32_t) * (grp[g].size() + 1));
  const size_t o_mm1 = L.add(sizeof(int) * 2 * grp[1].size());
  const size_t o_mm5 = L.add(sizeof(int) * 2 * grp[5].size());
  const size_t o_upd = L.add(sizeof(IndexRec) * nm);
  const size_t o_era = L.add(sizeof(IndexRec) * nd);
  CB_TRY(h_mscratch.ensure(L.off), "pinned scratch");
  CB_TRY(d_mscratch.ensure(L.off), "device scratch");
  uint8_t *h = static_cast<uint8_t *>(h_mscratch.ptr);
  CopyDesc *desc = reinterpret_cast<CopyDesc *>(h + o_desc);
  IndexRec *upd = reinterpret_cast<IndexRec *>(h + o_upd);
  IndexRec *era = reinterpret_cast<IndexRec *>(h + o_era);
  uint32_t total[kGroups] = {};
  uint64_t grp_bytes[kGroups] = {};
  int base[kGroups] = {};
  bool dev_only[kGroups] = {true, true, true, true, true, true};  // no host-memory side in the group
  int di = 0;
  for (int g = 0; g < kGroups; ++g) {
    uint32_t *us = reinterpret_cast<uint32_t *>(h + o_us[g]);
    base[g] = di;
    for (size_t j = 0; j < grp[g].size(); ++j) {
      const TierMove &m = *grp[g][j];
      const uint64_t src = m.src_tier == kTierDram ? (uint64_t)dram_dev + m.src_off : (uint64_t)pool + m.src_off;
      const uint64_t dst = m.dst_tier == kTierDram ? (uint64_t)dram_dev + m.dst_off : (uint64_t)pool + m.dst_off;
      if (g == 5) {
        desc[di + j] = CopyDesc{src, (uint64_t)d_pack.ptr + pslot[j] + kPackLead, m.size, 0};
      } else if (m.src_dev) {
        desc[di + j] = CopyDesc{m.src_dev, dst, m.size, 0};  // device -> HBM, already unpacked
      } else {
        desc[di + j] = CopyDesc{src, dst, m.size, kCopyHost | (m.op == kMoveUnpack ? kCopyUnpack : 0)};
        dev_only[g] = false;
      }
      us[j] = total[g];
      total[g] += units_of(m.size);
      grp_bytes[g] += m.size;
      const BlockMeta *bm = policy.find(m.key);
      const bool packed = m.op == kMovePack;
      upd[di + j] = IndexRec{m.key.lo, m.key.hi, m.dst_off | (m.dst_tier == kTierDram ? kLocDram : 0),
                             meta_word(packed ? (m.size & ~1ull) : m.size, bm ? bm->prefix : 0) |
                                 (packed ? kMetaPacked : 0)};
    }
    us[grp[g].size()] = total[g];
    di += (int)grp[g].size();
  }
  // (an empty group's region has the next one's offset: pair each with its count)
  for (const auto &oc : {std::make_pair(o_mm1, grp[1].size()), std::make_pair(o_mm5, grp[5].size())}) {
    int *mm = reinterpret_cast<int *>(h + oc.first);
    for (size_t j = 0; j < oc.second; ++j) {
      mm[2 * j] = INT_MAX;
      mm[2 * j + 1] = INT_MIN;
    }
  }
  for (int j = 0; j < nd; ++j) era[j] = IndexRec{dropped[j].lo, dropped[j].hi, 0, 0};
  uint8_t *d = static_cast<uint8_t *>(d_mscratch.ptr);
  CB_TRY(cudaMemcpyAsync(d, h, L.off, cudaMemcpyHostToDevice, st), "H2D moves");
  const CopyDesc *ddesc = reinterpret_cast<const CopyDesc *>(d + o_desc);
  // Demotions: on st, or on move_stream beside the caller's concurrent work.
  cudaStream_t ds = st;
  if (concurrent) {
    CB_TRY(cudaEventRecord(ev_move_in, st), "event");
    CB_TRY(cudaStreamWaitEvent(move_stream, ev_move_in, 0), "wait");
    ds = move_stream;
  }
  // Host-link-bound demotions beside a gather take 2 CTAs per SM, so that
  // the gather's CTAs fit next to them instead of waiting for them to drain.
  const int move_ctas = concurrent ? 2 : 8;
  auto launch_group = [&](int g, cudaStream_t gs) -> int {
    if (grp[g].empty()) return CB_OK;
    const CopyDesc *gd = ddesc + base[g];
    const uint32_t *gu = reinterpret_cast<const uint32_t *>(d + o_us[g]);
    const int gn = (int)grp[g].size();
    if (g == 1 || g == 5) {
      // group 5: the timed span covers the packing and the D2H copies of the
      // packed images to the arena, i.e. the whole move
      CB_TRY(timed(3, grp_bytes[g], gs,
                   [&] {
                     cudaError_t e = launch_kv_pack(gd, gu, gn, total[g],
                                                    reinterpret_cast<int *>(d + (g == 1 ? o_mm1 : o_mm5)), num_sms,
                                                    gs, g == 5 ? 8 : move_ctas);
                     for (size_t j = 0; g == 5 && e == cudaSuccess && j < grp[5].size(); ++j) {
                       const TierMove &m = *grp[5][j];
                       e = cudaMemcpyAsync(dram_host + m.dst_off,
                                           static_cast<uint8_t *>(d_pack.ptr) + pslot[j] + kPackLead,
                                           packed_bytes(m.size), cudaMemcpyDeviceToHost, gs);
                     }
                     return e;
                   }),
             "demote pack");
      launches++;  // two kernels
    } else {
      // host-link moves on the LSU engine; device-only groups on the store's
      const int engine = dev_only[g] ? copy_engine : 2;
      CB_TRY(timed(3, grp_bytes[g], gs,
                   [&] {
                     return launch_batch_copy(gd, gu, gn, total[g], engine, d_err, num_sms, gs,
                                              g == 2 ? 8 : move_ctas);
                   }),
             g ? "promote copy" : "demote copy");
    }
    return CB_OK;
  };
  // DMA groups: one cudaMemcpyAsync per run of moves contiguous on both
  // sides, bracketed by profiling events like a kernel (not counted as one).
  auto dma_group = [&](int g, cudaStream_t gs) -> int {
    if (grp[g].empty()) return CB_OK;
    const bool down = g == 3;
    cudaEvent_t a = nullptr, b = nullptr;
    if (profile) {
      CB_TRY(prof_event(a), "event");
      CB_TRY(prof_event(b), "event");
      CB_TRY(cudaEventRecord(a, gs), "event");
    }
    const auto &v = grp[g];
    size_t j = 0;
    while (j < v.size()) {
      uint64_t run = v[j]->size;
      size_t e = j + 1;
      while (e < v.size() && v[e]->src_off == v[j]->src_off + run && v[e]->dst_off == v[j]->dst_off + run) {
        run += v[e]->size;
        ++e;
      }
      if (down) {
        CB_TRY(cudaMemcpyAsync(dram_host + v[j]->dst_off, pool + v[j]->src_off, run, cudaMemcpyDeviceToHost, gs),
               "demote DMA");
      } else {
        CB_TRY(cudaMemcpyAsync(pool + v[j]->dst_off, dram_host + v[j]->src_off, run, cudaMemcpyHostToDevice, gs),
               "promote DMA");
      }
      j = e;
    }
    if (profile) {
      CB_TRY(cudaEventRecord(b, gs), "event");
      prof_pending.push_back(ProfRec{3, grp_bytes[g], a, b});
    }
    return CB_OK;
  };
  int rc = launch_group(0, ds);
  if (rc == CB_OK) rc = dma_group(3, ds);
  if (rc == CB_OK) rc = launch_group(5, ds);
  if (rc == CB_OK) rc = launch_group(1, ds);
  if (concurrent) {
    // join: whatever happens, st waits for the demotions before going on
    const cudaError_t e = cudaEventRecord(ev_move_done, move_stream);
    if (rc == CB_OK && e == cudaSuccess) rc = concurrent();
    if (e == cudaSuccess) cudaStreamWaitEvent(st, ev_move_done, 0);
    if (e != cudaSuccess) {
      cudaStreamSynchronize(move_stream);
      return cuda_fail(e, "event");
    }
  }
  if (rc) {
    cudaStreamSynchronize(move_stream);
    cudaStreamSynchronize(st);
    return rc;
  }
  rc = launch_group(2, st);
  if (rc == CB_OK) rc = dma_group(4, st);
  if (rc) {
    cudaStreamSynchronize(st);
    return rc;
  }
  if (nm) {
    CB_TRY(launch_index_update(table, table_slots - 1, reinterpret_cast<const IndexRec *>(d + o_upd), nm,
                               d_err, st),
           "index update");
    launches++;
  }
  if (nd) {
    CB_TRY(launch_index_erase(table, table_slots - 1, reinterpret_cast<const IndexRec *>(d + o_era), nd,
                              d_err, st),
           "index erase");
    launches++;
  }
  table_tombs += nd;
  table_used -= std::min<uint64_t>(table_used, nd);
  // The scratch buffers are reused by the next plan: wait for the copies
  // of this plan's descriptors to be consumed.
  CB_TRY(cudaStreamSynchronize(st), "moves");
  resolve_prof();
  return CB_OK;
}

// SHA-256 of device-resident blocks; digests (n*32 B) land in h_out.
int Store::hash_device(const uint64_t *ptrs, const uint64_t *sizes, int n, cudaStream_t st,
                       const HashProgress *pg, cudaEvent_t copies_done) {
  Trace tr("cb.sha256");
  Layout L;
  const size_t o_jobs = L.add(sizeof(HashJob) * n);
  const size_t o_dig = L.add(32ull * n);
  CB_TRY(h_scratch.ensure(L.off), "pinned scratch");
  CB_TRY(d_scratch.ensure(L.off), "device scratch");
  CB_TRY(h_out.ensure(32ull * n), "pinned out");
  HashJob *jobs = reinterpret_cast<HashJob *>(static_cast<uint8_t *>(h_scratch.ptr) + o_jobs);
  uint64_t total = 0;
  for (int i = 0; i < n; ++i) {
    jobs[i] = HashJob{ptrs[i], sizes[i]};
    total += sizes[i];
  }
  uint8_t *d = static_cast<uint8_t *>(d_scratch.ptr);
  CB_TRY(cudaMemcpyAsync(d + o_jobs, jobs, sizeof(HashJob) * n, cudaMemcpyHostToDevice, st), "H2D jobs");
  CB_TRY(timed(0, total, st,
               [&] {
                 return launch_sha256_batch(reinterpret_cast<const HashJob *>(d + o_jobs), n,
                                            reinterpret_cast<uint32_t *>(d + o_dig), hash_lanes, d_err, st, pg);
               }),
         "sha256 launch");
  // everything after the hash on st (scatter) also needs every copy done
  if (copies_done) CB_TRY(cudaStreamWaitEvent(st, copies_done, 0), "wait copies");
  CB_TRY(cudaMemcpyAsync(h_out.ptr, d + o_dig, 32ull * n, cudaMemcpyDeviceToHost, st), "D2H digests");
  return check_device_error(st);  // syncs; a timed-out hash is an error
}

// ---------------------------------------------------------------- put

// Scatter of a planned put into its tiers, stream-ordered on st: plain
// copies (HBM, or DRAM without packing), blocks packed to INT8 straight into
// the DRAM tier, then the index insert. Descriptors go through (hbuf, dbuf),
// which must stay untouched until the kernels have run.
int Store::enqueue_places(const PutPlan &plan, const uint64_t *ptrs, cudaStream_t st, PinnedBuf &hbuf,
                          DevBuf &dbuf, int engine, int lsu_ctas_per_sm) {
  const int np = (int)plan.places.size();
  if (!np) return CB_OK;
  {
    bool need_dram = false;
    for (const auto &p : plan.places) need_dram |= p.tier == kTierDram;
    if (need_dram) {
      cudaError_t e = ensure_dram();
      if (e != cudaSuccess) return cuda_fail(e, "pinned DRAM arena cudaHostAlloc");
    }
    // Two groups: blocks copied as they are (HBM, or DRAM without packing),
    // then blocks packed to INT8 straight into the DRAM tier.
    int npk = 0;
    for (const auto &p : plan.places) npk += p.packed ? 1 : 0;
    const int ncp = np - npk;
    Layout L;
    const size_t o_desc = L.add(sizeof(CopyDesc) * np);
    const size_t o_us = L.add(sizeof(uint32_t) * (ncp + 1));
    const size_t o_pus = L.add(sizeof(uint32_t) * (npk + 1));
    const size_t o_mm = L.add(sizeof(int) * 2 * npk);
    const size_t o_ins = L.add(sizeof(IndexRec) * np);
    CB_TRY(hbuf.ensure(L.off), "pinned scratch");
    CB_TRY(dbuf.ensure(L.off), "device scratch");
    uint8_t *h = static_cast<uint8_t *>(hbuf.ptr);
    CopyDesc *desc = reinterpret_cast<CopyDesc *>(h + o_desc);
    uint32_t *us = reinterpret_cast<uint32_t *>(h + o_us);
    uint32_t *pus = reinterpret_cast<uint32_t *>(h + o_pus);
    int *mm = reinterpret_cast<int *>(h + o_mm);
    IndexRec *ins = reinterpret_cast<IndexRec *>(h + o_ins);
    uint32_t total = 0, ptotal = 0;
    uint64_t bytes = 0, pbytes = 0;
    int jc = 0, jp = 0;
    for (int j = 0; j < np; ++j) {
      const Placement &p = plan.places[j];
      const bool dram = p.tier == kTierDram;
      const uint64_t dst = dram ? (uint64_t)dram_dev + p.off : (uint64_t)pool + p.off;
      const int slot = p.packed ? ncp + jp : jc;
      desc[slot] = CopyDesc{ptrs[p.idx], dst, p.size, dram ? kCopyHost : 0};
      if (p.packed) {
        pus[jp] = ptotal;
        ptotal += units_of(p.size);
        pbytes += p.size;
        mm[2 * jp] = INT_MAX;
        mm[2 * jp + 1] = INT_MIN;
        ++jp;
      } else {
        us[jc] = total;
        total += units_of(p.size);
        bytes += p.size;
        ++jc;
      }
      ins[j] = IndexRec{p.key.lo, p.key.hi, p.off | (dram ? kLocDram : 0),
                        meta_word(p.packed ? (p.size & ~1ull) : p.size, p.prefix) | (p.packed ? kMetaPacked : 0)};
    }
    us[ncp] = total;
    pus[npk] = ptotal;
    uint8_t *d = static_cast<uint8_t *>(dbuf.ptr);
    CB_TRY(cudaMemcpyAsync(d, h, L.off, cudaMemcpyHostToDevice, st), "H2D scatter");
    if (ncp) {
      CB_TRY(timed(1, bytes, st,
                   [&] {
                     return launch_batch_copy(reinterpret_cast<const CopyDesc *>(d + o_desc),
                                              reinterpret_cast<const uint32_t *>(d + o_us), ncp, total,
                                              engine, d_err, num_sms, st, lsu_ctas_per_sm);
                   }),
             "scatter");
    }
    if (npk) {
      CB_TRY(timed(1, pbytes, st,
                   [&] {
                     return launch_kv_pack(reinterpret_cast<const CopyDesc *>(d + o_desc) + ncp,
                                           reinterpret_cast<const uint32_t *>(d + o_pus), npk, ptotal,
                                           reinterpret_cast<int *>(d + o_mm), num_sms, st);
                   }),
             "scatter pack");
      launches++;  // two kernels
    }
    CB_TRY(launch_index_insert(table, table_slots - 1, reinterpret_cast<const IndexRec *>(d + o_ins), np,
                               d_err, st),
           "index insert");
    launches++;
    table_used += np;
  }
  return CB_OK;
}

int Store::put_device(const uint64_t *ptrs, const uint64_t *sizes, const uint8_t *is_prefix,
                      const uint8_t *keys_in, int n, uint8_t *keys_out, uint8_t *status_out,
                      cudaStream_t st, const HashProgress *pg, cudaEvent_t copies_done) {
  Trace tr("cb.put");
  std::vector<HKey> keys(n);
  if (keys_in) {
    if (copies_done) CB_TRY(cudaStreamWaitEvent(st, copies_done, 0), "wait copies");
    for (int i = 0; i < n; ++i) keys[i] = to_hkey(keys_in + 16 * i);
  } else {
    int rc = hash_device(ptrs, sizes, n, st, pg, copies_done);
    if (rc) return rc;
    const uint8_t *dig = static_cast<const uint8_t *>(h_out.ptr);
    for (int i = 0; i < n; ++i) keys[i] = to_hkey(dig + 32 * i);
  }
  int rc = reserve_index((uint64_t)n, st);
  if (rc) return rc;
  PutPlan &plan = put_plan;
  policy.plan_put(keys.data(), sizes, is_prefix, n, cfg.dedup_enabled != 0, plan);
  plan_open = true;
  rc = run_moves(plan.moves, plan.dropped, st);
  if (rc) return rc;

  rc = enqueue_places(plan, ptrs, st, h_scratch, d_scratch, copy_engine, 8);
  if (rc) return rc;
  rc = check_device_error(st);  // also the final sync of the batch
  policy.commit();
  if (rc) return rc;
  for (int i = 0; i < n; ++i) {
    if (keys_out) from_hkey(keys[i], keys_out + 16 * i);
    if (status_out) status_out[i] = plan.status[i];
  }
  return CB_OK;
}

// Host-memory blocks: copied into device staging in slices that fit it, each
// slice then takes the device path (sequential dedup is preserved because
// slices are processed in batch order).
int Store::put_host(const void *const *ptrs, const uint64_t *sizes, const uint8_t *is_prefix,
                    const uint8_t *keys_in, int n, uint8_t *keys_out, uint8_t *status_out,
                    cudaStream_t st) {
  const uint64_t cap = staging_capacity();
  int i = 0;
  std::vector<uint64_t> dptrs;
  while (i < n) {
    uint64_t bytes = 0;
    int j = i;
    while (j < n && (j == i || bytes + align_up(sizes[j], 256) <= cap)) bytes += align_up(sizes[j++], 256);
    CB_TRY(d_staging.ensure(bytes), "device staging");
    dptrs.resize(j - i);
    HashProgress pg;
    if (!keys_in && stage_overlapped(ptrs + i, sizes + i, j - i, dptrs.data(), pg, st) == CB_OK) {
      // Copies run on copy_stream; the hash reads each segment as it lands.
      int rc = put_device(dptrs.data(), sizes + i, is_prefix ? is_prefix + i : nullptr, nullptr, j - i,
                          keys_out ? keys_out + 16 * i : nullptr, status_out ? status_out + i : nullptr, st, &pg,
                          ev_copies);
      CB_TRY(cudaStreamSynchronize(copy_stream), "copy stream");
      if (rc) return rc;
      i = j;
      continue;
    }
    uint64_t off = 0;
    for (int k = i; k < j; ++k) {
      dptrs[k - i] = (uint64_t)d_staging.ptr + off;
      off += align_up(sizes[k], 256);
    }
    // Coalesce host-contiguous runs into single DMA copies.
    int k = i;
    while (k < j) {
      int e = k + 1;
      uint64_t run = sizes[k];
      const AddrRange rg = e < j ? alloc_range(ptrs[k]) : AddrRange{0, 0};
      while (e < j && static_cast<const uint8_t *>(ptrs[k]) + (dptrs[e - i] - dptrs[k - i]) == ptrs[e] &&
             dptrs[e - i] - dptrs[e - 1 - i] == sizes[e - 1] &&
             rg.holds(ptrs[k], dptrs[e - i] - dptrs[k - i] + sizes[e])) {
        run = dptrs[e - i] - dptrs[k - i] + sizes[e];
        ++e;
      }
      if (run) CB_TRY(cudaMemcpyAsync(reinterpret_cast<void *>(dptrs[k - i]), ptrs[k], run,
                                      cudaMemcpyHostToDevice, st),
                      "H2D block");
      k = e;
    }
    int rc = put_device(dptrs.data(), sizes + i, is_prefix ? is_prefix + i : nullptr,
                        keys_in ? keys_in + 16 * i : nullptr, j - i, keys_out ? keys_out + 16 * i : nullptr,
                        status_out ? status_out + i : nullptr, st);
    if (rc) return rc;
    i = j;
  }
  return CB_OK;
}

// Overlapped staging for host puts of equal-size blocks at a constant host
// stride (KV pages in one pinned buffer): the batch is copied segment-major
// (segment k = bytes [k*seg, (k+1)*seg) of every block) with one strided
// copy per segment on copy_stream, each followed by a 4-byte copy that
// publishes k+1 to d_progress. The SHA-256 kernel (which consumes every
// chain front to back at the same pace) reads a segment once it is
// published, so the host link and the hash overlap. Returns CB_ERR_ARG when
// the batch does not have that shape (the caller then copies plainly).
int Store::stage_overlapped(const void *const *ptrs, const uint64_t *sizes, int n, uint64_t *dptrs,
                            HashProgress &pg, cudaStream_t st) {
  constexpr uint64_t kSeg = 64 * 1024;
  if (n < 32) return CB_ERR_ARG;
  const uint64_t size = sizes[0];
  if (size < 4 * kSeg) return CB_ERR_ARG;
  const int64_t stride = static_cast<const uint8_t *>(ptrs[1]) - static_cast<const uint8_t *>(ptrs[0]);
  if (stride < (int64_t)size) return CB_ERR_ARG;
  for (int i = 1; i < n; ++i) {
    if (sizes[i] != size) return CB_ERR_ARG;
    if (static_cast<const uint8_t *>(ptrs[i]) - static_cast<const uint8_t *>(ptrs[i - 1]) != stride) return CB_ERR_ARG;
  }
  // the strided copies read the caller's blocks as one buffer
  if (!one_allocation(ptrs[0], (uint64_t)stride * (n - 1) + size)) return CB_ERR_ARG;
  const uint64_t slot = align_up(size, 256);
  for (int i = 0; i < n; ++i) dptrs[i] = (uint64_t)d_staging.ptr + slot * i;
  const uint32_t nseg = (uint32_t)((size + kSeg - 1) / kSeg);
  CB_TRY(h_progress.ensure(4ull * (nseg + 1)), "pinned progress");
  unsigned *vals = static_cast<unsigned *>(h_progress.ptr);
  for (uint32_t k = 0; k <= nseg; ++k) vals[k] = k;
  // The staging area may still be read by earlier work on st.
  CB_TRY(cudaEventRecord(ev_reset, st), "event");
  CB_TRY(cudaStreamWaitEvent(copy_stream, ev_reset, 0), "wait");
  CB_TRY(cudaMemcpyAsync(d_progress, &vals[0], 4, cudaMemcpyHostToDevice, copy_stream), "progress reset");
  CB_TRY(cudaEventRecord(ev_reset, copy_stream), "event");
  for (uint32_t k = 0; k < nseg; ++k) {
    const uint64_t off = (uint64_t)k * kSeg;
    const uint64_t w = std::min(kSeg, size - off);
    CB_TRY(cudaMemcpy2DAsync(reinterpret_cast<void *>(dptrs[0] + off), slot,
                             static_cast<const uint8_t *>(ptrs[0]) + off, (size_t)stride, w, n,
                             cudaMemcpyHostToDevice, copy_stream),
           "H2D segment");
    CB_TRY(cudaMemcpyAsync(d_progress, &vals[k + 1], 4, cudaMemcpyHostToDevice, copy_stream), "progress");
  }
  CB_TRY(cudaEventRecord(ev_copies, copy_stream), "event");
  // the hash must see the reset counter, not a stale one
  CB_TRY(cudaStreamWaitEvent(st, ev_reset, 0), "wait reset");
  pg = HashProgress{d_progress, (uint32_t)(kSeg / 64), (size + 63) / 64};
  return CB_OK;
}

// ---------------------------------------------------------------- get

int Store::get_device(const uint8_t *keys, int n, const uint64_t *outs, const uint64_t *caps,
                      uint64_t *sizes_out, uint8_t *found_out, cudaStream_t st) {
  Trace tr("cb.get");
  Layout L;
  const size_t o_keys = L.add(16ull * n);
  const size_t o_outs = L.add(8ull * n);
  const size_t o_caps = L.add(8ull * n);
  const size_t o_us = L.add(4ull * (n + 1));
  const size_t o_desc = L.add(sizeof(CopyDesc) * n);
  const size_t o_res = L.add(sizeof(GetResult) * n);
  const size_t o_udesc = L.add(sizeof(CopyDesc) * n);  // unpacks of DMA'd packed hits
  const size_t o_uus = L.add(4ull * (n + 1));
  CB_TRY(h_scratch.ensure(L.off), "pinned scratch");
  CB_TRY(d_scratch.ensure(L.off), "device scratch");
  CB_TRY(h_out.ensure(sizeof(GetResult) * n), "pinned out");
  uint8_t *h = static_cast<uint8_t *>(h_scratch.ptr);
  memcpy(h + o_keys, keys, 16ull * n);
  memcpy(h + o_outs, outs, 8ull * n);
  // DRAM hits of large plain blocks are copied by the H2D copy engine from
  // the location the host metadata holds (the engines move each direction at
  // the link rate, and beside the demotions' D2H DMA): the lookup kernel gets
  // a capacity of 0 for them, so it reports them without copying.
  // Large INT8-packed DRAM hits: their packed bytes come in by DMA to an HBM
  // staging area and are unpacked there into the caller's buffers.
  uint64_t *dcaps = reinterpret_cast<uint64_t *>(h + o_caps);
  std::vector<int> dma_req;
  std::vector<uint64_t> pk_slot;  // staging offset per dma_req entry (packed hits)
  uint32_t *us = reinterpret_cast<uint32_t *>(h + o_us);
  CopyDesc *udesc = reinterpret_cast<CopyDesc *>(h + o_udesc);
  uint32_t *uus = reinterpret_cast<uint32_t *>(h + o_uus);
  uint32_t total = 0, utotal = 0;
  int nu = 0;
  uint64_t bytes = 0, dma_bytes = 0, ustage = 0;
  for (int i = 0; i < n; ++i) {
    us[i] = total;
    dcaps[i] = caps[i];
    const BlockMeta *m = policy.find(to_hkey(keys + 16 * i));
    if (!m || m->size > caps[i]) continue;
    if (m->tier == kTierDram && m->size >= kDmaMinBytes) {
      const uint64_t slot = m->packed ? align_up(kPackLead + packed_bytes(m->size), 256) : 0;
      if (!m->packed || ustage + slot <= kPackStagingBytes) {
        dma_req.push_back(i);
        pk_slot.push_back(m->packed ? ustage : UINT64_MAX);
        ustage += slot;
        dma_bytes += m->packed ? packed_bytes(m->size) : m->size;
        dcaps[i] = 0;
        continue;
      }
    }
    total += units_of(m->size);
    bytes += m->size;
  }
  us[n] = total;
  if (ustage) CB_TRY(d_unpack.ensure(ustage), "unpacking staging");  // before any concurrent work
  std::vector<std::pair<uint64_t, uint64_t>> dma_src(dma_req.size());  // (arena offset, size)
  for (size_t j = 0; j < dma_req.size(); ++j) {
    const BlockMeta *m = policy.find(to_hkey(keys + 16 * dma_req[j]));
    dma_src[j] = {Policy::data_offset(*m), m->size};
    if (pk_slot[j] != UINT64_MAX) {
      uus[nu] = utotal;
      udesc[nu++] = CopyDesc{(uint64_t)d_unpack.ptr + pk_slot[j] + kPackLead, outs[dma_req[j]], m->size, kCopyUnpack};
      utotal += units_of(m->size);
    }
  }
  uus[nu] = utotal;
  // LRU touches first (CascadeStore::get touches on hit,
  // src/cascade_core.cpp:1281), so that blocks of this batch are the last
  // victims of the promotions below.
  for (int i = 0; i < n; ++i) policy.touch(to_hkey(keys + 16 * i));
  // Promotion on a DRAM hit. CB_PROMOTE_EVERY_HIT is CascadeStore's rule
  // (CascadeStore::get -> promote_to_gpu, src/cascade_core.cpp:1303-1307,
  // :1166-1185). CB_PROMOTE_LOCALITY is DistributedStore::get's
  // (src/distributed_backend.cpp:721-724): promote_to_local_gpu only when
  // locality_aware and should_promote_local (:1257-1265), i.e. after
  // >= promotion_threshold accesses with an EMA remote-access rate > 0.5.
  // Every access a store makes to its own DRAM tier is a local one, so the
  // EMA stays 0 and the rule never fires: such stores do not promote.
  // The host metadata already knows which requests are DRAM hits that will
  // be copied, so the promotions are planned before the lookup: the
  // demotions that make room for them (HBM -> DRAM, the device-to-host
  // direction of the host link) run on move_stream while the gather reads
  // the DRAM hits (host-to-device); the promotions then read the copy the
  // gather made in the caller's buffer (or the staging slot of a host get),
  // already unpacked, like the reference, instead of reading DRAM again.
  std::vector<TierMove> moves;
  std::vector<HKey> dropped;
  bool planned = false;
  const bool promote = cfg.promote_on_hit && cfg.promotion_rule == CB_PROMOTE_EVERY_HIT;
  if (promote && policy.dram_used() > 0) {
    std::unordered_map<HKey, uint64_t, HKeyHash> copy_of;
    std::vector<HKey> order;
    for (int i = 0; i < n; ++i) {
      const HKey k = to_hkey(keys + 16 * i);
      const BlockMeta *m = policy.find(k);
      if (m && m->tier == kTierDram && m->size && m->size <= caps[i] && copy_of.emplace(k, outs[i]).second)
        order.push_back(k);
    }
    // every DRAM block this get reads stays put (and its extent unused)
    // until the batch ends, whatever the plans for the others evict
    for (const HKey &k : order) policy.protect(k);
    for (const HKey &k : order) policy.plan_promote(k, moves, dropped);
    for (TierMove &mv : moves) {
      if (mv.src_tier != kTierDram || mv.dst_tier != kTierHbm) continue;
      auto it = copy_of.find(mv.key);
      if (it != copy_of.end()) mv.src_dev = it->second;
    }
    planned = !order.empty();
    plan_open |= planned;
  }
  uint8_t *d = static_cast<uint8_t *>(d_scratch.ptr);
  auto lookup_and_gather = [&]() -> int {
    if (!dma_req.empty()) {  // runs contiguous in the arena and in the caller's memory: one copy
      cudaEvent_t a = nullptr, b = nullptr;
      if (profile) {
        CB_TRY(prof_event(a), "event");
        CB_TRY(prof_event(b), "event");
        CB_TRY(cudaEventRecord(a, st), "event");
      }
      size_t j = 0;
      while (j < dma_req.size()) {
        if (pk_slot[j] != UINT64_MAX) {  // packed: its packed image into the staging area
          CB_TRY(cudaMemcpyAsync(static_cast<uint8_t *>(d_unpack.ptr) + pk_slot[j] + kPackLead,
                                 dram_host + dma_src[j].first, packed_bytes(dma_src[j].second), cudaMemcpyHostToDevice,
                                 st),
                 "packed DRAM hit DMA");
          ++j;
          continue;
        }
        uint64_t run = dma_src[j].second;
        size_t e = j + 1;
        const void *o0 = reinterpret_cast<const void *>(outs[dma_req[j]]);
        const AddrRange rg = e < dma_req.size() ? alloc_range(o0) : AddrRange{0, 0};
        while (e < dma_req.size() && pk_slot[e] == UINT64_MAX && dma_src[e].first == dma_src[j].first + run &&
               outs[dma_req[e]] == outs[dma_req[j]] + run && rg.holds(o0, run + dma_src[e].second)) {
          run += dma_src[e].second;
          ++e;
        }
        CB_TRY(cudaMemcpyAsync(reinterpret_cast<void *>(outs[dma_req[j]]), dram_host + dma_src[j].first, run,
                               cudaMemcpyHostToDevice, st),
               "DRAM hit DMA");
        j = e;
      }
      if (profile) {
        CB_TRY(cudaEventRecord(b, st), "event");
        prof_pending.push_back(ProfRec{2, dma_bytes, a, b});
      }
    }
    CB_TRY(cudaMemcpyAsync(d, h, L.off, cudaMemcpyHostToDevice, st), "H2D get");
    if (nu) {  // the DMA'd packed images, unpacked device to device
      CB_TRY(timed(2, 0, st,
                   [&] {
                     return launch_batch_copy(reinterpret_cast<const CopyDesc *>(d + o_udesc),
                                              reinterpret_cast<const uint32_t *>(d + o_uus), nu, utotal, 2, d_err,
                                              num_sms, st);
                   }),
             "unpack");
    }
    LookupArgs a;
    a.table = table;
    a.mask = table_slots - 1;
    a.keys = reinterpret_cast<const Key *>(d + o_keys);
    a.outs = reinterpret_cast<const uint64_t *>(d + o_outs);
    a.caps = reinterpret_cast<const uint64_t *>(d + o_caps);
    a.unit_start = reinterpret_cast<const uint32_t *>(d + o_us);
    a.n = n;
    a.pool_base = (uint64_t)pool;
    a.pool_bytes = pool_bytes;
    a.dram_base = (uint64_t)dram_dev;
    a.dram_bytes = dram_host ? dram_bytes : 0;
    a.code_hbm = CB_FOUND_LOCAL_HBM;
    a.code_dram = CB_FOUND_LOCAL_DRAM;
    a.desc = reinterpret_cast<CopyDesc *>(d + o_desc);
    a.res = reinterpret_cast<GetResult *>(d + o_res);
    a.err = d_err;
    CB_TRY(launch_index_lookup(a, st), "index lookup");
    launches++;
    if (total) {
      CB_TRY(timed(2, bytes, st,
                   [&] { return launch_batch_copy(a.desc, a.unit_start, n, total, copy_engine, d_err, num_sms, st); }),
             "gather");
    }
    CB_TRY(cudaMemcpyAsync(h_out.ptr, d + o_res, sizeof(GetResult) * n, cudaMemcpyDeviceToHost, st),
           "D2H results");
    return CB_OK;
  };
  int rc = run_moves(moves, dropped, st, lookup_and_gather);
  if (planned) policy.commit();
  if (rc) return rc;
  rc = check_device_error(st);
  if (rc) return rc;
  GetResult *res = static_cast<GetResult *>(h_out.ptr);
  for (size_t j = 0; j < dma_req.size(); ++j) {
    // copied by the DMA above; the lookup saw capacity 0
    const int i = dma_req[j];
    if ((res[i].code & 0x0f) != CB_FOUND_LOCAL_DRAM || res[i].size != dma_src[j].second)
      return fail(CB_ERR_STATE, "device index disagrees with the host metadata for request %d", i);
    res[i].code = CB_FOUND_LOCAL_DRAM;
  }
  for (int i = 0; i < n; ++i) {
    sizes_out[i] = res[i].size;
    found_out[i] = (uint8_t)res[i].code;
    const uint32_t tier = res[i].code & 0x0f;
    if (tier == CB_FOUND_MISS) {
      misses++;
    } else if (tier == CB_FOUND_LOCAL_HBM) {
      local_gpu_hits++;
    } else if (tier == CB_FOUND_LOCAL_DRAM) {
      local_dram_hits++;
    }
  }
  return CB_OK;
}

int Store::get_host(const uint8_t *keys, int n, void *const *outs, const uint64_t *caps,
                    uint64_t *sizes_out, uint8_t *found_out, cudaStream_t st) {
  const uint64_t cap = staging_capacity();
  std::vector<uint64_t> dptrs, dcaps;
  int i = 0;
  while (i < n) {
    uint64_t bytes = 0;
    int j = i;
    while (j < n) {
      const BlockMeta *m = policy.find(to_hkey(keys + 16 * j));
      const uint64_t need = (m && m->size <= caps[j]) ? align_up(m->size, 256) : 0;
      if (j > i && bytes + need > cap) break;
      bytes += need;
      ++j;
    }
    CB_TRY(d_staging.ensure(std::max<uint64_t>(bytes, 256)), "device staging");
    dptrs.resize(j - i);
    dcaps.resize(j - i);
    uint64_t off = 0;
    for (int k = i; k < j; ++k) {
      const BlockMeta *m = policy.find(to_hkey(keys + 16 * k));
      const uint64_t need = (m && m->size <= caps[k]) ? m->size : 0;
      dptrs[k - i] = (uint64_t)d_staging.ptr + off;
      dcaps[k - i] = m ? (m->size <= caps[k] ? m->size : 0) : 0;
      off += align_up(need, 256);
    }
    int rc = get_device(keys + 16 * i, j - i, dptrs.data(), dcaps.data(), sizes_out + i, found_out + i, st);
    if (rc) return rc;
    // Report "not copied" against the caller's real capacity, then DMA the
    // found blocks out, coalescing runs that are contiguous on both sides.
    int k = i;
    while (k < j) {
      const bool ok = (found_out[k] & 0x0f) != CB_FOUND_MISS && sizes_out[k] <= caps[k];
      if ((found_out[k] & 0x0f) != CB_FOUND_MISS && sizes_out[k] > caps[k]) {
        found_out[k] = (uint8_t)((found_out[k] & 0x0f) | CB_FOUND_NOT_COPIED);
      } else if ((found_out[k] & 0x0f) != CB_FOUND_MISS) {
        found_out[k] &= 0x0f;
      }
      if (!ok) {
        ++k;
        continue;
      }
      int e = k + 1;
      uint64_t run = sizes_out[k];
      const AddrRange rg = e < j ? alloc_range(outs[k]) : AddrRange{0, 0};
      while (e < j && (found_out[e] & 0x0f) != CB_FOUND_MISS && sizes_out[e] <= caps[e] &&
             static_cast<uint8_t *>(outs[k]) + (dptrs[e - i] - dptrs[k - i]) == outs[e] &&
             dptrs[e - i] - dptrs[e - 1 - i] == sizes_out[e - 1] &&
             rg.holds(outs[k], dptrs[e - i] - dptrs[k - i] + sizes_out[e])) {
        run = dptrs[e - i] - dptrs[k - i] + sizes_out[e];
        ++e;
      }
      if (run) CB_TRY(cudaMemcpyAsync(outs[k], reinterpret_cast<void *>(dptrs[k - i]), run,
                                      cudaMemcpyDeviceToHost, st),
                      "D2H block");
      k = e;
    }
    CB_TRY(cudaStreamSynchronize(st), "D2H blocks");
    i = j;
  }
  return CB_OK;
}

// ---------------------------------------------------------------- misc

// Failure-path self-test (cb_selftest): one 1 MiB hash whose input is
// announced as still arriving (progress word 0, never published). The
// producer warp's poll gives up after 4096 tries (~1 ms), raises
// kErrTimeout and sets the ring's abort word; the consumer warp sees it and
// leaves; the host reads the error word and reports CB_ERR_TIMEOUT. Nothing
// faults or hangs and the context stays usable.
int Store::selftest(int which, cudaStream_t st) {
  if (which == CB_SELFTEST_FAIL_MOVES) {
    fake_move_failures = 1;
    return CB_OK;
  }
  if (which == CB_SELFTEST_GET_ERROR) {
    inject_get_error = true;
    return CB_OK;
  }
  if (which != CB_SELFTEST_HASH_WAIT) return fail(CB_ERR_ARG, "unknown self-test %d", which);
  constexpr uint64_t kBytes = 1 << 20;
  CB_TRY(cudaStreamSynchronize(copy_stream), "copy stream");
  CB_TRY(d_staging.ensure(kBytes), "device staging");
  CB_TRY(cudaMemsetAsync(d_staging.ptr, 0, kBytes, st), "staging");
  CB_TRY(cudaMemsetAsync(d_progress, 0, 4, st), "progress");
  HashProgress pg{d_progress, 1024, kBytes / 64, 4096};
  const uint64_t ptr = (uint64_t)d_staging.ptr, size = kBytes;
  return hash_device(&ptr, &size, 1, st, &pg);
}

// Zero-copy get: the caller reads the blocks where they sit in the HBM pool
// (a torch view, an attention kernel reading KV pages in place) instead of
// receiving copies — the caller-side step after batch_get
// (DistributedStore::get_batch, src/distributed_backend.cpp:844-870) without
// its copy. HBM hits are resolved from the host metadata alone: no kernel, no
// device round trip. DRAM-tier hits are promoted first (with promote_on_hit;
// packed blocks are unpacked by the promotion) and then viewed. Each viewed
// block is pinned — never a victim, so neither moved nor dropped — until
// release_views drops the pin (one release per view).
int Store::get_views(const uint8_t *keys, int n, uint64_t *addrs_out, uint64_t *sizes_out, uint8_t *found_out,
                     cudaStream_t st) {
  std::vector<TierMove> moves;
  std::vector<HKey> dropped;
  bool planned = false;
  for (int i = 0; i < n; ++i) {
    const HKey k = to_hkey(keys + 16 * i);
    policy.touch(k);
    const BlockMeta *m = policy.find(k);
    if (m && m->tier == kTierDram && cfg.promote_on_hit) {
      policy.plan_promote(k, moves, dropped);
      planned = true;
    }
  }
  plan_open |= planned;
  int rc = run_moves(moves, dropped, st);
  if (planned) policy.commit();
  if (rc) return rc;
  rc = check_device_error(st);
  if (rc) return rc;
  for (int i = 0; i < n; ++i) {
    const HKey k = to_hkey(keys + 16 * i);
    const BlockMeta *m = policy.find(k);
    addrs_out[i] = 0;
    sizes_out[i] = m ? m->size : 0;
    if (!m) {
      found_out[i] = CB_FOUND_MISS;
      misses++;
    } else if (m->tier == kTierDram) {  // promotion off, or no HBM room
      found_out[i] = CB_FOUND_LOCAL_DRAM | CB_FOUND_NOT_COPIED;
      local_dram_hits++;
    } else {
      found_out[i] = CB_FOUND_LOCAL_HBM;
      addrs_out[i] = (uint64_t)pool + m->off;
      policy.pin(k);
      local_gpu_hits++;
    }
  }
  return CB_OK;
}

int Store::release_views(const uint8_t *keys, int n) {
  int bad = 0;
  for (int i = 0; i < n; ++i) bad += policy.unpin(to_hkey(keys + 16 * i)) ? 0 : 1;
  if (bad) return fail(CB_ERR_ARG, "%d key(s) had no outstanding view", bad);
  return CB_OK;
}

// KVCompressor::compress (src/cascade_core.cpp:908-944) of n device blocks:
// the pack kernels of the DRAM tier on caller buffers.
int Store::kv_compress(const uint64_t *srcs, const uint64_t *sizes, const uint64_t *dsts, int n, cudaStream_t st) {
  Layout L;
  const size_t o_desc = L.add(sizeof(CopyDesc) * n);
  const size_t o_us = L.add(sizeof(uint32_t) * (n + 1));
  const size_t o_mm = L.add(sizeof(int) * 2 * n);
  CB_TRY(h_scratch.ensure(L.off), "pinned scratch");
  CB_TRY(d_scratch.ensure(L.off), "device scratch");
  uint8_t *h = static_cast<uint8_t *>(h_scratch.ptr);
  CopyDesc *desc = reinterpret_cast<CopyDesc *>(h + o_desc);
  uint32_t *us = reinterpret_cast<uint32_t *>(h + o_us);
  int *mm = reinterpret_cast<int *>(h + o_mm);
  uint32_t total = 0;
  uint64_t bytes = 0;
  for (int i = 0; i < n; ++i) {
    if (sizes[i] < 2) return fail(CB_ERR_ARG, "block %d: compression needs at least one 16-bit value", i);
    desc[i] = CopyDesc{srcs[i], dsts[i], sizes[i], 0};
    us[i] = total;
    total += units_of(sizes[i]);
    bytes += sizes[i];
    mm[2 * i] = INT_MAX;
    mm[2 * i + 1] = INT_MIN;
  }
  us[n] = total;
  uint8_t *d = static_cast<uint8_t *>(d_scratch.ptr);
  CB_TRY(cudaMemcpyAsync(d, h, L.off, cudaMemcpyHostToDevice, st), "H2D pack");
  CB_TRY(timed(3, bytes, st,
               [&] {
                 return launch_kv_pack(reinterpret_cast<const CopyDesc *>(d + o_desc),
                                       reinterpret_cast<const uint32_t *>(d + o_us), n, total,
                                       reinterpret_cast<int *>(d + o_mm), num_sms, st);
               }),
         "pack");
  launches++;  // two kernels
  return check_device_error(st);
}

// KVCompressor::decompress (src/cascade_core.cpp:946-967) of n device
// blocks; ok_out[i] = 0 (nothing written) when block i is shorter than
// 8 + orig_sizes[i]/2 bytes, the reference's `return false`.
int Store::kv_decompress(const uint64_t *srcs, const uint64_t *comp_sizes, const uint64_t *orig_sizes,
                         const uint64_t *dsts, int n, uint8_t *ok_out, cudaStream_t st) {
  Layout L;
  const size_t o_desc = L.add(sizeof(CopyDesc) * n);
  const size_t o_us = L.add(sizeof(uint32_t) * (n + 1));
  CB_TRY(h_scratch.ensure(L.off), "pinned scratch");
  CB_TRY(d_scratch.ensure(L.off), "device scratch");
  uint8_t *h = static_cast<uint8_t *>(h_scratch.ptr);
  CopyDesc *desc = reinterpret_cast<CopyDesc *>(h + o_desc);
  uint32_t *us = reinterpret_cast<uint32_t *>(h + o_us);
  uint32_t total = 0;
  uint64_t bytes = 0;
  for (int i = 0; i < n; ++i) {
    const bool ok = comp_sizes[i] >= packed_bytes(orig_sizes[i]);
    if (ok_out) ok_out[i] = ok ? 1 : 0;
    const uint64_t out = ok ? orig_sizes[i] / 2 * 2 : 0;
    desc[i] = CopyDesc{srcs[i], dsts[i], out, kCopyHost | kCopyUnpack};
    us[i] = total;
    total += units_of(out);
    bytes += out;
  }
  us[n] = total;
  if (total == 0) return CB_OK;
  uint8_t *d = static_cast<uint8_t *>(d_scratch.ptr);
  CB_TRY(cudaMemcpyAsync(d, h, L.off, cudaMemcpyHostToDevice, st), "H2D unpack");
  CB_TRY(timed(3, bytes, st,
               [&] {
                 return launch_batch_copy(reinterpret_cast<const CopyDesc *>(d + o_desc),
                                          reinterpret_cast<const uint32_t *>(d + o_us), n, total, 2, d_err,
                                          num_sms, st);
               }),
         "unpack");
  return check_device_error(st);
}

int Store::evict(uint64_t bytes, uint64_t *evicted, cudaStream_t st) {
  std::vector<TierMove> moves;
  std::vector<HKey> dropped;
  const uint64_t freed = policy.plan_evict(bytes, moves, dropped);
  plan_flag() |= !moves.empty() || !dropped.empty();
  int rc = run_moves(moves, dropped, st);
  policy.commit();
  if (rc) return rc;
  rc = check_device_error(st);
  if (evicted) *evicted = freed;
  return rc;
}

int Store::clear(cudaStream_t st) {
  if (policy.pinned_blocks())  // a view would point at memory the store hands out again
    return fail(CB_ERR_STATE, "%llu block(s) have outstanding zero-copy views",
                (unsigned long long)policy.pinned_blocks());
  // Pipelined work first: batches submitted before the clear are placed
  // (and then cleared) like synchronous puts would have been; after a
  // failure the rest of them are dropped.
  if (settle() != CB_OK) drop_pipeline();
  plan_open = false;
  CB_TRY(cudaStreamSynchronize(st), "sync");
  if (dht) {  // collective, like DistributedStore::clear (barrier before and after)
    int rc = dht_barrier();
    if (rc) return rc;
  }
  policy.clear();
  CB_TRY(cudaMemsetAsync(table, 0, table_slots * sizeof(Slot), st), "index clear");
  CB_TRY(cudaStreamSynchronize(st), "sync");
  table_used = table_tombs = 0;
  lost.clear();  // metadata and memory agree again: both are empty
  fake_move_failures = 0;
  local_gpu_hits = local_dram_hits = remote_gpu_hits = remote_dram_hits = misses = 0;
  remote_dedup_hits = remote_dedup_bytes = 0;
  replica_promotions = 0;
  if (dht) {
    dht_clear_replicas();
    return dht_barrier();
  }
  return CB_OK;
}

void Store::fill_stats(cb_stats *o) const {
  memset(o, 0, sizeof *o);
  const PolicyCounters &c = policy.counters();
  o->local_gpu_used = policy.hbm_used();
  o->local_dram_used = policy.dram_used();
  o->cluster_gpu_used = o->local_gpu_used;
  o->cluster_dram_used = o->local_dram_used;
  o->local_gpu_hits = local_gpu_hits;
  o->local_dram_hits = local_dram_hits;
  o->remote_gpu_hits = remote_gpu_hits;
  o->remote_dram_hits = remote_dram_hits;
  o->misses = misses;
  // Dedup hits belong to the rank that put the block (like the reference's
  // per-rank counters); in a DHT the owner's policy sees other ranks' puts.
  o->dedup_hits = dht ? remote_dedup_hits : c.dedup_hits;
  o->dedup_bytes_saved = dht ? remote_dedup_bytes : c.dedup_bytes_saved;
  o->gpu_evictions = c.gpu_evictions;
  o->dram_evictions = c.dram_evictions;
  o->promotions_to_local = c.promotions + replica_promotions;
  o->compression_savings = c.compression_savings;
  o->total_blocks = policy.size();
  // the prefix registry (DistributedStore::Stats, distributed_backend.cpp:
  // 1405): prefix blocks this rank stored; after sync_metadata, the cluster's
  o->prefix_blocks = dht ? dht_registry_size() : c.prefix_blocks;
  o->prefix_replicated_blocks = dht_prefix_replicas();
  o->evicted_bytes = c.evicted_bytes;
  o->promoted_bytes = c.promoted_bytes;
  o->dropped_blocks = c.dropped_blocks;
  o->kernel_launches = launches;
  o->peer_bytes_read = peer_bytes_read;
  o->peer_bytes_written = peer_bytes_written;
  uint64_t *p = &o->sha_ns;  // sha, scatter, gather, tier: (ns, bytes, launches) each
  for (int k = 0; k < 4; ++k) {
    p[3 * k] = prof_ns[k];
    p[3 * k + 1] = prof_bytes[k];
    p[3 * k + 2] = prof_launches[k];
  }
  o->coll_ns = prof_ns[4];
  o->coll_bytes = prof_bytes[4];
  o->coll_calls = prof_launches[4];
}

uint64_t Store::staging_capacity() const {
  return cfg.staging_bytes ? cfg.staging_bytes : (1ull << 30);
}

}  // namespace cb

// =================================================================== C ABI

using cb::Store;

struct cb_store {
  Store *s;
};

namespace {

cudaStream_t pick_stream(Store *s, void *stream) {
  return stream ? static_cast<cudaStream_t>(stream) : s->own_stream;
}

// kData calls read or change stored blocks: they are refused once a call
// failed after planning (Store::lost) until clear(), and they first settle
// the stream-ordered work (pipelined puts are placed, stream-ordered gets
// waited for; an error of that work is the call's result). kAsync calls
// (the stream-ordered put and get) are refused in that state too but do not
// settle. kAny calls (statistics, barriers, syncs) run in that state and
// settle; kFree calls (hashing, KV compression, view releases, clear, which
// settles by itself) neither.
// kSubmit: a pipelined put's submission - the one call that runs beside a
// DHT member's placement thread; every other call first waits until that
// thread is idle.
enum Access { kData, kAsync, kAny, kFree, kSubmit };

template <class F>
int guarded(cb_store *h, F f, Access access = kData) {
  if (!h || !h->s) return CB_ERR_ARG;
  Store *s = h->s;
  std::lock_guard<std::mutex> g(s->mu);
  if (access != kSubmit) {
    const int prc = s->placer_idle();  // a failure of the placement thread is this call's error
    if (prc) return prc;
  }
  if ((access == kData || access == kAsync || access == kSubmit) && !s->lost.empty())
    return s->fail(CB_ERR_STATE, "store state lost after a failed call (%s); clear() resets it", s->lost.c_str());
  s->plan_open = false;
  int rc;
  try {
    cudaError_t e = cudaSetDevice(s->device);
    if (e != cudaSuccess) {
      rc = s->cuda_fail(e, "cudaSetDevice");
    } else {
      rc = (access == kData || access == kAny) ? s->settle() : CB_OK;
      if (rc == CB_OK) rc = f(s);
    }
  } catch (const std::bad_alloc &) {
    rc = s->fail(CB_ERR_NOSPACE, "host allocation failed");
  } catch (const std::exception &ex) {
    rc = s->fail(CB_ERR_STATE, "%s", ex.what());
  }
  if (rc != CB_OK && s->plan_open && s->lost.empty()) s->lost = s->last_error_copy();
  s->plan_open = false;
  return rc;
}

}  // namespace

extern "C" {

void cb_config_init(cb_config *c) {
  if (!c) return;
  memset(c, 0, sizeof *c);
  c->gpu_capacity_bytes = 32ull << 30;  // DistributedConfig default
  c->dram_capacity_bytes = 64ull << 30;
  c->device = 0;
  c->dedup_enabled = 1;
  c->semantic_eviction = 1;
  c->promote_on_hit = 1;
  c->promotion_rule = CB_PROMOTE_LOCALITY;  // DistributedStore::get's rule
  c->index_log2 = 16;
  c->copy_engine = 0;
  c->staging_bytes = 1ull << 30;
}

int cb_create(const cb_config *cfg, cb_store **out) {
  if (!cfg || !out) return CB_ERR_ARG;
  *out = nullptr;
  Store *s = nullptr;
  try {
    s = new Store(*cfg);
  } catch (...) {
    cb::g_create_error = "host allocation failed";
    return CB_ERR_NOSPACE;
  }
  s->copy_engine = cfg->copy_engine == 2 ? 2 : 1;
  int rc = s->init();
  if (rc) {
    cb::g_create_error = s->last_error_copy();
    delete s;
    return rc;
  }
  *out = new cb_store{s};
  return CB_OK;
}

int cb_destroy(cb_store *h) {
  if (!h) return CB_OK;
  delete h->s;
  delete h;
  return CB_OK;
}

// The message is copied under the store's mutex into a per-thread buffer: a
// call from another thread may replace the store's message meanwhile, and
// the pointer returned here must stay valid until this thread asks again.
const char *cb_last_error(const cb_store *h) {
  static thread_local std::string copy;
  if (!h || !h->s) return cb::g_create_error.c_str();
  std::lock_guard<std::mutex> g(h->s->mu);
  copy = h->s->last_error_copy();
  return copy.c_str();
}

int cb_selftest(cb_store *h, int32_t which) {
  return guarded(h, [&](Store *s) -> int { return s->selftest(which, s->own_stream); }, kAny);
}

int cb_put_batch_async(cb_store *h, const void *const *ptrs, const uint64_t *sizes, const uint8_t *is_prefix,
                       const uint8_t *keys_in, int32_t n, int32_t mem_kind, uint8_t *keys_out, uint8_t *status_out,
                       uint64_t *ticket_out, void *stream) {
  return guarded(h, [&](Store *s) -> int {
    if (n < 0 || (n > 0 && (!ptrs || !sizes)) || !ticket_out) return s->fail(CB_ERR_ARG, "bad arguments");
    if (mem_kind != CB_MEM_DEVICE && mem_kind != CB_MEM_HOST) return s->fail(CB_ERR_ARG, "unknown mem_kind %d", mem_kind);
    for (int i = 0; i < n; ++i)
      if (sizes[i] > cb::kSizeMask) return s->fail(CB_ERR_ARG, "block %d too large", i);
    cudaStream_t st = pick_stream(s, stream);
    if (mem_kind == CB_MEM_HOST) {
      // host blocks are staged and placed at once, after every earlier batch
      int rc = s->settle();
      if (rc) return rc;
      *ticket_out = s->next_ticket++;
      s->placed_ticket = *ticket_out;
      if (s->world > 1)
        return s->dht_put(ptrs, sizes, is_prefix, keys_in, n, mem_kind, keys_out, status_out, st);
      return n ? s->put_host(ptrs, sizes, is_prefix, keys_in, n, keys_out, status_out, st) : CB_OK;
    }
    std::vector<uint64_t> p(n);
    for (int i = 0; i < n; ++i) p[i] = (uint64_t)ptrs[i];
    return s->put_async(p.data(), sizes, is_prefix, keys_in, n, keys_out, status_out, ticket_out, st);
  }, kSubmit);
}

int cb_put_wait(cb_store *h, uint64_t ticket, uint64_t *placed_out) {
  return guarded(h, [&](Store *s) -> int {
    const int rc = s->put_wait(ticket ? ticket : UINT64_MAX);
    if (placed_out) {
      std::lock_guard<std::mutex> g(s->pmu);
      *placed_out = s->placed_ticket;
    }
    return rc;
  }, kAsync);
}

int cb_put_placed(cb_store *h, uint64_t *placed_out) {
  if (!h || !h->s || !placed_out) return CB_ERR_ARG;
  std::lock_guard<std::mutex> g(h->s->mu);
  std::lock_guard<std::mutex> g2(h->s->pmu);  // the placement thread advances it
  *placed_out = h->s->placed_ticket;
  return CB_OK;
}

int cb_get_batch_async(cb_store *h, const uint8_t *keys, int32_t n, void *const *outs, const uint64_t *out_caps,
                       uint64_t *sizes_out, uint8_t *found_out, void *stream) {
  return guarded(h, [&](Store *s) -> int {
    if (n < 0 || (n > 0 && (!keys || !outs || !out_caps || !sizes_out || !found_out)))
      return s->fail(CB_ERR_ARG, "bad arguments");
    cudaStream_t st = pick_stream(s, stream);
    if (s->world > 1) {  // DHT gets are collective and synchronous
      int rc = s->settle();
      if (rc) return rc;
      return s->dht_get(keys, n, outs, out_caps, CB_MEM_DEVICE, sizes_out, found_out, st);
    }
    if (n == 0) return CB_OK;
    std::vector<uint64_t> o(n);
    for (int i = 0; i < n; ++i) o[i] = (uint64_t)outs[i];
    return s->get_async(keys, n, o.data(), out_caps, sizes_out, found_out, st);
  }, kAsync);
}

int cb_get_views(cb_store *h, const uint8_t *keys, int32_t n, uint64_t *addrs_out, uint64_t *sizes_out,
                 uint8_t *found_out, void *stream) {
  return guarded(h, [&](Store *s) -> int {
    if (n < 0 || (n > 0 && (!keys || !addrs_out || !sizes_out || !found_out))) return s->fail(CB_ERR_ARG, "bad arguments");
    if (s->dht) return s->fail(CB_ERR_STATE, "zero-copy views are local to one store (not on a DHT member)");
    if (n == 0) return CB_OK;
    return s->get_views(keys, n, addrs_out, sizes_out, found_out, pick_stream(s, stream));
  });
}

int cb_release_views(cb_store *h, const uint8_t *keys, int32_t n) {
  return guarded(h, [&](Store *s) -> int {
    if (n < 0 || (n > 0 && !keys)) return s->fail(CB_ERR_ARG, "bad arguments");
    return s->release_views(keys, n);
  }, kFree);
}

int cb_kv_compress_batch(cb_store *h, const void *const *srcs, const uint64_t *sizes, void *const *dsts,
                         int32_t n, void *stream) {
  return guarded(h, [&](Store *s) -> int {
    if (n < 0 || (n > 0 && (!srcs || !sizes || !dsts))) return s->fail(CB_ERR_ARG, "bad arguments");
    if (n == 0) return CB_OK;
    std::vector<uint64_t> src(n), dst(n);
    for (int i = 0; i < n; ++i) {
      src[i] = (uint64_t)srcs[i];
      dst[i] = (uint64_t)dsts[i];
    }
    return s->kv_compress(src.data(), sizes, dst.data(), n, pick_stream(s, stream));
  }, kFree);
}

int cb_kv_decompress_batch(cb_store *h, const void *const *srcs, const uint64_t *comp_sizes,
                           const uint64_t *orig_sizes, void *const *dsts, int32_t n, uint8_t *ok_out,
                           void *stream) {
  return guarded(h, [&](Store *s) -> int {
    if (n < 0 || (n > 0 && (!srcs || !comp_sizes || !orig_sizes || !dsts))) return s->fail(CB_ERR_ARG, "bad arguments");
    if (n == 0) return CB_OK;
    std::vector<uint64_t> src(n), dst(n);
    for (int i = 0; i < n; ++i) {
      src[i] = (uint64_t)srcs[i];
      dst[i] = (uint64_t)dsts[i];
    }
    return s->kv_decompress(src.data(), comp_sizes, orig_sizes, dst.data(), n, ok_out, pick_stream(s, stream));
  }, kFree);
}

int cb_hash_batch(cb_store *h, const void *const *ptrs, const uint64_t *sizes, int32_t n,
                  int32_t mem_kind, uint8_t *digests_out, void *stream) {
  return guarded(h, [&](Store *s) -> int {
    if (n < 0 || (n > 0 && (!ptrs || !sizes || !digests_out))) return s->fail(CB_ERR_ARG, "bad arguments");
    if (mem_kind != CB_MEM_DEVICE && mem_kind != CB_MEM_HOST) return s->fail(CB_ERR_ARG, "unknown mem_kind %d", mem_kind);
    if (n == 0) return CB_OK;
    cudaStream_t st = pick_stream(s, stream);
    if (mem_kind == CB_MEM_DEVICE) {
      std::vector<uint64_t> p(n);
      for (int i = 0; i < n; ++i) p[i] = (uint64_t)ptrs[i];
      int rc = s->hash_device(p.data(), sizes, n, st);
      if (rc) return rc;
      memcpy(digests_out, s->h_out.ptr, 32ull * n);
      return CB_OK;
    }
    // Host blocks: stage slices into device memory and hash them there.
    const uint64_t cap = s->staging_capacity();
    std::vector<uint64_t> p;
    int i = 0;
    while (i < n) {
      uint64_t bytes = 0;
      int j = i;
      while (j < n && (j == i || bytes + cb::align_up(sizes[j], 256) <= cap)) bytes += cb::align_up(sizes[j++], 256);
      cudaError_t e = s->d_staging.ensure(std::max<uint64_t>(bytes, 256));
      if (e != cudaSuccess) return s->cuda_fail(e, "device staging");
      p.resize(j - i);
      uint64_t off = 0;
      for (int k = i; k < j; ++k) {
        p[k - i] = (uint64_t)s->d_staging.ptr + off;
        if (sizes[k]) {
          e = cudaMemcpyAsync(reinterpret_cast<void *>(p[k - i]), ptrs[k], sizes[k], cudaMemcpyHostToDevice, st);
          if (e != cudaSuccess) return s->cuda_fail(e, "H2D block");
        }
        off += cb::align_up(sizes[k], 256);
      }
      int rc = s->hash_device(p.data(), sizes + i, j - i, st);
      if (rc) return rc;
      memcpy(digests_out + 32ull * i, s->h_out.ptr, 32ull * (j - i));
      i = j;
    }
    return CB_OK;
  }, kFree);
}

int cb_put_batch(cb_store *h, const void *const *ptrs, const uint64_t *sizes, const uint8_t *is_prefix,
                 const uint8_t *keys_in, int32_t n, int32_t mem_kind, uint8_t *keys_out,
                 uint8_t *status_out, void *stream) {
  return guarded(h, [&](Store *s) -> int {
    if (n < 0 || (n > 0 && (!ptrs || !sizes))) return s->fail(CB_ERR_ARG, "bad arguments");
    if (mem_kind != CB_MEM_DEVICE && mem_kind != CB_MEM_HOST) return s->fail(CB_ERR_ARG, "unknown mem_kind %d", mem_kind);
    for (int i = 0; i < n; ++i)
      if (sizes[i] > cb::kSizeMask) return s->fail(CB_ERR_ARG, "block %d too large", i);
    cudaStream_t st = pick_stream(s, stream);
    // DHT calls are collective: a rank with nothing to put still takes part.
    if (s->world > 1) return s->dht_put(ptrs, sizes, is_prefix, keys_in, n, mem_kind, keys_out, status_out, st);
    if (n == 0) return CB_OK;
    if (mem_kind == CB_MEM_HOST) return s->put_host(ptrs, sizes, is_prefix, keys_in, n, keys_out, status_out, st);
    std::vector<uint64_t> p(n);
    for (int i = 0; i < n; ++i) p[i] = (uint64_t)ptrs[i];
    return s->put_device(p.data(), sizes, is_prefix, keys_in, n, keys_out, status_out, st);
  });
}

int cb_get_batch(cb_store *h, const uint8_t *keys, int32_t n, void *const *outs, const uint64_t *out_caps,
                 int32_t mem_kind, uint64_t *sizes_out, uint8_t *found_out, void *stream) {
  return guarded(h, [&](Store *s) -> int {
    if (n < 0 || (n > 0 && (!keys || !outs || !out_caps || !sizes_out || !found_out)))
      return s->fail(CB_ERR_ARG, "bad arguments");
    if (mem_kind != CB_MEM_DEVICE && mem_kind != CB_MEM_HOST) return s->fail(CB_ERR_ARG, "unknown mem_kind %d", mem_kind);
    cudaStream_t st = pick_stream(s, stream);
    if (s->world > 1) return s->dht_get(keys, n, outs, out_caps, mem_kind, sizes_out, found_out, st);
    if (n == 0) return CB_OK;
    if (mem_kind == CB_MEM_HOST) return s->get_host(keys, n, outs, out_caps, sizes_out, found_out, st);
    std::vector<uint64_t> o(n);
    for (int i = 0; i < n; ++i) o[i] = (uint64_t)outs[i];
    return s->get_device(keys, n, o.data(), out_caps, sizes_out, found_out, st);
  });
}

int cb_contains_batch(cb_store *h, const uint8_t *keys, int32_t n, uint8_t *found_out) {
  return guarded(h, [&](Store *s) -> int {
    if (n < 0 || (n > 0 && (!keys || !found_out))) return s->fail(CB_ERR_ARG, "bad arguments");
    if (s->world > 1) return s->dht_contains(keys, n, found_out, s->own_stream);
    for (int i = 0; i < n; ++i) found_out[i] = s->policy.find(cb::to_hkey(keys + 16 * i)) ? 1 : 0;
    return CB_OK;
  });
}

int cb_locate(cb_store *h, const uint8_t *key, cb_location *out, int32_t *found) {
  return guarded(h, [&](Store *s) -> int {
    if (!key || !out || !found) return s->fail(CB_ERR_ARG, "bad arguments");
    if (s->dht) return s->dht_locate(key, out, found);
    const cb::BlockMeta *m = s->policy.find(cb::to_hkey(key));
    *found = m ? 1 : 0;
    memset(out, 0, sizeof *out);
    if (!m) return CB_OK;
    out->node_id = s->rank;
    out->gpu_id = m->tier == cb::kTierHbm ? s->device : -1;
    out->offset = cb::Policy::data_offset(*m);
    out->size = m->size;
    out->is_gpu = m->tier == cb::kTierHbm;
    out->is_prefix = m->prefix;
    return CB_OK;
  });
}

int cb_evict(cb_store *h, uint64_t bytes, uint64_t *evicted_bytes) {
  return guarded(h, [&](Store *s) -> int { return s->evict(bytes, evicted_bytes, s->own_stream); });
}

int cb_get_stats(cb_store *h, cb_stats *out) {
  return guarded(h, [&](Store *s) -> int {
    if (!out) return s->fail(CB_ERR_ARG, "bad arguments");
    s->resolve_prof(true);  // records of batches that ended without a store-side sync
    s->fill_stats(out);
    if (s->world > 1) return s->dht_cluster_usage(out);
    return CB_OK;
  }, kAny);
}

int cb_clear(cb_store *h) {
  return guarded(h, [&](Store *s) -> int { return s->clear(s->own_stream); }, kFree);
}

int cb_sync(cb_store *h) {
  return guarded(h, [&](Store *s) -> int {
    cudaError_t e = cudaStreamSynchronize(s->own_stream);
    if (e != cudaSuccess) return s->cuda_fail(e, "sync");
    return CB_OK;
  }, kAny);
}

int cb_dht_attach(cb_store *h, int32_t rank, int32_t world, const uint8_t *uid) {
  return guarded(h, [&](Store *s) -> int {
    if (!uid) return s->fail(CB_ERR_ARG, "bad arguments");
    return s->dht_attach(rank, world, uid);
  }, kAny);
}

int cb_sync_metadata(cb_store *h) {
  return guarded(h, [&](Store *s) -> int {
    if (!s->dht) return CB_OK;  // one GPU: the registry is already complete
    return s->dht_sync_prefixes(s->own_stream);
  });
}

int cb_dht_barrier(cb_store *h) {
  return guarded(h, [&](Store *s) -> int { return s->world > 1 ? s->dht_barrier() : CB_OK; }, kAny);
}

int32_t cb_owner_rank(const uint8_t *key, int32_t world) {
  if (!key || world <= 0) return -1;
  const cb::HKey k = cb::to_hkey(key);
  return cb::owner_of(cb::Key{k.lo, k.hi}, world);
}

int cb_rank(const cb_store *h, int32_t *rank, int32_t *world) {
  if (!h || !h->s || !rank || !world) return CB_ERR_ARG;
  *rank = h->s->rank;
  *world = h->s->world;
  return CB_OK;
}

}  // extern "C"
