// Store object behind the C ABI (one per GPU per process).
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <condition_variable>
#include <deque>
#include <functional>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include <nvtx3/nvToolsExt.h>

#include "cascade_b200.h"
#include "common.cuh"
#include "kernels.cuh"
#include "policy.hpp"

// Returns from a Store member with CB_ERR_CUDA on a CUDA error.
#define CB_TRY_CUDA(call, what)                          \
  do {                                                   \
    cudaError_t _e = (call);                             \
    if (_e != cudaSuccess) return cuda_fail(_e, what);   \
  } while (0)

namespace cb {

// NVTX range over one phase of a batch (hash, tier moves, scatter, gather,
// DHT exchange): visible to nsys/ncu timelines, a no-op without a tool.
struct Trace {
  explicit Trace(const char *name) { nvtxRangePushA(name); }
  ~Trace() { nvtxRangePop(); }
  Trace(const Trace &) = delete;
  Trace &operator=(const Trace &) = delete;
};

struct PinnedBuf {
  void *ptr = nullptr;
  size_t cap = 0;
  unsigned flags = cudaHostAllocPortable;  // cudaHostAlloc flags of the next allocation
  cudaError_t ensure(size_t bytes);
  void release();
};

struct DevBuf {
  void *ptr = nullptr;
  size_t cap = 0;
  cudaError_t ensure(size_t bytes);
  void release();
};

struct DhtState;  // dht.cu

// A DHT member keeps kDhtSpareSms SMs free of hash launches (green context,
// cb_config.hash_sms = 0), and its NCCL communicator runs every collective
// with at most kDhtNcclCtas CTAs, so that a collective issued while the hash
// CTAs fill their SMs runs at once on the spare ones: an NCCL kernel whose
// CTAs (channels) cannot all be resident waits, on both ranks, until hash
// CTAs retire.
constexpr int kDhtSpareSms = 8;
constexpr int kDhtNcclCtas = 4;

struct Store {
  explicit Store(const cb_config &c);
  ~Store();
  int init();

  cb_config cfg;
  int device = -1;
  int num_sms = 148;
  int copy_engine = 1;  // 1 TMA bulk, 2 LSU
  int hash_lanes = 32;  // chains per warp in the SHA-256 kernel
  cudaStream_t own_stream = nullptr;
  // DHT puts: the peer stores of a put run on peer_stream beside the local
  // stores (TMA engine) on the put's stream; ev_peer_in/out join them.
  cudaStream_t peer_stream = nullptr;
  cudaEvent_t ev_peer_in = nullptr, ev_peer_out = nullptr;

  uint8_t *pool = nullptr;  // HBM slab pool
  uint64_t pool_bytes = 0;
  uint8_t *dram_host = nullptr;  // pinned DRAM arena (host address)
  uint8_t *dram_dev = nullptr;   // same arena, device address
  uint64_t dram_bytes = 0;

  Slot *table = nullptr;
  uint64_t table_slots = 0, table_used = 0, table_tombs = 0;
  unsigned *d_err = nullptr;

  PinnedBuf h_scratch, h_out, h_err;
  DevBuf d_scratch, d_staging;

  Policy policy;
  PutPlan put_plan;
  std::mutex mu;
  std::mutex err_mu;  // last_error: also written by the placement thread
  std::string last_error;
  std::string last_error_copy() {
    std::lock_guard<std::mutex> g(err_mu);
    return last_error;
  }
  // The host metadata records a batch's placements and tier moves when the
  // batch is planned. A call that fails after planning (plan_open still set
  // when it returns) may leave metadata that its memory does not match, so
  // the store refuses data calls (`lost` holds the first error) until clear().
  bool plan_open = false;
  bool placer_plan_open = false;  // the placement thread's own flag (its failures always lose the state)
  bool &plan_flag() { return std::this_thread::get_id() == placer_id ? placer_plan_open : plan_open; }
  std::string lost;
  int fake_move_failures = 0;  // CB_SELFTEST_FAIL_MOVES: host-side injection

  uint64_t local_gpu_hits = 0, local_dram_hits = 0, remote_gpu_hits = 0, remote_dram_hits = 0,
           misses = 0, remote_dedup_hits = 0, remote_dedup_bytes = 0;
  uint64_t peer_bytes_read = 0, peer_bytes_written = 0;  // not reset by clear (traffic counters)
  uint64_t replica_promotions = 0;  // DHT: hot remote blocks copied to local HBM

  int rank = 0, world = 1;
  DhtState *dht = nullptr;

  // Kernel accounting. kinds: 0 SHA-256, 1 scatter, 2 gather, 3 tier move,
  // 4 DHT collective (NCCL; not counted as a kernel launch of this store).
  // With profiling on, every launch is bracketed by two CUDA events on its
  // stream; the pairs are read after the batch's final synchronisation
  // (resolve_prof), so profiling does not serialise streams.
  bool profile = false;
  std::atomic<uint64_t> launches{0};
  static constexpr int kProfKinds = 5;
  uint64_t prof_ns[kProfKinds] = {}, prof_bytes[kProfKinds] = {}, prof_launches[kProfKinds] = {};
  struct ProfRec {
    int kind;
    uint64_t bytes;
    cudaEvent_t a, b;
  };
  std::vector<cudaEvent_t> prof_events;  // every event created (destroyed with the store)
  std::vector<ProfRec> prof_pending;
  cudaError_t prof_event(cudaEvent_t &e);
  std::vector<cudaEvent_t> prof_free;  // created, not in use
  // Reads the timing of finished launches; with `wait`, waits for all.
  void resolve_prof(bool wait = false);

  // Runs `launch` (one or two kernels on stream st) and, when profiling,
  // brackets it with events. `bytes` = payload bytes it processes.
  template <class F>
  cudaError_t timed(int kind, uint64_t bytes, cudaStream_t st, F launch) {
    launches++;
    if (!profile) return launch();
    cudaEvent_t a, b;
    cudaError_t e = prof_event(a);
    if (e == cudaSuccess) e = prof_event(b);
    if (e == cudaSuccess) e = cudaEventRecord(a, st);
    if (e != cudaSuccess) return e;
    e = launch();
    if (e != cudaSuccess) return e;
    e = cudaEventRecord(b, st);
    if (e == cudaSuccess) prof_pending.push_back(ProfRec{kind, bytes, a, b});
    return e;
  }

  // The same bracketing for a DHT collective step (`call` returns a CB_*
  // code); `bytes` = payload bytes this rank sends in it.
  template <class F>
  int timed_coll(uint64_t bytes, cudaStream_t st, F call) {
    if (!profile) return call();
    cudaEvent_t a, b;
    cudaError_t e = prof_event(a);
    if (e == cudaSuccess) e = prof_event(b);
    if (e == cudaSuccess) e = cudaEventRecord(a, st);
    if (e != cudaSuccess) return cuda_fail(e, "collective timing event");
    const int rc = call();
    if (rc) return rc;
    e = cudaEventRecord(b, st);
    if (e != cudaSuccess) return cuda_fail(e, "collective timing event");
    prof_pending.push_back(ProfRec{4, bytes, a, b});
    return 0;
  }

  int fail(int code, const char *fmt, ...);
  int cuda_fail(cudaError_t e, const char *what);

  cudaError_t alloc_table(uint64_t slots);
  cudaError_t ensure_dram();
  int reserve_index(uint64_t incoming, cudaStream_t st);
  int check_device_error(cudaStream_t st);
  // Runs a plan's tier moves on st. With `concurrent`, the demotions run on
  // move_stream while `concurrent()` issues other work on st; promotions
  // (which may reuse HBM the demotions vacate) and index updates follow both.
  int run_moves(const std::vector<TierMove> &moves, const std::vector<HKey> &dropped, cudaStream_t st,
                const std::function<int()> &concurrent = nullptr);
  cudaStream_t move_stream = nullptr;
  cudaEvent_t ev_move_in = nullptr, ev_move_done = nullptr;
  PinnedBuf h_mscratch;  // descriptors of run_moves (separate from the callers')
  DevBuf d_mscratch;
  DevBuf d_pack;    // packed images of large demotions, on their way to DRAM by DMA
  DevBuf d_unpack;  // packed DRAM hits of a get, brought in by DMA to be unpacked
  // pg/copies_done: the blocks are still arriving on copy_stream (see
  // put_host); the hash kernel waits per segment and later work on st waits
  // for copies_done.
  int hash_device(const uint64_t *ptrs, const uint64_t *sizes, int n, cudaStream_t st,
                  const HashProgress *pg = nullptr, cudaEvent_t copies_done = nullptr);
  int put_device(const uint64_t *ptrs, const uint64_t *sizes, const uint8_t *is_prefix,
                 const uint8_t *keys_in, int n, uint8_t *keys_out, uint8_t *status_out,
                 cudaStream_t st, const HashProgress *pg = nullptr, cudaEvent_t copies_done = nullptr);
  int stage_overlapped(const void *const *ptrs, const uint64_t *sizes, int n, uint64_t *dptrs,
                       HashProgress &pg, cudaStream_t st);

  // Host puts: a second stream copies blocks in while the hash runs.
  cudaStream_t copy_stream = nullptr;
  unsigned *d_progress = nullptr;
  PinnedBuf h_progress;
  cudaEvent_t ev_reset = nullptr, ev_copies = nullptr;
  int put_host(const void *const *ptrs, const uint64_t *sizes, const uint8_t *is_prefix,
               const uint8_t *keys_in, int n, uint8_t *keys_out, uint8_t *status_out,
               cudaStream_t st);
  int get_device(const uint8_t *keys, int n, const uint64_t *outs, const uint64_t *caps,
                 uint64_t *sizes_out, uint8_t *found_out, cudaStream_t st);
  int get_host(const uint8_t *keys, int n, void *const *outs, const uint64_t *caps,
               uint64_t *sizes_out, uint8_t *found_out, cudaStream_t st);
  int evict(uint64_t bytes, uint64_t *evicted, cudaStream_t st);
  int selftest(int which, cudaStream_t st);
  // Zero-copy gets: pool addresses of HBM blocks, pinned until released.
  int get_views(const uint8_t *keys, int n, uint64_t *addrs_out, uint64_t *sizes_out, uint8_t *found_out,
                cudaStream_t st);
  int release_views(const uint8_t *keys, int n);
  // INT8 KV packing of device blocks outside the store (KVCompressor).
  int kv_compress(const uint64_t *srcs, const uint64_t *sizes, const uint64_t *dsts, int n, cudaStream_t st);
  int kv_decompress(const uint64_t *srcs, const uint64_t *comp_sizes, const uint64_t *orig_sizes,
                    const uint64_t *dsts, int n, uint8_t *ok_out, cudaStream_t st);
  int clear(cudaStream_t st);
  void fill_stats(cb_stats *o) const;
  uint64_t staging_capacity() const;

  // pipeline.cu — stream-ordered (pipelined) puts and gets.
  //
  // Pipelined put: a batch's SHA-256 is launched at submission on one of
  // kHashSlots side streams (several queued small batches share one launch),
  // so many batches hash concurrently; batches are then placed (dedup plan,
  // tier moves, scatter, index insert) strictly in submission order, which
  // keeps the sequential dedup rule of put_batch exactly.
  struct HashSlot {
    PinnedBuf h;  // [HashJob x n][digests n x 32], mapped: the kernel writes the digests here
    DevBuf d;
    cudaStream_t stream = nullptr;
    int n = 0;                   // blocks of the launch
    int cap = 0;                 // blocks the slot's buffers hold
    int users = 0;               // batches of the launch not placed yet
    bool launched = false;
    bool finished = false;       // launched and its digests are back
  };
  struct AsyncPut {
    uint64_t ticket = 0;
    std::vector<uint64_t> ptrs, sizes;
    std::vector<uint8_t> prefix, keys_in;  // empty: none given
    uint8_t *keys_out = nullptr, *status_out = nullptr;
    int slot = -1, off = 0;  // its digests: slot's launch, from block `off`
  };
  // Ring of scratch buffers for stream-ordered kernels whose descriptors must
  // outlive the call (pipelined scatters, stream-ordered gathers).
  struct ScratchSlot {
    PinnedBuf h;
    DevBuf d;
    cudaEvent_t done = nullptr;
    bool pending = false;  // done is recorded and not yet waited for by the host
  };
  static constexpr int kHashSlots = 64;
  static constexpr int kScratchSlots = 16;
  HashSlot hslots[kHashSlots];
  int hslot_next = 0;
  std::deque<AsyncPut> aput;         // submitted, not placed (submission order); DHT: not yet assigned
  // DHT member: groups of pipelined batches are placed (collective DHT put)
  // by a placement thread of the store, in assignment order, while the
  // caller keeps submitting and the GPU keeps hashing. Assignment is
  // count-based, the same on every rank, so every rank's thread runs the
  // same sequence of collectives. Every other call that needs the store's
  // state or its communicator first waits until the thread is idle.
  std::thread placer;
  std::thread::id placer_id;
  std::mutex pmu;                    // guards the fields below and hslots[].users of a DHT member
  std::condition_variable pcv;
  std::deque<std::vector<AsyncPut>> pgroups;  // assigned, not placed (oldest first)
  bool placer_busy = false, placer_stop = false;
  int placer_rc = 0;                 // first failure of the thread (the state is then lost)
  std::string placer_err;
  int assign_dht_group(size_t count);  // caller: the `count` oldest unassigned batches to the thread
  int placer_idle();                 // caller: waits until nothing is assigned; reports a failure
  void placer_loop();
  void placer_join();
  int place_dht_batches(std::vector<AsyncPut> &g);  // placement thread
  int open_slot = -1;                // slot collecting batches not launched yet
  uint64_t next_ticket = 1, placed_ticket = 0;
  uint64_t inflight_blocks = 0;      // blocks submitted and not placed
  uint64_t hashing_blocks = 0;       // blocks of launches whose digests are not back yet
  void refresh_hashing();            // notes launches that finished (does not wait)
  bool front_ready() const;          // the oldest batch can be placed without waiting
  cudaStream_t put_stream = nullptr; // placements of pipelined puts
  // Hash streams may live in a green context holding part of the SMs, so
  // that collectives and copies always find free SMs beside a GPU full of
  // hash CTAs (cb_config.hash_sms). hash_sm_count = SMs they may use.
  void *green = nullptr;             // CUgreenCtx, or null: ordinary streams on every SM
  int hash_sm_count = 0;
  int make_hash_green_context(int sms);
  cudaError_t create_hash_stream(cudaStream_t &s);
  ScratchSlot sslots[kScratchSlots];
  int sslot_next = 0;
  bool pipeline_ready = false;
  int pipeline_init();
  void pipeline_release();
  int put_async(const uint64_t *ptrs, const uint64_t *sizes, const uint8_t *is_prefix, const uint8_t *keys_in,
                int n, uint8_t *keys_out, uint8_t *status_out, uint64_t *ticket, cudaStream_t st);
  int put_wait(uint64_t ticket);
  int place_until(uint64_t ticket);
  int launch_open_slot();
  int place_oldest();
  int place_batch(const std::vector<HKey> &keys, AsyncPut &b);
  // Scatter + INT8 packing + index insert of a plan's placements on st, with
  // descriptors in (h, d). Returns without waiting.
  int enqueue_places(const PutPlan &plan, const uint64_t *ptrs, cudaStream_t st, PinnedBuf &h, DevBuf &d,
                     int engine, int lsu_ctas_per_sm);
  ScratchSlot *take_scratch(size_t bytes, int &rc);
  // The next take_scratch would not wait.
  bool scratch_free() const;
  // Every pool extent a stream-ordered gather may still read is released
  // only after it: work that may write the pool waits for them first.
  int fence_reads(cudaStream_t st);
  // Settles everything stream-ordered: places every pipelined put, waits for
  // every stream-ordered gather, and reports a device error any of them
  // raised (CB_ERR_DEVICE / CB_ERR_TIMEOUT) before the caller goes on.
  int settle();
  int finish_placements();
  void drop_pipeline();
  unsigned *d_err_get = nullptr;  // device errors of stream-ordered gathers
  // Reads and clears a device error word (st is synchronised first).
  int read_error_word(unsigned *word, cudaStream_t st);
  int get_async(const uint8_t *keys, int n, const uint64_t *outs, const uint64_t *caps, uint64_t *sizes_out,
                uint8_t *found_out, cudaStream_t st);
  bool inject_get_error = false;  // CB_SELFTEST_GET_ERROR: host-side injection
  bool placed_unsettled = false;  // a pipelined batch was placed since the last settle()
  cudaEvent_t ev_submit = nullptr;

  // dht.cu
  int dht_attach(int rank, int world, const uint8_t *uid);
  void dht_detach();
  int dht_barrier();
  int dht_nccl(int nccl_result, const char *what);
  int dht_sync(cudaStream_t st);
  int dht_finish(cudaStream_t st);
  int dht_counts(const uint32_t *scount, uint32_t *rcount, cudaStream_t st);
  int dht_alltoallv(const void *d_send, const uint32_t *scount, void *d_recv, const uint32_t *rcount, size_t rec,
                    cudaStream_t st);
  int dht_alltoallv_group(const void *d_send, const uint32_t *scount, void *d_recv, const uint32_t *rcount,
                          size_t rec, cudaStream_t st);
  // stage: DRAM-tier blocks other ranks ask for go to the outbox (a get);
  // without it the replies only say where each block is (contains).
  int dht_lookup(const uint8_t *keys, int n, std::vector<uint64_t> &reps, std::vector<int> &owner,
                 cudaStream_t st, bool stage = true);
  int dht_locate(const uint8_t *key, cb_location *out, int32_t *found);
  void dht_clear_replicas();
  // step (may be null): per block, the index of its batch within a group of
  // pipelined batches placed in one collective step (non-decreasing).
  int dht_put(const void *const *ptrs, const uint64_t *sizes, const uint8_t *is_prefix,
              const uint8_t *keys_in, int n, int mem_kind, uint8_t *keys_out,
              uint8_t *status_out, cudaStream_t st, const uint16_t *step = nullptr);
  int dht_slot_free(int s);  // caller: waits until hash slot s is placed
  int dht_get(const uint8_t *keys, int n, void *const *outs, const uint64_t *caps, int mem_kind,
              uint64_t *sizes_out, uint8_t *found_out, cudaStream_t st);
  int dht_contains(const uint8_t *keys, int n, uint8_t *found_out, cudaStream_t st);
  int dht_cluster_usage(cb_stats *o);
  int dht_sync_prefixes(cudaStream_t st);
  int dht_drain_inbox(const std::vector<std::pair<const Placement *, uint64_t>> &inbox, cudaStream_t st);
  // Owner side of a get step when this rank's DRAM tier holds blocks: the
  // replies come from the host metadata, and DRAM-tier blocks other ranks
  // asked for are staged into the outbox for their peer loads.
  int dht_serve_host(const uint8_t *d_keys, uint32_t nrecv, const uint32_t *rcount, uint64_t *d_reps,
                     cudaStream_t st, bool stage);
  uint64_t dht_registry_size() const;
  uint64_t dht_prefix_replicas() const;
};

inline uint64_t align_up(uint64_t x, uint64_t a) { return (x + a - 1) / a * a; }

// Offsets of the parts of one scratch buffer, each 256-byte aligned.
struct Layout {
  size_t off = 0;
  size_t add(size_t bytes) {
    off = align_up(off, 256);
    const size_t o = off;
    off += bytes;
    return o;
  }
};

// dht.cu: the DHT's host-side routing and owner planning (also exported for
// host-only use through cb_dht_route / cb_dht_plan_put).
void dht_route(const HKey *keys, int n, int W, int *owner, int *order, uint32_t *scount);
void dht_owner_plan(Policy &policy, const HKey *keys, const uint64_t *sizes, const uint8_t *prefix, uint32_t n,
                    bool dedup, PutPlan &plan, uint32_t *status, uint64_t *loc);

// The address range one copy starting at p may cover: the CUDA allocation
// that contains p (device, pinned or managed), or everything when p is memory
// CUDA does not know (pageable host memory, copied through staging whatever
// its extent). Neighbouring caller buffers can be adjacent in the address
// space yet belong to different allocations; a copy must not span them.
// Returns [p, p) when the range cannot be determined.
struct AddrRange {
  uint64_t lo, hi;
  bool holds(const void *p, uint64_t bytes) const {
    const uint64_t a = reinterpret_cast<uint64_t>(p);
    return a >= lo && a <= hi && bytes <= hi - a;
  }
};
AddrRange alloc_range(const void *p);
inline bool one_allocation(const void *p, uint64_t bytes) { return alloc_range(p).holds(p, bytes); }

inline HKey to_hkey(const uint8_t *p) {
  HKey k;
  __builtin_memcpy(&k.lo, p, 8);
  __builtin_memcpy(&k.hi, p + 8, 8);
  return k;
}

}  // namespace cb
