/*
 * cascade_b200.h — C ABI of the B200-native Cascade block data path.
 *
 * One store per GPU per process. All array arguments are HOST arrays; the
 * block pointers inside them (ptrs / outs) point to device memory
 * (mem_kind = CB_MEM_DEVICE) or host memory (CB_MEM_HOST). Keys are the
 * 16-byte binary form of the 32-hex BlockId (first 16 bytes of SHA-256).
 * No function throws; every function returns a CB_* status and leaves a
 * message for cb_last_error(). Calls on one store are serialised internally.
 * `stream` is a cudaStream_t (NULL = the store's own stream, which is ordered
 * with the legacy default stream); work is ordered after prior work on it and
 * the call returns with its results final.
 */
#ifndef CASCADE_B200_H
#define CASCADE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes (reference returns bool: gpu_backend.cu:43-51) ------- */
#define CB_OK 0
#define CB_ERR_ARG 1      /* bad argument                                   */
#define CB_ERR_CUDA 2     /* CUDA runtime error                             */
#define CB_ERR_NOSPACE 3  /* HBM + DRAM tiers cannot hold the block         */
#define CB_ERR_BUFSIZE 4  /* an output buffer is smaller than the block     */
#define CB_ERR_TIMEOUT 5  /* a bounded device or collective wait ran out    */
#define CB_ERR_NCCL 6     /* NCCL error                                     */
#define CB_ERR_STATE 7    /* call not valid in the store's current state    */
#define CB_ERR_DEVICE 8   /* a device-side check failed (bounds, index)     */

/* ---- memory kind of the block pointers --------------------------------- */
#define CB_MEM_DEVICE 0
#define CB_MEM_HOST 1

/* ---- put status per block ---------------------------------------------- */
#define CB_PUT_STORED 0  /* new block stored                                */
#define CB_PUT_DEDUP 1   /* key already stored (or earlier in the batch)    */
#define CB_PUT_FAILED 2  /* no space in any tier                            */

/* ---- get result code per block (low 4 bits = tier the block came from) - */
#define CB_FOUND_MISS 0
#define CB_FOUND_LOCAL_HBM 1
#define CB_FOUND_LOCAL_DRAM 2
#define CB_FOUND_REMOTE_HBM 3
#define CB_FOUND_REMOTE_DRAM 4
#define CB_FOUND_NOT_COPIED 0x80 /* found, but out_cap < size: nothing written */

typedef struct cb_store cb_store;

/* Mirrors DistributedConfig (include/cascade_distributed.hpp:186-213) and
 * CascadeConfig (include/cascade.hpp:47-82) fields that apply to this path. */
typedef struct cb_config {
  uint64_t gpu_capacity_bytes;  /* HBM slab pool (gpu_capacity_per_device)  */
  uint64_t dram_capacity_bytes; /* pinned DRAM arena (dram_capacity); 0=none */
  int32_t device;               /* CUDA device ordinal                      */
  int32_t dedup_enabled;        /* dedup_enabled                            */
  int32_t semantic_eviction;    /* prefix-protected eviction                */
  int32_t promote_on_hit;       /* move DRAM-tier hits back to HBM          */
  int32_t index_log2;           /* initial device index slots = 2^index_log2 */
  int32_t copy_engine;          /* 0 auto, 1 TMA bulk, 2 vector LSU         */
  uint64_t staging_bytes;       /* device staging for host-memory callers   */
  int32_t profile;              /* 1: time each kernel with CUDA events     */
  int32_t hash_lanes;           /* reserved: the SHA-256 kernel always runs
                                   32 chains per warp; accepted, ignored   */
  uint64_t replica_bytes;       /* DHT: HBM for replicas of hot remote blocks */
  int32_t locality_aware;       /* DHT: replicate hot remote blocks locally */
  uint32_t promotion_threshold; /* accesses before a block may be replicated */
  int32_t kv_compression;       /* kv_compression: DRAM-tier copies of blocks
                                   >= 64 B in the INT8 KVCompressor format
                                   (src/cascade_core.cpp:908-967); a read of
                                   such a block returns (size/2)*2 bytes    */
  int32_t prefix_replication;   /* DHT: cb_sync_metadata copies every prefix
                                   block into each rank's local HBM
                                   (broadcast_prefix_data)                   */
  uint64_t collective_timeout_ms; /* DHT: a collective that does not finish in
                                   time aborts the communicator and fails
                                   with CB_ERR_TIMEOUT (0 = 600 s)          */
  int32_t promotion_rule;       /* which DRAM-tier get hits promote_on_hit
                                   moves back to HBM: CB_PROMOTE_*          */
  int32_t reserved32;
  uint64_t pipeline_blocks;     /* cb_put_batch_async: blocks whose SHA-256
                                   runs at once (0 = 65536) */
  int32_t hash_sms;             /* SMs the pipelined puts' SHA-256 launches
                                   may occupy (a green context; the rest stay
                                   free for collectives and copies): 0 = all
                                   on one GPU, all but 8 on a DHT member    */
  int32_t reserved32b;
} cb_config;

/* cb_config.promotion_rule. CB_PROMOTE_EVERY_HIT: every DRAM-tier hit of a
 * get (CascadeStore::get -> promote_to_gpu, src/cascade_core.cpp:1303-1307).
 * CB_PROMOTE_LOCALITY: DistributedStore::get's rule
 * (src/distributed_backend.cpp:721-724, :1224-1265): only with
 * locality_aware, after >= promotion_threshold accesses and an EMA (window
 * 8, alpha 0.3) of the block's remote-access rate above 0.5. Every access a
 * rank makes to a block in its own DRAM tier is local, so under this rule a
 * DRAM hit is never promoted (the reference's 1-rank DistributedStore never
 * promotes either). Zero-copy views (cb_get_views) promote whenever
 * promote_on_hit is set: a view must alias HBM. */
#define CB_PROMOTE_EVERY_HIT 0
#define CB_PROMOTE_LOCALITY 1

/* Mirrors DistributedStore::Stats (include/cascade_distributed.hpp:386-409). */
typedef struct cb_stats {
  uint64_t local_gpu_used, local_dram_used;
  uint64_t cluster_gpu_used, cluster_dram_used;
  uint64_t local_gpu_hits, local_dram_hits;
  uint64_t remote_gpu_hits, remote_dram_hits;
  uint64_t lustre_hits, misses;
  uint64_t dedup_hits, dedup_bytes_saved;
  uint64_t gpu_evictions, dram_evictions;
  uint64_t prefix_blocks_protected, promotions_to_local;
  uint64_t compression_savings;
  uint64_t total_blocks, prefix_blocks;
  /* B200 additions */
  uint64_t evicted_bytes, promoted_bytes, dropped_blocks;
  uint64_t kernel_launches; /* kernels this store launched                 */
  /* per-kernel device time (cb_config.profile = 1): ns, bytes, launches     */
  uint64_t sha_ns, sha_bytes, sha_launches;
  uint64_t scatter_ns, scatter_bytes, scatter_launches;
  uint64_t gather_ns, gather_bytes, gather_launches;
  uint64_t tier_ns, tier_bytes, tier_launches;
  /* DHT payload bytes this rank read from / wrote to peers' pools (NVLink) */
  uint64_t peer_bytes_read, peer_bytes_written;
  /* DHT: prefix blocks of other ranks held in this rank's HBM (replicated by
   * cb_sync_metadata)                                                       */
  uint64_t prefix_replicated_blocks;
  /* DHT collective steps (cb_config.profile = 1): CUDA-event time on the
   * store's stream of each count all-gather, key/reply all-to-all and put
   * barrier (waiting for the slowest peer included), payload bytes this rank
   * sent in them, and their number                                          */
  uint64_t coll_ns, coll_bytes, coll_calls;
} cb_stats;

/* Mirrors BlockLocation (include/cascade_distributed.hpp:62-80). */
typedef struct cb_location {
  int32_t node_id; /* owner rank                                            */
  int32_t gpu_id;  /* device ordinal, -1 when the block is in the DRAM tier */
  uint64_t offset; /* byte offset in the owner's HBM pool or DRAM arena     */
  uint64_t size;
  int32_t is_gpu;
  int32_t is_prefix;
} cb_location;

/* Fills defaults (replaces the struct initialisers of DistributedConfig). */
void cb_config_init(cb_config *cfg);

/* Replaces DistributedStore::DistributedStore
 * (src/distributed_backend.cpp:521-593) for one GPU of one rank. */
int cb_create(const cb_config *cfg, cb_store **out);

/* Replaces DistributedStore::~DistributedStore (src/distributed_backend.cpp:595). */
int cb_destroy(cb_store *s);

/* Message of the last failed call on this store (or of cb_create when s is
 * NULL). The string stays valid until the same thread calls cb_last_error
 * again. Replaces the CUDA_CHECK fprintf of src/gpu_backend.cu:43-51. */
const char *cb_last_error(const cb_store *s);

/* Zero-copy get: addrs_out[i] = device address of block i inside this
 * store's HBM pool, sizes_out[i] its size, found_out[i] a CB_FOUND_* code.
 * No copy and, for HBM hits, no kernel: the addresses come from the host
 * metadata. A DRAM-tier block is first promoted to HBM when promote_on_hit
 * is set (otherwise, or without HBM room, it is reported
 * CB_FOUND_LOCAL_DRAM | CB_FOUND_NOT_COPIED with address 0). Each returned
 * address stays valid — the block is neither evicted nor moved — until
 * cb_release_views is called for that key (one release per view). Views are
 * read-only by contract (a block is its content hash). Not available on a
 * DHT member. The caller-side step after DistributedStore::get_batch
 * (src/distributed_backend.cpp:844-870), without its copy. */
int cb_get_views(cb_store *s, const uint8_t *keys, int32_t n, uint64_t *addrs_out, uint64_t *sizes_out,
                 uint8_t *found_out, void *stream);

/* Releases one view of each key (CB_ERR_ARG if a key has none). */
int cb_release_views(cb_store *s, const uint8_t *keys, int32_t n);

/* Batched INT8 KV compression of n device blocks (srcs[i], sizes[i] >= 2
 * bytes) into dsts[i] (device memory, 8 + sizes[i]/2 bytes each) in the
 * format [f32 scale][i8 zero_point][3 zero bytes][sizes[i]/2 x i8] — the
 * format of DRAM-tier blocks under kv_compression. Replaces
 * KVCompressor::compress (src/cascade_core.cpp:908-944,
 * include/cascade.hpp:400-403). */
int cb_kv_compress_batch(cb_store *s, const void *const *srcs, const uint64_t *sizes, void *const *dsts,
                         int32_t n, void *stream);

/* Inverse of cb_kv_compress_batch: packed block i (srcs[i], comp_sizes[i]
 * bytes, device memory) -> (orig_sizes[i]/2)*2 bytes at dsts[i]. ok_out[i]
 * (may be NULL) = 0 and nothing written when comp_sizes[i] < 8 +
 * orig_sizes[i]/2. Replaces KVCompressor::decompress
 * (src/cascade_core.cpp:946-967, include/cascade.hpp:405-407). */
int cb_kv_decompress_batch(cb_store *s, const void *const *srcs, const uint64_t *comp_sizes,
                           const uint64_t *orig_sizes, void *const *dsts, int32_t n, uint8_t *ok_out,
                           void *stream);

/* Batched SHA-256 of n blocks on the GPU; digests_out = n*32 host bytes.
 * Replaces n calls of compute_block_id (src/cascade_core.cpp:47-58) /
 * python/bindings.cpp:176-179. */
int cb_hash_batch(cb_store *s, const void *const *ptrs, const uint64_t *sizes, int32_t n,
                  int32_t mem_kind, uint8_t *digests_out, void *stream);

/* Batched put. keys_in = n*16 caller keys (NULL: hash every block on the GPU
 * and use the digests). keys_out = n*16 (may be NULL), status_out = n
 * CB_PUT_* (may be NULL). Dedup is sequential in batch order: a block is a
 * dedup hit iff its key was stored before it.
 * Replaces DistributedStore::put_batch (src/distributed_backend.cpp:813-841)
 * and DistributedStore::put (src/distributed_backend.cpp:601-692). */
int cb_put_batch(cb_store *s, const void *const *ptrs, const uint64_t *sizes,
                 const uint8_t *is_prefix, const uint8_t *keys_in, int32_t n, int32_t mem_kind,
                 uint8_t *keys_out, uint8_t *status_out, void *stream);

/* Batched get into caller buffers outs[i] of out_caps[i] bytes.
 * sizes_out[i] = block size when found; found_out[i] = CB_FOUND_* code.
 * Replaces DistributedStore::get_batch (src/distributed_backend.cpp:844-870)
 * and DistributedStore::get (src/distributed_backend.cpp:698-795). */
int cb_get_batch(cb_store *s, const uint8_t *keys, int32_t n, void *const *outs,
                 const uint64_t *out_caps, int32_t mem_kind, uint64_t *sizes_out,
                 uint8_t *found_out, void *stream);

/* found_out[i] = 1 when key i is stored in any tier.
 * Replaces DistributedStore::contains (src/distributed_backend.cpp:797-802). */
int cb_contains_batch(cb_store *s, const uint8_t *keys, int32_t n, uint8_t *found_out);

/* Replaces DistributedStore::locate (src/distributed_backend.cpp:804-806). */
int cb_locate(cb_store *s, const uint8_t *key, cb_location *out, int32_t *found);

/* Demote least-recently-used HBM blocks (prefix blocks last) to the DRAM
 * tier until at least `bytes` have left HBM; *evicted_bytes = bytes moved.
 * Replaces DistributedStore::evict_gpu_to_dram
 * (src/distributed_backend.cpp:876-941, GPUBackend::evict_for_space
 * src/gpu_backend.cu:514-537). */
int cb_evict(cb_store *s, uint64_t bytes, uint64_t *evicted_bytes);

/* Replaces DistributedStore::get_stats (src/distributed_backend.cpp:1384-1427). */
int cb_get_stats(cb_store *s, cb_stats *out);

/* Replaces DistributedStore::clear (src/distributed_backend.cpp:1452-1477). */
int cb_clear(cb_store *s);

/* Waits for all work of the store. Replaces GPUBackend::sync_all
 * (src/gpu_backend.cu:556-562). */
int cb_sync(cb_store *s);

/* ---- multi-GPU DHT (replaces DistributedGPUBackend's MPI RMA tier,
 *      src/distributed_backend.cpp:303-514, and the metadata replication of
 *      sync_metadata, :1323-1382) ------------------------------------------ */

/* Failure-path self-tests that fault, trap or hang nothing.
 * CB_SELFTEST_HASH_WAIT: a hash whose input is announced as still arriving
 * but never published; the kernel's bounded poll gives up after ~1 ms and
 * the call returns CB_ERR_TIMEOUT; the store stays usable afterwards.
 * CB_SELFTEST_FAIL_MOVES: arms a host-side failure of the next tier-move
 * plan, before any of its copies is issued (as a failed pinned-arena
 * allocation would). The call that planned the moves returns
 * CB_ERR_NOSPACE; its planned placements are no longer backed by memory,
 * so every later put/get/contains/locate/evict/view call returns
 * CB_ERR_STATE until cb_clear() empties the store. Any failure of a call
 * after its batch was planned puts the store in that state. */
#define CB_SELFTEST_HASH_WAIT 1
#define CB_SELFTEST_FAIL_MOVES 2
/* CB_SELFTEST_GET_ERROR: the next cb_get_batch_async adds one descriptor
 * whose copy kernel reports a device-side error without touching memory;
 * the next settling call (cb_sync, any synchronous data call) returns
 * CB_ERR_DEVICE, and the store stays usable. */
#define CB_SELFTEST_GET_ERROR 3
int cb_selftest(cb_store *s, int32_t which);

/* ---- stream-ordered (pipelined) puts and gets --------------------------- */

/* Pipelined batched put: the GPU form of CascadeStore::put_batch's OpenMP
 * loop over the batch (src/cascade_core.cpp:1358-1373), with the results of
 * DistributedStore::put_batch (src/distributed_backend.cpp:813-841). The
 * call launches the batch's SHA-256 (after prior work on `stream`) and
 * returns at once with *ticket_out; batches are placed (sequential dedup,
 * tier moves, scatter, index insert) strictly in ticket order, so IDs,
 * statuses and dedup counts equal those of the same batches put one by one
 * with cb_put_batch. keys_out / status_out (may be NULL) are written when the
 * batch is placed: at the latest when cb_put_wait covers its ticket, or when
 * any other data call of the store runs; they must stay valid until then,
 * and the blocks must stay unchanged until then. Up to
 * cb_config.pipeline_blocks blocks hash at once. CB_MEM_HOST
 * blocks are placed before the call returns. On a DHT member every rank
 * must submit the same number of batches (n may be 0) and wait on the same
 * tickets: placement there is collective. */
int cb_put_batch_async(cb_store *s, const void *const *ptrs, const uint64_t *sizes,
                       const uint8_t *is_prefix, const uint8_t *keys_in, int32_t n, int32_t mem_kind,
                       uint8_t *keys_out, uint8_t *status_out, uint64_t *ticket_out, void *stream);

/* Places every batch up to `ticket` (0: every batch submitted) and waits for
 * their device work; *placed_out (may be NULL) = highest ticket placed. A
 * device-side error of a placement is returned here and leaves the store
 * refusing data calls until cb_clear. */
int cb_put_wait(cb_store *s, uint64_t ticket, uint64_t *placed_out);

/* Highest ticket placed so far, without waiting. */
int cb_put_placed(cb_store *s, uint64_t *placed_out);

/* Stream-ordered batched get into device buffers outs[i] (out_caps[i]
 * bytes): found_out / sizes_out are final when the call returns; the bytes
 * land in stream order on `stream`. When every requested block is in the
 * HBM tier (or missing) the call builds the gather from the host metadata -
 * no device lookup, no device round trip - and returns without waiting;
 * other batches (DRAM-tier blocks, DHT members) take the synchronous path
 * of cb_get_batch. A device-side error of the gather is returned by the next
 * settling call (cb_sync, cb_put_wait, any synchronous data call). Sees every
 * put submitted before it. Same results as cb_get_batch
 * (DistributedStore::get_batch, src/distributed_backend.cpp:844-870). */
int cb_get_batch_async(cb_store *s, const uint8_t *keys, int32_t n, void *const *outs,
                       const uint64_t *out_caps, uint64_t *sizes_out, uint8_t *found_out, void *stream);

/* Size of the opaque NCCL unique id blob. */
#define CB_UID_BYTES 128

/* Rank 0 creates the unique id; every rank passes the same blob. */
int cb_dht_unique_id(uint8_t uid_out[CB_UID_BYTES]);

/* Joins the DHT: NCCL communicator over `world` ranks, one GPU each; the HBM
 * pools are exported with CUDA IPC and mapped into every peer. Collective. */
int cb_dht_attach(cb_store *s, int32_t rank, int32_t world, const uint8_t uid[CB_UID_BYTES]);

/* Collective barrier over the DHT (ncclAllReduce of one word).
 * Replaces DistributedStore::barrier (src/distributed_backend.cpp:1310-1314). */
int cb_dht_barrier(cb_store *s);

/* Cluster-wide prefix registry and prefix replication. Collective in a DHT:
 * every rank learns every prefix block (cb_stats.prefix_blocks becomes the
 * cluster count) and, with cb_config.prefix_replication, copies each prefix
 * block another rank holds in HBM into its own replica region by peer loads
 * (as space allows; these replicas are never dropped for hot-block
 * replicas), after which gets of prefix blocks are served from local HBM.
 * A 1-GPU store has nothing to exchange and returns CB_OK.
 * Replaces DistributedStore::sync_metadata -> sync_prefix_registry ->
 * broadcast_prefix_data (src/distributed_backend.cpp:958-1217, :1323-1325). */
int cb_sync_metadata(cb_store *s);

/* Rank and world size (1-GPU stores: 0 and 1). */
int cb_rank(const cb_store *s, int32_t *rank, int32_t *world);

/* Writer side of the DHT routing, host-only: owner_out[i] = owner rank of
 * key i (cb_owner_rank), order_out = the batch indices in the order they
 * are sent (grouped by owner rank, batch order inside a group), counts_out
 * [world] = keys per owner. cb_put_batch / cb_get_batch on a DHT member route
 * with this function. Replaces the per-block target choice of
 * DistributedGPUBackend::get_target_node (src/distributed_backend.cpp:
 * 396-398) for a whole batch. */
int cb_dht_route(const uint8_t *keys, int32_t n, int32_t world, int32_t *owner_out, int32_t *order_out,
                 uint32_t *counts_out);

/* Owner side of a DHT put step without a GPU: a planner holds an owner's
 * host policy (HBM pool and DRAM arena capacities, prefix-protected
 * eviction, dedup); cb_dht_plan_put applies n requests (16-byte key, size,
 * prefix flag) received in (source rank, batch index) order with the
 * sequential dedup rule of DistributedStore::put
 * (src/distributed_backend.cpp:604-608) and returns status_out[i]
 * (CB_PUT_*) and loc_out[i] (pool offset of a stored block, bit 63 set for
 * the DRAM tier; 0 otherwise). It is the function a DHT owner runs inside
 * cb_put_batch; tier moves it plans are not executed here. */
typedef struct cb_planner cb_planner;
int cb_planner_create(uint64_t gpu_capacity_bytes, uint64_t dram_capacity_bytes, int32_t semantic_eviction,
                      int32_t dedup_enabled, cb_planner **out);
int cb_planner_destroy(cb_planner *p);
int cb_dht_plan_put(cb_planner *p, const uint8_t *keys, const uint64_t *sizes, const uint8_t *prefix,
                    int32_t n, uint8_t *status_out, uint64_t *loc_out);

/* Owner rank of a key in a `world`-rank DHT: the first 8 key bytes read as a
 * big-endian integer, modulo world. Host-only, no GPU needed. Replaces
 * DistributedGPUBackend::get_target_node (src/distributed_backend.cpp:396-398),
 * whose std::hash placement is not stable across builds. */
int32_t cb_owner_rank(const uint8_t *key, int32_t world);

/* ---- allocation-free hashing -------------------------------------------- */

/* Most blocks one cb_hash_batch_noalloc call accepts (its fixed scratch). */
#define CB_NOALLOC_MAX_BLOCKS 4096

/* Batched SHA-256 that allocates nothing; no counterpart in the reference.
 * For callers that may not allocate GPU memory while they run (an engine that
 * reserved nearly all HBM for its own pool and forbids cudaMalloc during
 * serving, or code inside an allocator callback): it needs no cb_store.
 * Blocks (ptrs[i], sizes[i]) are device memory on `device`; digests_out is a
 * caller-owned, 16-byte aligned device buffer of n*32 bytes. n above
 * CB_NOALLOC_MAX_BLOCKS is rejected with CB_ERR_ARG. Its scratch is one
 * static device array of ~66 KB that every GPU loading the library keeps
 * until exit; all calls share it, so calls that overlap on the GPU race.
 * The first call on a device (an empty call, n = 0, does only this) looks up
 * that array's address and, under lazy module loading, loads this entry
 * point's GPU code and the array's backing: the only device memory it ever
 * causes to be allocated, so make that first call at start-up. Later calls
 * allocate nothing. The looked-up address is kept for the process lifetime:
 * do not call this on a device after cudaDeviceReset of that device. A call
 * on a stream that is being captured is refused with CB_ERR_ARG before
 * anything is enqueued (each call copies from pageable host memory and waits
 * for its own completion). Results are final when the call returns; errors
 * are reported by cb_last_error(NULL). */
int cb_hash_batch_noalloc(int32_t device, const void *const *ptrs, const uint64_t *sizes, int32_t n,
                          uint8_t *digests_out, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* CASCADE_B200_H */
