// Launchers of the sm_100a kernels of the block data path.
#pragma once

#include "common.cuh"

namespace cb {

struct HashJob {
  uint64_t ptr;   // device (or mapped host) address of the block
  uint64_t size;  // bytes
};

// Blocks that are still being copied in: segment k (seg_chunks 64-byte
// chunks of every block) may be read once *counter > k. data_chunks =
// ceil(block size / 64) (uniform block size).
struct HashProgress {
  const unsigned *counter;
  uint32_t seg_chunks;
  uint64_t data_chunks;
  uint32_t wait_iters = 0;  // polls of the counter before giving up (0 = default)
};

// sha256.cu — digests: n * 8 words holding the 32 digest bytes in order.
// progress may be null. many_chains = false: one CTA (producer + consumer
// warp) per 32 blocks, the fastest chains when few run; true: the fused
// kernel (one warp per 32 blocks, half the issue resources per chain), the
// higher throughput when many chains run at once (pipelined puts).
cudaError_t launch_sha256_batch(const HashJob *d_jobs, int n, uint32_t *d_digests, int lanes,
                                unsigned *d_err, cudaStream_t stream, const HashProgress *progress = nullptr,
                                bool many_chains = false);
// Loads the SHA-256 kernel's module on the current device now (with lazy
// module loading it would otherwise load, and allocate, at its first launch).
cudaError_t prepare_sha256_kernel();

// copy.cu — batched copies. Descriptor i covers units
// [unit_start[i], unit_start[i+1]) of kCopyUnit bytes each; a unit past the
// descriptor's size is skipped. engine: 1 = TMA bulk (device memory only),
// 2 = vector LSU. Descriptors with flags bit 0 (host memory) always take the
// LSU path.
// lsu_ctas_per_sm bounds the LSU engine's grid (a host-link-bound move that
// runs beside other kernels leaves them room on every SM).
cudaError_t launch_batch_copy(const CopyDesc *d_desc, const uint32_t *d_unit_start, int n,
                              uint32_t total_units, int engine, unsigned *d_err, int num_sms,
                              cudaStream_t stream, int lsu_ctas_per_sm = 8);

// kvquant.cu — INT8 packing (KVCompressor::compress format) of blocks:
// descriptor i packs the d.size-byte block at d.src (device memory, d.size
// >= 2) into packed_size(d.size) bytes at d.dst (device or mapped pinned host
// memory); units as for launch_batch_copy over the source bytes. d_mm holds
// n (min, max) int pairs the caller initialised to (INT_MAX, INT_MIN). Two
// kernels (min/max, then pack). Unpacking is launch_batch_copy with
// kCopyUnpack descriptors.
cudaError_t launch_kv_pack(const CopyDesc *d_desc, const uint32_t *d_unit_start, int n, uint32_t total_units,
                           int *d_mm, int num_sms, cudaStream_t stream, int ctas_per_sm = 8);

// index.cu — device index mutations and lookups.
cudaError_t launch_index_insert(Slot *table, uint64_t mask, const IndexRec *recs, int n,
                                unsigned *d_err, cudaStream_t stream);
cudaError_t launch_index_update(Slot *table, uint64_t mask, const IndexRec *recs, int n,
                                unsigned *d_err, cudaStream_t stream);
cudaError_t launch_index_erase(Slot *table, uint64_t mask, const IndexRec *recs, int n,
                               unsigned *d_err, cudaStream_t stream);

// Lookup for gets: for each key resolves the source address in the HBM pool
// (pool_base) or DRAM arena (dram_base), checks it against the arena sizes
// and out_caps, and fills desc (size 0 when nothing is to be copied) and res.
struct LookupArgs {
  const Slot *table;
  uint64_t mask;
  const Key *keys;
  const uint64_t *outs;
  const uint64_t *caps;
  const uint32_t *unit_start;  // copy units the host reserved per request
  int n;
  uint64_t pool_base, pool_bytes;
  uint64_t dram_base, dram_bytes;
  uint32_t code_hbm, code_dram;  // CB_FOUND_* codes to report per tier
  CopyDesc *desc;
  GetResult *res;
  unsigned *err;
};
cudaError_t launch_index_lookup(const LookupArgs &a, cudaStream_t stream);

// DHT owner lookup: reps[2i] = location word, reps[2i+1] = meta word
// (0 when the key is absent).
cudaError_t launch_index_serve(const Slot *table, uint64_t mask, const Key *keys, int n, uint64_t *reps,
                               cudaStream_t stream);

}  // namespace cb
