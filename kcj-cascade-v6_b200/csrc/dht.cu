// Multi-GPU hash-sharded DHT (placeholder until the NCCL path lands).
#include "store.hpp"

namespace cb {

struct DhtState {};

int Store::dht_attach(int, int, const uint8_t *) {
  return fail(CB_ERR_STATE, "multi-GPU DHT not available in this build");
}
void Store::dht_detach() {}
int Store::dht_barrier() { return CB_OK; }
int Store::dht_put(const void *const *, const uint64_t *, const uint8_t *, const uint8_t *, int, int,
                   uint8_t *, uint8_t *, cudaStream_t) {
  return fail(CB_ERR_STATE, "multi-GPU DHT not available in this build");
}
int Store::dht_get(const uint8_t *, int, void *const *, const uint64_t *, int, uint64_t *, uint8_t *,
                   cudaStream_t) {
  return fail(CB_ERR_STATE, "multi-GPU DHT not available in this build");
}
int Store::dht_contains(const uint8_t *, int, uint8_t *, cudaStream_t) {
  return fail(CB_ERR_STATE, "multi-GPU DHT not available in this build");
}
int Store::dht_cluster_usage(cb_stats *) { return CB_OK; }

}  // namespace cb

extern "C" {
int cb_dht_unique_id(uint8_t *) { return CB_ERR_STATE; }
int cb_dht_attach(cb_store *, int32_t, int32_t, const uint8_t *) { return CB_ERR_STATE; }
int cb_dht_barrier(cb_store *) { return CB_OK; }
}
