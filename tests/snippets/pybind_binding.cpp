// C++ shown to maintainers in INTEGRATION.md: a pybind11 binding of the C
// ABI in place of the reference's DistributedStore / KVCompressor bindings
// (python/bindings.cpp). tests/test_capi.py compiles this file against
// include/cascade_b200.h.
#include <stdexcept>
#include <string>

#include "cascade_b200.h"
#include <pybind11/numpy.h>
namespace py = pybind11;

struct B200Store {
  cb_store* s = nullptr;
  explicit B200Store(uint64_t hbm, uint64_t dram, int device) {
    cb_config c; cb_config_init(&c);
    c.gpu_capacity_bytes = hbm; c.dram_capacity_bytes = dram; c.device = device;
    if (cb_create(&c, &s) != CB_OK) throw std::runtime_error(cb_last_error(nullptr));
  }
  ~B200Store() { cb_destroy(s); }
};

// DistributedStore::put (src/distributed_backend.cpp:601) -> cb_put_batch with n = 1
bool put(B200Store& st, const std::string& id32hex, py::array_t<uint8_t> data, bool is_prefix) {
  auto b = data.request();
  uint8_t key[16];  // 32 lowercase hex chars -> 16 bytes (other IDs: a 16-byte hash, see block_id_to_key)
  for (int i = 0; i < 16; ++i) key[i] = std::stoi(id32hex.substr(2 * i, 2), nullptr, 16);
  const void* ptr = b.ptr; uint64_t size = b.size; uint8_t pf = is_prefix, status = 0;
  int rc = cb_put_batch(st.s, &ptr, &size, &pf, key, 1, CB_MEM_HOST, nullptr, &status, nullptr);
  return rc == CB_OK && status != CB_PUT_FAILED;
}

// KVCompressor::compress (src/cascade_core.cpp:908) on device buffers: packs
// size bytes at dev_src into dev_dst and returns the packed size, 8 + size/2
uint64_t compress(B200Store& st, uint64_t dev_src, uint64_t size, uint64_t dev_dst) {
  const void* src = (const void*)dev_src; void* dst = (void*)dev_dst;
  if (cb_kv_compress_batch(st.s, &src, &size, &dst, 1, nullptr) != CB_OK)
    throw std::runtime_error(cb_last_error(st.s));
  return 8 + size / 2;
}
