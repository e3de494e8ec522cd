// ORACLE — test infrastructure only (checker and timed CPU baseline).
//
// A pybind11 shim over the reference's OWN compiled CPU path
// (cascade_Code/cpp/src/cascade_core.cpp, built from its sources in place by
// oracle/Makefile). It exposes what the reference's bindings.cpp does not:
//   * compute_block_ids: compute_block_id (cascade_core.cpp:47-58) over a batch
//     in an OpenMP loop — the reference drivers' CPU hashing pass;
//   * CascadeStore.put_batch / get_batch (cascade_core.cpp:1358-1390), the
//     reference's parallel OpenMP batch API, which bindings.cpp:68-85 leaves
//     unbound;
//   * kv_compress / kv_decompress: KVCompressor::compress / decompress
//     (cascade_core.cpp:908-967), the INT8 format of the DRAM tier when
//     kv_compression is on. The header's 3 padding bytes are indeterminate in
//     the reference; the shim zeroes the CompressionMeta it passes so they
//     come out as zero.
// The store is configured for the CPU path only: use_gpu = false, SHM tier
// (ShmBackend on /dev/shm, cascade_core.cpp:269-497), no Lustre, no prefetch.
#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <omp.h>

#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "cascade.hpp"

namespace py = pybind11;
using cascade::CascadeStore;

namespace {

using u8arr = py::array_t<uint8_t, py::array::c_style>;
using u64arr = py::array_t<uint64_t, py::array::c_style | py::array::forcecast>;

std::unique_ptr<CascadeStore> make_store(size_t shm_capacity, const std::string &shm_path,
                                         bool dedup, bool semantic) {
  cascade::CascadeConfig c;
  c.use_gpu = false;
  c.gpu_capacity_bytes = 0;
  c.shm_capacity_bytes = shm_capacity;
  c.shm_path = shm_path;
  c.lustre_path = "";
  c.prefetch_enabled = false;
  c.dedup_enabled = dedup;
  c.semantic_eviction = semantic;
  c.promotion_enabled = false;
  c.aggregated_lustre = false;
  return std::make_unique<CascadeStore>(c);
}

}  // namespace

PYBIND11_MODULE(cascade_ref, m) {
  m.doc() = "Reference Cascade CPU path (compiled from the reference sources) - oracle only";

  m.def("compute_block_id", [](u8arr a) {
    auto b = a.request();
    return cascade::compute_block_id(static_cast<const uint8_t *>(b.ptr), b.size);
  });

  m.def(
      "compute_block_ids",
      [](u8arr packed, u64arr offsets, u64arr sizes, int threads) {
        auto pb = packed.request();
        const uint8_t *base = static_cast<const uint8_t *>(pb.ptr);
        const uint64_t *off = offsets.data();
        const uint64_t *sz = sizes.data();
        const int64_t n = offsets.size();
        std::vector<std::string> out(n);
        {
          py::gil_scoped_release rel;
          if (threads > 0) omp_set_num_threads(threads);
#pragma omp parallel for schedule(dynamic)
          for (int64_t i = 0; i < n; ++i) out[i] = cascade::compute_block_id(base + off[i], sz[i]);
        }
        return out;
      },
      py::arg("packed"), py::arg("offsets"), py::arg("sizes"), py::arg("threads") = 0);

  m.def("max_threads", []() { return omp_get_max_threads(); });

  m.def("kv_compress", [](u8arr a) {
    auto b = a.request();
    cascade::CompressionMeta meta;
    std::memset(&meta, 0, sizeof(meta));
    std::vector<uint8_t> c = cascade::KVCompressor::compress(static_cast<const uint8_t *>(b.ptr), b.size, meta);
    return py::bytes(reinterpret_cast<const char *>(c.data()), c.size());
  });

  m.def("kv_decompress", [](u8arr comp, size_t orig_size) {
    auto b = comp.request();
    const uint8_t *p = static_cast<const uint8_t *>(b.ptr);
    cascade::CompressionMeta meta;
    std::memset(&meta, 0, sizeof(meta));
    std::memcpy(&meta, p, sizeof(meta));
    std::string out((orig_size / 2) * 2, '\0');
    const bool ok = cascade::KVCompressor::decompress(p, b.size, meta, reinterpret_cast<uint8_t *>(&out[0]),
                                                      orig_size);
    return py::make_tuple(ok, py::bytes(out));
  });

  py::class_<CascadeStore, std::unique_ptr<CascadeStore>>(m, "CascadeStore")
      .def(py::init(&make_store), py::arg("shm_capacity"), py::arg("shm_path"),
           py::arg("dedup") = true, py::arg("semantic_eviction") = true)
      .def(
          "put",
          [](CascadeStore &s, const std::string &id, u8arr data, bool is_prefix) {
            auto b = data.request();
            return s.put(id, static_cast<const uint8_t *>(b.ptr), b.size, is_prefix);
          },
          py::arg("block_id"), py::arg("data"), py::arg("is_prefix") = false)
      .def("get",
           [](CascadeStore &s, const std::string &id, u8arr out) {
             auto b = out.request();
             size_t size = 0;
             bool found = s.get(id, static_cast<uint8_t *>(b.ptr), &size);
             return py::make_tuple(found, size);
           })
      .def("contains", &CascadeStore::contains)
      .def(
          "put_batch",
          [](CascadeStore &s, const std::vector<std::string> &ids, u8arr packed, u64arr offsets,
             u64arr sizes) {
            auto pb = packed.request();
            const uint8_t *base = static_cast<const uint8_t *>(pb.ptr);
            const size_t n = ids.size();
            std::vector<const uint8_t *> ptrs(n);
            std::vector<size_t> sz(n);
            for (size_t i = 0; i < n; ++i) {
              ptrs[i] = base + offsets.data()[i];
              sz[i] = sizes.data()[i];
            }
            py::gil_scoped_release rel;
            return s.put_batch(ids, ptrs, sz);
          })
      .def("get_batch",
           [](CascadeStore &s, const std::vector<std::string> &ids, u8arr out_packed,
              u64arr offsets) {
             auto pb = out_packed.request();
             uint8_t *base = static_cast<uint8_t *>(pb.ptr);
             const size_t n = ids.size();
             std::vector<uint8_t *> outs(n);
             std::vector<size_t> sizes(n, 0);
             for (size_t i = 0; i < n; ++i) outs[i] = base + offsets.data()[i];
             size_t found;
             {
               py::gil_scoped_release rel;
               found = s.get_batch(ids, outs, sizes);
             }
             return py::make_tuple(found, sizes);
           })
      .def("stats",
           [](const CascadeStore &s) {
             auto st = s.get_stats();
             py::dict d;
             d["shm_used"] = st.shm_used;
             d["shm_hits"] = st.shm_hits;
             d["misses"] = st.misses;
             d["dedup_hits"] = st.dedup_hits;
             d["shm_evictions"] = st.shm_evictions;
             d["shm_puts"] = st.shm_puts;
             return d;
           })
      .def("clear", &CascadeStore::clear);
}
