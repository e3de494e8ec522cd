// Allocation-free block hashing: cb_hash_batch_noalloc.
//
// Some callers of this library must not allocate GPU memory at the moment
// they hash blocks: a serving engine that reserved nearly all of HBM for its
// own KV-cache pool at start-up and forbids further cudaMalloc while it
// serves (an allocation would fail, or carve into the engine's reservation),
// or code running in an allocator or memory-pressure callback, which must
// not re-enter the allocator. cb_hash_batch needs a store, and a store
// allocates its pool, index and scratch when it is created.
//
// This entry point needs no store. Its only scratch (the per-block job
// descriptors and the kernel's error word) lives in the file-scope device
// array below, which every GPU that loads the library holds until the
// process exits. The caller passes the blocks (device memory) and a device
// output buffer for the digests. The call makes no cudaMalloc / cudaFree /
// allocating library call.
//
// With lazy module loading (the CUDA 12 default) the GPU code of this file
// and of the SHA-256 kernel, and the backing of the array, are loaded on
// first use. The per-device set-up below forces that loading, so it happens
// in the first call on a device (an empty call, n = 0, does only the
// set-up); every later call allocates nothing at all.
#include <stdint.h>
#include <string.h>

#include <mutex>
#include <string>

#include "kernels.cuh"

namespace cb {

// Upper bound on blocks per call; the scratch array is sized for it.
constexpr int kNoAllocMaxBlocks = CB_NOALLOC_MAX_BLOCKS;
// Layout: [HashJob x kNoAllocMaxBlocks][error word, padded to 256 B].
constexpr size_t kNoAllocJobBytes = sizeof(HashJob) * kNoAllocMaxBlocks;
constexpr size_t kNoAllocBytes = kNoAllocJobBytes + 256;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

extern thread_local std::string g_create_error;  // store.cu: message of store-less calls

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_setup_mu;
void *g_scratch_addr[kMaxDevices] = {nullptr};  // device address of the array, per device

int noalloc_fail(int code, const char *msg, cudaError_t e = cudaSuccess) {
  g_create_error = msg;
  if (e != cudaSuccess) {
    g_create_error += ": ";
    g_create_error += cudaGetErrorString(e);
  }
  return code;
}

// The host-side name of g_noalloc_scratch is only a stand-in: its device
// address differs per device and must be looked up with that device current.
// Done once per device, on the first call that targets it, together with the
// loading of the SHA-256 kernel, so that no later call loads anything. The
// address is kept for the life of the process: a cudaDeviceReset of that
// device invalidates it.
int scratch_for(int device, unsigned char **out) {
  std::lock_guard<std::mutex> g(g_setup_mu);
  if (!g_scratch_addr[device]) {
    void *p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) return noalloc_fail(CB_ERR_CUDA, "cudaGetSymbolAddress(noalloc scratch)", e);
    if ((e = prepare_sha256_kernel()) != cudaSuccess)
      return noalloc_fail(CB_ERR_CUDA, "cb_hash_batch_noalloc: loading the SHA-256 kernel", e);
    g_scratch_addr[device] = p;
  }
  *out = static_cast<unsigned char *>(g_scratch_addr[device]);
  return CB_OK;
}

}  // namespace

}  // namespace cb

extern "C" int cb_hash_batch_noalloc(int32_t device, const void *const *ptrs, const uint64_t *sizes,
                                     int32_t n, uint8_t *digests_out, void *stream) {
  using namespace cb;
  if (n < 0 || (n > 0 && (!ptrs || !sizes || !digests_out)))
    return noalloc_fail(CB_ERR_ARG, "cb_hash_batch_noalloc: bad arguments");
  if (n > kNoAllocMaxBlocks)
    return noalloc_fail(CB_ERR_ARG,
                        "cb_hash_batch_noalloc: more blocks than CB_NOALLOC_MAX_BLOCKS (4096) in one call");
  if (device < 0 || device >= kMaxDevices) return noalloc_fail(CB_ERR_ARG, "cb_hash_batch_noalloc: bad device");
  if (reinterpret_cast<uintptr_t>(digests_out) & 15)
    return noalloc_fail(CB_ERR_ARG, "cb_hash_batch_noalloc: digests_out must be 16-byte aligned");
  for (int i = 0; i < n; ++i)
    if (sizes[i] > kSizeMask) return noalloc_fail(CB_ERR_ARG, "cb_hash_batch_noalloc: block too large");
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  int prev = -1;
  cudaError_t e = cudaGetDevice(&prev);
  if (e != cudaSuccess) return noalloc_fail(CB_ERR_CUDA, "cudaGetDevice", e);
  if (prev != device && (e = cudaSetDevice(device)) != cudaSuccess)
    return noalloc_fail(CB_ERR_CUDA, "cudaSetDevice", e);

  int rc = CB_OK;
  unsigned char *scratch = nullptr;
  unsigned host_err = 0;
  do {
    // Each call copies its descriptors from pageable host memory and waits
    // for its own completion; neither is allowed on a stream under capture,
    // so refuse before anything is enqueued (the caller's capture stays
    // valid).
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    if ((e = cudaStreamIsCapturing(st, &cap)) != cudaSuccess) {
      rc = noalloc_fail(CB_ERR_CUDA, "cb_hash_batch_noalloc: cudaStreamIsCapturing", e);
      break;
    }
    if (cap != cudaStreamCaptureStatusNone) {
      rc = noalloc_fail(CB_ERR_ARG, "cb_hash_batch_noalloc: the stream is being captured (not supported)");
      break;
    }
    if ((rc = scratch_for(device, &scratch)) != CB_OK || n == 0) break;
    HashJob *jobs = reinterpret_cast<HashJob *>(scratch);
    unsigned *err = reinterpret_cast<unsigned *>(scratch + kNoAllocJobBytes);
    // Job descriptors: the caller's two host arrays are interleaved into the
    // scratch by two strided copies (no host or device buffer is made).
    if ((e = cudaMemcpy2DAsync(&jobs[0].ptr, sizeof(HashJob), ptrs, sizeof(void *), sizeof(uint64_t), n,
                               cudaMemcpyHostToDevice, st)) != cudaSuccess ||
        (e = cudaMemcpy2DAsync(&jobs[0].size, sizeof(HashJob), sizes, sizeof(uint64_t), sizeof(uint64_t), n,
                               cudaMemcpyHostToDevice, st)) != cudaSuccess) {
      rc = noalloc_fail(CB_ERR_CUDA, "cb_hash_batch_noalloc: descriptor copy", e);
      break;
    }
    // The array keeps the previous call's contents: the error word must
    // start at zero.
    if ((e = cudaMemsetAsync(err, 0, sizeof(unsigned), st)) != cudaSuccess) {
      rc = noalloc_fail(CB_ERR_CUDA, "cb_hash_batch_noalloc: clear error word", e);
      break;
    }
    if ((e = launch_sha256_batch(jobs, n, reinterpret_cast<uint32_t *>(digests_out), 32, err, st)) !=
        cudaSuccess) {
      rc = noalloc_fail(CB_ERR_CUDA, "cb_hash_batch_noalloc: launch", e);
      break;
    }
    if ((e = cudaMemcpyAsync(&host_err, err, sizeof(unsigned), cudaMemcpyDeviceToHost, st)) != cudaSuccess ||
        (e = cudaStreamSynchronize(st)) != cudaSuccess) {
      rc = noalloc_fail(CB_ERR_CUDA, "cb_hash_batch_noalloc: completion", e);
      break;
    }
    if (host_err & kErrTimeout) rc = noalloc_fail(CB_ERR_TIMEOUT, "cb_hash_batch_noalloc: device wait timed out");
    else if (host_err) rc = noalloc_fail(CB_ERR_DEVICE, "cb_hash_batch_noalloc: device-side check failed");
  } while (false);

  if (prev != device) cudaSetDevice(prev);
  return rc;
}
