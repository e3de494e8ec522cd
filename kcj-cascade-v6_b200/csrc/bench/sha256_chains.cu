// Throughput of the two SHA-256 kernels against the number of chains (blocks)
// in flight: single launches of n blocks, and k concurrent 1024-block
// launches on their own streams (the pipelined put's launch pattern).
// Blocks are 917,504 bytes (one Qwen2.5-7B KV block); `distinct` source
// blocks (default 4096 = 3.76 GB, far larger than L2) are reused round robin
// beyond that.
//
//   nvcc -gencode arch=compute_100a,code=sm_100a -O3 -std=c++17 -Iinclude \
//        -Ikcj-cascade-v6_b200/csrc -o sha256_chains kcj-cascade-v6_b200/csrc/bench/sha256_chains.cu
//   ./sha256_chains [max_blocks = 65536] [distinct = 4096] [shuffled = 0]
//
// Prints whether both kernels give equal digests, then GB/s (block bytes /
// CUDA-event time) per configuration. Device memory: 917,504 B per distinct
// block, 32 B of digest and 16 B of job per block.
#include <cstdio>
#include <cstdlib>
#include <vector>

#include "../sha256.cu"

namespace chains_bench {

using cb::HashJob;

__global__ void fill_blocks(uint32_t *p, uint64_t words) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < words; i += (uint64_t)gridDim.x * blockDim.x)
    p[i] = (uint32_t)(i * 2654435761ull) ^ (uint32_t)(i >> 7);
}

bool launch(bool fused, const HashJob *jobs, int n, uint32_t *dig, unsigned *err, cudaStream_t s) {
  return cb::launch_sha256_batch(jobs, n, dig, 32, err, s, nullptr, fused) == cudaSuccess;
}

}  // namespace chains_bench

using namespace chains_bench;

int main(int argc, char **argv) {
  const int nmax = argc > 1 ? atoi(argv[1]) : 65536;
  const int nu = argc > 2 ? atoi(argv[2]) : 4096;  // distinct source blocks
  const int shuffled = argc > 3 ? atoi(argv[3]) : 0;  // 1: chains read blocks in a shuffled order
  if (nmax < 2048 || nmax > (1 << 20) || nu < 1 || nu > 65536) {
    fprintf(stderr, "max_blocks must be in [2048, 1048576], distinct blocks in [1, 65536]\n");
    return 1;
  }
  const uint64_t S = 917504;
  uint8_t *buf = nullptr;
  HashJob *jobs = nullptr;
  uint32_t *dig[2] = {nullptr, nullptr};
  unsigned *err = nullptr;
  if (cudaMalloc(&buf, nu * S) != cudaSuccess || cudaMalloc(&jobs, nmax * sizeof(HashJob)) != cudaSuccess ||
      cudaMalloc(&err, 4) != cudaSuccess || cudaMalloc(&dig[0], nmax * 32ull) != cudaSuccess ||
      cudaMalloc(&dig[1], nmax * 32ull) != cudaSuccess) {
    fprintf(stderr, "cudaMalloc failed\n");
    return 1;
  }
  cudaMemset(err, 0, 4);
  fill_blocks<<<1184, 256>>>(reinterpret_cast<uint32_t *>(buf), nu * S / 4);
  std::vector<HashJob> hj(nmax);
  for (int i = 0; i < nmax; ++i) hj[i] = HashJob{(uint64_t)(uintptr_t)(buf + (uint64_t)(i % nu) * S), S};
  if (shuffled) {  // the i-th chain reads a block at a random place of the buffer
    uint64_t x = 88172645463325252ull;
    for (int i = nmax - 1; i > 0; --i) {
      x ^= x << 13; x ^= x >> 7; x ^= x << 17;
      const int j = (int)(x % (uint64_t)(i + 1));
      const HashJob t = hj[i]; hj[i] = hj[j]; hj[j] = t;
    }
  }
  cudaMemcpy(jobs, hj.data(), nmax * sizeof(HashJob), cudaMemcpyHostToDevice);

  for (int v = 0; v < 2; ++v)
    if (!launch(v == 1, jobs, 2048, dig[v], err, 0)) return 2;
  cudaDeviceSynchronize();
  std::vector<uint32_t> a(2048 * 8), b(2048 * 8);
  cudaMemcpy(a.data(), dig[0], 2048 * 32, cudaMemcpyDeviceToHost);
  cudaMemcpy(b.data(), dig[1], 2048 * 32, cudaMemcpyDeviceToHost);
  printf("digests of both kernels equal: %d\n", a == b ? 1 : 0);

  const char *name[2] = {"sha256_pc_kernel   ", "sha256_fused_kernel"};
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  for (int v = 0; v < 2; ++v)
    for (int n : {1024, 16384, 18944, 32768, 37888, 49152, 65536}) {
      if (n > nmax) continue;
      launch(v == 1, jobs, n, dig[v], err, 0);  // warm-up
      cudaEventRecord(e0);
      launch(v == 1, jobs, n, dig[v], err, 0);
      cudaEventRecord(e1);
      cudaEventSynchronize(e1);
      float ms = 0.f;
      cudaEventElapsedTime(&ms, e0, e1);
      printf("%s one launch of %6d blocks: %7.1f GB/s %7.2f ms\n", name[v], n, n * (double)S / ms / 1e6, ms);
    }
  std::vector<cudaStream_t> st(64);
  std::vector<cudaEvent_t> fin(64);
  for (int j = 0; j < 64; ++j) {
    cudaStreamCreateWithFlags(&st[j], cudaStreamNonBlocking);
    cudaEventCreateWithFlags(&fin[j], cudaEventDisableTiming);
  }
  for (int v = 0; v < 2; ++v)
    for (int k : {16, 32, 48, 64}) {
      if (k * 1024 > nmax) continue;
      cudaDeviceSynchronize();
      cudaEventRecord(e0);
      for (int j = 0; j < k; ++j) {
        cudaStreamWaitEvent(st[j], e0, 0);
        launch(v == 1, jobs + 1024 * j, 1024, dig[v] + 8 * 1024 * j, err, st[j]);
        cudaEventRecord(fin[j], st[j]);
        cudaStreamWaitEvent(0, fin[j], 0);
      }
      cudaEventRecord(e1);
      cudaEventSynchronize(e1);
      float ms = 0.f;
      cudaEventElapsedTime(&ms, e0, e1);
      printf("%s %2d concurrent 1024-block launches: %7.1f GB/s %7.2f ms\n", name[v], k,
             k * 1024 * (double)S / ms / 1e6, ms);
    }
  unsigned he = 0;
  cudaMemcpy(&he, err, 4, cudaMemcpyDeviceToHost);
  const cudaError_t last = cudaGetLastError();
  printf("device error word %u, %s\n", he, cudaGetErrorString(last));
  return (he || last != cudaSuccess || a != b) ? 3 : 0;
}
