// Batched variable-size copies: the scatter (caller block -> pool slot) of
// put, the gather (pool slot -> caller buffer) of get, and the HBM<->pinned
// DRAM tier moves. They replace the per-block cudaMemcpy[Async] calls of the
// reference (src/gpu_backend.cu:327-343 put, :390-425 read_block_to_host,
// :469/:502 eviction reads) with one launch per batch.
//
// Work is cut into kCopyUnit (64 KiB) units; descriptor i owns units
// [unit_start[i], unit_start[i+1]). Each CTA takes a contiguous range of
// units, so a block is streamed by few CTAs front to back.
//
// Two engines:
//  * TMA bulk (engine 1): one CTA per SM, one elected lane drives a
//    kStages-deep pipeline of cp.async.bulk global->shared loads (mbarrier
//    completion) and cp.async.bulk shared->global stores (bulk groups). No
//    multicast anywhere: every byte is read by exactly one CTA.
//  * LSU (engine 2): 256-thread CTAs moving 16-byte vectors, 4 in flight per
//    thread, with streaming cache hints.
// Units touching host memory (tier moves), units whose addresses are not
// 16-byte aligned, and the sub-16-byte tail of a unit always use the LSU path.
// Descriptors flagged kCopyUnpack (reads of INT8-packed DRAM-tier blocks)
// are unpacked by the same LSU threads (kvquant.cuh).
#include "kernels.cuh"
#include "kvquant.cuh"
#include "units.cuh"

namespace cb {

namespace {

constexpr int kLsuThreads = 256;
constexpr int kLsuCtasPerSm = 8;
constexpr int kTmaStages = 6;
constexpr uint32_t kTmaStageBytes = 32 * 1024;
constexpr uint64_t kWaitLimit = 1ull << 24;  // try_wait rounds before giving up

CB_D uint4 ld_dev16(const uint4 *p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}
CB_D void st_dev16(uint4 *p, const uint4 &v) {
  asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}
CB_D uint4 ld_plain16(const uint4 *p) {
  uint4 r;
  asm volatile("ld.global.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}
CB_D uint4 ld_any16(const uint4 *p, bool host) { return host ? ld_plain16(p) : ld_dev16(p); }
CB_D void st_any16(uint4 *p, const uint4 &v, bool host) {
  if (host) {
    *p = v;
  } else {
    st_dev16(p, v);
  }
}

// Copies len bytes with threads tid = 0..nt-1 of the caller's group.
CB_D void copy_range_lsu(const uint8_t *s, uint8_t *d, uint64_t len, int tid, int nt, bool host) {
  const uintptr_t mis = (reinterpret_cast<uintptr_t>(s) | reinterpret_cast<uintptr_t>(d));
  if ((mis & 15) == 0) {
    const uint64_t nv = len >> 4;
    const uint4 *s4 = reinterpret_cast<const uint4 *>(s);
    uint4 *d4 = reinterpret_cast<uint4 *>(d);
    uint64_t j = tid;
    for (; j + 3 * (uint64_t)nt < nv; j += 4 * (uint64_t)nt) {
      const uint4 r0 = ld_any16(s4 + j, host);
      const uint4 r1 = ld_any16(s4 + j + nt, host);
      const uint4 r2 = ld_any16(s4 + j + 2 * nt, host);
      const uint4 r3 = ld_any16(s4 + j + 3 * nt, host);
      st_any16(d4 + j, r0, host);
      st_any16(d4 + j + nt, r1, host);
      st_any16(d4 + j + 2 * nt, r2, host);
      st_any16(d4 + j + 3 * nt, r3, host);
    }
    for (; j < nv; j += nt) st_any16(d4 + j, ld_any16(s4 + j, host), host);
    for (uint64_t b = (nv << 4) + tid; b < len; b += nt) d[b] = s[b];
  } else if ((mis & 3) == 0) {
    const uint64_t nw = len >> 2;
    const uint32_t *s1 = reinterpret_cast<const uint32_t *>(s);
    uint32_t *d1 = reinterpret_cast<uint32_t *>(d);
    for (uint64_t j = tid; j < nw; j += nt) d1[j] = s1[j];
    for (uint64_t b = (nw << 2) + tid; b < len; b += nt) d[b] = s[b];
  } else {
    for (uint64_t b = tid; b < len; b += nt) d[b] = s[b];
  }
}

// One unit of a descriptor through the LSU: a plain copy or an unpack (or,
// for a self-test descriptor, an error report without any memory access).
CB_D void lsu_unit(const CopyDesc &d, uint64_t off, uint64_t len, int tid, int nt, unsigned *err) {
  if (d.flags & kCopyFault) {
    if (tid == 0 && off == 0) atomicOr(err, kErrBounds);
  } else if (d.flags & kCopyUnpack) {
    unpack_range(reinterpret_cast<const uint8_t *>(d.src), reinterpret_cast<uint8_t *>(d.dst), off, len, tid,
                 nt);
  } else {
    copy_range_lsu(reinterpret_cast<const uint8_t *>(d.src) + off, reinterpret_cast<uint8_t *>(d.dst) + off,
                   len, tid, nt, (d.flags & kCopyHost) != 0);
  }
}

__global__ void __launch_bounds__(kLsuThreads, kLsuCtasPerSm) copy_lsu_kernel(const CopyDesc *__restrict__ desc,
                                                               const uint32_t *__restrict__ unit_start,
                                                               int n, uint32_t total_units, unsigned *err) {
  uint32_t u0, u1;
  cta_unit_range(total_units, u0, u1);
  if (u0 >= u1) return;
  int i = find_req(unit_start, n, u0);
  for (uint32_t u = u0; u < u1; ++u) {
    while (unit_start[i + 1] <= u) ++i;
    const CopyDesc d = desc[i];
    const uint64_t off = (uint64_t)(u - unit_start[i]) * kCopyUnit;
    if (off >= d.size) continue;
    const uint64_t len = min(kCopyUnit, d.size - off);
    lsu_unit(d, off, len, threadIdx.x, blockDim.x, err);
  }
}

// ---------------------------------------------------------------- TMA bulk

CB_D uint32_t smem_addr(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

CB_D void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

CB_D void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

CB_D bool mbar_wait(uint32_t bar, uint32_t parity) {
  for (uint64_t it = 0; it < kWaitLimit; ++it) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    if (ok) return true;
  }
  return false;
}

CB_D void bulk_load(uint32_t dst_smem, const void *src, uint32_t bytes, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          dst_smem),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

CB_D void bulk_store(void *dst, uint32_t src_smem, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst),
               "r"(src_smem), "r"(bytes)
               : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

CB_D void bulk_wait_read_le1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
CB_D void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
CB_D void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

struct PieceIter {
  int i;
  uint32_t u;
  uint64_t sub;
};

CB_D bool tma_unit(const CopyDesc &d, uint64_t off) {
  return !(d.flags & (kCopyHost | kCopyUnpack | kCopyFault)) && (((d.src + off) | (d.dst + off)) & 15) == 0;
}

// Next TMA piece (<= kTmaStageBytes, 16-byte multiple) of the CTA's range.
CB_D bool next_piece(PieceIter &it, uint32_t u1, const CopyDesc *desc, const uint32_t *unit_start,
                     uint64_t &src, uint64_t &dst, uint32_t &bytes) {
  while (it.u < u1) {
    while (unit_start[it.i + 1] <= it.u) ++it.i;
    const CopyDesc d = desc[it.i];
    const uint64_t off = (uint64_t)(it.u - unit_start[it.i]) * kCopyUnit;
    if (off < d.size && tma_unit(d, off)) {
      const uint64_t len = min(kCopyUnit, d.size - off) & ~15ull;
      if (it.sub < len) {
        src = d.src + off + it.sub;
        dst = d.dst + off + it.sub;
        bytes = (uint32_t)min((uint64_t)kTmaStageBytes, len - it.sub);
        it.sub += bytes;
        return true;
      }
    }
    ++it.u;
    it.sub = 0;
  }
  return false;
}

__global__ void __launch_bounds__(32) copy_tma_kernel(const CopyDesc *__restrict__ desc,
                                                      const uint32_t *__restrict__ unit_start, int n,
                                                      uint32_t total_units, unsigned *err) {
  extern __shared__ __align__(1024) uint8_t stage_mem[];
  __shared__ __align__(8) uint64_t bars[kTmaStages];
  uint32_t u0, u1;
  cta_unit_range(total_units, u0, u1);
  if (u0 >= u1) return;
  const int lane = threadIdx.x;

  // Pass 1 (whole warp): everything the TMA engine does not take.
  {
    int i = find_req(unit_start, n, u0);
    for (uint32_t u = u0; u < u1; ++u) {
      while (unit_start[i + 1] <= u) ++i;
      const CopyDesc d = desc[i];
      const uint64_t off = (uint64_t)(u - unit_start[i]) * kCopyUnit;
      if (off >= d.size) continue;
      const uint64_t len = min(kCopyUnit, d.size - off);
      if (!tma_unit(d, off)) {
        lsu_unit(d, off, len, lane, 32, err);
      } else if (len & 15) {
        const uint8_t *s = reinterpret_cast<const uint8_t *>(d.src) + off;
        uint8_t *t = reinterpret_cast<uint8_t *>(d.dst) + off;
        const uint64_t body = len & ~15ull;
        for (uint64_t b = body + lane; b < len; b += 32) t[b] = s[b];
      }
    }
  }

  // Pass 2 (lane 0): pipelined bulk copies of the aligned bodies.
  if (lane != 0) return;
  for (int s = 0; s < kTmaStages; ++s) mbar_init(smem_addr(&bars[s]), 1);
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  fence_proxy_async();

  PieceIter it{find_req(unit_start, n, u0), u0, 0};
  uint64_t ring_dst[kTmaStages];
  uint32_t ring_bytes[kTmaStages];
  uint32_t issued = 0;
  for (int s = 0; s < kTmaStages; ++s) {
    uint64_t src, dst;
    uint32_t bytes;
    if (!next_piece(it, u1, desc, unit_start, src, dst, bytes)) break;
    const uint32_t bar = smem_addr(&bars[s]);
    mbar_expect_tx(bar, bytes);
    bulk_load(smem_addr(stage_mem + (size_t)s * kTmaStageBytes), reinterpret_cast<const void *>(src),
              bytes, bar);
    ring_dst[s] = dst;
    ring_bytes[s] = bytes;
    ++issued;
  }
  bool more = issued == kTmaStages;
  for (uint32_t j = 0; j < issued; ++j) {
    const int s = (int)(j % kTmaStages);
    const uint32_t parity = (j / kTmaStages) & 1u;
    if (!mbar_wait(smem_addr(&bars[s]), parity)) {
      // A load never completed: report, give the remaining loads one more
      // bounded wait each, drain our stores, and leave.
      atomicOr(err, kErrTimeout);
      for (uint32_t k = j + 1; k < issued; ++k)
        mbar_wait(smem_addr(&bars[k % kTmaStages]), (k / kTmaStages) & 1u);
      bulk_wait_all();
      return;
    }
    fence_proxy_async();
    bulk_store(reinterpret_cast<void *>(ring_dst[s]), smem_addr(stage_mem + (size_t)s * kTmaStageBytes),
               ring_bytes[s]);
    // Store j-1 has finished reading its stage: refill that stage.
    bulk_wait_read_le1();
    if (j >= 1 && more) {
      uint64_t src, dst;
      uint32_t bytes;
      if (next_piece(it, u1, desc, unit_start, src, dst, bytes)) {
        const int fs = (int)((j - 1) % kTmaStages);
        const uint32_t bar = smem_addr(&bars[fs]);
        mbar_expect_tx(bar, bytes);
        bulk_load(smem_addr(stage_mem + (size_t)fs * kTmaStageBytes),
                  reinterpret_cast<const void *>(src), bytes, bar);
        ring_dst[fs] = dst;
        ring_bytes[fs] = bytes;
        ++issued;
      } else {
        more = false;
      }
    }
  }
  bulk_wait_all();
}

}  // namespace

cudaError_t launch_batch_copy(const CopyDesc *d_desc, const uint32_t *d_unit_start, int n,
                              uint32_t total_units, int engine, unsigned *d_err, int num_sms,
                              cudaStream_t stream, int lsu_ctas_per_sm) {
  if (n <= 0 || total_units == 0) return cudaSuccess;
  if (engine == 2) {
    const int cps = lsu_ctas_per_sm > 0 && lsu_ctas_per_sm < kLsuCtasPerSm ? lsu_ctas_per_sm : kLsuCtasPerSm;
    const uint32_t grid = min(total_units, (uint32_t)(num_sms * cps));
    copy_lsu_kernel<<<grid, kLsuThreads, 0, stream>>>(d_desc, d_unit_start, n, total_units, d_err);
    return cudaGetLastError();
  }
  static thread_local int configured_device = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  const size_t smem = (size_t)kTmaStages * kTmaStageBytes;
  if (configured_device != dev) {
    cudaError_t e =
        cudaFuncSetAttribute(copy_tma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    configured_device = dev;
  }
  const uint32_t grid = min(total_units, (uint32_t)num_sms);
  copy_tma_kernel<<<grid, 32, smem, stream>>>(d_desc, d_unit_start, n, total_units, d_err);
  return cudaGetLastError();
}

}  // namespace cb
