// INT8 packing of blocks into the DRAM-tier format (kv_compression): the GPU
// side of KVCompressor::compress (cascade_Code/cpp/src/cascade_core.cpp:
// 908-944) fused into the HBM -> DRAM tier move. The reference compresses each
// block with a CPU loop before its DRAM write (src/distributed_backend.cpp:
// 898-903); here the whole wave of demotions is packed by two launches that
// read the blocks from HBM and write only the packed bytes (8 + size/2) over
// the host link into the pinned DRAM arena:
//   1. kv_minmax_kernel: the int16 min/max of every block (warp reductions,
//      one atomicMin/atomicMax pair per warp and unit);
//   2. kv_pack_kernel: header + one int8 code per value (16-byte loads from
//      HBM, 16-byte stores to the arena: the store starts every packed block
//      8 bytes into its extent so that the int8 payload is 16-byte aligned).
// Both walk the same kCopyUnit units as the copy kernels (units.cuh). The
// inverse (unpack) runs inside the copy kernels on kCopyUnpack descriptors.
#include <climits>

#include "kernels.cuh"
#include "kvquant.cuh"
#include "units.cuh"

namespace cb {

namespace {

constexpr int kThreads = 256;
constexpr int kCtasPerSm = 8;

CB_D int ld_i16(const uint8_t *p) { return (int)(short)((uint32_t)p[0] | ((uint32_t)p[1] << 8)); }

CB_D void st_plain8(void *p, uint2 v) {
  asm volatile("st.global.v2.u32 [%0], {%1,%2};" ::"l"(p), "r"(v.x), "r"(v.y) : "memory");
}
CB_D void st_plain16(void *p, uint4 v) {
  asm volatile("st.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

// Values [e0, e1) of the unit that starts at source byte 2*e0.
CB_D void unit_values(const CopyDesc &d, uint64_t off, uint64_t &e0, uint64_t &e1) {
  e0 = off / 2;
  e1 = min(d.size / 2, (off + kCopyUnit) / 2);
}

__global__ void __launch_bounds__(kThreads) kv_minmax_kernel(const CopyDesc *__restrict__ desc,
                                                             const uint32_t *__restrict__ unit_start, int n,
                                                             uint32_t total_units, int *__restrict__ mm) {
  uint32_t u0, u1;
  cta_unit_range(total_units, u0, u1);
  if (u0 >= u1) return;
  int i = find_req(unit_start, n, u0);
  for (uint32_t u = u0; u < u1; ++u) {
    while (unit_start[i + 1] <= u) ++i;
    const CopyDesc d = desc[i];
    const uint64_t off = (uint64_t)(u - unit_start[i]) * kCopyUnit;
    if (off >= d.size) continue;  // uniform across the CTA
    uint64_t e0, e1;
    unit_values(d, off, e0, e1);
    const uint8_t *s = reinterpret_cast<const uint8_t *>(d.src);
    int mn = INT_MAX, mx = INT_MIN;
    uint64_t e = e0;
    if ((reinterpret_cast<uintptr_t>(s + 2 * e0) & 15) == 0) {
      // 8 values per 16-byte load, two per 32-bit word (per-halfword min/max)
      const uint64_t ng = (e1 - e0) / 8;
      const uint4 *s16 = reinterpret_cast<const uint4 *>(s + 2 * e0);
      uint32_t vmn = 0x7fff7fffu, vmx = 0x80008000u;
      for (uint64_t g = threadIdx.x; g < ng; g += blockDim.x) {
        const uint4 v = __ldg(s16 + g);
        vmn = __vmins2(vmn, __vmins2(__vmins2(v.x, v.y), __vmins2(v.z, v.w)));
        vmx = __vmaxs2(vmx, __vmaxs2(__vmaxs2(v.x, v.y), __vmaxs2(v.z, v.w)));
      }
      mn = min(lo16s(vmn), hi16s(vmn));
      mx = max(lo16s(vmx), hi16s(vmx));
      e = e0 + ng * 8;
    }
    for (uint64_t k = e + threadIdx.x; k < e1; k += blockDim.x) {
      const int v = ld_i16(s + 2 * k);
      mn = min(mn, v);
      mx = max(mx, v);
    }
    // Threads without values hold an identity (32767/-32768 or INT_MAX/INT_MIN).
    mn = __reduce_min_sync(0xffffffffu, mn);
    mx = __reduce_max_sync(0xffffffffu, mx);
    if ((threadIdx.x & 31) == 0 && mn <= mx) {
      atomicMin(&mm[2 * i], mn);
      atomicMax(&mm[2 * i + 1], mx);
    }
  }
}

// Eight values (one 16-byte word) -> eight codes (two 32-bit words).
CB_D uint2 pack8(const uint4 &v, const PackParams &p) {
  uint2 w;
  w.x = pack1(lo16s(v.x), p) | (pack1(hi16s(v.x), p) << 8) | (pack1(lo16s(v.y), p) << 16) |
        (pack1(hi16s(v.y), p) << 24);
  w.y = pack1(lo16s(v.z), p) | (pack1(hi16s(v.z), p) << 8) | (pack1(lo16s(v.w), p) << 16) |
        (pack1(hi16s(v.w), p) << 24);
  return w;
}

__global__ void __launch_bounds__(kThreads) kv_pack_kernel(const CopyDesc *__restrict__ desc,
                                                           const uint32_t *__restrict__ unit_start, int n,
                                                           uint32_t total_units, const int *__restrict__ mm) {
  uint32_t u0, u1;
  cta_unit_range(total_units, u0, u1);
  if (u0 >= u1) return;
  int i = find_req(unit_start, n, u0);
  for (uint32_t u = u0; u < u1; ++u) {
    while (unit_start[i + 1] <= u) ++i;
    const CopyDesc d = desc[i];
    const uint64_t off = (uint64_t)(u - unit_start[i]) * kCopyUnit;
    if (off >= d.size) continue;
    const PackParams p = pack_params(mm[2 * i], mm[2 * i + 1]);
    uint8_t *blk = reinterpret_cast<uint8_t *>(d.dst);
    if (off == 0 && threadIdx.x == 0) {
      const uint32_t sb = __float_as_uint(p.scale), zb = (uint32_t)p.zp & 0xffu;
      if ((reinterpret_cast<uintptr_t>(blk) & 7) == 0) {
        st_plain8(blk, make_uint2(sb, zb));
      } else {
        for (int k = 0; k < 4; ++k) blk[k] = (uint8_t)(sb >> (8 * k));
        blk[4] = (uint8_t)zb;
        blk[5] = blk[6] = blk[7] = 0;
      }
    }
    uint64_t e0, e1;
    unit_values(d, off, e0, e1);
    const uint8_t *s = reinterpret_cast<const uint8_t *>(d.src) + 2 * e0;
    uint8_t *q = blk + kPackHeaderBytes + e0;
    uint64_t done = 0;
    const uintptr_t sa = reinterpret_cast<uintptr_t>(s), qa = reinterpret_cast<uintptr_t>(q);
    const uint4 *s16 = reinterpret_cast<const uint4 *>(s);
    if (((sa | qa) & 15) == 0) {
      // 16 values (two 16-byte loads) -> 16 codes (one 16-byte store). The
      // store places packed blocks so that q is 16-byte aligned.
      const uint64_t ng = (e1 - e0) / 16;
      uint4 *q16 = reinterpret_cast<uint4 *>(q);
      uint64_t g = threadIdx.x;
      for (; g + blockDim.x < ng; g += 2 * (uint64_t)blockDim.x) {
        const uint64_t h = g + blockDim.x;
        const uint4 a0 = __ldg(s16 + 2 * g), a1 = __ldg(s16 + 2 * g + 1);
        const uint4 b0 = __ldg(s16 + 2 * h), b1 = __ldg(s16 + 2 * h + 1);
        const uint2 wa0 = pack8(a0, p), wa1 = pack8(a1, p), wb0 = pack8(b0, p), wb1 = pack8(b1, p);
        st_plain16(q16 + g, make_uint4(wa0.x, wa0.y, wa1.x, wa1.y));
        st_plain16(q16 + h, make_uint4(wb0.x, wb0.y, wb1.x, wb1.y));
      }
      for (; g < ng; g += blockDim.x) {
        const uint2 w0 = pack8(__ldg(s16 + 2 * g), p), w1 = pack8(__ldg(s16 + 2 * g + 1), p);
        st_plain16(q16 + g, make_uint4(w0.x, w0.y, w1.x, w1.y));
      }
      done = ng * 16;
    } else if ((sa & 15) == 0 && (qa & 7) == 0) {
      // 8 values (one 16-byte load) -> 8 codes (one 8-byte store)
      const uint64_t ng = (e1 - e0) / 8;
      uint2 *q8 = reinterpret_cast<uint2 *>(q);
      for (uint64_t g = threadIdx.x; g < ng; g += blockDim.x) st_plain8(q8 + g, pack8(__ldg(s16 + g), p));
      done = ng * 8;
    }
    for (uint64_t k = done + threadIdx.x; k < e1 - e0; k += blockDim.x)
      q[k] = (uint8_t)pack1(ld_i16(s + 2 * k), p);
  }
}

}  // namespace

cudaError_t launch_kv_pack(const CopyDesc *d_desc, const uint32_t *d_unit_start, int n, uint32_t total_units,
                           int *d_mm, int num_sms, cudaStream_t stream, int ctas_per_sm) {
  if (n <= 0 || total_units == 0) return cudaSuccess;
  const int cps = ctas_per_sm > 0 && ctas_per_sm < kCtasPerSm ? ctas_per_sm : kCtasPerSm;
  const uint32_t grid = min(total_units, (uint32_t)(num_sms * cps));
  kv_minmax_kernel<<<grid, kThreads, 0, stream>>>(d_desc, d_unit_start, n, total_units, d_mm);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  kv_pack_kernel<<<grid, kThreads, 0, stream>>>(d_desc, d_unit_start, n, total_units, d_mm);
  return cudaGetLastError();
}

}  // namespace cb
