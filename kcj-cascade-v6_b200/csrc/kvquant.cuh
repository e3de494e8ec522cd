// INT8 KV packing of DRAM-tier blocks (kv_compression), device side.
//
// Restates the reference's KVCompressor (cascade_Code/cpp/src/
// cascade_core.cpp:908-967; format in include/cascade.hpp:386-418):
//   * a block is n = size/2 little-endian int16 values (the raw bit patterns
//     of its fp16 data); an odd last byte is not kept;
//   * scale = (max - min)/255 (1 when max == min);
//     zero_point = int8(trunc(min/scale));
//   * q = clamp(trunc((v - min) * (1/scale) + 0.5), 0, 255) - 128;
//   * unpacked value = int16(trunc((q + 128) * scale + zero_point * scale));
//   * packed block = [f32 scale][i8 zero_point][3 zero bytes][n x i8].
// The arithmetic is the reference's Release build (-O3 -march=native on an
// FMA host, GCC's default fp-contract=fast): both "x*y + z" are one fused
// multiply-add, every other operation is one IEEE single-precision operation
// rounded to nearest, written with the _rn intrinsics so that nvcc cannot
// contract or reassociate them. Float-to-integer conversion truncates toward
// zero and keeps the low 8 or 16 bits (x86 cvttss2si followed by a narrowing
// store); the operands are finite and inside int32 range by construction
// (|v - min| <= 65535, 1/scale <= 255, |q + 128| * scale <= 65535 + 257).
#pragma once

#include "common.cuh"
#include "policy.hpp"  // kPackHeaderBytes, kPackMinBytes

namespace cb {

CB_HD uint64_t packed_size(uint64_t size) { return kPackHeaderBytes + size / 2; }

struct PackParams {
  float scale;  // header field
  float inv;    // 1/scale
  float min_f;  // min as float
  int zp;       // int8 zero point, sign-extended
};

CB_D PackParams pack_params(int mn, int mx) {
  PackParams p;
  const float range = __fsub_rn(__int2float_rn(mx), __int2float_rn(mn));
  p.scale = range > 0.0f ? __fdiv_rn(range, 255.0f) : 1.0f;
  p.zp = (int)(signed char)(__float2int_rz(__fdiv_rn(__int2float_rn(mn), p.scale)) & 0xff);
  p.inv = __fdiv_rn(1.0f, p.scale);
  p.min_f = __int2float_rn(mn);
  return p;
}

// One int16 value -> its int8 code (as the low byte of the result).
CB_D uint32_t pack1(int v, const PackParams &p) {
  int q = __float2int_rz(__fmaf_rn(__fsub_rn(__int2float_rn(v), p.min_f), p.inv, 0.5f));
  q = min(255, max(0, q));
  return (uint32_t)(q - 128) & 0xffu;
}

// One int8 code (sign-extended) -> the unpacked int16 (as the low 16 bits).
CB_D uint32_t unpack1(int q, float scale, float zmin) {
  return (uint32_t)__float2int_rz(__fmaf_rn(__fadd_rn(__int2float_rn(q), 128.0f), scale, zmin)) & 0xffffu;
}

CB_D int lo16s(uint32_t w) { return (int)(short)(w & 0xffffu); }
CB_D int hi16s(uint32_t w) { return (int)(short)(w >> 16); }
CB_D int byte_s(uint32_t w, int k) { return (int)(signed char)((w >> (8 * k)) & 0xffu); }

// Plain (coherent) loads: the packed side may be mapped pinned host memory.
CB_D uint2 ld_host8(const void *p) {
  uint2 r;
  asm volatile("ld.global.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
  return r;
}
CB_D uint4 ld_host16(const void *p) {
  uint4 r;
  asm volatile("ld.global.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}

// Four packed codes (one 32-bit word) -> four unpacked values (two words).
CB_D uint2 unpack4(uint32_t w, float scale, float zmin) {
  uint2 r;
  r.x = unpack1(byte_s(w, 0), scale, zmin) | (unpack1(byte_s(w, 1), scale, zmin) << 16);
  r.y = unpack1(byte_s(w, 2), scale, zmin) | (unpack1(byte_s(w, 3), scale, zmin) << 16);
  return r;
}

// Writes bytes [off, off + len) of the unpacked form of the packed block at
// blk into out + off, with threads tid = 0..nt-1 of the caller's group. off
// is a multiple of 16 (a copy unit boundary) and len is even. blk may be
// mapped pinned host memory (plain loads throughout). The store places packed
// blocks so that the payload (blk + 8) is 16-byte aligned; other alignments
// (caller buffers) take 8-byte or byte-wise paths.
CB_D void unpack_range(const uint8_t *blk, uint8_t *out, uint64_t off, uint64_t len, int tid, int nt) {
  float scale;
  int zp;
  if ((reinterpret_cast<uintptr_t>(blk) & 7) == 0) {
    const uint2 h = ld_host8(blk);
    scale = __uint_as_float(h.x);
    zp = byte_s(h.y, 0);
  } else {
    const uint32_t b = (uint32_t)blk[0] | ((uint32_t)blk[1] << 8) | ((uint32_t)blk[2] << 16) |
                       ((uint32_t)blk[3] << 24);
    scale = __uint_as_float(b);
    zp = (int)(signed char)blk[4];
  }
  const float zmin = __fmul_rn(__int2float_rn(zp), scale);
  const uint8_t *q = blk + kPackHeaderBytes + off / 2;
  uint8_t *o = out + off;
  const uint64_t ne = len / 2;
  const uintptr_t qa = reinterpret_cast<uintptr_t>(q), oa = reinterpret_cast<uintptr_t>(o);
  uint64_t done = 0;
  if (((qa | oa) & 15) == 0) {
    // 16 codes (one 16-byte load) -> 16 values (two 16-byte stores); 4 loads
    // in flight per thread to cover the host-link latency.
    const uint64_t ng = ne / 16;
    const uint4 *q16 = reinterpret_cast<const uint4 *>(q);
    uint4 *o16 = reinterpret_cast<uint4 *>(o);
    uint64_t g = tid;
    for (; g + 3 * (uint64_t)nt < ng; g += 4 * (uint64_t)nt) {
      uint4 w[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) w[k] = ld_host16(q16 + g + k * nt);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint2 a = unpack4(w[k].x, scale, zmin), b = unpack4(w[k].y, scale, zmin);
        const uint2 c = unpack4(w[k].z, scale, zmin), d = unpack4(w[k].w, scale, zmin);
        o16[2 * (g + k * nt)] = make_uint4(a.x, a.y, b.x, b.y);
        o16[2 * (g + k * nt) + 1] = make_uint4(c.x, c.y, d.x, d.y);
      }
    }
    for (; g < ng; g += nt) {
      const uint4 w = ld_host16(q16 + g);
      const uint2 a = unpack4(w.x, scale, zmin), b = unpack4(w.y, scale, zmin);
      const uint2 c = unpack4(w.z, scale, zmin), d = unpack4(w.w, scale, zmin);
      o16[2 * g] = make_uint4(a.x, a.y, b.x, b.y);
      o16[2 * g + 1] = make_uint4(c.x, c.y, d.x, d.y);
    }
    done = ng * 16;
  } else if ((qa & 7) == 0 && (oa & 15) == 0) {
    // 8 codes (one 8-byte load) -> 8 values (one 16-byte store)
    const uint64_t ng = ne / 8;
    const uint2 *q8 = reinterpret_cast<const uint2 *>(q);
    uint4 *o16 = reinterpret_cast<uint4 *>(o);
    for (uint64_t g = tid; g < ng; g += nt) {
      const uint2 w = ld_host8(q8 + g);
      const uint2 a = unpack4(w.x, scale, zmin), b = unpack4(w.y, scale, zmin);
      o16[g] = make_uint4(a.x, a.y, b.x, b.y);
    }
    done = ng * 8;
  }
  for (uint64_t e = done + tid; e < ne; e += nt) {
    const uint32_t v = unpack1((int)(signed char)q[e], scale, zmin);
    o[2 * e] = (uint8_t)(v & 0xffu);
    o[2 * e + 1] = (uint8_t)(v >> 8);
  }
}

}  // namespace cb
