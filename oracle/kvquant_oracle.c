/* ORACLE — test infrastructure only (the checker of the INT8 tier-move
 * kernels; never linked into the product).
 *
 * Plain-C restatement of the reference's INT8 KV compressor,
 * KVCompressor::compress / decompress
 * (cascade_Code/cpp/src/cascade_core.cpp:908-967, format and sizes in
 * cascade_Code/cpp/include/cascade.hpp:386-418):
 *
 *   compress:   the block is read as n = size/2 little-endian int16 values
 *               (the raw bit patterns of the fp16 data, not their values);
 *               min/max over them; scale = (max-min)/255 (1 when max == min);
 *               zero_point = int8(trunc(min/scale)); every value becomes
 *               int8(clamp(trunc((v-min)*(1/scale) + 0.5), 0, 255) - 128).
 *               Output: [f32 scale][i8 zero_point][3 pad][n x i8].
 *   decompress: v = int16(trunc((q + 128)*scale + zero_point*scale)),
 *               n = (compressed size - 8)/2 ... i.e. original size (size/2)*2.
 *
 * Arithmetic as the reference's Release build computes it
 * (cascade_Code/cpp/CMakeLists.txt:19, "-O3 -march=native", GCC): on any
 * x86-64 host with FMA (the reference's Perlmutter/Milan nodes included) GCC's
 * default -ffp-contract=fast fuses "x*y + z" into one fused multiply-add, so
 * both loops use fmaf here. Float-to-integer conversions follow x86
 * cvttss2si: truncation toward zero, then the integer's low 8 / 16 bits
 * (the narrowing of an out-of-range value is what the reference's machine
 * code does; C++ leaves it undefined). The 3 padding bytes of the header are
 * indeterminate in the reference; they are written as zero here.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

static int32_t cvtt_i32(float x) {
  if (!(x > -2147483904.0f && x < 2147483648.0f)) return INT32_MIN; /* x86 "integer indefinite" */
  return (int32_t)x;
}

static int16_t ld_i16(const uint8_t *p) {
  uint16_t u = (uint16_t)(p[0] | (p[1] << 8));
  int16_t v;
  memcpy(&v, &u, 2);
  return v;
}

/* Header fields for a block with raw int16 extremes mn, mx. */
void kvq_params(int32_t mn, int32_t mx, float *scale, int8_t *zero_point) {
  const float range = (float)mx - (float)mn;
  const float s = (range > 0.0f) ? range / 255.0f : 1.0f;
  *scale = s;
  *zero_point = (int8_t)(uint8_t)((uint32_t)cvtt_i32((float)mn / s) & 0xFFu);
}

uint64_t kvq_compressed_size(uint64_t size) { return 8 + size / 2; }

/* out: 8 + size/2 bytes. size >= 2. Returns the bytes written. */
uint64_t kvq_compress(const uint8_t *data, uint64_t size, uint8_t *out) {
  const uint64_t n = size / 2;
  int32_t mn = ld_i16(data), mx = mn;
  for (uint64_t i = 1; i < n; ++i) {
    const int32_t v = ld_i16(data + 2 * i);
    if (v < mn) mn = v;
    if (v > mx) mx = v;
  }
  float scale;
  int8_t zp;
  kvq_params(mn, mx, &scale, &zp);
  memcpy(out, &scale, 4);
  out[4] = (uint8_t)zp;
  out[5] = out[6] = out[7] = 0;
  const float inv = 1.0f / scale;
  const float min_f = (float)mn;
  for (uint64_t i = 0; i < n; ++i) {
    const float val = (float)ld_i16(data + 2 * i);
    int32_t q = cvtt_i32(fmaf(val - min_f, inv, 0.5f));
    q = q < 0 ? 0 : (q > 255 ? 255 : q);
    out[8 + i] = (uint8_t)(q - 128);
  }
  return 8 + n;
}

/* out: (orig_size/2)*2 bytes. Returns 0 when the compressed buffer is short
 * (the reference's `return false`), else 1. */
int kvq_decompress(const uint8_t *comp, uint64_t comp_size, uint64_t orig_size, uint8_t *out) {
  const uint64_t n = orig_size / 2;
  if (comp_size < 8 + n) return 0;
  float scale;
  memcpy(&scale, comp, 4);
  const int8_t zp = (int8_t)comp[4];
  const float min_f = (float)zp * scale;
  for (uint64_t i = 0; i < n; ++i) {
    const float q = (float)(int8_t)comp[8 + i];
    const uint16_t v = (uint16_t)((uint32_t)cvtt_i32(fmaf(q + 128.0f, scale, min_f)) & 0xFFFFu);
    out[2 * i] = (uint8_t)(v & 0xFF);
    out[2 * i + 1] = (uint8_t)(v >> 8);
  }
  return 1;
}
