/*
 * ORACLE — test infrastructure only. Nothing in the product links, loads or
 * calls this file; only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline leg use it, and only as the checker.
 *
 * Plain-C restatement of the block-ID computation on the Cascade hot path:
 *
 *   cascade_Code/cpp/src/cascade_core.cpp:47-58  compute_block_id():
 *       SHA256(data, size) (OpenSSL one-shot, third-party libcrypto, system
 *       OpenSSL 3.0.x; the algorithm is FIPS 180-4 SHA-256), keep the first
 *       16 digest bytes, format them as 32 lowercase hex characters.
 *
 * OpenSSL is not vendored by the reference. This file restates the published
 * FIPS 180-4 algorithm (sections 4.1.2, 4.2.2, 5.1.1, 5.3.3, 6.2) and is
 * pinned against the reference's compiled compute_block_id and against
 * Python's hashlib (the convention of benchmark/run_benchmark.py:119) by
 * tests/golden/make_golden.py and tests/test_oracle.py.
 *
 * The round constants are not typed in: they are derived at first use from
 * their definition (FIPS 180-4 4.2.2: first 32 bits of the fractional parts
 * of the cube roots of the first 64 primes; 5.3.3: square roots of the first
 * 8 primes) with exact integer root extraction, so a transcription error is
 * impossible by construction.
 */
#include <stdint.h>
#include <stddef.h>
#include <string.h>

static uint32_t K[64];
static uint32_t H0[8];
static int consts_ready = 0;

/* floor(x^(1/k)) for k in {2,3}, x < 2^128, exact (binary search on
 * unsigned __int128). */
static unsigned __int128 iroot(unsigned __int128 x, int k) {
    /* roots needed here are < 2^36 (x < 2^105), so hi = 2^40 keeps mid^2 far
     * from overflow; mid^3 is compared as mid^2 > x / mid. */
    unsigned __int128 lo = 0, hi = (unsigned __int128)1 << 40;
    while (lo < hi) {
        unsigned __int128 mid = (lo + hi + 1) >> 1;
        unsigned __int128 p = mid * mid;
        if (k == 3) {
            if (p > x / mid) { hi = mid - 1; continue; }
            p = p * mid;
        }
        if (p <= x) lo = mid; else hi = mid - 1;
    }
    return lo;
}

static void init_consts(void) {
    int primes[64];
    int count = 0;
    for (int c = 2; count < 64; ++c) {
        int is_p = 1;
        for (int d = 2; d * d <= c; ++d) if (c % d == 0) { is_p = 0; break; }
        if (is_p) primes[count++] = c;
    }
    for (int i = 0; i < 64; ++i) {
        /* frac(cbrt(p)) * 2^32 = cbrt(p * 2^96) mod 2^32 */
        unsigned __int128 x = (unsigned __int128)primes[i] << 96;
        K[i] = (uint32_t)iroot(x, 3);
    }
    for (int i = 0; i < 8; ++i) {
        /* frac(sqrt(p)) * 2^32 = sqrt(p * 2^64) mod 2^32 */
        unsigned __int128 x = (unsigned __int128)primes[i] << 64;
        H0[i] = (uint32_t)iroot(x, 2);
    }
    consts_ready = 1;
}

static inline uint32_t rotr(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }

/* FIPS 180-4 6.2.2: one compression of a 64-byte message block. */
static void compress(uint32_t h[8], const uint8_t blk[64]) {
    uint32_t w[64];
    for (int t = 0; t < 16; ++t)
        w[t] = ((uint32_t)blk[4 * t] << 24) | ((uint32_t)blk[4 * t + 1] << 16) |
               ((uint32_t)blk[4 * t + 2] << 8) | (uint32_t)blk[4 * t + 3];
    for (int t = 16; t < 64; ++t) {
        uint32_t s0 = rotr(w[t - 15], 7) ^ rotr(w[t - 15], 18) ^ (w[t - 15] >> 3);
        uint32_t s1 = rotr(w[t - 2], 17) ^ rotr(w[t - 2], 19) ^ (w[t - 2] >> 10);
        w[t] = w[t - 16] + s0 + w[t - 7] + s1;
    }
    uint32_t a = h[0], b = h[1], c = h[2], d = h[3], e = h[4], f = h[5], g = h[6], hh = h[7];
    for (int t = 0; t < 64; ++t) {
        uint32_t S1 = rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25);
        uint32_t ch = (e & f) ^ (~e & g);
        uint32_t t1 = hh + S1 + ch + K[t] + w[t];
        uint32_t S0 = rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22);
        uint32_t mj = (a & b) ^ (a & c) ^ (b & c);
        uint32_t t2 = S0 + mj;
        hh = g; g = f; f = e; e = d + t1; d = c; c = b; b = a; a = t1 + t2;
    }
    h[0] += a; h[1] += b; h[2] += c; h[3] += d;
    h[4] += e; h[5] += f; h[6] += g; h[7] += hh;
}

/* Full SHA-256 (FIPS 180-4 5.1.1 padding + 6.2). out = 32 digest bytes. */
void oracle_sha256(const uint8_t *data, uint64_t len, uint8_t out[32]) {
    if (!consts_ready) init_consts();
    uint32_t h[8];
    memcpy(h, H0, sizeof h);
    uint64_t full = len / 64;
    for (uint64_t i = 0; i < full; ++i) compress(h, data + 64 * i);
    uint8_t tail[128];
    uint64_t rem = len - 64 * full;
    memset(tail, 0, sizeof tail);
    if (rem) memcpy(tail, data + 64 * full, rem);
    tail[rem] = 0x80;
    uint64_t tlen = (rem < 56) ? 64 : 128;
    uint64_t bits = len * 8;
    for (int i = 0; i < 8; ++i) tail[tlen - 1 - i] = (uint8_t)(bits >> (8 * i));
    compress(h, tail);
    if (tlen == 128) compress(h, tail + 64);
    for (int i = 0; i < 8; ++i) {
        out[4 * i] = (uint8_t)(h[i] >> 24);
        out[4 * i + 1] = (uint8_t)(h[i] >> 16);
        out[4 * i + 2] = (uint8_t)(h[i] >> 8);
        out[4 * i + 3] = (uint8_t)h[i];
    }
}

/* Batch form over a packed buffer: block i is data[offsets[i] .. +sizes[i]).
 * digests: n * 32 bytes. */
void oracle_sha256_batch(const uint8_t *data, const uint64_t *offsets,
                         const uint64_t *sizes, int64_t n, uint8_t *digests) {
    for (int64_t i = 0; i < n; ++i)
        oracle_sha256(data + offsets[i], sizes[i], digests + 32 * i);
}

/* compute_block_id restated (cascade_core.cpp:47-58): 16 digest bytes as 32
 * lowercase hex chars + NUL into hex33. */
void oracle_block_id(const uint8_t *data, uint64_t len, char hex33[33]) {
    static const char *digits = "0123456789abcdef";
    uint8_t d[32];
    oracle_sha256(data, len, d);
    for (int i = 0; i < 16; ++i) {
        hex33[2 * i] = digits[d[i] >> 4];
        hex33[2 * i + 1] = digits[d[i] & 15];
    }
    hex33[32] = 0;
}

/* Exposes the derived constants so tests can compare them with the CUDA
 * source's table. */
void oracle_sha256_constants(uint32_t k_out[64], uint32_t h0_out[8]) {
    if (!consts_ready) init_consts();
    memcpy(k_out, K, sizeof K);
    memcpy(h0_out, H0, sizeof H0);
}
