/*
 * SHA-256 as specified by FIPS 180-4 section 6.2. Used by the JFM loader to
 * verify segment files against the manifest (the reference verifies with its
 * own sha256.c, runtime/engines/native/src/sha256.c, called from engine.c:262-276).
 */
#include "jetsonfabric/engine.h"
#include "sha256_stream.h"

#include <string.h>

typedef jfb_sha256_stream sha256_state;

/* First 32 bits of the fractional parts of the cube roots of the first 64
 * primes (FIPS 180-4 section 4.2.2). */
static const uint32_t round_constants[64] = {
    0x428a2f98u, 0x71374491u, 0xb5c0fbcfu, 0xe9b5dba5u, 0x3956c25bu, 0x59f111f1u,
    0x923f82a4u, 0xab1c5ed5u, 0xd807aa98u, 0x12835b01u, 0x243185beu, 0x550c7dc3u,
    0x72be5d74u, 0x80deb1feu, 0x9bdc06a7u, 0xc19bf174u, 0xe49b69c1u, 0xefbe4786u,
    0x0fc19dc6u, 0x240ca1ccu, 0x2de92c6fu, 0x4a7484aau, 0x5cb0a9dcu, 0x76f988dau,
    0x983e5152u, 0xa831c66du, 0xb00327c8u, 0xbf597fc7u, 0xc6e00bf3u, 0xd5a79147u,
    0x06ca6351u, 0x14292967u, 0x27b70a85u, 0x2e1b2138u, 0x4d2c6dfcu, 0x53380d13u,
    0x650a7354u, 0x766a0abbu, 0x81c2c92eu, 0x92722c85u, 0xa2bfe8a1u, 0xa81a664bu,
    0xc24b8b70u, 0xc76c51a3u, 0xd192e819u, 0xd6990624u, 0xf40e3585u, 0x106aa070u,
    0x19a4c116u, 0x1e376c08u, 0x2748774cu, 0x34b0bcb5u, 0x391c0cb3u, 0x4ed8aa4au,
    0x5b9cca4fu, 0x682e6ff3u, 0x748f82eeu, 0x78a5636fu, 0x84c87814u, 0x8cc70208u,
    0x90befffau, 0xa4506cebu, 0xbef9a3f7u, 0xc67178f2u,
};

static uint32_t rotr(uint32_t x, unsigned n) { return (x >> n) | (x << (32u - n)); }

static void compress(uint32_t h[8], const uint8_t block[64]) {
    uint32_t w[64];
    for (unsigned t = 0; t < 16; ++t) {
        w[t] = ((uint32_t) block[4 * t] << 24) | ((uint32_t) block[4 * t + 1] << 16) |
            ((uint32_t) block[4 * t + 2] << 8) | (uint32_t) block[4 * t + 3];
    }
    for (unsigned t = 16; t < 64; ++t) {
        const uint32_t s0 = rotr(w[t - 15], 7) ^ rotr(w[t - 15], 18) ^ (w[t - 15] >> 3);
        const uint32_t s1 = rotr(w[t - 2], 17) ^ rotr(w[t - 2], 19) ^ (w[t - 2] >> 10);
        w[t] = w[t - 16] + s0 + w[t - 7] + s1;
    }
    uint32_t a = h[0], b = h[1], c = h[2], d = h[3];
    uint32_t e = h[4], f = h[5], g = h[6], k = h[7];
    for (unsigned t = 0; t < 64; ++t) {
        const uint32_t big1 = rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25);
        const uint32_t choose = (e & f) ^ (~e & g);
        const uint32_t t1 = k + big1 + choose + round_constants[t] + w[t];
        const uint32_t big0 = rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22);
        const uint32_t majority = (a & b) ^ (a & c) ^ (b & c);
        const uint32_t t2 = big0 + majority;
        k = g; g = f; f = e; e = d + t1;
        d = c; c = b; b = a; a = t1 + t2;
    }
    h[0] += a; h[1] += b; h[2] += c; h[3] += d;
    h[4] += e; h[5] += f; h[6] += g; h[7] += k;
}

static void sha256_begin(sha256_state * s) {
    /* First 32 bits of the fractional parts of the square roots of the first
     * eight primes (FIPS 180-4 section 5.3.3). */
    static const uint32_t initial[8] = {
        0x6a09e667u, 0xbb67ae85u, 0x3c6ef372u, 0xa54ff53au,
        0x510e527fu, 0x9b05688cu, 0x1f83d9abu, 0x5be0cd19u,
    };
    memcpy(s->h, initial, sizeof(initial));
    s->total_bytes = 0;
    s->pending_bytes = 0;
}

static void sha256_feed(sha256_state * s, const uint8_t * data, size_t size) {
    s->total_bytes += size;
    if (s->pending_bytes > 0) {
        const size_t take = size < 64 - s->pending_bytes ? size : 64 - s->pending_bytes;
        memcpy(s->pending + s->pending_bytes, data, take);
        s->pending_bytes += take;
        data += take;
        size -= take;
        if (s->pending_bytes < 64) return;
        compress(s->h, s->pending);
        s->pending_bytes = 0;
    }
    while (size >= 64) {
        compress(s->h, data);
        data += 64;
        size -= 64;
    }
    memcpy(s->pending, data, size);
    s->pending_bytes = size;
}

static void sha256_end(sha256_state * s, uint8_t digest[32]) {
    const uint64_t bit_length = s->total_bytes * 8u;
    uint8_t tail[128];
    size_t tail_bytes = s->pending_bytes;
    memcpy(tail, s->pending, tail_bytes);
    tail[tail_bytes++] = 0x80;
    const size_t padded = tail_bytes <= 56 ? 64 : 128;
    memset(tail + tail_bytes, 0, padded - tail_bytes);
    for (unsigned i = 0; i < 8; ++i) {
        tail[padded - 1 - i] = (uint8_t) (bit_length >> (8u * i));
    }
    compress(s->h, tail);
    if (padded == 128) compress(s->h, tail + 64);
    for (unsigned i = 0; i < 8; ++i) {
        digest[4 * i] = (uint8_t) (s->h[i] >> 24);
        digest[4 * i + 1] = (uint8_t) (s->h[i] >> 16);
        digest[4 * i + 2] = (uint8_t) (s->h[i] >> 8);
        digest[4 * i + 3] = (uint8_t) s->h[i];
    }
}

void jf_sha256_buffer(const void * data, size_t size, uint8_t digest[32]) {
    sha256_state state;
    sha256_begin(&state);
    sha256_feed(&state, (const uint8_t *) data, size);
    sha256_end(&state, digest);
}

void jfb_sha256_stream_begin(jfb_sha256_stream * s) { sha256_begin(s); }

void jfb_sha256_stream_feed(jfb_sha256_stream * s, const void * data, size_t size) {
    sha256_feed(s, (const uint8_t *) data, size);
}

void jfb_sha256_stream_end(jfb_sha256_stream * s, uint8_t digest[32]) { sha256_end(s, digest); }
