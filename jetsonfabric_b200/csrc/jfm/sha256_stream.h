/*
 * Incremental SHA-256 (FIPS 180-4) over the same implementation as
 * jf_sha256_buffer, for inputs too large to hold in memory (the GGUF
 * importer hashes whole source files and every segment it writes).
 * Library-internal: not part of the public C ABI.
 */
#ifndef JFB_SHA256_STREAM_H
#define JFB_SHA256_STREAM_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct jfb_sha256_stream {
    uint32_t h[8];
    uint64_t total_bytes;
    uint8_t pending[64];
    size_t pending_bytes;
} jfb_sha256_stream;

void jfb_sha256_stream_begin(jfb_sha256_stream * s);
void jfb_sha256_stream_feed(jfb_sha256_stream * s, const void * data, size_t size);
void jfb_sha256_stream_end(jfb_sha256_stream * s, uint8_t digest[32]);

#ifdef __cplusplus
}
#endif

#endif
