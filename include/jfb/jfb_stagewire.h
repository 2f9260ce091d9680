/*
 * Stagewire v2 payload checksums on the device.
 *
 * A Stagewire v2 frame (reference internal/stagewire/frame.go:36-136) is a
 * 20-byte big-endian header, JSON metadata and the raw payload; the metadata
 * field `payload_crc32` holds crc32.ChecksumIEEE(payload) and a receiver
 * rejects a frame whose payload does not match it (frame.go:221-223). When
 * stage activations travel GPU to GPU over NVLink the payload never reaches
 * the host, so these entry points compute the checksum where the bytes are,
 * write it into the metadata bytes of an outgoing frame, and compare it with
 * the field of a received frame, all ordered on `stream` with no host sync.
 *
 * Conventions as in jfb_kernels.h: device pointers, `stream` is a
 * cudaStream_t passed as void*, a jfb_status is returned and never thrown.
 */
#ifndef JFB_STAGEWIRE_H
#define JFB_STAGEWIRE_H

#include <stdint.h>

#include "jfb/jfb_status.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Width of the checksum field the stamp writes: the decimal CRC right-aligned
 * in 10 characters, leading spaces being JSON whitespace before the number. */
#define JFB_STAGEWIRE_CRC_FIELD 10

/* Device scratch that jfb_crc32 needs for an `n`-byte input. */
uint64_t jfb_crc32_scratch_bytes(uint64_t n);

/* *crc_out (device word) = CRC-32/IEEE of data[0, n), the value of Go's
 * crc32.ChecksumIEEE and zlib's crc32 (replaces the host checksum of
 * frame.go:272 for a device payload). n = 0 writes 0. */
jfb_status jfb_crc32(const void * data, uint64_t n, uint32_t * crc_out, void * scratch, uint64_t scratch_bytes,
                     void * stream);

/* Writes *crc as JFB_STAGEWIRE_CRC_FIELD characters at frame[field_offset]:
 * the outgoing frame's `payload_crc32` value (metadata built on the host with
 * that many spaces in its place). */
jfb_status jfb_stagewire_stamp_crc(const uint32_t * crc, uint8_t * frame, uint32_t field_offset, void * stream);

/* Received-frame check: parses the JFB_STAGEWIRE_CRC_FIELD characters at
 * frame[field_offset] (optional leading spaces, then decimal digits) and sets
 * *mismatch = 1 when they are malformed or differ from *crc; leaves it
 * untouched otherwise, so one word can gather the checks of many frames. */
jfb_status jfb_stagewire_check_crc(const uint32_t * crc, const uint8_t * frame, uint32_t field_offset,
                                   int32_t * mismatch, void * stream);

#ifdef __cplusplus
}
#endif

#endif
