/*
 * Stagewire v2 frames between stages: payload checksums on the device, and
 * an in-box frame channel between processes.
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

/* ---- in-box frame channel ----------------------------------------------------
 *
 * Carries Stagewire v2 frames between processes on one host through POSIX
 * shared memory, in place of the reference's keep-alive HTTP connection
 * (runtime/transport/http_stage_transport.cpp:481-599: one POST of the
 * request frame answered by a status and a response frame). A stage server
 * creates a named channel; callers open it by name. Each call writes the
 * request frame in two pieces (the reference's EncodedStageFrameView prefix
 * and payload) and waits for the server's status, a flag telling a reply
 * frame from a JSON error body (the reference's non-Stagewire error
 * responses), and the reply bytes. Frames are opaque here. Every wait is
 * bounded by `timeout_ms` and ends with JFB_STATUS_TIMEOUT; one caller holds
 * the channel at a time. Nothing here touches a GPU. */
typedef struct jfb_frame_channel jfb_frame_channel;

/* Server side: creates channel `name` ([A-Za-z0-9._-], up to 200 characters)
 * with `capacity` bytes per direction (0: 513 MiB + 4 KiB, the largest
 * frame the Stagewire v2 limits allow; the segment is sparse). Fails if the
 * name is taken. */
jfb_status jfb_frame_channel_create(const char * name, uint64_t capacity, jfb_frame_channel ** out);

/* Caller side: opens channel `name`, waiting up to `timeout_ms` for a server
 * to create it (JFB_STATUS_NOT_FOUND after that). */
jfb_status jfb_frame_channel_open(const char * name, uint32_t timeout_ms, jfb_frame_channel ** out);

/* Bytes per direction of an opened or created channel. */
uint64_t jfb_frame_channel_capacity(const jfb_frame_channel * channel);

/* Caller: sends head || body as one request and waits for the reply. On
 * success *status is the server's status code (200, 400, 502, ...), *is_frame
 * is 1 for a Stagewire reply frame and 0 for a JSON error body, and *reply /
 * *reply_bytes stay valid until the next call or close on this handle. */
jfb_status jfb_frame_channel_call(jfb_frame_channel * channel, const void * head, uint64_t head_bytes,
                                  const void * body, uint64_t body_bytes, uint32_t timeout_ms, int32_t * status,
                                  int32_t * is_frame, const uint8_t ** reply, uint64_t * reply_bytes);

/* Server: waits up to `timeout_ms` for the next request; *frame stays valid
 * until jfb_frame_channel_reply. */
jfb_status jfb_frame_channel_receive(jfb_frame_channel * channel, uint32_t timeout_ms, const uint8_t ** frame,
                                     uint64_t * frame_bytes);

/* Server: answers the pending request with head || body. A reply larger than
 * the channel becomes a 502 JSON error body. */
jfb_status jfb_frame_channel_reply(jfb_frame_channel * channel, int32_t status, int32_t is_frame, const void * head,
                                   uint64_t head_bytes, const void * body, uint64_t body_bytes);

/* Unmaps the channel; a server's close also wakes its callers with an error
 * and removes the name. */
void jfb_frame_channel_close(jfb_frame_channel * channel);

#ifdef __cplusplus
}
#endif

#endif
