// CRC-32 of device buffers and the Stagewire v2 checksum field, on the device.
//
// Stagewire v2 (the reference's docs/stagewire-v2.md; internal/stagewire/
// frame.go:157-227) carries every stage payload with its CRC-32 (IEEE 802.3,
// the reflected polynomial 0xEDB88320, as Go's crc32.ChecksumIEEE and zlib's
// crc32 compute it) in the frame metadata, and a receiver rejects a payload
// whose checksum differs. Over NVLink the payload never visits the host, so
// the checksum is formed where the bytes are.
//
// Method (the published linearity of CRCs, as in zlib's crc32_combine): with
// F(s, data) the register after feeding `data` from register value s,
//   F(0, A || B) = x^(8 |B|) * F(0, A) xor F(0, B)      (mod P)
//   crc(data)    = ~(F(0, data) xor x^(8 |data|) * 0xFFFFFFFF)
// where products are of polynomials modulo P in the reflected representation
// (bit 31 is x^0). Every thread feeds one chunk (64 B to 1 KiB, a multiple of
// 16) from register 0 with a byte table in shared memory; blocks then join 256 consecutive items at a
// time in a tree, item lengths known, until one item is left, whose register
// becomes the CRC. x^(8n) comes from a host table of x^(8 * 2^j).
#include "common.cuh"
#include "jfb/jfb_stagewire.h"

#include <algorithm>

namespace jfb {
namespace {

constexpr uint32_t kCrcPoly = 0xEDB88320u;
constexpr uint64_t kCrcChunkMin = 64;    // bytes fed by one thread: 64 B for small inputs
constexpr uint64_t kCrcChunkMax = 1024;  // ... growing to 1 KiB once ~148 x 2048 threads are busy
constexpr uint64_t kCrcTargetItems = 148ull * 2048;
constexpr int kCrcThreads = 256;      // items joined per block
constexpr int kCrcPowers = 48;        // x^(8 * 2^j), j < 48: lengths below 2^48 bytes

struct CrcPowers {
    uint32_t x[kCrcPowers];
};

// a * b mod P, reflected polynomials (bit 31 = x^0)
__host__ __device__ inline uint32_t crc_mulmod(uint32_t a, uint32_t b) {
    uint32_t p = 0;
    for (int i = 0; i < 32; ++i) {
        if (a & (0x80000000u >> i)) p ^= b;
        b = (b & 1u) ? (b >> 1) ^ kCrcPoly : b >> 1;
    }
    return p;
}

// x^(8 n) mod P
__host__ __device__ inline uint32_t crc_xpow_bytes(uint64_t n, const CrcPowers & pw) {
    uint32_t r = 0x80000000u;  // x^0
    for (int j = 0; n != 0 && j < kCrcPowers; ++j, n >>= 1) {
        if (n & 1u) r = crc_mulmod(r, pw.x[j]);
    }
    return r;
}

__host__ inline CrcPowers crc_powers() {
    CrcPowers pw;
    pw.x[0] = 0x00800000u;  // x^8
    for (int j = 1; j < kCrcPowers; ++j) pw.x[j] = crc_mulmod(pw.x[j - 1], pw.x[j - 1]);
    return pw;
}

// Per join level, computed on the host: x^(8 item_bytes 2^s) for the
// tree's eight steps (every right-hand subtree but the one holding the
// ragged last item is that long), and 0xFFFFFFFF * x^(8 total) for the finish.
struct CrcJoinPowers {
    uint32_t step[8];
    uint32_t fin;
};

// Joins the block's 256 registers reg[] (item lengths len[], all
// `item_bytes` but a ragged last one, 0 past the end) in a tree; reg[0] ends
// as the register after all of them. Every thread of the block calls it.
__device__ inline void crc_join_block(uint32_t * reg, uint64_t * len, uint64_t item_bytes, const CrcPowers & pw,
                                      const CrcJoinPowers & jp) {
    __syncthreads();
    for (int s = 0, step = 1; step < kCrcThreads; ++s, step *= 2) {
        if ((threadIdx.x % (2 * step)) == 0) {
            const uint64_t lb = len[threadIdx.x + step];
            if (lb != 0) {
                const uint32_t xp = lb == (item_bytes << s) ? jp.step[s] : crc_xpow_bytes(lb, pw);
                reg[threadIdx.x] = crc_mulmod(reg[threadIdx.x], xp) ^ reg[threadIdx.x + step];
                len[threadIdx.x] += lb;
            }
        }
        __syncthreads();
    }
}

// Feeds each `chunk`-byte piece from register 0 (one per thread), then joins
// the block's 256 pieces: out[b] is the register after the block's bytes, or,
// with `finish` (a single block), the CRC of all `n` bytes in *crc_out.
__global__ void __launch_bounds__(kCrcThreads) crc_chunks_kernel(const uint8_t * __restrict__ data, uint64_t n,
                                                               uint64_t chunk, uint32_t * __restrict__ out,
                                                               CrcPowers pw, CrcJoinPowers jp, int finish,
                                                               uint32_t * __restrict__ crc_out) {
    __shared__ uint32_t table[256];
    __shared__ uint32_t reg[kCrcThreads];
    __shared__ uint64_t len[kCrcThreads];
    pdl_trigger();
    for (uint32_t i = threadIdx.x; i < 256; i += blockDim.x) {
        uint32_t c = i;
        for (int k = 0; k < 8; ++k) c = (c & 1u) ? (c >> 1) ^ kCrcPoly : c >> 1;
        table[i] = c;
    }
    __syncthreads();
    pdl_wait();
    const uint64_t item = uint64_t(blockIdx.x) * kCrcThreads + threadIdx.x;
    const uint64_t begin = item * chunk;
    uint32_t s = 0;
    uint64_t bytes = 0;
    if (begin < n) {
        const uint64_t end = begin + chunk < n ? begin + chunk : n;
        bytes = end - begin;
        uint64_t i = begin;
        // 16-byte loads where the address allows (payload buffers are 256-byte aligned)
        if ((reinterpret_cast<uintptr_t>(data + i) & 15u) == 0) {
            for (; i + 16 <= end; i += 16) {
                const uint4 v = *reinterpret_cast<const uint4 *>(data + i);
                const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int k = 0; k < 4; ++k) {
#pragma unroll
                    for (int b = 0; b < 4; ++b) s = (s >> 8) ^ table[(s ^ (w[k] >> (8 * b))) & 0xffu];
                }
            }
        }
        for (; i < end; ++i) s = (s >> 8) ^ table[(s ^ data[i]) & 0xffu];
    }
    reg[threadIdx.x] = s;
    len[threadIdx.x] = bytes;
    crc_join_block(reg, len, chunk, pw, jp);
    if (threadIdx.x == 0) {
        if (finish) *crc_out = ~(reg[0] ^ jp.fin);
        else out[blockIdx.x] = reg[0];
    }
}

// Joins `count` consecutive items (each `item_bytes` long, the last one
// `last_bytes`) 256 at a time: output item b is the register after items
// [256 b, 256 b + 256). With `finish`, the single output becomes the CRC of
// all the bytes and is written to `crc_out`.
__global__ void __launch_bounds__(kCrcThreads) crc_join_kernel(const uint32_t * __restrict__ in, uint64_t count,
                                                             uint64_t item_bytes, uint64_t last_bytes,
                                                             uint32_t * __restrict__ out, CrcPowers pw,
                                                             CrcJoinPowers jp, int finish,
                                                             uint32_t * __restrict__ crc_out) {
    __shared__ uint32_t reg[kCrcThreads];
    __shared__ uint64_t len[kCrcThreads];
    pdl_trigger();
    pdl_wait();
    const uint64_t i = uint64_t(blockIdx.x) * kCrcThreads + threadIdx.x;
    reg[threadIdx.x] = i < count ? in[i] : 0u;
    len[threadIdx.x] = i < count ? (i + 1 == count ? last_bytes : item_bytes) : 0u;
    crc_join_block(reg, len, item_bytes, pw, jp);
    if (threadIdx.x == 0) {
        if (finish) *crc_out = ~(reg[0] ^ jp.fin);
        else out[blockIdx.x] = reg[0];
    }
}

// The CRC of zero bytes.
__global__ void crc_empty_kernel(uint32_t * crc_out) {
    pdl_trigger();
    pdl_wait();
    if (threadIdx.x == 0) *crc_out = 0u;
}

// The 10-character checksum field of a frame's metadata: the decimal value,
// right-aligned with leading spaces (whitespace the JSON grammar allows).
__global__ void stamp_kernel(const uint32_t * __restrict__ crc, uint8_t * __restrict__ frame, uint32_t offset) {
    pdl_trigger();
    pdl_wait();
    if (threadIdx.x != 0) return;
    uint32_t v = *crc;
    for (int k = JFB_STAGEWIRE_CRC_FIELD - 1; k >= 0; --k) {
        if (v != 0 || k == JFB_STAGEWIRE_CRC_FIELD - 1) {
            frame[offset + k] = uint8_t('0' + v % 10);
            v /= 10;
        } else {
            frame[offset + k] = uint8_t(' ');
        }
    }
}

// Compares the checksum field of a received frame with the CRC of the
// received payload; a difference (or a malformed field) sets *mismatch.
__global__ void check_kernel(const uint32_t * __restrict__ crc, const uint8_t * __restrict__ frame, uint32_t offset,
                             int32_t * __restrict__ mismatch) {
    pdl_trigger();
    pdl_wait();
    if (threadIdx.x != 0) return;
    uint64_t v = 0;
    bool digits = false, bad = false;
    for (int k = 0; k < JFB_STAGEWIRE_CRC_FIELD; ++k) {
        const uint8_t ch = frame[offset + k];
        if (ch == ' ' && !digits) continue;
        if (ch < '0' || ch > '9') {
            bad = true;
            break;
        }
        digits = true;
        v = v * 10 + (ch - '0');
    }
    if (bad || !digits || v != uint64_t(*crc)) *mismatch = 1;
}

uint64_t crc_chunk_bytes(uint64_t n) {
    const uint64_t c = ((n + kCrcTargetItems - 1) / kCrcTargetItems + 15) / 16 * 16;
    return std::min(kCrcChunkMax, std::max(kCrcChunkMin, c));
}

uint64_t crc_items_total(uint64_t n) {
    const uint64_t chunk = crc_chunk_bytes(n);
    uint64_t items = (n + chunk - 1) / chunk, total = 0;
    while (items > 1) {
        total += items;
        items = (items + kCrcThreads - 1) / kCrcThreads;
    }
    return total + 1;
}

}  // namespace
}  // namespace jfb

using namespace jfb;

extern "C" uint64_t jfb_crc32_scratch_bytes(uint64_t n) { return crc_items_total(n) * sizeof(uint32_t) + 256; }

extern "C" jfb_status jfb_crc32(const void * data, uint64_t n, uint32_t * crc_out, void * scratch,
                                uint64_t scratch_bytes, void * stream) {
    if (crc_out == nullptr || (n > 0 && (data == nullptr || scratch == nullptr))) {
        return status_error(JFB_STATUS_INVALID_ARGUMENT, "crc32 needs data, scratch and an output word");
    }
    if (n >= (uint64_t(1) << kCrcPowers)) return status_error(JFB_STATUS_INVALID_ARGUMENT, "crc32 input is too long");
    cudaStream_t s = as_stream(stream);
    cudaError_t e;
    if (n == 0) {
        e = launch_k(crc_empty_kernel, dim3(1), dim3(32), 0, s, crc_out);
        if (e != cudaSuccess) return status_error(JFB_STATUS_CUDA_ERROR, "jfb_crc32: %s", cudaGetErrorString(e));
        return launch_status("jfb_crc32");
    }
    if (scratch_bytes < jfb_crc32_scratch_bytes(n)) {
        return status_error(JFB_STATUS_INVALID_ARGUMENT, "crc32 scratch is too small");
    }
    static const CrcPowers pw = crc_powers();
    uint32_t * buf = static_cast<uint32_t *>(scratch);
    const uint64_t chunk = crc_chunk_bytes(n);
    uint64_t items = (n + chunk - 1) / chunk;
    const uint64_t blocks0 = (items + kCrcThreads - 1) / kCrcThreads;
    if (blocks0 > 0x7fffffffu) return status_error(JFB_STATUS_INVALID_ARGUMENT, "crc32 input is too long");
    auto join_powers = [&](uint64_t item_bytes, int finish) {
        CrcJoinPowers jp;
        for (int k = 0; k < 8; ++k) jp.step[k] = crc_xpow_bytes(item_bytes << k, pw);
        jp.fin = finish ? crc_mulmod(0xFFFFFFFFu, crc_xpow_bytes(n, pw)) : 0u;
        return jp;
    };
    // chunks and their first join in one launch; one block finishes at once
    const int finish0 = blocks0 == 1 ? 1 : 0;
    e = launch_k(crc_chunks_kernel, dim3(uint32_t(blocks0)), dim3(kCrcThreads), 0, s, static_cast<const uint8_t *>(data),
                 n, chunk, buf, pw, join_powers(chunk, finish0), finish0, crc_out);
    if (e != cudaSuccess) return status_error(JFB_STATUS_CUDA_ERROR, "jfb_crc32: %s", cudaGetErrorString(e));
    if (finish0) return launch_status("jfb_crc32");
    items = blocks0;
    uint64_t item_bytes = chunk * kCrcThreads, last_bytes = n - (blocks0 - 1) * chunk * kCrcThreads;
    uint32_t * in = buf;
    // each level joins 256 items; the last level (one block) finishes
    while (e == cudaSuccess) {
        const uint64_t blocks = (items + kCrcThreads - 1) / kCrcThreads;
        uint32_t * out = in + items;
        const int finish = blocks == 1 ? 1 : 0;
        e = launch_k(crc_join_kernel, dim3(uint32_t(blocks)), dim3(kCrcThreads), 0, s, static_cast<const uint32_t *>(in),
                     items, item_bytes, last_bytes, out, pw, join_powers(item_bytes, finish), finish, crc_out);
        if (finish) break;
        // the joined items: full ones of 256 items, the last of the remainder
        const uint64_t full_bytes = item_bytes * kCrcThreads;
        last_bytes = n - (blocks - 1) * full_bytes;
        item_bytes = full_bytes;
        items = blocks;
        in = out;
    }
    if (e != cudaSuccess) return status_error(JFB_STATUS_CUDA_ERROR, "jfb_crc32: %s", cudaGetErrorString(e));
    return launch_status("jfb_crc32");
}

extern "C" jfb_status jfb_stagewire_stamp_crc(const uint32_t * crc, uint8_t * frame, uint32_t field_offset,
                                              void * stream) {
    if (crc == nullptr || frame == nullptr) return status_error(JFB_STATUS_INVALID_ARGUMENT, "crc and frame are required");
    const cudaError_t e = launch_k(stamp_kernel, dim3(1), dim3(32), 0, as_stream(stream), crc, frame, field_offset);
    if (e != cudaSuccess) return status_error(JFB_STATUS_CUDA_ERROR, "jfb_stagewire_stamp_crc: %s", cudaGetErrorString(e));
    return launch_status("jfb_stagewire_stamp_crc");
}

extern "C" jfb_status jfb_stagewire_check_crc(const uint32_t * crc, const uint8_t * frame, uint32_t field_offset,
                                              int32_t * mismatch, void * stream) {
    if (crc == nullptr || frame == nullptr || mismatch == nullptr) {
        return status_error(JFB_STATUS_INVALID_ARGUMENT, "crc, frame and the mismatch word are required");
    }
    const cudaError_t e = launch_k(check_kernel, dim3(1), dim3(32), 0, as_stream(stream), crc, frame, field_offset,
                                   mismatch);
    if (e != cudaSuccess) return status_error(JFB_STATUS_CUDA_ERROR, "jfb_stagewire_check_crc: %s", cudaGetErrorString(e));
    return launch_status("jfb_stagewire_check_crc");
}
