// K-quant block encoders for the synthetic package writer.
//
// Block byte layouts are the GGML K-quant formats the reference engine reads
// (sizes fixed by the JFM type table: Q2_K 256/84, Q4_K 256/144, Q6_K
// 256/210, docs/jfm-v2-format.md "Stable Tensor Types"):
//   Q4_K: f16 d, f16 dmin, 12 bytes of packed 6-bit (scale, min) pairs for
//         eight 32-element sub-blocks, 128 bytes of 4-bit codes.
//         value = d*scale_j*q - dmin*min_j.
//   Q6_K: 128 bytes low nibbles, 64 bytes high 2-bit pairs, 16 int8 scales
//         (one per 16 elements), f16 d.  value = d*scale_g*(q - 32).
//   Q2_K: 16 bytes of (scale | min << 4) nibbles (one per 16 elements),
//         64 bytes of 2-bit codes, f16 d, f16 dmin.
//         value = d*scale_g*q - dmin*min_g.
//
// The encoders are this project's own (min/max affine fit per sub-block, then
// 6-bit or 4-bit quantization of the sub-block scales); they do not reproduce
// GGML's iterative quantizers, which is fine because the packages they write
// are decoded by the same published formulas on every side. Q6_K scales use
// the whole signed int8 range the way GGML's do: each group's scale carries
// the sign that maps its largest-magnitude value to code -32 (the wide side of
// [-32, 31]), and d maps the block's largest group scale to -128.
#pragma once

#include "half.hpp"

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>

namespace jfb::kquant {

constexpr int kBlock = 256;

inline int round_clamp(float value, int lo, int hi) {
    const long r = std::lrint(value);
    return static_cast<int>(std::min<long>(hi, std::max<long>(lo, r)));
}

inline void encode_q4_k(const float * x, std::uint8_t * out) {
    float scale[8], offset[8];
    float max_scale = 0.0f, max_offset = 0.0f;
    for (int j = 0; j < 8; ++j) {
        float lo = 0.0f, hi = x[32 * j];
        for (int l = 0; l < 32; ++l) {
            lo = std::min(lo, x[32 * j + l]);
            hi = std::max(hi, x[32 * j + l]);
        }
        scale[j] = (hi - lo) / 15.0f;
        offset[j] = -lo;
        max_scale = std::max(max_scale, scale[j]);
        max_offset = std::max(max_offset, offset[j]);
    }
    const std::uint16_t d16 = float_to_half_rne(max_scale / 63.0f);
    const std::uint16_t m16 = float_to_half_rne(max_offset / 63.0f);
    const float d = half_to_float(d16), dmin = half_to_float(m16);
    int sc[8], mn[8];
    for (int j = 0; j < 8; ++j) {
        sc[j] = d > 0.0f ? round_clamp(scale[j] / d, 0, 63) : 0;
        mn[j] = dmin > 0.0f ? round_clamp(offset[j] / dmin, 0, 63) : 0;
    }
    std::memcpy(out, &d16, 2);
    std::memcpy(out + 2, &m16, 2);
    std::uint8_t * packed = out + 4;
    for (int j = 0; j < 4; ++j) {
        packed[j] = static_cast<std::uint8_t>((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
        packed[j + 4] = static_cast<std::uint8_t>((mn[j] & 63) | ((mn[j + 4] >> 4) << 6));
        packed[j + 8] = static_cast<std::uint8_t>((sc[j + 4] & 15) | ((mn[j + 4] & 15) << 4));
    }
    std::uint8_t * qs = out + 16;
    std::memset(qs, 0, 128);
    for (int e = 0; e < kBlock; ++e) {
        const int j = e / 32;
        const float step = d * static_cast<float>(sc[j]);
        const float base = dmin * static_cast<float>(mn[j]);
        const int q = step > 0.0f ? round_clamp((x[e] + base) / step, 0, 15) : 0;
        // element e = 64*c + 32*s + l lives in qs[32*c + l], nibble s
        const int c = e / 64, s = (e / 32) & 1, l = e % 32;
        qs[32 * c + l] |= static_cast<std::uint8_t>(q << (4 * s));
    }
}

inline void encode_q6_k(const float * x, std::uint8_t * out) {
    float scale[16];
    float max_scale = 0.0f;  // the signed group scale of largest magnitude
    for (int g = 0; g < 16; ++g) {
        float peak = 0.0f;
        for (int l = 0; l < 16; ++l) {
            if (std::fabs(x[16 * g + l]) > std::fabs(peak)) peak = x[16 * g + l];
        }
        scale[g] = -peak / 32.0f;
        if (std::fabs(scale[g]) > std::fabs(max_scale)) max_scale = scale[g];
    }
    const std::uint16_t d16 = float_to_half_rne(-max_scale / 128.0f);
    const float d = half_to_float(d16);
    std::uint8_t * ql = out;
    std::uint8_t * qh = out + 128;
    std::int8_t * sc = reinterpret_cast<std::int8_t *>(out + 192);
    std::memset(out, 0, 192);
    for (int g = 0; g < 16; ++g) sc[g] = static_cast<std::int8_t>(d != 0.0f ? round_clamp(scale[g] / d, -128, 127) : 0);
    for (int e = 0; e < kBlock; ++e) {
        const float step = d * static_cast<float>(sc[e / 16]);
        const int q = (step != 0.0f ? round_clamp(x[e] / step, -32, 31) : 0) + 32;
        // half h = e/128; within it e' : low nibble in ql[64h + e'%64] (nibble e'/64),
        // high two bits in qh[32h + e'%32] (bit pair e'/32)
        const int h = e / 128, r = e % 128;
        ql[64 * h + (r % 64)] |= static_cast<std::uint8_t>((q & 15) << (4 * (r / 64)));
        qh[32 * h + (r % 32)] |= static_cast<std::uint8_t>(((q >> 4) & 3) << (2 * (r / 32)));
    }
    std::memcpy(out + 208, &d16, 2);
}

inline void encode_q2_k(const float * x, std::uint8_t * out) {
    float scale[16], offset[16];
    float max_scale = 0.0f, max_offset = 0.0f;
    for (int g = 0; g < 16; ++g) {
        float lo = 0.0f, hi = x[16 * g];
        for (int l = 0; l < 16; ++l) {
            lo = std::min(lo, x[16 * g + l]);
            hi = std::max(hi, x[16 * g + l]);
        }
        scale[g] = (hi - lo) / 3.0f;
        offset[g] = -lo;
        max_scale = std::max(max_scale, scale[g]);
        max_offset = std::max(max_offset, offset[g]);
    }
    const std::uint16_t d16 = float_to_half_rne(max_scale / 15.0f);
    const std::uint16_t m16 = float_to_half_rne(max_offset / 15.0f);
    const float d = half_to_float(d16), dmin = half_to_float(m16);
    std::uint8_t * scales = out;
    std::uint8_t * qs = out + 16;
    std::memset(qs, 0, 64);
    int sc[16], mn[16];
    for (int g = 0; g < 16; ++g) {
        sc[g] = d > 0.0f ? round_clamp(scale[g] / d, 0, 15) : 0;
        mn[g] = dmin > 0.0f ? round_clamp(offset[g] / dmin, 0, 15) : 0;
        scales[g] = static_cast<std::uint8_t>(sc[g] | (mn[g] << 4));
    }
    for (int e = 0; e < kBlock; ++e) {
        const int g = e / 16;
        const float step = d * static_cast<float>(sc[g]);
        const float base = dmin * static_cast<float>(mn[g]);
        const int q = step > 0.0f ? round_clamp((x[e] + base) / step, 0, 3) : 0;
        // element e = 128*h + 32*s + l lives in qs[32*h + l], bit pair s
        const int h = e / 128, s = (e % 128) / 32, l = e % 32;
        qs[32 * h + l] |= static_cast<std::uint8_t>(q << (2 * s));
    }
    std::memcpy(out + 80, &d16, 2);
    std::memcpy(out + 82, &m16, 2);
}

}  // namespace jfb::kquant
