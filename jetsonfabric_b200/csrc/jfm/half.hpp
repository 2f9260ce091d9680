// IEEE 754 binary16 <-> binary32 conversion on the host, round to nearest
// even. Written from the binary16 definition (IEEE 754-2008 section 3.6); the
// GPU side uses the hardware conversions (__float2half_rn), which follow the
// same rounding, so host-encoded K-quant scales and device-side conversions
// agree bit for bit.
#pragma once

#include <cstdint>
#include <cstring>

namespace jfb {

inline std::uint32_t float_bits(float value) {
    std::uint32_t bits;
    std::memcpy(&bits, &value, sizeof(bits));
    return bits;
}

inline float bits_float(std::uint32_t bits) {
    float value;
    std::memcpy(&value, &bits, sizeof(value));
    return value;
}

inline std::uint16_t float_to_half_rne(float value) {
    const std::uint32_t x = float_bits(value);
    const std::uint16_t sign = static_cast<std::uint16_t>((x >> 16) & 0x8000u);
    const std::uint32_t biased = (x >> 23) & 0xffu;
    std::uint32_t frac = x & 0x7fffffu;
    if (biased == 0xffu) {  // inf / nan (nan keeps its top payload bits, made quiet)
        return static_cast<std::uint16_t>(sign | 0x7c00u | (frac != 0 ? (0x200u | (frac >> 13)) : 0u));
    }
    const int exponent = static_cast<int>(biased) - 127;
    if (exponent > 15) return static_cast<std::uint16_t>(sign | 0x7c00u);
    if (exponent >= -14) {  // normal half
        std::uint32_t half = (static_cast<std::uint32_t>(exponent + 15) << 10) | (frac >> 13);
        const std::uint32_t rest = frac & 0x1fffu;
        if (rest > 0x1000u || (rest == 0x1000u && (half & 1u))) ++half;  // may carry into inf: correct
        return static_cast<std::uint16_t>(sign | half);
    }
    if (exponent < -25) return sign;  // rounds to zero
    // subnormal half: value = frac' * 2^-24
    frac |= 0x800000u;
    const int shift = -exponent - 1;  // 14..24 -> bits dropped = 13 + (-14 - exponent)
    const unsigned drop = static_cast<unsigned>(13 + (-14 - exponent));
    (void) shift;
    std::uint32_t half = frac >> drop;
    const std::uint32_t rest = frac & ((1u << drop) - 1u);
    const std::uint32_t halfway = 1u << (drop - 1u);
    if (rest > halfway || (rest == halfway && (half & 1u))) ++half;
    return static_cast<std::uint16_t>(sign | half);
}

inline float half_to_float(std::uint16_t h) {
    const std::uint32_t sign = static_cast<std::uint32_t>(h & 0x8000u) << 16;
    const std::uint32_t exponent = (h >> 10) & 0x1fu;
    std::uint32_t frac = h & 0x3ffu;
    if (exponent == 0x1fu) return bits_float(sign | 0x7f800000u | (frac << 13));
    if (exponent != 0) return bits_float(sign | ((exponent + 112u) << 23) | (frac << 13));
    if (frac == 0) return bits_float(sign);
    int e = -14;
    while ((frac & 0x400u) == 0) {
        frac <<= 1;
        --e;
    }
    return bits_float(sign | (static_cast<std::uint32_t>(e + 127) << 23) | ((frac & 0x3ffu) << 13));
}

}  // namespace jfb
