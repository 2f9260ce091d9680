/*
 * CPU ORACLE — TEST INFRASTRUCTURE ONLY (see qwen2_oracle.h).
 *
 * Restates, in plain C with OpenMP, what the reference computes when its
 * native engine runs a Qwen2 stage on GGML's CPU backend:
 *   graph  runtime/engines/native/src/qwen2_architecture.cpp:522-598 (build),
 *          386-470 (attention), 499-506 (NEOX RoPE), 508-520 (feed forward),
 *          584-597 (output head), 697-747 (mask, cache indices),
 *          1056-1092 (F16 KV cache), 818-823/1029-1054 (session positions);
 *   ops    GGML-CPU semantics at llama.cpp bf2c86dd (third-party, not
 *          vendored): restated from the published K-quant block formats and
 *          op definitions, each at its use site below.
 *
 * Compiled with -ffp-contract=off so that every float expression rounds as
 * written (no fused multiply-add), which keeps the dequantizer bit-exact with
 * gguf-py's NumPy dequantizers.
 */
#include "qwen2_oracle.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <immintrin.h>
#ifdef _OPENMP
#include <omp.h>
#endif

enum { QK = 256 };
enum { T_F32 = 1, T_F16 = 2, T_Q2_K = 9, T_Q4_K = 11, T_Q6_K = 13 };

typedef struct q8k_block {
    float d;
    int8_t qs[QK];
    int16_t bsums[QK / 16];
} q8k_block;

void orc_set_threads(int threads) {
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#else
    (void) threads;
#endif
}

/* ---- exp ------------------------------------------------------------------
 * exp(x) by Cody-Waite argument reduction (x = n ln2 + r, ln2 split in a
 * short high part and a correction) and the degree-7 Taylor polynomial of
 * e^r in Horner form with fused multiply-adds, then an exact two-step scaling
 * by 2^n. Used for softmax and SiLU. The device kernels evaluate this same
 * restatement step for step (exp_cw in the kernels' common header), so both
 * produce identical bits (fmaf, rintf and the float multiplications are
 * correctly rounded on both). */
static float bitsf(uint32_t u);
static float pow2i(int e) { return bitsf((uint32_t) (e + 127) << 23); }  /* 2^e, -126 <= e <= 127 */

float orc_expf(float x) {
    if (x != x) return x;
    if (x > 88.72283935546875f) return INFINITY;
    if (x < -103.972084045410156f) return 0.0f;
    const float n = rintf(x * 1.44269502162933349609375f);
    float r = fmaf(-n, 0.693145751953125f, x);
    r = fmaf(-n, 1.4286068203094172e-06f, r);
    float p = 1.98412701138295233e-04f;            /* 1/7! */
    p = fmaf(p, r, 1.38888892251998186e-03f);      /* 1/6! */
    p = fmaf(p, r, 8.33333376795053482e-03f);      /* 1/5! */
    p = fmaf(p, r, 4.16666679084300995e-02f);      /* 1/4! */
    p = fmaf(p, r, 1.66666671633720398e-01f);      /* 1/3! */
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    const int e = (int) n;
    const int e1 = e / 2, e2 = e - e1;
    return (p * pow2i(e1)) * pow2i(e2);
}

/* ---- binary16 (IEEE 754, round to nearest even) ------------------------ */

static uint32_t fbits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static float bitsf(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* GGML_FP32_TO_FP16 is a round-to-nearest-even conversion (F16C vcvtps2ph
 * with imm 0 on x86); NaN handling is irrelevant here (no NaNs reach it). */
uint16_t orc_f32_to_f16(float value) {
    const uint32_t x = fbits(value);
    const uint16_t sign = (uint16_t) ((x >> 16) & 0x8000u);
    const uint32_t be = (x >> 23) & 0xffu;
    uint32_t frac = x & 0x7fffffu;
    if (be == 0xffu) return (uint16_t) (sign | 0x7c00u | (frac ? 0x200u | (frac >> 13) : 0u));
    const int e = (int) be - 127;
    if (e > 15) return (uint16_t) (sign | 0x7c00u);
    if (e >= -14) {
        uint32_t h = ((uint32_t) (e + 15) << 10) | (frac >> 13);
        const uint32_t rest = frac & 0x1fffu;
        if (rest > 0x1000u || (rest == 0x1000u && (h & 1u))) ++h;
        return (uint16_t) (sign | h);
    }
    if (e < -25) return sign;
    frac |= 0x800000u;
    const unsigned drop = (unsigned) (13 + (-14 - e));
    uint32_t h = frac >> drop;
    const uint32_t rest = frac & ((1u << drop) - 1u), half = 1u << (drop - 1u);
    if (rest > half || (rest == half && (h & 1u))) ++h;
    return (uint16_t) (sign | h);
}

float orc_f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t) (h & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 0x1fu;
    uint32_t m = h & 0x3ffu;
    if (e == 0x1fu) return bitsf(sign | 0x7f800000u | (m << 13));
    if (e) return bitsf(sign | ((e + 112u) << 23) | (m << 13));
    if (!m) return bitsf(sign);
    int ex = -14;
    while (!(m & 0x400u)) { m <<= 1; --ex; }
    return bitsf(sign | ((uint32_t) (ex + 127) << 23) | ((m & 0x3ffu) << 13));
}

/* The reference activation codec (runtime/activation/builtin_activation_codecs.cpp
 * :51-106): round to nearest even, NaN keeps its top payload bits plus the
 * quiet bit, overflow saturates to infinity, tiny values flush to signed zero. */
uint16_t orc_codec_float_to_half(float value) {
    const uint32_t bits = fbits(value);
    const uint16_t sign = (uint16_t) ((bits >> 16) & 0x8000u);
    const uint32_t exponent = (bits >> 23) & 0xffu;
    uint32_t mantissa = bits & 0x7fffffu;
    if (exponent == 0xffu) {
        if (mantissa == 0) return (uint16_t) (sign | 0x7c00u);
        return (uint16_t) (sign | 0x7c00u | (mantissa >> 13) | 0x0200u);
    }
    int he = (int) exponent - 127 + 15;
    if (he >= 31) return (uint16_t) (sign | 0x7c00u);
    if (he <= 0) {
        if (he < -10) return sign;
        mantissa |= 0x800000u;
        const unsigned shift = (unsigned) (14 - he);
        uint32_t hm = mantissa >> shift;
        const uint32_t rem = mantissa & ((1u << shift) - 1u), halfway = 1u << (shift - 1u);
        if (rem > halfway || (rem == halfway && (hm & 1u))) ++hm;
        return (uint16_t) (sign | hm);
    }
    uint32_t hm = mantissa >> 13;
    const uint32_t rem = mantissa & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (hm & 1u))) {
        ++hm;
        if (hm == 0x400u) {
            hm = 0;
            ++he;
            if (he >= 31) return (uint16_t) (sign | 0x7c00u);
        }
    }
    return (uint16_t) (sign | ((uint16_t) he << 10) | (uint16_t) hm);
}

/* builtin_activation_codecs.cpp:108-137: exact widening, NaN payload kept. */
float orc_codec_half_to_float(uint16_t value) { return orc_f16_to_f32(value); }

/* ---- K-quant dequantization ---------------------------------------------
 * GGML dequantize_row_{q2_K,q4_K,q6_K}; the arithmetic order follows the
 * published formulas (also gguf-py quants.py Q2_K/Q4_K/Q6_K.dequantize_blocks):
 * (d*scale)*q - (dmin*min), each product rounded to float. */

static void q4k_scale_min(const uint8_t * s, int j, int * sc, int * m) {
    if (j < 4) {
        *sc = s[j] & 63;
        *m = s[j + 4] & 63;
    } else {
        *sc = (s[j + 4] & 0x0f) | ((s[j - 4] >> 6) << 4);
        *m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

static void dequant_q4_k(const uint8_t * b, float * y) {
    uint16_t hd, hm;
    memcpy(&hd, b, 2);
    memcpy(&hm, b + 2, 2);
    const float d = orc_f16_to_f32(hd), dmin = orc_f16_to_f32(hm);
    const uint8_t * qs = b + 16;
    for (int j = 0; j < 8; ++j) {
        int sc, m;
        q4k_scale_min(b + 4, j, &sc, &m);
        const float d1 = d * (float) sc, m1 = dmin * (float) m;
        const int c = j / 2, shift = 4 * (j & 1);
        for (int l = 0; l < 32; ++l) {
            const float q = (float) ((qs[32 * c + l] >> shift) & 15);
            const float p = d1 * q;
            y[32 * j + l] = p - m1;
        }
    }
}

static int q6k_code(const uint8_t * b, int e) {
    const uint8_t * ql = b;
    const uint8_t * qh = b + 128;
    const int h = e / 128, r = e % 128;
    const int lo = (ql[64 * h + (r % 64)] >> (4 * (r / 64))) & 15;
    const int hi = (qh[32 * h + (r % 32)] >> (2 * (r / 32))) & 3;
    return (lo | (hi << 4)) - 32;
}

static void dequant_q6_k(const uint8_t * b, float * y) {
    uint16_t hd;
    memcpy(&hd, b + 208, 2);
    const float d = orc_f16_to_f32(hd);
    const int8_t * sc = (const int8_t *) (b + 192);
    for (int e = 0; e < QK; ++e) {
        const float ds = d * (float) sc[e / 16];
        y[e] = ds * (float) q6k_code(b, e);
    }
}

static int q2k_code(const uint8_t * b, int e) {
    const uint8_t * qs = b + 16;
    const int h = e / 128, s = (e % 128) / 32, l = e % 32;
    return (qs[32 * h + l] >> (2 * s)) & 3;
}

static void dequant_q2_k(const uint8_t * b, float * y) {
    uint16_t hd, hm;
    memcpy(&hd, b + 80, 2);
    memcpy(&hm, b + 82, 2);
    const float d = orc_f16_to_f32(hd), dmin = orc_f16_to_f32(hm);
    for (int e = 0; e < QK; ++e) {
        const uint8_t s = b[e / 16];
        const float dl = d * (float) (s & 15), ml = dmin * (float) (s >> 4);
        const float p = dl * (float) q2k_code(b, e);
        y[e] = p - ml;
    }
}

static size_t block_bytes(uint32_t type) {
    switch (type) {
    case T_Q2_K: return 84;
    case T_Q4_K: return 144;
    case T_Q6_K: return 210;
    default: return 0;
    }
}

void orc_dequantize_row(uint32_t type, const void * src, float * dst, int64_t k) {
    const uint8_t * p = src;
    switch (type) {
    case T_F32: memcpy(dst, src, (size_t) k * 4); return;
    case T_F16:
        for (int64_t i = 0; i < k; ++i) {
            uint16_t h;
            memcpy(&h, p + 2 * i, 2);
            dst[i] = orc_f16_to_f32(h);
        }
        return;
    case T_Q4_K: for (int64_t b = 0; b < k / QK; ++b) dequant_q4_k(p + 144 * b, dst + QK * b); return;
    case T_Q6_K: for (int64_t b = 0; b < k / QK; ++b) dequant_q6_k(p + 210 * b, dst + QK * b); return;
    case T_Q2_K: for (int64_t b = 0; b < k / QK; ++b) dequant_q2_k(p + 84 * b, dst + QK * b); return;
    default: memset(dst, 0, (size_t) k * 4); return;
    }
}

/* ---- Q8_K activation quantization ----------------------------------------
 * GGML-CPU converts the f32 src1 of every K-quant mul_mat to the weight's
 * vec_dot_type, which is Q8_K for Q2_K/Q4_K/Q6_K (quantize_row_q8_K_ref):
 * per 256 values, max = the signed value of largest magnitude (first one on
 * ties), iscale = -127/max, q = round-half-even(iscale*x) capped at 127,
 * d = 1/iscale, bsums = sums of 16 consecutive q. */
void orc_quantize_row_q8_k(const float * x, void * blocks, int64_t k) {
    q8k_block * y = blocks;
    for (int64_t b = 0; b < k / QK; ++b, x += QK) {
        float amax = 0.0f, max = 0.0f;
        for (int j = 0; j < QK; ++j) {
            const float ax = fabsf(x[j]);
            if (ax > amax) { amax = ax; max = x[j]; }
        }
        if (amax == 0.0f) {
            y[b].d = 0.0f;
            memset(y[b].qs, 0, sizeof(y[b].qs));
            memset(y[b].bsums, 0, sizeof(y[b].bsums));
            continue;
        }
        const float iscale = -127.0f / max;
        for (int j = 0; j < QK; ++j) {
            const long v = lrintf(iscale * x[j]);
            y[b].qs[j] = (int8_t) (v < 127 ? v : 127);
        }
        for (int g = 0; g < QK / 16; ++g) {
            int sum = 0;
            for (int l = 0; l < 16; ++l) sum += y[b].qs[16 * g + l];
            y[b].bsums[g] = (int16_t) sum;
        }
        y[b].d = 1.0f / iscale;
    }
}

/* ---- K-quant x Q8_K dot products -----------------------------------------
 * ggml_vec_dot_{q2_K,q4_K,q6_K}_q8_K: exact integer sums per sub-block,
 * scaled by the 6/4-bit sub-block scales, then one float scale per 256-block:
 *   sum += (d_w*d_a)*isum - (dmin_w*d_a)*msum. */

/* The per-block contributions are rounded to float exactly as written and
 * summed in double, which makes the row result independent of the order in
 * which blocks are added (the double sum of up to a few hundred floats is
 * exact or off by far less than a float ulp), so a GPU reduction in any order
 * reproduces it bit for bit. */
static float dot_q4_k(const uint8_t * w, const q8k_block * a, int64_t nb) {
    double sum = 0.0;
    for (int64_t b = 0; b < nb; ++b, w += 144) {
        const uint8_t * qs = w + 16;
        int32_t isum = 0, msum = 0;
        for (int j = 0; j < 8; ++j) {
            int sc, m;
            q4k_scale_min(w + 4, j, &sc, &m);
            const int c = j / 2, shift = 4 * (j & 1);
            int32_t s = 0;
            for (int l = 0; l < 32; ++l) s += ((qs[32 * c + l] >> shift) & 15) * a[b].qs[32 * j + l];
            isum += sc * s;
            msum += m * (a[b].bsums[2 * j] + a[b].bsums[2 * j + 1]);
        }
        uint16_t hd, hm;
        memcpy(&hd, w, 2);
        memcpy(&hm, w + 2, 2);
        const float d = orc_f16_to_f32(hd) * a[b].d;
        const float dmin = orc_f16_to_f32(hm) * a[b].d;
        const float c = d * (float) isum - dmin * (float) msum;
        sum += (double) c;
    }
    return (float) sum;
}

static float dot_q6_k(const uint8_t * w, const q8k_block * a, int64_t nb) {
    double sum = 0.0;
    for (int64_t b = 0; b < nb; ++b, w += 210) {
        const int8_t * sc = (const int8_t *) (w + 192);
        int32_t isum = 0;
        for (int g = 0; g < 16; ++g) {
            int32_t s = 0;
            for (int l = 0; l < 16; ++l) s += q6k_code(w, 16 * g + l) * a[b].qs[16 * g + l];
            isum += sc[g] * s;
        }
        uint16_t hd;
        memcpy(&hd, w + 208, 2);
        const float c = (orc_f16_to_f32(hd) * a[b].d) * (float) isum;
        sum += (double) c;
    }
    return (float) sum;
}

static float dot_q2_k(const uint8_t * w, const q8k_block * a, int64_t nb) {
    double sum = 0.0;
    for (int64_t b = 0; b < nb; ++b, w += 84) {
        int32_t isum = 0, msum = 0;
        for (int g = 0; g < 16; ++g) {
            int32_t s = 0;
            for (int l = 0; l < 16; ++l) s += q2k_code(w, 16 * g + l) * a[b].qs[16 * g + l];
            isum += (w[g] & 15) * s;
            msum += (w[g] >> 4) * a[b].bsums[g];
        }
        uint16_t hd, hm;
        memcpy(&hd, w + 80, 2);
        memcpy(&hm, w + 82, 2);
        const float d = orc_f16_to_f32(hd) * a[b].d;
        const float dmin = orc_f16_to_f32(hm) * a[b].d;
        const float c = d * (float) isum - dmin * (float) msum;
        sum += (double) c;
    }
    return (float) sum;
}

/* ---- the same dot products, vectorised ------------------------------------
 * orc_matmul unpacks each weight row once into codes in element order (Q4_K
 * and Q2_K codes as stored, Q6_K codes + 32, all in [0, 63]) with one scale
 * and one min per 16-value group, then forms every integer sub-block sum with
 * AVX2 byte products. Integer sums are exact in any order, so isum and msum
 * equal the scalar loops' values above (dot_q{4,6,2}_k, kept as the readable
 * statement and checked against this path by tests/test_oracle.py); the float
 * block terms are then rounded and summed exactly as there. */
typedef struct unpacked_row {
    uint8_t * codes;  /* [nb * 256], 32-byte aligned */
    int16_t * scale;  /* [nb * 16] per 16-value group */
    int16_t * min;    /* [nb * 16] (Q4_K, Q2_K) */
    float * d;        /* [nb] */
    float * dmin;     /* [nb] (Q4_K, Q2_K) */
} unpacked_row;

static void unpack_row(uint32_t type, const uint8_t * w, int64_t nb, unpacked_row * u) {
    const __m256i lo4 = _mm256_set1_epi8(0x0f), lo2 = _mm256_set1_epi8(0x03);
    for (int64_t b = 0; b < nb; ++b) {
        uint8_t * c = u->codes + 256 * b;
        int16_t * sc = u->scale + 16 * b, * mn = u->min + 16 * b;
        uint16_t hd, hm;
        if (type == T_Q4_K) {
            const uint8_t * blk = w + 144 * b;
            memcpy(&hd, blk, 2);
            memcpy(&hm, blk + 2, 2);
            for (int j = 0; j < 8; ++j) {
                int s, m;
                q4k_scale_min(blk + 4, j, &s, &m);
                sc[2 * j] = sc[2 * j + 1] = (int16_t) s;
                mn[2 * j] = mn[2 * j + 1] = (int16_t) m;
            }
            /* element 64c + l (l < 32): low nibble of qs[32c + l]; 64c + 32 + l: high nibble */
            for (int q = 0; q < 4; ++q) {
                const __m256i x = _mm256_loadu_si256((const __m256i *) (blk + 16 + 32 * q));
                _mm256_store_si256((__m256i *) (c + 64 * q), _mm256_and_si256(x, lo4));
                _mm256_store_si256((__m256i *) (c + 64 * q + 32), _mm256_and_si256(_mm256_srli_epi16(x, 4), lo4));
            }
            u->d[b] = orc_f16_to_f32(hd);
            u->dmin[b] = orc_f16_to_f32(hm);
        } else if (type == T_Q6_K) {
            const uint8_t * blk = w + 210 * b;
            memcpy(&hd, blk + 208, 2);
            for (int g = 0; g < 16; ++g) {
                sc[g] = (int16_t) (int8_t) blk[192 + g];
                mn[g] = 0;
            }
            /* element 128h + r: low nibble (r / 64) of ql[64h + r % 64], bits 2 (r / 32) of qh[32h + r % 32] */
            for (int h = 0; h < 2; ++h) {
                const __m256i l0 = _mm256_loadu_si256((const __m256i *) (blk + 64 * h));
                const __m256i l1 = _mm256_loadu_si256((const __m256i *) (blk + 64 * h + 32));
                const __m256i hh = _mm256_loadu_si256((const __m256i *) (blk + 128 + 32 * h));
                const __m256i lows[4] = {_mm256_and_si256(l0, lo4), _mm256_and_si256(l1, lo4),
                                         _mm256_and_si256(_mm256_srli_epi16(l0, 4), lo4),
                                         _mm256_and_si256(_mm256_srli_epi16(l1, 4), lo4)};
                for (int s = 0; s < 4; ++s) {
                    const __m256i hi = _mm256_and_si256(_mm256_srli_epi16(hh, 2 * s), lo2);
                    _mm256_store_si256((__m256i *) (c + 128 * h + 32 * s),
                                       _mm256_or_si256(lows[s], _mm256_slli_epi16(hi, 4)));
                }
            }
            u->d[b] = orc_f16_to_f32(hd);
            u->dmin[b] = 0.0f;
        } else {
            const uint8_t * blk = w + 84 * b;
            memcpy(&hd, blk + 80, 2);
            memcpy(&hm, blk + 82, 2);
            for (int g = 0; g < 16; ++g) {
                sc[g] = (int16_t) (blk[g] & 15);
                mn[g] = (int16_t) (blk[g] >> 4);
            }
            /* element 128h + 32s + l: bits 2s of qs[32h + l] */
            for (int h = 0; h < 2; ++h) {
                const __m256i x = _mm256_loadu_si256((const __m256i *) (blk + 16 + 32 * h));
                for (int s = 0; s < 4; ++s) {
                    _mm256_store_si256((__m256i *) (c + 128 * h + 32 * s), _mm256_and_si256(_mm256_srli_epi16(x, 2 * s), lo2));
                }
            }
            u->d[b] = orc_f16_to_f32(hd);
            u->dmin[b] = orc_f16_to_f32(hm);
        }
    }
}

static int32_t hsum_i32(__m256i v) {
    __m128i s = _mm_add_epi32(_mm256_castsi256_si128(v), _mm256_extracti128_si256(v, 1));
    s = _mm_add_epi32(s, _mm_shuffle_epi32(s, 0x4e));
    s = _mm_add_epi32(s, _mm_shuffle_epi32(s, 0xb1));
    return _mm_cvtsi128_si32(s);
}

static float dot_unpacked(uint32_t type, const unpacked_row * u, const q8k_block * a, int64_t nb) {
    double sum = 0.0;
    for (int64_t b = 0; b < nb; ++b) {
        const uint8_t * c = u->codes + 256 * b;
        const int16_t * sc = u->scale + 16 * b;
        __m256i acc = _mm256_setzero_si256();
        for (int v = 0; v < 8; ++v) {
            /* 16 pair sums code*q (|sum| <= 2*63*127), then times the group scale, pairs summed in int32 */
            const __m256i p = _mm256_maddubs_epi16(_mm256_load_si256((const __m256i *) (c + 32 * v)),
                                                   _mm256_loadu_si256((const __m256i *) (a[b].qs + 32 * v)));
            const __m256i s = _mm256_set_m128i(_mm_set1_epi16(sc[2 * v + 1]), _mm_set1_epi16(sc[2 * v]));
            acc = _mm256_add_epi32(acc, _mm256_madd_epi16(p, s));
        }
        int32_t isum = hsum_i32(acc);
        const __m256i bs = _mm256_loadu_si256((const __m256i *) a[b].bsums);
        if (type == T_Q6_K) {
            /* codes carry +32: sum (q6 + 32) q = sum q6 q + 32 bsum */
            isum -= 32 * hsum_i32(_mm256_madd_epi16(_mm256_loadu_si256((const __m256i *) sc), bs));
            const float c6 = (u->d[b] * a[b].d) * (float) isum;
            sum += (double) c6;
        } else {
            const int32_t msum = hsum_i32(_mm256_madd_epi16(_mm256_loadu_si256((const __m256i *) (u->min + 16 * b)), bs));
            const float d = u->d[b] * a[b].d;
            const float dmin = u->dmin[b] * a[b].d;
            const float cb = d * (float) isum - dmin * (float) msum;
            sum += (double) cb;
        }
    }
    return (float) sum;
}

float orc_dot_kquant_scalar(uint32_t type, const void * w, const void * a, int64_t nb) {
    if (type == T_Q4_K) return dot_q4_k(w, a, nb);
    if (type == T_Q6_K) return dot_q6_k(w, a, nb);
    return dot_q2_k(w, a, nb);
}

float orc_dot_kquant_vector(uint32_t type, const void * w, const void * a, int64_t nb) {
    unpacked_row u;
    u.codes = aligned_alloc(32, (size_t) nb * 256);
    u.scale = malloc(sizeof(int16_t) * 16 * (size_t) nb);
    u.min = malloc(sizeof(int16_t) * 16 * (size_t) nb);
    u.d = malloc(sizeof(float) * (size_t) nb);
    u.dmin = malloc(sizeof(float) * (size_t) nb);
    unpack_row(type, w, nb, &u);
    const float v = dot_unpacked(type, &u, a, nb);
    free(u.codes); free(u.scale); free(u.min); free(u.d); free(u.dmin);
    return v;
}

size_t orc_q8k_block_bytes(void) { return sizeof(q8k_block); }

/* ggml_mul_mat on the CPU backend (qwen2_architecture.cpp:347-371 builds it):
 * src1 rows are converted to the weight's vec_dot_type first (Q8_K for
 * K-quants, F16 for F16 weights, none for F32), then every output element is
 * one vec_dot. */
void orc_matmul(const orc_tensor * w, const float * x, int64_t rows, float * y) {
    const int64_t K = (int64_t) w->ne0, N = (int64_t) w->ne1;
    const uint8_t * base = w->data;
    if (w->type == T_Q4_K || w->type == T_Q6_K || w->type == T_Q2_K) {
        const int64_t nb = K / QK;
        const size_t bb = block_bytes(w->type);
        q8k_block * act = malloc(sizeof(q8k_block) * (size_t) (nb * rows));
        for (int64_t r = 0; r < rows; ++r) orc_quantize_row_q8_k(x + r * K, act + r * nb, K);
#pragma omp parallel
        {
            unpacked_row u;
            u.codes = aligned_alloc(32, (size_t) nb * 256);
            u.scale = malloc(sizeof(int16_t) * 16 * (size_t) nb);
            u.min = malloc(sizeof(int16_t) * 16 * (size_t) nb);
            u.d = malloc(sizeof(float) * (size_t) nb);
            u.dmin = malloc(sizeof(float) * (size_t) nb);
#pragma omp for schedule(static)
            for (int64_t n = 0; n < N; ++n) {
                unpack_row(w->type, base + (size_t) n * (size_t) nb * bb, nb, &u);
                for (int64_t r = 0; r < rows; ++r) y[r * N + n] = dot_unpacked(w->type, &u, act + r * nb, nb);
            }
            free(u.codes); free(u.scale); free(u.min); free(u.d); free(u.dmin);
        }
        free(act);
        return;
    }
    if (w->type == T_F16) {
        uint16_t * act = malloc(sizeof(uint16_t) * (size_t) (K * rows));
        for (int64_t i = 0; i < K * rows; ++i) act[i] = orc_f32_to_f16(x[i]);
#pragma omp parallel for schedule(static)
        for (int64_t n = 0; n < N; ++n) {
            const uint16_t * wr = (const uint16_t *) base + n * K;
            for (int64_t r = 0; r < rows; ++r) {
                double s = 0.0;
                for (int64_t k = 0; k < K; ++k) s += (double) (orc_f16_to_f32(wr[k]) * orc_f16_to_f32(act[r * K + k]));
                y[r * N + n] = (float) s;
            }
        }
        free(act);
        return;
    }
    /* F32 */
#pragma omp parallel for schedule(static)
    for (int64_t n = 0; n < N; ++n) {
        const float * wr = (const float *) base + n * K;
        for (int64_t r = 0; r < rows; ++r) {
            double s = 0.0;
            for (int64_t k = 0; k < K; ++k) s += (double) (wr[k] * x[r * K + k]);
            y[r * N + n] = (float) s;
        }
    }
}

/* ggml_rms_norm + ggml_mul (qwen2_architecture.cpp:373-376): the sum of
 * squares is accumulated in double, mean = (float)(sum/n),
 * scale = 1/sqrtf(mean + eps), y = (x*scale)*w. */
void orc_rms_norm(const float * x, const float * weight, int64_t n, float eps, float * y) {
    double sum = 0.0;
    for (int64_t i = 0; i < n; ++i) sum += (double) (x[i] * x[i]);
    const float mean = (float) (sum / (double) n);
    const float scale = 1.0f / sqrtf(mean + eps);
    for (int64_t i = 0; i < n; ++i) {
        const float v = x[i] * scale;
        y[i] = v * weight[i];
    }
}

/* ggml_rope_ext, NEOX mode, ext_factor 0, freq_scale 1, attn_factor 1
 * (qwen2_architecture.cpp:499-506): theta_scale = powf(base, -2/n_dims);
 * the angle of pair i is built by repeated float multiplication,
 * theta_0 = position, theta_{i+1} = theta_i * theta_scale; pair i rotates
 * elements (i, i + n_dims/2) of each head. */
void orc_rope_neox(float * x, int64_t heads, int64_t head_length, int64_t dims, int32_t position,
                   float freq_base) {
    const float theta_scale = powf(freq_base, -2.0f / (float) dims);
    float cosv[512], sinv[512];
    float theta = (float) position;
    for (int64_t i = 0; i < dims / 2; ++i) {
        cosv[i] = cosf(theta);
        sinv[i] = sinf(theta);
        theta *= theta_scale;
    }
    for (int64_t h = 0; h < heads; ++h) {
        float * v = x + h * head_length;
        for (int64_t i = 0; i < dims / 2; ++i) {
            const float x0 = v[i], x1 = v[i + dims / 2];
            v[i] = x0 * cosv[i] - x1 * sinv[i];
            v[i + dims / 2] = x0 * sinv[i] + x1 * cosv[i];
        }
    }
}

/* ggml_argmax: first index of the maximum (strict >). */
int32_t orc_argmax(const float * x, int64_t n) {
    int32_t best = 0;
    float max = -INFINITY;
    for (int64_t i = 0; i < n; ++i) {
        if (x[i] > max) { max = x[i]; best = (int32_t) i; }
    }
    return best;
}

/* ---- sessions --------------------------------------------------------- */

struct orc_session {
    const orc_model * m;
    size_t capacity;
    size_t position;
    size_t prefill_position;
    uint16_t * k_cache;  /* [layers][capacity][kv_dim] f16, token-major */
    uint16_t * v_cache;  /* [layers][capacity][kv_dim] f16, token-major */
};

orc_session * orc_session_create(const orc_model * model, size_t capacity) {
    if (model == NULL || capacity == 0 || capacity > model->context_length) return NULL;
    orc_session * s = calloc(1, sizeof(*s));
    if (s == NULL) return NULL;
    const size_t kvd = (size_t) model->embedding_length / model->head_count * model->kv_head_count;
    const size_t layers = model->layer_end - model->layer_start;
    s->m = model;
    s->capacity = capacity;
    /* qwen2_architecture.cpp:1091: the cache buffer is cleared at allocation */
    s->k_cache = calloc(layers * capacity * kvd, sizeof(uint16_t));
    s->v_cache = calloc(layers * capacity * kvd, sizeof(uint16_t));
    if (s->k_cache == NULL || s->v_cache == NULL) {
        orc_session_destroy(s);
        return NULL;
    }
    return s;
}

void orc_session_destroy(orc_session * s) {
    if (s == NULL) return;
    free(s->k_cache);
    free(s->v_cache);
    free(s);
}

size_t orc_session_position(const orc_session * s) { return s->position; }
size_t orc_session_capacity(const orc_session * s) { return s->capacity; }

/* Qwen2Session::rollback (qwen2_architecture.cpp:818-823). */
int orc_session_rollback(orc_session * s, size_t n) {
    if (n == 0 || n > s->position - s->prefill_position) return -1;
    s->position -= n;
    return 0;
}

static int fail_with(char * error, size_t size, const char * message) {
    if (error != NULL && size > 0) snprintf(error, size, "%s", message);
    return -1;
}

/* Attention of one query row at absolute position pos against cache keys
 * [0, pos] (the -inf mask of qwen2_architecture.cpp:697-708 removes the
 * rest). Scores: K (f16) . q rounded to f16, the products (exact in float)
 * summed in double and rounded to float once (ggml_vec_dot_f16 with src1
 * converted to F16, f32 result); soft_max_ext with scale 1/sqrt(head_dim):
 * x = score*scale, e = exp(x - max), sum in double, p = e * (float)(1/sum),
 * P rounded to f16 before the V product (src1 of the second mul_mat is
 * converted to F16); output = sum of exact f16*f16 products in double,
 * rounded once. GQA: query head h reads kv head h / (heads / kv_heads)
 * (ggml_mul_mat broadcast). */
void orc_attention_row(const float * q, const uint16_t * kc, const uint16_t * vc, int64_t pos, int64_t H,
                       int64_t KVH, int64_t hl, float * out) {
    const int64_t kvd = hl * KVH, group = H / KVH, keys = pos + 1;
    const float scale = 1.0f / sqrtf((float) hl);
    float * p = malloc(sizeof(float) * (size_t) keys);
    float qh[512];
    for (int64_t h = 0; h < H; ++h) {
        const int64_t g = h / group;
        for (int64_t d = 0; d < hl; ++d) qh[d] = orc_f16_to_f32(orc_f32_to_f16(q[h * hl + d]));
        float mx = -INFINITY;
        for (int64_t j = 0; j < keys; ++j) {
            const uint16_t * kr = kc + j * kvd + g * hl;
            double s = 0.0;
            for (int64_t d = 0; d < hl; ++d) s += (double) (orc_f16_to_f32(kr[d]) * qh[d]);
            p[j] = (float) s * scale;
            if (p[j] > mx) mx = p[j];
        }
        double sum = 0.0;
        for (int64_t j = 0; j < keys; ++j) {
            p[j] = orc_expf(p[j] - mx);
            sum += (double) p[j];
        }
        const float inv = (float) (1.0 / sum);
        for (int64_t j = 0; j < keys; ++j) p[j] = orc_f16_to_f32(orc_f32_to_f16(p[j] * inv));
        for (int64_t d = 0; d < hl; ++d) {
            double acc = 0.0;
            for (int64_t j = 0; j < keys; ++j) acc += (double) (orc_f16_to_f32(vc[j * kvd + g * hl + d]) * p[j]);
            out[h * hl + d] = (float) acc;
        }
    }
    free(p);
}

static void attention(const orc_model * m, const uint16_t * kc, const uint16_t * vc, const float * q,
                      size_t n, size_t p0, float * out) {
    const int64_t H = m->head_count, KVH = m->kv_head_count, hl = (int64_t) m->embedding_length / H;
#pragma omp parallel for schedule(dynamic)
    for (int64_t t = 0; t < (int64_t) n; ++t) {
        orc_attention_row(q + t * m->embedding_length, kc, vc, (int64_t) p0 + t, H, KVH, hl,
                          out + t * m->embedding_length);
    }
}

/* silu(g) * u with silu(g) = g / (1 + e^-g) (ggml_swiglu_split / ggml_silu). */
float orc_silu_mul(float g, float u) { return (g / (1.0f + orc_expf(-g))) * u; }

/* One transformer layer over n rows (qwen2_architecture.cpp:575-583). */
static void layer_forward(orc_session * s, size_t li, float * hidden, size_t n, size_t p0) {
    const orc_model * m = s->m;
    const orc_layer * L = &m->layers[li];
    const int64_t h = m->embedding_length, f = m->feed_forward_length;
    const int64_t H = m->head_count, KVH = m->kv_head_count, hl = h / H, kvd = hl * KVH;
    float * x = malloc(sizeof(float) * (size_t) (n * h));
    float * q = malloc(sizeof(float) * (size_t) (n * h));
    float * k = malloc(sizeof(float) * (size_t) (n * kvd));
    float * v = malloc(sizeof(float) * (size_t) (n * kvd));
    float * att = malloc(sizeof(float) * (size_t) (n * h));
    float * o = malloc(sizeof(float) * (size_t) (n * h));
    float * gate = malloc(sizeof(float) * (size_t) (n * f));
    float * up = malloc(sizeof(float) * (size_t) (n * f));
    uint16_t * kc = s->k_cache + li * s->capacity * (size_t) kvd;
    uint16_t * vc = s->v_cache + li * s->capacity * (size_t) kvd;

    for (size_t t = 0; t < n; ++t) orc_rms_norm(hidden + t * h, L->attn_norm.data, h, m->rms_epsilon, x + t * h);
    orc_matmul(&L->attn_q, x, (int64_t) n, q);
    orc_matmul(&L->attn_k, x, (int64_t) n, k);
    orc_matmul(&L->attn_v, x, (int64_t) n, v);
    const float * qb = L->attn_q_bias.data, * kb = L->attn_k_bias.data, * vb = L->attn_v_bias.data;
    for (size_t t = 0; t < n; ++t) {
        for (int64_t i = 0; i < h; ++i) q[t * h + i] += qb[i];
        for (int64_t i = 0; i < kvd; ++i) { k[t * kvd + i] += kb[i]; v[t * kvd + i] += vb[i]; }
        orc_rope_neox(q + t * h, H, hl, m->rope_dimension_count, (int32_t) (p0 + t), m->rope_freq_base);
        orc_rope_neox(k + t * kvd, KVH, hl, m->rope_dimension_count, (int32_t) (p0 + t), m->rope_freq_base);
        /* ggml_set_rows into the F16 caches (qwen2_architecture.cpp:405-424) */
        for (int64_t i = 0; i < kvd; ++i) {
            kc[(p0 + t) * (size_t) kvd + (size_t) i] = orc_f32_to_f16(k[t * kvd + i]);
            vc[(p0 + t) * (size_t) kvd + (size_t) i] = orc_f32_to_f16(v[t * kvd + i]);
        }
    }
    attention(m, kc, vc, q, n, p0, att);
    orc_matmul(&L->attn_output, att, (int64_t) n, o);
    for (size_t i = 0; i < n * (size_t) h; ++i) hidden[i] = o[i] + hidden[i];

    for (size_t t = 0; t < n; ++t) orc_rms_norm(hidden + t * h, L->ffn_norm.data, h, m->rms_epsilon, x + t * h);
    orc_matmul(&L->ffn_up, x, (int64_t) n, up);
    orc_matmul(&L->ffn_gate, x, (int64_t) n, gate);
    /* swiglu / silu*mul (qwen2_architecture.cpp:508-520): silu(g) = g/(1+e^-g) */
    for (size_t i = 0; i < n * (size_t) f; ++i) {
        const float g = gate[i];
        gate[i] = orc_silu_mul(g, up[i]);
    }
    orc_matmul(&L->ffn_down, gate, (int64_t) n, o);
    for (size_t i = 0; i < n * (size_t) h; ++i) hidden[i] = o[i] + hidden[i];
    free(x); free(q); free(k); free(v); free(att); free(o); free(gate); free(up);
}

int orc_session_forward(orc_session * s, int prefill, const int32_t * tokens, const float * activations,
                        size_t n, float * out_activations, float * out_logits, int32_t * out_token,
                        char * error, size_t error_size) {
    const orc_model * m = s->m;
    const int first = m->layer_start == 0, last = m->layer_end == m->layer_count;
    /* position rules: validate_prefill_count / validate_decode
     * (qwen2_architecture.cpp:1037-1054) */
    if (prefill) {
        if (s->position != 0 || n == 0 || n > s->capacity) {
            return fail_with(error, error_size, "native Qwen2 prefill is outside session capacity");
        }
    } else {
        if (n != 1) return fail_with(error, error_size, "native decode must contain one token row");
        if (s->position == 0 || s->position >= s->capacity) {
            return fail_with(error, error_size, "native Qwen2 decode is outside session capacity");
        }
    }
    if (first && tokens == NULL) return fail_with(error, error_size, "the first native stage requires tokens");
    if (!first && activations == NULL) return fail_with(error, error_size, "later native stages require activations");
    const int64_t h = m->embedding_length;
    if (first) {
        for (size_t t = 0; t < n; ++t) {
            if (tokens[t] < 0 || (uint32_t) tokens[t] >= m->vocabulary_size) {
                return fail_with(error, error_size, "native token ID is outside model vocabulary");
            }
        }
    }
    float * hidden = malloc(sizeof(float) * n * (size_t) h);
    if (first) {
        /* ggml_get_rows on token_embd (qwen2_architecture.cpp:564-568) */
        const size_t row_bytes = m->token_embd.type == T_F32 ? (size_t) h * 4
            : m->token_embd.type == T_F16 ? (size_t) h * 2
            : (size_t) h / QK * block_bytes(m->token_embd.type);
        for (size_t t = 0; t < n; ++t) {
            orc_dequantize_row(m->token_embd.type, (const uint8_t *) m->token_embd.data + (size_t) tokens[t] * row_bytes,
                               hidden + t * (size_t) h, h);
        }
    } else {
        memcpy(hidden, activations, sizeof(float) * n * (size_t) h);
    }
    const size_t p0 = s->position;
    for (size_t li = 0; li < m->layer_end - m->layer_start; ++li) layer_forward(s, li, hidden, n, p0);
    s->position = p0 + n;
    if (prefill) s->prefill_position = s->position;
    if (!last) {
        if (out_activations != NULL) memcpy(out_activations, hidden, sizeof(float) * n * (size_t) h);
        free(hidden);
        return 0;
    }
    /* output head (qwen2_architecture.cpp:584-597): last row, output norm,
     * projection (+ optional bias), argmax */
    float * normed = malloc(sizeof(float) * (size_t) h);
    orc_rms_norm(hidden + (n - 1) * (size_t) h, m->output_norm.data, h, m->rms_epsilon, normed);
    float * logits = malloc(sizeof(float) * m->output.ne1);
    orc_matmul(&m->output, normed, 1, logits);
    if (m->output_bias.data != NULL) {
        const float * ob = m->output_bias.data;
        for (uint64_t i = 0; i < m->output.ne1; ++i) logits[i] += ob[i];
    }
    if (out_logits != NULL) memcpy(out_logits, logits, sizeof(float) * m->output.ne1);
    if (out_token != NULL) *out_token = orc_argmax(logits, (int64_t) m->output.ne1);
    free(logits);
    free(normed);
    free(hidden);
    return 0;
}
