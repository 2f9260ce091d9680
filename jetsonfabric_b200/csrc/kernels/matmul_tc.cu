// K-quant x Q8_K matmul on the 5th-generation tensor cores (tcgen05), with
// the same bit-exact result as the CUDA-core path and the CPU oracle for every
// input.
//
// Exactness. Per 256-value block the CPU (ggml_vec_dot_{q4_K,q6_K,q2_K}_q8_K,
// restated in the oracle) forms the integers
//     isum = sum_j scale_j * sum_{k in sub-block j} q_w[k] * q_a[k]
//     msum = sum_g min_g * bsum_g                       (Q4_K, Q2_K)
// and one float term c = (d_w*d_a)*(float)isum - (dmin_w*d_a)*(float)msum.
// Here the activation operand B holds the Q8_K codes (|q_a| <= 127) as f16 and
// the weight operand A holds integer products, also as f16. A chain of MMAs
// into one f32 accumulator is exact when every partial sum stays below 2^24 in
// magnitude, so each type is split until that holds for any input:
//   Q4_K  A = scale*code <= 63*15 = 945. One accumulator per 128-value half:
//         at most 945*127*128 < 2^24. (float)isum = RN(D0 + D1), one add of
//         two exact integers.
//   Q6_K  A = scale*(code-32) reaches 128*32 = 4096, where odd values are not
//         f16 numbers. The int8 scale s is split into s = 16*hi + lo
//         (hi in [-8, 7], lo in [0, 15]); the planes hi*(code-32) and
//         lo*(code-32) stay within 256 and 480, their accumulators within
//         256*127*256 and 480*127*256, both < 2^24.
//         (float)isum = RN(16*Dhi + Dlo), one fused multiply-add.
//   Q2_K  A = scale*code <= 15*3 = 45: one accumulator.
//   mins  One K = 16 MMA per block of the mins (<= 63) with the Q8_K partial
//         sums (|bsum| <= 16*127): at most 16*63*2032 < 2^24.
// The epilogue rounds every block term exactly as the CPU does and adds it to
// a per-(row, token) double sum, as the CUDA-core kernel does.
//
// Schedule. Persistent stream-K: grid G = min(SMs, W) and CTA c walks the
// contiguous work range [c*W/G, (c+1)*W/G) of W = tiles * blocks units. A tile
// is 128 weight rows x 32 activation rows; a unit is one 256-block of K. When
// a tile's K range spans several CTAs, each epilogue warp writes its double
// partials and the last warp to arrive (a per-tile, per-warp counter) adds
// all contributors' partials in CTA order, so the result does not depend on
// timing and no CTA ever waits for another.
//
// Warp roles (13 warps, 416 threads):
//   warps 0-3   epilogue: warp w owns TMEM lanes 32w..32w+31 (weight rows)
//               and all 32 token columns;
//   warps 4-11  producers: per stage (half a block, 128 K values) thread
//               (m, part) writes 64 values of weight row m as f16 products in
//               the canonical no-swizzle K-major layout (core matrices of
//               8 rows x 16 bytes; LBO = 128 B between the two K-halves of one
//               16-wide MMA step, SBO = 2048 B between 8-row groups), and all
//               producers convert the activation codes (and, once per block,
//               the mins and partial sums) the same way;
//   warp 12     TMEM allocation and the single-thread tcgen05.mma issue.
// Accumulators are double-buffered in TMEM, so the MMAs of block i+1 overlap
// the epilogue of block i. Every mbarrier wait is bounded by a 2 s
// global-timer limit: on expiry the kernel records an error code, every role
// stops, in-flight MMAs are drained and TMEM is released.
#include <algorithm>
#include <mutex>

#include "common.cuh"

namespace jfb {
namespace {

constexpr int kThreads = 416;
constexpr int kEpilogueThreads = 128;  // warps 0-3
constexpr int kEpilogueWarps = 4;
constexpr int kProducerThreads = 256;  // warps 4-11
constexpr int kMmaWarp = 12;
constexpr int kRows = 128;             // MMA M: weight rows per tile
constexpr int kBN = 32;                // MMA N: activation rows per tile
constexpr int kKStage = 128;           // K values per pipeline stage
constexpr uint32_t kSbo = 2048;        // 8-row group stride of a 128-wide K tile
constexpr uint32_t kSbo16 = 256;       // same for the K = 16 mins tiles
constexpr uint32_t kTileBytes = kRows * kKStage * 2;  // one f16 A plane, 32 KB
constexpr uint32_t kBBytes = kBN * kKStage * 2;       // 8 KB
constexpr uint32_t kA2Bytes = kRows * 16 * 2;         // 4 KB
constexpr uint32_t kB2Bytes = kBN * 16 * 2;           // 1 KB
constexpr uint32_t kMaxSmem = 232448;                 // sm_100 opt-in limit per block
constexpr uint32_t kTailBytes = 1024;                 // barriers, TMEM slot, flags, activation scales
constexpr uint64_t kWaitNs = 2000000000ull;
constexpr uint32_t kSlotDoubles = kRows * kBN;        // one partial tile

enum : int {
    kErrWaitEmpty = 1,
    kErrWaitAccEmpty = 2,
    kErrWaitFull = 3,
    kErrWaitAccFull = 4,
};

template <uint32_t TYPE>
struct TypeTraits;
template <>
struct TypeTraits<JF_TENSOR_Q4_K> {
    static constexpr int kPlanes = 1, kAcc = 3;  // D(half 0), D(half 1), mins
    static constexpr bool kMins = true;
};
template <>
struct TypeTraits<JF_TENSOR_Q6_K> {
    static constexpr int kPlanes = 2, kAcc = 2;  // D(hi), D(lo)
    static constexpr bool kMins = false;
};
template <>
struct TypeTraits<JF_TENSOR_Q2_K> {
    static constexpr int kPlanes = 1, kAcc = 2;  // D, mins
    static constexpr bool kMins = true;
};

template <uint32_t TYPE>
__host__ __device__ constexpr uint32_t stage_bytes() {
    return TypeTraits<TYPE>::kPlanes * kTileBytes + kBBytes + (TypeTraits<TYPE>::kMins ? kA2Bytes + kB2Bytes : 0);
}
template <uint32_t TYPE>
__host__ __device__ constexpr int stage_count() {
    return int((kMaxSmem - kTailBytes) / stage_bytes<TYPE>()) < 6 ? int((kMaxSmem - kTailBytes) / stage_bytes<TYPE>()) : 6;
}
template <uint32_t TYPE>
__host__ __device__ constexpr uint32_t smem_bytes() {
    return stage_count<TYPE>() * stage_bytes<TYPE>() + kTailBytes;
}
template <uint32_t TYPE>
__host__ __device__ constexpr uint32_t tmem_columns() {
    const uint32_t need = 2 * TypeTraits<TYPE>::kAcc * kBN;
    return need <= 32 ? 32 : need <= 64 ? 64 : need <= 128 ? 128 : need <= 256 ? 256 : 512;
}

// ---- PTX wrappers -------------------------------------------------------------

__device__ __forceinline__ uint32_t smem_u32(const void * p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint64_t * bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_arrive(uint64_t * bar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t * bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.b32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait: false (with the abort flag raised and `code` recorded) when
// the phase has not completed within kWaitNs, or when another role aborted.
__device__ __noinline__ bool mbar_wait_slow(uint64_t * bar, uint32_t parity, volatile int * abort_flag, int * error,
                                            int code) {
    const uint64_t t0 = global_ns();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort_flag) return false;
        if ((i & 63u) == 0 && global_ns() - t0 > kWaitNs) break;
    }
    *abort_flag = 1;
    if (error != nullptr) *reinterpret_cast<volatile int *>(error) = code;  // device or host-mapped word
    return false;
}

__device__ __forceinline__ bool mbar_wait(uint64_t * bar, uint32_t parity, volatile int * abort_flag, int * error,
                                          int code) {
    if (mbar_try_wait(bar, parity)) return true;
    return mbar_wait_slow(bar, parity, abort_flag, error, code);
}

__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor: K-major, no swizzle, sm_100 version bit.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= uint64_t((addr & 0x3FFFF) >> 4);
    d |= uint64_t((lbo >> 4) & 0x3FFF) << 16;
    d |= uint64_t((sbo >> 4) & 0x3FFF) << 32;
    d |= uint64_t(1) << 46;
    return d;
}

// Instruction descriptor of kind::f16: D = f32, A = B = f16, both K-major.
__host__ __device__ constexpr uint32_t instr_desc(uint32_t m, uint32_t n) {
    return (1u << 4) | ((n >> 3) << 17) | ((m >> 4) << 24);
}

__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void mma_commit(uint64_t * bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// 8 consecutive f32 columns of this thread's TMEM lane (completes at tmem_wait_ld).
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// ---- operand construction ---------------------------------------------------------

__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t *>(&h); }
__device__ __forceinline__ __half2 bits_h2(uint32_t u) { return *reinterpret_cast<__half2 *>(&u); }

// Bytes 0,1 (sel 0x4140) or 2,3 (sel 0x4342) of w as the f16 pair
// (1024 + b0, 1024 + b1): 0x64 is the high byte of 1024.0 in f16.
__device__ __forceinline__ __half2 magic_pair(uint32_t w, uint32_t sel) { return bits_h2(__byte_perm(w, 0x64u, sel)); }

// Four bytes b of w as two f16 pairs fma(1024 + b, scale, nbias). With
// nbias = -(1024 + offset) * scale the exact value (b - offset) * scale is an
// f16 integer and the fused operation rounds once, so the result is exact.
__device__ __forceinline__ uint2 scaled4(uint32_t w, __half2 scale, __half2 nbias) {
    const __half2 lo = __hfma2(magic_pair(w, 0x4140u), scale, nbias);
    const __half2 hi = __hfma2(magic_pair(w, 0x4342u), scale, nbias);
    return make_uint2(h2_bits(lo), h2_bits(hi));
}

__device__ __forceinline__ __half2 h2_int(int v) { return __half2half2(__int2half_rn(v)); }

__device__ __forceinline__ uint32_t byte_at(const uint4 & v, int i) {
    const uint32_t w = i < 4 ? v.x : i < 8 ? v.y : i < 12 ? v.z : v.w;
    return (w >> (8 * (i & 3))) & 0xffu;
}

// 6-bit scale and min of Q4_K sub-block j from the 12 packed bytes at hdr[4..16).
__device__ __forceinline__ void q4k_scale_min_hdr(const uint4 & hdr, int j, int & sc, int & m) {
    auto s = [&](int k) { return int(byte_at(hdr, 4 + k)); };
    if (j < 4) {
        sc = s(j) & 63;
        m = s(j + 4) & 63;
    } else {
        sc = (s(j + 4) & 0x0f) | ((s(j - 4) >> 6) << 4);
        m = (s(j + 4) >> 4) | ((s(j) >> 6) << 4);
    }
}

struct TcParams {
    jfb_weight w;
    const int8_t * qs;      // Q8_K codes [n][cols]
    const float * da;       // [n][blocks]
    const int16_t * bsums;  // [n][cols/16]
    uint32_t n;
    uint32_t blocks;        // cols / 256
    uint32_t tiles_m;
    uint32_t tiles;
    uint64_t work;          // tiles * blocks
    uint32_t epilogue;
    const float * bias;
    const float * residual;
    float * out;            // [n][rows]
    double * partial;       // [2 * gridDim.x][kBN][kRows]
    uint32_t * counters;    // [tiles][kEpilogueWarps]
    int * error;
};

__host__ __device__ __forceinline__ uint64_t range_start(uint64_t c, uint64_t work, uint64_t g) {
    return c * work / g;
}
// The CTA whose range holds `unit`.
__device__ __forceinline__ uint32_t cta_of(uint64_t unit, uint64_t work, uint64_t g) {
    return uint32_t(((unit + 1) * g - 1) / work);
}

// Weight half-block `h`, values [64*part, 64*part + 64), of block `block` for
// tile row m, as f16 products in the A plane(s).
template <uint32_t TYPE>
__device__ __forceinline__ void produce_a(const jfb_weight & w, uint64_t block, int h, int part, uint8_t * a_tile,
                                          int m) {
    const uint8_t * p0 = static_cast<const uint8_t *>(w.plane[0]);
    const uint8_t * p1 = static_cast<const uint8_t *>(w.plane[1]);
    uint8_t * row_base = a_tile + (m >> 3) * kSbo + (m & 7) * 16;
    if constexpr (TYPE == JF_TENSOR_Q4_K) {
        // codes: byte 32c + l holds element 64c + l (low nibble) and 64c + 32 + l
        // (high nibble); this thread covers c = 2h + part.
        const int c = 2 * h + part;
        const uint4 hdr = __ldg(reinterpret_cast<const uint4 *>(p1 + block * 16));
        const uint4 * codes = reinterpret_cast<const uint4 *>(p0 + block * 128 + 32 * c);
        const uint4 v0 = __ldg(codes), v1 = __ldg(codes + 1);
        const uint32_t wv[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
#pragma unroll
        for (int nib = 0; nib < 2; ++nib) {
            int sc, mn;
            q4k_scale_min_hdr(hdr, 2 * c + nib, sc, mn);
            const __half2 scale = h2_int(sc), nbias = h2_int(-1024 * sc);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const uint2 a = scaled4((wv[2 * q] >> (4 * nib)) & 0x0f0f0f0fu, scale, nbias);
                const uint2 b = scaled4((wv[2 * q + 1] >> (4 * nib)) & 0x0f0f0f0fu, scale, nbias);
                const int chunk = 8 * part + 4 * nib + q;
                *reinterpret_cast<uint4 *>(row_base + chunk * 128) = make_uint4(a.x, a.y, b.x, b.y);
            }
        }
    } else if constexpr (TYPE == JF_TENSOR_Q6_K) {
        // element r (0..127) of half h: nibble r / 64 of ql[64h + r % 64] and
        // bits 2*(r / 32) of qh[32h + r % 32]; this thread covers
        // r in [64*part, 64*part + 64).
        const uint8_t * blk = p0 + block * 192;
        const uint4 * ql = reinterpret_cast<const uint4 *>(blk + 64 * h);
        const uint4 * qh = reinterpret_cast<const uint4 *>(blk + 128 + 32 * h);
        const uint4 scv = __ldg(reinterpret_cast<const uint4 *>(p1 + block * 16));
        const uint4 l0 = __ldg(ql), l1 = __ldg(ql + 1), l2 = __ldg(ql + 2), l3 = __ldg(ql + 3);
        const uint4 q0 = __ldg(qh), q1 = __ldg(qh + 1);
        const uint32_t L[16] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w,
                                l2.x, l2.y, l2.z, l2.w, l3.x, l3.y, l3.z, l3.w};
        const uint32_t H[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
        uint8_t * row_lo = row_base + kTileBytes;
#pragma unroll
        for (int ch = 0; ch < 8; ++ch) {
            const int r0 = 64 * part + 8 * ch;
            const int s = int(int8_t(byte_at(scv, (128 * h + r0) / 16)));
            const int s_lo = s & 15, s_hi = (s - s_lo) / 16;
            const __half2 shi = h2_int(s_hi), nhi = h2_int(-1056 * s_hi);  // 1056 = 1024 + 32
            const __half2 slo = h2_int(s_lo), nlo = h2_int(-1056 * s_lo);
            uint32_t q[2];
#pragma unroll
            for (int k = 0; k < 2; ++k) {
                const int r = r0 + 4 * k;
                q[k] = ((L[(r % 64) / 4] >> (4 * (r / 64))) & 0x0f0f0f0fu) |
                       (((H[(r % 32) / 4] >> (2 * (r / 32))) & 0x03030303u) << 4);
            }
            const int chunk = 8 * part + ch;
            const uint2 a0 = scaled4(q[0], shi, nhi), a1 = scaled4(q[1], shi, nhi);
            *reinterpret_cast<uint4 *>(row_base + chunk * 128) = make_uint4(a0.x, a0.y, a1.x, a1.y);
            const uint2 b0 = scaled4(q[0], slo, nlo), b1 = scaled4(q[1], slo, nlo);
            *reinterpret_cast<uint4 *>(row_lo + chunk * 128) = make_uint4(b0.x, b0.y, b1.x, b1.y);
        }
    } else {  // Q2_K: element 128h + 32s + l lives in bits 2s of qs[32h + l]
        const uint4 * qs = reinterpret_cast<const uint4 *>(p0 + block * 64 + 32 * h);
        const uint4 a0 = __ldg(qs), a1 = __ldg(qs + 1);
        const uint32_t Q[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
        const uint4 scv = __ldg(reinterpret_cast<const uint4 *>(p1 + block * 16));
#pragma unroll
        for (int ch = 0; ch < 8; ++ch) {
            const int r0 = 64 * part + 8 * ch;
            const int s = r0 / 32, l0 = r0 % 32;
            const int sc = int(byte_at(scv, (128 * h + r0) / 16) & 15);
            const __half2 scale = h2_int(sc), nbias = h2_int(-1024 * sc);
            const uint2 x = scaled4((Q[l0 / 4] >> (2 * s)) & 0x03030303u, scale, nbias);
            const uint2 y = scaled4((Q[l0 / 4 + 1] >> (2 * s)) & 0x03030303u, scale, nbias);
            *reinterpret_cast<uint4 *>(row_base + (8 * part + ch) * 128) = make_uint4(x.x, x.y, y.x, y.y);
        }
    }
}

// The 16 per-16-value mins of one block as a K = 16 f16 operand row (Q4_K:
// the 6-bit min of each 32-value sub-block, twice; Q2_K: the high nibble of
// each scale byte).
template <uint32_t TYPE>
__device__ __forceinline__ void produce_mins(const jfb_weight & w, uint64_t block, uint8_t * tile, int m) {
    const uint4 meta = __ldg(reinterpret_cast<const uint4 *>(static_cast<const uint8_t *>(w.plane[1]) + block * 16));
    uint32_t h2[8];
#pragma unroll
    for (int g = 0; g < 16; g += 2) {
        int m0, m1;
        if constexpr (TYPE == JF_TENSOR_Q4_K) {
            int sc;
            q4k_scale_min_hdr(meta, g / 2, sc, m0);
            m1 = m0;
        } else {
            m0 = int(byte_at(meta, g) >> 4);
            m1 = int(byte_at(meta, g + 1) >> 4);
        }
        h2[g / 2] = h2_bits(__halves2half2(__int2half_rn(m0), __int2half_rn(m1)));
    }
    uint8_t * base = tile + (m >> 3) * kSbo16 + (m & 7) * 16;
    *reinterpret_cast<uint4 *>(base) = make_uint4(h2[0], h2[1], h2[2], h2[3]);
    *reinterpret_cast<uint4 *>(base + 128) = make_uint4(h2[4], h2[5], h2[6], h2[7]);
}

template <uint32_t TYPE>
__global__ void __launch_bounds__(kThreads, 1) mmq_tc_kernel(TcParams p) {
    using T = TypeTraits<TYPE>;
    constexpr int NS = stage_count<TYPE>();
    constexpr uint32_t kStage = stage_bytes<TYPE>();
    constexpr uint32_t kBOff = T::kPlanes * kTileBytes;
    constexpr uint32_t kA2Off = kBOff + kBBytes;
    constexpr uint32_t kB2Off = kA2Off + kA2Bytes;
    constexpr uint32_t kTmemCols = tmem_columns<TYPE>();

    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t * tail = smem + NS * kStage;
    uint64_t * full = reinterpret_cast<uint64_t *>(tail);  // [NS]
    uint64_t * empty = full + NS;                          // [NS]
    uint64_t * acc_full = empty + NS;                      // [2]
    uint64_t * acc_empty = acc_full + 2;                   // [2]
    uint64_t * drain = acc_empty + 2;                      // [1]
    uint32_t * tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
    volatile int * abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
    float * da_rows = reinterpret_cast<float *>(tail + 512);  // [kEpilogueWarps][kBN]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint64_t g = gridDim.x;
    const uint64_t w_begin = range_start(blockIdx.x, p.work, g);
    const uint64_t w_end = range_start(blockIdx.x + 1, p.work, g);
    const uint32_t nb = p.blocks;

    if (threadIdx.x == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(&full[s], kProducerThreads);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&acc_full[a], 1);
            mbar_init(&acc_empty[a], kEpilogueThreads);
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == kMmaWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp >= kEpilogueWarps && warp < kMmaWarp) {
        // ---------------- producers ----------------
        const int pt = threadIdx.x - kEpilogueThreads;
        const int m = pt & (kRows - 1), part = pt >> 7;
        const __half2 act_nbias = h2_int(-1152);  // codes arrive as q + 128 after the sign flip
        const __half2 one = h2_int(1);
        uint32_t stage = 0, phase = 0;
        bool ok = true;
        for (uint64_t w = w_begin; w < w_end && ok && !*abort_flag; ++w) {
            const uint32_t tile = uint32_t(w / nb), b = uint32_t(w % nb);
            const uint32_t tm = tile % p.tiles_m, tn = tile / p.tiles_m;
            const uint32_t row = tm * kRows + uint32_t(m), tok0 = tn * kBN;
            const uint64_t block = uint64_t(row) * nb + b;
            for (int h = 0; h < 2; ++h) {
                if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, p.error, kErrWaitEmpty)) {
                    ok = false;
                    break;
                }
                uint8_t * st = smem + stage * kStage;
                if (row < p.w.rows) {
                    produce_a<TYPE>(p.w, block, h, part, st, m);
                    if (T::kMins && h == 0 && part == 0) produce_mins<TYPE>(p.w, block, st + kA2Off, m);
                } else {
#pragma unroll
                    for (int pl = 0; pl < T::kPlanes; ++pl) {
                        uint8_t * base = st + pl * kTileBytes + (m >> 3) * kSbo + (m & 7) * 16;
                        for (int c = 8 * part; c < 8 * part + 8; ++c) {
                            *reinterpret_cast<uint4 *>(base + c * 128) = make_uint4(0, 0, 0, 0);
                        }
                    }
                    if (T::kMins && h == 0 && part == 0) {
                        uint8_t * base = st + kA2Off + (m >> 3) * kSbo16 + (m & 7) * 16;
                        *reinterpret_cast<uint4 *>(base) = make_uint4(0, 0, 0, 0);
                        *reinterpret_cast<uint4 *>(base + 128) = make_uint4(0, 0, 0, 0);
                    }
                }
                // activation codes: kBN rows x 16 chunks of 8
                for (int idx = pt; idx < kBN * 16; idx += kProducerThreads) {
                    const int t = idx >> 4, c = idx & 15;
                    uint4 v = make_uint4(0, 0, 0, 0);
                    if (tok0 + t < p.n) {
                        const uint2 raw = __ldg(reinterpret_cast<const uint2 *>(
                            p.qs + uint64_t(tok0 + t) * (uint64_t(nb) * kQK) + uint64_t(b) * kQK + 128 * h + 8 * c));
                        const uint2 x = scaled4(raw.x ^ 0x80808080u, one, act_nbias);
                        const uint2 y = scaled4(raw.y ^ 0x80808080u, one, act_nbias);
                        v = make_uint4(x.x, x.y, y.x, y.y);
                    }
                    *reinterpret_cast<uint4 *>(st + kBOff + (t >> 3) * kSbo + c * 128 + (t & 7) * 16) = v;
                }
                if (T::kMins && h == 0 && pt < kBN * 2) {
                    const int t = pt >> 1, c = pt & 1;
                    uint32_t hv[4] = {0, 0, 0, 0};
                    if (tok0 + t < p.n) {
                        const uint4 raw = __ldg(reinterpret_cast<const uint4 *>(
                            p.bsums + uint64_t(tok0 + t) * (uint64_t(nb) * 16) + uint64_t(b) * 16 + 8 * c));
                        const uint32_t rw[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
                        for (int k = 0; k < 4; ++k) {
                            hv[k] = h2_bits(__halves2half2(__int2half_rn(int(int16_t(rw[k] & 0xffffu))),
                                                           __int2half_rn(int(int16_t(rw[k] >> 16)))));
                        }
                    }
                    *reinterpret_cast<uint4 *>(st + kB2Off + (t >> 3) * kSbo16 + c * 128 + (t & 7) * 16) =
                        make_uint4(hv[0], hv[1], hv[2], hv[3]);
                }
                fence_proxy_async();
                mbar_arrive(&full[stage]);
                if (++stage == NS) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
        }
    } else if (warp == kMmaWarp) {
        // ---------------- MMA issue (one thread) ----------------
        if (lane == 0) {
            constexpr uint32_t idesc = instr_desc(kRows, kBN);
            uint32_t stage = 0, phase = 0, i = 0;
            bool ok = true;
            for (uint64_t w = w_begin; w < w_end && ok && !*abort_flag; ++w, ++i) {
                const uint32_t acc = i & 1u, use = i >> 1;
                if (!mbar_wait(&acc_empty[acc], (use & 1u) ^ 1u, abort_flag, p.error, kErrWaitAccEmpty)) break;
                tc_fence_after();
                const uint32_t d = tmem + acc * (T::kAcc * kBN);
                for (int h = 0; h < 2; ++h) {
                    if (!mbar_wait(&full[stage], phase, abort_flag, p.error, kErrWaitFull)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t st = smem_u32(smem + stage * kStage);
#pragma unroll
                    for (int ks = 0; ks < kKStage / 16; ++ks) {
                        const uint64_t bdesc = smem_desc(st + kBOff + ks * 256, 128, kSbo);
                        if constexpr (TYPE == JF_TENSOR_Q4_K) {
                            mma_f16(d + h * kBN, smem_desc(st + ks * 256, 128, kSbo), bdesc, idesc, ks > 0 ? 1u : 0u);
                        } else if constexpr (TYPE == JF_TENSOR_Q6_K) {
                            const uint32_t accum = (h > 0 || ks > 0) ? 1u : 0u;
                            mma_f16(d, smem_desc(st + ks * 256, 128, kSbo), bdesc, idesc, accum);
                            mma_f16(d + kBN, smem_desc(st + kTileBytes + ks * 256, 128, kSbo), bdesc, idesc, accum);
                        } else {
                            mma_f16(d, smem_desc(st + ks * 256, 128, kSbo), bdesc, idesc, (h > 0 || ks > 0) ? 1u : 0u);
                        }
                    }
                    if (T::kMins && h == 0) {
                        mma_f16(d + (T::kAcc - 1) * kBN, smem_desc(st + kA2Off, 128, kSbo16),
                                smem_desc(st + kB2Off, 128, kSbo16), idesc, 0u);
                    }
                    mma_commit(&empty[stage]);  // frees the stage once these MMAs are done
                    if (++stage == NS) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (ok) mma_commit(&acc_full[acc]);
            }
            // every issued MMA completes before TMEM is released
            mma_commit(drain);
            volatile int no_abort = 0;
            (void) mbar_wait(drain, 0, &no_abort, nullptr, 0);
        }
        __syncwarp();
    } else {
        // ---------------- epilogue (warps 0-3) ----------------
        const int m = warp * 32 + lane;
        const uint32_t lane_base = uint32_t(warp * 32) << 16;
        float * da_s = da_rows + warp * kBN;
        const uint8_t * p1 = static_cast<const uint8_t *>(p.w.plane[1]);
        const uint8_t * p2 = static_cast<const uint8_t *>(p.w.plane[2]);
        const uint32_t first_tile = uint32_t(w_begin / nb);
        double sum[kBN];
        uint64_t seg_begin = w_begin;
        uint32_t i = 0;
        for (uint64_t w = w_begin; w < w_end; ++w, ++i) {
            // warp-uniform stop: the warp collectives below need every lane
            if (__any_sync(0xffffffffu, *abort_flag != 0)) break;
            const uint32_t tile = uint32_t(w / nb), b = uint32_t(w % nb);
            const uint32_t tm = tile % p.tiles_m, tn = tile / p.tiles_m;
            const uint32_t row = tm * kRows + uint32_t(m), tok0 = tn * kBN;
            if (w == seg_begin) {
#pragma unroll
                for (int t = 0; t < kBN; ++t) sum[t] = 0.0;
            }
            // per-block scales: this row's d (and dmin), the tile's activation d
            float dw = 0.0f, dmin = 0.0f;
            if (row < p.w.rows) {
                const uint64_t block = uint64_t(row) * nb + b;
                if constexpr (TYPE == JF_TENSOR_Q4_K) {
                    const uint32_t dd = __ldg(reinterpret_cast<const uint32_t *>(p1 + block * 16));
                    dw = half_bits_to_float(uint16_t(dd & 0xffffu));
                    dmin = half_bits_to_float(uint16_t(dd >> 16));
                } else if constexpr (TYPE == JF_TENSOR_Q6_K) {
                    dw = half_bits_to_float(__ldg(reinterpret_cast<const uint16_t *>(p2) + block));
                } else {
                    const uint32_t dd = __ldg(reinterpret_cast<const uint32_t *>(p2) + block);
                    dw = half_bits_to_float(uint16_t(dd & 0xffffu));
                    dmin = half_bits_to_float(uint16_t(dd >> 16));
                }
            }
            __syncwarp();
            da_s[lane] = tok0 + lane < p.n ? __ldg(p.da + uint64_t(tok0 + lane) * nb + b) : 0.0f;
            __syncwarp();

            const uint32_t acc = i & 1u, use = i >> 1;
            // the whole warp proceeds or stops together
            const bool ready = mbar_wait(&acc_full[acc], use & 1u, abort_flag, p.error, kErrWaitAccFull);
            if (!__all_sync(0xffffffffu, ready)) break;
            tc_fence_after();
            const uint32_t base = tmem + lane_base + acc * (T::kAcc * kBN);
#pragma unroll
            for (int ch = 0; ch < kBN / 8; ++ch) {
                uint32_t r0[8], r1[8], r2[8];
                tmem_ld8(base + 8 * ch, r0);
                tmem_ld8(base + kBN + 8 * ch, r1);
                if constexpr (T::kAcc == 3) tmem_ld8(base + 2 * kBN + 8 * ch, r2);
                tmem_wait_ld();
                if (ch == kBN / 8 - 1) {
                    tc_fence_before();
                    mbar_arrive(&acc_empty[acc]);  // the accumulators may be overwritten now
                }
                const float4 da0 = *reinterpret_cast<const float4 *>(da_s + 8 * ch);
                const float4 da1 = *reinterpret_cast<const float4 *>(da_s + 8 * ch + 4);
                const float das[8] = {da0.x, da0.y, da0.z, da0.w, da1.x, da1.y, da1.z, da1.w};
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    const float da = das[k];
                    float c;
                    if constexpr (TYPE == JF_TENSOR_Q4_K) {
                        const float isum = __fadd_rn(__uint_as_float(r0[k]), __uint_as_float(r1[k]));
                        c = __fsub_rn(__fmul_rn(__fmul_rn(dw, da), isum),
                                      __fmul_rn(__fmul_rn(dmin, da), __uint_as_float(r2[k])));
                    } else if constexpr (TYPE == JF_TENSOR_Q6_K) {
                        const float isum = __fmaf_rn(16.0f, __uint_as_float(r0[k]), __uint_as_float(r1[k]));
                        c = __fmul_rn(__fmul_rn(dw, da), isum);
                    } else {
                        c = __fsub_rn(__fmul_rn(__fmul_rn(dw, da), __uint_as_float(r0[k])),
                                      __fmul_rn(__fmul_rn(dmin, da), __uint_as_float(r1[k])));
                    }
                    sum[8 * ch + k] += double(c);
                }
            }

            // a segment ends where the CTA's range or the tile's K range ends
            if (w + 1 != w_end && (w + 1) % nb != 0) continue;
            const bool complete = seg_begin == uint64_t(tile) * nb && w + 1 == uint64_t(tile + 1) * nb;
            seg_begin = w + 1;
            if (!complete) {
                const uint32_t slot = 2 * blockIdx.x + (tile == first_tile ? 0 : 1);
                double * part = p.partial + uint64_t(slot) * kSlotDoubles;
#pragma unroll
                for (int t = 0; t < kBN; ++t) part[t * kRows + m] = sum[t];
                __threadfence();
                __syncwarp();
                const uint32_t lo = cta_of(uint64_t(tile) * nb, p.work, g);
                const uint32_t hi = cta_of(uint64_t(tile + 1) * nb - 1, p.work, g);
                uint32_t arrived = 0;
                if (lane == 0) {
                    uint32_t * counter = p.counters + uint64_t(tile) * kEpilogueWarps + warp;
                    arrived = atomicAdd(counter, 1u) + 1;
                    if (arrived == hi - lo + 1) *counter = 0;  // every contributor is in
                }
                arrived = __shfl_sync(0xffffffffu, arrived, 0);
                if (arrived != hi - lo + 1) continue;
                __threadfence();
#pragma unroll
                for (int t = 0; t < kBN; ++t) sum[t] = 0.0;
                for (uint32_t c = lo; c <= hi; ++c) {
                    const uint32_t c_first = uint32_t(range_start(c, p.work, g) / nb);
                    const uint64_t s = 2 * uint64_t(c) + (tile == c_first ? 0 : 1);
                    const double * src = p.partial + s * kSlotDoubles;
#pragma unroll
                    for (int t = 0; t < kBN; ++t) sum[t] += __ldcg(src + t * kRows + m);
                }
            }
            if (row < p.w.rows) {
#pragma unroll
                for (int t = 0; t < kBN; ++t) {
                    const uint32_t tok = tok0 + t;
                    if (tok >= p.n) break;
                    const uint64_t at = uint64_t(tok) * p.w.rows + row;
                    float v = __double2float_rn(sum[t]);
                    if (p.epilogue == JFB_EPILOGUE_BIAS) v = __fadd_rn(v, p.bias[row]);
                    else if (p.epilogue == JFB_EPILOGUE_RESIDUAL) v = __fadd_rn(v, p.residual[at]);
                    p.out[at] = v;
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == kMmaWarp) {
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
    }
}

int sm_count() {
    static std::mutex mu;
    static int cached[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    std::lock_guard<std::mutex> lock(mu);
    if (cached[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        cached[dev] = n;
    }
    return cached[dev];
}

struct Plan {
    uint32_t tiles_m, tiles, grid;
    uint64_t work;
};

Plan make_plan(uint32_t rows, uint32_t cols, uint32_t n) {
    Plan pl;
    pl.tiles_m = (rows + kRows - 1) / kRows;
    pl.tiles = pl.tiles_m * ((n + kBN - 1) / kBN);
    pl.work = uint64_t(pl.tiles) * (cols / kQK);
    pl.grid = uint32_t(std::min<uint64_t>(pl.work, uint64_t(sm_count())));
    return pl;
}

// Workspace: partial slots for the largest grid this device runs (two per
// SM), then the arrival counters. Both offsets are the same for every shape,
// so calls of different shapes can share one workspace on a stream.
uint64_t partial_bytes() { return uint64_t(2) * uint64_t(sm_count()) * kSlotDoubles * sizeof(double); }
uint64_t workspace_bytes(const Plan & pl) {
    return partial_bytes() + uint64_t(pl.tiles) * kEpilogueWarps * sizeof(uint32_t);
}

template <uint32_t TYPE>
jfb_status launch(const TcParams & p, uint32_t grid, cudaStream_t s) {
    constexpr uint32_t bytes = smem_bytes<TYPE>();
    static_assert(bytes <= kMaxSmem, "shared memory budget");
    static_assert(stage_count<TYPE>() >= 2, "pipeline depth");
    auto kernel = mmq_tc_kernel<TYPE>;
    const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(bytes));
    if (e != cudaSuccess) {
        return status_error(JFB_STATUS_CUDA_ERROR, "jfb_matmul_tc: shared memory attribute: %s", cudaGetErrorString(e));
    }
    kernel<<<grid, kThreads, bytes, s>>>(p);
    return launch_status("jfb_matmul_tc");
}

}  // namespace
}  // namespace jfb

using namespace jfb;

extern "C" uint64_t jfb_matmul_tc_workspace_bytes(uint32_t rows, uint32_t cols, uint32_t n) {
    if (rows == 0 || cols < kQK || n == 0) return 0;
    return workspace_bytes(make_plan(rows, cols, n));
}

extern "C" int jfb_matmul_tc_supported(const jfb_weight * w) {
    return w != nullptr && is_kquant(w->type) && w->rows > 0 && w->cols >= kQK && w->cols % kQK == 0 ? 1 : 0;
}

extern "C" jfb_status jfb_matmul_tc(const jfb_weight * weight, const jfb_q8k * x_q8, uint32_t n, uint32_t epilogue,
                                    const float * bias, const float * residual, float * out, void * workspace,
                                    uint64_t workspace_size, int32_t * error_flag, void * stream) {
    if (weight == nullptr || x_q8 == nullptr || out == nullptr) {
        return status_error(JFB_STATUS_INVALID_ARGUMENT, "weight, activations and output are required");
    }
    if (!jfb_matmul_tc_supported(weight)) {
        return status_error(JFB_STATUS_UNSUPPORTED, "jfb_matmul_tc needs a Q4_K, Q6_K or Q2_K weight");
    }
    if (epilogue > JFB_EPILOGUE_RESIDUAL || (epilogue == JFB_EPILOGUE_BIAS && bias == nullptr) ||
        (epilogue == JFB_EPILOGUE_RESIDUAL && residual == nullptr)) {
        return status_error(JFB_STATUS_INVALID_ARGUMENT, "matmul epilogue operands are missing");
    }
    if (n == 0) return status_ok();
    if (x_q8->qs == nullptr || x_q8->d == nullptr || x_q8->bsums == nullptr) {
        return status_error(JFB_STATUS_INVALID_ARGUMENT, "Q8_K activation planes are required");
    }
    if ((reinterpret_cast<uintptr_t>(x_q8->qs) & 7u) != 0 || (reinterpret_cast<uintptr_t>(x_q8->bsums) & 15u) != 0) {
        return status_error(JFB_STATUS_INVALID_ARGUMENT, "Q8_K codes must be 8-byte and partial sums 16-byte aligned");
    }
    for (int i = 0; i < 2; ++i) {
        if ((reinterpret_cast<uintptr_t>(weight->plane[i]) & 15u) != 0) {
            return status_error(JFB_STATUS_INVALID_ARGUMENT, "weight planes must be 16-byte aligned");
        }
    }
    const Plan pl = make_plan(weight->rows, weight->cols, n);
    const uint64_t need = workspace_bytes(pl);
    if (workspace == nullptr || workspace_size < need) {
        return status_error(JFB_STATUS_INVALID_ARGUMENT, "jfb_matmul_tc workspace needs %llu bytes",
                            static_cast<unsigned long long>(need));
    }
    if ((reinterpret_cast<uintptr_t>(workspace) & 15u) != 0) {
        return status_error(JFB_STATUS_INVALID_ARGUMENT, "jfb_matmul_tc workspace must be 16-byte aligned");
    }
    TcParams p;
    p.w = *weight;
    p.qs = x_q8->qs;
    p.da = x_q8->d;
    p.bsums = x_q8->bsums;
    p.n = n;
    p.blocks = weight->cols / kQK;
    p.tiles_m = pl.tiles_m;
    p.tiles = pl.tiles;
    p.work = pl.work;
    p.epilogue = epilogue;
    p.bias = bias;
    p.residual = residual;
    p.out = out;
    p.partial = static_cast<double *>(workspace);
    p.counters = reinterpret_cast<uint32_t *>(static_cast<uint8_t *>(workspace) + partial_bytes());
    p.error = error_flag;
    cudaStream_t s = as_stream(stream);
    switch (weight->type) {
    case JF_TENSOR_Q4_K: return launch<JF_TENSOR_Q4_K>(p, pl.grid, s);
    case JF_TENSOR_Q6_K: return launch<JF_TENSOR_Q6_K>(p, pl.grid, s);
    default: return launch<JF_TENSOR_Q2_K>(p, pl.grid, s);
    }
}
