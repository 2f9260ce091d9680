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
// Warp roles (18 warps, 576 threads):
//   warps 0-7   epilogue: warp w owns TMEM lanes 32(w % 4)..+31 (weight rows)
//               and token columns 16(w / 4)..+15;
//   warps 8-15  converters: per stage (half a block, 128 K values) thread
//               (m, part) turns 64 raw values of weight row m into f16
//               products and writes them to tensor memory (tcgen05.st): the A
//               operand lives in TMEM (lane = weight row, each 32-bit column
//               a pair of consecutive K values), so it never takes shared
//               memory bandwidth. All converters also turn the activation
//               codes (and, once per block, the mins and partial sums) into
//               f16 B tiles in shared memory, in the canonical no-swizzle
//               K-major layout (core matrices of 8 rows x 16 bytes; LBO = 128 B
//               between the two K-halves of one 16-wide MMA step, SBO between
//               8-row groups);
//   warp 16     TMEM allocation and the single-thread tcgen05.mma issue;
//   warp 17     one thread issuing the 2D TMA loads (cp.async.bulk.tensor, no
//               multicast) of the raw weight rows, activation codes and
//               partial sums into a ring of raw stages, several stages ahead
//               of the converters, completing on mbarrier transaction counts.
// Accumulators are double-buffered in TMEM, so the MMAs of block i+1 overlap
// the epilogue of block i. The epilogue stages its per-block scales (weight
// d/dmin of its row, activation d of its lane's token) with cp.async several
// blocks ahead. Every mbarrier wait is bounded by a 2 s
// global-timer limit: on expiry the kernel records an error code, every role
// stops, in-flight MMAs and TMA loads are drained and TMEM is released.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>

#include "common.cuh"

namespace jfb {
namespace {

constexpr int kThreads = 576;
constexpr int kEpilogueThreads = 256;   // warps 0-7
constexpr int kEpilogueWarps = 8;
constexpr int kConverterThreads = 256;  // warps 8-15
constexpr int kMmaWarp = 16;
constexpr int kTmaWarp = 17;
constexpr int kRows = 128;             // MMA M: weight rows per tile
constexpr int kBN = 32;                // MMA N: activation rows per tile
constexpr int kKStage = 128;           // K values per pipeline stage
constexpr uint32_t kSbo = 2048;        // 8-row group stride of a 128-wide K tile
constexpr uint32_t kSbo16 = 256;       // same for the K = 16 mins tiles
constexpr uint32_t kBBytes = kBN * kKStage * 2;       // 8 KB
constexpr uint32_t kA2Bytes = kRows * 16 * 2;         // 4 KB
constexpr uint32_t kB2Bytes = kBN * 16 * 2;           // 1 KB
constexpr uint32_t kMaxSmem = 232448;                 // sm_100 opt-in limit per block
constexpr uint32_t kTailBytes = 1024;                 // barriers, TMEM slot, flags, activation scales
constexpr uint64_t kWaitNs = 2000000000ull;            // bound of every pipeline wait
constexpr uint32_t kSuspendNs = 1000000;               // longest single suspension of a waiting thread
constexpr uint32_t kSlotDoubles = kRows * kBN;        // one partial tile

enum : int {
    kErrWaitEmpty = 1,
    kErrWaitAccEmpty = 2,
    kErrWaitFull = 3,
    kErrWaitAccFull = 4,
    kErrWaitRawEmpty = 5,
    kErrWaitRawFull = 6,
};

// Raw stage (TMA destination, per half-block): the weight boxes W0 (and W1)
// of 128 rows, the scale/header box of 128 x 16 bytes, the activation codes
// (32 x 128 bytes) and, for types with mins, the Q8_K partial sums (32 x 32).
template <uint32_t TYPE>
struct TypeTraits;
template <>
struct TypeTraits<JF_TENSOR_Q4_K> {
    static constexpr int kPlanes = 1, kAcc = 3;  // D(half 0), D(half 1), mins
    static constexpr bool kMins = true;
    static constexpr uint32_t kW0 = 64, kW1 = 0;  // bytes per row: codes of the half-block
    static constexpr uint32_t kBlockBytes = 128;  // plane-0 bytes per block
};
template <>
struct TypeTraits<JF_TENSOR_Q6_K> {
    static constexpr int kPlanes = 2, kAcc = 2;  // D(hi), D(lo)
    static constexpr bool kMins = false;
    static constexpr uint32_t kW0 = 64, kW1 = 32;  // ql, qh of the half-block
    static constexpr uint32_t kBlockBytes = 192;
};
template <>
struct TypeTraits<JF_TENSOR_Q2_K> {
    static constexpr int kPlanes = 1, kAcc = 2;  // D, mins
    static constexpr bool kMins = true;
    static constexpr uint32_t kW0 = 32, kW1 = 0;
    static constexpr uint32_t kBlockBytes = 64;
};

template <uint32_t TYPE>
struct RawLayout {
    using T = TypeTraits<TYPE>;
    static constexpr uint32_t kW0Off = 0;
    static constexpr uint32_t kW1Off = kW0Off + kRows * T::kW0;
    static constexpr uint32_t kScOff = kW1Off + kRows * T::kW1;
    static constexpr uint32_t kActOff = kScOff + kRows * 16;
    static constexpr uint32_t kBsOff = kActOff + kBN * 128;
    static constexpr uint32_t kBytes = kBsOff + (T::kMins ? kBN * 32 : 0);  // also the TMA transaction size
};

// Operand stage in shared memory: the f16 B tile (activation codes) and, for
// types with mins, the K = 16 mins (A2) and partial-sum (B2) tiles. The A
// operand of a stage lives in TMEM.
template <uint32_t TYPE>
__host__ __device__ constexpr uint32_t stage_bytes() {
    return kBBytes + (TypeTraits<TYPE>::kMins ? kA2Bytes + kB2Bytes : 0);
}
template <uint32_t TYPE>
__host__ __device__ constexpr uint32_t acc_columns() {  // both accumulator buffers
    return 2 * TypeTraits<TYPE>::kAcc * kBN;
}
template <uint32_t TYPE>
__host__ __device__ constexpr uint32_t a_columns() {  // one stage of A: 64 columns per plane
    return TypeTraits<TYPE>::kPlanes * (kKStage / 2);
}
// Operand stages: as many A stages as fit next to the accumulators in the
// 512 TMEM columns, at most 4.
template <uint32_t TYPE>
__host__ __device__ constexpr int stage_count() {
    return int((512 - acc_columns<TYPE>()) / a_columns<TYPE>()) < 4 ? int((512 - acc_columns<TYPE>()) / a_columns<TYPE>())
                                                                      : 4;
}
constexpr int kScaleRing = 4;  // blocks of epilogue scales staged ahead
constexpr uint32_t kScaleBytes = kEpilogueWarps * kScaleRing * (32 + 32) * 4;
template <uint32_t TYPE>
__host__ __device__ constexpr int raw_count() {
    return int((kMaxSmem - kTailBytes - kScaleBytes - stage_count<TYPE>() * stage_bytes<TYPE>()) / RawLayout<TYPE>::kBytes) < 10
               ? int((kMaxSmem - kTailBytes - kScaleBytes - stage_count<TYPE>() * stage_bytes<TYPE>()) / RawLayout<TYPE>::kBytes)
               : 10;
}
template <uint32_t TYPE>
__host__ __device__ constexpr uint32_t smem_bytes() {
    return stage_count<TYPE>() * stage_bytes<TYPE>() + raw_count<TYPE>() * RawLayout<TYPE>::kBytes + kScaleBytes +
           kTailBytes;
}
constexpr uint32_t kTmemCols = 512;  // one CTA per SM owns all of TMEM

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

// try_wait that lets the hardware suspend the thread until the phase
// completes, for at most `hint_ns`, so waiting roles take no issue slots.
__device__ __forceinline__ bool mbar_try_wait_suspend(uint64_t * bar, uint32_t parity, uint32_t hint_ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.b32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0;
}

// Bounded wait: false (with the abort flag raised and `code` recorded) when
// the phase has not completed within kWaitNs, or when another role aborted.
__device__ __noinline__ bool mbar_wait_slow(uint64_t * bar, uint32_t parity, volatile int * abort_flag, int * error,
                                            int code) {
    const uint64_t t0 = global_ns();
    for (;;) {
        if (mbar_try_wait_suspend(bar, parity, kSuspendNs)) return true;
        if (*abort_flag) return false;
        if (global_ns() - t0 > kWaitNs) break;
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

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t * bar, uint32_t bytes) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

// 2D tiled TMA load of one box into this CTA's shared memory (no multicast).
// x is the byte offset along the row: always a multiple of 16 here.
__device__ __forceinline__ void tma_load_2d(void * dst, const CUtensorMap * map, int32_t x, int32_t y, uint64_t * bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
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

// The same with the A operand read from TMEM (K-major: lane = row, each
// 32-bit column a pair of consecutive K values).
__device__ __forceinline__ void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate));
}

// 16 consecutive 32-bit columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t * v) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
        "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
        : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 4-byte asynchronous global -> shared copy (completes at cp_async_wait).
__device__ __forceinline__ void cp_async4(void * dst, const void * src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
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

// f16 pair (V, V) of an exactly representable integer constant.
template <int V>
__device__ __forceinline__ __half2 h2_int_const() {
    constexpr float f = float(V);
    return __float2half2_rn(f);
}

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

// Tensor maps of one launch: weight boxes W0/W1 and the scale box (128 rows
// each), the activation codes (32 x 128 bytes) and partial sums (32 x 32).
struct TcMaps {
    CUtensorMap w0, w1, sc, act, bsums;
};

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
    // output segments: rows [seg_end[k-1], seg_end[k]) -> seg_out[k] [n][rows of k]
    uint32_t nseg;
    uint32_t seg_end[JFB_MATMUL_MAX_SEGMENTS];
    uint32_t seg_epilogue[JFB_MATMUL_MAX_SEGMENTS];
    const float * seg_bias[JFB_MATMUL_MAX_SEGMENTS];
    const float * seg_residual[JFB_MATMUL_MAX_SEGMENTS];
    float * seg_out[JFB_MATMUL_MAX_SEGMENTS];
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

// Position of a work unit: tile = tn * tiles_m + tm, K block b. Advanced one
// unit at a time so that no role divides per unit.
struct Cursor {
    uint32_t tile, b, tm, tn;
    __device__ __forceinline__ void init(uint64_t w, uint32_t nb, uint32_t tiles_m) {
        tile = uint32_t(w / nb);
        b = uint32_t(w - uint64_t(tile) * nb);
        tn = tile / tiles_m;
        tm = tile - tn * tiles_m;
    }
    __device__ __forceinline__ void next(uint32_t nb, uint32_t tiles_m) {
        if (++b == nb) {
            b = 0;
            ++tile;
            if (++tm == tiles_m) {
                tm = 0;
                ++tn;
            }
        }
    }
};

// f16 pair (v, v) of a small integer v with v + BIAS in [0, 1024), without a
// conversion instruction: 0x6400 | u is the f16 number 1024 + u, and
// subtracting 1024 + BIAS is exact.
template <int BIAS>
__device__ __forceinline__ __half2 small_h2(int v) {
    const uint32_t u = uint32_t(v + BIAS) | 0x6400u;
    return __hsub2(bits_h2(u * 0x00010001u), h2_int_const<1024 + BIAS>());
}

// The scale-byte word of 16-value groups [8h + 4part, 8h + 4part + 4) of a
// block: bytes 0..3 of the result are the scales of those four groups.
__device__ __forceinline__ uint32_t scale_word(const uint4 & scv, int h, int part) {
    const int w = 2 * h + part;
    return w == 0 ? scv.x : w == 1 ? scv.y : w == 2 ? scv.z : scv.w;
}

// Converts values [64*part, 64*part + 64) of raw half-block h of tile row m
// (raw stage `r`) into f16 products and stores them into this thread's TMEM
// lane of the stage's A operand (`a_col`: address of plane 0, column 0; plane
// 1 follows 64 columns later). Value k of the half goes to column k / 2, two
// values per 32-bit column. h and part only move byte offsets and shift
// amounts, so every register-array index below is a compile-time constant and
// one body serves all four (h, part) cases. Warp-collective (tcgen05.st).
template <uint32_t TYPE>
__device__ __forceinline__ void convert_a(const uint8_t * r, int h, int part, uint32_t a_col, int m) {
    using RL = RawLayout<TYPE>;
    const uint4 scv = *reinterpret_cast<const uint4 *>(r + RL::kScOff + m * 16);
    const uint32_t col = a_col + 32 * part;
    if constexpr (TYPE == JF_TENSOR_Q4_K) {
        // raw row: code bytes [64h, 64h + 64) of the block; byte 32c' + l holds
        // element 64c' + l (low nibble) and 64c' + 32 + l (high nibble) of the
        // half; this thread covers c' = part, i.e. sub-blocks j = 4h + 2part
        // and j + 1 of the block. The packed 6-bit scale/min of sub-block j:
        // j < 4 (h = 0): low 6 bits of bytes j and j + 4 of the 12; j >= 4
        // (h = 1): nibbles of byte j + 4 with the top 2 bits of bytes j - 4
        // and j.
        const uint4 * codes = reinterpret_cast<const uint4 *>(r + RL::kW0Off + m * 64 + 32 * part);
        const uint4 v0 = codes[0], v1 = codes[1];
        const uint32_t wv[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
#pragma unroll
        for (int nib = 0; nib < 2; ++nib) {
            const int sh = 8 * (2 * part + nib);  // byte jj = j mod 4 of each 4-byte scale word
            const uint32_t b1 = scv.y >> sh, b2 = scv.z >> sh, b3 = scv.w >> sh;
            const int sc = h == 0 ? int(b1 & 63) : int((b3 & 0x0f) | (((b1 >> 6) & 3) << 4));
            const __half2 scale = small_h2<0>(sc);
            const __half2 nbias = __hmul2(scale, h2_int_const<-1024>());
            uint32_t w[16];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const uint2 a = scaled4((wv[2 * q] >> (4 * nib)) & 0x0f0f0f0fu, scale, nbias);
                const uint2 b = scaled4((wv[2 * q + 1] >> (4 * nib)) & 0x0f0f0f0fu, scale, nbias);
                w[4 * q + 0] = a.x;
                w[4 * q + 1] = a.y;
                w[4 * q + 2] = b.x;
                w[4 * q + 3] = b.y;
            }
            (void) b2;
            tmem_st16(col + 16 * nib, w);  // values [32*nib, 32*nib + 32) of this thread
        }
    } else if constexpr (TYPE == JF_TENSOR_Q6_K) {
        // raw rows: ql bytes [64h, 64h + 64) and qh bytes [32h, 32h + 32) of
        // the block. Element r' (0..127) of the half is nibble r' / 64 of
        // ql[r' % 64] with bits 2*(r' / 32) of qh[r' % 32]; this thread covers
        // r' in [64*part, 64*part + 64): nibble `part` of every ql byte and
        // bit pairs 2*part, 2*part + 1 of the qh bytes.
        const uint4 * ql = reinterpret_cast<const uint4 *>(r + RL::kW0Off + m * 64);
        const uint4 * qh = reinterpret_cast<const uint4 *>(r + RL::kW1Off + m * 32);
        const uint4 l0 = ql[0], l1 = ql[1], l2 = ql[2], l3 = ql[3];
        const uint4 q0 = qh[0], q1 = qh[1];
        const uint32_t L[16] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w,
                                l2.x, l2.y, l2.z, l2.w, l3.x, l3.y, l3.z, l3.w};
        const uint32_t Hq[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
        const uint32_t sw = scale_word(scv, h, part);
        const int lsh = 4 * part, hsh = 4 * part;
        const __half2 k1056 = h2_int_const<-1056>();  // 1056 = 1024 + 32
#pragma unroll
        for (int gp = 0; gp < 2; ++gp) {  // 32 values (two scale groups) per pass
            uint32_t whi[16], wlo[16];
#pragma unroll
            for (int g2 = 0; g2 < 2; ++g2) {
                const int grp = 2 * gp + g2;
                const int s = int(int8_t(uint8_t(sw >> (8 * grp))));
                const int s_lo = s & 15, s_hi = (s - s_lo) / 16;
                const __half2 shi = small_h2<8>(s_hi), nhi = __hmul2(shi, k1056);
                const __half2 slo = small_h2<0>(s_lo), nlo = __hmul2(slo, k1056);
#pragma unroll
                for (int half_grp = 0; half_grp < 2; ++half_grp) {
                    const int ch = 2 * grp + half_grp;  // 8-value chunk of this thread
                    uint32_t q[2];
#pragma unroll
                    for (int k = 0; k < 2; ++k) {
                        const int rr = 8 * ch + 4 * k;  // within the thread's 64 values
                        q[k] = ((L[rr / 4] >> lsh) & 0x0f0f0f0fu) |
                               (((Hq[(rr % 32) / 4] >> (hsh + 2 * (rr / 32))) & 0x03030303u) << 4);
                    }
                    const __half2 x0 = magic_pair(q[0], 0x4140u), x1 = magic_pair(q[0], 0x4342u);
                    const __half2 x2 = magic_pair(q[1], 0x4140u), x3 = magic_pair(q[1], 0x4342u);
                    const int o = 4 * (2 * g2 + half_grp);
                    whi[o + 0] = h2_bits(__hfma2(x0, shi, nhi));
                    whi[o + 1] = h2_bits(__hfma2(x1, shi, nhi));
                    whi[o + 2] = h2_bits(__hfma2(x2, shi, nhi));
                    whi[o + 3] = h2_bits(__hfma2(x3, shi, nhi));
                    wlo[o + 0] = h2_bits(__hfma2(x0, slo, nlo));
                    wlo[o + 1] = h2_bits(__hfma2(x1, slo, nlo));
                    wlo[o + 2] = h2_bits(__hfma2(x2, slo, nlo));
                    wlo[o + 3] = h2_bits(__hfma2(x3, slo, nlo));
                }
            }
            tmem_st16(col + 16 * gp, whi);
            tmem_st16(col + 64 + 16 * gp, wlo);
        }
    } else {
        // raw row: qs bytes [32h, 32h + 32); element 32s + l of the half lives
        // in bits 2s of byte l; this thread covers s = 2*part, 2*part + 1
        const uint4 * qs = reinterpret_cast<const uint4 *>(r + RL::kW0Off + m * 32);
        const uint4 a0 = qs[0], a1 = qs[1];
        const uint32_t Q[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
        const uint32_t sw = scale_word(scv, h, part);
#pragma unroll
        for (int gp = 0; gp < 2; ++gp) {
            uint32_t w[16];
#pragma unroll
            for (int g2 = 0; g2 < 2; ++g2) {
                const int grp = 2 * gp + g2;
                const __half2 scale = small_h2<0>(int((sw >> (8 * grp)) & 15));
                const __half2 nbias = __hmul2(scale, h2_int_const<-1024>());
#pragma unroll
                for (int half_grp = 0; half_grp < 2; ++half_grp) {
                    const int r0 = 16 * grp + 8 * half_grp;  // within the thread's 64 values
                    const int shift = 2 * (2 * part + r0 / 32), l0 = r0 % 32;
                    const uint2 x = scaled4((Q[l0 / 4] >> shift) & 0x03030303u, scale, nbias);
                    const uint2 y = scaled4((Q[l0 / 4 + 1] >> shift) & 0x03030303u, scale, nbias);
                    const int o = 4 * (2 * g2 + half_grp);
                    w[o + 0] = x.x;
                    w[o + 1] = x.y;
                    w[o + 2] = y.x;
                    w[o + 3] = y.y;
                }
            }
            tmem_st16(col + 16 * gp, w);
        }
    }
}

// Mins of 16-value groups [8*part, 8*part + 8) of one block as half of a
// K = 16 f16 operand row (Q4_K: the 6-bit min of each 32-value sub-block,
// twice; Q2_K: the high nibble of each scale byte), from the raw scale row of
// tile row m. The two parts of a row write the two 16-byte core columns.
template <uint32_t TYPE>
__device__ __forceinline__ void convert_mins(const uint8_t * r, int part, uint8_t * tile, int m) {
    const uint4 meta = *reinterpret_cast<const uint4 *>(r + RawLayout<TYPE>::kScOff + m * 16);
    uint32_t h2[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        int m0, m1;
        if constexpr (TYPE == JF_TENSOR_Q4_K) {
            // sub-block j = 4*part + k: j < 4 -> low 6 bits of byte j + 4 of the
            // 12; j >= 4 -> high nibble of byte j + 4 with the top 2 bits of byte j
            const int sh = 8 * k;
            const uint32_t b1 = meta.y >> sh, b2 = meta.z >> sh, b3 = meta.w >> sh;
            m0 = part == 0 ? int(b2 & 63) : int(((b3 >> 4) & 0x0f) | (((b2 >> 6) & 3) << 4));
            (void) b1;
            m1 = m0;
        } else {
            const uint32_t word = part == 0 ? (k < 2 ? meta.x : meta.y) : (k < 2 ? meta.z : meta.w);
            m0 = int((word >> (16 * (k & 1) + 4)) & 15);
            m1 = int((word >> (16 * (k & 1) + 12)) & 15);
        }
        const uint32_t u = (uint32_t(m0) | 0x6400u) | ((uint32_t(m1) | 0x6400u) << 16);  // mins < 64
        h2[k] = h2_bits(__hsub2(bits_h2(u), h2_int_const<1024>()));
    }
    *reinterpret_cast<uint4 *>(tile + (m >> 3) * kSbo16 + part * 128 + (m & 7) * 16) = make_uint4(h2[0], h2[1], h2[2], h2[3]);
}

template <uint32_t TYPE>
__global__ void __launch_bounds__(kThreads, 1) mmq_tc_kernel(const __grid_constant__ TcMaps maps, TcParams p) {
    using T = TypeTraits<TYPE>;
    using RL = RawLayout<TYPE>;
    constexpr int NS = stage_count<TYPE>();
    constexpr int NR = raw_count<TYPE>();
    constexpr uint32_t kStage = stage_bytes<TYPE>();
    constexpr uint32_t kBOff = 0;
    constexpr uint32_t kA2Off = kBOff + kBBytes;
    constexpr uint32_t kB2Off = kA2Off + kA2Bytes;
    constexpr uint32_t kAccCols = acc_columns<TYPE>();
    constexpr uint32_t kACols = a_columns<TYPE>();

    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t * raw = smem + NS * kStage;                    // [NR][RL::kBytes]
    uint8_t * scales = raw + NR * RL::kBytes;              // epilogue scale rings
    uint8_t * tail = scales + kScaleBytes;
    uint64_t * full = reinterpret_cast<uint64_t *>(tail);  // [NS]
    uint64_t * empty = full + NS;                          // [NS]
    uint64_t * raw_full = empty + NS;                      // [NR]
    uint64_t * raw_empty = raw_full + NR;                  // [NR]
    uint64_t * acc_full = raw_empty + NR;                  // [2]
    uint64_t * acc_empty = acc_full + 2;                   // [2]
    uint64_t * drain = acc_empty + 2;                      // [1]
    uint32_t * tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
    volatile int * abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint64_t g = gridDim.x;
    const uint64_t w_begin = range_start(blockIdx.x, p.work, g);
    const uint64_t w_end = range_start(blockIdx.x + 1, p.work, g);
    const uint32_t nb = p.blocks;

    if (threadIdx.x == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(&full[s], kConverterThreads);
            mbar_init(&empty[s], 1);
        }
        for (int s = 0; s < NR; ++s) {
            mbar_init(&raw_full[s], 1);
            mbar_init(&raw_empty[s], kConverterThreads);
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

    if (warp == kTmaWarp) {
        // ---------------- TMA loads of the raw stages (one thread) ----------------
        if (lane == 0) {
            uint32_t rs = 0, rph = 0;
            uint64_t issued = 0;
            bool ok = true;
            Cursor cur;
            cur.init(w_begin, nb, p.tiles_m);
            for (uint64_t w = w_begin; w < w_end && ok && !*abort_flag; ++w, cur.next(nb, p.tiles_m)) {
                const uint32_t b = cur.b;
                const int32_t y_w = int32_t(cur.tm * kRows), y_a = int32_t(cur.tn * kBN);
                for (int h = 0; h < 2; ++h) {
                    if (!mbar_wait(&raw_empty[rs], rph ^ 1u, abort_flag, p.error, kErrWaitRawEmpty)) {
                        ok = false;
                        break;
                    }
                    uint8_t * r = raw + rs * RL::kBytes;
                    mbar_arrive_expect_tx(&raw_full[rs], RL::kBytes);
                    const int32_t x_blk = int32_t(b * T::kBlockBytes);
                    tma_load_2d(r + RL::kW0Off, &maps.w0, x_blk + int32_t(T::kW0 * h), y_w, &raw_full[rs]);
                    if constexpr (T::kW1 > 0) {
                        tma_load_2d(r + RL::kW1Off, &maps.w1, x_blk + 128 + int32_t(T::kW1 * h), y_w, &raw_full[rs]);
                    }
                    tma_load_2d(r + RL::kScOff, &maps.sc, int32_t(b * 16), y_w, &raw_full[rs]);
                    tma_load_2d(r + RL::kActOff, &maps.act, int32_t(b * kQK + 128 * h), y_a, &raw_full[rs]);
                    if constexpr (T::kMins) tma_load_2d(r + RL::kBsOff, &maps.bsums, int32_t(b * 32), y_a, &raw_full[rs]);
                    ++issued;
                    if (++rs == NR) {
                        rs = 0;
                        rph ^= 1u;
                    }
                }
            }
            // a stopped kernel must not exit with loads still landing in its
            // shared memory: wait (bounded) for the last issue of every stage
            if (*abort_flag) {
                volatile int no_abort = 0;
                for (uint64_t j = issued > uint64_t(NR) ? issued - NR : 0; j < issued; ++j) {
                    (void) mbar_wait(&raw_full[j % NR], uint32_t((j / NR) & 1u), &no_abort, nullptr, 0);
                }
            }
        }
        __syncwarp();
    } else if (warp >= kEpilogueWarps && warp < kMmaWarp) {
        // ---------------- converters ----------------
        const int pt = threadIdx.x - kEpilogueThreads;
        const int m = pt & (kRows - 1), part = pt >> 7;  // part is uniform per warp
        const uint32_t lane_base = uint32_t((warp & 3) * 32) << 16;  // this warp's TMEM lane quarter
        const __half2 act_nbias = h2_int(-1152);  // codes arrive as q + 128 after the sign flip
        const __half2 one = h2_int(1);
        uint32_t stage = 0, phase = 0, rs = 0, rph = 0;
        for (uint64_t w = w_begin; w < w_end; ++w) {
            if (__any_sync(0xffffffffu, *abort_flag != 0)) break;
            bool ok = true;
            for (int h = 0; h < 2; ++h) {
                // the whole warp proceeds or stops together (TMEM stores are warp-collective)
                const bool ready = mbar_wait(&raw_full[rs], rph, abort_flag, p.error, kErrWaitRawFull) &&
                                   mbar_wait(&empty[stage], phase ^ 1u, abort_flag, p.error, kErrWaitEmpty);
                if (!__all_sync(0xffffffffu, ready)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint8_t * r = raw + rs * RL::kBytes;
                uint8_t * st = smem + stage * kStage;
                convert_a<TYPE>(r, h, part, tmem + lane_base + kAccCols + stage * kACols, m);
                if (T::kMins && h == 0) convert_mins<TYPE>(r, part, st + kA2Off, m);
                // activation codes: one token t and 16 codes (chunk pair c16) per
                // thread. The raw tile arrives 128-byte swizzled (16-byte chunk c
                // of token row t at chunk c ^ (t & 7)), so the 8 lanes that share
                // c16 read 8 different bank groups; they also write 128
                // contiguous bytes of the B tile.
                {
                    const int t_low = pt & 7, c16 = (pt >> 3) & 7, t = ((pt >> 6) << 3) | t_low;
                    const uint4 v = *reinterpret_cast<const uint4 *>(r + RL::kActOff + t * 128 + ((c16 ^ t_low) << 4));
                    const uint2 a = scaled4(v.x ^ 0x80808080u, one, act_nbias);
                    const uint2 b = scaled4(v.y ^ 0x80808080u, one, act_nbias);
                    const uint2 c = scaled4(v.z ^ 0x80808080u, one, act_nbias);
                    const uint2 d = scaled4(v.w ^ 0x80808080u, one, act_nbias);
                    uint8_t * dst = st + kBOff + (t >> 3) * kSbo + (2 * c16) * 128 + (t & 7) * 16;
                    *reinterpret_cast<uint4 *>(dst) = make_uint4(a.x, a.y, b.x, b.y);
                    *reinterpret_cast<uint4 *>(dst + 128) = make_uint4(c.x, c.y, d.x, d.y);
                }
                if (T::kMins && h == 0 && pt < kBN * 2) {
                    const int t = pt >> 1, c = pt & 1;
                    const uint4 v = *reinterpret_cast<const uint4 *>(r + RL::kBsOff + t * 32 + 16 * c);
                    const uint32_t rw[4] = {v.x, v.y, v.z, v.w};
                    uint32_t hv[4];
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        hv[k] = h2_bits(__halves2half2(__int2half_rn(int(int16_t(rw[k] & 0xffffu))),
                                                       __int2half_rn(int(int16_t(rw[k] >> 16)))));
                    }
                    *reinterpret_cast<uint4 *>(st + kB2Off + (t >> 3) * kSbo16 + c * 128 + (t & 7) * 16) =
                        make_uint4(hv[0], hv[1], hv[2], hv[3]);
                }
                tmem_wait_st();
                tc_fence_before();
                fence_proxy_async();
                mbar_arrive(&full[stage]);
                mbar_arrive(&raw_empty[rs]);
                if (++stage == NS) {
                    stage = 0;
                    phase ^= 1u;
                }
                if (++rs == NR) {
                    rs = 0;
                    rph ^= 1u;
                }
            }
            if (!ok) break;
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
                    const uint32_t a = tmem + kAccCols + stage * kACols;
#pragma unroll
                    for (int ks = 0; ks < kKStage / 16; ++ks) {
                        const uint64_t bdesc = smem_desc(st + kBOff + ks * 256, 128, kSbo);
                        if constexpr (TYPE == JF_TENSOR_Q4_K) {
                            mma_f16_ts(d + h * kBN, a + ks * 8, bdesc, idesc, ks > 0 ? 1u : 0u);
                        } else if constexpr (TYPE == JF_TENSOR_Q6_K) {
                            const uint32_t accum = (h > 0 || ks > 0) ? 1u : 0u;
                            mma_f16_ts(d, a + ks * 8, bdesc, idesc, accum);
                            mma_f16_ts(d + kBN, a + 64 + ks * 8, bdesc, idesc, accum);
                        } else {
                            mma_f16_ts(d, a + ks * 8, bdesc, idesc, (h > 0 || ks > 0) ? 1u : 0u);
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
        constexpr int kCols = kBN / 2;  // token columns of this thread
        const int m = (warp & 3) * 32 + lane;  // TMEM lane quarter of the warp = its 32 weight rows
        const int col0 = (warp >> 2) * kCols;
        const uint32_t lane_base = uint32_t((warp & 3) * 32) << 16;
        // scale rings of this warp: [kScaleRing][32] weight scale words (own row), [kScaleRing][32] activation d
        uint32_t * dring = reinterpret_cast<uint32_t *>(scales) + warp * kScaleRing * 64;
        float * aring = reinterpret_cast<float *>(dring + kScaleRing * 32);
        const uint8_t * p1 = static_cast<const uint8_t *>(p.w.plane[1]);
        const uint8_t * p2 = static_cast<const uint8_t *>(p.w.plane[2]);
        const uint32_t first_tile = uint32_t(w_begin / nb);
        Cursor ahead;  // the unit whose scales are staged next
        ahead.init(w_begin, nb, p.tiles_m);
        // stage unit w (at cursor `ahead`) into ring slot `slot` (one commit group per unit, possibly empty)
        auto stage_scales = [&](uint64_t w, int slot) {
            if (w < w_end) {
                const uint32_t b = ahead.b;
                const uint32_t row = ahead.tm * kRows + uint32_t(m), tok = ahead.tn * kBN + lane;
                if (row < p.w.rows) {
                    const uint64_t block = uint64_t(row) * nb + b;
                    const uint8_t * src = TYPE == JF_TENSOR_Q4_K ? p1 + block * 16        // d | dmin << 16
                                          : TYPE == JF_TENSOR_Q6_K ? p2 + ((block * 2) & ~uint64_t(3))  // word holding d
                                                                   : p2 + block * 4;      // d | dmin << 16
                    cp_async4(&dring[slot * 32 + lane], src);
                } else {
                    dring[slot * 32 + lane] = 0;
                }
                if (tok < p.n) cp_async4(&aring[slot * 32 + lane], p.da + uint64_t(tok) * nb + b);
                else aring[slot * 32 + lane] = 0.0f;
                ahead.next(nb, p.tiles_m);
            }
            cp_async_commit();
        };
#pragma unroll
        for (int k = 0; k < kScaleRing; ++k) stage_scales(w_begin + k, k);
        double sum[kCols];
        uint64_t seg_begin = w_begin;
        uint32_t i = 0;
        Cursor cur;
        cur.init(w_begin, nb, p.tiles_m);
        for (uint64_t w = w_begin; w < w_end; ++w, ++i, cur.next(nb, p.tiles_m)) {
            // warp-uniform stop: the warp collectives below need every lane
            if (__any_sync(0xffffffffu, *abort_flag != 0)) break;
            const uint32_t tile = cur.tile;
            const uint32_t row = cur.tm * kRows + uint32_t(m), tok0 = cur.tn * kBN;
            if (w == seg_begin) {
#pragma unroll
                for (int t = 0; t < kCols; ++t) sum[t] = 0.0;
            }
            const int slot = int(i % kScaleRing);
            cp_async_wait<kScaleRing - 1>();  // unit i's group is complete
            __syncwarp();
            float dw, dmin = 0.0f;
            {
                const uint32_t word = dring[slot * 32 + lane];
                if constexpr (TYPE == JF_TENSOR_Q6_K) {
                    const uint32_t odd = ((row & nb) + cur.b) & 1u;  // parity of block row * nb + b
                    dw = half_bits_to_float(uint16_t(odd ? word >> 16 : word & 0xffffu));
                } else {
                    dw = half_bits_to_float(uint16_t(word & 0xffffu));
                    dmin = half_bits_to_float(uint16_t(word >> 16));
                }
            }
            const float * da_s = aring + slot * 32;

            const uint32_t acc = i & 1u, use = i >> 1;
            // the whole warp proceeds or stops together
            const bool ready = mbar_wait(&acc_full[acc], use & 1u, abort_flag, p.error, kErrWaitAccFull);
            if (!__all_sync(0xffffffffu, ready)) break;
            tc_fence_after();
            const uint32_t base = tmem + lane_base + acc * (T::kAcc * kBN) + col0;
#pragma unroll
            for (int ch = 0; ch < kCols / 8; ++ch) {
                uint32_t r0[8], r1[8], r2[8];
                tmem_ld8(base + 8 * ch, r0);
                tmem_ld8(base + kBN + 8 * ch, r1);
                if constexpr (T::kAcc == 3) tmem_ld8(base + 2 * kBN + 8 * ch, r2);
                tmem_wait_ld();
                if (ch == kCols / 8 - 1) {
                    tc_fence_before();
                    mbar_arrive(&acc_empty[acc]);  // the accumulators may be overwritten now
                }
                const float4 da0 = *reinterpret_cast<const float4 *>(da_s + col0 + 8 * ch);
                const float4 da1 = *reinterpret_cast<const float4 *>(da_s + col0 + 8 * ch + 4);
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
            __syncwarp();  // every lane is done with slot `slot` before it is refilled
            stage_scales(w + kScaleRing, slot);

            // a segment ends where the CTA's range or the tile's K range ends
            if (w + 1 != w_end && cur.b + 1 != nb) continue;
            const bool complete = seg_begin == uint64_t(tile) * nb && w + 1 == uint64_t(tile + 1) * nb;
            seg_begin = w + 1;
            if (!complete) {
                const uint32_t slot_p = 2 * blockIdx.x + (tile == first_tile ? 0 : 1);
                double * part = p.partial + uint64_t(slot_p) * kSlotDoubles;
#pragma unroll
                for (int t = 0; t < kCols; ++t) part[(col0 + t) * kRows + m] = sum[t];
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
                // contributors after `lo` start inside this tile, so it is their
                // first tile (slot 2c); `lo` used slot 2lo + 1 unless its range
                // starts exactly at the tile. Partials are added in CTA order,
                // eight tokens at a time, with the loads of several
                // contributors in flight together.
                const uint64_t lo_slot = 2 * uint64_t(lo) + (range_start(lo, p.work, g) == uint64_t(tile) * nb ? 0 : 1);
                const double * lo_src = p.partial + lo_slot * kSlotDoubles + col0 * kRows + m;
                const double * rest = p.partial + 2 * uint64_t(lo + 1) * kSlotDoubles + col0 * kRows + m;
#pragma unroll
                for (int t0 = 0; t0 < kCols; t0 += 8) {
                    double acc8[8];
#pragma unroll
                    for (int k = 0; k < 8; ++k) acc8[k] = 0.0 + __ldcg(lo_src + (t0 + k) * kRows);
#pragma unroll 4
                    for (uint32_t c = 0; c < hi - lo; ++c) {
                        const double * src = rest + uint64_t(2 * c) * kSlotDoubles;
                        double v[8];
#pragma unroll
                        for (int k = 0; k < 8; ++k) v[k] = __ldcg(src + (t0 + k) * kRows);
#pragma unroll
                        for (int k = 0; k < 8; ++k) acc8[k] += v[k];
                    }
#pragma unroll
                    for (int k = 0; k < 8; ++k) sum[t0 + k] = acc8[k];
                }
            }
            if (row < p.w.rows) {
                // this row's output segment
                int k = 0;
#pragma unroll
                for (int j = 0; j < JFB_MATMUL_MAX_SEGMENTS - 1; ++j) k += (j < int(p.nseg) - 1 && row >= p.seg_end[j]) ? 1 : 0;
                const uint32_t seg_begin_row = k == 0 ? 0u : p.seg_end[k - 1];
                const uint32_t ld = p.seg_end[k] - seg_begin_row, r = row - seg_begin_row;
                const uint32_t ep = p.seg_epilogue[k];
                float * out = p.seg_out[k];
                const float * bias = p.seg_bias[k];
                const float * residual = p.seg_residual[k];
#pragma unroll
                for (int t = 0; t < kCols; ++t) {
                    const uint32_t tok = tok0 + col0 + t;
                    if (tok >= p.n) break;
                    const uint64_t at = uint64_t(tok) * ld + r;
                    float v = __double2float_rn(sum[t]);
                    if (ep == JFB_EPILOGUE_BIAS) v = __fadd_rn(v, bias[r]);
                    else if (ep == JFB_EPILOGUE_RESIDUAL) v = __fadd_rn(v, residual[at]);
                    out[at] = v;
                }
            }
        }
        cp_async_wait<0>();  // no copy may land after the kernel ends
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

// ---- tensor maps ----------------------------------------------------------------

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void * f = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess) {
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
        }
    });
    return fn;
}

// A tensor map is a pure function of its parameters, so encoded maps are
// cached by the full parameter tuple (bounded; cleared when it grows large).
bool byte_tensor_map(CUtensorMap & out, const void * base, uint64_t row_bytes, uint64_t rows, uint32_t box_bytes,
                     uint32_t box_rows, bool swizzle128 = false) {
    using Key = std::tuple<uintptr_t, uint64_t, uint64_t, uint32_t, uint32_t, bool>;
    static std::mutex mu;
    static std::map<Key, CUtensorMap> cache;
    const Key key{reinterpret_cast<uintptr_t>(base), row_bytes, rows, box_bytes, box_rows, swizzle128};
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) {
        out = it->second;
        return true;
    }
    PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
    if (encode == nullptr) return false;
    const cuuint64_t dims[2] = {row_bytes, rows};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {box_bytes, box_rows};
    const cuuint32_t elem[2] = {1, 1};
    CUtensorMap map;
    std::memset(&map, 0, sizeof(map));
    if (encode(&map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims, strides, box, elem,
               CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
               CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
        return false;
    }
    if (cache.size() >= 4096) cache.clear();
    cache.emplace(key, map);
    out = map;
    return true;
}

template <uint32_t TYPE>
jfb_status build_maps(TcMaps & maps, const TcParams & p, uint32_t cols) {
    using T = TypeTraits<TYPE>;
    const uint64_t nb = p.blocks;
    bool ok = byte_tensor_map(maps.w0, p.w.plane[0], nb * T::kBlockBytes, p.w.rows, T::kW0, kRows) &&
              byte_tensor_map(maps.w1, p.w.plane[0], nb * T::kBlockBytes, p.w.rows, T::kW1 > 0 ? T::kW1 : 16, kRows) &&
              byte_tensor_map(maps.sc, p.w.plane[1], nb * 16, p.w.rows, 16, kRows) &&
              byte_tensor_map(maps.act, p.qs, cols, p.n, 128, kBN, true) &&
              byte_tensor_map(maps.bsums, p.bsums, uint64_t(cols) / 8, p.n, 32, kBN);
    if (!ok) return status_error(JFB_STATUS_CUDA_ERROR, "jfb_matmul_tc: could not encode a TMA tensor map");
    return status_ok();
}

template <uint32_t TYPE>
jfb_status launch(TcParams & p, uint32_t cols, uint32_t grid, cudaStream_t s) {
    constexpr uint32_t bytes = smem_bytes<TYPE>();
    static_assert(bytes <= kMaxSmem, "shared memory budget");
    static_assert(raw_count<TYPE>() >= 2, "raw pipeline depth");
    static_assert(stage_count<TYPE>() >= 2, "operand pipeline depth");
    static_assert(acc_columns<TYPE>() + stage_count<TYPE>() * a_columns<TYPE>() <= kTmemCols, "TMEM budget");
    static_assert(RawLayout<TYPE>::kBytes % 1024 == 0 && RawLayout<TYPE>::kActOff % 1024 == 0,
                  "raw stages and the swizzled activation box stay 1024-byte aligned");
    static_assert(kConverterThreads == kBN * 8, "one converter thread per token and 16-code chunk");
    TcMaps maps;
    jfb_status st = build_maps<TYPE>(maps, p, cols);
    if (st.code != JFB_STATUS_OK) return st;
    auto kernel = mmq_tc_kernel<TYPE>;
    // the shared-memory opt-in is a per-device function attribute: set once
    static std::mutex mu;
    static bool attribute_set[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = 0;
    {
        std::lock_guard<std::mutex> lock(mu);
        if (!attribute_set[dev]) {
            const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(bytes));
            if (e != cudaSuccess) {
                return status_error(JFB_STATUS_CUDA_ERROR, "jfb_matmul_tc: shared memory attribute: %s",
                                    cudaGetErrorString(e));
            }
            attribute_set[dev] = true;
        }
    }
    kernel<<<grid, kThreads, bytes, s>>>(maps, p);
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

extern "C" jfb_status jfb_matmul_tc_segments(const jfb_weight * weight, const jfb_q8k * x_q8, uint32_t n,
                                             const jfb_matmul_segment * segments, uint32_t segment_count,
                                             void * workspace, uint64_t workspace_size, int32_t * error_flag,
                                             void * stream) {
    if (weight == nullptr || x_q8 == nullptr || segments == nullptr) {
        return status_error(JFB_STATUS_INVALID_ARGUMENT, "weight, activations and output segments are required");
    }
    if (!jfb_matmul_tc_supported(weight)) {
        return status_error(JFB_STATUS_UNSUPPORTED, "jfb_matmul_tc needs a Q4_K, Q6_K or Q2_K weight");
    }
    if (segment_count == 0 || segment_count > JFB_MATMUL_MAX_SEGMENTS) {
        return status_error(JFB_STATUS_INVALID_ARGUMENT, "1 to %d output segments are supported", JFB_MATMUL_MAX_SEGMENTS);
    }
    uint32_t prev = 0;
    for (uint32_t k = 0; k < segment_count; ++k) {
        const jfb_matmul_segment & g = segments[k];
        if (g.out == nullptr || g.row_end <= prev || g.epilogue > JFB_EPILOGUE_RESIDUAL ||
            (g.epilogue == JFB_EPILOGUE_BIAS && g.bias == nullptr) ||
            (g.epilogue == JFB_EPILOGUE_RESIDUAL && g.residual == nullptr)) {
            return status_error(JFB_STATUS_INVALID_ARGUMENT, "matmul output segment %u is invalid", k);
        }
        prev = g.row_end;
    }
    if (prev != weight->rows) {
        return status_error(JFB_STATUS_INVALID_ARGUMENT, "output segments must end at the weight's %u rows", weight->rows);
    }
    if (n == 0) return status_ok();
    if (x_q8->qs == nullptr || x_q8->d == nullptr || x_q8->bsums == nullptr) {
        return status_error(JFB_STATUS_INVALID_ARGUMENT, "Q8_K activation planes are required");
    }
    if ((reinterpret_cast<uintptr_t>(x_q8->qs) & 15u) != 0 || (reinterpret_cast<uintptr_t>(x_q8->bsums) & 15u) != 0) {
        return status_error(JFB_STATUS_INVALID_ARGUMENT, "Q8_K codes and partial sums must be 16-byte aligned");
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
    p.nseg = segment_count;
    for (uint32_t k = 0; k < JFB_MATMUL_MAX_SEGMENTS; ++k) {
        const bool used = k < segment_count;
        p.seg_end[k] = used ? segments[k].row_end : weight->rows;
        p.seg_epilogue[k] = used ? segments[k].epilogue : JFB_EPILOGUE_STORE;
        p.seg_bias[k] = used ? segments[k].bias : nullptr;
        p.seg_residual[k] = used ? segments[k].residual : nullptr;
        p.seg_out[k] = used ? segments[k].out : nullptr;
    }
    p.partial = static_cast<double *>(workspace);
    p.counters = reinterpret_cast<uint32_t *>(static_cast<uint8_t *>(workspace) + partial_bytes());
    p.error = error_flag;
    cudaStream_t s = as_stream(stream);
    switch (weight->type) {
    case JF_TENSOR_Q4_K: return launch<JF_TENSOR_Q4_K>(p, weight->cols, pl.grid, s);
    case JF_TENSOR_Q6_K: return launch<JF_TENSOR_Q6_K>(p, weight->cols, pl.grid, s);
    default: return launch<JF_TENSOR_Q2_K>(p, weight->cols, pl.grid, s);
    }
}

extern "C" jfb_status jfb_matmul_tc(const jfb_weight * weight, const jfb_q8k * x_q8, uint32_t n, uint32_t epilogue,
                                    const float * bias, const float * residual, float * out, void * workspace,
                                    uint64_t workspace_size, int32_t * error_flag, void * stream) {
    if (weight == nullptr || x_q8 == nullptr || out == nullptr) {
        return status_error(JFB_STATUS_INVALID_ARGUMENT, "weight, activations and output are required");
    }
    if (epilogue > JFB_EPILOGUE_RESIDUAL || (epilogue == JFB_EPILOGUE_BIAS && bias == nullptr) ||
        (epilogue == JFB_EPILOGUE_RESIDUAL && residual == nullptr)) {
        return status_error(JFB_STATUS_INVALID_ARGUMENT, "matmul epilogue operands are missing");
    }
    const jfb_matmul_segment seg{weight->rows, epilogue, bias, residual, out};
    return jfb_matmul_tc_segments(weight, x_q8, n, &seg, 1, workspace, workspace_size, error_flag, stream);
}
