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
// The epilogue rounds every block term exactly as the CPU does (the products
// with packed f32x2 multiplies, which round each lane like the scalar ones,
// the final difference with scalar non-contractible subtractions) and adds it
// to a per-(row, token) double sum, as the CUDA-core kernel does.
//
// Operands. The quantizers of this library also write the Q8_K codes and
// 16-value partial sums as f16 numbers and the block scales d transposed
// (jfb_q8k.qs_f16, bsums_f16, d_t). The activation operand therefore arrives
// by TMA already in the tensor cores' layout and is never converted here: the
// codes as 128-byte swizzled K-major boxes (SWIZZLE_128B, 64 codes per row),
// the partial sums as two 8-wide no-swizzle boxes that form the canonical
// K-major core-matrix layout, and each unit's activation scales as one row of
// d_t. Only the weights are converted: every weight code becomes its exact
// f16 product in tensor memory (the A operand, lane = weight row).
//
// Schedule. Persistent stream-K: grid G = min(SMs, W) and CTA c walks the
// contiguous work range [c*W/G, (c+1)*W/G) of W = tiles * blocks units. A tile
// is 128 weight rows x BN activation rows (BN = 32 for n <= 32, else 64); a
// unit is one 256-block of K. When a tile's K range spans several CTAs, each
// epilogue warp writes its double partials and the last warp to arrive (a
// per-tile, per-warp counter) adds all contributors' partials in CTA order, so
// the result does not depend on timing and no CTA ever waits for another.
//
// Warp roles (BN = 32: 19 warps; BN = 64: 15 warps):
//   epilogue    8 warps: warp w owns TMEM lanes 32(w % 4)..+31 (weight rows)
//               and token columns (BN/2)(w / 4)..+BN/2-1;
//   converters  8 warps for BN = 32 (two threads per weight row, 64 values
//               each per half-block), 4 for BN = 64 (one thread per row):
//               weight codes -> exact f16 products in TMEM (tcgen05.st), the
//               mins -> a K = 16 shared-memory tile, and each row's block
//               scale word -> the epilogue ring;
//   MMA         two warps, one issuing thread each, for the even and the odd
//               units (the first also allocates TMEM): the tcgen05.mma chain
//               of each half-block; commits free the A stage, the raw stage
//               (which holds B) and hand the accumulator to the epilogue;
//   TMA         one thread: the 2D loads (cp.async.bulk.tensor, no multicast)
//               of the raw stages (weights, scale bytes, f16 codes, f16
//               partial sums) and of each unit's activation scales, several
//               units ahead, completing on mbarrier transaction counts.
// Accumulators are double-buffered in TMEM, so the MMAs of unit i+1 overlap
// the epilogue of unit i. Every mbarrier wait is bounded by a 2 s global-timer
// limit: on expiry the kernel records an error code, every role stops,
// in-flight MMAs and TMA loads are drained and TMEM is released.
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

constexpr int kRows = 128;             // MMA M: weight rows per tile
constexpr int kKStage = 128;           // K values per pipeline stage (half a block)
constexpr uint32_t kSbo16 = 256;       // 8-row group stride of the K = 16 mins tile
constexpr uint32_t kA2Bytes = kRows * 16 * 2;         // 4 KB
constexpr uint32_t kMaxSmem = 232448;                 // sm_100 opt-in limit per block
constexpr uint32_t kTailBytes = 1024;                 // barriers, TMEM slot, flags
constexpr uint64_t kWaitNs = 2000000000ull;           // bound of every pipeline wait
constexpr uint32_t kSuspendNs = 1000000;              // longest single suspension of a waiting thread
constexpr uint32_t kTmemCols = 512;                   // one CTA per SM owns all of TMEM
constexpr int kEpiRing = 8;                           // units of activation scales staged ahead
constexpr uint32_t kEpiSlotBytes = 256;               // [BN] activation d

enum : int {
    kErrWaitEmpty = 1,
    kErrWaitAccEmpty = 2,
    kErrWaitFull = 3,
    kErrWaitAccFull = 4,
    kErrWaitRawEmpty = 5,
    kErrWaitRawFull = 6,
    kErrWaitEpiEmpty = 7,
    kErrWaitEpiFull = 8,
    kErrSmemAlign = 9,
    kErrWaitReduce = 10,
};

// Per type: A planes (Q6_K: hi and lo), accumulators per unit, raw weight
// bytes per row and half-block (W0, W1) and plane-0 bytes per block.
template <uint32_t TYPE>
struct TypeTraits;
template <>
struct TypeTraits<JF_TENSOR_Q4_K> {
    static constexpr int kPlanes = 1, kAcc = 3;  // D(half 0), D(half 1), mins
    static constexpr bool kMins = true;
    static constexpr uint32_t kW0 = 64, kW1 = 0;  // bytes per row: codes of the half-block
    static constexpr uint32_t kBlockBytes = 128;
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

// Warp roles for BN activation rows per tile.
template <int BN>
struct Roles {
    // 4 TMEM lane quarters x 2 (32-token tiles) or 4 (64-token tiles) column
    // groups: 16 token columns per epilogue thread either way, and four
    // epilogue warps per SM sub-partition on 64-token tiles to hide the TMEM
    // load latency of the per-block epilogue
    static constexpr int kEpiWarps = BN == 64 ? 16 : 8;
    static constexpr int kCols = BN * 4 / kEpiWarps;  // token columns per epilogue thread
    // converter groups: with two, group g converts half-block g of every
    // unit, so the two halves of a unit are converted concurrently
    static constexpr int kGroups = 2;
    static constexpr int kGroupWarps = BN == 32 ? 8 : 4;
    static constexpr int kConvWarps = kGroups * kGroupWarps;
    static constexpr int kParts = kGroupWarps * 32 / kRows;  // converter threads per weight row in a group
    // the epilogue's per-(row, token) double sums: shared memory for 32-token
    // tiles (which frees the registers for the second converter group),
    // registers for 64-token tiles
    static constexpr bool kSmemSums = BN == 32;
    // two alternating shared-memory sum buffers when the sums live there
    static constexpr uint32_t kSumBufs = kSmemSums ? 2 : 0;
    // cluster schedules (K slices of a tile added over distributed shared
    // memory) for 32-token tiles; 64-token launches always run stream-K
    static constexpr bool kClusters = kSmemSums;
    // two MMA warps issue alternate units: a memory read by an issuing
    // thread (its barrier waits) stalls its issue for hundreds of cycles, and
    // the other thread's MMAs keep the tensor pipe busy meanwhile
    static constexpr int kMmaWarp = kEpiWarps + kConvWarps;
    static constexpr int kMmaWarps = 2;
    static constexpr int kTmaWarp = kMmaWarp + kMmaWarps;
    static constexpr int kTmaWarps = 2;  // one TMA-issuing thread per half-block
    static constexpr int kWarps = kTmaWarp + kTmaWarps;
    static constexpr int kThreads = kWarps * 32;
    // registers per thread: each of the SM's 4 sub-partitions has 16 K
    // registers for the warps w with w % 4 == its index, allocated in
    // multiples of 8 per thread
    static constexpr int kRegs = (16384 / (((kWarps + 3) / 4) * 32)) / 8 * 8;
};

// Shared and tensor memory of one (type, BN):
//   raw stage (one TMA transaction per half-block): the f16 codes as two
//   swizzled 64-code boxes [BN][128 B], the weight boxes W0 (and W1) of 128
//   rows, the scale/header box [128][16 B] and, for types with mins in half 0,
//   the f16 partial sums as two boxes [BN][16 B];
//   operand stage: the K = 16 mins tile of A (types with mins);
//   epilogue sums (32-token tiles): two [BN][128] double buffers of running sums;
//   epilogue ring: per unit the activation scales d of the tile's tokens.
template <uint32_t TYPE, int BN>
struct Layout {
    using T = TypeTraits<TYPE>;
    static constexpr uint32_t kBOff = 0;
    static constexpr uint32_t kBHalf = uint32_t(BN) * 128;
    static constexpr uint32_t kW0Off = 2 * kBHalf;
    static constexpr uint32_t kW1Off = kW0Off + kRows * T::kW0;
    static constexpr uint32_t kScOff = kW1Off + kRows * T::kW1;
    static constexpr uint32_t kB2Off = kScOff + kRows * 16;
    static constexpr uint32_t kB2Bytes = T::kMins ? uint32_t(BN) * 32 : 0;
    static constexpr uint32_t kTx0 = kB2Off + kB2Bytes;  // transaction bytes of half 0
    static constexpr uint32_t kTx1 = kB2Off;             // half 1 (no partial sums)
    static constexpr uint32_t kRawBytes = (kTx0 + 1023) / 1024 * 1024;
    static constexpr uint32_t kAccCols = 2 * T::kAcc * uint32_t(BN);  // both accumulator buffers
    static constexpr uint32_t kACols = T::kPlanes * (kKStage / 2);    // one A stage: 64 columns per plane
    // with two converter groups each group owns every other A stage and raw
    // stage, so both counts are even
    static constexpr int kStep = Roles<BN>::kGroups;
    static constexpr int kNsFit = int((kTmemCols - kAccCols) / kACols);
    static constexpr int NS = (kNsFit < 4 ? kNsFit : 4) / kStep * kStep;
    static constexpr uint32_t kOpBytes = T::kMins ? kA2Bytes : 0;
    static constexpr uint32_t kSumBytes = Roles<BN>::kSumBufs * uint32_t(kRows) * BN * 8;
    static constexpr uint32_t kFixed = uint32_t(NS) * kOpBytes + kSumBytes + kEpiRing * kEpiSlotBytes + kTailBytes;
    static constexpr int kNrFit = int((kMaxSmem - kFixed) / kRawBytes);
    static constexpr int NR = (kNrFit < 12 ? kNrFit : 12) / kStep * kStep;
    static constexpr uint32_t kSmem = uint32_t(NR) * kRawBytes + kFixed;
};

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

// Two bounded waits whose first polls are issued together, so that two
// phases that have already completed cost one shared-memory round trip.
__device__ __forceinline__ bool mbar_wait2(uint64_t * bar_a, uint32_t parity_a, int code_a, uint64_t * bar_b,
                                           uint32_t parity_b, int code_b, volatile int * abort_flag, int * error) {
    const bool a = mbar_try_wait(bar_a, parity_a);
    const bool b = mbar_try_wait(bar_b, parity_b);
    if (a && b) return true;
    return (a || mbar_wait_slow(bar_a, parity_a, abort_flag, error, code_a)) &&
           (b || mbar_wait_slow(bar_b, parity_b, abort_flag, error, code_b));
}

// ---- clusters: the K slices of a tile are added over distributed shared memory

__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Shared-memory address of `p` in the CTA of cluster rank `rank`.
__device__ __forceinline__ uint32_t dsmem_addr(const void * p, uint32_t rank) {
    uint32_t out;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(smem_u32(p)), "r"(rank));
    return out;
}

__device__ __forceinline__ double dsmem_f64(uint32_t addr) {
    double v;
    asm volatile("ld.shared::cluster.f64 %0, [%1];" : "=d"(v) : "r"(addr) : "memory");
    return v;
}

// Arrival on the barrier at the same offset in the CTA of rank `rank`,
// releasing (at cluster scope) this thread's earlier shared-memory accesses
// and, through the fence and the warp barrier before it, its warp's.
__device__ __forceinline__ void mbar_arrive_remote(uint64_t * bar, uint32_t rank) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(dsmem_addr(bar, rank)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t * bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.b32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait with cluster-scope acquire (the arrivals come from the CTAs of
// the cluster); same limit and error reporting as mbar_wait.
__device__ __noinline__ bool mbar_wait_cluster(uint64_t * bar, uint32_t parity, volatile int * abort_flag, int * error,
                                               int code) {
    const uint64_t t0 = global_ns();
    for (;;) {
        if (mbar_try_wait_cluster(bar, parity)) return true;
        if (*abort_flag) return false;
        if (global_ns() - t0 > kWaitNs) break;
        __nanosleep(64);
    }
    *abort_flag = 1;
    if (error != nullptr) *reinterpret_cast<volatile int *>(error) = code;
    return false;
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

// 3D tiled TMA load (no multicast); x is always 0 here.
__device__ __forceinline__ void tma_load_3d(void * dst, const CUtensorMap * map, int32_t x, int32_t y, int32_t z,
                                            uint64_t * bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
        "[%5];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
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

// K-major operand in the 128-byte swizzled layout that a SWIZZLE_128B TMA
// box writes (rows of 64 f16 = 128 bytes, 16-byte chunk c of row r stored at
// chunk c ^ (r % 8), 8-row groups 1024 bytes apart). The atom must be
// 1024-byte aligned; a K step of 16 values inside it advances the start
// address by 32 bytes. Layout type 2 (bits 61-63) is SWIZZLE_128B.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr) {
    uint64_t d = 0;
    d |= uint64_t((addr & 0x3FFFF) >> 4);
    d |= uint64_t(1) << 16;          // leading byte offset: unused for swizzled K-major
    d |= uint64_t(1024 >> 4) << 32;  // stride byte offset: 8 rows x 128 bytes
    d |= uint64_t(1) << 46;
    d |= uint64_t(2) << 61;
    return d;
}

// Instruction descriptor of kind::f16: D = f32, A = B = f16, both K-major.
__host__ __device__ constexpr uint32_t instr_desc(uint32_t m, uint32_t n) {
    return (1u << 4) | ((n >> 3) << 17) | ((m >> 4) << 24);
}

// The MMA wrappers are executed by a whole converged warp: elect.sync picks
// one lane to issue. Measured on the B200, a 128 x 32 x 16 MMA chain issued
// this way streams at 17 cycles per MMA, against 46 when a single thread
// (inside lane-divergent code) issues the same chain.
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p, e;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
}

// The same with the A operand read from TMEM (K-major: lane = row, each
// 32-bit column a pair of consecutive K values).
__device__ __forceinline__ void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p, e;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
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

// Warp-collective like the MMA wrappers: one elected lane commits.
__device__ __forceinline__ void mma_commit(uint64_t * bar) {
    asm volatile(
        "{\n\t.reg .pred e;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(smem_u32(bar))
        : "memory");
}

// 8 consecutive f32 columns of this thread's TMEM lane (completes at tmem_wait_ld).
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
}
// 4 consecutive f32 columns of this thread's TMEM lane (completes at tmem_wait_ld).
__device__ __forceinline__ void tmem_ld4(uint32_t taddr, uint32_t (&r)[4]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(taddr));
}
template <int N>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, uint32_t (&r)[N]) {
    if constexpr (N == 8) tmem_ld8(taddr, r);
    else tmem_ld4(taddr, r);
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

// f16 pair (V, V) of an exactly representable integer constant.
template <int V>
__device__ __forceinline__ __half2 h2_int_const() {
    constexpr float f = float(V);
    return __float2half2_rn(f);
}

// Tensor maps of one launch: weight boxes W0/W1 and the scale box (128 rows
// each), the f16 codes (3D: 64 codes x BN rows x 2 chunks, 128-byte swizzle),
// the f16 partial sums (3D: 8 x BN x 2 chunks) and the transposed activation
// scales (BN x 1).
struct TcMaps {
    CUtensorMap w0, w1, sc, qs, b2, dt;
};

struct TcParams {
    jfb_weight w;
    uint32_t n;
    uint32_t blocks;        // cols / 256
    uint32_t tiles_m;
    uint32_t tiles;
    uint64_t work;          // tiles * blocks
    uint32_t csize;         // 1: stream-K over the grid; > 1: CTAs per cluster, the K slices of one tile
    // output segments: rows [seg_end[k-1], seg_end[k]) -> seg_out[k] [n][rows of k]
    uint32_t nseg;
    uint32_t seg_end[JFB_MATMUL_MAX_SEGMENTS];
    uint32_t seg_epilogue[JFB_MATMUL_MAX_SEGMENTS];
    const float * seg_bias[JFB_MATMUL_MAX_SEGMENTS];
    const float * seg_residual[JFB_MATMUL_MAX_SEGMENTS];
    float * seg_out[JFB_MATMUL_MAX_SEGMENTS];
    double * partial;       // stream-K: [2 * gridDim.x][BN][kRows]
    uint32_t * counters;    // stream-K: [tiles][epilogue warps]
    int * error;
};

__host__ __device__ __forceinline__ uint64_t range_start(uint64_t c, uint64_t work, uint64_t g) {
    return c * work / g;
}
// The CTA whose stream-K range holds `unit`.
__device__ __forceinline__ uint32_t cta_of(uint64_t unit, uint64_t work, uint64_t g) {
    return uint32_t(((unit + 1) * g - 1) / work);
}

// This CTA's work: U units, one (tile, K block) pair each, starting at
// (tile0, bstart); within a tile the blocks run from b0 to b1 - 1.
//   Stream-K (csize == 1): CTA c of G takes the contiguous unit range
//   [c*W/G, (c+1)*W/G) of the W = tiles * nb units (b0 = 0, b1 = nb); a tile
//   split between CTAs is finished by the last one to arrive, from partial
//   sums in global memory.
//   Clusters (csize > 1): cluster k of G takes the tiles [k*T/G, (k+1)*T/G)
//   and its CTA of rank r the blocks [r*nb/csize, (r+1)*nb/csize) of each;
//   the K slices of a tile are added over distributed shared memory.
struct Work {
    uint32_t tile0, bstart, b0, b1, units, rank;
};

__device__ __forceinline__ Work cta_work(const TcParams & p) {
    Work w;
    const uint32_t nb = p.blocks;
    if (p.csize == 1) {
        const uint64_t wb = range_start(blockIdx.x, p.work, gridDim.x);
        const uint64_t we = range_start(blockIdx.x + 1, p.work, gridDim.x);
        w.tile0 = uint32_t(wb / nb);
        w.bstart = uint32_t(wb - uint64_t(w.tile0) * nb);
        w.b0 = 0;
        w.b1 = nb;
        w.units = uint32_t(we - wb);
        w.rank = 0;
    } else {
        const uint32_t clusters = gridDim.x / p.csize, c = blockIdx.x / p.csize;
        w.rank = blockIdx.x - c * p.csize;
        const uint32_t t0 = uint32_t(uint64_t(c) * p.tiles / clusters);
        const uint32_t t1 = uint32_t(uint64_t(c + 1) * p.tiles / clusters);
        w.tile0 = t0;
        w.b0 = w.rank * nb / p.csize;
        w.b1 = (w.rank + 1) * nb / p.csize;
        w.bstart = w.b0;
        w.units = (t1 - t0) * (w.b1 - w.b0);
    }
    return w;
}

// Position of a work unit: tile = tn * tiles_m + tm, K block b. Advanced one
// unit at a time so that no role divides per unit.
struct Cursor {
    uint32_t tile, b, tm, tn;
    __device__ __forceinline__ void init(const Work & w, uint32_t tiles_m) {
        tile = w.tile0;
        b = w.bstart;
        tn = tile / tiles_m;
        tm = tile - tn * tiles_m;
    }
    __device__ __forceinline__ void next(const Work & w, uint32_t tiles_m) {
        if (++b == w.b1) {
            b = w.b0;
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
template <uint32_t TYPE, class RL>
__device__ __forceinline__ void convert_a(const uint8_t * r, int h, int part, uint32_t a_col, int m) {
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
template <uint32_t TYPE, class RL>
__device__ __forceinline__ void convert_mins(const uint8_t * r, int part, uint8_t * tile, int m) {
    const uint4 meta = *reinterpret_cast<const uint4 *>(r + RL::kScOff + m * 16);
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

// Packed f32x2 arithmetic (sm_100): each lane is rounded exactly as the
// scalar __fmul_rn / __fadd_rn / __fmaf_rn would round it. A packed product
// that feeds an addition can still be fused with it by the compiler (measured:
// the __fmul2_rn / __fadd2_rn intrinsics are), so every rounding-sensitive
// difference of two products below is a scalar __fsub_rn, which never is.
__device__ __forceinline__ float2 f2(float a, float b) { return make_float2(a, b); }

__device__ __forceinline__ float2 mul2_rn(float2 a, float2 b) {
    float2 d;
    asm("{\n\t.reg .b64 a, b, d;\n\tmov.b64 a, {%2, %3};\n\tmov.b64 b, {%4, %5};\n\t"
        "mul.rn.f32x2 d, a, b;\n\tmov.b64 {%0, %1}, d;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}

__device__ __forceinline__ float2 fma2_rn(float2 a, float2 b, float2 c) {
    float2 d;
    asm("{\n\t.reg .b64 a, b, c, d;\n\tmov.b64 a, {%2, %3};\n\tmov.b64 b, {%4, %5};\n\t"
        "mov.b64 c, {%6, %7};\n\tfma.rn.f32x2 d, a, b, c;\n\tmov.b64 {%0, %1}, d;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
    return d;
}

template <uint32_t TYPE, int BN>
__global__ void __launch_bounds__(Roles<BN>::kThreads) __maxnreg__(Roles<BN>::kRegs) mmq_tc_kernel(const __grid_constant__ TcMaps maps, TcParams p) {
    using T = TypeTraits<TYPE>;
    using L = Layout<TYPE, BN>;
    using R = Roles<BN>;
    constexpr int NS = L::NS;
    constexpr int NR = L::NR;
    constexpr uint32_t kAccCols = L::kAccCols;
    constexpr uint32_t kACols = L::kACols;

    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t * raw = smem;                                   // [NR][kRawBytes], 1024-byte aligned
    uint8_t * ops = raw + NR * L::kRawBytes;                // [NS][kOpBytes]
    double * sums = reinterpret_cast<double *>(ops + NS * L::kOpBytes);  // [BN][kRows] (shared-memory sums)
    uint8_t * ering = reinterpret_cast<uint8_t *>(sums) + L::kSumBytes;  // [kEpiRing][kEpiSlotBytes]
    uint8_t * tail = ering + kEpiRing * kEpiSlotBytes;
    uint64_t * full = reinterpret_cast<uint64_t *>(tail);  // [NS] A stage written (its converter group)
    uint64_t * empty = full + NS;                          // [NS] A stage consumed (MMA commit)
    uint64_t * raw_full = empty + NS;                      // [NR] TMA landed
    uint64_t * raw_empty = raw_full + NR;                  // [NR] converter group + MMA done with it
    uint64_t * acc_full = raw_empty + NR;                  // [2]
    uint64_t * acc_empty = acc_full + 2;                   // [2]
    uint64_t * epi_tx = acc_empty + 2;                     // [kEpiRing] activation d landed (TMA)
    uint64_t * epi_empty = epi_tx + kEpiRing;              // [kEpiRing]
    uint64_t * red_full = epi_empty + kEpiRing;            // [2] every CTA of the cluster wrote its tile sums
    uint64_t * red_empty = red_full + 2;                   // [2] every CTA of the cluster read them
    uint64_t * drain = red_empty + 2;                      // [kMmaWarps]
    uint32_t * tmem_slot = reinterpret_cast<uint32_t *>(drain + R::kMmaWarps);
    volatile int * abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    pdl_trigger();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t nb = p.blocks;
    const uint32_t csize = p.csize;
    const Work wk = cta_work(p);
    const uint32_t U = wk.units;

    if (threadIdx.x == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(&full[s], R::kGroupWarps);
            mbar_init(&empty[s], 1);
        }
        for (int s = 0; s < NR; ++s) {
            mbar_init(&raw_full[s], 1);
            mbar_init(&raw_empty[s], R::kGroupWarps + 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&acc_full[a], 1);
            mbar_init(&acc_empty[a], R::kEpiWarps);
        }
        for (int e = 0; e < kEpiRing; ++e) {
            mbar_init(&epi_tx[e], 1);
            mbar_init(&epi_empty[e], R::kEpiWarps);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&red_full[b], csize * R::kEpiWarps);
            mbar_init(&red_empty[b], csize * R::kEpiWarps);
        }
        for (int d = 0; d < R::kMmaWarps; ++d) mbar_init(&drain[d], 1);
        // the swizzled boxes need a 1024-byte aligned ring; stop before any load otherwise
        const bool aligned = (smem_u32(smem) & 1023u) == 0;
        *abort_flag = aligned ? 0 : 1;
        if (!aligned && p.error != nullptr) *reinterpret_cast<volatile int *>(p.error) = kErrSmemAlign;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == R::kMmaWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    // with clusters, every CTA's barriers are initialised before any remote arrival
    if (csize > 1) cluster_sync_all();
    else __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp >= R::kTmaWarp) {
        // ---------------- TMA loads (one thread per half-block) ----------------
        // Thread t issues the loads of half-block t of every unit (raw stages
        // rs with rs % 2 == t, NR is even); thread 0 also stages each unit's
        // activation scales in the epilogue ring.
        const int t = warp - R::kTmaWarp;
        if (lane == 0) {
            uint32_t es = 0, eph = 0;
            uint64_t e_issued = 0;
            bool ok = true;
            auto issue_weights = [&](uint8_t * r, const Cursor & c, int h, uint64_t * bar) {
                const int32_t y_w = int32_t(c.tm * kRows);
                const int32_t x_blk = int32_t(c.b * T::kBlockBytes);
                tma_load_2d(r + L::kW0Off, &maps.w0, x_blk + int32_t(T::kW0 * h), y_w, bar);
                if constexpr (T::kW1 > 0) tma_load_2d(r + L::kW1Off, &maps.w1, x_blk + 128 + int32_t(T::kW1 * h), y_w, bar);
                tma_load_2d(r + L::kScOff, &maps.sc, int32_t(c.b * 16), y_w, bar);
            };
            // one 3D box each: the two 64-code chunks of the half-block and
            // (half 0, types with mins) the two 8-wide partial-sum chunks; the
            // x coordinate is 0 and the chunk index is the third coordinate
            auto issue_activations = [&](uint8_t * r, const Cursor & c, int h, uint64_t * bar) {
                const int32_t y_a = int32_t(c.tn * BN);
                tma_load_3d(r + L::kBOff, &maps.qs, 0, y_a, int32_t(4 * c.b + 2 * h), bar);
                if (T::kMins && h == 0) tma_load_3d(r + L::kB2Off, &maps.b2, 0, y_a, int32_t(2 * c.b), bar);
            };
            // The weights of the first raw stages depend on no earlier kernel:
            // they are requested before waiting for the previous kernel, so
            // their latency overlaps its tail (programmatic dependent launch).
            const uint32_t pre = std::min<uint32_t>(uint32_t(NR), 2 * U);
            {
                Cursor c0;
                c0.init(wk, p.tiles_m);
                for (uint32_t k = uint32_t(t); k < pre; k += 2) {
                    mbar_arrive_expect_tx(&raw_full[k], t == 0 ? L::kTx0 : L::kTx1);  // fresh stages: nothing to wait for
                    issue_weights(raw + k * L::kRawBytes, c0, t, &raw_full[k]);
                    c0.next(wk, p.tiles_m);
                }
            }
            pdl_wait();
            Cursor cur;
            cur.init(wk, p.tiles_m);
            uint32_t hb = uint32_t(t);  // this thread's next half-block
            for (uint32_t u = 0; u < U && ok && !*abort_flag; ++u, hb += 2, cur.next(wk, p.tiles_m)) {
                if (t == 0) {
                    // the unit's activation scales d[tokens][b] (one row of d_t)
                    if (!mbar_wait(&epi_empty[es], eph ^ 1u, abort_flag, p.error, kErrWaitEpiEmpty)) break;
                    mbar_arrive_expect_tx(&epi_tx[es], uint32_t(BN) * 4);
                    tma_load_2d(ering + es * kEpiSlotBytes, &maps.dt, int32_t(cur.tn * BN), int32_t(cur.b), &epi_tx[es]);
                    ++e_issued;
                    if (++es == kEpiRing) {
                        es = 0;
                        eph ^= 1u;
                    }
                }
                const uint32_t rs = uint32_t(hb % NR), rph = uint32_t((hb / NR) & 1u);
                uint8_t * r = raw + rs * L::kRawBytes;
                if (hb >= pre) {
                    if (!mbar_wait(&raw_empty[rs], rph ^ 1u, abort_flag, p.error, kErrWaitRawEmpty)) break;
                    mbar_arrive_expect_tx(&raw_full[rs], t == 0 ? L::kTx0 : L::kTx1);
                    issue_weights(r, cur, t, &raw_full[rs]);
                }
                issue_activations(r, cur, t, &raw_full[rs]);
            }
            // a stopped kernel must not exit with loads still landing in its
            // shared memory: wait (bounded) for the last issue of every slot
            if (*abort_flag) {
                // pre-issued stages whose activation boxes were not requested yet
                // get them now, so that every transaction completes
                for (uint32_t j = hb; j < pre; j += 2) {
                    Cursor cj;
                    cj.init(wk, p.tiles_m);
                    for (uint32_t k = 0; k < j / 2; ++k) cj.next(wk, p.tiles_m);
                    issue_activations(raw + j * L::kRawBytes, cj, t, &raw_full[j]);
                }
                volatile int no_abort = 0;
                uint32_t last = hb;  // every half-block of this thread below `last` was issued
                while (last < pre) last += 2;
                for (uint32_t j = last >= uint32_t(NR) ? last - NR : uint32_t(t); j < last; j += 2) {
                    (void) mbar_wait(&raw_full[j % NR], uint32_t((j / NR) & 1u), &no_abort, nullptr, 0);
                }
                for (uint64_t j = e_issued > uint64_t(kEpiRing) ? e_issued - kEpiRing : 0; j < e_issued; ++j) {
                    (void) mbar_wait(&epi_tx[j % kEpiRing], uint32_t((j / kEpiRing) & 1u), &no_abort, nullptr, 0);
                }
            }
        }
        __syncwarp();
    } else if (warp >= R::kEpiWarps && warp < R::kMmaWarp) {
        // ---------------- converters ----------------
        // Group `grp` converts the half-blocks h with h % kGroups == grp (with
        // two groups: half 0 and half 1 of every unit, concurrently). A group
        // owns the A stages and raw stages of its halves (NS and NR are even
        // when there are two groups), so each of its barriers completes its
        // phases in the order the group waits for them.
        const int cw = warp - R::kEpiWarps;
        const int grp = cw / R::kGroupWarps;
        const int quarter = warp & 3;                                 // TMEM lane quarter of this warp
        const int part = (cw % R::kGroupWarps) >> 2;                  // uniform per warp
        const int m = quarter * 32 + lane;
        const uint32_t lane_base = uint32_t(quarter * 32) << 16;
        uint32_t hb = uint32_t(grp);  // half-block index of the CTA's range
        for (uint32_t u = 0; u < U; ++u) {
            if (__any_sync(0xffffffffu, *abort_flag != 0)) break;
            bool ok = true;
            for (int h = grp; h < 2; h += R::kGroups, hb += R::kGroups) {
                const uint32_t stage = uint32_t(hb % NS), phase = uint32_t((hb / NS) & 1u);
                const uint32_t rs = uint32_t(hb % NR), rph = uint32_t((hb / NR) & 1u);
                // the whole warp proceeds or stops together (TMEM stores are warp-collective)
                const bool ready = mbar_wait2(&raw_full[rs], rph, kErrWaitRawFull, &empty[stage], phase ^ 1u,
                                              kErrWaitEmpty, abort_flag, p.error);
                if (!__all_sync(0xffffffffu, ready)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint8_t * r = raw + rs * L::kRawBytes;
                const uint32_t a_col = tmem + lane_base + kAccCols + stage * kACols;
                uint8_t * op = ops + stage * L::kOpBytes;
                if constexpr (R::kParts == 2) {
                    convert_a<TYPE, L>(r, h, part, a_col, m);
                    if (T::kMins && h == 0) convert_mins<TYPE, L>(r, part, op, m);
                } else {
#pragma unroll 1
                    for (int pt = 0; pt < 2; ++pt) {
                        convert_a<TYPE, L>(r, h, pt, a_col, m);
                        if (T::kMins && h == 0) convert_mins<TYPE, L>(r, pt, op, m);
                    }
                }
                tmem_wait_st();
                tc_fence_before();
                if (T::kMins && h == 0) fence_proxy_async();  // the mins tile is read by the tensor cores
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&full[stage]);
                    mbar_arrive(&raw_empty[rs]);
                }
            }
            if (!ok) break;
        }
    } else if (warp >= R::kMmaWarp && warp < R::kTmaWarp) {
        // ---------------- MMA issue (one thread per MMA warp) ----------------
        // With A stages in a multiple of 4, MMA warp `mid` issues the units i
        // with i % 2 == mid: those are the units of accumulator buffer `mid`
        // and of A stages {2 mid, 2 mid + 1} (mod 4), so every barrier a thread
        // waits on is used by that thread alone and its phases come in order.
        // With fewer stages one thread issues every unit.
        constexpr uint32_t kIssuers = NS % 4 == 0 ? 2u : 1u;
        const uint32_t mid = uint32_t(warp - R::kMmaWarp);
        if (mid < kIssuers) {
            // the whole warp runs this loop (the MMA and commit wrappers elect
            // one lane), so every wait below ends warp-uniformly
            constexpr uint32_t idesc = instr_desc(kRows, BN);
            bool ok = true;
            uint32_t i = mid;
            for (; i < U && ok; i += kIssuers) {
                if (__any_sync(0xffffffffu, *abort_flag != 0)) break;
                const uint32_t acc = i & 1u, use = i >> 1;
                if (!__all_sync(0xffffffffu, mbar_wait(&acc_empty[acc], (use & 1u) ^ 1u, abort_flag, p.error,
                                                       kErrWaitAccEmpty))) {
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem + acc * (T::kAcc * BN);
                for (int h = 0; h < 2; ++h) {
                    const uint32_t hb = 2 * i + uint32_t(h);  // half-block index of the CTA's range
                    const uint32_t stage = uint32_t(hb % NS), phase = uint32_t((hb / NS) & 1u);
                    const uint32_t rs = uint32_t(hb % NR), rph = uint32_t((hb / NR) & 1u);
                    // (the converters waited for the raw stage before completing full[stage];
                    // with two issuers the raw barriers are shared, so only one waits on them)
                    const bool ready = kIssuers == 2
                                           ? mbar_wait(&full[stage], phase, abort_flag, p.error, kErrWaitFull)
                                           : mbar_wait2(&full[stage], phase, kErrWaitFull, &raw_full[rs], rph,
                                                        kErrWaitRawFull, abort_flag, p.error);
                    if (!__all_sync(0xffffffffu, ready)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t braw = smem_u32(raw + rs * L::kRawBytes);
                    const uint32_t a = tmem + kAccCols + stage * kACols;
#pragma unroll
                    for (int ks = 0; ks < kKStage / 16; ++ks) {
                        const uint64_t bdesc =
                            smem_desc_sw128(braw + L::kBOff + uint32_t(ks >> 2) * L::kBHalf + uint32_t(ks & 3) * 32);
                        if constexpr (TYPE == JF_TENSOR_Q4_K) {
                            mma_f16_ts(d + h * BN, a + ks * 8, bdesc, idesc, ks > 0 ? 1u : 0u);
                        } else if constexpr (TYPE == JF_TENSOR_Q6_K) {
                            const uint32_t accum = (h > 0 || ks > 0) ? 1u : 0u;
                            mma_f16_ts(d, a + ks * 8, bdesc, idesc, accum);
                            mma_f16_ts(d + BN, a + 64 + ks * 8, bdesc, idesc, accum);
                        } else {
                            mma_f16_ts(d, a + ks * 8, bdesc, idesc, (h > 0 || ks > 0) ? 1u : 0u);
                        }
                    }
                    if (T::kMins && h == 0) {
                        // A2 [128 x 16]: core matrices 128 B apart along K, 8-row groups kSbo16 apart;
                        // B2 [BN x 16]: the two 8-wide boxes BN*16 B apart, 8-row groups 128 B apart
                        mma_f16(d + (T::kAcc - 1) * BN, smem_desc(smem_u32(ops + stage * L::kOpBytes), 128, kSbo16),
                                smem_desc(braw + L::kB2Off, uint32_t(BN) * 16, 128), idesc, 0u);
                    }
                    mma_commit(&empty[stage]);   // the A stage is free once these MMAs are done
                    mma_commit(&raw_empty[rs]);  // and so is the raw stage that holds B
                }
                if (ok) mma_commit(&acc_full[acc]);
            }
            // every issued MMA completes before TMEM is released
            mma_commit(&drain[mid]);
            volatile int no_abort = 0;
            (void) mbar_wait(&drain[mid], 0, &no_abort, nullptr, 0);
        }
        __syncwarp();
    } else {
        // ---------------- epilogue ----------------
        // Each thread owns weight row m of the tile (its warp's TMEM lane
        // quarter) and kCols token columns. It reads its row's scale word of
        // each block from the weight planes itself, one unit ahead; the TMA
        // thread stages each unit's activation scales in the epilogue ring.
        // The per-(row, token) double sums of a segment (the CTA's blocks of
        // one tile) live in shared memory ([BN][kRows], two buffers
        // alternating by segment) for 32-token tiles and in registers for
        // 64-token tiles. Stream-K finishes a split tile in the last CTA to
        // arrive, from partials in global memory; with clusters (32-token
        // tiles), the K slices of a tile are added over distributed shared
        // memory: CTA r adds slices 0..csize-1, in that order, for its
        // 1/csize of the tile's outputs. Either way the result does not depend
        // on timing.
        constexpr int kCols = R::kCols;  // token columns of this thread
        constexpr uint32_t kTileOut = uint32_t(kRows) * BN;
        const int quarter = warp & 3;
        const int m = quarter * 32 + lane;  // the warp's TMEM lane quarter = its 32 weight rows
        const int col0 = (warp >> 2) * kCols;
        const uint32_t et = uint32_t(warp) * 32 + uint32_t(lane);  // 0..255
        const uint32_t lane_base = uint32_t(quarter * 32) << 16;
        double rsum[R::kSmemSums ? 1 : kCols] = {};
        uint32_t bi = 0;  // sums / staging buffer of the current tile
        auto sbuf = [&](uint32_t k) { return sums + k * kTileOut; };
        auto sum_get = [&](int t) -> double {
            if constexpr (R::kSmemSums) return sbuf(bi)[uint32_t(col0 + t) * kRows + uint32_t(m)];
            else return rsum[t];
        };
        auto sum_set = [&](int t, double v) {
            if constexpr (R::kSmemSums) sbuf(bi)[uint32_t(col0 + t) * kRows + uint32_t(m)] = v;
            else rsum[t] = v;
        };
        const uint8_t * p1 = static_cast<const uint8_t *>(p.w.plane[1]);
        const uint8_t * p2 = static_cast<const uint8_t *>(p.w.plane[2]);
        // this row's scale word of the unit's block: Q4_K (d | dmin << 16) from
        // the 16-byte header, Q6_K d, Q2_K (d | dmin << 16); 0 past the last row
        auto load_word = [&](const Cursor & c) -> uint32_t {
            const uint32_t row = c.tm * kRows + uint32_t(m);
            if (row >= p.w.rows) return 0u;
            const uint64_t block = uint64_t(row) * nb + c.b;
            if constexpr (TYPE == JF_TENSOR_Q4_K) return __ldg(reinterpret_cast<const uint32_t *>(p1 + block * 16));
            else if constexpr (TYPE == JF_TENSOR_Q6_K) return uint32_t(__ldg(reinterpret_cast<const uint16_t *>(p2) + block));
            else return __ldg(reinterpret_cast<const uint32_t *>(p2) + block);
        };
        // one output row: its segment's output, epilogue and row stride, looked
        // up once per row; store(tok, sum) then writes token tok of the row
        struct OutRow {
            float * out;
            const float * bias;
            const float * residual;
            uint32_t ld, r, ep;
            bool valid;
        };
        auto out_row = [&](uint32_t row) {
            OutRow o;
            o.valid = row < p.w.rows;
            int k = 0;
#pragma unroll
            for (int j = 0; j < JFB_MATMUL_MAX_SEGMENTS - 1; ++j) k += (j < int(p.nseg) - 1 && row >= p.seg_end[j]) ? 1 : 0;
            const uint32_t seg_begin_row = k == 0 ? 0u : p.seg_end[k - 1];
            o.ld = p.seg_end[k] - seg_begin_row;
            o.r = row - seg_begin_row;
            o.ep = p.seg_epilogue[k];
            o.out = p.seg_out[k];
            o.bias = p.seg_bias[k];
            o.residual = p.seg_residual[k];
            return o;
        };
        auto store = [&](const OutRow & o, uint32_t tok, double sum) {
            if (!o.valid || tok >= p.n) return;
            const uint64_t at = uint64_t(tok) * o.ld + o.r;
            float v = __double2float_rn(sum);
            if (o.ep == JFB_EPILOGUE_BIAS) v = __fadd_rn(v, o.bias[o.r]);
            else if (o.ep == JFB_EPILOGUE_RESIDUAL) v = __fadd_rn(v, o.residual[at]);
            o.out[at] = v;
        };
        uint32_t i = 0, es = 0, eph = 0, tix = 0;  // unit, ring slot, segment (tile slice) of this CTA
        uint32_t seg_b = 0;                         // first block of the current segment
        const uint32_t first_tile = wk.tile0;
        bool ok = true;
        Cursor cur;
        cur.init(wk, p.tiles_m);
        uint32_t word_next = U > 0 ? load_word(cur) : 0u;  // weights: written by no earlier kernel
        pdl_wait();  // outputs and residuals are shared with earlier kernels
        for (; i < U && ok; ++i, cur.next(wk, p.tiles_m)) {
            // warp-uniform stop: the warp collectives below need every lane
            if (__any_sync(0xffffffffu, *abort_flag != 0)) break;
            if (i == 0 || cur.b == wk.b0) {
                // a new segment: its sums buffer must be free (with clusters:
                // read by every CTA of the cluster two tiles ago)
                seg_b = cur.b;
                if constexpr (R::kSmemSums) {
                    bi = tix % R::kSumBufs;
                    if (R::kClusters && csize > 1 && tix >= R::kSumBufs) {
                        const uint32_t use = tix / R::kSumBufs - 1;
                        if (!__all_sync(0xffffffffu, mbar_wait_cluster(&red_empty[bi], use & 1u, abort_flag, p.error,
                                                                        kErrWaitReduce))) {
                            break;
                        }
                    }
                }
#pragma unroll
                for (int t = 0; t < kCols; ++t) sum_set(t, 0.0);
            }
            const uint32_t word = word_next;
            if (i + 1 < U) {
                Cursor nx = cur;
                nx.next(wk, p.tiles_m);
                word_next = load_word(nx);
            }
            const uint32_t acc = i & 1u, use = i >> 1;
            // the whole warp proceeds or stops together
            const bool ready = mbar_wait2(&epi_tx[es], eph, kErrWaitEpiFull, &acc_full[acc], use & 1u, kErrWaitAccFull,
                                          abort_flag, p.error);
            if (!__all_sync(0xffffffffu, ready)) break;
            tc_fence_after();
            const float * da_s = reinterpret_cast<const float *>(ering + es * kEpiSlotBytes) + col0;
            const float dw = half_bits_to_float(uint16_t(word & 0xffffu));
            const float dmin = half_bits_to_float(uint16_t(word >> 16));  // unused for Q6_K
            const float2 dw2 = f2(dw, dw), dmin2 = f2(dmin, dmin);
            const uint32_t base = tmem + lane_base + acc * (T::kAcc * BN) + col0;
#pragma unroll
            // The unit's accumulator columns come in chunks of kCw, double
            // buffered: chunk ch + 1 is requested before chunk ch is worked on,
            // so its TMEM load latency overlaps that arithmetic (wait::ld
            // waits for every earlier load of the thread, so the request is
            // issued after the wait that completes chunk ch).
            constexpr int kCw = R::kSmemSums ? 8 : 4;
            constexpr int kChunks = kCols / kCw;
            uint32_t rb[2][3][kCw];
            auto request = [&](int ch, uint32_t (&r)[3][kCw]) {
                tmem_ld_cols<kCw>(base + kCw * ch, r[0]);
                tmem_ld_cols<kCw>(base + BN + kCw * ch, r[1]);
                if constexpr (T::kAcc == 3) tmem_ld_cols<kCw>(base + 2 * BN + kCw * ch, r[2]);
            };
            request(0, rb[0]);
#pragma unroll
            for (int ch = 0; ch < kChunks; ++ch) {
                uint32_t (&r0)[kCw] = rb[ch & 1][0];
                uint32_t (&r1)[kCw] = rb[ch & 1][1];
                uint32_t (&r2)[kCw] = rb[ch & 1][2];
                float2 das[kCw / 2];
#pragma unroll
                for (int q = 0; q < kCw / 4; ++q) {
                    const float4 d4 = *reinterpret_cast<const float4 *>(da_s + kCw * ch + 4 * q);
                    das[2 * q] = f2(d4.x, d4.y);
                    das[2 * q + 1] = f2(d4.z, d4.w);
                }
                tmem_wait_ld();
                if (ch + 1 < kChunks) request(ch + 1, rb[(ch + 1) & 1]);
                if (ch == kChunks - 1) {
                    // the accumulators and the ring slot may be reused now
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) {
                        mbar_arrive(&acc_empty[acc]);
                        mbar_arrive(&epi_empty[es]);
                    }
                }
#pragma unroll
                for (int k = 0; k < kCw / 2; ++k) {
                    const float2 da2 = das[k];
                    const float2 a0 = f2(__uint_as_float(r0[2 * k]), __uint_as_float(r0[2 * k + 1]));
                    const float2 a1 = f2(__uint_as_float(r1[2 * k]), __uint_as_float(r1[2 * k + 1]));
                    float2 c;
                    if constexpr (TYPE == JF_TENSOR_Q4_K) {
                        // c = (dw*da)*RN(D0 + D1) - (dmin*da)*msum
                        const float2 a2 = f2(__uint_as_float(r2[2 * k]), __uint_as_float(r2[2 * k + 1]));
                        const float2 isum = f2(__fadd_rn(a0.x, a1.x), __fadd_rn(a0.y, a1.y));
                        const float2 t1 = mul2_rn(mul2_rn(dw2, da2), isum);
                        const float2 t2 = mul2_rn(mul2_rn(dmin2, da2), a2);
                        c = f2(__fsub_rn(t1.x, t2.x), __fsub_rn(t1.y, t2.y));
                    } else if constexpr (TYPE == JF_TENSOR_Q6_K) {
                        // 16*Dhi is exact, so the fused form rounds once, like RN(isum)
                        const float2 isum = fma2_rn(f2(16.0f, 16.0f), a0, a1);
                        c = mul2_rn(mul2_rn(dw2, da2), isum);
                    } else {
                        const float2 t1 = mul2_rn(mul2_rn(dw2, da2), a0);
                        const float2 t2 = mul2_rn(mul2_rn(dmin2, da2), a1);
                        c = f2(__fsub_rn(t1.x, t2.x), __fsub_rn(t1.y, t2.y));
                    }
                    const int t = kCw * ch + 2 * k;
                    sum_set(t, sum_get(t) + double(c.x));
                    sum_set(t + 1, sum_get(t + 1) + double(c.y));
                }
            }
            if (++es == kEpiRing) {
                es = 0;
                eph ^= 1u;
            }

            // a segment ends where this CTA's blocks of the tile or its range end
            if (i + 1 != U && cur.b + 1 != wk.b1) continue;
            const uint32_t tile_ix = tix++;
            const uint32_t tile = cur.tile;
            if (csize == 1) {
                if (seg_b != 0 || cur.b + 1 != nb) {
                    // stream-K: part of a tile. Every contributor adds its double
                    // partials into the tile's slot in the workspace (device-scope
                    // f64 reductions, which return nothing to wait for); the last
                    // warp to arrive (per tile and warp) reads the sums, clears the
                    // slot for the next call and stores the outputs. The slot is
                    // that of the tile's first contributor `lo`: 2 lo + 1 when lo's
                    // range starts before the tile (the tile is lo's last), 2 lo
                    // when it starts exactly at the tile; no CTA is the first
                    // contributor of two split tiles, so slots are never shared.
                    // The block terms' double sums are exact whatever the order of
                    // the additions, as for the CPU's sequential sum.
                    const uint64_t g = gridDim.x;
                    const uint32_t lo = cta_of(uint64_t(tile) * nb, p.work, g);
                    const uint32_t hi = cta_of(uint64_t(tile + 1) * nb - 1, p.work, g);
                    const uint64_t lo_slot =
                        2 * uint64_t(lo) + (range_start(lo, p.work, g) == uint64_t(tile) * nb ? 0 : 1);
                    double * slot = p.partial + lo_slot * (uint64_t(kRows) * BN) + col0 * kRows + m;
#pragma unroll
                    for (int t = 0; t < kCols; ++t) {
                        asm volatile("red.global.add.f64 [%0], %1;" ::"l"(slot + t * kRows), "d"(sum_get(t)) : "memory");
                    }
                    __threadfence();
                    __syncwarp();
                    uint32_t arrived = 0;
                    if (lane == 0) {
                        uint32_t * counter = p.counters + uint64_t(tile) * R::kEpiWarps + warp;
                        arrived = atomicAdd(counter, 1u) + 1;
                        if (arrived == hi - lo + 1) *counter = 0;  // every contributor is in
                    }
                    arrived = __shfl_sync(0xffffffffu, arrived, 0);
                    if (arrived != hi - lo + 1) continue;
                    __threadfence();
                    double v[kCols];
#pragma unroll
                    for (int t = 0; t < kCols; ++t) v[t] = __ldcg(slot + t * kRows);
#pragma unroll
                    for (int t = 0; t < kCols; ++t) {
                        __stcg(slot + t * kRows, 0.0);
                        sum_set(t, v[t]);
                    }
                }
#pragma unroll
                {
                    const OutRow orow = out_row(cur.tm * kRows + uint32_t(m));
#pragma unroll
                    for (int t = 0; t < kCols; ++t) store(orow, cur.tn * BN + uint32_t(col0 + t), sum_get(t));
                }
                continue;
            }
            if constexpr (R::kClusters) {
                // clusters (32-token tiles only): add the csize K slices of the tile
                const uint32_t ph = (tile_ix / R::kSumBufs) & 1u;
                asm volatile("fence.acq_rel.cluster;" ::: "memory");
                __syncwarp();
                if (lane < csize) mbar_arrive_remote(&red_full[bi], lane);  // release: this warp's sums are written
                if (!__all_sync(0xffffffffu, mbar_wait_cluster(&red_full[bi], ph, abort_flag, p.error, kErrWaitReduce))) {
                    ok = false;
                    break;
                }
                // this CTA's share of the tile's outputs, element o = token * kRows + row
                // (the pass stride 256 is a multiple of kRows: a thread keeps its row)
                const uint32_t share = kTileOut / csize;
                const double * buf = sbuf(bi);
                const OutRow orow = out_row(cur.tm * kRows + (wk.rank * share + et) % kRows);
                for (uint32_t o = wk.rank * share + et; o < (wk.rank + 1) * share; o += 32 * R::kEpiWarps) {
                    double v = 0.0;
                    for (uint32_t c = 0; c < csize; ++c) v += dsmem_f64(dsmem_addr(buf + o, c));
                    store(orow, cur.tn * BN + o / kRows, v);
                }
                asm volatile("fence.acq_rel.cluster;" ::: "memory");
                __syncwarp();
                if (lane < csize) mbar_arrive_remote(&red_empty[bi], lane);  // release: this warp's reads are done
            }
        }
    }
    tc_fence_before();
    // no CTA leaves while another CTA of its cluster may still read its shared
    // memory or arrive on its barriers
    if (csize > 1) cluster_sync_all();
    else __syncthreads();
    tc_fence_after();
    if (warp == R::kMmaWarp) {
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

// Activation rows per tile: 32 for decode-sized calls, 64 above (each weight
// conversion then feeds twice the tokens).
uint32_t tile_tokens(uint32_t n) { return n <= 32 ? 32u : 64u; }

struct Plan {
    uint32_t bn, tiles_m, tiles;
    uint64_t work;
};

Plan make_plan(uint32_t rows, uint32_t cols, uint32_t n) {
    Plan pl;
    pl.bn = tile_tokens(n);
    pl.tiles_m = (rows + kRows - 1) / kRows;
    pl.tiles = pl.tiles_m * ((n + pl.bn - 1) / pl.bn);
    pl.work = uint64_t(pl.tiles) * (cols / kQK);
    return pl;
}

// Workspace (stream-K launches): partial slots for the largest grid and tile
// this device runs (two per SM), then the arrival counters. Both offsets are
// the same for every shape, so calls of different shapes can share one
// workspace on a stream.
constexpr uint32_t kMaxBN = 64;
uint64_t partial_bytes() { return uint64_t(2) * uint64_t(sm_count()) * uint64_t(kRows) * kMaxBN * sizeof(double); }
uint64_t workspace_bytes(const Plan & pl) {
    return partial_bytes() + uint64_t(pl.tiles) * Roles<64>::kEpiWarps * sizeof(uint32_t);
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

// 2D tensor map of [rows][width] elements of `elem_bytes` bytes with a row
// stride of `stride` elements. A tensor map is a pure function of its
// parameters, so encoded maps are cached by the full parameter tuple
// (bounded; cleared when it grows large).
bool tensor_map_2d(CUtensorMap & out, const void * base, uint32_t elem_bytes, uint64_t width, uint64_t stride,
                   uint64_t rows, uint32_t box_w, uint32_t box_rows, bool swizzle128 = false) {
    using Key = std::tuple<uintptr_t, uint32_t, uint64_t, uint64_t, uint64_t, uint32_t, uint32_t, bool>;
    static std::mutex mu;
    static std::map<Key, CUtensorMap> cache;
    const Key key{reinterpret_cast<uintptr_t>(base), elem_bytes, width, stride, rows, box_w, box_rows, swizzle128};
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) {
        out = it->second;
        return true;
    }
    PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
    if (encode == nullptr) return false;
    const CUtensorMapDataType type = elem_bytes == 1   ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                     : elem_bytes == 2 ? CU_TENSOR_MAP_DATA_TYPE_UINT16
                                                       : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
    const cuuint64_t dims[2] = {width, rows};
    const cuuint64_t strides[1] = {stride * elem_bytes};
    const cuuint32_t box[2] = {box_w, box_rows};
    const cuuint32_t elem[2] = {1, 1};
    CUtensorMap map;
    std::memset(&map, 0, sizeof(map));
    if (encode(&map, type, 2, const_cast<void *>(base), dims, strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE,
               swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
        return false;
    }
    if (cache.size() >= 4096) cache.clear();
    cache.emplace(key, map);
    out = map;
    return true;
}

// 3D tensor map over f16 rows [rows][width] that views each row as chunks of
// `chunk` elements: dims (chunk, rows, width / chunk), strides (row pitch,
// chunk bytes). A box (chunk, box_rows, 2) lands in shared memory as two
// consecutive [box_rows][chunk] tiles, exactly as two 2D boxes would. Cached
// like tensor_map_2d.
bool tensor_map_chunks(CUtensorMap & out, const void * base, uint32_t chunk, uint64_t width, uint64_t rows,
                       uint32_t box_rows, bool swizzle128) {
    using Key = std::tuple<uintptr_t, uint32_t, uint64_t, uint64_t, uint32_t, bool>;
    static std::mutex mu;
    static std::map<Key, CUtensorMap> cache;
    const Key key{reinterpret_cast<uintptr_t>(base), chunk, width, rows, box_rows, swizzle128};
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) {
        out = it->second;
        return true;
    }
    PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
    if (encode == nullptr || width % chunk != 0) return false;
    const cuuint64_t dims[3] = {chunk, rows, width / chunk};
    const cuuint64_t strides[2] = {width * 2, uint64_t(chunk) * 2};
    const cuuint32_t box[3] = {chunk, box_rows, 2};
    const cuuint32_t elem[3] = {1, 1, 1};
    CUtensorMap map;
    std::memset(&map, 0, sizeof(map));
    if (encode(&map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, const_cast<void *>(base), dims, strides, box, elem,
               CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
               CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
        return false;
    }
    if (cache.size() >= 4096) cache.clear();
    cache.emplace(key, map);
    out = map;
    return true;
}

template <uint32_t TYPE, int BN>
jfb_status build_maps(TcMaps & maps, const TcParams & p, const jfb_q8k & x, uint32_t cols) {
    using T = TypeTraits<TYPE>;
    const uint64_t nb = p.blocks, wb = nb * T::kBlockBytes;
    const bool ok = tensor_map_2d(maps.w0, p.w.plane[0], 1, wb, wb, p.w.rows, T::kW0, kRows) &&
                    tensor_map_2d(maps.w1, p.w.plane[0], 1, wb, wb, p.w.rows, T::kW1 > 0 ? T::kW1 : 16, kRows) &&
                    tensor_map_2d(maps.sc, p.w.plane[1], 1, nb * 16, nb * 16, p.w.rows, 16, kRows) &&
                    tensor_map_chunks(maps.qs, x.qs_f16, 64, cols, p.n, BN, true) &&
                    tensor_map_chunks(maps.b2, x.bsums_f16, 8, cols / 16, p.n, BN, false) &&
                    tensor_map_2d(maps.dt, x.d_t, 4, p.n, x.d_stride, nb, BN, 1);
    if (!ok) return status_error(JFB_STATUS_CUDA_ERROR, "jfb_matmul_tc: could not encode a TMA tensor map");
    return status_ok();
}

// Clusters of `csize` CTAs of this kernel that fit on the device at once.
template <uint32_t TYPE, int BN>
int max_clusters(uint32_t csize) {
    using L = Layout<TYPE, BN>;
    using R = Roles<BN>;
    if (csize == 1) return sm_count();  // one CTA per SM (shared memory)
    static std::mutex mu;
    static std::map<std::pair<int, uint32_t>, int> cache;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) dev = 0;
    std::lock_guard<std::mutex> lock(mu);
    const auto key = std::make_pair(dev, csize);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(csize);
    cfg.blockDim = dim3(R::kThreads);
    cfg.dynamicSmemBytes = L::kSmem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = csize;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, mmq_tc_kernel<TYPE, BN>, &cfg) != cudaSuccess) {
        (void) cudaGetLastError();
        n = 0;
    }
    cache.emplace(key, n);
    return n;
}

// Schedule. With at least half as many tiles as SMs, stream-K over the whole
// grid (csize = 1): its unit ranges balance any shape and few tiles are
// split. With fewer tiles, every tile would be split across several CTAs and
// finished through global memory, so tiles go to clusters instead: each of G
// = min(clusters, T) clusters takes ceil(T / G) tiles of ceil(nb / csize)
// units per CTA, and a tile's slices are added on chip (about one unit more).
// The smallest cluster size of least cost wins.
template <uint32_t TYPE, int BN>
void choose_schedule(uint32_t tiles, uint32_t nb, uint64_t work, uint32_t & csize, uint32_t & grid) {
    const uint32_t sms = uint32_t(max_clusters<TYPE, BN>(1));
    csize = 1;
    grid = uint32_t(std::min<uint64_t>(work, uint64_t(sms)));
    if (!Roles<BN>::kClusters || 2 * uint64_t(tiles) >= sms) return;
    uint64_t best = ~uint64_t(0);
    for (uint32_t c = 2; c <= 8 && c <= nb; c *= 2) {
        const int mc = max_clusters<TYPE, BN>(c);
        if (mc <= 0) continue;
        const uint32_t g = std::min<uint32_t>(tiles, uint32_t(mc));
        const uint64_t cost = uint64_t((tiles + g - 1) / g) * ((nb + c - 1) / c + 1);
        if (cost < best) {
            best = cost;
            csize = c;
            grid = g * c;
        }
    }
}

template <uint32_t TYPE, int BN>
jfb_status launch(TcParams & p, const jfb_q8k & x, uint32_t cols, cudaStream_t s) {
    using L = Layout<TYPE, BN>;
    using R = Roles<BN>;
    constexpr uint32_t bytes = L::kSmem;
    static_assert(bytes <= kMaxSmem, "shared memory budget");
    static_assert(L::NR >= 4, "raw pipeline depth: two units");
    static_assert(L::NS >= 2, "operand pipeline depth");
    static_assert(L::kAccCols + L::NS * L::kACols <= kTmemCols, "TMEM budget");
    static_assert(L::kRawBytes % 1024 == 0 && L::kBHalf % 1024 == 0, "swizzled boxes stay 1024-byte aligned");
    static_assert(L::kOpBytes % 1024 == 0 && kEpiSlotBytes % 128 == 0 && L::kSumBytes % 1024 == 0,
                  "TMA destinations stay 128-byte aligned");
    static_assert(BN * 4 <= kEpiSlotBytes, "epilogue slot layout");
    static_assert(R::kGroupWarps % 4 == 0 && R::kParts * kRows == R::kGroupWarps * 32 && R::kParts <= 2,
                  "converter lanes cover the rows");
    static_assert(L::NS % R::kGroups == 0 && L::NR % R::kGroups == 0, "each converter group owns its stages");
    static_assert(R::kEpiWarps * 32 * R::kCols == kRows * BN && R::kCols % 8 == 0, "epilogue threads cover the tile");
    static_assert((kRows * BN) % (8 * R::kEpiWarps * 32) == 0, "every cluster share is a whole number of passes");
    TcMaps maps;
    jfb_status st = build_maps<TYPE, BN>(maps, p, x, cols);
    if (st.code != JFB_STATUS_OK) return st;
    auto kernel = mmq_tc_kernel<TYPE, BN>;
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
    uint32_t csize = 1, grid = 1;
    choose_schedule<TYPE, BN>(p.tiles, p.blocks, p.work, csize, grid);
    p.csize = csize;
    // programmatic dependent launch: the prologue (barriers, TMEM, the first
    // weight loads) overlaps the previous kernel; every write follows the
    // kernel's griddepcontrol.wait
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(R::kThreads);
    cfg.dynamicSmemBytes = bytes;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    unsigned na = 0;
    if (csize > 1) {
        attr[na].id = cudaLaunchAttributeClusterDimension;
        attr[na].val.clusterDim.x = csize;
        attr[na].val.clusterDim.y = 1;
        attr[na].val.clusterDim.z = 1;
        ++na;
    }
    if (pdl_enabled()) {
        attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[na].val.programmaticStreamSerializationAllowed = 1;
        ++na;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, maps, p);
    if (e != cudaSuccess) return status_error(JFB_STATUS_CUDA_ERROR, "jfb_matmul_tc: %s", cudaGetErrorString(e));
    return launch_status("jfb_matmul_tc");
}

template <uint32_t TYPE>
jfb_status launch_type(TcParams & p, const jfb_q8k & x, uint32_t cols, const Plan & pl, cudaStream_t s) {
    return pl.bn == 32 ? launch<TYPE, 32>(p, x, cols, s) : launch<TYPE, 64>(p, x, cols, s);
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
    if (x_q8->qs_f16 == nullptr || x_q8->bsums_f16 == nullptr || x_q8->d_t == nullptr) {
        return status_error(JFB_STATUS_INVALID_ARGUMENT,
                            "jfb_matmul_tc needs the Q8_K tensor-core planes (qs_f16, bsums_f16, d_t)");
    }
    jfb_status chk = check_q8_tensor_core(x_q8, n);
    if (chk.code != JFB_STATUS_OK) return chk;
    for (int i = 0; i < 2; ++i) {
        if ((reinterpret_cast<uintptr_t>(weight->plane[i]) & 15u) != 0) {
            return status_error(JFB_STATUS_INVALID_ARGUMENT, "weight planes must be 16-byte aligned");
        }
    }
    if (weight->type != JF_TENSOR_Q4_K && weight->plane[2] == nullptr) {
        return status_error(JFB_STATUS_INVALID_ARGUMENT, "Q6_K and Q2_K weights need their scale plane");
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
    p.n = n;
    p.blocks = weight->cols / kQK;
    p.tiles_m = pl.tiles_m;
    p.tiles = pl.tiles;
    p.work = pl.work;
    p.csize = 1;
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
    case JF_TENSOR_Q4_K: return launch_type<JF_TENSOR_Q4_K>(p, *x_q8, weight->cols, pl, s);
    case JF_TENSOR_Q6_K: return launch_type<JF_TENSOR_Q6_K>(p, *x_q8, weight->cols, pl, s);
    default: return launch_type<JF_TENSOR_Q2_K>(p, *x_q8, weight->cols, pl, s);
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
