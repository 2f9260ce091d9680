// Causal GQA attention over the F16 KV cache with GGML-CPU semantics,
// computed exactly enough to reproduce the CPU result bit for bit.
//
// The reference graph's unfused path, which GGML-CPU executes
// (qwen2_architecture.cpp:425-470, mask 697-708), is: scores = K . q with q
// converted to f16 and an f32 result; soft_max_ext: x = score * scale + mask,
// e = exp(x - max), p = e / sum; P converted to f16; out = V . P with an f32
// result. Here:
//   - every product of two f16 values is exact in f32 and the products are
//     summed in double, then rounded to f32 once, so the order of the
//     additions (and the split of a row over CTAs) does not change the result;
//   - the softmax normaliser is the double sum of exp(x - max) over all keys
//     of the row, and p is rounded to f16 exactly as GGML does before P V;
//   - exp is exp_cw (common.cuh), the same method the CPU oracle implements.
//
// Head dims 64 and 128 with at most 8 query heads per kv head take a single
// launch on the FP64 tensor cores (see the single-launch path below) for rows
// of up to 32768 keys (4096 with 8 rows per CTA). Otherwise four launches over
// a (row, kv head, 64-key chunk) grid:
//   1. scores x_j (and each chunk's maximum) -> scratch
//   2. per (row, head): max over chunks, sum_j exp(x_j - max) in double
//   3. P V partial sums per chunk in double -> scratch
//   4. per row: sum of the chunk partials, f32 output (+ Q8_K quantization)
// A CTA of launches 1 and 3 serves the G = heads/kv_heads query heads that
// share its kv head, so each K and V row is read once for G heads.
#include "common.cuh"

#include <algorithm>
#include <mutex>

namespace jfb {
namespace {

constexpr int kThreads = 128;
constexpr int kChunk = 64;      // keys per CTA
constexpr int kMaxGroup = 16;   // query heads per kv head
constexpr int kMaxHeadDim = 256;
constexpr uint32_t kMaxSplits = 65535;  // grid z of the four-launch form

struct Scratch {
    float * scores;      // [n][heads][keys_cap]
    float * chunk_max;   // [n][heads][splits]
    float2 * stats;      // [n][heads] (max, 1/sum)
    double * partial;    // [n][heads][splits][head_dim]
};

__host__ __device__ inline uint64_t align_up(uint64_t v) { return (v + 255) / 256 * 256; }

__host__ __device__ inline Scratch carve(void * base, uint32_t n, uint32_t heads, uint32_t head_dim, uint32_t splits) {
    uint8_t * p = static_cast<uint8_t *>(base);
    const uint64_t keys_cap = uint64_t(splits) * kChunk;
    Scratch s;
    s.scores = reinterpret_cast<float *>(p);
    p += align_up(uint64_t(n) * heads * keys_cap * sizeof(float));
    s.chunk_max = reinterpret_cast<float *>(p);
    p += align_up(uint64_t(n) * heads * splits * sizeof(float));
    s.stats = reinterpret_cast<float2 *>(p);
    p += align_up(uint64_t(n) * heads * sizeof(float2));
    s.partial = reinterpret_cast<double *>(p);
    return s;
}

uint64_t scratch_size(uint32_t n, uint32_t heads, uint32_t head_dim, uint32_t splits) {
    const uint64_t keys_cap = uint64_t(splits) * kChunk;
    return align_up(uint64_t(n) * heads * keys_cap * sizeof(float)) + align_up(uint64_t(n) * heads * splits * sizeof(float)) +
           align_up(uint64_t(n) * heads * sizeof(float2)) + uint64_t(n) * heads * splits * head_dim * sizeof(double);
}

// Keys of row r: positions 0..pos[r], clamped to the splits * kChunk keys the
// scratch was carved for, so a position beyond the call's max_keys (a broken
// caller contract) reads and writes nothing outside this call's scratch.
__device__ __forceinline__ uint32_t split_row_keys(int32_t p, uint32_t splits) {
    const uint64_t keys = uint64_t(uint32_t(p)) + 1u;
    const uint64_t cap = uint64_t(splits) * kChunk;
    return uint32_t(keys < cap ? keys : cap);
}

// Launch 1: x_j = f32(sum_d k_jd * f16(q_d)) * scale for the chunk's keys.
__global__ void __launch_bounds__(kThreads) scores_kernel(const float * __restrict__ q, const int32_t * __restrict__ seq,
                                                        const int32_t * __restrict__ pos, uint32_t heads, uint32_t kv_heads,
                                                        uint32_t head_dim, const jfb_kv_slot * __restrict__ slots,
                                                        uint32_t layer, float scale, uint32_t splits, Scratch sc) {
    __shared__ float q_s[kMaxGroup * kMaxHeadDim];
    __shared__ float x_s[kMaxGroup][kChunk];
    pdl_trigger();
    pdl_wait();
    const uint32_t r = blockIdx.x, kvh = blockIdx.y, split = blockIdx.z;
    const uint32_t keys = split_row_keys(pos[r], splits);
    const uint32_t j0 = split * kChunk;
    if (j0 >= keys) return;
    const uint32_t j1 = min(keys, j0 + kChunk);
    const uint32_t G = heads / kv_heads, D = head_dim, kvd = kv_heads * D;
    const jfb_kv_slot slot = slots[seq[r]];
    const uint16_t * kbase = slot.k + uint64_t(layer) * slot.capacity * kvd + kvh * D;
    for (uint32_t i = threadIdx.x; i < G * D; i += kThreads) {
        const uint32_t g = i / D, d = i % D;
        q_s[i] = __half2float(__float2half_rn(q[uint64_t(r) * heads * D + (kvh * G + g) * D + d]));
    }
    __syncthreads();
    const uint32_t kk = threadIdx.x >> 1, half = threadIdx.x & 1;
    const uint32_t j = j0 + kk;
    double acc[kMaxGroup];
#pragma unroll
    for (int g = 0; g < kMaxGroup; ++g) acc[g] = 0.0;
    if (j < j1) {
        const uint16_t * krow = kbase + uint64_t(j) * kvd;
        const uint32_t d_begin = half * (D / 2), d_end = half ? D : D / 2;
        if ((D % 16) == 0) {
            for (uint32_t d = d_begin; d < d_end; d += 8) {
                const uint4 raw = __ldg(reinterpret_cast<const uint4 *>(krow + d));
                const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float k0 = half_bits_to_float(uint16_t(w[e] & 0xffffu));
                    const float k1 = half_bits_to_float(uint16_t(w[e] >> 16));
#pragma unroll
                    for (int g = 0; g < kMaxGroup; ++g) {
                        if (uint32_t(g) < G) {
                            acc[g] += double(__fmul_rn(k0, q_s[g * D + d + 2 * e]));
                            acc[g] += double(__fmul_rn(k1, q_s[g * D + d + 2 * e + 1]));
                        }
                    }
                }
            }
        } else {
            for (uint32_t d = d_begin; d < d_end; ++d) {
                const float kv = half_bits_to_float(krow[d]);
#pragma unroll
                for (int g = 0; g < kMaxGroup; ++g) {
                    if (uint32_t(g) < G) acc[g] += double(__fmul_rn(kv, q_s[g * D + d]));
                }
            }
        }
    }
#pragma unroll
    for (int g = 0; g < kMaxGroup; ++g) {
        const double total = acc[g] + __shfl_xor_sync(0xffffffffu, acc[g], 1);
        if (uint32_t(g) < G && half == 0) {
            x_s[g][kk] = j < j1 ? __fmul_rn(__double2float_rn(total), scale) : -INFINITY;
        }
    }
    __syncthreads();
    const uint32_t keys_cap = splits * kChunk;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (uint32_t g = warp; g < G; g += kThreads / 32) {
        const uint32_t h = kvh * G + g;
        float * dst = sc.scores + (uint64_t(r) * heads + h) * keys_cap + j0;
        float mx = -INFINITY;
        for (uint32_t k = lane; k < uint32_t(kChunk); k += 32) {
            const float x = x_s[g][k];
            if (j0 + k < j1) dst[k] = x;
            mx = fmaxf(mx, x);
        }
        mx = warp_max(mx);
        if (lane == 0) sc.chunk_max[(uint64_t(r) * heads + h) * splits + split] = mx;
    }
}

__device__ __forceinline__ double block_sum(double v, double * shared) {
    v = warp_sum(v);
    if ((threadIdx.x & 31) == 0) shared[threadIdx.x >> 5] = v;
    __syncthreads();
    double t = 0.0;
    if (threadIdx.x < 32) {
        t = threadIdx.x < kThreads / 32 ? shared[threadIdx.x] : 0.0;
        t = warp_sum(t);
        if (threadIdx.x == 0) shared[0] = t;
    }
    __syncthreads();
    return shared[0];
}

// Launch 2: per (row, head) maximum and 1 / sum_j exp(x_j - max).
__global__ void __launch_bounds__(kThreads) stats_kernel(const int32_t * __restrict__ pos, uint32_t heads, uint32_t splits,
                                                       Scratch sc) {
    __shared__ double red[kThreads / 32];
    pdl_trigger();
    pdl_wait();
    const uint32_t r = blockIdx.x, h = blockIdx.y;
    const uint32_t keys = split_row_keys(pos[r], splits);
    const uint32_t used = (keys + kChunk - 1) / kChunk;
    const uint64_t rh = uint64_t(r) * heads + h;
    float mx = -INFINITY;
    for (uint32_t c = threadIdx.x; c < used; c += kThreads) mx = fmaxf(mx, sc.chunk_max[rh * splits + c]);
    mx = warp_max(mx);
    __shared__ float mx_s[kThreads / 32];
    if ((threadIdx.x & 31) == 0) mx_s[threadIdx.x >> 5] = mx;
    __syncthreads();
    mx = -INFINITY;
    for (int w = 0; w < kThreads / 32; ++w) mx = fmaxf(mx, mx_s[w]);
    const float * x = sc.scores + rh * (uint64_t(splits) * kChunk);
    double sum = 0.0;
    for (uint32_t j = threadIdx.x; j < keys; j += kThreads) sum += double(exp_cw(__fsub_rn(x[j], mx)));
    sum = block_sum(sum, red);
    if (threadIdx.x == 0) sc.stats[rh] = make_float2(mx, __double2float_rn(__ddiv_rn(1.0, sum)));  // sum >= 1
}

// Launch 3: P V over the chunk, p = f16(exp(x - max) * inv), sums in double.
__global__ void __launch_bounds__(kThreads) pv_kernel(const int32_t * __restrict__ seq, const int32_t * __restrict__ pos,
                                                    uint32_t heads, uint32_t kv_heads, uint32_t head_dim,
                                                    const jfb_kv_slot * __restrict__ slots, uint32_t layer,
                                                    uint32_t splits, Scratch sc) {
    __shared__ float p_s[kMaxGroup][kChunk];
    pdl_trigger();
    pdl_wait();
    const uint32_t r = blockIdx.x, kvh = blockIdx.y, split = blockIdx.z;
    const uint32_t keys = split_row_keys(pos[r], splits);
    const uint32_t j0 = split * kChunk;
    if (j0 >= keys) return;
    const uint32_t j1 = min(keys, j0 + kChunk);
    const uint32_t G = heads / kv_heads, D = head_dim, kvd = kv_heads * D;
    const uint32_t keys_cap = splits * kChunk;
    for (uint32_t i = threadIdx.x; i < G * kChunk; i += kThreads) {
        const uint32_t g = i / kChunk, k = i % kChunk;
        const uint64_t rh = uint64_t(r) * heads + kvh * G + g;
        float p = 0.0f;
        if (j0 + k < j1) {
            const float2 st = sc.stats[rh];
            const float e = exp_cw(__fsub_rn(sc.scores[rh * keys_cap + j0 + k], st.x));
            p = __half2float(__float2half_rn(__fmul_rn(e, st.y)));
        }
        p_s[g][k] = p;
    }
    __syncthreads();
    const jfb_kv_slot slot = slots[seq[r]];
    const uint16_t * vbase = slot.v + uint64_t(layer) * slot.capacity * kvd + kvh * D;
    for (uint32_t d = threadIdx.x; d < D; d += kThreads) {
        double acc[kMaxGroup];
#pragma unroll
        for (int g = 0; g < kMaxGroup; ++g) acc[g] = 0.0;
        for (uint32_t j = j0; j < j1; ++j) {
            const float vv = half_bits_to_float(vbase[uint64_t(j) * kvd + d]);
#pragma unroll
            for (int g = 0; g < kMaxGroup; ++g) {
                if (uint32_t(g) < G) acc[g] += double(__fmul_rn(p_s[g][j - j0], vv));
            }
        }
#pragma unroll
        for (int g = 0; g < kMaxGroup; ++g) {
            if (uint32_t(g) < G) {
                const uint64_t rh = uint64_t(r) * heads + kvh * G + g;
                sc.partial[(rh * splits + split) * D + d] = acc[g];
            }
        }
    }
}

// Launch 4: out[r][h*D + d] = f32(sum of the chunk partials); Q8_K of the row.
__global__ void __launch_bounds__(256) combine_kernel(const int32_t * __restrict__ pos, uint32_t heads, uint32_t head_dim,
                                                    uint32_t splits, Scratch sc, float * __restrict__ out, jfb_q8k q8,
                                                    int quantize) {
    __shared__ unsigned long long keys_s[8];
    pdl_trigger();
    pdl_wait();
    const uint32_t r = blockIdx.x;
    const uint32_t D = head_dim, width = heads * D;
    const uint32_t used = (split_row_keys(pos[r], splits) + kChunk - 1) / kChunk;
    for (uint32_t i = threadIdx.x; i < width; i += blockDim.x) {
        const uint32_t h = i / D, d = i % D;
        const double * base = sc.partial + ((uint64_t(r) * heads + h) * splits) * D + d;
        double acc = 0.0;
        for (uint32_t c = 0; c < used; ++c) acc += base[uint64_t(c) * D];
        out[uint64_t(r) * width + i] = __double2float_rn(acc);
    }
    if (!quantize) return;
    __syncthreads();
    for (uint32_t c = 0; c < width / kQK; ++c) {
        const float y = out[uint64_t(r) * width + c * kQK + threadIdx.x];
        q8k_block_256(y, q8_dest(q8, r, c, width / kQK), keys_s);
    }
}

// ---- single-launch path on the FP64 tensor cores -------------------------------
//
// Exactness needs every score and output as the double sum of exact f16*f16
// products, rounded to float once. The FP64 MMA (mma.sync m8n8k4 .f64)
// computes such sums eight query heads at a time: the 8 x 4 A fragment holds
// f16(q) of the G <= 8 query heads that share a kv head (the rows beyond G
// are zero), the 4 x 8 B fragment eight keys of the K cache, and the 8 x 8
// accumulator the scores of those heads and keys. Every product is exact in
// double and each MMA rounds its sums in double, so the float scores equal
// the CPU's (the order of the additions changes only bits far below a float
// ulp). P V is the same product with A = f16(p) and B = eight V columns.
//
// Operands. A K or V value (f16) becomes a double with integer operations:
// its 15 magnitude bits shifted into a double's exponent and mantissa fields
// give the value times 2^-1008 (f16 subnormals become double subnormals, also
// exact), and q and p carry the factor 2^1008, so every product is the exact
// f16 product. The dimension order inside the dot products is free, so lane
// (g, t) of a warp (g = lane / 4, t = lane % 4) holds dimensions
// [D/4 * t, D/4 * (t + 1)) of q and of key g of each 8-key group: one
// contiguous load of the K row per lane.
//
// Work split. A CTA (8 warps) serves R query rows and one kv head: R = 8 rows
// (a warp per row) for prefill-sized calls, R = 1 row (8 warps splitting its
// keys) for decode-sized ones. The keys of a row are split into contiguous
// ranges of at most KC over a thread-block cluster of C CTAs, which exchange
// the softmax maximum, the double sums of exp and the P V partial sums
// through distributed shared memory, each added in cluster-rank order.
// Scores and probabilities stay in shared memory ([R][8][KC + 4] floats).
constexpr int kDThreads = 256;
constexpr int kDWarps = kDThreads / 32;
constexpr uint32_t kDMaxKeysRow8 = 512;    // KC limit with 8 rows per CTA
constexpr uint32_t kDMaxKeysRow1 = 4096;   // KC limit with 1 row per CTA
// KC limit with R rows per CTA (R = 1, 2, 4, 8): the score array is
// R x 8 heads x (KC + 4) floats, about 128 KB at each limit
__host__ __device__ constexpr uint32_t dmma_max_keys(uint32_t rows) { return kDMaxKeysRow1 / rows; }
constexpr uint32_t kDMaxCluster = 8;       // portable cluster size

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

__device__ __forceinline__ uint32_t cluster_ctas() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
    return r;
}

// All threads of all CTAs of the cluster; release/acquire orders the shared
// memory each CTA wrote before it for the reads of the others after it.
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t dsmem_addr(const void * p, uint32_t rank) {
    uint32_t out;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;"
                 : "=r"(out)
                 : "r"(static_cast<uint32_t>(__cvta_generic_to_shared(p))), "r"(rank));
    return out;
}

__device__ __forceinline__ float dsmem_f32(uint32_t addr) {
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
    return v;
}

__device__ __forceinline__ double dsmem_f64(uint32_t addr) {
    double v;
    asm volatile("ld.shared::cluster.f64 %0, [%1];" : "=d"(v) : "r"(addr) : "memory");
    return v;
}

// D (8 x 8) += A (8 x 4) B (4 x 8) in double; this lane's elements:
// a = A[lane / 4][lane % 4], b = B[lane % 4][lane / 4],
// d0, d1 = D[lane / 4][2 (lane % 4) + 0, 1].
__device__ __forceinline__ void dmma(double & d0, double & d1, double a, double b) {
    asm volatile("mma.sync.aligned.m8n8k4.row.col.f64.f64.f64.f64 {%0, %1}, {%2}, {%3}, {%0, %1};"
                 : "+d"(d0), "+d"(d1)
                 : "d"(a), "d"(b));
}

// The two f16 values of w as doubles times 2^-1008, exactly.
__device__ __forceinline__ void h2_scaled_doubles(uint32_t w, double & lo, double & hi) {
    const uint32_t h0 = ((w & 0x7fffu) << 10) | ((w & 0x8000u) << 16);
    const uint32_t h1 = ((w >> 6) & 0x01fffc00u) | (w & 0x80000000u);
    lo = __hiloint2double(static_cast<int>(h0), 0);
    hi = __hiloint2double(static_cast<int>(h1), 0);
}

constexpr double kTwo1008 = 0x1p1008;  // 2^1008

struct DmmaLayout {
    uint32_t rows, kc, kcp;  // R, keys per CTA, row stride of the score array
    uint32_t x_bytes;        // scores / probabilities, later the warps' P V partials and the output rows
    uint32_t o_bytes;        // the CTA's P V partial sums [R][8][D] (read by the cluster)
    uint32_t total;
};

__host__ __device__ inline DmmaLayout dmma_layout(uint32_t rows, uint32_t kc, uint32_t head_dim) {
    DmmaLayout l;
    l.rows = rows;
    l.kc = kc;
    l.kcp = kc + 4;  // == 4 mod 8: the 8 head rows of a P fragment load hit distinct banks
    uint32_t x = rows * 8 * l.kcp * 4;
    // several warps per row (R < 8) add their P V partials through shared memory
    const uint32_t warp_partials = rows < kDWarps ? kDWarps * 8 * head_dim * 8 : 0;
    const uint32_t out_rows = rows * 8 * head_dim * 4;
    x = x > warp_partials ? x : warp_partials;
    x = x > out_rows ? x : out_rows;
    l.x_bytes = (x + 15) / 16 * 16;
    l.o_bytes = rows * 8 * head_dim * 8;
    // + wmax [8][8] f32, wsum [8][8] f64, lmax [8][8] f32, lsum [8][8] f64, gmax/ginv [8][8] f32 each,
    // key counts [8] u32
    l.total = l.x_bytes + l.o_bytes + 8 * 8 * (4 + 8 + 4 + 8 + 4 + 4) + 8 * 4;
    return l;
}

// MINB = 2 for decode-sized plans (one row per CTA) with more CTAs than SMs:
// two CTAs per SM keep, for example, a 64-sequence 7B decode call (256 CTAs)
// in one wave with twice the warps of loads in flight. With fewer CTAs than
// SMs the MINB = 1 kernel is faster (more registers, no spills, deeper load
// ring).
template <int D, int MINB>
__global__ void __launch_bounds__(kDThreads, MINB) dmma_attention_kernel(
    const float * __restrict__ q, const int32_t * __restrict__ seq, const int32_t * __restrict__ pos, uint32_t n,
    uint32_t heads, uint32_t kv_heads, const jfb_kv_slot * __restrict__ slots, uint32_t layer, float scale,
    uint32_t keys_cap, uint32_t R, uint32_t KC, float * __restrict__ out, jfb_q8k q8, int quantize) {
    constexpr int KS = D / 4;  // k-steps of a score (dimensions per lane)
    constexpr int NT = D / 8;  // n-tiles of P V (dimensions per lane)
    // K / V loads in flight per warp: three steps with one CTA per SM, two
    // with two (whose register budget is half)
    constexpr int RING = MINB >= 2 ? 2 : 3;
    extern __shared__ __align__(16) uint8_t smem_raw[];
    const DmmaLayout lay = dmma_layout(R, KC, D);
    float * xs = reinterpret_cast<float *>(smem_raw);                                // [R][8][kcp]
    double * wpart = reinterpret_cast<double *>(smem_raw);                           // [8 warps][8][D] (R = 1)
    float * orow = reinterpret_cast<float *>(smem_raw);                              // [R][8][D] final values
    double * octa = reinterpret_cast<double *>(smem_raw + lay.x_bytes);              // [R][8][D]
    float * wmax = reinterpret_cast<float *>(smem_raw + lay.x_bytes + lay.o_bytes);  // [8][8]
    double * wsum = reinterpret_cast<double *>(wmax + 64);                          // [8][8]
    float * lmax = reinterpret_cast<float *>(wsum + 64);                            // [8][8] per (row, head)
    double * lsum = reinterpret_cast<double *>(lmax + 64);                          // [8][8]
    float * gmax = reinterpret_cast<float *>(lsum + 64);                            // [8][8]
    float * ginv = gmax + 64;                                                       // [8][8]

    const uint32_t C = cluster_ctas(), crank = cluster_rank();
    const uint32_t tile = blockIdx.x / C, kvh = blockIdx.y;
    const uint32_t G = heads / kv_heads, h0 = kvh * G, kvd = kv_heads * D;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gq = lane >> 2, tq = lane & 3;
    const uint32_t S = kDWarps / R;                    // warps per row
    const uint32_t row_local = uint32_t(warp) / S, slice = uint32_t(warp) % S;
    const uint32_t kc0 = crank * KC;

    // keys of row `rl` of the tile that fall in this CTA's range [kc0, kc0 + KC)
    auto row_keys = [&](uint32_t rl) -> uint32_t {
        const uint32_t r = tile * R + rl;
        if (r >= n) return 0u;
        const uint32_t keys = min(uint32_t(pos[r]) + 1u, keys_cap);
        return keys > kc0 ? min(keys - kc0, KC) : 0u;
    };

    pdl_trigger();
    // positions, sequence ids and KV slots are per-call metadata, written
    // before the first kernel of the call: read them before waiting for the
    // previous kernel (whose output is q and the appended K/V rows)
    uint32_t * nk_s = reinterpret_cast<uint32_t *>(ginv + 64);  // [8] keys of each tile row in this CTA
    if (threadIdx.x < R) nk_s[threadIdx.x] = row_keys(threadIdx.x);
    const uint32_t r = tile * R + row_local;
    const uint32_t nk = row_keys(row_local);
    const uint32_t ng = (nk + 7) / 8;                  // 8-key groups of the row in this CTA
    const uint32_t gs = (ng + S - 1) / S;               // groups per warp of the row
    const uint32_t g_begin = min(ng, slice * gs), g_end = min(ng, g_begin + gs);
    const jfb_kv_slot slot = r < n ? slots[seq[r]] : jfb_kv_slot{};
    const uint16_t * kbase = slot.k + uint64_t(layer) * slot.capacity * kvd + kvh * D;
    const uint16_t * vbase = slot.v + uint64_t(layer) * slot.capacity * kvd + kvh * D;
    float * xrow = xs + row_local * 8 * lay.kcp;
    if (R == 1) {
        // decode-sized calls: this CTA's K and V rows into L2 while the
        // previous kernel finishes. The newest row may still be in flight
        // from that kernel; a prefetch cannot make it stale, as L2 is the
        // point every SM's stores reach and the rows are read after the wait.
        // With two CTAs per SM all CTAs are resident at once and their whole
        // caches can exceed L2, so those prefetch only their first 256 keys.
        constexpr uint32_t kLines = (D * 2 + 127) / 128;
        const uint32_t npre = MINB >= 2 ? min(nk, 256u) : nk;
        for (uint32_t i = threadIdx.x; i < npre * kLines; i += kDThreads) {
            const uint64_t at = uint64_t(kc0 + i / kLines) * kvd + (i % kLines) * 64;
            asm volatile("prefetch.global.L2 [%0];" ::"l"(kbase + at));
            asm volatile("prefetch.global.L2 [%0];" ::"l"(vbase + at));
        }
    }
    pdl_wait();

    // ---- scores of this warp's key groups. Four independent accumulator
    // chains per score (k-steps of each residue mod 4) keep several FP64 MMAs
    // in flight; the next group's K row is loaded while this one is summed.
    float mx = -INFINITY;  // this lane's maximum for head gq
    if (g_begin < g_end) {
        double qa[KS];
        {
            const bool live = uint32_t(gq) < G;
            const float * qh = q + uint64_t(r) * heads * D + uint64_t(h0 + (live ? gq : 0)) * D + KS * tq;
#pragma unroll
            for (int k = 0; k < KS; ++k) {
                qa[k] = live ? double(__half2float(__float2half_rn(qh[k]))) * kTwo1008 : 0.0;
            }
        }
        auto load_k = [&](uint32_t g, uint4 (&raw)[KS / 8]) {
            const uint32_t key = 8 * g + uint32_t(gq);  // this lane's K row (relative to kc0)
#pragma unroll
            for (int c = 0; c < KS / 8; ++c) {
                raw[c] = key < nk ? __ldg(reinterpret_cast<const uint4 *>(kbase + uint64_t(kc0 + key) * kvd + KS * tq) + c)
                                  : make_uint4(0, 0, 0, 0);
            }
        };
        auto score_group = [&](uint32_t g, const uint4 (&cur)[KS / 8]) {
            double acc[4][2];
#pragma unroll
            for (int a = 0; a < 4; ++a) acc[a][0] = acc[a][1] = 0.0;
#pragma unroll
            for (int c = 0; c < KS / 8; ++c) {
                const uint32_t w[4] = {cur[c].x, cur[c].y, cur[c].z, cur[c].w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    double b0, b1;
                    h2_scaled_doubles(w[e], b0, b1);
                    const int k0 = 8 * c + 2 * e;
                    dmma(acc[k0 & 3][0], acc[k0 & 3][1], qa[k0], b0);
                    dmma(acc[(k0 + 1) & 3][0], acc[(k0 + 1) & 3][1], qa[k0 + 1], b1);
                }
            }
            const double d0 = (acc[0][0] + acc[1][0]) + (acc[2][0] + acc[3][0]);
            const double d1 = (acc[0][1] + acc[1][1]) + (acc[2][1] + acc[3][1]);
            // d0, d1: scores of head gq for keys 8g + 2tq + {0, 1} (relative to kc0)
            const uint32_t j = 8 * g + 2 * uint32_t(tq);
            const float x0 = j < nk ? __fmul_rn(__double2float_rn(d0), scale) : -INFINITY;
            const float x1 = j + 1 < nk ? __fmul_rn(__double2float_rn(d1), scale) : -INFINITY;
            if (uint32_t(gq) < G) {
                xrow[gq * lay.kcp + j] = x0;
                xrow[gq * lay.kcp + j + 1] = x1;
            }
            mx = fmaxf(mx, fmaxf(x0, x1));
        };
        // K rows of RING groups in flight per warp (a ring of register buffers)
        uint4 kb[RING][KS / 8];
#pragma unroll
        for (int u = 0; u < RING - 1; ++u) {
            if (g_begin + u < g_end) load_k(g_begin + u, kb[u]);
        }
        for (uint32_t g = g_begin; g < g_end; g += RING) {
#pragma unroll
            for (int u = 0; u < RING; ++u) {
                if (g + u >= g_end) break;
                if (g + u + RING - 1 < g_end) load_k(g + u + RING - 1, kb[(u + RING - 1) % RING]);
                score_group(g + u, kb[u]);
            }
        }
    }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    if (tq == 0) wmax[warp * 8 + gq] = mx;
    __syncthreads();
    if (threadIdx.x < R * 8) {  // (row, head) maximum over the row's warps
        const uint32_t rl = threadIdx.x / 8, h = threadIdx.x % 8;
        float m = -INFINITY;
        for (uint32_t s = 0; s < S; ++s) m = fmaxf(m, wmax[(rl * S + s) * 8 + h]);
        lmax[threadIdx.x] = m;
    }
    cluster_sync_all();
    if (threadIdx.x < R * 8) {  // maximum over the cluster
        float m = -INFINITY;
        for (uint32_t c = 0; c < C; ++c) m = fmaxf(m, dsmem_f32(dsmem_addr(lmax + threadIdx.x, c)));
        gmax[threadIdx.x] = m;
    }
    __syncthreads();

    // ---- e = exp(x - max) and its double sum per (row, head); zero the key
    // tail up to the next multiple of 8 (read by the P V k-steps)
    for (uint32_t pr = uint32_t(warp); pr < R * 8; pr += kDWarps) {
        const uint32_t rl = pr / 8, h = pr % 8;
        double acc = 0.0;
        if (h < G) {
            const uint32_t keys = nk_s[rl];
            float * xr = xs + (rl * 8 + h) * lay.kcp;
            const float m = gmax[pr];
            for (uint32_t j = uint32_t(lane); j < (keys + 7) / 8 * 8; j += 32) {
                if (j < keys) {
                    const float e = exp_cw(__fsub_rn(xr[j], m));
                    xr[j] = e;
                    acc += double(e);
                } else {
                    xr[j] = 0.0f;
                }
            }
        }
        acc = warp_sum(acc);
        if (lane == 0) lsum[pr] = acc;
    }
    cluster_sync_all();
    if (threadIdx.x < R * 8) {  // total in cluster-rank order; 1 / total as the CPU rounds it
        double t = 0.0;
        for (uint32_t c = 0; c < C; ++c) t += dsmem_f64(dsmem_addr(lsum + threadIdx.x, c));
        ginv[threadIdx.x] = t > 0.0 ? __double2float_rn(__ddiv_rn(1.0, t)) : 0.0f;
    }
    __syncthreads();

    // ---- P V over this warp's keys: o[t][i] = O[head gq][dim 16 (2 tq + i) + t],
    // each probability p = f16(e * (1 / sum)) formed as it is used (the zeroed
    // key tail stays 0)
    double o[NT][2];
#pragma unroll
    for (int t = 0; t < NT; ++t) o[t][0] = o[t][1] = 0.0;
    {
        const uint32_t k_begin = 8 * g_begin, k_end = 8 * g_end;  // multiples of 8, within the zeroed tail
        const float * prow = xrow + gq * lay.kcp;
        const bool live = uint32_t(gq) < G;
        const float inv = live ? ginv[row_local * 8 + uint32_t(gq)] : 0.0f;
        auto load_v = [&](uint32_t kk, uint4 (&raw)[NT / 8]) {
            const uint32_t j = kk + uint32_t(tq);  // this lane's V row (relative to kc0)
#pragma unroll
            for (int c = 0; c < NT / 8; ++c) {
                raw[c] = j < nk ? __ldg(reinterpret_cast<const uint4 *>(vbase + uint64_t(kc0 + j) * kvd + NT * gq) + c)
                                : make_uint4(0, 0, 0, 0);
            }
        };
        auto pv_step = [&](uint32_t kk, const uint4 (&cur)[NT / 8]) {
            const double a =
                live ? double(__half2float(__float2half_rn(__fmul_rn(prow[kk + uint32_t(tq)], inv)))) * kTwo1008 : 0.0;
#pragma unroll
            for (int c = 0; c < NT / 8; ++c) {
                const uint32_t w[4] = {cur[c].x, cur[c].y, cur[c].z, cur[c].w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    double b0, b1;
                    h2_scaled_doubles(w[e], b0, b1);
                    dmma(o[8 * c + 2 * e][0], o[8 * c + 2 * e][1], a, b0);
                    dmma(o[8 * c + 2 * e + 1][0], o[8 * c + 2 * e + 1][1], a, b1);
                }
            }
        };
        // V rows of RING key steps in flight per warp
        uint4 vb[RING][NT / 8];
#pragma unroll
        for (int u = 0; u < RING - 1; ++u) {
            if (k_begin + 4 * uint32_t(u) < k_end) load_v(k_begin + 4 * uint32_t(u), vb[u]);
        }
        for (uint32_t kk = k_begin; kk < k_end; kk += 4 * RING) {
#pragma unroll
            for (int u = 0; u < RING; ++u) {
                const uint32_t k = kk + 4 * uint32_t(u);
                if (k >= k_end) break;
                if (k + 4 * (RING - 1) < k_end) load_v(k + 4 * (RING - 1), vb[(u + RING - 1) % RING]);
                pv_step(k, vb[u]);
            }
        }
    }
    __syncthreads();  // every warp is done with the probabilities: the score array is reused below

    // ---- the CTA's partial sums [R][8][D]
    if (S > 1) {
        // the S warps of a row add their partials in slice order
        double * wp = wpart + uint64_t(warp) * 8 * D + gq * D;
#pragma unroll
        for (int t = 0; t < NT; ++t) {
#pragma unroll
            for (int i = 0; i < 2; ++i) wp[NT * (2 * tq + i) + t] = o[t][i];
        }
        __syncthreads();
        for (uint32_t e = threadIdx.x; e < R * 8 * D; e += kDThreads) {
            const uint32_t rl = e / (8 * D), at = e % (8 * D);
            double t = 0.0;
            for (uint32_t w = 0; w < S; ++w) t += wpart[uint64_t(rl * S + w) * 8 * D + at];
            octa[e] = t;
        }
    } else {
        double * op = octa + uint64_t(row_local) * 8 * D + gq * D;
#pragma unroll
        for (int t = 0; t < NT; ++t) {
#pragma unroll
            for (int i = 0; i < 2; ++i) op[NT * (2 * tq + i) + t] = o[t][i];
        }
    }
    cluster_sync_all();

    // ---- rank 0 adds the cluster's partials in rank order, writes the rows
    // and quantizes them to Q8_K
    if (crank == 0) {
        const uint32_t width = G * D;
        for (uint32_t e = threadIdx.x; e < R * 8 * D; e += kDThreads) {
            const uint32_t rl = e / (8 * D), h = (e / D) % 8, d = e % D;
            const uint32_t rr = tile * R + rl;
            if (h >= G || rr >= n) continue;
            double t = 0.0;
            for (uint32_t c = 0; c < C; ++c) t += dsmem_f64(dsmem_addr(octa + e, c));
            const float v = __double2float_rn(t);
            orow[rl * width + h * D + d] = v;
            out[uint64_t(rr) * heads * D + uint64_t(h0) * D + h * D + d] = v;
        }
        if (quantize) {
            __syncthreads();
            const uint32_t per_row = width / kQK;  // Q8_K blocks of this kv head's heads
            for (uint32_t b = uint32_t(warp); b < R * per_row; b += kDWarps) {
                const uint32_t rl = b / per_row, blk = b % per_row;
                const uint32_t rr = tile * R + rl;
                if (rr >= n) continue;
                const float * src = orow + rl * width + blk * kQK + 8 * lane;
                const float4 a = *reinterpret_cast<const float4 *>(src);
                const float4 c = *reinterpret_cast<const float4 *>(src + 4);
                const Vals8 y = {{a.x, a.y, a.z, a.w, c.x, c.y, c.z, c.w}};
                q8k_block_warp(y, q8_dest(q8, rr, (h0 * D) / kQK + blk, heads * D / kQK));
            }
        }
    }
    cluster_sync_all();  // no CTA leaves while another may still read its shared memory
}

struct DmmaPlan {
    bool ok;
    bool two_per_sm;  // the MINB = 2 kernel: one-row CTAs that would not fit in one wave at one per SM
    uint32_t rows, kc, cluster, tiles;
    DmmaLayout layout;
};

DmmaPlan dmma_plan(uint32_t n, uint32_t heads, uint32_t kv_heads, uint32_t head_dim, uint32_t max_keys, int sms) {
    DmmaPlan pl{};
    pl.ok = false;
    if ((head_dim != 64 && head_dim != 128) || heads / kv_heads > 8 || n == 0) return pl;
    // prefill-sized calls: as many rows per CTA as keep the longest row's keys
    // in one CTA (8 rows up to 512 keys, 4 up to 1024, 2 up to 2048), so that
    // no cluster CTA sits beside a partner that has all the keys of a causal
    // row; beyond 2048 keys, 8 rows over a cluster. Decode-sized calls: 1 row.
    if (uint64_t(n) * kv_heads >= uint64_t(8) * uint64_t(sms)) {
        pl.rows = max_keys <= dmma_max_keys(8) ? 8u : max_keys <= dmma_max_keys(4) ? 4u
                  : max_keys <= dmma_max_keys(2) ? 2u : 8u;
    } else {
        pl.rows = 1u;
    }
    const uint32_t kc_max = dmma_max_keys(pl.rows);
    const uint32_t c_min = (max_keys + kc_max - 1) / kc_max;
    if (c_min > kDMaxCluster) return pl;
    pl.tiles = (n + pl.rows - 1) / pl.rows;
    uint32_t c = c_min;
    if (pl.rows == 1) {  // about one CTA per SM for decode-sized calls
        const uint64_t ctas = uint64_t(pl.tiles) * kv_heads;
        const uint32_t want = uint32_t(std::min<uint64_t>(kDMaxCluster, std::max<uint64_t>(1, uint64_t(sms) / ctas)));
        c = std::max(c, want);
    }
    c = std::min(c, std::max(1u, (max_keys + 7) / 8));  // no CTA without keys at all
    pl.cluster = std::max(c, c_min);
    pl.kc = ((max_keys + pl.cluster - 1) / pl.cluster + 7) / 8 * 8;
    if (pl.kc > kc_max) return pl;
    pl.layout = dmma_layout(pl.rows, pl.kc, head_dim);
    if (uint64_t(pl.tiles) * pl.cluster > 0x7fffffffu || kv_heads > 65535u) return pl;
    pl.two_per_sm = pl.rows == 1 && uint64_t(pl.tiles) * pl.cluster * kv_heads > uint64_t(sms);
    pl.ok = true;
    return pl;
}

template <int D, int MINB>
jfb_status launch_dmma_kernel(const DmmaPlan & pl, const float * q, uint32_t n, const int32_t * seq,
                              const int32_t * pos, uint32_t heads, uint32_t kv_heads, const jfb_kv_slot * slots,
                              uint32_t layer, float scale, uint32_t keys_cap, float * out, jfb_q8k q8, int quantize,
                              cudaStream_t s) {
    auto kernel = dmma_attention_kernel<D, MINB>;
    static std::mutex mu;
    static uint32_t attribute_bytes[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = 0;
    {
        std::lock_guard<std::mutex> lock(mu);
        if (attribute_bytes[dev] < pl.layout.total) {
            // the largest layout of any plan: one attribute for every later call
            uint32_t bytes = pl.layout.total;
            for (uint32_t r = 1; r <= 8; r *= 2) bytes = std::max<uint32_t>(bytes, dmma_layout(r, dmma_max_keys(r), D).total);
            cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(bytes));
            if (e != cudaSuccess) {
                return status_error(JFB_STATUS_CUDA_ERROR, "attention shared memory attribute: %s", cudaGetErrorString(e));
            }
            attribute_bytes[dev] = bytes;
        }
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(pl.tiles * pl.cluster, kv_heads, 1);
    cfg.blockDim = dim3(kDThreads, 1, 1);
    cfg.dynamicSmemBytes = pl.layout.total;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = pl.cluster;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (pdl_enabled()) {
        attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[1].val.programmaticStreamSerializationAllowed = 1;
        cfg.numAttrs = 2;
    }
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, q, seq, pos, n, heads, kv_heads, slots, layer, scale, keys_cap,
                                             pl.rows, pl.kc, out, q8, quantize);
    if (e != cudaSuccess) return status_error(JFB_STATUS_CUDA_ERROR, "jfb_attention: %s", cudaGetErrorString(e));
    return launch_status("jfb_attention");
}

template <int D>
jfb_status launch_dmma(const DmmaPlan & pl, const float * q, uint32_t n, const int32_t * seq, const int32_t * pos,
                       uint32_t heads, uint32_t kv_heads, const jfb_kv_slot * slots, uint32_t layer, float scale,
                       uint32_t keys_cap, float * out, jfb_q8k q8, int quantize, cudaStream_t s) {
    if (pl.two_per_sm) {
        return launch_dmma_kernel<D, 2>(pl, q, n, seq, pos, heads, kv_heads, slots, layer, scale, keys_cap, out, q8,
                                        quantize, s);
    }
    return launch_dmma_kernel<D, 1>(pl, q, n, seq, pos, heads, kv_heads, slots, layer, scale, keys_cap, out, q8,
                                    quantize, s);
}

int device_sms() {
    static std::mutex mu;
    static int cached[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    std::lock_guard<std::mutex> lock(mu);
    if (cached[dev] == 0) {
        int v = 0;
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
        cached[dev] = v;
    }
    return cached[dev];
}

}  // namespace
}  // namespace jfb

using namespace jfb;

extern "C" uint64_t jfb_attention_scratch_bytes(uint32_t n, uint32_t heads, uint32_t head_dim, uint32_t max_keys) {
    const uint64_t splits = (uint64_t(max_keys) + kChunk - 1) / kChunk;
    if (splits > kMaxSplits) return UINT64_MAX;  // beyond any supported call
    return scratch_size(n, heads, head_dim, uint32_t(splits));
}

extern "C" uint64_t jfb_attention_call_scratch_bytes(uint32_t n, uint32_t heads, uint32_t kv_heads, uint32_t head_dim,
                                                     uint32_t max_keys) {
    if (n == 0 || kv_heads == 0 || heads % kv_heads != 0 || max_keys == 0) return 0;
    if (uint64_t(max_keys) > uint64_t(kMaxSplits) * kChunk) return UINT64_MAX;
    if (dmma_plan(n, heads, kv_heads, head_dim, max_keys, device_sms()).ok) return 0;
    return jfb_attention_scratch_bytes(n, heads, head_dim, max_keys);
}

extern "C" jfb_status jfb_attention(const float * q, uint32_t n, const int32_t * seq, const int32_t * pos,
                                    uint32_t heads, uint32_t kv_heads, uint32_t head_dim, uint32_t max_keys,
                                    const jfb_kv_slot * slots, uint32_t layer, void * scratch, uint64_t scratch_bytes,
                                    float * out, const jfb_q8k * out_q8, void * stream) {
    if (q == nullptr || seq == nullptr || pos == nullptr || slots == nullptr || out == nullptr) {
        return status_error(JFB_STATUS_INVALID_ARGUMENT, "attention operands are required");
    }
    if (heads == 0 || kv_heads == 0 || heads % kv_heads != 0 || heads / kv_heads > uint32_t(kMaxGroup) ||
        head_dim == 0 || head_dim > uint32_t(kMaxHeadDim) || head_dim % 2 != 0 || max_keys == 0) {
        return status_error(JFB_STATUS_INVALID_ARGUMENT, "attention dimensions are unsupported");
    }
    if (out_q8 != nullptr && (heads * head_dim) % kQK != 0) {
        return status_error(JFB_STATUS_INVALID_ARGUMENT, "Q8_K attention output needs a width multiple of 256");
    }
    if (out_q8 != nullptr) {
        const jfb_status tc = check_q8_tensor_core(out_q8, n);
        if (tc.code != JFB_STATUS_OK) return tc;
    }
    // every ceil-division below stays far from the uint32 range
    if (uint64_t(max_keys) > uint64_t(kMaxSplits) * kChunk || kv_heads > 65535u || heads > 65535u) {
        return status_error(JFB_STATUS_INVALID_ARGUMENT, "attention grid too large");
    }
    if (n == 0) return status_ok();
    const uint32_t splits = (max_keys + kChunk - 1) / kChunk;
    cudaStream_t s = as_stream(stream);
    const DmmaPlan plan = dmma_plan(n, heads, kv_heads, head_dim, max_keys, device_sms());
    // only the four-launch form below uses the scratch
    if (!plan.ok && (scratch == nullptr || scratch_bytes < jfb_attention_scratch_bytes(n, heads, head_dim, max_keys))) {
        return status_error(JFB_STATUS_INVALID_ARGUMENT, "attention scratch is too small");
    }
    if (plan.ok) {
        const bool fused_q8 = out_q8 != nullptr && ((heads / kv_heads) * head_dim) % kQK == 0;
        const jfb_q8k q8_fused = fused_q8 ? *out_q8 : jfb_q8k{};
        const float fscale = 1.0f / sqrtf(float(head_dim));
        jfb_status st = head_dim == 64 ? launch_dmma<64>(plan, q, n, seq, pos, heads, kv_heads, slots, layer, fscale,
                                                         max_keys, out, q8_fused, fused_q8 ? 1 : 0, s)
                                       : launch_dmma<128>(plan, q, n, seq, pos, heads, kv_heads, slots, layer, fscale,
                                                          max_keys, out, q8_fused, fused_q8 ? 1 : 0, s);
        if (st.code != JFB_STATUS_OK || out_q8 == nullptr || fused_q8) return st;
        return jfb_quantize_q8k(out, n, heads * head_dim, out_q8, stream);
    }
    const Scratch sc = carve(scratch, n, heads, head_dim, splits);
    const float scale = 1.0f / sqrtf(float(head_dim));
    cudaError_t e = launch_k(scores_kernel, dim3(n, kv_heads, splits), dim3(kThreads), 0, s, q, seq, pos, heads, kv_heads,
                             head_dim, slots, layer, scale, splits, sc);
    if (e == cudaSuccess) e = launch_k(stats_kernel, dim3(n, heads), dim3(kThreads), 0, s, pos, heads, splits, sc);
    if (e == cudaSuccess) {
        e = launch_k(pv_kernel, dim3(n, kv_heads, splits), dim3(kThreads), 0, s, seq, pos, heads, kv_heads, head_dim, slots,
                     layer, splits, sc);
    }
    const jfb_q8k q8 = out_q8 != nullptr ? *out_q8 : jfb_q8k{};
    if (e == cudaSuccess) {
        e = launch_k(combine_kernel, dim3(n), dim3(256), 0, s, pos, heads, head_dim, splits, sc, out, q8,
                     out_q8 != nullptr ? 1 : 0);
    }
    if (e != cudaSuccess) return status_error(JFB_STATUS_CUDA_ERROR, "jfb_attention: %s", cudaGetErrorString(e));
    return launch_status("jfb_attention");
}

// ---- attention without caller-provided scratch --------------------------------

// The scratch of jfb_attention_static_scratch: allocated with the module on
// every device that loads this library, never by a call.
static __device__ __align__(256) unsigned char g_attention_scratch[JFB_ATTENTION_STATIC_SCRATCH_BYTES];

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mutex;
void * g_scratch_address[kMaxDevices] = {};

// Device address of g_attention_scratch on the current device. In host code
// the symbol's name is only a host-side handle, so the address is looked up
// once per device with that device current, and cached.
jfb_status static_scratch_address(void ** address) {
    int device = -1;
    cudaError_t e = cudaGetDevice(&device);
    if (e != cudaSuccess) return status_error(JFB_STATUS_CUDA_ERROR, "cudaGetDevice: %s", cudaGetErrorString(e));
    if (device < 0 || device >= kMaxDevices) {
        return status_error(JFB_STATUS_UNSUPPORTED, "device ordinal %d is beyond the static scratch table", device);
    }
    std::lock_guard lock(g_scratch_mutex);
    if (g_scratch_address[device] == nullptr) {
        void * p = nullptr;
        e = cudaGetSymbolAddress(&p, g_attention_scratch);
        if (e != cudaSuccess || p == nullptr) {
            return status_error(JFB_STATUS_CUDA_ERROR, "cudaGetSymbolAddress(attention scratch): %s",
                                cudaGetErrorString(e));
        }
        g_scratch_address[device] = p;
    }
    *address = g_scratch_address[device];
    return status_ok();
}

}  // namespace

extern "C" jfb_status jfb_attention_static_scratch(const float * q, uint32_t n, const int32_t * seq, const int32_t * pos,
                                                   uint32_t heads, uint32_t kv_heads, uint32_t head_dim,
                                                   uint32_t max_keys, const jfb_kv_slot * slots, uint32_t layer,
                                                   float * out, const jfb_q8k * out_q8, void * stream) {
    if (heads == 0 || head_dim == 0 || max_keys == 0) {
        return status_error(JFB_STATUS_INVALID_ARGUMENT, "attention dimensions are unsupported");
    }
    if (uint64_t(max_keys) > uint64_t(kMaxSplits) * kChunk) {
        return status_error(JFB_STATUS_INVALID_ARGUMENT, "attention grid too large");
    }
    const uint64_t needed = jfb_attention_scratch_bytes(n, heads, head_dim, max_keys);
    if (needed > JFB_ATTENTION_STATIC_SCRATCH_BYTES) {
        return status_error(JFB_STATUS_INVALID_ARGUMENT,
                            "attention needs %llu scratch bytes, more than the %u-byte static scratch array",
                            static_cast<unsigned long long>(needed), JFB_ATTENTION_STATIC_SCRATCH_BYTES);
    }
    void * scratch = nullptr;
    const jfb_status s = static_scratch_address(&scratch);
    if (s.code != JFB_STATUS_OK) return s;
    return jfb_attention(q, n, seq, pos, heads, kv_heads, head_dim, max_keys, slots, layer, scratch,
                         JFB_ATTENTION_STATIC_SCRATCH_BYTES, out, out_q8, stream);
}
