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
// Rows of up to 8192 keys with head_dim 64 or 128 take a single launch (see
// the single-launch path below). Otherwise four launches over a
// (row, kv head, 64-key chunk) grid:
//   1. scores x_j (and each chunk's maximum) -> scratch
//   2. per (row, head): max over chunks, sum_j exp(x_j - max) in double
//   3. P V partial sums per chunk in double -> scratch
//   4. per row: sum of the chunk partials, f32 output (+ Q8_K quantization)
// A CTA of launches 1 and 3 serves the G = heads/kv_heads query heads that
// share its kv head, so each K and V row is read once for G heads.
#include "common.cuh"

#include <mutex>

namespace jfb {
namespace {

constexpr int kThreads = 128;
constexpr int kChunk = 64;      // keys per CTA
constexpr int kMaxGroup = 16;   // query heads per kv head
constexpr int kMaxHeadDim = 256;

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

// Launch 1: x_j = f32(sum_d k_jd * f16(q_d)) * scale for the chunk's keys.
__global__ void __launch_bounds__(kThreads) scores_kernel(const float * __restrict__ q, const int32_t * __restrict__ seq,
                                                        const int32_t * __restrict__ pos, uint32_t heads, uint32_t kv_heads,
                                                        uint32_t head_dim, const jfb_kv_slot * __restrict__ slots,
                                                        uint32_t layer, float scale, uint32_t splits, Scratch sc) {
    __shared__ float q_s[kMaxGroup * kMaxHeadDim];
    __shared__ float x_s[kMaxGroup][kChunk];
    const uint32_t r = blockIdx.x, kvh = blockIdx.y, split = blockIdx.z;
    const uint32_t keys = uint32_t(pos[r]) + 1u;
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
    const uint32_t r = blockIdx.x, h = blockIdx.y;
    const uint32_t keys = uint32_t(pos[r]) + 1u;
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
    const uint32_t r = blockIdx.x, kvh = blockIdx.y, split = blockIdx.z;
    const uint32_t keys = uint32_t(pos[r]) + 1u;
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
    const uint32_t r = blockIdx.x;
    const uint32_t D = head_dim, width = heads * D;
    const uint32_t used = (uint32_t(pos[r]) + kChunk) / kChunk;
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

// ---- single-launch path -------------------------------------------------------
//
// One CTA per (row, kv head, group of HPC query heads) does the whole row:
//   scores   16 lanes per key for D = 128 (each lane 8 dims, one 16-byte load
//            of the K row, so a K row is one coalesced 256-byte read); each
//            lane keeps its 8 dims of f16(q) for the HPC heads in registers
//            as doubles and accumulates k*q with DFMA (the f16*f16 product is
//            exact, so this equals adding the exact products in double); the
//            lane partials are added by a shuffle tree;
//   softmax  block reductions for the maximum and the double sum of exp;
//   P V      each thread owns 4 dims x HPC heads in double over an interleaved
//            share of the keys; the shares are added in a fixed order.
// The exact semantics are those of the four-launch path above. Scores and
// probabilities live in shared memory, so the row's key count is bounded by
// kFusedMaxKeys; longer rows use the four-launch path.
constexpr int kFusedThreads = 256;
constexpr uint32_t kFusedMaxKeys = 8192;

template <int HPC, int D>
__host__ __device__ constexpr uint32_t fused_smem_bytes(uint32_t keys_cap) {
    return (kFusedThreads / (D / 4)) * HPC * D * 8  // PV partials [S][HPC][D] double
           + HPC * D * 4                             // output values of the CTA
           + HPC * keys_cap * 4;                     // scores / probabilities [HPC][keys_cap]
}

template <int HPC, int D>
__global__ void __launch_bounds__(kFusedThreads, 1) fused_kernel(const float * __restrict__ q, const int32_t * __restrict__ seq,
                                                            const int32_t * __restrict__ pos, uint32_t heads,
                                                            uint32_t kv_heads, const jfb_kv_slot * __restrict__ slots,
                                                            uint32_t layer, float scale, uint32_t keys_cap,
                                                            float * __restrict__ out, jfb_q8k q8, int quantize) {
    constexpr int L = D / 8;                  // lanes per key in the score pass
    constexpr int KPW = 32 / L;               // keys per warp step
    constexpr int DT = D / 4;                 // threads per key share in the P V pass
    constexpr int S = kFusedThreads / DT;     // key shares
    constexpr int W = kFusedThreads / 32;
    extern __shared__ __align__(16) uint8_t smem_raw[];
    double * red = reinterpret_cast<double *>(smem_raw);   // [S][HPC][D]
    float * outs = reinterpret_cast<float *>(red + S * HPC * D);  // [HPC * D]
    float * xs = outs + HPC * D;                            // [HPC][keys_cap]
    __shared__ float wmax[W][HPC];
    __shared__ double wsum[W][HPC];
    __shared__ float stat[HPC][2];  // max, 1 / sum
    __shared__ unsigned long long q8_keys[8];

    const uint32_t r = blockIdx.x;
    const uint32_t G = heads / kv_heads, groups = G / HPC;
    const uint32_t kvh = blockIdx.y / groups;
    const uint32_t h0 = kvh * G + (blockIdx.y % groups) * HPC;  // first query head of this CTA
    // keys beyond the caller's max_keys are ignored, as on the four-launch path
    const uint32_t keys = min(uint32_t(pos[r]) + 1u, keys_cap), kvd = kv_heads * D;
    const jfb_kv_slot slot = slots[seq[r]];
    const uint16_t * kbase = slot.k + uint64_t(layer) * slot.capacity * kvd + kvh * D;
    const uint16_t * vbase = slot.v + uint64_t(layer) * slot.capacity * kvd + kvh * D;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    // ---- scores
    {
        const int sub = lane / L, li = lane % L;
        double qr[HPC][8];
#pragma unroll
        for (int h = 0; h < HPC; ++h) {
            const float * qh = q + uint64_t(r) * heads * D + uint64_t(h0 + h) * D + 8 * li;
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                qr[h][e] = double(__half2float(__float2half_rn(qh[e])));
                asm volatile("" : "+d"(qr[h][e]));  // keep in a register: no reload inside the key loop
            }
        }
        float mx[HPC];
#pragma unroll
        for (int h = 0; h < HPC; ++h) mx[h] = -INFINITY;
        constexpr int U = 8;  // key steps whose loads are in flight together
        for (uint32_t jb = uint32_t(warp) * KPW; jb < keys; jb += W * KPW * U) {
            uint4 raw[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const uint32_t j = jb + uint32_t(u * W * KPW + sub);
                raw[u] = j < keys ? __ldg(reinterpret_cast<const uint4 *>(kbase + uint64_t(j) * kvd + 8 * li))
                                  : make_uint4(0, 0, 0, 0);
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const uint32_t j = jb + uint32_t(u * W * KPW + sub);
                double acc[HPC];
#pragma unroll
                for (int h = 0; h < HPC; ++h) acc[h] = 0.0;
                const uint32_t wv[4] = {raw[u].x, raw[u].y, raw[u].z, raw[u].w};
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    const double kd = double(half_bits_to_float(uint16_t(wv[e / 2] >> (16 * (e & 1)))));
#pragma unroll
                    for (int h = 0; h < HPC; ++h) acc[h] = fma(kd, qr[h][e], acc[h]);
                }
#pragma unroll
                for (int o = L / 2; o > 0; o >>= 1) {
#pragma unroll
                    for (int h = 0; h < HPC; ++h) acc[h] += __shfl_xor_sync(0xffffffffu, acc[h], o);
                }
                if (li == 0 && j < keys) {
#pragma unroll
                    for (int h = 0; h < HPC; ++h) {
                        const float x = __fmul_rn(__double2float_rn(acc[h]), scale);
                        xs[h * keys_cap + j] = x;
                        mx[h] = fmaxf(mx[h], x);
                    }
                }
            }
        }
#pragma unroll
        for (int h = 0; h < HPC; ++h) {
            const float m = warp_max(mx[h]);
            if (lane == 0) wmax[warp][h] = m;
        }
    }
    __syncthreads();
    if (threadIdx.x < HPC) {
        float m = -INFINITY;
        for (int w = 0; w < W; ++w) m = fmaxf(m, wmax[w][threadIdx.x]);
        stat[threadIdx.x][0] = m;
    }
    __syncthreads();

    // ---- softmax: e = exp(x - max), 1 / double sum, p = f16(e * inv)
    {
        double sum[HPC];
#pragma unroll
        for (int h = 0; h < HPC; ++h) {
            const float m = stat[h][0];
            double acc = 0.0;
            for (uint32_t j = threadIdx.x; j < keys; j += kFusedThreads) {
                const float e = exp_cw(__fsub_rn(xs[h * keys_cap + j], m));
                xs[h * keys_cap + j] = e;
                acc += double(e);
            }
            sum[h] = warp_sum(acc);
        }
        if (lane == 0) {
#pragma unroll
            for (int h = 0; h < HPC; ++h) wsum[warp][h] = sum[h];
        }
    }
    __syncthreads();
    if (threadIdx.x < HPC) {
        double t = 0.0;
        for (int w = 0; w < W; ++w) t += wsum[w][threadIdx.x];
        stat[threadIdx.x][1] = __double2float_rn(__ddiv_rn(1.0, t));  // t >= 1 (the maximum contributes 1)
    }
    __syncthreads();
#pragma unroll
    for (int h = 0; h < HPC; ++h) {
        const float inv = stat[h][1];
        for (uint32_t j = threadIdx.x; j < keys; j += kFusedThreads) {
            xs[h * keys_cap + j] = __half2float(__float2half_rn(__fmul_rn(xs[h * keys_cap + j], inv)));
        }
    }
    __syncthreads();

    // ---- P V
    {
        const int dq = threadIdx.x % DT, share = threadIdx.x / DT;
        double acc[HPC][4];
#pragma unroll
        for (int h = 0; h < HPC; ++h) {
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[h][e] = 0.0;
        }
        constexpr int U = 8;  // keys whose V loads are in flight together
        for (uint32_t jb = uint32_t(share); jb < keys; jb += S * U) {
            uint2 raw[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const uint32_t j = jb + uint32_t(u * S);
                raw[u] = j < keys ? __ldg(reinterpret_cast<const uint2 *>(vbase + uint64_t(j) * kvd + 4 * dq))
                                  : make_uint2(0, 0);
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const uint32_t j = jb + uint32_t(u * S);
                if (j >= keys) break;
                const double v0 = double(half_bits_to_float(uint16_t(raw[u].x & 0xffffu)));
                const double v1 = double(half_bits_to_float(uint16_t(raw[u].x >> 16)));
                const double v2 = double(half_bits_to_float(uint16_t(raw[u].y & 0xffffu)));
                const double v3 = double(half_bits_to_float(uint16_t(raw[u].y >> 16)));
#pragma unroll
                for (int h = 0; h < HPC; ++h) {
                    const double pj = double(xs[h * keys_cap + j]);
                    acc[h][0] = fma(v0, pj, acc[h][0]);
                    acc[h][1] = fma(v1, pj, acc[h][1]);
                    acc[h][2] = fma(v2, pj, acc[h][2]);
                    acc[h][3] = fma(v3, pj, acc[h][3]);
                }
            }
        }
#pragma unroll
        for (int h = 0; h < HPC; ++h) {
#pragma unroll
            for (int e = 0; e < 4; ++e) red[(share * HPC + h) * D + 4 * dq + e] = acc[h][e];
        }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < HPC * D; i += kFusedThreads) {
        double t = 0.0;
#pragma unroll
        for (int sh = 0; sh < S; ++sh) t += red[sh * HPC * D + i];
        const float v = __double2float_rn(t);
        outs[i] = v;
        out[uint64_t(r) * heads * D + uint64_t(h0) * D + i] = v;
    }
    if (!quantize) return;
    __syncthreads();
    const uint32_t blocks_per_row = heads * D / kQK;
#pragma unroll 1
    for (int c = 0; c < HPC * D / kQK; ++c) {
        const uint32_t blk = uint32_t((uint64_t(h0) * D) / kQK) + uint32_t(c);
        q8k_block_256(outs[c * kQK + threadIdx.x], q8_dest(q8, r, blk, blocks_per_row), q8_keys);
    }
}

template <int D>
jfb_status launch_fused_d(int hpc, const float * q, uint32_t n, const int32_t * seq, const int32_t * pos, uint32_t heads,
                          uint32_t kv_heads, const jfb_kv_slot * slots, uint32_t layer, float scale,
                          uint32_t keys_cap, float * out, jfb_q8k q8, int quantize, cudaStream_t s) {
    const dim3 grid(n, kv_heads * ((heads / kv_heads) / uint32_t(hpc)));
    auto go = [&](auto kernel, uint32_t bytes) -> jfb_status {
        const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(bytes));
        if (e != cudaSuccess) {
            return status_error(JFB_STATUS_CUDA_ERROR, "attention shared memory attribute: %s", cudaGetErrorString(e));
        }
        kernel<<<grid, kFusedThreads, bytes, s>>>(q, seq, pos, heads, kv_heads, slots, layer, scale, keys_cap, out, q8,
                                                  quantize);
        return launch_status("jfb_attention");
    };
    switch (hpc) {
    case 4: return go(fused_kernel<4, D>, fused_smem_bytes<4, D>(keys_cap));
    case 3: return go(fused_kernel<3, D>, fused_smem_bytes<3, D>(keys_cap));
    case 2: return go(fused_kernel<2, D>, fused_smem_bytes<2, D>(keys_cap));
    default: return go(fused_kernel<1, D>, fused_smem_bytes<1, D>(keys_cap));
    }
}

// Query heads per CTA of the single-launch path: the largest of 4, 3, 2, 1
// dividing the group, halved while that leaves the GPU without a full wave.
int fused_heads_per_cta(uint32_t n, uint32_t heads, uint32_t kv_heads) {
    const uint32_t G = heads / kv_heads;
    int hpc = 1;
    for (int c = 4; c >= 1; --c) {
        if (G % uint32_t(c) == 0) {
            hpc = c;
            break;
        }
    }
    while (hpc % 2 == 0 && uint64_t(n) * kv_heads * (G / uint32_t(hpc)) < 148) hpc /= 2;
    return hpc;
}

}  // namespace
}  // namespace jfb

using namespace jfb;

extern "C" uint64_t jfb_attention_scratch_bytes(uint32_t n, uint32_t heads, uint32_t head_dim, uint32_t max_keys) {
    const uint32_t splits = (max_keys + kChunk - 1) / kChunk;
    return scratch_size(n, heads, head_dim, splits);
}

extern "C" jfb_status jfb_attention(const float * q, uint32_t n, const int32_t * seq, const int32_t * pos,
                                    uint32_t heads, uint32_t kv_heads, uint32_t head_dim, uint32_t max_keys,
                                    const jfb_kv_slot * slots, uint32_t layer, void * scratch, uint64_t scratch_bytes,
                                    float * out, const jfb_q8k * out_q8, void * stream) {
    if (q == nullptr || seq == nullptr || pos == nullptr || slots == nullptr || out == nullptr || scratch == nullptr) {
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
    if (scratch_bytes < jfb_attention_scratch_bytes(n, heads, head_dim, max_keys)) {
        return status_error(JFB_STATUS_INVALID_ARGUMENT, "attention scratch is too small");
    }
    if (n == 0) return status_ok();
    const uint32_t splits = (max_keys + kChunk - 1) / kChunk;
    if (splits > 65535u || kv_heads > 65535u || heads > 65535u) {
        return status_error(JFB_STATUS_INVALID_ARGUMENT, "attention grid too large");
    }
    cudaStream_t s = as_stream(stream);
    const jfb_q8k q8_fused = out_q8 != nullptr ? *out_q8 : jfb_q8k{};
    if ((head_dim == 64 || head_dim == 128) && max_keys <= kFusedMaxKeys) {
        const int hpc = fused_heads_per_cta(n, heads, kv_heads);
        const uint32_t keys_cap = (max_keys + 3) / 4 * 4;
        const bool fused_q8 = out_q8 != nullptr && (uint32_t(hpc) * head_dim) % kQK == 0;
        const float fscale = 1.0f / sqrtf(float(head_dim));
        jfb_status st = head_dim == 64 ? launch_fused_d<64>(hpc, q, n, seq, pos, heads, kv_heads, slots, layer, fscale,
                                                            keys_cap, out, q8_fused, fused_q8 ? 1 : 0, s)
                                       : launch_fused_d<128>(hpc, q, n, seq, pos, heads, kv_heads, slots, layer, fscale,
                                                             keys_cap, out, q8_fused, fused_q8 ? 1 : 0, s);
        if (st.code != JFB_STATUS_OK || out_q8 == nullptr || fused_q8) return st;
        return jfb_quantize_q8k(out, n, heads * head_dim, out_q8, stream);
    }
    const Scratch sc = carve(scratch, n, heads, head_dim, splits);
    const float scale = 1.0f / sqrtf(float(head_dim));
    scores_kernel<<<dim3(n, kv_heads, splits), kThreads, 0, s>>>(q, seq, pos, heads, kv_heads, head_dim, slots, layer,
                                                                  scale, splits, sc);
    stats_kernel<<<dim3(n, heads), kThreads, 0, s>>>(pos, heads, splits, sc);
    pv_kernel<<<dim3(n, kv_heads, splits), kThreads, 0, s>>>(seq, pos, heads, kv_heads, head_dim, slots, layer, splits, sc);
    const jfb_q8k q8 = out_q8 != nullptr ? *out_q8 : jfb_q8k{};
    combine_kernel<<<n, 256, 0, s>>>(pos, heads, head_dim, splits, sc, out, q8, out_q8 != nullptr);
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
