// Causal GQA attention over the F16 KV cache, split over key chunks, plus the
// combine step (fused with the Q8_K quantization of the result, which the
// O-projection consumes).
//
// Semantics follow the reference graph's unfused path, which is what GGML-CPU
// executes (qwen2_architecture.cpp:425-470): scores = K . q with q rounded to
// f16 and f32 accumulation; x = score * (1/sqrt(head_dim)); keys after the
// query's position are masked out (697-708); softmax in f32; output = P V
// accumulated in f32. One deliberate difference: GGML rounds the normalized
// probabilities to f16 before the V product; this kernel keeps them in f32
// (online softmax across chunks), a relative difference below 2^-11 per
// probability.
//
// Grid: (query row, kv head, key chunk). A CTA owns the G = heads/kv_heads
// query heads that share one kv head, so every K and V row it reads serves G
// heads. Two threads per key compute the scores (half of head_dim each); one
// thread per output dimension accumulates P V.
#include "common.cuh"

namespace jfb {
namespace {

constexpr int kThreads = 128;
constexpr int kChunk = 64;      // keys per CTA
constexpr int kMaxGroup = 16;   // query heads per kv head
constexpr int kMaxHeadDim = 256;

__global__ void __launch_bounds__(kThreads) attention_chunk_kernel(
    const float * __restrict__ q, const int32_t * __restrict__ seq, const int32_t * __restrict__ pos, uint32_t heads,
    uint32_t kv_heads, uint32_t head_dim, const jfb_kv_slot * __restrict__ slots, uint32_t layer, float scale,
    uint32_t max_splits, float * __restrict__ partial) {
    __shared__ float q_s[kMaxGroup * kMaxHeadDim];
    __shared__ float p_s[kMaxGroup][kChunk];
    __shared__ float m_s[kMaxGroup], l_s[kMaxGroup];
    const uint32_t r = blockIdx.x, kvh = blockIdx.y, split = blockIdx.z;
    const int32_t p = pos[r];
    const uint32_t keys = uint32_t(p) + 1u;
    const uint32_t j0 = split * kChunk;
    if (j0 >= keys) return;
    const uint32_t j1 = min(keys, j0 + kChunk);
    const uint32_t G = heads / kv_heads;
    const uint32_t D = head_dim;
    const jfb_kv_slot slot = slots[seq[r]];
    const uint32_t kvd = kv_heads * D;
    const uint16_t * kbase = slot.k + (uint64_t(layer) * slot.capacity) * kvd + kvh * D;
    const uint16_t * vbase = slot.v + (uint64_t(layer) * slot.capacity) * kvd + kvh * D;

    // q rounded to f16 (GGML converts src1 of the F16 mul_mat to F16)
    for (uint32_t i = threadIdx.x; i < G * D; i += kThreads) {
        const uint32_t g = i / D, d = i % D;
        q_s[i] = __half2float(__float2half_rn(q[uint64_t(r) * heads * D + (kvh * G + g) * D + d]));
    }
    __syncthreads();

    // scores: thread pair (2k, 2k+1) handles key j0 + k, each over half of D
    {
        const uint32_t kk = threadIdx.x >> 1, half = threadIdx.x & 1;
        const uint32_t j = j0 + kk;
        float acc[kMaxGroup];
#pragma unroll
        for (int g = 0; g < kMaxGroup; ++g) acc[g] = 0.0f;
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
                                acc[g] = fmaf(k0, q_s[g * D + d + 2 * e], acc[g]);
                                acc[g] = fmaf(k1, q_s[g * D + d + 2 * e + 1], acc[g]);
                            }
                        }
                    }
                }
            } else {
                for (uint32_t d = d_begin; d < d_end; ++d) {
                    const float kv = half_bits_to_float(krow[d]);
#pragma unroll
                    for (int g = 0; g < kMaxGroup; ++g) {
                        if (uint32_t(g) < G) acc[g] = fmaf(kv, q_s[g * D + d], acc[g]);
                    }
                }
            }
        }
#pragma unroll
        for (int g = 0; g < kMaxGroup; ++g) {
            const float total = acc[g] + __shfl_xor_sync(0xffffffffu, acc[g], 1);
            if (uint32_t(g) < G && half == 0 && kk < uint32_t(kChunk)) {
                p_s[g][kk] = j < j1 ? __fmul_rn(total, scale) : -INFINITY;
            }
        }
    }
    __syncthreads();

    // per-head chunk max and exponentials: warp w handles heads w, w+4, ...
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (uint32_t g = warp; g < G; g += kThreads / 32) {
        float mx = -INFINITY;
        for (uint32_t k = lane; k < uint32_t(kChunk); k += 32) mx = fmaxf(mx, p_s[g][k]);
        mx = warp_max(mx);
        float sum = 0.0f;
        for (uint32_t k = lane; k < uint32_t(kChunk); k += 32) {
            const float e = (j0 + k < j1) ? expf(p_s[g][k] - mx) : 0.0f;
            p_s[g][k] = e;
            sum += e;
        }
        sum = warp_sum(sum);
        if (lane == 0) {
            m_s[g] = mx;
            l_s[g] = sum;
        }
    }
    __syncthreads();

    // P V: thread d (and d + 128 for head_dim 256)
    const uint64_t part_row = (uint64_t(r) * heads + kvh * G) * max_splits;  // head (kvh*G + g) at + g*max_splits
    for (uint32_t d = threadIdx.x; d < D; d += kThreads) {
        float acc[kMaxGroup];
#pragma unroll
        for (int g = 0; g < kMaxGroup; ++g) acc[g] = 0.0f;
        for (uint32_t j = j0; j < j1; ++j) {
            const float vv = half_bits_to_float(vbase[uint64_t(j) * kvd + d]);
#pragma unroll
            for (int g = 0; g < kMaxGroup; ++g) {
                if (uint32_t(g) < G) acc[g] = fmaf(p_s[g][j - j0], vv, acc[g]);
            }
        }
#pragma unroll
        for (int g = 0; g < kMaxGroup; ++g) {
            if (uint32_t(g) < G) {
                float * rec = partial + ((part_row + uint64_t(g) * max_splits + split) * (D + 2));
                rec[2 + d] = acc[g];
            }
        }
    }
    if (threadIdx.x < G) {
        float * rec = partial + ((part_row + uint64_t(threadIdx.x) * max_splits + split) * (D + 2));
        rec[0] = m_s[threadIdx.x];
        rec[1] = l_s[threadIdx.x];
    }
}

// Merges the chunk partials of one query row, writes out[r][heads*D] and
// optionally its Q8_K quantization (then heads*D % 256 == 0).
__global__ void __launch_bounds__(256) attention_combine_kernel(const int32_t * __restrict__ pos, uint32_t heads,
                                                              uint32_t head_dim, uint32_t max_splits,
                                                              const float * __restrict__ partial,
                                                              float * __restrict__ out, jfb_q8k q8, int quantize) {
    __shared__ unsigned long long keys[8];
    const uint32_t r = blockIdx.x;
    const uint32_t D = head_dim, width = heads * D;
    const uint32_t splits = (uint32_t(pos[r]) + kChunk) / kChunk;  // ceil((pos + 1) / chunk)
    for (uint32_t i = threadIdx.x; i < width; i += blockDim.x) {
        const uint32_t h = i / D, d = i % D;
        const float * base = partial + (uint64_t(r) * heads + h) * max_splits * (D + 2);
        float M = -INFINITY;
        for (uint32_t c = 0; c < splits; ++c) M = fmaxf(M, base[c * (D + 2)]);
        float L = 0.0f, O = 0.0f;
        for (uint32_t c = 0; c < splits; ++c) {
            const float w = expf(base[c * (D + 2)] - M);
            L = fmaf(w, base[c * (D + 2) + 1], L);
            O = fmaf(w, base[c * (D + 2) + 2 + d], O);
        }
        out[uint64_t(r) * width + i] = __fdiv_rn(O, L);
    }
    if (!quantize) return;
    __syncthreads();
    for (uint32_t c = 0; c < width / kQK; ++c) {
        const float y = out[uint64_t(r) * width + c * kQK + threadIdx.x];
        const uint64_t block = uint64_t(r) * (width / kQK) + c;
        q8k_block_256(y, q8.qs + block * kQK, q8.d + block, q8.bsums + block * 16, keys);
    }
}

}  // namespace
}  // namespace jfb

using namespace jfb;

extern "C" uint64_t jfb_attention_scratch_bytes(uint32_t n, uint32_t heads, uint32_t head_dim, uint32_t max_keys) {
    const uint64_t splits = (uint64_t(max_keys) + kChunk - 1) / kChunk;
    return uint64_t(n) * heads * splits * (uint64_t(head_dim) + 2) * sizeof(float);
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
    if (scratch_bytes < jfb_attention_scratch_bytes(n, heads, head_dim, max_keys)) {
        return status_error(JFB_STATUS_INVALID_ARGUMENT, "attention scratch is too small");
    }
    if (n == 0) return status_ok();
    const uint32_t splits = (max_keys + kChunk - 1) / kChunk;
    if (splits > 65535u || kv_heads > 65535u) return status_error(JFB_STATUS_INVALID_ARGUMENT, "attention grid too large");
    cudaStream_t s = as_stream(stream);
    const float scale = 1.0f / sqrtf(float(head_dim));
    attention_chunk_kernel<<<dim3(n, kv_heads, splits), kThreads, 0, s>>>(q, seq, pos, heads, kv_heads, head_dim, slots,
                                                                          layer, scale, splits,
                                                                          static_cast<float *>(scratch));
    jfb_status st = launch_status("jfb_attention(chunks)");
    if (st.code != JFB_STATUS_OK) return st;
    const jfb_q8k q8 = out_q8 != nullptr ? *out_q8 : jfb_q8k{nullptr, nullptr, nullptr};
    attention_combine_kernel<<<n, 256, 0, s>>>(pos, heads, head_dim, splits, static_cast<const float *>(scratch), out,
                                               q8, out_q8 != nullptr);
    return launch_status("jfb_attention(combine)");
}
