// Row-wise kernels that produce the activations the matmuls consume:
// RMSNorm (+weight) and SwiGLU, each optionally fused with the Q8_K
// quantization GGML-CPU applies to the src1 of every K-quant mul_mat.
//
// Q8_K blocks are quantized one per warp (q8k_block_warp): lane l owns the
// eight consecutive values 8l..8l+7 of its block, so the row kernels never
// wait on a block-wide barrier per 256 values. SwiGLU and plain quantization
// spread a row's blocks over many warps and CTAs; RMSNorm keeps one CTA per
// row (the mean needs the whole row) and each of its warps quantizes its own
// blocks straight from registers.
#include "common.cuh"

#include <algorithm>

namespace jfb {
namespace {

constexpr int kThreads = 256;
constexpr int kMaxRowChunks = 32;  // rows up to 8192 values

__device__ __forceinline__ bool aligned16(const void * p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Eight consecutive floats at a 16-byte aligned address, as two vectors.
__device__ __forceinline__ void load8(const float * p, float (&v)[8]) {
    const float4 a = reinterpret_cast<const float4 *>(p)[0], b = reinterpret_cast<const float4 *>(p)[1];
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

// row[col .. col + 8) = v, clipped to the row length; two vectors when the
// whole group is inside a row that starts 16-byte aligned.
__device__ __forceinline__ void store8(float * row, uint32_t col, uint32_t cols, bool vec, const float (&v)[8]) {
    if (vec && col + 8 <= cols) {
        reinterpret_cast<float4 *>(row + col)[0] = make_float4(v[0], v[1], v[2], v[3]);
        reinterpret_cast<float4 *>(row + col)[1] = make_float4(v[4], v[5], v[6], v[7]);
        return;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        if (col + j < cols) row[col + j] = v[j];
    }
}

__device__ __forceinline__ double block_sum_double(double v, double * shared) {
    v = warp_sum(v);
    if ((threadIdx.x & 31) == 0) shared[threadIdx.x >> 5] = v;
    __syncthreads();
    double total = 0.0;
    if (threadIdx.x < 32) {
        total = threadIdx.x < (kThreads / 32) ? shared[threadIdx.x] : 0.0;
        total = warp_sum(total);
        if (threadIdx.x == 0) shared[0] = total;
    }
    __syncthreads();
    total = shared[0];
    __syncthreads();
    return total;
}

// ggml_rms_norm (sum of float squares accumulated in double, mean rounded to
// float, scale = 1/sqrtf(mean + eps), y = x*scale) followed by ggml_mul with
// the norm weight (qwen2_architecture.cpp:373-376). Thread t = 32w + l holds
// elements 256(w + 8c) + 8l .. +8 for c = 0, 1, ..., so warp w's values of
// round c are exactly Q8_K block w + 8c.
__global__ void __launch_bounds__(kThreads) rmsnorm_quant_kernel(
    const float * __restrict__ x, const int32_t * __restrict__ row_index, const float * __restrict__ w,
    uint32_t cols, float eps, float * __restrict__ out_f32, jfb_q8k q8, int quantize) {
    constexpr int kRounds = kMaxRowChunks / 8;  // 2048 values per round
    __shared__ double red[kThreads / 32];
    pdl_trigger();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // the norm weight is written by no earlier kernel: its loads overlap the
    // wait for the previous one
    // whole 8-value groups move as two 16-byte vectors when every row starts
    // 16-byte aligned (aligned buffers, a row length that is a multiple of 4);
    // otherwise, and for ragged tails, element by element. The arithmetic and
    // its order are the same either way.
    const bool vec = (cols & 3u) == 0 && aligned16(x) && aligned16(w) && aligned16(out_f32);
    float wv[kRounds][8];
#pragma unroll
    for (int c = 0; c < kRounds; ++c) {
        const uint32_t base = uint32_t(warp + 8 * c) * kQK + 8 * lane;
        if (vec && base + 8 <= cols) {
            load8(w + base, wv[c]);
        } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) wv[c][j] = base + j < cols ? w[base + j] : 0.0f;
        }
    }
    pdl_wait();
    const uint32_t row = blockIdx.x;
    const uint64_t src_row = row_index != nullptr ? uint64_t(row_index[row]) : uint64_t(row);
    const float * xr = x + src_row * cols;
    float v[kRounds][8];
    double sq = 0.0;
#pragma unroll
    for (int c = 0; c < kRounds; ++c) {
        const uint32_t base = uint32_t(warp + 8 * c) * kQK + 8 * lane;
        if (vec && base + 8 <= cols) {
            load8(xr + base, v[c]);
        } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) v[c][j] = base + j < cols ? xr[base + j] : 0.0f;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            if (base + j < cols) sq += double(__fmul_rn(v[c][j], v[c][j]));
        }
    }
    const double sum = block_sum_double(sq, red);
    const float mean = float(sum / double(cols));
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
#pragma unroll
    for (int c = 0; c < kRounds; ++c) {
        const uint32_t blk = uint32_t(warp + 8 * c);
        if (blk * kQK >= cols) break;  // warp-uniform
        const uint32_t base = blk * kQK + 8 * lane;
        Vals8 y;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            y.v[j] = base + j < cols ? __fmul_rn(__fmul_rn(v[c][j], scale), wv[c][j]) : 0.0f;
        }
        if (out_f32 != nullptr) store8(out_f32 + uint64_t(row) * cols, base, cols, vec, y.v);
        if (quantize) q8k_block_warp(y, q8_dest(q8, row, blk, cols / kQK));
    }
}

// One warp per Q8_K block: grid (ceil(blocks / 8), rows).
// grid (ceil(blocks / 8), min(rows, 65535)); rows beyond the grid's y extent
// are taken in strides of gridDim.y (warp-uniform loop)
__global__ void __launch_bounds__(kThreads) quantize_kernel(const float * __restrict__ x, uint32_t n, uint32_t cols,
                                                         jfb_q8k q8) {
    pdl_trigger();
    pdl_wait();
    const uint32_t blk = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (blk >= cols / kQK) return;  // warp-uniform
    for (uint32_t row = blockIdx.y; row < n; row += gridDim.y) {
        const float4 * src = reinterpret_cast<const float4 *>(x + uint64_t(row) * cols + blk * kQK + 8 * lane);
        const float4 a = src[0], b = src[1];
        const Vals8 y = {{a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w}};
        q8k_block_warp(y, q8_dest(q8, row, blk, cols / kQK));
    }
}

// silu(g) * u with silu(g) = g / (1 + e^-g), each step rounded
// (ggml_swiglu_split / ggml_silu + ggml_mul, qwen2_architecture.cpp:508-520).
__device__ __forceinline__ float swiglu(float g, float u) {
    return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, exp_cw(-g))), u);
}

// One warp per 256 values: grid (ceil(cols / 2048), min(rows, 65535)), rows
// beyond the grid's y extent in strides of gridDim.y. With Q8_K output (cols
// a multiple of 256) each warp quantizes its block; the f32-only form also
// takes rows of any length.
__global__ void __launch_bounds__(kThreads) swiglu_quant_kernel(const float * __restrict__ gate, const float * __restrict__ up,
                                                             uint32_t n, uint32_t cols, float * __restrict__ out_f32,
                                                             jfb_q8k q8, int quantize) {
    pdl_trigger();
    pdl_wait();
    const uint32_t blk = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (blk * kQK >= cols) return;  // warp-uniform
    const uint32_t col = blk * kQK + 8 * lane;
    // two 16-byte vectors per 8 values when every row starts 16-byte aligned
    const bool vec = (cols & 3u) == 0 && aligned16(gate) && aligned16(up) && aligned16(out_f32);
    for (uint32_t row = blockIdx.y; row < n; row += gridDim.y) {
        const uint64_t rbase = uint64_t(row) * cols;
        float g[8], u[8];
        if (vec && col + 8 <= cols) {
            load8(gate + rbase + col, g);
            load8(up + rbase + col, u);
        } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const bool in = col + j < cols;
                g[j] = in ? gate[rbase + col + j] : 0.0f;
                u[j] = in ? up[rbase + col + j] : 0.0f;
            }
        }
        Vals8 y;
#pragma unroll
        for (int j = 0; j < 8; ++j) y.v[j] = col + j < cols ? swiglu(g[j], u[j]) : 0.0f;
        if (out_f32 != nullptr) store8(out_f32 + rbase, col, cols, vec, y.v);
        if (quantize) q8k_block_warp(y, q8_dest(q8, row, blk, cols / kQK));
    }
}

jfb_status check_q8(const jfb_q8k * q8, uint32_t n, uint32_t cols) {
    if (q8 == nullptr) return status_ok();
    if (q8->qs == nullptr || q8->d == nullptr || q8->bsums == nullptr) {
        return status_error(JFB_STATUS_INVALID_ARGUMENT, "Q8_K output planes are required");
    }
    const jfb_status tc = check_q8_tensor_core(q8, n);
    if (tc.code != JFB_STATUS_OK) return tc;
    if (cols % kQK != 0) return status_error(JFB_STATUS_INVALID_ARGUMENT, "Q8_K rows must be a multiple of 256");
    return status_ok();
}

}  // namespace
}  // namespace jfb

using namespace jfb;

extern "C" jfb_status jfb_rmsnorm_quant(const float * x, const int32_t * row_index, const float * norm_weight,
                                        uint32_t n, uint32_t cols, float eps, float * out_f32, const jfb_q8k * out_q8,
                                        void * stream) {
    if (x == nullptr || norm_weight == nullptr || (out_f32 == nullptr && out_q8 == nullptr)) {
        return status_error(JFB_STATUS_INVALID_ARGUMENT, "rmsnorm needs input, weight and an output");
    }
    if (cols == 0 || cols > uint32_t(kMaxRowChunks * kThreads)) {
        return status_error(JFB_STATUS_INVALID_ARGUMENT, "rmsnorm row length %u is outside 1..8192", cols);
    }
    jfb_status s = check_q8(out_q8, n, cols);
    if (s.code != JFB_STATUS_OK) return s;
    if (n == 0) return status_ok();
    const jfb_q8k q8 = out_q8 != nullptr ? *out_q8 : jfb_q8k{};
    const cudaError_t e = launch_k(rmsnorm_quant_kernel, dim3(n), dim3(kThreads), 0, as_stream(stream), x, row_index,
                                   norm_weight, cols, eps, out_f32, q8, out_q8 != nullptr ? 1 : 0);
    if (e != cudaSuccess) return status_error(JFB_STATUS_CUDA_ERROR, "jfb_rmsnorm_quant: %s", cudaGetErrorString(e));
    return launch_status("jfb_rmsnorm_quant");
}

extern "C" jfb_status jfb_quantize_q8k(const float * x, uint32_t n, uint32_t cols, const jfb_q8k * out, void * stream) {
    if (x == nullptr || out == nullptr) return status_error(JFB_STATUS_INVALID_ARGUMENT, "input and output are required");
    jfb_status s = check_q8(out, n, cols);
    if (s.code != JFB_STATUS_OK) return s;
    if (n == 0) return status_ok();
    const cudaError_t e = launch_k(quantize_kernel, dim3((cols / kQK + 7) / 8, std::min(n, 65535u)), dim3(kThreads), 0,
                                   as_stream(stream), x, n, cols, *out);
    if (e != cudaSuccess) return status_error(JFB_STATUS_CUDA_ERROR, "jfb_quantize_q8k: %s", cudaGetErrorString(e));
    return launch_status("jfb_quantize_q8k");
}

extern "C" jfb_status jfb_swiglu_quant(const float * gate, const float * up, uint32_t n, uint32_t cols, float * out_f32,
                                       const jfb_q8k * out_q8, void * stream) {
    if (gate == nullptr || up == nullptr || (out_f32 == nullptr && out_q8 == nullptr)) {
        return status_error(JFB_STATUS_INVALID_ARGUMENT, "swiglu needs gate, up and an output");
    }
    jfb_status s = check_q8(out_q8, n, cols);
    if (s.code != JFB_STATUS_OK) return s;
    if (n == 0 || cols == 0) return status_ok();
    const jfb_q8k q8 = out_q8 != nullptr ? *out_q8 : jfb_q8k{};
    const cudaError_t e = launch_k(swiglu_quant_kernel, dim3((cols + 8 * kQK - 1) / (8 * kQK), std::min(n, 65535u)),
                                   dim3(kThreads), 0, as_stream(stream), gate, up, n, cols, out_f32, q8,
                                   out_q8 != nullptr ? 1 : 0);
    if (e != cudaSuccess) return status_error(JFB_STATUS_CUDA_ERROR, "jfb_swiglu_quant: %s", cudaGetErrorString(e));
    return launch_status("jfb_swiglu_quant");
}
