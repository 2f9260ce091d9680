// Row-wise kernels that produce the activations the matmuls consume:
// RMSNorm (+weight) and SwiGLU, each optionally fused with the Q8_K
// quantization GGML-CPU applies to the src1 of every K-quant mul_mat.
//
// One 256-thread CTA per row; for rows whose length is a multiple of 256 the
// row is walked one 256-value Q8_K block at a time with thread t owning
// element t of the block, so the quantizer needs no data exchange beyond the
// block reductions.
#include "common.cuh"

namespace jfb {
namespace {

constexpr int kThreads = 256;
constexpr int kMaxRowChunks = 32;  // rows up to 8192 values

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
// the norm weight (qwen2_architecture.cpp:373-376).
__global__ void __launch_bounds__(kThreads) rmsnorm_quant_kernel(
    const float * __restrict__ x, const int32_t * __restrict__ row_index, const float * __restrict__ w,
    uint32_t cols, float eps, float * __restrict__ out_f32, jfb_q8k q8, int quantize) {
    __shared__ double red[kThreads / 32];
    __shared__ unsigned long long keys[8];
    const uint32_t row = blockIdx.x;
    const uint64_t src_row = row_index != nullptr ? uint64_t(row_index[row]) : uint64_t(row);
    const float * xr = x + src_row * cols;
    float v[kMaxRowChunks];
    double sq = 0.0;
#pragma unroll
    for (int c = 0; c < kMaxRowChunks; ++c) {
        const uint32_t i = uint32_t(c) * kThreads + threadIdx.x;
        v[c] = i < cols ? xr[i] : 0.0f;
        if (i < cols) sq += double(__fmul_rn(v[c], v[c]));
    }
    const double sum = block_sum_double(sq, red);
    const float mean = float(sum / double(cols));
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
#pragma unroll
    for (int c = 0; c < kMaxRowChunks; ++c) {
        const uint32_t i = uint32_t(c) * kThreads + threadIdx.x;
        if (uint32_t(c) * kThreads >= cols) break;
        const float y = i < cols ? __fmul_rn(__fmul_rn(v[c], scale), w[i]) : 0.0f;
        if (out_f32 != nullptr && i < cols) out_f32[uint64_t(row) * cols + i] = y;
        if (quantize) {
            const uint64_t block = uint64_t(row) * (cols / kQK) + c;
            q8k_block_256(y, q8.qs + block * kQK, q8.d + block, q8.bsums + block * 16, keys);
        }
    }
}

__global__ void __launch_bounds__(kThreads) quantize_kernel(const float * __restrict__ x, uint32_t cols, jfb_q8k q8) {
    __shared__ unsigned long long keys[8];
    const uint32_t row = blockIdx.x;
    for (uint32_t c = 0; c < cols / kQK; ++c) {
        const float y = x[uint64_t(row) * cols + c * kQK + threadIdx.x];
        const uint64_t block = uint64_t(row) * (cols / kQK) + c;
        q8k_block_256(y, q8.qs + block * kQK, q8.d + block, q8.bsums + block * 16, keys);
    }
}

// silu(g) * u with silu(g) = g / (1 + e^-g), each step rounded
// (ggml_swiglu_split / ggml_silu + ggml_mul, qwen2_architecture.cpp:508-520).
__device__ __forceinline__ float swiglu(float g, float u) {
    return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, exp_cw(-g))), u);
}

__global__ void __launch_bounds__(kThreads) swiglu_quant_kernel(const float * __restrict__ gate, const float * __restrict__ up,
                                                             uint32_t cols, float * __restrict__ out_f32, jfb_q8k q8,
                                                             int quantize) {
    __shared__ unsigned long long keys[8];
    const uint32_t row = blockIdx.x;
    const uint32_t chunks = (cols + kThreads - 1) / kThreads;
    for (uint32_t c = 0; c < chunks; ++c) {
        const uint32_t i = c * kThreads + threadIdx.x;
        const uint64_t at = uint64_t(row) * cols + i;
        const float y = i < cols ? swiglu(gate[at], up[at]) : 0.0f;
        if (out_f32 != nullptr && i < cols) out_f32[at] = y;
        if (quantize) {
            const uint64_t block = uint64_t(row) * (cols / kQK) + c;
            q8k_block_256(y, q8.qs + block * kQK, q8.d + block, q8.bsums + block * 16, keys);
        }
    }
}

jfb_status check_q8(const jfb_q8k * q8, uint32_t cols) {
    if (q8 == nullptr) return status_ok();
    if (q8->qs == nullptr || q8->d == nullptr || q8->bsums == nullptr) {
        return status_error(JFB_STATUS_INVALID_ARGUMENT, "Q8_K output planes are required");
    }
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
    jfb_status s = check_q8(out_q8, cols);
    if (s.code != JFB_STATUS_OK) return s;
    if (n == 0) return status_ok();
    const jfb_q8k q8 = out_q8 != nullptr ? *out_q8 : jfb_q8k{nullptr, nullptr, nullptr};
    rmsnorm_quant_kernel<<<n, kThreads, 0, as_stream(stream)>>>(x, row_index, norm_weight, cols, eps, out_f32, q8,
                                                                 out_q8 != nullptr);
    return launch_status("jfb_rmsnorm_quant");
}

extern "C" jfb_status jfb_quantize_q8k(const float * x, uint32_t n, uint32_t cols, const jfb_q8k * out, void * stream) {
    if (x == nullptr || out == nullptr) return status_error(JFB_STATUS_INVALID_ARGUMENT, "input and output are required");
    jfb_status s = check_q8(out, cols);
    if (s.code != JFB_STATUS_OK) return s;
    if (n == 0) return status_ok();
    quantize_kernel<<<n, kThreads, 0, as_stream(stream)>>>(x, cols, *out);
    return launch_status("jfb_quantize_q8k");
}

extern "C" jfb_status jfb_swiglu_quant(const float * gate, const float * up, uint32_t n, uint32_t cols, float * out_f32,
                                       const jfb_q8k * out_q8, void * stream) {
    if (gate == nullptr || up == nullptr || (out_f32 == nullptr && out_q8 == nullptr)) {
        return status_error(JFB_STATUS_INVALID_ARGUMENT, "swiglu needs gate, up and an output");
    }
    jfb_status s = check_q8(out_q8, cols);
    if (s.code != JFB_STATUS_OK) return s;
    if (n == 0 || cols == 0) return status_ok();
    const jfb_q8k q8 = out_q8 != nullptr ? *out_q8 : jfb_q8k{nullptr, nullptr, nullptr};
    swiglu_quant_kernel<<<n, kThreads, 0, as_stream(stream)>>>(gate, up, cols, out_f32, q8, out_q8 != nullptr);
    return launch_status("jfb_swiglu_quant");
}
