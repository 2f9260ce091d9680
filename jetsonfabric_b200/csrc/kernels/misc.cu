// Output-side kernels: greedy argmax over the logits and the F16 activation
// codec used for stage-to-stage handoff.
#include "common.cuh"

namespace jfb {
namespace {

// ggml_argmax (qwen2_architecture.cpp:594): first index of the maximum,
// comparisons with `>` so NaNs never win.
__device__ __forceinline__ void better(float & v, int & i, float ov, int oi) {
    if (ov > v || (ov == v && oi < i)) {
        v = ov;
        i = oi;
    }
}

__global__ void __launch_bounds__(1024) argmax_kernel(const float * __restrict__ x, uint32_t cols, int32_t * out) {
    __shared__ float sv[32];
    __shared__ int si[32];
    pdl_trigger();
    pdl_wait();
    const float * row = x + uint64_t(blockIdx.x) * cols;
    float v = -INFINITY;
    int idx = 0x7fffffff;
    // eight loads in flight per thread; each thread visits its indices in
    // increasing order, so `>` keeps the first index of its maximum
    constexpr uint32_t kUnroll = 8;
    uint32_t c = threadIdx.x;
    for (; c + (kUnroll - 1) * blockDim.x < cols; c += kUnroll * blockDim.x) {
        float e[kUnroll];
#pragma unroll
        for (uint32_t u = 0; u < kUnroll; ++u) e[u] = __ldg(row + c + u * blockDim.x);
#pragma unroll
        for (uint32_t u = 0; u < kUnroll; ++u) {
            if (e[u] > v) {
                v = e[u];
                idx = int(c + u * blockDim.x);
            }
        }
    }
    for (; c < cols; c += blockDim.x) {
        const float e = row[c];
        if (e > v) {
            v = e;
            idx = int(c);
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) better(v, idx, __shfl_xor_sync(0xffffffffu, v, o), __shfl_xor_sync(0xffffffffu, idx, o));
    if ((threadIdx.x & 31) == 0) {
        sv[threadIdx.x >> 5] = v;
        si[threadIdx.x >> 5] = idx;
    }
    __syncthreads();
    if (threadIdx.x < 32) {
        const int warps = int(blockDim.x >> 5);
        v = int(threadIdx.x) < warps ? sv[threadIdx.x] : -INFINITY;
        idx = int(threadIdx.x) < warps ? si[threadIdx.x] : 0x7fffffff;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) better(v, idx, __shfl_xor_sync(0xffffffffu, v, o), __shfl_xor_sync(0xffffffffu, idx, o));
        if (threadIdx.x == 0) out[blockIdx.x] = idx == 0x7fffffff ? 0 : idx;
    }
}

// The reference F16 activation codec (builtin_activation_codecs.cpp:51-106),
// in integer arithmetic so NaN payloads survive exactly.
__device__ __forceinline__ uint16_t codec_float_to_half(float value) {
    const uint32_t bits = __float_as_uint(value);
    const uint16_t sign = uint16_t((bits >> 16) & 0x8000u);
    const uint32_t exponent = (bits >> 23) & 0xffu;
    uint32_t mantissa = bits & 0x7fffffu;
    if (exponent == 0xffu) {
        if (mantissa == 0) return uint16_t(sign | 0x7c00u);
        return uint16_t(sign | 0x7c00u | (mantissa >> 13) | 0x0200u);
    }
    int he = int(exponent) - 127 + 15;
    if (he >= 31) return uint16_t(sign | 0x7c00u);
    if (he <= 0) {
        if (he < -10) return sign;
        mantissa |= 0x800000u;
        const unsigned shift = unsigned(14 - he);
        uint32_t hm = mantissa >> shift;
        const uint32_t rem = mantissa & ((1u << shift) - 1u), halfway = 1u << (shift - 1u);
        if (rem > halfway || (rem == halfway && (hm & 1u))) ++hm;
        return uint16_t(sign | hm);
    }
    uint32_t hm = mantissa >> 13;
    const uint32_t rem = mantissa & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (hm & 1u))) {
        ++hm;
        if (hm == 0x400u) {
            hm = 0;
            ++he;
            if (he >= 31) return uint16_t(sign | 0x7c00u);
        }
    }
    return uint16_t(sign | (uint32_t(he) << 10) | hm);
}

// builtin_activation_codecs.cpp:108-137: exact widening, NaN payload kept.
__device__ __forceinline__ float codec_half_to_float(uint16_t value) {
    const uint32_t sign = uint32_t(value & 0x8000u) << 16;
    const uint32_t exponent = (value >> 10) & 0x1fu;
    uint32_t mantissa = value & 0x03ffu;
    uint32_t bits;
    if (exponent == 0) {
        if (mantissa == 0) {
            bits = sign;
        } else {
            int e = -14;
            while ((mantissa & 0x0400u) == 0) {
                mantissa <<= 1;
                --e;
            }
            bits = sign | (uint32_t(e + 127) << 23) | ((mantissa & 0x3ffu) << 13);
        }
    } else if (exponent == 0x1fu) {
        bits = sign | 0x7f800000u | (mantissa << 13);
    } else {
        bits = sign | ((exponent + 112u) << 23) | (mantissa << 13);
    }
    return __uint_as_float(bits);
}

__global__ void encode_kernel(const float * __restrict__ in, uint16_t * __restrict__ out, uint64_t count) {
    pdl_trigger();
    pdl_wait();
    for (uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < count; i += uint64_t(gridDim.x) * blockDim.x) {
        out[i] = codec_float_to_half(in[i]);
    }
}

__global__ void decode_kernel(const uint16_t * __restrict__ in, float * __restrict__ out, uint64_t count) {
    pdl_trigger();
    pdl_wait();
    for (uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < count; i += uint64_t(gridDim.x) * blockDim.x) {
        out[i] = codec_half_to_float(in[i]);
    }
}

unsigned grid_for(uint64_t count) {
    const uint64_t g = (count + 255) / 256;
    return unsigned(g < 148u * 32u ? (g == 0 ? 1 : g) : 148u * 32u);
}

}  // namespace
}  // namespace jfb

using namespace jfb;

extern "C" jfb_status jfb_argmax(const float * logits, uint32_t n, uint32_t cols, int32_t * out, void * stream) {
    if (logits == nullptr || out == nullptr || cols == 0) return status_error(JFB_STATUS_INVALID_ARGUMENT, "argmax operands are required");
    if (n == 0) return status_ok();
    const cudaError_t e = launch_k(argmax_kernel, dim3(n), dim3(1024), 0, as_stream(stream), logits, cols, out);
    if (e != cudaSuccess) return status_error(JFB_STATUS_CUDA_ERROR, "jfb_argmax: %s", cudaGetErrorString(e));
    return launch_status("jfb_argmax");
}

extern "C" jfb_status jfb_codec_f32_to_f16(const float * in, uint16_t * out, uint64_t count, void * stream) {
    if (count == 0) return status_ok();
    if (in == nullptr || out == nullptr) return status_error(JFB_STATUS_INVALID_ARGUMENT, "codec buffers are required");
    const cudaError_t e = launch_k(encode_kernel, dim3(grid_for(count)), dim3(256), 0, as_stream(stream), in, out, count);
    if (e != cudaSuccess) return status_error(JFB_STATUS_CUDA_ERROR, "jfb_codec_f32_to_f16: %s", cudaGetErrorString(e));
    return launch_status("jfb_codec_f32_to_f16");
}

extern "C" jfb_status jfb_codec_f16_to_f32(const uint16_t * in, float * out, uint64_t count, void * stream) {
    if (count == 0) return status_ok();
    if (in == nullptr || out == nullptr) return status_error(JFB_STATUS_INVALID_ARGUMENT, "codec buffers are required");
    const cudaError_t e = launch_k(decode_kernel, dim3(grid_for(count)), dim3(256), 0, as_stream(stream), in, out, count);
    if (e != cudaSuccess) return status_error(JFB_STATUS_CUDA_ERROR, "jfb_codec_f16_to_f32: %s", cudaGetErrorString(e));
    return launch_status("jfb_codec_f16_to_f32");
}
