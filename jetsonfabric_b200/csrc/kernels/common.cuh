// Shared helpers of the sm_100a kernel library: status construction, launch
// checks and the small device-side building blocks (binary16 conversion,
// Q8_K quantization of one 256-value block, block reductions).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <utility>

#include "jetsonfabric/engine.h"
#include "jfb/jfb_kernels.h"

namespace jfb {

constexpr int kQK = 256;  // K-quant / Q8_K super-block length

inline jfb_status status_ok() {
    jfb_status s;
    s.code = JFB_STATUS_OK;
    s.message[0] = '\0';
    return s;
}

inline jfb_status status_error(jfb_status_code code, const char * format, ...) {
    jfb_status s;
    s.code = code;
    va_list args;
    va_start(args, format);
    std::vsnprintf(s.message, sizeof(s.message), format, args);
    va_end(args);
    return s;
}

inline jfb_status launch_status(const char * what) {
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return status_error(JFB_STATUS_CUDA_ERROR, "%s: %s", what, cudaGetErrorString(e));
    return status_ok();
}

inline cudaStream_t as_stream(void * s) { return static_cast<cudaStream_t>(s); }

// The tensor-core operands of a Q8_K buffer: all three planes or none,
// 16-byte aligned, d_t wide enough for `rows` rows.
inline jfb_status check_q8_tensor_core(const jfb_q8k * q8, uint32_t rows) {
    const int present = (q8->qs_f16 != nullptr) + (q8->bsums_f16 != nullptr) + (q8->d_t != nullptr);
    if (present == 0) return status_ok();
    if (present != 3) {
        return status_error(JFB_STATUS_INVALID_ARGUMENT, "Q8_K tensor-core planes must be given all together");
    }
    if ((reinterpret_cast<uintptr_t>(q8->qs_f16) & 15u) != 0 || (reinterpret_cast<uintptr_t>(q8->bsums_f16) & 15u) != 0 ||
        (reinterpret_cast<uintptr_t>(q8->d_t) & 15u) != 0) {
        return status_error(JFB_STATUS_INVALID_ARGUMENT, "Q8_K tensor-core planes must be 16-byte aligned");
    }
    if (q8->d_stride % 4 != 0 || q8->d_stride < rows) {
        return status_error(JFB_STATUS_INVALID_ARGUMENT, "Q8_K d_stride %u must be a multiple of 4 and >= %u rows",
                            q8->d_stride, rows);
    }
    return status_ok();
}

// ---- programmatic dependent launch ---------------------------------------------
//
// The kernels of the per-step path are launched with programmatic stream
// serialization (off with JFB_PDL=0): a kernel may start while its predecessor
// in the stream drains, runs its prologue (barriers, tensor memory, weight
// loads, per-call metadata), and calls pdl_wait() before it touches anything
// an earlier kernel writes. Every such kernel also calls pdl_trigger() on
// entry, which lets the next kernel start as soon as all of its CTAs run.
// Without the launch attribute both instructions return at once.
inline bool pdl_enabled() {
    static const bool on = [] {
        const char * e = std::getenv("JFB_PDL");
        return e == nullptr || e[0] != '0';
    }();
    return on;
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                            Args &&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    if (pdl_enabled()) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

inline bool is_kquant(uint32_t type) {
    return type == JF_TENSOR_Q4_K || type == JF_TENSOR_Q6_K || type == JF_TENSOR_Q2_K;
}

// ---- device helpers --------------------------------------------------------

// Wait until the kernels before this one in the stream have completed and
// their writes are visible (programmatic dependent launch).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Allow the next kernel in the stream to start launching.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ float half_bits_to_float(uint16_t h) {
    return __half2float(__ushort_as_half(h));
}

__device__ __forceinline__ uint16_t float_to_half_bits(float f) {
    return __half_as_ushort(__float2half_rn(f));
}

// exp(x) by Cody-Waite argument reduction (x = n ln2 + r with ln2 split into
// a short high part and a correction) and the degree-7 Taylor polynomial of
// e^r evaluated in Horner form with fused multiply-adds, then an exact
// two-step scaling by 2^n (max error below 1 ulp over the normal range). Every
// step is a correctly rounded IEEE operation, so the CPU oracle's
// implementation of the same method gives identical bits.
__device__ __forceinline__ float pow2i(int e) { return __uint_as_float(static_cast<unsigned>(e + 127) << 23); }

__device__ __forceinline__ float exp_cw(float x) {
    if (x != x) return x;
    if (x > 88.72283935546875f) return __int_as_float(0x7f800000);
    if (x < -103.972084045410156f) return 0.0f;
    const float n = rintf(__fmul_rn(x, 1.44269502162933349609375f));
    float r = fmaf(-n, 0.693145751953125f, x);
    r = fmaf(-n, 1.4286068203094172e-06f, r);
    float p = 1.98412701138295233e-04f;
    p = fmaf(p, r, 1.38888892251998186e-03f);
    p = fmaf(p, r, 8.33333376795053482e-03f);
    p = fmaf(p, r, 4.16666679084300995e-02f);
    p = fmaf(p, r, 1.66666671633720398e-01f);
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    const int e = static_cast<int>(n);
    const int e1 = e / 2, e2 = e - e1;
    return __fmul_rn(__fmul_rn(p, pow2i(e1)), pow2i(e2));
}

// Warp-wide sum.
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// (|value| max, first index on ties) reduction key packed for a shuffle: the
// magnitude's bits (non-negative floats order like their bit patterns) in the
// high word and the complement of the index in the low word, so a plain
// unsigned max picks the largest magnitude and, among equals, the smallest
// index.
__device__ __forceinline__ unsigned long long amax_key(float magnitude, int index) {
    return (static_cast<unsigned long long>(__float_as_uint(magnitude)) << 32) |
           static_cast<unsigned long long>(0xffffffffu - static_cast<unsigned>(index));
}

__device__ __forceinline__ unsigned long long warp_max_u64(unsigned long long v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, v, o);
        v = other > v ? other : v;
    }
    return v;
}

// Quantizes one 256-value block held one value per thread by a 256-thread
// block (thread t holds element t) with GGML's quantize_row_q8_K rule:
// max = signed value of largest magnitude (first on ties), iscale = -127/max,
// q = round-half-even(iscale * x) capped at 127, d = 1/iscale, bsums over 16.
// `shared` must hold 8 unsigned long long + 16 int. Every thread of the block
// must call it.
// Where one Q8_K block of a jfb_q8k goes: row r, block b of nb per row.
struct Q8Dest {
    int8_t * qs;
    float * d;
    int16_t * bsums;
    uint16_t * qs_f16;     // nullptr when the tensor-core operands are not kept
    uint16_t * bsums_f16;
    float * d_t;
};

__device__ __forceinline__ Q8Dest q8_dest(const jfb_q8k & q8, uint64_t r, uint32_t b, uint32_t nb) {
    const uint64_t block = r * nb + b;
    Q8Dest o;
    o.qs = q8.qs + block * kQK;
    o.d = q8.d + block;
    o.bsums = q8.bsums + block * 16;
    const bool tc = q8.qs_f16 != nullptr;
    o.qs_f16 = tc ? q8.qs_f16 + block * kQK : nullptr;
    o.bsums_f16 = tc ? q8.bsums_f16 + block * 16 : nullptr;
    o.d_t = tc ? q8.d_t + uint64_t(b) * q8.d_stride + r : nullptr;
    return o;
}

// f16 bits of a small integer (|v| < 2048: exact).
__device__ __forceinline__ uint16_t int_to_half_bits(int v) { return __half_as_ushort(__int2half_rn(v)); }

__device__ __forceinline__ void q8k_block_256(float x, const Q8Dest & dst, unsigned long long * shared_keys) {
    int8_t * qs = dst.qs;
    float * d = dst.d;
    int16_t * bsums = dst.bsums;
    const int t = threadIdx.x;
    unsigned long long key = warp_max_u64(amax_key(fabsf(x), t));
    if ((t & 31) == 0) shared_keys[t >> 5] = key;
    __syncthreads();
    if (t < 32) {
        unsigned long long k2 = t < 8 ? shared_keys[t] : 0ull;
        k2 = warp_max_u64(k2);
        if (t == 0) shared_keys[0] = k2;
    }
    __syncthreads();
    const unsigned long long best = shared_keys[0];
    const float amax = __uint_as_float(static_cast<unsigned>(best >> 32));
    int q = 0;
    float dval = 0.0f;
    // All threads read the winner's value by broadcast through a shuffle-free
    // path: the winner writes it.
    __shared__ float winner_value;
    const int winner = static_cast<int>(0xffffffffu - static_cast<unsigned>(best & 0xffffffffull));
    if (t == winner) winner_value = x;
    __syncthreads();
    if (amax != 0.0f) {
        const float mx = winner_value;
        const float iscale = __fdiv_rn(-127.0f, mx);
        const int v = __float2int_rn(__fmul_rn(iscale, x));
        q = v < 127 ? v : 127;
        dval = __fdiv_rn(1.0f, iscale);
    }
    qs[t] = static_cast<int8_t>(q);
    if (dst.qs_f16 != nullptr) dst.qs_f16[t] = int_to_half_bits(q);
    // bsums: 16 consecutive values -> half-warp segments
    int s = q;
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if ((t & 15) == 0) {
        bsums[t >> 4] = static_cast<int16_t>(s);
        if (dst.bsums_f16 != nullptr) dst.bsums_f16[t >> 4] = int_to_half_bits(s);
    }
    if (t == 0) {
        *d = dval;
        if (dst.d_t != nullptr) *dst.d_t = dval;
    }
    __syncthreads();  // shared_keys / winner_value reuse safety
}

// The same Q8_K quantization of one 256-value block by one warp: lane l holds
// elements 8l..8l+7 in v[]. Identical arithmetic to q8k_block_256 (the amax
// key picks the signed value of largest magnitude, first on ties), with
// shuffles only, so any number of warps of a CTA quantize blocks
// independently. qs must be 8-byte aligned and qs_f16 16-byte aligned.
struct Vals8 {
    float v[8];
};

__device__ __forceinline__ void q8k_block_warp(const Vals8 vals, const Q8Dest & dst) {
    int8_t * qs = dst.qs;
    float * d = dst.d;
    int16_t * bsums = dst.bsums;
    const int lane = threadIdx.x & 31;
    unsigned long long key = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const unsigned long long k = amax_key(fabsf(vals.v[j]), 8 * lane + j);
        key = k > key ? k : key;
    }
    key = warp_max_u64(key);
    const float amax = __uint_as_float(static_cast<unsigned>(key >> 32));
    const int winner = static_cast<int>(0xffffffffu - static_cast<unsigned>(key & 0xffffffffull));
    float mine = vals.v[0];
#pragma unroll
    for (int j = 1; j < 8; ++j) mine = (winner & 7) == j ? vals.v[j] : mine;
    const float mx = __shfl_sync(0xffffffffu, mine, winner >> 3);
    int q[8];
    float dval = 0.0f;
    if (amax != 0.0f) {
        const float iscale = __fdiv_rn(-127.0f, mx);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int t = __float2int_rn(__fmul_rn(iscale, vals.v[j]));
            q[j] = t < 127 ? t : 127;
        }
        dval = __fdiv_rn(1.0f, iscale);
    } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) q[j] = 0;
    }
    uint32_t lo = 0, hi = 0;
    int s = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        lo |= (static_cast<uint32_t>(q[j]) & 0xffu) << (8 * j);
        hi |= (static_cast<uint32_t>(q[j + 4]) & 0xffu) << (8 * j);
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) s += q[j];
    *reinterpret_cast<uint2 *>(qs + 8 * lane) = make_uint2(lo, hi);
    if (dst.qs_f16 != nullptr) {
        uint32_t h[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            h[j] = uint32_t(int_to_half_bits(q[2 * j])) | (uint32_t(int_to_half_bits(q[2 * j + 1])) << 16);
        }
        *reinterpret_cast<uint4 *>(dst.qs_f16 + 8 * lane) = make_uint4(h[0], h[1], h[2], h[3]);
    }
    s += __shfl_xor_sync(0xffffffffu, s, 1);  // 16-value group = lanes 2g, 2g + 1
    if ((lane & 1) == 0) {
        bsums[lane >> 1] = static_cast<int16_t>(s);
        if (dst.bsums_f16 != nullptr) dst.bsums_f16[lane >> 1] = int_to_half_bits(s);
    }
    if (lane == 0) {
        *d = dval;
        if (dst.d_t != nullptr) *dst.d_t = dval;
    }
}

}  // namespace jfb
