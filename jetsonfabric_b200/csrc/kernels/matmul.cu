// ggml_mul_mat replacement for K-quant and float weights (CUDA cores).
//
// K-quant x Q8_K: GGML-CPU's vec_dot_{q2_K,q4_K,q6_K}_q8_K computes, per
// 256-value block, exact integer dot products of the weight codes with the
// Q8_K activation bytes inside each 16- or 32-value sub-block, multiplies them
// by the integer sub-block scales, and applies one float scale per block:
//     c_b = (d_w * d_a) * isum - (dmin_w * d_a) * msum
// This kernel computes the same integers with dp4a and each c_b with the same
// rounded float operations; the c_b of a row are summed in double and
// rounded to float once, which makes the result independent of the order in
// which lanes add blocks, so it equals the CPU oracle bit for bit.
//
// Work split: one warp per weight row, four lanes per 256-block (each lane
// owns 64 values: 32 bytes of Q4_K codes, 64 bytes of Q6_K ql/qh, or the
// 32 Q2_K code bytes it shares with its neighbour), eight consecutive blocks
// per warp step so a warp reads 1-1.5 KB of contiguous codes per step.
// Activation rows are processed eight at a time (blockIdx.y); the weight
// re-reads of further groups hit L2.
#include "common.cuh"

namespace jfb {
namespace {

constexpr int kWarps = 4;       // rows per CTA
constexpr int kGroup = 8;       // activation rows per CTA

struct Epilogue {
    uint32_t kind;
    const float * bias;
    const float * residual;
};

__device__ __forceinline__ void store_out(float v, uint32_t row, uint32_t t, uint32_t rows, float * out,
                                          const Epilogue & ep) {
    const uint64_t at = uint64_t(t) * rows + row;
    if (ep.kind == JFB_EPILOGUE_BIAS) v = __fadd_rn(v, ep.bias[row]);
    else if (ep.kind == JFB_EPILOGUE_RESIDUAL) v = __fadd_rn(v, ep.residual[at]);
    out[at] = v;
}

__device__ __forceinline__ int dp4a(int a, int b, int c) { return __dp4a(a, b, c); }

__device__ __forceinline__ uint32_t byte_of(const uint4 & v, int i) {
    const uint32_t w = i < 4 ? v.x : i < 8 ? v.y : i < 12 ? v.z : v.w;
    return (w >> (8 * (i & 3))) & 0xffu;
}

// Q4_K 6-bit (scale, min) of sub-block j from the 12 packed bytes that follow
// d and dmin in the 16-byte header.
__device__ __forceinline__ void q4k_scale_min(const uint4 & hdr, int j, int & sc, int & m) {
    // header bytes: 0-1 d, 2-3 dmin, 4..15 scales[0..11]
    auto s = [&](int k) { return int(byte_of(hdr, 4 + k)); };
    if (j < 4) {
        sc = s(j) & 63;
        m = s(j + 4) & 63;
    } else {
        sc = (s(j + 4) & 0x0f) | ((s(j - 4) >> 6) << 4);
        m = (s(j + 4) >> 4) | ((s(j) >> 6) << 4);
    }
}

__device__ __forceinline__ uint4 ldg16(const void * p) { return __ldg(static_cast<const uint4 *>(p)); }

struct ActView {
    const int8_t * qs;
    const float * d;
    const int16_t * bsums;
    uint32_t cols;
};

// Sums an integer over the four lanes that share one 256-block (lanes 4k..4k+3).
__device__ __forceinline__ int block_lanes_sum(int v) {
    v += __shfl_xor_sync(0xffffffffu, v, 1);
    v += __shfl_xor_sync(0xffffffffu, v, 2);
    return v;
}

// The weight bytes one lane reads for one 256-block (its 64 values plus the
// block's scales), loaded one warp step ahead of their use so that a warp
// keeps two steps of weight loads in flight.
struct WRegs {
    uint4 a, b, c, d, e;
    uint32_t x;
};

template <uint32_t TYPE>
__device__ __forceinline__ WRegs load_weights(const jfb_weight & w, uint64_t block, int c, bool valid) {
    const uint8_t * p0 = static_cast<const uint8_t *>(w.plane[0]);
    const uint8_t * p1 = static_cast<const uint8_t *>(w.plane[1]);
    const uint8_t * p2 = static_cast<const uint8_t *>(w.plane[2]);
    const uint4 zero = make_uint4(0, 0, 0, 0);
    WRegs r{zero, zero, zero, zero, zero, 0u};
    if (!valid) return r;
    if constexpr (TYPE == JF_TENSOR_Q4_K) {
        r.a = ldg16(p0 + block * 128 + 32 * c);
        r.b = ldg16(p0 + block * 128 + 32 * c + 16);
        r.c = ldg16(p1 + block * 16);
    } else if constexpr (TYPE == JF_TENSOR_Q6_K) {
        const int h = c >> 1, part = c & 1;
        const uint8_t * blk = p0 + block * 192;
        r.a = ldg16(blk + 64 * h + 32 * part);
        r.b = ldg16(blk + 64 * h + 32 * part + 16);
        r.c = ldg16(blk + 128 + 32 * h);
        r.d = ldg16(blk + 128 + 32 * h + 16);
        r.e = ldg16(p1 + block * 16);
        r.x = uint32_t(__ldg(reinterpret_cast<const uint16_t *>(p2) + block));
    } else {
        const int h = c >> 1;
        r.a = ldg16(p0 + block * 64 + 32 * h);
        r.b = ldg16(p0 + block * 64 + 32 * h + 16);
        r.c = ldg16(p1 + block * 16);
        r.x = __ldg(reinterpret_cast<const uint32_t *>(p2) + block);
    }
    return r;
}

// One 256-block of one weight row against up to kGroup activation rows. The
// four lanes of a block each own 64 values; their integer partial sums are
// combined first so the block's float term is formed once, as on the CPU.
// Every lane of the warp must call this (the shuffles are warp-wide);
// `valid` is false for lanes whose block index is past the row end.
template <uint32_t TYPE>
__device__ __forceinline__ void lane_block(const WRegs & wr, int c, const ActView & a, uint32_t b, uint32_t t0, int nt,
                                           bool valid, double * acc) {
    const uint32_t nb = a.cols / kQK;
    if constexpr (TYPE == JF_TENSOR_Q4_K) {
        const uint4 q0 = wr.a, q1 = wr.b, hdr = wr.c;
        const float d = half_bits_to_float(uint16_t(hdr.x & 0xffffu));
        const float dmin = half_bits_to_float(uint16_t(hdr.x >> 16));
        int sc_lo, m_lo, sc_hi, m_hi;
        q4k_scale_min(hdr, 2 * c, sc_lo, m_lo);
        q4k_scale_min(hdr, 2 * c + 1, sc_hi, m_hi);
        const uint32_t q[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
        for (int t = 0; t < kGroup; ++t) {
            if (t >= nt) break;
            const uint64_t row = uint64_t(t0 + t);
            int isum = 0, msum = 0;
            float da = 0.0f;
            if (valid) {
                const int8_t * aq = a.qs + row * a.cols + uint64_t(b) * kQK + 64 * c;
                const int4 a0 = __ldg(reinterpret_cast<const int4 *>(aq));
                const int4 a1 = __ldg(reinterpret_cast<const int4 *>(aq + 16));
                const int4 a2 = __ldg(reinterpret_cast<const int4 *>(aq + 32));
                const int4 a3 = __ldg(reinterpret_cast<const int4 *>(aq + 48));
                const int av[16] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w,
                                    a2.x, a2.y, a2.z, a2.w, a3.x, a3.y, a3.z, a3.w};
                int s_lo = 0, s_hi = 0;
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    s_lo = dp4a(int(q[i] & 0x0f0f0f0fu), av[i], s_lo);
                    s_hi = dp4a(int((q[i] >> 4) & 0x0f0f0f0fu), av[8 + i], s_hi);
                }
                const int2 bs = __ldg(reinterpret_cast<const int2 *>(a.bsums + row * (a.cols / 16) + uint64_t(b) * 16 + 4 * c));
                const int b0 = int(int16_t(bs.x & 0xffff)), b1 = int(int16_t(uint32_t(bs.x) >> 16));
                const int b2 = int(int16_t(bs.y & 0xffff)), b3 = int(int16_t(uint32_t(bs.y) >> 16));
                isum = sc_lo * s_lo + sc_hi * s_hi;
                msum = m_lo * (b0 + b1) + m_hi * (b2 + b3);
                da = __ldg(a.d + row * nb + b);
            }
            isum = block_lanes_sum(isum);
            msum = block_lanes_sum(msum);
            if (valid && c == 0) {
                const float cb = __fsub_rn(__fmul_rn(__fmul_rn(d, da), float(isum)),
                                           __fmul_rn(__fmul_rn(dmin, da), float(msum)));
                acc[t] += double(cb);
            }
        }
    } else if constexpr (TYPE == JF_TENSOR_Q6_K) {
        const int h = c >> 1, part = c & 1;
        const uint4 l0 = wr.a, l1 = wr.b, h0 = wr.c, h1 = wr.d, scv = wr.e;
        const float d = valid ? half_bits_to_float(uint16_t(wr.x)) : 0.0f;
        const uint32_t L[8] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w};
        const uint32_t H[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
        int qa[8], qb[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            qa[i] = int((L[i] & 0x0f0f0f0fu) | (((H[i] >> (2 * part)) & 0x03030303u) << 4));
            qb[i] = int(((L[i] >> 4) & 0x0f0f0f0fu) | (((H[i] >> (4 + 2 * part)) & 0x03030303u) << 4));
        }
        const int ga = 8 * h + 2 * part, gb = 8 * h + 4 + 2 * part;  // 16-value groups
        const int sa0 = int(int8_t(byte_of(scv, ga))), sa1 = int(int8_t(byte_of(scv, ga + 1)));
        const int sb0 = int(int8_t(byte_of(scv, gb))), sb1 = int(int8_t(byte_of(scv, gb + 1)));
#pragma unroll
        for (int t = 0; t < kGroup; ++t) {
            if (t >= nt) break;
            const uint64_t row = uint64_t(t0 + t);
            int isum = 0;
            float da = 0.0f;
            if (valid) {
                const int8_t * aq = a.qs + row * a.cols + uint64_t(b) * kQK + 128 * h + 32 * part;
                const int4 x0 = __ldg(reinterpret_cast<const int4 *>(aq));
                const int4 x1 = __ldg(reinterpret_cast<const int4 *>(aq + 16));
                const int4 y0 = __ldg(reinterpret_cast<const int4 *>(aq + 64));
                const int4 y1 = __ldg(reinterpret_cast<const int4 *>(aq + 80));
                const int ax[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
                const int ay[8] = {y0.x, y0.y, y0.z, y0.w, y1.x, y1.y, y1.z, y1.w};
                int s[4] = {0, 0, 0, 0};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    s[0] = dp4a(qa[i], ax[i], s[0]);
                    s[1] = dp4a(qa[4 + i], ax[4 + i], s[1]);
                    s[2] = dp4a(qb[i], ay[i], s[2]);
                    s[3] = dp4a(qb[4 + i], ay[4 + i], s[3]);
                }
                const int16_t * bs = a.bsums + row * (a.cols / 16) + uint64_t(b) * 16;
                // codes are stored +32: subtract 32 * (sum of the group's activations)
                s[0] -= 32 * int(__ldg(bs + ga));
                s[1] -= 32 * int(__ldg(bs + ga + 1));
                s[2] -= 32 * int(__ldg(bs + gb));
                s[3] -= 32 * int(__ldg(bs + gb + 1));
                isum = sa0 * s[0] + sa1 * s[1] + sb0 * s[2] + sb1 * s[3];
                da = __ldg(a.d + row * nb + b);
            }
            isum = block_lanes_sum(isum);
            if (valid && c == 0) acc[t] += double(__fmul_rn(__fmul_rn(d, da), float(isum)));
        }
    } else {  // Q2_K
        const int h = c >> 1, sp = c & 1;
        const uint4 c0 = wr.a, c1 = wr.b, scv = wr.c;
        const uint32_t dd = wr.x;
        const float d = half_bits_to_float(uint16_t(dd & 0xffffu));
        const float dmin = half_bits_to_float(uint16_t(dd >> 16));
        const uint32_t Q[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
        int qe[8], qo[8];  // s = 2sp (even) and s = 2sp + 1 (odd)
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            qe[i] = int((Q[i] >> (4 * sp)) & 0x03030303u);
            qo[i] = int((Q[i] >> (4 * sp + 2)) & 0x03030303u);
        }
        const int g0 = 8 * h + 4 * sp;  // groups g0..g0+3
        int scl[4], mnl[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint32_t sb = byte_of(scv, g0 + k);
            scl[k] = int(sb & 15);
            mnl[k] = int(sb >> 4);
        }
#pragma unroll
        for (int t = 0; t < kGroup; ++t) {
            if (t >= nt) break;
            const uint64_t row = uint64_t(t0 + t);
            int isum = 0, msum = 0;
            float da = 0.0f;
            if (valid) {
                const int8_t * aq = a.qs + row * a.cols + uint64_t(b) * kQK + 128 * h + 64 * sp;
                const int4 x0 = __ldg(reinterpret_cast<const int4 *>(aq));
                const int4 x1 = __ldg(reinterpret_cast<const int4 *>(aq + 16));
                const int4 x2 = __ldg(reinterpret_cast<const int4 *>(aq + 32));
                const int4 x3 = __ldg(reinterpret_cast<const int4 *>(aq + 48));
                const int ax[16] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w,
                                    x2.x, x2.y, x2.z, x2.w, x3.x, x3.y, x3.z, x3.w};
                int s[4] = {0, 0, 0, 0};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    s[0] = dp4a(qe[i], ax[i], s[0]);
                    s[1] = dp4a(qe[4 + i], ax[4 + i], s[1]);
                    s[2] = dp4a(qo[i], ax[8 + i], s[2]);
                    s[3] = dp4a(qo[4 + i], ax[12 + i], s[3]);
                }
                const int16_t * bs = a.bsums + row * (a.cols / 16) + uint64_t(b) * 16 + g0;
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    isum += scl[k] * s[k];
                    msum += mnl[k] * int(__ldg(bs + k));
                }
                da = __ldg(a.d + row * nb + b);
            }
            isum = block_lanes_sum(isum);
            msum = block_lanes_sum(msum);
            if (valid && c == 0) {
                const float cb = __fsub_rn(__fmul_rn(__fmul_rn(d, da), float(isum)),
                                           __fmul_rn(__fmul_rn(dmin, da), float(msum)));
                acc[t] += double(cb);
            }
        }
    }
}

template <uint32_t TYPE>
__global__ void __launch_bounds__(kWarps * 32) mmv_kquant_kernel(jfb_weight w, ActView a, uint32_t n, float * out,
                                                               Epilogue ep) {
    pdl_trigger();
    pdl_wait();
    const uint32_t row = blockIdx.x * kWarps + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    const uint32_t t0 = blockIdx.y * kGroup;
    if (row >= w.rows || t0 >= n) return;
    const int nt = int(min(uint32_t(kGroup), n - t0));
    const uint32_t nb = w.cols / kQK;
    double acc[kGroup];
#pragma unroll
    for (int t = 0; t < kGroup; ++t) acc[t] = 0.0;
    const int c = lane & 3;
    // warp-uniform trip count (the block lanes shuffle); the next step's
    // weights are requested before this step's arithmetic
    uint32_t b = uint32_t(lane >> 2);
    WRegs cur = load_weights<TYPE>(w, uint64_t(row) * nb + (b < nb ? b : 0), c, b < nb);
    for (uint32_t b0 = 0; b0 < nb; b0 += 8) {
        const uint32_t bn = b0 + 8 + uint32_t(lane >> 2);
        WRegs nxt{};
        if (b0 + 8 < nb) nxt = load_weights<TYPE>(w, uint64_t(row) * nb + (bn < nb ? bn : 0), c, bn < nb);
        b = b0 + uint32_t(lane >> 2);
        lane_block<TYPE>(cur, c, a, b, t0, nt, b < nb, acc);
        cur = nxt;
    }
#pragma unroll
    for (int t = 0; t < kGroup; ++t) {
        if (t >= nt) break;
        const double v = warp_sum(acc[t]);
        if (lane == 0) store_out(float(v), row, t0 + t, w.rows, out, ep);
    }
}

// F32 / F16 weights: plain dot products; F16 weights see f16-rounded
// activations (GGML converts src1 to the F16 vec_dot_type).
template <bool HALF>
__global__ void __launch_bounds__(kWarps * 32) mmv_float_kernel(jfb_weight w, const float * __restrict__ x, uint32_t n,
                                                              float * out, Epilogue ep) {
    pdl_trigger();
    pdl_wait();
    const uint32_t row = blockIdx.x * kWarps + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    const uint32_t t0 = blockIdx.y * kGroup;
    if (row >= w.rows || t0 >= n) return;
    const int nt = int(min(uint32_t(kGroup), n - t0));
    for (int t = 0; t < nt; ++t) {
        const float * xr = x + uint64_t(t0 + t) * w.cols;
        double acc = 0.0;
        for (uint32_t k = lane; k < w.cols; k += 32) {
            float wv, xv = xr[k];
            if constexpr (HALF) {
                wv = half_bits_to_float(static_cast<const uint16_t *>(w.plane[0])[uint64_t(row) * w.cols + k]);
                xv = __half2float(__float2half_rn(xv));
            } else {
                wv = static_cast<const float *>(w.plane[0])[uint64_t(row) * w.cols + k];
            }
            acc += double(__fmul_rn(wv, xv));  // products rounded to float, summed in double
        }
        acc = warp_sum(acc);
        if (lane == 0) store_out(float(acc), row, t0 + t, w.rows, out, ep);
    }
}

}  // namespace
}  // namespace jfb

using namespace jfb;

extern "C" jfb_status jfb_matmul(const jfb_weight * weight, const jfb_q8k * x_q8, const float * x_f32, uint32_t n,
                                 uint32_t epilogue, const float * bias, const float * residual, float * out,
                                 void * stream) {
    if (weight == nullptr || out == nullptr) return status_error(JFB_STATUS_INVALID_ARGUMENT, "weight and output are required");
    if (epilogue > JFB_EPILOGUE_RESIDUAL || (epilogue == JFB_EPILOGUE_BIAS && bias == nullptr) ||
        (epilogue == JFB_EPILOGUE_RESIDUAL && residual == nullptr)) {
        return status_error(JFB_STATUS_INVALID_ARGUMENT, "matmul epilogue operands are missing");
    }
    if (n == 0) return status_ok();
    const jfb_weight w = *weight;
    const Epilogue ep{epilogue, bias, residual};
    const dim3 grid((w.rows + kWarps - 1) / kWarps, (n + kGroup - 1) / kGroup);
    if (grid.y > 65535u) return status_error(JFB_STATUS_INVALID_ARGUMENT, "too many activation rows (%u)", n);
    cudaStream_t s = as_stream(stream);
    if (is_kquant(w.type)) {
        if (x_q8 == nullptr || x_q8->qs == nullptr || x_q8->d == nullptr || x_q8->bsums == nullptr) {
            return status_error(JFB_STATUS_INVALID_ARGUMENT, "K-quant matmul needs Q8_K activations");
        }
        if (w.cols % kQK != 0) return status_error(JFB_STATUS_INVALID_ARGUMENT, "K-quant columns must be a multiple of 256");
        const ActView a{x_q8->qs, x_q8->d, x_q8->bsums, w.cols};
        cudaError_t e;
        switch (w.type) {
        case JF_TENSOR_Q4_K: e = launch_k(mmv_kquant_kernel<JF_TENSOR_Q4_K>, grid, dim3(kWarps * 32), 0, s, w, a, n, out, ep); break;
        case JF_TENSOR_Q6_K: e = launch_k(mmv_kquant_kernel<JF_TENSOR_Q6_K>, grid, dim3(kWarps * 32), 0, s, w, a, n, out, ep); break;
        default: e = launch_k(mmv_kquant_kernel<JF_TENSOR_Q2_K>, grid, dim3(kWarps * 32), 0, s, w, a, n, out, ep); break;
        }
        if (e != cudaSuccess) return status_error(JFB_STATUS_CUDA_ERROR, "jfb_matmul: %s", cudaGetErrorString(e));
        return launch_status("jfb_matmul(kquant)");
    }
    if (x_f32 == nullptr) return status_error(JFB_STATUS_INVALID_ARGUMENT, "float matmul needs f32 activations");
    if (w.type == JF_TENSOR_F32) {
        const cudaError_t e = launch_k(mmv_float_kernel<false>, grid, dim3(kWarps * 32), 0, s, w, x_f32, n, out, ep);
        if (e != cudaSuccess) return status_error(JFB_STATUS_CUDA_ERROR, "jfb_matmul: %s", cudaGetErrorString(e));
    } else if (w.type == JF_TENSOR_F16) {
        const cudaError_t e = launch_k(mmv_float_kernel<true>, grid, dim3(kWarps * 32), 0, s, w, x_f32, n, out, ep);
        if (e != cudaSuccess) return status_error(JFB_STATUS_CUDA_ERROR, "jfb_matmul: %s", cudaGetErrorString(e));
    } else {
        return status_error(JFB_STATUS_UNSUPPORTED, "matmul weight type %u is not supported", w.type);
    }
    return launch_status("jfb_matmul(float)");
}
