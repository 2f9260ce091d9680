// NEOX rotary embedding of q and k, and the F16 append of k and v to the
// per-sequence KV cache (ggml_rope_ext + ggml_set_rows,
// qwen2_architecture.cpp:400-424, 499-506).
//
// GGML's rope cache builds the angle of pair i as theta_0 = position,
// theta_{i+1} = theta_i * theta_scale in float, and rotates (x_i, x_{i+d/2}):
//     y_i       = x_i * cos - x_{i+d/2} * sin
//     y_{i+d/2} = x_i * sin + x_{i+d/2} * cos
// Every product and sum is rounded separately here (no fused multiply-add)
// so the result matches the CPU oracle's float evaluation.
#include "common.cuh"

namespace jfb {
namespace {

constexpr int kThreads = 128;
constexpr int kMaxPairs = 256;  // rope_dims up to 512

__global__ void __launch_bounds__(kThreads) rope_kv_kernel(float * __restrict__ q, const float * __restrict__ k,
                                                         const float * __restrict__ v, const int32_t * __restrict__ seq,
                                                         const int32_t * __restrict__ pos, uint32_t heads,
                                                         uint32_t kv_heads, uint32_t head_dim, uint32_t rope_dims,
                                                         float theta_scale, const jfb_kv_slot * __restrict__ slots,
                                                         uint32_t layer) {
    __shared__ float cos_s[kMaxPairs], sin_s[kMaxPairs];
    const uint32_t r = blockIdx.x;
    const int32_t p = pos[r];
    const jfb_kv_slot slot = slots[seq[r]];
    const uint32_t pairs = rope_dims / 2;
    for (uint32_t i = threadIdx.x; i < pairs; i += kThreads) {
        float theta = float(p);
        for (uint32_t s = 0; s < i; ++s) theta = __fmul_rn(theta, theta_scale);
        cos_s[i] = cosf(theta);
        sin_s[i] = sinf(theta);
    }
    __syncthreads();
    const uint32_t hd = heads * head_dim, kvd = kv_heads * head_dim;
    float * qr = q + uint64_t(r) * hd;
    for (uint32_t idx = threadIdx.x; idx < heads * pairs; idx += kThreads) {
        const uint32_t h = idx / pairs, i = idx % pairs;
        float * x = qr + h * head_dim;
        const float x0 = x[i], x1 = x[i + pairs];
        x[i] = __fsub_rn(__fmul_rn(x0, cos_s[i]), __fmul_rn(x1, sin_s[i]));
        x[i + pairs] = __fadd_rn(__fmul_rn(x0, sin_s[i]), __fmul_rn(x1, cos_s[i]));
    }
    if (p < 0 || uint32_t(p) >= slot.capacity) return;  // the engine never issues these
    const uint64_t row = (uint64_t(layer) * slot.capacity + uint64_t(p)) * kvd;
    const float * kr = k + uint64_t(r) * kvd;
    const float * vr = v + uint64_t(r) * kvd;
    for (uint32_t idx = threadIdx.x; idx < kvd; idx += kThreads) {
        const uint32_t h = idx / head_dim, e = idx % head_dim;
        float y;
        if (e < rope_dims) {
            const uint32_t i = e % pairs;
            const float x0 = kr[h * head_dim + i], x1 = kr[h * head_dim + i + pairs];
            y = e < pairs ? __fsub_rn(__fmul_rn(x0, cos_s[i]), __fmul_rn(x1, sin_s[i]))
                          : __fadd_rn(__fmul_rn(x0, sin_s[i]), __fmul_rn(x1, cos_s[i]));
        } else {
            y = kr[idx];
        }
        slot.k[row + idx] = float_to_half_bits(y);
        slot.v[row + idx] = float_to_half_bits(vr[idx]);
    }
}

}  // namespace
}  // namespace jfb

using namespace jfb;

extern "C" jfb_status jfb_rope_kv_append(float * q, const float * k, const float * v, uint32_t n, const int32_t * seq,
                                         const int32_t * pos, uint32_t heads, uint32_t kv_heads, uint32_t head_dim,
                                         uint32_t rope_dims, float theta_scale, const jfb_kv_slot * slots,
                                         uint32_t layer, void * stream) {
    if (q == nullptr || k == nullptr || v == nullptr || seq == nullptr || pos == nullptr || slots == nullptr) {
        return status_error(JFB_STATUS_INVALID_ARGUMENT, "rope/kv append operands are required");
    }
    if (heads == 0 || kv_heads == 0 || heads % kv_heads != 0 || head_dim == 0 || rope_dims == 0 ||
        rope_dims > head_dim || rope_dims % 2 != 0 || rope_dims / 2 > uint32_t(kMaxPairs)) {
        return status_error(JFB_STATUS_INVALID_ARGUMENT, "rope/kv append dimensions are inconsistent");
    }
    if (n == 0) return status_ok();
    rope_kv_kernel<<<n, kThreads, 0, as_stream(stream)>>>(q, k, v, seq, pos, heads, kv_heads, head_dim, rope_dims,
                                                          theta_scale, slots, layer);
    return launch_status("jfb_rope_kv_append");
}
