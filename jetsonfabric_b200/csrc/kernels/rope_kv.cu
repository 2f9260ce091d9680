// NEOX rotary embedding of q and k, and the F16 append of k and v to the
// per-sequence KV cache (ggml_rope_ext + ggml_set_rows,
// qwen2_architecture.cpp:400-424, 499-506).
//
// GGML's rope cache builds the angle of pair i as theta_0 = position,
// theta_{i+1} = theta_i * theta_scale in float and stores cosf/sinf of it;
// the pair (x_i, x_{i+d/2}) becomes
//     y_i       = x_i * cos - x_{i+d/2} * sin
//     y_{i+d/2} = x_i * sin + x_{i+d/2} * cos
// The (cos, sin) table is computed once on the host with the same C library
// calls (jfb_rope_table_host) and read here; every product and sum is
// rounded separately (no fused multiply-add) like the CPU evaluation.
#include "common.cuh"

#include <cmath>

namespace jfb {
namespace {

constexpr int kThreads = 256;

// One element per thread: grid (rows, ceil((heads * rope_dims / 2 + kv_dim) / 256)). Items
// [0, heads * pairs) are the rotated pairs of q (in place); the next kv_dim
// items are the k elements (rotated or passed through) and v elements of the
// appended cache row. Each thread does one round of independent loads.
__global__ void __launch_bounds__(kThreads) rope_kv_kernel(float * __restrict__ q, const float * __restrict__ k,
                                                         const float * __restrict__ v, const int32_t * __restrict__ seq,
                                                         const int32_t * __restrict__ pos, uint32_t heads,
                                                         uint32_t kv_heads, uint32_t head_dim, uint32_t rope_dims,
                                                         const float2 * __restrict__ table, uint32_t table_positions,
                                                         const jfb_kv_slot * __restrict__ slots, uint32_t layer) {
    pdl_trigger();
    const uint32_t r = blockIdx.x;
    const int32_t p = pos[r];                 // per-call metadata: written before the first kernel of the call
    const jfb_kv_slot slot = slots[seq[r]];
    if (p < 0 || uint32_t(p) >= slot.capacity || uint32_t(p) >= table_positions) return;  // never issued by the engine
    const uint32_t pairs = rope_dims / 2;
    const float2 * cs = table + uint64_t(p) * pairs;
    const uint32_t hd = heads * head_dim, kvd = kv_heads * head_dim;
    const uint32_t idx = blockIdx.y * kThreads + threadIdx.x;
    const uint32_t qitems = heads * pairs;
    // this item's (cos, sin): the table is written by no earlier kernel
    float2 c = make_float2(0.0f, 0.0f);
    if (idx < qitems) c = cs[idx % pairs];
    else if (idx < qitems + kvd && (idx - qitems) % head_dim < rope_dims) c = cs[(idx - qitems) % head_dim % pairs];
    pdl_wait();                                // q, k, v come from the projection before this kernel
    if (idx < qitems) {
        const uint32_t h = idx / pairs, i = idx % pairs;
        float * x = q + uint64_t(r) * hd + h * head_dim;
        const float x0 = x[i], x1 = x[i + pairs];
        x[i] = __fsub_rn(__fmul_rn(x0, c.x), __fmul_rn(x1, c.y));
        x[i + pairs] = __fadd_rn(__fmul_rn(x0, c.y), __fmul_rn(x1, c.x));
    } else if (idx < qitems + kvd) {
        const uint32_t e_all = idx - qitems;
        const uint32_t h = e_all / head_dim, e = e_all % head_dim;
        const float * kr = k + uint64_t(r) * kvd;
        float y;
        if (e < rope_dims) {
            const uint32_t i = e % pairs;
            const float x0 = kr[h * head_dim + i], x1 = kr[h * head_dim + i + pairs];
            y = e < pairs ? __fsub_rn(__fmul_rn(x0, c.x), __fmul_rn(x1, c.y))
                          : __fadd_rn(__fmul_rn(x0, c.y), __fmul_rn(x1, c.x));
        } else {
            y = kr[e_all];
        }
        const uint64_t row = (uint64_t(layer) * slot.capacity + uint64_t(p)) * kvd;
        slot.k[row + e_all] = float_to_half_bits(y);
        slot.v[row + e_all] = float_to_half_bits(v[uint64_t(r) * kvd + e_all]);
    }
}

}  // namespace
}  // namespace jfb

using namespace jfb;

extern "C" void jfb_rope_table_host(float * table, uint32_t positions, uint32_t rope_dims, float freq_base) {
    const uint32_t pairs = rope_dims / 2;
    const float theta_scale = ::powf(freq_base, -2.0f / float(rope_dims));
    for (uint32_t p = 0; p < positions; ++p) {
        float theta = float(p);
        float * row = table + uint64_t(p) * pairs * 2;
        for (uint32_t i = 0; i < pairs; ++i) {
            row[2 * i] = ::cosf(theta);
            row[2 * i + 1] = ::sinf(theta);
            theta = theta * theta_scale;
        }
    }
}

extern "C" jfb_status jfb_rope_kv_append(float * q, const float * k, const float * v, uint32_t n, const int32_t * seq,
                                         const int32_t * pos, uint32_t heads, uint32_t kv_heads, uint32_t head_dim,
                                         uint32_t rope_dims, const float * rope_table, uint32_t table_positions,
                                         const jfb_kv_slot * slots, uint32_t layer, void * stream) {
    if (q == nullptr || k == nullptr || v == nullptr || seq == nullptr || pos == nullptr || slots == nullptr ||
        rope_table == nullptr) {
        return status_error(JFB_STATUS_INVALID_ARGUMENT, "rope/kv append operands are required");
    }
    if (heads == 0 || kv_heads == 0 || heads % kv_heads != 0 || head_dim == 0 || rope_dims == 0 ||
        rope_dims > head_dim || rope_dims % 2 != 0) {
        return status_error(JFB_STATUS_INVALID_ARGUMENT, "rope/kv append dimensions are inconsistent");
    }
    if (n == 0) return status_ok();
    const uint32_t items = heads * (rope_dims / 2) + kv_heads * head_dim;
    const cudaError_t e = launch_k(rope_kv_kernel, dim3(n, (items + kThreads - 1) / kThreads), dim3(kThreads), 0,
                                   as_stream(stream), q, k, v, seq, pos, heads,
                                   kv_heads, head_dim, rope_dims, reinterpret_cast<const float2 *>(rope_table),
                                   table_positions, slots, layer);
    if (e != cudaSuccess) return status_error(JFB_STATUS_CUDA_ERROR, "jfb_rope_kv_append: %s", cudaGetErrorString(e));
    return launch_status("jfb_rope_kv_append");
}
