// Weight residency kernels: planar repack of GGML K-quant blocks, bit-exact
// dequantization and the embedding-row gather.
//
// Dequantization follows the published K-quant formulas with every product
// rounded separately (__fmul_rn / __fsub_rn, no fused multiply-add), which is
// the order GGML's dequantize_row_{q2_K,q4_K,q6_K} and gguf-py's NumPy
// dequantizers evaluate: value = (d * scale) * q - (dmin * min).
#include "common.cuh"

namespace jfb {
namespace {

constexpr uint64_t kPlaneAlign = 256;

uint64_t align_up(uint64_t v, uint64_t a) { return (v + a - 1) / a * a; }

struct PlaneSizes {
    uint64_t bytes[3];
};

// Bytes of each plane per 256-block.
__host__ __device__ inline void plane_block_bytes(uint32_t type, uint32_t * b0, uint32_t * b1, uint32_t * b2) {
    switch (type) {
    case JF_TENSOR_Q4_K: *b0 = 128; *b1 = 16; *b2 = 0; break;
    case JF_TENSOR_Q6_K: *b0 = 192; *b1 = 16; *b2 = 2; break;
    case JF_TENSOR_Q2_K: *b0 = 64; *b1 = 16; *b2 = 4; break;
    default: *b0 = 0; *b1 = 0; *b2 = 0; break;
    }
}

PlaneSizes plane_sizes(uint32_t type, uint32_t rows, uint32_t cols) {
    PlaneSizes p{{0, 0, 0}};
    if (type == JF_TENSOR_F32) {
        p.bytes[0] = uint64_t(rows) * cols * 4;
    } else if (type == JF_TENSOR_F16) {
        p.bytes[0] = uint64_t(rows) * cols * 2;
    } else {
        uint32_t b0, b1, b2;
        plane_block_bytes(type, &b0, &b1, &b2);
        const uint64_t blocks = uint64_t(rows) * (cols / kQK);
        p.bytes[0] = blocks * b0;
        p.bytes[1] = blocks * b1;
        p.bytes[2] = blocks * b2;
    }
    return p;
}

// One thread per 16-byte piece of an output plane would be ideal; blocks are
// small enough that one warp per GGML block keeps this simple and coalesced.
__global__ void repack_kernel(uint32_t type, uint64_t blocks, const uint8_t * __restrict__ src,
                              uint8_t * __restrict__ p0, uint8_t * __restrict__ p1, uint8_t * __restrict__ p2) {
    const uint64_t block = (uint64_t(blockIdx.x) * blockDim.x + threadIdx.x) / 32;
    const int lane = threadIdx.x & 31;
    if (block >= blocks) return;
    if (type == JF_TENSOR_Q4_K) {
        const uint8_t * b = src + block * 144;  // d, dmin, scales[12], qs[128]
        for (int i = lane; i < 16; i += 32) p1[block * 16 + i] = b[i];
        for (int i = lane; i < 128; i += 32) p0[block * 128 + i] = b[16 + i];
    } else if (type == JF_TENSOR_Q6_K) {
        const uint8_t * b = src + block * 210;  // ql[128], qh[64], scales[16], d
        for (int i = lane; i < 192; i += 32) p0[block * 192 + i] = b[i];
        for (int i = lane; i < 16; i += 32) p1[block * 16 + i] = b[192 + i];
        if (lane < 2) p2[block * 2 + lane] = b[208 + lane];
    } else {  // Q2_K: scales[16], qs[64], d, dmin
        const uint8_t * b = src + block * 84;
        for (int i = lane; i < 64; i += 32) p0[block * 64 + i] = b[16 + i];
        for (int i = lane; i < 16; i += 32) p1[block * 16 + i] = b[i];
        if (lane < 4) p2[block * 4 + lane] = b[80 + lane];
    }
}

// ---- dequantization ---------------------------------------------------------

__device__ __forceinline__ void q4k_scale_min(const uint8_t * s, int j, int & sc, int & m) {
    if (j < 4) {
        sc = s[j] & 63;
        m = s[j + 4] & 63;
    } else {
        sc = (s[j + 4] & 0x0f) | ((s[j - 4] >> 6) << 4);
        m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

// Element e (0..255) of block `block` of a planar weight.
__device__ __forceinline__ float dequant_element(const jfb_weight & w, uint64_t block, int e) {
    const uint8_t * p0 = static_cast<const uint8_t *>(w.plane[0]);
    const uint8_t * p1 = static_cast<const uint8_t *>(w.plane[1]);
    const uint8_t * p2 = static_cast<const uint8_t *>(w.plane[2]);
    if (w.type == JF_TENSOR_Q4_K) {
        const uint8_t * hdr = p1 + block * 16;
        const float d = half_bits_to_float(uint16_t(hdr[0] | (hdr[1] << 8)));
        const float dmin = half_bits_to_float(uint16_t(hdr[2] | (hdr[3] << 8)));
        const int j = e / 32;
        int sc, m;
        q4k_scale_min(hdr + 4, j, sc, m);
        const uint8_t byte = p0[block * 128 + 32 * (j / 2) + (e % 32)];
        const int q = (byte >> (4 * (j & 1))) & 15;
        const float d1 = __fmul_rn(d, float(sc));
        const float m1 = __fmul_rn(dmin, float(m));
        return __fsub_rn(__fmul_rn(d1, float(q)), m1);
    }
    if (w.type == JF_TENSOR_Q6_K) {
        const uint8_t * ql = p0 + block * 192;
        const uint8_t * qh = ql + 128;
        const int h = e / 128, r = e % 128;
        const int lo = (ql[64 * h + (r % 64)] >> (4 * (r / 64))) & 15;
        const int hi = (qh[32 * h + (r % 32)] >> (2 * (r / 32))) & 3;
        const int q = (lo | (hi << 4)) - 32;
        const int8_t sc = static_cast<int8_t>(p1[block * 16 + e / 16]);
        const float d = half_bits_to_float(uint16_t(p2[block * 2] | (p2[block * 2 + 1] << 8)));
        return __fmul_rn(__fmul_rn(d, float(sc)), float(q));
    }
    // Q2_K
    const uint8_t s = p1[block * 16 + e / 16];
    const float d = half_bits_to_float(uint16_t(p2[block * 4] | (p2[block * 4 + 1] << 8)));
    const float dmin = half_bits_to_float(uint16_t(p2[block * 4 + 2] | (p2[block * 4 + 3] << 8)));
    const int h = e / 128, sh = (e % 128) / 32, l = e % 32;
    const int q = (p0[block * 64 + 32 * h + l] >> (2 * sh)) & 3;
    const float dl = __fmul_rn(d, float(s & 15));
    const float ml = __fmul_rn(dmin, float(s >> 4));
    return __fsub_rn(__fmul_rn(dl, float(q)), ml);
}

__device__ __forceinline__ float weight_element(const jfb_weight & w, uint64_t row, uint32_t col) {
    if (w.type == JF_TENSOR_F32) return static_cast<const float *>(w.plane[0])[row * w.cols + col];
    if (w.type == JF_TENSOR_F16) {
        return half_bits_to_float(static_cast<const uint16_t *>(w.plane[0])[row * w.cols + col]);
    }
    return dequant_element(w, row * (w.cols / kQK) + col / kQK, int(col % kQK));
}

__global__ void dequantize_kernel(jfb_weight w, float * __restrict__ out) {
    const uint64_t total = uint64_t(w.rows) * w.cols;
    for (uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += uint64_t(gridDim.x) * blockDim.x) {
        out[i] = weight_element(w, i / w.cols, uint32_t(i % w.cols));
    }
}

__global__ void embed_kernel(jfb_weight w, const int32_t * __restrict__ tokens, float * __restrict__ hidden,
                             int32_t * error_flag) {
    pdl_trigger();
    pdl_wait();  // the token ids may be the previous step's greedy tokens
    const int r = blockIdx.x;
    const int32_t tok = tokens[r];
    float * out = hidden + uint64_t(r) * w.cols;
    const bool valid = tok >= 0 && uint32_t(tok) < w.rows;
    if (!valid && threadIdx.x == 0 && error_flag != nullptr) *error_flag = 1;
    for (uint32_t c = threadIdx.x; c < w.cols; c += blockDim.x) {
        out[c] = valid ? weight_element(w, uint64_t(tok), c) : 0.0f;
    }
}

}  // namespace
}  // namespace jfb

using namespace jfb;

extern "C" uint64_t jfb_weight_device_bytes(uint32_t type, uint32_t rows, uint32_t cols) {
    const PlaneSizes p = plane_sizes(type, rows, cols);
    // K-quant weights keep 16 bytes past the last plane, so kernels may read
    // the whole aligned 4-byte word that holds a block's 2-byte scale
    const uint64_t tail = is_kquant(type) ? 16 : 0;
    return align_up(p.bytes[0], kPlaneAlign) + align_up(p.bytes[1], kPlaneAlign) + align_up(p.bytes[2] + tail, kPlaneAlign);
}

extern "C" jfb_status jfb_weight_row_view(const jfb_weight * weight, uint32_t row_begin, uint32_t rows,
                                          jfb_weight * view) {
    if (weight == nullptr || view == nullptr || !is_kquant(weight->type)) {
        return status_error(JFB_STATUS_INVALID_ARGUMENT, "row views need a K-quant weight");
    }
    if (rows == 0 || uint64_t(row_begin) + rows > weight->rows) {
        return status_error(JFB_STATUS_INVALID_ARGUMENT, "row view [%u, %u) is outside the weight's %u rows", row_begin,
                            row_begin + rows, weight->rows);
    }
    uint32_t b[3];
    plane_block_bytes(weight->type, &b[0], &b[1], &b[2]);
    const uint64_t blocks_before = uint64_t(row_begin) * (weight->cols / kQK);
    *view = *weight;
    view->rows = rows;
    for (int i = 0; i < 3; ++i) {
        view->plane[i] = weight->plane[i] == nullptr
                             ? nullptr
                             : static_cast<const uint8_t *>(weight->plane[i]) + blocks_before * b[i];
    }
    return status_ok();
}

static jfb_status check_weight_shape(uint32_t type, uint32_t rows, uint32_t cols) {
    if (rows == 0 || cols == 0) return status_error(JFB_STATUS_INVALID_ARGUMENT, "weight shape must be positive");
    if (type != JF_TENSOR_F32 && type != JF_TENSOR_F16 && !is_kquant(type)) {
        return status_error(JFB_STATUS_UNSUPPORTED, "weight type %u is not supported by the CUDA engine", type);
    }
    if (is_kquant(type) && cols % kQK != 0) {
        return status_error(JFB_STATUS_INVALID_ARGUMENT, "K-quant weight columns must be a multiple of 256");
    }
    return status_ok();
}

extern "C" jfb_status jfb_weight_repack(uint32_t type, uint32_t rows, uint32_t cols, const void * src, void * dst,
                                        jfb_weight * weight, void * stream) {
    jfb_status s = check_weight_shape(type, rows, cols);
    if (s.code != JFB_STATUS_OK) return s;
    if (src == nullptr || dst == nullptr || weight == nullptr) {
        return status_error(JFB_STATUS_INVALID_ARGUMENT, "repack needs source, destination and descriptor");
    }
    const PlaneSizes p = plane_sizes(type, rows, cols);
    uint8_t * base = static_cast<uint8_t *>(dst);
    weight->type = type;
    weight->rows = rows;
    weight->cols = cols;
    weight->reserved = 0;
    weight->plane[0] = base;
    weight->plane[1] = p.bytes[1] ? base + align_up(p.bytes[0], kPlaneAlign) : nullptr;
    weight->plane[2] = p.bytes[2] ? base + align_up(p.bytes[0], kPlaneAlign) + align_up(p.bytes[1], kPlaneAlign)
                                  : nullptr;
    if (!is_kquant(type)) {
        const cudaError_t e = cudaMemcpyAsync(dst, src, p.bytes[0], cudaMemcpyDeviceToDevice, as_stream(stream));
        if (e != cudaSuccess) return status_error(JFB_STATUS_CUDA_ERROR, "repack copy: %s", cudaGetErrorString(e));
        return status_ok();
    }
    const uint64_t blocks = uint64_t(rows) * (cols / kQK);
    const unsigned threads = 256;
    const uint64_t grid = (blocks * 32 + threads - 1) / threads;
    repack_kernel<<<unsigned(grid), threads, 0, as_stream(stream)>>>(
        type, blocks, static_cast<const uint8_t *>(src), static_cast<uint8_t *>(const_cast<void *>(weight->plane[0])),
        static_cast<uint8_t *>(const_cast<void *>(weight->plane[1])),
        static_cast<uint8_t *>(const_cast<void *>(weight->plane[2])));
    return launch_status("jfb_weight_repack");
}

extern "C" jfb_status jfb_dequantize(const jfb_weight * weight, float * out, void * stream) {
    if (weight == nullptr || out == nullptr) return status_error(JFB_STATUS_INVALID_ARGUMENT, "weight and output are required");
    jfb_status s = check_weight_shape(weight->type, weight->rows, weight->cols);
    if (s.code != JFB_STATUS_OK) return s;
    const uint64_t total = uint64_t(weight->rows) * weight->cols;
    const unsigned grid = unsigned(std::min<uint64_t>((total + 255) / 256, 148u * 16u));
    dequantize_kernel<<<grid, 256, 0, as_stream(stream)>>>(*weight, out);
    return launch_status("jfb_dequantize");
}

extern "C" jfb_status jfb_embed_rows(const jfb_weight * embd, const int32_t * tokens, uint32_t n, float * hidden,
                                     int32_t * error_flag, void * stream) {
    if (embd == nullptr || tokens == nullptr || hidden == nullptr) {
        return status_error(JFB_STATUS_INVALID_ARGUMENT, "embedding, tokens and output are required");
    }
    if (n == 0) return status_ok();
    jfb_status s = check_weight_shape(embd->type, embd->rows, embd->cols);
    if (s.code != JFB_STATUS_OK) return s;
    const cudaError_t e = launch_k(embed_kernel, dim3(n), dim3(256), 0, as_stream(stream), *embd, tokens, hidden, error_flag);
    if (e != cudaSuccess) return status_error(JFB_STATUS_CUDA_ERROR, "jfb_embed_rows: %s", cudaGetErrorString(e));
    return launch_status("jfb_embed_rows");
}
