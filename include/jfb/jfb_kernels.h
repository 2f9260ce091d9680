/*
 * jfb kernel library: the hand-written sm_100a kernels of the native Qwen2
 * stage engine behind a thin C ABI.
 *
 * Conventions: every pointer argument is a device pointer unless its name ends
 * in _host; sizes are element counts; `stream` is a cudaStream_t passed as
 * void* (NULL = the legacy default stream); every call validates its shapes on
 * the host and returns a jfb_status instead of throwing. Nothing here
 * allocates device memory: scratch buffers are caller-owned, and their
 * required sizes are returned by the *_scratch_bytes queries.
 *
 * Each entry point replaces one GGML op (or a chain of them) of the reference
 * graph runtime/engines/native/src/qwen2_architecture.cpp; the op it replaces
 * is cited on its declaration. The reference has no C ABI at this level (it
 * calls into GGML), so these signatures are new; the engine ABI in
 * jfb_engine.h is the drop-in boundary.
 */
#ifndef JFB_KERNELS_H
#define JFB_KERNELS_H

#include <stddef.h>
#include <stdint.h>

#include "jfb/jfb_status.h"

#ifdef __cplusplus
extern "C" {
#endif

/* A weight matrix resident in HBM in the engine's planar layout.
 * rows = output features (GGML ne1), cols = input features (GGML ne0).
 *   F32, F16 : plane[0] = [rows][cols] values (GGML layout, unchanged)
 *   Q4_K     : plane[0] = [rows][cols/256][128] 4-bit codes,
 *              plane[1] = [rows][cols/256][16]  f16 d, f16 dmin, 12 scale bytes
 *   Q6_K     : plane[0] = [rows][cols/256][192] ql (128 B) then qh (64 B),
 *              plane[1] = [rows][cols/256][16]  int8 scales,
 *              plane[2] = [rows][cols/256]      f16 d
 *   Q2_K     : plane[0] = [rows][cols/256][64]  2-bit codes,
 *              plane[1] = [rows][cols/256][16]  scale | min << 4 bytes,
 *              plane[2] = [rows][cols/256][2]   f16 d, f16 dmin
 * The bytes inside each plane are the GGML block bytes, only regrouped, so
 * dequantized values are bit-identical to GGML's. */
typedef struct jfb_weight {
    uint32_t type;      /* JF_TENSOR_* id */
    uint32_t rows;
    uint32_t cols;
    uint32_t reserved;
    const void * plane[3];
} jfb_weight;

/* Activations quantized to GGML's Q8_K (per 256 values: f32 d, 256 int8,
 * 16 int16 partial sums), stored as three planes for [rows][cols]. */
typedef struct jfb_q8k {
    int8_t * qs;        /* [rows][cols] */
    float * d;          /* [rows][cols/256] */
    int16_t * bsums;    /* [rows][cols/16] */
    /* Operands of jfb_matmul_tc, written by every quantizer of this library
     * when non-NULL (all three or none): the same codes and partial sums as
     * f16 numbers (both are exact: |q| <= 127, |bsum| <= 2032) and the block
     * scales transposed, so the tensor cores load them without conversion. */
    uint16_t * qs_f16;     /* [rows][cols] */
    uint16_t * bsums_f16;  /* [rows][cols/16] */
    float * d_t;           /* [cols/256][d_stride]: d_t[b * d_stride + r] = d[r][b] */
    uint32_t d_stride;     /* row stride of d_t in floats: >= rows, a multiple of 4 */
    uint32_t reserved;
} jfb_q8k;

/* Per-sequence KV cache: token-major F16 rows for every resident layer,
 * K and V in separate buffers laid out [layers][capacity][kv_dim]. The
 * reference keeps K token-major and V transposed
 * (qwen2_architecture.cpp:1072-1079); here both are token-major so decode
 * never re-transposes V. */
typedef struct jfb_kv_slot {
    uint16_t * k;
    uint16_t * v;
    uint32_t capacity;
    uint32_t reserved;
} jfb_kv_slot;

/* Bytes of device memory a weight of this type and shape occupies (all
 * planes, each plane 256-byte aligned). */
uint64_t jfb_weight_device_bytes(uint32_t type, uint32_t rows, uint32_t cols);

/* Regroups GGML block bytes (src, device) into the planar layout at dst
 * (device, jfb_weight_device_bytes long) and fills *weight. */
jfb_status jfb_weight_repack(uint32_t type, uint32_t rows, uint32_t cols, const void * src, void * dst,
                             jfb_weight * weight, void * stream);

/* out[rows][cols] = dequantized weight, bit-exact with GGML's dequantize_row_*
 * (used by get_rows on token_embd, qwen2_architecture.cpp:564-568). */
jfb_status jfb_dequantize(const jfb_weight * weight, float * out, void * stream);

/* hidden[r][:] = dequantized row tokens[r] of the embedding table
 * (ggml_get_rows(token_embd, ids), qwen2_architecture.cpp:564-568).
 * Tokens outside [0, rows) are rejected on the device: the row is zeroed and
 * *error_flag (may be NULL) is set to 1. */
jfb_status jfb_embed_rows(const jfb_weight * embd, const int32_t * tokens, uint32_t n, float * hidden,
                          int32_t * error_flag, void * stream);

/* RMSNorm times weight (ggml_rms_norm + ggml_mul, qwen2_architecture.cpp:373-376)
 * of rows [n][cols] of x, optionally gathered by row_index (NULL = identity).
 * Writes the f32 result to out_f32 (may be NULL) and its Q8_K quantization
 * to out_q8 (may be NULL; cols % 256 == 0). */
jfb_status jfb_rmsnorm_quant(const float * x, const int32_t * row_index, const float * norm_weight,
                             uint32_t n, uint32_t cols, float eps, float * out_f32, const jfb_q8k * out_q8,
                             void * stream);

/* Q8_K quantization of f32 rows (GGML quantize_row_q8_K semantics). */
jfb_status jfb_quantize_q8k(const float * x, uint32_t n, uint32_t cols, const jfb_q8k * out, void * stream);

/* out[r][i] = silu(gate[r][i]) * up[r][i] (ggml_swiglu_split or silu+mul,
 * qwen2_architecture.cpp:508-520); also quantizes the result to Q8_K when
 * out_q8 != NULL. */
jfb_status jfb_swiglu_quant(const float * gate, const float * up, uint32_t n, uint32_t cols, float * out_f32,
                            const jfb_q8k * out_q8, void * stream);

/* Epilogue applied to y = W x by jfb_matmul. */
typedef enum jfb_epilogue {
    JFB_EPILOGUE_STORE = 0,        /* out = Wx */
    JFB_EPILOGUE_BIAS = 1,         /* out = Wx + bias */
    JFB_EPILOGUE_RESIDUAL = 2,     /* out = Wx + residual (out may alias residual) */
} jfb_epilogue;

/* ggml_mul_mat(W, x) for n activation rows (qwen2_architecture.cpp:361-371):
 * K-quant weights consume the Q8_K activations (exact integer sub-block dot
 * products, one float scale per 256-block); F32/F16 weights consume x_f32.
 * out[r][rows] row-major. */
jfb_status jfb_matmul(const jfb_weight * weight, const jfb_q8k * x_q8, const float * x_f32, uint32_t n,
                      uint32_t epilogue, const float * bias, const float * residual, float * out,
                      void * stream);

/* The same product as jfb_matmul for K-quant weights (Q4_K, Q6_K, Q2_K) on
 * the tcgen05 tensor cores, bit-identical to it for every input. Per 256-value
 * block the weight operand holds integer scale*code values in f16 and the
 * activation operand the Q8_K codes in f16. Each f32 accumulator chain is
 * bounded below 2^24 in magnitude, so it holds an exact integer sum:
 *   - Q4_K: one accumulator per 128-value half;
 *   - Q6_K: the 8-bit scale is split into 16*hi + lo, with two operands and
 *     two accumulators;
 *   - Q4_K and Q2_K: the mins term is one more K=16 product of the mins with
 *     the Q8_K partial sums.
 * The epilogue applies the per-block float terms exactly as the CPU rounds
 * them and sums them in double. The kernel is persistent: one CTA per SM walks
 * a contiguous range of (tile, block) work (stream-K, tiles of 128 weight rows
 * x 32 activation rows for n <= 32, x 64 above). A tile shared by several CTAs
 * is finished by the last contributor: every contributor adds its double
 * partials into the tile's workspace slot with f64 reductions, and the last
 * one reads the sums, clears the slot and writes the outputs (double sums of
 * the block terms are exact in any order). x_q8 must carry the tensor-core operands (qs_f16, bsums_f16, d_t),
 * all 16-byte aligned, with d_stride >= n.
 *
 * The workspace holds the partials and the per-tile arrival counters at
 * offsets that do not depend on the shape, so one workspace (sized for the
 * largest call) serves calls of any shape on one stream. It must be
 * zero-filled before its first use; every successful call leaves it that way,
 * and a call that reports an error through error_flag may not, so clear it
 * again after one. error_flag (may be NULL; device memory or host memory
 * mapped into the device address space) receives a nonzero code when a
 * bounded pipeline wait gave up. */
int jfb_matmul_tc_supported(const jfb_weight * weight);

/* Output segments of one tensor-core launch over a weight whose rows stack
 * several matrices (fused Q/K/V, gate/up): rows [previous row_end, row_end)
 * are written to `out` [n][segment rows] with their own epilogue, bias
 * [segment rows] and residual [n][segment rows]. */
typedef struct jfb_matmul_segment {
    uint32_t row_end;
    uint32_t epilogue;
    const float * bias;
    const float * residual;
    float * out;
} jfb_matmul_segment;
#define JFB_MATMUL_MAX_SEGMENTS 4
uint64_t jfb_matmul_tc_workspace_bytes(uint32_t rows, uint32_t cols, uint32_t n);
jfb_status jfb_matmul_tc(const jfb_weight * weight, const jfb_q8k * x_q8, uint32_t n, uint32_t epilogue,
                         const float * bias, const float * residual, float * out, void * workspace,
                         uint64_t workspace_bytes, int32_t * error_flag, void * stream);
/* The same with 1..JFB_MATMUL_MAX_SEGMENTS output segments (the last
 * segment's row_end must be weight->rows). */
jfb_status jfb_matmul_tc_segments(const jfb_weight * weight, const jfb_q8k * x_q8, uint32_t n,
                                  const jfb_matmul_segment * segments, uint32_t segment_count, void * workspace,
                                  uint64_t workspace_bytes, int32_t * error_flag, void * stream);

/* A view of rows [row_begin, row_begin + rows) of a K-quant weight: the same
 * device planes offset to that row range (planes are row-major), no copy. */
jfb_status jfb_weight_row_view(const jfb_weight * weight, uint32_t row_begin, uint32_t rows, jfb_weight * view);

/* NEOX rotary embedding of q and k plus the F16 KV-cache append
 * (ggml_rope_ext NEOX + ggml_set_rows, qwen2_architecture.cpp:400-424,
 * 499-506). Row r belongs to slots[seq[r]] at absolute position pos[r]; its K
 * and V rows are written at [layer][pos[r]] of that slot. q is rotated in
 * place. rope_table holds (cos, sin) pairs [table_positions][rope_dims/2]:
 * GGML's rope cache values, angle_i = pos * theta_scale^i built by repeated
 * float multiplication, theta_scale = powf(freq_base, -2/rope_dims), computed
 * once on the host with the C library's cosf/sinf (the functions GGML-CPU
 * calls), so device and CPU rotate with identical coefficients. */
jfb_status jfb_rope_kv_append(float * q, const float * k, const float * v, uint32_t n, const int32_t * seq,
                              const int32_t * pos, uint32_t heads, uint32_t kv_heads, uint32_t head_dim,
                              uint32_t rope_dims, const float * rope_table, uint32_t table_positions,
                              const jfb_kv_slot * slots, uint32_t layer, void * stream);

/* Host helper: fills table[positions][rope_dims/2][2] with GGML's rope cache
 * (cosf/sinf of pos * theta_scale^i, angles by repeated multiplication). */
void jfb_rope_table_host(float * table, uint32_t positions, uint32_t rope_dims, float freq_base);

/* Scratch bytes jfb_attention's four-launch form needs for n query rows with
 * at most max_keys keys each (UINT64_MAX beyond 65535 * 64 keys, which no
 * call supports). */
uint64_t jfb_attention_scratch_bytes(uint32_t n, uint32_t heads, uint32_t head_dim, uint32_t max_keys);

/* Scratch bytes one jfb_attention call with these dimensions needs on the
 * current device: 0 when the call runs as the single launch (no scratch
 * read or written; scratch may then be NULL), else
 * jfb_attention_scratch_bytes. Lets a caller size its scratch per call
 * instead of for the worst case. */
uint64_t jfb_attention_call_scratch_bytes(uint32_t n, uint32_t heads, uint32_t kv_heads, uint32_t head_dim,
                                          uint32_t max_keys);

/* Causal GQA attention of query rows over the F16 caches
 * (qwen2_architecture.cpp:425-470, GGML-CPU semantics of the unfused path):
 * row r attends keys [0, pos[r]] of slots[seq[r]] at `layer`; query head h
 * reads kv head h / (heads / kv_heads); scores are K . f16(q) with the exact
 * f16 products summed in double and rounded to f32 once; x = score *
 * 1/sqrt(head_dim); softmax with exp(x - max) summed in double over all keys,
 * p = e * (float)(1/sum) rounded to f16; output = exact p*v products summed
 * in double, rounded once. One launch on the FP64 tensor cores where the
 * shape allows (no scratch used), else four launches: scores (+chunk maxima),
 * row statistics, P V partials, combine (+Q8_K quantization of the result
 * when out_q8 != NULL). max_keys above 65535 * 64 is rejected; a row whose
 * pos[r] + 1 exceeds max_keys is clamped to the keys the call was sized for. */
jfb_status jfb_attention(const float * q, uint32_t n, const int32_t * seq, const int32_t * pos, uint32_t heads,
                         uint32_t kv_heads, uint32_t head_dim, uint32_t max_keys, const jfb_kv_slot * slots,
                         uint32_t layer, void * scratch, uint64_t scratch_bytes, float * out,
                         const jfb_q8k * out_q8, void * stream);

/* Attention for callers that cannot allocate device memory.
 *
 * No counterpart in the reference. Same computation and arguments as
 * jfb_attention, minus the scratch buffer: the scratch comes from a
 * file-scope device array of JFB_ATTENTION_STATIC_SCRATCH_BYTES that every
 * GPU loading this library holds until the process exits. It serves callers
 * that may not call cudaMalloc at all: a stage hosted inside a process whose
 * device memory is owned by another allocator (a framework's caching pool
 * that must see every byte), or a latency-critical step where cudaMalloc's
 * implicit device synchronisation is not acceptable.
 *
 * The first call on a device looks up the array's device address
 * (cudaGetSymbolAddress, which may load the module); make that first call
 * before any stream capture. Calls that need more scratch than the array
 * holds (see jfb_attention_scratch_bytes) are rejected with
 * JFB_STATUS_INVALID_ARGUMENT. All calls on a device share the one array and
 * the array keeps the last call's contents; nothing in it needs to start at
 * zero (each call writes every scratch value before reading it). Calls whose
 * work overlaps on the GPU (different streams, or host threads without
 * ordering) race on the array. */
#define JFB_ATTENTION_STATIC_SCRATCH_BYTES (16u * 1024u * 1024u)
jfb_status jfb_attention_static_scratch(const float * q, uint32_t n, const int32_t * seq, const int32_t * pos,
                                        uint32_t heads, uint32_t kv_heads, uint32_t head_dim, uint32_t max_keys,
                                        const jfb_kv_slot * slots, uint32_t layer, float * out,
                                        const jfb_q8k * out_q8, void * stream);

/* First index of the maximum of each row (ggml_argmax, qwen2_architecture.cpp:594). */
jfb_status jfb_argmax(const float * logits, uint32_t n, uint32_t cols, int32_t * out, void * stream);

/* The reference F16 activation codec on the device, bit-exact with
 * runtime/activation/builtin_activation_codecs.cpp:51-137 (round to nearest
 * even, NaN payload kept and made quiet). */
jfb_status jfb_codec_f32_to_f16(const float * in, uint16_t * out, uint64_t count, void * stream);
jfb_status jfb_codec_f16_to_f32(const uint16_t * in, float * out, uint64_t count, void * stream);

#ifdef __cplusplus
}
#endif

#endif
