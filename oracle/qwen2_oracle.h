/*
 * CPU ORACLE — TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the reference native engine's Qwen2 stage forward
 * (runtime/engines/native/src/qwen2_architecture.cpp:361-598) with the op
 * semantics of GGML's CPU backend, which the reference runs it on. It is the
 * parity checker for the CUDA engine and the timed CPU baseline; nothing in
 * the product links, loads or calls it. Only tests/, __graft_entry__.smoke()
 * and bench.py's CPU-baseline leg may use it.
 *
 * GGML itself (llama.cpp bf2c86ddc0685f580595954056c2e77ebabfab4f) is not
 * vendored in the reference and cannot be fetched here, so each GGML-CPU
 * semantic below is restated from the published K-quant formats and op
 * definitions and cited at its use site in qwen2_oracle.c.
 */
#ifndef QWEN2_ORACLE_H
#define QWEN2_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* A tensor in its on-disk (GGML block) encoding; type is the JFM type id. */
typedef struct orc_tensor {
    uint32_t type;
    uint32_t pad_;
    uint64_t ne0;           /* elements along the input dimension */
    uint64_t ne1;           /* rows */
    const void * data;      /* NULL when absent (optional tensors) */
} orc_tensor;

typedef struct orc_layer {
    orc_tensor attn_norm, attn_q, attn_q_bias, attn_k, attn_k_bias, attn_v, attn_v_bias,
        attn_output, ffn_norm, ffn_gate, ffn_up, ffn_down;
} orc_layer;

typedef struct orc_model {
    uint32_t layer_count;
    uint32_t embedding_length;
    uint32_t head_count;
    uint32_t kv_head_count;
    uint32_t feed_forward_length;
    uint32_t context_length;
    uint32_t vocabulary_size;
    uint32_t rope_dimension_count;
    float rope_freq_base;
    float rms_epsilon;
    uint32_t layer_start;
    uint32_t layer_end;
    orc_tensor token_embd;    /* first stage only */
    orc_tensor output_norm;   /* last stage only */
    orc_tensor output;        /* last stage only */
    orc_tensor output_bias;   /* optional */
    const orc_layer * layers; /* layer_end - layer_start entries */
} orc_model;

typedef struct orc_session orc_session;

void orc_set_threads(int threads);

/* ---- primitives (exposed for unit tests) ---- */
void orc_dequantize_row(uint32_t type, const void * src, float * dst, int64_t k);
/* GGML block_q8_K: float d, int8 qs[256], int16 bsums[16]  (292 bytes) */
void orc_quantize_row_q8_k(const float * x, void * blocks, int64_t k);
/* One row of nb K-quant blocks (type 9, 11 or 13) times nb Q8_K blocks: the
 * readable scalar loops and the vectorised path orc_matmul runs. The two must
 * agree bit for bit (the integer sums are exact in any order). */
float orc_dot_kquant_scalar(uint32_t type, const void * w, const void * a, int64_t nb);
float orc_dot_kquant_vector(uint32_t type, const void * w, const void * a, int64_t nb);
size_t orc_q8k_block_bytes(void);
/* y[r * ne1 + n] = sum_k W[n, k] * x[r * ne0 + k] with GGML-CPU mul_mat semantics */
void orc_matmul(const orc_tensor * w, const float * x, int64_t rows, float * y);
void orc_rms_norm(const float * x, const float * weight, int64_t n, float eps, float * y);
void orc_rope_neox(float * x, int64_t heads, int64_t head_length, int64_t dims, int32_t position,
                   float freq_base);
int32_t orc_argmax(const float * x, int64_t n);
uint16_t orc_f32_to_f16(float value);
/* exp by Cody-Waite reduction + degree-7 Taylor polynomial (see the .c file) */
float orc_expf(float x);
float orc_silu_mul(float g, float u);
/* Attention of one query row (heads*head_dim floats, already rotated) at
 * absolute position pos over token-major f16 caches [pos+1][kv_heads*head_dim]. */
void orc_attention_row(const float * q, const uint16_t * k_cache, const uint16_t * v_cache, int64_t pos,
                       int64_t heads, int64_t kv_heads, int64_t head_dim, float * out);
float orc_f16_to_f32(uint16_t value);
/* The reference's F16 activation codec (builtin_activation_codecs.cpp:51-137). */
uint16_t orc_codec_float_to_half(float value);
float orc_codec_half_to_float(uint16_t value);

/* ---- stage sessions ---- */
orc_session * orc_session_create(const orc_model * model, size_t capacity);
void orc_session_destroy(orc_session * session);
size_t orc_session_position(const orc_session * session);
size_t orc_session_capacity(const orc_session * session);
/* 0 on success, -1 when token_count is outside the decoded suffix. */
int orc_session_rollback(orc_session * session, size_t token_count);

/*
 * Runs n rows through the stage. prefill=1 requires position 0 and leaves the
 * position at n; prefill=0 is one decode row (n == 1) at the current position.
 * The first stage takes tokens, later stages take f32 activations [n, h].
 * Non-final stages write activations [n, h] to out_activations. The final
 * stage writes the last row's logits (if out_logits) and its greedy token.
 * Returns 0, or -1 with a message (invalid input, like std::invalid_argument).
 */
int orc_session_forward(orc_session * session, int prefill, const int32_t * tokens,
                        const float * activations, size_t n, float * out_activations,
                        float * out_logits, int32_t * out_token, char * error, size_t error_size);

#ifdef __cplusplus
}
#endif

#endif
