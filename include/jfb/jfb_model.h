/*
 * Model-package side of the jetsonfabric_b200 C ABI (host only, no CUDA):
 * the GGUF importer and the seeded synthetic Qwen2 package writer used by
 * tests and the benchmark.
 *
 * The reference builds test packages with a GGML-based GGUF fixture writer
 * (runtime/compiler/model_fixture.cpp:76-133) and converts real models with a
 * GGML-based importer (runtime/compiler/jf_model_compile.cpp:547-645). Neither
 * can be built without GGML. These entry points write JFM v2 packages
 * directly: GGUF metadata segment, an optional shared segment, one input, one
 * output and one segment per layer, with the manifest hashes the loader
 * verifies.
 */
#ifndef JFB_MODEL_H
#define JFB_MODEL_H

#include <stddef.h>
#include <stdint.h>

#include "jfb/jfb_status.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef enum jfb_synth_kind {
    /* Seeded N(0, weight_std) weights quantized with this library's K-quant
     * encoders. */
    JFB_SYNTH_RANDOM = 0,
    /* The reference's 2-layer constant F32 fixture: hidden 4, FFN 8, one
     * head, context 16, vocabulary 8; token_embd rows 0.1*(row+1), output rows
     * 0.01*(row+1), layer matrices 0.01, norms 1, biases 0
     * (runtime/compiler/model_fixture.cpp:76-133). Dimension fields of the
     * spec are ignored. */
    JFB_SYNTH_REFERENCE_FIXTURE = 1,
} jfb_synth_kind;

typedef struct jfb_synth_spec {
    uint32_t kind;                 /* jfb_synth_kind */
    uint32_t layer_count;
    uint32_t embedding_length;
    uint32_t head_count;
    uint32_t kv_head_count;
    uint32_t feed_forward_length;
    uint32_t vocabulary_size;
    uint32_t context_length;
    float rope_freq_base;
    float rms_epsilon;
    /* JFM type ids (JF_TENSOR_*): F32, F16, Q2_K, Q4_K or Q6_K. */
    uint32_t layer_type;
    uint32_t embedding_type;
    uint32_t output_type;
    /* 1: Q6_K attn_v and ffn_down on the "more bits" layers
     * (i < L/8 || i >= 7L/8 || (i - L/8) % 3 == 2), the Q4_K_M recipe. */
    uint32_t more_bits_q6k;
    uint64_t seed;
    float weight_std;
    /* 0: norms are 1.0; 1: norms are 1 + N(0, weight_std). */
    uint32_t draw_norms;
    /* 0: biases are 0; 1: biases are N(0, weight_std). */
    uint32_t draw_biases;
    uint32_t threads;              /* 0 = hardware concurrency */
} jfb_synth_spec;

typedef struct jfb_synth_report {
    uint64_t weight_bytes;         /* sum of tensor payload bytes */
    uint64_t tensor_count;
    uint64_t file_bytes;           /* sum of segment file sizes */
} jfb_synth_report;

/* Writes a complete JFM v2 package into `directory` (created if missing;
 * existing package files are overwritten). */
jfb_status jfb_write_synthetic_package(
    const jfb_synth_spec * spec,
    const char * directory,
    jfb_synth_report * report
);

typedef struct jfb_import_report {
    uint32_t layer_count;
    uint32_t reserved;
    uint64_t tensor_count;
    uint64_t tensor_bytes;         /* sum of tensor payload bytes */
    uint64_t package_bytes;        /* every package file, manifest included */
    uint8_t source_sha256[32];
    char architecture[64];         /* general.architecture, NUL-terminated */
} jfb_import_report;

/* Converts an unsplit GGUF (v2 or v3) into a new JFM v2 package directory
 * `package_dir`, replacing the reference's jf-model-compile
 * (runtime/compiler/jf_model_compile.cpp:547-645): the same segment
 * assignment, byte layout and manifest, built in an exclusive staging
 * directory next to the output and published by one no-replace rename.
 * Fails (and leaves nothing behind) if the output exists, the source is not a
 * regular file, the GGUF is malformed or split, a tensor type has no JFM v2
 * geometry, a layer or the input has no tensors, output.weight is missing
 * (tied embeddings), or the source changes while it is being read.
 * `report` may be NULL. */
jfb_status jfb_import_gguf(const char * gguf_path, const char * package_dir, jfb_import_report * report);

/* Encodes `count` floats (a multiple of 256) into GGML K-quant blocks of the
 * given JFM type (Q2_K, Q4_K or Q6_K) with this library's encoders. Exposed so
 * tests can build quantized tensors without writing a package. */
jfb_status jfb_quantize_blocks(
    uint32_t type,
    const float * values,
    size_t count,
    void * blocks,
    size_t blocks_capacity
);

#ifdef __cplusplus
}
#endif

#endif
