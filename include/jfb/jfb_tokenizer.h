/*
 * C ABI of the package tokenizer (include/jetsonfabric/tokenizer.hpp) for FFI
 * callers: the three operations of the reference's tokenizer interface
 * (runtime/tokenization/tokenizer.hpp:9-16) over an opaque handle.
 */
#ifndef JFB_TOKENIZER_H
#define JFB_TOKENIZER_H

#include <stddef.h>
#include <stdint.h>

#include "jfb/jfb_status.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct jfb_tokenizer jfb_tokenizer;

/* Opens the tokenizer of the JFM package directory `package_dir`
 * (its metadata.gguf). */
jfb_status jfb_tokenizer_open(const char * package_dir, jfb_tokenizer ** out);

void jfb_tokenizer_close(jfb_tokenizer * tokenizer);

/* Tokens of `text` (`length` bytes of UTF-8), special tokens parsed and the
 * BOS/EOS added as the vocabulary asks. Writes min(count, capacity) ids to
 * `tokens` and the full count to *count; a capacity below the count is not an
 * error (call again with a larger buffer). Text that yields no tokens is
 * JFB_STATUS_INVALID_ARGUMENT. */
jfb_status jfb_tokenizer_tokenize(const jfb_tokenizer * tokenizer, const char * text, size_t length, int32_t * tokens,
                                  size_t capacity, size_t * count);

/* The bytes the token stands for (special tokens as their text). Writes
 * min(length, capacity) bytes and the full length to *length. */
jfb_status jfb_tokenizer_token_piece(const jfb_tokenizer * tokenizer, int32_t token, char * piece, size_t capacity,
                                     size_t * length);

/* 1 for -1 and the vocabulary's end-of-generation tokens, else 0. */
int jfb_tokenizer_is_end_token(const jfb_tokenizer * tokenizer, int32_t token);

#ifdef __cplusplus
}
#endif

#endif
