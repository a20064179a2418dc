/*
 * Packed GGUF tensor view, declared with the same name, field order and types
 * as the reference engine's `GgufQuantizedTensorView`
 * (src/gguf_reader.h:31-40) so that a pointer built by the reference's
 * `gguf_get_quantized_tensor_view` (src/gguf_reader.cpp:573-637) can be passed
 * to this library unchanged.  The GGML type ids match src/gguf_reader.h:7-11.
 *
 * When this library is linked into the reference build, include the
 * reference's own gguf_reader.h instead: define GGUF_READER_H before this
 * header, or include gguf_reader.h first, and this declaration is skipped.
 */
#ifndef QMV_GGUF_QUANTIZED_VIEW_H
#define QMV_GGUF_QUANTIZED_VIEW_H

#include <stdint.h>

#ifndef GGUF_READER_H
#define ENGINE_GGML_TYPE_F32 0u
#define ENGINE_GGML_TYPE_Q5_0 6u
#define ENGINE_GGML_TYPE_Q8_0 8u
#define ENGINE_GGML_TYPE_Q4_K 12u
#define ENGINE_GGML_TYPE_Q6_K 14u

/* Read-only packed data.  dimensions[0] = columns, dimensions[1] = rows. */
typedef struct GgufQuantizedTensorView {
    const unsigned char *data;  /* first packed byte; only byte-aligned */
    uint32_t ggml_type;         /* ENGINE_GGML_TYPE_* */
    uint32_t dimension_count;   /* 2 for a matrix */
    uint64_t dimensions[4];
    uint64_t element_count;     /* columns * rows */
    uint64_t block_elements;    /* 32 (Q5_0, Q8_0) or 256 (Q4_K, Q6_K) */
    uint64_t block_bytes;       /* 22, 34, 144 or 210 */
    uint64_t block_count;       /* element_count / block_elements */
} GgufQuantizedTensorView;
#endif

#endif
