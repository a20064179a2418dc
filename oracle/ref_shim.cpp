// TEST INFRASTRUCTURE ONLY — compiled together with the reference engine's own
// hot-path sources (src/quantization.cpp, src/quantized_matvec.cpp,
// src/sampler.cpp, read in place from the reference checkout) by
// oracle/Makefile into oracle/_ref/.  It exposes the reference functions under
// plain C names so the Python tests can call the reference itself through
// ctypes.  Nothing in the product links this file.
#include <stdint.h>
#include <string.h>

#include "gguf_reader.h"
#include "quantization.h"
#include "quantized_matvec.h"
#include "sampler.h"

#ifdef _OPENMP
#include <omp.h>
#endif

extern "C" {

int ref_f16_to_f32(uint16_t bits, float *out) { return f16_bits_to_f32(bits, out); }

static int block_shape(uint32_t type, uint64_t *be, uint64_t *bb)
{
    switch (type) {
    case ENGINE_GGML_TYPE_Q5_0: *be = Q5_0_BLOCK_ELEMENTS; *bb = Q5_0_BLOCK_BYTES; return 1;
    case ENGINE_GGML_TYPE_Q8_0: *be = Q8_0_BLOCK_ELEMENTS; *bb = Q8_0_BLOCK_BYTES; return 1;
    case ENGINE_GGML_TYPE_Q4_K: *be = Q4_K_BLOCK_ELEMENTS; *bb = Q4_K_BLOCK_BYTES; return 1;
    case ENGINE_GGML_TYPE_Q6_K: *be = Q6_K_BLOCK_ELEMENTS; *bb = Q6_K_BLOCK_BYTES; return 1;
    default: return 0;
    }
}

// Dequantize nblocks raw blocks with the reference's *_dequantize_block.
int ref_dequant_blocks(uint32_t type, const unsigned char *data, uint64_t nblocks, float *out)
{
    uint64_t be, bb;
    if (!block_shape(type, &be, &bb)) return 0;
    for (uint64_t b = 0; b < nblocks; b++) {
        const unsigned char *p = data + b * bb;
        float *o = out + b * be;
        int ok = 0;
        switch (type) {
        case ENGINE_GGML_TYPE_Q5_0: { Q5_0Block k; memcpy(&k, p, sizeof k); ok = q5_0_dequantize_block(&k, o); break; }
        case ENGINE_GGML_TYPE_Q8_0: { Q8_0Block k; memcpy(&k, p, sizeof k); ok = q8_0_dequantize_block(&k, o); break; }
        case ENGINE_GGML_TYPE_Q4_K: { Q4_KBlock k; memcpy(&k, p, sizeof k); ok = q4_k_dequantize_block(&k, o); break; }
        case ENGINE_GGML_TYPE_Q6_K: { Q6_KBlock k; memcpy(&k, p, sizeof k); ok = q6_k_dequantize_block(&k, o); break; }
        }
        if (!ok) return 0;
    }
    return 1;
}

// One block dot with the reference's *_dot_f32.
int ref_block_dot(uint32_t type, const unsigned char *blk, const float *x, float *out)
{
    switch (type) {
    case ENGINE_GGML_TYPE_Q5_0: { Q5_0Block k; memcpy(&k, blk, sizeof k); return q5_0_dot_f32(&k, x, out); }
    case ENGINE_GGML_TYPE_Q8_0: { Q8_0Block k; memcpy(&k, blk, sizeof k); return q8_0_dot_f32(&k, x, out); }
    case ENGINE_GGML_TYPE_Q4_K: { Q4_KBlock k; memcpy(&k, blk, sizeof k); return q4_k_dot_f32(&k, x, out); }
    case ENGINE_GGML_TYPE_Q6_K: { Q6_KBlock k; memcpy(&k, blk, sizeof k); return q6_k_dot_f32(&k, x, out); }
    default: return 0;
    }
}

int ref_q4_k_unpack_scale_min(const uint8_t *sm, int j, uint8_t *sc, uint8_t *mn)
{
    return q4_k_unpack_scale_min(sm, j, sc, mn);
}

int ref_q6_k_unpack_value(const unsigned char *blk, int index, int8_t *q, int8_t *sc)
{
    Q6_KBlock k;
    memcpy(&k, blk, sizeof k);
    return q6_k_unpack_value(&k, index, q, sc);
}

// The reference's matvec/matmul entry points, called with a caller-built view
// (so tests can hand both implementations the same invalid views).
int ref_matvec_view(const GgufQuantizedTensorView *view, const float *x, int xn, float *y, int yn)
{
    return quantized_tensor_matvec_f32(view, x, xn, y, yn);
}

int ref_matmul_view(const GgufQuantizedTensorView *view, const float *X, int xn, int batch,
                    float *Y, int yn)
{
    return quantized_tensor_matmul_f32(view, X, xn, batch, Y, yn);
}

static GgufQuantizedTensorView make_view(uint32_t type, const unsigned char *data, int rows, int cols)
{
    GgufQuantizedTensorView v;
    memset(&v, 0, sizeof v);
    uint64_t be = 0, bb = 0;
    block_shape(type, &be, &bb);
    v.data = data;
    v.ggml_type = type;
    v.dimension_count = 2;
    v.dimensions[0] = (uint64_t)cols;
    v.dimensions[1] = (uint64_t)rows;
    v.element_count = (uint64_t)cols * (uint64_t)rows;
    v.block_elements = be;
    v.block_bytes = bb;
    v.block_count = be ? v.element_count / be : 0;
    return v;
}

int ref_matvec(uint32_t type, const unsigned char *data, int rows, int cols, const float *x, float *y)
{
    GgufQuantizedTensorView v = make_view(type, data, rows, cols);
    return quantized_tensor_matvec_f32(&v, x, cols, y, rows);
}

int ref_matmul(uint32_t type, const unsigned char *data, int rows, int cols, const float *X,
               int batch, float *Y)
{
    GgufQuantizedTensorView v = make_view(type, data, rows, cols);
    return quantized_tensor_matmul_f32(&v, X, cols, batch, Y, rows);
}

int ref_greedy(const float *logits, int n, int *id, char *err, int cap)
{
    return sampler_greedy_sample(logits, n, id, err, cap);
}

int ref_set_threads(int n)
{
#ifdef _OPENMP
    omp_set_dynamic(0);
    omp_set_num_threads(n);
    return omp_get_max_threads();
#else
    (void)n;
    return 1;
#endif
}

int ref_view_size(void) { return (int)sizeof(GgufQuantizedTensorView); }

}  // extern "C"
