/*
 * Drop-in replacement for the reference engine's src/quantized_matvec.h.
 *
 * The two functions keep the reference's exact C++ signatures
 * (src/quantized_matvec.h:32-38 and :42-50), argument meaning, validation and
 * 0/1 return convention (src/quantized_matvec.cpp:86-149, :164-191).  They are
 * implemented in my-inference-engine_b200/csrc/quantized_matvec.cpp on top of
 * the B200 C-ABI in qmv_b200.h:
 *
 *   - the packed tensor behind matrix->data is uploaded to the current CUDA
 *     device on first use and kept resident (keyed by matrix->data, shape and
 *     type), exactly once per process;
 *   - input/output stay host pointers: each call copies the input to the
 *     device, runs the sm_100a kernel, and copies the output back before it
 *     returns;
 *   - on any CUDA error the call returns 0 (never aborts) and
 *     qmv_last_error() holds the message.
 *
 * A caller that keeps activations on the device uses qmv_matvec/qmv_matmul
 * from qmv_b200.h instead.
 */
#ifndef QUANTIZED_MATVEC_H
#define QUANTIZED_MATVEC_H

#include "gguf_quantized_view.h"

/* y[row] = sum over blocks of block_dot(W[row, b], input[b-slice]);
 * input_count == dimensions[0], output_count == dimensions[1].
 * Returns 1 on success, 0 for invalid arguments/views or a device error. */
int quantized_tensor_matvec_f32(
    const GgufQuantizedTensorView *matrix,
    const float *input,
    int input_count,
    float *output,
    int output_count
);

/* outputs[p, row] for p < batch_count; inputs [batch_count, input_count]
 * token-major, outputs [batch_count, output_count]. */
int quantized_tensor_matmul_f32(
    const GgufQuantizedTensorView *matrix,
    const float *inputs,
    int input_count,
    int batch_count,
    float *outputs,
    int output_count
);

#endif
