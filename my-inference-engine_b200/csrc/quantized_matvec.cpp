// Drop-in replacement for the reference engine's src/quantized_matvec.cpp.
//
// Same C++ signatures as src/quantized_matvec.h:32-50, so the reference's
// callers (qwen2_weight_matvec / qwen2_weight_matmul,
// src/qwen2_architecture.cpp:605, :612, :686) link against it unchanged.  The
// work runs on the current CUDA device through the C ABI (qmv_b200.h); there
// is no CPU fallback: a missing or failing device makes the call return 0.
#include "quantized_matvec.h"

#include "qmv_b200.h"

__attribute__((visibility("default"))) int quantized_tensor_matvec_f32(
    const GgufQuantizedTensorView *matrix, const float *input, int input_count, float *output,
    int output_count)
{
    return qmv_quantized_tensor_matvec_f32(matrix, input, input_count, output, output_count);
}

__attribute__((visibility("default"))) int quantized_tensor_matmul_f32(
    const GgufQuantizedTensorView *matrix, const float *inputs, int input_count, int batch_count,
    float *outputs, int output_count)
{
    return qmv_quantized_tensor_matmul_f32(matrix, inputs, input_count, batch_count, outputs,
                                           output_count);
}
