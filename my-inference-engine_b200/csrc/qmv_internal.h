// Internal interface between the C ABI (qmv_capi.cpp) and the sm_100a kernels
// (qmv_kernels.cu).  Not installed; no torch or CUDA types leak into the
// public headers.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace qmv {

enum : uint32_t { kQ5_0 = 6u, kQ8_0 = 8u, kQ4_K = 12u, kQ6_K = 14u };

// Largest column count the kernels stage in shared memory (x is quantized to
// 2.375 B/column per position): 65536 columns = 152 KiB for one position.
constexpr int kMaxCols = 65536;
// Upper bound on CTAs of one argmax-producing launch (size of the workspace
// key array).
constexpr int kMaxArgmaxCtas = 2048;
constexpr size_t kArgmaxWorkspaceBytes = 16 + 8 * (size_t)kMaxArgmaxCtas;

// Device layout of one resident tensor.  Rows are contiguous and every row
// starts on a 16-byte boundary; the odd-sized fp16 block scales of Q8_0, Q5_0
// and Q6_K are moved to the end of their row so the quant payload can be read
// with 128-bit loads:
//   Q8_0 row: qs[32*nb] | d[nb] (fp16, padded to 16 B)
//   Q5_0 row: qs[16*nb] | qh[4*nb] (padded) | d[nb] (padded)
//   Q4_K row: raw 144-byte blocks (already 9 x 16 B)
//   Q6_K row: {ql[128] qh[64] sc[16]}[nb] (208 B each) | d[nb] (padded)
struct Layout {
    uint32_t type;
    int rows;
    int cols;
    int nb;               // blocks per row
    uint64_t row_stride;  // bytes, multiple of 16
    uint32_t off_qh;      // Q5_0 qh segment
    uint32_t off_d;       // Q8_0/Q5_0/Q6_K fp16 scale segment
};

int block_elements(uint32_t type);
int block_bytes(uint32_t type);
bool make_layout(uint32_t type, int rows, int cols, Layout *out);

// raw (device, byte-aligned) GGUF blocks of `rows` rows -> layout.
cudaError_t launch_repack(const Layout &L, const uint8_t *raw, uint8_t *dst, cudaStream_t s);
// Bit-exact dequant of a resident tensor into out[rows*cols].
cudaError_t launch_dequant_layout(const Layout &L, const uint8_t *w, float *out, cudaStream_t s);
// Bit-exact dequant of raw device blocks.
cudaError_t launch_dequant_raw(uint32_t type, const uint8_t *raw, uint64_t nblocks, float *out,
                               cudaStream_t s);

// Argmax output of a launch (all device pointers; workspace from the caller).
struct ArgmaxOut {
    unsigned long long *key;  // final key
    void *workspace;          // kArgmaxWorkspaceBytes, zeroed once
    int index_base;           // global index of row 0
};

// y = W x (and optionally the argmax key of y).
cudaError_t launch_gemv(const Layout &L, const uint8_t *w, const float *x, float *y,
                        const ArgmaxOut *am, cudaStream_t s);
// Y[p] = W X[p], p < batch.
cudaError_t launch_matmul(const Layout &L, const uint8_t *w, const float *X, int batch, float *Y,
                          cudaStream_t s);
// Argmax key of logits[0..n).
cudaError_t launch_argmax(const float *logits, int n, const ArgmaxOut &am, cudaStream_t s);

}  // namespace qmv
