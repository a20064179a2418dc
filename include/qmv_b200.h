/*
 * qmv_b200 — C ABI of the B200 (sm_100a) quantized matrix-vector library.
 *
 * Plain C types only: pointers, sizes, ints.  CUDA streams are passed as
 * `void *` (a cudaStream_t / CUstream; NULL = the legacy default stream).
 * Every function returns 1 on success and 0 on failure; on failure
 * qmv_last_error() (per calling thread) holds a one-line message.  No
 * function aborts the process.
 *
 * Citations name the reference engine's interface each entry point replaces
 * or backs (paths inside trungnguyen21/my-inference-engine).
 */
#ifndef QMV_B200_H
#define QMV_B200_H

#include <stddef.h>
#include <stdint.h>

#include "gguf_quantized_view.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Device-resident packed tensor (opaque). */
typedef struct QmvWeight QmvWeight;

/* ---- errors, devices ---------------------------------------------------- */

/* Last error of the calling thread ("" if none).  Replaces the reference's
 * set_error/error-buffer convention (src/sampler.cpp:7-12,
 * src/qwen2_architecture.cpp:62-67) for the device path. */
const char *qmv_last_error(void);

/* Copy the last error into buf (always NUL-terminated when capacity > 0). */
int qmv_copy_last_error(char *buf, int capacity);

/* Library ABI version (increments on any signature change). */
int qmv_abi_version(void);

/* Number of visible CUDA devices. */
int qmv_device_count(int *count);

/* Make `device` current for the calling thread (all later calls of this
 * thread allocate and launch there). */
int qmv_set_device(int device);

/* Device status of the current device: bit 0 = a consumer's pipeline wait
 * expired, bit 1 = a producer's wait expired, bit 2 = draining in-flight
 * copies timed out, bit 3 = a peer's exchange flag never arrived, bit 4 = a
 * tensor-core matmul's wait for its MMAs expired.  0 means every bounded
 * wait completed.  clear != 0 resets the word.  No counterpart in the reference (its kernels never wait). */
int qmv_device_status(uint32_t *flags, int clear);

/* GEMV kernel selection for the calling process: 0 = automatic (the
 * resident-row-range kernel when one CTA's rows fit in its shared memory
 * whole -- a small CTA, so the CTAs of the next launches of a stream are
 * resident beside it and copy their weights while it computes -- else the
 * TMA bulk-copy pipeline with the exclusive plan when its shared-memory
 * stages fit, direct loads otherwise),
 * 1 = direct loads, 2 = TMA pipeline only (shapes it cannot stage fail),
 * 3 = the exclusive TMA plan (one CTA per SM using all of its shared
 * memory; direct loads where no stages fit), 4 = the shared TMA plan where
 * its stages fit in half an SM (a CTA that leaves half of the SM to the next
 * launch, so consecutive launches overlap), else as 3, 5 = the
 * resident-row-range kernel only (shapes it cannot hold fail).  No
 * counterpart in the reference; every path computes the same function. */
int qmv_set_gemv_path(int path);

/* Batched-matmul kernel selection for the calling process: 0 = automatic
 * (tensor cores, tcgen05 with bf16 hi/lo operand splits and fp32
 * accumulation, from 32 positions when X is 16-byte aligned; CUDA-core dp4a
 * kernel otherwise), 1 = CUDA cores only, 2 = tensor cores only (a misaligned
 * X then fails), 64 / 128 / 176 / 256 = tensor cores with that many positions
 * per tile (normally chosen from the shape).  No counterpart in the
 * reference; all paths compute the same function within the parity bound. */
int qmv_set_matmul_path(int path);

/* ---- residency of packed tensors ----------------------------------------
 * Backs the packed-weight source of the reference: the borrowed mmap views
 * returned by gguf_get_quantized_tensor_view (src/gguf_reader.cpp:573-637,
 * struct src/gguf_reader.h:31-40).  Validation follows
 * src/quantized_matvec.cpp:94-149. */

/* Upload rows [row_begin, row_end) of `view` to the current device, repacked
 * into 16-byte-aligned rows.  row_begin = 0, row_end = rows uploads the whole
 * tensor; a sub-range is one rank's shard of a row-partitioned projection. */
int qmv_weight_upload(const GgufQuantizedTensorView *view, int row_begin, int row_end,
                      QmvWeight **out);

/* Free a weight from qmv_weight_upload (not one owned by the registry). */
int qmv_weight_free(QmvWeight *weight);

/* Shape of a resident weight.  Any output pointer may be NULL. */
int qmv_weight_info(const QmvWeight *weight, uint32_t *ggml_type, int *rows, int *cols,
                    int *row_begin, uint64_t *device_bytes);

/* Registry lookup-or-upload keyed by (view->data, type, shape) on the current
 * device; thread-safe, uploads once.  The registry owns the weight. */
int qmv_resident_weight(const GgufQuantizedTensorView *view, QmvWeight **out);

/* Free every registry-owned weight (no call may be using them). */
int qmv_resident_release_all(void);

/* ---- compute on device buffers ----------------------------------------- */

/* y = W x.  x: x_count floats (== columns), y: y_count floats (== rows of
 * this weight).  Device pointers.  Device form of quantized_tensor_matvec_f32
 * (src/quantized_matvec.h:32-38, src/quantized_matvec.cpp:86-162). */
int qmv_matvec(const QmvWeight *weight, const float *x, int x_count, float *y, int y_count,
               void *stream);

/* Y[p, :] = W X[p, :] for p < batch.  X: [batch, x_count], Y: [batch, y_count],
 * token-major, device pointers.  Device form of quantized_tensor_matmul_f32
 * (src/quantized_matvec.h:42-50, src/quantized_matvec.cpp:164-224). */
int qmv_matmul(const QmvWeight *weight, const float *X, int x_count, int batch, float *Y,
               int y_count, void *stream);

/* H[p, :] += W X[p, :] (the residual projections of the reference's prefill,
 * src/qwen2_architecture.cpp:1650-1655, :1679-1686): on the tensor cores from
 * 32 positions, with K split across CTAs when that fills more SMs and the
 * partial products summed into H in split order.  Device pointers. */
int qmv_matmul_residual(const QmvWeight *weight, const float *X, int x_count, int batch, float *H,
                        int h_count, void *stream);

/* Bit-exact dequantisation of a resident weight into out[rows * cols]
 * (row-major).  Same bits as the reference's *_dequantize_block
 * (src/quantization.cpp:54-67, 161-184, 380-409, 588-615). */
int qmv_dequantize(const QmvWeight *weight, float *out, uint64_t out_count, void *stream);

/* Bit-exact dequantisation of block_count raw GGUF blocks already in device
 * memory (any byte alignment) into out[block_count * block_elements].
 * Used for single rows such as an embedding lookup
 * (src/qwen2_architecture.cpp:375-475). */
int qmv_dequantize_raw(uint32_t ggml_type, const void *blocks, uint64_t block_count,
                       float *out, void *stream);

/* ---- greedy argmax -------------------------------------------------------
 * Argmax results are 64-bit keys: the high word orders the float value, the
 * low word is 0xFFFFFFFF - index, so the maximum key is the largest logit with
 * the lowest index on ties (src/sampler.cpp:29-31).  Any NaN/Inf makes the key
 * QMV_KEY_NONFINITE.  Keys combine across shards with an unsigned 64-bit max
 * (one NCCL all-reduce). */
#define QMV_KEY_NONFINITE 0xFFFFFFFFFFFFFFFFull

/* Bytes of device workspace the argmax entry points need (zero it once
 * before first use; the kernels leave it zeroed). */
size_t qmv_argmax_workspace_bytes(void);

/* *key (device) = argmax key of logits[0..n) with indices offset by
 * index_base.  Device form of sampler_greedy_sample (src/sampler.cpp:14-36). */
int qmv_argmax(const float *logits, int n, int index_base, uint64_t *key, void *workspace,
               void *stream);

/* Fused vocab projection + greedy argmax: logits = W x (device, y_count ==
 * rows of this weight) and *key (device) = argmax key over those rows with
 * indices offset by the weight's row_begin.  Output projection
 * (src/qwen2_architecture.cpp:1504-1523) followed by the sampler. */
int qmv_matvec_argmax(const QmvWeight *weight, const float *x, int x_count, float *logits,
                      int y_count, uint64_t *key, void *workspace, void *stream);

/* ---- row-sharded projection over peer memory (one node, 2..8 GPUs) -------
 * The vocabulary projection split by rows across ranks, one process per GPU
 * (the reference runs it on one CPU: src/qwen2_architecture.cpp:1504-1523 +
 * src/sampler.cpp:14-36).  Each rank owns an exchange buffer of
 * qmv_exchange_bytes() allocated with qmv_ipc_alloc: a 256-byte control block
 * (the rank's device-side step counter) and two parity regions
 * (logits[world * slot_rows] f32 | one argmax key and one flag per source
 * CTA).  The ranks share their IPC handles and open each other's with
 * qmv_ipc_open.  All ranks run the same GPU model. */

/* Bytes of one rank's exchange buffer. */
int qmv_exchange_bytes(int world, int slot_rows, size_t *bytes);

/* cudaMalloc + zero + IPC handle (64 bytes written to `handle`). */
int qmv_ipc_alloc(size_t bytes, void **dev_ptr, void *handle);
/* Map a peer's buffer from its 64-byte IPC handle / unmap it. */
int qmv_ipc_open(const void *handle, void **dev_ptr);
int qmv_ipc_close(void *dev_ptr);
/* Free a buffer from qmv_ipc_alloc. */
int qmv_ipc_free(void *dev_ptr);

/* Copy `bytes` between any host/device pointers (direction from unified
 * addressing) on `stream` and wait for it: reads exchange buffers, which are
 * raw device pointers owned by this library. */
int qmv_memcpy(void *dst, const void *src, size_t bytes, void *stream);

/* Gathered logits of the `epoch`-th call (1, 2, ...) inside a rank's own
 * buffer: logits[world * slot_rows], rank r's rows at r * slot_rows. */
int qmv_exchange_logits(void *buffer, int world, int slot_rows, uint32_t epoch, float **logits);

/* One kernel per rank: this rank's rows of W x (the weight must hold rows
 * [rank * slot_rows, ...)) and its argmax key.  Every CTA stores its logits
 * and its key into every rank's buffer over NVLink and release-stores its
 * flag there; the rank's last CTA waits (bounded) until every rank's CTAs of
 * this step have delivered and folds their keys.  The step counter lives in the
 * buffer (device side), so the call can be captured in a CUDA graph and
 * replayed.  On completion *key (device) is the global argmax key on every
 * rank and every rank's buffer holds all logits of the step.  `buffers` is a
 * host array of world device pointers (own + opened peers).  Read a step's
 * gathered logits on the same stream before the call after next.  A rank that
 * never arrives within 2 s leaves key 0 (no token) and sets bit 3 of
 * qmv_device_status. */
int qmv_matvec_argmax_exchange(const QmvWeight *weight, const float *x, int x_count, int rank, int world,
                               void *const *buffers, int slot_rows, uint64_t *key, void *workspace,
                               void *stream);

/* Greedy argmax that allocates nothing and needs no workspace: same result
 * as qmv_argmax, for callers that cannot call cudaMalloc -- for example a host
 * that owns every device allocation through its own pool and gives a plugin
 * only the logits and the key buffer.  No counterpart in the reference (its
 * sampler runs on the host).  The scratch is a static device array of
 * 16 + 8 * 2048 bytes, held on every GPU that loads this library until the
 * process exits, so n is limited to QMV_ARGMAX_NOALLOC_MAX_LOGITS; larger n
 * is rejected with an error.  The first call on a device looks up the array's
 * device address in that device's primary context (the CUDA runtime's) and
 * keeps it for the life of the process: make that first call before any
 * stream capture, and do not use this entry point after a cudaDeviceReset or
 * from a context other than the primary one.  All calls
 * on a device share the array: each call clears its counter first, and calls
 * that overlap on the GPU (e.g. on concurrent streams) race. */
#define QMV_ARGMAX_NOALLOC_MAX_LOGITS (2048 * 4096)
int qmv_argmax_noalloc(const float *logits, int n, int index_base, uint64_t *key, void *stream);

/* Host: decode a key into a token id.  Returns 0 (id = -1) for
 * QMV_KEY_NONFINITE or a key with no valid index. */
int qmv_key_to_token(uint64_t key, int *token_id);

/* Host-facing greedy sampler over DEVICE logits with the reference's contract
 * (src/sampler.h:4-13): synchronises `stream`, writes the id, and on failure
 * returns 0, sets *token_id = -1 when writable and fills `error`. */
int qmv_greedy_sample(const float *logits, int vocab_size, int *token_id, char *error,
                      int error_capacity, void *stream);

/* ---- drop-in entry points with C linkage ---------------------------------
 * Same arguments and results as the C++ functions in quantized_matvec.h
 * (host input/output; see there), for C/cgo/ctypes callers. */
int qmv_quantized_tensor_matvec_f32(const GgufQuantizedTensorView *matrix, const float *input,
                                    int input_count, float *output, int output_count);
int qmv_quantized_tensor_matmul_f32(const GgufQuantizedTensorView *matrix, const float *inputs,
                                    int input_count, int batch_count, float *outputs,
                                    int output_count);
/* Kernel-only timing of the calling thread's drop-in calls above, for the
 * reference's per-format weight profile (OperationProfile.weight_*_seconds,
 * include/metrics.h:15-20, filled around quantized_tensor_matvec_f32 at
 * src/qwen2_architecture.cpp:603-614): with profiling on, each call
 * brackets its kernels (not its host<->device copies) with CUDA events, and
 * qmv_last_kernel_seconds returns that device time of the latest call. */
int qmv_set_profiling(int enabled);
int qmv_last_kernel_seconds(double *seconds);

/* ---- device-resident Qwen2 decode step ------------------------------------
 * Replaces the Qwen2 implementation of ArchitectureOps.forward_token
 * (src/architecture.h:67-80, qwen2_forward_token_cached_impl
 * src/qwen2_architecture.cpp:1195-1531) with one GPU-resident step: embedding,
 * per layer RMSNorm + Q/K/V (+ biases) + RoPE + KV append + grouped-query
 * attention + output projection + residual + RMSNorm + SwiGLU FFN + residual,
 * then final RMSNorm, vocabulary projection and greedy argmax
 * (src/sampler.cpp:14-36).  The step is captured once in a CUDA graph; the
 * token and position live on the device, so generation replays the graph
 * without host round trips.  Head dimension 64 and at most 16 query heads per
 * KV head are supported.  Projections take the packed formats of this
 * library; results follow the parity bound of the matvec path per projection.
 * Calls on one decoder must not overlap. */
typedef struct QmvQwen2Config {
    int dim, hidden_dim, n_layers, n_heads, n_kv_heads, vocab_size; /* ModelConfig, include/engine.h:17-27 */
    int max_context;                                                  /* KV-cache positions */
    float rms_norm_epsilon, rope_frequency_base;
} QmvQwen2Config;

/* One tensor of the model under its GGUF name (token_embd.weight,
 * blk.<l>.attn_norm.weight, blk.<l>.attn_q.weight / .bias, attn_k, attn_v,
 * attn_output.weight, ffn_norm.weight, ffn_gate / ffn_up / ffn_down.weight,
 * output_norm.weight, output.weight).  Matrices: packed type, cols (K), rows
 * (N) and host bytes of rows x cols/block_elements blocks; vectors: type 0
 * (F32), rows 0, cols floats. */
typedef struct QmvQwen2Tensor {
    const char *name;
    uint32_t ggml_type;
    uint64_t cols, rows;
    const void *data;
} QmvQwen2Tensor;

typedef struct QmvQwen2 QmvQwen2;

/* Upload every tensor to the current device and capture the step graph. */
int qmv_qwen2_create(const QmvQwen2Config *config, const QmvQwen2Tensor *tensors, int count,
                     QmvQwen2 **decoder);
/* Pre-fill positions [0, token_count) of every layer's KV cache from host
 * keys/values laid out [layer][token_count][n_kv_heads * head_dim]; the next
 * step writes position token_count. */
int qmv_qwen2_set_kv(QmvQwen2 *decoder, const float *keys, const float *values, int token_count);
/* One step for `token`: logits[vocab_size] (host, may be NULL) and the greedy
 * next token.  0 on a non-finite logit or a full context, as the reference. */
int qmv_qwen2_forward(QmvQwen2 *decoder, int token, float *logits, int *next_token);
/* `steps` greedy steps from first_token without host round trips;
 * tokens[steps] receives the produced ids. */
int qmv_qwen2_generate(QmvQwen2 *decoder, int first_token, int steps, int *tokens);
/* Split form of qmv_qwen2_generate for timing: begin sets the first token,
 * replay enqueues `steps` graph launches on `stream` (no synchronisation),
 * read synchronises the device and copies the first `count` produced ids and
 * the next position (may be NULL). */
int qmv_qwen2_begin(QmvQwen2 *decoder, int first_token);
int qmv_qwen2_replay(QmvQwen2 *decoder, int steps, void *stream);
int qmv_qwen2_read(QmvQwen2 *decoder, int *tokens, int count, int *position);
/* Host copy of one layer's cached key and value at `position`. */
int qmv_qwen2_get_kv(QmvQwen2 *decoder, int layer, int position, float *key, float *value);
/* The reference's prefill_tokens (src/architecture.h:78-79,
 * qwen2_prefill_tokens, src/qwen2_architecture.cpp:1550-1729): append
 * `count` prompt tokens at the current position -- their keys and values in
 * every layer's cache -- and return the last position's logits (may be NULL)
 * and greedy token.  Positions go through each layer in chunks of up to 1024,
 * every projection one batched matmul (tensor cores from 32 positions).
 * Same checks as the reference (ids, context capacity, non-finite logits);
 * on failure the position is unchanged.  Continue with qmv_qwen2_generate /
 * qmv_qwen2_forward from the returned token. */
int qmv_qwen2_prefill(QmvQwen2 *decoder, const int *ids, int count, float *logits, int *next_token);
/* The reference's state_reset (src/architecture.h:80-81): position 0. */
int qmv_qwen2_reset(QmvQwen2 *decoder);
/* The (non-blocking) stream the decoder's work runs on, as a cudaStream_t. */
int qmv_qwen2_stream(const QmvQwen2 *decoder, void **stream);
/* Kernel launches in one captured step (0 on a null decoder). */
int qmv_qwen2_kernels_per_step(const QmvQwen2 *decoder);
/* How decoders created afterwards in this process run a step: 0 (default) =
 * one launch per projection and attention, captured in a CUDA graph;
 * 1 = the layer stack as one persistent cooperative launch (one CTA per SM,
 * grid barriers between the phases of each layer, each CTA copying its rows
 * of the next two projections into shared memory ahead of use), then the
 * output projection with its fused argmax and the advance kernel: 3 launches
 * per token; falls back to 0 where the device cannot keep every CTA
 * resident.  Same results within the parity bound (mode 1 adds a row's
 * partial sums in another order).  No counterpart in the reference. */
int qmv_set_decode_mode(int mode);
/* Decode attention kernel for steps captured afterwards in this process
 * (one launch per layer, decode mode 0): 0 (default) = one cluster of 16
 * CTAs per KV head, each CTA a range of the cached positions, the ranges'
 * softmax partials merged in the leader CTA's shared memory (groups of up to
 * 8 query heads, where the device places 16-CTA clusters; else as 1);
 * 1 = KV head x 64-position chunks merged through global memory by the last
 * CTA of each head.  Same function within the parity bound.  No counterpart
 * in the reference. */
int qmv_set_attention_path(int path);

/* The reference's per-request operation profile, field for field
 * (OperationProfile, include/metrics.h:6-25; per-format arrays indexed
 * F32, Q5_0, Q8_0, Q4_K, Q6_K), so a pointer to the reference's struct may
 * be passed.  Seconds here are device time from CUDA events. */
typedef struct QmvOperationProfile {
    int enabled;
    double matvec_seconds;
    double attention_seconds;
    double rmsnorm_seconds;
    double rope_seconds;
    double output_seconds;
    double sampling_seconds;
    double weight_layer_seconds[5];
    double weight_output_seconds[5];
    unsigned long long weight_layer_calls[5];
    unsigned long long weight_output_calls[5];
    double forward_seconds;
    unsigned long long forward_calls;
    unsigned long long sampling_calls;
} QmvOperationProfile;

/* qmv_qwen2_forward with the step's device time added to `profile` by stage
 * and weight format when profile->enabled (the reference's --profile
 * accounting, src/qwen2_architecture.cpp:1225-1525 and :603-614).  The step
 * runs un-captured with an event after each launch.  RMSNorm and RoPE are
 * fused into the projection and attention kernels (their rows stay 0); a
 * launch covering two formats splits its time by weight bytes; calls count
 * weight matrices as the reference's per-matrix matvec calls do. */
int qmv_qwen2_forward_profiled(QmvQwen2 *decoder, int token, float *logits, int *next_token,
                               QmvOperationProfile *profile);

/* ---- GGUF model images ---------------------------------------------------
 * The reference opens a model with gguf_open (src/gguf_reader.h:71,
 * src/gguf_reader.cpp:617-786) and derives a packed view per projection call
 * (gguf_get_quantized_tensor_view, src/gguf_reader.h:136-140, called from
 * src/qwen2_architecture.cpp:585-595).  These parse the same GGUF v3 image
 * with the same acceptance rules, walk its tensor directory once to make
 * every packed tensor resident, and configure the Qwen2 decoder from its
 * metadata. */
typedef struct QmvGguf QmvGguf;

/* One directory entry; name and data point into the handle / the image. */
typedef struct QmvGgufTensor {
    const char *name;
    uint32_t ggml_type;        /* 0 F32, 6 Q5_0, 8 Q8_0, 12 Q4_K, 14 Q6_K */
    uint32_t dimension_count;  /* 1..4; dimensions[0] is the row length */
    uint64_t dimensions[4];
    uint64_t offset;           /* from the start of the data section */
    uint64_t byte_size;
    const void *data;
} QmvGgufTensor;

/* Parse an image the caller keeps mapped for the handle's lifetime
 * (e.g. the reference's GgufFile::data / file_size). */
int qmv_gguf_open(const void *data, uint64_t size, QmvGguf **gguf);
/* Map `path` read-only and parse it; the handle owns the mapping. */
int qmv_gguf_open_file(const char *path, QmvGguf **gguf);
/* Also frees the resident weights keyed by addresses inside the image
 * (made by qmv_gguf_upload or by drop-in calls on its views). */
int qmv_gguf_close(QmvGguf *gguf);
int qmv_gguf_info(const QmvGguf *gguf, uint64_t *tensor_count, uint64_t *metadata_count,
                  uint64_t *data_offset, uint32_t *alignment);
int qmv_gguf_tensor(const QmvGguf *gguf, uint64_t index, QmvGgufTensor *tensor);
int qmv_gguf_find_tensor(const QmvGguf *gguf, const char *name, QmvGgufTensor *tensor);
/* Metadata reads with the reference's rules (gguf_get_uint / _float /
 * _string / _array_info, src/gguf_reader.h:73-90): 0 when the key is missing
 * or of another type (no message; the output is left unchanged). */
int qmv_gguf_get_uint(const QmvGguf *gguf, const char *key, uint64_t *value);
int qmv_gguf_get_float(const QmvGguf *gguf, const char *key, double *value);
int qmv_gguf_get_string(const QmvGguf *gguf, const char *key, const char **value, uint64_t *length);
int qmv_gguf_get_array_info(const QmvGguf *gguf, const char *key, uint32_t *element_type, uint64_t *count);
/* gguf_get_bool (src/gguf_reader.h:89). */
int qmv_gguf_get_bool(const QmvGguf *gguf, const char *key, int *value);
/* Sequential reads of one top-level array (GgufArrayCursor and
 * gguf_array_cursor_init / gguf_array_next_string / _uint / _int,
 * src/gguf_reader.h:64-69, :89-94): each read checks the element type and
 * the image bounds; strings point into the image. */
typedef struct QmvGgufArrayCursor {
    const QmvGguf *gguf;
    uint64_t position;
    uint64_t remaining;
    uint32_t element_type;
} QmvGgufArrayCursor;
int qmv_gguf_array_cursor_init(const QmvGguf *gguf, const char *key, QmvGgufArrayCursor *cursor);
int qmv_gguf_array_next_string(QmvGgufArrayCursor *cursor, const char **value, uint64_t *length);
int qmv_gguf_array_next_uint(QmvGgufArrayCursor *cursor, uint64_t *value);
int qmv_gguf_array_next_int(QmvGgufArrayCursor *cursor, int64_t *value);
/* gguf_get_f32_tensor_view (src/gguf_reader.h:99-118; same fields as its
 * GgufF32TensorView): F32 tensors only, cleared on every failure. */
typedef struct QmvGgufF32View {
    const float *data;
    uint32_t dimension_count;
    uint64_t dimensions[4];
    uint64_t element_count;
} QmvGgufF32View;
int qmv_gguf_f32_view(const QmvGguf *gguf, const char *name, QmvGgufF32View *view);
/* gguf_get_quantized_tensor_view (src/gguf_reader.h:136-140): the view is
 * cleared on every failure (0, no message). */
int qmv_gguf_quantized_view(const QmvGguf *gguf, const char *name, GgufQuantizedTensorView *view);
/* Make every packed 2-D tensor resident on the calling thread's device,
 * keyed by its mapped address (qmv_resident_weight); counts what is now
 * resident.  For the reference: call after gguf_open in engine_load_model
 * (src/engine.cpp:45-51) with the GgufFile's data and size. */
int qmv_gguf_upload(const QmvGguf *gguf, int *tensors, uint64_t *device_bytes);
/* A decoder configured from the image's qwen2.* metadata and vocabulary
 * size (qwen2_configure_model, src/qwen2_architecture.cpp:105-257;
 * engine_load_model, src/engine.cpp:64-72); 1 <= max_context <=
 * qwen2.context_length (qwen2_state_init, :286-291). */
int qmv_qwen2_create_from_gguf(const QmvGguf *gguf, int max_context, QmvQwen2 **decoder);
int qmv_qwen2_destroy(QmvQwen2 *decoder);

#ifdef __cplusplus
}
#endif

#endif
