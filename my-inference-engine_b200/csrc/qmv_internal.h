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
// 2.5 B/column per position): 65536 columns = 160 KiB for one position.
constexpr int kMaxCols = 65536;
// Upper bound on CTAs of one argmax-producing launch (size of the workspace
// key array).
constexpr int kMaxArgmaxCtas = 2048;
constexpr size_t kArgmaxWorkspaceBytes = 16 + 8 * (size_t)kMaxArgmaxCtas;

// Device layout of one resident tensor ("chunk-major").  Rows are contiguous
// and start on 16-byte boundaries.  A row is cut into C chunks, the unit one
// GEMV lane handles (a 32-weight block for Q8_0/Q5_0, 64 weights for
// Q4_K/Q6_K), and each chunk's 16-byte pieces are stored piece-major:
// piece j of chunk c sits at (j * C + c) * 16, so the 32 lanes of a warp
// reading piece j of chunks c..c+31 read one contiguous 512-byte run.
// Per-row segments (bytes, C = chunks per row, nb = blocks per row):
//   Q8_0 (C = nb):    q[0..15] pieces | q[16..31] pieces | d[C] fp16      (32 C + pad)
//   Q5_0 (C = nb):    qs pieces | qh[C] u32 (off_a) | d[C] fp16 (off_b)    (22 nb + pad)
//   Q4_K (C = 4 nb):  qs bytes 0-15 of group g | bytes 16-31 | raw 16-byte
//                     headers {d, dmin, 12 scale bytes}[nb] (off_a)        (144 nb, no pad)
//   Q6_K (C = 4 nb):  chunk (sb, g, h) = 4 sb + 2 g + h holds weights
//                     {128 g + 32 r + 16 h + o}: ql[64g+16h..] | ql[64g+32+16h..]
//                     | qh[32g+16h..] pieces | sc[8g+2r+h] r=0..3 as 4 bytes (off_a)
//                     | d[nb] fp16 (off_b)                                 (208 nb + pad)
// Every byte of the GGUF blocks is kept; only the Q8_0/Q5_0/Q6_K padding to
// 16 bytes per row is added.
struct Layout {
    uint32_t type;
    int rows;
    int cols;
    int nb;               // blocks per row
    int C;                // chunks per row
    uint64_t row_stride;  // bytes, multiple of 16
    uint32_t off_a;       // Q8_0 d, Q5_0 qh, Q4_K headers, Q6_K scales
    uint32_t off_b;       // Q5_0 d, Q6_K d
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

// Row-sharded exchange over peer memory (one node, up to kMaxPeers GPUs).
// Each rank's exchange buffer starts with a 256-byte control block whose
// first word is the rank's step counter (epoch, device-side), followed by two
// parity regions: logits[world * slot_rows] f32 | keys[world][kMaxExCtas] u64
// | flags[world][kMaxExCtas] u32 (one key and one flag per source CTA).  A
// kernel runs epoch = counter + 1, uses parity region epoch & 1 and stores
// the counter back when its exchange completed, so repeated launches
// (including CUDA-graph replays) need no host epoch.  Every rank launches
// ncta = min(SMs, slot_rows) CTAs (the GPUs of a node are one model).
constexpr int kMaxPeers = 8;
constexpr int kMaxExCtas = 256;
constexpr size_t kExchangeHeader = 256;
struct Exchange {
    int world;  // <= 1: no exchange
    int rank;
    int slot_rows;
    int ncta;             // CTAs per rank (set by the launcher)
    unsigned int *epoch;  // this rank's counter
    float *logits[2][kMaxPeers];
    unsigned long long *keys[2][kMaxPeers];  // rank p's keys: [source rank][CTA]
    unsigned int *flags[2][kMaxPeers];       // rank p's flags: [source rank][CTA], = epoch when delivered
};
size_t exchange_parity_bytes(int world, int slot_rows);

// x of a batched matmul: x[p][k] = x[p * ldx + k], or, with up set,
// up[p * ldu + k] * silu(x[p * ldx + k]) (a SwiGLU formed as x is read).
struct XSource {
    const float *x;
    const float *up;
    int ldx;
    int ldu;
};

// Fused prologue / epilogue of a GEMV (the decode step's RMSNorm, SwiGLU,
// bias and residual additions); device pointers.  Zero-initialised: none.
enum : int { kPreNone = 0, kPreRmsNorm = 1, kPreSwiGlu = 2, kPreScale = 3 };
struct Fuse {
    int pre;            // kPreRmsNorm: x <- (x / sqrt(mean(x^2) + eps)) * norm
                        // kPreSwiGlu:  x <- up * x / (1 + exp(-x))   (x is the gate)
                        // kPreScale:   x <- x * norm (the persistent step's RMSNorm,
                        //              whose 1 / sqrt(mean(x^2) + eps) scales the dot)
    const float *norm;  // kPreRmsNorm: weight[cols]
    float eps;
    const float *up;    // kPreSwiGlu: up[cols]
    const float *add;   // y[row] = (W x)[row] + add[row] when non-null (add == y: residual in place)
    // L2 prefetch of the launch that follows in the stream (the decode step's
    // next projection): each CTA prefetches its share of these byte ranges
    // once its own copies are issued.  Null: none.
    const uint8_t *pf[2];
    uint64_t pf_bytes[2];
};

// y = W x (and optionally the argmax key of y).
cudaError_t launch_gemv(const Layout &L, const uint8_t *w, const float *x, float *y,
                        const ArgmaxOut *am, cudaStream_t s);
// The same with a fused prologue / epilogue; needs the TMA pipeline
// (cudaErrorNotSupported when its stages do not fit).
cudaError_t launch_gemv_fused(const Layout &L, const uint8_t *w, const float *x, float *y,
                              const ArgmaxOut *am, const Fuse &fu, cudaStream_t s);
// Two matrices of different formats and equal columns over one x in one
// launch (ya = Wa x', yb = Wb x', x' = x through fu's RMSNorm prologue, no
// epilogue); the SMs are split between them by bytes.  cudaErrorNotSupported
// when no common 16-warp plan fits (launch the two separately).
cudaError_t launch_gemv_pair(const Layout &La, const uint8_t *wa, float *ya, const Layout &Lb, const uint8_t *wb,
                             float *yb, const float *x, const Fuse &fu, cudaStream_t s);
// Fused projection + argmax + exchange: y is this rank's slot in its own
// buffer; needs the TMA pipeline (cudaErrorNotSupported when its stages do
// not fit).
cudaError_t launch_gemv_exchange(const Layout &L, const uint8_t *w, const float *x, float *y,
                                 const ArgmaxOut &am, const Exchange &ex, cudaStream_t s);
// Y[p] = W X[p], p < batch.
// H [batch][rows] += W X (the prefill's residual projections): on the tensor
// cores with K split across CTAs when that fills more SMs, the partial
// products summed into H in split order; scratch from the stream-ordered pool.
cudaError_t launch_matmul_residual(const Layout &L, const uint8_t *w, const float *X, int batch, float *H,
                                   cudaStream_t s);
// The same product left as *ks partial slices of batch x rows floats in
// stream-ordered scratch (free with cudaFreeAsync on s after summing them):
// launch_rmsnorm_residual folds them into the residual stream and normalises
// it in one pass; launch_add_partials only adds them.
cudaError_t launch_matmul_partials(const Layout &L, const uint8_t *w, const float *X, int batch, float **part,
                                   int *ks, cudaStream_t s);
// The same with x = up * silu(gate) formed as x is read (the prefill's down
// projection): gate and up rows g_ld / u_ld floats apart.
cudaError_t launch_matmul_partials_swiglu(const Layout &L, const uint8_t *w, const float *gate, int g_ld,
                                          const float *up, int u_ld, int batch, float **part, int *ks, cudaStream_t s);
cudaError_t launch_rmsnorm_residual(float *h, const float *part, int ks, const float *w, float eps, int cols,
                                    int rows, float *out, cudaStream_t s);
cudaError_t launch_add_partials(float *h, const float *part, size_t n, int ks, cudaStream_t s);
cudaError_t launch_matmul(const Layout &L, const uint8_t *w, const float *X, int batch, float *Y,
                          cudaStream_t s);
// GEMV kernel selection: 0 automatic (TMA pipeline when its stages fit in
// shared memory, direct loads otherwise), 1 direct loads, 2 TMA pipeline only.
void set_gemv_path(int path);
// Matmul kernel selection: 0 automatic (tensor cores from 32 positions when X
// is 16-byte aligned), 1 CUDA cores (dp4a), 2 tensor cores only, 64 / 128 /
// 176 / 256 tensor cores with that position-tile width.
void set_matmul_path(int path);
// Device status bits set by bounded waits that expired (0 = healthy).
cudaError_t read_status(unsigned int *out, bool clear);
// A device-visible word that the calling thread's later launches also set
// their expired-wait bits in (null: the device-wide word only).
void set_call_status(unsigned int *word);
// Stream-ordered scratch from the library's per-device pool (no device-wide
// synchronisation; steady-state allocations do not reach the driver).
cudaError_t stream_alloc(void **ptr, size_t bytes, cudaStream_t s);
cudaError_t stream_free(void *ptr, cudaStream_t s);
// ---- device-resident decode step (Qwen2 architecture)
// Step state in device memory, so one step replays from a CUDA graph.
struct DecodeState {
    int pos;             // position the next step writes
    int tok;             // token of the next step
    int steps;           // tokens produced so far (index into the history)
    unsigned int error;  // 1 token out of range, 2 context full, 4 no finite logit, 8 barrier expired,
                         // 16 the attention cluster's wait for its partials expired
};
// h = row st->tok of the resident embedding matrix (bit-exact dequant).
cudaError_t launch_embed(const Layout &L, const uint8_t *w, DecodeState *st, float *h, cudaStream_t s);
// RoPE, KV-cache append and grouped-query attention for one layer at
// position st->pos.  qkv = [q (heads x hd) | k (kv_heads x hd) | v] after the
// biases; kc / vc: this layer's cache [max_ctx][kv_heads x hd]; att: output
// [heads x hd].  head_dim must be 64.
size_t attention_workspace_floats(int heads, int kv_heads, int head_dim, int max_ctx);
cudaError_t launch_attention(const float *qkv, int heads, int kv_heads, int head_dim, float *kc, float *vc,
                             int max_ctx, float rope_base, DecodeState *st, float *part, unsigned int *counter,
                             float *att, cudaStream_t s);
// Decode attention kernel: 0 automatic (one 16-CTA cluster per KV head,
// merged in distributed shared memory, where the group has at most 8 query
// heads and the device places such clusters), 1 the chunked kernel (KV head
// x 64-position chunks, merged by the last CTA through global memory).
void set_attention_path(int path);
// The layer stack of one decode step as one cooperative launch (one CTA per
// SM, grid barriers between the phases of each layer): embedding, then per
// layer [q; k; v] (RMSNorm prologue, biases), attention, o (residual),
// [gate; up] (RMSNorm prologue), down (SwiGLU prologue, residual).  Leaves h
// for the output projection.  head_dim must be 64.
struct PGemv {
    Layout L;
    const uint8_t *w;  // resident rows (null: absent)
};
struct PLayer {
    PGemv qkv[3];  // [q; k; v] as one matrix (n_qkv = 1) or q, k, v (3)
    int n_qkv;
    PGemv o;
    PGemv gu[2];  // [gate; up] as one matrix (n_gu = 1) or gate, up (2)
    int n_gu;
    PGemv down;
    const float *attn_norm, *ffn_norm, *bias_qkv;
    float *kc, *vc;  // this layer's cache [max_ctx][kv_heads * 64]
};
struct GridBar {  // zeroed before the first launch
    unsigned int count;  // arrivals of the current step
    unsigned int abort;  // a barrier expired: every later one returns at once
    unsigned int pad[2];
};
struct PStep {
    const PLayer *layers;  // device array of n_layers
    int n_layers;
    int dim, hid, heads, kv_heads, max_ctx;
    float eps, rope_base;
    PGemv embd;
    float *h, *qkv, *att, *gate, *up;  // up: the up output of layers with n_gu == 2
    float *part;                       // attention_workspace_floats
    unsigned int *attn_cnt;            // kv_heads zeroed words
    DecodeState *st;                   // error bit 8: a grid barrier expired
    GridBar *bar;                      // count re-armed by launch_advance
    uint32_t slot_bytes;               // decode_layers_slot_bytes
};
uint32_t decode_layers_slot_bytes(int dim, int hid);
size_t decode_layers_smem(int dim, int hid, uint32_t slot_bytes);
cudaError_t launch_decode_layers(const PStep &P, cudaStream_t s);
// next token from the step's argmax key; history[st->steps] = token; pos += 1
cudaError_t launch_advance(const unsigned long long *key, DecodeState *st, int *history, int max_steps,
                           cudaStream_t s, unsigned int *bar_count = nullptr);
// Prefill steps (the reference's qwen2_prefill_tokens between its
// projections), over n consecutive positions of one chunk; row-major
// activations, device pointers.
cudaError_t launch_embed_rows(const Layout &L, const uint8_t *w, const int *ids, int n, float *h,
                              unsigned int *err, cudaStream_t s);
cudaError_t launch_rmsnorm_rows(const float *x, const float *w, float eps, int cols, int rows, float *out,
                                cudaStream_t s);
// biases, RoPE (q in place) and the keys/values of positions pos0.. appended
cudaError_t launch_rope_kv(float *q, int q_ld, const float *k, int k_ld, const float *v, int v_ld,
                           const float *bias_q, const float *bias_k, const float *bias_v, int heads, int kv_heads,
                           int head_dim, int pos0, int n, float rope_base, float *kc, float *vc, cudaStream_t s);
// causal attention of positions pos0..pos0+n-1 over the cache; att [n][heads*hd];
// part: prefill_attention_part_floats(heads, head_dim, n) floats of scratch
// (partials of rows whose keys are split across CTAs)
size_t prefill_attention_part_floats(int heads, int head_dim, int positions);
// counter: kv_heads x n zeroed words (arrivals of a block's split CTAs;
// each block's merging CTA re-arms its own)
cudaError_t launch_prefill_attention(const float *q, int q_ld, const float *kc, const float *vc, int heads,
                                     int kv_heads, int head_dim, int pos0, int n, float *att, float *part,
                                     unsigned int *counter, cudaStream_t s);


// Argmax key of logits[0..n).
cudaError_t launch_argmax(const float *logits, int n, const ArgmaxOut &am, cudaStream_t s);
// Same, with the scratch in a static device array (no allocation, no caller
// workspace); n <= noalloc_max_logits().
int noalloc_max_logits();
cudaError_t launch_argmax_noalloc(const float *logits, int n, int index_base, unsigned long long *key,
                                  cudaStream_t s);

// Per-thread error message of the C ABI (qmv_last_error); both return 0.
int set_error(const char *msg);
int set_cuda_error(const char *what, cudaError_t e);
// Free every registry-owned resident weight whose host key lies in
// [begin, end) (an image that is being unmapped); returns how many.
int release_resident_range(const void *begin, const void *end);

}  // namespace qmv

// A resident packed tensor (rows [row_begin, row_begin + L.rows) of the
// uploaded matrix), the opaque handle of the C ABI.
struct QmvWeight {
    qmv::Layout L;
    uint8_t *dev;
    size_t bytes;
    int device;
    int row_begin;
    bool registry_owned;
};
