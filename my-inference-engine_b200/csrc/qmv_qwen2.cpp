// Device-resident Qwen2 decode step behind the C ABI (qmv_qwen2_*, declared
// in include/qmv_b200.h).
//
// The reference runs one token through qwen2_forward_token_cached_impl
// (src/qwen2_architecture.cpp:1195-1531) on the host, calling the packed
// matvec once per projection and moving every activation through host
// memory.  Here the whole step stays on one GPU:
//
//   embed_kernel                       token row of token_embd (bit-exact)
//   per layer:
//     GEMV [q; k; v]   RMSNorm(attn_norm) prologue, bias epilogue
//     attention_kernel RoPE, KV-cache append, grouped-query attention
//     GEMV o           residual epilogue (h += W_o att)
//     GEMV [gate; up]  RMSNorm(ffn_norm) prologue (one paired launch when
//                      their formats differ)
//     GEMV down        SwiGLU prologue (up * silu(gate)), residual epilogue
//   GEMV output        RMSNorm(output_norm) prologue, fused greedy argmax
//   advance_kernel     argmax key -> next token, position + 1
//
// Token and position live in device memory, so the step is captured once into
// a CUDA graph and replayed: generation runs token after token without the
// host.  Weights are uploaded once (Q, K and V, and gate and up, concatenated
// into one resident tensor each when they share a format); the KV cache is f32
// [layer][max_context][n_kv_heads * head_dim] like the reference's
// (src/qwen2_internal.h:33-39).
#include <cuda_runtime.h>

#include <stdint.h>
#include <string.h>

#include <map>
#include <string>
#include <vector>

#include "qmv_b200.h"
#include "qmv_internal.h"

#define QMV_EXPORT extern "C" __attribute__((visibility("default")))

namespace {

struct Layer {
    QmvWeight *qkv = nullptr;                            // [q; k; v] when they share a format
    QmvWeight *q = nullptr, *k = nullptr, *v = nullptr;  // otherwise
    QmvWeight *gate_up = nullptr;                        // [gate; up] when they share a format
    QmvWeight *o = nullptr, *gate = nullptr, *up = nullptr, *down = nullptr;
    float *attn_norm = nullptr, *ffn_norm = nullptr, *bias_qkv = nullptr;
};

int cuda_err(const char *what, cudaError_t e) { return qmv::set_cuda_error(what, e); }

#define QW_CUDA(call, what)                          \
    do {                                             \
        cudaError_t e_ = (call);                     \
        if (e_ != cudaSuccess) return cuda_err(what, e_); \
    } while (0)

}  // namespace

struct QmvQwen2 {
    QmvQwen2Config cfg{};
    int device = 0, head_dim = 0, kvd = 0;
    QmvWeight *embd = nullptr, *out = nullptr;
    std::vector<Layer> layers;
    float *out_norm = nullptr;
    float *h = nullptr, *qkv = nullptr, *att = nullptr, *gate = nullptr, *up = nullptr, *logits = nullptr;
    float *kc = nullptr, *vc = nullptr;
    float *attn_part = nullptr;
    unsigned int *attn_cnt = nullptr;
    unsigned long long *key = nullptr;
    void *am_ws = nullptr;
    qmv::DecodeState *st = nullptr;
    int *history = nullptr;
    cudaStream_t stream = nullptr;
    cudaGraphExec_t exec = nullptr;
    int kernels_per_step = 0;  // kernel nodes of the captured step
    // prefill chunk buffers (allocated on first use), pf_cap positions each
    int pf_cap = 0;
    int *pf_ids = nullptr;
    float *pf_h = nullptr, *pf_xn = nullptr, *pf_qkv = nullptr, *pf_att = nullptr, *pf_y = nullptr;
    float *pf_gu = nullptr, *pf_part = nullptr;
    unsigned int *pf_cnt = nullptr;
    cudaStream_t pf_side = nullptr;  // up projection beside gate (different formats)
    cudaEvent_t pf_fork = nullptr, pf_join = nullptr;
    // persistent step (decode_layers_kernel): descriptors and grid barrier
    bool persistent = false;
    qmv::PStep ps{};
    qmv::GridBar *bar = nullptr;
    std::vector<cudaEvent_t> prof_events;  // profiled steps (created on first use)
    std::vector<void *> allocs;
    std::vector<QmvWeight *> weights;
};

namespace {

// 0: one launch per projection and attention; 1: the layer stack as one
// persistent cooperative launch where the device allows it (process-wide,
// read when a decoder is created).
int g_decode_mode = 0;

int dalloc(QmvQwen2 *m, void **p, size_t bytes, const char *what)
{
    QW_CUDA(cudaMalloc(p, bytes), what);
    m->allocs.push_back(*p);
    QW_CUDA(cudaMemset(*p, 0, bytes), what);
    return 1;
}

int upload_rows(QmvQwen2 *m, uint32_t type, uint64_t cols, uint64_t rows, const void *data, QmvWeight **out)
{
    const int be = qmv::block_elements(type), bb = qmv::block_bytes(type);
    if (be == 0) return qmv::set_error("unsupported projection format");
    GgufQuantizedTensorView v{};
    v.data = (const unsigned char *)data;
    v.ggml_type = type;
    v.dimension_count = 2;
    v.dimensions[0] = cols;
    v.dimensions[1] = rows;
    v.element_count = cols * rows;
    v.block_elements = (uint64_t)be;
    v.block_bytes = (uint64_t)bb;
    v.block_count = v.element_count / (uint64_t)be;
    if (!qmv_weight_upload(&v, 0, (int)rows, out)) return 0;
    m->weights.push_back(*out);
    return 1;
}

int upload_vector(QmvQwen2 *m, const float *host, size_t n, float **out, const char *what)
{
    if (!dalloc(m, (void **)out, n * sizeof(float), what)) return 0;
    QW_CUDA(cudaMemcpy(*out, host, n * sizeof(float), cudaMemcpyHostToDevice), what);
    return 1;
}

const QmvQwen2Tensor *find(const std::map<std::string, const QmvQwen2Tensor *> &by, const std::string &name,
                           uint64_t cols, uint64_t rows)
{
    auto it = by.find(name);
    if (it == by.end()) {
        qmv::set_error(("missing tensor " + name).c_str());
        return nullptr;
    }
    const QmvQwen2Tensor *t = it->second;
    const bool vec = rows == 0;
    if (t->cols != cols || t->rows != rows || t->data == nullptr || (vec && t->ggml_type != 0) ||
        (!vec && qmv::block_elements(t->ggml_type) == 0) || (!vec && cols % qmv::block_elements(t->ggml_type))) {
        qmv::set_error(("tensor " + name + " has the wrong shape or format").c_str());
        return nullptr;
    }
    return t;
}

size_t tensor_bytes(const QmvQwen2Tensor *t)
{
    return (size_t)(t->cols / qmv::block_elements(t->ggml_type)) * t->rows * qmv::block_bytes(t->ggml_type);
}

cudaError_t gemv(QmvQwen2 *m, const QmvWeight *w, const float *x, float *y, const qmv::Fuse &fu,
                 const qmv::ArgmaxOut *am = nullptr)
{
    return qmv::launch_gemv_fused(w->L, w->dev, x, y, am, fu, m->stream);
}

// Profiled steps (never captured): an event after each launch, tagged with
// the reference's stage it belongs to (include/metrics.h:6-25).  A launch of
// two formats (the gate/up pair) splits its time between them by weight
// bytes; `calls` counts weight matrices, as the reference counts its
// per-matrix matvec calls.
enum Stage : int { kStageEmbed, kStageLayerGemv, kStageAttention, kStageOutput, kStageSampling };
struct Mark {
    int stage;
    uint32_t type[2];
    double share0;  // of the time, to type[0]
    int calls[2];
};
struct Marks {
    int used = 0;  // events recorded; event 0 precedes the first launch
    std::vector<Mark> what;  // what[i] ends at event i + 1
};

cudaError_t record(QmvQwen2 *m, Marks *mk)
{
    if ((size_t)mk->used == m->prof_events.size()) {
        cudaEvent_t ev = nullptr;
        const cudaError_t e = cudaEventCreate(&ev);
        if (e != cudaSuccess) return e;
        m->prof_events.push_back(ev);
    }
    return cudaEventRecord(m->prof_events[(size_t)mk->used++], m->stream);
}

// After a successful launch, close its stage (no-op when not profiling).
cudaError_t mark(QmvQwen2 *m, Marks *mk, cudaError_t launched, const Mark &w)
{
    if (mk == nullptr || launched != cudaSuccess) return launched;
    mk->what.push_back(w);
    return record(m, mk);
}

Mark layer_mark(const QmvWeight *w, int calls) { return Mark{kStageLayerGemv, {w->L.type, 0}, 1.0, {calls, 0}}; }

// One decode step as three launches: the persistent layer stack, the output
// projection with its fused greedy argmax, and the advance kernel.
cudaError_t enqueue_step_persistent(QmvQwen2 *m)
{
    const QmvQwen2Config &c = m->cfg;
    cudaError_t e = qmv::launch_decode_layers(m->ps, m->stream);
    const qmv::ArgmaxOut am{m->key, m->am_ws, 0};
    if (e == cudaSuccess)
        e = gemv(m, m->out, m->h, m->logits,
                 qmv::Fuse{qmv::kPreRmsNorm, m->out_norm, c.rms_norm_epsilon, nullptr, nullptr}, &am);
    if (e == cudaSuccess)
        e = qmv::launch_advance(m->key, m->st, m->history, c.max_context, m->stream, &m->bar->count);
    return e;
}

// One decode step, enqueued on m->stream; mk != nullptr records the
// profiling events of an un-captured step (always one launch per projection,
// so each stage has its own events).
// The step's projections in launch order (gate and up of a paired launch
// as one entry each), for the L2 prefetch of the ones ahead.
std::vector<const QmvWeight *> step_weights(const QmvQwen2 *m)
{
    std::vector<const QmvWeight *> seq;
    for (const Layer &L : m->layers) {
        if (L.qkv) {
            seq.push_back(L.qkv);
        } else {
            seq.push_back(L.q);
            seq.push_back(L.k);
            seq.push_back(L.v);
        }
        seq.push_back(L.o);
        if (L.gate_up) {
            seq.push_back(L.gate_up);
        } else {
            seq.push_back(L.gate);
            seq.push_back(L.up);
        }
        seq.push_back(L.down);
    }
    return seq;
}

// Prefetch ranges of a launch whose last weight matrix is seq[i]: the next
// two matrices (the output projection, hundreds of MB, is never prefetched).
qmv::Fuse with_prefetch(qmv::Fuse fu, const std::vector<const QmvWeight *> &seq, size_t i)
{
    constexpr size_t kMaxPrefetch = 16u << 20;
    for (int j = 0; j < 2; ++j) {
        const size_t n = i + 1 + (size_t)j;
        if (n < seq.size() && seq[n]->bytes <= kMaxPrefetch) {
            fu.pf[j] = seq[n]->dev;
            fu.pf_bytes[j] = seq[n]->bytes;
        }
    }
    return fu;
}

cudaError_t enqueue_step(QmvQwen2 *m, Marks *mk = nullptr)
{
    if (m->persistent && mk == nullptr) return enqueue_step_persistent(m);
    const QmvQwen2Config &c = m->cfg;
    const int dim = c.dim, kvd = m->kvd;
    const std::vector<const QmvWeight *> seq = step_weights(m);
    size_t si = 0;  // index in seq of the next launch's first matrix
    cudaError_t e = mk ? record(m, mk) : cudaSuccess;
    if (e == cudaSuccess)
        e = mark(m, mk, qmv::launch_embed(m->embd->L, m->embd->dev, m->st, m->h, m->stream),
                 Mark{kStageEmbed, {0, 0}, 1.0, {0, 0}});
    for (int l = 0; l < c.n_layers && e == cudaSuccess; ++l) {
        const Layer &L = m->layers[(size_t)l];
        qmv::Fuse pre_attn{qmv::kPreRmsNorm, L.attn_norm, c.rms_norm_epsilon, nullptr, L.bias_qkv};
        if (L.qkv) {
            e = mark(m, mk, gemv(m, L.qkv, m->h, m->qkv, with_prefetch(pre_attn, seq, si)), layer_mark(L.qkv, 3));
            si += 1;
        } else {
            e = mark(m, mk, gemv(m, L.q, m->h, m->qkv, with_prefetch(pre_attn, seq, si)), layer_mark(L.q, 1));
            pre_attn.add = L.bias_qkv + dim;
            if (e == cudaSuccess)
                e = mark(m, mk, gemv(m, L.k, m->h, m->qkv + dim, with_prefetch(pre_attn, seq, si + 1)),
                         layer_mark(L.k, 1));
            pre_attn.add = L.bias_qkv + dim + kvd;
            if (e == cudaSuccess)
                e = mark(m, mk, gemv(m, L.v, m->h, m->qkv + dim + kvd, with_prefetch(pre_attn, seq, si + 2)),
                         layer_mark(L.v, 1));
            si += 3;
        }
        const size_t layer_off = (size_t)l * (size_t)c.max_context * (size_t)kvd;
        if (e == cudaSuccess)
            e = mark(m, mk,
                     qmv::launch_attention(m->qkv, c.n_heads, c.n_kv_heads, m->head_dim, m->kc + layer_off,
                                           m->vc + layer_off, c.max_context, c.rope_frequency_base, m->st,
                                           m->attn_part, m->attn_cnt, m->att, m->stream),
                     Mark{kStageAttention, {0, 0}, 1.0, {0, 0}});
        if (e == cudaSuccess)
            e = mark(m, mk,
                     gemv(m, L.o, m->att, m->h,
                          with_prefetch(qmv::Fuse{qmv::kPreNone, nullptr, 0.f, nullptr, m->h}, seq, si)),
                     layer_mark(L.o, 1));
        si += 1;
        const qmv::Fuse pre_ffn{qmv::kPreRmsNorm, L.ffn_norm, c.rms_norm_epsilon, nullptr, nullptr};
        // With [gate; up] resident as one matrix, up lands right after gate.
        float *up = L.gate_up ? m->gate + c.hidden_dim : m->up;
        if (L.gate_up) {
            if (e == cudaSuccess)
                e = mark(m, mk, gemv(m, L.gate_up, m->h, m->gate, with_prefetch(pre_ffn, seq, si)),
                         layer_mark(L.gate_up, 2));
            si += 1;
        } else {
            if (e == cudaSuccess) {
                // different formats: one paired launch, else two
                e = qmv::launch_gemv_pair(L.gate->L, L.gate->dev, m->gate, L.up->L, L.up->dev, m->up, m->h,
                                          with_prefetch(pre_ffn, seq, si + 1), m->stream);
                if (e == cudaErrorNotSupported) {
                    e = mark(m, mk, gemv(m, L.gate, m->h, m->gate, with_prefetch(pre_ffn, seq, si)),
                             layer_mark(L.gate, 1));
                    if (e == cudaSuccess)
                        e = mark(m, mk, gemv(m, L.up, m->h, m->up, with_prefetch(pre_ffn, seq, si + 1)),
                                 layer_mark(L.up, 1));
                } else {
                    const double bg = (double)L.gate->bytes, bu = (double)L.up->bytes;
                    e = mark(m, mk, e,
                             Mark{kStageLayerGemv, {L.gate->L.type, L.up->L.type}, bg / (bg + bu), {1, 1}});
                }
            }
            si += 2;
        }
        if (e == cudaSuccess)
            e = mark(m, mk,
                     gemv(m, L.down, m->gate, m->h,
                          with_prefetch(qmv::Fuse{qmv::kPreSwiGlu, nullptr, 0.f, up, m->h}, seq, si)),
                     layer_mark(L.down, 1));
        si += 1;
    }
    const qmv::ArgmaxOut am{m->key, m->am_ws, 0};
    if (e == cudaSuccess)
        e = mark(m, mk,
                 gemv(m, m->out, m->h, m->logits,
                      qmv::Fuse{qmv::kPreRmsNorm, m->out_norm, c.rms_norm_epsilon, nullptr, nullptr}, &am),
                 Mark{kStageOutput, {m->out->L.type, 0}, 1.0, {1, 0}});
    if (e == cudaSuccess)
        e = mark(m, mk, qmv::launch_advance(m->key, m->st, m->history, c.max_context, m->stream),
                 Mark{kStageSampling, {0, 0}, 1.0, {0, 0}});
    return e;
}

int set_token(QmvQwen2 *m, int token)
{
    if (token < 0 || token >= m->cfg.vocab_size) return qmv::set_error("token id is out of range");
    if (m->bar) QW_CUDA(cudaMemsetAsync(m->bar, 0, sizeof(qmv::GridBar), m->stream), "set token");
    const int tok_steps[2] = {token, 0};
    QW_CUDA(cudaMemcpyAsync(&m->st->tok, tok_steps, sizeof tok_steps, cudaMemcpyHostToDevice, m->stream),
            "set token");
    QW_CUDA(cudaStreamSynchronize(m->stream), "set token");
    return 1;
}

int check_state(QmvQwen2 *m, qmv::DecodeState *out)
{
    qmv::DecodeState s{};
    QW_CUDA(cudaMemcpy(&s, m->st, sizeof s, cudaMemcpyDeviceToHost), "read decode state");
    if (out) *out = s;
    if (s.error & 1u) return qmv::set_error("decode step: token id out of range");
    if (s.error & 2u) return qmv::set_error("decode step: context capacity is exhausted");
    if (s.error & 4u) return qmv::set_error("decode step: output contains a non-finite logit");
    if (s.error & 8u) return qmv::set_error("decode step: a grid barrier of the persistent step expired");
    if (s.error & 16u) return qmv::set_error("decode step: the attention cluster's wait for its partials expired");
    return 1;
}

void release(QmvQwen2 *m)
{
    for (cudaEvent_t ev : m->prof_events) cudaEventDestroy(ev);
    if (m->pf_fork) cudaEventDestroy(m->pf_fork);
    if (m->pf_join) cudaEventDestroy(m->pf_join);
    if (m->pf_side) cudaStreamDestroy(m->pf_side);
    if (m->exec) cudaGraphExecDestroy(m->exec);
    for (QmvWeight *w : m->weights) qmv_weight_free(w);
    for (void *p : m->allocs) cudaFree(p);
    if (m->stream) cudaStreamDestroy(m->stream);
    delete m;
}

qmv::PGemv pg(const QmvWeight *w) { return w ? qmv::PGemv{w->L, w->dev} : qmv::PGemv{qmv::Layout{}, nullptr}; }

// Descriptors of the persistent step (decode_layers_kernel) in device memory.
int build_persistent(QmvQwen2 *m)
{
    const QmvQwen2Config &c = m->cfg;
    std::vector<qmv::PLayer> host((size_t)c.n_layers);
    const size_t kvd = (size_t)m->kvd;
    for (int l = 0; l < c.n_layers; ++l) {
        const Layer &L = m->layers[(size_t)l];
        qmv::PLayer &p = host[(size_t)l];
        p = qmv::PLayer{};
        if (L.qkv) {
            p.qkv[0] = pg(L.qkv);
            p.n_qkv = 1;
        } else {
            p.qkv[0] = pg(L.q);
            p.qkv[1] = pg(L.k);
            p.qkv[2] = pg(L.v);
            p.n_qkv = 3;
        }
        p.o = pg(L.o);
        if (L.gate_up) {
            p.gu[0] = pg(L.gate_up);
            p.n_gu = 1;
        } else {
            p.gu[0] = pg(L.gate);
            p.gu[1] = pg(L.up);
            p.n_gu = 2;
        }
        p.down = pg(L.down);
        p.attn_norm = L.attn_norm;
        p.ffn_norm = L.ffn_norm;
        p.bias_qkv = L.bias_qkv;
        const size_t off = (size_t)l * (size_t)c.max_context * kvd;
        p.kc = m->kc + off;
        p.vc = m->vc + off;
    }
    qmv::PLayer *dev_layers = nullptr;
    if (!dalloc(m, (void **)&dev_layers, host.size() * sizeof(qmv::PLayer), "persistent step") ||
        !dalloc(m, (void **)&m->bar, sizeof(qmv::GridBar), "grid barrier"))
        return 0;
    QW_CUDA(cudaMemcpy(dev_layers, host.data(), host.size() * sizeof(qmv::PLayer), cudaMemcpyHostToDevice),
            "persistent step");
    qmv::PStep &P = m->ps;
    P.slot_bytes = qmv::decode_layers_slot_bytes(c.dim, c.hidden_dim);
    if (P.slot_bytes < 16u) return 1;  // no room for the weight slots: one launch per projection
    P.layers = dev_layers;
    P.n_layers = c.n_layers;
    P.dim = c.dim;
    P.hid = c.hidden_dim;
    P.heads = c.n_heads;
    P.kv_heads = c.n_kv_heads;
    P.max_ctx = c.max_context;
    P.eps = c.rms_norm_epsilon;
    P.rope_base = c.rope_frequency_base;
    P.embd = pg(m->embd);
    P.h = m->h;
    P.qkv = m->qkv;
    P.att = m->att;
    P.gate = m->gate;
    P.up = m->up;
    P.part = m->attn_part;
    P.attn_cnt = m->attn_cnt;
    P.st = m->st;
    P.bar = m->bar;
    m->persistent = true;
    return 1;
}

int build(QmvQwen2 *m, const QmvQwen2Tensor *tensors, int count)
{
    const QmvQwen2Config &c = m->cfg;
    std::map<std::string, const QmvQwen2Tensor *> by;
    for (int i = 0; i < count; ++i)
        if (tensors[i].name) by[tensors[i].name] = &tensors[i];
    const uint64_t dim = (uint64_t)c.dim, hid = (uint64_t)c.hidden_dim, kvd = (uint64_t)m->kvd;
    const QmvQwen2Tensor *t = find(by, "token_embd.weight", dim, (uint64_t)c.vocab_size);
    if (!t || !upload_rows(m, t->ggml_type, t->cols, t->rows, t->data, &m->embd)) return 0;
    t = find(by, "output.weight", dim, (uint64_t)c.vocab_size);
    if (!t || !upload_rows(m, t->ggml_type, t->cols, t->rows, t->data, &m->out)) return 0;
    t = find(by, "output_norm.weight", dim, 0);
    if (!t || !upload_vector(m, (const float *)t->data, dim, &m->out_norm, "output_norm")) return 0;
    m->layers.resize((size_t)c.n_layers);
    for (int l = 0; l < c.n_layers; ++l) {
        Layer &L = m->layers[(size_t)l];
        const std::string p = "blk." + std::to_string(l) + ".";
        const QmvQwen2Tensor *q = find(by, p + "attn_q.weight", dim, dim);
        const QmvQwen2Tensor *k = find(by, p + "attn_k.weight", dim, kvd);
        const QmvQwen2Tensor *v = find(by, p + "attn_v.weight", dim, kvd);
        const QmvQwen2Tensor *qb = find(by, p + "attn_q.bias", dim, 0);
        const QmvQwen2Tensor *kb = find(by, p + "attn_k.bias", kvd, 0);
        const QmvQwen2Tensor *vb = find(by, p + "attn_v.bias", kvd, 0);
        if (!q || !k || !v || !qb || !kb || !vb) return 0;
        if (q->ggml_type == k->ggml_type && k->ggml_type == v->ggml_type) {
            const size_t bq = tensor_bytes(q), bk = tensor_bytes(k), bv = tensor_bytes(v);
            std::vector<unsigned char> cat(bq + bk + bv);
            memcpy(cat.data(), q->data, bq);
            memcpy(cat.data() + bq, k->data, bk);
            memcpy(cat.data() + bq + bk, v->data, bv);
            if (!upload_rows(m, q->ggml_type, dim, dim + 2 * kvd, cat.data(), &L.qkv)) return 0;
        } else if (!upload_rows(m, q->ggml_type, dim, dim, q->data, &L.q) ||
                   !upload_rows(m, k->ggml_type, dim, kvd, k->data, &L.k) ||
                   !upload_rows(m, v->ggml_type, dim, kvd, v->data, &L.v)) {
            return 0;
        }
        std::vector<float> bias(dim + 2 * kvd);
        memcpy(bias.data(), qb->data, dim * sizeof(float));
        memcpy(bias.data() + dim, kb->data, kvd * sizeof(float));
        memcpy(bias.data() + dim + kvd, vb->data, kvd * sizeof(float));
        if (!upload_vector(m, bias.data(), bias.size(), &L.bias_qkv, "qkv bias")) return 0;
        const QmvQwen2Tensor *o = find(by, p + "attn_output.weight", dim, dim);
        const QmvQwen2Tensor *g = find(by, p + "ffn_gate.weight", dim, hid);
        const QmvQwen2Tensor *u = find(by, p + "ffn_up.weight", dim, hid);
        const QmvQwen2Tensor *d = find(by, p + "ffn_down.weight", hid, dim);
        const QmvQwen2Tensor *an = find(by, p + "attn_norm.weight", dim, 0);
        const QmvQwen2Tensor *fn = find(by, p + "ffn_norm.weight", dim, 0);
        if (!o || !g || !u || !d || !an || !fn) return 0;
        if (g->ggml_type == u->ggml_type) {
            const size_t bg = tensor_bytes(g), bu = tensor_bytes(u);
            std::vector<unsigned char> cat(bg + bu);
            memcpy(cat.data(), g->data, bg);
            memcpy(cat.data() + bg, u->data, bu);
            if (!upload_rows(m, g->ggml_type, dim, 2 * hid, cat.data(), &L.gate_up)) return 0;
        } else if (!upload_rows(m, g->ggml_type, dim, hid, g->data, &L.gate) ||
                   !upload_rows(m, u->ggml_type, dim, hid, u->data, &L.up)) {
            return 0;
        }
        if (!upload_rows(m, o->ggml_type, dim, dim, o->data, &L.o) ||
            !upload_rows(m, d->ggml_type, hid, dim, d->data, &L.down) ||
            !upload_vector(m, (const float *)an->data, dim, &L.attn_norm, "attn_norm") ||
            !upload_vector(m, (const float *)fn->data, dim, &L.ffn_norm, "ffn_norm"))
            return 0;
    }
    const size_t cache = (size_t)c.n_layers * (size_t)c.max_context * kvd * sizeof(float);
    const size_t wide = (size_t)(hid > dim ? hid : dim);
    if (!dalloc(m, (void **)&m->h, dim * sizeof(float), "activations") ||
        !dalloc(m, (void **)&m->qkv, (dim + 2 * kvd) * sizeof(float), "activations") ||
        !dalloc(m, (void **)&m->att, dim * sizeof(float), "activations") ||
        !dalloc(m, (void **)&m->gate, 2 * wide * sizeof(float), "activations") ||
        !dalloc(m, (void **)&m->up, wide * sizeof(float), "activations") ||
        !dalloc(m, (void **)&m->logits, (size_t)c.vocab_size * sizeof(float), "logits") ||
        !dalloc(m, (void **)&m->kc, cache, "key cache") || !dalloc(m, (void **)&m->vc, cache, "value cache") ||
        !dalloc(m, (void **)&m->attn_part,
                qmv::attention_workspace_floats(c.n_heads, c.n_kv_heads, m->head_dim, c.max_context) * sizeof(float),
                "attention workspace") ||
        !dalloc(m, (void **)&m->attn_cnt, (size_t)c.n_kv_heads * sizeof(unsigned int), "attention counters") ||
        !dalloc(m, (void **)&m->key, sizeof(unsigned long long), "argmax key") ||
        !dalloc(m, &m->am_ws, qmv::kArgmaxWorkspaceBytes, "argmax workspace") ||
        !dalloc(m, (void **)&m->st, sizeof(qmv::DecodeState), "decode state") ||
        !dalloc(m, (void **)&m->history, (size_t)c.max_context * sizeof(int), "token history"))
        return 0;
    QW_CUDA(cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking), "decoder stream");
    if (g_decode_mode == 1 && m->head_dim == 64 && !build_persistent(m)) return 0;
    // One step outside capture sets every kernel's launch attributes, then the
    // state and cache are cleared and the step is captured.  A persistent step
    // the device refuses (its CTAs cannot all be resident) or that cannot be
    // captured falls back to one launch per projection.
    cudaError_t e0 = enqueue_step(m);
    if (e0 != cudaSuccess && m->persistent) {
        cudaGetLastError();
        m->persistent = false;
        e0 = enqueue_step(m);
    }
    QW_CUDA(e0, "decode step");
    QW_CUDA(cudaStreamSynchronize(m->stream), "decode step");
    QW_CUDA(cudaMemset(m->st, 0, sizeof(qmv::DecodeState)), "decode state");
    QW_CUDA(cudaMemset(m->kc, 0, cache), "key cache");
    QW_CUDA(cudaMemset(m->vc, 0, cache), "value cache");
    cudaGraph_t graph = nullptr;
    QW_CUDA(cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal), "graph capture");
    cudaError_t e = enqueue_step(m);
    cudaError_t e2 = cudaStreamEndCapture(m->stream, &graph);
    if ((e != cudaSuccess || e2 != cudaSuccess) && m->persistent) {
        if (graph) cudaGraphDestroy(graph);
        graph = nullptr;
        cudaGetLastError();
        m->persistent = false;
        QW_CUDA(cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal), "graph capture");
        e = enqueue_step(m);
        e2 = cudaStreamEndCapture(m->stream, &graph);
    }
    if (e != cudaSuccess) {
        if (graph) cudaGraphDestroy(graph);
        return cuda_err("graph capture", e);
    }
    QW_CUDA(e2, "graph capture");
    size_t n_nodes = 0;
    cudaError_t e4 = cudaGraphGetNodes(graph, nullptr, &n_nodes);
    std::vector<cudaGraphNode_t> nodes(n_nodes);
    if (e4 == cudaSuccess && n_nodes > 0) e4 = cudaGraphGetNodes(graph, nodes.data(), &n_nodes);
    for (size_t i = 0; e4 == cudaSuccess && i < n_nodes; ++i) {
        cudaGraphNodeType t;
        e4 = cudaGraphNodeGetType(nodes[i], &t);
        if (e4 == cudaSuccess && t == cudaGraphNodeTypeKernel) ++m->kernels_per_step;
    }
    if (e4 != cudaSuccess) {
        cudaGraphDestroy(graph);
        return cuda_err("graph nodes", e4);
    }
    const cudaError_t e3 = cudaGraphInstantiate(&m->exec, graph, 0);
    cudaGraphDestroy(graph);
    QW_CUDA(e3, "graph instantiate");
    return 1;
}

}  // namespace

QMV_EXPORT int qmv_qwen2_create(const QmvQwen2Config *cfg, const QmvQwen2Tensor *tensors, int count,
                                QmvQwen2 **out)
{
    if (out == nullptr) return qmv::set_error("output handle pointer is null");
    *out = nullptr;
    if (cfg == nullptr || tensors == nullptr || count <= 0) return qmv::set_error("null configuration or tensors");
    const QmvQwen2Config &c = *cfg;
    if (c.dim <= 0 || c.hidden_dim <= 0 || c.n_layers <= 0 || c.n_heads <= 0 || c.n_kv_heads <= 0 ||
        c.vocab_size <= 0 || c.max_context <= 0 || c.dim % c.n_heads != 0 || c.n_heads % c.n_kv_heads != 0 ||
        !(c.rms_norm_epsilon > 0.f) || !(c.rope_frequency_base > 0.f))
        return qmv::set_error("invalid Qwen2 configuration");
    if (c.dim / c.n_heads != 64 || c.n_heads / c.n_kv_heads > 16 || c.dim % 4 || c.hidden_dim % 4)
        return qmv::set_error("unsupported shape: head dimension 64 and at most 16 query heads per KV head");
    QmvQwen2 *m = new QmvQwen2();
    m->cfg = c;
    m->head_dim = c.dim / c.n_heads;
    m->kvd = c.n_kv_heads * m->head_dim;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        delete m;
        return qmv::set_error("no CUDA device");
    }
    m->device = dev;
    if (!build(m, tensors, count)) {
        release(m);
        return 0;
    }
    *out = m;
    return 1;
}

QMV_EXPORT int qmv_qwen2_set_kv(QmvQwen2 *m, const float *keys, const float *values, int token_count)
{
    if (m == nullptr || keys == nullptr || values == nullptr) return qmv::set_error("null argument");
    if (token_count < 0 || token_count >= m->cfg.max_context) return qmv::set_error("token count out of range");
    const size_t kvd = (size_t)m->kvd, T = (size_t)token_count;
    for (int l = 0; l < m->cfg.n_layers; ++l) {
        const size_t dst = (size_t)l * (size_t)m->cfg.max_context * kvd, src = (size_t)l * T * kvd;
        QW_CUDA(cudaMemcpy(m->kc + dst, keys + src, T * kvd * sizeof(float), cudaMemcpyHostToDevice), "set kv");
        QW_CUDA(cudaMemcpy(m->vc + dst, values + src, T * kvd * sizeof(float), cudaMemcpyHostToDevice), "set kv");
    }
    const qmv::DecodeState s{token_count, 0, 0, 0u};
    QW_CUDA(cudaMemcpy(m->st, &s, sizeof s, cudaMemcpyHostToDevice), "set kv");
    return 1;
}

// The stream every call of this decoder runs on (for callers timing it with
// their own events).
QMV_EXPORT int qmv_qwen2_stream(const QmvQwen2 *m, void **stream)
{
    if (m == nullptr || stream == nullptr) return qmv::set_error("null argument");
    *stream = (void *)m->stream;
    return 1;
}

// The reference's state_reset (src/architecture.h:80-81): back to position
// zero; the cache is overwritten as positions are written again.
QMV_EXPORT int qmv_qwen2_reset(QmvQwen2 *m)
{
    if (m == nullptr) return qmv::set_error("null decoder");
    const qmv::DecodeState s{0, 0, 0, 0u};
    QW_CUDA(cudaMemcpy(m->st, &s, sizeof s, cudaMemcpyHostToDevice), "reset");
    return 1;
}

QMV_EXPORT int qmv_qwen2_replay(QmvQwen2 *m, int steps, void *stream)
{
    if (m == nullptr || steps < 0) return qmv::set_error("bad replay request");
    for (int i = 0; i < steps; ++i) QW_CUDA(cudaGraphLaunch(m->exec, (cudaStream_t)stream), "graph launch");
    return 1;
}

QMV_EXPORT int qmv_qwen2_begin(QmvQwen2 *m, int token)
{
    if (m == nullptr) return qmv::set_error("null decoder");
    return set_token(m, token);
}

QMV_EXPORT int qmv_qwen2_read(QmvQwen2 *m, int *tokens, int count, int *position)
{
    if (m == nullptr || count < 0 || (count > 0 && tokens == nullptr)) return qmv::set_error("bad read request");
    QW_CUDA(cudaDeviceSynchronize(), "decode steps");
    qmv::DecodeState s{};
    if (!check_state(m, &s)) return 0;
    if (count > s.steps || count > m->cfg.max_context) return qmv::set_error("fewer tokens were produced");
    if (count > 0) QW_CUDA(cudaMemcpy(tokens, m->history, (size_t)count * sizeof(int), cudaMemcpyDeviceToHost), "read");
    if (position) *position = s.pos;
    return 1;
}

QMV_EXPORT int qmv_qwen2_forward(QmvQwen2 *m, int token, float *logits, int *next_token)
{
    if (m == nullptr) return qmv::set_error("null decoder");
    if (!set_token(m, token) || !qmv_qwen2_replay(m, 1, m->stream)) return 0;
    QW_CUDA(cudaStreamSynchronize(m->stream), "decode step");
    if (!check_state(m, nullptr)) return 0;
    if (logits)
        QW_CUDA(cudaMemcpy(logits, m->logits, (size_t)m->cfg.vocab_size * sizeof(float), cudaMemcpyDeviceToHost),
                "read logits");
    if (next_token) QW_CUDA(cudaMemcpy(next_token, m->history, sizeof(int), cudaMemcpyDeviceToHost), "read token");
    return 1;
}

namespace {

// Index of a weight format in the profile's per-format arrays
// (PROFILE_F32 .. PROFILE_Q6_K, include/metrics.h:6-7); -1 otherwise.
int profile_format(uint32_t type)
{
    switch (type) {
    case 0: return 0;
    case qmv::kQ5_0: return 1;
    case qmv::kQ8_0: return 2;
    case qmv::kQ4_K: return 3;
    case qmv::kQ6_K: return 4;
    default: return -1;
    }
}

void add_weight(double *seconds, unsigned long long *calls, uint32_t type, double dt, int n)
{
    const int f = profile_format(type);
    if (f < 0) return;
    seconds[f] += dt;
    calls[f] += (unsigned long long)n;
}

}  // namespace

// One step like qmv_qwen2_forward, run un-captured with an event after each
// launch; device times accumulate into `profile` by the reference's stages
// when profile->enabled (otherwise a plain step).  RMSNorm and RoPE run inside
// the projection and attention kernels, so their rows stay 0 and their time
// is in matvec / attention; the fused greedy argmax is in output, and the
// advance kernel that turns it into the next token is sampling.
QMV_EXPORT int qmv_qwen2_forward_profiled(QmvQwen2 *m, int token, float *logits, int *next_token,
                                          QmvOperationProfile *profile)
{
    if (m == nullptr) return qmv::set_error("null decoder");
    if (profile == nullptr || !profile->enabled) return qmv_qwen2_forward(m, token, logits, next_token);
    if (!set_token(m, token)) return 0;
    Marks mk;
    QW_CUDA(enqueue_step(m, &mk), "profiled decode step");
    QW_CUDA(cudaStreamSynchronize(m->stream), "profiled decode step");
    if (!check_state(m, nullptr)) return 0;
    double forward = 0.0;
    for (size_t i = 0; i < mk.what.size(); ++i) {
        float ms = 0.f;
        QW_CUDA(cudaEventElapsedTime(&ms, m->prof_events[i], m->prof_events[i + 1]), "profile events");
        const double dt = (double)ms * 1e-3;
        const Mark &w = mk.what[i];
        switch (w.stage) {
        case kStageLayerGemv:
            profile->matvec_seconds += dt;
            add_weight(profile->weight_layer_seconds, profile->weight_layer_calls, w.type[0], dt * w.share0,
                       w.calls[0]);
            if (w.calls[1] > 0)
                add_weight(profile->weight_layer_seconds, profile->weight_layer_calls, w.type[1],
                           dt * (1.0 - w.share0), w.calls[1]);
            break;
        case kStageAttention: profile->attention_seconds += dt; break;
        case kStageOutput:
            profile->output_seconds += dt;
            add_weight(profile->weight_output_seconds, profile->weight_output_calls, w.type[0], dt, w.calls[0]);
            break;
        case kStageSampling:
            profile->sampling_seconds += dt;
            ++profile->sampling_calls;
            break;
        default: break;
        }
        if (w.stage != kStageSampling) forward += dt;  // forward stages exclude sampling
    }
    profile->forward_seconds += forward;
    ++profile->forward_calls;
    if (logits)
        QW_CUDA(cudaMemcpy(logits, m->logits, (size_t)m->cfg.vocab_size * sizeof(float), cudaMemcpyDeviceToHost),
                "read logits");
    if (next_token) QW_CUDA(cudaMemcpy(next_token, m->history, sizeof(int), cudaMemcpyDeviceToHost), "read token");
    return 1;
}

namespace {

constexpr int kPrefillChunk = 1024;  // positions per chunk (activation buffers scale with it)

int prefill_buffers(QmvQwen2 *m)
{
    if (m->pf_cap > 0) return 1;
    const QmvQwen2Config &c = m->cfg;
    const size_t C = (size_t)(c.max_context < kPrefillChunk ? c.max_context : kPrefillChunk);
    const size_t dim = (size_t)c.dim, hid = (size_t)c.hidden_dim, kvd = (size_t)m->kvd;
    if (!dalloc(m, (void **)&m->pf_ids, C * sizeof(int), "prefill ids") ||
        !dalloc(m, (void **)&m->pf_h, C * dim * sizeof(float), "prefill activations") ||
        !dalloc(m, (void **)&m->pf_xn, C * dim * sizeof(float), "prefill activations") ||
        !dalloc(m, (void **)&m->pf_qkv, C * (dim + 2 * kvd) * sizeof(float), "prefill activations") ||
        !dalloc(m, (void **)&m->pf_att, C * dim * sizeof(float), "prefill activations") ||
        !dalloc(m, (void **)&m->pf_y, C * dim * sizeof(float), "prefill activations") ||
        !dalloc(m, (void **)&m->pf_gu, C * 2 * hid * sizeof(float), "prefill activations") ||
        !dalloc(m, (void **)&m->pf_part,
                qmv::prefill_attention_part_floats(c.n_heads, m->head_dim, (int)C) * sizeof(float),
                "prefill attention partials") ||
        !dalloc(m, (void **)&m->pf_cnt, (size_t)c.n_kv_heads * C * sizeof(unsigned int), "prefill counters"))
        return 0;
    QW_CUDA(cudaStreamCreateWithFlags(&m->pf_side, cudaStreamNonBlocking), "prefill stream");
    QW_CUDA(cudaEventCreateWithFlags(&m->pf_fork, cudaEventDisableTiming), "prefill event");
    QW_CUDA(cudaEventCreateWithFlags(&m->pf_join, cudaEventDisableTiming), "prefill event");
    m->pf_cap = (int)C;
    return 1;
}

cudaError_t matmul(QmvQwen2 *m, const QmvWeight *w, const float *X, int n, float *Y)
{
    return qmv::launch_matmul(w->L, w->dev, X, n, Y, m->stream);
}

// Positions pos0 .. pos0 + n - 1 (ids already on the device) through every
// layer: the reference's per-chunk schedule (src/qwen2_architecture.cpp:
// 1586-1690) with the chunk's positions batched in every projection.  The
// residual projections (o, down) leave split-K partial products that the next
// RMSNorm folds into the residual stream; gate and up of different formats
// run on two streams so their CTAs share the SMs.
cudaError_t enqueue_prefill_chunk(QmvQwen2 *m, int pos0, int n)
{
    const QmvQwen2Config &c = m->cfg;
    const int dim = c.dim, hid = c.hidden_dim, kvd = m->kvd;
    cudaStream_t st = m->stream;
    float *pend = nullptr;  // the previous down projection's partials, not yet in h
    int pend_ks = 0;
    auto fold = [&](const float *norm) {  // h += pending partials; xn = rmsnorm(h)
        cudaError_t e = pend ? qmv::launch_rmsnorm_residual(m->pf_h, pend, pend_ks, norm, c.rms_norm_epsilon, dim, n,
                                                            m->pf_xn, st)
                             : qmv::launch_rmsnorm_rows(m->pf_h, norm, c.rms_norm_epsilon, dim, n, m->pf_xn, st);
        if (pend) {
            const cudaError_t f = cudaFreeAsync(pend, st);
            if (e == cudaSuccess) e = f;
            pend = nullptr;
        }
        return e;
    };
    cudaError_t e = qmv::launch_embed_rows(m->embd->L, m->embd->dev, m->pf_ids, n, m->pf_h, &m->st->error, st);
    for (int l = 0; l < c.n_layers && e == cudaSuccess; ++l) {
        const Layer &L = m->layers[(size_t)l];
        e = fold(L.attn_norm);
        float *q = m->pf_qkv, *k, *v;
        int q_ld, k_ld, v_ld;
        if (L.qkv) {
            if (e == cudaSuccess) e = matmul(m, L.qkv, m->pf_xn, n, m->pf_qkv);
            k = q + dim;
            v = k + kvd;
            q_ld = k_ld = v_ld = dim + 2 * kvd;
        } else {
            k = q + (size_t)n * dim;
            v = k + (size_t)n * kvd;
            q_ld = dim;
            k_ld = v_ld = kvd;
            if (e == cudaSuccess) e = matmul(m, L.q, m->pf_xn, n, q);
            if (e == cudaSuccess) e = matmul(m, L.k, m->pf_xn, n, k);
            if (e == cudaSuccess) e = matmul(m, L.v, m->pf_xn, n, v);
        }
        const size_t off = (size_t)l * (size_t)c.max_context * (size_t)kvd;
        if (e == cudaSuccess)
            e = qmv::launch_rope_kv(q, q_ld, k, k_ld, v, v_ld, L.bias_qkv, L.bias_qkv + dim, L.bias_qkv + dim + kvd,
                                    c.n_heads, c.n_kv_heads, m->head_dim, pos0, n, c.rope_frequency_base, m->kc + off,
                                    m->vc + off, st);
        if (e == cudaSuccess)
            e = qmv::launch_prefill_attention(q, q_ld, m->kc + off, m->vc + off, c.n_heads, c.n_kv_heads, m->head_dim,
                                              pos0, n, m->pf_att, m->pf_part, m->pf_cnt, st);
        if (e == cudaSuccess) e = qmv::launch_matmul_partials(L.o->L, L.o->dev, m->pf_att, n, &pend, &pend_ks, st);
        if (e == cudaSuccess) e = fold(L.ffn_norm);
        // the down projection reads x = up * silu(gate) straight from the
        // gate / up outputs (the SwiGLU is formed as its x is split)
        const float *gate = m->pf_gu, *upv = m->pf_gu + hid;
        int g_ld = 2 * hid, u_ld = 2 * hid;
        if (L.gate_up) {  // [gate | up] rows of 2 * hid
            if (e == cudaSuccess) e = matmul(m, L.gate_up, m->pf_xn, n, m->pf_gu);
        } else {
            float *up = m->pf_gu + (size_t)n * hid;
            if (e == cudaSuccess) e = cudaEventRecord(m->pf_fork, st);
            if (e == cudaSuccess) e = cudaStreamWaitEvent(m->pf_side, m->pf_fork, 0);
            if (e == cudaSuccess) e = qmv::launch_matmul(L.up->L, L.up->dev, m->pf_xn, n, up, m->pf_side);
            if (e == cudaSuccess) e = matmul(m, L.gate, m->pf_xn, n, m->pf_gu);
            if (e == cudaSuccess) e = cudaEventRecord(m->pf_join, m->pf_side);
            if (e == cudaSuccess) e = cudaStreamWaitEvent(st, m->pf_join, 0);
            upv = up;
            g_ld = u_ld = hid;
        }
        if (e == cudaSuccess)
            e = qmv::launch_matmul_partials_swiglu(L.down->L, L.down->dev, gate, g_ld, upv, u_ld, n, &pend, &pend_ks,
                                                   st);
    }
    if (pend) {  // the last layer's down projection
        if (e == cudaSuccess) e = qmv::launch_add_partials(m->pf_h, pend, (size_t)n * dim, pend_ks, st);
        const cudaError_t f = cudaFreeAsync(pend, st);
        if (e == cudaSuccess) e = f;
    }
    return e;
}

}  // namespace

// The reference's prefill_tokens (qwen2_prefill_tokens,
// src/qwen2_architecture.cpp:1550-1729): append `count` tokens at the current
// position, writing their keys and values into every layer's cache, and
// publish the logits of the last one (plus its greedy token).  Same checks and
// messages; on failure the position is unchanged.  One token is one decode
// step, as in the reference.
QMV_EXPORT int qmv_qwen2_prefill(QmvQwen2 *m, const int *ids, int count, float *logits, int *next_token)
{
    if (m == nullptr || ids == nullptr || count <= 0) return qmv::set_error("Qwen2 prefill arguments are invalid.");
    const QmvQwen2Config &c = m->cfg;
    qmv::DecodeState st{};
    if (!check_state(m, &st)) return 0;
    const int pos0 = st.pos;
    if (pos0 < 0 || pos0 > c.max_context || count > c.max_context - pos0)
        return qmv::set_error("Qwen2 prefill context capacity is exhausted.");
    for (int i = 0; i < count; ++i)
        if (ids[i] < 0 || ids[i] >= c.vocab_size) return qmv::set_error("Qwen2 prefill token ID is out of range.");
    if (count == 1) return qmv_qwen2_forward(m, ids[0], logits, next_token);
    if (!prefill_buffers(m)) return 0;
    int last_n = 0;
    for (int start = 0; start < count; start += m->pf_cap) {
        const int n = count - start < m->pf_cap ? count - start : m->pf_cap;
        QW_CUDA(cudaMemcpyAsync(m->pf_ids, ids + start, (size_t)n * sizeof(int), cudaMemcpyHostToDevice, m->stream),
                "prefill ids");
        QW_CUDA(enqueue_prefill_chunk(m, pos0 + start, n), "prefill");
        last_n = n;
    }
    // the last position's logits: output_norm, output projection, greedy argmax
    const qmv::ArgmaxOut am{m->key, m->am_ws, 0};
    QW_CUDA(gemv(m, m->out, m->pf_h + (size_t)(last_n - 1) * c.dim, m->logits,
                 qmv::Fuse{qmv::kPreRmsNorm, m->out_norm, c.rms_norm_epsilon, nullptr, nullptr}, &am),
            "prefill output");
    unsigned long long key = 0;
    QW_CUDA(cudaMemcpyAsync(&key, m->key, sizeof key, cudaMemcpyDeviceToHost, m->stream), "prefill output");
    QW_CUDA(cudaStreamSynchronize(m->stream), "prefill");
    if (!check_state(m, nullptr)) return 0;
    if (key == 0ull || key == ~0ull) return qmv::set_error("Output contains a non-finite logit.");
    const int pos = pos0 + count;
    QW_CUDA(cudaMemcpy(&m->st->pos, &pos, sizeof pos, cudaMemcpyHostToDevice), "prefill position");
    if (logits)
        QW_CUDA(cudaMemcpy(logits, m->logits, (size_t)c.vocab_size * sizeof(float), cudaMemcpyDeviceToHost),
                "read logits");
    if (next_token) *next_token = (int)(0xffffffffu - (unsigned int)(key & 0xffffffffull));
    return 1;
}

QMV_EXPORT int qmv_qwen2_generate(QmvQwen2 *m, int first_token, int steps, int *tokens)
{
    if (m == nullptr || steps <= 0 || tokens == nullptr) return qmv::set_error("bad generate request");
    if (!set_token(m, first_token) || !qmv_qwen2_replay(m, steps, m->stream)) return 0;
    QW_CUDA(cudaStreamSynchronize(m->stream), "decode steps");
    return qmv_qwen2_read(m, tokens, steps, nullptr);
}

QMV_EXPORT int qmv_qwen2_get_kv(QmvQwen2 *m, int layer, int position, float *key, float *value)
{
    if (m == nullptr || key == nullptr || value == nullptr || layer < 0 || layer >= m->cfg.n_layers || position < 0 ||
        position >= m->cfg.max_context)
        return qmv::set_error("bad KV request");
    const size_t off = ((size_t)layer * (size_t)m->cfg.max_context + (size_t)position) * (size_t)m->kvd;
    QW_CUDA(cudaMemcpy(key, m->kc + off, (size_t)m->kvd * sizeof(float), cudaMemcpyDeviceToHost), "read kv");
    QW_CUDA(cudaMemcpy(value, m->vc + off, (size_t)m->kvd * sizeof(float), cudaMemcpyDeviceToHost), "read kv");
    return 1;
}

QMV_EXPORT int qmv_set_decode_mode(int mode)
{
    if (mode < 0 || mode > 1) return qmv::set_error("decode mode must be 0 or 1");
    g_decode_mode = mode;
    return 1;
}

QMV_EXPORT int qmv_set_attention_path(int path)
{
    if (path < 0 || path > 1) return qmv::set_error("attention path must be 0 or 1");
    qmv::set_attention_path(path);
    return 1;
}

QMV_EXPORT int qmv_qwen2_kernels_per_step(const QmvQwen2 *m)
{
    if (m == nullptr) return qmv::set_error("null decoder");
    return m->kernels_per_step;
}

QMV_EXPORT int qmv_qwen2_destroy(QmvQwen2 *m)
{
    if (m == nullptr) return qmv::set_error("null decoder");
    release(m);
    return 1;
}
