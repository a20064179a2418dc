// TEST INFRASTRUCTURE ONLY — compiled by oracle/Makefile together with the
// reference engine's own sources (src/qwen2_architecture.cpp, gguf_reader.cpp,
// tensor.cpp, transformer_ops.cpp, quantization.cpp, quantized_matvec.cpp, read
// in place from the reference checkout) into oracle/_ref/.  It runs the
// reference's Qwen2 decode step (qwen2_forward_token_cached_impl,
// src/qwen2_architecture.cpp:1195-1531) on an in-memory model assembled the way
// tests/forward_quantized_reference_test.cpp:26-117 assembles its fixture, with
// the KV cache pre-filled through the private state
// (src/qwen2_internal.h:21-52).  Nothing in the product links this file.
#include <stddef.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "engine.h"
#include "engine_internal.h"
#include "qwen2_architecture.h"
#include "qwen2_internal.h"
#include "architecture.h"

extern "C" {

// One tensor of the in-memory model: a 2-D matrix (rows > 0) or a 1-D F32
// vector (rows == 0), with its raw bytes.
typedef struct RefTensor {
    const char *name;
    uint32_t type;
    uint64_t cols;
    uint64_t rows;
    const void *data;
    uint64_t bytes;
} RefTensor;

struct RefQwen2 {
    Model model;
    EngineModel impl;
    GgufTensorInfo *tensors;
    char **names;
    int count;
    unsigned char *data;
    InferenceState state;
    int max_context;
};

// cfg = {dim, hidden_dim, n_layers, n_heads, n_kv_heads, vocab_size, seq_len}
void *ref_qwen2_create(const int *cfg, float eps, float rope_base, const RefTensor *t, int n, int max_context)
{
    RefQwen2 *m = (RefQwen2 *)calloc(1, sizeof(RefQwen2));
    if (m == nullptr) return nullptr;
    size_t total = 0;
    for (int i = 0; i < n; ++i) total = ((total + 31) & ~(size_t)31) + (size_t)t[i].bytes;
    m->data = (unsigned char *)calloc(total + 32, 1);
    m->tensors = (GgufTensorInfo *)calloc((size_t)n, sizeof(GgufTensorInfo));
    m->names = (char **)calloc((size_t)n, sizeof(char *));
    if (m->data == nullptr || m->tensors == nullptr || m->names == nullptr) return nullptr;
    size_t used = 0;
    for (int i = 0; i < n; ++i) {
        used = (used + 31) & ~(size_t)31;
        memcpy(m->data + used, t[i].data, (size_t)t[i].bytes);
        m->names[i] = strdup(t[i].name);
        GgufTensorInfo *g = &m->tensors[i];
        g->name = m->names[i];
        g->type = t[i].type;
        g->dimension_count = t[i].rows == 0 ? 1 : 2;
        g->dimensions[0] = t[i].cols;
        g->dimensions[1] = t[i].rows;
        g->offset = used;
        g->byte_size = t[i].bytes;
        used += (size_t)t[i].bytes;
    }
    m->count = n;
    m->impl.gguf.data = m->data;
    m->impl.gguf.file_size = used;
    m->impl.gguf.tensor_count = (uint64_t)n;
    m->impl.gguf.tensors = m->tensors;
    m->impl.architecture = qwen2_architecture_ops();
    m->model.implementation = &m->impl;
    m->model.config.dim = cfg[0];
    m->model.config.hidden_dim = cfg[1];
    m->model.config.n_layers = cfg[2];
    m->model.config.n_heads = cfg[3];
    m->model.config.n_kv_heads = cfg[4];
    m->model.config.vocab_size = cfg[5];
    m->model.config.seq_len = cfg[6];
    m->model.config.rms_norm_epsilon = eps;
    m->model.config.rope_frequency_base = rope_base;
    m->max_context = max_context;
    char error[512] = {};
    if (!qwen2_architecture_ops()->state_init(&m->model, &m->state, max_context, error, sizeof(error))) return nullptr;
    return m;
}

// Pre-fill positions [0, token_count) of every layer's KV cache from
// keys/values laid out [layer][token_count][n_kv_heads * head_dim].
int ref_qwen2_set_kv(void *h, const float *keys, const float *values, int token_count)
{
    RefQwen2 *m = (RefQwen2 *)h;
    Qwen2InferenceState *s = (Qwen2InferenceState *)m->state.implementation;
    if (token_count < 0 || token_count >= s->max_context_tokens) return 0;
    const size_t kvd = (size_t)s->key_value_dimension;
    for (int layer = 0; layer < m->model.config.n_layers; ++layer) {
        const size_t dst = (size_t)layer * (size_t)s->max_context_tokens * kvd;
        const size_t src = (size_t)layer * (size_t)token_count * kvd;
        memcpy(s->keys + dst, keys + src, (size_t)token_count * kvd * sizeof(float));
        memcpy(s->values + dst, values + src, (size_t)token_count * kvd * sizeof(float));
    }
    for (int p = 0; p < token_count; ++p) s->token_ids[p] = 0;
    s->token_count = token_count;
    return 1;
}

// One decode step at the current position; logits[vocab] on success.
int ref_qwen2_forward(void *h, int token, float *logits)
{
    RefQwen2 *m = (RefQwen2 *)h;
    char error[512] = {};
    if (!qwen2_architecture_ops()->forward_token(&m->model, &m->state, token, error, sizeof(error))) return 0;
    memcpy(logits, m->state.logits, (size_t)m->model.config.vocab_size * sizeof(float));
    return 1;
}

// The reference's profile of this decoder state (enabled on first call):
// its OperationProfile bytes are copied to `out` after the next
// ref_qwen2_forward calls accumulate into it.
void ref_qwen2_enable_profile(void *h)
{
    RefQwen2 *m = (RefQwen2 *)h;
    memset(&m->state.profile, 0, sizeof(m->state.profile));
    m->state.profile.enabled = 1;
}

void ref_qwen2_read_profile(void *h, void *out)
{
    RefQwen2 *m = (RefQwen2 *)h;
    memcpy(out, &m->state.profile, sizeof(m->state.profile));
}

// The reference's prefill_tokens (qwen2_prefill_tokens) on `count` ids at the
// state's position; the last position's logits on success.
int ref_qwen2_prefill(void *h, const int *ids, int count, float *logits)
{
    RefQwen2 *m = (RefQwen2 *)h;
    char error[512] = {};
    if (!qwen2_architecture_ops()->prefill_tokens(&m->model, &m->state, ids, count, error, sizeof(error))) return 0;
    memcpy(logits, m->state.logits, (size_t)m->model.config.vocab_size * sizeof(float));
    return 1;
}

// The reference's state_reset: back to position zero.
void ref_qwen2_reset(void *h)
{
    RefQwen2 *m = (RefQwen2 *)h;
    qwen2_architecture_ops()->state_reset(&m->state);
}

// KV entries of one layer and position (after a forward step wrote them).
int ref_qwen2_get_kv(void *h, int layer, int position, float *key, float *value)
{
    RefQwen2 *m = (RefQwen2 *)h;
    Qwen2InferenceState *s = (Qwen2InferenceState *)m->state.implementation;
    const size_t kvd = (size_t)s->key_value_dimension;
    const size_t off = ((size_t)layer * (size_t)s->max_context_tokens + (size_t)position) * kvd;
    memcpy(key, s->keys + off, kvd * sizeof(float));
    memcpy(value, s->values + off, kvd * sizeof(float));
    return 1;
}

// sizeof(OperationProfile) and the offset of each field in declaration
// order (include/metrics.h:8-25): 15 values.
int ref_operation_profile_layout(uint64_t *out)
{
    out[0] = sizeof(OperationProfile);
    out[1] = offsetof(OperationProfile, enabled);
    out[2] = offsetof(OperationProfile, matvec_seconds);
    out[3] = offsetof(OperationProfile, attention_seconds);
    out[4] = offsetof(OperationProfile, rmsnorm_seconds);
    out[5] = offsetof(OperationProfile, rope_seconds);
    out[6] = offsetof(OperationProfile, output_seconds);
    out[7] = offsetof(OperationProfile, sampling_seconds);
    out[8] = offsetof(OperationProfile, weight_layer_seconds);
    out[9] = offsetof(OperationProfile, weight_output_seconds);
    out[10] = offsetof(OperationProfile, weight_layer_calls);
    out[11] = offsetof(OperationProfile, weight_output_calls);
    out[12] = offsetof(OperationProfile, forward_seconds);
    out[13] = offsetof(OperationProfile, forward_calls);
    out[14] = offsetof(OperationProfile, sampling_calls);
    return PROFILE_WEIGHT_FORMAT_COUNT;
}

void ref_qwen2_destroy(void *h)
{
    RefQwen2 *m = (RefQwen2 *)h;
    if (m == nullptr) return;
    qwen2_architecture_ops()->state_destroy(&m->state);
    for (int i = 0; i < m->count; ++i) free(m->names[i]);
    free(m->names);
    free(m->tensors);
    free(m->data);
    free(m);
}

}  // extern "C"
