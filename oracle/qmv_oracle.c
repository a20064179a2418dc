/*
 * CPU ORACLE — TEST INFRASTRUCTURE ONLY.
 *
 * This file restates, in plain C, the scalar (non-SIMD) arithmetic of the
 * reference engine's quantized matrix-vector path so that tests can check the
 * CUDA path against it.  Only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline leg may load it; the product library never links or calls it.
 *
 * Parity pin: every function here is compared bit-for-bit with the reference's
 * own sources compiled from the reference checkout by oracle/Makefile (the
 * `_ref` libraries), and with the known-answer blocks of the reference's tests
 * (tests/q8_0_reference_test.cpp, q5_0_..., q4_k_..., q6_k_...,
 * quantized_matvec_reference_test.cpp, sampler_greedy_test.cpp), see
 * tests/test_oracle.py.
 *
 * Packed blocks are passed as raw bytes (GGUF little-endian layout); the
 * reference's struct layouts are restated as byte offsets.
 *
 * Build: cc -O2 -ffp-contract=off -fPIC -shared (no FMA contraction, so every
 * product and sum rounds exactly as the reference's scalar build does).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

/* GGML type ids: src/gguf_reader.h:7-11. */
#define OR_Q5_0 6u
#define OR_Q8_0 8u
#define OR_Q4_K 12u
#define OR_Q6_K 14u

static uint16_t rd16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* IEEE binary16 -> binary32 by bit expansion.
 * Follows src/quantization.cpp:11-52 (portable branch :23-49): subnormals are
 * renormalised, Inf keeps its sign, NaN payloads are shifted up and quieted. */
float or_f16_to_f32(uint16_t h)
{
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1fu;
    uint32_t m = h & 0x3ffu;
    uint32_t bits;
    if (e == 0u) {
        if (m == 0u) {
            bits = sign;
        } else {
            /* value = m * 2^-24; find the leading one and renormalise */
            int exp32 = 127 - 15 + 1;
            while ((m & 0x400u) == 0u) { m <<= 1; exp32--; }
            bits = sign | ((uint32_t)exp32 << 23) | ((m & 0x3ffu) << 13);
        }
    } else if (e == 31u) {
        bits = sign | 0x7f800000u | (m << 13) | (m ? 0x00400000u : 0u);
    } else {
        bits = sign | ((e + (127u - 15u)) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* ---------------- Q8_0: 2 B fp16 d + 32 x int8 (quantization.h:33-36) ---- */

/* quantization.cpp:54-67: out[i] = d * q[i] */
void or_q8_0_dequant(const uint8_t *blk, float *out)
{
    float d = or_f16_to_f32(rd16(blk));
    const int8_t *q = (const int8_t *)(blk + 2);
    for (int i = 0; i < 32; i++) out[i] = d * (float)q[i];
}

/* quantization.cpp:150-156 (scalar branch): acc += (d * q[i]) * x[i] */
float or_q8_0_dot(const uint8_t *blk, const float *x)
{
    float d = or_f16_to_f32(rd16(blk));
    const int8_t *q = (const int8_t *)(blk + 2);
    float acc = 0.0f;
    for (int i = 0; i < 32; i++) acc += d * (float)q[i] * x[i];
    return acc;
}

/* ---------------- Q5_0: d (2) + qh (4) + qs (16) (quantization.h:93-97) --- */

static int q5_0_value(const uint8_t *blk, int i)
{
    const uint8_t *qh = blk + 2;
    const uint8_t *qs = blk + 6;
    int nib = (i < 16) ? (qs[i] & 0x0f) : (qs[i - 16] >> 4);
    int hi = (qh[i >> 3] >> (i & 7)) & 1;
    return (nib | (hi << 4)) - 16;
}

/* quantization.cpp:161-184: out[i] = d * (v - 16) */
void or_q5_0_dequant(const uint8_t *blk, float *out)
{
    float d = or_f16_to_f32(rd16(blk));
    for (int i = 0; i < 32; i++) out[i] = d * (float)q5_0_value(blk, i);
}

/* quantization.cpp:332-346 (scalar branch): acc += (d * v) * x[i] */
float or_q5_0_dot(const uint8_t *blk, const float *x)
{
    float d = or_f16_to_f32(rd16(blk));
    float acc = 0.0f;
    for (int i = 0; i < 32; i++) acc += d * (float)q5_0_value(blk, i) * x[i];
    return acc;
}

/* ---------------- Q4_K: d, dmin, 12 B scales, 128 B nibbles (h:152-157) --- */

/* 6-bit scale/min of sub-block j from the 12-byte field.
 * quantization.cpp:351-378 (layout described at quantization.h:169-179). */
void or_q4_k_scale_min(const uint8_t *sm, int j, uint8_t *sc, uint8_t *mn)
{
    if (j < 4) {
        *sc = sm[j] & 63;
        *mn = sm[j + 4] & 63;
    } else {
        *sc = (uint8_t)((sm[j + 4] & 0x0f) | ((sm[j - 4] >> 6) << 4));
        *mn = (uint8_t)((sm[j + 4] >> 4) | ((sm[j] >> 6) << 4));
    }
}

/* quantization.cpp:380-409: out = (d*sc) * nib - (dmin*m), two roundings
 * for the products and one for the difference (no fused multiply-add). */
void or_q4_k_dequant(const uint8_t *blk, float *out)
{
    float d = or_f16_to_f32(rd16(blk));
    float dmin = or_f16_to_f32(rd16(blk + 2));
    const uint8_t *sm = blk + 4;
    const uint8_t *qs = blk + 16;
    for (int j = 0; j < 8; j++) {
        uint8_t sc, mn;
        or_q4_k_scale_min(sm, j, &sc, &mn);
        float scale = d * (float)sc;
        float minimum = dmin * (float)mn;
        const uint8_t *p = qs + 32 * (j >> 1);
        int shift = (j & 1) * 4;
        for (int o = 0; o < 32; o++) {
            float t = scale * (float)((p[o] >> shift) & 0x0f);
            out[32 * j + o] = t - minimum;
        }
    }
}

/* quantization.cpp:536-554 (scalar branch): sub-block order, then offset. */
float or_q4_k_dot(const uint8_t *blk, const float *x)
{
    float d = or_f16_to_f32(rd16(blk));
    float dmin = or_f16_to_f32(rd16(blk + 2));
    const uint8_t *sm = blk + 4;
    const uint8_t *qs = blk + 16;
    float acc = 0.0f;
    for (int j = 0; j < 8; j++) {
        uint8_t sc, mn;
        or_q4_k_scale_min(sm, j, &sc, &mn);
        float scale = d * (float)sc;
        float minimum = dmin * (float)mn;
        const uint8_t *p = qs + 32 * (j >> 1);
        int shift = (j & 1) * 4;
        for (int o = 0; o < 32; o++) {
            float w = scale * (float)((p[o] >> shift) & 0x0f) - minimum;
            acc += w * x[32 * j + o];
        }
    }
    return acc;
}

/* ---------------- Q6_K: ql 128, qh 64, sc 16 x int8, d (h:236-241) ------- */

/* Weight index i -> signed 6-bit value and int8 scale multiplier.
 * quantization.cpp:559-586 (layout quantization.h:220-234, 254-258). */
void or_q6_k_value(const uint8_t *blk, int i, int *q, int *sc)
{
    const uint8_t *ql = blk;
    const uint8_t *qh = blk + 128;
    const int8_t *scales = (const int8_t *)(blk + 192);
    int g = i >> 7, local = i & 127, r = local >> 5, o = local & 31;
    int lo = (ql[64 * g + 32 * (r & 1) + o] >> (4 * (r >> 1))) & 0x0f;
    int hi = (qh[32 * g + o] >> (2 * r)) & 0x03;
    *q = (lo | (hi << 4)) - 32;
    *sc = scales[8 * g + 2 * r + (o >> 4)];
}

/* quantization.cpp:588-615: out = (d * sc) * q, evaluated left to right. */
void or_q6_k_dequant(const uint8_t *blk, float *out)
{
    float d = or_f16_to_f32(rd16(blk + 208));
    for (int i = 0; i < 256; i++) {
        int q, sc;
        or_q6_k_value(blk, i, &q, &sc);
        out[i] = d * (float)sc * (float)q;
    }
}

/* quantization.cpp:734-753 (scalar branch); index order = natural order. */
float or_q6_k_dot(const uint8_t *blk, const float *x)
{
    float d = or_f16_to_f32(rd16(blk + 208));
    float acc = 0.0f;
    for (int i = 0; i < 256; i++) {
        int q, sc;
        or_q6_k_value(blk, i, &q, &sc);
        acc += (d * (float)sc * (float)q) * x[i];
    }
    return acc;
}

/* ---------------- tensor-level helpers ----------------------------------- */

int or_block_elements(uint32_t type)
{
    switch (type) {
    case OR_Q5_0: case OR_Q8_0: return 32;
    case OR_Q4_K: case OR_Q6_K: return 256;
    default: return 0;
    }
}

int or_block_bytes(uint32_t type)
{
    switch (type) {
    case OR_Q5_0: return 22;
    case OR_Q8_0: return 34;
    case OR_Q4_K: return 144;
    case OR_Q6_K: return 210;
    default: return 0;
    }
}

static float block_dot(uint32_t type, const uint8_t *blk, const float *x)
{
    switch (type) {
    case OR_Q5_0: return or_q5_0_dot(blk, x);
    case OR_Q8_0: return or_q8_0_dot(blk, x);
    case OR_Q4_K: return or_q4_k_dot(blk, x);
    default: return or_q6_k_dot(blk, x);
    }
}

static void block_dequant(uint32_t type, const uint8_t *blk, float *out)
{
    switch (type) {
    case OR_Q5_0: or_q5_0_dequant(blk, out); break;
    case OR_Q8_0: or_q8_0_dequant(blk, out); break;
    case OR_Q4_K: or_q4_k_dequant(blk, out); break;
    default: or_q6_k_dequant(blk, out); break;
    }
}

/* Dequantize nblocks consecutive blocks. Returns 0 for an unknown type. */
int or_dequant_blocks(uint32_t type, const uint8_t *data, uint64_t nblocks, float *out)
{
    int be = or_block_elements(type), bb = or_block_bytes(type);
    if (be == 0) return 0;
    for (uint64_t b = 0; b < nblocks; b++) block_dequant(type, data + b * bb, out + b * be);
    return 1;
}

/* Rows [row_begin, row_end) of y = W x.  Per row, block dots are summed in
 * block order starting from 0.0f: quantized_matvec.cpp:10-84 (accumulation
 * :36,49,62,75), driven row by row as in :151-160. */
int or_matvec_rows(uint32_t type, const uint8_t *data, int rows, int cols,
                   const float *x, float *y, int row_begin, int row_end)
{
    int be = or_block_elements(type), bb = or_block_bytes(type);
    if (be == 0 || cols % be != 0 || row_begin < 0 || row_end > rows) return 0;
    int nb = cols / be;
    for (int r = row_begin; r < row_end; r++) {
        float acc = 0.0f;
        const uint8_t *row = data + (uint64_t)r * nb * bb;
        for (int b = 0; b < nb; b++) acc += block_dot(type, row + (uint64_t)b * bb, x + b * be);
        y[r] = acc;
    }
    return 1;
}

int or_matvec(uint32_t type, const uint8_t *data, int rows, int cols,
              const float *x, float *y)
{
    return or_matvec_rows(type, data, rows, cols, x, y, 0, rows);
}

/* Y[p, r] for p < batch: quantized_matvec.cpp:164-224.  Y starts at 0.0f and
 * each block's dot for position p is added in block order (:197-211). */
int or_matmul(uint32_t type, const uint8_t *data, int rows, int cols,
              const float *X, int batch, float *Y)
{
    int be = or_block_elements(type), bb = or_block_bytes(type);
    if (be == 0 || cols % be != 0) return 0;
    int nb = cols / be;
    for (int r = 0; r < rows; r++) {
        for (int p = 0; p < batch; p++) Y[(uint64_t)p * rows + r] = 0.0f;
        for (int b = 0; b < nb; b++) {
            const uint8_t *blk = data + ((uint64_t)r * nb + b) * bb;
            for (int p = 0; p < batch; p++)
                Y[(uint64_t)p * rows + r] += block_dot(type, blk, X + (uint64_t)p * cols + b * be);
        }
    }
    return 1;
}

/* Per-row tolerance scale S[r] = sum_k |w_rk * x_k| with w the reference's
 * dequantized weight, accumulated in double (tolerance = 1e-4 * S[r]). */
int or_row_abs_dot(uint32_t type, const uint8_t *data, int rows, int cols,
                   const float *x, double *s)
{
    int be = or_block_elements(type), bb = or_block_bytes(type);
    if (be == 0 || cols % be != 0) return 0;
    int nb = cols / be;
    float w[256];
    for (int r = 0; r < rows; r++) {
        double acc = 0.0;
        for (int b = 0; b < nb; b++) {
            block_dequant(type, data + ((uint64_t)r * nb + b) * bb, w);
            for (int i = 0; i < be; i++) acc += fabs((double)w[i] * (double)x[b * be + i]);
        }
        s[r] = acc;
    }
    return 1;
}

/* Greedy argmax: src/sampler.cpp:14-36.  Strict '>' keeps the lowest id on
 * ties; any NaN/Inf anywhere fails (returns 0, *id = -1). */
int or_argmax(const float *logits, int n, int *id)
{
    if (id) *id = -1;
    if (logits == 0 || n <= 0 || id == 0) return 0;
    int best = 0;
    for (int i = 0; i < n; i++) {
        if (!isfinite(logits[i])) return 0;
        if (logits[i] > logits[best]) best = i;
    }
    *id = best;
    return 1;
}

/* ------------------------------------------------------------------------
 * Qwen2 decode step (configuration 4): the reference's
 * qwen2_forward_token_cached_impl (src/qwen2_architecture.cpp:1195-1531) with
 * its helpers tensor_rms_norm_f32 (src/tensor.cpp:99-136), tensor_dot_f32
 * (:25-45), tensor_add_f32 (:5-23), transformer_apply_rope_f32 and
 * transformer_attention_f32 (src/transformer_ops.cpp:16-153) and
 * transformer_swiglu_f32 (:155-178), restated in the same operation order.
 * ---------------------------------------------------------------------- */

/* type 0: F32 rows */
typedef struct OrTensor {
    uint32_t type;
    const uint8_t *data;
} OrTensor;

typedef struct OrQwen2Layer {
    const float *attn_norm, *ffn_norm, *q_bias, *k_bias, *v_bias;
    OrTensor q, k, v, o, gate, up, down;
} OrQwen2Layer;

typedef struct OrQwen2 {
    int dim, hidden, layers, heads, kv_heads, vocab, max_ctx;
    float eps, rope_base;
    OrTensor embd;
    const float *out_norm;
    OrTensor out;
    const OrQwen2Layer *layer;
} OrQwen2;

static int or_tensor_matvec(OrTensor t, int rows, int cols, const float *x, float *y)
{
    if (t.type == 0) {
        const float *w = (const float *)t.data;
        for (int r = 0; r < rows; r++) {
            float acc = 0.0f;
            for (int c = 0; c < cols; c++) acc += w[(size_t)r * cols + c] * x[c];
            y[r] = acc;
        }
        return 1;
    }
    return or_matvec(t.type, t.data, rows, cols, x, y);
}

/* tensor_rms_norm_f32: sum of squares in order, sqrtf(mean + eps), then
 * (x / denom) * weight. */
static void or_rms_norm(const float *x, const float *w, int n, float eps, float *out)
{
    float denom = 0.0f;
    for (int j = 0; j < n; j++) denom += x[j] * x[j];
    denom = sqrtf((denom / n) + eps);
    for (int i = 0; i < n; i++) out[i] = (x[i] / denom) * w[i];
}

/* rotate_array_helper: pairs (i, i + d/2) of every head. */
static void or_rope(float *v, int heads, int d, int pos, float base)
{
    for (int h = 0; h < heads; h++) {
        int s = h * d;
        for (int i = 0; i < d / 2; i++) {
            float x = v[s + i];
            float y = v[s + i + d / 2];
            float angle = (float)pos / powf(base, (2.0f * (float)i / (float)d));
            float rx = x * cosf(angle) - y * sinf(angle);
            float ry = x * sinf(angle) + y * cosf(angle);
            v[s + i] = rx;
            v[s + i + d / 2] = ry;
        }
    }
}

/* transformer_attention_f32 over tokens [0, T) of one layer's cache. */
static int or_attention(const float *q, int heads, int kv_heads, int d, const float *keys,
                        const float *values, int T, float *prob, float *out)
{
    for (int h = 0; h < heads; h++) {
        const float *qh = q + h * d;
        int kvh = h / (heads / kv_heads);
        for (int t = 0; t < T; t++) {
            const float *k = keys + ((size_t)t * kv_heads + kvh) * d;
            float score = 0.0f;
            for (int i = 0; i < d; i++) score += qh[i] * k[i];
            score /= sqrtf((float)d);
            prob[h * T + t] = score;
        }
        float mx = prob[h * T];
        for (int t = 1; t < T; t++)
            if (prob[h * T + t] > mx) mx = prob[h * T + t];
        float sum = 0.0f;
        for (int t = 0; t < T; t++) {
            prob[h * T + t] = expf(prob[h * T + t] - mx);
            sum += prob[h * T + t];
        }
        if (!isfinite(sum) || sum <= 0.0f) return 0;
        for (int t = 0; t < T; t++) prob[h * T + t] /= sum;
        for (int i = 0; i < d; i++) out[h * d + i] = 0.0f;
        for (int t = 0; t < T; t++) {
            float p = prob[h * T + t];
            const float *v = values + ((size_t)t * kv_heads + kvh) * d;
            for (int i = 0; i < d; i++) out[h * d + i] += p * v[i];
        }
    }
    return 1;
}

/* Workspace floats or_qwen2_forward needs. */
int or_qwen2_scratch_floats(const OrQwen2 *m)
{
    int big = m->hidden > m->dim ? m->hidden : m->dim;
    return 5 * m->dim + 2 * m->kv_heads * (m->dim / m->heads) + m->heads * m->max_ctx + 3 * big;
}

/* One decode step at position pos for token: keys/values are the caller's
 * cache [layers][max_ctx][kv_heads * head_dim] (positions < pos filled; the
 * step writes position pos), logits[vocab] out.  0 on a non-finite softmax
 * sum or logit, as the reference fails. */
int or_qwen2_forward(const OrQwen2 *m, float *keys, float *values, int pos, int token,
                     float *logits, float *scratch)
{
    const int dim = m->dim, hd = dim / m->heads, kvd = m->kv_heads * hd;
    const int big = m->hidden > dim ? m->hidden : dim;
    float *h = scratch, *xn = h + dim, *q = xn + dim, *att = q + dim, *tmp = att + dim;
    float *k = tmp + dim, *v = k + kvd, *prob = v + kvd;
    float *gate = prob + m->heads * m->max_ctx, *up = gate + big, *mv = up + big;
    if (pos < 0 || pos >= m->max_ctx || token < 0 || token >= m->vocab) return 0;

    /* embedding row (qwen2_lookup_embedding, :477-528) */
    if (m->embd.type == 0) {
        memcpy(h, (const float *)m->embd.data + (size_t)token * dim, (size_t)dim * sizeof(float));
    } else {
        int be = or_block_elements(m->embd.type), bb = or_block_bytes(m->embd.type);
        int nb = dim / be;
        or_dequant_blocks(m->embd.type, m->embd.data + (size_t)token * nb * bb, (uint64_t)nb, h);
    }
    for (int l = 0; l < m->layers; l++) {
        const OrQwen2Layer *L = &m->layer[l];
        float *kc = keys + (size_t)l * m->max_ctx * kvd, *vc = values + (size_t)l * m->max_ctx * kvd;
        or_rms_norm(h, L->attn_norm, dim, m->eps, xn);
        /* qwen2_layer_project: matvec, then output + bias */
        or_tensor_matvec(L->q, dim, dim, xn, q);
        for (int i = 0; i < dim; i++) q[i] = q[i] + L->q_bias[i];
        or_tensor_matvec(L->k, kvd, dim, xn, k);
        for (int i = 0; i < kvd; i++) k[i] = k[i] + L->k_bias[i];
        or_tensor_matvec(L->v, kvd, dim, xn, v);
        for (int i = 0; i < kvd; i++) v[i] = v[i] + L->v_bias[i];
        or_rope(q, m->heads, hd, pos, m->rope_base);
        or_rope(k, m->kv_heads, hd, pos, m->rope_base);
        memcpy(kc + (size_t)pos * kvd, k, (size_t)kvd * sizeof(float));
        memcpy(vc + (size_t)pos * kvd, v, (size_t)kvd * sizeof(float));
        if (!or_attention(q, m->heads, m->kv_heads, hd, kc, vc, pos + 1, prob, att)) return 0;
        or_tensor_matvec(L->o, dim, dim, att, mv);
        for (int i = 0; i < dim; i++) h[i] = mv[i] + h[i];
        or_rms_norm(h, L->ffn_norm, dim, m->eps, xn);
        or_tensor_matvec(L->gate, m->hidden, dim, xn, gate);
        or_tensor_matvec(L->up, m->hidden, dim, xn, up);
        for (int i = 0; i < m->hidden; i++) gate[i] = up[i] * (gate[i] / (1.0f + expf(-gate[i])));
        or_tensor_matvec(L->down, dim, m->hidden, gate, mv);
        for (int i = 0; i < dim; i++) h[i] = h[i] + mv[i];
    }
    or_rms_norm(h, m->out_norm, dim, m->eps, xn);
    or_tensor_matvec(m->out, m->vocab, dim, xn, logits);
    for (int j = 0; j < m->vocab; j++)
        if (!isfinite(logits[j])) return 0;
    return 1;
}
