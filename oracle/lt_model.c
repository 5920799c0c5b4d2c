/*
 * lt_model.c -- TEST INFRASTRUCTURE ONLY (the C1 end-to-end workload).
 *
 * CPU restatement of the reference engine's Llama forward pass
 * (engine/crates/native/src/model.rs:366-518) over Q8_0 weights
 * (engine/crates/native/src/quant.rs: Q8_0 repack :265-273, row_dot Q8
 * branch :405-423, QActs::quantize :771-783, quantize_block :785-795),
 * with the KV cache behind a callback interface so the same forward runs
 * with the oracle's KvCache or with the GPU cache through the C ABI.  The
 * weights are random (seeded) Q8_0 blocks, as BASELINE.json configs[0]
 * specifies; the model is never read from a file.
 *
 * Arithmetic order follows the reference (no fused multiply-add):
 *   row_dot:  sum += (ws[b] * xs[b]) * (float)dot32            quant.rs:418-421
 *   quantize: amax fold, d = amax/127, q = round(x * (1/d))      quant.rs:785-795
 *   rms_norm: ms = sequential sum(v*v)/dim, o = (v*inv)*g      model.rs:174-183
 *   rope:     (2i, 2i+1) pairs, sin/cos of pos*inv_freq[i]     model.rs:291-308
 *   silu:     g / (1 + exp(-g)) * u                            model.rs:492-494
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "lt_model.h"

#define QK 32

typedef struct {
    int rows, cols;
    float* scales; /* per 32-block, rounded through f16 as a GGUF file stores it */
    int8_t* qs;
} qmat;

typedef struct {
    float* attn_norm;
    float* ffn_norm;
    qmat q, k, v, o, gate, up, down;
} olayer;

struct omodel {
    int dim, n_layers, n_heads, n_kv_heads, head_dim, ffn_dim, vocab;
    float eps, rope_base;
    qmat embed, output;
    float* output_norm;
    olayer* layers;
    float* inv_freq;
};

/* ------------------------------------------------------------- weights ---- */

static uint64_t splitmix(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

/* Normal(0, 1) from a counter (Box-Muller on two hashed uniforms). */
static float gauss(uint64_t seed, uint64_t i) {
    uint64_t a = splitmix(seed ^ (2 * i)), b = splitmix(seed ^ (2 * i + 1));
    double u1 = ((a >> 11) + 0.5) * (1.0 / 9007199254740992.0);
    double u2 = (b >> 11) * (1.0 / 9007199254740992.0);
    return (float)(sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2));
}

/* quantize_block (quant.rs:785-795). */
static float quantize_block(const float* x, int8_t* q) {
    float amax = 0.0f;
    for (int i = 0; i < QK; i++) amax = fmaxf(amax, fabsf(x[i]));
    float d = amax / 127.0f;
    float id = d > 0.0f ? 1.0f / d : 0.0f;
    for (int i = 0; i < QK; i++) {
        float r = roundf(x[i] * id);
        q[i] = r != r ? 0 : (r > 127.0f ? 127 : (r < -128.0f ? -128 : (int8_t)r));
    }
    return d;
}

static int make_qmat(qmat* m, int rows, int cols, uint64_t seed, float sigma) {
    m->rows = rows;
    m->cols = cols;
    size_t n = (size_t)rows * cols, nb = n / QK;
    m->qs = (int8_t*)malloc(n);
    m->scales = (float*)malloc(nb * sizeof(float));
    if (!m->qs || !m->scales) return -1;
#pragma omp parallel for schedule(static)
    for (long long b = 0; b < (long long)nb; b++) {
        float x[QK];
        for (int i = 0; i < QK; i++) x[i] = sigma * gauss(seed, (uint64_t)b * QK + i);
        float d = quantize_block(x, m->qs + b * QK);
        m->scales[b] = okv_f16_to_f32(okv_f32_to_f16(d)); /* a GGUF Q8_0 block stores d as f16 */
    }
    return 0;
}

static void free_qmat(qmat* m) {
    free(m->qs);
    free(m->scales);
}

static float* ones(int n) {
    float* v = (float*)malloc(sizeof(float) * n);
    for (int i = 0; i < n; i++) v[i] = 1.0f;
    return v;
}

omodel* om_new_random(int dim, int n_layers, int n_heads, int n_kv_heads, int head_dim, int ffn_dim, int vocab,
                      uint64_t seed) {
    omodel* m = (omodel*)calloc(1, sizeof(omodel));
    if (!m) return NULL;
    m->dim = dim;
    m->n_layers = n_layers;
    m->n_heads = n_heads;
    m->n_kv_heads = n_kv_heads;
    m->head_dim = head_dim;
    m->ffn_dim = ffn_dim;
    m->vocab = vocab;
    m->eps = 1e-5f;        /* model.rs: layer_norm_rms_epsilon default */
    m->rope_base = 10000.0f; /* model.rs: rope.freq_base default */
    const float sd = 0.02f;
    uint64_t s = seed * 1000003ull;
    int rc = make_qmat(&m->embed, vocab, dim, s + 1, 1.0f);
    rc |= make_qmat(&m->output, vocab, dim, s + 2, sd);
    m->output_norm = ones(dim);
    m->layers = (olayer*)calloc((size_t)n_layers, sizeof(olayer));
    int qd = n_heads * head_dim, kvd = n_kv_heads * head_dim;
    for (int l = 0; l < n_layers && !rc; l++) {
        olayer* L = &m->layers[l];
        uint64_t b = s + 100 + 16ull * l;
        L->attn_norm = ones(dim);
        L->ffn_norm = ones(dim);
        rc |= make_qmat(&L->q, qd, dim, b + 0, sd);
        rc |= make_qmat(&L->k, kvd, dim, b + 1, sd);
        rc |= make_qmat(&L->v, kvd, dim, b + 2, sd);
        rc |= make_qmat(&L->o, dim, qd, b + 3, sd);
        rc |= make_qmat(&L->gate, ffn_dim, dim, b + 4, sd);
        rc |= make_qmat(&L->up, ffn_dim, dim, b + 5, sd);
        rc |= make_qmat(&L->down, dim, ffn_dim, b + 6, sd);
    }
    m->inv_freq = (float*)malloc(sizeof(float) * (head_dim / 2));
    for (int i = 0; i < head_dim / 2; i++) /* model.rs:271-273 */
        m->inv_freq[i] = powf(m->rope_base, -2.0f * (float)i / (float)head_dim);
    if (rc) {
        om_delete(m);
        return NULL;
    }
    return m;
}

void om_delete(omodel* m) {
    if (!m) return;
    free_qmat(&m->embed);
    free_qmat(&m->output);
    free(m->output_norm);
    if (m->layers)
        for (int l = 0; l < m->n_layers; l++) {
            olayer* L = &m->layers[l];
            free(L->attn_norm);
            free(L->ffn_norm);
            free_qmat(&L->q);
            free_qmat(&L->k);
            free_qmat(&L->v);
            free_qmat(&L->o);
            free_qmat(&L->gate);
            free_qmat(&L->up);
            free_qmat(&L->down);
        }
    free(m->layers);
    free(m->inv_freq);
    free(m);
}

/* ------------------------------------------------------------- kernels ---- */

typedef struct {
    int n, cols;
    int8_t* qs;
    float* scales;
} qacts;

static void qacts_quantize(qacts* a, const float* x, int n, int cols) { /* quant.rs:771-783 */
    a->n = n;
    a->cols = cols;
    a->qs = (int8_t*)realloc(a->qs, (size_t)n * cols);
    a->scales = (float*)realloc(a->scales, sizeof(float) * ((size_t)n * cols / QK));
    for (size_t b = 0; b < (size_t)n * cols / QK; b++) a->scales[b] = quantize_block(x + b * QK, a->qs + b * QK);
}

static inline int32_t dot32(const int8_t* a, const int8_t* b) {
    int32_t s = 0;
    for (int i = 0; i < QK; i++) s += (int32_t)a[i] * (int32_t)b[i];
    return s;
}

/* out[t][r] = W[r] . x[t] (QMatrix::matmul via row_dot, quant.rs:405-423, 492-533). */
static void matmul(const qmat* w, const qacts* x, float* out, int n_threads) {
    int nb = w->cols / QK, rows = w->rows, n = x->n;
#pragma omp parallel for schedule(static) num_threads(n_threads)
    for (int r = 0; r < rows; r++) {
        const int8_t* wq = w->qs + (size_t)r * w->cols;
        const float* ws = w->scales + (size_t)r * nb;
        for (int t = 0; t < n; t++) {
            const int8_t* xq = x->qs + (size_t)t * w->cols;
            const float* xs = x->scales + (size_t)t * nb;
            float sum = 0.0f;
            for (int b = 0; b < nb; b++) sum += ws[b] * xs[b] * (float)dot32(wq + b * QK, xq + b * QK);
            out[(size_t)t * rows + r] = sum;
        }
    }
}

static void rms_norm(const float* x, const float* w, int dim, int n, float eps, float* out) {
    for (int t = 0; t < n; t++) {
        const float* xr = x + (size_t)t * dim;
        float* o = out + (size_t)t * dim;
        float ms = -0.0f;
        for (int i = 0; i < dim; i++) ms += xr[i] * xr[i];
        ms /= (float)dim;
        float inv = 1.0f / sqrtf(ms + eps);
        for (int i = 0; i < dim; i++) o[i] = xr[i] * inv * w[i];
    }
}

static void rope(const omodel* m, float* x, int n_heads, uint32_t pos) {
    int hd = m->head_dim;
    for (int h = 0; h < n_heads; h++) {
        float* v = x + (size_t)h * hd;
        for (int i = 0; i < hd / 2; i++) {
            float a = (float)pos * m->inv_freq[i];
            float sn = sinf(a), cs = cosf(a);
            float x0 = v[2 * i], x1 = v[2 * i + 1];
            v[2 * i] = x0 * cs - x1 * sn;
            v[2 * i + 1] = x0 * sn + x1 * cs;
        }
    }
}

static void dequant_row(const qmat* m, int r, float* out) { /* quant.rs:464-490 */
    int nb = m->cols / QK;
    for (int b = 0; b < nb; b++) {
        float s = m->scales[(size_t)r * nb + b];
        const int8_t* q = m->qs + (size_t)r * m->cols + b * QK;
        for (int j = 0; j < QK; j++) out[b * QK + j] = s * (float)q[j];
    }
}

/* ---- op-level entry points (the per-op parity tests call these) ---- */

void om_quantize(const float* x, uint32_t n, uint32_t cols, int8_t* qs, float* scales) {
    for (size_t b = 0; b < (size_t)n * cols / QK; b++) scales[b] = quantize_block(x + b * QK, qs + b * QK);
}

void om_matmul_q8(const int8_t* wq, const float* ws, uint32_t rows, uint32_t cols, const int8_t* xq, const float* xs,
                  uint32_t n, float* out, int n_threads) {
    qmat w = {(int)rows, (int)cols, (float*)ws, (int8_t*)wq};
    qacts a = {(int)n, (int)cols, (int8_t*)xq, (float*)xs};
    matmul(&w, &a, out, n_threads > 0 ? n_threads : 1);
}

void om_rms_norm(const float* x, const float* w, uint32_t dim, uint32_t n, float eps, float* out) {
    rms_norm(x, w, (int)dim, (int)n, eps, out);
}

void om_rope(const omodel* m, float* x, uint32_t n_heads, uint32_t pos) { rope(m, x, (int)n_heads, pos); }

void om_silu_mul(float* g, const float* u, size_t n) {
    for (size_t e = 0; e < n; e++) g[e] = g[e] / (1.0f + expf(-g[e])) * u[e];
}

const float* om_inv_freq(const omodel* m) { return m->inv_freq; }

static const qmat* tensor_qmat(const omodel* m, int which, int layer) {
    if (which == OM_T_EMBED) return &m->embed;
    if (which == OM_T_OUTPUT) return &m->output;
    if (layer < 0 || layer >= m->n_layers) return NULL;
    const olayer* L = &m->layers[layer];
    switch (which) {
        case OM_T_Q: return &L->q;
        case OM_T_K: return &L->k;
        case OM_T_V: return &L->v;
        case OM_T_O: return &L->o;
        case OM_T_GATE: return &L->gate;
        case OM_T_UP: return &L->up;
        case OM_T_DOWN: return &L->down;
        default: return NULL;
    }
}

/* One tensor in its GGUF encoding: Q8_0 blocks {f16 d; i8 qs[32]} (34 bytes,
 * the layout quant.rs:265-273 repacks) for matrices, F32 for norm vectors.
 * Returns the byte count (0 for an unknown tensor); writes only if out. */
size_t om_export_tensor(const omodel* m, int which, int layer, void* out) {
    const float* vec = NULL;
    if (which == OM_T_OUTPUT_NORM) vec = m->output_norm;
    if (which == OM_T_ATTN_NORM && layer >= 0 && layer < m->n_layers) vec = m->layers[layer].attn_norm;
    if (which == OM_T_FFN_NORM && layer >= 0 && layer < m->n_layers) vec = m->layers[layer].ffn_norm;
    if (vec) {
        if (out) memcpy(out, vec, sizeof(float) * m->dim);
        return sizeof(float) * m->dim;
    }
    const qmat* q = tensor_qmat(m, which, layer);
    if (!q) return 0;
    size_t nb = (size_t)q->rows * q->cols / QK;
    if (out) {
        uint8_t* o = (uint8_t*)out;
        for (size_t b = 0; b < nb; b++) {
            uint16_t d = okv_f32_to_f16(q->scales[b]);
            memcpy(o + 34 * b, &d, 2);
            memcpy(o + 34 * b + 2, q->qs + b * QK, QK);
        }
    }
    return 34 * nb;
}

/* Model::forward (model.rs:366-518).  Returns 0, or the KV append error. */
int om_forward(const omodel* m, const om_kv* kv, const int32_t* tokens, const uint32_t* seqs, const uint32_t* pos,
               uint32_t n, const uint32_t* want, uint32_t n_want, float* logits, int n_threads) {
    int dim = m->dim, hd = m->head_dim;
    int qd = m->n_heads * hd, kvd = m->n_kv_heads * hd, ffn = m->ffn_dim;
    int32_t* blocks = (int32_t*)malloc(sizeof(int32_t) * (n ? n : 1));
    int32_t* slots = (int32_t*)malloc(sizeof(int32_t) * (n ? n : 1));
    int rc = kv->append(kv->ctx, seqs, pos, n, blocks, slots); /* claim first, model.rs:380-383 */
    if (rc) {
        free(blocks);
        free(slots);
        return rc;
    }
    float* x = (float*)malloc(sizeof(float) * (size_t)n * dim);
    float* h = (float*)malloc(sizeof(float) * (size_t)n * dim);
    float* q = (float*)malloc(sizeof(float) * (size_t)n * qd);
    float* k = (float*)malloc(sizeof(float) * (size_t)n * kvd);
    float* v = (float*)malloc(sizeof(float) * (size_t)n * kvd);
    float* att = (float*)malloc(sizeof(float) * (size_t)n * qd);
    float* o = (float*)malloc(sizeof(float) * (size_t)n * dim);
    float* gate = (float*)malloc(sizeof(float) * (size_t)n * ffn);
    float* up = (float*)malloc(sizeof(float) * (size_t)n * ffn);
    qacts xq = {0, 0, NULL, NULL};
    for (uint32_t i = 0; i < n; i++) dequant_row(&m->embed, tokens[i], x + (size_t)i * dim);
    for (int li = 0; li < m->n_layers; li++) {
        const olayer* L = &m->layers[li];
        rms_norm(x, L->attn_norm, dim, n, m->eps, h);
        qacts_quantize(&xq, h, n, dim);
        matmul(&L->q, &xq, q, n_threads);
        matmul(&L->k, &xq, k, n_threads);
        matmul(&L->v, &xq, v, n_threads);
        for (uint32_t i = 0; i < n; i++) {
            rope(m, q + (size_t)i * qd, m->n_heads, pos[i]);
            rope(m, k + (size_t)i * kvd, m->n_kv_heads, pos[i]);
        }
        kv->write(kv->ctx, li, blocks, slots, n, k, v);
        kv->attend(kv->ctx, li, q, seqs, pos, n, att);
        qacts_quantize(&xq, att, n, qd);
        matmul(&L->o, &xq, o, n_threads);
        for (size_t e = 0; e < (size_t)n * dim; e++) x[e] += o[e];
        rms_norm(x, L->ffn_norm, dim, n, m->eps, h);
        qacts_quantize(&xq, h, n, dim);
        matmul(&L->gate, &xq, gate, n_threads);
        matmul(&L->up, &xq, up, n_threads);
        for (size_t e = 0; e < (size_t)n * ffn; e++) gate[e] = gate[e] / (1.0f + expf(-gate[e])) * up[e];
        qacts_quantize(&xq, gate, n, ffn);
        matmul(&L->down, &xq, o, n_threads);
        for (size_t e = 0; e < (size_t)n * dim; e++) x[e] += o[e];
    }
    if (n_want) { /* model.rs:502-517 */
        float* sel = (float*)malloc(sizeof(float) * (size_t)n_want * dim);
        float* normed = (float*)malloc(sizeof(float) * (size_t)n_want * dim);
        for (uint32_t j = 0; j < n_want; j++) memcpy(sel + (size_t)j * dim, x + (size_t)want[j] * dim, sizeof(float) * dim);
        rms_norm(sel, m->output_norm, dim, n_want, m->eps, normed);
        qacts_quantize(&xq, normed, n_want, dim);
        matmul(&m->output, &xq, logits, n_threads);
        free(sel);
        free(normed);
    }
    free(xq.qs);
    free(xq.scales);
    free(x);
    free(h);
    free(q);
    free(k);
    free(v);
    free(att);
    free(o);
    free(gate);
    free(up);
    free(blocks);
    free(slots);
    return 0;
}

/* Greedy token: argmax with f32::total_cmp, the last index among equal
 * maxima (engine/crates/engine/src/sampling.rs:161-163). */
int32_t om_argmax(const float* logits, int n) {
    int32_t best = 0;
    int64_t bk = INT64_MIN;
    for (int i = 0; i < n; i++) {
        int32_t b;
        memcpy(&b, &logits[i], 4);
        int64_t key = b < 0 ? (int64_t)(b ^ 0x7FFFFFFF) : (int64_t)b; /* total order on f32 bits */
        if (key >= bk) {
            bk = key;
            best = i;
        }
    }
    return best;
}

/* ---- the oracle KvCache as an om_kv ---- */

typedef struct {
    okv* kv;
    int n_heads, n_kv_heads, head_dim, n_threads;
} okv_adapter;

static int oa_append(void* c, const uint32_t* seq, const uint32_t* pos, uint32_t n, int32_t* block, int32_t* slot) {
    uint32_t done;
    return okv_append_batch(((okv_adapter*)c)->kv, seq, pos, n, block, slot, &done);
}
static void oa_write(void* c, uint32_t layer, const int32_t* block, const int32_t* slot, uint32_t n, const float* k,
                     const float* v) {
    okv_write_batch(((okv_adapter*)c)->kv, layer, block, slot, n, k, v);
}
static void oa_attend(void* c, uint32_t layer, const float* q, const uint32_t* seq, const uint32_t* pos, uint32_t n,
                      float* out) {
    okv_adapter* a = (okv_adapter*)c;
    float scale = 1.0f / sqrtf((float)a->head_dim); /* model.rs:402 */
    okv_attend(a->kv, layer, q, seq, pos, n, a->n_heads, a->n_kv_heads, a->head_dim, scale, out, a->n_threads);
}

om_kv* om_kv_oracle(okv* kv, int n_heads, int n_kv_heads, int head_dim, int n_threads) {
    om_kv* w = (om_kv*)calloc(1, sizeof(om_kv));
    okv_adapter* a = (okv_adapter*)calloc(1, sizeof(okv_adapter));
    a->kv = kv;
    a->n_heads = n_heads;
    a->n_kv_heads = n_kv_heads;
    a->head_dim = head_dim;
    a->n_threads = n_threads;
    w->ctx = a;
    w->append = oa_append;
    w->write = oa_write;
    w->attend = oa_attend;
    return w;
}

void om_kv_free(om_kv* w) {
    if (!w) return;
    free(w->ctx);
    free(w);
}
