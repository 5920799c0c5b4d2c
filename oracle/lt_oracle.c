/*
 * lt_oracle.c -- TEST INFRASTRUCTURE ONLY (the checker and the timed CPU
 * baseline; never part of the product path).
 *
 * A plain-C restatement of the reference engine's paged KV cache
 * (engine/crates/native/src/kv.rs) and attention closure
 * (engine/crates/native/src/model.rs:431-476).  The reference is Rust and
 * cannot be compiled in this environment (no cargo/rustc, crates not
 * vendored), so this file follows its algorithm step by step, keeping the
 * same operation order wherever it affects results:
 *   - free list is a stack initialised to (0..n_blocks).rev()   kv.rs:45
 *   - append/CoW/truncate/share exactly as kv.rs:85-183
 *   - f32 -> f16 round-to-nearest-even (half 2.7.1)             kv.rs:126,129
 *   - dot with 8 partial sums + tail                            model.rs:159-172
 *   - scores * scale, max fold, expf, sequential sum, 1/sum     model.rs:447-463
 *   - V accumulation  o += w * v  (no contraction)              model.rs:464-473
 * A Q8_0 cache (okv_new_q8) keeps each row as 32-value groups of int8 + an
 * f16 scale: the Q8_0 block of the reference's GGUF reader (quant.rs:254-275)
 * filled by the engine's own int8 quantiser (quant.rs:785-795); reads widen
 * q * d, which is exact in f32 (8-bit q times an 11-bit scale).
 * Build with -ffp-contract=off and without fast-math (Rust does not fuse).
 */
#define _GNU_SOURCE
#include "lt_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdatomic.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>
#if defined(__F16C__)
#include <immintrin.h>
#endif

typedef struct {
    int32_t* blocks;
    uint32_t n, cap;
    uint32_t len;
} oseq;

struct okv {
    uint32_t n_layers, kv_dim, n_blocks, max_seqs;
    uint16_t* k;
    uint16_t* v;
    int q8;           /* Q8_0 rows: kq/vq values, kd/vd f16 scales (k, v unused) */
    int8_t* kq;
    int8_t* vq;
    uint16_t* kd;
    uint16_t* vd;
    uint32_t* refs;
    int32_t* free_list;
    uint32_t n_free;
    oseq* seqs;
};

/* ---------------------------------------------------------------- f16 ---- */

/* IEEE binary16 round-to-nearest-even, the semantics of half 2.7.1's
 * f16::from_f32 (hardware F16C or its software path give the same bits):
 * overflow -> inf, f32 subnormals -> signed zero, NaN -> quiet NaN keeping
 * the top 10 payload bits. */
uint16_t okv_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    uint32_t e = (x >> 23) & 0xFFu;
    uint32_t man = x & 0x007FFFFFu;
    if (e == 0xFFu) {
        uint16_t nan_bit = man ? 0x0200u : 0u;
        return (uint16_t)(sign | 0x7C00u | nan_bit | (man >> 13));
    }
    if (e == 0) return sign; /* zero or f32 subnormal: far below half range */
    int32_t unb = (int32_t)e - 127;
    if (unb > 15) return (uint16_t)(sign | 0x7C00u);
    if (unb >= -14) {
        uint32_t hm = man >> 13, rem = man & 0x1FFFu;
        uint32_t h = ((uint32_t)(unb + 15) << 10) + hm;
        if (rem > 0x1000u || (rem == 0x1000u && (hm & 1u))) h += 1; /* carry may reach inf */
        return (uint16_t)(sign | h);
    }
    /* half subnormal: value = full * 2^(unb-23), result m * 2^-24 */
    uint32_t full = man | 0x00800000u;
    int32_t shift = -unb - 1; /* >= 14 */
    if (shift > 24) return sign;
    uint32_t m = full >> shift;
    uint32_t rem = full & ((1u << shift) - 1u), half = 1u << (shift - 1);
    if (rem > half || (rem == half && (m & 1u))) m += 1;
    return (uint16_t)(sign | m);
}

float okv_f16_to_f32(uint16_t h) {
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1Fu, m = h & 0x3FFu, x;
    if (e == 0) {
        if (m == 0) {
            x = sign;
        } else { /* subnormal: normalise */
            int32_t ee = -1;
            do { m <<= 1; ee++; } while (!(m & 0x400u));
            x = sign | ((uint32_t)(127 - 15 - ee) << 23) | ((m & 0x3FFu) << 13);
        }
    } else if (e == 0x1Fu) {
        x = sign | 0x7F800000u | (m << 13);
    } else {
        x = sign | ((e + 127 - 15) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &x, 4);
    return f;
}

void okv_f32_to_f16_array(const float* x, uint16_t* out, size_t n) {
    for (size_t i = 0; i < n; i++) out[i] = okv_f32_to_f16(x[i]);
}

/* convert_to_f32_slice (model.rs:448,466): exact widening. */
static void widen(const uint16_t* src, float* dst, uint32_t n) {
    uint32_t i = 0;
#if defined(__F16C__)
    for (; i + 8 <= n; i += 8)
        _mm256_storeu_ps(dst + i, _mm256_cvtph_ps(_mm_loadu_si128((const __m128i*)(src + i))));
#endif
    for (; i < n; i++) dst[i] = okv_f16_to_f32(src[i]);
}

/* ------------------------------------------------------------ KvCache ---- */

static okv* okv_new_fmt(uint32_t n_layers, uint32_t kv_dim, uint32_t n_tokens, uint32_t max_seqs, int q8) {
    if (q8 && kv_dim % 32) return NULL;
    okv* kv = (okv*)calloc(1, sizeof(okv));
    if (!kv) return NULL;
    kv->n_layers = n_layers;
    kv->kv_dim = kv_dim;
    kv->n_blocks = (n_tokens + OKV_BLOCK - 1) / OKV_BLOCK; /* div_ceil, kv.rs:36 */
    kv->max_seqs = max_seqs;
    kv->q8 = q8;
    size_t size = (size_t)n_layers * kv->n_blocks * OKV_BLOCK * kv_dim; /* kv.rs:37 */
    size_t fsize = q8 ? 1 : (size ? size : 1);
    kv->k = (uint16_t*)calloc(fsize, 2);
    kv->v = (uint16_t*)calloc(fsize, 2);
    if (q8) {
        kv->kq = (int8_t*)calloc(size ? size : 1, 1);
        kv->vq = (int8_t*)calloc(size ? size : 1, 1);
        kv->kd = (uint16_t*)calloc(size / 32 ? size / 32 : 1, 2);
        kv->vd = (uint16_t*)calloc(size / 32 ? size / 32 : 1, 2);
    }
    kv->refs = (uint32_t*)calloc(kv->n_blocks ? kv->n_blocks : 1, 4);
    kv->free_list = (int32_t*)malloc((kv->n_blocks ? kv->n_blocks : 1) * 4);
    kv->seqs = (oseq*)calloc(max_seqs ? max_seqs : 1, sizeof(oseq));
    if (!kv->k || !kv->v || !kv->refs || !kv->free_list || !kv->seqs ||
        (q8 && (!kv->kq || !kv->vq || !kv->kd || !kv->vd))) {
        okv_delete(kv);
        return NULL;
    }
    for (uint32_t i = 0; i < kv->n_blocks; i++) kv->free_list[i] = (int32_t)(kv->n_blocks - 1 - i);
    kv->n_free = kv->n_blocks;
    return kv;
}

okv* okv_new(uint32_t n_layers, uint32_t kv_dim, uint32_t n_tokens, uint32_t max_seqs) {
    return okv_new_fmt(n_layers, kv_dim, n_tokens, max_seqs, 0);
}

okv* okv_new_q8(uint32_t n_layers, uint32_t kv_dim, uint32_t n_tokens, uint32_t max_seqs) {
    return okv_new_fmt(n_layers, kv_dim, n_tokens, max_seqs, 1);
}

void okv_delete(okv* kv) {
    if (!kv) return;
    if (kv->seqs)
        for (uint32_t s = 0; s < kv->max_seqs; s++) free(kv->seqs[s].blocks);
    free(kv->seqs);
    free(kv->k);
    free(kv->v);
    free(kv->kq);
    free(kv->vq);
    free(kv->kd);
    free(kv->vd);
    free(kv->refs);
    free(kv->free_list);
    free(kv);
}

uint32_t okv_capacity(const okv* kv) { return kv->n_blocks * OKV_BLOCK; }
uint64_t okv_bytes(const okv* kv) {
    const uint64_t rows = (uint64_t)kv->n_layers * kv->n_blocks * OKV_BLOCK;
    if (kv->q8) return rows * 2u * (kv->kv_dim + kv->kv_dim / 32 * 2u);
    return rows * kv->kv_dim * 2u * 2u;
}
uint32_t okv_len(const okv* kv, uint32_t seq) { return seq < kv->max_seqs ? kv->seqs[seq].len : 0; }
uint32_t okv_free_blocks(const okv* kv) { return kv->n_free; }
uint32_t okv_n_blocks(const okv* kv) { return kv->n_blocks; }

static size_t offset(const okv* kv, uint32_t layer, uint32_t block, uint32_t slot) { /* kv.rs:63-65 */
    return (((size_t)layer * kv->n_blocks + block) * OKV_BLOCK + slot) * kv->kv_dim;
}

/* All K and V bytes of block src onto block dst in every layer. */
static void copy_block(okv* kv, uint32_t src, uint32_t dst) {
    for (uint32_t l = 0; l < kv->n_layers; l++) {
        size_t so = offset(kv, l, src, 0), dof = offset(kv, l, dst, 0);
        size_t n = (size_t)OKV_BLOCK * kv->kv_dim;
        if (kv->q8) {
            memmove(kv->kq + dof, kv->kq + so, n);
            memmove(kv->vq + dof, kv->vq + so, n);
            memmove(kv->kd + dof / 32, kv->kd + so / 32, n / 32 * 2);
            memmove(kv->vd + dof / 32, kv->vd + so / 32, n / 32 * 2);
        } else {
            memmove(kv->k + dof, kv->k + so, n * 2);
            memmove(kv->v + dof, kv->v + so, n * 2);
        }
    }
}

static int alloc_block(okv* kv, int32_t* out) { /* kv.rs:67-74 */
    if (kv->n_free == 0) return OKV_FULL;
    int32_t b = kv->free_list[--kv->n_free];
    kv->refs[b] = 1;
    *out = b;
    return OKV_OK;
}

static void release_block(okv* kv, int32_t b) { /* kv.rs:76-82 */
    kv->refs[b] -= 1;
    if (kv->refs[b] == 0) kv->free_list[kv->n_free++] = b;
}

static void seq_push(oseq* s, int32_t b) {
    if (s->n == s->cap) {
        s->cap = s->cap ? s->cap * 2 : 8;
        s->blocks = (int32_t*)realloc(s->blocks, s->cap * 4);
    }
    s->blocks[s->n++] = b;
}

int okv_append(okv* kv, uint32_t seq, uint32_t pos, int32_t* block, int32_t* slot_out) {
    if (seq >= kv->max_seqs) return OKV_ARG;
    oseq* s = &kv->seqs[seq];
    if (pos != s->len) return OKV_NONCONTIG; /* kv.rs:87-92, state unchanged */
    uint32_t slot = pos % OKV_BLOCK;
    if (slot == 0) {
        int32_t b;
        if (alloc_block(kv, &b)) return OKV_FULL; /* kv.rs:96: state unchanged */
        seq_push(s, b);
    } else {
        int32_t last = s->blocks[s->n - 1];
        if (kv->refs[last] > 1) { /* copy-on-write, kv.rs:99-110 */
            int32_t nb;
            if (alloc_block(kv, &nb)) return OKV_FULL;
            copy_block(kv, (uint32_t)last, (uint32_t)nb);
            release_block(kv, last);
            s->blocks[s->n - 1] = nb;
        }
    }
    s->len = pos + 1;
    *block = s->blocks[s->n - 1];
    *slot_out = (int32_t)slot;
    return OKV_OK;
}

int okv_append_batch(okv* kv, const uint32_t* seq, const uint32_t* pos, uint32_t n, int32_t* block,
                     int32_t* slot, uint32_t* n_done) {
    uint32_t i = 0;
    int rc = OKV_OK;
    for (; i < n; i++) {
        rc = okv_append(kv, seq[i], pos[i], &block[i], &slot[i]);
        if (rc) break;
    }
    if (n_done) *n_done = i;
    return rc;
}

float okv_q8_group(const float* x, int8_t* q) { /* quant.rs:785-795 */
    float amax = 0.0f;
    for (int i = 0; i < 32; i++) {
        float a = fabsf(x[i]);
        if (a > amax) amax = a; /* f32::max: a NaN operand loses */
    }
    float d = amax / 127.0f;
    float id = d > 0.0f ? 1.0f / d : 0.0f;
    for (int i = 0; i < 32; i++) {
        float r = roundf(x[i] * id); /* f32::round: half away from zero */
        q[i] = r != r ? 0 : r >= 127.0f ? 127 : r <= -128.0f ? -128 : (int8_t)r; /* `as i8` saturates */
    }
    return d;
}

static void q8_row(const float* x, uint32_t n, int8_t* q, uint16_t* d) {
    for (uint32_t g = 0; g < n / 32; g++) d[g] = okv_f32_to_f16(okv_q8_group(x + 32 * g, q + 32 * g));
}

void okv_write(okv* kv, uint32_t layer, int32_t block, int32_t slot, const float* k, const float* v) {
    size_t o = offset(kv, layer, (uint32_t)block, (uint32_t)slot);
    if (kv->q8) {
        q8_row(k, kv->kv_dim, kv->kq + o, kv->kd + o / 32);
        q8_row(v, kv->kv_dim, kv->vq + o, kv->vd + o / 32);
        return;
    }
    for (uint32_t d = 0; d < kv->kv_dim; d++) kv->k[o + d] = okv_f32_to_f16(k[d]);
    for (uint32_t d = 0; d < kv->kv_dim; d++) kv->v[o + d] = okv_f32_to_f16(v[d]);
}

void okv_write_batch(okv* kv, uint32_t layer, const int32_t* block, const int32_t* slot, uint32_t n,
                     const float* k, const float* v) {
    for (uint32_t i = 0; i < n; i++)
        okv_write(kv, layer, block[i], slot[i], k + (size_t)i * kv->kv_dim, v + (size_t)i * kv->kv_dim);
}

void okv_write_batch_f16(okv* kv, uint32_t layer, const int32_t* block, const int32_t* slot,
                         uint32_t n, const uint16_t* k, const uint16_t* v) {
    if (kv->q8) {
        float* kf = (float*)malloc(kv->kv_dim * sizeof(float));
        float* vf = (float*)malloc(kv->kv_dim * sizeof(float));
        for (uint32_t i = 0; i < n; i++) {
            widen(k + (size_t)i * kv->kv_dim, kf, kv->kv_dim);
            widen(v + (size_t)i * kv->kv_dim, vf, kv->kv_dim);
            okv_write(kv, layer, block[i], slot[i], kf, vf);
        }
        free(kf);
        free(vf);
        return;
    }
    for (uint32_t i = 0; i < n; i++) {
        size_t o = offset(kv, layer, (uint32_t)block[i], (uint32_t)slot[i]);
        memcpy(kv->k + o, k + (size_t)i * kv->kv_dim, kv->kv_dim * 2);
        memcpy(kv->v + o, v + (size_t)i * kv->kv_dim, kv->kv_dim * 2);
    }
}

void okv_truncate(okv* kv, uint32_t seq, uint32_t from) {
    if (seq >= kv->max_seqs) return;
    oseq* s = &kv->seqs[seq];
    if (from >= s->len) return; /* also covers a missing seq (len 0) */
    uint32_t keep = (from + OKV_BLOCK - 1) / OKV_BLOCK;
    for (uint32_t i = keep; i < s->n; i++) release_block(kv, s->blocks[i]); /* ascending */
    s->n = keep;
    s->len = from;
}

void okv_share(okv* kv, uint32_t src, uint32_t dst, uint32_t len) {
    if (dst < kv->max_seqs) okv_truncate(kv, dst, 0);
    if (src >= kv->max_seqs || dst >= kv->max_seqs) return;
    oseq* s = &kv->seqs[src];
    if (s->len == 0) return; /* missing source (share(x, x, _) lands here too) */
    if (len > s->len) len = s->len;
    uint32_t nb = (len + OKV_BLOCK - 1) / OKV_BLOCK;
    for (uint32_t i = 0; i < nb; i++) kv->refs[s->blocks[i]] += 1;
    if (len > 0) {
        oseq* d = &kv->seqs[dst];
        d->n = 0;
        for (uint32_t i = 0; i < nb; i++) seq_push(d, s->blocks[i]);
        d->len = len;
    }
}

uint32_t okv_compact(okv* kv, int32_t* moves) {
    uint32_t nb = kv->n_blocks, nf = 0, nl = 0, moved = 0;
    int32_t* fr = (int32_t*)malloc((nb ? nb : 1) * 4);
    int32_t* lv = (int32_t*)malloc((nb ? nb : 1) * 4);
    int32_t* remap = (int32_t*)malloc((nb ? nb : 1) * 4);
    for (uint32_t b = 0; b < nb; b++) {
        remap[b] = (int32_t)b;
        if (kv->refs[b] == 0) fr[nf++] = (int32_t)b;
    }
    for (uint32_t b = nb; b-- > 0;)
        if (kv->refs[b] != 0) lv[nl++] = (int32_t)b;
    for (uint32_t j = 0; j < nf && j < nl && fr[j] < lv[j]; j++) {
        int32_t src = lv[j], dst = fr[j];
        copy_block(kv, (uint32_t)src, (uint32_t)dst);
        kv->refs[dst] = kv->refs[src];
        kv->refs[src] = 0;
        remap[src] = dst;
        if (moves) {
            moves[2 * moved] = src;
            moves[2 * moved + 1] = dst;
        }
        moved++;
    }
    for (uint32_t s = 0; s < kv->max_seqs; s++)
        for (uint32_t i = 0; i < kv->seqs[s].n; i++) kv->seqs[s].blocks[i] = remap[kv->seqs[s].blocks[i]];
    kv->n_free = 0;
    for (uint32_t b = nb; b-- > 0;)
        if (kv->refs[b] == 0) kv->free_list[kv->n_free++] = (int32_t)b;
    free(fr);
    free(lv);
    free(remap);
    return moved;
}

uint32_t okv_seq_blocks(const okv* kv, uint32_t seq, int32_t* out, uint32_t cap) {
    if (seq >= kv->max_seqs) return 0;
    const oseq* s = &kv->seqs[seq];
    for (uint32_t i = 0; i < s->n && i < cap; i++) out[i] = s->blocks[i];
    return s->n;
}

void okv_refs(const okv* kv, uint32_t* out) { memcpy(out, kv->refs, (size_t)kv->n_blocks * 4); }

uint32_t okv_free_list(const okv* kv, int32_t* out, uint32_t cap) {
    for (uint32_t i = 0; i < kv->n_free && i < cap; i++) out[i] = kv->free_list[i];
    return kv->n_free;
}

const uint16_t* okv_pool_k(const okv* kv) { return kv->k; }
const uint16_t* okv_pool_v(const okv* kv) { return kv->v; }
const int8_t* okv_pool_kq(const okv* kv) { return kv->kq; }
const int8_t* okv_pool_vq(const okv* kv) { return kv->vq; }
const uint16_t* okv_pool_kd(const okv* kv) { return kv->kd; }
const uint16_t* okv_pool_vd(const okv* kv) { return kv->vd; }

/* q * d of n values of a Q8_0 row (exact in f32). */
static void dequant(const int8_t* q, const uint16_t* d, float* out, uint32_t n) {
    for (uint32_t i = 0; i < n; i++) out[i] = (float)q[i] * okv_f16_to_f32(d[i / 32]);
}

/* Row o (element offset) of K or V, head `kvh`, widened to f32. */
static void read_row(const okv* kv, int is_v, size_t o, uint32_t kvh, uint32_t hd, float* row) {
    o += (size_t)kvh * hd;
    if (kv->q8)
        dequant((is_v ? kv->vq : kv->kq) + o, (is_v ? kv->vd : kv->kd) + o / 32, row, hd);
    else
        widen((is_v ? kv->v : kv->k) + o, row, hd);
}

void okv_rows(const okv* kv, uint32_t layer, uint32_t seq, uint32_t n, uint16_t* k_out, uint16_t* v_out) {
    const oseq* s = &kv->seqs[seq];
    float* row = kv->q8 ? (float*)malloc(kv->kv_dim * sizeof(float)) : NULL;
    for (uint32_t p = 0; p < n; p++) {
        size_t o = offset(kv, layer, (uint32_t)s->blocks[p / OKV_BLOCK], p % OKV_BLOCK);
        if (kv->q8) {
            read_row(kv, 0, o, 0, kv->kv_dim, row);
            okv_f32_to_f16_array(row, k_out + (size_t)p * kv->kv_dim, kv->kv_dim);
            read_row(kv, 1, o, 0, kv->kv_dim, row);
            okv_f32_to_f16_array(row, v_out + (size_t)p * kv->kv_dim, kv->kv_dim);
            continue;
        }
        memcpy(k_out + (size_t)p * kv->kv_dim, kv->k + o, kv->kv_dim * 2);
        memcpy(v_out + (size_t)p * kv->kv_dim, kv->v + o, kv->kv_dim * 2);
    }
    free(row);
}

/* ---------------------------------------------------------- attention ---- */

/* model.rs:159-172: 8 independent partial sums, then the tail, then
 * acc.iter().sum() + tail.  Float Sum folds from -0.0 in current Rust; the
 * start value cannot change a result that is later scaled and exp'd. */
static float dot(const float* a, const float* b, uint32_t n) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    uint32_t n8 = n / 8 * 8;
    for (uint32_t i = 0; i < n8; i += 8)
        for (int k = 0; k < 8; k++) acc[k] += a[i + k] * b[i + k];
    float tail = -0.0f;
    for (uint32_t i = n8; i < n; i++) tail += a[i] * b[i];
    float s = -0.0f;
    for (int k = 0; k < 8; k++) s += acc[k];
    return s + tail;
}

typedef struct {
    const okv* kv;
    uint32_t layer, n, n_heads, n_kv_heads, hd;
    const float* q;
    const uint32_t* seq;
    const uint32_t* pos;
    float scale;
    float* out;
    atomic_uint next;
} attn_job;

static void attend_task(const attn_job* j, uint32_t idx, float** scores, size_t* scores_cap, float* row) {
    const okv* kv = j->kv;
    uint32_t hd = j->hd, group = j->n_heads / j->n_kv_heads;
    uint32_t q_dim = j->n_heads * hd;
    uint32_t i = idx / j->n_kv_heads, kvh = idx % j->n_kv_heads; /* model.rs:436 */
    const float* qs = j->q + (size_t)i * q_dim + (size_t)kvh * group * hd;
    float* out = j->out + (size_t)i * q_dim + (size_t)kvh * group * hd;
    uint32_t len = j->pos[i] + 1;
    const oseq* s = &kv->seqs[j->seq[i]];
    size_t need = (size_t)group * len;
    if (need > *scores_cap) {
        *scores = (float*)realloc(*scores, need * sizeof(float));
        *scores_cap = need;
    }
    float* sc = *scores;
    for (uint32_t p = 0; p < len; p++) { /* K pass, model.rs:447-452 */
        size_t o = offset(kv, j->layer, (uint32_t)s->blocks[p / OKV_BLOCK], p % OKV_BLOCK);
        read_row(kv, 0, o, kvh, hd, row);
        for (uint32_t g = 0; g < group; g++) sc[(size_t)g * len + p] = dot(qs + (size_t)g * hd, row, hd) * j->scale;
    }
    for (uint32_t g = 0; g < group; g++) { /* softmax, model.rs:453-463 */
        float* sg = sc + (size_t)g * len;
        float mx = -INFINITY;
        for (uint32_t p = 0; p < len; p++) mx = fmaxf(mx, sg[p]);
        float sum = 0.0f;
        for (uint32_t p = 0; p < len; p++) {
            sg[p] = expf(sg[p] - mx);
            sum += sg[p];
        }
        float inv = 1.0f / sum;
        for (uint32_t p = 0; p < len; p++) sg[p] *= inv;
    }
    for (uint32_t e = 0; e < group * hd; e++) out[e] = 0.0f;
    for (uint32_t p = 0; p < len; p++) { /* V pass, model.rs:464-473 */
        size_t o = offset(kv, j->layer, (uint32_t)s->blocks[p / OKV_BLOCK], p % OKV_BLOCK);
        read_row(kv, 1, o, kvh, hd, row);
        for (uint32_t g = 0; g < group; g++) {
            float w = sc[(size_t)g * len + p];
            float* og = out + (size_t)g * hd;
            for (uint32_t d = 0; d < hd; d++) og[d] += w * row[d];
        }
    }
}

static void* attend_worker(void* arg) {
    attn_job* j = (attn_job*)arg;
    float* scores = NULL;
    size_t cap = 0;
    float* row = (float*)malloc(j->hd * sizeof(float));
    uint32_t total = j->n * j->n_kv_heads;
    for (;;) {
        uint32_t idx = atomic_fetch_add(&j->next, 1u);
        if (idx >= total) break;
        attend_task(j, idx, &scores, &cap, row);
    }
    free(scores);
    free(row);
    return NULL;
}

void okv_attend(const okv* kv, uint32_t layer, const float* q, const uint32_t* seq, const uint32_t* pos,
                uint32_t n, uint32_t n_heads, uint32_t n_kv_heads, uint32_t head_dim, float scale, float* out,
                int n_threads) {
    attn_job j;
    j.kv = kv;
    j.layer = layer;
    j.n = n;
    j.n_heads = n_heads;
    j.n_kv_heads = n_kv_heads;
    j.hd = head_dim;
    j.q = q;
    j.seq = seq;
    j.pos = pos;
    j.scale = scale;
    j.out = out;
    atomic_init(&j.next, 0u);
    if (n_threads <= 0) n_threads = (int)sysconf(_SC_NPROCESSORS_ONLN);
    if (n_threads < 1) n_threads = 1;
    if (n_threads == 1) {
        attend_worker(&j);
        return;
    }
    pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)n_threads);
    int started = 0;
    for (int t = 1; t < n_threads; t++)
        if (pthread_create(&th[started], NULL, attend_worker, &j) == 0) started++;
    attend_worker(&j);
    for (int t = 0; t < started; t++) pthread_join(th[t], NULL);
    free(th);
}
