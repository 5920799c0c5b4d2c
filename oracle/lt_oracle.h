/*
 * lt_oracle.h -- TEST INFRASTRUCTURE ONLY.
 *
 * CPU restatement of the reference engine's paged KV cache
 * (engine/crates/native/src/kv.rs) and of its decode/prefill attention
 * closure (engine/crates/native/src/model.rs:431-476, dot at :159-172).
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may
 * load this code, and only as the checker or the timed CPU baseline.  The
 * product path (include/lt_kv.h, langtrain_studio_b200/) never calls it.
 *
 * Parity pins: the bookkeeping is checked against the reference's own
 * known-answer tests (kv.rs:202-229, ported verbatim in tests/); the
 * f32->f16 conversion against numpy's IEEE round-to-nearest-even.  The
 * attention arithmetic has no golden vector in the reference (none exists),
 * so its parity is pinned only by this restatement.
 */
#ifndef LT_ORACLE_H
#define LT_ORACLE_H
#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#define OKV_BLOCK 16

typedef struct okv okv;

enum { OKV_OK = 0, OKV_FULL = 1, OKV_NONCONTIG = 2, OKV_ARG = 3 };

/* KvCache::new (kv.rs:35-48).  Sequence ids must be < max_seqs. */
okv* okv_new(uint32_t n_layers, uint32_t kv_dim, uint32_t n_tokens, uint32_t max_seqs);
/* The same cache with Q8_0 rows (lt_kv.h, LT_KV_Q8_0): every kv_dim row is
 * kept as kv_dim/32 groups of int8 values + one f16 scale each; kv_dim must
 * be a multiple of 32.  Bookkeeping is unchanged; writes quantise, reads
 * (rows, attention) use q * d. */
okv* okv_new_q8(uint32_t n_layers, uint32_t kv_dim, uint32_t n_tokens, uint32_t max_seqs);

/* One 32-value group as the engine's int8 quantiser does it
 * (quant.rs:785-795): amax folded from 0 with f32::max (NaN ignored),
 * d = amax / 127, id = d > 0 ? 1 / d : 0, q = round(x * id) half away from
 * zero, cast to int8 saturating (NaN -> 0).  Returns d (f32); the cache
 * keeps okv_f32_to_f16(d). */
float okv_q8_group(const float* x, int8_t* q);
void okv_delete(okv* kv);

uint32_t okv_capacity(const okv* kv);            /* kv.rs:50 */
uint64_t okv_bytes(const okv* kv);               /* kv.rs:54 */
uint32_t okv_len(const okv* kv, uint32_t seq);   /* kv.rs:58 */
uint32_t okv_free_blocks(const okv* kv);         /* kv.rs:185 */
uint32_t okv_n_blocks(const okv* kv);

/* KvCache::append (kv.rs:85-121): 0, OKV_FULL or OKV_NONCONTIG. */
int okv_append(okv* kv, uint32_t seq, uint32_t pos, int32_t* block, int32_t* slot);
/* The claim loop of Model::forward (model.rs:380-383): stops at the first
 * error; *n_done tokens were claimed. */
int okv_append_batch(okv* kv, const uint32_t* seq, const uint32_t* pos, uint32_t n,
                     int32_t* block, int32_t* slot, uint32_t* n_done);

/* KvCache::write (kv.rs:123-131), f32 -> f16 round-to-nearest-even. */
void okv_write(okv* kv, uint32_t layer, int32_t block, int32_t slot, const float* k, const float* v);
void okv_write_batch(okv* kv, uint32_t layer, const int32_t* block, const int32_t* slot, uint32_t n,
                     const float* k, const float* v);
/* Same, for inputs that are already f16 bit patterns (stored unchanged). */
void okv_write_batch_f16(okv* kv, uint32_t layer, const int32_t* block, const int32_t* slot,
                         uint32_t n, const uint16_t* k, const uint16_t* v);

void okv_truncate(okv* kv, uint32_t seq, uint32_t from);            /* kv.rs:153-169 */
void okv_share(okv* kv, uint32_t src, uint32_t dst, uint32_t len);  /* kv.rs:172-183 */

/* Compaction (no counterpart in the reference): pair free ids ascending with
 * live ids descending while free < live, move each such live block onto the
 * free id (all layers, K and V; the source keeps its bytes), move its
 * refcount, rewrite every table entry, then rebuild the free list as all
 * free ids in descending order so the next alloc returns the lowest.
 * Returns the number of blocks moved; (src, dst) pairs go to moves[] if
 * non-NULL (capacity n_blocks pairs). */
uint32_t okv_compact(okv* kv, int32_t* moves);

/* Introspection for parity checks. */
uint32_t okv_seq_blocks(const okv* kv, uint32_t seq, int32_t* out, uint32_t cap);
void okv_refs(const okv* kv, uint32_t* out);
uint32_t okv_free_list(const okv* kv, int32_t* out, uint32_t cap);
/* Pool in reference layout [layer][block][slot][kv_dim] (f16 bits). */
const uint16_t* okv_pool_k(const okv* kv);
const uint16_t* okv_pool_v(const okv* kv);
/* Q8_0 pool: int8 [layer][block][slot][kv_dim] and f16 scales
 * [layer][block][slot][kv_dim/32]; NULL for an f16 cache. */
const int8_t* okv_pool_kq(const okv* kv);
const int8_t* okv_pool_vq(const okv* kv);
const uint16_t* okv_pool_kd(const okv* kv);
const uint16_t* okv_pool_vd(const okv* kv);

/* Rows 0..n of seq (KvCache::rows, kv.rs:135-150) copied out as f16 bits
 * (Q8_0: q * d rounded to f16). */
void okv_rows(const okv* kv, uint32_t layer, uint32_t seq, uint32_t n, uint16_t* k_out, uint16_t* v_out);

/* Attention closure of Model::forward (model.rs:431-476) for n tokens:
 * q [n][n_heads*head_dim] f32, out [n][n_heads*head_dim] f32, len = pos+1.
 * One task per (token, kv head) as pool::for_chunks splits it
 * (model.rs:435), spread over n_threads threads (<=0: all cores). */
void okv_attend(const okv* kv, uint32_t layer, const float* q, const uint32_t* seq,
                const uint32_t* pos, uint32_t n, uint32_t n_heads, uint32_t n_kv_heads,
                uint32_t head_dim, float scale, float* out, int n_threads);

/* half 2.7.1 f16::from_f32 / to_f32 semantics (IEEE binary16, RNE). */
uint16_t okv_f32_to_f16(float x);
float okv_f16_to_f32(uint16_t h);
void okv_f32_to_f16_array(const float* x, uint16_t* out, size_t n);

#ifdef __cplusplus
}
#endif
#endif
