/*
 * lt_sched.h -- the KV-cache side of the reference's continuous-batching
 * scheduler as a native driver over lt_kv.h.
 *
 * Restates the slot / prefix policy of engine/crates/engine/src/scheduler.rs
 * (admit :252-275, ensure_kv_room :321-334, the step :356-451, retire :452-473) and
 * engine/crates/engine/src/prefix.rs (LRU slot cache :58-125) in blocks:
 *   - a request waits in a FIFO queue; it is admitted into the least
 *     recently used idle slot once its prompt plus min(output,
 *     decode_headroom) tokens fit, evicting idle slots' cached KV least
 *     recently used first (kv_remove(slot, 0) = lt_kv_truncate(slot, 0));
 *   - each step: one decode token for every sequence past its prompt, a
 *     prompt chunk of at most prefill_chunk tokens for the others;
 *   - before the step, enough blocks are freed for it: evict LRU idle slots,
 *     then preempt the youngest running sequence (it ends with Length);
 *   - a finished sequence keeps its KV in its now idle slot for prefix reuse;
 *   - optionally lt_kv_compact after every step (no reference counterpart).
 * Length-only requests (lt_sched_submit) stand for random prompts: no prefix
 * is ever reused and the driver never calls kv_copy.
 *
 * Requests that carry token ids (lt_sched_submit_tokens) go through the
 * reference's token-level admission instead (a driver takes one kind or the
 * other):
 *   - placement by the slot-level prefix cache (lt_prefix.h, prefix.rs:58-92):
 *     the free slot with the longest common prefix keeps it
 *     (kv_remove(slot, reuse)); when another slot matches at least 16 tokens
 *     more, its KV is copied (kv_remove(slot, 0) + kv_copy = lt_kv_share);
 *   - admission while the prompt suffix plus min(output, decode_headroom)
 *     fits, evicting idle prefixes LRU, re-planning after eviction
 *     (scheduler.rs:252-317);
 *   - one batch per step: decode tokens, then prompt chunks, in the order of
 *     the active list (scheduler.rs:356-407); its blocks include one
 *     copy-on-write block per first write into a shared partial block;
 *   - a step that does not fit evicts idle prefixes, else marks the
 *     youngest sequence finished and skips the step (scheduler.rs:321-334,
 *     409-411);
 *   - retire keeps exactly the tokens in KV in the idle slot for reuse
 *     (prefix.rs:105-112, scheduler.rs:452-473; Vec::swap_remove order).
 * Generated tokens get negative ids, which no prompt uses.  Adapter ids only
 * separate prefixes; adapter-group scheduling is not restated.
 *
 * The step's K/V rows and q rows are cut from caller-provided device arrays
 * (synthetic inputs of the benchmark): prompt tokens are appended and their
 * rows written (lt_kv_write), decode tokens run the fused append + attention
 * (lt_kv_write_attend).  With cfg.data == 0 only the bookkeeping runs, on a
 * host-only handle too.
 *
 * Threading: a driver and its cache belong to one thread.
 */
#ifndef LT_SCHED_H
#define LT_SCHED_H

#include <stdint.h>

#include "lt_kv.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct lt_sched lt_sched;

typedef struct lt_sched_config {
    uint32_t n_slots;         /* parallel slots: sequence ids [0, n_slots) (Backend::n_seq_max) */
    uint32_t decode_headroom; /* scheduler.rs DECODE_HEADROOM (256) */
    uint32_t prefill_chunk;   /* EngineConfig::prefill_chunk (256) */
    int32_t compact;          /* 1: lt_kv_compact after every step */
    int32_t data;             /* 1: write K/V rows and attend; 0: bookkeeping only */
} lt_sched_config;

typedef struct lt_sched_stats {
    uint64_t steps, admitted, finished, evicted, preempted;
    uint64_t decode_tokens, prefill_tokens, moved_blocks;
    uint32_t running, queued;
    uint64_t attended_positions;  /* sum over decode tokens of pos + 1: cached rows the attention reads */
    /* token requests: prefix copies (kv_copy), prompt tokens admitted, and
     * those already in KV at admission (the reference's cached_tokens) */
    uint64_t copies, prompt_tokens, cached_tokens;
} lt_sched_stats;

lt_status lt_sched_create(lt_kv* kv, const lt_sched_config* cfg, lt_sched** out);
void lt_sched_destroy(lt_sched* s);
const char* lt_sched_last_error(const lt_sched* s);

/* Queue a request of prompt_len prompt tokens and out_len output tokens. */
lt_status lt_sched_submit(lt_sched* s, uint32_t prompt_len, uint32_t out_len);
/* Queue a request with its prompt token ids (ids >= 0), out_len output
 * tokens and an adapter id (LT_NO_ADAPTER for none); see the header
 * comment.  LT_E_ARG when the driver already took length-only requests, or
 * when the prompt plus one token exceeds the context window (the pool, or
 * max_blocks_per_seq blocks; scheduler.rs:234-237). */
lt_status lt_sched_submit_tokens(lt_sched* s, const int32_t* tokens, uint32_t n, uint32_t out_len, int32_t adapter);

/* One scheduler step (see the header comment).  kv_src: device f16
 * [src_rows][n_kv_heads*head_dim] rows for the appended tokens (a contiguous
 * window of them per call); q_src: device f16 [n_slots][n_heads*head_dim],
 * row i is the i-th decode token's q; out: device f16 [n_slots][n_heads*
 * head_dim].  Unused (may be NULL) with cfg.data == 0.  *n_decode receives
 * the step's decode tokens (may be NULL). */
lt_status lt_sched_step(lt_sched* s, const void* kv_src, uint32_t src_rows, const void* q_src, void* out,
                        uint32_t* n_decode, void* stream);

lt_status lt_sched_get_stats(const lt_sched* s, lt_sched_stats* out);

#ifdef __cplusplus
}
#endif
#endif
