/*
 * lt_prefix.h -- the reference engine's slot-level prefix cache
 * (engine/crates/engine/src/prefix.rs), native, over token ids.
 *
 * Every KV slot remembers the tokens its cache holds after its request
 * finishes.  A new prompt is placed on the free slot sharing the longest
 * prefix with it, so only the suffix is prefilled; when another slot (busy or
 * not) holds at least LT_MIN_COPY_GAIN more matching tokens, its KV is copied
 * (Backend::kv_copy = lt_kv_share).  KV computed under one adapter is never
 * reused for another.  The decisions, tie-breaks included, are the
 * reference's:
 *   place    prefix.rs:58-92   free slot with the longest match, the least
 *                              recently used among equal matches (the last
 *                              slot on a full tie); match capped at len - 1
 *                              so one prompt token is evaluated; copy from the
 *                              other slot with the longest match (the last on
 *                              ties) when it gains >= LT_MIN_COPY_GAIN
 *   acquire  prefix.rs:94-102  tick the clock, mark busy, keep prompt[..reuse]
 *   release  prefix.rs:105-112 tick the clock, mark idle, keep the KV tokens
 *   evict    prefix.rs:115-125 least recently used idle slot holding tokens
 *                              (the first on ties); its tokens are dropped
 * Adapters are ids (LT_NO_ADAPTER for none) compared for equality, as the
 * reference compares Option<String>.
 *
 * Host-only bookkeeping: no device memory, no CUDA calls.  A cache belongs to
 * one thread.  place() scans every slot and compares prompts token by token,
 * O(slots x prompt), as the reference does: sized for the engine's parallel
 * slots (hardware.rs picks 2-16), not for thousands of slots.
 */
#ifndef LT_PREFIX_H
#define LT_PREFIX_H

#include <stdint.h>

#include "lt_kv.h"

#ifdef __cplusplus
extern "C" {
#endif

#define LT_MIN_COPY_GAIN 16 /* prefix.rs:13 */
#define LT_NO_ADAPTER (-1)

typedef struct lt_slot_cache lt_slot_cache;

/* prefix.rs:25-31 Placement: copy_src < 0 means no copy. */
typedef struct lt_placement {
    uint32_t slot;
    uint32_t reuse;    /* prompt tokens already in KV after any copy */
    int32_t copy_src;  /* slot whose first copy_len tokens are copied into `slot`, or -1 */
    uint32_t copy_len;
} lt_placement;

/* SlotCache::new (prefix.rs:44-46). */
lt_status lt_slot_cache_create(uint32_t n_slots, lt_slot_cache** out);
void lt_slot_cache_destroy(lt_slot_cache* c);

/* SlotCache::place (prefix.rs:58-92): LT_OK with *out, or LT_E_FULL when
 * every slot is busy (the reference's None). */
lt_status lt_slot_cache_place(const lt_slot_cache* c, const int32_t* prompt, uint32_t n, int32_t adapter,
                              lt_placement* out);
/* SlotCache::acquire (prefix.rs:94-102); p->reuse <= n. */
lt_status lt_slot_cache_acquire(lt_slot_cache* c, const lt_placement* p, const int32_t* prompt, uint32_t n,
                                int32_t adapter);
/* SlotCache::release (prefix.rs:105-112): the slot's KV now holds tokens[0, n). */
lt_status lt_slot_cache_release(lt_slot_cache* c, uint32_t slot, const int32_t* tokens, uint32_t n);
/* SlotCache::evict_lru (prefix.rs:115-125): the evicted slot, or -1. */
int32_t lt_slot_cache_evict_lru(lt_slot_cache* c);
/* SlotCache::idle_cells (prefix.rs:53-55): tokens held by idle slots. */
uint64_t lt_slot_cache_idle_cells(const lt_slot_cache* c);
/* SlotCache::has_free (prefix.rs:48-50). */
int lt_slot_cache_has_free(const lt_slot_cache* c);

/* Introspection for parity checks: the slot's tokens (count returned, at
 * most cap copied), busy flag, adapter and last-used clock. */
uint32_t lt_slot_cache_tokens(const lt_slot_cache* c, uint32_t slot, int32_t* out, uint32_t cap);
lt_status lt_slot_cache_slot_state(const lt_slot_cache* c, uint32_t slot, int32_t* busy, int32_t* adapter,
                                   uint64_t* last_used);
/* Test hook: overwrite a slot's tokens and adapter without ticking the clock
 * (the reference's own tests assign slot fields directly, prefix.rs:159, 169). */
lt_status lt_slot_cache_set_slot(lt_slot_cache* c, uint32_t slot, const int32_t* tokens, uint32_t n,
                                 int32_t adapter);

#ifdef __cplusplus
}
#endif
#endif /* LT_PREFIX_H */
