/*
 * A plain C client of the library, linked the way the engine's Rust FFI would
 * link it (no Python, no CUDA headers).  On a bookkeeping-only handle
 * (device = -1) it runs the reference's own KvCache known-answer tests,
 * engine/crates/native/src/kv.rs:202-217 and :219-229 (bookkeeping half),
 * the SlotCache placement test prefix.rs:136-144, and the reference
 * scheduler's tests of KV behaviour (scheduler.rs:584-592, 615-621, 623-636,
 * 675-682) through the native driver (lt_sched.h) with token requests on
 * byte-level tokens, as the reference's MockBackend tests use.  Exit status 0
 * on success.
 */
#include <stdio.h>
#include <string.h>

#include "lt_kv.h"
#include "lt_prefix.h"
#include "lt_sched.h"

#define CHECK(cond)                                                          \
    do {                                                                     \
        if (!(cond)) {                                                       \
            fprintf(stderr, "%s:%d: check failed: %s\n", __FILE__, __LINE__, #cond); \
            return 1;                                                        \
        }                                                                    \
    } while (0)

static lt_kv* make(uint32_t n_tokens) {
    lt_kv_config c;
    memset(&c, 0, sizeof c);
    c.n_layers = 1;
    c.n_kv_heads = 1;
    c.head_dim = 64;
    c.n_heads = 1;
    c.n_tokens = n_tokens;
    c.max_seqs = 8;
    c.max_batch = 1024;
    c.device = -1;
    lt_kv* kv = NULL;
    return lt_kv_create(&c, &kv) == LT_OK ? kv : NULL;
}

static lt_status append(lt_kv* kv, uint32_t seq, uint32_t pos, int32_t* block, int32_t* slot) {
    uint32_t done = 0;
    return lt_kv_append(kv, &seq, &pos, 1, block, slot, &done, NULL);
}

static int share_then_diverge(void) { /* kv.rs:202-217 */
    lt_kv* kv = make(256);
    CHECK(kv);
    int32_t b, s;
    for (uint32_t p = 0; p < 20; ++p) CHECK(append(kv, 0, p, &b, &s) == LT_OK);
    lt_kv_share(kv, 0, 1, 20);
    const uint32_t free_before = lt_kv_free_blocks(kv);
    CHECK(append(kv, 1, 20, &b, &s) == LT_OK); /* copy-on-write of the shared partial block */
    CHECK(lt_kv_free_blocks(kv) == free_before - 1);
    CHECK(s == 4);
    int32_t b0[4], b1[4];
    CHECK(lt_kv_seq_blocks(kv, 0, b0, 4) == 2 && lt_kv_seq_blocks(kv, 1, b1, 4) == 2);
    CHECK(b1[0] == b0[0] && b1[1] != b0[1] && b1[1] == b);
    CHECK(lt_kv_len(kv, 0) == 20 && lt_kv_len(kv, 1) == 21);
    lt_kv_destroy(kv);
    return 0;
}

static int truncate_frees_blocks(void) { /* kv.rs:219-229 */
    lt_kv* kv = make(64);
    CHECK(kv);
    int32_t b, s;
    for (uint32_t p = 0; p < 40; ++p) CHECK(append(kv, 3, p, &b, &s) == LT_OK);
    CHECK(lt_kv_free_blocks(kv) == 1);
    lt_kv_truncate(kv, 3, 10);
    CHECK(lt_kv_free_blocks(kv) == 3);
    lt_kv_truncate(kv, 3, 0);
    CHECK(lt_kv_free_blocks(kv) == 4);
    CHECK(append(kv, 3, 5, &b, &s) == LT_E_NONCONTIG);
    CHECK(strstr(lt_kv_last_error(kv), "not contiguous") != NULL);
    lt_kv_destroy(kv);
    return 0;
}

static int prefers_slot_with_longest_prefix(void) { /* prefix.rs:136-144 */
    lt_slot_cache* c = NULL;
    CHECK(lt_slot_cache_create(3, &c) == LT_OK);
    int32_t toks[52];
    for (int i = 0; i < 50; ++i) toks[i] = i;
    CHECK(lt_slot_cache_release(c, 1, toks, 50) == LT_OK);
    toks[50] = 999;
    toks[51] = 998;
    lt_placement p;
    CHECK(lt_slot_cache_place(c, toks, 52, LT_NO_ADAPTER, &p) == LT_OK);
    CHECK(p.slot == 1 && p.reuse == 50 && p.copy_src == -1);
    lt_slot_cache_destroy(c);
    return 0;
}

/* ---- scheduler.rs tests of KV behaviour, through lt_sched ---- */

static lt_kv* make_engine_kv(uint32_t n_ctx, uint32_t n_seq) {
    lt_kv_config c;
    memset(&c, 0, sizeof c);
    c.n_layers = 1;
    c.n_kv_heads = 2;
    c.head_dim = 64;
    c.n_heads = 4;
    c.n_tokens = n_ctx;
    c.max_seqs = n_seq;
    c.max_batch = 1u << 14;
    c.device = -1;
    lt_kv* kv = NULL;
    return lt_kv_create(&c, &kv) == LT_OK ? kv : NULL;
}

static lt_sched* make_sched(lt_kv* kv, uint32_t n_seq, uint32_t chunk) {
    lt_sched_config c;
    memset(&c, 0, sizeof c);
    c.n_slots = n_seq;
    c.decode_headroom = 256;
    c.prefill_chunk = chunk;
    c.compact = 1;
    c.data = 0; /* bookkeeping only */
    lt_sched* s = NULL;
    return lt_sched_create(kv, &c, &s) == LT_OK ? s : NULL;
}

/* A chat prompt as byte-level token ids: a shared system prompt, the
 * question, role tags. */
static uint32_t chat(const char* question, int32_t* out, uint32_t cap) {
    char text[512];
    strcpy(text, "<|system|>");
    for (int i = 0; i < 8; ++i) strcat(text, "You are helpful. ");
    strcat(text, "<|user|>");
    strcat(text, question);
    strcat(text, "<|assistant|>");
    uint32_t n = (uint32_t)strlen(text);
    if (n > cap) n = cap;
    for (uint32_t i = 0; i < n; ++i) out[i] = (int32_t)(unsigned char)text[i];
    return n;
}

/* Step until n_requests have finished (bounded). */
static int drive(lt_sched* s, uint64_t n_requests, lt_sched_stats* st) {
    for (int i = 0; i < 10000; ++i) {
        if (lt_sched_step(s, NULL, 0, NULL, NULL, NULL, NULL) != LT_OK) return 1;
        if (lt_sched_get_stats(s, st) != LT_OK) return 1;
        if (st->finished >= n_requests) return 0;
    }
    return 1;
}

static int second_request_reuses_prefix(void) { /* scheduler.rs:584-592 */
    lt_kv* kv = make_engine_kv(4096, 2);
    CHECK(kv);
    lt_sched* s = make_sched(kv, 2, 32);
    CHECK(s);
    int32_t t[256];
    lt_sched_stats st;
    uint32_t n = chat("first question", t, 256);
    CHECK(lt_sched_submit_tokens(s, t, n, 20, LT_NO_ADAPTER) == LT_OK);
    CHECK(drive(s, 1, &st) == 0);
    CHECK(st.cached_tokens == 0);
    n = chat("second question", t, 256);
    CHECK(lt_sched_submit_tokens(s, t, n, 20, LT_NO_ADAPTER) == LT_OK);
    CHECK(drive(s, 2, &st) == 0);
    CHECK(st.cached_tokens > 100); /* the system prompt and role tags come from the cache */
    lt_sched_destroy(s);
    lt_kv_destroy(kv);
    return 0;
}

static int long_prompt_is_chunked(void) { /* scheduler.rs:615-621 */
    lt_kv* kv = make_engine_kv(4096, 2);
    CHECK(kv);
    lt_sched* s = make_sched(kv, 2, 32);
    CHECK(s);
    int32_t t[1000];
    for (int i = 0; i < 1000; ++i) t[i] = 'x';
    lt_sched_stats st;
    CHECK(lt_sched_submit_tokens(s, t, 1000, 20, LT_NO_ADAPTER) == LT_OK);
    CHECK(lt_sched_step(s, NULL, 0, NULL, NULL, NULL, NULL) == LT_OK);
    CHECK(lt_sched_get_stats(s, &st) == LT_OK);
    CHECK(st.prefill_tokens == 32); /* one chunk per step */
    CHECK(drive(s, 1, &st) == 0);
    CHECK(st.prompt_tokens == 1000 && st.prefill_tokens == 1000 && st.finished == 1);
    lt_sched_destroy(s);
    lt_kv_destroy(kv);
    return 0;
}

static int context_pressure_ends_youngest_gracefully(void) { /* scheduler.rs:623-636 */
    lt_kv* kv = make_engine_kv(600, 3); /* three prompts fit, not their replies too */
    CHECK(kv);
    lt_sched* s = make_sched(kv, 3, 32);
    CHECK(s);
    int32_t t[256];
    char q[8];
    for (int i = 0; i < 3; ++i) {
        snprintf(q, sizeof q, "q%d", i);
        const uint32_t n = chat(q, t, 256);
        CHECK(lt_sched_submit_tokens(s, t, n, 200, LT_NO_ADAPTER) == LT_OK);
    }
    lt_sched_stats st;
    CHECK(drive(s, 3, &st) == 0); /* every request ends (Stop or Length), no error */
    CHECK(st.finished == 3 && st.admitted == 3);
    lt_sched_destroy(s);
    lt_kv_destroy(kv);
    return 0;
}

static int rejects_prompt_larger_than_context(void) { /* scheduler.rs:675-682 */
    lt_kv* kv = make_engine_kv(64, 1);
    CHECK(kv);
    lt_sched* s = make_sched(kv, 1, 32);
    CHECK(s);
    int32_t t[100];
    for (int i = 0; i < 100; ++i) t[i] = 'y';
    CHECK(lt_sched_submit_tokens(s, t, 100, 10, LT_NO_ADAPTER) == LT_E_ARG);
    CHECK(strstr(lt_sched_last_error(s), "context window") != NULL);
    lt_sched_destroy(s);
    lt_kv_destroy(kv);
    return 0;
}

int main(void) {
    if (share_then_diverge() || truncate_frees_blocks() || prefers_slot_with_longest_prefix()) return 1;
    if (second_request_reuses_prefix() || long_prompt_is_chunked() || context_pressure_ends_youngest_gracefully() ||
        rejects_prompt_larger_than_context())
        return 1;
    printf("C client: kv.rs, prefix.rs and scheduler.rs known-answer tests passed\n");
    return 0;
}
