/*
 * A plain C client of the library, linked the way the engine's Rust FFI would
 * link it (no Python, no CUDA headers).  On a bookkeeping-only handle
 * (device = -1) it runs the reference's own KvCache known-answer tests,
 * engine/crates/native/src/kv.rs:202-217 and :219-229 (bookkeeping half), and
 * the SlotCache placement test prefix.rs:136-144.  Exit status 0 on success.
 */
#include <stdio.h>
#include <string.h>

#include "lt_kv.h"
#include "lt_prefix.h"

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

int main(void) {
    if (share_then_diverge() || truncate_frees_blocks() || prefers_slot_with_longest_prefix()) return 1;
    printf("C client: kv.rs and prefix.rs known-answer tests passed\n");
    return 0;
}
