// Native continuous-batching driver over the KV-cache C ABI: the reference
// scheduler's KV policy (scheduler.rs:252-473, prefix.rs:58-125) in blocks.
// See include/lt_sched.h for the policy.
//
// Data structures keep every per-step decision O(log n) or O(changed):
//   - idle slots ordered by (last use, slot) -- admission takes the least
//     recently used, lowest slot on ties, as an argmin over slot order does;
//   - idle slots still holding KV ordered the same way -- LRU eviction;
//   - running sequences in admission order (a vector; removals are rare
//     relative to the step) -- batch order, youngest-first preemption.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <deque>
#include <set>
#include <string>
#include <utility>
#include <vector>

#include "lt_kv.h"
#include "lt_kv_internal.h"
#include "lt_prefix.h"
#include "lt_sched.h"

namespace {
constexpr uint32_t kBlock = LT_KV_BLOCK;

uint32_t blocks_for(uint32_t tokens) { return (tokens + kBlock - 1) / kBlock; }
}  // namespace

// Token requests (lt_sched_submit_tokens).
struct TokReq {
    std::vector<int32_t> toks;
    uint32_t out;
    int32_t adapter;
};
struct TokSeq {  // scheduler.rs Seq, the KV side
    uint32_t slot;
    std::vector<int32_t> tokens;  // prompt, then sampled tokens
    uint32_t n_prompt, n_past, max_total;
    uint64_t admit;  // admission order (youngest = largest)
    bool finished;
};

struct lt_sched {
    lt_kv* kv = nullptr;
    int mode = 0;  // 0: no request yet, 1: length-only requests, 2: token requests
    lt_slot_cache* sc = nullptr;
    std::deque<TokReq> tqueue;
    std::vector<TokSeq> tactive;  // the reference's active list (swap_remove on retire)
    uint64_t admit_seq = 0;
    int32_t gen_id = -2;          // next sampled token id (prompt ids are >= 0)
    lt_sched_config cfg{};
    std::string err;
    std::vector<uint8_t> busy;
    std::vector<uint32_t> held;       // tokens an idle slot keeps (prefix cache)
    std::vector<uint64_t> last_used;  // LRU clock of the slot
    uint64_t clock = 0, step_no = 0;
    std::set<std::pair<uint64_t, uint32_t>> idle;       // not busy
    std::set<std::pair<uint64_t, uint32_t>> evictable;  // not busy and held > 0
    std::deque<std::pair<uint32_t, uint32_t>> queue;    // (prompt, out)
    std::vector<uint32_t> order;                        // running slots, admission order
    std::vector<uint32_t> n_past, prompt, total;
    std::vector<uint64_t> admit_step;
    lt_sched_stats st{};
    // scratch
    std::vector<uint32_t> seqs, pos;
    std::vector<int32_t> blocks, slots;
    std::vector<uint32_t> dec, pre;  // running slots of the step, in admission order
};

namespace {

lt_status fail(lt_sched* s, lt_status rc, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    s->err = buf;
    return rc;
}

void set_idle(lt_sched* s, uint32_t slot) {
    s->idle.insert({s->last_used[slot], slot});
    if (s->held[slot] > 0) s->evictable.insert({s->last_used[slot], slot});
}

void clear_idle(lt_sched* s, uint32_t slot) {
    s->idle.erase({s->last_used[slot], slot});
    s->evictable.erase({s->last_used[slot], slot});
}

// Evict the least recently used idle slot's KV (prefix.rs:115-125 + kv_remove(slot, 0)).
bool evict_lru_idle(lt_sched* s) {
    if (s->evictable.empty()) return false;
    const uint32_t slot = s->evictable.begin()->second;
    s->evictable.erase(s->evictable.begin());
    lt_kv_truncate(s->kv, slot, 0);
    s->held[slot] = 0;
    s->st.evicted++;
    return true;
}

void retire(lt_sched* s, uint32_t slot) {  // a finished sequence keeps its KV, idle
    s->busy[slot] = 0;
    s->held[slot] = s->n_past[slot];
    s->last_used[slot] = ++s->clock;
    set_idle(s, slot);
}

void erase_running(lt_sched* s, uint32_t slot) {
    for (size_t i = 0; i < s->order.size(); ++i)
        if (s->order[i] == slot) {
            s->order.erase(s->order.begin() + (std::ptrdiff_t)i);
            return;
        }
}

// admit (scheduler.rs:252-275): FIFO, into the LRU idle slot, while it fits.
void admit(lt_sched* s) {
    while (!s->queue.empty() && !s->idle.empty()) {
        const auto [p, o] = s->queue.front();
        const uint32_t need = blocks_for(p + std::min(o, s->cfg.decode_headroom));
        while (lt_kv_free_blocks(s->kv) < need && evict_lru_idle(s)) {
        }
        if (lt_kv_free_blocks(s->kv) < need && !s->order.empty()) break;
        s->queue.pop_front();
        const uint32_t slot = s->idle.begin()->second;
        clear_idle(s, slot);
        lt_kv_truncate(s->kv, slot, 0);  // kv_remove(slot, reuse = 0): random prompts share nothing
        s->held[slot] = 0;
        s->busy[slot] = 1;
        s->last_used[slot] = ++s->clock;
        s->order.push_back(slot);
        s->n_past[slot] = 0;
        s->prompt[slot] = p;
        s->total[slot] = p + o;
        s->admit_step[slot] = s->step_no;
        s->st.admitted++;
    }
}

// New blocks the slot's work item of this step takes.
uint32_t item_blocks(const lt_sched* s, uint32_t slot) {
    const uint32_t p0 = s->n_past[slot];
    const uint32_t cnt = p0 >= s->prompt[slot] ? 1 : std::min(s->cfg.prefill_chunk, s->prompt[slot] - p0);
    return blocks_for(p0 + cnt) - blocks_for(p0);
}

// ensure_kv_room (scheduler.rs:321-334): evict LRU idle, then preempt the youngest.
void ensure_room(lt_sched* s) {
    uint64_t need = 0;
    for (uint32_t slot : s->order) need += item_blocks(s, slot);
    while (lt_kv_free_blocks(s->kv) < need) {
        if (evict_lru_idle(s)) continue;
        if (s->order.empty()) break;
        size_t yi = 0;
        for (size_t i = 1; i < s->order.size(); ++i)
            if (s->admit_step[s->order[i]] > s->admit_step[s->order[yi]]) yi = i;
        const uint32_t slot = s->order[yi];
        need -= item_blocks(s, slot);
        s->order.erase(s->order.begin() + (std::ptrdiff_t)yi);
        lt_kv_truncate(s->kv, slot, 0);  // preempted: finishes with Length, nothing kept
        s->busy[slot] = 0;
        s->held[slot] = 0;
        set_idle(s, slot);
        s->st.preempted++;
    }
}

// ---- token requests: the reference's admission with prefix reuse ----

bool tok_evict(lt_sched* s) {  // prefix.rs:115-125 + Backend::kv_remove(i, 0)
    const int32_t i = lt_slot_cache_evict_lru(s->sc);
    if (i < 0) return false;
    lt_kv_truncate(s->kv, (uint32_t)i, 0);
    s->st.evicted++;
    return true;
}

// scheduler.rs:252-317, KV room in blocks.
void tok_admit(lt_sched* s) {
    while (!s->tqueue.empty()) {
        const TokReq& r = s->tqueue.front();
        const uint32_t n = (uint32_t)r.toks.size();
        lt_placement pl{};
        if (lt_slot_cache_place(s->sc, r.toks.data(), n, r.adapter, &pl) != LT_OK) break;  // every slot busy
        const int64_t need = (int64_t)blocks_for(n + std::min(r.out, s->cfg.decode_headroom)) - pl.reuse / kBlock;
        while ((int64_t)lt_kv_free_blocks(s->kv) < need && tok_evict(s)) {
        }
        if ((int64_t)lt_kv_free_blocks(s->kv) < need && !s->tactive.empty()) break;
        TokReq req = std::move(s->tqueue.front());
        s->tqueue.pop_front();
        lt_slot_cache_place(s->sc, req.toks.data(), n, req.adapter, &pl);  // eviction may have cleared the prefix
        if (pl.copy_src >= 0) {
            lt_kv_truncate(s->kv, pl.slot, 0);
            lt_kv_share(s->kv, (uint32_t)pl.copy_src, pl.slot, pl.copy_len);  // Backend::kv_copy
            s->st.copies++;
        } else {
            lt_kv_truncate(s->kv, pl.slot, pl.reuse);
        }
        lt_slot_cache_acquire(s->sc, &pl, req.toks.data(), n, req.adapter);
        TokSeq q;
        q.slot = pl.slot;
        q.n_prompt = n;
        q.n_past = pl.reuse;
        q.max_total = n + req.out;
        q.admit = ++s->admit_seq;
        q.finished = false;
        q.tokens = std::move(req.toks);
        s->tactive.push_back(std::move(q));
        s->st.admitted++;
        s->st.prompt_tokens += n;
        s->st.cached_tokens += pl.reuse;
    }
}

// Blocks a work item (p0, cnt) of the slot takes: the blocks its tokens open,
// plus a copy-on-write block when it first writes into a shared partial
// block (kv.rs:99-110).
uint32_t tok_item_blocks(const lt_sched* s, uint32_t slot, uint32_t p0, uint32_t cnt) {
    uint32_t b = blocks_for(p0 + cnt) - blocks_for(p0);
    if (p0 % kBlock && ltkv::block_refs(s->kv, ltkv::seq_block_at(s->kv, slot, p0 / kBlock)) > 1) b += 1;
    return b;
}

// scheduler.rs:321-334: evict idle prefixes; else the youngest live sequence
// finishes (Length) and the step is skipped.
bool tok_ensure_room(lt_sched* s, uint64_t need) {
    while (lt_kv_free_blocks(s->kv) < need) {
        if (tok_evict(s)) continue;
        TokSeq* y = nullptr;
        for (TokSeq& q : s->tactive)
            if (!q.finished && (!y || q.admit > y->admit)) y = &q;
        if (y) {
            y->finished = true;
            s->st.preempted++;
        }
        return false;
    }
    return true;
}

// scheduler.rs:452-473: the slot keeps exactly the tokens in KV.
void tok_retire(lt_sched* s) {
    for (size_t i = 0; i < s->tactive.size();) {
        if (!s->tactive[i].finished) {
            ++i;
            continue;
        }
        TokSeq q = std::move(s->tactive[i]);
        if (i + 1 != s->tactive.size()) s->tactive[i] = std::move(s->tactive.back());  // Vec::swap_remove
        s->tactive.pop_back();
        lt_slot_cache_release(s->sc, q.slot, q.tokens.data(), q.n_past);
        if (q.n_past < q.tokens.size()) lt_kv_truncate(s->kv, q.slot, q.n_past);
        s->st.finished++;
    }
}

lt_status tok_step(lt_sched* s, const void* kv_src, uint32_t src_rows, const void* q_src, void* out,
                   uint32_t* n_decode, void* stream);

}  // namespace

extern "C" {

lt_status lt_sched_create(lt_kv* kv, const lt_sched_config* cfg, lt_sched** out) {
    if (!kv || !cfg || !out || cfg->n_slots == 0 || cfg->prefill_chunk == 0) return LT_E_ARG;
    if (cfg->n_slots > ltkv::handle_config(kv)->max_seqs) return LT_E_ARG;
    auto* s = new lt_sched();
    s->kv = kv;
    s->cfg = *cfg;
    const uint32_t n = cfg->n_slots;
    s->busy.assign(n, 0);
    s->held.assign(n, 0);
    s->last_used.assign(n, 0);
    s->n_past.assign(n, 0);
    s->prompt.assign(n, 0);
    s->total.assign(n, 0);
    s->admit_step.assign(n, 0);
    for (uint32_t i = 0; i < n; ++i) s->idle.insert({0, i});
    *out = s;
    return LT_OK;
}

void lt_sched_destroy(lt_sched* s) {
    if (s) lt_slot_cache_destroy(s->sc);
    delete s;
}

const char* lt_sched_last_error(const lt_sched* s) { return s ? s->err.c_str() : "null handle"; }

lt_status lt_sched_submit(lt_sched* s, uint32_t prompt_len, uint32_t out_len) {
    if (!s || prompt_len == 0) return LT_E_ARG;
    if (s->mode == 2) return fail(s, LT_E_ARG, "this driver takes token requests (lt_sched_submit_tokens)");
    s->mode = 1;
    s->queue.emplace_back(prompt_len, out_len);
    return LT_OK;
}

lt_status lt_sched_submit_tokens(lt_sched* s, const int32_t* tokens, uint32_t n, uint32_t out_len, int32_t adapter) {
    if (!s || !tokens || n == 0) return LT_E_ARG;
    if (s->mode == 1) return fail(s, LT_E_ARG, "this driver takes length-only requests (lt_sched_submit)");
    for (uint32_t i = 0; i < n; ++i)
        if (tokens[i] < 0) return fail(s, LT_E_ARG, "prompt token ids must be >= 0");
    // scheduler.rs:234-237 (enqueue): the prompt and one generated token must fit
    const lt_kv_config* kc = ltkv::handle_config(s->kv);
    const uint64_t n_ctx = std::min<uint64_t>(lt_kv_capacity(s->kv),
                                              (uint64_t)(kc->max_blocks_per_seq ? std::min(kc->max_blocks_per_seq,
                                                                                           lt_kv_n_blocks(s->kv))
                                                                                : lt_kv_n_blocks(s->kv)) *
                                                  kBlock);
    if ((uint64_t)n + 1 > n_ctx)
        return fail(s, LT_E_ARG, "prompt has %u tokens; context window is %llu", n, (unsigned long long)n_ctx);
    if (!s->sc) {
        lt_status rc = lt_slot_cache_create(s->cfg.n_slots, &s->sc);
        if (rc != LT_OK) return fail(s, rc, "slot cache");
    }
    s->mode = 2;
    s->tqueue.push_back(TokReq{std::vector<int32_t>(tokens, tokens + n), out_len, adapter});
    return LT_OK;
}

lt_status lt_sched_get_stats(const lt_sched* s, lt_sched_stats* out) {
    if (!s || !out) return LT_E_ARG;
    *out = s->st;
    out->running = (uint32_t)(s->mode == 2 ? s->tactive.size() : s->order.size());
    out->queued = (uint32_t)(s->mode == 2 ? s->tqueue.size() : s->queue.size());
    return LT_OK;
}

lt_status lt_sched_step(lt_sched* s, const void* kv_src, uint32_t src_rows, const void* q_src, void* out,
                        uint32_t* n_decode, void* stream) {
    ltkv::NvtxRange nv("lt_sched_step");
    if (!s) return LT_E_ARG;
    if (s->cfg.data && (!kv_src || !q_src || !out || src_rows == 0))
        return fail(s, LT_E_ARG, "data mode needs kv_src, q_src and out");
    if (s->mode == 2) return tok_step(s, kv_src, src_rows, q_src, out, n_decode, stream);
    s->step_no++;
    s->st.steps++;
    admit(s);
    ensure_room(s);
    s->dec.clear();
    s->pre.clear();
    for (uint32_t slot : s->order) (s->n_past[slot] >= s->prompt[slot] ? s->dec : s->pre).push_back(slot);
    const lt_kv_config* kc = ltkv::handle_config(s->kv);
    const size_t kv_row = (size_t)kc->n_kv_heads * kc->head_dim * 2;  // f16 bytes
    const size_t q_row = (size_t)kc->n_heads * kc->head_dim * 2;
    auto src_off = [&](uint32_t n) -> uint64_t {  // a window of n rows of kv_src, moving each step
        return src_rows > n ? (s->step_no * 2654435761ull) % (src_rows - n + 1) : 0;
    };
    // prompt chunks: claim, write
    if (!s->pre.empty()) {
        s->seqs.clear();
        s->pos.clear();
        for (uint32_t slot : s->pre) {
            const uint32_t p0 = s->n_past[slot], cnt = std::min(s->cfg.prefill_chunk, s->prompt[slot] - p0);
            for (uint32_t i = 0; i < cnt; ++i) {
                s->seqs.push_back(slot);
                s->pos.push_back(p0 + i);
            }
        }
        const uint32_t n = (uint32_t)s->seqs.size();
        s->blocks.resize(n);
        s->slots.resize(n);
        uint32_t done = 0;
        lt_status rc = lt_kv_append(s->kv, s->seqs.data(), s->pos.data(), n, s->blocks.data(), s->slots.data(), &done,
                                    stream);
        if (rc != LT_OK) return fail(s, rc, "prefill claim: %s", lt_kv_last_error(s->kv));
        if (s->cfg.data) {
            if (n > src_rows) return fail(s, LT_E_ARG, "kv_src holds %u rows, the step writes %u", src_rows, n);
            const char* k = static_cast<const char*>(kv_src) + src_off(n) * kv_row;
            rc = lt_kv_write(s->kv, 0, s->blocks.data(), s->slots.data(), n, k, k, LT_F16, stream);
            if (rc != LT_OK) return fail(s, rc, "prefill write: %s", lt_kv_last_error(s->kv));
        }
        s->st.prefill_tokens += n;
    }
    // decode tokens: claim, fused write + attention
    const uint32_t nd = (uint32_t)s->dec.size();
    if (nd) {
        s->seqs.assign(s->dec.begin(), s->dec.end());
        s->pos.resize(nd);
        for (uint32_t i = 0; i < nd; ++i) s->pos[i] = s->n_past[s->dec[i]];
        s->blocks.resize(nd);
        s->slots.resize(nd);
        uint32_t done = 0;
        lt_status rc = lt_kv_append(s->kv, s->seqs.data(), s->pos.data(), nd, s->blocks.data(), s->slots.data(),
                                    &done, stream);
        if (rc != LT_OK) return fail(s, rc, "decode claim: %s", lt_kv_last_error(s->kv));
        if (s->cfg.data) {
            if (nd > src_rows || nd > s->cfg.n_slots) return fail(s, LT_E_ARG, "source arrays too small");
            const char* k = static_cast<const char*>(kv_src) + src_off(nd) * kv_row;
            (void)q_row;
            const float scale = 1.0f / std::sqrt((float)kc->head_dim);
            rc = lt_kv_write_attend(s->kv, 0, s->blocks.data(), s->slots.data(), k, k, LT_F16, q_src, LT_F16,
                                    s->seqs.data(), s->pos.data(), nd, out, LT_F16, scale, stream);
            if (rc != LT_OK) return fail(s, rc, "decode attention: %s", lt_kv_last_error(s->kv));
        }
        s->st.decode_tokens += nd;
        for (uint32_t i = 0; i < nd; ++i) s->st.attended_positions += (uint64_t)s->pos[i] + 1;
    }
    if (n_decode) *n_decode = nd;
    // advance, retire (scheduler.rs:452-473)
    auto advance = [&](uint32_t slot, uint32_t cnt) {
        s->n_past[slot] += cnt;
        if (s->n_past[slot] >= s->total[slot]) {
            erase_running(s, slot);
            retire(s, slot);
            s->st.finished++;
        }
    };
    for (uint32_t slot : s->dec) advance(slot, 1);
    for (uint32_t slot : s->pre) advance(slot, std::min(s->cfg.prefill_chunk, s->prompt[slot] - s->n_past[slot]));
    if (s->cfg.compact) {
        uint32_t moved = 0;
        lt_status rc = lt_kv_compact(s->kv, &moved, stream);
        if (rc != LT_OK) return fail(s, rc, "compaction: %s", lt_kv_last_error(s->kv));
        s->st.moved_blocks += moved;
    }
    return LT_OK;
}

}  // extern "C"

namespace {

// One engine iteration for token requests: admit, one batch (decode tokens,
// then prompt chunks, in active order), sampling's bookkeeping, retire.
lt_status tok_step(lt_sched* s, const void* kv_src, uint32_t src_rows, const void* q_src, void* out,
                   uint32_t* n_decode, void* stream) {
    s->step_no++;
    s->st.steps++;
    tok_admit(s);
    uint32_t nd = 0;
    if (!s->tactive.empty()) {
        std::vector<uint32_t>& dec = s->dec;  // indices into tactive
        std::vector<uint32_t>& pre = s->pre;
        dec.clear();
        pre.clear();
        uint64_t need = 0;
        for (uint32_t i = 0; i < s->tactive.size(); ++i) {
            const TokSeq& q = s->tactive[i];
            if (q.finished) continue;
            if (q.n_past >= q.n_prompt) {
                dec.push_back(i);
                need += tok_item_blocks(s, q.slot, q.n_past, 1);
            }
        }
        for (uint32_t i = 0; i < s->tactive.size(); ++i) {
            const TokSeq& q = s->tactive[i];
            if (q.finished || q.n_past >= q.n_prompt) continue;
            pre.push_back(i);
            need += tok_item_blocks(s, q.slot, q.n_past, std::min(q.n_prompt - q.n_past, s->cfg.prefill_chunk));
        }
        if ((!dec.empty() || !pre.empty()) && tok_ensure_room(s, need)) {
            s->seqs.clear();
            s->pos.clear();
            for (uint32_t i : dec) {
                s->seqs.push_back(s->tactive[i].slot);
                s->pos.push_back(s->tactive[i].n_past);
            }
            nd = (uint32_t)dec.size();
            for (uint32_t i : pre) {
                const TokSeq& q = s->tactive[i];
                const uint32_t cnt = std::min(q.n_prompt - q.n_past, s->cfg.prefill_chunk);
                for (uint32_t k = 0; k < cnt; ++k) {
                    s->seqs.push_back(q.slot);
                    s->pos.push_back(q.n_past + k);
                }
            }
            const uint32_t n = (uint32_t)s->seqs.size();
            s->blocks.resize(n);
            s->slots.resize(n);
            uint32_t done = 0;
            lt_status rc = lt_kv_append(s->kv, s->seqs.data(), s->pos.data(), n, s->blocks.data(), s->slots.data(),
                                        &done, stream);
            if (rc != LT_OK) return fail(s, rc, "batch claim: %s", lt_kv_last_error(s->kv));
            if (s->cfg.data) {
                const lt_kv_config* kc = ltkv::handle_config(s->kv);
                const size_t kv_row = (size_t)kc->n_kv_heads * kc->head_dim * 2;  // f16 bytes
                if (n > src_rows || nd > s->cfg.n_slots) return fail(s, LT_E_ARG, "source arrays too small");
                const char* k = static_cast<const char*>(kv_src) +
                                (src_rows > n ? (s->step_no * 2654435761ull) % (src_rows - n + 1) : 0) * kv_row;
                if (n > nd) {
                    rc = lt_kv_write(s->kv, 0, s->blocks.data() + nd, s->slots.data() + nd, n - nd, k + nd * kv_row,
                                     k + nd * kv_row, LT_F16, stream);
                    if (rc != LT_OK) return fail(s, rc, "prefill write: %s", lt_kv_last_error(s->kv));
                }
                if (nd) {
                    const float scale = 1.0f / std::sqrt((float)kc->head_dim);
                    rc = lt_kv_write_attend(s->kv, 0, s->blocks.data(), s->slots.data(), k, k, LT_F16, q_src, LT_F16,
                                            s->seqs.data(), s->pos.data(), nd, out, LT_F16, scale, stream);
                    if (rc != LT_OK) return fail(s, rc, "decode attention: %s", lt_kv_last_error(s->kv));
                }
            }
            s->st.decode_tokens += nd;
            s->st.prefill_tokens += n - nd;
            for (uint32_t j = 0; j < nd; ++j) s->st.attended_positions += (uint64_t)s->pos[j] + 1;
            for (uint32_t i : pre) {
                TokSeq& q = s->tactive[i];
                q.n_past += std::min(q.n_prompt - q.n_past, s->cfg.prefill_chunk);
            }
            // sample_at order: the decode tokens, then the prompts whose last chunk ran
            auto sample = [&](TokSeq& q) {
                if (q.n_past >= q.n_prompt && q.n_past < q.tokens.size()) q.n_past += 1;  // pending token now in KV
                q.tokens.push_back(s->gen_id--);
                if (q.tokens.size() >= q.max_total) q.finished = true;
            };
            for (uint32_t i : dec) sample(s->tactive[i]);
            for (uint32_t i : pre)
                if (s->tactive[i].n_past == s->tactive[i].n_prompt) sample(s->tactive[i]);
        }
    }
    if (n_decode) *n_decode = nd;
    tok_retire(s);
    if (s->cfg.compact) {
        uint32_t moved = 0;
        lt_status rc = lt_kv_compact(s->kv, &moved, stream);
        if (rc != LT_OK) return fail(s, rc, "compaction: %s", lt_kv_last_error(s->kv));
        s->st.moved_blocks += moved;
    }
    return LT_OK;
}

}  // namespace
