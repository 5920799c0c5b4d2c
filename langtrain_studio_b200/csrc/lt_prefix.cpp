// The reference engine's slot-level prefix cache (engine/crates/engine/src/
// prefix.rs) over token ids; see include/lt_prefix.h.  Host-only.
//
// Tie-breaks follow the Rust iterator adaptors the reference uses:
// Iterator::max_by / max_by_key keep the LAST of equal maxima, min_by_key
// keeps the FIRST of equal minima.
#include <algorithm>
#include <cstdint>
#include <cstring>
#include <new>
#include <vector>

#include "lt_prefix.h"

namespace {

struct Slot {  // prefix.rs:15-22
    std::vector<int32_t> tokens;
    int32_t adapter = LT_NO_ADAPTER;
    bool busy = false;
    uint64_t last_used = 0;
};

uint32_t common_prefix(const std::vector<int32_t>& a, const int32_t* b, uint32_t nb) {  // prefix.rs:39-41
    const uint32_t n = std::min<uint32_t>((uint32_t)a.size(), nb);
    uint32_t i = 0;
    while (i < n && a[i] == b[i]) ++i;
    return i;
}

}  // namespace

struct lt_slot_cache {
    std::vector<Slot> slots;
    uint64_t clock = 0;
};

extern "C" {

lt_status lt_slot_cache_create(uint32_t n_slots, lt_slot_cache** out) {
    if (!out || n_slots == 0) return LT_E_ARG;
    auto* c = new (std::nothrow) lt_slot_cache();
    if (!c) return LT_E_ARG;
    c->slots.resize(n_slots);
    *out = c;
    return LT_OK;
}

void lt_slot_cache_destroy(lt_slot_cache* c) { delete c; }

lt_status lt_slot_cache_place(const lt_slot_cache* c, const int32_t* prompt, uint32_t n, int32_t adapter,
                              lt_placement* out) {
    if (!c || !out || (n && !prompt)) return LT_E_ARG;
    const uint32_t cap = n > 0 ? n - 1 : 0;  // one prompt token is always evaluated
    auto matches = [&](const Slot& s) -> uint32_t {
        return s.adapter == adapter ? std::min(common_prefix(s.tokens, prompt, n), cap) : 0u;
    };
    // free slot: longest match; among equal matches the least recently used;
    // the last of full ties (max_by)
    int best = -1;
    uint32_t own = 0;
    for (uint32_t i = 0; i < c->slots.size(); ++i) {
        const Slot& s = c->slots[i];
        if (s.busy) continue;
        const uint32_t m = matches(s);
        if (best < 0 || m > own || (m == own && s.last_used <= c->slots[(size_t)best].last_used)) {
            best = (int)i;
            own = m;
        }
    }
    if (best < 0) return LT_E_FULL;
    // any other slot, busy or not: the longest match, the last of ties (max_by_key)
    int other = -1;
    uint32_t on = 0;
    for (uint32_t i = 0; i < c->slots.size(); ++i) {
        if ((int)i == best) continue;
        const uint32_t m = matches(c->slots[i]);
        if (other < 0 || m >= on) {
            other = (int)i;
            on = m;
        }
    }
    out->slot = (uint32_t)best;
    if (other >= 0 && on >= own + LT_MIN_COPY_GAIN) {
        out->reuse = on;
        out->copy_src = other;
        out->copy_len = on;
    } else {
        out->reuse = own;
        out->copy_src = -1;
        out->copy_len = 0;
    }
    return LT_OK;
}

lt_status lt_slot_cache_acquire(lt_slot_cache* c, const lt_placement* p, const int32_t* prompt, uint32_t n,
                                int32_t adapter) {
    if (!c || !p || p->slot >= c->slots.size() || p->reuse > n || (n && !prompt)) return LT_E_ARG;
    c->clock += 1;
    Slot& s = c->slots[p->slot];
    s.busy = true;
    s.last_used = c->clock;
    s.adapter = adapter;
    s.tokens.assign(prompt, prompt + p->reuse);
    return LT_OK;
}

lt_status lt_slot_cache_release(lt_slot_cache* c, uint32_t slot, const int32_t* tokens, uint32_t n) {
    if (!c || slot >= c->slots.size() || (n && !tokens)) return LT_E_ARG;
    c->clock += 1;
    Slot& s = c->slots[slot];
    s.busy = false;
    s.last_used = c->clock;
    s.tokens.assign(tokens, tokens + n);
    return LT_OK;
}

int32_t lt_slot_cache_evict_lru(lt_slot_cache* c) {
    if (!c) return -1;
    int best = -1;
    for (uint32_t i = 0; i < c->slots.size(); ++i) {  // min_by_key: the first of equal minima
        const Slot& s = c->slots[i];
        if (s.busy || s.tokens.empty()) continue;
        if (best < 0 || s.last_used < c->slots[(size_t)best].last_used) best = (int)i;
    }
    if (best >= 0) c->slots[(size_t)best].tokens.clear();
    return best;
}

uint64_t lt_slot_cache_idle_cells(const lt_slot_cache* c) {
    uint64_t n = 0;
    if (c)
        for (const Slot& s : c->slots)
            if (!s.busy) n += s.tokens.size();
    return n;
}

int lt_slot_cache_has_free(const lt_slot_cache* c) {
    if (!c) return 0;
    for (const Slot& s : c->slots)
        if (!s.busy) return 1;
    return 0;
}

uint32_t lt_slot_cache_tokens(const lt_slot_cache* c, uint32_t slot, int32_t* out, uint32_t cap) {
    if (!c || slot >= c->slots.size()) return 0;
    const auto& t = c->slots[slot].tokens;
    const size_t k = std::min<size_t>(t.size(), cap);
    if (out && k) std::memcpy(out, t.data(), k * sizeof(int32_t));  // an empty vector's data() may be null
    return (uint32_t)t.size();
}

lt_status lt_slot_cache_slot_state(const lt_slot_cache* c, uint32_t slot, int32_t* busy, int32_t* adapter,
                                   uint64_t* last_used) {
    if (!c || slot >= c->slots.size()) return LT_E_ARG;
    const Slot& s = c->slots[slot];
    if (busy) *busy = s.busy ? 1 : 0;
    if (adapter) *adapter = s.adapter;
    if (last_used) *last_used = s.last_used;
    return LT_OK;
}

lt_status lt_slot_cache_set_slot(lt_slot_cache* c, uint32_t slot, const int32_t* tokens, uint32_t n,
                                 int32_t adapter) {
    if (!c || slot >= c->slots.size() || (n && !tokens)) return LT_E_ARG;
    c->slots[slot].tokens.assign(tokens, tokens + n);
    c->slots[slot].adapter = adapter;
    return LT_OK;
}

}  // extern "C"
