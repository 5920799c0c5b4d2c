// Host side of the B200 paged KV cache: the reference's KvCache bookkeeping
// (engine/crates/native/src/kv.rs) kept bit-identical on the host, the
// device mirror of the block tables, and the C ABI of include/lt_kv.h.
//
// Host/device split.  Allocation, refcounts, the LIFO free list and every
// sequence's block list live here (they are O(tokens/16) integer work and
// their order must match the reference exactly).  Their device-side effects
// -- copy-on-write block copies, compaction moves and block-table entries --
// are queued and applied by one kv_apply_plan launch right before the next
// kernel that reads them, on that kernel's stream.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <initializer_list>
#include <string>
#include <vector>

#include "lt_kv.h"
#include "lt_kv_internal.h"

using ltkv::kBlock;

namespace {

constexpr int kSlots = 8;  // staging ring depth (pinned host + device pairs)
constexpr uint32_t kCascadeMaxTokens = 1024;  // tokens of one call the prefix pass serves
constexpr int kCascadeMinBlocks = 4;          // shortest shared prefix worth a pass (64 positions)
constexpr uint32_t kClean = 0xFFFFFFFFu;

struct Slot {
    void* host = nullptr;
    void* dev = nullptr;
    cudaEvent_t ev = nullptr;
    uint64_t gen = 0;
    bool used = false;
};

// Device copy of a small host array, reused while the contents are unchanged
// (e.g. the same batch cells for every layer of a forward pass).
struct UploadCache {
    std::vector<char> key;
    int slot = -1;
    uint64_t gen = 0;
};

struct DeviceGuard {
    int prev = -1;
    bool ok = true;
    // dev < 0 (bookkeeping-only handle): touch no CUDA state at all.
    explicit DeviceGuard(int dev) {
        if (dev < 0) return;
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) ok = cudaSetDevice(dev) == cudaSuccess;
    }
    ~DeviceGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

}  // namespace

// Head-sharded gather over NVLink (lt_kv_peer_*): this rank's exported
// buffer is [flags: u32 per rank][done counter][half 0][half 1], each half
// [max_tokens][nranks * n_heads][head_dim] of f32 (f16 rows use half of it),
// of which this rank writes its own heads; calls alternate halves (epoch
// parity).  Peers' buffers are IPC mappings, read after their flags.
struct PeerGather {
    int rank = -1, nranks = 0;
    uint32_t max_tokens = 0;
    size_t half_bytes = 0;
    unsigned char* d_buf = nullptr;                 // own allocation (exported)
    unsigned char* base[ltkv::kMaxPeers] = {};      // every rank's buffer in this process (own: d_buf)
    bool mapped[ltkv::kMaxPeers] = {};              // opened with cudaIpcOpenMemHandle
    uint32_t epoch = 0;                             // gather calls so far (same on every rank)
    bool ready = false;
    // Set by export, cleared by import: the flags in a buffer hold the epochs
    // of every call made through it, so a second import of the same buffers
    // (epoch back at 0) would see stale flags as raised.
    bool fresh = false;
};
constexpr size_t kPeerFlagsBytes = 256, kPeerHeaderBytes = 512;
static_assert(sizeof(cudaIpcMemHandle_t) == LT_IPC_HANDLE_BYTES, "IPC handle size");
static_assert(ltkv::kMaxPeers * sizeof(uint32_t) <= kPeerFlagsBytes, "peer flags");

// Device timing of one kind of launch: (start, end) event pairs in a ring,
// folded into the totals when read or when the ring is full.
struct ProfRing {
    std::vector<cudaEvent_t> ev;
    size_t head = 0, pending = 0;
    double ms = 0.0;
    uint64_t count = 0;
};

struct lt_kv {
    lt_kv_config cfg{};
    PeerGather peer;
    uint32_t min_tiles_per_warp = 8;  // attention launch sizing (lt_kv_set_min_tiles_per_warp)
    // shared-prefix (cascade) pass: groups of >= cascade_min_tokens tokens
    // whose sequences share >= kCascadeMinBlocks leading blocks (0: off)
    uint32_t cascade_min_tokens = 8;
    uint32_t pre_cap = 0;          // tokens the prefix partial buffers hold
    int sm_count = 0;              // of the device: the prefix pass splits blocks to fill it
    float* d_pre_o = nullptr;      // [pre_cap][n_heads][head_dim]
    float* d_pre_ml = nullptr;     // [pre_cap][n_heads][2]
    std::vector<uint32_t> casc_order;
    std::vector<int32_t> casc_buf;  // upload image: PrefixItems then the token list
    uint64_t cascade_launches = 0;
    int casc_splits = 1;
    size_t casc_ntok = 0;  // tokens in the upload image's token list
    uint32_t n_blocks = 0, kv_dim = 0, group = 0, max_blocks = 0;
    bool q8 = false;          // LT_KV_Q8_0 pool
    size_t block_elems = 0;   // 16-bit units of one block in one layer (all heads, K and V)
    size_t layer_elems = 0;   // 16-bit units of one layer of the pool

    // ---- reference bookkeeping (kv.rs:15-26) ----
    std::vector<std::vector<int32_t>> blocks;  // per sequence
    std::vector<uint32_t> lens;
    std::vector<uint32_t> refs;
    std::vector<int32_t> free_list;  // stack: back() is popped first
    // free_list[0, free_run) is the run nb-1, nb-2, ..., nb-free_run (ids no
    // one touched since the last compaction): compaction only sorts the rest.
    size_t free_run = 0;
    // The sequence and table index that took a block (alloc, copy-on-write,
    // compaction move), and whether it was ever shared (then a move falls back
    // to scanning every table).
    std::vector<int32_t> owner_seq, owner_idx;
    std::vector<uint8_t> ever_shared;
    std::vector<int32_t> cmp_low;  // compaction scratch

    std::string err;
    bool dev = false;

    // ---- device state ----
    uint16_t* d_pool = nullptr;
    int32_t* d_tables = nullptr;
    float* d_part_o = nullptr;
    float* d_part_ml = nullptr;
    int32_t* d_err = nullptr;
    uint32_t* d_flags = nullptr;  // attention: per-warp range-done flags (epoch values)
    uint32_t attn_epoch = 0;
    size_t ws_slots = 0;  // split-K partial slots (one per split piece)
    size_t slot_bytes = 0;
    Slot slots[kSlots];
    int next_slot = 0;

    // ---- queued device work ----
    std::vector<int2> pend_copies;
    std::vector<uint32_t> mark_src, mark_dst;
    uint32_t epoch = 1;
    std::vector<uint32_t> dirty_from;  // per seq, first table index to re-upload
    std::vector<uint32_t> dirty_list;
    std::vector<int2> tw_tmp;

    std::vector<int32_t> dev_shadow;  // what the device tables hold (host copy)

    // launch timing (lt_kv_profile): attention launches, and plan launches
    // (copy-on-write copies, compaction moves, table entries)
    bool profiling = false;
    ProfRing prof_attn, prof_plan, prof_write;
    uint64_t plan_blocks = 0, plan_entries = 0;  // block copies and table entries of the timed plan launches
    uint64_t write_rows = 0, write_in_bytes = 0;  // rows and input bytes of the timed write launches

    UploadCache cells_cache, items_cache, casc_cache;
    std::vector<ltkv::TokenDesc> toks_tmp;
    std::vector<std::pair<size_t, int32_t>> fold_tmp;  // (table index, previous shadow value)
    std::vector<uint32_t> fold_mark, fold_pos;         // per sequence, for one call
    uint32_t fold_epoch = 0;
    ltkv::AttnParams params{};                         // large (inline descriptors): kept here
    std::vector<int2> cells_tmp;
    uint64_t launches = 0;
};

namespace {

lt_status fail(lt_kv* kv, lt_status s, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    if (kv) kv->err = buf;
    return s;
}

#define LT_CUDA(kv, call)                                                                              \
    do {                                                                                               \
        cudaError_t e_ = (call);                                                                       \
        if (e_ != cudaSuccess) return fail((kv), LT_E_CUDA, "%s: %s", #call, cudaGetErrorString(e_)); \
    } while (0)

void peer_unmap(lt_kv* kv) {
    PeerGather& pg = kv->peer;
    for (int r = 0; r < ltkv::kMaxPeers; ++r) {
        if (pg.mapped[r]) cudaIpcCloseMemHandle(pg.base[r]);
        pg.mapped[r] = false;
        pg.base[r] = nullptr;
    }
    pg.ready = false;
}

void free_device(lt_kv* kv) {
    peer_unmap(kv);
    cudaFree(kv->peer.d_buf);
    kv->peer = PeerGather{};
    cudaFree(kv->d_pool);
    cudaFree(kv->d_tables);
    cudaFree(kv->d_part_o);
    cudaFree(kv->d_part_ml);
    cudaFree(kv->d_pre_o);
    cudaFree(kv->d_pre_ml);
    kv->d_pre_o = kv->d_pre_ml = nullptr;
    cudaFree(kv->d_err);
    cudaFree(kv->d_flags);
    kv->d_flags = nullptr;
    for (auto& s : kv->slots) {
        if (s.host) cudaFreeHost(s.host);
        if (s.dev) cudaFree(s.dev);
        if (s.ev) cudaEventDestroy(s.ev);
        s = Slot{};
    }
    for (ProfRing* r : {&kv->prof_attn, &kv->prof_plan, &kv->prof_write}) {
        for (cudaEvent_t e : r->ev) cudaEventDestroy(e);
        r->ev.clear();
    }
    kv->d_pool = nullptr;
    kv->d_tables = nullptr;
    kv->d_part_o = kv->d_part_ml = nullptr;
    kv->d_err = nullptr;
}

// Next staging slot; waits until every kernel that read its previous
// contents has finished (the slot's event).
int acquire_slot(lt_kv* kv) {
    const int s = kv->next_slot;
    kv->next_slot = (s + 1) % kSlots;
    Slot& sl = kv->slots[s];
    if (sl.used) cudaEventSynchronize(sl.ev);
    sl.gen++;
    sl.used = true;
    return s;
}

lt_status mark_slot_use(lt_kv* kv, int s, cudaStream_t st) {
    LT_CUDA(kv, cudaEventRecord(kv->slots[s].ev, st));
    return LT_OK;
}

// Upload `bytes` of `src` through the staging ring, reusing the previous
// upload of the same contents while its slot has not been recycled.
lt_status upload(lt_kv* kv, UploadCache& cache, const void* src, size_t bytes, cudaStream_t st, const void** dptr,
                 int* slot_out) {
    if (bytes > kv->slot_bytes) return fail(kv, LT_E_ARG, "upload of %zu bytes exceeds staging slot", bytes);
    if (cache.slot >= 0 && kv->slots[cache.slot].gen == cache.gen && cache.key.size() == bytes &&
        std::memcmp(cache.key.data(), src, bytes) == 0) {
        *dptr = kv->slots[cache.slot].dev;
        *slot_out = cache.slot;
        return LT_OK;
    }
    const int s = acquire_slot(kv);
    std::memcpy(kv->slots[s].host, src, bytes);
    LT_CUDA(kv, cudaMemcpyAsync(kv->slots[s].dev, kv->slots[s].host, bytes, cudaMemcpyHostToDevice, st));
    cache.key.assign(static_cast<const char*>(src), static_cast<const char*>(src) + bytes);
    cache.slot = s;
    cache.gen = kv->slots[s].gen;
    *dptr = kv->slots[s].dev;
    *slot_out = s;
    return LT_OK;
}

lt_status prof_begin(lt_kv* kv, ProfRing& r, cudaStream_t st, cudaEvent_t* end);

// Launch kv_apply_plan for `copies` and table writes `tw`, split to fit the
// staging slots.  All copies in one call are independent of each other.
lt_status run_plan(lt_kv* kv, const std::vector<int2>& copies, const std::vector<int2>& tw, cudaStream_t st) {
    const size_t cap = kv->slot_bytes / sizeof(int2);
    size_t ci = 0, ti = 0;
    while (ci < copies.size() || ti < tw.size()) {
        const size_t nc = std::min(copies.size() - ci, cap);
        const size_t nt = std::min(tw.size() - ti, cap - nc);
        const int s = acquire_slot(kv);
        int2* h = static_cast<int2*>(kv->slots[s].host);
        if (nc) std::memcpy(h, copies.data() + ci, nc * sizeof(int2));
        if (nt) std::memcpy(h + nc, tw.data() + ti, nt * sizeof(int2));
        LT_CUDA(kv, cudaMemcpyAsync(kv->slots[s].dev, h, (nc + nt) * sizeof(int2), cudaMemcpyHostToDevice, st));
        const int2* d = static_cast<const int2*>(kv->slots[s].dev);
        cudaEvent_t ev_end = nullptr;
        if (kv->profiling) {  // the kernel alone: after the plan's upload
            lt_status prc = prof_begin(kv, kv->prof_plan, st, &ev_end);
            if (prc) return prc;
            kv->plan_blocks += nc;
            kv->plan_entries += nt;
        }
        LT_CUDA(kv, ltkv::launch_apply_plan(kv->d_pool, kv->layer_elems, kv->block_elems, (int)kv->cfg.n_layers, d,
                                            (int)nc, kv->d_tables, d + nc, (int)nt, (int)kv->n_blocks,
                                            (long long)kv->cfg.max_seqs * kv->max_blocks, kv->d_err, st));
        if (ev_end) LT_CUDA(kv, cudaEventRecord(ev_end, st));
        kv->launches++;
        lt_status rc = mark_slot_use(kv, s, st);
        if (rc) return rc;
        ci += nc;
        ti += nt;
    }
    return LT_OK;
}

lt_status flush(lt_kv* kv, cudaStream_t st) {
    if (!kv->dev) {
        kv->pend_copies.clear();
        for (uint32_t s : kv->dirty_list) kv->dirty_from[s] = kClean;
        kv->dirty_list.clear();
        return LT_OK;
    }
    if (kv->pend_copies.empty() && kv->dirty_list.empty()) return LT_OK;
    kv->tw_tmp.clear();
    for (uint32_t s : kv->dirty_list) {
        const auto& bl = kv->blocks[s];
        const size_t row = (size_t)s * kv->max_blocks;
        for (size_t i = kv->dirty_from[s]; i < bl.size(); ++i) {
            if (kv->dev_shadow[row + i] == bl[i]) continue;  // device already holds it
            kv->dev_shadow[row + i] = bl[i];
            kv->tw_tmp.push_back(make_int2((int)(row + i), bl[i]));
        }
        kv->dirty_from[s] = kClean;
    }
    kv->dirty_list.clear();
    lt_status rc = run_plan(kv, kv->pend_copies, kv->tw_tmp, st);
    kv->pend_copies.clear();
    kv->epoch++;
    return rc;
}

void mark_dirty(lt_kv* kv, uint32_t seq, uint32_t idx) {
    if (!kv->dev) return;
    if (kv->dirty_from[seq] == kClean) {
        kv->dirty_list.push_back(seq);
        kv->dirty_from[seq] = idx;
    } else if (idx < kv->dirty_from[seq]) {
        kv->dirty_from[seq] = idx;
    }
}

void release_block(lt_kv* kv, int32_t b) {  // kv.rs:76-82
    kv->refs[b] -= 1;
    if (kv->refs[b] == 0) kv->free_list.push_back(b);
}

// KvCache::append for one token (kv.rs:85-121).
lt_status append_one(lt_kv* kv, uint32_t seq, uint32_t pos, int32_t* block_out, int32_t* slot_out,
                     cudaStream_t st) {
    if (seq >= kv->cfg.max_seqs) return fail(kv, LT_E_ARG, "seq %u out of range (max_seqs %u)", seq, kv->cfg.max_seqs);
    auto& bl = kv->blocks[seq];
    const uint32_t len = kv->lens[seq];
    if (pos != len) return fail(kv, LT_E_NONCONTIG, "seq %u: position %u is not contiguous (length %u)", seq, pos, len);
    const uint32_t slot = pos % kBlock;
    if (slot == 0) {
        if (bl.size() >= kv->max_blocks)
            return fail(kv, LT_E_ARG, "seq %u exceeds max_blocks_per_seq (%u)", seq, kv->max_blocks);
        if (kv->free_list.empty()) return fail(kv, LT_E_FULL, "KV cache full");
        const int32_t b = kv->free_list.back();  // kv.rs:67-74
        kv->free_list.pop_back();
        kv->free_run = std::min(kv->free_run, kv->free_list.size());
        kv->refs[b] = 1;
        bl.push_back(b);
        kv->owner_seq[b] = (int32_t)seq;
        kv->owner_idx[b] = (int32_t)bl.size() - 1;
        kv->ever_shared[b] = 0;
        mark_dirty(kv, seq, (uint32_t)bl.size() - 1);
    } else {
        const int32_t last = bl.back();
        if (kv->refs[last] > 1) {  // copy-on-write, kv.rs:99-110
            if (kv->free_list.empty()) return fail(kv, LT_E_FULL, "KV cache full");
            const int32_t nb = kv->free_list.back();
            if (kv->dev) {
                // A queued copy that reads `nb` or writes `last`/`nb` must land first.
                if (kv->mark_dst[last] == kv->epoch || kv->mark_dst[nb] == kv->epoch || kv->mark_src[nb] == kv->epoch) {
                    lt_status rc = flush(kv, st);
                    if (rc) return rc;
                }
                kv->pend_copies.push_back(make_int2(last, nb));
                kv->mark_src[last] = kv->epoch;
                kv->mark_dst[nb] = kv->epoch;
            }
            kv->free_list.pop_back();
            kv->free_run = std::min(kv->free_run, kv->free_list.size());
            kv->refs[nb] = 1;
            release_block(kv, last);
            bl.back() = nb;
            kv->owner_seq[nb] = (int32_t)seq;
            kv->owner_idx[nb] = (int32_t)bl.size() - 1;
            kv->ever_shared[nb] = 0;
            mark_dirty(kv, seq, (uint32_t)bl.size() - 1);
        }
    }
    kv->lens[seq] = pos + 1;
    *block_out = bl.back();
    *slot_out = (int32_t)slot;
    return LT_OK;
}

void truncate_impl(lt_kv* kv, uint32_t seq, uint32_t from) {  // kv.rs:153-169
    if (seq >= kv->cfg.max_seqs) return;
    auto& bl = kv->blocks[seq];
    if (from >= kv->lens[seq]) return;
    const size_t keep = (from + kBlock - 1) / kBlock;
    for (size_t i = keep; i < bl.size(); ++i) release_block(kv, bl[i]);  // ascending order
    bl.resize(keep);
    kv->lens[seq] = from;
}

// lt_dtype arguments must name one of the enum's values: anything else is
// refused rather than read as f16.  Checked at the extern "C" entry, through
// the arguments' addresses, before any copy of them.
lt_status check_dtypes(lt_kv* kv, std::initializer_list<const lt_dtype*> ds) {
    for (const lt_dtype* d : ds)
        if (!ltkv::dtype_valid(*d)) {
            int32_t v;
            std::memcpy(&v, d, sizeof v);
            return fail(kv, LT_E_ARG, "dtype %d is neither LT_F32 nor LT_F16", (int)v);
        }
    return LT_OK;
}

lt_status require_device(lt_kv* kv) {
    if (!kv->dev) return fail(kv, LT_E_ARG, "handle was created without a device (device = -1)");
    return LT_OK;
}

lt_status check_tokens(lt_kv* kv, const uint32_t* seq, const uint32_t* pos, uint32_t n) {
    if (n > kv->cfg.max_batch) return fail(kv, LT_E_ARG, "batch of %u tokens exceeds max_batch %u", n, kv->cfg.max_batch);
    for (uint32_t i = 0; i < n; ++i) {
        if (seq[i] >= kv->cfg.max_seqs) return fail(kv, LT_E_ARG, "seq %u out of range", seq[i]);
        if (pos[i] >= kv->lens[seq[i]])
            return fail(kv, LT_E_ARG, "seq %u: position %u not in the cache (length %u)", seq[i], pos[i],
                        kv->lens[seq[i]]);
    }
    return LT_OK;
}

lt_status check_cells(lt_kv* kv, const int32_t* block, const int32_t* slot, uint32_t n) {
    if (n > kv->cfg.max_batch) return fail(kv, LT_E_ARG, "batch of %u tokens exceeds max_batch %u", n, kv->cfg.max_batch);
    for (uint32_t i = 0; i < n; ++i) {
        if (block[i] < 0 || (uint32_t)block[i] >= kv->n_blocks || slot[i] < 0 || slot[i] >= kBlock)
            return fail(kv, LT_E_ARG, "cell %u (block %d, slot %d) out of range", i, block[i], slot[i]);
    }
    return LT_OK;
}

constexpr size_t kProfPairs = 512;

// Fold the oldest `n` recorded (start, end) pairs of a ring into its totals.
lt_status prof_drain(lt_kv* kv, ProfRing& r, size_t n) {
    while (n-- && r.pending) {
        const size_t tail = (r.head + kProfPairs - r.pending) % kProfPairs;
        float ms = 0.f;
        LT_CUDA(kv, cudaEventSynchronize(r.ev[2 * tail + 1]));
        LT_CUDA(kv, cudaEventElapsedTime(&ms, r.ev[2 * tail], r.ev[2 * tail + 1]));
        r.ms += ms;
        r.count++;
        r.pending--;
    }
    return LT_OK;
}

// Record the start event of the next launch of a ring's kind; *end gets its
// end event.
lt_status prof_begin(lt_kv* kv, ProfRing& r, cudaStream_t st, cudaEvent_t* end) {
    if (r.pending == kProfPairs) {
        lt_status rc = prof_drain(kv, r, 1);
        if (rc) return rc;
    }
    const size_t i = r.head;
    r.head = (r.head + 1) % kProfPairs;
    r.pending++;
    LT_CUDA(kv, cudaEventRecord(r.ev[2 * i], st));
    *end = r.ev[2 * i + 1];
    return LT_OK;
}

// Shared-prefix groups of one attention call: tokens whose sequences start
// with the same block, at least cascade_min_tokens of them, sharing at least
// kCascadeMinBlocks leading blocks (all strictly before every member token's
// own block).  Each group's tokens get skip = its shared block count.  When
// every token of a group belongs to one sequence (a prefill chunk), each
// token's skip is instead its own block index: the pass then covers, row by
// row, every block before the token's own one (causally masked), and the
// stream-K launch only the token's own block.  The prefix pass items (KV
// head x chunks of the group's tokens, each over [0, its tokens' largest
// skip)), the token list and the tokens' skips go to casc_buf.  Returns the
// number of items (0: no pass).
int plan_cascade(lt_kv* kv, const uint32_t* seq, const uint32_t* pos, uint32_t n) {
    if (kv->cascade_min_tokens == 0 || n < kv->cascade_min_tokens || n > kv->pre_cap) return 0;
    auto& ord = kv->casc_order;
    ord.resize(n);
    for (uint32_t i = 0; i < n; ++i) ord[i] = i;
    std::sort(ord.begin(), ord.end(), [&](uint32_t a, uint32_t b) {
        const int32_t fa = kv->blocks[seq[a]][0], fb = kv->blocks[seq[b]][0];
        return fa != fb ? fa < fb : a < b;
    });
    const int tpc = ltkv::prefix_tokens_per_cta((int)kv->group);
    const uint32_t hkv = kv->cfg.n_kv_heads;
    struct Group {
        int32_t root, P, off, cnt;
        bool one_seq;  // every token of the group is of sequence root
    };
    std::vector<Group> groups;
    std::vector<int32_t> toks;
    for (uint32_t a = 0; a < n;) {
        const int32_t first = kv->blocks[seq[ord[a]]][0];
        uint32_t b = a + 1;
        while (b < n && kv->blocks[seq[ord[b]]][0] == first) ++b;
        if (b - a >= kv->cascade_min_tokens) {
            const uint32_t root = seq[ord[a]];
            const std::vector<int32_t>& rb = kv->blocks[root];
            size_t P = pos[ord[a]] / kBlock;
            for (uint32_t k = a; k < b && P >= (size_t)kCascadeMinBlocks; ++k) {
                const uint32_t i = ord[k];
                P = std::min<size_t>(P, pos[i] / kBlock);
                if (seq[i] != root) {
                    const std::vector<int32_t>& sb = kv->blocks[seq[i]];
                    const size_t lim = std::min(P, std::min(sb.size(), rb.size()));
                    P = (size_t)(std::mismatch(rb.begin(), rb.begin() + lim, sb.begin()).first - rb.begin());
                }
            }
            if (P >= (size_t)kCascadeMinBlocks) {
                bool one_seq = true;
                for (uint32_t k = a; k < b && one_seq; ++k) one_seq = seq[ord[k]] == root;
                groups.push_back({(int32_t)root, (int32_t)P, (int32_t)toks.size(), (int32_t)(b - a), one_seq});
                for (uint32_t k = a; k < b; ++k) {
                    toks.push_back((int32_t)ord[k]);
                    kv->toks_tmp[ord[k]].skip = one_seq ? (int32_t)(pos[ord[k]] / kBlock) : (int32_t)P;
                }
            }
        }
        a = b;
    }
    // Blocks each chunk of tpc tokens covers: its tokens' largest skip.
    auto chunk_blocks = [&](const Group& g, int32_t c0) {
        int32_t L = 0;
        for (int32_t k = c0; k < std::min(g.cnt, c0 + tpc); ++k) L = std::max(L, kv->toks_tmp[toks[g.off + k]].skip);
        return L;
    };
    // Split every chunk's blocks over S CTAs so the pass fills the SMs; each
    // split keeps at least one 4-block step.
    long long base_items = 0;
    int min_p = 1 << 30;
    for (const Group& g : groups) {
        base_items += (long long)hkv * ((g.cnt + tpc - 1) / tpc);
        for (int32_t c0 = 0; c0 < g.cnt; c0 += tpc) min_p = std::min(min_p, (int)chunk_blocks(g, c0));
    }
    int S = 1;
    if (base_items > 0)
        S = (int)std::max<long long>(1, std::min<long long>(ltkv::kPreMaxSplits, kv->sm_count / base_items));
    S = std::max(1, std::min(S, min_p / 4));
    kv->casc_splits = S;
    std::vector<ltkv::PrefixItem> items;
    for (const Group& g : groups)
        for (int32_t c0 = 0; c0 < g.cnt; c0 += tpc) {
            const int32_t L = chunk_blocks(g, c0);
            for (uint32_t h = 0; h < hkv; ++h)
                for (int sp = 0; sp < S; ++sp) {
                    const int32_t b0 = (int32_t)((long long)L * sp / S), b1 = (int32_t)((long long)L * (sp + 1) / S);
                    items.push_back({g.root, b0, b1, sp, (int32_t)h, g.off + c0, std::min(tpc, g.cnt - c0)});
                }
        }
    const size_t item_words = items.size() * (sizeof(ltkv::PrefixItem) / 4);
    kv->casc_buf.resize(item_words + 2 * toks.size());
    if (!items.empty()) std::memcpy(kv->casc_buf.data(), items.data(), items.size() * sizeof(ltkv::PrefixItem));
    for (size_t k = 0; k < toks.size(); ++k) {
        kv->casc_buf[item_words + k] = toks[k];
        kv->casc_buf[item_words + toks.size() + k] = kv->toks_tmp[toks[k]].skip;
    }
    kv->casc_ntok = toks.size();
    return (int)items.size();
}

lt_status attend_impl(lt_kv* kv, uint32_t layer, const void* q, lt_dtype q_dtype, const uint32_t* seq,
                      const uint32_t* pos, uint32_t n, void* out, lt_dtype out_dtype, float scale, const void* k,
                      const void* v, lt_dtype kv_dtype, bool fused, cudaStream_t st, bool gather = false) {
    if ((reinterpret_cast<uintptr_t>(q) & 15) || (reinterpret_cast<uintptr_t>(out) & 15) ||
        (k && (reinterpret_cast<uintptr_t>(k) & 15)) || (v && (reinterpret_cast<uintptr_t>(v) & 15)))
        return fail(kv, LT_E_ARG, "q, out, k and v must be 16-byte aligned device pointers");
    if (gather) {
        if (!kv->peer.ready) return fail(kv, LT_E_ARG, "attend_gather before lt_kv_peer_import");
        if (n > kv->peer.max_tokens)
            return fail(kv, LT_E_ARG, "attend_gather of %u tokens exceeds the exported max_tokens %u", n,
                        kv->peer.max_tokens);
    }
    if (n == 0) return flush(kv, st);
    // Per-token descriptors; the kernel derives its stream-K partition from them.
    const int q_f32 = q_dtype == LT_F32;
    const int max_warps = ltkv::attend_warps(kv->cfg.device, (int)kv->group, (int)kv->cfg.head_dim, q_f32, kv->q8);
    if (max_warps <= 0) return fail(kv, LT_E_CUDA, "could not size the attention launch on device %d", kv->cfg.device);
    kv->toks_tmp.resize(n);
    for (uint32_t i = 0; i < n; ++i) {
        ltkv::TokenDesc& t = kv->toks_tmp[i];
        t.seq = (int32_t)seq[i];
        t.pos = (int32_t)pos[i];
        t.last_block = kv->blocks[seq[i]][pos[i] / kBlock];
        t.skip = 0;
    }
    // sets skip of the tokens it covers; Q8_0 tiles are not f16 tensor-core operands
    const int n_items = kv->q8 ? 0 : plan_cascade(kv, seq, pos, n);
    long long tiles = 0;
    for (uint32_t i = 0; i < n; ++i) {
        ltkv::TokenDesc& t = kv->toks_tmp[i];
        t.prefix = (int32_t)tiles;
        tiles += pos[i] / kBlock + 1 - t.skip;
    }
    if (tiles > 0x7FFFFFFFll / kv->cfg.n_kv_heads) return fail(kv, LT_E_ARG, "attention call too large");
    // The kernel writes every token's last table entry itself.  For the
    // highest position of each sequence in the call that entry is read by no
    // other token from the table, so its pending upload is dropped; the
    // shadow is restored if the launch fails.
    kv->fold_tmp.clear();
    if (++kv->fold_epoch == 0) {  // wrapped: start the marks afresh
        std::fill(kv->fold_mark.begin(), kv->fold_mark.end(), 0u);
        kv->fold_epoch = 1;
    }
    for (uint32_t i = n; i-- > 0;) {
        if (kv->fold_mark[seq[i]] == kv->fold_epoch && kv->fold_pos[seq[i]] >= pos[i]) continue;
        kv->fold_mark[seq[i]] = kv->fold_epoch;
        kv->fold_pos[seq[i]] = pos[i];
    }
    for (uint32_t i = 0; i < n; ++i) {
        if (kv->fold_pos[seq[i]] != pos[i] || kv->fold_mark[seq[i]] != kv->fold_epoch) continue;
        kv->fold_mark[seq[i]] = 0;  // once per sequence
        const size_t idx = (size_t)seq[i] * kv->max_blocks + pos[i] / kBlock;
        const int32_t val = kv->toks_tmp[i].last_block;
        if (kv->dev_shadow[idx] != val) {
            kv->fold_tmp.push_back(std::make_pair(idx, kv->dev_shadow[idx]));
            kv->dev_shadow[idx] = val;
        }
    }
    lt_status rc = flush(kv, st);
    auto rollback = [&]() {
        for (auto& f : kv->fold_tmp) kv->dev_shadow[f.first] = f.second;
    };
    if (rc) {
        rollback();
        return rc;
    }
    ltkv::AttnParams& p = kv->params;
    p.pool_layer = kv->d_pool + (size_t)layer * kv->layer_elems;
    p.pool_layer_w = kv->d_pool + (size_t)layer * kv->layer_elems;
    p.tables = kv->d_tables;
    p.max_blocks = (int32_t)kv->max_blocks;
    p.n_blocks = (int32_t)kv->n_blocks;
    p.check_ids = 0;  // this handle's bookkeeping wrote the tables
    p.n_tok = (int32_t)n;
    p.tiles_per_head = (int32_t)tiles;
    // At least min_tiles_per_warp tiles a warp: a small step (few tokens, short
    // contexts) runs on fewer warps with fewer split merges instead of
    // paying every warp's ramp for one tile.
    const long long total_tiles = tiles * kv->cfg.n_kv_heads;
    const long long want = (total_tiles + kv->min_tiles_per_warp - 1) / kv->min_tiles_per_warp;
    p.n_warps = (int32_t)std::min<long long>(max_warps, std::max<long long>(want, total_tiles ? 1 : 0));
    p.n_kv_heads = (int32_t)kv->cfg.n_kv_heads;
    p.group = (int32_t)kv->group;
    p.q = q;
    p.q_f32 = q_f32;
    p.out = out;
    p.out_f32 = out_dtype == LT_F32;
    p.scale_log2 = scale * 1.4426950408889634f;
    p.part_o = kv->d_part_o;
    p.part_ml = kv->d_part_ml;
    p.flags = kv->d_flags;
    p.part2_o = kv->d_part_o + kv->ws_slots * kv->group * kv->cfg.head_dim;
    p.part2_ml = kv->d_part_ml + kv->ws_slots * kv->group * 2;
    p.flags2 = kv->d_flags + kv->ws_slots;
    // A waiter tests flag == epoch.  When the count wraps, a warp slot that
    // only large launches reach may still hold any earlier epoch, so the
    // flags restart from zero (0 is never an epoch).  On failure the count is
    // left as it was and the next launch tries again.
    uint32_t epoch = kv->attn_epoch + 1;
    if (epoch == 0) {
        const cudaError_t e = cudaMemsetAsync(kv->d_flags, 0, 2 * kv->ws_slots * sizeof(uint32_t) + 4, st);
        if (e != cudaSuccess) {
            rollback();
            return fail(kv, LT_E_CUDA, "cudaMemsetAsync(flags): %s", cudaGetErrorString(e));
        }
        epoch = 1;
    }
    kv->attn_epoch = epoch;
    p.epoch = epoch;
    p.err = kv->d_err;
    p.k_new = k;
    p.v_new = v;
    p.kv_f32 = kv_dtype == LT_F32;
    int s_plan = -1;
    if (n <= (uint32_t)ltkv::kInlineTokens) {
        p.toks = nullptr;  // descriptors travel in the kernel parameters
        std::memcpy(p.inl, kv->toks_tmp.data(), n * sizeof(ltkv::TokenDesc));
    } else {
        const void* d_toks = nullptr;
        rc = upload(kv, kv->items_cache, kv->toks_tmp.data(), n * sizeof(ltkv::TokenDesc), st, &d_toks, &s_plan);
        if (rc) {
            rollback();
            return rc;
        }
        p.toks = static_cast<const ltkv::TokenDesc*>(d_toks);
    }
    p.pre_o = kv->d_pre_o;
    p.pre_ml = kv->d_pre_ml;
    p.pre_splits = n_items > 0 ? kv->casc_splits : 0;
    p.q8 = kv->q8;
    p.pre_split_rows = (int64_t)kv->pre_cap * kv->cfg.n_heads;
    p.n_peers = 0;
    uint32_t g_epoch = 0;
    if (gather) {
        PeerGather& pg = kv->peer;
        if (++pg.epoch == 0) pg.epoch = 1;  // flags start at 0
        g_epoch = pg.epoch;
        p.n_peers = pg.nranks;
        p.peer_rank = pg.rank;
        p.peer_epoch = g_epoch;
        p.done_count = reinterpret_cast<uint32_t*>(pg.d_buf + kPeerFlagsBytes);
        p.gather_out = pg.d_buf + kPeerHeaderBytes + (g_epoch & 1) * pg.half_bytes;
        for (int r = 0; r < pg.nranks; ++r) p.peer_flag[r] = reinterpret_cast<uint32_t*>(pg.base[r]) + pg.rank;
        p.out = nullptr;
    }
    cudaEvent_t ev_end = nullptr;
    if (kv->profiling) {
        lt_status prc = prof_begin(kv, kv->prof_attn, st, &ev_end);
        if (prc) return prc;
    }
    int s_casc = -1;
    if (n_items > 0) {
        const void* d_casc = nullptr;
        rc = upload(kv, kv->casc_cache, kv->casc_buf.data(), kv->casc_buf.size() * sizeof(int32_t), st, &d_casc,
                    &s_casc);
        if (rc) {
            rollback();
            return rc;
        }
        ltkv::PrefixParams pp{};
        pp.pool_layer = p.pool_layer;
        pp.tables = kv->d_tables;
        pp.max_blocks = (int32_t)kv->max_blocks;
        pp.n_blocks = (int32_t)kv->n_blocks;
        pp.items = static_cast<const ltkv::PrefixItem*>(d_casc);
        pp.tok_list = static_cast<const int32_t*>(d_casc) + (size_t)n_items * (sizeof(ltkv::PrefixItem) / 4);
        pp.tok_lim = pp.tok_list + kv->casc_ntok;
        pp.n_kv_heads = (int32_t)kv->cfg.n_kv_heads;
        pp.group = (int32_t)kv->group;
        pp.q = q;
        pp.q_f32 = q_f32;
        pp.scale_log2 = p.scale_log2;
        pp.pre_o = kv->d_pre_o;
        pp.pre_ml = kv->d_pre_ml;
        pp.split_rows = p.pre_split_rows;
        pp.err = kv->d_err;
        const cudaError_t pe = ltkv::launch_prefix(pp, n_items, (int)kv->cfg.head_dim, st);
        if (pe != cudaSuccess) {
            rollback();
            return fail(kv, LT_E_CUDA, "prefix launch: %s", cudaGetErrorString(pe));
        }
        kv->launches++;
        kv->cascade_launches++;
    }
    const cudaError_t le = ltkv::launch_attend(p, (int)kv->cfg.head_dim, st);
    if (le != cudaSuccess) {
        rollback();
        return fail(kv, LT_E_CUDA, "attention launch: %s", cudaGetErrorString(le));
    }
    kv->launches += ltkv::attend_launches(p);
    if (ev_end) LT_CUDA(kv, cudaEventRecord(ev_end, st));
    if (gather) {
        const PeerGather& pg = kv->peer;
        const size_t slice = (size_t)kv->cfg.n_heads * kv->cfg.head_dim * (out_dtype == LT_F32 ? 4 : 2);
        void* srcs[ltkv::kMaxPeers] = {};
        for (int r = 0; r < pg.nranks; ++r) srcs[r] = pg.base[r] + kPeerHeaderBytes + (g_epoch & 1) * pg.half_bytes;
        LT_CUDA(kv, ltkv::launch_gather_wait_copy(reinterpret_cast<const uint32_t*>(pg.d_buf), pg.nranks, g_epoch,
                                                  srcs, out, n, slice, kv->d_err, st));
        kv->launches++;
    }
    if (s_casc >= 0 && (rc = mark_slot_use(kv, s_casc, st)) != LT_OK) return rc;
    return s_plan >= 0 ? mark_slot_use(kv, s_plan, st) : LT_OK;
}

}  // namespace

namespace ltkv {
size_t local_out_row_bytes(const lt_kv* kv, int dtype) {
    return (size_t)kv->cfg.n_heads * kv->cfg.head_dim * (dtype == LT_F32 ? 4 : 2);
}
int handle_device(const lt_kv* kv) { return kv->cfg.device; }
const lt_kv_config* handle_config(const lt_kv* kv) { return &kv->cfg; }
void count_launch(lt_kv* kv) { kv->launches++; }
int32_t seq_block_at(const lt_kv* kv, uint32_t seq, uint32_t idx) { return kv->blocks[seq][idx]; }
uint32_t block_refs(const lt_kv* kv, int32_t block) { return kv->refs[(size_t)block]; }
}  // namespace ltkv

// ============================================================== C ABI ====

extern "C" {

lt_status lt_kv_create(const lt_kv_config* cfg, lt_kv** out) {
    if (!cfg || !out) return LT_E_ARG;
    *out = nullptr;
    const lt_kv_config c = *cfg;
    if (c.n_layers == 0 || c.n_kv_heads == 0 || c.n_heads == 0 || c.max_seqs == 0 || c.max_batch == 0)
        return LT_E_ARG;
    if (c.n_heads % c.n_kv_heads != 0) return LT_E_ARG;
    if (c.head_dim != 64 && c.head_dim != 128) return LT_E_UNSUPPORTED;
    if (c.n_heads / c.n_kv_heads > (uint32_t)ltkv::kMaxGroup) return LT_E_UNSUPPORTED;
    if (c.kv_format != LT_KV_F16 && c.kv_format != LT_KV_Q8_0) return LT_E_ARG;
    lt_kv* kv = new (std::nothrow) lt_kv();
    if (!kv) return LT_E_ARG;
    kv->cfg = c;
    kv->n_blocks = (c.n_tokens + kBlock - 1) / kBlock;  // kv.rs:36
    kv->kv_dim = c.n_kv_heads * c.head_dim;
    kv->group = c.n_heads / c.n_kv_heads;
    kv->max_blocks = c.max_blocks_per_seq ? std::min(c.max_blocks_per_seq, kv->n_blocks) : kv->n_blocks;
    if (kv->max_blocks == 0) kv->max_blocks = 1;
    if ((uint64_t)c.max_seqs * kv->max_blocks > 0x7FFFFFFFull) {
        delete kv;
        return LT_E_ARG;
    }
    // 16-bit units of one block (all heads, K and V): f16 tiles of 2*16*D
    // values, or Q8_0 tiles of 34*D bytes.
    kv->q8 = c.kv_format == LT_KV_Q8_0;
    kv->block_elems = (size_t)c.n_kv_heads * (kv->q8 ? 17 : 2 * kBlock) * c.head_dim;
    kv->layer_elems = (size_t)kv->n_blocks * kv->block_elems;
    kv->blocks.resize(c.max_seqs);
    kv->lens.assign(c.max_seqs, 0);
    kv->refs.assign(kv->n_blocks, 0);
    kv->free_list.resize(kv->n_blocks);
    for (uint32_t i = 0; i < kv->n_blocks; ++i) kv->free_list[i] = (int32_t)(kv->n_blocks - 1 - i);  // kv.rs:45
    kv->free_run = kv->n_blocks;
    kv->owner_seq.assign(kv->n_blocks, -1);
    kv->owner_idx.assign(kv->n_blocks, -1);
    kv->ever_shared.assign(kv->n_blocks, 0);
    kv->dirty_from.assign(c.max_seqs, kClean);
    kv->fold_mark.assign(c.max_seqs, 0);
    kv->fold_pos.assign(c.max_seqs, 0);

    if (c.device >= 0) {
        kv->dev = true;
        kv->mark_src.assign(kv->n_blocks, 0);
        kv->mark_dst.assign(kv->n_blocks, 0);
        kv->dev_shadow.assign((size_t)c.max_seqs * kv->max_blocks, 0);  // tables are zeroed below
        DeviceGuard g(c.device);
        lt_status rc = LT_OK;
        auto ck = [&](cudaError_t e, const char* what) {
            if (e != cudaSuccess && rc == LT_OK) rc = fail(kv, LT_E_CUDA, "%s: %s", what, cudaGetErrorString(e));
        };
        if (!g.ok) ck(cudaErrorInvalidDevice, "cudaSetDevice");
        const size_t pool_bytes = (size_t)c.n_layers * kv->layer_elems * 2;
        // Partial slots: a warp's first piece may be part of a split sequence.
        const int max_warps = std::max(ltkv::attend_warps(c.device, (int)kv->group, (int)c.head_dim, 1, kv->q8),
                                       ltkv::attend_warps(c.device, (int)kv->group, (int)c.head_dim, 0, kv->q8));
        if (max_warps <= 0) ck(cudaErrorInvalidDevice, "attend_warps");
        kv->ws_slots = (size_t)std::max(max_warps, 0);  // one partial slot per warp
        const size_t gd = (size_t)kv->group * c.head_dim;
        if (rc == LT_OK) ck(cudaMalloc(&kv->d_pool, std::max<size_t>(pool_bytes, 16)), "cudaMalloc(pool)");
        if (rc == LT_OK) ck(cudaMemset(kv->d_pool, 0, std::max<size_t>(pool_bytes, 16)), "cudaMemset(pool)");
        const size_t tbytes = (size_t)c.max_seqs * kv->max_blocks * 4;
        if (rc == LT_OK) ck(cudaMalloc(&kv->d_tables, tbytes), "cudaMalloc(tables)");
        if (rc == LT_OK) ck(cudaMemset(kv->d_tables, 0, tbytes), "cudaMemset(tables)");
        // Two sets: the warps' partials and the group partials of the two-level merge.
        if (rc == LT_OK) ck(cudaMalloc(&kv->d_part_o, 2 * kv->ws_slots * gd * sizeof(float)), "cudaMalloc(partials)");
        if (rc == LT_OK)
            ck(cudaMalloc(&kv->d_part_ml, 2 * kv->ws_slots * kv->group * 2 * sizeof(float)), "cudaMalloc(partials)");
        if (rc == LT_OK) ck(cudaMalloc(&kv->d_flags, 2 * kv->ws_slots * sizeof(uint32_t) + 4), "cudaMalloc(flags)");
        if (rc == LT_OK) ck(cudaMemset(kv->d_flags, 0, 2 * kv->ws_slots * sizeof(uint32_t) + 4), "cudaMemset(flags)");
        kv->pre_cap = std::min<uint32_t>(c.max_batch, kCascadeMaxTokens);
        const size_t pre_rows = (size_t)kv->pre_cap * c.n_heads * ltkv::kPreMaxSplits;
        if (rc == LT_OK) ck(cudaDeviceGetAttribute(&kv->sm_count, cudaDevAttrMultiProcessorCount, c.device),
                            "cudaDeviceGetAttribute");
        if (rc == LT_OK) ck(cudaMalloc(&kv->d_pre_o, pre_rows * c.head_dim * sizeof(float) + 16), "cudaMalloc(prefix)");
        if (rc == LT_OK) ck(cudaMalloc(&kv->d_pre_ml, pre_rows * 2 * sizeof(float) + 16), "cudaMalloc(prefix)");
        if (rc == LT_OK) ck(cudaMalloc(&kv->d_err, sizeof(int32_t)), "cudaMalloc(err)");
        if (rc == LT_OK) ck(cudaMemset(kv->d_err, 0, sizeof(int32_t)), "cudaMemset(err)");
        kv->slot_bytes = std::max<size_t>(1u << 20, sizeof(ltkv::TokenDesc) * (size_t)c.max_batch + 64);
        for (auto& s : kv->slots) {
            if (rc != LT_OK) break;
            ck(cudaHostAlloc(&s.host, kv->slot_bytes, cudaHostAllocDefault), "cudaHostAlloc(staging)");
            if (rc == LT_OK) ck(cudaMalloc(&s.dev, kv->slot_bytes), "cudaMalloc(staging)");
            if (rc == LT_OK) ck(cudaEventCreateWithFlags(&s.ev, cudaEventDisableTiming), "cudaEventCreate");
        }
        if (rc == LT_OK) ck(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
        if (rc != LT_OK) {
            free_device(kv);
            delete kv;
            return rc;
        }
    }
    *out = kv;
    return LT_OK;
}

void lt_kv_destroy(lt_kv* kv) {
    if (!kv) return;
    if (kv->dev) {
        DeviceGuard g(kv->cfg.device);
        cudaDeviceSynchronize();
        free_device(kv);
    }
    delete kv;
}

const char* lt_kv_last_error(const lt_kv* kv) { return kv ? kv->err.c_str() : "null handle"; }

uint32_t lt_kv_capacity(const lt_kv* kv) { return kv ? kv->n_blocks * kBlock : 0; }

uint64_t lt_kv_bytes(const lt_kv* kv) { return kv ? (uint64_t)kv->cfg.n_layers * kv->layer_elems * 2 : 0; }

uint32_t lt_kv_len(const lt_kv* kv, uint32_t seq) { return kv && seq < kv->cfg.max_seqs ? kv->lens[seq] : 0; }

uint32_t lt_kv_free_blocks(const lt_kv* kv) { return kv ? (uint32_t)kv->free_list.size() : 0; }

uint32_t lt_kv_n_blocks(const lt_kv* kv) { return kv ? kv->n_blocks : 0; }

lt_status lt_kv_append(lt_kv* kv, const uint32_t* seq, const uint32_t* pos, uint32_t n, int32_t* block_out,
                       int32_t* slot_out, uint32_t* n_done, void* stream) {
    ltkv::NvtxRange nv("lt_kv_append");
    if (!kv) return LT_E_ARG;
    DeviceGuard g(kv->dev ? kv->cfg.device : -1);
    uint32_t i = 0;
    lt_status rc = LT_OK;
    for (; i < n; ++i) {
        rc = append_one(kv, seq[i], pos[i], &block_out[i], &slot_out[i], static_cast<cudaStream_t>(stream));
        if (rc) break;
    }
    if (n_done) *n_done = i;
    return rc;
}

lt_status lt_kv_write(lt_kv* kv, uint32_t layer, const int32_t* block, const int32_t* slot, uint32_t n,
                      const void* k, const void* v, lt_dtype dtype, void* stream) {
    ltkv::NvtxRange nv("lt_kv_write");
    if (!kv) return LT_E_ARG;
    lt_status rc = check_dtypes(kv, {&dtype});
    if (rc || (rc = require_device(kv))) return rc;
    if (layer >= kv->cfg.n_layers) return fail(kv, LT_E_ARG, "layer %u out of range", layer);
    if ((rc = check_cells(kv, block, slot, n))) return rc;
    DeviceGuard g(kv->cfg.device);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if ((rc = flush(kv, st))) return rc;
    if (n == 0) return LT_OK;
    kv->cells_tmp.resize(n);
    for (uint32_t i = 0; i < n; ++i) kv->cells_tmp[i] = make_int2(block[i], slot[i]);
    const void* d_cells = nullptr;
    int s = -1;
    if ((rc = upload(kv, kv->cells_cache, kv->cells_tmp.data(), n * sizeof(int2), st, &d_cells, &s))) return rc;
    cudaEvent_t ev_end = nullptr;
    if (kv->profiling) {  // the kernel alone: after the cells' upload
        if ((rc = prof_begin(kv, kv->prof_write, st, &ev_end))) return rc;
        kv->write_rows += n;
        kv->write_in_bytes += (uint64_t)n * 2 * kv->cfg.n_kv_heads * kv->cfg.head_dim * (dtype == LT_F32 ? 4 : 2);
    }
    LT_CUDA(kv, ltkv::launch_write(kv->d_pool + (size_t)layer * kv->layer_elems, static_cast<const int2*>(d_cells),
                                   (int)n, (int)kv->cfg.n_kv_heads, (int)kv->cfg.head_dim, k, v, dtype == LT_F32, kv->q8,
                                   st));
    if (ev_end) LT_CUDA(kv, cudaEventRecord(ev_end, st));
    kv->launches++;
    return mark_slot_use(kv, s, st);
}

}  // extern "C"

namespace {

lt_status attend_entry(lt_kv* kv, uint32_t layer, const void* q, lt_dtype q_dtype, const uint32_t* seq,
                       const uint32_t* pos, uint32_t n, void* out, lt_dtype out_dtype, float scale, void* stream,
                       bool gather) {
    if (!kv) return LT_E_ARG;
    lt_status rc = require_device(kv);
    if (rc) return rc;
    if (layer >= kv->cfg.n_layers) return fail(kv, LT_E_ARG, "layer %u out of range", layer);
    if ((rc = check_tokens(kv, seq, pos, n))) return rc;
    DeviceGuard g(kv->cfg.device);
    return attend_impl(kv, layer, q, q_dtype, seq, pos, n, out, out_dtype, scale, nullptr, nullptr, LT_F32, false,
                       static_cast<cudaStream_t>(stream), gather);
}

lt_status write_attend_entry(lt_kv* kv, uint32_t layer, const int32_t* block, const int32_t* slot, const void* k,
                             const void* v, lt_dtype kv_dtype, const void* q, lt_dtype q_dtype, const uint32_t* seq,
                             const uint32_t* pos, uint32_t n, void* out, lt_dtype out_dtype, float scale,
                             void* stream, bool gather) {
    if (!kv) return LT_E_ARG;
    lt_status rc = require_device(kv);
    if (rc) return rc;
    if (layer >= kv->cfg.n_layers) return fail(kv, LT_E_ARG, "layer %u out of range", layer);
    if ((rc = check_tokens(kv, seq, pos, n))) return rc;
    if ((rc = check_cells(kv, block, slot, n))) return rc;
    // One kernel is only equivalent to write-then-attend when every token's
    // new row is the only new row its attention reads: one token per
    // sequence, written to its own sequence's last cell, in a block no other
    // sequence references.
    bool fusable = true;
    for (uint32_t i = 0; i < n && fusable; ++i) {
        const auto& bl = kv->blocks[seq[i]];
        if (pos[i] + 1 != kv->lens[seq[i]] || bl[pos[i] / kBlock] != block[i] ||
            (int32_t)(pos[i] % kBlock) != slot[i] || kv->refs[block[i]] != 1)
            fusable = false;
    }
    if (fusable && n > 1) {
        std::vector<uint32_t> sorted(seq, seq + n);
        std::sort(sorted.begin(), sorted.end());
        fusable = std::adjacent_find(sorted.begin(), sorted.end()) == sorted.end();
    }
    if (!fusable) {
        if ((rc = lt_kv_write(kv, layer, block, slot, n, k, v, kv_dtype, stream))) return rc;
        return attend_entry(kv, layer, q, q_dtype, seq, pos, n, out, out_dtype, scale, stream, gather);
    }
    DeviceGuard g(kv->cfg.device);
    return attend_impl(kv, layer, q, q_dtype, seq, pos, n, out, out_dtype, scale, k, v, kv_dtype, true,
                       static_cast<cudaStream_t>(stream), gather);
}

}  // namespace

extern "C" {

lt_status lt_kv_attend(lt_kv* kv, uint32_t layer, const void* q, lt_dtype q_dtype, const uint32_t* seq,
                       const uint32_t* pos, uint32_t n, void* out, lt_dtype out_dtype, float scale, void* stream) {
    ltkv::NvtxRange nv("lt_kv_attend");
    if (!kv) return LT_E_ARG;
    if (lt_status rc = check_dtypes(kv, {&q_dtype, &out_dtype})) return rc;
    return attend_entry(kv, layer, q, q_dtype, seq, pos, n, out, out_dtype, scale, stream, false);
}

lt_status lt_kv_write_attend(lt_kv* kv, uint32_t layer, const int32_t* block, const int32_t* slot, const void* k,
                             const void* v, lt_dtype kv_dtype, const void* q, lt_dtype q_dtype, const uint32_t* seq,
                             const uint32_t* pos, uint32_t n, void* out, lt_dtype out_dtype, float scale,
                             void* stream) {
    ltkv::NvtxRange nv("lt_kv_write_attend");
    if (!kv) return LT_E_ARG;
    if (lt_status rc = check_dtypes(kv, {&kv_dtype, &q_dtype, &out_dtype})) return rc;
    return write_attend_entry(kv, layer, block, slot, k, v, kv_dtype, q, q_dtype, seq, pos, n, out, out_dtype, scale,
                              stream, false);
}

lt_status lt_kv_attend_gather(lt_kv* kv, uint32_t layer, const void* q, lt_dtype q_dtype, const uint32_t* seq,
                              const uint32_t* pos, uint32_t n, void* out, lt_dtype out_dtype, float scale,
                              void* stream) {
    ltkv::NvtxRange nv("lt_kv_attend_gather");
    if (!kv) return LT_E_ARG;
    if (lt_status rc = check_dtypes(kv, {&q_dtype, &out_dtype})) return rc;
    return attend_entry(kv, layer, q, q_dtype, seq, pos, n, out, out_dtype, scale, stream, true);
}

lt_status lt_kv_write_attend_gather(lt_kv* kv, uint32_t layer, const int32_t* block, const int32_t* slot,
                                    const void* k, const void* v, lt_dtype kv_dtype, const void* q, lt_dtype q_dtype,
                                    const uint32_t* seq, const uint32_t* pos, uint32_t n, void* out,
                                    lt_dtype out_dtype, float scale, void* stream) {
    ltkv::NvtxRange nv("lt_kv_write_attend_gather");
    if (!kv) return LT_E_ARG;
    if (lt_status rc = check_dtypes(kv, {&kv_dtype, &q_dtype, &out_dtype})) return rc;
    return write_attend_entry(kv, layer, block, slot, k, v, kv_dtype, q, q_dtype, seq, pos, n, out, out_dtype, scale,
                              stream, true);
}

lt_status lt_kv_peer_export(lt_kv* kv, int rank, int nranks, uint32_t max_tokens, void* ipc_handle_out) {
    if (!kv || !ipc_handle_out) return LT_E_ARG;
    lt_status rc = require_device(kv);
    if (rc) return rc;
    if (nranks < 1 || nranks > ltkv::kMaxPeers || rank < 0 || rank >= nranks || max_tokens == 0)
        return fail(kv, LT_E_ARG, "peer_export: rank %d of %d (at most %d ranks), max_tokens %u", rank, nranks,
                    ltkv::kMaxPeers, max_tokens);
    DeviceGuard g(kv->cfg.device);
    PeerGather& pg = kv->peer;
    peer_unmap(kv);
    LT_CUDA(kv, cudaDeviceSynchronize());
    cudaFree(pg.d_buf);
    pg = PeerGather{};
    const size_t half = ((size_t)max_tokens * nranks * kv->cfg.n_heads * kv->cfg.head_dim * 4 + 255) & ~(size_t)255;
    LT_CUDA(kv, cudaMalloc(&pg.d_buf, kPeerHeaderBytes + 2 * half));
    // Flags and the done counter start at zero before any peer can see the buffer.
    LT_CUDA(kv, cudaMemset(pg.d_buf, 0, kPeerHeaderBytes));
    LT_CUDA(kv, cudaDeviceSynchronize());
    cudaIpcMemHandle_t h;
    LT_CUDA(kv, cudaIpcGetMemHandle(&h, pg.d_buf));
    std::memcpy(ipc_handle_out, &h, sizeof h);
    pg.rank = rank;
    pg.nranks = nranks;
    pg.max_tokens = max_tokens;
    pg.half_bytes = half;
    pg.fresh = true;
    return LT_OK;
}

lt_status lt_kv_peer_import(lt_kv* kv, const void* ipc_handles) {
    if (!kv || !ipc_handles) return LT_E_ARG;
    PeerGather& pg = kv->peer;
    if (!pg.d_buf) return fail(kv, LT_E_ARG, "peer_import before peer_export");
    if (!pg.fresh)
        return fail(kv, LT_E_ARG, "peer_import needs a new peer_export on every rank (the buffers hold the flags of "
                                  "earlier calls)");
    DeviceGuard g(kv->cfg.device);
    peer_unmap(kv);
    const unsigned char* hs = static_cast<const unsigned char*>(ipc_handles);
    for (int r = 0; r < pg.nranks; ++r) {
        if (r == pg.rank) {
            pg.base[r] = pg.d_buf;
            continue;
        }
        cudaIpcMemHandle_t h;
        std::memcpy(&h, hs + (size_t)r * LT_IPC_HANDLE_BYTES, sizeof h);
        void* ptr = nullptr;
        const cudaError_t e = cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            peer_unmap(kv);
            return fail(kv, LT_E_CUDA, "cudaIpcOpenMemHandle(rank %d): %s", r, cudaGetErrorString(e));
        }
        pg.base[r] = static_cast<unsigned char*>(ptr);
        pg.mapped[r] = true;
    }
    pg.epoch = 0;  // export zeroed every rank's flags
    pg.ready = true;
    pg.fresh = false;
    return LT_OK;
}

lt_status lt_kv_peer_close(lt_kv* kv) {
    if (!kv) return LT_E_ARG;
    if (!kv->dev) return LT_OK;
    DeviceGuard g(kv->cfg.device);
    LT_CUDA(kv, cudaDeviceSynchronize());
    peer_unmap(kv);
    return LT_OK;
}

void lt_kv_truncate(lt_kv* kv, uint32_t seq, uint32_t from) {
    if (kv) truncate_impl(kv, seq, from);
}

void lt_kv_share(lt_kv* kv, uint32_t src, uint32_t dst, uint32_t len) {  // kv.rs:172-183
    if (!kv) return;
    truncate_impl(kv, dst, 0);
    if (src >= kv->cfg.max_seqs || dst >= kv->cfg.max_seqs) return;
    const uint32_t slen = kv->lens[src];
    if (slen == 0) return;  // unknown source (share(x, x, _) lands here as well)
    len = std::min(len, slen);
    const size_t nb = (len + kBlock - 1) / kBlock;
    for (size_t i = 0; i < nb; ++i) {
        kv->refs[kv->blocks[src][i]] += 1;
        kv->ever_shared[kv->blocks[src][i]] = 1;
    }
    if (len > 0) {
        kv->blocks[dst].assign(kv->blocks[src].begin(), kv->blocks[src].begin() + nb);
        kv->lens[dst] = len;
        mark_dirty(kv, dst, 0);
    }
}

lt_status lt_kv_compact(lt_kv* kv, uint32_t* n_moved, void* stream) {
    ltkv::NvtxRange nv("lt_kv_compact");
    if (!kv) return LT_E_ARG;
    DeviceGuard g(kv->dev ? kv->cfg.device : -1);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    lt_status rc = flush(kv, st);
    if (rc) return rc;
    // The rule: the j-th lowest free block receives the j-th highest live
    // block while it is lower (so live blocks end up as [0, n_live)).  Free
    // ids at or above W = nb - free_run were untouched since the last
    // compaction; only the free ids below W (released since) need sorting,
    // and the live ids are found by walking down from W - 1.
    const uint32_t nb = kv->n_blocks;
    const size_t r = std::min(kv->free_run, kv->free_list.size());
    const int32_t W = (int32_t)(nb - r);
    std::vector<int32_t>& low = kv->cmp_low;
    low.assign(kv->free_list.begin() + (std::ptrdiff_t)r, kv->free_list.end());
    std::sort(low.begin(), low.end());
    std::vector<int2> moves;
    {
        int32_t cand = W - 1;     // next live candidate from the top
        size_t top = low.size();  // low[top - 1] is the highest free id not yet passed by cand
        for (size_t j = 0; j < low.size(); ++j) {
            while (cand >= 0 && top > 0 && low[top - 1] == cand) {
                --cand;
                --top;
            }
            if (cand < 0 || low[j] >= cand) break;
            const int32_t src = cand--, dst = low[j];
            moves.push_back(make_int2(src, dst));
            kv->refs[dst] = kv->refs[src];
            kv->refs[src] = 0;
            kv->owner_seq[dst] = kv->owner_seq[src];
            kv->owner_idx[dst] = kv->owner_idx[src];
            kv->ever_shared[dst] = kv->ever_shared[src];
        }
    }
    std::vector<int2> tw;
    auto remap_entry = [&](uint32_t s, size_t i, int32_t nbk) {
        kv->blocks[s][i] = nbk;
        const size_t idx = (size_t)s * kv->max_blocks + i;
        if (kv->dev && kv->dev_shadow[idx] != nbk) {
            kv->dev_shadow[idx] = nbk;
            tw.push_back(make_int2((int)idx, nbk));
        }
    };
    // The owner entry is used only when it still holds the moved block (it
    // always does for a block never shared; checked anyway).
    bool shared = false;
    for (const int2& m : moves) {
        const int32_t s = kv->owner_seq[m.y], i = kv->owner_idx[m.y];
        shared |= kv->ever_shared[m.y] != 0 || s < 0 || (uint32_t)s >= kv->cfg.max_seqs || i < 0 ||
                  (size_t)i >= kv->blocks[(size_t)s].size() || kv->blocks[(size_t)s][(size_t)i] != m.x;
    }
    if (!shared) {
        // each moved block sits in exactly one table entry: the one that took it
        for (const int2& m : moves) {
            const int32_t s = kv->owner_seq[m.y], i = kv->owner_idx[m.y];
            remap_entry((uint32_t)s, (size_t)i, m.y);
        }
    } else if (!moves.empty()) {
        std::vector<int32_t> remap(nb);
        for (uint32_t b = 0; b < nb; ++b) remap[b] = (int32_t)b;
        for (const int2& m : moves) remap[m.x] = m.y;
        for (uint32_t s = 0; s < kv->cfg.max_seqs; ++s) {
            auto& bl = kv->blocks[s];
            for (size_t i = 0; i < bl.size(); ++i)
                if (remap[bl[i]] != bl[i]) remap_entry(s, i, remap[bl[i]]);
        }
    }
    // Free blocks are now exactly [n_live, nb): the list nb-1, ..., n_live,
    // whose first r entries are already in place.
    const size_t F = kv->free_list.size();
    for (size_t i = r; i < F; ++i) kv->free_list[i] = (int32_t)(nb - 1 - i);
    kv->free_run = F;
    if (n_moved) *n_moved = (uint32_t)moves.size();
    if (kv->dev && (!moves.empty() || !tw.empty())) {
        rc = run_plan(kv, moves, tw, st);
        kv->epoch++;
    }
    return rc;
}

lt_status lt_kv_flush(lt_kv* kv, void* stream) {
    if (!kv) return LT_E_ARG;
    DeviceGuard g(kv->dev ? kv->cfg.device : -1);
    return flush(kv, static_cast<cudaStream_t>(stream));
}

lt_status lt_kv_rows(lt_kv* kv, uint32_t layer, uint32_t seq, uint32_t n, void* k_out, void* v_out, void* stream) {
    if (!kv) return LT_E_ARG;
    lt_status rc = require_device(kv);
    if (rc) return rc;
    if (layer >= kv->cfg.n_layers || seq >= kv->cfg.max_seqs || n > kv->lens[seq])
        return fail(kv, LT_E_ARG, "rows(layer %u, seq %u, n %u) out of range", layer, seq, n);
    DeviceGuard g(kv->cfg.device);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if ((rc = flush(kv, st))) return rc;
    LT_CUDA(kv, ltkv::launch_rows(kv->d_pool + (size_t)layer * kv->layer_elems,
                                  kv->d_tables + (size_t)seq * kv->max_blocks, (int)n, (int)kv->cfg.n_kv_heads,
                                  (int)kv->cfg.head_dim, static_cast<uint16_t*>(k_out), static_cast<uint16_t*>(v_out),
                                  kv->q8, (int)kv->n_blocks, kv->d_err, st));
    kv->launches++;
    return LT_OK;
}

lt_status lt_kv_check(lt_kv* kv, void* stream) {
    if (!kv) return LT_E_ARG;
    if (!kv->dev) return LT_OK;
    DeviceGuard g(kv->cfg.device);
    LT_CUDA(kv, cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
    int32_t flag = 0;
    LT_CUDA(kv, cudaMemcpy(&flag, kv->d_err, sizeof flag, cudaMemcpyDeviceToHost));
    if (flag) {
        LT_CUDA(kv, cudaMemset(kv->d_err, 0, sizeof(int32_t)));
        LT_CUDA(kv, cudaDeviceSynchronize());
        if (flag & ltkv::kErrBounds)
            return fail(kv, LT_E_BOUNDS, "a device block table named a block outside the pool (access redirected "
                                         "to block 0); the affected outputs are invalid");
        return fail(kv, LT_E_TIMEOUT, "a bounded device wait timed out; the affected outputs are invalid");
    }
    return LT_OK;
}

lt_status lt_kv_selftest_wait(lt_kv* kv, uint32_t limit_us, void* stream) {
    if (!kv) return LT_E_ARG;
    lt_status rc = require_device(kv);
    if (rc) return rc;
    if (limit_us == 0 || limit_us > 2000000u)
        return fail(kv, LT_E_ARG, "selftest_wait: limit %u us outside [1, 2000000]", limit_us);
    DeviceGuard g(kv->cfg.device);
    LT_CUDA(kv, ltkv::launch_wait_selftest((uint64_t)limit_us * 1000u, kv->d_err, static_cast<cudaStream_t>(stream)));
    kv->launches++;
    return LT_OK;
}

uint32_t lt_kv_build_features(void) { return ltkv::bounds_checked_build() ? LT_FEATURE_BOUNDS_CHECK : 0u; }

uint32_t lt_kv_seq_blocks(const lt_kv* kv, uint32_t seq, int32_t* out, uint32_t cap) {
    if (!kv || seq >= kv->cfg.max_seqs) return 0;
    const auto& bl = kv->blocks[seq];
    for (size_t i = 0; i < bl.size() && i < cap; ++i) out[i] = bl[i];
    return (uint32_t)bl.size();
}

uint32_t lt_kv_refs(const lt_kv* kv, uint32_t* out, uint32_t cap) {
    if (!kv) return 0;
    for (uint32_t b = 0; b < kv->n_blocks && b < cap; ++b) out[b] = kv->refs[b];
    return kv->n_blocks;
}

uint32_t lt_kv_free_list(const lt_kv* kv, int32_t* out, uint32_t cap) {
    if (!kv) return 0;
    for (size_t i = 0; i < kv->free_list.size() && i < cap; ++i) out[i] = kv->free_list[i];
    return (uint32_t)kv->free_list.size();
}

void* lt_kv_device_pool(const lt_kv* kv) { return kv ? kv->d_pool : nullptr; }

const int32_t* lt_kv_device_tables(const lt_kv* kv, uint32_t* max_blocks_per_seq) {
    if (!kv) return nullptr;
    if (max_blocks_per_seq) *max_blocks_per_seq = kv->max_blocks;
    return kv->d_tables;
}

lt_status lt_kv_read_pool(lt_kv* kv, uint32_t layer, uint32_t block0, uint32_t count, void* out) {
    if (!kv) return LT_E_ARG;
    lt_status rc = require_device(kv);
    if (rc) return rc;
    if (layer >= kv->cfg.n_layers || block0 > kv->n_blocks || count > kv->n_blocks - block0)
        return fail(kv, LT_E_ARG, "read_pool(layer %u, blocks %u+%u) out of range", layer, block0, count);
    DeviceGuard g(kv->cfg.device);
    LT_CUDA(kv, cudaDeviceSynchronize());
    LT_CUDA(kv, cudaMemcpy(out, kv->d_pool + (size_t)layer * kv->layer_elems + (size_t)block0 * kv->block_elems,
                           (size_t)count * kv->block_elems * 2, cudaMemcpyDeviceToHost));
    return LT_OK;
}

lt_status lt_kv_profile(lt_kv* kv, int enable) {
    if (!kv) return LT_E_ARG;
    lt_status rc = require_device(kv);
    if (rc) return rc;
    DeviceGuard g(kv->cfg.device);
    for (ProfRing* r : {&kv->prof_attn, &kv->prof_plan, &kv->prof_write}) {
        if (r->ev.empty()) {
            r->ev.resize(2 * kProfPairs);
            for (auto& e : r->ev) LT_CUDA(kv, cudaEventCreate(&e));
        }
        if ((rc = prof_drain(kv, *r, kProfPairs))) return rc;
        r->ms = 0.0;
        r->count = 0;
    }
    kv->plan_blocks = kv->plan_entries = 0;
    kv->write_rows = kv->write_in_bytes = 0;
    kv->profiling = enable != 0;
    return LT_OK;
}

lt_status lt_kv_profile_read(lt_kv* kv, double* total_ms, uint64_t* launches) {
    if (!kv) return LT_E_ARG;
    DeviceGuard g(kv->dev ? kv->cfg.device : -1);
    lt_status rc = prof_drain(kv, kv->prof_attn, kProfPairs);
    if (rc) return rc;
    if (total_ms) *total_ms = kv->prof_attn.ms;
    if (launches) *launches = kv->prof_attn.count;
    return LT_OK;
}

lt_status lt_kv_profile_read_plan(lt_kv* kv, double* total_ms, uint64_t* launches, uint64_t* copied_blocks,
                                  uint64_t* table_entries) {
    if (!kv) return LT_E_ARG;
    DeviceGuard g(kv->dev ? kv->cfg.device : -1);
    lt_status rc = prof_drain(kv, kv->prof_plan, kProfPairs);
    if (rc) return rc;
    if (total_ms) *total_ms = kv->prof_plan.ms;
    if (launches) *launches = kv->prof_plan.count;
    if (copied_blocks) *copied_blocks = kv->plan_blocks;
    if (table_entries) *table_entries = kv->plan_entries;
    return LT_OK;
}

lt_status lt_kv_profile_read_write(lt_kv* kv, double* total_ms, uint64_t* launches, uint64_t* rows,
                                   uint64_t* in_bytes) {
    if (!kv) return LT_E_ARG;
    DeviceGuard g(kv->dev ? kv->cfg.device : -1);
    lt_status rc = prof_drain(kv, kv->prof_write, kProfPairs);
    if (rc) return rc;
    if (total_ms) *total_ms = kv->prof_write.ms;
    if (launches) *launches = kv->prof_write.count;
    if (rows) *rows = kv->write_rows;
    if (in_bytes) *in_bytes = kv->write_in_bytes;
    return LT_OK;
}

lt_status lt_kv_set_cascade(lt_kv* kv, uint32_t min_group_tokens) {
    if (!kv) return LT_E_ARG;
    kv->cascade_min_tokens = min_group_tokens;
    return LT_OK;
}

uint64_t lt_kv_cascade_launches(const lt_kv* kv) { return kv ? kv->cascade_launches : 0; }

lt_status lt_kv_set_min_tiles_per_warp(lt_kv* kv, uint32_t tiles) {
    if (!kv || tiles == 0) return LT_E_ARG;
    kv->min_tiles_per_warp = tiles;
    return LT_OK;
}

uint64_t lt_kv_launch_count(const lt_kv* kv) { return kv ? kv->launches : 0; }

}  // extern "C"
