// Internal interface between the host bookkeeping (lt_kv.cpp) and the sm_100a
// kernels (lt_kv_kernels.cu).  Not part of the C ABI.
#pragma once
#include <cuda_runtime.h>
#include <nvtx3/nvToolsExt.h>
#include <stdint.h>
#include <string.h>

#include "lt_kv.h"

namespace ltkv {

// Whether an lt_dtype argument names LT_F32 or LT_F16.  A C caller may pass
// any 32-bit value; reading an out-of-range value through the C++ enum type
// is undefined, so the argument's bytes are read instead.
static_assert(sizeof(lt_dtype) == sizeof(int32_t), "lt_dtype is passed as a 32-bit int");
inline bool dtype_valid(const lt_dtype& d) {
    int32_t v;
    memcpy(&v, &d, sizeof v);
    return v == (int32_t)LT_F32 || v == (int32_t)LT_F16;
}

constexpr int kBlock = 16;           // tokens per block (kv.rs:13)
constexpr int kMaxGroup = 8;         // q heads per KV head the attention kernel handles

// Bits of the device error word (lt_kv_check turns them into statuses).
constexpr int32_t kErrTimeout = 1;   // a bounded wait gave up -> LT_E_TIMEOUT
constexpr int32_t kErrBounds = 2;    // a table entry named no block of the pool -> LT_E_BOUNDS
                                     // (tested by LT_BOUNDS_CHECK builds, and by every build
                                     // for tables the caller owns)

// Per-token input of one attention launch: the token's sequence, its
// position (it attends over blocks [0, pos/16]), the physical id of its last
// block, the tile prefix P = sum of (pos_j/16 + 1 - skip_j) over tokens
// j < i, and skip: its first `skip` blocks are a shared prefix whose
// attention the prefix pass already computed (partial in pre_o / pre_ml).
struct TokenDesc {
    int32_t seq, pos, last_block, prefix, skip;
};

constexpr int kInlineTokens = 512;  // tokens passed inside the kernel parameters
constexpr int kMaxPeers = 8;        // ranks of a head-sharded peer gather
constexpr int kMergeGroup = 8;      // partials a group leader combines (two-level merge)

struct AttnParams {
    const uint16_t* pool_layer;  // pool + layer offset
    uint16_t* pool_layer_w;      // same, for the fused append
    int32_t* tables;             // [max_seqs][max_blocks]; each token's last entry is (re)written
    int32_t max_blocks;
    int32_t n_blocks;            // blocks in the pool, for LT_BOUNDS_CHECK builds (0: not checked)
    int32_t check_ids;           // test every block id read from `tables` against n_blocks in every
                                 // build (caller-owned tables, lt_paged_attend_noalloc)
    const TokenDesc* toks;       // n_tok entries in global memory, or null: use inl
    int32_t n_tok;
    int32_t tiles_per_head;      // prefix of n_tok (total blocks over the tokens)
    int32_t n_warps;             // stream-K ranges; tile total = tiles_per_head * n_kv_heads
    int32_t n_kv_heads;
    int32_t group;
    const void* q;               // [n][n_heads*D]
    int32_t q_f32;
    void* out;                   // [n][n_heads*D]
    int32_t out_f32;
    float scale_log2;            // scale * log2(e)
    float* part_o;               // [n_warps][group][D]: partial of warp w's first piece
    float* part_ml;              // [n_warps][group][2]
    uint32_t* flags;             // [n_warps]: warp w stores `epoch` once its range is done
    // Two-level merge of (token, head)s cut into more than kMergeGroup + 1
    // pieces: the helper warps' partials are first combined in groups of
    // kMergeGroup by each group's first warp (into slot w of part2_*, flag
    // flags2[w]); the merging warp then reads one partial per group.  Null:
    // one level (the merging warp reads every helper's partial).
    float* part2_o;
    float* part2_ml;
    uint32_t* flags2;
    uint32_t epoch;              // distinct per launch on a flags array
    int32_t* err;                // device error flag
    const void* k_new;           // fused append: new K/V rows [n][n_kv_heads*D], or null
    const void* v_new;
    int32_t kv_f32;
    const float* pre_o;          // [pre_splits][rows][D]: shared-prefix partial O (tokens with skip > 0),
    const float* pre_ml;         // [pre_splits][rows][2]: its (m, l); row = (token*n_kv_heads + h)*group + g
    int32_t pre_splits;          // partials per row (the prefix blocks split over that many CTAs)
    int64_t pre_split_rows;      // rows between split slabs
    int32_t q8;                  // pool tiles are Q8_0 (lt_kv.h LT_KV_Q8_0); no prefix partials then
    // Head-sharded gather over NVLink (lt_kv_attend_gather).  With n_peers > 0
    // every output row goes, instead of to `out`, to this rank's gather half
    // gather_out at row tok*(n_peers*n_heads) + peer_rank*n_heads + head, and
    // the (token, head) that completes the count publishes peer_epoch into
    // every rank's flag for this rank (peer_flag[r]); the ranks then read
    // each other's rows (launch_gather_wait_copy).
    int32_t n_peers;
    int32_t peer_rank;
    uint32_t peer_epoch;
    uint32_t* done_count;        // this rank's count of stored (token, head)s (zero between launches)
    void* gather_out;
    uint32_t* peer_flag[kMaxPeers];
    TokenDesc inl[kInlineTokens];
};

// Shared-prefix (cascade) pass: one CTA per item attends up to
// prefix_tokens_per_cta(group) tokens of one prefix group (128 query rows on
// the tensor cores) to the group's first n_blocks blocks for one KV head,
// each K/V tile staged once for all of them, and writes (m, l, O) partials
// that the stream-K launch folds into the tokens' outputs.
struct PrefixItem {
    int32_t root_seq;  // a member whose table row holds the shared blocks
    int32_t blk0;      // this item's part of the shared blocks: [blk0, blk1)
    int32_t blk1;
    int32_t split;     // which partial slab it writes
    int32_t head;      // KV head
    int32_t tok_off;   // first of the item's tokens in the token list
    int32_t n_tok;     // tokens of this item
};
constexpr int kPreMaxSplits = 4;
struct PrefixParams {
    const uint16_t* pool_layer;
    const int32_t* tables;
    int32_t max_blocks;
    int32_t n_blocks;  // blocks in the pool, for LT_BOUNDS_CHECK builds (0: not checked)
    const PrefixItem* items;
    const int32_t* tok_list;  // token indices of the call (into q, pre_o, pre_ml)
    const int32_t* tok_lim;   // parallel to tok_list: the token attends blocks [0, tok_lim) here
    int32_t n_kv_heads, group;
    const void* q;
    int32_t q_f32;
    float scale_log2;
    float* pre_o;
    float* pre_ml;
    int64_t split_rows;  // rows between split slabs of pre_o / pre_ml
    int32_t* err;
};
// Tokens one prefix CTA covers: 128 query rows / group.
inline int prefix_tokens_per_cta(int group) { return 128 / group; }
cudaError_t launch_prefix(const PrefixParams& p, int n_items, int head_dim, cudaStream_t s);

// Warps of one attention launch on `device` (all resident at once), or 0.
int attend_warps(int device, int group, int head_dim, int q_f32, int q8);
cudaError_t launch_attend(const AttnParams& p, int head_dim, cudaStream_t s);
// Kernel launches made by launch_attend(p).
int attend_launches(const AttnParams& p);

// Head-sharded output assembly: gathered [nranks][n][row bytes] ->
// out [n][nranks][row bytes] (row = one token's local heads).
cudaError_t launch_gather_permute(const void* gathered, void* out, int nranks, uint32_t n, size_t row_bytes,
                                  cudaStream_t s);

cudaError_t launch_write(uint16_t* pool_layer, const int2* cells, int n, int n_kv_heads, int head_dim,
                         const void* k, const void* v, int in_f32, int q8, cudaStream_t s);

// Block copies (copy-on-write and compaction moves) and table scatter.
// copies: (src, dst) pairs; tw: (flat table index, value) pairs.  n_blocks
// and n_entries (pool blocks, table entries) bound the indices in
// LT_BOUNDS_CHECK builds, which report a bad one through err.
cudaError_t launch_apply_plan(uint16_t* pool, size_t layer_stride_elems, size_t block_elems, int n_layers,
                              const int2* copies, int n_copies, int32_t* tables, const int2* tw, int n_tw,
                              int n_blocks, long long n_entries, int32_t* err, cudaStream_t s);

cudaError_t launch_rows(const uint16_t* pool_layer, const int32_t* table_row, int n, int n_kv_heads,
                        int head_dim, uint16_t* k_out, uint16_t* v_out, int q8, int n_blocks, int32_t* err,
                        cudaStream_t s);

// One warp waits, through the kernels' bounded flag wait with a limit of
// limit_ns, for a device word that nothing sets, then raises kErrTimeout in
// err: the failure path of every bounded wait, made to run out on purpose.
cudaError_t launch_wait_selftest(uint64_t limit_ns, int32_t* err, cudaStream_t s);
// Whether this build checks table entries on the device (LT_BOUNDS_CHECK).
bool bounds_checked_build();

// Peer gather, receiving side: wait (bounded, system-scope acquire) until
// every rank's flag in `flags` has reached `epoch`, then assemble `out`
// [n][nranks][slice_bytes]: slice r of every token comes from rank r's
// gather half srcs[r] (the same layout; over NVLink for the other ranks).
// A wait that gives up raises kErrTimeout and copies nothing.
cudaError_t launch_gather_wait_copy(const uint32_t* flags, int nranks, uint32_t epoch, void* const* srcs, void* out,
                                    uint32_t n, size_t slice_bytes, int32_t* err, cudaStream_t s);

}  // namespace ltkv

// Accessors of the opaque handle for the other translation units.
struct lt_kv;
struct lt_kv_config;
namespace ltkv {
size_t local_out_row_bytes(const lt_kv* kv, int dtype);  // n_heads*head_dim*elem of this handle
int handle_device(const lt_kv* kv);
const lt_kv_config* handle_config(const lt_kv* kv);
void count_launch(lt_kv* kv);
// Host bookkeeping reads for the scheduler driver: entry idx of seq's block
// list, and a block's refcount.
int32_t seq_block_at(const lt_kv* kv, uint32_t seq, uint32_t idx);
uint32_t block_refs(const lt_kv* kv, int32_t block);
}  // namespace ltkv

namespace ltkv {
// NVTX range over one C ABI call, named after it, so a timeline from a
// profiler shows the host bookkeeping and launches of each call.  With no
// profiler attached the push/pop cost one test of a null pointer each.
struct NvtxRange {
    explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
    ~NvtxRange() { nvtxRangePop(); }
    NvtxRange(const NvtxRange&) = delete;
    NvtxRange& operator=(const NvtxRange&) = delete;
};
}  // namespace ltkv
