/*
 * lt_kv.h -- C ABI of the B200 paged KV-cache path.
 *
 * Drop-in replacement for the reference engine's KV cache API
 * (engine/crates/native/src/kv.rs, struct KvCache) and the attention closure
 * of Model::forward (engine/crates/native/src/model.rs:431-476), exposed as
 * plain `extern "C"` functions over pointers and sizes so that the Rust host
 * (NativeBackend, engine/crates/native/src/lib.rs:45-198) can bind it through
 * a thin FFI module.  No torch or C++ types cross this boundary.
 *
 * Model.  One handle owns one paged cache on one CUDA device: the K/V block
 * pool in HBM, the device copy of every sequence's block table, and the host
 * bookkeeping (refcounts, LIFO free list, per-sequence block lists) that the
 * reference keeps in KvCache.  The bookkeeping runs on the host thread and
 * is bit-identical to the reference's; the data work (copy-on-write block
 * copies, K/V append, attention, compaction) runs as sm_100a kernels on the
 * stream the caller passes.
 *
 * Threading.  A handle is not thread-safe (KvCache is owned by the single
 * engine thread, engine/crates/engine/src/scheduler.rs:103-119).  Issue all
 * kernel-launching calls of one handle on one stream, or synchronise when
 * switching streams.  Bookkeeping-only calls (truncate, share) take no
 * stream; their device-side effect is applied, in call order, right before
 * the next kernel-launching call.
 *
 * Pointers.  Arguments named *_host are host memory; `k`, `v`, `q`, `out`
 * and the pointers of lt_kv_rows are device memory.  seq / pos / block /
 * slot arrays are host memory (they are the reference's Vec arguments).
 *
 * Errors.  Every fallible call returns an lt_status; the message of the last
 * error is kept per handle (lt_kv_last_error).
 */
#ifndef LT_KV_H
#define LT_KV_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Tokens per block: kv.rs:13 (BLOCK = 16). */
#define LT_KV_BLOCK 16

typedef enum lt_status {
    LT_OK = 0,
    LT_E_FULL = 1,        /* "KV cache full" (kv.rs:71)                         */
    LT_E_NONCONTIG = 2,   /* "position not contiguous" (kv.rs:87-92)            */
    LT_E_ARG = 3,         /* invalid argument (id out of range, bad size, ...)  */
    LT_E_CUDA = 4,        /* a CUDA runtime call failed                         */
    LT_E_NCCL = 5,        /* an NCCL call failed                                */
    LT_E_TIMEOUT = 6,     /* a bounded device wait gave up (kernel error flag)  */
    LT_E_UNSUPPORTED = 7, /* shape outside what the kernels implement           */
    LT_E_SCRATCH = 8,     /* request too large for lt_paged_attend_noalloc's
                             fixed scratch (see LT_NOALLOC_*)                   */
    LT_E_BOUNDS = 9       /* a device block table named a block outside the
                             pool (only LT_FEATURE_BOUNDS_CHECK builds test)    */
} lt_status;

/* Element type of a device array argument.  Any other value is refused with
 * LT_E_ARG before the call does anything. */
typedef enum lt_dtype {
    LT_F32 = 0,
    LT_F16 = 1
} lt_dtype;

/* Storage format of the cached K/V rows (lt_kv_config.kv_format).
 *   LT_KV_F16   the reference's cache (kv.rs:20-21): f16 per value.
 *   LT_KV_Q8_0  each row cut into 32-value groups, stored as the Q8_0 block
 *               of the reference's GGUF reader (quant.rs:254-275: one f16
 *               scale d + 32 int8) -- the "q8_0" KV type the engine's
 *               llama.cpp profile selects (engine/crates/engine/src/
 *               hardware.rs:173) and its roadmap asks of the native cache
 *               (engine/README.md:115).  A group x is quantised by the
 *               engine's own int8 quantiser (quant.rs:785-795): d =
 *               max|x| / 127, q = round(x / d) half away from zero, saturating
 *               to int8 (q = 0 when d = 0); d is kept as f16 (round to
 *               nearest even) and a value reads back as q * d.  0.53 of the
 *               f16 bytes per cached token. */
typedef enum lt_kv_format {
    LT_KV_F16 = 0,
    LT_KV_Q8_0 = 1
} lt_kv_format;

typedef struct lt_kv lt_kv;

/* Creation parameters.  KvCache::new(n_layers, kv_dim, n_tokens) (kv.rs:35-48)
 * with kv_dim = n_kv_heads * head_dim, plus the sizes the device buffers are
 * planned for, so no call after lt_kv_create allocates device memory. */
typedef struct lt_kv_config {
    uint32_t n_layers;
    uint32_t n_kv_heads;        /* KV heads held by this handle                  */
    uint32_t head_dim;          /* 64 or 128                                     */
    uint32_t n_heads;           /* query heads for those KV heads; n_heads /
                                   n_kv_heads = GQA group (model.rs:401), <= 8   */
    uint32_t n_tokens;          /* pool capacity in tokens (rounded up to blocks) */
    uint32_t max_seqs;          /* sequence ids are in [0, max_seqs): seq == slot
                                   (engine/crates/engine/src/backend.rs:19-20)   */
    uint32_t max_batch;         /* most tokens per append / write / attend call  */
    uint32_t max_blocks_per_seq;/* 0: n_blocks (never limits)                    */
    int32_t device;             /* CUDA ordinal; -1 = bookkeeping only (no GPU)  */
    uint32_t kv_format;         /* lt_kv_format; 0 (f16) when zero-initialised    */
} lt_kv_config;

/* KvCache::new (kv.rs:35-48): zero-filled pool, free list (0..n_blocks).rev()
 * so the first allocation returns block 0. */
lt_status lt_kv_create(const lt_kv_config* cfg, lt_kv** out);
/* Drop (frees device and host memory; synchronises the device first). */
void lt_kv_destroy(lt_kv* kv);
/* Message of the last failed call on this handle ("" if none). */
const char* lt_kv_last_error(const lt_kv* kv);

/* The accessors below return 0 for a null handle. */
/* KvCache::capacity (kv.rs:50-52): n_blocks * 16 tokens. Backend::n_ctx. */
uint32_t lt_kv_capacity(const lt_kv* kv);
/* KvCache::bytes (kv.rs:54-56): K + V pool bytes (LT_KV_Q8_0: values and
 * scales). */
uint64_t lt_kv_bytes(const lt_kv* kv);
/* KvCache::len (kv.rs:58-60): 0 for an unknown sequence. */
uint32_t lt_kv_len(const lt_kv* kv, uint32_t seq);
/* KvCache::free_blocks (kv.rs:185-187). */
uint32_t lt_kv_free_blocks(const lt_kv* kv);

/* KvCache::append (kv.rs:85-121) for a batch, as Model::forward claims every
 * batch token before any layer runs (model.rs:380-383).  For token i:
 * pos[i] must equal the sequence's length (else LT_E_NONCONTIG); a new block
 * is taken at slot 0 (else LT_E_FULL); a write into a shared last block
 * copies it first (copy-on-write, all layers, K and V).  Returns the (block,
 * slot) cell of each token.  Stops at the first error: *n_done tokens were
 * claimed and stay claimed, the failing sequence is unchanged -- exactly the
 * reference's `collect::<Result<Vec<_>>>()`.  The copy-on-write copies are
 * enqueued on `stream`. */
lt_status lt_kv_append(lt_kv* kv, const uint32_t* seq_host, const uint32_t* pos_host, uint32_t n,
                       int32_t* block_host, int32_t* slot_host, uint32_t* n_done, void* stream);

/* KvCache::write (kv.rs:123-131) for n cells of one layer, as the per-layer
 * loop of Model::forward does (model.rs:414-429).  k and v are device arrays
 * [n][n_kv_heads * head_dim] of `dtype`.  LT_KV_F16: f32 is rounded to f16
 * with round-to-nearest-even (bit-identical to half::f16::from_f32), f16 is
 * stored unchanged.  LT_KV_Q8_0: each 32-value group of the given values
 * (f16 widened exactly) is quantised as lt_kv_format describes. */
lt_status lt_kv_write(lt_kv* kv, uint32_t layer, const int32_t* block_host, const int32_t* slot_host,
                      uint32_t n, const void* k, const void* v, lt_dtype dtype, void* stream);

/* Attention closure of Model::forward (model.rs:431-476) for n tokens of one
 * layer: token i attends over positions [0, pos[i]] of sequence seq[i]
 * through its block table, GQA with group n_heads / n_kv_heads.
 * q and out are device arrays [n][n_heads * head_dim] (q: f32 or f16; out:
 * f32 or f16), head h*group+g reads KV head h.  scale is the reference's
 * 1/sqrt(head_dim) (model.rs:402).  Softmax and accumulation are f32. */
lt_status lt_kv_attend(lt_kv* kv, uint32_t layer, const void* q, lt_dtype q_dtype,
                       const uint32_t* seq_host, const uint32_t* pos_host, uint32_t n, void* out,
                       lt_dtype out_dtype, float scale, void* stream);

/* write + attend in one kernel launch (the K/V rows of each token are
 * written by the attention work item that covers them, then attended to).
 * Same results as lt_kv_write followed by lt_kv_attend with the same
 * arguments.  k/v dtype: `kv_dtype`. */
lt_status lt_kv_write_attend(lt_kv* kv, uint32_t layer, const int32_t* block_host,
                             const int32_t* slot_host, const void* k, const void* v, lt_dtype kv_dtype,
                             const void* q, lt_dtype q_dtype, const uint32_t* seq_host,
                             const uint32_t* pos_host, uint32_t n, void* out, lt_dtype out_dtype,
                             float scale, void* stream);

/* KvCache::truncate (kv.rs:153-169): drop positions [from, len) of seq,
 * releasing whole blocks past ceil(from/16) in ascending order; no-op for an
 * unknown seq or from >= len.  Backend::kv_remove (native/src/lib.rs:192). */
void lt_kv_truncate(lt_kv* kv, uint32_t seq, uint32_t from);

/* KvCache::share (kv.rs:172-183): truncate(dst, 0), then let dst start with
 * the first min(len, len(src)) tokens of src by sharing its blocks (refcount
 * + 1 each).  Backend::kv_copy (native/src/lib.rs:196). */
void lt_kv_share(lt_kv* kv, uint32_t src, uint32_t dst, uint32_t len);

/* Compaction (no counterpart in the reference, which never moves blocks):
 * free ids ascending are paired with live ids descending while free < live;
 * each such live block is moved (all layers, K and V) onto the free id, its
 * refcount moves with it and every block-table entry is remapped, on host
 * and device alike; the free list is rebuilt descending so the next
 * allocation returns the lowest free id.  Every sequence's rows() are
 * byte-identical before and after.  *n_moved (optional) = blocks moved. */
lt_status lt_kv_compact(lt_kv* kv, uint32_t* n_moved, void* stream);

/* Apply every pending bookkeeping change to the device (block tables,
 * pending copies) on `stream` now. */
lt_status lt_kv_flush(lt_kv* kv, void* stream);

/* KvCache::rows (kv.rs:135-150): gather rows [0, n) of seq in `layer` into
 * device arrays k_out / v_out [n][n_kv_heads * head_dim] (f16, reference
 * row layout).  LT_KV_Q8_0: each value is q * d rounded to f16 (nearest
 * even). */
lt_status lt_kv_rows(lt_kv* kv, uint32_t layer, uint32_t seq, uint32_t n, void* k_out, void* v_out,
                     void* stream);

/* Reads (and clears) the device error flag set by bounded waits in the
 * kernels; synchronises `stream`.  LT_OK or LT_E_TIMEOUT / LT_E_CUDA, or
 * LT_E_BOUNDS from a bounds-checked build. */
lt_status lt_kv_check(lt_kv* kv, void* stream);

/* ---- failure paths and debug builds ---------------------------------------
 * No counterpart in the reference, whose path has no device code.  Every
 * device wait in these kernels (pipeline barriers, the stream-K merge's
 * neighbour flags) is bounded: when its limit runs out the kernel raises the
 * handle's error flag and returns instead of hanging, and lt_kv_check reports
 * LT_E_TIMEOUT. */

/* Failure-path self-test: one warp waits, through the same bounded flag
 * wait as the attention merge, for a device word that nothing ever sets,
 * with a limit of limit_us microseconds (1 .. 2,000,000).  When the limit
 * runs out the error flag is raised; the next lt_kv_check returns
 * LT_E_TIMEOUT and clears it, and the handle stays usable.  Asynchronous on
 * `stream`. */
lt_status lt_kv_selftest_wait(lt_kv* kv, uint32_t limit_us, void* stream);

/* Build features of the loaded library.  LT_FEATURE_BOUNDS_CHECK: compiled
 * with -DLT_BOUNDS_CHECK (liblt_kv_checked.so): every block id the kernels
 * read from a device table is tested against the pool; a bad one raises
 * LT_E_BOUNDS at the next lt_kv_check and block 0 is read in its place. */
#define LT_FEATURE_BOUNDS_CHECK 1u
uint32_t lt_kv_build_features(void);

/* ---- introspection (parity checks, debugging) ---------------------------- */

/* Block ids of seq's table; returns the count, copies min(count, cap). */
uint32_t lt_kv_seq_blocks(const lt_kv* kv, uint32_t seq, int32_t* out_host, uint32_t cap);
/* Refcount of every block (n_blocks entries). */
uint32_t lt_kv_refs(const lt_kv* kv, uint32_t* out_host, uint32_t cap);
/* Free list, bottom of the stack first; returns its length. */
uint32_t lt_kv_free_list(const lt_kv* kv, int32_t* out_host, uint32_t cap);
uint32_t lt_kv_n_blocks(const lt_kv* kv);

/* Device pool layout, for tools that read it directly.
 * LT_KV_F16: f16 [layer][block][kv_head][2 (K, V)][head_dim/64][16 slots][64]:
 * each K or V part is head_dim/64 sub-tiles of 16 rows x 128 bytes, and
 * inside a sub-tile the 16-byte chunk c of row `slot` is stored at chunk
 * position (c ^ (slot & 7)) -- the 128-byte-swizzled layout of the
 * tensor-core operand descriptors, bank-conflict free for ldmatrix once
 * bulk-copied.
 * LT_KV_Q8_0: [layer][block][kv_head] tiles of 34*head_dim bytes, D =
 * head_dim, with the order within 16 of a 16-byte run
 * pos(i) = ((i & 7) >> 1) * 4 + ((i >> 3) << 1) + (i & 1):
 *   [0, 16D)    K int8, row-major [16 slots][D]: the 16-byte run that holds
 *               values 16k..16k+15 of slot s is run L = (s*D)/16 + k of the
 *               part, stored at byte 128*(L/8) + 16*((L%8) ^ ((L/8) & 7)),
 *               value 16k+i at byte pos(i) of the run;
 *   [16D, 32D)  V int8, transposed: 16 bytes per column d, slot s at byte
 *               16*d + pos(s);
 *   [32D, 33D)  K scales, f16 [D/32 groups][16]: group c of slot s at
 *               element 16*c + pos(s);
 *   [33D, 34D)  V scales, the same.
 * Returns the device base address. */
void* lt_kv_device_pool(const lt_kv* kv);
/* Device block tables: int32 [max_seqs][max_blocks_per_seq]. */
const int32_t* lt_kv_device_tables(const lt_kv* kv, uint32_t* max_blocks_per_seq);

/* Copy the raw device pool bytes of `layer`, blocks [block0, block0+count),
 * into host memory (layout of lt_kv_device_pool); synchronous.  For parity
 * checks of whole pools against the reference layout. */
lt_status lt_kv_read_pool(lt_kv* kv, uint32_t layer, uint32_t block0, uint32_t count, void* out_host);

/* Launch timing.  While enabled, CUDA events bracket every attention launch
 * (lt_kv_attend, lt_kv_write_attend), every plan launch (the kernel that
 * applies copy-on-write copies, compaction moves and block-table entries;
 * after the plan's upload) and every K/V write launch (lt_kv_write) on its
 * own stream; enabling resets the totals. */
lt_status lt_kv_profile(lt_kv* kv, int enable);
/* Total duration (ms) and count of the bracketed attention launches since
 * profiling was enabled; waits for the recorded events. */
lt_status lt_kv_profile_read(lt_kv* kv, double* total_ms, uint64_t* launches);
/* The same for the plan launches, with the block copies (copy-on-write and
 * compaction; each moves one block of every layer) and table entries they
 * applied.  New: the reference copies on the host (kv.rs:99-110). */
lt_status lt_kv_profile_read_plan(lt_kv* kv, double* total_ms, uint64_t* launches, uint64_t* copied_blocks,
                                  uint64_t* table_entries);
/* The same for the K/V write launches of lt_kv_write (KvCache::write,
 * kv.rs:123-131; the kernel alone, after the cells' upload), with the rows
 * written and the input bytes they read. */
lt_status lt_kv_profile_read_write(lt_kv* kv, double* total_ms, uint64_t* launches, uint64_t* rows,
                                   uint64_t* in_bytes);

/* Kernel launches made by this handle since creation (all kinds). */
uint64_t lt_kv_launch_count(const lt_kv* kv);

/* Attention launch sizing: each warp of the stream-K attention launch takes
 * at least `tiles` 16-position tiles (default 8), so small steps run on fewer
 * warps; large steps use every resident warp regardless.  Results do not
 * depend on it beyond f32 summation order of split merges. */
lt_status lt_kv_set_min_tiles_per_warp(lt_kv* kv, uint32_t tiles);

/* Shared-prefix (cascade) attention.  In an attention call, tokens whose
 * sequences begin with the same physical blocks (prefix sharing, kv.rs:172)
 * -- at least `min_group_tokens` of them, sharing at least 4 leading blocks
 * before every member's own last block -- have those blocks attended in one
 * extra launch that stages each shared K/V tile once for the whole group;
 * the decode launch then covers only each token's own blocks and folds the
 * prefix result in (online-softmax merge, f32).  Default 8; 0 turns it off.
 * Calls of more than 1024 tokens (or max_batch) never use it, nor does an
 * LT_KV_Q8_0 cache (its tiles are not tensor-core f16 operands). */
lt_status lt_kv_set_cascade(lt_kv* kv, uint32_t min_group_tokens);

/* Prefix-pass launches issued by this handle since creation. */
uint64_t lt_kv_cascade_launches(const lt_kv* kv);

/* ---- KV-head sharding across GPUs (NCCL) ---------------------------------- */
/* No counterpart in the reference, which runs one process.  For long
 * contexts the KV heads are split across ranks: rank r's handle holds KV
 * heads [r*hl, (r+1)*hl) of every sequence (n_kv_heads = hl, n_heads = hl*G),
 * every rank makes the same bookkeeping calls, and after each attention the
 * ranks' outputs are all-gathered.  NCCL is resolved at run time from
 * libnccl.so.2 (an already-loaded copy is reused); LT_E_NCCL if absent. */

/* ncclGetUniqueId into 128 bytes, to be shared with every rank. */
lt_status lt_kv_nccl_unique_id(void* id_out);
/* ncclCommInitRank on `device`; blocks until all nranks ranks join. */
lt_status lt_kv_nccl_init(void** comm_out, int nranks, const void* id, int rank, int device);
void lt_kv_nccl_destroy(void* comm);
/* Join the head-sharded attention outputs: `local` [n][n_heads*head_dim]
 * (this rank's heads, from lt_kv_attend / lt_kv_write_attend) is
 * all-gathered over `comm` into `gathered` [nranks][n][n_heads*head_dim] and
 * permuted into `out` [n][nranks*n_heads*head_dim] -- the layout of the
 * unsharded attention (head h*group+g of the full model).  Device buffers,
 * 16-byte aligned; ordered on `stream`. */
lt_status lt_kv_gather_heads(lt_kv* kv, const void* local, void* gathered, void* out, uint32_t n, lt_dtype dtype,
                             void* comm, int nranks, void* stream);

/* ---- KV-head sharding with the gather fused into attention (NVLink) ------
 * The same head-sharded decode without a collective launch: each rank's
 * attention kernel stores every output row straight into every rank's
 * gather buffer over NVLink (peer memory, CUDA IPC), and the launch's last
 * warp raises this rank's flag on every rank; one small kernel per rank then
 * waits (bounded) for all ranks' flags and copies the gathered rows to
 * `out`.  Replaces lt_kv_attend + lt_kv_gather_heads; no counterpart in the
 * reference (one process).  Set-up, on every rank:
 *   1. lt_kv_peer_export: allocate this rank's gather buffer (max_tokens
 *      tokens a call) and write its 64-byte CUDA IPC handle;
 *   2. exchange the handles between ranks (any host transport);
 *   3. lt_kv_peer_import with all nranks handles in rank order.
 * Every rank then makes the same sequence of *_gather calls (the gather
 * buffer alternates halves between calls, so a rank may run one call ahead).
 * A rank that misses a call leaves the others' waits to run out:
 * lt_kv_check then reports LT_E_TIMEOUT.  Tear-down: lt_kv_peer_close on
 * every rank, a host barrier, then lt_kv_destroy (which frees the buffer the
 * peers had mapped).  Each import follows a new export (LT_E_ARG otherwise):
 * the buffers keep the flags of earlier calls.  After LT_E_TIMEOUT the ranks'
 * call counts may differ; recover with lt_kv_peer_close on every rank, a
 * host barrier, and set-up steps 1-3 again. */
#define LT_IPC_HANDLE_BYTES 64
lt_status lt_kv_peer_export(lt_kv* kv, int rank, int nranks, uint32_t max_tokens, void* ipc_handle_out);
lt_status lt_kv_peer_import(lt_kv* kv, const void* ipc_handles /* nranks * LT_IPC_HANDLE_BYTES */);
lt_status lt_kv_peer_close(lt_kv* kv);
/* lt_kv_attend / lt_kv_write_attend of this rank's KV heads with the gather
 * fused in: `out` receives [n][nranks * n_heads * head_dim], the layout of
 * the unsharded attention (rank r's heads at [r * n_heads, (r+1) * n_heads)),
 * as lt_kv_gather_heads produces it.  n <= max_tokens. */
lt_status lt_kv_attend_gather(lt_kv* kv, uint32_t layer, const void* q, lt_dtype q_dtype, const uint32_t* seq,
                              const uint32_t* pos, uint32_t n, void* out, lt_dtype out_dtype, float scale,
                              void* stream);
lt_status lt_kv_write_attend_gather(lt_kv* kv, uint32_t layer, const int32_t* block, const int32_t* slot,
                                    const void* k, const void* v, lt_dtype kv_dtype, const void* q, lt_dtype q_dtype,
                                    const uint32_t* seq, const uint32_t* pos, uint32_t n, void* out,
                                    lt_dtype out_dtype, float scale, void* stream);

/* ---- allocation-free attention ------------------------------------------- */

/* No counterpart in the reference.  The same paged decode attention as
 * lt_kv_attend, for callers that cannot call cudaMalloc: hosts whose device
 * memory is wholly owned by their own allocator or fixed budget, and hosts
 * that cannot pay for cudaMalloc's possible device-wide synchronisation on
 * their step path.  The caller passes everything:
 *   - pool_layer: the K/V tiles of one layer in the lt_kv_device_pool layout
 *     (lt_kv_device_pool(kv) + layer * n_blocks * n_kv_heads * 2 * 16 *
 *     head_dim halves), 16-byte aligned, holding n_blocks blocks;
 *     kv_format states its format and must be LT_KV_F16 (LT_KV_Q8_0 pools
 *     are refused with LT_E_UNSUPPORTED);
 *   - tables: device block tables, int32 [n_table_rows][max_blocks_per_seq],
 *     4-byte aligned;
 *   - host seq/pos arrays, device q and out (16-byte aligned).
 * Every seq must be below n_table_rows and every pos below
 * 16 * max_blocks_per_seq (and below 2^31 - 16): anything else is refused
 * with LT_E_ARG before any work.  The block ids in entries [0, pos/16] of
 * each token's row are read on the device and tested against n_blocks; an
 * id outside the pool reads block 0 instead (that token's output is then
 * wrong) and raises LT_E_BOUNDS, reported by lt_paged_attend_noalloc_check.
 *
 * Nothing is allocated: the kernel's scratch (split-K partials and
 * range-done flags) lives in one static device array of
 * LT_NOALLOC_SCRATCH_BYTES that every GPU loading this library holds until
 * the process exits.
 *   - At most LT_NOALLOC_MAX_TOKENS tokens per call; larger requests return
 *     LT_E_SCRATCH before any work.  Calls of more than 512 tokens run as
 *     consecutive launches on `stream`.
 *   - The first call on a device looks up the array's address with that
 *     device current; make that first call before any stream capture.
 *   - All calls share the array and it keeps the last call's contents; each
 *     launch tags its flags with a fresh epoch and rewrites the partials it
 *     reads.  Calls that overlap on the GPU race: issue them in order on
 *     one stream.
 *   - The call does not synchronise.  Device-side failures of every call on
 *     the current device (a bounded wait that gave up, a block id past the
 *     pool) accumulate in the array's error word until
 *     lt_paged_attend_noalloc_check reads it. */
#define LT_NOALLOC_SCRATCH_BYTES (8u << 20)
#define LT_NOALLOC_MAX_TOKENS 1024u
lt_status lt_paged_attend_noalloc(const void* pool_layer, uint32_t kv_format, uint32_t n_blocks,
                                  uint32_t n_kv_heads, uint32_t head_dim, uint32_t n_heads,
                                  const int32_t* tables, uint32_t n_table_rows, uint32_t max_blocks_per_seq,
                                  const uint32_t* seq_host, const uint32_t* pos_host, uint32_t n,
                                  const void* q, lt_dtype q_dtype, void* out, lt_dtype out_dtype,
                                  float scale, void* stream);
/* No counterpart in the reference.  Synchronises `stream`, then reads and
 * clears the error word of lt_paged_attend_noalloc on the current device:
 * LT_OK when no call since the last check failed on the device,
 * LT_E_TIMEOUT when a bounded wait gave up (those calls' outputs are
 * invalid), else LT_E_BOUNDS (a table named a block outside the pool). */
lt_status lt_paged_attend_noalloc_check(void* stream);

#ifdef __cplusplus
}
#endif
#endif /* LT_KV_H */
