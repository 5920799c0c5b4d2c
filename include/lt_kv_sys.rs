//! lt_kv_sys.rs -- the Rust FFI binding of liblt_kv.so, as the reference engine's
//! native crate would add it (engine/crates/native/src/lt_kv_sys.rs).
//!
//! Every declaration mirrors include/lt_kv.h, lt_llama.h, lt_sched.h and
//! lt_prefix.h: the same symbols, argument order, integer widths and struct
//! layouts.  Statuses are returned as i32 (lt_status), dtypes and formats are
//! passed as i32/u32 (lt_dtype / lt_kv_format).  The engine's KvCache
//! (engine/crates/native/src/kv.rs) becomes a thin owner of `*mut LtKv` whose
//! Drop calls lt_kv_destroy; `build.rs` links liblt_kv.so with
//! `cargo:rustc-link-search` pointing at the directory that holds it.
#![allow(non_camel_case_types, dead_code)]

use std::ffi::{c_char, c_void, CStr};

// ---- the KV cache: include/lt_kv.h ----------------------------------------

#[repr(C)]
pub struct LtKvConfig {
    pub n_layers: u32, pub n_kv_heads: u32, pub head_dim: u32, pub n_heads: u32,
    pub n_tokens: u32, pub max_seqs: u32, pub max_batch: u32, pub max_blocks_per_seq: u32,
    pub device: i32,
    pub kv_format: u32,  // LT_KV_F16 (0, the reference's cache) or LT_KV_Q8_0 (1)
}
#[repr(C)] pub struct LtKv { _p: [u8; 0] }
pub const LT_F32: i32 = 0;
pub const LT_F16: i32 = 1;
pub const LT_KV_F16: u32 = 0;
pub const LT_KV_Q8_0: u32 = 1;
pub const LT_E_FULL: i32 = 1;
pub const LT_E_NONCONTIG: i32 = 2;
pub const LT_E_ARG: i32 = 3;
pub const LT_E_TIMEOUT: i32 = 6;
pub const LT_E_UNSUPPORTED: i32 = 7;
pub const LT_E_SCRATCH: i32 = 8;
pub const LT_E_BOUNDS: i32 = 9;
pub const LT_FEATURE_BOUNDS_CHECK: u32 = 1;

#[link(name = "lt_kv")]
extern "C" {
    pub fn lt_kv_create(cfg: *const LtKvConfig, out: *mut *mut LtKv) -> i32;
    pub fn lt_kv_destroy(kv: *mut LtKv);
    pub fn lt_kv_last_error(kv: *const LtKv) -> *const c_char;
    pub fn lt_kv_capacity(kv: *const LtKv) -> u32;
    pub fn lt_kv_bytes(kv: *const LtKv) -> u64;
    pub fn lt_kv_len(kv: *const LtKv, seq: u32) -> u32;
    pub fn lt_kv_free_blocks(kv: *const LtKv) -> u32;
    pub fn lt_kv_append(kv: *mut LtKv, seq: *const u32, pos: *const u32, n: u32,
                        block: *mut i32, slot: *mut i32, n_done: *mut u32, stream: *mut c_void) -> i32;
    pub fn lt_kv_write(kv: *mut LtKv, layer: u32, block: *const i32, slot: *const i32, n: u32,
                       k: *const c_void, v: *const c_void, dtype: i32, stream: *mut c_void) -> i32;
    pub fn lt_kv_attend(kv: *mut LtKv, layer: u32, q: *const c_void, q_dtype: i32,
                        seq: *const u32, pos: *const u32, n: u32, out: *mut c_void, out_dtype: i32,
                        scale: f32, stream: *mut c_void) -> i32;
    // write + attention of the same tokens, one kernel when the batch allows it
    pub fn lt_kv_write_attend(kv: *mut LtKv, layer: u32, block: *const i32, slot: *const i32,
                              k: *const c_void, v: *const c_void, kv_dtype: i32,
                              q: *const c_void, q_dtype: i32, seq: *const u32, pos: *const u32,
                              n: u32, out: *mut c_void, out_dtype: i32, scale: f32,
                              stream: *mut c_void) -> i32;
    pub fn lt_kv_truncate(kv: *mut LtKv, seq: u32, from: u32);
    pub fn lt_kv_share(kv: *mut LtKv, src: u32, dst: u32, len: u32);
    pub fn lt_kv_compact(kv: *mut LtKv, moved: *mut u32, stream: *mut c_void) -> i32;
    // pending table updates and copies to the device now
    pub fn lt_kv_flush(kv: *mut LtKv, stream: *mut c_void) -> i32;
    // synchronises `stream`; reads and clears the device error flag (LT_E_TIMEOUT, LT_E_BOUNDS)
    pub fn lt_kv_check(kv: *mut LtKv, stream: *mut c_void) -> i32;
    pub fn lt_kv_selftest_wait(kv: *mut LtKv, limit_us: u32, stream: *mut c_void) -> i32;
    pub fn lt_kv_build_features() -> u32;
    pub fn lt_kv_set_cascade(kv: *mut LtKv, min_group_tokens: u32) -> i32;
    pub fn lt_kv_set_min_tiles_per_warp(kv: *mut LtKv, tiles: u32) -> i32;
}

pub fn check(kv: *const LtKv, rc: i32) -> anyhow::Result<()> {
    if rc == 0 { return Ok(()); }
    let msg = unsafe { CStr::from_ptr(lt_kv_last_error(kv)) }.to_string_lossy().into_owned();
    anyhow::bail!(msg)
}

// ---- KV-head sharding across GPUs: NCCL gather, or the gather fused into attention ----

extern "C" {
    pub fn lt_kv_nccl_unique_id(id_out: *mut u8 /* 128 bytes */) -> i32;
    pub fn lt_kv_nccl_init(comm_out: *mut *mut c_void, nranks: i32, id: *const u8, rank: i32,
                           device: i32) -> i32;
    pub fn lt_kv_nccl_destroy(comm: *mut c_void);
    pub fn lt_kv_gather_heads(kv: *mut LtKv, local: *const c_void, gathered: *mut c_void,
                              out: *mut c_void, n: u32, dtype: i32, comm: *mut c_void, nranks: i32,
                              stream: *mut c_void) -> i32;
}

extern "C" {
    pub fn lt_kv_peer_export(kv: *mut LtKv, rank: i32, nranks: i32, max_tokens: u32,
                             ipc_handle_out: *mut u8 /* 64 bytes */) -> i32;
    pub fn lt_kv_peer_import(kv: *mut LtKv, ipc_handles: *const u8 /* nranks * 64 */) -> i32;
    pub fn lt_kv_peer_close(kv: *mut LtKv) -> i32;
    pub fn lt_kv_attend_gather(kv: *mut LtKv, layer: u32, q: *const c_void, q_dtype: i32,
                               seq: *const u32, pos: *const u32, n: u32, out: *mut c_void,
                               out_dtype: i32, scale: f32, stream: *mut c_void) -> i32;
    pub fn lt_kv_write_attend_gather(kv: *mut LtKv, layer: u32, block: *const i32, slot: *const i32,
                                     k: *const c_void, v: *const c_void, kv_dtype: i32,
                                     q: *const c_void, q_dtype: i32, seq: *const u32, pos: *const u32,
                                     n: u32, out: *mut c_void, out_dtype: i32, scale: f32,
                                     stream: *mut c_void) -> i32;
}

// ---- attention for hosts that cannot allocate device memory ----

pub const LT_NOALLOC_MAX_TOKENS: u32 = 1024;
extern "C" {
    pub fn lt_paged_attend_noalloc(pool_layer: *const c_void, kv_format: u32, n_blocks: u32,
                                   n_kv_heads: u32, head_dim: u32, n_heads: u32,
                                   tables: *const i32, n_table_rows: u32, max_blocks_per_seq: u32,
                                   seq_host: *const u32, pos_host: *const u32, n: u32,
                                   q: *const c_void, q_dtype: i32, out: *mut c_void, out_dtype: i32,
                                   scale: f32, stream: *mut c_void) -> i32;
    // synchronises `stream`; reads and clears the error word of every call since the last check
    pub fn lt_paged_attend_noalloc_check(stream: *mut c_void) -> i32;
}

// ---- the model step around the cache: include/lt_llama.h ----

#[repr(C)]
pub struct LtLlamaConfig {
    pub n_layers: u32, pub dim: u32, pub n_heads: u32, pub n_kv_heads: u32, pub head_dim: u32,
    pub ffn_dim: u32, pub vocab: u32, pub rope_dim: u32, pub rope_neox: i32, pub eps: f32,
    pub rope_base: f32, pub max_batch: u32, pub device: i32,
}
#[repr(C)] pub struct LtLlama { _p: [u8; 0] }

#[link(name = "lt_kv")]
extern "C" {
    pub fn lt_llama_create(cfg: *const LtLlamaConfig, out: *mut *mut LtLlama) -> i32;
    pub fn lt_llama_destroy(m: *mut LtLlama);
    pub fn lt_llama_last_error(m: *const LtLlama) -> *const c_char;
    // which: 0 token_embd, 1 output, 2 output_norm, 3 attn_norm, 4 ffn_norm, 5 attn_q,
    // 6 attn_k, 7 attn_v, 8 attn_output, 9 ffn_gate, 10 ffn_up, 11 ffn_down (model.rs:236-262);
    // data = the tensor's GGUF bytes (Q8_0 blocks or F32)
    pub fn lt_llama_set_tensor(m: *mut LtLlama, which: i32, layer: u32, data: *const c_void,
                               bytes: usize) -> i32;
    pub fn lt_llama_forward(m: *mut LtLlama, kv: *mut LtKv, tokens: *const i32, seqs: *const u32,
                            pos: *const u32, n: u32, want: *const u32, n_want: u32,
                            logits_dev: *mut f32, stream: *mut c_void) -> i32;
    pub fn lt_llama_step_greedy(m: *mut LtLlama, kv: *mut LtKv, tokens: *const i32,
                                seqs: *const u32, pos: *const u32, n: u32, want: *const u32,
                                n_want: u32, next: *mut i32, stream: *mut c_void) -> i32;
}

// ---- the scheduler's KV policy: include/lt_sched.h ----

#[repr(C)]
pub struct LtSchedConfig {
    pub n_slots: u32, pub decode_headroom: u32, pub prefill_chunk: u32,
    pub compact: i32,  // 1: lt_kv_compact after every step
    pub data: i32,     // 1: write K/V rows and attend; 0: bookkeeping only
}
#[repr(C)]
pub struct LtSchedStats {
    pub steps: u64, pub admitted: u64, pub finished: u64, pub evicted: u64, pub preempted: u64,
    pub decode_tokens: u64, pub prefill_tokens: u64, pub moved_blocks: u64,
    pub running: u32, pub queued: u32,
    pub attended_positions: u64, pub copies: u64, pub prompt_tokens: u64, pub cached_tokens: u64,
}
#[repr(C)] pub struct LtSched { _p: [u8; 0] }

extern "C" {
    pub fn lt_sched_create(kv: *mut LtKv, cfg: *const LtSchedConfig, out: *mut *mut LtSched) -> i32;
    pub fn lt_sched_destroy(s: *mut LtSched);
    pub fn lt_sched_last_error(s: *const LtSched) -> *const c_char;
    pub fn lt_sched_submit(s: *mut LtSched, prompt_len: u32, out_len: u32) -> i32;
    pub fn lt_sched_submit_tokens(s: *mut LtSched, tokens: *const i32, n: u32, out_len: u32,
                                  adapter: i32) -> i32;
    pub fn lt_sched_step(s: *mut LtSched, kv_src: *const c_void, src_rows: u32, q_src: *const c_void,
                         out: *mut c_void, n_decode: *mut u32, stream: *mut c_void) -> i32;
    pub fn lt_sched_get_stats(s: *const LtSched, out: *mut LtSchedStats) -> i32;
}

// ---- the slot-level prefix cache: include/lt_prefix.h ----

#[repr(C)]
pub struct LtPlacement { pub slot: u32, pub reuse: u32, pub copy_src: i32, pub copy_len: u32 }
#[repr(C)] pub struct LtSlotCache { _p: [u8; 0] }
pub const LT_NO_ADAPTER: i32 = -1;

extern "C" {
    pub fn lt_slot_cache_create(n_slots: u32, out: *mut *mut LtSlotCache) -> i32;
    pub fn lt_slot_cache_destroy(c: *mut LtSlotCache);
    // 0 and *out, or LT_E_FULL (1) when every slot is busy (the reference's None)
    pub fn lt_slot_cache_place(c: *const LtSlotCache, prompt: *const i32, n: u32, adapter: i32,
                               out: *mut LtPlacement) -> i32;
    pub fn lt_slot_cache_acquire(c: *mut LtSlotCache, p: *const LtPlacement, prompt: *const i32, n: u32,
                                 adapter: i32) -> i32;
    pub fn lt_slot_cache_release(c: *mut LtSlotCache, slot: u32, tokens: *const i32, n: u32) -> i32;
    pub fn lt_slot_cache_evict_lru(c: *mut LtSlotCache) -> i32;  // -1: none
    pub fn lt_slot_cache_idle_cells(c: *const LtSlotCache) -> u64;
}
