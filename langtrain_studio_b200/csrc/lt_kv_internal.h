// Internal interface between the host bookkeeping (lt_kv.cpp) and the sm_100a
// kernels (lt_kv_kernels.cu).  Not part of the C ABI.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace ltkv {

constexpr int kBlock = 16;           // tokens per block (kv.rs:13)
constexpr int kMaxGroup = 8;         // q heads per KV head the attention kernel handles

// One warp's share of one (token, KV head): blocks [b0, b1) of the token's
// sequence, which has length pos + 1.  slot >= 0: the (token, head) is split
// across warps and this piece writes partial `slot`; slot < 0: the piece
// covers the whole sequence and writes the output.  last_block >= 0: the
// piece holds the token's last block (physical id last_block) and writes
// the token's new K/V row there (fused append).
struct Piece {
    int32_t tok, h, seq, pos;
    int32_t b0, b1;
    int32_t slot;
    int32_t last_block;
};

struct AttnParams {
    const uint16_t* pool_layer;  // pool + layer offset
    uint16_t* pool_layer_w;      // same, for the fused append
    const int32_t* tables;       // [max_seqs][max_blocks]
    int32_t max_blocks;
    const Piece* pieces;         // grouped by warp
    const int32_t* warp_off;     // warp w owns pieces [warp_off[w], warp_off[w+1])
    int32_t n_warps;
    const int4* combine;         // (tok, h, n_pieces, first_slot) per split (token, head)
    int32_t n_combine;
    int32_t n_kv_heads;
    int32_t group;
    const void* q;               // [n][n_heads*D]
    int32_t q_f32;
    void* out;                   // [n][n_heads*D]
    int32_t out_f32;
    float scale_log2;            // scale * log2(e)
    float* part_o;               // [slots][group][D]
    float* part_ml;              // [slots][group][2]
    int32_t* err;                // device error flag
    const void* k_new;           // fused append: new K/V rows [n][n_kv_heads*D]
    const void* v_new;
    int32_t kv_f32;
};

// Warps of one attention launch on `device` (all resident at once), or 0.
int attend_warps(int device, int group, int head_dim, int q_f32);
cudaError_t launch_attend(const AttnParams& p, int head_dim, cudaStream_t s);
// Kernel launches made by launch_attend(p).
int attend_launches(const AttnParams& p);

cudaError_t launch_write(uint16_t* pool_layer, const int2* cells, int n, int n_kv_heads, int head_dim,
                         const void* k, const void* v, int in_f32, cudaStream_t s);

// Block copies (copy-on-write and compaction moves) and table scatter.
// copies: (src, dst) pairs; tw: (flat table index, value) pairs.
cudaError_t launch_apply_plan(uint16_t* pool, size_t layer_stride_elems, size_t block_elems, int n_layers,
                              const int2* copies, int n_copies, int32_t* tables, const int2* tw, int n_tw,
                              cudaStream_t s);

cudaError_t launch_rows(const uint16_t* pool_layer, const int32_t* table_row, int n, int n_kv_heads,
                        int head_dim, uint16_t* k_out, uint16_t* v_out, cudaStream_t s);

}  // namespace ltkv
