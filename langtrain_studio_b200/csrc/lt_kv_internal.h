// Internal interface between the host bookkeeping (lt_kv.cpp) and the sm_100a
// kernels (lt_kv_kernels.cu).  Not part of the C ABI.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace ltkv {

constexpr int kBlock = 16;           // tokens per block (kv.rs:13)
constexpr int kMaxGroup = 8;         // q heads per KV head the attention kernel handles

// One attention work item: token `tok` (index into q/out), sequence `seq`
// with length pos+1, blocks [chunk*cb, min((chunk+1)*cb, nb)) of its table.
// nchunks > 1 means the item writes a partial to slot part_base + chunk and
// the last item of (tok, head) to finish combines them.
struct WorkItem {
    int32_t tok;
    int32_t seq;
    int32_t pos;
    int32_t chunk;
    int32_t nchunks;
    int32_t part_base;
    int32_t cb;
    int32_t write_row;  // fused append: 1 if this item writes token tok's K/V row
};

struct AttnParams {
    const uint16_t* pool_layer;  // pool + layer offset
    const int32_t* tables;       // [max_seqs][max_blocks]
    int32_t max_blocks;
    const WorkItem* items;
    int32_t n_items;
    int32_t n_kv_heads;
    int32_t group;
    const void* q;               // [n][n_heads*D]
    int32_t q_f32;
    void* out;                   // [n][n_heads*D]
    int32_t out_f32;
    float scale_log2;            // scale * log2(e)
    float* part_o;               // [slots][n_kv_heads][group][D]
    float* part_ml;              // [slots][n_kv_heads][group][2]
    int32_t* counters;           // [max_batch][n_kv_heads]
    int32_t* err;                // device error flag
    // fused append (write_row items): new K/V rows [n][n_kv_heads*D]
    uint16_t* pool_layer_w;
    const void* k_new;
    const void* v_new;
    int32_t kv_f32;
    const int2* cells;           // (block, slot) per token
};

int attn_smem_bytes(int head_dim);
cudaError_t launch_attend(const AttnParams& p, int head_dim, cudaStream_t s);

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
