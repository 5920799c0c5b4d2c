// Internal interface of the persistent decode step (lt_llama_decode.cu):
// the whole of Model::forward (model.rs:366-518) for a small decode batch in
// one cooperative launch.  Not part of the C ABI.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace lldec {

// The Q8_0 matrices of one layer (int8 [rows][cols] + f16 scales
// [rows][cols/32]) and its two norm vectors.
enum { kQkv = 0, kO = 1, kGateUp = 2, kDown = 3 };
struct Layer {
    const int8_t* wq[4];
    const __half* ws[4];
    const float* attn_norm;
    const float* ffn_norm;
};

struct Params {
    const Layer* layers;  // device [n_layers]
    int n_layers, dim, q_dim, kv_dim, qkv_rows, ffn, vocab, head_dim, group, n_kv_heads, half, neox;
    float eps, scale_log2;
    const int8_t* emb_q;
    const __half* emb_s;
    const int8_t* out_q;
    const __half* out_s;
    const float* out_norm;
    int n, n_want;
    const int32_t* tokens;  // device [n]
    const int32_t* want;    // device [n_want]: rows whose logits are wanted
    const int32_t* seq;     // device [n]: one token per sequence
    const int32_t* pos;     // device [n]: the cell each token was appended at (its last position)
    const float* sincos;    // device [n][half][2]: sin, cos of pos * inv_freq
    uint16_t* pool;         // f16 block pool, layer l at pool + l * layer_elems
    size_t layer_elems;
    const int32_t* tables;  // [max_seqs][max_blocks]
    int max_blocks;
    float* x;               // [n][dim] residual stream
    float* qkv;             // [n][qkv_rows]
    float* att;             // [n][q_dim]
    float* act;             // [n][ffn]: SiLU(gate) * up
    float* logits;          // [n_want][vocab]
    int32_t* ids;           // [0]: error word (1: a bounded wait gave up); [1 + j]: argmax of logits row j
    int argmax;             // also write the greedy picks
    // [0] barrier arrivals (counted up through the launch; zeroed by the
    // host before it), [1] unused, [2] abort
    uint32_t* sync;
};

// Words of `sync`.
constexpr int kSyncWords = 3;
// Tokens per step the kernel takes (one mma N tile).
constexpr int kMaxTokens = 8;

// Whether the shapes fit the kernel (dims, shared memory); `smem` receives
// the dynamic shared memory a CTA needs.
bool supported(int dim, int q_dim, int ffn, int head_dim, int group, size_t* smem);
// Launch one decode step on `grid` co-resident CTAs.
cudaError_t launch(const Params& p, int grid, cudaStream_t st);
// CTAs a launch uses on the current device (one per SM), or 0 when the
// kernel cannot be made co-resident.
int grid_size(const Params& p);

}  // namespace lldec
