/*
 * lt_llama.h -- C ABI of the Llama step around the paged KV cache (sm_100a).
 *
 * Drop-in for the reference engine's Model::forward
 * (engine/crates/native/src/model.rs:366-518) over Q8_0 weights
 * (engine/crates/native/src/quant.rs), with the KV cache of lt_kv.h as its
 * cache: the same claim-first append (model.rs:380-383), the same per-layer
 * RoPE + K/V write + attention (model.rs:404-476), the same Q8_0 matmuls,
 * int8 activation quantizer, RMSNorm and SiLU, all on the device.
 *
 * Arithmetic.  Bit-identical to the reference's x86 path:
 *   - QMatrix::matmul (quant.rs:405-428, 492-533): per block
 *     (ws * xs) * (float)dot32, summed block by block from 0 in order;
 *   - QActs::quantize (quant.rs:771-795): amax / 127, round half away from
 *     zero, saturating to int8;
 *   - RoPE (model.rs:291-308): sin/cos of pos * inv_freq computed on the host
 *     with the C library, as the reference does, the rotation on the device;
 *   - embedding rows (quant.rs:464-490), residual adds, argmax
 *     (engine/crates/engine/src/sampling.rs:161-163).
 * Within a few ulps or a small relative error:
 *   - SiLU (model.rs:492-494): the exponential is correctly rounded to f32;
 *     the C library expf the reference calls is one ulp off on ~0.03 % of
 *     inputs, which moves the SiLU output by at most 2 ulps;
 *   - RMSNorm (model.rs:174-183): the sum of squares is a tree reduction,
 *     the reference's is sequential (its rounding error grows with dim);
 *     outputs agree within 1e-5 relative.
 * Attention matches within the lt_kv.h tolerance.
 *
 * Pointers.  *_host arguments are host memory; logits and the op-level
 * arrays are device memory.  Weights are given in their GGUF encoding and
 * copied to the device (Q8_0 blocks {f16 d; int8 qs[32]} for matrices, F32
 * for norm vectors).
 */
#ifndef LT_LLAMA_H
#define LT_LLAMA_H

#include <stddef.h>
#include <stdint.h>

#include "lt_kv.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct lt_llama lt_llama;

/* model.rs Config (model.rs:14-31) for a llama-architecture model. */
typedef struct lt_llama_config {
    uint32_t n_layers, dim, n_heads, n_kv_heads, head_dim, ffn_dim, vocab;
    uint32_t rope_dim;  /* rotary dims per head (model.rs:220-223); 0 = head_dim */
    int32_t rope_neox;  /* 1: pairs (i, i + rope_dim/2); 0: pairs (2i, 2i+1), llama */
    float eps;          /* attention.layer_norm_rms_epsilon (model.rs:218) */
    float rope_base;    /* rope.freq_base (model.rs:219) */
    uint32_t max_batch; /* tokens per forward call (n_batch, server/src/state.rs:220) */
    int32_t device;
} lt_llama_config;

/* Tensor ids (GGUF names per model.rs:236-262). */
typedef enum lt_tensor {
    LT_T_EMBED = 0,       /* token_embd.weight    [vocab][dim]  Q8_0 */
    LT_T_OUTPUT = 1,      /* output.weight        [vocab][dim]  Q8_0 */
    LT_T_OUTPUT_NORM = 2, /* output_norm.weight   [dim]         F32  */
    LT_T_ATTN_NORM = 3,   /* blk.L.attn_norm      [dim]         F32  */
    LT_T_FFN_NORM = 4,    /* blk.L.ffn_norm       [dim]         F32  */
    LT_T_Q = 5,           /* blk.L.attn_q         [q_dim][dim]  Q8_0 */
    LT_T_K = 6,           /* blk.L.attn_k         [kv_dim][dim] Q8_0 */
    LT_T_V = 7,           /* blk.L.attn_v         [kv_dim][dim] Q8_0 */
    LT_T_O = 8,           /* blk.L.attn_output    [dim][q_dim]  Q8_0 */
    LT_T_GATE = 9,        /* blk.L.ffn_gate       [ffn][dim]    Q8_0 */
    LT_T_UP = 10,         /* blk.L.ffn_up         [ffn][dim]    Q8_0 */
    LT_T_DOWN = 11        /* blk.L.ffn_down       [dim][ffn]    Q8_0 */
} lt_tensor;

/* Model::load's allocation (model.rs:184-289) without the file: device
 * buffers for every weight and for max_batch tokens of activations.
 * Dimensions must be multiples of 32; head_dim 64 or 128. */
lt_status lt_llama_create(const lt_llama_config* cfg, lt_llama** out);
void lt_llama_destroy(lt_llama* m);
const char* lt_llama_last_error(const lt_llama* m);

/* Copy one tensor (GGUF encoding, `bytes` long) to the device.  Every
 * tensor must be set before the first forward. */
lt_status lt_llama_set_tensor(lt_llama* m, lt_tensor which, uint32_t layer, const void* data_host, size_t bytes);

/* Model::forward (model.rs:366-518) for n tokens on `kv`, whose shape must
 * match (n_layers, n_kv_heads, head_dim, n_heads).  Claims every token's KV
 * cell first (errors as lt_kv_append; nothing else runs then).  Writes the
 * logits of the tokens listed in want_host to `logits` (device f32
 * [n_want][vocab]); logits may be NULL when n_want is 0.  Asynchronous on
 * `stream` after the host bookkeeping. */
lt_status lt_llama_forward(lt_llama* m, lt_kv* kv, const int32_t* tokens_host, const uint32_t* seq_host,
                           const uint32_t* pos_host, uint32_t n, const uint32_t* want_host, uint32_t n_want,
                           float* logits, void* stream);

/* forward + greedy pick (sampling.rs:161-163) of every token in want_host:
 * next_host[j] receives the argmax of want_host[j]'s logits.  Synchronises
 * `stream` (the ids are copied to the host). */
lt_status lt_llama_step_greedy(lt_llama* m, lt_kv* kv, const int32_t* tokens_host, const uint32_t* seq_host,
                               const uint32_t* pos_host, uint32_t n, const uint32_t* want_host, uint32_t n_want,
                               int32_t* next_host, void* stream);

/* Kernel launches issued by this handle since creation. */
uint64_t lt_llama_launch_count(const lt_llama* m);

/* The persistent decode step.  A forward of up to 8 tokens, each of a
 * different sequence, on an f16 cache runs as one cooperative launch (one
 * CTA per SM): every layer's matmuls, norms, RoPE, K/V append and attention,
 * then the output matrix and, for lt_llama_step_greedy, the greedy pick.  Its
 * matmul outputs and appended K/V bytes equal the multi-launch path's bit for
 * bit; attention is within the attention tolerance.  On by default;
 * enable = 0 runs every forward on the multi-launch path (for comparison).
 * lt_llama_persistent_available returns 1 when the model's shapes and the
 * device allow the persistent step. */
lt_status lt_llama_set_persistent(lt_llama* m, int enable);
int lt_llama_persistent_available(const lt_llama* m);

/* Profiling of the Q8_0 matmul launches of lt_llama_forward: when enabled,
 * each is bracketed by CUDA events on its stream (a persistent decode step
 * counts as one launch that carries every matmul of the step).
 * profile_read waits for the recorded launches, returns their summed device
 * time, count and algorithmic bytes (weights + scales, activations,
 * outputs), and starts a new window. */
lt_status lt_llama_profile(lt_llama* m, int enable);
lt_status lt_llama_profile_read(lt_llama* m, double* matmul_ms, uint64_t* matmul_launches, uint64_t* matmul_bytes);

/* ---- op-level entry points (device arrays; the same kernels the forward
 * runs), for per-op parity checks and for hosts that run their own loop ---- */

/* QActs::quantize (quant.rs:771-795): x [n][cols] f32 -> qs [n][cols] int8,
 * scales [n][cols/32] f32. */
lt_status lt_q8_quantize(const float* x, uint32_t n, uint32_t cols, int8_t* qs, float* scales, void* stream);

/* QMatrix::matmul (quant.rs:492-533): out[t][r] (+)= W[r] . x[t] for
 * weights w_qs [rows][cols] int8 and w_scales [rows][cols/32] f16 bits,
 * activations x_qs [n][cols], x_scales [n][cols/32] f32; out row stride
 * out_stride floats; accumulate != 0 adds into out (the residual add). */
lt_status lt_q8_matmul(const int8_t* w_qs, const uint16_t* w_scales, uint32_t rows, uint32_t cols,
                       const int8_t* x_qs, const float* x_scales, uint32_t n, float* out, uint32_t out_stride,
                       int accumulate, void* stream);

/* One projection of the forward on device arrays: an activation prologue on
 * f32 input x, then the Q8_0 matmul (as lt_q8_matmul):
 *   LT_PRO_QUANT    quantize x [n][cols];
 *   LT_PRO_SILU     SiLU(x[:, :cols]) * x[:, cols:] (x is [n][2*cols]), quantize;
 *   LT_PRO_RMSNORM  rms_norm of rows x[rows_idx[i]] (rows_idx NULL: 0..n-1)
 *                   with weight gamma [cols] and eps, quantize.
 * fused != 0 runs both in one launch when n <= 8 and cols % 256 == 0 (the
 * decode path of lt_llama_forward); otherwise, or with fused == 0, as two
 * launches.  Results are identical either way. */
enum { LT_PRO_QUANT = 1, LT_PRO_SILU = 2, LT_PRO_RMSNORM = 3 };
lt_status lt_q8_project(int prologue, const int8_t* w_qs, const uint16_t* w_scales, uint32_t rows, uint32_t cols,
                        const float* x, const int32_t* rows_idx, const float* gamma, float eps, uint32_t n,
                        float* out, uint32_t out_stride, int fused, int accumulate, void* stream);

/* Synchronises `stream` and reports whether an op-level matmul's bounded
 * wait for its weight copies gave up since the last check (LT_E_TIMEOUT). */
lt_status lt_q8_check(void* stream);

/* rms_norm (model.rs:174-183) of rows x[rows_idx[i]] (rows_idx NULL: rows
 * 0..n-1) with weight w [dim], then QActs::quantize; `normed` (may be NULL)
 * receives the f32 normalised rows [n][dim]. */
lt_status lt_rms_norm_q8(const float* x, const int32_t* rows_idx, const float* w, uint32_t dim, uint32_t n,
                         float eps, float* normed, int8_t* qs, float* scales, void* stream);

/* SiLU(gate) * up (model.rs:492-494) then QActs::quantize: gu [n][2*ffn]
 * holds gate in columns [0, ffn) and up in [ffn, 2*ffn); `h` (may be NULL)
 * receives the f32 product [n][ffn]. */
lt_status lt_silu_q8(const float* gu, uint32_t n, uint32_t ffn, float* h, int8_t* qs, float* scales, void* stream);

/* Greedy pick per row of x [n][cols] (sampling.rs:161-163: f32 total order,
 * the last index among equal maxima) -> idx [n] int32. */
lt_status lt_argmax_f32(const float* x, uint32_t n, uint32_t cols, int32_t* idx, void* stream);

#ifdef __cplusplus
}
#endif
#endif
