/*
 * lt_model.h -- TEST INFRASTRUCTURE ONLY: the C1 end-to-end workload.
 *
 * A CPU restatement of the reference engine's Llama forward pass
 * (engine/crates/native/src/model.rs:366-518) over Q8_0 weights
 * (engine/crates/native/src/quant.rs), with its KV cache behind om_kv so
 * the same forward runs against the oracle's KvCache or the GPU cache.
 * Parity of the forward itself is unpinned (the reference is Rust and is not
 * built here); only the KV cache and attention it drives are pinned.
 */
#ifndef LT_MODEL_H
#define LT_MODEL_H
#include <stddef.h>
#include <stdint.h>

#include "lt_oracle.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct omodel omodel;

/* The KV cache calls Model::forward makes (model.rs:380-383, 428, 431-476).
 * append claims all n cells first and returns 0 or an error code; write
 * stores f32 K/V rows [n][kv_dim]; attend fills out [n][n_heads*head_dim]. */
typedef struct {
    void* ctx;
    int (*append)(void* ctx, const uint32_t* seq, const uint32_t* pos, uint32_t n, int32_t* block, int32_t* slot);
    void (*write)(void* ctx, uint32_t layer, const int32_t* block, const int32_t* slot, uint32_t n, const float* k,
                  const float* v);
    void (*attend)(void* ctx, uint32_t layer, const float* q, const uint32_t* seq, const uint32_t* pos, uint32_t n,
                   float* out);
} om_kv;

/* Random-init Llama with Q8_0 weights: every weight ~ N(0, 0.02), the token
 * embedding ~ N(0, 1), norms 1, rope base 10000, eps 1e-5, an output matrix
 * of its own.  Deterministic in seed; dims must be multiples of 32. */
omodel* om_new_random(int dim, int n_layers, int n_heads, int n_kv_heads, int head_dim, int ffn_dim, int vocab,
                      uint64_t seed);
void om_delete(omodel* m);

/* Model::forward for n tokens (any mix of sequences and positions).  Logits
 * [n_want][vocab] for the tokens whose indices are in want.  n_threads
 * bounds the matmul threads (<=0: all). Returns 0 or append's error. */
int om_forward(const omodel* m, const om_kv* kv, const int32_t* tokens, const uint32_t* seqs, const uint32_t* pos,
               uint32_t n, const uint32_t* want, uint32_t n_want, float* logits, int n_threads);

/* argmax under f32 total order, last index among equal maxima
 * (engine/crates/engine/src/sampling.rs:161-163). */
int32_t om_argmax(const float* logits, int n);

/* Tensor ids, the same numbering as the product's lt_tensor. */
enum {
    OM_T_EMBED = 0, OM_T_OUTPUT, OM_T_OUTPUT_NORM, OM_T_ATTN_NORM, OM_T_FFN_NORM,
    OM_T_Q, OM_T_K, OM_T_V, OM_T_O, OM_T_GATE, OM_T_UP, OM_T_DOWN
};
size_t om_export_tensor(const omodel* m, int which, int layer, void* out);
const float* om_inv_freq(const omodel* m);

/* Op-level restatements, for per-op parity checks. */
void om_quantize(const float* x, uint32_t n, uint32_t cols, int8_t* qs, float* scales); /* quant.rs:771-795 */
void om_matmul_q8(const int8_t* wq, const float* ws, uint32_t rows, uint32_t cols, const int8_t* xq, const float* xs,
                  uint32_t n, float* out, int n_threads);                                 /* quant.rs:405-428 */
void om_rms_norm(const float* x, const float* w, uint32_t dim, uint32_t n, float eps, float* out); /* model.rs:174-183 */
void om_rope(const omodel* m, float* x, uint32_t n_heads, uint32_t pos);                  /* model.rs:291-308 */
void om_silu_mul(float* g, const float* u, size_t n);                                     /* model.rs:492-494 */

/* The oracle KvCache as an om_kv (attention over n_threads threads). */
om_kv* om_kv_oracle(okv* kv, int n_heads, int n_kv_heads, int head_dim, int n_threads);
void om_kv_free(om_kv* w);

#ifdef __cplusplus
}
#endif
#endif
