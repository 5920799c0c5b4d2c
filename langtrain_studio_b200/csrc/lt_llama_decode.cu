// Persistent decode step of the Llama forward: Model::forward
// (model.rs:366-518) for up to 8 tokens, one per sequence, in one
// cooperative launch of one CTA per SM.
//
// The step's work is a chain of phases, each needing the whole output of the
// one before: per layer
//   A  RMSNorm + quantise of x, q|k|v = Wqkv . x          (model.rs:404-413)
//   B  RoPE, append of K/V into the paged pool, attention (model.rs:414-476)
//   C  quantise of att, x += Wo . att                     (model.rs:478-484)
//   D  RMSNorm + quantise of x, gate|up = Wgu . x, and SiLU(gate) * up +
//      quantise of every 32-column group once its four 16-row tiles are in
//   E  x += Wdown . act                                   (model.rs:486-498)
// then the output norm and matrix (model.rs:502-517) and the greedy pick.
// A grid-wide barrier separates the phases; nothing else does.
//
// Weights.  The rows of every matrix are cut into 16-row tiles, dealt
// round-robin to the CTAs with an offset that rotates from phase to phase so
// each CTA's total stays within a tile of the mean.  A producer warp per CTA
// streams the CTA's tiles -- all layers, in phase order -- through a 4-slot
// shared-memory ring with bulk copies (16 rows x up to 2048 columns and
// their f16 scales per slot), limited only by free slots: weights for the
// next phases arrive while the CTA waits at a barrier.  The 16 compute warps
// form 2 groups of 8; a CTA's tiles go to the groups in turn, so each group
// multiplies one slot while the next tile it gets is loading into another.
//
// Attention.  Each (token, KV head)'s blocks are cut into up to 32 pieces,
// and the pieces of all of them are dealt over every CTA's warps.  A warp
// attends its piece (online softmax, f32), writes the piece's (m, l, O) to
// global memory, and the warp that completes a (token, head) merges its
// pieces into att.
//
// Arithmetic.  Every matmul output is the reference's row_dot
// (quant.rs:418-421): one s8 mma per 32-wide block gives the exact int
// dot, the products (ws * xs) * dot are written over the block's weight bytes
// in the slot, and one warp adds them block by block from 0.0f -- across
// chunks for matrices wider than 2048 columns.  The activation prologues use
// the grouping and reduction tree of the multi-launch kernels, RoPE the
// host's sin/cos table without contraction, and the pool rows the same
// f32 -> f16 conversion and cell layout as the K/V write, so matmul outputs
// and pool bytes equal those of the multi-launch path bit for bit.  Attention
// is f32 with an online softmax (exp2 of log2e-scaled scores) and stays
// within the attention tolerance of the reference's result.
//
// Waits.  Every wait (slot barriers, the grid barrier) is bounded.  One that
// gives up raises the error word and an abort flag that every other wait
// polls, so the whole grid leaves within one limit; each CTA drains its
// copies in flight before it exits.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include <algorithm>

#include "lt_kv_layout.cuh"
#include "lt_llama_decode.h"
#include "lt_q8_device.cuh"

namespace lldec {
namespace {

using ltq8::kQK;
constexpr int kWarps = 16;                 // compute warps
constexpr int kGroups = 2;                 // warp groups that multiply different tiles at once
constexpr int kGroupWarps = kWarps / kGroups;
constexpr int kThreads = kWarps * 32;      // compute threads (named barrier 1)
constexpr int kCtaThreads = kThreads + 32; // + the weight producer warp
constexpr int kRows = 16;                  // weight rows per tile (mma M)
constexpr int kChunk = 2048;               // columns per ring slot
constexpr int kStages = 4;                 // ring slots
constexpr int kWPitch = kChunk + 16;       // bytes between weight rows in a slot (16-byte rows of 8
                                           // consecutive weight rows fall in 8 different bank groups)
constexpr int kSPitch = kChunk / kQK * 2 + 16;  // bytes between scale rows in a slot
constexpr int kSlotBytes = kRows * kWPitch + kRows * kSPitch;
constexpr int kHeader = 128;               // mbarriers and a few words
constexpr int kNormItems = 4;              // RMSNorm items a thread holds (8 tokens x 2048 / 8 over 512 threads)
constexpr uint64_t kWaitNs = 2000000000ull;  // 2 s
constexpr uint64_t kDrainNs = 100000000ull;  // 0.1 s per copy still in flight when a CTA gives up
constexpr unsigned kFull = 0xffffffffu;

struct Smem {
    int x_pitch, xs_pitch;  // activation rows (int8 bytes), their scales (floats)
    size_t xq, xs, red, total;
    __host__ __device__ Smem(int maxc) {
        x_pitch = maxc + 32;
        xs_pitch = maxc / kQK + 4;
        xq = kHeader + (size_t)kStages * kSlotBytes;
        xs = xq + (size_t)kMaxTokens * x_pitch;
        red = xs + (size_t)kMaxTokens * xs_pitch * 4;
        total = red + kWarps * 32 * 4;
    }
};

// ------------------------------------------------------------ helpers -----

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ uint32_t ld_volatile(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.volatile.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ uint32_t ld_acquire(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Raise the error word and the abort flag that every bounded wait polls.
__device__ __forceinline__ void raise_abort(const Params& p) {
    atomicOr(p.ids, 1);
    atomicExch(p.sync + 2, 1u);
}

// Wait for a phase of an mbarrier; gives up after kWaitNs or once another
// CTA raised the abort flag.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, const Params& p, bool backoff = false) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if (backoff) __nanosleep(128);  // a producer waiting for a free slot leaves the issue slots to the math
        if ((it & 63) == 0) {
            if (ld_volatile(p.sync + 2)) return false;
            if (global_ns() - t0 > kWaitNs) {
                raise_abort(p);
                return false;
            }
        }
    }
}

// The compute warps' barrier (the producer warp never takes part), and one
// barrier per warp group.
__device__ __forceinline__ void bar_compute() { asm volatile("bar.sync 1, %0;" ::"n"(kThreads) : "memory"); }
__device__ __forceinline__ void bar_group(int grp) {
    asm volatile("bar.sync %0, %1;" ::"r"(2 + grp), "n"(kGroupWarps * 32) : "memory");
}

__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}

// 8 consecutive f32 from memory that other CTAs wrote in an earlier phase
// (read at L2, never from a stale L1 line).
__device__ __forceinline__ void load8_cg(const float* p, float (&v)[8]) {
    const float4 a = __ldcg(reinterpret_cast<const float4*>(p));
    const float4 b = __ldcg(reinterpret_cast<const float4*>(p) + 1);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

// ------------------------------------------------------ work partition ----

struct Mat {
    const int8_t* q;
    const __half* s;
    int rows, cols;
};

// Phase ph = 4 * layer + matrix kind; ph = 4 * n_layers is the output matrix.
__device__ __forceinline__ Mat phase_mat(const Params& p, int ph) {
    if (ph == 4 * p.n_layers) return {p.out_q, p.out_s, p.vocab, p.dim};
    const Layer& L = p.layers[ph >> 2];
    const int k = ph & 3;
    const int rows = k == kQkv ? p.qkv_rows : k == kGateUp ? 2 * p.ffn : p.dim;
    const int cols = k == kO ? p.q_dim : k == kDown ? p.ffn : p.dim;
    return {L.wq[k], L.ws[k], rows, cols};
}

__device__ __forceinline__ int n_phases(const Params& p) { return 4 * p.n_layers + (p.n_want > 0 ? 1 : 0); }
__device__ __forceinline__ int tiles_of(const Mat& m) { return (m.rows + kRows - 1) / kRows; }
__device__ __forceinline__ int chunks_of(const Mat& m) { return (m.cols + kChunk - 1) / kChunk; }
// First tile of this CTA in a phase whose deal starts `off` CTAs along.
__device__ __forceinline__ int first_tile(int off) { return ((int)blockIdx.x - off + (int)gridDim.x) % (int)gridDim.x; }
// Tiles of this CTA in such a phase.
__device__ __forceinline__ int local_tiles(int tiles, int off) {
    const int t0 = first_tile(off);
    return t0 < tiles ? (tiles - t0 + (int)gridDim.x - 1) / (int)gridDim.x : 0;
}

// ------------------------------------------------------------ producer ----

// Issue every chunk of this CTA's tiles, in phase order, into the ring.
__device__ void produce(const Params& p, uint8_t* sm) {
    const int lane = threadIdx.x & 31;
    const uint32_t full0 = smem_u32(sm), empty0 = full0 + 8 * kStages;
    volatile uint32_t* issued = reinterpret_cast<volatile uint32_t*>(sm + 16 * kStages);
    uint32_t c = 0;
    int off = 0;
    bool ok = true;
    for (int ph = 0; ph < n_phases(p) && ok; ++ph) {
        const Mat m = phase_mat(p, ph);
        const int tiles = tiles_of(m), nck = chunks_of(m);
        for (int t = first_tile(off); t < tiles && ok; t += gridDim.x) {
            for (int j = 0; j < nck; ++j, ++c) {
                const int s = c % kStages;
                int go = 1;
                if (lane == 0 && c >= kStages) go = mbar_wait(empty0 + 8 * s, ((c / kStages) - 1) & 1, p, true);
                go = __shfl_sync(kFull, go, 0);
                if (!go) {
                    ok = false;
                    break;
                }
                const int k0 = j * kChunk, kc = min(kChunk, m.cols - k0);
                const uint32_t bar = full0 + 8 * s;
                if (lane == 0)
                    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar),
                                 "r"((uint32_t)(kRows * (kc + kc / kQK * 2)))
                                 : "memory");
                __syncwarp();
                if (lane < kRows) {  // one lane per weight row: its bytes and its scales
                    const int r = min(t * kRows + lane, m.rows - 1);
                    uint8_t* slot = sm + kHeader + (size_t)s * kSlotBytes;
                    bulk_g2s(smem_u32(slot + lane * kWPitch), m.q + (size_t)r * m.cols + k0, (uint32_t)kc, bar);
                    bulk_g2s(smem_u32(slot + kRows * kWPitch + lane * kSPitch),
                             m.s + (size_t)r * (m.cols / kQK) + k0 / kQK, (uint32_t)(kc / kQK * 2), bar);
                }
                __syncwarp();
                if (lane == 0) *issued = c + 1;
            }
        }
        off = (off + tiles) % (int)gridDim.x;
    }
    __syncwarp();
    if (lane == 0) *reinterpret_cast<volatile uint32_t*>(sm + 16 * kStages + 4) = 1;  // done issuing
}

// ----------------------------------------------------------- prologues ----

// RMSNorm + quantise of rows of x into the activation tile, all tokens in
// one pass.  Item (t, i) is the 8 columns [8i, 8i + 8) of token t; its
// squares are summed in order, the items of a warp (32 consecutive i of one
// token) by an xor tree, and the dim/256 warp partials of a token by an xor
// tree over 32 lanes (lanes past them add 0.0f): rms_norm_q8_kernel's tree,
// so the result is the multi-launch path's bit for bit.  Every item's loads
// are issued before any arithmetic.
__device__ void prologue_norm(const Params& p, const Smem& L, uint8_t* sm, const int32_t* rows_idx,
                              const float* gamma, int n_tok) {
    const int cols = p.dim, tpt = cols / 8, nw = tpt / 32, items = n_tok * tpt;
    const int tid = threadIdx.x, lane = tid & 31;
    float* red = reinterpret_cast<float*>(sm + L.red);  // [8 tokens][nw] warp partials; totals at [256 + t]
    int8_t* xq = reinterpret_cast<int8_t*>(sm + L.xq);
    float* xs = reinterpret_cast<float*>(sm + L.xs);
    float v[kNormItems][8];
#pragma unroll
    for (int k = 0; k < kNormItems; ++k) {
        const int it = tid + k * kThreads;
#pragma unroll
        for (int e = 0; e < 8; ++e) v[k][e] = 0.f;
        if (it < items) {
            const int t = it / tpt, i = it % tpt;
            load8_cg(p.x + (size_t)(rows_idx ? __ldg(rows_idx + t) : t) * cols + i * 8, v[k]);
        }
    }
#pragma unroll
    for (int k = 0; k < kNormItems; ++k) {
        const int it = tid + k * kThreads;
        if (k * kThreads >= items) break;  // block-uniform
        float ss = 0.0f;
#pragma unroll
        for (int e = 0; e < 8; e++) ss = __fadd_rn(ss, __fmul_rn(v[k][e], v[k][e]));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(kFull, ss, o));
        if (lane == 0 && it < items) red[(it / tpt) * nw + (it % tpt) / 32] = ss;
    }
    bar_compute();
    const int warp = tid >> 5;
    if (warp < n_tok) {  // token `warp`: the tree over its nw warp partials
        float s2 = lane < nw ? red[warp * nw + lane] : 0.0f;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s2 = __fadd_rn(s2, __shfl_xor_sync(kFull, s2, o));
        if (lane == 0) red[256 + warp] = s2;
    }
    bar_compute();
#pragma unroll
    for (int k = 0; k < kNormItems; ++k) {
        const int it = tid + k * kThreads;
        if (k * kThreads >= items) break;
        const bool live = it < items;
        const int t = live ? it / tpt : 0, i = live ? it % tpt : 0;
        const float ms = __fdiv_rn(red[256 + t], (float)cols);
        const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, p.eps)));
        float gv[8];
        ltq8::load8(gamma + i * 8, gv);
#pragma unroll
        for (int e = 0; e < 8; e++) v[k][e] = __fmul_rn(__fmul_rn(v[k][e], inv), gv[e]);
        ltq8::quant8_store(v[k], xq + (size_t)t * L.x_pitch + i * 8, xs + (size_t)t * L.xs_pitch + i / 4,
                           (i & 3) == 0, live);
    }
}

// Quantise of the attention output rows (the QUANT prologue's mapping).
__device__ void prologue_quant(const Params& p, const Smem& L, uint8_t* sm) {
    const int per_row = p.q_dim / 8, total = p.n * per_row;
    int8_t* xq = reinterpret_cast<int8_t*>(sm + L.xq);
    float* xs = reinterpret_cast<float*>(sm + L.xs);
    for (int base = 0; base < total; base += kThreads) {  // every lane takes every pass (group shuffles)
        const int item = base + (int)threadIdx.x;
        const bool live = item < total;
        const int t = live ? item / per_row : 0, c = live ? (item % per_row) * 8 : 0;
        float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        if (live) load8_cg(p.att + (size_t)t * p.q_dim + c, v);
        ltq8::quant8_store(v, xq + (size_t)t * L.x_pitch + c, xs + (size_t)t * L.xs_pitch + c / kQK,
                           (threadIdx.x & 3) == 0, live);
    }
}

// The quantised SiLU(gate) * up rows, as the D phase's last arrivers wrote them.
__device__ void prologue_act(const Params& p, const Smem& L, uint8_t* sm) {
    const int per_row = p.ffn / 16, nb = p.ffn / kQK;
    int8_t* xq = reinterpret_cast<int8_t*>(sm + L.xq);
    float* xs = reinterpret_cast<float*>(sm + L.xs);
    for (int idx = threadIdx.x; idx < p.n * per_row; idx += kThreads) {
        const int t = idx / per_row, c = (idx % per_row) * 16;
        *reinterpret_cast<int4*>(xq + (size_t)t * L.x_pitch + c) =
            __ldcg(reinterpret_cast<const int4*>(p.act_q + (size_t)t * p.ffn + c));
    }
    for (int idx = threadIdx.x; idx < p.n * nb; idx += kThreads)
        xs[(idx / nb) * L.xs_pitch + idx % nb] = __ldcg(p.act_s + idx);
}

// Tokens n_tok..7 of the activation tile read as zeros over `cols` columns.
__device__ void zero_tail(const Smem& L, uint8_t* sm, int n_tok, int cols) {
    int8_t* xq = reinterpret_cast<int8_t*>(sm + L.xq);
    float* xs = reinterpret_cast<float*>(sm + L.xs);
    const int per = cols / 16, nb = cols / kQK;
    for (int idx = threadIdx.x; idx < (kMaxTokens - n_tok) * per; idx += kThreads)
        *reinterpret_cast<int4*>(xq + (size_t)(n_tok + idx / per) * L.x_pitch + (idx % per) * 16) =
            make_int4(0, 0, 0, 0);
    for (int idx = threadIdx.x; idx < (kMaxTokens - n_tok) * nb; idx += kThreads)
        xs[(n_tok + idx / nb) * L.xs_pitch + idx % nb] = 0.f;
}

// SiLU(gate) * up + quantise of one 32-column group for every token, by one
// warp (silu_q8_kernel's arithmetic: exp rounded once from double precision).
__device__ void silu_group(const Params& p, int j) {
    const int lane = threadIdx.x & 31, tok = lane >> 2, part = lane & 3;
    const bool live = tok < p.n;
    const int c = j * kQK + part * 8;
    float g[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f}, u[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (live) {
        load8_cg(p.gu + (size_t)tok * 2 * p.ffn + c, g);
        load8_cg(p.gu + (size_t)tok * 2 * p.ffn + p.ffn + c, u);
    }
#pragma unroll
    for (int k = 0; k < 8; k++) {
        const float e = (float)exp(-(double)g[k]);
        g[k] = __fmul_rn(__fdiv_rn(g[k], __fadd_rn(1.0f, e)), u[k]);
    }
    ltq8::quant8_store(g, p.act_q + (size_t)tok * p.ffn + c, p.act_s + ((size_t)tok * p.ffn + c) / kQK, part == 0,
                       live);
}

// -------------------------------------------------------------- barrier ---

// Grid-wide barrier of the compute warps.  The arrival count rises through
// the launch (the host zeroes it before): barrier k of the launch is passed
// once it reaches k * gridDim.x.  Thread 0 of each CTA keeps that target.
__device__ bool grid_sync(const Params& p, uint32_t& target, volatile int* flag) {
    bar_compute();
    if (threadIdx.x == 0) {
        target += gridDim.x;
        int ok = 1;
        // release: this CTA's writes (ordered before by the barrier above) before the arrival
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(p.sync) : "memory");
        if (ld_acquire(p.sync) < target) {
            const uint64_t t0 = global_ns();
            for (uint32_t it = 0;; ++it) {
                if (ld_acquire(p.sync) >= target) break;
                if ((it & 15) == 15) {
                    if (ld_volatile(p.sync + 2)) {
                        ok = 0;
                        break;
                    }
                    if (global_ns() - t0 > kWaitNs) {
                        raise_abort(p);
                        ok = 0;
                        break;
                    }
                }
            }
        }
        *flag = ok;
    }
    bar_compute();
    return *flag != 0;
}

// ------------------------------------------------------------- matmuls ----

// This CTA's tiles of phase ph, local tile i to warp group i % kGroups; its
// chunks are ring chunks c_base + i * chunks + j.  Per chunk: the group's
// leader waits for it; one s8 mma per 32-wide block (block b to the group's
// warp b % 8, four blocks' operands loaded before their mmas), the products
// over the block's weight bytes; the group's first warp adds them in block
// order; the slot goes back to the producer.  After a tile's last chunk that
// warp writes its 16 rows x n_tok outputs.  D phases also run the SiLU of
// every group of columns whose fourth tile this CTA completes.  flags[0]
// (set to 1 by the caller before the prologue's barrier) falls to 0 when a
// wait gave up; the result is that flag.
__device__ bool consume(const Params& p, const Smem& L, uint8_t* sm, int ph, uint32_t c_base, int off, int n_tok,
                        volatile int* flags) {
    const Mat m = phase_mat(p, ph);
    const int kind = ph == 4 * p.n_layers ? 4 : (ph & 3), layer = ph >> 2;
    const int nck = chunks_of(m);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int grp = warp / kGroupWarps, gw = warp % kGroupWarps, gtid = tid % (kGroupWarps * 32);
    const int g = lane >> 2, q = lane & 3;
    const uint32_t full0 = smem_u32(sm), empty0 = full0 + 8 * kStages;
    const int8_t* xq = reinterpret_cast<const int8_t*>(sm + L.xq);
    const float* xs = reinterpret_cast<const float*>(sm + L.xs);
    volatile int* gflag = flags + 1 + grp;
    bool ok = true;
    const int n_local = local_tiles(tiles_of(m), off);
    for (int i = grp; i < n_local && ok; i += kGroups) {
        const int t = first_tile(off) + i * (int)gridDim.x;
        float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);  // the group's first warp: running sums of the tile
        for (int j = 0; j < nck; ++j) {
            const uint32_t c = c_base + (uint32_t)(i * nck + j);
            const int s = c % kStages;
            if (gtid == 0) *gflag = mbar_wait(full0 + 8 * s, (c / kStages) & 1, p);
            bar_group(grp);
            if (!*gflag) {
                ok = false;
                break;
            }
            uint8_t* w = sm + kHeader + (size_t)s * kSlotBytes;
            const __half* ws = reinterpret_cast<const __half*>(w + kRows * kWPitch);
            const int k0 = j * kChunk, nb = min(kChunk, m.cols - k0) / kQK, kb0 = k0 / kQK;
            for (int b0 = gw; b0 < nb; b0 += 4 * kGroupWarps) {
                uint2 A0[4], A1[4], B[4];
                float wsa[4], wsb[4], xsa[4], xsc[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int b = min(b0 + u * kGroupWarps, nb - 1);
                    A0[u] = *reinterpret_cast<const uint2*>(w + (size_t)g * kWPitch + 32 * b + 8 * q);
                    A1[u] = *reinterpret_cast<const uint2*>(w + (size_t)(g + 8) * kWPitch + 32 * b + 8 * q);
                    B[u] = *reinterpret_cast<const uint2*>(xq + (size_t)g * L.x_pitch + 32 * (kb0 + b) + 8 * q);
                    wsa[u] = __half2float(ws[g * (kSPitch / 2) + b]);
                    wsb[u] = __half2float(ws[(g + 8) * (kSPitch / 2) + b]);
                    xsa[u] = xs[(2 * q) * L.xs_pitch + kb0 + b];
                    xsc[u] = xs[(2 * q + 1) * L.xs_pitch + kb0 + b];
                }
                float4 pr[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    int d[4];
                    ltq8::mma_s8(d, A0[u].x, A1[u].x, A0[u].y, A1[u].y, B[u].x, B[u].y);
                    pr[u].x = __fmul_rn(__fmul_rn(wsa[u], xsa[u]), __int2float_rn(d[0]));
                    pr[u].y = __fmul_rn(__fmul_rn(wsa[u], xsc[u]), __int2float_rn(d[1]));
                    pr[u].z = __fmul_rn(__fmul_rn(wsb[u], xsa[u]), __int2float_rn(d[2]));
                    pr[u].w = __fmul_rn(__fmul_rn(wsb[u], xsc[u]), __int2float_rn(d[3]));
                }
                __syncwarp();  // every lane has read these blocks before they are overwritten
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int b = b0 + u * kGroupWarps;
                    if (b < nb)
                        *reinterpret_cast<float4*>(w + (size_t)(lane >> 1) * kWPitch + 32 * b + 16 * (lane & 1)) = pr[u];
                }
            }
            bar_group(grp);
            if (gw == 0) {
                const uint8_t* slot = w + (size_t)(lane >> 1) * kWPitch + 16 * (lane & 1);
#pragma unroll 8
                for (int b = 0; b < nb; b++) {
                    const float4 pb = *reinterpret_cast<const float4*>(slot + 32 * b);
                    acc.x = __fadd_rn(acc.x, pb.x);
                    acc.y = __fadd_rn(acc.y, pb.y);
                    acc.z = __fadd_rn(acc.z, pb.z);
                    acc.w = __fadd_rn(acc.w, pb.w);
                }
            }
            // the slot's generic reads and writes before the next bulk copy into it
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            bar_group(grp);
            if (gtid == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(empty0 + 8 * s) : "memory");
        }
        if (!ok) break;
        if (gw == 0) {
            const float v[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const int r = t * kRows + g + 8 * (e >> 1), tok = 2 * q + (e & 1);
                if (r >= m.rows || tok >= n_tok) continue;
                if (kind == kQkv) {
                    p.qkv[(size_t)tok * p.qkv_rows + r] = v[e];
                } else if (kind == kGateUp) {
                    p.gu[(size_t)tok * 2 * p.ffn + r] = v[e];
                } else if (kind == 4) {
                    p.logits[(size_t)tok * p.vocab + r] = v[e];
                } else {  // o, down: residual add into x (model.rs:484, 498)
                    float* o = p.x + (size_t)tok * p.dim + r;
                    *o = __fadd_rn(__ldcg(o), v[e]);
                }
            }
        }
        if (kind == kGateUp) {
            // The SiLU group of this tile: its two gate and two up tiles; the
            // warp group that completes the fourth computes it.
            __threadfence();
            bar_group(grp);
            if (gtid == 0) {
                const int half_tiles = p.ffn / kRows;
                const int sg = t < half_tiles ? t / 2 : (t - half_tiles) / 2;
                const uint32_t old = atomicAdd(p.sync + kSyncHeader + sg, 1u);
                __threadfence();
                *gflag = old == 4u * (uint32_t)(layer + 1) - 1u ? sg : -1;
            }
            bar_group(grp);
            const int sg = *gflag;
            if (sg >= 0 && gw == 0) silu_group(p, sg);
            bar_group(grp);
        }
    }
    if (gtid == 0 && !ok) flags[0] = 0;  // this group gave up
    bar_compute();
    return flags[0] != 0;
}

// --------------------------------------------------------- attention -----

// RoPE of the head-aligned range [base, base + count) of a token's q|k row
// into dst[0, count), by one warp: each rotated pair (non-NeoX: 2i, 2i+1;
// NeoX: i, i + half; model.rs:291-308) once, with rope_split_kernel's
// arithmetic, columns past the rotary part copied.  Four items a lane per
// round, all their loads issued before the arithmetic.
__device__ void rope_range(const Params& p, const float* row, const float* sc, int base, int count, float* dst) {
    const int lane = threadIdx.x & 31, hd = p.head_dim, half = p.half;
    const int per_head = half + (hd - 2 * half), total = (count / hd) * per_head;
    for (int r0 = 0; r0 < total; r0 += 4 * 32) {
        float a[4], b[4], sn[4], cs[4];
        int ia[4], ib[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int it = r0 + u * 32 + lane;
            ia[u] = -1;
            ib[u] = -1;
            if (it < total) {
                const int h = it / per_head, k = it % per_head, hb = h * hd;
                if (k < half) {
                    ia[u] = hb + (p.neox ? k : 2 * k);
                    ib[u] = hb + (p.neox ? k + half : 2 * k + 1);
                    a[u] = __ldcg(row + base + ia[u]);
                    b[u] = __ldcg(row + base + ib[u]);
                    sn[u] = __ldg(sc + 2 * k);
                    cs[u] = __ldg(sc + 2 * k + 1);
                } else {
                    ia[u] = hb + 2 * half + (k - half);
                    a[u] = __ldcg(row + base + ia[u]);
                }
            }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            if (ia[u] < 0) continue;
            if (ib[u] < 0) {
                dst[ia[u]] = a[u];
            } else {
                dst[ia[u]] = __fsub_rn(__fmul_rn(a[u], cs[u]), __fmul_rn(b[u], sn[u]));  // x0 cos - x1 sin
                dst[ib[u]] = __fadd_rn(__fmul_rn(a[u], sn[u]), __fmul_rn(b[u], cs[u]));  // x0 sin + x1 cos
            }
        }
    }
}

// Pieces of (token, KV head) unit u: its blocks [0, pos/16] cut into up to
// kMaxPieces ranges of near-equal length.
__device__ __forceinline__ int unit_pieces(const Params& p, int u) {
    return min(__ldg(p.pos + u / p.n_kv_heads) / ltkv::kBlock + 1, kMaxPieces);
}

// One attention piece, by one warp: RoPE of the unit's q heads into the
// warp's buffer; the new K/V row into the token's pool cell when the piece
// holds the last block (f16, the write kernel's layout and conversion);
// attention over the piece's blocks (a block's K loads issued together, then
// its V loads); the piece's (m, l, O) to att_part.  The warp that
// completes the unit's pieces merges them into att.
template <int D>
__device__ void attend_piece(const Params& p, int layer, int u, int piece, float* q_w) {
    constexpr int DV = D / 32;  // output dims per lane
    const int lane = threadIdx.x & 31;
    const int G = p.group, Hkv = p.n_kv_heads;
    const int t = u / Hkv, h = u % Hkv;
    const float* row = p.qkv + (size_t)t * p.qkv_rows;
    const float* sc = p.sincos + (size_t)t * p.half * 2;
    const int seq = __ldg(p.seq + t), pos = __ldg(p.pos + t);
    const int nb = pos / ltkv::kBlock + 1, np = unit_pieces(p, u);
    const int b0 = (int)((long long)piece * nb / np), b1 = (int)((long long)(piece + 1) * nb / np);
    const int32_t* trow = p.tables + (size_t)seq * p.max_blocks;
    uint16_t* pool_l = p.pool + (size_t)layer * p.layer_elems;
    rope_range(p, row, sc, h * G * D, G * D, q_w);  // the group's q heads
    if (b1 == nb) rope_range(p, row, sc, p.q_dim + h * D, D, q_w + G * D);  // the new K row
    __syncwarp();
    if (b1 == nb && lane < 2 * (D / 8)) {  // the new row of (token, head): K roped, V as is
        const int blk = __ldg(trow + pos / ltkv::kBlock), slot = pos % ltkv::kBlock;
        uint16_t* tile = pool_l + ((size_t)blk * Hkv + h) * 2 * ltkv::kBlock * D;
        const int kvsel = lane / (D / 8), c = lane % (D / 8);
        float x[8];
        if (kvsel == 0) {
#pragma unroll
            for (int e = 0; e < 8; ++e) x[e] = q_w[G * D + c * 8 + e];
        } else {
            load8_cg(row + p.q_dim + p.kv_dim + h * D + c * 8, x);
        }
        uint32_t wv[4];
#pragma unroll
        for (int e = 0; e < 4; ++e)
            wv[e] = ltkv::f32_to_f16_ref(x[2 * e]) | (uint32_t(ltkv::f32_to_f16_ref(x[2 * e + 1])) << 16);
        *reinterpret_cast<uint4*>(tile + kvsel * ltkv::kBlock * D + ltkv::chunk_off(c, slot)) =
            make_uint4(wv[0], wv[1], wv[2], wv[3]);
    }
    __syncwarp();  // q_w and the new row are visible to the whole warp
    const int s = lane & 15, hs = lane >> 4, d0 = lane * DV;
    float m[4], l[4], o[8][DV];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        m[i] = -INFINITY;
        l[i] = 0.0f;
    }
#pragma unroll
    for (int gg = 0; gg < 8; gg++)
#pragma unroll
        for (int dd = 0; dd < DV; dd++) o[gg][dd] = 0.0f;
    for (int b = b0; b < b1; ++b) {
        const int blk = __ldg(trow + b);
        const uint16_t* kt = pool_l + ((size_t)blk * Hkv + h) * 2 * ltkv::kBlock * D;
        const uint16_t* vt = kt + ltkv::kBlock * D;
        uint4 kr[D / 8];
#pragma unroll
        for (int c = 0; c < D / 8; ++c) kr[c] = *reinterpret_cast<const uint4*>(kt + ltkv::chunk_off(c, s));
        float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int c = 0; c < D / 8; ++c) {
            const uint32_t kw[4] = {kr[c].x, kr[c].y, kr[c].z, kr[c].w};
            float kf[8];
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&kw[e]));
                kf[2 * e] = f.x;
                kf[2 * e + 1] = f.y;
            }
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const int gq = hs + 2 * i;
                if (gq < G) {
                    const float* qg = q_w + gq * D + c * 8;
#pragma unroll
                    for (int e = 0; e < 8; e++) acc[i] = fmaf(qg[e], kf[e], acc[i]);
                }
            }
        }
        const bool valid = b * ltkv::kBlock + s <= pos;
        float pr[4], al[4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const float sv = valid ? acc[i] * p.scale_log2 : -INFINITY;
            float bm = sv;
#pragma unroll
            for (int o2 = 1; o2 < 16; o2 <<= 1) bm = fmaxf(bm, __shfl_xor_sync(kFull, bm, o2));
            const float mn = fmaxf(m[i], bm);  // finite: slot 0 of every block is at or before pos
            al[i] = exp2f(m[i] - mn);
            pr[i] = exp2f(sv - mn);
            float bs = pr[i];
#pragma unroll
            for (int o2 = 1; o2 < 16; o2 <<= 1) bs += __shfl_xor_sync(kFull, bs, o2);
            l[i] = l[i] * al[i] + bs;
            m[i] = mn;
        }
        uint32_t vr[ltkv::kBlock][DV / 2];  // this lane's columns of the block's 16 V rows
#pragma unroll
        for (int ss = 0; ss < ltkv::kBlock; ++ss) {
            const uint16_t* vp = vt + ltkv::chunk_off(d0 / 8, ss) + (d0 % 8);
            if (DV == 2) {
                vr[ss][0] = *reinterpret_cast<const uint32_t*>(vp);
            } else {
                const uint2 uu = *reinterpret_cast<const uint2*>(vp);
                vr[ss][0] = uu.x;
                vr[ss][DV / 2 - 1] = uu.y;
            }
        }
#pragma unroll
        for (int gg = 0; gg < 8; gg++) {
            if (gg < G) {
                const float a = __shfl_sync(kFull, al[gg >> 1], (gg & 1) * 16);
#pragma unroll
                for (int dd = 0; dd < DV; dd++) o[gg][dd] *= a;
            }
        }
#pragma unroll
        for (int ss = 0; ss < ltkv::kBlock; ++ss) {
            float vv[DV];
#pragma unroll
            for (int e = 0; e < DV / 2; ++e) {
                const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&vr[ss][e]));
                vv[2 * e] = f.x;
                vv[2 * e + 1] = f.y;
            }
#pragma unroll
            for (int gg = 0; gg < 8; gg++) {
                if (gg < G) {
                    const float pg = __shfl_sync(kFull, pr[gg >> 1], ss + (gg & 1) * 16);
#pragma unroll
                    for (int dd = 0; dd < DV; dd++) o[gg][dd] = fmaf(pg, vv[dd], o[gg][dd]);
                }
            }
        }
    }
    const size_t stride = (size_t)2 * G + (size_t)G * D;
    float* mine = p.att_part + ((size_t)u * kMaxPieces + piece) * stride;
    if (s == 0) {
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int gq = hs + 2 * i;
            if (gq < G) {
                mine[gq] = m[i];
                mine[G + gq] = l[i];
            }
        }
    }
#pragma unroll
    for (int gg = 0; gg < 8; gg++)
        if (gg < G)
#pragma unroll
            for (int dd = 0; dd < DV; dd++) mine[2 * G + gg * D + d0 + dd] = o[gg][dd];
    // the warp that completes the unit's pieces merges them
    __threadfence();
    __syncwarp();
    int last = 0;
    if (lane == 0) {
        const uint32_t old = atomicAdd(p.sync + kSyncHeader + p.ffn / kQK + u, 1u);
        last = old == (uint32_t)np * (uint32_t)(layer + 1) - 1u;
        __threadfence();
    }
    if (!__shfl_sync(kFull, last, 0)) return;
    __threadfence();
    const float* part = p.att_part + (size_t)u * kMaxPieces * stride;
    for (int e = lane; e < G * D; e += 32) {
        const int gq = e / D, d = e % D;
        float mx = -INFINITY;
        for (int w = 0; w < np; w++) mx = fmaxf(mx, __ldcg(part + w * stride + gq));
        float ls = 0.0f, os = 0.0f;
        for (int w = 0; w < np; w++) {
            const float* pw = part + w * stride;
            const float f = exp2f(__ldcg(pw + gq) - mx);
            ls += __ldcg(pw + G + gq) * f;
            os += __ldcg(pw + 2 * G + gq * D + d) * f;
        }
        p.att[(size_t)t * p.q_dim + (size_t)(h * G + gq) * D + d] = os / ls;
    }
}

// The attention phase of this CTA: piece k of the enumeration over units
// (unit-major) goes to CTA k % gridDim.x, its warp (k / gridDim.x) % aw.
template <int D>
__device__ void attend_phase(const Params& p, const Smem& L, uint8_t* sm, int layer, int aw) {
    const int warp = threadIdx.x >> 5;
    if (warp >= aw) return;
    float* q_w = reinterpret_cast<float*>(sm + L.xq) + (size_t)warp * (p.group + 1) * D;
    const int units = p.n * p.n_kv_heads;
    int k = 0;  // running piece index
    for (int u = 0; u < units; ++u) {
        const int np = unit_pieces(p, u);
        for (int pc = 0; pc < np; ++pc, ++k)
            if (k % (int)gridDim.x == (int)blockIdx.x && (k / (int)gridDim.x) % aw == warp)
                attend_piece<D>(p, layer, u, pc, q_w);
    }
}

// Greedy pick over one logits row: max under f32 total order, the last index
// among equal keys (sampling.rs:161-163; argmax_kernel's rule).
__device__ __forceinline__ int32_t total_key(float f) {
    const int32_t b = __float_as_int(f);
    return b < 0 ? (b ^ 0x7fffffff) : b;
}

__device__ void argmax_row(const Params& p, const Smem& L, uint8_t* sm, int j) {
    int32_t* sk = reinterpret_cast<int32_t*>(sm + L.red);
    int32_t* si = sk + kWarps;
    const float* row = p.logits + (size_t)j * p.vocab;
    int32_t bk = INT32_MIN, bi = -1;
    for (int c = threadIdx.x; c < p.vocab; c += kThreads) {
        const int32_t k = total_key(__ldcg(row + c));
        if (k >= bk) {
            bk = k;
            bi = c;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const int32_t k2 = __shfl_xor_sync(kFull, bk, o), i2 = __shfl_xor_sync(kFull, bi, o);
        if (k2 > bk || (k2 == bk && i2 > bi)) {
            bk = k2;
            bi = i2;
        }
    }
    if ((threadIdx.x & 31) == 0) {
        sk[threadIdx.x >> 5] = bk;
        si[threadIdx.x >> 5] = bi;
    }
    bar_compute();
    if (threadIdx.x == 0) {
        for (int w = 1; w < kWarps; w++)
            if (sk[w] > bk || (sk[w] == bk && si[w] > bi)) {
                bk = sk[w];
                bi = si[w];
            }
        p.ids[1 + j] = bi < 0 ? 0 : bi;
    }
    bar_compute();
}

// ---------------------------------------------------------------- kernel --

// One CTA of kCtaThreads per SM.  Its 17 warps put 5 on one of the SM's four
// sub-partitions, whose register file holds 16384: at most 96 registers a
// thread, which the launch bound makes the compiler keep to.
template <int D>
__global__ void __launch_bounds__(kCtaThreads, 1) decode_kernel(const __grid_constant__ Params p) {
    extern __shared__ __align__(128) uint8_t sm[];
    const Smem L(max(max(p.dim, p.q_dim), p.ffn));
    const int tid = threadIdx.x, warp = tid >> 5;
    const uint32_t full0 = smem_u32(sm), empty0 = full0 + 8 * kStages;
    volatile uint32_t* issued = reinterpret_cast<volatile uint32_t*>(sm + 16 * kStages);
    volatile uint32_t* prod_done = issued + 1;
    // flags[0]: the phase's matmuls went through; [1..4]: per warp group; [5]: grid barrier
    volatile int* flags = reinterpret_cast<volatile int*>(sm + 16 * kStages + 8);
    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(full0 + 8 * s) : "memory");
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(empty0 + 8 * s) : "memory");
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        *issued = 0;
        *prod_done = 0;
    }
    __syncthreads();
    if (warp == kWarps) {
        produce(p, sm);
        return;
    }
    // ---- compute warps ----
    uint32_t target = 0;  // thread 0: arrivals that pass the next grid barrier
    uint32_t c = 0;       // ring chunks consumed
    int off = 0;          // deal offset of the next phase
    bool ok = true;
    // embedding rows (quant.rs:464-490); the completion counters start at zero
    {
        const int total = p.n * p.dim, stride = gridDim.x * kThreads;
        for (int e = blockIdx.x * kThreads + tid; e < total; e += stride) {
            const int t = e / p.dim, j = e % p.dim;
            const size_t tok = (size_t)__ldg(p.tokens + t);
            p.x[e] = __fmul_rn(__half2float(p.emb_s[tok * (p.dim / kQK) + j / kQK]), (float)p.emb_q[tok * p.dim + j]);
        }
        if (blockIdx.x == 0)
            for (int g = tid; g < p.ffn / kQK + kMaxTokens * p.n_kv_heads; g += kThreads) p.sync[kSyncHeader + g] = 0u;
    }
    ok = grid_sync(p, target, flags + 5);
    // attention warps: their q buffers (and one K row) share the activation tile
    const int aw = min(kWarps, (int)((size_t)kMaxTokens * L.x_pitch / ((size_t)(p.group + 1) * D * 4)));
    // one matmul phase: this CTA's tiles, then the chunk count and the deal
    // offset move on (identically in the producer)
    auto matmul = [&](int ph, int n_tok) -> bool {
        const Mat m = phase_mat(p, ph);
        const bool r = consume(p, L, sm, ph, c, off, n_tok, flags);
        c += (uint32_t)(local_tiles(tiles_of(m), off) * chunks_of(m));
        off = (off + tiles_of(m)) % (int)gridDim.x;
        return r;
    };
    for (int l = 0; l < p.n_layers && ok; ++l) {
        const Layer& Ly = p.layers[l];
        // A: q|k|v
        if (tid == 0) flags[0] = 1;
        prologue_norm(p, L, sm, nullptr, Ly.attn_norm, p.n);
        zero_tail(L, sm, p.n, p.dim);
        bar_compute();
        ok = matmul(4 * l + kQkv, p.n) && grid_sync(p, target, flags + 5);
        if (!ok) break;
        // B: RoPE, append, attention
        attend_phase<D>(p, L, sm, l, aw);
        ok = grid_sync(p, target, flags + 5);
        if (!ok) break;
        // C: x += Wo . quant(att)
        if (tid == 0) flags[0] = 1;
        prologue_quant(p, L, sm);
        zero_tail(L, sm, p.n, p.q_dim);
        bar_compute();
        ok = matmul(4 * l + kO, p.n) && grid_sync(p, target, flags + 5);
        if (!ok) break;
        // D: gate|up, SiLU
        if (tid == 0) flags[0] = 1;
        prologue_norm(p, L, sm, nullptr, Ly.ffn_norm, p.n);
        zero_tail(L, sm, p.n, p.dim);
        bar_compute();
        ok = matmul(4 * l + kGateUp, p.n) && grid_sync(p, target, flags + 5);
        if (!ok) break;
        // E: x += Wdown . act
        if (tid == 0) flags[0] = 1;
        prologue_act(p, L, sm);
        zero_tail(L, sm, p.n, p.ffn);
        bar_compute();
        ok = matmul(4 * l + kDown, p.n) && grid_sync(p, target, flags + 5);
    }
    if (ok && p.n_want > 0) {
        if (tid == 0) flags[0] = 1;
        prologue_norm(p, L, sm, p.want, p.out_norm, p.n_want);
        zero_tail(L, sm, p.n_want, p.dim);
        bar_compute();
        ok = matmul(4 * p.n_layers, p.n_want);
        if (ok && p.argmax) {
            ok = grid_sync(p, target, flags + 5);
            if (ok)
                for (int j = blockIdx.x; j < p.n_want; j += gridDim.x) argmax_row(p, L, sm, j);
        }
    }
    if (!ok && tid == 0) {
        // Drain: the producer stops at the abort flag; wait (bounded) for the
        // last copies it issued before shared memory is released.
        const uint64_t t0 = global_ns();
        while (!*prod_done && global_ns() - t0 < kWaitNs) __nanosleep(1000);
        const uint32_t n_issued = *issued;
        const uint32_t first = n_issued > (uint32_t)kStages ? n_issued - kStages : 0u;
        for (uint32_t k = first; k < n_issued; ++k) {
            const uint64_t t1 = global_ns();
            while (!mbar_try_wait(full0 + 8 * (k % kStages), (k / kStages) & 1) && global_ns() - t1 < kDrainNs) {
            }
        }
    }
}

}  // namespace

bool supported(int dim, int q_dim, int ffn, int head_dim, int group, size_t* smem) {
    if (head_dim != 64 && head_dim != 128) return false;
    if (group < 1 || group > 8) return false;
    // every matrix width a multiple of 256 (16-byte scale rows per chunk), and
    // RMSNorm's dim/8 items a token in warps of one token, kNormItems a thread
    if (dim % 256 || q_dim % 256 || ffn % 256) return false;
    const int tpt = dim / 8;
    if (tpt < 32 || tpt > kThreads || kThreads % tpt) return false;
    if (kMaxTokens * tpt > kNormItems * kThreads) return false;
    const Smem L(std::max(std::max(dim, q_dim), ffn));
    if (L.total > 227 * 1024) return false;
    // the attention warps' q buffers (one warp at least) fit the activation tile
    if ((size_t)kMaxTokens * L.x_pitch < (size_t)(group + 1) * head_dim * 4) return false;
    if (smem) *smem = L.total;
    return true;
}

template <int D>
static cudaError_t launch_d(const Params& p, int grid, size_t smem, cudaStream_t st) {
    static bool attr_set[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!attr_set[dev]) {
        e = cudaFuncSetAttribute(decode_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        if (e != cudaSuccess) return e;
        attr_set[dev] = true;
    }
    void* args[] = {const_cast<Params*>(&p)};
    return cudaLaunchCooperativeKernel(reinterpret_cast<const void*>(&decode_kernel<D>), dim3(grid),
                                       dim3(kCtaThreads), args, smem, st);
}

int grid_size(const Params& p) {
    size_t smem = 0;
    if (!supported(p.dim, p.q_dim, p.ffn, p.head_dim, p.group, &smem)) return 0;
    int dev = 0, sms = 0, per_sm = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
    const void* fn = p.head_dim == 64 ? reinterpret_cast<const void*>(&decode_kernel<64>)
                                      : reinterpret_cast<const void*>(&decode_kernel<128>);
    if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024) != cudaSuccess) return 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kCtaThreads, smem) != cudaSuccess) return 0;
    return per_sm >= 1 ? sms : 0;
}

cudaError_t launch(const Params& p, int grid, cudaStream_t st) {
    size_t smem = 0;
    if (!supported(p.dim, p.q_dim, p.ffn, p.head_dim, p.group, &smem) || grid <= 0 || p.n < 1 ||
        p.n > kMaxTokens || p.n_want < 0 || p.n_want > p.n)
        return cudaErrorInvalidValue;
    return p.head_dim == 64 ? launch_d<64>(p, grid, smem, st) : launch_d<128>(p, grid, smem, st);
}

}  // namespace lldec
