// Persistent decode step of the Llama forward: Model::forward
// (model.rs:366-518) for up to 8 tokens, one per sequence, in one
// cooperative launch of one CTA per SM.
//
// The step's work is a chain of phases, each needing the whole output of the
// one before: per layer
//   A  RMSNorm + quantise of x, q|k|v = Wqkv . x          (model.rs:404-413)
//   B  RoPE, append of K/V into the paged pool, attention (model.rs:414-476)
//   C  quantise of att, x += Wo . att                     (model.rs:478-484)
//   D  RMSNorm + quantise of x, gate|up = Wgu . x, act = SiLU(gate) * up
//      (gate tile k is dealt with up tile k, so act's 16 columns are formed
//      in the registers that summed them)
//   E  quantise of act, x += Wdown . act                  (model.rs:486-498)
// then the output norm and matrix (model.rs:502-517) and the greedy pick.
// A grid-wide barrier separates the phases; nothing else does.
//
// Weights.  The rows of every matrix are cut into 16-row tiles, dealt
// round-robin to the CTAs with an offset that rotates from phase to phase so
// each CTA's total stays within a tile of the mean.  A producer warp per CTA
// streams the CTA's tiles -- all layers, in phase order -- through a 4-slot
// shared-memory ring with bulk copies (16 rows x up to 2048 columns and
// their f16 scales per slot), limited only by free slots: weights for the
// next phases arrive while the CTA waits at a barrier.  All 16 compute warps
// work on each chunk: each takes 4 of its 64 blocks and writes their
// products to a shared buffer, and 128 threads add them up in block order.
//
// Attention.  (token, KV head) unit u goes to CTA u % gridDim.x: its 16
// warps take the unit's blocks round-robin (online softmax, f32), and their
// (m, l, O) are merged in shared memory, so the attention output needs no
// grid barrier of its own.  For non-NeoX models RoPE is applied in the
// q|k|v matmul's epilogue (the partner row sits in the neighbouring lane
// group).
//
// Arithmetic.  Every matmul output is the reference's row_dot
// (quant.rs:418-421): one s8 mma per 32-wide block gives the exact int
// dot, and the owning warp adds the products (ws * xs) * dot block by block
// from 0.0f -- across chunks for matrices wider than 2048 columns.  The activation prologues use
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

// Shared-memory floats the attention of one unit takes from the activation
// tile: its q heads and new K row, then each warp's (m[8], l[8], O[8][D]).
__host__ __device__ constexpr size_t unit_floats(int group, int head_dim) {
    return (size_t)(group + 1) * head_dim + (size_t)kWarps * (16 + 8 * head_dim);
}

// Dynamic shared memory: header, ring slots, the activation tile (which the
// attention phase reuses for a unit's q heads and warp partials), its
// scales, a reduction scratch, the matmul's product buffer (a chunk's
// 64 blocks x 32 lanes x 4 products).
struct Smem {
    int x_pitch, xs_pitch;  // activation rows (int8 bytes), their scales (floats)
    size_t xq, xs, red, prod, total;
    __host__ __device__ Smem(int maxc, int group, int head_dim) {
        x_pitch = maxc + 32;
        xs_pitch = maxc / kQK + 4;
        xq = kHeader + (size_t)kStages * kSlotBytes;
        const size_t act = (size_t)kMaxTokens * x_pitch, att = unit_floats(group, head_dim) * 4;
        xs = xq + (act > att ? act : att);
        red = xs + (size_t)kMaxTokens * xs_pitch * 4;
        prod = red + kWarps * 32 * 4;
        total = prod + (size_t)(kChunk / kQK) * 32 * 16;
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

// Wait until the producer has issued ring chunk c (its `issued` count passed
// c); bounded like mbar_wait.  Only then is the slot's full barrier in the
// phase of chunk c or the one after, so its parity names chunk c alone: a
// warp may reach chunk c while the chunk kStages earlier in the same slot,
// owned by another warp, is still unread.
__device__ __forceinline__ bool wait_issued(const volatile uint32_t* issued, uint32_t c, const Params& p) {
    if (*issued > c) return true;
    const uint64_t t0 = global_ns();
    for (uint32_t it = 1;; ++it) {
        if (*issued > c) return true;
        if ((it & 63) == 0) {
            if (ld_volatile(p.sync + 2)) return false;
            if (global_ns() - t0 > kWaitNs) {
                raise_abort(p);
                return false;
            }
        }
    }
}

// The compute warps' barrier (the producer warp never takes part).
__device__ __forceinline__ void bar_compute() { asm volatile("bar.sync 1, %0;" ::"n"(kThreads) : "memory"); }

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
// The deal hands out units of one tile, or for gate|up of two: gate tile k
// (rows 16k..) and up tile k (rows ffn + 16k..), whose outputs are the gate
// and up values of the same 16 columns of act.
__device__ __forceinline__ int unit_tiles(const Params& p, int ph) {
    return ph != 4 * p.n_layers && (ph & 3) == kGateUp ? 2 : 1;
}
__device__ __forceinline__ int unit_tile(const Params& p, int ut, int u, int k) {
    return ut == 2 && k == 1 ? u + p.ffn / kRows : u;
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
        const int ut = unit_tiles(p, ph), units = tiles_of(m) / ut, nck = chunks_of(m);
        for (int it = 0; it < local_tiles(units, off) * ut && ok; ++it) {
            const int t = unit_tile(p, ut, first_tile(off) + (it / ut) * (int)gridDim.x, it % ut);
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
                if (lane == 0) {
                    __threadfence_block();  // the arrive above before the count
                    *issued = c + 1;
                }
            }
        }
        off = (off + units) % (int)gridDim.x;
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
// (and the thread's gamma slice) are issued before any arithmetic.
__device__ __noinline__ void prologue_norm(const Params& p, const Smem& L, uint8_t* sm, const int32_t* rows_idx,
                              const float* gamma, int n_tok) {
    const int cols = p.dim, tpt = cols / 8, nw = tpt / 32, items = n_tok * tpt;
    const int tid = threadIdx.x, lane = tid & 31;
    float* red = reinterpret_cast<float*>(sm + L.red);  // [8 tokens][nw] warp partials; totals at [256 + t]
    int8_t* xq = reinterpret_cast<int8_t*>(sm + L.xq);
    float* xs = reinterpret_cast<float*>(sm + L.xs);
    // a thread's items are columns (tid % tpt) of different tokens (tpt divides
    // the thread count): one gamma slice, loaded with x
    float gv[8];
    ltq8::load8(gamma + (tid % tpt) * 8, gv);
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
#pragma unroll
        for (int e = 0; e < 8; e++) v[k][e] = __fmul_rn(__fmul_rn(v[k][e], inv), gv[e]);
        ltq8::quant8_store(v[k], xq + (size_t)t * L.x_pitch + i * 8, xs + (size_t)t * L.xs_pitch + i / 4,
                           (i & 3) == 0, live);
    }
}

// Quantise of n rows of `cols` f32 (att, or act) into the activation tile:
// the QUANT prologue's mapping, 8 columns a lane, 32-column groups over 4
// consecutive lanes.  Token rows past n are left as they are: their
// products only reach outputs that are never written.
__device__ __noinline__ void prologue_quant(const Params& p, const Smem& L, uint8_t* sm, const float* src, int cols) {
    const int per_row = cols / 8, total = p.n * per_row;
    int8_t* xq = reinterpret_cast<int8_t*>(sm + L.xq);
    float* xs = reinterpret_cast<float*>(sm + L.xs);
    for (int base = 0; base < total; base += kThreads) {  // every lane takes every pass (group shuffles)
        const int item = base + (int)threadIdx.x;
        const bool live = item < total;
        const int t = live ? item / per_row : 0, c = live ? (item % per_row) * 8 : 0;
        float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        if (live) load8_cg(src + (size_t)t * cols + c, v);
        ltq8::quant8_store(v, xq + (size_t)t * L.x_pitch + c, xs + (size_t)t * L.xs_pitch + c / kQK,
                           (threadIdx.x & 3) == 0, live);
    }
}

// -------------------------------------------------------------- barrier ---

// Grid-wide barrier of the compute warps.  The arrival count rises through
// the launch (the host zeroes it before): barrier k of the launch is passed
// once it reaches k * gridDim.x.  Thread 0 of each CTA keeps that target.
__device__ __noinline__ bool grid_sync(const Params& p, uint32_t& target, volatile int* flag) {
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

// Tile outputs are held by the summing threads t < 128: thread t has row
// g = t / 16 (+ 8 when bit 1 of t is set) and token 2 ((t / 4) % 4) + t % 2
// of the tile, so the RoPE partner row r ^ 1 (rows g and g ^ 1) sits in
// thread t ^ 16 of the same warp.
__device__ __forceinline__ int out_row(int t) { return (t >> 4) + 8 * ((t >> 1) & 1); }
__device__ __forceinline__ int out_tok(int t) { return 2 * ((t >> 2) & 3) + (t & 1); }

// RoPE of a q|k value held by summing thread t, non-NeoX: row r pairs with
// row r ^ 1 (rope_split_kernel's arithmetic).  Every lane of the warp calls
// it (the shuffle); only rows in the q|k part inside the rotary columns
// change.
__device__ __forceinline__ float rope_epilogue(const Params& p, float v, int r, int tok, int n_tok) {
    const float other = __shfl_xor_sync(kFull, v, 16);
    const int c = r % p.head_dim;
    if (r >= p.q_dim + p.kv_dim || c >= 2 * p.half || tok >= n_tok) return v;
    const float* sc = p.sincos + ((size_t)tok * p.half + (c >> 1)) * 2;
    const float sn = __ldg(sc), cs = __ldg(sc + 1);
    return (c & 1) == 0 ? __fsub_rn(__fmul_rn(v, cs), __fmul_rn(other, sn))   // x0 cos - x1 sin
                        : __fadd_rn(__fmul_rn(other, sn), __fmul_rn(v, cs));  // x0 sin + x1 cos
}

// int32 -> f32 for |d| < 2^22, exactly __int2float_rn(d): d added into the
// mantissa of 1.5 * 2^23, which is then subtracted.  An s8 block dot is at
// most 32 * 128 * 128 = 2^19 in size.
__device__ __forceinline__ float small_int_to_float(int d) {
    return __fsub_rn(__int_as_float(0x4B400000 + d), 12582912.0f);
}

// This CTA's tiles of phase ph, one after the other, every chunk by all 16
// compute warps.  Warp w takes blocks [w * bpw, (w + 1) * bpw) of the chunk:
// per 32-wide block one s8 mma gives the exact int dots of 16 rows x 8
// tokens, and the lane writes the four products (ws * xs) * dot of its
// fragment to the product buffer, then hands the slot back to the producer.
// After a CTA barrier the summing threads (t < 128, one output each) add
// the chunk's products block by block onto their running sums -- from 0.0f
// at the tile's first block, in block order across chunks: row_dot's order.
// After the last chunk they write the tile's outputs (q|k rows RoPE'd first
// for non-NeoX models); gate|up units end with act = SiLU(gate) * up of
// their 16 columns.  Returns false when a wait gave up (every warp of the
// CTA returns together).
__device__ __noinline__ bool consume(const Params& p, const Smem& L, uint8_t* sm, int ph, uint32_t c_base, int off,
                                     int n_tok, volatile int* flags) {
    const Mat m = phase_mat(p, ph);
    const int kind = ph == 4 * p.n_layers ? 4 : (ph & 3);
    const int nck = chunks_of(m);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, q = lane & 3;
    const uint32_t full0 = smem_u32(sm), empty0 = full0 + 8 * kStages;
    const volatile uint32_t* issued = reinterpret_cast<const volatile uint32_t*>(sm + 16 * kStages);
    const int8_t* xq = reinterpret_cast<const int8_t*>(sm + L.xq);
    const float* xs = reinterpret_cast<const float*>(sm + L.xs);
    float4* prod = reinterpret_cast<float4*>(sm + L.prod);  // [block][lane]
    const float* prod_f = reinterpret_cast<const float*>(sm + L.prod);
    const int ut = unit_tiles(p, ph), n_local = local_tiles(tiles_of(m) / ut, off) * ut;
    float gate = 0.0f;  // summing threads, gate|up: the gate value of the unit's first tile
    for (int i = 0; i < n_local; ++i) {
        const int u = first_tile(off) + (i / ut) * (int)gridDim.x, t = unit_tile(p, ut, u, i % ut);
        float acc = 0.0f;  // summing threads: the output's running row_dot
        for (int j = 0; j < nck; ++j) {
            const uint32_t c = c_base + (uint32_t)(i * nck + j);
            const int s = c % kStages;
            int w_ok = 1;
            if (lane == 0) w_ok = wait_issued(issued, c, p) && mbar_wait(full0 + 8 * s, (c / kStages) & 1, p);
            w_ok = __shfl_sync(kFull, w_ok, 0);
            const int k0 = j * kChunk, nb = min(kChunk, m.cols - k0) / kQK, kb0 = k0 / kQK;
            if (w_ok) {
                (void)mbar_try_wait(full0 + 8 * s, (c / kStages) & 1);  // every lane observes the completed phase
                const uint8_t* w = sm + kHeader + (size_t)s * kSlotBytes;
                const __half* ws = reinterpret_cast<const __half*>(w + kRows * kWPitch);
                const int bpw = (nb + kWarps - 1) / kWarps, b0 = warp * bpw, b1 = min(nb, b0 + bpw);
                const uint8_t* wa = w + (size_t)g * kWPitch + 8 * q;
                const uint8_t* wb = w + (size_t)(g + 8) * kWPitch + 8 * q;
                const int8_t* xb = xq + (size_t)g * L.x_pitch + 32 * kb0 + 8 * q;
                const float* xsa_p = xs + (2 * q) * L.xs_pitch + kb0;
                const float* xsc_p = xs + (2 * q + 1) * L.xs_pitch + kb0;
#pragma unroll 4
                for (int b = b0; b < b1; ++b) {
                    const uint2 A0 = *reinterpret_cast<const uint2*>(wa + 32 * b);
                    const uint2 A1 = *reinterpret_cast<const uint2*>(wb + 32 * b);
                    const uint2 B = *reinterpret_cast<const uint2*>(xb + 32 * b);
                    int d[4];
                    ltq8::mma_s8(d, A0.x, A1.x, A0.y, A1.y, B.x, B.y);
                    const float wsa = __half2float(ws[g * (kSPitch / 2) + b]);
                    const float wsb = __half2float(ws[(g + 8) * (kSPitch / 2) + b]);
                    const float xsa = xsa_p[b], xsc = xsc_p[b];
                    prod[b * 32 + lane] = make_float4(__fmul_rn(__fmul_rn(wsa, xsa), small_int_to_float(d[0])),
                                                      __fmul_rn(__fmul_rn(wsa, xsc), small_int_to_float(d[1])),
                                                      __fmul_rn(__fmul_rn(wsb, xsa), small_int_to_float(d[2])),
                                                      __fmul_rn(__fmul_rn(wsb, xsc), small_int_to_float(d[3])));
                }
            } else if (lane == 0) {
                flags[0] = 0;  // this warp gave up: the CTA leaves after the barrier
            }
            __syncwarp();  // every lane has read the slot
            if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(empty0 + 8 * s) : "memory");
            bar_compute();
            if (!flags[0]) return false;
            if (tid < 128) {  // output (lane tid / 4, fragment element tid % 4) of the products
                const float* pp = prod_f + tid;
#pragma unroll 8
                for (int b = 0; b < nb; ++b) acc = __fadd_rn(acc, pp[b * 128]);
            }
            bar_compute();  // the product buffer is free again
        }
        if (tid < 128) {
            const int r = t * kRows + out_row(tid), tok = out_tok(tid);
            float v = acc;
            if (kind == kQkv && !p.neox) v = rope_epilogue(p, v, r, tok, n_tok);
            if (kind == kGateUp) {
                if (i % ut == 0) {
                    gate = v;
                } else if (tok < n_tok) {  // act = SiLU(gate) * up (silu_q8_kernel's arithmetic: exp
                                           // rounded once from double precision)
                    const float e = (float)exp(-(double)gate);
                    p.act[(size_t)tok * p.ffn + u * kRows + out_row(tid)] =
                        __fmul_rn(__fdiv_rn(gate, __fadd_rn(1.0f, e)), v);
                }
            } else if (r < m.rows && tok < n_tok) {
                if (kind == kQkv) {
                    p.qkv[(size_t)tok * p.qkv_rows + r] = v;
                } else if (kind == 4) {
                    p.logits[(size_t)tok * p.vocab + r] = v;
                } else {  // o, down: residual add into x (model.rs:484, 498)
                    float* o = p.x + (size_t)tok * p.dim + r;
                    *o = __fadd_rn(__ldcg(o), v);
                }
            }
        }
    }
    bar_compute();
    return flags[0] != 0;
}

// --------------------------------------------------------- attention -----

// RoPE of the head-aligned range [base, base + count) of a token's q|k row
// into dst[0, count), by one warp: each rotated pair (non-NeoX: 2i, 2i+1;
// NeoX: i, i + half; model.rs:291-308) once, with rope_split_kernel's
// arithmetic, columns past the rotary part copied.  Four items a lane per
// round, all their loads issued before the arithmetic.
__device__ __noinline__ void rope_range(const Params& p, const float* row, const float* sc, int base, int count, float* dst) {
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

// f16 tensor-core helpers of the attention phase.
__device__ __forceinline__ void mma_f16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Transpose of an 8 x 8 f16 matrix held one 32-bit pair a lane (row
// lane / 4, columns 2 (lane % 4) + {0, 1}).
__device__ __forceinline__ uint32_t transpose8(uint32_t x) {
    uint32_t y;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
    return y;
}

__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }

// (a, b) as an f16 pair `hi` plus the f16 pair of what rounding left out,
// so that hi + lo carries about 22 bits of each value.
__device__ __forceinline__ void split_h2(float a, float b, uint32_t& hi, uint32_t& lo) {
    const __half2 h = __floats2half2_rn(a, b);
    const float2 f = __half22float2(h);
    hi = h2_bits(h);
    lo = h2_bits(__floats2half2_rn(a - f.x, b - f.y));
}

__device__ __forceinline__ uint32_t word_of(const uint4& v, int w) {
    return w == 0 ? v.x : w == 1 ? v.y : w == 2 ? v.z : v.w;
}

// One warp's share of a unit's attention: blocks warp, warp + 16, ... of the
// unit, online softmax in f32 over exp2 of log2e-scaled scores, both
// products on the tensor cores (f16 in, f32 accumulate).
//
// Scores.  S^T (16 positions x 8 heads) = K (16 x D) . Q^T, K straight from
// the pool as the A operand: lane (g, q) loads the 16-byte chunks 4j + q of
// rows g and g + 8, and k-step (j, u) takes words 2u, 2u + 1 of them, so
// the step's k index 2q + e stands for column 8 (4j + q) + 4u + e and
// 2q + 8 + e for 8 (4j + q) + 4u + 2 + e; the B operand (the q heads,
// heads past the group zero) is read with the same column order.  q is f32:
// it goes in as an f16 pair hi + lo, two mma per step.
//
// Output.  O^T (D x 8 heads) += V^T (D x 16 positions) . P^T.  The 8 x 8
// pieces of V that lane (g, q) loads the same way (word w of chunk 4j + q
// of rows g and g + 8) are transposed in registers into V^T's A fragments:
// m-tile (j, v) has rows 8 (4j + r/2) + 4v + 2 (r / 8) + r % 2 ... written
// out below as dim_of.  P^T's B fragments are the score fragments rounded to
// f16 (hi + lo) and transposed.  A block's table entry is read one block
// ahead; for D = 64 its V rows are loaded together with its K rows.
template <int D>
__device__ __forceinline__ void attend_blocks(const Params& p, const float* qs, const uint16_t* pool_l,
                                              const int32_t* trow, int h, int pos, int nb, float* mine) {
    constexpr int NJ = D / 32;  // chunk groups: chunk 4j + q of a row per lane
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, q = lane & 3;
    const int G = p.group, Hkv = p.n_kv_heads;
    // B fragments of the q heads for k-step (j, u): head g, columns 8 (4j + q) + 4u + [0, 4)
    auto q_frag = [&](int j, int u, uint32_t (&hi)[2], uint32_t (&lo)[2]) {
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (g < G) v = *reinterpret_cast<const float4*>(qs + g * D + 8 * (4 * j + q) + 4 * u);
        split_h2(v.x, v.y, hi[0], lo[0]);
        split_h2(v.z, v.w, hi[1], lo[1]);
    };
    uint32_t qh[D == 64 ? NJ : 1][2][2], ql[D == 64 ? NJ : 1][2][2];
    if constexpr (D == 64) {
#pragma unroll
        for (int j = 0; j < NJ; ++j)
#pragma unroll
            for (int u = 0; u < 2; ++u) q_frag(j, u, qh[j][u], ql[j][u]);
    }
    float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.0f, 0.0f};  // heads 2q, 2q + 1
    float o[NJ][2][4];
#pragma unroll
    for (int j = 0; j < NJ; ++j)
#pragma unroll
        for (int v = 0; v < 2; ++v)
#pragma unroll
            for (int e = 0; e < 4; ++e) o[j][v][e] = 0.0f;
    int blk = warp < nb ? __ldg(trow + warp) : 0;
    for (int b = warp; b < nb; b += kWarps) {
        const int blk_next = b + kWarps < nb ? __ldg(trow + b + kWarps) : 0;
        const uint16_t* kt = pool_l + ((size_t)blk * Hkv + h) * 2 * ltkv::kBlock * D;
        const uint16_t* vt = kt + ltkv::kBlock * D;
        uint4 ka[NJ], kb[NJ], va[NJ], vb[NJ];
#pragma unroll
        for (int j = 0; j < NJ; ++j) {
            ka[j] = *reinterpret_cast<const uint4*>(kt + ltkv::chunk_off(4 * j + q, g));
            kb[j] = *reinterpret_cast<const uint4*>(kt + ltkv::chunk_off(4 * j + q, g + 8));
        }
        auto load_v = [&]() {
#pragma unroll
            for (int j = 0; j < NJ; ++j) {
                va[j] = *reinterpret_cast<const uint4*>(vt + ltkv::chunk_off(4 * j + q, g));
                vb[j] = *reinterpret_cast<const uint4*>(vt + ltkv::chunk_off(4 * j + q, g + 8));
            }
        };
        if constexpr (D == 64) load_v();  // registers allow V in flight with K
        float s[4] = {0.0f, 0.0f, 0.0f, 0.0f};  // S^T: [position g | g + 8][head 2q | 2q + 1]
#pragma unroll
        for (int j = 0; j < NJ; ++j)
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                const uint32_t a[4] = {word_of(ka[j], 2 * u), word_of(kb[j], 2 * u), word_of(ka[j], 2 * u + 1),
                                       word_of(kb[j], 2 * u + 1)};
                if constexpr (D == 64) {
                    mma_f16(s, a, qh[j][u][0], qh[j][u][1]);
                    mma_f16(s, a, ql[j][u][0], ql[j][u][1]);
                } else {
                    uint32_t hi[2], lo[2];
                    q_frag(j, u, hi, lo);
                    mma_f16(s, a, hi[0], hi[1]);
                    mma_f16(s, a, lo[0], lo[1]);
                }
            }
        if constexpr (D != 64) load_v();
        const int p0 = b * ltkv::kBlock + g;
        float pr[4];
        float al[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            const float s0 = p0 <= pos ? s[e] * p.scale_log2 : -INFINITY;
            const float s1 = p0 + 8 <= pos ? s[2 + e] * p.scale_log2 : -INFINITY;
            float bm = fmaxf(s0, s1);
            bm = fmaxf(bm, __shfl_xor_sync(kFull, bm, 4));
            bm = fmaxf(bm, __shfl_xor_sync(kFull, bm, 8));
            bm = fmaxf(bm, __shfl_xor_sync(kFull, bm, 16));
            const float mn = fmaxf(m[e], bm);  // finite: position 0 of every block is at or before pos
            al[e] = exp2f(m[e] - mn);
            pr[e] = exp2f(s0 - mn);
            pr[2 + e] = exp2f(s1 - mn);
            float bs = pr[e] + pr[2 + e];
            bs += __shfl_xor_sync(kFull, bs, 4);
            bs += __shfl_xor_sync(kFull, bs, 8);
            bs += __shfl_xor_sync(kFull, bs, 16);
            l[e] = l[e] * al[e] + bs;
            m[e] = mn;
        }
        // P^T's B fragments: [positions 2q, 2q + 1 | 8 + 2q, 9 + 2q][head g], hi and lo
        uint32_t h0, l0, h1, l1;
        split_h2(pr[0], pr[1], h0, l0);
        split_h2(pr[2], pr[3], h1, l1);
        h0 = transpose8(h0);
        l0 = transpose8(l0);
        h1 = transpose8(h1);
        l1 = transpose8(l1);
#pragma unroll
        for (int j = 0; j < NJ; ++j)
#pragma unroll
            for (int v = 0; v < 2; ++v) {
                o[j][v][0] *= al[0];
                o[j][v][1] *= al[1];
                o[j][v][2] *= al[0];
                o[j][v][3] *= al[1];
                const uint32_t a[4] = {transpose8(word_of(va[j], 2 * v)), transpose8(word_of(va[j], 2 * v + 1)),
                                       transpose8(word_of(vb[j], 2 * v)), transpose8(word_of(vb[j], 2 * v + 1))};
                mma_f16(o[j][v], a, h0, h1);
                mma_f16(o[j][v], a, l0, l1);
            }
        blk = blk_next;
    }
    // m = -inf, l = 0 for a warp without blocks: it drops out of the merge
#pragma unroll
    for (int e = 0; e < 2; ++e) {
        const int hd = 2 * q + e;
        if (g == 0 && hd < G) {
            mine[hd] = m[e];
            mine[8 + hd] = l[e];
        }
    }
    // O^T fragment rows: row g of m-tile (j, v) is column 8 (4j + g/2) + 4v + g%2, row g + 8 that + 2
#pragma unroll
    for (int j = 0; j < NJ; ++j)
#pragma unroll
        for (int v = 0; v < 2; ++v) {
            const int d = 8 * (4 * j + g / 2) + 4 * v + (g & 1);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int hd = 2 * q + (e & 1);
                if (hd < G) mine[16 + hd * D + d + 2 * (e >> 1)] = o[j][v][e];
            }
        }
}

// Attention of (token, KV head) unit u by the whole CTA (model.rs:414-476).
// The unit's q heads and its new K row go to shared memory: RoPE'd here
// for NeoX models (rows half a head apart lie in different tiles of the
// q|k|v matmul), as the matmul's epilogue left them otherwise.  The warp
// that owns the last block writes the new K/V row into the token's pool
// cell (f16, the write kernel's layout and conversion) before it reads the
// block.  Every warp attends its blocks; the warps' (m, l, O) are merged in
// shared memory, one output element a thread, and written to att.
template <int D>
__device__ __noinline__ void attend_unit(const Params& p, const Smem& L, uint8_t* sm, int layer, int u) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = p.group, Hkv = p.n_kv_heads;
    const int t = u / Hkv, h = u % Hkv;
    const float* row = p.qkv + (size_t)t * p.qkv_rows;
    const int seq = __ldg(p.seq + t), pos = __ldg(p.pos + t);
    const int nb = pos / ltkv::kBlock + 1;
    const int32_t* trow = p.tables + (size_t)seq * p.max_blocks;
    uint16_t* pool_l = p.pool + (size_t)layer * p.layer_elems;
    float* qs = reinterpret_cast<float*>(sm + L.xq);  // [G][D] q heads, then [D] the new K row
    float* part = qs + (size_t)(G + 1) * D;           // [kWarps][16 + 8 * D]
    if (p.neox) {
        const float* sc = p.sincos + (size_t)t * p.half * 2;
        if (warp < G) rope_range(p, row, sc, (h * G + warp) * D, D, qs + warp * D);
        else if (warp == G) rope_range(p, row, sc, p.q_dim + h * D, D, qs + G * D);
    } else {
        for (int e = tid; e < G * D / 4; e += kThreads)
            reinterpret_cast<float4*>(qs)[e] = __ldcg(reinterpret_cast<const float4*>(row + h * G * D) + e);
        for (int e = tid; e < D / 4; e += kThreads)
            reinterpret_cast<float4*>(qs + G * D)[e] = __ldcg(reinterpret_cast<const float4*>(row + p.q_dim + h * D) + e);
    }
    bar_compute();
    if (warp == (nb - 1) % kWarps) {
        if (lane < 2 * (D / 8)) {  // the new row of (token, head): K roped, V as is
            const int blk = __ldg(trow + pos / ltkv::kBlock), slot = pos % ltkv::kBlock;
            uint16_t* tile = pool_l + ((size_t)blk * Hkv + h) * 2 * ltkv::kBlock * D;
            const int kvsel = lane / (D / 8), c = lane % (D / 8);
            float x[8];
            if (kvsel == 0) {
#pragma unroll
                for (int e = 0; e < 8; ++e) x[e] = qs[G * D + c * 8 + e];
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
        __syncwarp();  // the new row is visible to the whole warp before it reads the block
    }
    attend_blocks<D>(p, qs, pool_l, trow, h, pos, nb, part + (size_t)warp * (16 + 8 * D));
    bar_compute();
    const int nw = min(kWarps, nb);
    for (int o = tid; o < G * D; o += kThreads) {
        const int gq = o / D, d = o % D;
        float mx = -INFINITY;
        for (int w = 0; w < nw; w++) mx = fmaxf(mx, part[w * (16 + 8 * D) + gq]);
        float ls = 0.0f, os = 0.0f;
        for (int w = 0; w < nw; w++) {
            const float* pw = part + w * (16 + 8 * D);
            const float f = exp2f(pw[gq] - mx);
            ls += pw[8 + gq] * f;
            os += pw[16 + gq * D + d] * f;
        }
        p.att[(size_t)t * p.q_dim + (size_t)(h * G + gq) * D + d] = os / ls;
    }
    bar_compute();  // the next unit reuses qs and part
}

// The attention phase: unit u = t * n_kv_heads + h to CTA u % gridDim.x.
template <int D>
__device__ void attend_phase(const Params& p, const Smem& L, uint8_t* sm, int layer) {
    for (int u = blockIdx.x; u < p.n * p.n_kv_heads; u += gridDim.x) attend_unit<D>(p, L, sm, layer, u);
}

// Greedy pick over one logits row: max under f32 total order, the last index
// among equal keys (sampling.rs:161-163; argmax_kernel's rule).
__device__ __forceinline__ int32_t total_key(float f) {
    const int32_t b = __float_as_int(f);
    return b < 0 ? (b ^ 0x7fffffff) : b;
}

__device__ __noinline__ void argmax_row(const Params& p, const Smem& L, uint8_t* sm, int j) {
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
    const Smem L(max(max(p.dim, p.q_dim), p.ffn), p.group, D);
    const int tid = threadIdx.x, warp = tid >> 5;
    const uint32_t full0 = smem_u32(sm), empty0 = full0 + 8 * kStages;
    volatile uint32_t* issued = reinterpret_cast<volatile uint32_t*>(sm + 16 * kStages);
    volatile uint32_t* prod_done = issued + 1;
    // flags[0]: the phase's matmuls went through; [5]: grid barrier
    volatile int* flags = reinterpret_cast<volatile int*>(sm + 16 * kStages + 8);
    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(full0 + 8 * s) : "memory");
            asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(empty0 + 8 * s), "n"(kWarps) : "memory");
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
    // embedding rows (quant.rs:464-490)
    {
        const int total = p.n * p.dim, stride = gridDim.x * kThreads;
        for (int e = blockIdx.x * kThreads + tid; e < total; e += stride) {
            const int t = e / p.dim, j = e % p.dim;
            const size_t tok = (size_t)__ldg(p.tokens + t);
            p.x[e] = __fmul_rn(__half2float(p.emb_s[tok * (p.dim / kQK) + j / kQK]), (float)p.emb_q[tok * p.dim + j]);
        }
    }
    ok = grid_sync(p, target, flags + 5);
    // one matmul phase: this CTA's tiles, then the chunk count and the deal
    // offset move on (identically in the producer)
    auto matmul = [&](int ph, int n_tok) -> bool {
        const Mat m = phase_mat(p, ph);
        const bool r = consume(p, L, sm, ph, c, off, n_tok, flags);
        const int ut = unit_tiles(p, ph);
        c += (uint32_t)(local_tiles(tiles_of(m) / ut, off) * ut * chunks_of(m));
        off = (off + tiles_of(m) / ut) % (int)gridDim.x;
        return r;
    };
    for (int l = 0; l < p.n_layers && ok; ++l) {
        const Layer& Ly = p.layers[l];
        // A: q|k|v
        if (tid == 0) flags[0] = 1;
        prologue_norm(p, L, sm, nullptr, Ly.attn_norm, p.n);
        bar_compute();
        ok = matmul(4 * l + kQkv, p.n) && grid_sync(p, target, flags + 5);
        if (!ok) break;
        // B: RoPE, append, attention
        attend_phase<D>(p, L, sm, l);
        ok = grid_sync(p, target, flags + 5);
        if (!ok) break;
        // C: x += Wo . quant(att)
        if (tid == 0) flags[0] = 1;
        prologue_quant(p, L, sm, p.att, p.q_dim);
        bar_compute();
        ok = matmul(4 * l + kO, p.n) && grid_sync(p, target, flags + 5);
        if (!ok) break;
        // D: gate|up, act = SiLU(gate) * up
        if (tid == 0) flags[0] = 1;
        prologue_norm(p, L, sm, nullptr, Ly.ffn_norm, p.n);
        bar_compute();
        ok = matmul(4 * l + kGateUp, p.n) && grid_sync(p, target, flags + 5);
        if (!ok) break;
        // E: x += Wdown . quant(act)
        if (tid == 0) flags[0] = 1;
        prologue_quant(p, L, sm, p.act, p.ffn);
        bar_compute();
        ok = matmul(4 * l + kDown, p.n) && grid_sync(p, target, flags + 5);
    }
    if (ok && p.n_want > 0) {
        if (tid == 0) flags[0] = 1;
        prologue_norm(p, L, sm, p.want, p.out_norm, p.n_want);
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
    const Smem L(std::max(std::max(dim, q_dim), ffn), group, head_dim);
    if (L.total > 227 * 1024) return false;
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
