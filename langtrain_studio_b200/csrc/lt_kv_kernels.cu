// sm_100a kernels of the paged KV-cache path.
//
//   kv_write_kernel      K1  KvCache::write (kv.rs:123-131): f32/f16 rows -> f16 pool cells
//   paged_attn_kernel    K2  attention closure of Model::forward (model.rs:431-476)
//   apply_plan_kernel    K3/K4  whole-block copies (copy-on-write kv.rs:99-110,
//                            compaction moves) + block-table scatter
//   rows_kernel              KvCache::rows (kv.rs:135-150) gather, for parity/debug
//
// Pool layout (per layer): f16 [block][kv_head][2 (K,V)][D/64][16 slots][64].
// Within each 16 x 64 sub-tile, the 16-byte chunk c of the row of slot s
// sits at chunk position c ^ (s & 7) (the 128-byte swizzle of the tensor-core
// operand layouts): one (block, head) K+V tile is a contiguous 4*D*16-byte run
// whose bulk-copied shared-memory image is bank-conflict free for ldmatrix
// and, 64-wide sub-tile by sub-tile, a valid tcgen05 operand.
//
// Q8_0 pool (LT_KV_Q8_0): one 34*D-byte tile per (block, head) -- K int8
// row-major with 128-byte-swizzled 16-byte runs, V int8 transposed (one
// 16-byte run per column), then the f16 scales of K and of V, one per
// (32-value group, slot).  Inside every 16-byte run the 16 entries sit in the
// order of the mma.sync B-fragment (pos(i) below), so one ldmatrix of the
// int8 bytes hands each lane exactly the four values of its fragment.
#include <cuda_fp16.h>
#include <stdint.h>

#include <algorithm>

#include "lt_kv_internal.h"
#include "lt_kv_layout.cuh"

namespace ltkv {
namespace {

constexpr int kWarps = 4;                         // warps per attention CTA
constexpr int kStages = 3;                        // bulk-copy stages per warp (f16 tiles)
constexpr int kStagesQ8 = 5;                      // the same for Q8_0 tiles (about half the bytes;
                                                  // 5 keeps two group-8 CTAs per SM)
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // bounded mbarrier wait: 2 s
constexpr unsigned kFull = 0xffffffffu;

// ------------------------------------------------------------- helpers ----

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
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

// Wait for `parity` of an mbarrier, giving up after kWaitLimitNs.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 15u) == 0 && global_ns() - t0 > kWaitLimitNs) return false;
    }
}

// Non-multicast 1-D bulk copy global -> this CTA's shared memory.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(bar)
        : "memory");
}

__device__ __forceinline__ void st_release_gpu(uint32_t* p, uint32_t v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// System scope (another GPU over NVLink reads or writes the word).
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

__device__ __forceinline__ void st_relaxed_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ uint32_t atom_add_acq_rel_gpu(uint32_t* p, uint32_t v) {
    uint32_t old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}


// Wait until *flag == epoch, giving up after limit_ns.
__device__ __forceinline__ int wait_flag_bounded(const uint32_t* flag, uint32_t epoch,
                                                 uint64_t limit_ns = kWaitLimitNs) {
    if (ld_acquire_gpu(flag) == epoch) return 1;
    const uint64_t t0 = global_ns();
    for (;;) {
        __nanosleep(64);
        if (ld_acquire_gpu(flag) == epoch) return 1;
        if (global_ns() - t0 > limit_ns) return 0;
    }
}

// A block id read from a block table.  Builds with LT_BOUNDS_CHECK test it
// against the pool (n_blocks > 0), and so does every build when `check` is
// set (tables the caller owns): a bad id raises kErrBounds and block 0
// stands in for it, so the access stays inside the pool and only the
// output is wrong (and reported).  Otherwise the host bookkeeping that
// wrote the table is trusted.
__device__ __forceinline__ int checked_block(int b, int n_blocks, int32_t* err, bool check = false) {
#ifdef LT_BOUNDS_CHECK
    check = true;
#endif
    if (check && n_blocks > 0 && (unsigned)b >= (unsigned)n_blocks) {
        atomicOr(err, kErrBounds);
        return 0;
    }
    return b;
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

// D(16x8 f32) += A(16x16 f16, row) * B(16x8 f16, col)
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// 2^x on the SFU (hardware instruction; relative error ~2^-22).
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }

// Load 8 consecutive input values (f32 or f16) and return them as 8 f16.
__device__ __forceinline__ uint4 load8_as_f16(const void* base, size_t idx, int in_f32) {
    uint4 r;
    if (in_f32) {
        const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(base) + idx);
        const float4 a = __ldg(p), b = __ldg(p + 1);
        r.x = f32_to_f16_ref(a.x) | (uint32_t(f32_to_f16_ref(a.y)) << 16);
        r.y = f32_to_f16_ref(a.z) | (uint32_t(f32_to_f16_ref(a.w)) << 16);
        r.z = f32_to_f16_ref(b.x) | (uint32_t(f32_to_f16_ref(b.y)) << 16);
        r.w = f32_to_f16_ref(b.z) | (uint32_t(f32_to_f16_ref(b.w)) << 16);
    } else {
        r = __ldg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(base) + idx));
    }
    return r;
}

// ---------------------------------------------------------- Q8_0 tile ----
__host__ __device__ constexpr int q8_tile_bytes(int D) { return 34 * D; }

// Position of entry i (0..15) inside a 16-byte run: the order
// 0,1,8,9, 2,3,10,11, 4,5,12,13, 6,7,14,15, so bytes 4t..4t+3 of a run hold
// entries 2t, 2t+1, 2t+8, 2t+9 -- one lane's part of an m16n8k16 B fragment.
__device__ __forceinline__ int q8_pos(int i) { return ((i & 7) >> 1) * 4 + ((i >> 3) << 1) + (i & 1); }

// Byte offset of the 16-byte run of K values 16k..16k+15 of slot s: run
// L = s*D/16 + k of the row-major K part, 128-byte lines swizzled by line.
template <int D>
__device__ __forceinline__ int q8_krun(int s, int k) {
    const int L = s * (D / 16) + k;
    return ((L >> 3) << 7) + (((L & 7) ^ ((L >> 3) & 7)) << 4);
}

// Four int8 (one 32-bit word) -> two f16x2, exactly: each biased byte
// b = x + 128 becomes the f16 1024 + b (exponent 10, b in the mantissa),
// then 1152 is subtracted.
__device__ __forceinline__ void i8x4_to_f16x2(uint32_t w, uint32_t& lo, uint32_t& hi) {
    const uint32_t u = w ^ 0x80808080u;
    const __half2 bias = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));
    uint32_t a = __byte_perm(u, 0x64646464u, 0x5140), b = __byte_perm(u, 0x64646464u, 0x7362);
    const __half2 ha = __hsub2(*reinterpret_cast<__half2*>(&a), bias);
    const __half2 hb = __hsub2(*reinterpret_cast<__half2*>(&b), bias);
    lo = h2_bits(ha);
    hi = h2_bits(hb);
}

// Load 8 consecutive input values (f32, or f16 widened exactly).
__device__ __forceinline__ void load8_f32(const void* base, size_t idx, int in_f32, float (&x)[8]) {
    if (in_f32) {
        const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(base) + idx);
        const float4 a = __ldg(p), b = __ldg(p + 1);
        x[0] = a.x, x[1] = a.y, x[2] = a.z, x[3] = a.w, x[4] = b.x, x[5] = b.y, x[6] = b.z, x[7] = b.w;
    } else {
        const uint4 r = __ldg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(base) + idx));
        const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[j]));
            x[2 * j] = f.x;
            x[2 * j + 1] = f.y;
        }
    }
}

// One 32-value group held as 8 values by each of the lanes 4j..4j+3 (all 32
// lanes call this): the engine's int8 quantiser (quant.rs:785-795) --
// d = max|x| / 127 (NaN ignored), q = round(x / d) half away from zero via
// the reciprocal id, saturating to int8, NaN -> 0.  Returns d; the lane's
// eight values come back packed in w0 (values 0-3) and w1 (4-7).
__device__ __forceinline__ float q8_quant8(const float (&x)[8], uint32_t& w0, uint32_t& w1) {
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(x[i]));
    amax = fmaxf(amax, __shfl_xor_sync(kFull, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(kFull, amax, 2));
    const float d = amax / 127.0f;
    const float id = d > 0.f ? 1.0f / d : 0.f;
    uint32_t w[2] = {0u, 0u};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float r = roundf(x[i] * id);
        const int q = r != r ? 0 : r >= 127.f ? 127 : r <= -128.f ? -128 : (int)r;
        w[i >> 2] |= (uint32_t)(q & 0xff) << (8 * (i & 3));
    }
    w0 = w[0];
    w1 = w[1];
    return d;
}

// Store the lane's eight quantised values (value unit c = values 8c..8c+7 of
// the row) of slot `slot` into a Q8_0 tile (K part for kvsel 0, V part for
// 1), plus the group scale from the group's first lane.  Lane c^1 holds the
// other half of the same K run; p0/p1 are its w0/w1.
template <int D>
__device__ __forceinline__ void q8_store8(uint8_t* tile, int kvsel, int c, int slot, uint32_t w0, uint32_t w1,
                                          uint32_t p0, uint32_t p1, float d) {
    if (kvsel == 0) {
        const bool odd = c & 1;
        const uint32_t A0 = odd ? p0 : w0, A1 = odd ? p1 : w1, B0 = odd ? w0 : p0, B1 = odd ? w1 : p1;
        const uint2 val = odd ? make_uint2(__byte_perm(A1, B1, 0x5410), __byte_perm(A1, B1, 0x7632))
                              : make_uint2(__byte_perm(A0, B0, 0x5410), __byte_perm(A0, B0, 0x7632));
        *reinterpret_cast<uint2*>(tile + q8_krun<D>(slot, c >> 1) + (odd ? 8 : 0)) = val;
    } else {
        const int sp = q8_pos(slot);
#pragma unroll
        for (int i = 0; i < 8; ++i)
            tile[16 * D + (8 * c + i) * 16 + sp] = (uint8_t)(((i < 4 ? w0 : w1) >> (8 * (i & 3))) & 0xff);
    }
    if ((c & 3) == 0)
        *reinterpret_cast<uint16_t*>(tile + (kvsel ? 33 : 32) * D + ((c >> 2) * 16 + q8_pos(slot)) * 2) =
            __half_as_ushort(__float2half_rn(d));
}

// ------------------------------------------------------------------ K1 ----
// One thread per 16-byte chunk of one (token, head, K|V) row.
template <int D>
__global__ void __launch_bounds__(256) kv_write_kernel(uint16_t* __restrict__ pool_layer,
                                                       const int2* __restrict__ cells, int n, int n_kv_heads,
                                                       const void* __restrict__ k, const void* __restrict__ v,
                                                       int in_f32) {
    constexpr int CH = D / 8;
    const int gid = blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= n * n_kv_heads * 2 * CH) return;
    const int c = gid % CH;
    int r = gid / CH;
    const int kvsel = r & 1;
    r >>= 1;
    const int h = r % n_kv_heads;
    const int i = r / n_kv_heads;
    const int2 cell = cells[i];
    const size_t src = (size_t)i * n_kv_heads * D + (size_t)h * D + (size_t)c * 8;
    const uint4 val = load8_as_f16(kvsel ? v : k, src, in_f32);
    uint16_t* dst = pool_layer + (((size_t)cell.x * n_kv_heads + h) * 2 + kvsel) * (kBlock * D) + chunk_off(c, cell.y);
    *reinterpret_cast<uint4*>(dst) = val;
}

// Q8_0 pool: the same thread mapping (eight values a thread, c fastest), so
// lanes 4j..4j+3 share a 32-value group and lanes c, c^1 a K run.  Every lane
// of a warp takes part in the shuffles; lanes past the end only compute.
template <int D>
__global__ void __launch_bounds__(256) kv_write_q8_kernel(uint8_t* __restrict__ pool_layer,
                                                          const int2* __restrict__ cells, int n, int n_kv_heads,
                                                          const void* __restrict__ k, const void* __restrict__ v,
                                                          int in_f32) {
    constexpr int CH = D / 8;
    const int gid = blockIdx.x * blockDim.x + threadIdx.x;
    const bool live = gid < n * n_kv_heads * 2 * CH;
    const int c = gid % CH;
    int r = gid / CH;
    const int kvsel = r & 1;
    r >>= 1;
    const int h = r % n_kv_heads;
    const int i = r / n_kv_heads;
    float x[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (live) load8_f32(kvsel ? v : k, (size_t)i * n_kv_heads * D + (size_t)h * D + (size_t)c * 8, in_f32, x);
    uint32_t w0, w1;
    const float d = q8_quant8(x, w0, w1);
    const uint32_t p0 = __shfl_xor_sync(kFull, w0, 1), p1 = __shfl_xor_sync(kFull, w1, 1);
    if (!live) return;
    const int2 cell = cells[i];
    q8_store8<D>(pool_layer + ((size_t)cell.x * n_kv_heads + h) * q8_tile_bytes(D), kvsel, c, cell.y, w0, w1, p0, p1,
                 d);
}

// ------------------------------------------------------------------ K2 ----
// Stream-K decode attention.  The tokens of a call are laid end to end --
// tokens in order, KV heads within a token, blocks within a head -- and the
// tile sequence is cut into n_warps contiguous ranges of equal length (+-1
// tile).  Every warp derives its range and its pieces (token, head, blocks
// [b0, b1)) from the per-token descriptors alone; those travel inside the
// kernel parameters for up to kInlineTokens tokens, so a decode step needs
// no upload.  An uncut (token, head) writes its output.  A cut one is merged
// by the warp whose range holds its start: there it is that warp's last
// piece, whose (m, l, O) stays in registers; its other pieces are the first
// pieces of the following warps, which write an (m, l, O) partial to their
// own slot.  Each warp publishes an epoch flag (release) once its range is
// done; a merging warp then waits (bounded) for its neighbours' flags and
// combines.  The launch is cooperative, so every warp it waits for is
// resident (after a shared-prefix pass it is instead a programmatic
// dependent of that pass, whose CTAs all become resident as the pass's
// retire).  No atomics, fences or CTA barriers sit on the streaming path.
//
// Each warp streams its (block, head) tiles -- 4*16*D contiguous bytes, one
// cp.async.bulk each, completion on an mbarrier -- through its own
// kStages-deep ring.  The issuer runs up to kStages tiles ahead of the
// consumer and at most one piece ahead of it; a piece's q rows are bulk-
// copied next to its first tile into one of two q buffers (piece parity).
// Block ids are read 32 at a time (one per lane) a whole window ahead; a
// token's last block id comes from its descriptor, and the warp holding it
// (head 0) writes that table entry, so new blocks need no separate table
// upload.  Scores S = Q K^T and O += P V use mma.sync m16n8k16: rows 0..7
// of the A operand hold the (up to 8) query heads of the KV head rounded to
// f16, rows 8..15 the f16 rounding residual of the same values, so S and O
// carry ~22-bit q and P at no extra MMA cost.

// kind: 0 the whole (token, head) -> output; 1 it started before this
// warp's range (this is the warp's first piece) -> partial slot; 2 it
// starts in this range and runs past its end (the warp's last piece) ->
// this warp merges it.
struct PieceRegs {
    int tok, h, seq, pos, b0, b1, kind, last_block, skip;  // b0, b1 count from block `skip`
    long long ps;  // first tile of the (token, head)
};

// Fold the shared-prefix partial (m, l, O) of row (tok, h, g) into the
// running (M, L, acc) of the rest of the token's blocks (same log2 units).
template <int D>
__device__ __forceinline__ void fold_prefix(const AttnParams& p, int tok, int h, int g, int t4, float& M, float& L,
                                            float (&acc)[D / 8][2]) {
    // The prefix pass that wrote these partials is the launch this one is a
    // programmatic dependent of: wait for its completion (and the visibility
    // of its writes).  Nothing before this point reads what it writes.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const size_t r = ((size_t)tok * p.n_kv_heads + h) * p.group + g;
    for (int sp = 0; sp < p.pre_splits; ++sp) {
        const size_t rs = r + (size_t)sp * p.pre_split_rows;
        const float mp = __ldcg(p.pre_ml + rs * 2), lp = __ldcg(p.pre_ml + rs * 2 + 1);
        const float M2 = fmaxf(M, mp);
        const float a = ex2(M - M2), b = ex2(mp - M2);
        L = L * a + lp * b;
        M = M2;
        const float* po = p.pre_o + rs * D + 2 * t4;
#pragma unroll
        for (int nt = 0; nt < D / 8; ++nt) {
            const float2 v = __ldcg(reinterpret_cast<const float2*>(po + nt * 8));
            acc[nt][0] = acc[nt][0] * a + v.x * b;
            acc[nt][1] = acc[nt][1] * a + v.y * b;
        }
    }
}

// Final output row (tok, h, g) of a lane: acc * inv at columns nt*8 + 2*t4.
// Plain calls store to p.out [n][n_heads][D]; a peer gather stores the row
// to this rank's gather half, at its place among all ranks' heads.
template <int D>
__device__ __forceinline__ void store_out(const AttnParams& p, int tok, int h, int g, int t4,
                                          const float (&acc)[D / 8][2], float inv) {
    constexpr int NT = D / 8;
    const int hl = p.n_kv_heads * p.group;  // this rank's q heads
    if (p.n_peers == 0) {
        const size_t ob = ((size_t)tok * hl + (size_t)h * p.group + g) * D + 2 * t4;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const float v0 = acc[nt][0] * inv, v1 = acc[nt][1] * inv;
            if (p.out_f32)
                *reinterpret_cast<float2*>(static_cast<float*>(p.out) + ob + nt * 8) = make_float2(v0, v1);
            else
                *reinterpret_cast<__half2*>(static_cast<__half*>(p.out) + ob + nt * 8) = __floats2half2_rn(v0, v1);
        }
        return;
    }
    const size_t row = (size_t)tok * p.n_peers * hl + (size_t)p.peer_rank * hl + (size_t)h * p.group + g;
    const size_t ob = row * D + 2 * t4;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        const float v0 = acc[nt][0] * inv, v1 = acc[nt][1] * inv;
        if (p.out_f32)
            *reinterpret_cast<float2*>(static_cast<float*>(p.gather_out) + ob + nt * 8) = make_float2(v0, v1);
        else
            *reinterpret_cast<__half2*>(static_cast<__half*>(p.gather_out) + ob + nt * 8) = __floats2half2_rn(v0, v1);
    }
}

// Peer gather: a warp is done and stored the output rows of `items`
// (token, head) items into this rank's gather half (local memory).  Only
// such warps take part: after the warp barrier, lane 0 adds the items to
// this launch's count with an acq_rel RMW on this GPU, so the warp that
// completes the count (n_tok * n_kv_heads items) has every row ordered
// before it, in this GPU's memory.  It publishes this launch's epoch into
// every rank's flag for this rank: one system-scope fence, then relaxed
// system-scope stores (fence + store is a release; a release store per rank
// would pay the fence once per rank).  A rank that acquires the flag then
// reads the rows from here over NVLink.
__device__ __forceinline__ void peer_done(const AttnParams& p, int lane, int items) {
    if (p.n_peers == 0 || items == 0) return;
    __syncwarp();
    const uint32_t total = (uint32_t)p.n_tok * (uint32_t)p.n_kv_heads;
    if (lane == 0 && atom_add_acq_rel_gpu(p.done_count, (uint32_t)items) + (uint32_t)items == total) {
        *p.done_count = 0u;  // ready for the next launch (which starts after this one ends)
        fence_acq_rel_sys();
        for (int r = 0; r < p.n_peers; ++r) st_relaxed_sys(p.peer_flag[r], p.peer_epoch);
    }
}

// Wait (bounded) until flags[w] == epoch for w = first, first + stride, ...
// <= last; lane j polls every 32nd of them, so the round trips overlap.
// Warp-uniform result.
__device__ __forceinline__ bool wait_flags(const uint32_t* flags, uint32_t epoch, int first, int last, int stride,
                                           int lane) {
    int ready = 1;
    for (int w0 = first; w0 <= last && ready; w0 += 32 * stride) {
        int ok = 1;
        const int w = w0 + lane * stride;
        if (w <= last) ok = wait_flag_bounded(flags + w, epoch);
        ready = __all_sync(kFull, ok);
    }
    return ready != 0;
}

// Fold the (m, l, O) partials in slots first, first + stride, ... <= last of
// (po, pml) into the running (M, L, acc) of row g (log2 units; acc is the
// unnormalised sum at maximum M), in one pass: each batch of U partials is
// loaded together (one L2 round trip; indices past the set clamp to its last
// member and get weight 0), the running maximum moves to the batch's, and
// the partials are added in slot order.
template <int D>
__device__ __forceinline__ void merge_slots(const float* po, const float* pml, int G, int g, int t4, int first,
                                            int last, int stride, float& M, float& L, float (&acc)[D / 8][2]) {
    constexpr int NT = D / 8;
    constexpr int U = D == 64 ? 8 : 4;
    const size_t GD = (size_t)G * D;
    const int lastv = first + ((last - first) / stride) * stride;  // last member of the set
    for (int w = first; w <= lastv; w += U * stride) {
        float pm[U], pl[U];
        float2 v2[U][NT];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const size_t ww = (size_t)min(w + u * stride, lastv);
            pm[u] = __ldcg(pml + (ww * G + g) * 2);
            pl[u] = __ldcg(pml + (ww * G + g) * 2 + 1);
            const float* src = po + ww * GD + (size_t)g * D + 2 * t4;
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) v2[u][nt] = __ldcg(reinterpret_cast<const float2*>(src + nt * 8));
        }
        float Mn = M;
#pragma unroll
        for (int u = 0; u < U; ++u)
            if (w + u * stride <= lastv) Mn = fmaxf(Mn, pm[u]);
        const float own = M == -INFINITY ? 0.f : ex2(M - Mn);
        M = Mn;
        L *= own;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            acc[nt][0] *= own;
            acc[nt][1] *= own;
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const float sw = w + u * stride <= lastv ? ex2(pm[u] - M) : 0.f;
            L += pl[u] * sw;
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                acc[nt][0] += v2[u][nt].x * sw;
                acc[nt][1] += v2[u][nt].y * sw;
            }
        }
    }
}

// S = Q K^T, online softmax and O += P V for one staged (block, head) tile.
template <int D>
__device__ __forceinline__ void attend_tile(const uint8_t* tile, int valid, const uint32_t (&qa)[D / 16][4],
                                            float (&o)[D / 8][4], float& m_run, float& l_run, float scale_log2,
                                            int lane) {
    constexpr int ROW = D * 2;
    constexpr int KS = D / 16;
    constexpr int NT = D / 8;
    const int t = lane & 3;
    float s0[4] = {0.f, 0.f, 0.f, 0.f}, s1[4] = {0.f, 0.f, 0.f, 0.f};
    const uint32_t kbase = smem_u32(tile);
    {
        const int mi = lane >> 3;
        const int tok = ((mi >> 1) << 3) + (lane & 7);
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
            const int c = 2 * ks + (mi & 1);
            uint32_t b0, b1, b2, b3;
            ldsm_x4(kbase + chunk_off(c, tok) * 2, b0, b1, b2, b3);
            mma16816(s0, qa[ks], b0, b1);
            mma16816(s1, qa[ks], b2, b3);
        }
    }
    float sc[4] = {(s0[0] + s0[2]) * scale_log2, (s0[1] + s0[3]) * scale_log2, (s1[0] + s1[2]) * scale_log2,
                   (s1[1] + s1[3]) * scale_log2};
    if (valid < kBlock) {
        if (2 * t >= valid) sc[0] = -INFINITY;
        if (2 * t + 1 >= valid) sc[1] = -INFINITY;
        if (2 * t + 8 >= valid) sc[2] = -INFINITY;
        if (2 * t + 9 >= valid) sc[3] = -INFINITY;
    }
    float mx = fmaxf(fmaxf(sc[0], sc[1]), fmaxf(sc[2], sc[3]));
    mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, 2));
    const bool grow = mx > m_run;
    const float m_new = grow ? mx : m_run;
    const float alpha = grow ? ex2(m_run - m_new) : 1.f;
    float pr[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) pr[e] = ex2(sc[e] - m_new);
    l_run = l_run * alpha + ((pr[0] + pr[1]) + (pr[2] + pr[3]));
    m_run = m_new;
    if (__any_sync(kFull, grow)) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            o[nt][0] *= alpha;
            o[nt][1] *= alpha;
            o[nt][2] *= alpha;
            o[nt][3] *= alpha;
        }
    }
    uint32_t pa[4];
    {
        const __half2 h01 = __floats2half2_rn(pr[0], pr[1]);
        const __half2 h23 = __floats2half2_rn(pr[2], pr[3]);
        const float2 f01 = __half22float2(h01), f23 = __half22float2(h23);
        pa[0] = h2_bits(h01);
        pa[1] = h2_bits(__floats2half2_rn(pr[0] - f01.x, pr[1] - f01.y));
        pa[2] = h2_bits(h23);
        pa[3] = h2_bits(__floats2half2_rn(pr[2] - f23.x, pr[3] - f23.y));
    }
    {
        const uint32_t vbase = kbase + kBlock * ROW;
        const int mi = lane >> 3;
        const int tok = ((mi & 1) << 3) + (lane & 7);
#pragma unroll
        for (int np = 0; np < NT / 2; ++np) {
            const int c = 2 * np + (mi >> 1);
            uint32_t b0, b1, b2, b3;
            ldsm_x4_t(vbase + chunk_off(c, tok) * 2, b0, b1, b2, b3);
            mma16816(o[2 * np], pa, b0, b1);
            mma16816(o[2 * np + 1], pa, b2, b3);
        }
    }
}

// The same step for a staged Q8_0 tile.  S: per 32-value group c, one
// ldmatrix hands each lane its K bytes for two k-steps (slots 0-7 and 8-15),
// converted to f16 exactly; the group's partial scores are scaled by the
// slots' K scales in f32.  O += P V: per group c the P row is multiplied by
// the slots' V scales (in f32, then split into f16 value + residual), so the
// V bytes (again exact f16) go to the MMA unscaled.  Slots past `valid`
// are masked out of S and contribute nothing to O, whatever their bytes.
template <int D>
__device__ __forceinline__ void attend_tile_q8(const uint8_t* tile, int valid, const uint32_t (&qa)[D / 16][4],
                                               float (&o)[D / 8][4], float& m_run, float& l_run, float scale_log2,
                                               int lane) {
    constexpr int G32 = D / 32;
    const int t = lane & 3;
    const int mi = lane >> 3, r = lane & 7;
    const uint32_t base = smem_u32(tile);
    float sc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int c = 0; c < G32; ++c) {
        float t0[4] = {0.f, 0.f, 0.f, 0.f}, t1[4] = {0.f, 0.f, 0.f, 0.f};
        uint32_t w0, w1, w2, w3, b0, b1;
        // matrices: (slots 0-7, run 2c), (8-15, 2c), (0-7, 2c+1), (8-15, 2c+1)
        ldsm_x4(base + q8_krun<D>(((mi & 1) << 3) + r, 2 * c + (mi >> 1)), w0, w1, w2, w3);
        i8x4_to_f16x2(w0, b0, b1);
        mma16816(t0, qa[2 * c], b0, b1);
        i8x4_to_f16x2(w1, b0, b1);
        mma16816(t1, qa[2 * c], b0, b1);
        i8x4_to_f16x2(w2, b0, b1);
        mma16816(t0, qa[2 * c + 1], b0, b1);
        i8x4_to_f16x2(w3, b0, b1);
        mma16816(t1, qa[2 * c + 1], b0, b1);
        // K scales of slots 2t, 2t+1, 2t+8, 2t+9 (entries 4t..4t+3 of group c)
        const uint2 kd = *reinterpret_cast<const uint2*>(tile + 32 * D + (c * 16 + 4 * t) * 2);
        const float2 d01 = __half22float2(*reinterpret_cast<const __half2*>(&kd.x));
        const float2 d23 = __half22float2(*reinterpret_cast<const __half2*>(&kd.y));
        sc[0] += d01.x * (t0[0] + t0[2]);
        sc[1] += d01.y * (t0[1] + t0[3]);
        sc[2] += d23.x * (t1[0] + t1[2]);
        sc[3] += d23.y * (t1[1] + t1[3]);
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) sc[e] *= scale_log2;
    // Slots past `valid` (only in a sequence's last block) are masked out of
    // S and weigh exactly 0 in O, whatever their stale bytes and scales.
    const bool part = valid < kBlock;  // warp-uniform
    const bool ok0 = !part || 2 * t < valid, ok1 = !part || 2 * t + 1 < valid, ok2 = !part || 2 * t + 8 < valid,
               ok3 = !part || 2 * t + 9 < valid;
    if (part) {
        if (!ok0) sc[0] = -INFINITY;
        if (!ok1) sc[1] = -INFINITY;
        if (!ok2) sc[2] = -INFINITY;
        if (!ok3) sc[3] = -INFINITY;
    }
    float mx = fmaxf(fmaxf(sc[0], sc[1]), fmaxf(sc[2], sc[3]));
    mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, 2));
    const bool grow = mx > m_run;
    const float m_new = grow ? mx : m_run;
    const float alpha = grow ? ex2(m_run - m_new) : 1.f;
    float pr[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) pr[e] = ex2(sc[e] - m_new);
    l_run = l_run * alpha + ((pr[0] + pr[1]) + (pr[2] + pr[3]));
    m_run = m_new;
    if (__any_sync(kFull, grow)) {
#pragma unroll
        for (int nt = 0; nt < D / 8; ++nt) {
            o[nt][0] *= alpha;
            o[nt][1] *= alpha;
            o[nt][2] *= alpha;
            o[nt][3] *= alpha;
        }
    }
#pragma unroll
    for (int c = 0; c < G32; ++c) {
        const uint2 vd = *reinterpret_cast<const uint2*>(tile + 33 * D + (c * 16 + 4 * t) * 2);
        const float2 d01 = __half22float2(*reinterpret_cast<const __half2*>(&vd.x));
        const float2 d23 = __half22float2(*reinterpret_cast<const __half2*>(&vd.y));
        float p0 = pr[0] * d01.x, p1 = pr[1] * d01.y, p2 = pr[2] * d23.x, p3 = pr[3] * d23.y;
        if (part) {
            p0 = ok0 ? p0 : 0.f;
            p1 = ok1 ? p1 : 0.f;
            p2 = ok2 ? p2 : 0.f;
            p3 = ok3 ? p3 : 0.f;
        }
        uint32_t pa[4];
        {
            const __half2 h01 = __floats2half2_rn(p0, p1), h23 = __floats2half2_rn(p2, p3);
            const float2 f01 = __half22float2(h01), f23 = __half22float2(h23);
            pa[0] = h2_bits(h01);
            pa[1] = h2_bits(__floats2half2_rn(p0 - f01.x, p1 - f01.y));
            pa[2] = h2_bits(h23);
            pa[3] = h2_bits(__floats2half2_rn(p2 - f23.x, p3 - f23.y));
        }
        // columns 32c + 8*mi + r: one 16-byte run (16 slots) each
        uint32_t w0, w1, w2, w3, b0, b1;
        ldsm_x4(base + 16 * D + (32 * c + 8 * mi + r) * 16, w0, w1, w2, w3);
        i8x4_to_f16x2(w0, b0, b1);
        mma16816(o[4 * c], pa, b0, b1);
        i8x4_to_f16x2(w1, b0, b1);
        mma16816(o[4 * c + 1], pa, b0, b1);
        i8x4_to_f16x2(w2, b0, b1);
        mma16816(o[4 * c + 2], pa, b0, b1);
        i8x4_to_f16x2(w3, b0, b1);
        mma16816(o[4 * c + 3], pa, b0, b1);
    }
}

// Shared memory of one warp: its tile ring plus two q buffers (pieces of
// even / odd index) of group*D elements of the q dtype.
__host__ __device__ inline int qbuf_bytes(int group, int head_dim, int q_f32) {
    return (group * head_dim * (q_f32 ? 4 : 2) + 127) & ~127;
}

__host__ __device__ inline int stage_count(int q8) { return q8 ? kStagesQ8 : kStages; }
__host__ __device__ inline int tile_bytes(int head_dim, int q8) {
    return q8 ? q8_tile_bytes(head_dim) : 2 * kBlock * head_dim * 2;
}

__host__ __device__ inline int warp_smem(int group, int head_dim, int q_f32, int q8) {
    return stage_count(q8) * tile_bytes(head_dim, q8) + 2 * qbuf_bytes(group, head_dim, q_f32);
}

__host__ __device__ inline int attn_smem(int group, int head_dim, int q_f32, int q8) {
    return kWarps * warp_smem(group, head_dim, q_f32, q8) + kWarps * stage_count(q8) * 8;
}

template <int D, bool Q8>
__global__ void __launch_bounds__(kWarps * 32, 1) paged_attn_kernel(const __grid_constant__ AttnParams p) {
    constexpr int TILE = Q8 ? q8_tile_bytes(D) : 2 * kBlock * D * 2;
    constexpr int ROW = D * 2;
    constexpr int KS = D / 16;
    constexpr int NT = D / 8;
    constexpr int S = Q8 ? kStagesQ8 : kStages;
    extern __shared__ __align__(1024) uint8_t smem[];

    // A kernel launched after this one as a programmatic dependent (the
    // decode matmul that consumes the output, the peer-gather wait) may start
    // as this launch's CTAs retire; it still waits for this grid's completion
    // (griddepcontrol.wait) before it reads what this grid wrote.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gw = blockIdx.x * kWarps + warp;
    const int Hkv = p.n_kv_heads, G = p.group;
    const int QBUF = qbuf_bytes(G, D, p.q_f32);
    uint8_t* stages = smem + (size_t)warp * warp_smem(G, D, p.q_f32, Q8);
    uint8_t* qbufs = stages + S * TILE;
    const uint32_t bar0 =
        smem_u32(reinterpret_cast<uint64_t*>(smem + (size_t)kWarps * warp_smem(G, D, p.q_f32, Q8)) + warp * S);
    if (lane < S) mbar_init(bar0 + 8u * lane, 1);
    fence_mbar_init();
    __syncwarp();
    if (gw >= p.n_warps) return;

    const TokenDesc* toks = p.toks ? p.toks : p.inl;
    const long long T = (long long)p.tiles_per_head * Hkv;
    const long long t0 = T * gw / p.n_warps, t1 = T * (gw + 1) / p.n_warps;
    const int g = lane >> 2, t4 = lane & 3;
    const size_t tile_elems = TILE / 2;  // pool addressing in 16-bit units
    const int qelem = p.q_f32 ? 4 : 2;
    const uint32_t qbytes = (uint32_t)(G * D * qelem);

    // ---- piece generator over [t0, t1) ----
    int gi, gh, gb;  // token, head, block of tile gt
    long long gt = t0;
    {
        int lo = 0, hi = p.n_tok - 1;  // last token whose first tile is <= t0
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if ((long long)toks[mid].prefix * Hkv <= t0) lo = mid; else hi = mid - 1;
        }
        gi = lo;
        const TokenDesc td = toks[gi];
        const int nb = td.pos / kBlock + 1 - td.skip;
        const long long off = t0 - (long long)td.prefix * Hkv;
        gh = (int)(off / nb);
        gb = (int)(off % nb);
    }
    auto gen_piece = [&](PieceRegs& r) {  // the piece at the generator, then advance past it
        const TokenDesc td = toks[gi];
        const int nb = td.pos / kBlock + 1 - td.skip;
        const int len = (int)min((long long)(nb - gb), t1 - gt);
        r.tok = gi;
        r.skip = td.skip;
        r.h = gh;
        r.seq = td.seq;
        r.pos = td.pos;
        r.b0 = gb;
        r.b1 = gb + len;
        r.ps = (long long)td.prefix * Hkv + (long long)gh * nb;
        r.kind = r.ps < t0 ? 1 : (r.ps + nb > t1 ? 2 : 0);
        r.last_block = r.b1 == nb ? td.last_block : -1;
        gt += len;
        gb += len;
        if (gb == nb) {
            gb = 0;
            if (++gh == Hkv) {
                gh = 0;
                ++gi;
            }
        }
    };
    // block ids [b, min(b + 32, b1)) of a piece, lane j holding b + j
    auto load_window = [&](const PieceRegs& r, int b) {
        const int bb = b + lane;
        if (bb >= r.b1) return 0;
        if (bb == r.b1 - 1 && r.last_block >= 0) return r.last_block;
        return checked_block(__ldg(p.tables + (size_t)r.seq * p.max_blocks + r.skip + bb), p.n_blocks, p.err,
                             p.check_ids != 0);
    };

    // ---- issuer state ----
    PieceRegs di{}, dn{};
    gen_piece(di);
    // The range's first piece: a warp whose first piece continues a cut
    // (token, head) may lead a group of its helpers in the two-level merge.
    const long long f_ps = di.ps;
    const int f_nb = di.pos / kBlock + 1 - di.skip, f_kind = di.kind;
    bool dn_valid = gt < t1;
    if (dn_valid) gen_piece(dn);
    int ii = 0;  // issuer piece ordinal
    int it = 0;  // next tile of piece di to issue (relative to b0)
    int wb = 0;  // window base (relative to b0)
    int win = load_window(di, di.b0);
    int win_n = 0;  // next window: same piece (wb + 32) or first of piece dn
    auto prefetch_window = [&]() {
        if (wb + 32 < di.b1 - di.b0) win_n = load_window(di, di.b0 + wb + 32);
        else if (dn_valid) win_n = load_window(dn, dn.b0);
    };
    prefetch_window();
    auto table_write = [&](const PieceRegs& r) {
        // the token's last block entry, written once per token (head 0)
        if (r.h == 0 && r.last_block >= 0 && lane == 0)
            p.tables[(size_t)r.seq * p.max_blocks + r.skip + r.b1 - 1] = r.last_block;
    };
    table_write(di);

    int issued = 0, consumed = 0;
    int istage = 0;              // ring stage of the next copy (issued % S)
    int cstage = 0, cphase = 0;  // ring stage and barrier phase of the next tile consumed
    auto issue_one = [&]() {
        if (it - wb >= 32) {
            win = win_n;
            wb += 32;
            prefetch_window();
        }
        const int b = __shfl_sync(kFull, win, it - wb);
        if (lane == 0) {
            const int s = istage;
            const uint32_t bar = bar0 + 8u * s;
            mbar_arrive_expect_tx(bar, TILE + (it == 0 ? qbytes : 0u));
            bulk_g2s(smem_u32(stages + (size_t)s * TILE), p.pool_layer + ((size_t)b * Hkv + di.h) * tile_elems, TILE,
                     bar);
            if (it == 0)
                bulk_g2s(smem_u32(qbufs + (ii & 1) * QBUF),
                         static_cast<const uint8_t*>(p.q) + ((size_t)di.tok * Hkv + di.h) * G * D * qelem, qbytes,
                         bar);
        }
        ++it;
        ++issued;
        istage = istage + 1 == S ? 0 : istage + 1;
    };
    auto issuer_advance = [&]() {  // piece di is fully issued; move to dn
        ++ii;
        di = dn;
        dn_valid = gt < t1;
        if (dn_valid) gen_piece(dn);
        it = 0;
        wb = 0;
        win = win_n;
        prefetch_window();
        table_write(di);
    };

    // ---- consumer state ----
    int ci = 0;
    PieceRegs dc = di;
    int ct = 0;
    // The issuer stays within one piece of the consumer (two q buffers).
    auto try_issue = [&]() {
        while (issued - consumed < S) {
            if (it < di.b1 - di.b0) {
                issue_one();
                continue;
            }
            if (ii != ci || !dn_valid) break;
            issuer_advance();
        }
    };
    try_issue();

    uint32_t qa[KS][4];
    float o[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.f;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    int items_out = 0;   // (token, head) outputs this warp stored
    for (;;) {
        const int s = cstage;
        if (!mbar_wait_bounded(bar0 + 8u * s, (uint32_t)cphase)) {
            ok = false;
            break;
        }
        uint8_t* tile = stages + (size_t)s * TILE;
        if (ct == 0) {
            // q rows of this piece: rows 0..G-1 rounded to f16, rows 8.. the residual
            const uint8_t* qb = qbufs + (ci & 1) * QBUF;
#pragma unroll
            for (int ks = 0; ks < KS; ++ks) {
#pragma unroll
                for (int hf = 0; hf < 2; ++hf) {
                    float x0 = 0.f, x1 = 0.f;
                    if (g < G) {
                        const int e = g * D + ks * 16 + hf * 8 + 2 * t4;
                        if (p.q_f32) {
                            const float2 f = *reinterpret_cast<const float2*>(qb + e * 4);
                            x0 = f.x;
                            x1 = f.y;
                        } else {
                            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(qb + e * 2));
                            x0 = f.x;
                            x1 = f.y;
                        }
                    }
                    const __half2 hi = __floats2half2_rn(x0, x1);
                    const float2 hf2 = __half22float2(hi);
                    qa[ks][2 * hf] = h2_bits(hi);
                    qa[ks][2 * hf + 1] = h2_bits(__floats2half2_rn(x0 - hf2.x, x1 - hf2.y));
                }
            }
        }
        const int b = dc.b0 + ct;  // from block dc.skip
        const int valid = min(kBlock, dc.pos + 1 - (dc.skip + b) * kBlock);
        bool touched = false;
        if (Q8 && p.k_new && dc.last_block >= 0 && b == dc.b1 - 1) {
            // Fused append, Q8_0: lanes 0..2*CH-1 quantise this token's new
            // K (then V) row for head h, eight values each, and store it to
            // its pool cell and into the staged tile.
            constexpr int CH = D / 8;
            const int slot = dc.pos % kBlock;
            const bool live = lane < 2 * CH;
            const int kvsel = lane / CH, c = lane % CH;
            float x[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
            if (live)
                load8_f32(kvsel ? p.v_new : p.k_new, (size_t)dc.tok * Hkv * D + (size_t)dc.h * D + (size_t)c * 8,
                          p.kv_f32, x);
            uint32_t w0, w1;
            const float d = q8_quant8(x, w0, w1);
            const uint32_t p0 = __shfl_xor_sync(kFull, w0, 1), p1 = __shfl_xor_sync(kFull, w1, 1);
            if (live) {
                q8_store8<D>(tile, kvsel, c, slot, w0, w1, p0, p1, d);
                q8_store8<D>(reinterpret_cast<uint8_t*>(p.pool_layer_w + ((size_t)dc.last_block * Hkv + dc.h) *
                                                                             tile_elems),
                             kvsel, c, slot, w0, w1, p0, p1, d);
            }
            touched = true;
        }
        if (!Q8 && p.k_new && dc.last_block >= 0 && b == dc.b1 - 1) {
            // Fused append: this token's new K/V row for head h goes to its
            // pool cell and into the staged tile (the copy read the old bytes).
            constexpr int CH = D / 8;
            const int slot = dc.pos % kBlock;
            if (lane < 2 * CH) {
                const int kvsel = lane / CH, c = lane % CH;
                const size_t src = (size_t)dc.tok * Hkv * D + (size_t)dc.h * D + (size_t)c * 8;
                const uint4 val = load8_as_f16(kvsel ? p.v_new : p.k_new, src, p.kv_f32);
                const int off = chunk_off(c, slot);
                *reinterpret_cast<uint4*>(tile + kvsel * kBlock * ROW + off * 2) = val;
                *reinterpret_cast<uint4*>(p.pool_layer_w + ((size_t)dc.last_block * Hkv + dc.h) * tile_elems +
                                          (size_t)kvsel * kBlock * D + off) = val;
            }
            touched = true;
        }
        if (!Q8 && valid < kBlock) {
            // Rows past the sequence end were never written for it: zero V so
            // 0 * (stale NaN/Inf) cannot reach O; K rows are masked.
            const int per_half = (kBlock - valid) * 8;  // 16-byte chunks past the end in each 64-wide sub-tile
            for (int e = lane; e < per_half * (D / 64); e += 32) {
                uint4* vz = reinterpret_cast<uint4*>(tile + kBlock * ROW + (e / per_half) * (kBlock * 128) + valid * 128);
                vz[e % per_half] = make_uint4(0, 0, 0, 0);
            }
            touched = true;
        }
        __syncwarp();
        if constexpr (Q8)
            attend_tile_q8<D>(tile, valid, qa, o, m_run, l_run, p.scale_log2, lane);
        else
            attend_tile<D>(tile, valid, qa, o, m_run, l_run, p.scale_log2, lane);
        ++consumed;
        if (++cstage == S) {
            cstage = 0;
            cphase ^= 1;
        }
        ++ct;
        // Generic-proxy writes into this stage must be ordered before the
        // async-proxy copy that may refill it.
        if (touched) fence_proxy_async_smem();
        __syncwarp();

        if (ct == dc.b1 - dc.b0) {
            // ---- piece done ----
            if (dc.kind == 2) break;  // the range's last piece: merged after the loop
            float l = l_run;
            l += __shfl_xor_sync(kFull, l, 1);
            l += __shfl_xor_sync(kFull, l, 2);
            const size_t GD = (size_t)G * D;
            if (dc.kind == 0) ++items_out;
            if (g < G) {
                if (dc.kind == 0) {
                    float acc[NT][2];
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt) {
                        acc[nt][0] = o[nt][0] + o[nt][2];
                        acc[nt][1] = o[nt][1] + o[nt][3];
                    }
                    if (dc.skip > 0) fold_prefix<D>(p, dc.tok, dc.h, g, t4, m_run, l, acc);
                    store_out<D>(p, dc.tok, dc.h, g, t4, acc, 1.f / l);
                } else {
                    const size_t sl = (size_t)gw;  // partial slot of this warp (its first piece)
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt)
                        *reinterpret_cast<float2*>(p.part_o + sl * GD + (size_t)g * D + nt * 8 + 2 * t4) =
                            make_float2(o[nt][0] + o[nt][2], o[nt][1] + o[nt][3]);
                    if (t4 == 0) {
                        p.part_ml[(sl * G + g) * 2] = m_run;
                        p.part_ml[(sl * G + g) * 2 + 1] = l;
                    }
                }
            }
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.f;
            m_run = -INFINITY;
            l_run = 0.f;
            if (ii == ci) {
                if (!dn_valid) break;  // last piece of the range: every issued tile is consumed
                issuer_advance();
            }
            ++ci;
            dc = di;
            ct = 0;
        }
        try_issue();
    }
    if (!ok) {
        // bounded drain of the copies still in flight, then report
        for (int jj = consumed + 1; jj < issued; ++jj) mbar_wait_bounded(bar0 + 8u * (jj % S), (jj / S) & 1);
        if (lane == 0) atomicOr(p.err, kErrTimeout);
    }
    // Publish: every partial this warp wrote is visible before its flag.
    __syncwarp();
    if (lane == 0) st_release_gpu(p.flags + gw, p.epoch);
    const long long NW = p.n_warps;

    // ---- two-level merge: lead a group of helpers of a long cut (token, head) ----
    // Helpers of a (token, head) are the warps after the one holding its first
    // tile; with more than kMergeGroup of them, every kMergeGroup-th helper
    // combines its own partial and its next kMergeGroup-1 neighbours' into a
    // group partial, so the merging warp reads one partial per group.
    if (ok && f_kind == 1 && p.part2_o) {
        const int ws = (int)(((f_ps + 1) * NW - 1) / T), we = (int)(((f_ps + f_nb) * NW - 1) / T);
        if (we - ws > kMergeGroup && (gw - ws - 1) % kMergeGroup == 0) {
            const int last = min(gw + kMergeGroup - 1, we);
            const bool rd = wait_flags(p.flags, p.epoch, gw + 1, last, 1, lane);
            __syncwarp();
            if (rd && g < G) {
                float M = -INFINITY, L = 0.f, acc[NT][2];
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) acc[nt][0] = acc[nt][1] = 0.f;
                merge_slots<D>(p.part_o, p.part_ml, G, g, t4, gw, last, 1, M, L, acc);
                const size_t GD = (size_t)G * D;
#pragma unroll
                for (int nt = 0; nt < NT; ++nt)
                    *reinterpret_cast<float2*>(p.part2_o + (size_t)gw * GD + (size_t)g * D + nt * 8 + 2 * t4) =
                        make_float2(acc[nt][0], acc[nt][1]);
                if (t4 == 0) {
                    p.part2_ml[((size_t)gw * G + g) * 2] = M;
                    p.part2_ml[((size_t)gw * G + g) * 2 + 1] = L;
                }
            }
            if (!rd && lane == 0) atomicOr(p.err, kErrTimeout);
            __syncwarp();
            if (lane == 0) st_release_gpu(p.flags2 + gw, p.epoch);  // published either way: no second wait
        }
    }
    // After a prefix pass every warp leaves only once that pass has
    // completed, so this grid's completion implies the pass's: work queued
    // after this launch may then reuse the prefix partials.
    if (!ok || dc.kind != 2 || ct != dc.b1 - dc.b0) {
        peer_done(p, lane, items_out);
        if (p.pre_splits > 0) asm volatile("griddepcontrol.wait;" ::: "memory");
        return;
    }

    // ---- merge the cut (token, head) this range ends with ----
    const int nb = dc.pos / kBlock + 1 - dc.skip;
    const int w_last = (int)(((dc.ps + nb) * NW - 1) / T);  // warp holding its last tile
    const bool grouped = p.part2_o && w_last - gw > kMergeGroup;
    const int stride = grouped ? kMergeGroup : 1;
    const bool ready = wait_flags(grouped ? p.flags2 : p.flags, p.epoch, gw + 1, w_last, stride, lane);
    __syncwarp();
    if (!ready) {
        if (lane == 0) atomicOr(p.err, kErrTimeout);
        peer_done(p, lane, items_out + 1);  // its item stays unwritten; the error flag says so
        if (p.pre_splits > 0) asm volatile("griddepcontrol.wait;" ::: "memory");
        return;
    }
    float l = l_run;
    l += __shfl_xor_sync(kFull, l, 1);
    l += __shfl_xor_sync(kFull, l, 2);
    if (g < G) {
        float M = m_run, L = l, acc[NT][2];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            acc[nt][0] = o[nt][0] + o[nt][2];
            acc[nt][1] = o[nt][1] + o[nt][3];
        }
        merge_slots<D>(grouped ? p.part2_o : p.part_o, grouped ? p.part2_ml : p.part_ml, G, g, t4, gw + 1, w_last,
                       stride, M, L, acc);
        if (dc.skip > 0) fold_prefix<D>(p, dc.tok, dc.h, g, t4, M, L, acc);
        store_out<D>(p, dc.tok, dc.h, g, t4, acc, 1.f / L);
    }
    peer_done(p, lane, items_out + 1);
    if (p.pre_splits > 0) asm volatile("griddepcontrol.wait;" ::: "memory");
}

// ------------------------------------------------------------ prefix ----
// Shared-prefix (cascade) pass on the 5th-generation tensor cores.
//
// One CTA per PrefixItem: one KV head and up to 128 query rows (row r =
// item token r / G, q head r % G), tcgen05 M = 128 with row r in TMEM lane r.
// The group's shared blocks stream through a 3-stage shared-memory ring, four
// blocks (64 positions) a step, each (block, head) K and V sub-tile
// bulk-copied once for all 128 rows.  Per step:
//   S = Q K^T      tcgen05.mma, A = Q (f16 value, then its f16 residual,
//                  both accumulating into S: ~22-bit q), B = K, D = S in TMEM;
//   softmax        thread r reads its S row from TMEM, keeps a running
//                  maximum m that only moves up by more than 2^8 (so O and l
//                  are rescaled rarely), writes P = 2^(s*scale - m) as f16
//                  value + residual rows into shared memory;
//   O += P V       tcgen05.mma, A = P (value, then residual), B = V (MN-major),
//                  D = O in TMEM.
// The pool's 16 x 64 sub-tiles are already the 128-byte-swizzled K-major (K)
// and MN-major (V) operand layouts, so the tiles go from the bulk copy
// straight to the tensor cores.  At the end each row writes (m, l, O).
// Every wait is bounded; on a timeout the CTA sets the error flag, drains
// its copies and still frees its TMEM.  The warp-collective tcgen05 ops
// (alloc, ld, st, wait, dealloc) are only ever reached by whole warps.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1 << 46;  // descriptor version (sm_100)
    d |= (uint64_t)2 << 61;  // 128-byte swizzle
    return d;
}

// kind::f16 instruction descriptor: f16 A/B, f32 D, M = 128, N = n.
__device__ __forceinline__ uint32_t f16_idesc(int n, bool b_mn_major) {
    return (1u << 4) | ((b_mn_major ? 1u : 0u) << 16) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0)
        : "memory");
}

__device__ __forceinline__ void umma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Warp-collective: every lane of the warp calls these with the same column.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    __syncwarp();
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
    __syncwarp();
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
        "%14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
        "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
        "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
        "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])),
        "r"(__float_as_uint(v[11])), "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])),
        "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])),
        "r"(__float_as_uint(v[17])), "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])),
        "r"(__float_as_uint(v[20])), "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])),
        "r"(__float_as_uint(v[23])), "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])),
        "r"(__float_as_uint(v[26])), "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])),
        "r"(__float_as_uint(v[29])), "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
        : "memory");
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

constexpr int kPreRows = 128;        // tcgen05 M: query rows of a CTA
constexpr int kPreStepBlocks = 4;    // blocks (16 positions each) per step: N = 64
constexpr int kPreStages = 3;        // K/V ring: copies run kPreStages - 2 steps ahead of their use
constexpr int kPreThreads = 192;     // warps 0..3: softmax of rows 32w..32w+31; warp 4: MMA issue; warp 5: copies
constexpr int kPreTmemCols = 256;    // S buffers at columns 0 and 64, O at 128
constexpr float kRescaleLog2 = 8.f;  // a row's maximum moves only when it grows by more than this

// Shared-memory layout of the prefix CTA (offsets from a 1024-aligned base):
// Q value and residual [D/64][128 rows][128 B]; kPreStages K/V stages, each
// K [D/64][64 rows][128 B] then V alike; two P buffers, each value and
// residual [128 rows][128 B]; the mbarriers.
struct PreSmem {
    uint32_t q_hi, q_lo, stage0, stage_bytes, p0, bars, total;
    __host__ __device__ explicit PreSmem(int D) {
        const uint32_t qbytes = (uint32_t)kPreRows * D * 2;
        stage_bytes = (uint32_t)2 * kPreStepBlocks * kBlock * D * 2;
        q_hi = 0;
        q_lo = q_hi + qbytes;
        stage0 = q_lo + qbytes;
        p0 = stage0 + kPreStages * stage_bytes;  // P buffer b: value at p0 + b*2*16K, residual +16K
        bars = p0 + 2 * 2 * kPreRows * 128;
        total = bars + 256;
    }
};

// mbarrier arrive (count 1) from a thread.
__device__ __forceinline__ void mbar_arrive1(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

template <int D>
__global__ void __launch_bounds__(kPreThreads, 1) prefix_attn_kernel(const __grid_constant__ PrefixParams p) {
    // The decode launch that folds these partials in may start on the SMs
    // this launch leaves free; it waits for this grid before the fold.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    constexpr int HALVES = D / 64;
    constexpr uint32_t HALF_ROWS_BYTES = kPreStepBlocks * kBlock * 128;  // one 64-wide sub-tile column of a stage
    constexpr uint32_t PBUF = 2 * kPreRows * 128;                         // one P buffer: value + residual
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
    uint8_t* sbase = smem_raw + (base - smem_u32(smem_raw));
    const PreSmem L(D);
    const uint32_t STAGE = L.stage_bytes, KPART = STAGE / 2;
    const PrefixItem item = p.items[blockIdx.x];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = p.group, Hkv = p.n_kv_heads;
    // barriers: kv_full[3], kv_empty[3], s_full[2], s_free[2], p_full[2], p_free[2], pv_done, tmem word
    const uint32_t kv_full = base + L.bars, kv_empty = kv_full + 8u * kPreStages;
    const uint32_t s_full = kv_empty + 8u * kPreStages, s_free = s_full + 16u, p_full = s_free + 16u,
                   p_free = p_full + 16u, pv_done = p_free + 16u;
    uint32_t* tmem_word = reinterpret_cast<uint32_t*>(sbase + L.bars + 8 * (2 * kPreStages + 9));
    if (tid == 0) {
        for (int st = 0; st < kPreStages; ++st) {
            mbar_init(kv_full + 8u * st, 1);
            mbar_init(kv_empty + 8u * st, 1);
        }
        for (int bb = 0; bb < 2; ++bb) {
            mbar_init(s_full + 8u * bb, 1);
            mbar_init(s_free + 8u * bb, 4);  // one arrival per softmax warp
            mbar_init(p_full + 8u * bb, 4);
            mbar_init(p_free + 8u * bb, 1);
        }
        mbar_init(pv_done, 1);
        fence_mbar_init();
    }
    __syncwarp();  // tcgen05.alloc is warp-collective: warp 0 converged after thread 0's setup
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_word)),
                     "r"(kPreTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_word;
    const uint32_t tmem_o = tmem + 128;

    const int nbk = item.blk1 - item.blk0;  // >= 1: the host gives every split at least one step
    const int n_steps = (nbk + kPreStepBlocks - 1) / kPreStepBlocks;
    const int32_t* trow = p.tables + (size_t)item.root_seq * p.max_blocks + item.blk0;
    const size_t tile_elems = 2 * kBlock * D;
    auto step_blocks = [&](int j) { return min(kPreStepBlocks, nbk - j * kPreStepBlocks); };
    int issued = 0;  // warp 5 lane 0: steps whose copies were issued
    // The step's block ids, loaded together (independent loads) a step ahead
    // of the copies that use them.
    auto load_ids = [&](int j, int (&ids)[kPreStepBlocks]) {
        if (j >= n_steps) return;
        const int nblk = step_blocks(j);
#pragma unroll
        for (int bb = 0; bb < kPreStepBlocks; ++bb)
            ids[bb] = bb < nblk ? checked_block(__ldg(trow + j * kPreStepBlocks + bb), p.n_blocks, p.err) : 0;
    };
    auto issue_step = [&](int j, const int (&ids)[kPreStepBlocks]) {
        const int st = j % kPreStages;
        const int nblk = step_blocks(j);
        const uint32_t bar = kv_full + 8u * st;
        mbar_arrive_expect_tx(bar, (uint32_t)nblk * 2 * kBlock * D * 2);
        const uint32_t sk = base + L.stage0 + st * STAGE;
        for (int bb = 0; bb < nblk; ++bb) {
            const uint16_t* src = p.pool_layer + ((size_t)ids[bb] * Hkv + item.head) * tile_elems;
            for (int hh = 0; hh < HALVES; ++hh) {
                bulk_g2s(sk + hh * HALF_ROWS_BYTES + bb * (kBlock * 128), src + hh * (kBlock * 64), kBlock * 128, bar);
                bulk_g2s(sk + KPART + hh * HALF_ROWS_BYTES + bb * (kBlock * 128), src + kBlock * D + hh * (kBlock * 64),
                         kBlock * 128, bar);
            }
        }
        ++issued;
    };
    int nxt_ids[kPreStepBlocks] = {};  // ids of the next refill (step kPreStages, ...)
    if (tid == kPreRows + 32) {
        for (int j = 0; j < min(kPreStages, n_steps); ++j) {
            int ids[kPreStepBlocks] = {};
            load_ids(j, ids);
            issue_step(j, ids);
        }
        load_ids(kPreStages, nxt_ids);
    }

    // Q rows (warps 0..3): row r = token r / G, head r % G; value and f16 residual
    const int r = tid;
    const int t_item = r / G, hg = r % G;
    const bool live = r < kPreRows && t_item < item.n_tok && t_item < kPreRows / G;
    const int tok = live ? p.tok_list[item.tok_off + t_item] : 0;
    // Row r attends positions [0, lim) of the item's blocks: the token's own
    // skip (a prefill chunk's tokens, causally), or all of them.
    const int lim = live ? p.tok_lim[item.tok_off + t_item] * kBlock : 0x7fffffff;
    if (r < kPreRows) {
        const int qelem = p.q_f32 ? 4 : 2;
        const uint8_t* qrow = static_cast<const uint8_t*>(p.q) + (((size_t)tok * Hkv + item.head) * G + hg) * D * qelem;
#pragma unroll 1
        for (int c = 0; c < D / 8; ++c) {
            float x[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) x[e] = 0.f;
            if (live) {
                if (p.q_f32) {
                    const float4 a = *reinterpret_cast<const float4*>(qrow + c * 32);
                    const float4 b2 = *reinterpret_cast<const float4*>(qrow + c * 32 + 16);
                    x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w; x[4] = b2.x; x[5] = b2.y; x[6] = b2.z; x[7] = b2.w;
                } else {
                    const uint4 u = *reinterpret_cast<const uint4*>(qrow + c * 16);
                    const __half2* h2 = reinterpret_cast<const __half2*>(&u);
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float2 f = __half22float2(h2[e]);
                        x[2 * e] = f.x;
                        x[2 * e + 1] = f.y;
                    }
                }
            }
            uint32_t hi[4], lo[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const __half2 h = __floats2half2_rn(x[2 * e], x[2 * e + 1]);
                const float2 hf = __half22float2(h);
                hi[e] = h2_bits(h);
                lo[e] = h2_bits(__floats2half2_rn(x[2 * e] - hf.x, x[2 * e + 1] - hf.y));
            }
            const uint32_t off = (uint32_t)(c >> 3) * (kPreRows * 128) + r * 128 + (((c & 7) ^ (r & 7)) << 4);
            *reinterpret_cast<uint4*>(sbase + L.q_hi + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
            *reinterpret_cast<uint4*>(sbase + L.q_lo + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
        }
    }
    fence_proxy_async_smem();  // Q -> visible to the tensor core
    tc_fence_before();
    __syncthreads();
    tc_fence_after();

    bool ok = true;
    int j_fail = 0;
    if (warp == 5) {
        // ===== copy producer (one lane): refill a stage once its MMAs have read it =====
        if (lane == 0) {
            for (int j = 0; j + kPreStages < n_steps && ok; ++j) {
                ok = mbar_wait_bounded(kv_empty + 8u * (j % kPreStages), (j / kPreStages) & 1);
                if (!ok) { j_fail = j + kPreStages; break; }
                issue_step(j + kPreStages, nxt_ids);
                load_ids(j + kPreStages + 1, nxt_ids);
            }
            if (!ok) {
                // bounded drain of the copies still in flight, then report
                for (int jj = 0; jj < issued; ++jj)
                    mbar_wait_bounded(kv_full + 8u * (jj % kPreStages), (jj / kPreStages) & 1);
                atomicOr(p.err, kErrTimeout);
            }
        }
    } else if (warp == 4) {
        // ===== MMA issuer (one lane) =====
        if (lane == 0) {
            // descriptors: the start-address field is the low 14 bits (address >> 4),
            // so offsets inside shared memory are added to a base descriptor
            const uint64_t dq_hi = sw128_desc(base + L.q_hi, 16, 1024), dq_lo = sw128_desc(base + L.q_lo, 16, 1024);
            const uint64_t dp0 = sw128_desc(base + L.p0, 16, 1024);
            const uint32_t idesc_pv = f16_idesc(D, true);
            auto issue_pv = [&](int j) {  // O += P(j) V(j), then free its stage and P buffer
                const int st = j % kPreStages, bb = j & 1;
                const int nblk = step_blocks(j);
                const uint64_t dv = sw128_desc(base + L.stage0 + st * STAGE + KPART, HALF_ROWS_BYTES, 1024);
                const uint64_t dp = dp0 + ((uint64_t)(bb * PBUF) >> 4);
                for (int ks = 0; ks < nblk; ++ks) {
                    const uint64_t bdesc = dv + ((uint64_t)(ks * (kBlock * 128)) >> 4);
                    umma_f16(tmem_o, dp + (uint64_t)(ks * 2), bdesc, idesc_pv, (j > 0 || ks > 0) ? 1u : 0u);
                    umma_f16(tmem_o, dp + ((uint64_t)(kPreRows * 128 + ks * 32) >> 4), bdesc, idesc_pv, 1u);
                }
                umma_commit(kv_empty + 8u * st);
                umma_commit(p_free + 8u * bb);
                umma_commit(pv_done);
            };
            // S(j) = Q K(j)^T into S buffer j&1, once its copies landed and
            // softmax(j-2) has read that buffer
            auto issue_s = [&](int j) -> bool {
                const int st = j % kPreStages, bb = j & 1;
                if (!mbar_wait_bounded(kv_full + 8u * st, (j / kPreStages) & 1)) return false;
                if (j >= 2 && !mbar_wait_bounded(s_free + 8u * bb, ((j - 2) >> 1) & 1)) return false;
                tc_fence_after();
                const uint64_t dk = sw128_desc(base + L.stage0 + st * STAGE, 16, 1024);
                const uint32_t idesc_s = f16_idesc(step_blocks(j) * kBlock, false);
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk) {
                    const uint64_t qoff = ((uint64_t)(kk >> 2) * (kPreRows * 128) + (kk & 3) * 32) >> 4;
                    const uint64_t koff = ((uint64_t)(kk >> 2) * HALF_ROWS_BYTES + (kk & 3) * 32) >> 4;
                    umma_f16(tmem + 64 * bb, dq_hi + qoff, dk + koff, idesc_s, kk > 0 ? 1u : 0u);
                    umma_f16(tmem + 64 * bb, dq_lo + qoff, dk + koff, idesc_s, 1u);
                }
                umma_commit(s_full + 8u * bb);
                return true;
            };
            // The tensor cores run S two steps ahead of P V: S(0), S(1), PV(0),
            // S(2), PV(1), ... so softmax(j+1) never waits on PV(j).
            for (int j = 0; j < min(2, n_steps) && ok; ++j) ok = issue_s(j);
            for (int j = 0; j < n_steps && ok; ++j) {
                ok = mbar_wait_bounded(p_full + 8u * (j & 1), (j >> 1) & 1);
                if (!ok) { j_fail = j; break; }
                tc_fence_after();
                issue_pv(j);
                if (j + 2 < n_steps && !(ok = issue_s(j + 2))) { j_fail = j; break; }
            }
            if (!ok) atomicOr(p.err, kErrTimeout);
        }
    } else {
        // ===== softmax warps: thread r owns query row r (TMEM lane r) =====
        const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
        const float scale_log2 = p.scale_log2;
        float m_use = -INFINITY, l_run = 0.f;
        for (int j = 0; j < n_steps; ++j) {
            const int bb = j & 1;
            const int npos = step_blocks(j) * kBlock;
            bool w_ok = mbar_wait_bounded(s_full + 8u * bb, (j >> 1) & 1);
            if (!__all_sync(0xffffffffu, w_ok)) { ok = false; break; }
            tc_fence_after();
            float sv_[64];
            {
                float tmp[32];
                tmem_ld32(tmem + 64 * bb + lane_off, tmp);
#pragma unroll
                for (int i = 0; i < 32; ++i) sv_[i] = tmp[i];
                if (npos > 32) {
                    tmem_ld32(tmem + 64 * bb + lane_off + 32, tmp);
#pragma unroll
                    for (int i = 0; i < 32; ++i) sv_[32 + i] = tmp[i];
                } else {
#pragma unroll
                    for (int i = 0; i < 32; ++i) sv_[32 + i] = 0.f;
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive1(s_free + 8u * bb);  // S buffer bb may be overwritten
            float mx = -INFINITY;
            const int pos0 = (item.blk0 + j * kPreStepBlocks) * kBlock;
#pragma unroll
            for (int i = 0; i < 64; ++i) {
                sv_[i] = i < npos && pos0 + i < lim ? sv_[i] * scale_log2 : -INFINITY;
                mx = fmaxf(mx, sv_[i]);
            }
            float alpha = 1.f;
            bool rescale = false;
            if (mx > m_use + kRescaleLog2 || m_use == -INFINITY) {
                alpha = m_use == -INFINITY ? 0.f : ex2(m_use - mx);
                rescale = m_use != -INFINITY;
                m_use = mx;
            }
            // P buffer bb is free once PV(j-2) has read it (waited before the
            // rescale, so pv_done is at most one phase behind PV(j-1))
            if (j >= 2) {
                w_ok = mbar_wait_bounded(p_free + 8u * bb, ((j - 2) >> 1) & 1);
                if (!__all_sync(0xffffffffu, w_ok)) { ok = false; break; }
            }
            if (__any_sync(0xffffffffu, rescale)) {
                // this warp's O rows are scaled once PV(j-1) has finished
                w_ok = mbar_wait_bounded(pv_done, (j - 1) & 1);
                if (!__all_sync(0xffffffffu, w_ok)) { ok = false; break; }
                tc_fence_after();
#pragma unroll 1
                for (int c0 = 0; c0 < D; c0 += 32) {
                    float o[32];
                    tmem_ld32(tmem_o + lane_off + c0, o);
#pragma unroll
                    for (int i = 0; i < 32; ++i) o[i] *= alpha;
                    tmem_st32(tmem_o + lane_off + c0, o);
                }
            }
            const uint32_t pb = L.p0 + bb * PBUF;
            // A row that has had no position yet (every one masked) keeps
            // m = -inf; its P is 0, taken against 0 rather than -inf.
            const float m_ref = m_use == -INFINITY ? 0.f : m_use;
            float lsum = 0.f;
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                uint32_t hi[4], lo[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float p0 = ex2(sv_[8 * c + 2 * e] - m_ref), p1 = ex2(sv_[8 * c + 2 * e + 1] - m_ref);
                    lsum += p0 + p1;
                    const __half2 h = __floats2half2_rn(p0, p1);
                    const float2 hf = __half22float2(h);
                    hi[e] = h2_bits(h);
                    lo[e] = h2_bits(__floats2half2_rn(p0 - hf.x, p1 - hf.y));
                }
                const uint32_t off = r * 128 + (((c & 7) ^ (r & 7)) << 4);
                *reinterpret_cast<uint4*>(sbase + pb + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
                *reinterpret_cast<uint4*>(sbase + pb + kPreRows * 128 + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
            }
            l_run = l_run * alpha + lsum;
            fence_proxy_async_smem();  // P rows (and O rescale) -> visible to the tensor core
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive1(p_full + 8u * bb);
        }
        if (ok && n_steps > 0) {
            const bool w_ok = mbar_wait_bounded(pv_done, (n_steps - 1) & 1);
            ok = __all_sync(0xffffffffu, w_ok);
        }
        if (ok) {
            tc_fence_after();
            const size_t row = ((size_t)tok * Hkv + item.head) * G + hg + (size_t)item.split * p.split_rows;
#pragma unroll 1
            for (int c0 = 0; c0 < D; c0 += 32) {
                float o[32];
                tmem_ld32(tmem_o + lane_off + c0, o);
                if (live) {
#pragma unroll
                    for (int i = 0; i < 32; i += 4)
                        *reinterpret_cast<float4*>(p.pre_o + row * D + c0 + i) =
                            make_float4(o[i], o[i + 1], o[i + 2], o[i + 3]);
                }
            }
            if (live) {
                p.pre_ml[row * 2] = m_use;
                p.pre_ml[row * 2 + 1] = l_run;
            }
        } else if (lane == 0) {
            atomicOr(p.err, kErrTimeout);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kPreTmemCols) : "memory");
    }
}

// -------------------------------------------------------------- K3/K4 ----
// CTAs [0, n_copies*n_layers): one (copy, layer) each, a contiguous block
// region of block_elems f16.  Remaining CTAs scatter table entries.
__global__ void __launch_bounds__(256) apply_plan_kernel(uint16_t* __restrict__ pool, size_t layer_stride,
                                                         size_t block_elems, int n_layers,
                                                         const int2* __restrict__ copies, int n_copies,
                                                         int32_t* __restrict__ tables, const int2* __restrict__ tw,
                                                         int n_tw, int n_blocks, long long n_entries, int32_t* err,
                                                         int parts) {
    // One CTA per (copy, layer, part): a block's bytes are split into
    // `parts` runs so a burst of copies keeps enough loads in flight.
    const int n_copy_ctas = n_copies * n_layers * parts;
    if ((int)blockIdx.x < n_copy_ctas) {
        const int part = blockIdx.x % parts;
        const int ci = blockIdx.x / (n_layers * parts), l = (blockIdx.x / parts) % n_layers;
        const int2 cp = copies[ci];
#ifdef LT_BOUNDS_CHECK
        if ((unsigned)cp.x >= (unsigned)n_blocks || (unsigned)cp.y >= (unsigned)n_blocks) {
            if (threadIdx.x == 0) atomicOr(err, kErrBounds);
            return;
        }
#endif
        const uint4* src = reinterpret_cast<const uint4*>(pool + (size_t)l * layer_stride + (size_t)cp.x * block_elems);
        uint4* dst = reinterpret_cast<uint4*>(pool + (size_t)l * layer_stride + (size_t)cp.y * block_elems);
        // this part's 16-byte words, up to 4 independent loads in flight per
        // thread before their stores
        const size_t n16 = block_elems * 2 / 16;
        const size_t per = (n16 + parts - 1) / parts;
        const size_t i0 = (size_t)part * per, i1 = min(n16, i0 + per);
        constexpr int U = 4;
        size_t i = i0 + threadIdx.x;
        for (; i + (U - 1) * blockDim.x < i1; i += U * blockDim.x) {
            uint4 t[U];
#pragma unroll
            for (int u = 0; u < U; ++u) t[u] = __ldg(src + i + u * blockDim.x);
#pragma unroll
            for (int u = 0; u < U; ++u) dst[i + u * blockDim.x] = t[u];
        }
        for (; i < i1; i += blockDim.x) dst[i] = __ldg(src + i);
    } else {
        const int i = (blockIdx.x - n_copy_ctas) * blockDim.x + threadIdx.x;
        if (i < n_tw) {
            const int2 w = tw[i];
#ifdef LT_BOUNDS_CHECK
            if (w.x < 0 || w.x >= n_entries || w.y >= n_blocks) {
                atomicOr(err, kErrBounds);
                return;
            }
#endif
            tables[w.x] = w.y;
        }
    }
}

// ---------------------------------------------------------- selftest ----
// A word that no code ever sets: the failure-path self-test waits on it.
__device__ uint32_t g_never_set;

// Lane 0 waits for g_never_set == 1 through the same bounded flag wait the
// attention merge uses, with the caller's limit; when the limit runs out it
// raises kErrTimeout and the kernel returns, leaving the context usable.
__global__ void wait_selftest_kernel(uint64_t limit_ns, int32_t* err) {
    if (threadIdx.x != 0) return;
    if (!wait_flag_bounded(&g_never_set, 1u, limit_ns)) atomicOr(err, kErrTimeout);
}

// ------------------------------------------------------ peer gather ----
struct GatherSrcs {
    const uint4* r[kMaxPeers];  // each rank's gather half (this process's mapping)
};

// Thread 0 of every CTA waits (bounded, system-scope acquire) for each
// rank's flag to reach `epoch` (wrap-safe comparison: a rank may already be
// one call ahead); the CTA then copies its share of out [n][nranks][slice],
// slice r of each token from rank r's gather half (NVLink loads for the
// other ranks; the acquire orders them after that rank's stores).  Launched
// as a programmatic dependent of the attention launch, so it starts polling
// while that launch's last CTAs retire; griddepcontrol.wait before it exits
// keeps "this kernel done" meaning "the attention launch done" for the work
// after it.
__global__ void __launch_bounds__(256) gather_wait_copy_kernel(const uint32_t* flags, int nranks, uint32_t epoch,
                                                               const __grid_constant__ GatherSrcs srcs, uint4* dst,
                                                               uint32_t n, uint32_t slice16, int32_t* err) {
    __shared__ int ok;
    if (threadIdx.x == 0) {
        int good = 1;
        const uint64_t t0 = global_ns();
        for (int r = 0; r < nranks && good; ++r) {
            while ((int32_t)(ld_acquire_sys(flags + r) - epoch) < 0) {
                if (global_ns() - t0 > kWaitLimitNs) {
                    good = 0;
                    break;
                }
                __nanosleep(200);  // gentle: this polls while the attention launch still streams
            }
        }
        if (!good) atomicOr(err, kErrTimeout);
        ok = good;
    }
    __syncthreads();
    if (ok) {
        const size_t row16 = (size_t)nranks * slice16, total = (size_t)n * row16;
        for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
            const int r = (int)((i % row16) / slice16);
            dst[i] = __ldcg(srcs.r[r] + i);
        }
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

// ---------------------------------------------------------- gather ----
// out[t][r] = gathered[r][t] for 16-byte chunks of one token's local heads.
__global__ void __launch_bounds__(256) gather_permute_kernel(const uint4* __restrict__ gathered, uint4* __restrict__ out,
                                                             int nranks, uint32_t n, uint32_t row16) {
    const size_t total = (size_t)nranks * n * row16;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const size_t c = i % row16, rt = i / row16;
        const size_t t = rt % n, r = rt / n;  // source order: [r][t][c]
        out[(t * nranks + r) * row16 + c] = gathered[i];
    }
}

// ------------------------------------------------------------- rows ----
template <int D>
__global__ void __launch_bounds__(256) rows_kernel(const uint16_t* __restrict__ pool_layer,
                                                   const int32_t* __restrict__ trow, int n, int n_kv_heads,
                                                   uint16_t* __restrict__ k_out, uint16_t* __restrict__ v_out,
                                                   int n_blocks, int32_t* err) {
    constexpr int CH = D / 8;
    const int gid = blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= n * n_kv_heads * 2 * CH) return;
    const int c = gid % CH;
    int r = gid / CH;
    const int kvsel = r & 1;
    r >>= 1;
    const int h = r % n_kv_heads;
    const int pos = r / n_kv_heads;
    const int b = checked_block(trow[pos / kBlock], n_blocks, err), slot = pos % kBlock;
    const uint16_t* src = pool_layer + (((size_t)b * n_kv_heads + h) * 2 + kvsel) * (kBlock * D) + chunk_off(c, slot);
    uint16_t* dst = (kvsel ? v_out : k_out) + (size_t)pos * n_kv_heads * D + (size_t)h * D + (size_t)c * 8;
    *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(src);
}

// Q8_0 pool: value q * d of each cell, rounded to f16 (nearest even).
template <int D>
__global__ void __launch_bounds__(256) rows_q8_kernel(const uint8_t* __restrict__ pool_layer,
                                                      const int32_t* __restrict__ trow, int n, int n_kv_heads,
                                                      uint16_t* __restrict__ k_out, uint16_t* __restrict__ v_out,
                                                      int n_blocks, int32_t* err) {
    constexpr int CH = D / 8;
    const int gid = blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= n * n_kv_heads * 2 * CH) return;
    const int c = gid % CH;
    int r = gid / CH;
    const int kvsel = r & 1;
    r >>= 1;
    const int h = r % n_kv_heads;
    const int pos = r / n_kv_heads;
    const int b = checked_block(trow[pos / kBlock], n_blocks, err), slot = pos % kBlock;
    const uint8_t* tile = pool_layer + ((size_t)b * n_kv_heads + h) * q8_tile_bytes(D);
    const float d = __half2float(__ushort_as_half(
        *reinterpret_cast<const uint16_t*>(tile + (kvsel ? 33 : 32) * D + ((c >> 2) * 16 + q8_pos(slot)) * 2)));
    uint16_t vals[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int e = 8 * c + i;
        const int off = kvsel ? 16 * D + e * 16 + q8_pos(slot) : q8_krun<D>(slot, e >> 4) + q8_pos(e & 15);
        vals[i] = f32_to_f16_ref((float)(int8_t)tile[off] * d);
    }
    uint16_t* dst = (kvsel ? v_out : k_out) + (size_t)pos * n_kv_heads * D + (size_t)h * D + (size_t)c * 8;
    *reinterpret_cast<uint4*>(dst) = make_uint4(vals[0] | (uint32_t(vals[1]) << 16), vals[2] | (uint32_t(vals[3]) << 16),
                                                vals[4] | (uint32_t(vals[5]) << 16), vals[6] | (uint32_t(vals[7]) << 16));
}

}  // namespace

namespace {

int sm_count(int dev) {
    static int sms[64] = {};
    if (sms[dev] == 0) cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
    return sms[dev];
}

template <int D, bool Q8>
cudaError_t ensure_attr(int dev) {
    // opt-in shared memory is a per-device attribute; size it for the largest
    // layout (f32 q, group 8)
    static bool set[64] = {};
    if (set[dev]) return cudaSuccess;
    const cudaError_t e = cudaFuncSetAttribute(paged_attn_kernel<D, Q8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               attn_smem(kMaxGroup, D, 1, Q8));
    if (e == cudaSuccess) set[dev] = true;
    return e;
}

template <int D, bool Q8>
int warps_for(int dev, int group, int q_f32) {
    // resident CTAs per SM for this layout, cached per (device, group, dtype)
    static int cache[64][kMaxGroup + 1][2] = {};
    int& c = cache[dev][group][q_f32 ? 1 : 0];
    if (c == 0) {
        if (ensure_attr<D, Q8>(dev) != cudaSuccess) return 0;
        int per_sm = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, paged_attn_kernel<D, Q8>, kWarps * 32,
                                                          attn_smem(group, D, q_f32, Q8)) != cudaSuccess)
            return 0;
        c = (per_sm < 1 ? 1 : per_sm) * sm_count(dev) * kWarps;
    }
    return c;
}

template <int D, bool Q8>
cudaError_t launch_attend_d(const AttnParams& p, cudaStream_t s) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if ((e = ensure_attr<D, Q8>(dev)) != cudaSuccess) return e;
    // Cooperative: merging warps wait for other CTAs' flags, so the whole
    // grid (sized to the resident capacity) must be co-resident.
    const dim3 grid((p.n_warps + kWarps - 1) / kWarps), block(kWarps * 32);
    if (p.pre_splits == 0) {
        void* args[] = {const_cast<AttnParams*>(&p)};
        return cudaLaunchCooperativeKernel(reinterpret_cast<const void*>(&paged_attn_kernel<D, Q8>), grid, block,
                                           args, attn_smem(p.group, D, p.q_f32, Q8), s);
    }
    // After a prefix pass: a programmatic dependent of it, so its first CTAs
    // stream the tokens' own blocks on the SMs the pass leaves free while the
    // pass runs, and the rest take the pass's SMs as its CTAs retire.  It can
    // start only once every CTA of the pass has started, and it reads the
    // pass's partials only after griddepcontrol.wait (fold_prefix).  Not
    // cooperative: that attribute holds the launch until the whole grid fits
    // at once.  Every CTA still becomes resident within the pass's run, since
    // the pass never waits on this launch; the merges' waits are bounded.
    // Config 3 (256 sequences on a 2048-token shared prefix): 0.104 ms per
    // launch pair against 0.114 ms with the launches in series.
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = attn_smem(p.group, D, p.q_f32, Q8);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, paged_attn_kernel<D, Q8>, p);
}

}  // namespace

int attend_warps(int device, int group, int head_dim, int q_f32, int q8) {
    if (device < 0 || device >= 64 || group < 1 || group > kMaxGroup) return 0;
    int prev = -1;
    cudaGetDevice(&prev);
    if (prev != device) cudaSetDevice(device);
    int w;
    if (q8)
        w = head_dim == 64 ? warps_for<64, true>(device, group, q_f32) : warps_for<128, true>(device, group, q_f32);
    else
        w = head_dim == 64 ? warps_for<64, false>(device, group, q_f32) : warps_for<128, false>(device, group, q_f32);
    if (prev != device && prev >= 0) cudaSetDevice(prev);
    return w;
}

cudaError_t launch_attend(const AttnParams& p, int head_dim, cudaStream_t s) {
    if (p.n_warps == 0) return cudaSuccess;
    if (p.q8) return head_dim == 64 ? launch_attend_d<64, true>(p, s) : launch_attend_d<128, true>(p, s);
    return head_dim == 64 ? launch_attend_d<64, false>(p, s) : launch_attend_d<128, false>(p, s);
}

int attend_launches(const AttnParams& p) { return p.n_warps == 0 ? 0 : 1; }

cudaError_t launch_prefix(const PrefixParams& p, int n_items, int head_dim, cudaStream_t s) {
    if (n_items <= 0) return cudaSuccess;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    static bool attr[64][2] = {};
    const size_t smem = PreSmem(head_dim).total + 1024;  // + alignment slack
    const int hi = head_dim == 64 ? 0 : 1;
    if (!attr[dev][hi]) {
        e = head_dim == 64
                ? cudaFuncSetAttribute(prefix_attn_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)
                : cudaFuncSetAttribute(prefix_attn_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        attr[dev][hi] = true;
    }
    if (head_dim == 64)
        prefix_attn_kernel<64><<<n_items, kPreThreads, smem, s>>>(p);
    else
        prefix_attn_kernel<128><<<n_items, kPreThreads, smem, s>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_gather_permute(const void* gathered, void* out, int nranks, uint32_t n, size_t row_bytes,
                                  cudaStream_t s) {
    const uint32_t row16 = (uint32_t)(row_bytes / 16);
    const size_t total = (size_t)nranks * n * row16;
    if (total == 0) return cudaSuccess;
    const unsigned blocks = (unsigned)std::min<size_t>((total + 255) / 256, 4096);
    gather_permute_kernel<<<blocks, 256, 0, s>>>(static_cast<const uint4*>(gathered), static_cast<uint4*>(out), nranks,
                                                 n, row16);
    return cudaGetLastError();
}

cudaError_t launch_write(uint16_t* pool_layer, const int2* cells, int n, int n_kv_heads, int head_dim, const void* k,
                         const void* v, int in_f32, int q8, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    const int threads = n * n_kv_heads * 2 * (head_dim / 8);
    const int blocks = (threads + 255) / 256;
    uint8_t* pool_bytes = reinterpret_cast<uint8_t*>(pool_layer);
    if (q8 && head_dim == 64)
        kv_write_q8_kernel<64><<<blocks, 256, 0, s>>>(pool_bytes, cells, n, n_kv_heads, k, v, in_f32);
    else if (q8)
        kv_write_q8_kernel<128><<<blocks, 256, 0, s>>>(pool_bytes, cells, n, n_kv_heads, k, v, in_f32);
    else if (head_dim == 64)
        kv_write_kernel<64><<<blocks, 256, 0, s>>>(pool_layer, cells, n, n_kv_heads, k, v, in_f32);
    else
        kv_write_kernel<128><<<blocks, 256, 0, s>>>(pool_layer, cells, n, n_kv_heads, k, v, in_f32);
    return cudaGetLastError();
}

cudaError_t launch_apply_plan(uint16_t* pool, size_t layer_stride_elems, size_t block_elems, int n_layers,
                              const int2* copies, int n_copies, int32_t* tables, const int2* tw, int n_tw,
                              int n_blocks, long long n_entries, int32_t* err, cudaStream_t s) {
    // a part of 16 KiB: one round of four 16-byte loads per thread
    const int parts = (int)std::max<size_t>(1, (block_elems * 2 + 16383) / 16384);
    const long long ctas = (long long)n_copies * n_layers * parts + (n_tw + 255) / 256;
    if (ctas == 0) return cudaSuccess;
    if (ctas > 0x7FFFFFFFll) return cudaErrorInvalidValue;
    apply_plan_kernel<<<(unsigned)ctas, 256, 0, s>>>(pool, layer_stride_elems, block_elems, n_layers, copies, n_copies,
                                                     tables, tw, n_tw, n_blocks, n_entries, err, parts);
    return cudaGetLastError();
}

cudaError_t launch_rows(const uint16_t* pool_layer, const int32_t* table_row, int n, int n_kv_heads, int head_dim,
                        uint16_t* k_out, uint16_t* v_out, int q8, int n_blocks, int32_t* err, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    const int threads = n * n_kv_heads * 2 * (head_dim / 8);
    const int blocks = (threads + 255) / 256;
    const uint8_t* pool_bytes = reinterpret_cast<const uint8_t*>(pool_layer);
    if (q8 && head_dim == 64)
        rows_q8_kernel<64><<<blocks, 256, 0, s>>>(pool_bytes, table_row, n, n_kv_heads, k_out, v_out, n_blocks, err);
    else if (q8)
        rows_q8_kernel<128><<<blocks, 256, 0, s>>>(pool_bytes, table_row, n, n_kv_heads, k_out, v_out, n_blocks, err);
    else if (head_dim == 64)
        rows_kernel<64><<<blocks, 256, 0, s>>>(pool_layer, table_row, n, n_kv_heads, k_out, v_out, n_blocks, err);
    else
        rows_kernel<128><<<blocks, 256, 0, s>>>(pool_layer, table_row, n, n_kv_heads, k_out, v_out, n_blocks, err);
    return cudaGetLastError();
}

cudaError_t launch_gather_wait_copy(const uint32_t* flags, int nranks, uint32_t epoch, void* const* srcs, void* out,
                                    uint32_t n, size_t slice_bytes, int32_t* err, cudaStream_t s) {
    if (nranks < 1 || nranks > kMaxPeers) return cudaErrorInvalidValue;
    GatherSrcs gs{};
    for (int r = 0; r < nranks; ++r) gs.r[r] = static_cast<const uint4*>(srcs[r]);
    const uint32_t slice16 = (uint32_t)(slice_bytes / 16);
    const size_t n16 = (size_t)n * nranks * slice16;
    const unsigned blocks = (unsigned)std::max<size_t>(1, std::min<size_t>((n16 + 255) / 256, 148));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(blocks);
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, gather_wait_copy_kernel, flags, nranks, epoch, gs, static_cast<uint4*>(out), n,
                              slice16, err);
}

cudaError_t launch_wait_selftest(uint64_t limit_ns, int32_t* err, cudaStream_t s) {
    wait_selftest_kernel<<<1, 32, 0, s>>>(limit_ns, err);
    return cudaGetLastError();
}

bool bounds_checked_build() {
#ifdef LT_BOUNDS_CHECK
    return true;
#else
    return false;
#endif
}

}  // namespace ltkv
