// sm_100a kernels of the paged KV-cache path.
//
//   kv_write_kernel      K1  KvCache::write (kv.rs:123-131): f32/f16 rows -> f16 pool cells
//   paged_attn_kernel    K2  attention closure of Model::forward (model.rs:431-476)
//   apply_plan_kernel    K3/K4  whole-block copies (copy-on-write kv.rs:99-110,
//                            compaction moves) + block-table scatter
//   rows_kernel              KvCache::rows (kv.rs:135-150) gather, for parity/debug
//
// Pool layout (per layer): f16 [block][kv_head][2 (K,V)][16 slots][D].  The
// 16-byte chunk c of the row of slot s sits at chunk position c ^ (s & 7):
// one (block, head) K+V tile is a contiguous 4*D*16-byte run whose
// bulk-copied shared-memory image is bank-conflict free for ldmatrix.
#include <cuda_fp16.h>
#include <stdint.h>

#include "lt_kv_internal.h"

namespace ltkv {
namespace {

constexpr int kWarps = 4;                       // warps per attention CTA
constexpr int kStages = 3;                      // bulk-copy stages per warp
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // bounded mbarrier wait: 2 s

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

// f32 -> f16 with the bit semantics of half 2.7.1's f16::from_f32: IEEE
// round-to-nearest-even (the hardware cvt.rn), and NaN -> quiet NaN that
// keeps the top 10 payload bits (the hardware returns a canonical NaN).
__device__ __forceinline__ uint16_t f32_to_f16_ref(float x) {
    const uint32_t u = __float_as_uint(x);
    if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x007FFFFFu))
        return static_cast<uint16_t>(((u >> 16) & 0x8000u) | 0x7E00u | ((u & 0x007FFFFFu) >> 13));
    return __half_as_ushort(__float2half_rn(x));
}

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

__device__ __forceinline__ int swz(int chunk, int slot) { return chunk ^ (slot & 7); }

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
    uint16_t* dst = pool_layer + (((size_t)cell.x * n_kv_heads + h) * 2 + kvsel) * (kBlock * D) +
                    (size_t)cell.y * D + (size_t)swz(c, cell.y) * 8;
    *reinterpret_cast<uint4*>(dst) = val;
}

// ------------------------------------------------------------------ K2 ----
// grid (n_items, n_kv_heads), kWarps warps.  Warp w of an item handles
// blocks b_begin + w, + kWarps, ... through its own kStages-deep ring of
// bulk copies.  Scores S = Q K^T and O += P V run on mma.sync m16n8k16:
// rows 0..7 of the A operand hold the (up to 8) query heads of this KV head
// rounded to f16, rows 8..15 hold the f16 rounding residual of the same
// values, so S and O carry ~22-bit q and P at no extra MMA cost.
template <int D>
__global__ void __launch_bounds__(kWarps * 32, 2) paged_attn_kernel(const AttnParams p) {
    constexpr int TILE = 2 * kBlock * D * 2;  // bytes of one (block, head) K+V tile
    constexpr int ROW = D * 2;                // bytes per row
    constexpr int KS = D / 16;                // k-steps of S = Q K^T
    constexpr int NT = D / 8;                 // n-tiles of O
    extern __shared__ __align__(1024) uint8_t smem[];
    __shared__ int s_flag[2];

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int h = blockIdx.y;
    const WorkItem it = p.items[blockIdx.x];
    const int Hkv = p.n_kv_heads, G = p.group;
    const int len = it.pos + 1;
    const int nb = (len + kBlock - 1) / kBlock;
    const int b_begin = it.chunk * it.cb;
    const int b_end = min(b_begin + it.cb, nb);
    const int32_t* trow = p.tables + (size_t)it.seq * p.max_blocks;
    const size_t tile_elems = 2 * kBlock * D;

    uint8_t* my_stages = smem + (size_t)warp * kStages * TILE;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + (size_t)kWarps * kStages * TILE);
    const uint32_t my_bar0 = smem_u32(bars + warp * kStages);

    if (threadIdx.x < kWarps * kStages) mbar_init(smem_u32(bars + threadIdx.x), 1);
    if (threadIdx.x == 0) s_flag[0] = 0;
    fence_mbar_init();
    __syncthreads();

    const int n_mine = (b_end - b_begin - warp + kWarps - 1) / kWarps;  // may be <= 0
    auto issue = [&](int j) {
        const int b = b_begin + warp + j * kWarps;
        const int pb = __ldg(trow + b);
        const uint16_t* src = p.pool_layer + ((size_t)pb * Hkv + h) * tile_elems;
        const int s = j % kStages;
        const uint32_t bar = my_bar0 + 8u * s;
        mbar_arrive_expect_tx(bar, TILE);
        bulk_g2s(smem_u32(my_stages + (size_t)s * TILE), src, TILE, bar);
    };
    int issued = 0;
    if (n_mine > 0) {
        issued = min(kStages, n_mine);
        if (lane == 0)
            for (int j = 0; j < issued; ++j) issue(j);
    }

    // Q fragments (A operand), loaded while the first copies are in flight.
    const int g = lane >> 2, t = lane & 3;
    uint32_t qa[KS][4];
    {
        const size_t qrow = ((size_t)it.tok * Hkv * G + (size_t)h * G + g) * D;
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {
                float x0 = 0.f, x1 = 0.f;
                if (g < G) {
                    const size_t e = qrow + ks * 16 + hf * 8 + 2 * t;
                    if (p.q_f32) {
                        const float2 f = *reinterpret_cast<const float2*>(static_cast<const float*>(p.q) + e);
                        x0 = f.x;
                        x1 = f.y;
                    } else {
                        const float2 f =
                            __half22float2(*reinterpret_cast<const __half2*>(static_cast<const __half*>(p.q) + e));
                        x0 = f.x;
                        x1 = f.y;
                    }
                }
                const __half2 hi = __floats2half2_rn(x0, x1);
                const float2 hf2 = __half22float2(hi);
                const __half2 lo = __floats2half2_rn(x0 - hf2.x, x1 - hf2.y);
                qa[ks][2 * hf] = h2_bits(hi);
                qa[ks][2 * hf + 1] = h2_bits(lo);
            }
        }
    }

    float o[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.f;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    int j = 0;
    for (; j < n_mine; ++j) {
        const int s = j % kStages;
        if (!mbar_wait_bounded(my_bar0 + 8u * s, (j / kStages) & 1)) {
            ok = false;
            break;
        }
        const int b = b_begin + warp + j * kWarps;
        uint8_t* tile = my_stages + (size_t)s * TILE;
        const int valid = min(kBlock, len - b * kBlock);
        bool touched = false;
        if (it.write_row && b == nb - 1) {
            // Fused append: this token's new K/V row for head h goes to the
            // pool cell and into the staged tile (the copy read the old bytes).
            constexpr int CH = D / 8;
            const int slot = it.pos % kBlock;
            if (lane < 2 * CH) {
                const int kvsel = lane / CH, c = lane % CH;
                const size_t src = (size_t)it.tok * Hkv * D + (size_t)h * D + (size_t)c * 8;
                const uint4 val = load8_as_f16(kvsel ? p.v_new : p.k_new, src, p.kv_f32);
                const int pc = swz(c, slot);
                uint16_t* dst = p.pool_layer_w + ((size_t)__ldg(trow + b) * Hkv + h) * tile_elems +
                                (size_t)kvsel * kBlock * D + (size_t)slot * D + (size_t)pc * 8;
                *reinterpret_cast<uint4*>(dst) = val;
                *reinterpret_cast<uint4*>(tile + kvsel * kBlock * ROW + slot * ROW + pc * 16) = val;
            }
            touched = true;
        }
        if (valid < kBlock) {
            // Rows past the sequence end were never written for it: zero V so
            // 0 * (stale NaN/Inf) cannot reach O; K rows are masked below.
            const int n16 = (kBlock - valid) * ROW / 16;
            uint4* vz = reinterpret_cast<uint4*>(tile + kBlock * ROW + valid * ROW);
            for (int e = lane; e < n16; e += 32) vz[e] = make_uint4(0, 0, 0, 0);
            touched = true;
        }
        __syncwarp();

        // S = Q K^T over this block's 16 tokens (two n-tiles of 8 tokens).
        float s0[4] = {0.f, 0.f, 0.f, 0.f}, s1[4] = {0.f, 0.f, 0.f, 0.f};
        const uint32_t kbase = smem_u32(tile);
        {
            const int mi = lane >> 3;
            const int tok = ((mi >> 1) << 3) + (lane & 7);
#pragma unroll
            for (int ks = 0; ks < KS; ++ks) {
                const int c = 2 * ks + (mi & 1);
                uint32_t b0, b1, b2, b3;
                ldsm_x4(kbase + tok * ROW + (swz(c, tok) << 4), b0, b1, b2, b3);
                mma16816(s0, qa[ks], b0, b1);
                mma16816(s1, qa[ks], b2, b3);
            }
        }
        float sc[4] = {(s0[0] + s0[2]) * p.scale_log2, (s0[1] + s0[3]) * p.scale_log2,
                       (s1[0] + s1[2]) * p.scale_log2, (s1[1] + s1[3]) * p.scale_log2};
        if (valid < kBlock) {
            if (2 * t >= valid) sc[0] = -INFINITY;
            if (2 * t + 1 >= valid) sc[1] = -INFINITY;
            if (2 * t + 8 >= valid) sc[2] = -INFINITY;
            if (2 * t + 9 >= valid) sc[3] = -INFINITY;
        }
        float mx = fmaxf(fmaxf(sc[0], sc[1]), fmaxf(sc[2], sc[3]));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const float m_new = fmaxf(m_run, mx);
        const float alpha = ex2(m_run - m_new);
        float pr[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) pr[e] = ex2(sc[e] - m_new);
        l_run = l_run * alpha + ((pr[0] + pr[1]) + (pr[2] + pr[3]));
        m_run = m_new;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            o[nt][0] *= alpha;
            o[nt][1] *= alpha;
            o[nt][2] *= alpha;
            o[nt][3] *= alpha;
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
        // O += P V (V^T fragments via ldmatrix.trans).
        {
            const uint32_t vbase = kbase + kBlock * ROW;
            const int mi = lane >> 3;
            const int tok = ((mi & 1) << 3) + (lane & 7);
#pragma unroll
            for (int np = 0; np < NT / 2; ++np) {
                const int c = 2 * np + (mi >> 1);
                uint32_t b0, b1, b2, b3;
                ldsm_x4_t(vbase + tok * ROW + (swz(c, tok) << 4), b0, b1, b2, b3);
                mma16816(o[2 * np], pa, b0, b1);
                mma16816(o[2 * np + 1], pa, b2, b3);
            }
        }
        // Generic-proxy writes into this stage must be ordered before the
        // async-proxy copy that may refill it.
        if (touched) fence_proxy_async_smem();
        __syncwarp();
        if (j + kStages < n_mine) {
            if (lane == 0) issue(j + kStages);
            ++issued;
        }
    }
    if (!ok) {
        // Give the copies still in flight a bounded chance to land before
        // this CTA's shared memory is released, then report the failure.
        for (int jj = j + 1; jj < issued; ++jj) mbar_wait_bounded(my_bar0 + 8u * (jj % kStages), (jj / kStages) & 1);
        if (lane == 0) {
            s_flag[0] = 1;
            atomicExch(p.err, 1);
        }
    }
    __syncthreads();
    if (s_flag[0]) return;

    // Combine the warps of this CTA (stage memory is free: every copy landed).
    float* cm = reinterpret_cast<float*>(smem);
    float* cl = cm + kWarps * kMaxGroup;
    float* co = cl + kWarps * kMaxGroup;
    float l_tot = l_run;
    l_tot += __shfl_xor_sync(0xffffffffu, l_tot, 1);
    l_tot += __shfl_xor_sync(0xffffffffu, l_tot, 2);
    if (g < G) {
        if (t == 0) {
            cm[warp * kMaxGroup + g] = m_run;
            cl[warp * kMaxGroup + g] = l_tot;
        }
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
            *reinterpret_cast<float2*>(co + (size_t)(warp * kMaxGroup + g) * D + nt * 8 + 2 * t) =
                make_float2(o[nt][0] + o[nt][2], o[nt][1] + o[nt][3]);
    }
    __syncthreads();

    const int GD = G * D;
    const size_t out_base = ((size_t)it.tok * Hkv + h) * GD;  // == tok*Hq*D + h*G*D
    if (it.nchunks == 1) {
        for (int e = threadIdx.x; e < GD; e += blockDim.x) {
            const int gg = e / D, d = e % D;
            float M = -INFINITY;
#pragma unroll
            for (int w = 0; w < kWarps; ++w) M = fmaxf(M, cm[w * kMaxGroup + gg]);
            float L = 0.f, O = 0.f;
#pragma unroll
            for (int w = 0; w < kWarps; ++w) {
                const float sw = ex2(cm[w * kMaxGroup + gg] - M);
                L += cl[w * kMaxGroup + gg] * sw;
                O += co[(size_t)(w * kMaxGroup + gg) * D + d] * sw;
            }
            const float r = O / L;
            if (p.out_f32)
                static_cast<float*>(p.out)[out_base + e] = r;
            else
                static_cast<__half*>(p.out)[out_base + e] = __float2half_rn(r);
        }
        return;
    }

    const size_t slot = (size_t)(it.part_base + it.chunk) * Hkv + h;
    for (int e = threadIdx.x; e < GD; e += blockDim.x) {
        const int gg = e / D, d = e % D;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) M = fmaxf(M, cm[w * kMaxGroup + gg]);
        float L = 0.f, O = 0.f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) {
            const float sw = ex2(cm[w * kMaxGroup + gg] - M);
            L += cl[w * kMaxGroup + gg] * sw;
            O += co[(size_t)(w * kMaxGroup + gg) * D + d] * sw;
        }
        p.part_o[slot * GD + e] = O;
        if (d == 0) {
            p.part_ml[(slot * G + gg) * 2] = M;
            p.part_ml[(slot * G + gg) * 2 + 1] = L;
        }
    }
    __threadfence();
    __syncthreads();
    int32_t* counter = p.counters + (size_t)it.tok * Hkv + h;
    if (threadIdx.x == 0) s_flag[1] = (atomicAdd(counter, 1) == it.nchunks - 1);
    __syncthreads();
    if (!s_flag[1]) return;
    __threadfence();
    // Last item of (tok, head): merge all chunks' (m, l, o).
    const size_t base = (size_t)it.part_base * Hkv + h;
    for (int e = threadIdx.x; e < GD; e += blockDim.x) {
        const int gg = e / D;
        float M = -INFINITY;
        for (int c = 0; c < it.nchunks; ++c)
            M = fmaxf(M, __ldcg(p.part_ml + ((base + (size_t)c * Hkv) * G + gg) * 2));
        float L = 0.f, O = 0.f;
        for (int c = 0; c < it.nchunks; ++c) {
            const size_t sl = base + (size_t)c * Hkv;
            const float sw = ex2(__ldcg(p.part_ml + (sl * G + gg) * 2) - M);
            L += __ldcg(p.part_ml + (sl * G + gg) * 2 + 1) * sw;
            O += __ldcg(p.part_o + sl * GD + e) * sw;
        }
        const float r = O / L;
        if (p.out_f32)
            static_cast<float*>(p.out)[out_base + e] = r;
        else
            static_cast<__half*>(p.out)[out_base + e] = __float2half_rn(r);
    }
    if (threadIdx.x == 0) *counter = 0;
}

// -------------------------------------------------------------- K3/K4 ----
// CTAs [0, n_copies*n_layers): one (copy, layer) each, a contiguous block
// region of block_elems f16.  Remaining CTAs scatter table entries.
__global__ void __launch_bounds__(256) apply_plan_kernel(uint16_t* __restrict__ pool, size_t layer_stride,
                                                         size_t block_elems, int n_layers,
                                                         const int2* __restrict__ copies, int n_copies,
                                                         int32_t* __restrict__ tables, const int2* __restrict__ tw,
                                                         int n_tw) {
    const int n_copy_ctas = n_copies * n_layers;
    if ((int)blockIdx.x < n_copy_ctas) {
        const int ci = blockIdx.x / n_layers, l = blockIdx.x % n_layers;
        const int2 cp = copies[ci];
        const uint4* src = reinterpret_cast<const uint4*>(pool + (size_t)l * layer_stride + (size_t)cp.x * block_elems);
        uint4* dst = reinterpret_cast<uint4*>(pool + (size_t)l * layer_stride + (size_t)cp.y * block_elems);
        const size_t n16 = block_elems * 2 / 16;
        for (size_t i = threadIdx.x; i < n16; i += blockDim.x) dst[i] = __ldg(src + i);
    } else {
        const int i = (blockIdx.x - n_copy_ctas) * blockDim.x + threadIdx.x;
        if (i < n_tw) {
            const int2 w = tw[i];
            tables[w.x] = w.y;
        }
    }
}

// ------------------------------------------------------------- rows ----
template <int D>
__global__ void __launch_bounds__(256) rows_kernel(const uint16_t* __restrict__ pool_layer,
                                                   const int32_t* __restrict__ trow, int n, int n_kv_heads,
                                                   uint16_t* __restrict__ k_out, uint16_t* __restrict__ v_out) {
    constexpr int CH = D / 8;
    const int gid = blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= n * n_kv_heads * 2 * CH) return;
    const int c = gid % CH;
    int r = gid / CH;
    const int kvsel = r & 1;
    r >>= 1;
    const int h = r % n_kv_heads;
    const int pos = r / n_kv_heads;
    const int b = trow[pos / kBlock], slot = pos % kBlock;
    const uint16_t* src = pool_layer + (((size_t)b * n_kv_heads + h) * 2 + kvsel) * (kBlock * D) + (size_t)slot * D +
                          (size_t)swz(c, slot) * 8;
    uint16_t* dst = (kvsel ? v_out : k_out) + (size_t)pos * n_kv_heads * D + (size_t)h * D + (size_t)c * 8;
    *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(src);
}

template <int D>
int smem_bytes_for() {
    return kWarps * kStages * (2 * kBlock * D * 2) + kWarps * kStages * 8;
}

}  // namespace

int attn_smem_bytes(int head_dim) { return head_dim == 64 ? smem_bytes_for<64>() : smem_bytes_for<128>(); }

template <int D>
cudaError_t launch_attend_d(const AttnParams& p, cudaStream_t s) {
    // The opt-in shared-memory size is a per-device function attribute.
    static bool attr_set[64] = {};
    const int sm = smem_bytes_for<D>();
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!attr_set[dev]) {
        e = cudaFuncSetAttribute(paged_attn_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm);
        if (e != cudaSuccess) return e;
        attr_set[dev] = true;
    }
    paged_attn_kernel<D><<<dim3(p.n_items, p.n_kv_heads), kWarps * 32, sm, s>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_attend(const AttnParams& p, int head_dim, cudaStream_t s) {
    if (p.n_items == 0) return cudaSuccess;
    return head_dim == 64 ? launch_attend_d<64>(p, s) : launch_attend_d<128>(p, s);
}

cudaError_t launch_write(uint16_t* pool_layer, const int2* cells, int n, int n_kv_heads, int head_dim, const void* k,
                         const void* v, int in_f32, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    const int threads = n * n_kv_heads * 2 * (head_dim / 8);
    const int blocks = (threads + 255) / 256;
    if (head_dim == 64)
        kv_write_kernel<64><<<blocks, 256, 0, s>>>(pool_layer, cells, n, n_kv_heads, k, v, in_f32);
    else
        kv_write_kernel<128><<<blocks, 256, 0, s>>>(pool_layer, cells, n, n_kv_heads, k, v, in_f32);
    return cudaGetLastError();
}

cudaError_t launch_apply_plan(uint16_t* pool, size_t layer_stride_elems, size_t block_elems, int n_layers,
                              const int2* copies, int n_copies, int32_t* tables, const int2* tw, int n_tw,
                              cudaStream_t s) {
    const int ctas = n_copies * n_layers + (n_tw + 255) / 256;
    if (ctas == 0) return cudaSuccess;
    apply_plan_kernel<<<ctas, 256, 0, s>>>(pool, layer_stride_elems, block_elems, n_layers, copies, n_copies, tables,
                                           tw, n_tw);
    return cudaGetLastError();
}

cudaError_t launch_rows(const uint16_t* pool_layer, const int32_t* table_row, int n, int n_kv_heads, int head_dim,
                        uint16_t* k_out, uint16_t* v_out, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    const int threads = n * n_kv_heads * 2 * (head_dim / 8);
    const int blocks = (threads + 255) / 256;
    if (head_dim == 64)
        rows_kernel<64><<<blocks, 256, 0, s>>>(pool_layer, table_row, n, n_kv_heads, k_out, v_out);
    else
        rows_kernel<128><<<blocks, 256, 0, s>>>(pool_layer, table_row, n, n_kv_heads, k_out, v_out);
    return cudaGetLastError();
}

}  // namespace ltkv
