// sm_100a Llama step around the paged KV cache: the operations on either
// side of the attention path in Model::forward (model.rs:366-518).
//
//   q8_matmul_kernel   QMatrix::matmul (quant.rs:405-428, 492-533): int8 dot
//                      products on the tensor cores (mma.sync m16n8k32 s8,
//                      one 32-wide Q8_0 block per instruction), scales applied
//                      per block and summed block by block in the reference's
//                      order, so results are bit-identical to row_dot
//   quantize_kernel    QActs::quantize (quant.rs:771-795)
//   rms_norm_q8_kernel rms_norm (model.rs:174-183) + quantize
//   rope_split_kernel  RoPE of q and k (model.rs:291-308, 414-421) and the
//                      split of the fused q|k|v projection into q, k, v
//   silu_q8_kernel     SiLU(gate) * up (model.rs:492-494) + quantize
//   embed_kernel       Q8_0 embedding rows (quant.rs:464-490)
//   argmax_kernel      greedy pick (sampling.rs:161-163)
//
// Weights live on the device in a split Q8_0 layout: int8 [rows][cols] and
// f16 scales [rows][cols/32] (the GGUF block's d, unchanged).  Projections
// that share an input are stored as one matrix: q|k|v rows, and gate|up rows,
// so each is one launch (the reference's matmul_many, quant.rs:722).
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "lt_kv.h"
#include "lt_kv_internal.h"
#include "lt_llama.h"
#include "lt_llama_decode.h"
#include "lt_q8_device.cuh"

using namespace ltq8;

namespace {

constexpr int kMmWarps = 16;     // warps per matmul CTA (K blocks dealt round-robin)
constexpr int kMmRows = 16;      // weight rows per matmul CTA (mma M)
constexpr int kMmToks = 8;       // tokens per matmul CTA (mma N)

// ------------------------------------------------------------ helpers -----

__device__ __forceinline__ uint2 ld_stream(const void* p) {  // weights: read once
    uint2 v;
    asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
    return v;
}

// ------------------------------------------------------------ kernels -----

// out[t][r] (+)= sum_b (ws[r][b] * xs[t][b]) * dot32(W[r][b], X[t][b]),
// summed over b = 0, 1, ... from 0.0f (row_dot, quant.rs:418-421).
// CTA: 16 rows x 8 tokens.  Its 16 warps take the 32-wide blocks round-robin
// and run one s8 mma per block: lane (g, q) loads bytes [8q, 8q+8) of its
// block for rows g and g+8 and token g; the same k permutation on both
// operands leaves each dot32 unchanged.  The four f32 products of every lane
// and block go to shared memory; warp 0 then adds them block by block.
__global__ void __launch_bounds__(kMmWarps * 32) q8_matmul_kernel(
    const int8_t* __restrict__ wq, const __half* __restrict__ ws, int rows, int cols,
    const int8_t* __restrict__ xq, const float* __restrict__ xs, int n, float* __restrict__ out, int out_stride,
    int accumulate) {
    extern __shared__ float4 prod[];  // [nb][32]
    const int nb = cols / kQK;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, q = lane & 3;
    const int r0 = blockIdx.x * kMmRows, t0 = blockIdx.y * kMmToks;
    const int ra = min(r0 + g, rows - 1), rb = min(r0 + g + 8, rows - 1);
    const int tb_op = min(t0 + g, n - 1);                                // B operand token
    const int ta = min(t0 + 2 * q, n - 1), tc = min(t0 + 2 * q + 1, n - 1);  // C columns
    const int8_t* wa = wq + (size_t)ra * cols + 8 * q;
    const int8_t* wb = wq + (size_t)rb * cols + 8 * q;
    const int8_t* xb = xq + (size_t)tb_op * cols + 8 * q;
    const __half* sa = ws + (size_t)ra * nb;
    const __half* sb = ws + (size_t)rb * nb;
    const float* xa = xs + (size_t)ta * nb;
    const float* xc = xs + (size_t)tc * nb;
#pragma unroll 4
    for (int b = warp; b < nb; b += kMmWarps) {
        const uint2 A0 = ld_stream(wa + (size_t)b * kQK);
        const uint2 A1 = ld_stream(wb + (size_t)b * kQK);
        const uint2 B = __ldg(reinterpret_cast<const uint2*>(xb + (size_t)b * kQK));
        int d[4];
        mma_s8(d, A0.x, A1.x, A0.y, A1.y, B.x, B.y);
        const float wsa = __half2float(sa[b]), wsb = __half2float(sb[b]);
        const float xsa = __ldg(xa + b), xsc = __ldg(xc + b);
        float4 p;
        p.x = __fmul_rn(__fmul_rn(wsa, xsa), __int2float_rn(d[0]));  // row g,   token 2q
        p.y = __fmul_rn(__fmul_rn(wsa, xsc), __int2float_rn(d[1]));  // row g,   token 2q+1
        p.z = __fmul_rn(__fmul_rn(wsb, xsa), __int2float_rn(d[2]));  // row g+8, token 2q
        p.w = __fmul_rn(__fmul_rn(wsb, xsc), __int2float_rn(d[3]));  // row g+8, token 2q+1
        prod[b * 32 + lane] = p;
    }
    __syncthreads();
    if (warp != 0) return;
    float4 s = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll 8
    for (int b = 0; b < nb; b++) {
        const float4 p = prod[b * 32 + lane];
        s.x = __fadd_rn(s.x, p.x);
        s.y = __fadd_rn(s.y, p.y);
        s.z = __fadd_rn(s.z, p.z);
        s.w = __fadd_rn(s.w, p.w);
    }
    const int rr[2] = {r0 + g, r0 + g + 8};
    const int tt[2] = {t0 + 2 * q, t0 + 2 * q + 1};
    const float v[4] = {s.x, s.y, s.z, s.w};
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int r = rr[i >> 1], t = tt[i & 1];
        if (r < rows && t < n) {
            float* o = out + (size_t)t * out_stride + r;
            *o = accumulate ? __fadd_rn(*o, v[i]) : v[i];
        }
    }
}

// QActs::quantize over n*cols/8 threads, 8 values each.
__global__ void quantize_kernel(const float* __restrict__ x, size_t n_threads, int8_t* __restrict__ qs,
                                float* __restrict__ scales) {
    // Lanes past the end stay for the group shuffles (n_threads is a multiple
    // of 4, so a group is wholly in or out) but neither load nor store.
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    const bool live = i < n_threads;
    float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (live) load8(x + i * 8, v);
    quant8_store(v, qs + i * 8, scales + i / 4, (threadIdx.x & 3) == 0, live);
}

// rms_norm then quantize: one CTA per output row, dim/8 threads.  The sum of
// squares is a tree (the reference's is sequential: a few ulps apart).
__global__ void rms_norm_q8_kernel(const float* __restrict__ x, const int32_t* __restrict__ rows_idx,
                                   const float* __restrict__ w, int dim, float eps, float* __restrict__ normed,
                                   int8_t* __restrict__ qs, float* __restrict__ scales) {
    __shared__ float red[32];
    const int row = blockIdx.x;
    const int src = rows_idx ? rows_idx[row] : row;
    const int i = threadIdx.x;
    float v[8];
    load8(x + (size_t)src * dim + i * 8, v);
    float ss = 0.0f;
#pragma unroll
    for (int k = 0; k < 8; k++) ss = __fadd_rn(ss, __fmul_rn(v[k], v[k]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
    if ((i & 31) == 0) red[i >> 5] = ss;
    __syncthreads();
    const int nw = blockDim.x >> 5;
    if (i < 32) {
        float t = i < nw ? red[i] : 0.0f;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) t = __fadd_rn(t, __shfl_xor_sync(0xffffffffu, t, o));
        if (i == 0) red[0] = t;
    }
    __syncthreads();
    const float ms = __fdiv_rn(red[0], (float)dim);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, eps)));
    float wv[8];
    load8(w + i * 8, wv);
#pragma unroll
    for (int k = 0; k < 8; k++) v[k] = __fmul_rn(__fmul_rn(v[k], inv), wv[k]);
    if (normed) store8(normed + (size_t)row * dim + i * 8, v);
    quant8_store(v, qs + (size_t)row * dim + i * 8, scales + ((size_t)row * dim + i * 8) / kQK, (i & 3) == 0);
}

// SiLU(g) * u = g / (1 + exp(-g)) * u, then quantize.  exp is rounded once
// to f32 from a double-precision exp: the correctly rounded f32 value.  The
// C library expf that the reference calls is one ulp away from it on about
// 0.03 % of inputs (near rounding midpoints).
__global__ void silu_q8_kernel(const float* __restrict__ gu, int n, int ffn, float* __restrict__ h,
                               int8_t* __restrict__ qs, float* __restrict__ scales) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");  // no-ops unless launched as a dependent
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    const size_t per_row = (size_t)ffn / 8;  // a multiple of 4: groups are wholly in or out
    const bool live = i < per_row * n;
    const size_t t = live ? i / per_row : 0, c = live ? (i % per_row) * 8 : 0;
    float gv[8], uv[8];
    load8(gu + t * 2 * ffn + c, gv);  // past the end: reload row 0, store nothing
    load8(gu + t * 2 * ffn + ffn + c, uv);
#pragma unroll
    for (int k = 0; k < 8; k++) {
        const float e = (float)exp(-(double)gv[k]);
        gv[k] = __fmul_rn(__fdiv_rn(gv[k], __fadd_rn(1.0f, e)), uv[k]);
    }
    if (h && live) store8(h + t * ffn + c, gv);
    quant8_store(gv, qs + t * ffn + c, scales + (t * ffn + c) / kQK, (threadIdx.x & 3) == 0, live);
}

// RoPE of the q and k parts of one token's q|k|v row and the split into q,
// k, v rows.  sincos [n][half][2] (sin, cos) of pos * inv_freq[i].  Grid:
// (tokens, ceil(row / 256)), one element a thread.  Launched as a dependent
// of the q|k|v matmul: it waits for it before reading.
__global__ void rope_split_kernel(const float* __restrict__ qkv, int q_dim, int kv_dim, int hd, int half, int neox,
                                  const float* __restrict__ sincos, float* __restrict__ qo, float* __restrict__ ko,
                                  float* __restrict__ vo) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int t = blockIdx.x;
    const int j = blockIdx.y * blockDim.x + threadIdx.x;
    if (j >= q_dim + 2 * kv_dim) return;
    const float* row = qkv + (size_t)t * (q_dim + 2 * kv_dim);
    const float* sc = sincos + (size_t)t * half * 2;
    float r = row[j];
    if (j < q_dim + kv_dim) {
        const int base = j - j % hd, c = j % hd;
        int i = -1, partner = 0;
        bool first = true;
        if (neox) {
            if (c < half) { i = c; partner = c + half; }
            else if (c < 2 * half) { i = c - half; partner = c - half; first = false; }
        } else if (c < 2 * half) {
            i = c >> 1; partner = c ^ 1; first = (c & 1) == 0;
        }
        if (i >= 0) {
            const float sn = sc[2 * i], cs = sc[2 * i + 1];
            const float other = row[base + partner];
            r = first ? __fsub_rn(__fmul_rn(r, cs), __fmul_rn(other, sn))     // x0 cos - x1 sin
                      : __fadd_rn(__fmul_rn(other, sn), __fmul_rn(r, cs));    // x0 sin + x1 cos
        }
    }
    if (j < q_dim) qo[(size_t)t * q_dim + j] = r;
    else if (j < q_dim + kv_dim) ko[(size_t)t * kv_dim + (j - q_dim)] = r;
    else vo[(size_t)t * kv_dim + (j - q_dim - kv_dim)] = r;
}

// Embedding rows: x[i][j] = d[tok][j/32] * q[tok][j].
__global__ void embed_kernel(const int8_t* __restrict__ qs, const __half* __restrict__ sc, int dim,
                             const int32_t* __restrict__ tokens, float* __restrict__ x) {
    const int i = blockIdx.x;
    const size_t tok = (size_t)tokens[i];
    for (int j = threadIdx.x; j < dim; j += blockDim.x)
        x[(size_t)i * dim + j] = __fmul_rn(__half2float(sc[tok * (dim / kQK) + j / kQK]), (float)qs[tok * dim + j]);
}

// Greedy pick: max under f32 total order, the last index among equal keys.
__device__ __forceinline__ int32_t total_key(float f) {
    const int32_t b = __float_as_int(f);
    return b < 0 ? (b ^ 0x7fffffff) : b;
}

__global__ void argmax_kernel(const float* __restrict__ x, int cols, int32_t* __restrict__ idx) {
    __shared__ int32_t sk[32], si[32];
    const float* row = x + (size_t)blockIdx.x * cols;
    int32_t bk = INT32_MIN, bi = -1;
    for (int j = threadIdx.x; j < cols; j += blockDim.x) {
        const int32_t k = total_key(row[j]);
        if (k >= bk) { bk = k; bi = j; }  // j rises: ties keep the later index
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const int32_t k2 = __shfl_xor_sync(0xffffffffu, bk, o), i2 = __shfl_xor_sync(0xffffffffu, bi, o);
        if (k2 > bk || (k2 == bk && i2 > bi)) { bk = k2; bi = i2; }
    }
    if ((threadIdx.x & 31) == 0) { sk[threadIdx.x >> 5] = bk; si[threadIdx.x >> 5] = bi; }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); w++)
            if (sk[w] > bk || (sk[w] == bk && si[w] > bi)) { bk = sk[w]; bi = si[w]; }
        idx[blockIdx.x] = bi < 0 ? 0 : bi;
    }
}

// ------------------------------------------------------------ launchers ---

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

cudaError_t launch_matmul(const int8_t* wq, const __half* ws, int rows, int cols, const int8_t* xq, const float* xs,
                          int n, float* out, int out_stride, int accumulate, cudaStream_t st) {
    if (rows <= 0 || n <= 0) return cudaSuccess;
    static bool attr_set[64] = {};
    const size_t smem = (size_t)(cols / kQK) * 32 * sizeof(float4);
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!attr_set[dev]) {
        const cudaError_t e = cudaFuncSetAttribute(q8_matmul_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   200 * 1024);
        if (e != cudaSuccess) return e;
        attr_set[dev] = true;
    }
    dim3 grid((rows + kMmRows - 1) / kMmRows, (n + kMmToks - 1) / kMmToks);
    q8_matmul_kernel<<<grid, kMmWarps * 32, smem, st>>>(wq, ws, rows, cols, xq, xs, n, out, out_stride, accumulate);
    return cudaGetLastError();
}

cudaError_t launch_quantize(const float* x, size_t n_elems, int8_t* qs, float* scales, cudaStream_t st) {
    const size_t threads = n_elems / 8;
    if (!threads) return cudaSuccess;
    quantize_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, st>>>(x, threads, qs, scales);
    return cudaGetLastError();
}

cudaError_t launch_rms_norm_q8(const float* x, const int32_t* rows_idx, const float* w, int dim, int n, float eps,
                               float* normed, int8_t* qs, float* scales, cudaStream_t st) {
    if (!n) return cudaSuccess;
    rms_norm_q8_kernel<<<n, dim / 8, 0, st>>>(x, rows_idx, w, dim, eps, normed, qs, scales);
    return cudaGetLastError();
}

cudaError_t launch_silu_q8(const float* gu, int n, int ffn, float* h, int8_t* qs, float* scales, cudaStream_t st,
                           bool dependent = false) {
    const size_t threads = (size_t)n * ffn / 8;
    if (!threads) return cudaSuccess;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((threads + 255) / 256));
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = dependent ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, silu_q8_kernel, gu, n, ffn, h, qs, scales);
}

cudaError_t launch_rope_split(const float* qkv, int n, int q_dim, int kv_dim, int hd, int half, int neox,
                              const float* sincos, float* qo, float* ko, float* vo, cudaStream_t st) {
    if (!n) return cudaSuccess;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(n, (q_dim + 2 * kv_dim + 255) / 256);
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, rope_split_kernel, qkv, q_dim, kv_dim, hd, half, neox, sincos, qo, ko, vo);
}

cudaError_t launch_argmax(const float* x, int n, int cols, int32_t* idx, cudaStream_t st) {
    if (!n) return cudaSuccess;
    argmax_kernel<<<n, 1024, 0, st>>>(x, cols, idx);
    return cudaGetLastError();
}


// ---------------------------------------------------------------------------
// Decode matmul: q8_gemv_kernel, for n <= 8 tokens and cols % 256 == 0.
//
// One CTA owns 16 weight rows.  Lanes 0-15 bulk-copy one row each and its
// f16 scales into shared memory (cp.async.bulk, one mbarrier) before the CTA
// waits for the kernel that produced its activations (programmatic
// dependent launch: griddepcontrol), so the weight stream of this matmul
// overlaps the tail of the previous kernel.  The activation prologue is fused:
// the CTA builds the int8 activations of its (up to 8) tokens in shared memory
// from the producer's f32 output -- RMSNorm + quantize, quantize, or
// SiLU * up + quantize -- with the same arithmetic, thread mapping and
// reduction tree as the standalone kernels, so results are identical to
// running them separately.  Then 16 warps run one s8 mma per 32-wide block
// (block b to warp b % 16), overwrite the block's weight bytes with their f32
// products, and warp 0 adds the products block by block from 0.0f in the
// reference's order.

constexpr int kGvWarps = 16;
constexpr int kGvThreads = kGvWarps * 32;
__device__ uint32_t g_op_err;  // error flag of the op-level entry points
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // bounded mbarrier wait: 2 s
enum { PRO_Q8 = 0, PRO_QUANT = 1, PRO_SILU = 2, PRO_NORM = 3 };

struct GemvArgs {
    const int8_t* wq;
    const __half* ws;
    int rows, cols;
    float* out;
    int out_stride, accumulate, n;
    const float* x;           // QUANT [n][cols]; SILU [n][2*cols]; NORM rows of [*][cols]
    const int32_t* rows_idx;  // NORM: source row of each token (NULL: 0..n-1)
    const float* gamma;       // NORM weight
    float eps;
    const int8_t* xq;         // Q8: activations given
    const float* xs;
    uint32_t* err;            // set to 1 when a bounded wait gives up
};

struct GemvSmem {
    int pitch, ws_pitch, xs_pitch;
    size_t off_w, off_ws, off_xq, off_xs, off_red, total;
    __host__ __device__ explicit GemvSmem(int cols) {
        const int nb = cols / kQK;
        pitch = cols + 32;        // conflict-free 8-byte operand reads
        ws_pitch = nb * 2 + 16;   // bytes; keeps the bulk-copy destinations 16-byte aligned
        xs_pitch = nb + 4;        // floats
        off_w = 128;
        off_ws = off_w + (size_t)16 * pitch;
        off_xq = off_ws + (size_t)16 * ws_pitch;
        off_xs = off_xq + (size_t)8 * pitch;
        off_red = off_xs + (size_t)8 * xs_pitch * 4;
        total = off_red + 16 * 32 * 4;
    }
};

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

__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 15u) == 0 && global_ns() - t0 > kWaitLimitNs) return false;
    }
}

__device__ __forceinline__ void pdl_trigger_and_wait() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

// RMSNorm + quantize of token rows into shared memory: cols/8 threads per
// token, the reduction tree of rms_norm_q8_kernel.
__device__ __forceinline__ void prologue_norm(const GemvArgs& a, const GemvSmem& L, uint8_t* sm) {
    const int tpt = a.cols / 8, per_pass = kGvThreads / tpt;
    const int slot = threadIdx.x / tpt, i = threadIdx.x % tpt, nw = tpt / 32;
    float* red = reinterpret_cast<float*>(sm + L.off_red);
    for (int t0 = 0; t0 < a.n; t0 += per_pass) {
        const int t = t0 + slot;
        const bool live = t < a.n;
        float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        if (live) load8(a.x + (size_t)(a.rows_idx ? a.rows_idx[t] : t) * a.cols + i * 8, v);
        float ss = 0.0f;
#pragma unroll
        for (int k = 0; k < 8; k++) ss = __fadd_rn(ss, __fmul_rn(v[k], v[k]));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
        if ((i & 31) == 0) red[slot * 32 + (i >> 5)] = ss;
        __syncthreads();
        if (i < 32) {
            float s2 = i < nw ? red[slot * 32 + i] : 0.0f;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) s2 = __fadd_rn(s2, __shfl_xor_sync(0xffffffffu, s2, o));
            if (i == 0) red[slot * 32] = s2;
        }
        __syncthreads();
        const float ms = __fdiv_rn(red[slot * 32], (float)a.cols);
        const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, a.eps)));
        float gv[8];
        load8(a.gamma + i * 8, gv);
#pragma unroll
        for (int k = 0; k < 8; k++) v[k] = __fmul_rn(__fmul_rn(v[k], inv), gv[k]);
        const int tt = live ? t : 0;
        quant8_store(v, reinterpret_cast<int8_t*>(sm + L.off_xq) + (size_t)tt * L.pitch + i * 8,
                     reinterpret_cast<float*>(sm + L.off_xs) + (size_t)tt * L.xs_pitch + i / 4, (i & 3) == 0, live);
        __syncthreads();  // red is reused by the next pass
    }
}

// Quantize (PRO_QUANT) or SiLU * up + quantize (PRO_SILU), 8 values a thread.
template <int PRO>
__device__ __forceinline__ void prologue_elementwise(const GemvArgs& a, const GemvSmem& L, uint8_t* sm) {
    const int per_row = a.cols / 8;
    const int total = a.n * per_row;
    for (int base = 0; base < total; base += kGvThreads) {  // every lane takes every pass (group shuffles)
        const int item = base + threadIdx.x;
        const bool live = item < total;
        const int t = live ? item / per_row : 0, c = live ? (item % per_row) * 8 : 0;
        float v[8];
        if (PRO == PRO_QUANT) {
            load8(a.x + (size_t)t * a.cols + c, v);
        } else {
            float u[8];
            load8(a.x + (size_t)t * 2 * a.cols + c, v);
            load8(a.x + (size_t)t * 2 * a.cols + a.cols + c, u);
#pragma unroll
            for (int k = 0; k < 8; k++) {
                const float e = (float)exp(-(double)v[k]);
                v[k] = __fmul_rn(__fdiv_rn(v[k], __fadd_rn(1.0f, e)), u[k]);
            }
        }
        quant8_store(v, reinterpret_cast<int8_t*>(sm + L.off_xq) + (size_t)t * L.pitch + c,
                     reinterpret_cast<float*>(sm + L.off_xs) + (size_t)t * L.xs_pitch + c / kQK,
                     (threadIdx.x & 3) == 0, live);
    }
}

template <int PRO>
__global__ void __launch_bounds__(kGvThreads) q8_gemv_kernel(const __grid_constant__ GemvArgs a) {
    extern __shared__ __align__(128) uint8_t sm[];
    const GemvSmem L(a.cols);
    const int nb = a.cols / kQK;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, q = lane & 3;
    const int r0 = blockIdx.x * 16;
    const uint32_t bar = smem_u32(sm);
    if (tid == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar) : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar),
                     "r"((uint32_t)(16 * (a.cols + nb * 2)))
                     : "memory");
    }
    __syncwarp();
    if (tid < 16) {  // one lane per weight row: the 32 copies are issued side by side
        const int r = tid;
        const int rr = min(r0 + r, a.rows - 1);
        asm volatile(
            "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                smem_u32(sm + L.off_w + (size_t)r * L.pitch)),
            "l"(a.wq + (size_t)rr * a.cols), "r"((uint32_t)a.cols), "r"(bar)
            : "memory");
        asm volatile(
            "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                smem_u32(sm + L.off_ws + (size_t)r * L.ws_pitch)),
            "l"(a.ws + (size_t)rr * nb), "r"((uint32_t)(nb * 2)), "r"(bar)
            : "memory");
    }
    pdl_trigger_and_wait();  // activations come from the previous kernel
    int8_t* xq_s = reinterpret_cast<int8_t*>(sm + L.off_xq);
    float* xs_s = reinterpret_cast<float*>(sm + L.off_xs);
    if (PRO == PRO_Q8) {
        const int per_row = a.cols / 16;
        for (int idx = tid; idx < a.n * per_row; idx += kGvThreads) {
            const int t = idx / per_row, c = (idx % per_row) * 16;
            *reinterpret_cast<int4*>(xq_s + (size_t)t * L.pitch + c) =
                *reinterpret_cast<const int4*>(a.xq + (size_t)t * a.cols + c);
        }
        for (int idx = tid; idx < a.n * nb; idx += kGvThreads)
            xs_s[(idx / nb) * L.xs_pitch + idx % nb] = a.xs[idx];
    } else if (PRO == PRO_NORM) {
        prologue_norm(a, L, sm);
    } else {
        prologue_elementwise<PRO>(a, L, sm);
    }
    // tokens n..7 read as zeros
    for (int idx = tid; idx < (8 - a.n) * (a.cols / 16); idx += kGvThreads) {
        const int t = a.n + idx / (a.cols / 16), c = (idx % (a.cols / 16)) * 16;
        *reinterpret_cast<int4*>(xq_s + (size_t)t * L.pitch + c) = make_int4(0, 0, 0, 0);
    }
    for (int idx = tid; idx < (8 - a.n) * nb; idx += kGvThreads) xs_s[(a.n + idx / nb) * L.xs_pitch + idx % nb] = 0.f;
    __syncthreads();
    const bool ok = mbar_wait_bounded(bar, 0);
    if (__syncthreads_or(!ok)) {
        if (tid == 0) atomicExch(a.err, 1u);
        return;
    }
    uint8_t* w_s = sm + L.off_w;
    const __half* ws_s = reinterpret_cast<const __half*>(sm + L.off_ws);
    for (int b = warp; b < nb; b += kGvWarps) {
        const uint2 A0 = *reinterpret_cast<const uint2*>(w_s + (size_t)g * L.pitch + 32 * b + 8 * q);
        const uint2 A1 = *reinterpret_cast<const uint2*>(w_s + (size_t)(g + 8) * L.pitch + 32 * b + 8 * q);
        const uint2 B = *reinterpret_cast<const uint2*>(xq_s + (size_t)g * L.pitch + 32 * b + 8 * q);
        int d[4];
        mma_s8(d, A0.x, A1.x, A0.y, A1.y, B.x, B.y);
        const float wsa = __half2float(ws_s[g * (L.ws_pitch / 2) + b]);
        const float wsb = __half2float(ws_s[(g + 8) * (L.ws_pitch / 2) + b]);
        const float xsa = xs_s[(2 * q) * L.xs_pitch + b], xsc = xs_s[(2 * q + 1) * L.xs_pitch + b];
        float4 p;
        p.x = __fmul_rn(__fmul_rn(wsa, xsa), __int2float_rn(d[0]));
        p.y = __fmul_rn(__fmul_rn(wsa, xsc), __int2float_rn(d[1]));
        p.z = __fmul_rn(__fmul_rn(wsb, xsa), __int2float_rn(d[2]));
        p.w = __fmul_rn(__fmul_rn(wsb, xsc), __int2float_rn(d[3]));
        __syncwarp();  // every lane has read block b before it is overwritten
        *reinterpret_cast<float4*>(w_s + (size_t)(lane >> 1) * L.pitch + 32 * b + 16 * (lane & 1)) = p;
    }
    __syncthreads();
    if (warp != 0) return;
    float4 s = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    const uint8_t* slot = w_s + (size_t)(lane >> 1) * L.pitch + 16 * (lane & 1);
#pragma unroll 8
    for (int b = 0; b < nb; b++) {
        const float4 p = *reinterpret_cast<const float4*>(slot + 32 * b);
        s.x = __fadd_rn(s.x, p.x);
        s.y = __fadd_rn(s.y, p.y);
        s.z = __fadd_rn(s.z, p.z);
        s.w = __fadd_rn(s.w, p.w);
    }
    const float v[4] = {s.x, s.y, s.z, s.w};
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int r = r0 + g + 8 * (i >> 1), t = 2 * q + (i & 1);
        if (r < a.rows && t < a.n) {
            float* o = a.out + (size_t)t * a.out_stride + r;
            *o = a.accumulate ? __fadd_rn(*o, v[i]) : v[i];
        }
    }
}

bool gemv_ok(int cols, int n) {
    return n >= 1 && n <= 8 && cols % 256 == 0 && GemvSmem(cols).total <= 220 * 1024;
}

bool norm_fusable(int cols) {
    const int tpt = cols / 8;
    return tpt >= 32 && tpt <= kGvThreads && kGvThreads % tpt == 0;
}

template <int PRO>
cudaError_t launch_gemv_t(const GemvArgs& a, cudaStream_t st) {
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!attr_set[dev]) {
        const cudaError_t e =
            cudaFuncSetAttribute(q8_gemv_kernel<PRO>, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024);
        if (e != cudaSuccess) return e;
        attr_set[dev] = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((a.rows + 15) / 16);
    cfg.blockDim = dim3(kGvThreads);
    cfg.dynamicSmemBytes = GemvSmem(a.cols).total;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, q8_gemv_kernel<PRO>, a);
}

cudaError_t launch_gemv(int pro, const GemvArgs& a, cudaStream_t st) {
    switch (pro) {
        case PRO_Q8: return launch_gemv_t<PRO_Q8>(a, st);
        case PRO_QUANT: return launch_gemv_t<PRO_QUANT>(a, st);
        case PRO_SILU: return launch_gemv_t<PRO_SILU>(a, st);
        default: return launch_gemv_t<PRO_NORM>(a, st);
    }
}

}  // namespace

// ------------------------------------------------------------ the handle --

struct QMat {
    int8_t* qs = nullptr;
    __half* sc = nullptr;
    uint32_t rows = 0, cols = 0;
};

struct lt_llama {
    lt_llama_config cfg{};
    std::string err;
    uint32_t q_dim = 0, kv_dim = 0, qkv_rows = 0, half = 0, maxc = 0;
    QMat embed, output;
    float* out_norm = nullptr;
    std::vector<QMat> wqkv, wo, wgu, wdown;
    std::vector<float*> attn_norm, ffn_norm;
    std::vector<uint8_t> set;  // which (tensor, layer) were given
    std::vector<float> inv_freq;
    float *x = nullptr, *qkv = nullptr, *qb = nullptr, *kb = nullptr, *vb = nullptr, *att = nullptr, *gu = nullptr;
    float *xs = nullptr, *logits = nullptr;
    int8_t* xq = nullptr;
    int32_t* ids = nullptr;
    char* meta_dev = nullptr;
    char* meta_host = nullptr;
    int32_t* ids_host = nullptr;
    size_t meta_bytes = 0;
    cudaEvent_t meta_ev = nullptr;
    std::vector<int32_t> blocks, slots;
    uint64_t launches = 0;
    std::vector<void*> allocs;
    bool use_gemv = true;     // fused decode matmuls for up to 8 tokens
    // the persistent decode step (lt_llama_decode.cu) for up to 8 tokens, one per sequence
    bool persistent = true;
    int dec_grid = 0;                  // its CTAs (0: the shapes do not fit it)
    lldec::Layer* d_layers = nullptr;  // device table of every layer's weights
    uint32_t* d_sync = nullptr;        // its grid barrier and abort flag
    size_t sync_bytes = 0;
    uint32_t* d_err = nullptr;  // device flag: a bounded wait gave up (ids[0], copied with the picks)
    // matmul profiling: an event pair around each q8_matmul launch
    bool prof = false;
    std::vector<cudaEvent_t> prof_ev;
    size_t prof_used = 0;
    uint64_t prof_bytes = 0;
};

namespace {

lt_status fail(lt_llama* m, lt_status rc, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    m->err = buf;
    return rc;
}

#define LL_CUDA(m, call)                                                                             \
    do {                                                                                             \
        cudaError_t e_ = (call);                                                                     \
        if (e_ != cudaSuccess) return fail((m), LT_E_CUDA, "%s: %s", #call, cudaGetErrorString(e_)); \
    } while (0)

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        cudaGetDevice(&prev);
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        cudaGetDevice(&cur);
        if (prev >= 0 && cur != prev) cudaSetDevice(prev);
    }
};

// One projection of the forward: the activation prologue (RMSNorm +
// quantize, quantize, or SiLU * up + quantize of the f32 input `x`) and the
// Q8_0 matmul.  For up to 8 tokens both run in one q8_gemv_kernel launch;
// otherwise the standalone prologue kernel, then q8_matmul_kernel.  With
// profiling on, the matmul (or the fused launch) is bracketed by events.
// Algorithmic bytes: weights and their f16 scales, the activations as the
// matmul reads them, the f32 output (read too when accumulating).
lt_status project(lt_llama* m, int pro, const QMat& w, const float* x, const int32_t* rows_idx, const float* gamma,
                  int n, float* out, int out_stride, int accumulate, cudaStream_t st) {
    const bool fused = m->use_gemv && gemv_ok((int)w.cols, n) && (pro != PRO_NORM || norm_fusable((int)w.cols));
    if (fused && pro == PRO_SILU) {
        // SiLU * up + quantize once, as a dependent launch, rather than in every
        // matmul CTA (its double-precision exp is not cheap at ffn width)
        LL_CUDA(m, launch_silu_q8(x, n, (int)w.cols, nullptr, m->xq, m->xs, st, true));
        m->launches++;
        pro = PRO_Q8;
    }
    if (!fused) {  // standalone prologue into m->xq / m->xs
        cudaError_t e = cudaSuccess;
        if (pro == PRO_NORM)
            e = launch_rms_norm_q8(x, rows_idx, gamma, (int)w.cols, n, m->cfg.eps, nullptr, m->xq, m->xs, st);
        else if (pro == PRO_QUANT)
            e = launch_quantize(x, (size_t)n * w.cols, m->xq, m->xs, st);
        else if (pro == PRO_SILU)
            e = launch_silu_q8(x, n, (int)w.cols, nullptr, m->xq, m->xs, st);
        if (e != cudaSuccess) return fail(m, LT_E_CUDA, "prologue launch: %s", cudaGetErrorString(e));
        if (pro != PRO_Q8) m->launches++;
    }
    if (m->prof) {
        if (m->prof_used + 2 > m->prof_ev.size()) {
            for (int i = 0; i < 2; i++) {
                cudaEvent_t e;
                LL_CUDA(m, cudaEventCreate(&e));
                m->prof_ev.push_back(e);
            }
        }
        LL_CUDA(m, cudaEventRecord(m->prof_ev[m->prof_used], st));
    }
    if (fused) {
        GemvArgs a = {};
        a.wq = w.qs;
        a.ws = w.sc;
        a.rows = (int)w.rows;
        a.cols = (int)w.cols;
        a.out = out;
        a.out_stride = out_stride;
        a.accumulate = accumulate;
        a.n = n;
        a.x = x;
        a.rows_idx = rows_idx;
        a.gamma = gamma;
        a.eps = m->cfg.eps;
        a.xq = m->xq;
        a.xs = m->xs;
        a.err = m->d_err;
        LL_CUDA(m, launch_gemv(pro, a, st));
    } else {
        LL_CUDA(m, launch_matmul(w.qs, w.sc, (int)w.rows, (int)w.cols, m->xq, m->xs, n, out, out_stride, accumulate,
                                 st));
    }
    m->launches++;
    if (m->prof) {
        LL_CUDA(m, cudaEventRecord(m->prof_ev[m->prof_used + 1], st));
        m->prof_used += 2;
        const uint64_t rc = (uint64_t)w.rows * w.cols;
        m->prof_bytes += rc + rc / kQK * 2 + (uint64_t)n * w.cols + (uint64_t)n * w.cols / kQK * 4 +
                         (uint64_t)n * w.rows * 4 * (accumulate ? 2 : 1);
    }
    return LT_OK;
}

template <typename T>
lt_status dalloc(lt_llama* m, T** p, size_t count) {
    void* q = nullptr;
    if (cudaMalloc(&q, count * sizeof(T) + 16) != cudaSuccess) {
        cudaGetLastError();
        return fail(m, LT_E_CUDA, "cudaMalloc of %zu bytes failed", count * sizeof(T));
    }
    m->allocs.push_back(q);
    *p = static_cast<T*>(q);
    return LT_OK;
}

lt_status alloc_mat(lt_llama* m, QMat& w, uint32_t rows, uint32_t cols) {
    w.rows = rows;
    w.cols = cols;
    lt_status rc = dalloc(m, &w.qs, (size_t)rows * cols);
    if (rc == LT_OK) rc = dalloc(m, &w.sc, (size_t)rows * cols / kQK);
    return rc;
}

enum { kTensorKinds = 12 };

size_t set_index(const lt_llama* m, int which, uint32_t layer) {
    return which <= LT_T_OUTPUT_NORM ? (size_t)which : 3 + (size_t)layer * (kTensorKinds - 3) + (which - 3);
}

}  // namespace

extern "C" {

lt_status lt_llama_create(const lt_llama_config* cfg, lt_llama** out) {
    if (!cfg || !out) return LT_E_ARG;
    *out = nullptr;
    const lt_llama_config& c = *cfg;
    if (!c.n_layers || !c.dim || !c.n_heads || !c.n_kv_heads || !c.vocab || !c.max_batch || !c.ffn_dim)
        return LT_E_ARG;
    if (c.dim % kQK || c.ffn_dim % kQK || c.n_heads % c.n_kv_heads || (c.head_dim != 64 && c.head_dim != 128))
        return LT_E_UNSUPPORTED;
    if (c.dim / 8 > 1024 || (c.dim / 8) % 32) return LT_E_UNSUPPORTED;  // rms_norm: one CTA of dim/8 threads
    const uint32_t rope_dim = c.rope_dim ? c.rope_dim : c.head_dim;
    if (rope_dim > c.head_dim || rope_dim % 2) return LT_E_ARG;
    if ((size_t)c.ffn_dim / kQK * 32 * sizeof(float4) > 200 * 1024) return LT_E_UNSUPPORTED;
    auto* m = new lt_llama();
    m->cfg = c;
    m->cfg.rope_dim = rope_dim;
    m->q_dim = c.n_heads * c.head_dim;
    m->kv_dim = c.n_kv_heads * c.head_dim;
    m->qkv_rows = m->q_dim + 2 * m->kv_dim;
    m->half = rope_dim / 2;
    m->maxc = std::max(std::max(c.dim, m->q_dim), c.ffn_dim);
    if (m->q_dim % kQK || (size_t)m->q_dim / kQK * 32 * sizeof(float4) > 200 * 1024) {
        delete m;
        return LT_E_UNSUPPORTED;
    }
    for (uint32_t i = 0; i < m->half; i++)  // model.rs:263-265
        m->inv_freq.push_back(powf(c.rope_base, -2.0f * (float)i / (float)rope_dim));
    m->set.assign(3 + (size_t)c.n_layers * (kTensorKinds - 3), 0);
    DeviceGuard dg(c.device);
    const size_t B = c.max_batch;
    lt_status rc = alloc_mat(m, m->embed, c.vocab, c.dim);
    if (rc == LT_OK) rc = alloc_mat(m, m->output, c.vocab, c.dim);
    if (rc == LT_OK) rc = dalloc(m, &m->out_norm, c.dim);
    m->wqkv.resize(c.n_layers);
    m->wo.resize(c.n_layers);
    m->wgu.resize(c.n_layers);
    m->wdown.resize(c.n_layers);
    m->attn_norm.assign(c.n_layers, nullptr);
    m->ffn_norm.assign(c.n_layers, nullptr);
    for (uint32_t l = 0; l < c.n_layers && rc == LT_OK; l++) {
        rc = alloc_mat(m, m->wqkv[l], m->qkv_rows, c.dim);
        if (rc == LT_OK) rc = alloc_mat(m, m->wo[l], c.dim, m->q_dim);
        if (rc == LT_OK) rc = alloc_mat(m, m->wgu[l], 2 * c.ffn_dim, c.dim);
        if (rc == LT_OK) rc = alloc_mat(m, m->wdown[l], c.dim, c.ffn_dim);
        if (rc == LT_OK) rc = dalloc(m, &m->attn_norm[l], c.dim);
        if (rc == LT_OK) rc = dalloc(m, &m->ffn_norm[l], c.dim);
    }
    if (rc == LT_OK) rc = dalloc(m, &m->x, B * c.dim);
    if (rc == LT_OK) rc = dalloc(m, &m->qkv, B * m->qkv_rows);
    if (rc == LT_OK) rc = dalloc(m, &m->qb, B * m->q_dim);
    if (rc == LT_OK) rc = dalloc(m, &m->kb, B * m->kv_dim);
    if (rc == LT_OK) rc = dalloc(m, &m->vb, B * m->kv_dim);
    if (rc == LT_OK) rc = dalloc(m, &m->att, B * m->q_dim);
    if (rc == LT_OK) rc = dalloc(m, &m->gu, B * 2 * c.ffn_dim);
    if (rc == LT_OK) rc = dalloc(m, &m->xq, B * m->maxc);
    if (rc == LT_OK) rc = dalloc(m, &m->xs, B * m->maxc / kQK);
    if (rc == LT_OK) rc = dalloc(m, &m->logits, B * c.vocab);
    if (rc == LT_OK) rc = dalloc(m, &m->ids, B + 1);  // [0]: error flag, [1..]: picks
    if (rc == LT_OK) {
        m->d_err = reinterpret_cast<uint32_t*>(m->ids);
        if (cudaMemset(m->ids, 0, sizeof(int32_t)) != cudaSuccess) rc = fail(m, LT_E_CUDA, "cudaMemset failed");
    }
    // step metadata: tokens [B] | want [B] | seq [B] | pos [B] | sincos [B][half][2]
    m->meta_bytes = B * 4 * 4 + B * m->half * 2 * sizeof(float);
    if (rc == LT_OK) rc = dalloc(m, &m->meta_dev, m->meta_bytes);
    if (rc == LT_OK && (cudaMallocHost(&m->meta_host, m->meta_bytes) != cudaSuccess ||
                        cudaMallocHost(&m->ids_host, (B + 1) * sizeof(int32_t)) != cudaSuccess ||
                        cudaEventCreateWithFlags(&m->meta_ev, cudaEventDisableTiming) != cudaSuccess))
        rc = fail(m, LT_E_CUDA, "pinned staging allocation failed");
    if (rc != LT_OK) {
        lt_llama_destroy(m);
        return rc;
    }
    m->blocks.resize(B);
    m->slots.resize(B);
    // The persistent decode step: a device table of the layers' weights (the
    // matrices stay where alloc_mat put them), its synchronisation words and
    // its attention partials.
    const int group = (int)(c.n_heads / c.n_kv_heads);
    if (lldec::supported((int)c.dim, (int)m->q_dim, (int)c.ffn_dim, (int)c.head_dim, group, nullptr)) {
        std::vector<lldec::Layer> layers(c.n_layers);
        for (uint32_t l = 0; l < c.n_layers; l++) {
            const QMat* mats[4] = {&m->wqkv[l], &m->wo[l], &m->wgu[l], &m->wdown[l]};
            for (int k = 0; k < 4; k++) {
                layers[l].wq[k] = mats[k]->qs;
                layers[l].ws[k] = mats[k]->sc;
            }
            layers[l].attn_norm = m->attn_norm[l];
            layers[l].ffn_norm = m->ffn_norm[l];
        }
        m->sync_bytes = lldec::kSyncWords * sizeof(uint32_t);
        rc = dalloc(m, &m->d_layers, c.n_layers);
        if (rc == LT_OK) rc = dalloc(m, &m->d_sync, m->sync_bytes / sizeof(uint32_t));
        if (rc == LT_OK && (cudaMemcpy(m->d_layers, layers.data(), c.n_layers * sizeof(lldec::Layer),
                                       cudaMemcpyHostToDevice) != cudaSuccess ||
                            cudaMemset(m->d_sync, 0, m->sync_bytes) != cudaSuccess))
            rc = fail(m, LT_E_CUDA, "persistent decode set-up failed");
        if (rc != LT_OK) {
            lt_llama_destroy(m);
            return rc;
        }
        lldec::Params probe{};
        probe.dim = (int)c.dim;
        probe.q_dim = (int)m->q_dim;
        probe.ffn = (int)c.ffn_dim;
        probe.head_dim = (int)c.head_dim;
        probe.group = group;
        m->dec_grid = lldec::grid_size(probe);
        cudaGetLastError();  // a failed occupancy query leaves the step on the multi-launch path
    }
    *out = m;
    return LT_OK;
}

void lt_llama_destroy(lt_llama* m) {
    if (!m) return;
    DeviceGuard dg(m->cfg.device);
    if (m->meta_ev) {
        cudaEventSynchronize(m->meta_ev);
        cudaEventDestroy(m->meta_ev);
    }
    for (cudaEvent_t e : m->prof_ev) cudaEventDestroy(e);
    for (void* p : m->allocs) cudaFree(p);
    if (m->meta_host) cudaFreeHost(m->meta_host);
    if (m->ids_host) cudaFreeHost(m->ids_host);
    delete m;
}

const char* lt_llama_last_error(const lt_llama* m) { return m ? m->err.c_str() : "null handle"; }

uint64_t lt_llama_launch_count(const lt_llama* m) { return m ? m->launches : 0; }

lt_status lt_llama_profile(lt_llama* m, int enable) {
    if (!m) return LT_E_ARG;
    m->prof = enable != 0;
    m->prof_used = 0;
    m->prof_bytes = 0;
    return LT_OK;
}

lt_status lt_llama_profile_read(lt_llama* m, double* matmul_ms, uint64_t* matmul_launches, uint64_t* matmul_bytes) {
    if (!m || !matmul_ms || !matmul_launches || !matmul_bytes) return LT_E_ARG;
    DeviceGuard dg(m->cfg.device);
    double ms = 0.0;
    for (size_t i = 0; i + 1 < m->prof_used; i += 2) {
        float t = 0.0f;
        LL_CUDA(m, cudaEventSynchronize(m->prof_ev[i + 1]));
        LL_CUDA(m, cudaEventElapsedTime(&t, m->prof_ev[i], m->prof_ev[i + 1]));
        ms += t;
    }
    *matmul_ms = ms;
    *matmul_launches = m->prof_used / 2;
    *matmul_bytes = m->prof_bytes;
    m->prof_used = 0;
    m->prof_bytes = 0;
    return LT_OK;
}

lt_status lt_llama_set_tensor(lt_llama* m, lt_tensor which, uint32_t layer, const void* data, size_t bytes) {
    if (!m || !data) return LT_E_ARG;
    const lt_llama_config& c = m->cfg;
    if ((int)which < 0 || (int)which >= kTensorKinds) return fail(m, LT_E_ARG, "unknown tensor %d", (int)which);
    if (which > LT_T_OUTPUT_NORM && layer >= c.n_layers) return fail(m, LT_E_ARG, "layer %u out of range", layer);
    DeviceGuard dg(c.device);
    if (which == LT_T_OUTPUT_NORM || which == LT_T_ATTN_NORM || which == LT_T_FFN_NORM) {
        if (bytes != (size_t)c.dim * sizeof(float)) return fail(m, LT_E_ARG, "norm vector: %zu bytes", bytes);
        float* dst = which == LT_T_OUTPUT_NORM ? m->out_norm
                     : which == LT_T_ATTN_NORM ? m->attn_norm[layer] : m->ffn_norm[layer];
        LL_CUDA(m, cudaMemcpy(dst, data, bytes, cudaMemcpyHostToDevice));
        m->set[set_index(m, which, layer)] = 1;
        return LT_OK;
    }
    QMat* dst = nullptr;
    uint32_t row0 = 0, rows = 0, cols = c.dim;
    switch (which) {
        case LT_T_EMBED: dst = &m->embed; rows = c.vocab; break;
        case LT_T_OUTPUT: dst = &m->output; rows = c.vocab; break;
        case LT_T_Q: dst = &m->wqkv[layer]; rows = m->q_dim; break;
        case LT_T_K: dst = &m->wqkv[layer]; row0 = m->q_dim; rows = m->kv_dim; break;
        case LT_T_V: dst = &m->wqkv[layer]; row0 = m->q_dim + m->kv_dim; rows = m->kv_dim; break;
        case LT_T_O: dst = &m->wo[layer]; rows = c.dim; cols = m->q_dim; break;
        case LT_T_GATE: dst = &m->wgu[layer]; rows = c.ffn_dim; break;
        case LT_T_UP: dst = &m->wgu[layer]; row0 = c.ffn_dim; rows = c.ffn_dim; break;
        case LT_T_DOWN: dst = &m->wdown[layer]; rows = c.dim; cols = c.ffn_dim; break;
        default: return fail(m, LT_E_ARG, "unknown tensor %d", (int)which);
    }
    const size_t nb = (size_t)rows * cols / kQK;
    if (bytes != nb * 34) return fail(m, LT_E_ARG, "Q8_0 tensor %d: %zu bytes, expected %zu", (int)which, bytes, nb * 34);
    // quant.rs:265-273: split each 34-byte block into its f16 d and 32 int8
    std::vector<int8_t> qs((size_t)rows * cols);
    std::vector<uint16_t> sc(nb);
    const uint8_t* src = static_cast<const uint8_t*>(data);
    for (size_t b = 0; b < nb; b++) {
        std::memcpy(&sc[b], src + 34 * b, 2);
        std::memcpy(&qs[b * kQK], src + 34 * b + 2, kQK);
    }
    LL_CUDA(m, cudaMemcpy(dst->qs + (size_t)row0 * cols, qs.data(), qs.size(), cudaMemcpyHostToDevice));
    LL_CUDA(m, cudaMemcpy(dst->sc + (size_t)row0 * cols / kQK, sc.data(), nb * 2, cudaMemcpyHostToDevice));
    m->set[set_index(m, which, layer)] = 1;
    return LT_OK;
}

}  // extern "C"

namespace {

// Whether a forward call can run as one persistent decode launch: up to 8
// tokens, each of a different sequence (so each appends to its own last
// cell), on an f16 cache, with shapes the kernel takes.
bool decode_eligible(const lt_llama* m, const lt_kv* kv, const uint32_t* seqs, uint32_t n) {
    if (!m->persistent || m->dec_grid <= 0 || n == 0 || n > (uint32_t)lldec::kMaxTokens) return false;
    if (ltkv::handle_config(kv)->kv_format != LT_KV_F16) return false;
    for (uint32_t i = 0; i < n; i++)
        for (uint32_t j = i + 1; j < n; j++)
            if (seqs[i] == seqs[j]) return false;
    return true;
}

// Algorithmic bytes of one matmul as the profiling counts them: weights and
// their f16 scales, the int8 activations and scales read, the f32 outputs
// (read too when accumulating).
uint64_t matmul_bytes(const QMat& w, uint32_t n, bool accumulate) {
    const uint64_t rc = (uint64_t)w.rows * w.cols;
    return rc + rc / kQK * 2 + (uint64_t)n * w.cols + (uint64_t)n * w.cols / kQK * 4 +
           (uint64_t)n * w.rows * 4 * (accumulate ? 2 : 1);
}

// Model::forward (model.rs:366-518).  `greedy`: also pick the argmax of each
// wanted row into m->ids[1..] when the persistent step runs (*picked is then
// set); otherwise the caller launches the pick.
lt_status forward_impl(lt_llama* m, lt_kv* kv, const int32_t* tokens, const uint32_t* seqs, const uint32_t* pos,
                       uint32_t n, const uint32_t* want, uint32_t n_want, float* logits, void* stream, bool greedy,
                       bool* picked) {
    ltkv::NvtxRange nv("lt_llama_forward");
    if (picked) *picked = false;
    if (!m || !kv) return LT_E_ARG;
    const lt_llama_config& c = m->cfg;
    if (n == 0) return LT_OK;
    if (!tokens || !seqs || !pos) return fail(m, LT_E_ARG, "null token/seq/pos array");
    if (n > c.max_batch) return fail(m, LT_E_ARG, "batch of %u tokens exceeds max_batch %u", n, c.max_batch);
    if (n_want > n || (n_want && (!want || !logits))) return fail(m, LT_E_ARG, "bad logits request");
    for (uint32_t j = 0; j < n_want; j++)
        if (want[j] >= n) return fail(m, LT_E_ARG, "want[%u] = %u out of range", j, want[j]);
    const lt_kv_config* kc = ltkv::handle_config(kv);
    if (kc->n_layers != c.n_layers || kc->n_kv_heads != c.n_kv_heads || kc->head_dim != c.head_dim ||
        kc->n_heads != c.n_heads || kc->device != c.device)
        return fail(m, LT_E_ARG, "KV cache shape does not match the model");
    for (uint8_t s : m->set)
        if (!s) return fail(m, LT_E_ARG, "not every tensor was set");
    DeviceGuard dg(c.device);
    cudaStream_t st = static_cast<cudaStream_t>(stream);

    // Claim every cell first (model.rs:380-383).
    uint32_t done = 0;
    lt_status rc = lt_kv_append(kv, seqs, pos, n, m->blocks.data(), m->slots.data(), &done, stream);
    if (rc != LT_OK) return fail(m, rc, "%s", lt_kv_last_error(kv));
    for (uint32_t i = 0; i < n; i++)  // embed_row (model.rs:520-526), after the claim as in the reference
        if (tokens[i] < 0 || (uint32_t)tokens[i] >= c.vocab)
            return fail(m, LT_E_ARG, "token id %d out of range", tokens[i]);

    // Step metadata in one copy: tokens, want, seq, pos, RoPE sin/cos (host libm, as model.rs:297).
    LL_CUDA(m, cudaEventSynchronize(m->meta_ev));  // the previous copy has left the staging buffer
    const size_t B = c.max_batch;
    int32_t* h_tok = reinterpret_cast<int32_t*>(m->meta_host);
    int32_t* h_want = h_tok + B;
    int32_t* h_seq = h_want + B;
    int32_t* h_pos = h_seq + B;
    float* h_sc = reinterpret_cast<float*>(h_pos + B);
    std::memcpy(h_tok, tokens, n * sizeof(int32_t));
    for (uint32_t j = 0; j < n_want; j++) h_want[j] = (int32_t)want[j];
    for (uint32_t i = 0; i < n; i++) {
        h_seq[i] = (int32_t)seqs[i];
        h_pos[i] = (int32_t)pos[i];
    }
    for (uint32_t i = 0; i < n; i++)
        for (uint32_t k = 0; k < m->half; k++) {
            const float a = (float)pos[i] * m->inv_freq[k];
            h_sc[((size_t)i * m->half + k) * 2] = sinf(a);
            h_sc[((size_t)i * m->half + k) * 2 + 1] = cosf(a);
        }
    int32_t* d_tok = reinterpret_cast<int32_t*>(m->meta_dev);
    int32_t* d_want = d_tok + B;
    int32_t* d_seq = d_want + B;
    int32_t* d_pos = d_seq + B;
    float* d_sc = reinterpret_cast<float*>(d_pos + B);
    LL_CUDA(m, cudaMemcpyAsync(m->meta_dev, m->meta_host, B * 16 + (size_t)n * m->half * 2 * sizeof(float),
                               cudaMemcpyHostToDevice, st));
    LL_CUDA(m, cudaEventRecord(m->meta_ev, st));

    const int dim = (int)c.dim, ffn = (int)c.ffn_dim, qd = (int)m->q_dim, kvd = (int)m->kv_dim;
    const float scale = 1.0f / sqrtf((float)c.head_dim);  // model.rs:402

    if (decode_eligible(m, kv, seqs, n)) {
        // The whole step in one launch: the cache's queued plan (new table
        // entries, copy-on-write copies) goes first.
        if ((rc = lt_kv_flush(kv, stream)) != LT_OK) return fail(m, rc, "%s", lt_kv_last_error(kv));
        uint32_t max_blocks = 0;
        const int32_t* tables = lt_kv_device_tables(kv, &max_blocks);
        lldec::Params p{};
        p.layers = m->d_layers;
        p.n_layers = (int)c.n_layers;
        p.dim = dim;
        p.q_dim = qd;
        p.kv_dim = kvd;
        p.qkv_rows = (int)m->qkv_rows;
        p.ffn = ffn;
        p.vocab = (int)c.vocab;
        p.head_dim = (int)c.head_dim;
        p.group = (int)(c.n_heads / c.n_kv_heads);
        p.n_kv_heads = (int)c.n_kv_heads;
        p.half = (int)m->half;
        p.neox = c.rope_neox;
        p.eps = c.eps;
        p.scale_log2 = scale * 1.4426950408889634f;
        p.emb_q = m->embed.qs;
        p.emb_s = m->embed.sc;
        p.out_q = m->output.qs;
        p.out_s = m->output.sc;
        p.out_norm = m->out_norm;
        p.n = (int)n;
        p.n_want = (int)n_want;
        p.tokens = d_tok;
        p.want = d_want;
        p.seq = d_seq;
        p.pos = d_pos;
        p.sincos = d_sc;
        p.pool = static_cast<uint16_t*>(lt_kv_device_pool(kv));
        p.layer_elems = (size_t)lt_kv_n_blocks(kv) * c.n_kv_heads * 2 * LT_KV_BLOCK * c.head_dim;
        p.tables = tables;
        p.max_blocks = (int)max_blocks;
        p.x = m->x;
        p.qkv = m->qkv;
        p.att = m->att;
        p.act = m->gu;  // the multi-launch path's gate|up buffer holds act here
        p.logits = logits;
        p.ids = m->ids;
        p.argmax = greedy ? 1 : 0;
        p.sync = m->d_sync;
        // the barrier count and abort flag start at zero (a launch that gave up may have left them set)
        LL_CUDA(m, cudaMemsetAsync(m->d_sync, 0, lldec::kSyncWords * sizeof(uint32_t), st));
        if (m->prof) {
            if (m->prof_used + 2 > m->prof_ev.size()) {
                for (int i = 0; i < 2; i++) {
                    cudaEvent_t e;
                    LL_CUDA(m, cudaEventCreate(&e));
                    m->prof_ev.push_back(e);
                }
            }
            LL_CUDA(m, cudaEventRecord(m->prof_ev[m->prof_used], st));
        }
        LL_CUDA(m, lldec::launch(p, m->dec_grid, st));
        m->launches++;
        if (m->prof) {
            LL_CUDA(m, cudaEventRecord(m->prof_ev[m->prof_used + 1], st));
            m->prof_used += 2;
            for (uint32_t l = 0; l < c.n_layers; l++)
                m->prof_bytes += matmul_bytes(m->wqkv[l], n, false) + matmul_bytes(m->wo[l], n, true) +
                                 matmul_bytes(m->wgu[l], n, false) + matmul_bytes(m->wdown[l], n, true);
            if (n_want) m->prof_bytes += matmul_bytes(m->output, n_want, false);
        }
        if (picked) *picked = greedy && n_want > 0;
        return LT_OK;
    }

    embed_kernel<<<n, 256, 0, st>>>(m->embed.qs, m->embed.sc, dim, d_tok, m->x);
    LL_CUDA(m, cudaGetLastError());
    m->launches++;
    for (uint32_t l = 0; l < c.n_layers; l++) {
        rc = project(m, PRO_NORM, m->wqkv[l], m->x, nullptr, m->attn_norm[l], (int)n, m->qkv, (int)m->qkv_rows, 0, st);
        if (rc != LT_OK) return rc;
        LL_CUDA(m, launch_rope_split(m->qkv, (int)n, qd, kvd, (int)c.head_dim, (int)m->half, c.rope_neox, d_sc, m->qb,
                                     m->kb, m->vb, st));
        m->launches++;
        rc = lt_kv_write_attend(kv, l, m->blocks.data(), m->slots.data(), m->kb, m->vb, LT_F32, m->qb, LT_F32, seqs,
                                pos, n, m->att, LT_F32, scale, stream);
        if (rc != LT_OK) return fail(m, rc, "%s", lt_kv_last_error(kv));
        if ((rc = project(m, PRO_QUANT, m->wo[l], m->att, nullptr, nullptr, (int)n, m->x, dim, 1, st)) != LT_OK) return rc;
        rc = project(m, PRO_NORM, m->wgu[l], m->x, nullptr, m->ffn_norm[l], (int)n, m->gu, 2 * ffn, 0, st);
        if (rc != LT_OK) return rc;
        if ((rc = project(m, PRO_SILU, m->wdown[l], m->gu, nullptr, nullptr, (int)n, m->x, dim, 1, st)) != LT_OK)
            return rc;
    }
    if (n_want) {  // model.rs:502-517
        rc = project(m, PRO_NORM, m->output, m->x, d_want, m->out_norm, (int)n_want, logits, (int)c.vocab, 0, st);
        if (rc != LT_OK) return rc;
    }
    return LT_OK;
}

}  // namespace

extern "C" {

lt_status lt_llama_forward(lt_llama* m, lt_kv* kv, const int32_t* tokens, const uint32_t* seqs, const uint32_t* pos,
                           uint32_t n, const uint32_t* want, uint32_t n_want, float* logits, void* stream) {
    return forward_impl(m, kv, tokens, seqs, pos, n, want, n_want, logits, stream, false, nullptr);
}

lt_status lt_llama_step_greedy(lt_llama* m, lt_kv* kv, const int32_t* tokens, const uint32_t* seqs,
                               const uint32_t* pos, uint32_t n, const uint32_t* want, uint32_t n_want,
                               int32_t* next_host, void* stream) {
    if (!m) return LT_E_ARG;
    if (n_want && !next_host) return fail(m, LT_E_ARG, "null next_host");
    bool picked = false;
    lt_status rc = forward_impl(m, kv, tokens, seqs, pos, n, want, n_want, m->logits, stream, true, &picked);
    if (rc != LT_OK || n_want == 0) return rc;
    DeviceGuard dg(m->cfg.device);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (!picked) {
        LL_CUDA(m, launch_argmax(m->logits, (int)n_want, (int)m->cfg.vocab, m->ids + 1, st));
        m->launches++;
    }
    LL_CUDA(m, cudaMemcpyAsync(m->ids_host, m->ids, (n_want + 1) * sizeof(int32_t), cudaMemcpyDeviceToHost, st));
    LL_CUDA(m, cudaStreamSynchronize(st));
    if (m->ids_host[0] != 0) {
        cudaMemsetAsync(m->ids, 0, sizeof(int32_t), st);
        return fail(m, LT_E_TIMEOUT, "a bounded device wait of the step gave up");
    }
    std::memcpy(next_host, m->ids_host + 1, n_want * sizeof(int32_t));
    return LT_OK;
}

lt_status lt_llama_set_persistent(lt_llama* m, int enable) {
    if (!m) return LT_E_ARG;
    m->persistent = enable != 0;
    return LT_OK;
}

int lt_llama_persistent_available(const lt_llama* m) { return m && m->dec_grid > 0 ? 1 : 0; }

// ---- op-level entry points ----

lt_status lt_q8_quantize(const float* x, uint32_t n, uint32_t cols, int8_t* qs, float* scales, void* stream) {
    if (!x || !qs || !scales || cols % kQK) return LT_E_ARG;
    if (!aligned16(x) || !aligned16(qs)) return LT_E_ARG;
    return launch_quantize(x, (size_t)n * cols, qs, scales, static_cast<cudaStream_t>(stream)) == cudaSuccess
               ? LT_OK : LT_E_CUDA;
}

lt_status lt_q8_matmul(const int8_t* w_qs, const uint16_t* w_scales, uint32_t rows, uint32_t cols, const int8_t* x_qs,
                       const float* x_scales, uint32_t n, float* out, uint32_t out_stride, int accumulate,
                       void* stream) {
    if (!w_qs || !w_scales || !x_qs || !x_scales || !out || cols % kQK || out_stride < rows) return LT_E_ARG;
    if ((reinterpret_cast<uintptr_t>(w_qs) | reinterpret_cast<uintptr_t>(x_qs)) & 7) return LT_E_ARG;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (gemv_ok((int)cols, (int)n) && !((reinterpret_cast<uintptr_t>(w_qs) | reinterpret_cast<uintptr_t>(w_scales) |
                                         reinterpret_cast<uintptr_t>(x_qs)) & 15)) {
        GemvArgs a = {};
        a.wq = w_qs;
        a.ws = reinterpret_cast<const __half*>(w_scales);
        a.rows = (int)rows;
        a.cols = (int)cols;
        a.out = out;
        a.out_stride = (int)out_stride;
        a.accumulate = accumulate;
        a.n = (int)n;
        a.xq = x_qs;
        a.xs = x_scales;
        if (cudaGetSymbolAddress(reinterpret_cast<void**>(&a.err), g_op_err) != cudaSuccess) return LT_E_CUDA;
        return launch_gemv(PRO_Q8, a, st) == cudaSuccess ? LT_OK : LT_E_CUDA;
    }
    if ((size_t)cols / kQK * 32 * sizeof(float4) > 200 * 1024) return LT_E_UNSUPPORTED;
    return launch_matmul(w_qs, reinterpret_cast<const __half*>(w_scales), (int)rows, (int)cols, x_qs, x_scales, (int)n,
                         out, (int)out_stride, accumulate, st) == cudaSuccess
               ? LT_OK : LT_E_CUDA;
}

lt_status lt_rms_norm_q8(const float* x, const int32_t* rows_idx, const float* w, uint32_t dim, uint32_t n, float eps,
                         float* normed, int8_t* qs, float* scales, void* stream) {
    if (!x || !w || !qs || !scales || dim % 256 || dim / 8 > 1024) return LT_E_ARG;
    if (!aligned16(x) || !aligned16(w) || (normed && !aligned16(normed)) || !aligned16(qs)) return LT_E_ARG;
    return launch_rms_norm_q8(x, rows_idx, w, (int)dim, (int)n, eps, normed, qs, scales,
                              static_cast<cudaStream_t>(stream)) == cudaSuccess ? LT_OK : LT_E_CUDA;
}

lt_status lt_silu_q8(const float* gu, uint32_t n, uint32_t ffn, float* h, int8_t* qs, float* scales, void* stream) {
    if (!gu || !qs || !scales || ffn % kQK) return LT_E_ARG;
    if (!aligned16(gu) || (h && !aligned16(h)) || !aligned16(qs)) return LT_E_ARG;
    return launch_silu_q8(gu, (int)n, (int)ffn, h, qs, scales, static_cast<cudaStream_t>(stream)) == cudaSuccess
               ? LT_OK : LT_E_CUDA;
}

lt_status lt_argmax_f32(const float* x, uint32_t n, uint32_t cols, int32_t* idx, void* stream) {
    if (!x || !idx || !cols) return LT_E_ARG;
    return launch_argmax(x, (int)n, (int)cols, idx, static_cast<cudaStream_t>(stream)) == cudaSuccess ? LT_OK
                                                                                                      : LT_E_CUDA;
}

lt_status lt_q8_project(int prologue, const int8_t* w_qs, const uint16_t* w_scales, uint32_t rows, uint32_t cols,
                        const float* x, const int32_t* rows_idx, const float* gamma, float eps, uint32_t n,
                        float* out, uint32_t out_stride, int fused, int accumulate, void* stream) {
    if (prologue < LT_PRO_QUANT || prologue > LT_PRO_RMSNORM || !w_qs || !w_scales || !x || !out || cols % kQK ||
        out_stride < rows || n == 0)
        return LT_E_ARG;
    if (prologue == LT_PRO_RMSNORM && (!gamma || cols % 256 || cols / 8 > 1024)) return LT_E_ARG;
    if ((reinterpret_cast<uintptr_t>(w_qs) | reinterpret_cast<uintptr_t>(w_scales) | reinterpret_cast<uintptr_t>(x)) &
        15)
        return LT_E_ARG;
    const int pro = prologue == LT_PRO_QUANT ? PRO_QUANT : prologue == LT_PRO_SILU ? PRO_SILU : PRO_NORM;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (fused && gemv_ok((int)cols, (int)n) && (pro != PRO_NORM || norm_fusable((int)cols))) {
        GemvArgs a = {};
        a.wq = w_qs;
        a.ws = reinterpret_cast<const __half*>(w_scales);
        a.rows = (int)rows;
        a.cols = (int)cols;
        a.out = out;
        a.out_stride = (int)out_stride;
        a.accumulate = accumulate;
        a.n = (int)n;
        a.x = x;
        a.rows_idx = rows_idx;
        a.gamma = gamma;
        a.eps = eps;
        if (cudaGetSymbolAddress(reinterpret_cast<void**>(&a.err), g_op_err) != cudaSuccess) return LT_E_CUDA;
        return launch_gemv(pro, a, st) == cudaSuccess ? LT_OK : LT_E_CUDA;
    }
    // two launches: the standalone prologue kernel into scratch, then the matmul
    int8_t* xq = nullptr;
    float* xs = nullptr;
    if (cudaMallocAsync(reinterpret_cast<void**>(&xq), (size_t)n * cols + 16, st) != cudaSuccess) return LT_E_CUDA;
    if (cudaMallocAsync(reinterpret_cast<void**>(&xs), (size_t)n * cols / kQK * 4 + 16, st) != cudaSuccess) {
        cudaFreeAsync(xq, st);
        return LT_E_CUDA;
    }
    cudaError_t e;
    if (pro == PRO_NORM)
        e = launch_rms_norm_q8(x, rows_idx, gamma, (int)cols, (int)n, eps, nullptr, xq, xs, st);
    else if (pro == PRO_QUANT)
        e = launch_quantize(x, (size_t)n * cols, xq, xs, st);
    else
        e = launch_silu_q8(x, (int)n, (int)cols, nullptr, xq, xs, st);
    lt_status rc = e == cudaSuccess ? lt_q8_matmul(w_qs, w_scales, rows, cols, xq, xs, n, out, out_stride, accumulate,
                                                   stream)
                                    : LT_E_CUDA;
    cudaFreeAsync(xq, st);
    cudaFreeAsync(xs, st);
    return rc;
}

lt_status lt_q8_check(void* stream) {
    uint32_t* p = nullptr;
    if (cudaGetSymbolAddress(reinterpret_cast<void**>(&p), g_op_err) != cudaSuccess) return LT_E_CUDA;
    uint32_t v = 0;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (cudaMemcpyAsync(&v, p, 4, cudaMemcpyDeviceToHost, st) != cudaSuccess || cudaStreamSynchronize(st) != cudaSuccess)
        return LT_E_CUDA;
    if (v) {
        cudaMemsetAsync(p, 0, 4, st);
        return LT_E_TIMEOUT;
    }
    return LT_OK;
}

}  // extern "C"
