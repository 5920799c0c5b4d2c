// Device helpers of the Q8_0 arithmetic shared by the Llama kernels: the
// s8 tensor-core dot, the engine's int8 activation quantiser and 8-wide
// f32 loads and stores.
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

namespace ltq8 {

constexpr int kQK = 32;  // Q8_0 block

__device__ __forceinline__ void mma_s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                       uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%10, %10, %10, %10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

// QActs::quantize of one 32-element block held as 8 values by each of 4
// consecutive lanes (quantize_block, quant.rs:785-795): amax folded from 0
// with f32::max (NaN-ignoring, as fmaxf), d = amax / 127, q = round(v * (1/d))
// half away from zero, saturated to int8 (Rust `as i8`: NaN -> 0).
// Every lane of the warp must call it (the group shuffles); only `live`
// lanes store.
__device__ __forceinline__ void quant8_store(const float (&v)[8], int8_t* q_dst, float* scale_dst, bool leader,
                                             bool live = true) {
    float a = 0.0f;
#pragma unroll
    for (int k = 0; k < 8; k++) a = fmaxf(a, fabsf(v[k]));
    a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 1));
    a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 2));
    const float d = __fdiv_rn(a, 127.0f);
    const float id = d > 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    uint32_t w[2] = {0u, 0u};
#pragma unroll
    for (int k = 0; k < 8; k++) {
        const float r = roundf(__fmul_rn(v[k], id));
        int qi = 0;
        if (!(r != r)) qi = (int)fminf(fmaxf(r, -128.0f), 127.0f);
        w[k >> 2] |= (uint32_t)(qi & 0xff) << (8 * (k & 3));
    }
    if (!live) return;
    *reinterpret_cast<uint2*>(q_dst) = make_uint2(w[0], w[1]);
    if (leader) *scale_dst = d;
}

__device__ __forceinline__ void load8(const float* p, float (&v)[8]) {
    const float4 a = *reinterpret_cast<const float4*>(p);
    const float4 b = *reinterpret_cast<const float4*>(p + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

__device__ __forceinline__ void store8(float* p, const float (&v)[8]) {
    *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
    *reinterpret_cast<float4*>(p + 4) = make_float4(v[4], v[5], v[6], v[7]);
}

}  // namespace ltq8
