// Device-side cell layout of the f16 block pool and the f32 -> f16
// conversion of its rows, shared by every kernel that writes or reads pool
// cells (the K/V write, attention, and the Llama decode step), so they agree
// bit for bit.
//
// Pool layout (per layer): f16 [block][kv_head][2 (K,V)][D/64][16 slots][64].
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

#include "lt_kv_internal.h"

namespace ltkv {

// f32 -> f16 with the bit semantics of half 2.7.1's f16::from_f32: IEEE
// round-to-nearest-even (the hardware cvt.rn), and NaN -> quiet NaN that
// keeps the top 10 payload bits (the hardware returns a canonical NaN).
__device__ __forceinline__ uint16_t f32_to_f16_ref(float x) {
    const uint32_t u = __float_as_uint(x);
    if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x007FFFFFu))
        return static_cast<uint16_t>(((u >> 16) & 0x8000u) | 0x7E00u | ((u & 0x007FFFFFu) >> 13));
    return __half_as_ushort(__float2half_rn(x));
}

// Element offset of 16-byte chunk c (8 f16) of slot s inside the K (or V)
// part of a (block, head) tile: the part is head_dim/64 sub-tiles of 16 rows
// x 128 bytes, chunk c in sub-tile c/8, at chunk position (c%8) ^ (s%8).
// Each sub-tile is the 128-byte-swizzled row-major layout of the tensor-core
// operand descriptors, and ldmatrix over it is bank-conflict free.
__device__ __forceinline__ int chunk_off(int c, int slot) {
    return (c >> 3) * (kBlock * 64) + slot * 64 + (((c & 7) ^ (slot & 7)) << 3);
}

}  // namespace ltkv
