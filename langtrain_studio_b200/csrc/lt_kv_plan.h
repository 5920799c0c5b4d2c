// Host-side stream-K partition of one attention call (shared by lt_kv.cpp
// and lt_kv_noalloc.cu).  Writes only into caller-provided arrays.
#pragma once
#include <stdint.h>

#include <algorithm>

#include "lt_kv_internal.h"

namespace ltkv {

struct StreamPlan {
    int n_pieces = 0;
    int n_combine = 0;
    int n_slots = 0;  // partial slots used
    int n_warps = 0;  // warps of the launch (each owns >= 1 tile)
};

// Lay the (token, KV head) sequences of n tokens end to end -- tokens in
// order, heads within a token, blocks within a head -- and cut the tile
// sequence into n_warps ranges of equal length (+-1).  Token i attends over
// blocks [0, (pos[i] + 16) / 16).
//   pieces:   capacity n*n_kv_heads + max_warps (every piece ends a
//             (token, head) or a warp range)
//   warp_off: capacity max_warps + 1
//   combine:  capacity n*n_kv_heads
// last_block (optional, per token): physical id of the token's last block;
// the piece holding that block then performs the fused K/V append.
inline StreamPlan plan_stream_k(const uint32_t* seq, const uint32_t* pos, uint32_t n, int n_kv_heads,
                                int max_warps, const int32_t* last_block, Piece* pieces, int32_t* warp_off,
                                int4* combine) {
    StreamPlan pl;
    long long total = 0;
    for (uint32_t i = 0; i < n; ++i) total += (long long)((pos[i] + kBlock) / kBlock) * n_kv_heads;
    if (total == 0 || max_warps <= 0) return pl;
    const long long nw = std::min<long long>(max_warps, total);
    auto start = [&](long long w) { return total * w / nw; };
    long long t = 0, w = 0, next = start(1);
    int np = 0, nc = 0, slots = 0;
    warp_off[0] = 0;
    for (uint32_t i = 0; i < n; ++i) {
        const int nb = (int)((pos[i] + kBlock) / kBlock);
        for (int h = 0; h < n_kv_heads; ++h) {
            const int first = np;
            int b = 0;
            while (b < nb) {
                while (t >= next) {  // move on to the next warp's range
                    ++w;
                    warp_off[w] = np;
                    next = start(w + 1);
                }
                const int take = (int)std::min<long long>(nb - b, next - t);
                Piece& pc = pieces[np++];
                pc.tok = (int32_t)i;
                pc.h = h;
                pc.seq = (int32_t)seq[i];
                pc.pos = (int32_t)pos[i];
                pc.b0 = b;
                pc.b1 = b + take;
                pc.slot = -1;
                pc.last_block = -1;
                b += take;
                t += take;
            }
            const int k = np - first;
            if (k > 1) {
                for (int j = 0; j < k; ++j) pieces[first + j].slot = slots + j;
                combine[nc++] = make_int4((int)i, h, k, slots);
                slots += k;
            }
            if (last_block) pieces[np - 1].last_block = last_block[i];
        }
    }
    for (long long ww = w + 1; ww <= nw; ++ww) warp_off[ww] = np;
    pl.n_pieces = np;
    pl.n_combine = nc;
    pl.n_slots = slots;
    pl.n_warps = (int)nw;
    return pl;
}

}  // namespace ltkv
