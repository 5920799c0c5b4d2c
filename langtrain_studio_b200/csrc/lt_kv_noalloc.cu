// lt_paged_attend_noalloc: paged decode attention for callers that cannot
// allocate device memory.
//
// Some hosts own every byte of device memory themselves: an engine that
// reserves HBM for its weights and KV pool up front and hands nothing else
// out, or a plugin host whose allocator is the only one allowed to call
// cudaMalloc.  Others cannot pay for cudaMalloc/cudaFree at all on their
// step path, because those calls may synchronise the whole device.  Such a
// caller has the block pool and block tables already (in the layout of
// lt_kv_device_pool / lt_kv_device_tables) and only needs the attention
// kernel.  That kernel needs scratch beyond its inputs and outputs (split-K
// partials and the work plan), so this entry point keeps it in one fixed,
// file-scope device array instead of allocating.
//
// The array is LT_NOALLOC_SCRATCH_BYTES (8 MiB).  Every GPU on which the
// library's module is loaded holds it until the process exits.  The first
// call on a device looks up the array's device address with that device
// current (cudaGetSymbolAddress) and caches it; make that first call before
// any stream capture.  Every call shares the array and it keeps the last
// call's contents, so each call clears its error word before its launch,
// keeps its range-done flags at a fixed place where they only ever hold
// epochs (a fresh one per call), and overwrites everything else it reads;
// calls that overlap on the GPU (different streams, no ordering) race on it
// -- issue them in order on one stream.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstring>
#include <mutex>

#include "lt_kv.h"
#include "lt_kv_internal.h"

namespace {

constexpr size_t kScratchBytes = LT_NOALLOC_SCRATCH_BYTES;
constexpr int kMaxDevices = 64;
// The range-done flags sit at a fixed place and only ever hold epochs: the
// descriptors and partials after them move with the call's size, and a flag
// placed over an earlier call's descriptor word (a small integer) could
// already equal the new epoch.
constexpr size_t kFlagsOffset = 256;
constexpr size_t kMaxFlagWarps = 16384;
constexpr size_t kFlagsBytes = kMaxFlagWarps * sizeof(uint32_t);

static __device__ __align__(256) unsigned char lt_noalloc_scratch[kScratchBytes];

std::atomic<void*> g_scratch[kMaxDevices];
// Host-side descriptors of one call (file scope, guarded by a mutex): the
// launch parameters carry up to kInlineTokens of them, the rest go through
// the scratch array.
std::mutex g_mu;
uint32_t g_epoch[kMaxDevices];  // per-device launch epoch for the range-done flags
ltkv::AttnParams g_params;
ltkv::TokenDesc g_toks[LT_NOALLOC_MAX_TOKENS];

size_t round256(size_t x) { return (x + 255) & ~size_t(255); }

// Device address of the scratch array on the current device (set up once).
cudaError_t scratch_ptr(void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    void* p = g_scratch[dev].load(std::memory_order_acquire);
    if (!p) {
        e = cudaGetSymbolAddress(&p, lt_noalloc_scratch);
        if (e != cudaSuccess) return e;
        g_scratch[dev].store(p, std::memory_order_release);
    }
    *out = p;
    return cudaSuccess;
}

}  // namespace

extern "C" lt_status lt_paged_attend_noalloc(const void* pool_layer, uint32_t n_kv_heads, uint32_t head_dim,
                                             uint32_t n_heads, const int32_t* tables, uint32_t max_blocks_per_seq,
                                             const uint32_t* seq, const uint32_t* pos, uint32_t n, const void* q,
                                             lt_dtype q_dtype, void* out, lt_dtype out_dtype, float scale,
                                             void* stream) {
    if (!pool_layer || !tables || !q || !out || (n && (!seq || !pos))) return LT_E_ARG;
    if (!ltkv::dtype_valid(q_dtype) || !ltkv::dtype_valid(out_dtype)) return LT_E_ARG;
    if (n_kv_heads == 0 || n_heads == 0 || n_heads % n_kv_heads) return LT_E_ARG;
    if (head_dim != 64 && head_dim != 128) return LT_E_UNSUPPORTED;
    const uint32_t group = n_heads / n_kv_heads;
    if (group > (uint32_t)ltkv::kMaxGroup) return LT_E_UNSUPPORTED;
    if ((reinterpret_cast<uintptr_t>(q) & 15) || (reinterpret_cast<uintptr_t>(out) & 15)) return LT_E_ARG;
    if (n == 0) return LT_OK;
    if (n > LT_NOALLOC_MAX_TOKENS) return LT_E_SCRATCH;
    long long tiles = 0;
    for (uint32_t i = 0; i < n; ++i) {
        if ((pos[i] + ltkv::kBlock) / ltkv::kBlock > max_blocks_per_seq) return LT_E_ARG;
        tiles += pos[i] / ltkv::kBlock + 1;
    }
    if (tiles > 0x7FFFFFFFll / n_kv_heads) return LT_E_SCRATCH;

    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return LT_E_CUDA;
    const int q_f32 = q_dtype == LT_F32;
    int n_warps = ltkv::attend_warps(dev, (int)group, (int)head_dim, q_f32, 0);
    if (n_warps <= 0) return LT_E_CUDA;
    n_warps = (int)std::min<long long>(n_warps, tiles * n_kv_heads);

    // Scratch layout: [error word][range-done flags, fixed][descriptors
    // beyond the inline ones][partial (m, l)][partial O], 256-byte aligned;
    // one flag and one partial slot per warp.  Fewer warps are used when the
    // partials would not fit.
    const size_t gd = (size_t)group * head_dim;
    const size_t o_toks = kFlagsOffset + kFlagsBytes;
    const size_t o_ml = o_toks + round256(n > (uint32_t)ltkv::kInlineTokens ? n * sizeof(ltkv::TokenDesc) : 0);
    const size_t per_warp = group * 2 * sizeof(float) + gd * sizeof(float);
    if (o_ml + 512 + per_warp > kScratchBytes) return LT_E_SCRATCH;
    n_warps = (int)std::min<size_t>({(size_t)n_warps, kMaxFlagWarps, (kScratchBytes - o_ml - 512) / per_warp});
    const size_t o_o = o_ml + round256((size_t)n_warps * group * 2 * sizeof(float));

    void* base = nullptr;
    if (scratch_ptr(&base) != cudaSuccess) return LT_E_CUDA;
    unsigned char* b = static_cast<unsigned char*>(base);
    cudaStream_t st = static_cast<cudaStream_t>(stream);

    std::lock_guard<std::mutex> lock(g_mu);
    ltkv::AttnParams& p = g_params;
    long long prefix = 0;
    ltkv::TokenDesc* td = n <= (uint32_t)ltkv::kInlineTokens ? p.inl : g_toks;
    for (uint32_t i = 0; i < n; ++i) {
        td[i].seq = (int32_t)seq[i];
        td[i].pos = (int32_t)pos[i];
        td[i].last_block = -1;  // unknown here: the kernel reads every block id from the tables
        td[i].prefix = (int32_t)prefix;
        td[i].skip = 0;
        prefix += pos[i] / ltkv::kBlock + 1;
    }
    // The error word must start at zero; the array keeps the previous call's bytes.
    if (cudaMemsetAsync(b, 0, sizeof(int32_t), st) != cudaSuccess) return LT_E_CUDA;
    if (td == g_toks) {
        // Pageable source: the call returns once the bytes are staged.
        if (cudaMemcpyAsync(b + o_toks, g_toks, n * sizeof(ltkv::TokenDesc), cudaMemcpyHostToDevice, st) !=
            cudaSuccess)
            return LT_E_CUDA;
        p.toks = reinterpret_cast<const ltkv::TokenDesc*>(b + o_toks);
    } else {
        p.toks = nullptr;
    }
    p.pool_layer = static_cast<const uint16_t*>(pool_layer);
    p.pool_layer_w = nullptr;  // no fused append on this entry point
    p.tables = const_cast<int32_t*>(tables);  // not written: no descriptor carries a last block id
    p.max_blocks = (int32_t)max_blocks_per_seq;
    p.n_tok = (int32_t)n;
    p.tiles_per_head = (int32_t)tiles;
    p.n_warps = n_warps;
    p.n_kv_heads = (int32_t)n_kv_heads;
    p.group = (int32_t)group;
    p.q = q;
    p.q_f32 = q_f32;
    p.out = out;
    p.out_f32 = out_dtype == LT_F32;
    p.scale_log2 = scale * 1.4426950408889634f;
    p.part_ml = reinterpret_cast<float*>(b + o_ml);
    p.part_o = reinterpret_cast<float*>(b + o_o);
    // The flags keep earlier calls' epochs: a fresh epoch per call on this
    // device (the array starts zeroed, and 0 is never used).  When the count
    // wraps, any earlier epoch may still be there, so the flags are cleared.
    p.flags = reinterpret_cast<uint32_t*>(b + kFlagsOffset);
    uint32_t epoch = g_epoch[dev] + 1;
    if (epoch == 0) {
        if (cudaMemsetAsync(b + kFlagsOffset, 0, kFlagsBytes, st) != cudaSuccess) return LT_E_CUDA;
        epoch = 1;
    }
    g_epoch[dev] = epoch;
    p.epoch = epoch;
    // A bounded wait that gives up sets the error word (first int32 of the
    // array) and leaves this call's outputs invalid; nothing synchronises
    // here to report it, and the next call clears it.
    p.err = reinterpret_cast<int32_t*>(b);
    p.k_new = nullptr;
    p.v_new = nullptr;
    p.kv_f32 = 0;
    p.pre_o = nullptr;
    p.pre_ml = nullptr;
    p.pre_splits = 0;
    p.pre_split_rows = 0;
    p.q8 = 0;  // f16 pool layout only
    if (ltkv::launch_attend(p, (int)head_dim, st) != cudaSuccess) return LT_E_CUDA;
    return LT_OK;
}
