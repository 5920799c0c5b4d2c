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
// partials and range-done flags), so this entry point keeps it in one fixed,
// file-scope device array instead of allocating.
//
// The array is LT_NOALLOC_SCRATCH_BYTES (8 MiB).  Every GPU on which the
// library's module is loaded holds it until the process exits.  The first
// call on a device looks up the array's device address with that device
// current (cudaGetSymbolAddress) and caches it; make that first call before
// any stream capture.  Every call shares the array and it keeps the last
// call's contents: the range-done flags sit at a fixed place where they only
// ever hold epochs (a fresh one per launch), each launch overwrites the
// partials it reads, and the error word collects the failures of every call
// until lt_paged_attend_noalloc_check reads and clears it.  Calls that
// overlap on the GPU (different streams, no ordering) race on the array --
// issue them in order on one stream.
//
// The tables and block ids come from the caller, not from this library's
// bookkeeping, so everything the kernel would index with is checked: on the
// host, before any work, every sequence id against the table rows and every
// position against the row length; on the device, every block id read from
// the tables against the caller's pool size (an id past it reads block 0
// instead and raises LT_E_BOUNDS in the error word).
//
// The per-token work descriptors travel inside the kernel parameters, up to
// 512 tokens a launch; a call with more tokens is issued as consecutive
// launches on the caller's stream, so no host buffer is ever copied.
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
// Scratch layout: [error word][range-done flags][partial (m, l)][partial O],
// 256-byte aligned.  The flags sit at a fixed place and only ever hold
// epochs, so a later launch never finds a stale word equal to its epoch.
constexpr size_t kFlagsOffset = 256;
constexpr size_t kMaxFlagWarps = 16384;
constexpr size_t kFlagsBytes = kMaxFlagWarps * sizeof(uint32_t);
constexpr size_t kPartialsOffset = kFlagsOffset + kFlagsBytes;

static __device__ __align__(256) unsigned char lt_noalloc_scratch[kScratchBytes];

std::atomic<void*> g_scratch[kMaxDevices];
std::mutex g_mu;                  // guards g_epoch and g_params
uint32_t g_epoch[kMaxDevices];    // per-device launch epoch for the range-done flags
ltkv::AttnParams g_params;        // one launch's parameters (large: kept off the stack)

size_t round256(size_t x) { return (x + 255) & ~size_t(255); }

// Device address of the scratch array on the current device (set up once).
cudaError_t scratch_ptr(int* dev_out, void** out) {
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
    *dev_out = dev;
    *out = p;
    return cudaSuccess;
}

bool misaligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) != 0; }

}  // namespace

extern "C" lt_status lt_paged_attend_noalloc(const void* pool_layer, uint32_t kv_format, uint32_t n_blocks,
                                             uint32_t n_kv_heads, uint32_t head_dim, uint32_t n_heads,
                                             const int32_t* tables, uint32_t n_table_rows,
                                             uint32_t max_blocks_per_seq, const uint32_t* seq, const uint32_t* pos,
                                             uint32_t n, const void* q, lt_dtype q_dtype, void* out,
                                             lt_dtype out_dtype, float scale, void* stream) {
    // ---- every argument, before any device work ----
    if (!pool_layer || !tables || !q || !out || (n && (!seq || !pos))) return LT_E_ARG;
    if (!ltkv::dtype_valid(q_dtype) || !ltkv::dtype_valid(out_dtype)) return LT_E_ARG;
    if (kv_format == LT_KV_Q8_0) return LT_E_UNSUPPORTED;  // the kernel below reads f16 tiles only
    if (kv_format != LT_KV_F16) return LT_E_ARG;
    if (n_blocks == 0 || n_blocks > 0x7FFFFFFFu) return LT_E_ARG;
    if (n_table_rows == 0 || max_blocks_per_seq == 0 || max_blocks_per_seq > 0x7FFFFFFFu) return LT_E_ARG;
    if (n_kv_heads == 0 || n_heads == 0 || n_heads % n_kv_heads) return LT_E_ARG;
    if (head_dim != 64 && head_dim != 128) return LT_E_UNSUPPORTED;
    const uint32_t group = n_heads / n_kv_heads;
    if (group > (uint32_t)ltkv::kMaxGroup) return LT_E_UNSUPPORTED;
    // Bulk copies read pool tiles and q rows from 16-byte boundaries.
    if (misaligned(pool_layer, 16) || misaligned(q, 16) || misaligned(out, 16) || misaligned(tables, 4))
        return LT_E_ARG;
    if (n == 0) return LT_OK;
    if (n > LT_NOALLOC_MAX_TOKENS) return LT_E_SCRATCH;
    for (uint32_t i = 0; i < n; ++i) {
        if (seq[i] >= n_table_rows) return LT_E_ARG;
        // pos is carried as int32 and attends over table entries [0, pos/16].
        if (pos[i] > 0x7FFFFFFFu - ltkv::kBlock || pos[i] / ltkv::kBlock >= max_blocks_per_seq) return LT_E_ARG;
    }
    const uint32_t kInline = (uint32_t)ltkv::kInlineTokens;
    for (uint32_t c0 = 0; c0 < n; c0 += kInline) {
        long long tiles = 0;
        for (uint32_t i = c0; i < std::min(n, c0 + kInline); ++i) tiles += pos[i] / ltkv::kBlock + 1;
        if (tiles > 0x7FFFFFFFll / n_kv_heads) return LT_E_SCRATCH;
    }
    const size_t gd = (size_t)group * head_dim;
    const size_t per_warp = group * 2 * sizeof(float) + gd * sizeof(float);

    // ---- set-up (first call on this device: look up the array's address) ----
    int dev = 0;
    void* base = nullptr;
    if (scratch_ptr(&dev, &base) != cudaSuccess) return LT_E_CUDA;
    unsigned char* b = static_cast<unsigned char*>(base);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int q_f32 = q_dtype == LT_F32;
    const int max_warps = ltkv::attend_warps(dev, (int)group, (int)head_dim, q_f32, 0);
    if (max_warps <= 0) return LT_E_CUDA;
    const size_t warp_cap =
        std::min<size_t>({(size_t)max_warps, kMaxFlagWarps, (kScratchBytes - kPartialsOffset - 256) / per_warp});
    const size_t q_row = (size_t)n_heads * head_dim * (q_f32 ? 4 : 2);
    const size_t out_row = (size_t)n_heads * head_dim * (out_dtype == LT_F32 ? 4 : 2);

    std::lock_guard<std::mutex> lock(g_mu);
    ltkv::AttnParams& p = g_params;
    for (uint32_t c0 = 0; c0 < n; c0 += kInline) {
        const uint32_t cn = std::min(n - c0, kInline);
        long long prefix = 0;
        for (uint32_t i = 0; i < cn; ++i) {
            ltkv::TokenDesc& td = p.inl[i];
            td.seq = (int32_t)seq[c0 + i];
            td.pos = (int32_t)pos[c0 + i];
            td.last_block = -1;  // every block id is read (and checked) from the caller's tables
            td.prefix = (int32_t)prefix;
            td.skip = 0;
            prefix += pos[c0 + i] / ltkv::kBlock + 1;
        }
        const int n_warps = (int)std::min<long long>((long long)warp_cap, prefix * n_kv_heads);
        p.toks = nullptr;  // descriptors travel in the kernel parameters
        p.pool_layer = static_cast<const uint16_t*>(pool_layer);
        p.pool_layer_w = nullptr;                 // no fused append on this entry point
        p.tables = const_cast<int32_t*>(tables);  // not written: no descriptor carries a last block id
        p.max_blocks = (int32_t)max_blocks_per_seq;
        p.n_blocks = (int32_t)n_blocks;
        p.check_ids = 1;
        p.n_tok = (int32_t)cn;
        p.tiles_per_head = (int32_t)prefix;
        p.n_warps = n_warps;
        p.n_kv_heads = (int32_t)n_kv_heads;
        p.group = (int32_t)group;
        p.q = static_cast<const uint8_t*>(q) + (size_t)c0 * q_row;
        p.q_f32 = q_f32;
        p.out = static_cast<uint8_t*>(out) + (size_t)c0 * out_row;
        p.out_f32 = out_dtype == LT_F32;
        p.scale_log2 = scale * 1.4426950408889634f;
        p.part_ml = reinterpret_cast<float*>(b + kPartialsOffset);
        p.part_o = reinterpret_cast<float*>(b + kPartialsOffset + round256((size_t)n_warps * group * 2 * sizeof(float)));
        p.part2_o = nullptr;  // one-level merge
        p.part2_ml = nullptr;
        p.flags2 = nullptr;
        // The flags keep earlier launches' epochs: a fresh epoch per launch on
        // this device (the array starts zeroed, and 0 is never used).  When the
        // count wraps, any earlier epoch may still be there, so the flags are
        // cleared.
        p.flags = reinterpret_cast<uint32_t*>(b + kFlagsOffset);
        uint32_t epoch = g_epoch[dev] + 1;
        if (epoch == 0) {
            if (cudaMemsetAsync(b + kFlagsOffset, 0, kFlagsBytes, st) != cudaSuccess) return LT_E_CUDA;
            epoch = 1;
        }
        g_epoch[dev] = epoch;
        p.epoch = epoch;
        // Failures (a bounded wait that gave up, a block id past the pool) are
        // OR-ed into the array's first word and stay there until
        // lt_paged_attend_noalloc_check reads and clears it.
        p.err = reinterpret_cast<int32_t*>(b);
        p.k_new = nullptr;
        p.v_new = nullptr;
        p.kv_f32 = 0;
        p.pre_o = nullptr;
        p.pre_ml = nullptr;
        p.pre_splits = 0;
        p.pre_split_rows = 0;
        p.q8 = 0;
        p.n_peers = 0;
        if (ltkv::launch_attend(p, (int)head_dim, st) != cudaSuccess) return LT_E_CUDA;
    }
    return LT_OK;
}

extern "C" lt_status lt_paged_attend_noalloc_check(void* stream) {
    int dev = 0;
    void* base = nullptr;
    if (scratch_ptr(&dev, &base) != cudaSuccess) return LT_E_CUDA;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    int32_t word = 0;
    if (cudaMemcpyAsync(&word, base, sizeof word, cudaMemcpyDeviceToHost, st) != cudaSuccess) return LT_E_CUDA;
    if (cudaStreamSynchronize(st) != cudaSuccess) return LT_E_CUDA;
    if (word == 0) return LT_OK;
    if (cudaMemsetAsync(base, 0, sizeof word, st) != cudaSuccess) return LT_E_CUDA;
    if (cudaStreamSynchronize(st) != cudaSuccess) return LT_E_CUDA;
    return (word & ltkv::kErrTimeout) ? LT_E_TIMEOUT : LT_E_BOUNDS;
}
