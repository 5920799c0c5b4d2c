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
// call's contents, so each call clears its error word before its launch and
// overwrites everything else it reads; calls that overlap on the GPU
// (different streams, no ordering) race on it -- issue them in order on one
// stream.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstring>
#include <mutex>

#include "lt_kv.h"
#include "lt_kv_internal.h"
#include "lt_kv_plan.h"

namespace {

constexpr size_t kScratchBytes = LT_NOALLOC_SCRATCH_BYTES;
constexpr int kMaxDevices = 64;
// Host-side plan buffers (file scope, guarded by a mutex): the stream-K
// pieces, per-warp offsets and split list of one call.
constexpr int kMaxPieces = 8192;
constexpr int kMaxWarps = 4096;

static __device__ __align__(256) unsigned char lt_noalloc_scratch[kScratchBytes];

std::atomic<void*> g_scratch[kMaxDevices];
std::mutex g_plan_mu;
ltkv::Piece g_pieces[kMaxPieces];
int32_t g_warp_off[kMaxWarps + 1];
int4 g_combine[kMaxPieces];

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
    if (n_kv_heads == 0 || n_heads == 0 || n_heads % n_kv_heads) return LT_E_ARG;
    if (head_dim != 64 && head_dim != 128) return LT_E_UNSUPPORTED;
    const uint32_t group = n_heads / n_kv_heads;
    if (group > (uint32_t)ltkv::kMaxGroup) return LT_E_UNSUPPORTED;
    if ((reinterpret_cast<uintptr_t>(q) & 15) || (reinterpret_cast<uintptr_t>(out) & 15)) return LT_E_ARG;
    if (n == 0) return LT_OK;
    if (n > LT_NOALLOC_MAX_TOKENS) return LT_E_SCRATCH;
    for (uint32_t i = 0; i < n; ++i)
        if ((pos[i] + ltkv::kBlock) / ltkv::kBlock > max_blocks_per_seq) return LT_E_ARG;

    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return LT_E_CUDA;
    const int q_f32 = q_dtype == LT_F32;
    const int max_warps = std::min(ltkv::attend_warps(dev, (int)group, (int)head_dim, q_f32), kMaxWarps);
    if (max_warps <= 0) return LT_E_CUDA;
    const size_t pairs = (size_t)n * n_kv_heads;
    if (pairs + (size_t)max_warps > (size_t)kMaxPieces) return LT_E_SCRATCH;

    std::lock_guard<std::mutex> lock(g_plan_mu);
    const ltkv::StreamPlan pl =
        ltkv::plan_stream_k(seq, pos, n, (int)n_kv_heads, max_warps, nullptr, g_pieces, g_warp_off, g_combine);

    // Scratch layout: [error word][pieces][warp offsets][split list]
    // [partial (m, l)][partial O], each 256-byte aligned.
    const size_t gd = (size_t)group * head_dim;
    const size_t o_pieces = 256;
    const size_t o_warp = o_pieces + round256((size_t)pl.n_pieces * sizeof(ltkv::Piece));
    const size_t o_comb = o_warp + round256(((size_t)pl.n_warps + 1) * sizeof(int32_t));
    const size_t o_ml = o_comb + round256((size_t)pl.n_combine * sizeof(int4));
    const size_t o_o = o_ml + round256((size_t)pl.n_slots * group * 2 * sizeof(float));
    const size_t need = o_o + round256((size_t)pl.n_slots * gd * sizeof(float));
    if (need > kScratchBytes) return LT_E_SCRATCH;

    void* base = nullptr;
    if (scratch_ptr(&base) != cudaSuccess) return LT_E_CUDA;
    unsigned char* b = static_cast<unsigned char*>(base);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    // The error word must start at zero; the array keeps the previous call's bytes.
    if (cudaMemsetAsync(b, 0, sizeof(int32_t), st) != cudaSuccess) return LT_E_CUDA;
    // Pageable sources: each call returns once its bytes are staged.
    if (cudaMemcpyAsync(b + o_pieces, g_pieces, (size_t)pl.n_pieces * sizeof(ltkv::Piece), cudaMemcpyHostToDevice,
                        st) != cudaSuccess ||
        cudaMemcpyAsync(b + o_warp, g_warp_off, ((size_t)pl.n_warps + 1) * sizeof(int32_t), cudaMemcpyHostToDevice,
                        st) != cudaSuccess ||
        (pl.n_combine && cudaMemcpyAsync(b + o_comb, g_combine, (size_t)pl.n_combine * sizeof(int4),
                                         cudaMemcpyHostToDevice, st) != cudaSuccess))
        return LT_E_CUDA;

    ltkv::AttnParams p{};
    p.pool_layer = static_cast<const uint16_t*>(pool_layer);
    p.pool_layer_w = nullptr;  // no fused append on this entry point
    p.tables = tables;
    p.max_blocks = (int32_t)max_blocks_per_seq;
    p.pieces = reinterpret_cast<const ltkv::Piece*>(b + o_pieces);
    p.warp_off = reinterpret_cast<const int32_t*>(b + o_warp);
    p.n_warps = pl.n_warps;
    p.combine = reinterpret_cast<const int4*>(b + o_comb);
    p.n_combine = pl.n_combine;
    p.n_kv_heads = (int32_t)n_kv_heads;
    p.group = (int32_t)group;
    p.q = q;
    p.q_f32 = q_f32;
    p.out = out;
    p.out_f32 = out_dtype == LT_F32;
    p.scale_log2 = scale * 1.4426950408889634f;
    p.part_ml = reinterpret_cast<float*>(b + o_ml);
    p.part_o = reinterpret_cast<float*>(b + o_o);
    // A bounded wait that gives up sets the error word (first int32 of the
    // array) and leaves this call's outputs invalid; nothing synchronises
    // here to report it, and the next call clears it.
    p.err = reinterpret_cast<int32_t*>(b);
    p.k_new = nullptr;
    p.v_new = nullptr;
    p.kv_f32 = 0;
    if (ltkv::launch_attend(p, (int)head_dim, st) != cudaSuccess) return LT_E_CUDA;
    return LT_OK;
}
