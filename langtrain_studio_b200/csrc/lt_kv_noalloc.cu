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
// partials, per-(token, head) arrival counters, the work list), so this entry
// point keeps it in one fixed, file-scope device array instead of allocating.
//
// The array is LT_NOALLOC_SCRATCH_BYTES (8 MiB).  Every GPU on which the
// library's module is loaded holds it until the process exits.  The first
// call on a device looks up the array's device address with that device
// current (cudaGetSymbolAddress) and caches it; make that first call before
// any stream capture.  Every call shares the array and it keeps the last
// call's contents, so each call clears the counters it uses before its
// launch; calls that overlap on the GPU (different streams, no ordering)
// race on it -- issue them in order on one stream.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstring>

#include "lt_kv.h"
#include "lt_kv_internal.h"

namespace {

constexpr size_t kScratchBytes = LT_NOALLOC_SCRATCH_BYTES;
constexpr int kMaxDevices = 64;
constexpr uint32_t kMaxItems = 2048;  // host-side work-list buffer (64 KiB of stack)

static __device__ __align__(256) unsigned char lt_noalloc_scratch[kScratchBytes];

std::atomic<void*> g_scratch[kMaxDevices];

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
    if (n == 0) return LT_OK;
    if (n > LT_NOALLOC_MAX_TOKENS) return LT_E_SCRATCH;
    for (uint32_t i = 0; i < n; ++i)
        if ((pos[i] + ltkv::kBlock) / ltkv::kBlock > max_blocks_per_seq) return LT_E_ARG;

    // Scratch plan: [error word + counters][work items][partial (m, l)]
    // [partial O], each 256-byte aligned.  Start at 32 blocks per chunk and
    // double the chunk until the partials fit; reject what does not fit even
    // unsplit.
    const size_t gd = (size_t)group * head_dim;
    const size_t counters_bytes = round256((1 + (size_t)n * n_kv_heads) * sizeof(int32_t));
    uint32_t cb = 32;
    size_t parts = 0, items = 0;
    for (;;) {
        parts = 0;
        items = 0;
        for (uint32_t i = 0; i < n; ++i) {
            const uint32_t nb = (pos[i] + ltkv::kBlock) / ltkv::kBlock;
            const uint32_t nc = (nb + cb - 1) / cb;
            items += nc;
            if (nc > 1) parts += nc;
        }
        const size_t need = counters_bytes + round256(items * sizeof(ltkv::WorkItem)) +
                            round256(parts * n_kv_heads * group * 2 * sizeof(float)) +
                            round256(parts * n_kv_heads * gd * sizeof(float));
        if (items <= kMaxItems && need <= kScratchBytes) break;
        if (parts == 0) return LT_E_SCRATCH;  // one chunk per token and still too large
        cb *= 2;
    }

    ltkv::WorkItem host_items[kMaxItems];
    size_t k = 0;
    int32_t part_base = 0;
    for (uint32_t i = 0; i < n; ++i) {
        const uint32_t nb = (pos[i] + ltkv::kBlock) / ltkv::kBlock;
        const int32_t nc = (int32_t)((nb + cb - 1) / cb);
        for (int32_t c = 0; c < nc; ++c) {
            ltkv::WorkItem& w = host_items[k++];
            w.tok = (int32_t)i;
            w.seq = (int32_t)seq[i];
            w.pos = (int32_t)pos[i];
            w.chunk = c;
            w.nchunks = nc;
            w.part_base = nc > 1 ? part_base : 0;
            w.cb = (int32_t)cb;
            w.write_row = 0;
        }
        if (nc > 1) part_base += nc;
    }

    void* base = nullptr;
    if (scratch_ptr(&base) != cudaSuccess) return LT_E_CUDA;
    unsigned char* b = static_cast<unsigned char*>(base);
    int32_t* d_err = reinterpret_cast<int32_t*>(b);
    int32_t* d_counters = d_err + 1;
    ltkv::WorkItem* d_items = reinterpret_cast<ltkv::WorkItem*>(b + counters_bytes);
    float* d_part_ml = reinterpret_cast<float*>(b + counters_bytes + round256(items * sizeof(ltkv::WorkItem)));
    float* d_part_o = reinterpret_cast<float*>(reinterpret_cast<unsigned char*>(d_part_ml) +
                                               round256(parts * n_kv_heads * group * 2 * sizeof(float)));
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    // The error word and the counters must start at zero; the array keeps
    // the previous call's bytes.
    if (cudaMemsetAsync(d_err, 0, (1 + (size_t)n * n_kv_heads) * sizeof(int32_t), st) != cudaSuccess)
        return LT_E_CUDA;
    // Pageable source: the call returns once the bytes are staged, so the
    // stack buffer may go out of scope.
    if (cudaMemcpyAsync(d_items, host_items, items * sizeof(ltkv::WorkItem), cudaMemcpyHostToDevice, st) !=
        cudaSuccess)
        return LT_E_CUDA;

    ltkv::AttnParams p{};
    p.pool_layer = static_cast<const uint16_t*>(pool_layer);
    p.pool_layer_w = nullptr;  // no fused append on this entry point
    p.tables = tables;
    p.max_blocks = (int32_t)max_blocks_per_seq;
    p.items = d_items;
    p.n_items = (int32_t)items;
    p.n_kv_heads = (int32_t)n_kv_heads;
    p.group = (int32_t)group;
    p.q = q;
    p.q_f32 = q_dtype == LT_F32;
    p.out = out;
    p.out_f32 = out_dtype == LT_F32;
    p.scale_log2 = scale * 1.4426950408889634f;
    p.part_o = d_part_o;
    p.part_ml = d_part_ml;
    p.counters = d_counters;
    // A bounded wait that gives up sets the error word (first int32 of the
    // array) and leaves this call's outputs invalid; nothing synchronises
    // here to report it, and the next call clears it.
    p.err = d_err;
    p.k_new = nullptr;
    p.v_new = nullptr;
    p.kv_f32 = 0;
    if (ltkv::launch_attend(p, (int)head_dim, st) != cudaSuccess) return LT_E_CUDA;
    return LT_OK;
}
