// KV-head sharding over NCCL: communicator set-up and the all-gather of the
// per-rank attention outputs (the one collective of the path).  The reference
// engine is single-process and has no counterpart; its KvCache API is kept
// per rank and these calls only join the ranks' outputs.
//
// NCCL is resolved at run time from libnccl.so.2: a process that already
// loaded NCCL (a framework, or the engine itself) shares that copy.
#include <cuda_runtime.h>
#include <dlfcn.h>

#include <cstring>
#include <mutex>

#include "lt_kv.h"
#include "lt_kv_internal.h"

namespace {

struct UniqueId {
    char internal[128];
};

struct NcclApi {
    bool ok = false;
    int (*get_unique_id)(UniqueId*) = nullptr;
    int (*comm_init_rank)(void**, int, UniqueId, int) = nullptr;
    int (*comm_destroy)(void*) = nullptr;
    int (*all_gather)(const void*, void*, size_t, int, void*, cudaStream_t) = nullptr;
};

constexpr int kNcclUint8 = 1;  // ncclDataType_t: bytes

NcclApi& nccl() {
    static std::once_flag once;
    static NcclApi api;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW);
        if (!h) return;
        api.get_unique_id = reinterpret_cast<int (*)(UniqueId*)>(dlsym(h, "ncclGetUniqueId"));
        api.comm_init_rank = reinterpret_cast<int (*)(void**, int, UniqueId, int)>(dlsym(h, "ncclCommInitRank"));
        api.comm_destroy = reinterpret_cast<int (*)(void*)>(dlsym(h, "ncclCommDestroy"));
        api.all_gather =
            reinterpret_cast<int (*)(const void*, void*, size_t, int, void*, cudaStream_t)>(dlsym(h, "ncclAllGather"));
        api.ok = api.get_unique_id && api.comm_init_rank && api.comm_destroy && api.all_gather;
    });
    return api;
}

}  // namespace

extern "C" {

lt_status lt_kv_nccl_unique_id(void* id_out) {
    if (!id_out) return LT_E_ARG;
    NcclApi& api = nccl();
    if (!api.ok) return LT_E_NCCL;
    UniqueId id;
    if (api.get_unique_id(&id) != 0) return LT_E_NCCL;
    std::memcpy(id_out, id.internal, sizeof id.internal);
    return LT_OK;
}

lt_status lt_kv_nccl_init(void** comm_out, int nranks, const void* id_in, int rank, int device) {
    if (!comm_out || !id_in || nranks < 1 || rank < 0 || rank >= nranks) return LT_E_ARG;
    NcclApi& api = nccl();
    if (!api.ok) return LT_E_NCCL;
    int prev = -1;
    cudaGetDevice(&prev);
    if (cudaSetDevice(device) != cudaSuccess) return LT_E_CUDA;
    UniqueId id;
    std::memcpy(id.internal, id_in, sizeof id.internal);
    void* comm = nullptr;
    const int rc = api.comm_init_rank(&comm, nranks, id, rank);
    if (prev >= 0) cudaSetDevice(prev);
    if (rc != 0) return LT_E_NCCL;
    *comm_out = comm;
    return LT_OK;
}

void lt_kv_nccl_destroy(void* comm) {
    NcclApi& api = nccl();
    if (comm && api.ok) api.comm_destroy(comm);
}

lt_status lt_kv_gather_heads(lt_kv* kv, const void* local, void* gathered, void* out, uint32_t n, lt_dtype dtype,
                             void* comm, int nranks, void* stream) {
    ltkv::NvtxRange nv("lt_kv_gather_heads");
    if (!kv || !local || !gathered || !out || !comm || nranks < 1) return LT_E_ARG;
    if (!ltkv::dtype_valid(dtype)) return LT_E_ARG;
    NcclApi& api = nccl();
    if (!api.ok) return LT_E_NCCL;
    const size_t row = ltkv::local_out_row_bytes(kv, dtype);  // one token's local heads
    if (row == 0 || (row & 15)) return LT_E_ARG;
    if ((reinterpret_cast<uintptr_t>(local) | reinterpret_cast<uintptr_t>(gathered) |
         reinterpret_cast<uintptr_t>(out)) & 15)
        return LT_E_ARG;
    if (n == 0) return LT_OK;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int dev = ltkv::handle_device(kv);
    int prev = -1;
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
    lt_status rc = LT_OK;
    if (api.all_gather(local, gathered, row * n, kNcclUint8, comm, st) != 0) {
        rc = LT_E_NCCL;
    } else if (ltkv::launch_gather_permute(gathered, out, nranks, n, row, st) != cudaSuccess) {
        rc = LT_E_CUDA;
    } else {
        ltkv::count_launch(kv);
    }
    if (prev >= 0 && prev != dev) cudaSetDevice(prev);
    return rc;
}

}  // extern "C"
