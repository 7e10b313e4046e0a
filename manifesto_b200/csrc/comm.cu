// comm.cu -- the NCCL communicator used by the checkpoint quantisation for
// its one exchange step: an in-place max all-reduce of the per-tensor amax
// vector (a few hundred floats) between pass 1 and pass 2.
//
// NCCL is bound at run time with dlopen("libnccl.so.2") so the library loads
// (and its CPU-side entry points work) on machines without NCCL; the first
// mf_comm_* call reports MF_ERR_NEEDS_PLATFORM_SETUP if it is missing.  In a
// process that already loaded NCCL (e.g. through torch.distributed) dlopen
// returns that copy.
#include <dlfcn.h>

#include <cstring>
#include <mutex>

#include "mf_internal.h"
#include "mf_runtime.h"

namespace {

// The subset of nccl.h this file uses (NCCL 2.x ABI).
typedef struct ncclComm* ncclComm_t;
typedef struct {
    char internal[128];
} ncclUniqueId;
typedef enum { ncclSuccess = 0 } ncclResult_t;
constexpr int kNcclFloat32 = 7;  // ncclFloat32
constexpr int kNcclMax = 2;      // ncclMax

struct NcclApi {
    ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*all_reduce)(const void*, void*, size_t, int, int, ncclComm_t, cudaStream_t) = nullptr;
    const char* (*get_error_string)(ncclResult_t) = nullptr;
    bool loaded = false;
};

NcclApi g_nccl;
std::mutex g_nccl_mutex;

int load_nccl() {
    std::lock_guard<std::mutex> lock(g_nccl_mutex);
    if (g_nccl.loaded) return MF_OK;
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return mf::fail(MF_ERR_NEEDS_PLATFORM_SETUP, "mfcuda: NCCL not available (%s)", dlerror());
    g_nccl.get_unique_id = reinterpret_cast<decltype(g_nccl.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    g_nccl.comm_init_rank = reinterpret_cast<decltype(g_nccl.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
    g_nccl.comm_destroy = reinterpret_cast<decltype(g_nccl.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    g_nccl.all_reduce = reinterpret_cast<decltype(g_nccl.all_reduce)>(dlsym(h, "ncclAllReduce"));
    g_nccl.get_error_string = reinterpret_cast<decltype(g_nccl.get_error_string)>(dlsym(h, "ncclGetErrorString"));
    if (!g_nccl.get_unique_id || !g_nccl.comm_init_rank || !g_nccl.comm_destroy || !g_nccl.all_reduce ||
        !g_nccl.get_error_string)
        return mf::fail(MF_ERR_NEEDS_PLATFORM_SETUP, "mfcuda: libnccl lacks a required symbol");
    g_nccl.loaded = true;
    return MF_OK;
}

int nccl_fail(ncclResult_t r, const char* what) {
    return mf::fail(MF_ERR_NCCL, "%s: %s", what, g_nccl.get_error_string ? g_nccl.get_error_string(r) : "error");
}

}  // namespace

struct mf_comm_s {
    ncclComm_t comm = nullptr;
    int world = 0;
    int rank = 0;
};

namespace mf {

int comm_allreduce_max(mf_comm comm, float* d_vec, int64_t count, cudaStream_t s) {
    if (!comm || !comm->comm) return fail(MF_ERR_INVALID_ARGUMENT, "allreduce: communicator is not initialised");
    if (count <= 0) return MF_OK;
    const ncclResult_t r = g_nccl.all_reduce(d_vec, d_vec, static_cast<size_t>(count), kNcclFloat32, kNcclMax,
                                             comm->comm, s);
    if (r != ncclSuccess) return nccl_fail(r, "ncclAllReduce");
    return MF_OK;
}

}  // namespace mf

using namespace mf;

extern "C" int mf_comm_unique_id(void* id128) {
    if (!id128) return fail(MF_ERR_INVALID_ARGUMENT, "mf_comm_unique_id: NULL buffer");
    int rc = load_nccl();
    if (rc) return rc;
    ncclUniqueId id;
    const ncclResult_t r = g_nccl.get_unique_id(&id);
    if (r != ncclSuccess) return nccl_fail(r, "ncclGetUniqueId");
    std::memcpy(id128, &id, sizeof id);
    return MF_OK;
}

extern "C" int mf_comm_init(mf_comm* comm, int32_t world, int32_t rank, const void* id128) {
    MF_ENTER();
    if (!comm || !id128) return fail(MF_ERR_INVALID_ARGUMENT, "mf_comm_init: NULL argument");
    *comm = nullptr;
    if (world < 1 || rank < 0 || rank >= world)
        return fail(MF_ERR_INVALID_ARGUMENT, "mf_comm_init: rank %d outside world %d", rank, world);
    int rc = load_nccl();
    if (rc) return rc;
    ncclUniqueId id;
    std::memcpy(&id, id128, sizeof id);
    mf_comm_s* c = new mf_comm_s();
    const ncclResult_t r = g_nccl.comm_init_rank(&c->comm, world, id, rank);
    if (r != ncclSuccess) {
        delete c;
        return nccl_fail(r, "ncclCommInitRank");
    }
    c->world = world;
    c->rank = rank;
    *comm = c;
    return MF_OK;
}

extern "C" int mf_comm_destroy(mf_comm comm) {
    if (!comm) return MF_OK;
    int rc = MF_OK;
    if (comm->comm) {
        const ncclResult_t r = g_nccl.comm_destroy(comm->comm);
        if (r != ncclSuccess) rc = nccl_fail(r, "ncclCommDestroy");
    }
    delete comm;
    return rc;
}

extern "C" int mf_comm_allreduce_max_f32(mf_comm comm, float* d_vec, int64_t count, mf_stream stream) {
    MF_ENTER();
    if (count < 0) return fail(MF_ERR_SHAPE_INVALID, "mf_comm_allreduce_max_f32: negative count");
    if (count > 0 && !d_vec) return fail(MF_ERR_INVALID_ARGUMENT, "mf_comm_allreduce_max_f32: NULL vector");
    return comm_allreduce_max(comm, d_vec, count, static_cast<cudaStream_t>(stream));
}
