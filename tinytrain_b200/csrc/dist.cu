// Collectives for data parallelism: NCCL over NVLink 5 / NVSwitch, one
// communicator per rank (one process per GPU). The reference has no
// distributed code; this is the exchange step of the data-parallel path
// (gradient all-reduce between backward and the optimizer step).
//
// libnccl.so.2 is opened at first use (dlopen), so the kernel library has no
// link-time dependency on it; in a process that already loaded NCCL (e.g.
// through torch) the loaded copy is reused.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <stdint.h>

#include <cstdio>
#include <cstring>
#include <mutex>

#include "ttk_internal.h"

namespace {

// The subset of nccl.h used here (ABI-stable across NCCL 2.x).
typedef struct {
    char internal[128];
} NcclUniqueId;
typedef void* NcclComm;
enum { kNcclFloat32 = 7, kNcclFloat64 = 9, kNcclSum = 0 };

struct Nccl {
    int (*GetUniqueId)(NcclUniqueId*) = nullptr;
    int (*CommInitRank)(NcclComm*, int, NcclUniqueId, int) = nullptr;
    int (*CommDestroy)(NcclComm) = nullptr;
    int (*CommAbort)(NcclComm) = nullptr;
    int (*CommGetAsyncError)(NcclComm, int*) = nullptr;
    int (*AllReduce)(const void*, void*, size_t, int, int, NcclComm, cudaStream_t) = nullptr;
    const char* (*GetErrorString)(int) = nullptr;
    bool ok = false;
};

Nccl& nccl() {
    static Nccl n;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h)
            h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h)
            return;
        n.GetUniqueId = reinterpret_cast<decltype(n.GetUniqueId)>(dlsym(h, "ncclGetUniqueId"));
        n.CommInitRank = reinterpret_cast<decltype(n.CommInitRank)>(dlsym(h, "ncclCommInitRank"));
        n.CommDestroy = reinterpret_cast<decltype(n.CommDestroy)>(dlsym(h, "ncclCommDestroy"));
        n.CommAbort = reinterpret_cast<decltype(n.CommAbort)>(dlsym(h, "ncclCommAbort"));
        n.CommGetAsyncError =
            reinterpret_cast<decltype(n.CommGetAsyncError)>(dlsym(h, "ncclCommGetAsyncError"));
        n.AllReduce = reinterpret_cast<decltype(n.AllReduce)>(dlsym(h, "ncclAllReduce"));
        n.GetErrorString =
            reinterpret_cast<decltype(n.GetErrorString)>(dlsym(h, "ncclGetErrorString"));
        n.ok = n.GetUniqueId && n.CommInitRank && n.CommDestroy && n.AllReduce && n.CommAbort &&
               n.CommGetAsyncError;
    });
    return n;
}

int nccl_status(int r, const char* what) {
    if (r == 0)
        return TTK_OK;
    static thread_local char buf[256];
    const char* m = nccl().GetErrorString ? nccl().GetErrorString(r) : "nccl error";
    snprintf(buf, sizeof(buf), "%s: %s", what, m);
    return ttk::set_error(TTK_ERR_NCCL, buf);
}

int need_nccl() {
    if (!nccl().ok)
        return ttk::set_error(TTK_ERR_NCCL, "libnccl.so.2 not found or incomplete");
    return TTK_OK;
}

}  // namespace

extern "C" {

int ttk_dist_unique_id(unsigned char out[128]) {
    int rc = need_nccl();
    if (rc)
        return rc;
    NcclUniqueId id;
    rc = nccl_status(nccl().GetUniqueId(&id), "ncclGetUniqueId");
    if (!rc)
        std::memcpy(out, id.internal, 128);
    return rc;
}

int ttk_dist_init(int rank, int world, const unsigned char id[128], void** comm) {
    int rc = need_nccl();
    if (rc)
        return rc;
    if (world < 1 || rank < 0 || rank >= world || !comm)
        return ttk::set_error(TTK_ERR_ARG, "dist_init: bad rank/world");
    NcclUniqueId uid;
    std::memcpy(uid.internal, id, 128);
    NcclComm c = nullptr;
    rc = nccl_status(nccl().CommInitRank(&c, world, uid, rank), "ncclCommInitRank");
    *comm = c;
    return rc;
}

int ttk_dist_destroy(void* comm) {
    if (!comm)
        return TTK_OK;
    int rc = need_nccl();
    if (rc)
        return rc;
    return nccl_status(nccl().CommDestroy(comm), "ncclCommDestroy");
}

int ttk_dist_abort(void* comm) {
    if (!comm)
        return TTK_OK;
    int rc = need_nccl();
    if (rc)
        return rc;
    return nccl_status(nccl().CommAbort(comm), "ncclCommAbort");
}

int ttk_dist_async_error(void* comm, int* err) {
    int rc = need_nccl();
    if (rc)
        return rc;
    int e = 0;
    rc = nccl_status(nccl().CommGetAsyncError(comm, &e), "ncclCommGetAsyncError");
    *err = e;
    return rc;
}

int ttk_dist_allreduce_f32(void* comm, float* buf, int64_t n, void* stream) {
    int rc = need_nccl();
    if (rc)
        return rc;
    if (n <= 0)
        return TTK_OK;
    return nccl_status(nccl().AllReduce(buf, buf, static_cast<size_t>(n), kNcclFloat32, kNcclSum,
                                        comm, static_cast<cudaStream_t>(stream)),
                       "ncclAllReduce");
}

int ttk_dist_allreduce_f64(void* comm, double* buf, int64_t n, void* stream) {
    int rc = need_nccl();
    if (rc)
        return rc;
    if (n <= 0)
        return TTK_OK;
    return nccl_status(nccl().AllReduce(buf, buf, static_cast<size_t>(n), kNcclFloat64, kNcclSum,
                                        comm, static_cast<cudaStream_t>(stream)),
                       "ncclAllReduce");
}

}  // extern "C"
