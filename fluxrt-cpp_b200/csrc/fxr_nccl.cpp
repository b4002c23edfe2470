// fxr_nccl.cpp — NCCL entry points of the head-split frame, with NCCL resolved at run time.
//
// The library does not link NCCL: a process that already holds a libnccl.so.2 (for example through
// PyTorch's distributed package) must drive communicators created by that same copy, so the
// functions are looked up with dlopen(RTLD_NOLOAD) first and only then from the loader's search
// path. Types and signatures come from the installed nccl.h.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "fxr.h"

extern "C" void fxr_internal_set_error(const char* msg);

namespace {

static_assert(sizeof(ncclUniqueId) == 128, "fxr_nccl_unique_id hands out 128-byte ids");
typedef int NcclResult;

struct NcclApi {
    decltype(&ncclGetUniqueId) get_unique_id = nullptr;
    decltype(&ncclCommInitRank) comm_init_rank = nullptr;
    decltype(&ncclCommDestroy) comm_destroy = nullptr;
    decltype(&ncclAllGather) all_gather = nullptr;
    decltype(&ncclGetErrorString) error_string = nullptr;
    bool ok = false;
    std::string why;
};

const NcclApi& api() {
    static NcclApi a;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_LOCAL);
        if (!h) {
            a.why = "libnccl.so.2 not found";
            return;
        }
        a.get_unique_id = reinterpret_cast<decltype(a.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
        a.comm_init_rank = reinterpret_cast<decltype(a.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
        a.comm_destroy = reinterpret_cast<decltype(a.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
        a.all_gather = reinterpret_cast<decltype(a.all_gather)>(dlsym(h, "ncclAllGather"));
        a.error_string = reinterpret_cast<decltype(a.error_string)>(dlsym(h, "ncclGetErrorString"));
        a.ok = a.get_unique_id && a.comm_init_rank && a.comm_destroy && a.all_gather;
        if (!a.ok) a.why = "libnccl.so.2 lacks a required symbol";
    });
    return a;
}

int32_t nccl_fail(const char* what, NcclResult r) {
    const NcclApi& a = api();
    char buf[256];
    std::snprintf(buf, sizeof(buf), "%s: NCCL error %d (%s)", what, r,
                  a.error_string ? a.error_string(static_cast<ncclResult_t>(r)) : "?");
    fxr_internal_set_error(buf);
    return FXR_ERR_NCCL;
}

int32_t no_nccl() {
    fxr_internal_set_error(("NCCL unavailable: " + api().why).c_str());
    return FXR_ERR_NCCL;
}

}  // namespace

extern "C" {

int32_t fxr_nccl_unique_id(unsigned char id_out[128]) {
    if (!id_out) return FXR_ERR_INVALID;
    const NcclApi& a = api();
    if (!a.ok) return no_nccl();
    ncclUniqueId id;
    NcclResult r = a.get_unique_id(&id);
    if (r != 0) return nccl_fail("ncclGetUniqueId", r);
    std::memcpy(id_out, id.internal, sizeof(id.internal));
    return FXR_OK;
}

int32_t fxr_nccl_comm_init(int32_t world, int32_t rank, const unsigned char id[128], void** comm) {
    if (!id || !comm || world < 1 || rank < 0 || rank >= world) return FXR_ERR_INVALID;
    const NcclApi& a = api();
    if (!a.ok) return no_nccl();
    ncclUniqueId uid;
    std::memcpy(uid.internal, id, sizeof(uid.internal));
    ncclComm_t c = nullptr;
    NcclResult r = a.comm_init_rank(&c, world, uid, rank);
    if (r != 0) return nccl_fail("ncclCommInitRank", r);
    *comm = c;
    return FXR_OK;
}

int32_t fxr_nccl_comm_destroy(void* comm) {
    if (!comm) return FXR_OK;
    const NcclApi& a = api();
    if (!a.ok) return no_nccl();
    NcclResult r = a.comm_destroy(static_cast<ncclComm_t>(comm));
    return r == 0 ? FXR_OK : nccl_fail("ncclCommDestroy", r);
}

// Byte all-gather on `comm` (used by fxr_allgather_heads).
int32_t fxr_internal_nccl_allgather(const void* send, void* recv, size_t bytes, void* comm,
                                    void* stream) {
    const NcclApi& a = api();
    if (!a.ok) return no_nccl();
    NcclResult r = a.all_gather(send, recv, bytes, ncclInt8, static_cast<ncclComm_t>(comm),
                                static_cast<cudaStream_t>(stream));
    return r == 0 ? FXR_OK : nccl_fail("ncclAllGather", r);
}

}  // extern "C"
