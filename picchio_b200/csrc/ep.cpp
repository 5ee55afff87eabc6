// ep.cpp - NCCL for expert parallelism, resolved with dlopen so the library
// loads (and a single GPU runs) without NCCL on the machine.  When torch has
// already loaded libnccl.so.2 into the process, dlopen returns that copy.
#include "ep.h"

#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>
#include <string>

namespace pc {

namespace {

struct NcclApi {
    void *h = nullptr;
    decltype(&ncclGetUniqueId) get_id = nullptr;
    decltype(&ncclCommInitRank) init = nullptr;
    decltype(&ncclAllReduce) allreduce = nullptr;
    decltype(&ncclCommDestroy) destroy = nullptr;
    decltype(&ncclGetErrorString) errstr = nullptr;
    bool ok = false;
};

NcclApi &api() {
    static NcclApi a;
    static std::once_flag once;
    std::call_once(once, [] {
        const char *names[] = {"libnccl.so.2", "libnccl.so"};
        for (const char *n : names) {
            a.h = dlopen(n, RTLD_NOW | RTLD_GLOBAL);
            if (a.h) break;
        }
        if (!a.h) return;
        a.get_id = (decltype(a.get_id))dlsym(a.h, "ncclGetUniqueId");
        a.init = (decltype(a.init))dlsym(a.h, "ncclCommInitRank");
        a.allreduce = (decltype(a.allreduce))dlsym(a.h, "ncclAllReduce");
        a.destroy = (decltype(a.destroy))dlsym(a.h, "ncclCommDestroy");
        a.errstr = (decltype(a.errstr))dlsym(a.h, "ncclGetErrorString");
        a.ok = a.get_id && a.init && a.allreduce && a.destroy && a.errstr;
    });
    return a;
}

pc_status nccl_fail(ncclResult_t r, const char *what) {
    return fail(PC_ERR_NCCL, std::string(what) + ": " + (api().errstr ? api().errstr(r) : "nccl error"));
}

}  // namespace

pc_status ep_init(pc_ctx *c) {
    NcclApi &a = api();
    if (!a.ok) return fail(PC_ERR_NCCL, "libnccl.so.2 not found: expert parallelism needs NCCL");
    if (!c->opts.nccl_id) return fail(PC_ERR_INVALID_ARG, "ep_size > 1 needs opts.nccl_id");
    if (c->opts.ep_rank < 0 || c->opts.ep_rank >= c->opts.ep_size) return fail(PC_ERR_INVALID_ARG, "ep_rank outside [0, ep_size)");
    ncclUniqueId id;
    memcpy(&id, c->opts.nccl_id, sizeof id);
    ncclComm_t comm = nullptr;
    ncclResult_t r = a.init(&comm, c->opts.ep_size, id, c->opts.ep_rank);
    if (r != ncclSuccess) return nccl_fail(r, "ncclCommInitRank");
    c->nccl_comm = comm;
    return PC_OK;
}

void ep_destroy(pc_ctx *c) {
    if (c->nccl_comm && api().ok) api().destroy((ncclComm_t)c->nccl_comm);
    c->nccl_comm = nullptr;
}

pc_status ep_allreduce_sum(pc_ctx *c, float *buf, size_t n) {
    ncclResult_t r = api().allreduce(buf, buf, n, ncclFloat32, ncclSum, (ncclComm_t)c->nccl_comm, c->st);
    if (r != ncclSuccess) return nccl_fail(r, "ncclAllReduce");
    return PC_OK;
}

}  // namespace pc

extern "C" pc_status pc_nccl_unique_id(void *out128) {
    if (!out128) return pc::fail(PC_ERR_INVALID_ARG, "null output");
    pc::NcclApi &a = pc::api();
    if (!a.ok) return pc::fail(PC_ERR_NCCL, "libnccl.so.2 not found");
    ncclUniqueId id;
    ncclResult_t r = a.get_id(&id);
    if (r != ncclSuccess) return pc::nccl_fail(r, "ncclGetUniqueId");
    static_assert(sizeof(id) == 128, "ncclUniqueId is 128 bytes");
    memcpy(out128, &id, sizeof id);
    return PC_OK;
}
