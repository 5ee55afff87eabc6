// ep.cpp - expert-parallel set-up and the combine exchange.
//
// NCCL is resolved with dlopen so the library loads (and a single GPU runs)
// without NCCL on the machine; when torch has already loaded libnccl.so.2
// into the process, dlopen returns that copy.  NCCL is used at set-up only:
// two all-gathers (GPU identities, CUDA IPC handles of the exchange blocks).
// Each step's exchange is the ep_push kernel writing into the other GPUs'
// memory through those mappings, with no NCCL call per layer.
#include "ep.h"

#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>
#include <string>
#include <vector>

namespace pc {

namespace {

struct NcclApi {
    void *h = nullptr;
    decltype(&ncclGetUniqueId) get_id = nullptr;
    decltype(&ncclCommInitRank) init = nullptr;
    decltype(&ncclAllGather) allgather = nullptr;
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
        a.allgather = (decltype(a.allgather))dlsym(a.h, "ncclAllGather");
        a.destroy = (decltype(a.destroy))dlsym(a.h, "ncclCommDestroy");
        a.errstr = (decltype(a.errstr))dlsym(a.h, "ncclGetErrorString");
        a.ok = a.get_id && a.init && a.allgather && a.destroy && a.errstr;
    });
    return a;
}

pc_status nccl_fail(ncclResult_t r, const char *what) {
    return fail(PC_ERR_NCCL, std::string(what) + ": " + (api().errstr ? api().errstr(r) : "nccl error"));
}

// Every rank's `bytes` bytes at `mine`, in rank order, through a device
// buffer (set-up only).
pc_status allgather_host(pc_ctx *c, const void *mine, size_t bytes, std::vector<char> &all) {
    const int n = c->opts.ep_size;
    char *d = nullptr;
    PC_CU(cudaMalloc(&d, bytes * (n + 1)));
    pc_status s = PC_OK;
    cudaError_t e = cudaMemcpyAsync(d + bytes * n, mine, bytes, cudaMemcpyHostToDevice, c->st);
    if (e != cudaSuccess) s = cuda_fail(e, "cudaMemcpy");
    if (s == PC_OK) {
        ncclResult_t r = api().allgather(d + bytes * n, d, bytes, ncclUint8, (ncclComm_t)c->nccl_comm, c->st);
        if (r != ncclSuccess) s = nccl_fail(r, "ncclAllGather");
    }
    if (s == PC_OK && (e = cudaStreamSynchronize(c->st)) != cudaSuccess) s = cuda_fail(e, "ncclAllGather");
    all.assign(bytes * n, 0);
    if (s == PC_OK && (e = cudaMemcpy(all.data(), d, bytes * n, cudaMemcpyDeviceToHost)) != cudaSuccess)
        s = cuda_fail(e, "cudaMemcpy");
    cudaFree(d);
    return s;
}

}  // namespace

pc_status ep_init(pc_ctx *c) {
    NcclApi &a = api();
    if (!a.ok) return fail(PC_ERR_NCCL, "libnccl.so.2 not found: expert parallelism needs NCCL");
    if (!c->opts.nccl_id) return fail(PC_ERR_INVALID_ARG, "ep_size > 1 needs opts.nccl_id");
    const int n = c->opts.ep_size, rank = c->opts.ep_rank;
    if (rank < 0 || rank >= n) return fail(PC_ERR_INVALID_ARG, "ep_rank outside [0, ep_size)");
    if (n > EP_MAX_RANKS) return fail(PC_ERR_RANGE, "ep_size above " + std::to_string(EP_MAX_RANKS));
    ncclUniqueId id;
    memcpy(&id, c->opts.nccl_id, sizeof id);
    ncclComm_t comm = nullptr;
    ncclResult_t r = a.init(&comm, n, id, rank);
    if (r != ncclSuccess) return nccl_fail(r, "ncclCommInitRank");
    c->nccl_comm = comm;
    c->ep_n = n;
    c->ep_rank = rank;

    // One GPU per rank: ranks sharing a GPU would each wait inside a kernel
    // for the other's kernel, which that GPU need not run at the same time.
    cudaDeviceProp prop;
    PC_CU(cudaGetDeviceProperties(&prop, c->dev));
    std::vector<char> uuids;
    PC_TRY(allgather_host(c, prop.uuid.bytes, 16, uuids));
    for (int p = 0; p < n; ++p)
        for (int q = p + 1; q < n; ++q)
            if (!memcmp(&uuids[16 * p], &uuids[16 * q], 16))
                return fail(PC_ERR_INVALID_ARG, "expert-parallel ranks " + std::to_string(p) + " and " +
                                                    std::to_string(q) + " share one GPU");

    // This rank's exchange block: flags, then two receive buffers for the
    // output rows of every (token, k) pair of a step.
    const pc_model_cfg &k = c->cfg;
    c->ep_rx_bytes = ((int64_t)c->maxm * k.topk * k.hidden * 4 + 255) & ~(int64_t)255;
    const size_t blk_bytes = EP_FLAG_BYTES + 2 * (size_t)c->ep_rx_bytes;
    char *blk = nullptr;
    PC_CU(cudaMalloc(&blk, blk_bytes));
    c->ep_blk[rank] = blk;
    PC_CU(cudaMemset(blk, 0, blk_bytes));
    PC_TRY(dalloc(c, 16, (void **)&c->ep_state));
    PC_CU(cudaDeviceSynchronize());  // zeroed before any peer can write into it
    cudaIpcMemHandle_t h;
    PC_CU(cudaIpcGetMemHandle(&h, blk));
    std::vector<char> handles;
    PC_TRY(allgather_host(c, &h, sizeof h, handles));
    for (int q = 0; q < n; ++q) {
        if (q == rank) continue;
        cudaIpcMemHandle_t hq;
        memcpy(&hq, &handles[sizeof hq * q], sizeof hq);
        void *p = nullptr;
        PC_CU(cudaIpcOpenMemHandle(&p, hq, cudaIpcMemLazyEnablePeerAccess));
        c->ep_blk[q] = (char *)p;
    }
    return PC_OK;
}

void ep_destroy(pc_ctx *c) {
    for (int q = 0; q < EP_MAX_RANKS; ++q) {
        if (!c->ep_blk[q]) continue;
        if (q == c->ep_rank) cudaFree(c->ep_blk[q]);
        else cudaIpcCloseMemHandle(c->ep_blk[q]);
        c->ep_blk[q] = nullptr;
    }
    if (c->nccl_comm && api().ok) api().destroy((ncclComm_t)c->nccl_comm);
    c->nccl_comm = nullptr;
}

pc_status ep_exchange(pc_ctx *c, int P) {
    EpPushParams p{};
    p.eo = c->eo;
    p.pair_local = c->pair_local;
    p.P = P;
    p.D = c->cfg.hidden;
    p.rank = c->ep_rank;
    p.n = c->ep_n;
    for (int q = 0; q < c->ep_n; ++q) p.blk[q] = c->ep_blk[q];
    p.rx_bytes = c->ep_rx_bytes;
    p.state = c->ep_state;
    PC_CU(launch_ep_push(p, c->nsm, c->st));
    ++c->launches;
    return PC_OK;
}

EpWait ep_wait_view(const pc_ctx *c) {
    EpWait w{};
    w.blk = c->ep_blk[c->ep_rank];
    w.rx_bytes = c->ep_rx_bytes;
    w.state = c->ep_state;
    w.n = c->ep_n;
    w.err = c->err;
    return w;
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
