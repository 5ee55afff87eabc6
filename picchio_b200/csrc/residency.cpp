// residency.cpp - streamed expert residency (residency.h).
#include "residency.h"

#include <cuda_runtime.h>

#include <algorithm>

#include "context.h"

namespace pc {

namespace {

__global__ void emap_set_kernel(const uint8_t **entry, const uint8_t *addr) { *entry = addr; }

const uint8_t *host_copy(const pc_ctx *c, int l, int e) {
    return c->res.host[l] + (int64_t)(e - c->e_lo) * c->eg.stride;
}

// Picks a slot for expert e of layer l: a free one, else the least recently
// used (lowest slot on ties), whose expert is read from the host again.  The
// map mirror keeps e on its host copy; returns the slot.
int claim_slot(pc_ctx *c, int l, int e) {
    Residency &r = c->res;
    std::vector<int> &own = r.owner[l];
    int victim = -1;
    for (int s = 0; s < r.slots && victim < 0; ++s)
        if (own[s] < 0) victim = s;
    if (victim < 0) {
        victim = 0;
        for (int s = 1; s < r.slots; ++s)
            if (r.last[l][own[s]] < r.last[l][own[victim]]) victim = s;
        const int old = own[victim];
        r.slot_of[l][old] = -1;
        r.h_emap[(size_t)l * r.E + old] = host_copy(c, l, old);
    }
    own[victim] = e;
    r.slot_of[l][e] = victim;
    return victim;
}

uint8_t *slot_addr(pc_ctx *c, int l, int s) { return c->L[l].experts + (int64_t)s * c->eg.stride; }

pc_status publish_map(pc_ctx *c) {
    Residency &r = c->res;
    const size_t n = (size_t)c->cfg.n_layers * r.E;
    PC_CU(cudaMemcpyAsync(r.emap, r.h_emap, n * sizeof(uint8_t *), cudaMemcpyHostToDevice, c->st));
    PC_CU(cudaStreamSynchronize(c->st));
    return PC_OK;
}

}  // namespace

pc_status res_init(pc_ctx *c) {
    Residency &r = c->res;
    PC_CU(cudaStreamCreateWithFlags(&r.side, cudaStreamNonBlocking));
    const int L = c->cfg.n_layers, E = c->cfg.n_experts, El = c->e_hi - c->e_lo;
    const int64_t stride = c->eg.stride;
    if (c->opts.expert_cache_slots < 1) return fail(PC_ERR_INVALID_ARG, "expert_cache_slots must be >= 1");
    r.E = E;
    r.slots = std::min(c->opts.expert_cache_slots, El);
    r.host.assign(L, nullptr);
    for (int l = 0; l < L; ++l) {
        if (cudaHostAlloc((void **)&r.host[l], (size_t)El * stride, cudaHostAllocMapped | cudaHostAllocPortable) !=
            cudaSuccess) {
            r.host[l] = nullptr;
            return fail(PC_ERR_OOM, "pinned host expert table");
        }
        PC_TRY(dalloc(c, (size_t)r.slots * stride, (void **)&c->L[l].experts));
    }
    const size_t n = (size_t)L * E;
    PC_TRY(dalloc(c, n * sizeof(uint8_t *), (void **)&r.emap));
    PC_TRY(dalloc(c, n, (void **)&r.used));
    PC_CU(cudaMemset(r.used, 0, n));
    PC_TRY(dalloc(c, (size_t)stride, (void **)&r.stage));
    if (cudaHostAlloc((void **)&r.h_emap, n * sizeof(uint8_t *), cudaHostAllocDefault) != cudaSuccess ||
        cudaHostAlloc((void **)&r.h_used, n, cudaHostAllocDefault) != cudaSuccess)
        return fail(PC_ERR_OOM, "pinned expert map");
    r.owner.assign(L, std::vector<int>(r.slots, -1));
    r.slot_of.assign(L, std::vector<int>(E, -1));
    r.last.assign(L, std::vector<uint64_t>(E, 0));
    r.on = true;
    return PC_OK;
}

pc_status res_store(pc_ctx *c, int l, int e) {
    PC_CU(cudaStreamSynchronize(c->st));
    PC_CU(cudaMemcpy(c->res.host[l] + (int64_t)(e - c->e_lo) * c->eg.stride, c->res.stage, (size_t)c->eg.stride,
                     cudaMemcpyDeviceToHost));
    return PC_OK;
}

pc_status res_finish_load(pc_ctx *c) {
    Residency &r = c->res;
    for (int l = 0; l < c->cfg.n_layers; ++l)
        for (int e = 0; e < r.E; ++e)
            r.h_emap[(size_t)l * r.E + e] = (e >= c->e_lo && e < c->e_hi) ? host_copy(c, l, e) : nullptr;
    return publish_map(c);
}

pc_status res_after_step(pc_ctx *c) {
    Residency &r = c->res;
    if (!r.on) return PC_OK;
    const int L = c->cfg.n_layers;
    const size_t n = (size_t)L * r.E;
    // the previous round's slot copies and map switches are done before any
    // of their slots can be evicted again
    PC_CU(cudaStreamSynchronize(r.side));
    PC_CU(cudaMemcpyAsync(r.h_used, r.used, n, cudaMemcpyDeviceToHost, c->st));
    PC_CU(cudaStreamSynchronize(c->st));
    ++r.round;
    struct Load { int l, e, s; };
    std::vector<Load> loads;
    bool missed = false;
    for (int l = 0; l < L; ++l)
        for (int e = c->e_lo; e < c->e_hi; ++e) {
            if (!r.h_used[(size_t)l * r.E + e]) continue;
            r.last[l][e] = r.round;
            if (r.slot_of[l][e] >= 0) {
                ++r.hits;
            } else {
                ++r.misses;
                missed = true;
                loads.push_back({l, e, claim_slot(c, l, e)});
            }
        }
    // a round with more misses than slots evicts some of its own loads again:
    // only the experts still owning their slot are copied (the others stay on
    // their host copies in the map)
    loads.erase(std::remove_if(loads.begin(), loads.end(),
                               [&](const Load &ld) { return r.owner[ld.l][ld.s] != ld.e; }),
                loads.end());
    if (loads.empty()) {
        PC_CU(cudaMemsetAsync(r.used, 0, n, c->st));
        return missed ? publish_map(c) : PC_OK;
    }
    // 1. evicted experts back on their host copies before the next step
    PC_TRY(publish_map(c));
    PC_CU(cudaMemsetAsync(r.used, 0, n, c->st));
    // 2. copies on the side stream, each entry switched after its copy
    for (const Load &ld : loads) {
        uint8_t *dst = slot_addr(c, ld.l, ld.s);
        PC_CU(cudaMemcpyAsync(dst, host_copy(c, ld.l, ld.e), (size_t)c->eg.stride, cudaMemcpyHostToDevice, r.side));
        const uint8_t **entry = r.emap + (size_t)ld.l * r.E + ld.e;
        emap_set_kernel<<<1, 1, 0, r.side>>>(entry, dst);
        PC_CU(cudaGetLastError());
        r.h_emap[(size_t)ld.l * r.E + ld.e] = dst;
        r.bytes += (uint64_t)c->eg.stride;
    }
    return PC_OK;
}

pc_status res_prefetch(pc_ctx *c, int l, const int *eids, int n) {
    Residency &r = c->res;
    if (!r.on) return PC_OK;
    PC_CU(cudaStreamSynchronize(r.side));
    ++r.round;
    bool moved = false;
    for (int i = 0; i < n; ++i) {
        const int e = eids[i];
        if (e < c->e_lo || e >= c->e_hi) continue;  // another rank's expert, or eid -1
        r.last[l][e] = r.round;
        if (r.slot_of[l][e] >= 0) continue;
        const int s = claim_slot(c, l, e);
        // resident on return (cache_load_batch): copied on the compute stream
        PC_CU(cudaMemcpyAsync(slot_addr(c, l, s), host_copy(c, l, e), (size_t)c->eg.stride, cudaMemcpyHostToDevice,
                              c->st));
        r.h_emap[(size_t)l * r.E + e] = slot_addr(c, l, s);
        r.bytes += (uint64_t)c->eg.stride;
        moved = true;
    }
    return moved ? publish_map(c) : PC_OK;
}

void res_free(pc_ctx *c) {
    Residency &r = c->res;
    if (r.side) {
        cudaStreamSynchronize(r.side);
        cudaStreamDestroy(r.side);
    }
    for (uint8_t *p : r.host)
        if (p) cudaFreeHost(p);
    if (r.h_emap) cudaFreeHost((void *)r.h_emap);
    if (r.h_used) cudaFreeHost(r.h_used);
    r = Residency{};
}

}  // namespace pc
