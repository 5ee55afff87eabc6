// residency.h - streamed expert residency (opts.expert_residency == 1): the
// counterpart of the reference's expert cache (ESlot / cache_load_batch /
// the LRU, picchio.c:121-136, 1000-1068) for models whose expert tables do
// not fit HBM.
//
// Every local expert lives in pinned, device-mapped host memory; each layer
// keeps `expert_cache_slots` experts in HBM slots.  The router reads each
// expert's address from a device map (slot or host copy) and flags the
// experts its jobs read, so a step never waits for the host: a miss is read
// over the host link inside the step.  After the step the host picks slots
// for the flagged misses (least recently used first): the evicted experts'
// map entries go back to their host copies before the next step starts, and
// the copies into the slots run on a side stream (cudaMemcpyAsync) that
// overlaps the next step; each entry switches to its slot (one 8-byte store
// by a one-thread kernel) only after its copy has landed, so a concurrent
// router reads either address, both valid.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>
#include <vector>

#include "../../include/picchio_b200.h"

namespace pc {

struct Residency {
    bool on = false;
    int slots = 0;                      // HBM slots per layer
    int E = 0;                          // experts per layer (global count; map is indexed by id)
    std::vector<uint8_t *> host;        // per layer: pinned [E_local][stride]
    const uint8_t **emap = nullptr;     // device [L][E]: address of each expert's bytes
    const uint8_t **h_emap = nullptr;   // pinned mirror
    unsigned char *used = nullptr;      // device [L][E]: experts read since the last update
    unsigned char *h_used = nullptr;    // pinned
    uint8_t *stage = nullptr;           // device: one expert, for loading
    cudaStream_t side = nullptr;        // slot copies
    std::vector<std::vector<int>> owner;     // [L][slots] expert id or -1
    std::vector<std::vector<int>> slot_of;   // [L][E] slot or -1
    std::vector<std::vector<uint64_t>> last; // [L][E] update round of the last use
    uint64_t round = 0, hits = 0, misses = 0, bytes = 0;
};

}  // namespace pc

struct pc_ctx;

namespace pc {

// After the expert geometry is known: pinned tables, HBM slots (one region
// per layer, assigned to the layer's `experts`), maps.
pc_status res_init(pc_ctx *c);
// Copies the expert assembled in c->res.stage to layer l's host table.
pc_status res_store(pc_ctx *c, int l, int e);
// Every expert starts on the host: the map points at the host copies.
pc_status res_finish_load(pc_ctx *c);
// After a step has completed: counts hits and misses of the flagged experts,
// moves the misses into slots (LRU), rewrites the map, clears the flags.
pc_status res_after_step(pc_ctx *c);
// Makes the given experts of layer l resident now (cache_load_batch).
pc_status res_prefetch(pc_ctx *c, int l, const int *eids, int n);
void res_free(pc_ctx *c);

}  // namespace pc
