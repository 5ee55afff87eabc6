// ep.h - expert parallelism: one rank per GPU, the experts of every layer
// split in contiguous ranges, everything else replicated.  NCCL (loaded at
// run time) sets the group up; the per-layer combine exchange is a kernel
// that writes each rank's expert output rows into every rank's receive
// buffer over NVLink (kernels.h, ep_push).
#pragma once
#include "context.h"

namespace pc {

// ncclCommInitRank from opts.nccl_id; checks that the ranks drive distinct
// GPUs; allocates this rank's exchange block and maps every other rank's
// (CUDA IPC handles gathered over NCCL).
pc_status ep_init(pc_ctx *c);
void ep_destroy(pc_ctx *c);
// After the down projection of P (token, k) pairs whose outputs (this rank's
// pairs only) are in c->eo: pushes them to every rank.  The combine that
// follows reads them through ep_wait_view.
pc_status ep_exchange(pc_ctx *c, int P);
EpWait ep_wait_view(const pc_ctx *c);

}  // namespace pc
