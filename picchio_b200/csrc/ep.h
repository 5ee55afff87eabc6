// ep.h - expert parallelism: NCCL (loaded at run time) for the one exchange
// of the MoE block.
#pragma once
#include "context.h"

namespace pc {

pc_status ep_init(pc_ctx *c);        // ncclCommInitRank from opts.nccl_id
void ep_destroy(pc_ctx *c);
// In-place sum over the expert-parallel group on the context stream.  Each
// element of the expert-output buffer is non-zero on exactly one rank (the
// owner of that (token, k) pair's expert), so the sum is exact.
pc_status ep_allreduce_sum(pc_ctx *c, float *buf, size_t n);

}  // namespace pc
