// gemv.h - host interface of the dequant-fused streaming GEMV (gemv.cu).
#pragma once
#include <cuda_runtime.h>

#include "layout.h"

namespace pc {

constexpr int GEMV_CONSUMERS = 12;
// k-blocks per step of a warp (64-column T4 or 32-column T8 blocks), and the
// depth of its shared-memory ring of steps; both shrink with the N-tiles so
// that the B operand and the rings fit in one CTA's shared memory.  4-bit
// blocks with two N-tiles (batched decode jobs) take 8-block steps in a
// 2-deep ring: the same bytes in flight as 4-block steps 3 deep, half the
// per-step work (bs64 decode +13 %); a padded input row of up to ~4100
// columns fits (gs32), longer ones run as one-N-tile jobs (pc_qt_matmul).
// With one N-tile, 5-block steps 3 deep: a GPT-OSS expert unit (45 blocks)
// split over 3 warps is then three full steps per warp (bs1 decode +0.6 %).
__host__ __device__ constexpr int gemv_step_blocks(int fmt, int nt) {
    return nt == 4 ? 2 : (tf_4bit(fmt) ? (nt == 2 ? 8 : 5) : 8);
}
__host__ __device__ constexpr int gemv_ring_depth(int fmt, int nt) { return nt == 1 ? 3 : 2; }
// N-tiles (8 MMA columns = 2 input rows x 4 digit columns) for a job of `rows` input rows
inline int gemv_nt_for_rows(int rows) { return rows <= 2 ? 1 : rows <= 4 ? 2 : 4; }
constexpr int GEMV_THREADS = 32 * GEMV_CONSUMERS;

// Dynamic shared memory of one GEMV launch.
size_t gemv_smem_bytes(int fmt, int nt, int Ip, int blk_bytes);
cudaError_t gemv_configure(int max_smem);
bool gemv_plan(GemvParams &p, int nt, int max_smem);
cudaError_t gemv_launch(const GemvParams &p, int nt, int grid, cudaStream_t st);

}  // namespace pc
