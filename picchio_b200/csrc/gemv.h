// gemv.h - host interface of the dequant-fused streaming GEMV (gemv.cu).
#pragma once
#include <cuda_runtime.h>

#include "layout.h"

namespace pc {

constexpr int GEMV_CONSUMERS = 12;
constexpr int GEMV_STEP_BLOCKS = 4;  // k-blocks a warp holds in registers per step
constexpr int GEMV_THREADS = 32 * GEMV_CONSUMERS;

size_t gemv_smem_bytes(int nt, int Ip, int stages, int stage_bytes);
cudaError_t gemv_configure(int max_smem);
bool gemv_plan(GemvParams &p, int nt, int max_smem);
cudaError_t gemv_launch(const GemvParams &p, int nt, int grid, cudaStream_t st);

}  // namespace pc
