// gemv.cu - launches of the dequant-fused GEMV (gemv_core.cuh): one
// persistent CTA of GEMV_THREADS threads per SM, programmatic dependent
// launch, and the host-side plan.
#include <algorithm>

#include "gemv_core.cuh"

namespace pc {

namespace {

template <int FMT, int NT, int GS>
__global__ void __launch_bounds__(GEMV_THREADS, 1) gemv_kernel(const GemvParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    gemv_cta<FMT, NT, GS, true>(p, smem, blockIdx.x, gridDim.x);
}

template <int FMT, int NT, int GS>
cudaError_t set_smem(int max_smem) {
    return cudaFuncSetAttribute(gemv_kernel<FMT, NT, GS>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
}

template <int FMT, int NT, int GS>
cudaError_t go(const GemvParams &p, int grid, size_t smem, cudaStream_t st) {
    return launch_k(gemv_kernel<FMT, NT, GS>, grid, GEMV_THREADS, smem, st, p);
}

template <int NT>
cudaError_t go_nt(const GemvParams &p, int grid, size_t smem, cudaStream_t st) {
    if (p.fmt == TF_T8) return go<TF_T8, NT, 0>(p, grid, smem, st);
    if (p.fmt == TF_F4) return p.gs == 32 ? go<TF_F4, NT, 32>(p, grid, smem, st) : cudaErrorInvalidValue;
    switch (p.gs) {
        case 32: return go<TF_T4, NT, 32>(p, grid, smem, st);
        case 64: return go<TF_T4, NT, 64>(p, grid, smem, st);
        case 16: return go<TF_T4, NT, 16>(p, grid, smem, st);
        case 0: return go<TF_T4, NT, 0>(p, grid, smem, st);
    }
    return cudaErrorInvalidValue;
}

template <int NT>
cudaError_t set_nt(int max_smem) {
    cudaError_t e = set_smem<TF_T8, NT, 0>(max_smem);
    if (e == cudaSuccess) e = set_smem<TF_T4, NT, 0>(max_smem);
    if (e == cudaSuccess) e = set_smem<TF_T4, NT, 16>(max_smem);
    if (e == cudaSuccess) e = set_smem<TF_T4, NT, 32>(max_smem);
    if (e == cudaSuccess) e = set_smem<TF_T4, NT, 64>(max_smem);
    if (e == cudaSuccess) e = set_smem<TF_F4, NT, 32>(max_smem);
    return e;
}

}  // namespace

size_t gemv_smem_bytes(int fmt, int nt, int Ip, int blk_bytes) {
    return (size_t)gemv_smem_need(fmt, nt, Ip, blk_bytes);
}

cudaError_t gemv_configure(int max_smem) {
    cudaError_t e = set_nt<1>(max_smem);
    if (e == cudaSuccess) e = set_nt<2>(max_smem);
    if (e == cudaSuccess) e = set_nt<4>(max_smem);
    return e;
}

// Launch plan: false if the B operand (nt * Ip * 8 bytes) and the warps'
// rings of weight steps do not fit in one CTA's shared memory.
bool gemv_plan(GemvParams &p, int nt, int max_smem) {
    if (gemv_smem_bytes(p.fmt, nt, p.Ip, p.blk_bytes) > (size_t)max_smem) return false;
    p.stages = gemv_ring_depth(p.fmt, nt);
    p.stage_bytes = GEMV_CONSUMERS * gemv_step_blocks(p.fmt, nt) * p.blk_bytes;
    return true;
}

cudaError_t gemv_launch(const GemvParams &p, int nt, int grid, cudaStream_t st) {
    const size_t smem = gemv_smem_bytes(p.fmt, nt, p.Ip, p.blk_bytes);
    switch (nt) {
        case 1: return go_nt<1>(p, grid, smem, st);
        case 2: return go_nt<2>(p, grid, smem, st);
        case 4: return go_nt<4>(p, grid, smem, st);
    }
    return cudaErrorInvalidValue;
}

}  // namespace pc
