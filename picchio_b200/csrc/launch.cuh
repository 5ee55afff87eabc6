// launch.cuh - kernel launches with programmatic dependent launch (PDL).
//
// Every kernel of the step starts with pdl_wait() before it reads anything an
// earlier kernel wrote, and calls pdl_trigger() once it no longer needs its
// launch slot to be exclusive.  Launched with the programmatic-serialization
// attribute, a kernel's CTAs can then be scheduled while its predecessor is
// still finishing (on the SMs the predecessor frees), which hides launch
// latency and, for the GEMV, the first weight fetches: weights do not depend
// on earlier kernels and are streamed before the wait.
#pragma once
#include <cuda_runtime.h>

#include <cstdlib>

namespace pc {

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

inline bool pdl_enabled() {
    static const bool on = [] {
        const char *v = getenv("PICCHIO_PDL");
        return !(v && v[0] == '0');
    }();
    return on;
}

template <typename... KArgs, typename... Args>
cudaError_t launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                     Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace pc
