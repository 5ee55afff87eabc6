// attention.cu - the decode attention launch: one CTA of 256 threads per
// work item (attention_core.cuh), grid (spans, KV heads, rows).
#include "attention_core.cuh"
#include "launch.cuh"

namespace pc {

namespace {

template <typename T, int HD>
__global__ void __launch_bounds__(NT) attn_kernel(const AttnParams a) {
    pdl_trigger();
    __shared__ AttnSmem<HD> sm;
    attn_item<T, HD, true>(a, blockIdx.x, blockIdx.y, blockIdx.z, sm, 0);  // waits inside
}

template <typename T>
cudaError_t launch_hd(const AttnParams &a, dim3 grid, cudaStream_t st) {
    switch (a.hd) {
        case 16: return launch_k(attn_kernel<T, 16>, grid, dim3(NT), 0, st, a);
        case 32: return launch_k(attn_kernel<T, 32>, grid, dim3(NT), 0, st, a);
        case 64: return launch_k(attn_kernel<T, 64>, grid, dim3(NT), 0, st, a);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace

cudaError_t launch_attention(const AttnParams &a, cudaStream_t st) {
    if (a.H / a.KVH > MAXG || a.nsplit > 64) return cudaErrorInvalidValue;
    if (attention_tc_ok(a)) return launch_attention_tc(a, st);
    dim3 grid(a.nsplit, a.KVH, a.M);
    return a.kv_bf16 ? launch_hd<__nv_bfloat16>(a, grid, st) : launch_hd<float>(a, grid, st);
}

}  // namespace pc
