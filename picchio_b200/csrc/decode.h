// decode.h - host interface of the persistent batch-1 decode kernel
// (decode.cu).
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

#include "kernels.h"
#include "layout.h"

namespace pc {

// Per layer, in device memory: the two dense GEMVs with their job tables and
// epilogue fields filled in, and the attention parameters (nsplit is set per
// step inside the kernel).
struct DecodeLayer {
    GemvParams qkv;  // x set per CTA to its shared-memory row
    GemvParams o;    // x = attention output, y = hA, res_src = hB
    AttnParams attn;
    const float *in_ln, *post_ln;
    const float *router_w, *router_b;
    const uint8_t *experts;  // the layer's expert table
};

// Parameter blocks too large for the kernel's parameter space, in device
// memory.
struct DecodeBlocks {
    GemvParams gu, dn, lm;  // expert GEMV templates (jobs filled per layer), lm_head
};

// The kernel parameter.
struct DecodeArgs {
    const DecodeLayer *layers;
    const DecodeBlocks *blocks;
    int L, D, E, K, V;
    float eps, routed_scale;
    // embedding (picchio.c:1472-1503)
    int emb_fmt, emb_gs;
    const void *emb;
    const float *emb_s;
    const float *final_norm;
    // expert table geometry
    int64_t ex_stride, ex_off_gu, ex_off_dn, ex_off_gu_rs, ex_off_dn_rs, ex_off_gu_b, ex_off_dn_b;
    int gu_rt, dn_rt, gu_O, dn_O;
    // step buffers
    float *hA, *hB;             // residual stream, alternating (see decode.cu)
    float *eo, *rlogits;        // [K][D] expert outputs, [E] router logits
    unsigned long long *argmax; // packed lm_head argmax, zero between steps
    int *d_tok, *d_pos, *d_next, *d_gen;
    unsigned *gbar;             // grid barrier counter, zeroed before each launch
    int *err;                   // device error word
};

// Shared-memory layout of the kernel for row length D: the row, a small state
// block and a copy of the arguments, one GEMV parameter block, then the GEMV /
// attention work area.
__host__ __device__ inline int decode_off_s(int D) { return (D * 4 + 127) & ~127; }
__host__ __device__ inline int decode_off_p(int D) {
    return (decode_off_s(D) + 512 + (int)sizeof(DecodeArgs) + 127) & ~127;
}
__host__ __device__ inline int decode_off_w(int D) {
    return (decode_off_p(D) + (int)sizeof(GemvParams) + 127) & ~127;
}

cudaError_t decode_configure(int max_smem);
// Instantiated for INT8 dense weights and INT4 experts with head_dim 64
// (expert group size 32 or 64) or head_dim 32 (group size 32).
bool decode_supported(int head_dim, int expert_gs);
// Dynamic shared memory for row length D and the largest GEMV work area.
size_t decode_smem_bytes(int D, int gemv_need);
// nsteps greedy tokens in one cooperative launch of ncta CTAs (one per SM).
cudaError_t decode_launch(const DecodeArgs &a, int head_dim, int kv_bf16, int expert_gs, int nsteps, int ncta,
                          size_t smem, cudaStream_t st);

}  // namespace pc
