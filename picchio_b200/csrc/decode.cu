// decode.cu - the persistent batch-1 decode kernel: every layer of
// forward_token (picchio.c:1655-1756), the final norm, the lm_head and the
// greedy argmax, for one or more tokens, in ONE cooperative launch.
//
// A bs1 decode step is ~330 small dependent operations; as separate launches
// each pays a launch hand-off and cold instruction and data caches, together
// far more than the step's ~0.6 ms of weight bytes.  Here one CTA of
// GEMV_THREADS threads runs on every SM for the whole step, and the stages
// are separated by grid barriers (~1.2 us each on B200):
//
//   S1  h = h + combine(previous layer's experts)       (every CTA, whole row)
//       x = rmsnorm(h, input_layernorm)                  (every CTA, in smem)
//       q/k/v GEMV with RoPE and the KV store            (row tiles over CTAs)
//   S2  attention work items (span, KV head)             (items over CTAs)
//   S3  o_proj GEMV, + residual                          (row tiles over CTAs)
//   S4  x = rmsnorm(h, post_attention_layernorm)         (every CTA)
//       router logits                                    (experts over CTAs)
//   S5  top-k + softmax                                  (every CTA, same result)
//       gate_up GEMV of the K experts, clamped SwiGLU    (row tiles over CTAs)
//   S6  down GEMV of the K experts                       (row tiles over CTAs)
//   then combine, final norm, lm_head GEMV with the packed argmax, and CTA 0
//   turns the argmax into the next token.
//
// What every CTA needs whole (norms, combine, top-k) is computed redundantly
// per CTA instead of paying a barrier.  The residual stream alternates between
// two buffers (S1 writes hB from hA, S3 writes hA from hB) so that no CTA
// overwrites values another CTA is still reading.  While a stage runs, each
// CTA asks L2 for the weights of its part of the next dense GEMV.
//
// Every grid-barrier wait is bounded (200 ms); a failure sets the context's
// error word, after which every CTA leaves at its next barrier.
#include <cuda_bf16.h>

#include <algorithm>

#include "attention_core.cuh"
#include "decode.h"
#include "gemv_core.cuh"

namespace pc {

namespace {

constexpr int NTHR = GEMV_THREADS;
constexpr int ATTN_BAR = 15;  // named barrier of the attention items (warps 0-7)
constexpr unsigned long long BARRIER_NS = 200ull * 1000 * 1000;
constexpr int V4MAX = 4;      // float4 per thread in the row helpers: D <= 4 * 4 * NTHR

struct DecState {
    int sel[16];
    float w[16];
    int ok;
    int tok, pos;
};
static_assert(sizeof(DecState) <= 256, "state block");

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void red_release_add_u32(unsigned *p, unsigned v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned long long globaltimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Grid barrier on a monotonically growing counter (zeroed before the launch):
// the g-th barrier completes when the counter reaches g * gridDim.x.  Returns
// false when this or another CTA has failed (error word set): leave.
__device__ __forceinline__ bool grid_sync(unsigned *gbar, int *err, unsigned &gen, DecState *S) {
    __syncthreads();
    ++gen;
    if (threadIdx.x == 0) {
        __threadfence();
        red_release_add_u32(gbar, 1u);
        const unsigned target = gen * gridDim.x;
        const unsigned long long t0 = globaltimer();
        int ok = 1;
        while (ld_acquire_u32(gbar) < target) {
            if (*reinterpret_cast<volatile int *>(err) != 0) { ok = 0; break; }
            if (globaltimer() - t0 > BARRIER_NS) {
                atomicExch(err, 2);
                ok = 0;
                break;
            }
        }
        if (*reinterpret_cast<volatile int *>(err) != 0) ok = 0;
        __threadfence();
        S->ok = ok;
    }
    __syncthreads();
    return S->ok != 0;
}

// L2 prefetch of this CTA's row tiles of a dense GEMV (the unit split of
// gemv_cta), spread over all threads.
__device__ __forceinline__ void prefetch_gemv(const GemvParams &p, int cta, int ncta) {
    const int nj = p.n_inline;
    int U = 0;
    for (int j = 0; j < nj; ++j) U += p.ijobs[j].n_rt;
    const int u0 = (int)((int64_t)U * cta / ncta), u1 = (int)((int64_t)U * (cta + 1) / ncta);
    const int64_t ub = (int64_t)p.kblocks * p.blk_bytes;
    int base = 0;
    for (int j = 0; j < nj; ++j) {
        const int nrt = p.ijobs[j].n_rt;
        const int lo = max(u0, base), hi = min(u1, base + nrt);
        if (lo < hi) {
            const uint8_t *s = p.ijobs[j].tiles + (int64_t)(lo - base) * ub;
            const int64_t n = (int64_t)(hi - lo) * ub;
            for (int64_t o = (int64_t)threadIdx.x * 128; o < n; o += (int64_t)NTHR * 128) prefetch_l2(s + o);
        }
        base += nrt;
    }
}

// *dst (shared memory) = *src, copied by all threads
__device__ __forceinline__ void copy_params(GemvParams *dst, const GemvParams *src) {
    const int n = (int)(sizeof(GemvParams) / 4);
    const uint32_t *s = reinterpret_cast<const uint32_t *>(src);
    uint32_t *d = reinterpret_cast<uint32_t *>(dst);
    for (int i = threadIdx.x; i < n; i += NTHR) d[i] = s[i];
}

// Block-wide sum of one double per thread, in a fixed order.
__device__ __forceinline__ double block_sum_d(double v, double *red) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    double s = 0.0;
    for (int w = 0; w < NTHR / 32; ++w) s += red[w];
    __syncthreads();
    return s;
}

// x <- rmsnorm(x) * w in place, x in shared memory (quant.h:396-402: double
// sum of squares, fp32 scale).  The weights are loaded before the reduction.
__device__ __forceinline__ void rmsnorm_smem(float *x, const float *w, int D, float eps, double *red) {
    const int n4 = D >> 2;
    float4 wv[V4MAX];
    double s = 0.0;
#pragma unroll
    for (int j = 0; j < V4MAX; ++j) {
        const int i = threadIdx.x + j * NTHR;
        wv[j] = i < n4 ? reinterpret_cast<const float4 *>(w)[i] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int j = 0; j < V4MAX; ++j) {
        const int i = threadIdx.x + j * NTHR;
        if (i < n4) {
            const float4 v = reinterpret_cast<const float4 *>(x)[i];
            s += (double)v.x * v.x + (double)v.y * v.y + (double)v.z * v.z + (double)v.w * v.w;
        }
    }
    s = block_sum_d(s, red);
    const float r = __fdiv_rn(1.0f, sqrtf(__fadd_rn((float)(s / D), eps)));
#pragma unroll
    for (int j = 0; j < V4MAX; ++j) {
        const int i = threadIdx.x + j * NTHR;
        if (i < n4) {
            float4 v = reinterpret_cast<float4 *>(x)[i];
            v.x = __fmul_rn(__fmul_rn(v.x, r), wv[j].x);
            v.y = __fmul_rn(__fmul_rn(v.y, r), wv[j].y);
            v.z = __fmul_rn(__fmul_rn(v.z, r), wv[j].z);
            v.w = __fmul_rn(__fmul_rn(v.w, r), wv[j].w);
            reinterpret_cast<float4 *>(x)[i] = v;
        }
    }
    __syncthreads();
}

// embed_token (picchio.c:1472-1503) into shared memory
__device__ __forceinline__ void embed_smem(const DecodeArgs &a, int tok, float *x) {
    const int D = a.D;
    if (tok < 0 || tok >= a.V) {  // picchio.c:1478-1481
        for (int i = threadIdx.x; i < D; i += NTHR) x[i] = 0.0f;
    } else if (a.emb_fmt == TF_T8) {
        const char4 *q = reinterpret_cast<const char4 *>(reinterpret_cast<const int8_t *>(a.emb) + (int64_t)tok * D);
        const float s = a.emb_s[tok];
        char4 v[V4MAX];
#pragma unroll
        for (int j = 0; j < V4MAX; ++j) {
            const int i = threadIdx.x + j * NTHR;
            v[j] = i < (D >> 2) ? q[i] : make_char4(0, 0, 0, 0);
        }
#pragma unroll
        for (int j = 0; j < V4MAX; ++j) {
            const int i = threadIdx.x + j * NTHR;
            if (i < (D >> 2))
                reinterpret_cast<float4 *>(x)[i] = make_float4(__fmul_rn((float)v[j].x, s), __fmul_rn((float)v[j].y, s),
                                                               __fmul_rn((float)v[j].z, s), __fmul_rn((float)v[j].w, s));
        }
    } else if (a.emb_fmt == TF_F32) {
        const float *q = reinterpret_cast<const float *>(a.emb) + (int64_t)tok * D;
        for (int i = threadIdx.x; i < D; i += NTHR) x[i] = q[i];
    } else {  // INT4 rows, picchio.c:1492-1502
        const uint8_t *q = reinterpret_cast<const uint8_t *>(a.emb) + (int64_t)tok * ((D + 1) / 2);
        const int ng = a.emb_gs > 0 ? (D + a.emb_gs - 1) / a.emb_gs : 1;
        const float *sc = a.emb_s + (int64_t)tok * ng;
        for (int i = threadIdx.x; i < D; i += NTHR) {
            const uint8_t b = q[i >> 1];
            const int n = (i & 1) ? (b >> 4) : (b & 0xF);
            x[i] = __fmul_rn((float)(n - 8), sc[a.emb_gs > 0 ? i / a.emb_gs : 0]);
        }
    }
    __syncthreads();
}

// x = hA + sum_k w_k * eo_k, the fma chain in k order (picchio.c:1445-1454):
// the previous layer's MoE residual, every load in flight at once
__device__ __forceinline__ void combine_smem(const DecodeArgs &a, const DecState *S, float *x) {
    const int n4 = a.D >> 2;
    const float4 *h4 = reinterpret_cast<const float4 *>(a.hA);
    float4 acc[V4MAX], hv[V4MAX];
#pragma unroll
    for (int j = 0; j < V4MAX; ++j) {
        const int i = threadIdx.x + j * NTHR;
        acc[j] = make_float4(0.f, 0.f, 0.f, 0.f);
        hv[j] = i < n4 ? __ldcg(h4 + i) : acc[j];
    }
    for (int k0 = 0; k0 < a.K; k0 += 4) {
        float4 e[4][V4MAX];
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
#pragma unroll
            for (int j = 0; j < V4MAX; ++j) {
                const int i = threadIdx.x + j * NTHR;
                e[kk][j] = (k0 + kk < a.K && i < n4)
                               ? __ldcg(reinterpret_cast<const float4 *>(a.eo + (int64_t)(k0 + kk) * a.D) + i)
                               : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
            if (k0 + kk >= a.K) break;
            const float c = __fmul_rn(S->w[k0 + kk], a.routed_scale);
#pragma unroll
            for (int j = 0; j < V4MAX; ++j) {
                acc[j].x = __fmaf_rn(c, e[kk][j].x, acc[j].x);
                acc[j].y = __fmaf_rn(c, e[kk][j].y, acc[j].y);
                acc[j].z = __fmaf_rn(c, e[kk][j].z, acc[j].z);
                acc[j].w = __fmaf_rn(c, e[kk][j].w, acc[j].w);
            }
        }
    }
#pragma unroll
    for (int j = 0; j < V4MAX; ++j) {
        const int i = threadIdx.x + j * NTHR;
        if (i < n4)
            reinterpret_cast<float4 *>(x)[i] = make_float4(__fadd_rn(hv[j].x, acc[j].x), __fadd_rn(hv[j].y, acc[j].y),
                                                           __fadd_rn(hv[j].z, acc[j].z), __fadd_rn(hv[j].w, acc[j].w));
    }
    __syncthreads();
}

// this CTA's share of a row, shared memory -> global
__device__ __forceinline__ void store_slice(const float *x, float *dst, int D, int cta, int ncta) {
    const int c0 = (int)((int64_t)D * cta / ncta), c1 = (int)((int64_t)D * (cta + 1) / ncta);
    for (int i = c0 + threadIdx.x; i < c1; i += NTHR) dst[i] = x[i];
}

// Router logits of experts cta, cta + ncta, ... (picchio.c:1316-1324): the dot
// split over the 12 warps (all 16-byte loads of a lane in flight at once), the
// partials added in a fixed order, the bias last.
__device__ __forceinline__ void router_stage(const DecodeArgs &a, const DecodeLayer &ly, const float *x, float *part,
                                             int cta, int ncta) {
    const int n4 = a.D >> 2, warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = NTHR / 32;
    const int i0 = n4 * warp / nw, i1 = n4 * (warp + 1) / nw;
    for (int e = cta; e < a.E; e += ncta) {
        const float4 *r4 = reinterpret_cast<const float4 *>(ly.router_w + (int64_t)e * a.D);
        float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
        for (int b = i0 + lane; b < i1; b += 32 * V4MAX) {
            float4 rv[V4MAX];
#pragma unroll
            for (int j = 0; j < V4MAX; ++j) rv[j] = b + 32 * j < i1 ? r4[b + 32 * j] : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int j = 0; j < V4MAX; ++j) {
                if (b + 32 * j >= i1) break;
                const float4 xv = reinterpret_cast<const float4 *>(x)[b + 32 * j];
                s0 = __fmaf_rn(xv.x, rv[j].x, s0);
                s1 = __fmaf_rn(xv.y, rv[j].y, s1);
                s2 = __fmaf_rn(xv.z, rv[j].z, s2);
                s3 = __fmaf_rn(xv.w, rv[j].w, s3);
            }
        }
        float s = __fadd_rn(__fadd_rn(s0, s1), __fadd_rn(s2, s3));
        for (int o = 16; o > 0; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
        if (lane == 0) part[warp] = s;
        __syncthreads();
        if (threadIdx.x == 0) {
            float v = 0.0f;
            for (int w = 0; w < nw; ++w) v = __fadd_rn(v, part[w]);
            if (ly.router_b) v = __fadd_rn(v, ly.router_b[e]);  // decode: bias after the dot
            a.rlogits[e] = v;
        }
        __syncthreads();
    }
}

// top-k with strict '>' (ties to the lowest index, picchio.c:1326-1340) and
// softmax over the K logits (quant.h:406-412), by warp 0; result in S
__device__ __forceinline__ void topk_smem(const DecodeArgs &a, DecState *S) {
    const int lane = threadIdx.x & 31;
    if (threadIdx.x < 32) {
        float vals[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            const int e = lane + 32 * q;
            vals[q] = e < a.E ? __ldcg(a.rlogits + e) : -INFINITY;
        }
        float wk[16];
        int sk[16];
        for (int k = 0; k < a.K; ++k) {
            float bv = -1e30f;
            int bi = -1;
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                const int e = lane + 32 * q;
                if (e < a.E && vals[q] > bv) { bv = vals[q]; bi = e; }
            }
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                if (ov > bv || (ov == bv && oi >= 0 && (bi < 0 || oi < bi))) { bv = ov; bi = oi; }
            }
            sk[k < 16 ? k : 15] = bi;
            wk[k < 16 ? k : 15] = bv;
#pragma unroll
            for (int q = 0; q < 8; ++q)
                if (bi >= 0 && bi == lane + 32 * q) vals[q] = -INFINITY;
        }
        if (lane == 0) {
            float mx = -1e30f;
            for (int k = 0; k < a.K; ++k) if (wk[k] > mx) mx = wk[k];
            float sum = 0.0f;
            for (int k = 0; k < a.K; ++k) { wk[k] = expf(__fsub_rn(wk[k], mx)); sum = __fadd_rn(sum, wk[k]); }
            for (int k = 0; k < a.K; ++k) {
                S->sel[k] = sk[k];
                S->w[k] = __fdiv_rn(wk[k], sum);
            }
        }
    }
    __syncthreads();
}

// Inline jobs of the K routed experts in P (gate_up: every job reads x row 0;
// down: expert k reads act row k); out row k either way.
__device__ __forceinline__ void expert_jobs(const DecodeArgs &a, const DecodeLayer &ly, const DecState *S,
                                            GemvParams *P, bool down) {
    if (threadIdx.x < a.K) {
        const int k = threadIdx.x;
        const uint8_t *base = ly.experts + (int64_t)S->sel[k] * a.ex_stride;
        GemvJob &j = P->ijobs[k];
        j.tiles = base + (down ? a.ex_off_dn : a.ex_off_gu);
        const int64_t rs = down ? a.ex_off_dn_rs : a.ex_off_gu_rs, b = down ? a.ex_off_dn_b : a.ex_off_gu_b;
        j.rs = rs >= 0 ? reinterpret_cast<const float *>(base + rs) : nullptr;
        j.bias = b >= 0 ? reinterpret_cast<const float *>(base + b) : nullptr;
        j.n_rt = down ? a.dn_rt : a.gu_rt;
        j.O = down ? a.dn_O : a.gu_O;
        j.nrows = 1;
        j.seg = 0;
        j.in_row[0] = down ? k : 0;
        j.out_row[0] = k;
    }
    if (threadIdx.x == 0) P->n_inline = a.K;
    __syncthreads();
}

// Stage kinds of one step, in order: per layer S1..S6, then the head.
enum StageKind { ST_QKV = 0, ST_ATTN, ST_O, ST_ROUTER, ST_GATE_UP, ST_DOWN, ST_HEAD };

// Prepares stage `kind` of layer l (everything but its GEMV / attention work).
__device__ __noinline__ void stage_prepare(const DecodeArgs *a, int kind, int l, DecState *S, float *x, GemvParams *P,
                                           double *dred, float *fred, int cta, int ncta) {
    const DecodeLayer *ly = a->layers + (l < a->L ? l : 0);
    switch (kind) {
        case ST_QKV:
            if (l > 0) combine_smem(*a, S, x);
            store_slice(x, a->hB, a->D, cta, ncta);
            rmsnorm_smem(x, ly->in_ln, a->D, a->eps, dred);
            copy_params(P, &ly->qkv);
            __syncthreads();
            if (threadIdx.x == 0) P->x = x;
            __syncthreads();
            break;
        case ST_O:
            copy_params(P, &ly->o);
            __syncthreads();
            break;
        case ST_ROUTER: {
            const int n4 = a->D >> 2;
            for (int i = threadIdx.x; i < n4; i += NTHR)
                reinterpret_cast<float4 *>(x)[i] = __ldcg(reinterpret_cast<const float4 *>(a->hA) + i);
            __syncthreads();
            rmsnorm_smem(x, ly->post_ln, a->D, a->eps, dred);
            router_stage(*a, *ly, x, fred, cta, ncta);
            break;
        }
        case ST_GATE_UP:
        case ST_DOWN: {
            const bool down = kind == ST_DOWN;
            if (!down) topk_smem(*a, S);
            copy_params(P, down ? &a->blocks->dn : &a->blocks->gu);
            __syncthreads();
            expert_jobs(*a, *ly, S, P, down);
            if (!down && threadIdx.x == 0) P->x = x;
            __syncthreads();
            break;
        }
        case ST_HEAD:
            combine_smem(*a, S, x);
            store_slice(x, a->hB, a->D, cta, ncta);
            rmsnorm_smem(x, a->final_norm, a->D, a->eps, dred);
            copy_params(P, &a->blocks->lm);
            __syncthreads();
            if (threadIdx.x == 0) P->x = x;
            __syncthreads();
            break;
        default:
            break;
    }
}

// L2 prefetch for what follows stage `kind` of layer l: the o_proj tiles
// during attention, the next layer's q/k/v tiles after o_proj.
__device__ __noinline__ void stage_prefetch(const DecodeArgs *a, int kind, int l, int cta, int ncta) {
    if (kind == ST_QKV) prefetch_gemv(a->layers[l].o, cta, ncta);
    else if (kind == ST_O && l + 1 < a->L) prefetch_gemv(a->layers[l + 1].qkv, cta, ncta);
}

template <int HD, typename KVT>
__device__ __noinline__ void stage_attention(const AttnParams *src, int pos, uint8_t *work, int cta, int ncta) {
    if (threadIdx.x >= ATTN_SPLIT) return;  // warps 0-7
    AttnParams at = *src;
    const int end = pos < at.ctx ? pos : at.ctx - 1;
    const int start = at.window > 0 ? max(0, end - at.window + 1) : 0;
    at.nsplit = (end - start + ATTN_SPLIT) / ATTN_SPLIT;
    const int items = at.nsplit * at.KVH;
    AttnSmem<HD> &sm = *reinterpret_cast<AttnSmem<HD> *>(work);
    for (int it = cta; it < items; it += ncta) attn_item<KVT, HD>(at, it % at.nsplit, it / at.nsplit, 0, sm, ATTN_BAR);
}

__device__ __noinline__ void stage_embed(const DecodeArgs *a, int tok, float *x) { embed_smem(*a, tok, x); }

// One loop over the stages of every step, so that each GEMV instance (INT8
// dense, INT4 experts) is inlined once into the kernel.
template <int HD, typename KVT, int EGS>
__global__ void __launch_bounds__(NTHR, 1) decode_kernel(const DecodeArgs args, int nsteps) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int cta = blockIdx.x, ncta = gridDim.x, D = args.D;
    float *x = reinterpret_cast<float *>(smem);
    DecState *S = reinterpret_cast<DecState *>(smem + decode_off_s(D));
    double *dred = reinterpret_cast<double *>(smem + decode_off_s(D) + 256);
    float *fred = reinterpret_cast<float *>(smem + decode_off_s(D) + 384);
    DecodeArgs *a = reinterpret_cast<DecodeArgs *>(smem + decode_off_s(D) + 512);
    GemvParams *P = reinterpret_cast<GemvParams *>(smem + decode_off_p(D));
    uint8_t *work = smem + decode_off_w(D);
    if (threadIdx.x == 0) {
        *a = args;
        S->tok = __ldcg(args.d_tok);
        S->pos = __ldcg(args.d_pos);
    }
    __syncthreads();
    const int per_step = 6 * args.L + 1;
    unsigned gen = 0;
    int step = 0, l = 0, kind = ST_QKV;
    for (int st = 0; st < nsteps * per_step; ++st) {
        if (st % per_step == 0) {
            step = st / per_step;
            l = 0;
            kind = ST_QKV;
            stage_embed(a, S->tok, x);
        }
        stage_prepare(a, kind, l, S, x, P, dred, fred, cta, ncta);
        if (kind == ST_QKV || kind == ST_O || kind == ST_HEAD) {
            gemv_cta<TF_T8, 1, 0, false>(*P, work, cta, ncta);
        } else if (kind == ST_GATE_UP || kind == ST_DOWN) {
            gemv_cta<TF_T4, 1, EGS, false>(*P, work, cta, ncta);
        } else if (kind == ST_ATTN) {
            stage_attention<HD, KVT>(&args.layers[l].attn, S->pos, work, cta, ncta);
        }
        stage_prefetch(a, kind, l, cta, ncta);
        if (!grid_sync(args.gbar, args.err, gen, S)) return;
        if (kind == ST_HEAD) {
            // the next token (first maximum wins, picchio.c:1555-1561)
            const int pos = S->pos;
            if (cta == 0 && threadIdx.x == 0) {
                const unsigned long long v = __ldcg(args.argmax);
                const int id = v ? (int)(0xFFFFFFFFu - (uint32_t)(v & 0xFFFFFFFFull)) : 0;
                *args.argmax = 0ull;
                args.d_next[0] = id;
                if (args.d_gen) args.d_gen[step] = id;
                args.d_tok[0] = id;
                args.d_pos[0] = pos + 1;
            }
            if (step + 1 < nsteps) {
                if (!grid_sync(args.gbar, args.err, gen, S)) return;
                if (threadIdx.x == 0) {
                    S->tok = __ldcg(args.d_tok);
                    S->pos = pos + 1;
                }
                __syncthreads();
            }
        } else if (kind == ST_DOWN) {
            ++l;
            kind = l < args.L ? ST_QKV : ST_HEAD;
        } else {
            ++kind;
        }
    }
}

template <int HD, typename KVT, int EGS>
cudaError_t launch_t(const DecodeArgs &a, int nsteps, int ncta, size_t smem, cudaStream_t st) {
    void *args[] = {const_cast<DecodeArgs *>(&a), &nsteps};
    return cudaLaunchCooperativeKernel((const void *)decode_kernel<HD, KVT, EGS>, dim3(ncta), dim3(NTHR), args, smem,
                                       st);
}

template <int HD, typename KVT, int EGS>
cudaError_t set_t(int max_smem) {
    return cudaFuncSetAttribute(decode_kernel<HD, KVT, EGS>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
}

}  // namespace

cudaError_t decode_configure(int max_smem) {
    cudaError_t e = cudaSuccess;
#define PC_SET(HD, T, G) if (e == cudaSuccess) e = set_t<HD, T, G>(max_smem)
    PC_SET(64, float, 32); PC_SET(64, __nv_bfloat16, 32); PC_SET(64, float, 64); PC_SET(64, __nv_bfloat16, 64);
    PC_SET(32, float, 32); PC_SET(32, __nv_bfloat16, 32);
#undef PC_SET
    return e;
}

bool decode_supported(int hd, int egs) { return (hd == 64 && (egs == 32 || egs == 64)) || (hd == 32 && egs == 32); }

size_t decode_smem_bytes(int D, int gemv_need) {
    return (size_t)decode_off_w(D) + (size_t)std::max(gemv_need, (int)sizeof(AttnSmem<64>));
}

cudaError_t decode_launch(const DecodeArgs &a, int hd, int kv_bf16, int egs, int nsteps, int ncta, size_t smem,
                          cudaStream_t st) {
    if (hd == 64 && egs == 32)
        return kv_bf16 ? launch_t<64, __nv_bfloat16, 32>(a, nsteps, ncta, smem, st)
                       : launch_t<64, float, 32>(a, nsteps, ncta, smem, st);
    if (hd == 64 && egs == 64)
        return kv_bf16 ? launch_t<64, __nv_bfloat16, 64>(a, nsteps, ncta, smem, st)
                       : launch_t<64, float, 64>(a, nsteps, ncta, smem, st);
    if (hd == 32 && egs == 32)
        return kv_bf16 ? launch_t<32, __nv_bfloat16, 32>(a, nsteps, ncta, smem, st)
                       : launch_t<32, float, 32>(a, nsteps, ncta, smem, st);
    return cudaErrorInvalidValue;
}

}  // namespace pc
