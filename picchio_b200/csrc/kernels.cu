// kernels.cu - the per-step kernels around the dequant GEMV: embedding,
// RMSNorm, decode attention with sinks and sliding window, router + top-k +
// expert job tables, weighted expert combine, fp32 GEMV, greedy argmax.
//
// This library is compiled with -fmad=false: every fused multiply-add below
// is an explicit __fmaf_rn, written where the reference's own build fuses
// (see oracle/oracle.c), so products and sums round as the reference's do.
#include <cuda_bf16.h>

#include <cfloat>

#include "kernels.h"
#include "launch.cuh"

namespace pc {

namespace {

__device__ __forceinline__ float ldf(const void *base, int64_t i, int bf16) {
    return bf16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(base)[i])
                : reinterpret_cast<const float *>(base)[i];
}

__device__ __forceinline__ void stf(void *base, int64_t i, float v, int bf16) {
    if (bf16)
        reinterpret_cast<__nv_bfloat16 *>(base)[i] = __float2bfloat16_rn(v);
    else
        reinterpret_cast<float *>(base)[i] = v;
}

// ---------------------------------------------------------------- embed ----
__global__ void embed_kernel(int fmt, const void *table, const float *scales, int gs, int V, int D,
                             const int *tok, float *h) {
    pdl_wait();
    pdl_trigger();
    const int m = blockIdx.x;
    const int t = tok[m];
    float *out = h + (int64_t)m * D;
    if (t < 0 || t >= V) {  // picchio.c:1478-1481
        for (int i = threadIdx.x; i < D; i += blockDim.x) out[i] = 0.0f;
        return;
    }
    if (fmt == TF_T8) {
        const int8_t *q = reinterpret_cast<const int8_t *>(table) + (int64_t)t * D;
        const float s = scales[t];
        for (int i = threadIdx.x; i < D; i += blockDim.x) out[i] = __fmul_rn((float)q[i], s);
    } else if (fmt == TF_F32) {
        const float *q = reinterpret_cast<const float *>(table) + (int64_t)t * D;
        for (int i = threadIdx.x; i < D; i += blockDim.x) out[i] = q[i];
    } else {  // INT4 rows, picchio.c:1492-1502
        const uint8_t *q = reinterpret_cast<const uint8_t *>(table) + (int64_t)t * ((D + 1) / 2);
        const int ng = gs > 0 ? (D + gs - 1) / gs : 1;
        const float *sc = scales + (int64_t)t * ng;
        for (int i = threadIdx.x; i < D; i += blockDim.x) {
            const uint8_t b = q[i >> 1];
            const int n = (i & 1) ? (b >> 4) : (b & 0xF);
            out[i] = __fmul_rn((float)(n - 8), sc[gs > 0 ? i / gs : 0]);
        }
    }
}

// -------------------------------------------------------------- rmsnorm ----
// One block per row.  On B200 an L2 round trip costs ~0.7 us, so every
// thread issues all of its loads (x and w, 16 bytes each) before using any:
// one round trip in, one out.
constexpr int NORM_THREADS = 256, NORM_V4 = 4;  // up to 4 float4 per thread (D <= 4096)

// 1/sqrt(mean + eps) of a row from each thread's partial sum of squares.
// The sum is taken in double, as quant.h:396-402 accumulates it; the
// per-thread element order is the same wherever this is used, so fused and
// unfused norms of one row agree bit for bit.
__device__ float norm_scale(double s, int D, float eps) {
    __shared__ double red[NORM_THREADS / 32];
    __shared__ float rs;
    const int tid = threadIdx.x;
    for (int q = 16; q > 0; q >>= 1) s += __shfl_xor_sync(0xffffffffu, s, q);
    if ((tid & 31) == 0) red[tid >> 5] = s;
    __syncthreads();
    if (tid < 32) {
        double v = tid < NORM_THREADS / 32 ? red[tid] : 0.0;
        for (int q = 16; q > 0; q >>= 1) v += __shfl_xor_sync(0xffffffffu, v, q);
        if (tid == 0) rs = __fdiv_rn(1.0f, sqrtf(__fadd_rn((float)(v / D), eps)));
    }
    __syncthreads();
    return rs;
}

__global__ void __launch_bounds__(NORM_THREADS) rmsnorm_kernel(const float *x, const float *w, float *out, int D,
                                                                float eps) {
    pdl_wait();
    pdl_trigger();
    const int m = blockIdx.x, tid = threadIdx.x;
    const float *xr = x + (int64_t)m * D;
    float *o = out + (int64_t)m * D;
    double s = 0.0;
    const bool vec = (D & 3) == 0 && D <= 4 * NORM_V4 * NORM_THREADS;
    float4 xv[NORM_V4], wv[NORM_V4];
    if (vec) {
        const int n4 = D >> 2;
#pragma unroll
        for (int j = 0; j < NORM_V4; ++j) {
            const int i = tid + j * NORM_THREADS;
            xv[j] = i < n4 ? reinterpret_cast<const float4 *>(xr)[i] : make_float4(0.f, 0.f, 0.f, 0.f);
            wv[j] = i < n4 ? reinterpret_cast<const float4 *>(w)[i] : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int j = 0; j < NORM_V4; ++j)
            s += (double)xv[j].x * xv[j].x + (double)xv[j].y * xv[j].y + (double)xv[j].z * xv[j].z +
                 (double)xv[j].w * xv[j].w;
    } else {
        for (int i = tid; i < D; i += NORM_THREADS) s += (double)xr[i] * (double)xr[i];
    }
    const float r = norm_scale(s, D, eps);
    if (vec) {
        const int n4 = D >> 2;
#pragma unroll
        for (int j = 0; j < NORM_V4; ++j) {
            const int i = tid + j * NORM_THREADS;
            if (i < n4)
                reinterpret_cast<float4 *>(o)[i] =
                    make_float4(__fmul_rn(__fmul_rn(xv[j].x, r), wv[j].x), __fmul_rn(__fmul_rn(xv[j].y, r), wv[j].y),
                                __fmul_rn(__fmul_rn(xv[j].z, r), wv[j].z), __fmul_rn(__fmul_rn(xv[j].w, r), wv[j].w));
        }
    } else {
        for (int i = tid; i < D; i += NORM_THREADS) o[i] = __fmul_rn(__fmul_rn(xr[i], r), w[i]);
    }
}

// --------------------------------------------------------------- router ----
// Dot products: four warps per expert (two experts and up to ROUTER_ROWS
// input rows per block, rows spread over blockIdx.y), each lane
// with all of its 16-byte loads of R and x in flight at once; the quarters
// are added in a fixed order.  The last block to finish (atomic ticket) does
// the top-k, the softmax and the expert job tables, reading the selection
// from shared memory.
// The expert job tables (and, with pair_start, the expert-sorted pair
// lists) from the selection in ssel[0..P): pairs grouped by expert in
// ascending pair order, at most per_job pairs per job.  Run by the 256
// threads of the block that finishes the routing: a shared-memory histogram
// of pairs per expert, scans, one warp placing the pairs 32 at a time (ranks
// within a step from match-any groups), then one thread per expert filling
// its jobs.  sorted: shared scratch of ROUTER_MAX_PAIRS ints.
__device__ void router_jobs(const RouterParams &r, const int *ssel, int P, int *cnt, int *jstart, int *pstart,
                            int *sorted) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
    const int Ps = min(P, ROUTER_MAX_PAIRS);
    const int pj = (r.per_job > 0 && r.per_job < GEMV_MAXR) ? r.per_job : GEMV_MAXR;
    const int e = tid;
    pstart[e] = 0;
    __syncthreads();
    for (int p = tid; p < Ps; p += blockDim.x) {
        const int ep = ssel[p];
        const bool loc = ep >= r.e_lo && ep < r.e_hi;
        r.pair_local[p] = loc ? 1 : 0;
        if (loc) atomicAdd(&pstart[ep], 1);
    }
    __syncthreads();
    const int n = e < r.E ? pstart[e] : 0;  // pairs of local expert e
    cnt[e] = (n + pj - 1) / pj;
    __syncthreads();
    if (warp == 1) {  // exclusive scan of pairs per expert: 8 experts per lane
        int v[8], tot = 0;
#pragma unroll
        for (int q = 0; q < 8; ++q) { v[q] = tot; tot += pstart[lane * 8 + q]; }
        int inc = tot;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int nn = __shfl_up_sync(0xffffffffu, inc, o);
            if (lane >= o) inc += nn;
        }
        const int base = inc - tot;
        __syncwarp();
#pragma unroll
        for (int q = 0; q < 8; ++q) pstart[lane * 8 + q] = base + v[q];
        if (lane == 31) pstart[256] = inc;
    }
    if (warp == 0) {  // exclusive scan of jobs per expert
        int v[8], tot = 0;
#pragma unroll
        for (int q = 0; q < 8; ++q) { v[q] = tot; tot += cnt[lane * 8 + q]; }
        int inc = tot;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int nn = __shfl_up_sync(0xffffffffu, inc, o);
            if (lane >= o) inc += nn;
        }
        const int base = inc - tot;
#pragma unroll
        for (int q = 0; q < 8; ++q) jstart[lane * 8 + q] = base + v[q];
        if (lane == 31) {
            jstart[256] = inc;
            r.njobs[0] = r.njobs[1] = min(inc, GEMV_MAX_JOBS);
        }
    }
    __syncthreads();
    if (warp == 0) {  // stable placement; cnt becomes the running offset per expert
#pragma unroll
        for (int q = 0; q < 8; ++q) cnt[lane * 8 + q] = 0;
        __syncwarp();
        for (int b = 0; b < Ps; b += 32) {
            const int p = b + lane;
            const int ep = p < Ps ? ssel[p] : -1;
            const bool loc = ep >= r.e_lo && ep < r.e_hi;
            const unsigned grp = __match_any_sync(0xffffffffu, loc ? ep : -1);
            int off = 0;
            if (loc) {
                off = cnt[ep];
                sorted[pstart[ep] + off + __popc(grp & ((1u << lane) - 1u))] = p;
            }
            __syncwarp();
            if (loc && lane == 31 - __clz(grp)) cnt[ep] = off + __popc(grp);
            __syncwarp();
        }
    }
    __syncthreads();
    if (r.pair_start) {
        if (e < r.E) r.pair_start[e] = pstart[e];
        if (e == 0) r.pair_start[r.E] = pstart[256];
        for (int q = tid; q < pstart[256]; q += blockDim.x) r.pair_list[q] = sorted[q];
    }
    if (n == 0) return;
    if (r.used) r.used[e] = 1;
    const uint8_t *base = r.emap ? r.emap[e] : r.table + (int64_t)(e - r.e_lo) * r.stride;
    const int *mine = sorted + pstart[e];
    for (int k = 0; k * pj < n; ++k) {
        const int j = jstart[e] + k;
        if (j >= GEMV_MAX_JOBS) break;
        const int fill = min(pj, n - k * pj);
        GemvJob &gu = r.jobs_gu[j];
        GemvJob &dn = r.jobs_dn[j];
        gu.tiles = base + r.off_gu;
        gu.rs = r.off_gu_rs >= 0 ? reinterpret_cast<const float *>(base + r.off_gu_rs) : nullptr;
        gu.bias = r.off_gu_b >= 0 ? reinterpret_cast<const float *>(base + r.off_gu_b) : nullptr;
        gu.n_rt = r.gu_rt; gu.O = r.gu_O; gu.seg = 0;
        dn.tiles = base + r.off_dn;
        dn.rs = r.off_dn_rs >= 0 ? reinterpret_cast<const float *>(base + r.off_dn_rs) : nullptr;
        dn.bias = r.off_dn_b >= 0 ? reinterpret_cast<const float *>(base + r.off_dn_b) : nullptr;
        dn.n_rt = r.dn_rt; dn.O = r.dn_O; dn.seg = 0;
        for (int f = 0; f < fill; ++f) {
            const int p = mine[k * pj + f];
            gu.in_row[f] = p / r.K;
            gu.out_row[f] = p;
            dn.in_row[f] = p;
            dn.out_row[f] = p;
        }
        gu.nrows = dn.nrows = fill;
    }
}

// Top-k of row m from its E logits lg (global memory: read past L1; else
// shared memory), one warp: K rounds of strict '>' argmax, ties to the lowest
// index (picchio.c:1330-1340), then the softmax over the K selected logits
// (quant.h:406-412).  Writes sel and w (and ssel when not null).
template <bool GLOBAL>
__device__ void router_topk_row(const RouterParams &r, const float *lg, int m, int *ssel) {
    const int lane = threadIdx.x & 31;
    float vals[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
        const int e = lane + 32 * q;
        vals[q] = e < r.E ? (GLOBAL ? __ldcg(lg + e) : lg[e]) : -INFINITY;
    }
    float wk[16];
    int sk[16];
    for (int k = 0; k < r.K; ++k) {
        float bv = -1e30f;
        int bi = -1;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            const int e = lane + 32 * q;
            if (e < r.E && vals[q] > bv) { bv = vals[q]; bi = e; }
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
        for (int k = 0; k < r.K; ++k) if (wk[k] > mx) mx = wk[k];
        float sum = 0.0f;
        for (int k = 0; k < r.K; ++k) { wk[k] = expf(__fsub_rn(wk[k], mx)); sum = __fadd_rn(sum, wk[k]); }
        for (int k = 0; k < r.K; ++k) {
            r.sel[m * r.K + k] = sk[k];
            if (ssel && m * r.K + k < ROUTER_MAX_PAIRS) ssel[m * r.K + k] = sk[k];
            r.w[m * r.K + k] = __fdiv_rn(wk[k], sum);
        }
    }
}

constexpr int ROUTER_RV = 6;    // float4 per lane per operand in flight
constexpr int ROUTER_ROWS = 2;  // input rows per block (blockIdx.y = row group)

__global__ void __launch_bounds__(256) router_kernel(const RouterParams r) {
    __shared__ bool last;
    __shared__ float part[8];
    __shared__ int cnt[256], jstart[257], pstart[257];
    __shared__ int ssel[ROUTER_MAX_PAIRS], sorted[ROUTER_MAX_PAIRS];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int P = r.M * r.K;
    // R does not depend on earlier kernels: when a quarter of D is one pass of
    // the lanes (D <= 3072), this lane's part of its expert row is loaded
    // before the dependency wait, once for all rows of the block
    const int n4p = r.D >> 2, ep = blockIdx.x * 2 + (warp >> 2), qp = warp & 3;
    const bool rpre_on = !r.sel_in && (r.D & 3) == 0 && ep < r.E && (n4p + 3) / 4 <= 32 * ROUTER_RV;
    float4 rpre[ROUTER_RV];
    if (rpre_on) {
        const int i0 = n4p * qp / 4, i1 = n4p * (qp + 1) / 4;
        const float4 *r4 = reinterpret_cast<const float4 *>(r.R + (int64_t)ep * r.D);
#pragma unroll
        for (int j = 0; j < ROUTER_RV; ++j) {
            const int i = i0 + lane + 32 * j;
            rpre[j] = i < i1 ? r4[i] : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
    pdl_wait();
    pdl_trigger();
    if (!r.sel_in) {
        const int e = blockIdx.x * 2 + (warp >> 2), q = warp & 3;
        const bool vec = (r.D & 3) == 0;
        const int m1 = min(r.M, (int)(blockIdx.y + 1) * ROUTER_ROWS);
        const bool fused = r.ln_w != nullptr;
        for (int m = blockIdx.y * ROUTER_ROWS; m < m1; ++m) {
            float rn = 1.0f;
            if (fused) {  // the input norm of this row, as rmsnorm_kernel computes it
                const int n4 = r.D >> 2;
                const float4 *h4 = reinterpret_cast<const float4 *>(r.h_in + (int64_t)m * r.D);
                const float4 *w4 = reinterpret_cast<const float4 *>(r.ln_w);
                float4 hv[NORM_V4];
                double ss = 0.0;
#pragma unroll
                for (int j = 0; j < NORM_V4; ++j) {
                    const int i = threadIdx.x + j * NORM_THREADS;
                    hv[j] = i < n4 ? h4[i] : make_float4(0.f, 0.f, 0.f, 0.f);
                    ss += (double)hv[j].x * hv[j].x + (double)hv[j].y * hv[j].y + (double)hv[j].z * hv[j].z +
                          (double)hv[j].w * hv[j].w;
                }
                rn = norm_scale(ss, r.D, r.eps);
                if (blockIdx.x == 0) {
                    float4 *o4 = reinterpret_cast<float4 *>(r.hn_out + (int64_t)m * r.D);
#pragma unroll
                    for (int j = 0; j < NORM_V4; ++j) {
                        const int i = threadIdx.x + j * NORM_THREADS;
                        if (i < n4) {
                            const float4 w = w4[i];
                            o4[i] = make_float4(__fmul_rn(__fmul_rn(hv[j].x, rn), w.x), __fmul_rn(__fmul_rn(hv[j].y, rn), w.y),
                                                __fmul_rn(__fmul_rn(hv[j].z, rn), w.z), __fmul_rn(__fmul_rn(hv[j].w, rn), w.w));
                        }
                    }
                }
            }
            float s = 0.0f;
            if (e < r.E) {
                const float *re = r.R + (int64_t)e * r.D;
                const float *xr = fused ? r.h_in + (int64_t)m * r.D : r.x + (int64_t)m * r.D;
                if (vec) {
                    const int n4 = r.D >> 2, i0 = n4 * q / 4, i1 = n4 * (q + 1) / 4;
                    const float4 *r4 = reinterpret_cast<const float4 *>(re);
                    const float4 *x4 = reinterpret_cast<const float4 *>(xr);
                    const float4 *w4 = reinterpret_cast<const float4 *>(r.ln_w);
                    float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
                    for (int base = i0 + lane; base < i1; base += 32 * ROUTER_RV) {
                        float4 rv[ROUTER_RV], xv[ROUTER_RV];
#pragma unroll
                        for (int j = 0; j < ROUTER_RV; ++j) {
                            const int i = base + 32 * j;
                            rv[j] = rpre_on ? rpre[j] : (i < i1 ? r4[i] : make_float4(0.f, 0.f, 0.f, 0.f));
                            xv[j] = i < i1 ? x4[i] : make_float4(0.f, 0.f, 0.f, 0.f);
                        }
                        if (fused) {
#pragma unroll
                            for (int j = 0; j < ROUTER_RV; ++j) {
                                const int i = base + 32 * j;
                                const float4 w = i < i1 ? w4[i] : make_float4(0.f, 0.f, 0.f, 0.f);
                                xv[j] = make_float4(__fmul_rn(__fmul_rn(xv[j].x, rn), w.x),
                                                    __fmul_rn(__fmul_rn(xv[j].y, rn), w.y),
                                                    __fmul_rn(__fmul_rn(xv[j].z, rn), w.z),
                                                    __fmul_rn(__fmul_rn(xv[j].w, rn), w.w));
                            }
                        }
#pragma unroll
                        for (int j = 0; j < ROUTER_RV; ++j) {
                            s0 = __fmaf_rn(xv[j].x, rv[j].x, s0);
                            s1 = __fmaf_rn(xv[j].y, rv[j].y, s1);
                            s2 = __fmaf_rn(xv[j].z, rv[j].z, s2);
                            s3 = __fmaf_rn(xv[j].w, rv[j].w, s3);
                        }
                    }
                    s = __fadd_rn(__fadd_rn(s0, s1), __fadd_rn(s2, s3));
                } else {
                    const int i0 = r.D * q / 4, i1 = r.D * (q + 1) / 4;
                    for (int i = i0 + lane; i < i1; i += 32) s = __fmaf_rn(xr[i], re[i], s);
                }
            }
            for (int o = 16; o > 0; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
            if (lane == 0) part[warp] = s;
            __syncthreads();
            if (threadIdx.x < 2) {
                const int ee = blockIdx.x * 2 + threadIdx.x;
                if (ee < r.E) {
                    const float *pp = part + 4 * threadIdx.x;
                    float v = __fadd_rn(__fadd_rn(pp[0], pp[1]), __fadd_rn(pp[2], pp[3]));
                    // decode adds the bias after the dot, prefill starts from it;
                    // with a parallel dot both become one final add.
                    if (r.bias) v = r.bias_first ? __fadd_rn(r.bias[ee], v) : __fadd_rn(v, r.bias[ee]);
                    r.logits[(int64_t)m * r.E + ee] = v;
                }
            }
            __syncthreads();
        }
        __threadfence();
        if (threadIdx.x == 0) {
            last = atomicAdd(r.counter, 1u) == gridDim.x * gridDim.y - 1;
            if (last) *r.counter = 0u;
        }
        __syncthreads();
        if (!last) return;
        __threadfence();
        // top-k, K rounds of strict '>' argmax; ties -> lowest index
        for (int m = warp; m < r.M; m += 8) router_topk_row<true>(r, r.logits + (int64_t)m * r.E, m, ssel);
        __syncthreads();
    } else {
        if (blockIdx.x != 0) return;
        for (int i = threadIdx.x; i < P; i += blockDim.x) {
            const int v = r.sel_in[i];
            r.sel[i] = v;
            if (i < ROUTER_MAX_PAIRS) ssel[i] = v;
            r.w[i] = r.w_in[i];
        }
        __syncthreads();
    }
    router_jobs(r, ssel, P, cnt, jstart, pstart, sorted);
}

// Many rows (batched decode, prefill): one block per RB rows instead.  The
// block normalises its rows once into shared memory (rmsnorm_kernel's
// arithmetic), then warp w takes experts w, w + 8, ... and forms each
// (row, expert) dot exactly as router_kernel does (four quarters of D, lanes
// strided by 32 float4 with four component sums, the same shuffle tree, the
// quarters added as (q0 + q1) + (q2 + q3)), so the logits are bit-identical;
// the next quarter's R loads are in flight while a quarter is summed.  Below
// 256 rows the experts are split over blockIdx.y (ROUTER_EPB per block); the
// last expert block of a row block (ticket) takes those rows' top-k, and the
// last row block the job tables.  D % 4 == 0 and one 32 x ROUTER_RV float4 pass per quarter
// (D <= 3072).
constexpr int ROUTER_RB_MIN_ROWS = 16;  // from this many rows the row-block form is used
constexpr int ROUTER_EPB = 16;          // experts per block of the row-block form (blockIdx.y)

// Row-block router helpers: R of task t ((expert warp + 8 (t / 4), quarter
// t % 4)) into registers, and the task's dots for the block's RB rows.
__device__ __forceinline__ void rr_load(const RouterParams &r, int n4, int ebase, int warp, int lane, int t,
                                        float4 (&rv)[ROUTER_RV]) {
    const int e = ebase + warp + 8 * (t >> 2), q = t & 3;
    const int i0 = n4 * q / 4, i1 = n4 * (q + 1) / 4;
    const float4 *r4 = reinterpret_cast<const float4 *>(r.R + (int64_t)e * r.D);
#pragma unroll
    for (int j = 0; j < ROUTER_RV; ++j) {
        const int i = i0 + lane + 32 * j;
        rv[j] = i < i1 ? r4[i] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
}

template <int RB>
__device__ __forceinline__ void rr_task(const RouterParams &r, const float4 *xn4, int n4, int ebase, int warp, int lane,
                                        int t, int nr, int m0, const float4 (&rv)[ROUTER_RV], float (&p0)[RB],
                                        float (&a01)[RB], float (&p2)[RB]) {
    const int e = ebase + warp + 8 * (t >> 2), q = t & 3;
    const int i0 = n4 * q / 4, i1 = n4 * (q + 1) / 4;
#pragma unroll
    for (int rr = 0; rr < RB; ++rr) {
        float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
        const float4 *xr = xn4 + (size_t)rr * n4;
#pragma unroll
        for (int j = 0; j < ROUTER_RV; ++j) {
            const int i = i0 + lane + 32 * j;
            const float4 xv = i < i1 ? xr[i] : make_float4(0.f, 0.f, 0.f, 0.f);
            s0 = __fmaf_rn(xv.x, rv[j].x, s0);
            s1 = __fmaf_rn(xv.y, rv[j].y, s1);
            s2 = __fmaf_rn(xv.z, rv[j].z, s2);
            s3 = __fmaf_rn(xv.w, rv[j].w, s3);
        }
        float v = __fadd_rn(__fadd_rn(s0, s1), __fadd_rn(s2, s3));
        for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
        v = __shfl_sync(0xffffffffu, v, 0);  // lane 0's sum, the one router_kernel keeps
        if (q == 0) {
            p0[rr] = v;
        } else if (q == 1) {
            a01[rr] = __fadd_rn(p0[rr], v);
        } else if (q == 2) {
            p2[rr] = v;
        } else if (lane == 0 && rr < nr) {
            float lv = __fadd_rn(a01[rr], __fadd_rn(p2[rr], v));
            if (r.bias) lv = r.bias_first ? __fadd_rn(r.bias[e], lv) : __fadd_rn(lv, r.bias[e]);
            r.logits[(int64_t)(m0 + rr) * r.E + e] = lv;
        }
    }
}

template <int RB>
__global__ void __launch_bounds__(256) router_rows_kernel(const RouterParams r) {
    extern __shared__ float4 rsm4[];
    float4 *xn4 = rsm4;  // [RB][D / 4]
    __shared__ bool last, rowlast;
    __shared__ int cnt[256], jstart[257], pstart[257];
    __shared__ int ssel[ROUTER_MAX_PAIRS], sorted[ROUTER_MAX_PAIRS];
    pdl_wait();
    pdl_trigger();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
    const int m0 = blockIdx.x * RB, nr = min(RB, r.M - m0);
    const int n4 = r.D >> 2;
    const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int rr = 0; rr < RB; ++rr) {
        float4 *dst = xn4 + (size_t)rr * n4;
        if (rr >= nr) {
            for (int i = tid; i < n4; i += NORM_THREADS) dst[i] = z4;
            continue;
        }
        const int m = m0 + rr;
        if (r.ln_w) {
            const float4 *h4 = reinterpret_cast<const float4 *>(r.h_in + (int64_t)m * r.D);
            const float4 *w4 = reinterpret_cast<const float4 *>(r.ln_w);
            float4 hv[NORM_V4];
            double ss = 0.0;
#pragma unroll
            for (int j = 0; j < NORM_V4; ++j) {
                const int i = tid + j * NORM_THREADS;
                hv[j] = i < n4 ? h4[i] : z4;
                ss += (double)hv[j].x * hv[j].x + (double)hv[j].y * hv[j].y + (double)hv[j].z * hv[j].z +
                      (double)hv[j].w * hv[j].w;
            }
            const float rn = norm_scale(ss, r.D, r.eps);
            float4 *o4 = reinterpret_cast<float4 *>(r.hn_out + (int64_t)m * r.D);
#pragma unroll
            for (int j = 0; j < NORM_V4; ++j) {
                const int i = tid + j * NORM_THREADS;
                if (i < n4) {
                    const float4 w = w4[i];
                    const float4 v = make_float4(__fmul_rn(__fmul_rn(hv[j].x, rn), w.x), __fmul_rn(__fmul_rn(hv[j].y, rn), w.y),
                                                 __fmul_rn(__fmul_rn(hv[j].z, rn), w.z), __fmul_rn(__fmul_rn(hv[j].w, rn), w.w));
                    dst[i] = v;
                    if (blockIdx.y == 0) o4[i] = v;
                }
            }
        } else {
            const float4 *x4 = reinterpret_cast<const float4 *>(r.x + (int64_t)m * r.D);
            for (int i = tid; i < n4; i += NORM_THREADS) dst[i] = x4[i];
        }
    }
    __syncthreads();
    // (expert, quarter) tasks of this warp over this block's experts
    // [ebase, ebase + ROUTER_EPB), R of the next task in flight
    const int epb = (r.E + gridDim.y - 1) / gridDim.y;
    const int ebase = blockIdx.y * epb, eend = min(r.E, ebase + epb);
    const int ne = (eend - ebase - warp + 7) / 8, T = 4 * max(ne, 0);
    float4 ra[ROUTER_RV], rb[ROUTER_RV];
    float p0[RB], a01[RB], p2[RB];
    if (T > 0) rr_load(r, n4, ebase, warp, lane, 0, ra);
    for (int t = 0; t < T; t += 2) {
        if (t + 1 < T) rr_load(r, n4, ebase, warp, lane, t + 1, rb);
        rr_task<RB>(r, xn4, n4, ebase, warp, lane, t, nr, m0, ra, p0, a01, p2);
        if (t + 1 < T) {
            if (t + 2 < T) rr_load(r, n4, ebase, warp, lane, t + 2, ra);
            rr_task<RB>(r, xn4, n4, ebase, warp, lane, t + 1, nr, m0, rb, p0, a01, p2);
        }
    }
    // the last expert block of this row block takes its rows' top-k
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        unsigned *c = r.counter + 1 + blockIdx.x;
        rowlast = atomicAdd(c, 1u) == gridDim.y - 1;
        if (rowlast) *c = 0u;
    }
    __syncthreads();
    if (!rowlast) return;
    __threadfence();
    for (int rr = warp; rr < nr; rr += 8)
        router_topk_row<true>(r, r.logits + (int64_t)(m0 + rr) * r.E, m0 + rr, nullptr);
    // ... and the last row block the job tables
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        last = atomicAdd(r.counter, 1u) == gridDim.x - 1;
        if (last) *r.counter = 0u;
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    const int P = r.M * r.K, Ps = min(P, ROUTER_MAX_PAIRS);
    for (int p = tid; p < Ps; p += blockDim.x) ssel[p] = __ldcg(r.sel + p);
    __syncthreads();
    router_jobs(r, ssel, P, cnt, jstart, pstart, sorted);
}

// ---------------------------------------------------- expert-parallel ----
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(unsigned *p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ns_now() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Waits (bounded by EP_WAIT_NS) until every rank's flag reached exchange e;
// false when the bound ran out.
__device__ bool ep_wait_all(const unsigned *flags, int n, unsigned e) {
    const unsigned long long t0 = ns_now();
    for (int q = 0; q < n; ++q) {
        while ((int)(ld_acquire_sys(flags + q) - e) < 0) {
            if (ns_now() - t0 > (unsigned long long)EP_WAIT_NS) return false;
            __nanosleep(64);
        }
    }
    return true;
}

// Copies the output rows of this rank's (token, k) pairs into receive buffer
// (e & 1) of every rank (itself included), e = this rank's exchange number
// + 1; the last block to finish then publishes e in every rank's flag array.
__global__ void __launch_bounds__(256) ep_push_kernel(const EpPushParams p) {
    pdl_wait();
    pdl_trigger();
    const unsigned e = *reinterpret_cast<const volatile unsigned *>(p.state) + 1u;
    const int64_t rx_off = EP_FLAG_BYTES + (int64_t)(e & 1u) * p.rx_bytes;
    const bool v4 = (p.D & 3) == 0;
    for (int pr = blockIdx.x; pr < p.P; pr += gridDim.x) {
        if (!p.pair_local[pr]) continue;
        if (v4) {
            const int n4 = p.D >> 2;
            const float4 *src = reinterpret_cast<const float4 *>(p.eo + (int64_t)pr * p.D);
            for (int i = threadIdx.x; i < n4; i += blockDim.x) {
                const float4 v = __ldcg(src + i);
                for (int q = 0; q < p.n; ++q)
                    reinterpret_cast<float4 *>(p.blk[q] + rx_off)[(int64_t)pr * n4 + i] = v;
            }
        } else {
            for (int i = threadIdx.x; i < p.D; i += blockDim.x) {
                const float v = __ldcg(p.eo + (int64_t)pr * p.D + i);
                for (int q = 0; q < p.n; ++q) reinterpret_cast<float *>(p.blk[q] + rx_off)[(int64_t)pr * p.D + i] = v;
            }
        }
    }
    __threadfence_system();  // this thread's rows are visible to every rank
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned t = atomicAdd(p.state + 1, 1u);
        if (t == gridDim.x - 1) {  // last block: every row of this rank has been written
            p.state[1] = 0u;
            p.state[0] = e;
            __threadfence_system();
            for (int q = 0; q < p.n; ++q) st_release_sys(reinterpret_cast<unsigned *>(p.blk[q]) + p.rank, e);
        }
    }
}

// -------------------------------------------------------------- combine ----
// One block per row; expert rows are taken four at a time with all their
// loads in flight.  The fma chain runs in k order, as picchio.c:1445-1454
// accumulates it; a failed expert (sel < 0) is skipped (picchio.c:1394).
// With ln_w set (and h), the updated residual row is also normalised into
// hn: the next layer's input RMSNorm (picchio.c:1680) or the final norm
// (picchio.c:1712), computed exactly as rmsnorm_kernel computes it.
__global__ void __launch_bounds__(NORM_THREADS) combine_kernel(const float *eo, const float *w, const int *sel,
                                                                float scale, int K, int D, float *out, float *h,
                                                                const float *ln_w, float eps, float *hn,
                                                                const EpWait ep) {
    pdl_wait();
    pdl_trigger();
    const int m = blockIdx.x, tid = threadIdx.x;
    if (ep.n > 0) {  // expert parallelism: the rows of every rank's pairs, once all have pushed
        const unsigned e = *reinterpret_cast<const volatile unsigned *>(ep.state);
        if (tid == 0 && !ep_wait_all(reinterpret_cast<const unsigned *>(ep.blk), ep.n, e))
            atomicExch(ep.err, EP_ERR_WAIT);
        __syncthreads();
        eo = reinterpret_cast<const float *>(ep.blk + EP_FLAG_BYTES + (int64_t)(e & 1u) * ep.rx_bytes);
    }
    const bool norm = ln_w && h;
    float wk[16];
    bool ok[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) {
        ok[k] = k < K && !(sel && sel[m * K + k] < 0);
        wk[k] = k < K ? __fmul_rn(w[m * K + k], scale) : 0.0f;
    }
    const bool vec = (D & 3) == 0 && D <= 4 * 3 * NORM_THREADS;
    if (vec) {
        const int n4 = D >> 2;
        float4 acc[3], hv[3];
#pragma unroll
        for (int j = 0; j < 3; ++j) {
            acc[j] = make_float4(0.f, 0.f, 0.f, 0.f);
            const int i = tid + j * NORM_THREADS;
            hv[j] = (h && i < n4) ? reinterpret_cast<const float4 *>(h + (int64_t)m * D)[i] : acc[j];
        }
#pragma unroll
        for (int k0 = 0; k0 < 16; k0 += 4) {
            if (k0 >= K) break;
            float4 e[4][3];
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
#pragma unroll
                for (int j = 0; j < 3; ++j) {
                    const int i = tid + j * NORM_THREADS;
                    e[kk][j] = (k0 + kk < K && i < n4)
                                   ? __ldcg(reinterpret_cast<const float4 *>(eo + ((int64_t)m * K + k0 + kk) * D) + i)
                                   : make_float4(0.f, 0.f, 0.f, 0.f);
                }
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
                if (!ok[k0 + kk]) continue;
                const float c = wk[k0 + kk];
#pragma unroll
                for (int j = 0; j < 3; ++j) {
                    acc[j].x = __fmaf_rn(c, e[kk][j].x, acc[j].x);
                    acc[j].y = __fmaf_rn(c, e[kk][j].y, acc[j].y);
                    acc[j].z = __fmaf_rn(c, e[kk][j].z, acc[j].z);
                    acc[j].w = __fmaf_rn(c, e[kk][j].w, acc[j].w);
                }
            }
        }
        float4 wv[3];
#pragma unroll
        for (int j = 0; j < 3; ++j) {
            const int i = tid + j * NORM_THREADS;
            wv[j] = (norm && i < n4) ? reinterpret_cast<const float4 *>(ln_w)[i] : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        double s = 0.0;
#pragma unroll
        for (int j = 0; j < 3; ++j) {
            const int i = tid + j * NORM_THREADS;
            hv[j] = make_float4(__fadd_rn(hv[j].x, acc[j].x), __fadd_rn(hv[j].y, acc[j].y),
                                __fadd_rn(hv[j].z, acc[j].z), __fadd_rn(hv[j].w, acc[j].w));
            if (i >= n4) continue;
            if (out) reinterpret_cast<float4 *>(out + (int64_t)m * D)[i] = acc[j];
            if (h) reinterpret_cast<float4 *>(h + (int64_t)m * D)[i] = hv[j];
            s += (double)hv[j].x * hv[j].x + (double)hv[j].y * hv[j].y + (double)hv[j].z * hv[j].z +
                 (double)hv[j].w * hv[j].w;
        }
        if (!norm) return;
        const float r = norm_scale(s, D, eps);
#pragma unroll
        for (int j = 0; j < 3; ++j) {
            const int i = tid + j * NORM_THREADS;
            if (i < n4)
                reinterpret_cast<float4 *>(hn + (int64_t)m * D)[i] =
                    make_float4(__fmul_rn(__fmul_rn(hv[j].x, r), wv[j].x), __fmul_rn(__fmul_rn(hv[j].y, r), wv[j].y),
                                __fmul_rn(__fmul_rn(hv[j].z, r), wv[j].z), __fmul_rn(__fmul_rn(hv[j].w, r), wv[j].w));
        }
        return;
    }
    float *hr = h ? h + (int64_t)m * D : nullptr;
    double s = 0.0;
    for (int i = tid; i < D; i += NORM_THREADS) {
        float acc = 0.0f;
        for (int k = 0; k < K; ++k)
            if (ok[k < 16 ? k : 15]) acc = __fmaf_rn(wk[k < 16 ? k : 15], __ldcg(eo + ((int64_t)m * K + k) * D + i), acc);
        if (out) out[(int64_t)m * D + i] = acc;
        if (hr) {
            const float v = __fadd_rn(hr[i], acc);
            hr[i] = v;
            s += (double)v * (double)v;
        }
    }
    if (!norm) return;
    const float r = norm_scale(s, D, eps);
    for (int i = tid; i < D; i += NORM_THREADS) hn[(int64_t)m * D + i] = __fmul_rn(__fmul_rn(hr[i], r), ln_w[i]);
}

// ------------------------------------------------------------- f32 gemv ----
__global__ void gemv_f32_kernel(const F32GemvParams p) {
    pdl_wait();
    pdl_trigger();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int o = blockIdx.x * 8 + warp;
    if (o >= p.O) return;
    const float *w = p.W + (int64_t)o * p.I;
    for (int m = 0; m < p.M; ++m) {
        const float *xr = p.x + (int64_t)m * p.ldx;
        float s = 0.0f;
        for (int i = lane; i < p.I; i += 32) s = __fmaf_rn(xr[i], w[i], s);
        for (int q = 16; q > 0; q >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, q));
        if (lane == 0) {
            if (p.bias) s = __fadd_rn(s, p.bias[o]);
            float *dst = p.y + (int64_t)m * p.ldy + o;
            *dst = p.residual ? __fadd_rn(*dst, s) : s;
        }
    }
}

__global__ void qkv_post_kernel(const QkvPostParams p) {
    pdl_wait();
    pdl_trigger();
    const int m = blockIdx.y;
    const int half = p.hd / 2, Oq = p.H * p.hd, Ok = p.KVH * p.hd;
    const float *raw = p.raw + (int64_t)m * (Oq + 2 * Ok);
    const int pos = p.row_pos[m];
    const int64_t kvb = (int64_t)p.row_seq[m] * p.seq_stride + (int64_t)pos * Ok;
    const bool store = pos >= 0 && pos < p.ctx;
    const int nq = p.H * half, nk = p.KVH * half;
    for (int idx = blockIdx.x * blockDim.x + threadIdx.x; idx < nq + nk + Ok; idx += gridDim.x * blockDim.x) {
        if (idx < nq + nk) {
            const bool isq = idx < nq;
            const int li = isq ? idx : idx - nq;
            const int h = li / half, j = li % half;
            const int o = h * p.hd + j;
            const float *src = isq ? raw : raw + Oq;
            const float *b = isq ? p.bq : p.bk;
            float a = src[o], c = src[o + half];
            if (b) { a = __fadd_rn(a, b[o]); c = __fadd_rn(c, b[o + half]); }
            const float cs = p.rope_cs[(int64_t)pos * half + j], sn = p.rope_sn[(int64_t)pos * half + j];
            const float lo = __fmaf_rn(a, cs, -__fmul_rn(c, sn));
            const float hi = __fmaf_rn(a, sn, __fmul_rn(c, cs));
            if (isq) {
                p.q[(int64_t)m * Oq + o] = lo;
                p.q[(int64_t)m * Oq + o + half] = hi;
            } else if (store) {
                stf(p.kc, kvb + o, lo, p.kv_bf16);
                stf(p.kc, kvb + o + half, hi, p.kv_bf16);
            }
        } else {
            const int o = idx - nq - nk;
            float v = raw[Oq + Ok + o];
            if (p.bv) v = __fadd_rn(v, p.bv[o]);
            if (store) stf(p.vc, kvb + o, v, p.kv_bf16);
        }
    }
}

__global__ void argmax_rows_kernel(const float *logits, int V, unsigned long long *packed) {
    pdl_wait();
    pdl_trigger();
    const int m = blockIdx.y;
    unsigned long long best = 0ull;
    for (int o = blockIdx.x * blockDim.x + threadIdx.x; o < V; o += gridDim.x * blockDim.x) {
        float v = logits[(int64_t)m * V + o];
        if (v != v) continue;
        if (v == 0.0f) v = 0.0f;
        const uint32_t u = __float_as_uint(v);
        const uint32_t key = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
        const unsigned long long k = ((unsigned long long)key << 32) | (0xFFFFFFFFu - (uint32_t)o);
        best = k > best ? k : best;
    }
    for (int q = 16; q > 0; q >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, q);
        best = other > best ? other : best;
    }
    if ((threadIdx.x & 31) == 0 && best) atomicMax(packed + m, best);
}

__global__ void argmax_finish_kernel(unsigned long long *packed, int n, int *ids, int *ids2) {
    pdl_wait();
    pdl_trigger();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const unsigned long long v = packed[i];
    const int id = v ? (int)(0xFFFFFFFFu - (uint32_t)(v & 0xFFFFFFFFull)) : 0;
    ids[i] = id;
    if (ids2) ids2[i] = id;
    packed[i] = 0ull;
}

}  // namespace

cudaError_t launch_embed(int fmt, const void *table, const float *scales, int gs, int V, int D,
                         const int *tok, int M, float *h, cudaStream_t st) {
    return launch_k(embed_kernel, dim3(M), dim3(256), 0, st, fmt, table, scales, gs, V, D, tok, h);
    return cudaGetLastError();
}

cudaError_t launch_rmsnorm(const float *x, const float *w, float *out, int M, int D, float eps,
                           cudaStream_t st) {
    return launch_k(rmsnorm_kernel, dim3(M), dim3(NORM_THREADS), 0, st, x, w, out, D, eps);
    return cudaGetLastError();
}


cudaError_t launch_router(const RouterParams &r, cudaStream_t st) {
    // more pairs than one job table holds only with the expert-sorted pair
    // lists (the tensor-core expert path reads those, not the jobs)
    // pairs are grouped at most 8 (or 4) per job: 4096 pairs of <= 256
    // experts make at most 768 jobs, within GEMV_MAX_JOBS
    if (r.E > 256 || r.K > 16 || r.M * r.K > ROUTER_MAX_PAIRS)
        return cudaErrorInvalidValue;
    if (r.ln_w && ((r.D & 3) || r.D > 4 * NORM_V4 * NORM_THREADS || !r.h_in || !r.hn_out)) return cudaErrorInvalidValue;
    if (!r.sel_in && r.M >= ROUTER_RB_MIN_ROWS && (r.D & 3) == 0 && r.D <= 4 * 32 * ROUTER_RV * 4 &&
        r.D <= 4 * NORM_V4 * NORM_THREADS) {
        // many rows: 4 per block, all experts (enough blocks already); fewer:
        // 2 rows per block and the experts split ROUTER_EPB per block
        const int rb = r.M >= 256 ? 4 : 2;
        const dim3 grid((r.M + rb - 1) / rb, r.M >= 256 ? 1 : (r.E + ROUTER_EPB - 1) / ROUTER_EPB);
        const size_t smem = (size_t)rb * r.D * 4;
        return rb == 4 ? launch_k(router_rows_kernel<4>, grid, dim3(256), smem, st, r)
                       : launch_k(router_rows_kernel<2>, grid, dim3(256), smem, st, r);
    }
    const dim3 grid = r.sel_in ? dim3(1) : dim3((r.E + 1) / 2, (r.M + ROUTER_ROWS - 1) / ROUTER_ROWS);
    return launch_k(router_kernel, grid, dim3(256), 0, st, r);
    return cudaGetLastError();
}

cudaError_t kernels_configure() {
    // the row-block router keeps RB normalised rows of up to 3072 floats
    cudaError_t e = cudaFuncSetAttribute(router_rows_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, 2 * 3072 * 4);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(router_rows_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, 4 * 3072 * 4);
    return e;
}

cudaError_t launch_combine(const float *eo, const float *w, const int *sel, float scale, int M, int K,
                           int D, float *out, float *h, cudaStream_t st, const float *ln_w, float eps,
                           float *hn, const EpWait *ep) {
    if (ln_w && (!h || !hn)) return cudaErrorInvalidValue;
    EpWait none{};
    return launch_k(combine_kernel, dim3(M), dim3(NORM_THREADS), 0, st, eo, w, sel, scale, K, D, out, h, ln_w,
                    eps, hn, ep ? *ep : none);
}

cudaError_t launch_ep_push(const EpPushParams &p, int nsm, cudaStream_t st) {
    if (p.n < 1 || p.n > EP_MAX_RANKS || p.P < 1) return cudaErrorInvalidValue;
    const int grid = p.P < 2 * nsm ? p.P : 2 * nsm;
    return launch_k(ep_push_kernel, dim3(grid), dim3(256), 0, st, p);
}

cudaError_t launch_gemv_f32(const F32GemvParams &p, cudaStream_t st) {
    return launch_k(gemv_f32_kernel, dim3((p.O + 7) / 8), dim3(256), 0, st, p);
    return cudaGetLastError();
}

cudaError_t launch_qkv_post(const QkvPostParams &p, cudaStream_t st) {
    dim3 grid(8, p.M);
    return launch_k(qkv_post_kernel, dim3(grid), dim3(256), 0, st, p);
    return cudaGetLastError();
}

cudaError_t launch_argmax_rows(const float *logits, int M, int V, unsigned long long *packed, cudaStream_t st) {
    dim3 grid(64, M);
    return launch_k(argmax_rows_kernel, dim3(grid), dim3(256), 0, st, logits, V, packed);
    return cudaGetLastError();
}

__global__ void gen_advance_kernel(const int *next, int *pos, int *gen, int *step) {
    pdl_wait();
    pdl_trigger();
    const int s = *step;
    gen[s] = next[0];
    *step = s + 1;
    pos[0] += 1;
}

cudaError_t launch_gen_advance(const int *next, int *pos, int *gen, int *step, cudaStream_t st) {
    return launch_k(gen_advance_kernel, dim3(1), dim3(1), 0, st, next, pos, gen, step);
    return cudaGetLastError();
}

cudaError_t launch_argmax_finish(unsigned long long *packed, int n, int *ids, int *ids2, cudaStream_t st) {
    return launch_k(argmax_finish_kernel, dim3((n + 127) / 128), dim3(128), 0, st, packed, n, ids, ids2);
    return cudaGetLastError();
}

}  // namespace pc
