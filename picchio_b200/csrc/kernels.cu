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
__global__ void rmsnorm_kernel(const float *x, const float *w, float *out, int D, float eps) {
    pdl_wait();
    pdl_trigger();
    __shared__ double red[32];
    const int m = blockIdx.x;
    const float *xr = x + (int64_t)m * D;
    double s = 0.0;
    for (int i = threadIdx.x; i < D; i += blockDim.x) s += (double)xr[i] * (double)xr[i];
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x < 32) {
        double v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0;
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (threadIdx.x == 0) red[0] = v;
    }
    __syncthreads();
    const float r = __fdiv_rn(1.0f, sqrtf(__fadd_rn((float)(red[0] / D), eps)));
    float *o = out + (int64_t)m * D;
    for (int i = threadIdx.x; i < D; i += blockDim.x) o[i] = __fmul_rn(__fmul_rn(xr[i], r), w[i]);
}

// --------------------------------------------------------------- router ----
__global__ void __launch_bounds__(256) router_kernel(const RouterParams r) {
    pdl_wait();
    pdl_trigger();
    __shared__ bool last;
    __shared__ int cnt[256], jstart[257];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (!r.sel_in) {
        const int e = blockIdx.x * 8 + warp;
        if (e < r.E) {
            const float *re = r.R + (int64_t)e * r.D;
            const bool vec = (r.D & 3) == 0;
            for (int m = 0; m < r.M; ++m) {
                const float *xr = r.x + (int64_t)m * r.D;
                float s = 0.0f;
                if (vec) {
                    // 16-byte loads, 8 in flight per lane, 4 partial sums
                    const float4 *r4 = reinterpret_cast<const float4 *>(re);
                    const float4 *x4 = reinterpret_cast<const float4 *>(xr);
                    const int n4 = r.D >> 2;
                    float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
                    for (int i0 = lane; i0 < n4; i0 += 32 * 8) {
                        float4 rv[8], xv[8];
#pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            const int i = i0 + 32 * j;
                            rv[j] = i < n4 ? r4[i] : make_float4(0.f, 0.f, 0.f, 0.f);
                            xv[j] = i < n4 ? x4[i] : make_float4(0.f, 0.f, 0.f, 0.f);
                        }
#pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            s0 = __fmaf_rn(xv[j].x, rv[j].x, s0);
                            s1 = __fmaf_rn(xv[j].y, rv[j].y, s1);
                            s2 = __fmaf_rn(xv[j].z, rv[j].z, s2);
                            s3 = __fmaf_rn(xv[j].w, rv[j].w, s3);
                        }
                    }
                    s = __fadd_rn(__fadd_rn(s0, s1), __fadd_rn(s2, s3));
                } else {
                    for (int i = lane; i < r.D; i += 32) s = __fmaf_rn(xr[i], re[i], s);
                }
                for (int o = 16; o > 0; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
                if (lane == 0) {
                    // decode adds the bias after the dot, prefill starts from it;
                    // with a parallel dot both become one final add.
                    if (r.bias) s = r.bias_first ? __fadd_rn(r.bias[e], s) : __fadd_rn(s, r.bias[e]);
                    r.logits[(int64_t)m * r.E + e] = s;
                }
            }
        }
        __threadfence();
        __syncthreads();
        if (threadIdx.x == 0) {
            last = atomicAdd(r.counter, 1u) == gridDim.x - 1;
            if (last) *r.counter = 0u;
        }
        __syncthreads();
        if (!last) return;
        __threadfence();
        // top-k, K rounds of strict '>' argmax; ties -> lowest index
        for (int m = warp; m < r.M; m += 8) {
            const float *lg = r.logits + (int64_t)m * r.E;
            float vals[8];
            for (int q = 0; q < 8; ++q) {
                const int e = lane + 32 * q;
                vals[q] = e < r.E ? __ldcg(lg + e) : -INFINITY;
            }
            float wk[16];
            int sk[16];
            for (int k = 0; k < r.K; ++k) {
                float bv = -1e30f;
                int bi = -1;
                for (int q = 0; q < 8; ++q) {
                    const int e = lane + 32 * q;
                    if (e < r.E && vals[q] > bv) { bv = vals[q]; bi = e; }
                }
                for (int o = 16; o > 0; o >>= 1) {
                    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                    if (ov > bv || (ov == bv && oi >= 0 && (bi < 0 || oi < bi))) { bv = ov; bi = oi; }
                }
                sk[k] = bi;
                wk[k] = bv;
                if (bi >= 0 && (bi & 31) == lane) vals[bi >> 5] = -INFINITY;
            }
            if (lane == 0) {
                // softmax over the K selected logits (quant.h:406-412)
                float mx = -1e30f;
                for (int k = 0; k < r.K; ++k) if (wk[k] > mx) mx = wk[k];
                float sum = 0.0f;
                for (int k = 0; k < r.K; ++k) { wk[k] = expf(__fsub_rn(wk[k], mx)); sum = __fadd_rn(sum, wk[k]); }
                for (int k = 0; k < r.K; ++k) {
                    r.sel[m * r.K + k] = sk[k];
                    r.w[m * r.K + k] = __fdiv_rn(wk[k], sum);
                }
            }
        }
        __syncthreads();
        __threadfence_block();
    } else {
        if (blockIdx.x != 0) return;
        for (int i = threadIdx.x; i < r.M * r.K; i += blockDim.x) {
            r.sel[i] = r.sel_in[i];
            r.w[i] = r.w_in[i];
        }
        __syncthreads();
    }
    // expert job tables: pairs grouped by expert, at most 8 pairs per job
    const int P = r.M * r.K;
    const int e = threadIdx.x;
    int n = 0;
    if (e < r.E && e >= r.e_lo && e < r.e_hi) {
        for (int p = 0; p < P; ++p) n += (__ldcg(r.sel + p) == e);
    }
    cnt[e] = (n + GEMV_MAXR - 1) / GEMV_MAXR;
    __syncthreads();
    if (warp == 0) {  // exclusive scan of jobs per expert: 8 experts per lane
        int v[8], tot = 0;
#pragma unroll
        for (int q = 0; q < 8; ++q) { v[q] = tot; tot += cnt[lane * 8 + q]; }
        int inc = tot;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int n = __shfl_up_sync(0xffffffffu, inc, o);
            if (lane >= o) inc += n;
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
    for (int p = threadIdx.x; p < P; p += blockDim.x) {
        const int ep = __ldcg(r.sel + p);
        r.pair_local[p] = (ep >= r.e_lo && ep < r.e_hi) ? 1 : 0;
    }
    if (n == 0) return;
    const int slot = r.slot_of ? r.slot_of[e] : e - r.e_lo;
    const uint8_t *base = r.table + (int64_t)slot * r.stride;
    int j = jstart[e], fill = 0;
    for (int p = 0; p < P && j < GEMV_MAX_JOBS; ++p) {
        if (__ldcg(r.sel + p) != e) continue;
        GemvJob &gu = r.jobs_gu[j];
        GemvJob &dn = r.jobs_dn[j];
        if (fill == 0) {
            gu.tiles = base + r.off_gu;
            gu.rs = r.off_gu_rs >= 0 ? reinterpret_cast<const float *>(base + r.off_gu_rs) : nullptr;
            gu.bias = r.off_gu_b >= 0 ? reinterpret_cast<const float *>(base + r.off_gu_b) : nullptr;
            gu.n_rt = r.gu_rt; gu.O = r.gu_O; gu.seg = 0;
            dn.tiles = base + r.off_dn;
            dn.rs = r.off_dn_rs >= 0 ? reinterpret_cast<const float *>(base + r.off_dn_rs) : nullptr;
            dn.bias = r.off_dn_b >= 0 ? reinterpret_cast<const float *>(base + r.off_dn_b) : nullptr;
            dn.n_rt = r.dn_rt; dn.O = r.dn_O; dn.seg = 0;
        }
        gu.in_row[fill] = p / r.K;
        gu.out_row[fill] = p;
        dn.in_row[fill] = p;
        dn.out_row[fill] = p;
        ++fill;
        gu.nrows = dn.nrows = fill;
        if (fill == GEMV_MAXR) { fill = 0; ++j; }
    }
}

// -------------------------------------------------------------- combine ----
__global__ void combine_kernel(const float *eo, const float *w, const int *sel, float scale, int K,
                               int D, float *out, float *h) {
    pdl_wait();
    pdl_trigger();
    const int m = blockIdx.x;
    for (int i = threadIdx.x; i < D; i += blockDim.x) {
        float acc = 0.0f;
        for (int k = 0; k < K; ++k) {
            if (sel && sel[m * K + k] < 0) continue;  // failed expert is skipped (picchio.c:1394)
            const float wk = __fmul_rn(w[m * K + k], scale);
            acc = __fmaf_rn(wk, eo[((int64_t)m * K + k) * D + i], acc);
        }
        if (out) out[(int64_t)m * D + i] = acc;
        if (h) h[(int64_t)m * D + i] = __fadd_rn(h[(int64_t)m * D + i], acc);
    }
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
    return launch_k(rmsnorm_kernel, dim3(M), dim3(256), 0, st, x, w, out, D, eps);
    return cudaGetLastError();
}


cudaError_t launch_router(const RouterParams &r, cudaStream_t st) {
    if (r.E > 256 || r.K > 16) return cudaErrorInvalidValue;
    const int blocks = r.sel_in ? 1 : (r.E + 7) / 8;
    return launch_k(router_kernel, dim3(blocks), dim3(256), 0, st, r);
    return cudaGetLastError();
}

cudaError_t launch_combine(const float *eo, const float *w, const int *sel, float scale, int M, int K,
                           int D, float *out, float *h, cudaStream_t st) {
    return launch_k(combine_kernel, dim3(M), dim3(256), 0, st, eo, w, sel, scale, K, D, out, h);
    return cudaGetLastError();
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
