// attention_core.cuh - decode attention over the KV cache with attention
// sinks and the alternating sliding window: the score / softmax / P.V part of
// gqa_attention (picchio.c:556-607) for one (row, KV head, span) work item.
//
// A work item takes one KV head of one row and a span of up to 256 positions
// (split-K over positions), for all G <= 8 query heads that share the KV head
// (GQA, picchio.c:568); 256 threads:
//  scores: thread t owns one position; it loads the whole K row with 16-byte
//    loads first, then forms each head's dot in the reference's sequential
//    order (dot = dot + q[i]*k[i], i = 0..hd-1, unfused), times 1/sqrt(hd);
//  softmax: per-head max and sum over the span (block reductions);
//  P.V: thread (4 dims, position group) loads its V rows (16 bytes each) up
//    front and accumulates p[g][t] * V[t][d..d+3] for all G heads; the 16
//    position groups are then summed in a fixed order.
// The last item of a (row, KV head) to finish (atomic ticket) merges the
// spans with the sink, which joins the max and the denominator only
// (picchio.c:586-596); a row whose positions fit one span merges in place.
#pragma once
#include <cuda_bf16.h>

#include "kernels.h"
#include "launch.cuh"
#include "ptx.cuh"

namespace pc {

namespace {


constexpr int MAXG = 8, NT = ATTN_SPLIT, PG = 16;  // PG: position groups in P.V

// 4 consecutive elements as floats
__device__ __forceinline__ float4 load4(const float *p) { return *reinterpret_cast<const float4 *>(p); }
__device__ __forceinline__ float4 load4(const __nv_bfloat16 *p) {
    const uint2 a = *reinterpret_cast<const uint2 *>(p);
    const float2 x = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&a.x));
    const float2 y = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&a.y));
    return make_float4(x.x, x.y, y.x, y.y);
}

// A K row's 4 elements as loaded (no conversion, so the load does not block)
__device__ __forceinline__ float4 load4_raw(const float *p) { return *reinterpret_cast<const float4 *>(p); }
__device__ __forceinline__ uint2 load4_raw(const __nv_bfloat16 *p) { return *reinterpret_cast<const uint2 *>(p); }
__device__ __forceinline__ float4 raw_to_f4(float4 v) { return v; }
__device__ __forceinline__ float4 raw_to_f4(uint2 a) {
    const float2 x = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&a.x));
    const float2 y = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&a.y));
    return make_float4(x.x, x.y, y.x, y.y);
}
template <typename T> struct Raw4 { using type = float4; };
template <> struct Raw4<__nv_bfloat16> { using type = uint2; };

// Shared memory of one work item.
template <int HD>
struct alignas(16) AttnSmem {
    float qs[MAXG][HD];
    float ps[MAXG][NT];
    float wred[MAXG][NT / 32];
    float mloc[MAXG], lloc[MAXG];
    float ored[NT / 32][MAXG][HD];
    float mrec[MAXG][64], lrec[MAXG][64];
    float lsum[MAXG];
    bool last;
};

// One work item: span s of KV head kh of row m, run by NT threads (t =
// threadIdx.x < NT) that synchronize on named barrier `bar`.  PDL: the item
// runs in a programmatic dependent launch: for a single row, the K rows of
// earlier positions (written by earlier steps) are requested before waiting
// for the kernel that writes this step's q and K/V row.
template <typename T, int HD, bool PDL = false>
__device__ __forceinline__ void attn_item(const AttnParams &a, int s, int kh, int m, AttnSmem<HD> &sm, int bar) {
    auto &qs = sm.qs;
    auto &ps = sm.ps;
    auto &wred = sm.wred;
    auto &mloc = sm.mloc;
    auto &lloc = sm.lloc;
    auto &ored = sm.ored;
    auto &mrec = sm.mrec;
    auto &lrec = sm.lrec;
    bool &last = sm.last;
    const T *Kc = reinterpret_cast<const T *>(a.kc);
    const T *Vc = reinterpret_cast<const T *>(a.vc);
    const int G = a.H / a.KVH, kvd = a.KVH * HD;
    const int pos = a.row_pos[m];
    int end = pos;
    if (end >= a.ctx) end = a.ctx - 1;  // picchio.c:559-560
    int start = 0;
    if (a.window > 0) {
        start = end - a.window + 1;
        if (start < 0) start = 0;
    }
    // spans that hold positions; a launch may have more (a power-of-two
    // bucket shared by nearby positions), which leave at once
    const int nsp = (end - start + NT) / NT;
    if (s >= nsp) return;
    const int p0 = start + s * NT;
    const int cnt = max(0, min(NT, end + 1 - p0));
    const int64_t cache0 = (int64_t)a.row_seq[m] * a.seq_stride + kh * HD;
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    // The KV rows of the span do not depend on q: this thread's K row goes
    // into registers and its V row into L2 before q is even loaded, so the
    // cache's HBM latency is paid once, overlapped with q and the scores.
    typename Raw4<T>::type k4[HD / 4];
    auto load_kv = [&]() {
        const T *kr = Kc + cache0 + (int64_t)(p0 + t) * kvd;
#pragma unroll
        for (int i = 0; i < HD / 4; ++i) k4[i] = load4_raw(kr + 4 * i);
        const char *vr = reinterpret_cast<const char *>(Vc + cache0 + (int64_t)(p0 + t) * kvd);
        for (int o = 0; o < (int)(HD * sizeof(T)); o += 128) prefetch_l2(vr + o);
    };
    // Rows of this step write K/V at their own positions: with one row that is
    // only position pos; with several (a prefill chunk shares one sequence)
    // every load waits.
    const bool fresh = a.M > 1 || p0 + t == pos;
    if (t < cnt && !fresh) load_kv();
    if (PDL) pdl_wait();
    if (t < cnt && fresh) load_kv();
    for (int i = t; i < G * HD; i += NT) qs[i / HD][i % HD] = a.q[(int64_t)m * a.H * HD + (kh * G) * HD + i];
    named_bar_sync(bar, NT);
    const float scale = __fdiv_rn(1.0f, sqrtf((float)HD));
    if (t < cnt) {
        float dot[MAXG];
#pragma unroll
        for (int g = 0; g < MAXG; ++g) dot[g] = 0.0f;
        // per head the sequential order of the reference (i = 0..hd-1); q is
        // read from shared memory 4 elements at a time
#pragma unroll
        for (int i = 0; i < HD / 4; ++i) {
            const float4 kv = raw_to_f4(k4[i]);
#pragma unroll
            for (int g = 0; g < MAXG; ++g)
                if (g < G) {
                    const float4 qv = *reinterpret_cast<const float4 *>(&qs[g][4 * i]);
                    dot[g] = __fadd_rn(dot[g], __fmul_rn(qv.x, kv.x));
                    dot[g] = __fadd_rn(dot[g], __fmul_rn(qv.y, kv.y));
                    dot[g] = __fadd_rn(dot[g], __fmul_rn(qv.z, kv.z));
                    dot[g] = __fadd_rn(dot[g], __fmul_rn(qv.w, kv.w));
                }
        }
#pragma unroll
        for (int g = 0; g < MAXG; ++g)
            if (g < G) ps[g][t] = __fmul_rn(dot[g], scale);
    }
    named_bar_sync(bar, NT);
    for (int g = 0; g < G; ++g) {
        float v = t < cnt ? ps[g][t] : -INFINITY;
        for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
        if (lane == 0) wred[g][warp] = v;
    }
    named_bar_sync(bar, NT);
    if (t < G) {
        float v = -INFINITY;
        for (int w = 0; w < NT / 32; ++w) v = fmaxf(v, wred[t][w]);
        mloc[t] = v;
    }
    named_bar_sync(bar, NT);
    for (int g = 0; g < G; ++g) {
        float e = 0.0f;
        if (t < cnt) {
            e = expf(__fsub_rn(ps[g][t], mloc[g]));
            ps[g][t] = e;
        }
        for (int o = 16; o > 0; o >>= 1) e = __fadd_rn(e, __shfl_xor_sync(0xffffffffu, e, o));
        if (lane == 0) wred[g][warp] = e;
    }
    named_bar_sync(bar, NT);
    if (t < G) {
        float v = 0.0f;
        for (int w = 0; w < NT / 32; ++w) v = __fadd_rn(v, wred[t][w]);
        lloc[t] = v;
    }
    // P.V: thread = (dq: 4 dims, pg: position group); positions pg, pg+16, ...
    constexpr int DQ = HD / 4;            // dim quads per row
    constexpr int TPG = NT / PG;          // threads per position group (16)
    float4 acc[MAXG];
#pragma unroll
    for (int g = 0; g < MAXG; ++g) acc[g] = make_float4(0.f, 0.f, 0.f, 0.f);
    {
        const int dq0 = t % TPG, pg = t / TPG;
        {  // HD <= 64: one quad of dims per thread; all lanes run the shuffles
            const int dq = dq0;
            const bool act = dq < DQ;
            float4 vv[NT / PG];
#pragma unroll
            for (int k = 0; k < NT / PG; ++k) {
                const int u = pg + PG * k;
                vv[k] = (act && u < cnt) ? load4(Vc + cache0 + (int64_t)(p0 + u) * kvd + 4 * dq)
                                         : make_float4(0.f, 0.f, 0.f, 0.f);
            }
            float4 ac[MAXG];
#pragma unroll
            for (int g = 0; g < MAXG; ++g) ac[g] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int k = 0; k < NT / PG; ++k) {
                const int u = pg + PG * k;
                if (u >= cnt) break;
#pragma unroll
                for (int g = 0; g < MAXG; ++g)
                    if (g < G) {
                        const float pg_ = ps[g][u];
                        ac[g].x = __fmaf_rn(pg_, vv[k].x, ac[g].x);
                        ac[g].y = __fmaf_rn(pg_, vv[k].y, ac[g].y);
                        ac[g].z = __fmaf_rn(pg_, vv[k].z, ac[g].z);
                        ac[g].w = __fmaf_rn(pg_, vv[k].w, ac[g].w);
                    }
            }
            // the two position groups of a warp (lanes l and l^16) first
#pragma unroll
            for (int g = 0; g < MAXG; ++g) {
                ac[g].x = __fadd_rn(ac[g].x, __shfl_xor_sync(0xffffffffu, ac[g].x, 16));
                ac[g].y = __fadd_rn(ac[g].y, __shfl_xor_sync(0xffffffffu, ac[g].y, 16));
                ac[g].z = __fadd_rn(ac[g].z, __shfl_xor_sync(0xffffffffu, ac[g].z, 16));
                ac[g].w = __fadd_rn(ac[g].w, __shfl_xor_sync(0xffffffffu, ac[g].w, 16));
            }
            if (lane < 16 && act)
#pragma unroll
                for (int g = 0; g < MAXG; ++g)
                    if (g < G) *reinterpret_cast<float4 *>(&ored[warp][g][4 * dq]) = ac[g];
        }
    }
    named_bar_sync(bar, NT);
    if (nsp == 1) {
        // one span: the merge below for a single span, in the same arithmetic
        // (so results equal the multi-span path's), without the round trip
        // through the partial records
        for (int idx = t; idx < G * HD; idx += NT) {
            const int g = idx / HD, d = idx % HD, h = kh * G + g;
            float o = 0.0f;
#pragma unroll
            for (int w = 0; w < NT / 32; ++w) o = __fadd_rn(o, ored[w][g][d]);
            float M = a.sinks ? a.sinks[h] : -INFINITY;
            M = fmaxf(M, mloc[g]);
            float L = a.sinks ? expf(__fsub_rn(a.sinks[h], M)) : 0.0f;
            float O = 0.0f;
            if (lloc[g] != 0.0f) {
                const float f = expf(__fsub_rn(mloc[g], M));
                L = __fmaf_rn(lloc[g], f, L);
                O = __fmaf_rn(o, f, O);
            }
            a.out[(int64_t)m * a.H * HD + h * HD + d] = __fdiv_rn(O, L);
        }
        return;
    }
    const int stride = HD + 2;
    for (int idx = t; idx < G * HD; idx += NT) {
        const int g = idx / HD, d = idx % HD;
        float o = 0.0f;
#pragma unroll
        for (int w = 0; w < NT / 32; ++w) o = __fadd_rn(o, ored[w][g][d]);
        float *rec = a.part + (((int64_t)m * a.H + kh * G + g) * a.nsplit + s) * stride;
        rec[2 + d] = o;
        if (d == 0) {
            rec[0] = cnt > 0 ? mloc[g] : -INFINITY;
            rec[1] = cnt > 0 ? lloc[g] : 0.0f;
        }
    }
    __threadfence();
    named_bar_sync(bar, NT);
    if (t == 0) {
        unsigned *c = a.counter + m * a.KVH + kh;
        last = atomicAdd(c, 1u) == (unsigned)(nsp - 1);
        if (last) *c = 0u;
    }
    named_bar_sync(bar, NT);
    if (!last) return;
    __threadfence();
    // merge the spans: (m, l) of every span into shared memory first
    for (int idx = t; idx < G * nsp; idx += NT) {
        const int g = idx / nsp, k = idx % nsp;
        const float *rec = a.part + (((int64_t)m * a.H + kh * G + g) * a.nsplit + k) * stride;
        if (k < 64) {
            mrec[g][k] = __ldcg(rec);
            lrec[g][k] = __ldcg(rec + 1);
        }
    }
    named_bar_sync(bar, NT);
    // per head, once: the max M over the sink and the spans, the span weights
    // f_k = exp(m_k - M) (in place of m_k) and the denominator
    if (t < G) {
        const int g = t, h = kh * G + g;
        float M = a.sinks ? a.sinks[h] : -INFINITY;
        for (int k = 0; k < nsp; ++k) M = fmaxf(M, mrec[g][k]);
        float L = a.sinks ? expf(__fsub_rn(a.sinks[h], M)) : 0.0f;
        for (int k = 0; k < nsp; ++k) {
            float f = 0.0f;
            if (lrec[g][k] != 0.0f) {
                f = expf(__fsub_rn(mrec[g][k], M));
                L = __fmaf_rn(lrec[g][k], f, L);
            }
            mrec[g][k] = f;
        }
        sm.lsum[g] = L;
    }
    named_bar_sync(bar, NT);
    for (int idx = t; idx < G * HD; idx += NT) {
        const int g = idx / HD, d = idx % HD, h = kh * G + g;
        const float *rec0 = a.part + (((int64_t)m * a.H + h) * a.nsplit) * stride;
        float O = 0.0f;
        for (int k0 = 0; k0 < nsp; k0 += 16) {
            float ov[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) ov[j] = k0 + j < nsp ? __ldcg(rec0 + (k0 + j) * stride + 2 + d) : 0.0f;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const int k = k0 + j;
                if (k >= nsp || lrec[g][k] == 0.0f) continue;
                O = __fmaf_rn(ov[j], mrec[g][k], O);
            }
        }
        a.out[(int64_t)m * a.H * HD + h * HD + d] = __fdiv_rn(O, sm.lsum[g]);
    }
}


}  // namespace

}  // namespace pc
