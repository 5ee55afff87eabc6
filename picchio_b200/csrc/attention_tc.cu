// attention_tc.cu - decode attention for steps of many rows (batched decode,
// prefill chunks) on the tensor cores: the score / softmax-with-sink / P.V
// part of gqa_attention (picchio.c:556-607) for a bf16 KV cache, head size 64
// and 8 query heads per KV head (the GPT-OSS shape).
//
// One CTA per (row, KV head), 4 warps.  Warp w takes the 64-position tiles
// w, w + 4, ... of the row's positions [start, end]; each tile's K and V rows
// (128 bytes each) are copied into a 2-stage shared-memory ring with cp.async
// (16-byte chunks, XOR-swizzled by row so ldmatrix reads are conflict-free).
// S = Q K^T and O += P V are mma.sync m16n8k16 bf16 products with fp32
// accumulation; the 8 query heads are rows 0-7 of the 16-row A operand.  Q
// and P enter as two bf16 halves each (x = hi + lo, hi = bf16(x), lo =
// bf16(x - hi)), K and V are exact in bf16, so each product carries ~16
// mantissa bits of Q or P: close to the fp32 path.  The softmax is online
// per warp (running max and sum per head); the four warps' (max, sum, O) are
// merged with the sink in shared memory, as the span merge of the one-row
// kernel does (picchio.c:586-596).
//
// With few rows the positions are also split over CTAs (blockIdx.z: spans of
// 512 positions, two tiles per warp): each span's CTA writes its (max, sum,
// O) per head and the last one (atomic ticket) merges the spans with the sink.
#include <cuda_bf16.h>

#include <algorithm>
#include <cstdlib>

#include "kernels.h"
#include "launch.cuh"
#include "ptx.cuh"

namespace pc {

namespace {

constexpr int AT_WARPS = 4, AT_TILE = 64, AT_HD = 64, AT_G = 8;
constexpr int AT_SPAN = AT_WARPS * 2 * AT_TILE;    // positions per CTA when split (512)
constexpr int AT_TILE_BYTES = AT_TILE * AT_HD * 2;  // 8 KB: 64 positions x 128 bytes
constexpr int AT_STAGE = 2 * AT_TILE_BYTES;         // K and V of one tile
constexpr int AT_MERGE = AT_WARPS * AT_G * (AT_HD + 2) * 4;
constexpr int AT_SMEM = AT_WARPS * 2 * AT_STAGE + AT_MERGE;

__device__ __forceinline__ void cp_async16_zfill(void *dst, const void *src, int src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes)
                 : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

// D += A B, A rows 8-15 zero (a1 = a3 = 0)
__device__ __forceinline__ void mma8(float (&c)[4], uint32_t a0, uint32_t a2, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
}

// (x0, x1) as two packed bf16 halves: hi = bf16(x), lo = bf16(x - hi)
__device__ __forceinline__ void split2(float x0, float x1, uint32_t &hi, uint32_t &lo) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(x0, x1);
    const float2 hf = __bfloat1622float2(h);
    const __nv_bfloat162 l = __floats2bfloat162_rn(__fsub_rn(x0, hf.x), __fsub_rn(x1, hf.y));
    hi = *reinterpret_cast<const uint32_t *>(&h);
    lo = *reinterpret_cast<const uint32_t *>(&l);
}

// byte offset of 16-byte chunk ch of tile row `row` (128-byte rows, swizzled)
__device__ __forceinline__ uint32_t at_off(int row, int ch) { return row * 128 + ((ch ^ (row & 7)) << 4); }

// FEW: the few-row form (span split over blockIdx.z, early tile requests for
// one row); the many-row instance compiles without either.
template <bool FEW>
__global__ void __launch_bounds__(AT_WARPS * 32) attn_tc_kernel(const AttnParams a) {
    extern __shared__ __align__(128) uint8_t at_smem[];
    pdl_trigger();
    const int m = blockIdx.x, kh = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const __nv_bfloat16 *Kc = reinterpret_cast<const __nv_bfloat16 *>(a.kc);
    const __nv_bfloat16 *Vc = reinterpret_cast<const __nv_bfloat16 *>(a.vc);
    const int kvd = a.KVH * AT_HD;
    const int pos = a.row_pos[m];
    int end = pos;
    if (end >= a.ctx) end = a.ctx - 1;  // picchio.c:559-560
    int start = 0;
    if (a.window > 0) {
        start = end - a.window + 1;
        if (start < 0) start = 0;
    }
    const int64_t cache0 = (int64_t)a.row_seq[m] * a.seq_stride + kh * AT_HD;
    // this CTA's positions [r0, r1]: the whole row, or span blockIdx.z
    const int split = FEW && gridDim.z > 1, sp = FEW ? blockIdx.z : 0;
    const int nsp = split ? (end - start + AT_SPAN) / AT_SPAN : 1;
    if (sp >= nsp) return;  // uniform: spans past the row's positions
    const int r0 = start + sp * AT_SPAN;
    const int r1 = split ? min(end, r0 + AT_SPAN - 1) : end;
    const int ntiles = (r1 - r0 + AT_TILE) / AT_TILE;
    const int nloc = ntiles > warp ? (ntiles - warp + AT_WARPS - 1) / AT_WARPS : 0;
    uint8_t *wsm = at_smem + warp * 2 * AT_STAGE;

    auto issue = [&](int i) {  // this warp's i-th tile into stage i % 2
        const int p0 = r0 + AT_TILE * (warp + AT_WARPS * i);
        uint8_t *ks = wsm + (i & 1) * AT_STAGE, *vs = ks + AT_TILE_BYTES;
        for (int c = lane; c < AT_TILE * 8; c += 32) {
            const int row = c >> 3, ch = c & 7, p = p0 + row;
            const bool ok = p <= r1;
            const int64_t off = cache0 + (int64_t)(ok ? p : start) * kvd + ch * 8;
            cp_async16_zfill(ks + at_off(row, ch), Kc + off, ok ? 16 : 0);
            cp_async16_zfill(vs + at_off(row, ch), Vc + off, ok ? 16 : 0);
        }
        cp_async_commit();
    };
    // q and this step's K/V row come from the q/k/v kernel; with one row,
    // this warp's first tiles that end before the row's position (rows of
    // earlier steps) are requested before waiting for it
    int issued = 0;
    while (FEW && a.M == 1 && issued < 2 && issued < nloc &&
           min(r0 + AT_TILE * (warp + AT_WARPS * issued) + AT_TILE - 1, r1) < pos)
        issue(issued++);
    pdl_wait();
    if (issued == 0 && nloc > 0) issue(issued++);

    // Q of head g (A rows 0-7), dims 16 ks + 2t (+1) and 16 ks + 8 + 2t (+1)
    const float *q = a.q + (int64_t)m * a.H * AT_HD + (int64_t)(kh * AT_G + g) * AT_HD;
    uint32_t qh[4][2], ql[4][2];
#pragma unroll
    for (int ks = 0; ks < 4; ++ks)
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
            const float2 x = *reinterpret_cast<const float2 *>(q + ks * 16 + hf * 8 + 2 * t);
            split2(x.x, x.y, qh[ks][hf], ql[ks][hf]);
        }
    const float scale = __fdiv_rn(1.0f, sqrtf((float)AT_HD));
    float mrun = -INFINITY, lrun = 0.0f;
    float o[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int j = 0; j < 4; ++j) o[nt][j] = 0.0f;

    for (int i = 0; i < nloc; ++i) {
        if (i + 1 < nloc && i + 1 >= issued) issue(i + 1);
        else cp_async_commit();
        cp_async_wait<1>();
        __syncwarp();
        const uint32_t ks = smem_u32(wsm + (i & 1) * AT_STAGE), vs = ks + AT_TILE_BYTES;
        const int p0 = r0 + AT_TILE * (warp + AT_WARPS * i);
        // S = Q K^T: n-tile nt = positions 8 nt .. 8 nt + 7
        float s[8][4];
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
            for (int j = 0; j < 4; ++j) s[nt][j] = 0.0f;
#pragma unroll
            for (int kp = 0; kp < 2; ++kp) {  // dims 32 kp .. 32 kp + 31: k-steps 2 kp, 2 kp + 1
                uint32_t b[4];
                ldsm_x4(b, ks + at_off(nt * 8 + (lane & 7), kp * 4 + (lane >> 3)));
                mma8(s[nt], qh[2 * kp][0], qh[2 * kp][1], b[0], b[1]);
                mma8(s[nt], ql[2 * kp][0], ql[2 * kp][1], b[0], b[1]);
                mma8(s[nt], qh[2 * kp + 1][0], qh[2 * kp + 1][1], b[2], b[3]);
                mma8(s[nt], ql[2 * kp + 1][0], ql[2 * kp + 1][1], b[2], b[3]);
            }
        }
        // online softmax of head g over this tile (the quad t = 0..3 holds the row)
        float tmax = -INFINITY;
#pragma unroll
        for (int nt = 0; nt < 8; ++nt)
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const int p = p0 + nt * 8 + 2 * t + j;
                const float v = p <= r1 ? __fmul_rn(s[nt][j], scale) : -INFINITY;
                s[nt][j] = v;
                tmax = fmaxf(tmax, v);
            }
        tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 1));
        tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 2));
        const float mnew = fmaxf(mrun, tmax);  // finite: position p0 <= r1 is in the tile
        const float corr = expf(__fsub_rn(mrun, mnew));
        float psum = 0.0f;
#pragma unroll
        for (int nt = 0; nt < 8; ++nt)
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const float p = expf(__fsub_rn(s[nt][j], mnew));
                s[nt][j] = p;
                psum = __fadd_rn(psum, p);
            }
        psum = __fadd_rn(psum, __shfl_xor_sync(0xffffffffu, psum, 1));
        psum = __fadd_rn(psum, __shfl_xor_sync(0xffffffffu, psum, 2));
        lrun = __fmaf_rn(lrun, corr, psum);
        mrun = mnew;
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
            o[nt][0] = __fmul_rn(o[nt][0], corr);
            o[nt][1] = __fmul_rn(o[nt][1], corr);
        }
        // O += P V: k-step kk = positions 16 kk .. 16 kk + 15 (S n-tiles 2 kk, 2 kk + 1)
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
            uint32_t ph0, pl0, ph2, pl2;
            split2(s[2 * kk][0], s[2 * kk][1], ph0, pl0);
            split2(s[2 * kk + 1][0], s[2 * kk + 1][1], ph2, pl2);
#pragma unroll
            for (int nn = 0; nn < 4; ++nn) {  // dims 16 nn .. 16 nn + 15: O n-tiles 2 nn, 2 nn + 1
                uint32_t b[4];
                const int j = lane >> 3;
                ldsm_x4_t(b, vs + at_off(16 * kk + (lane & 7) + 8 * (j & 1), 2 * nn + (j >> 1)));
                mma8(o[2 * nn], ph0, ph2, b[0], b[1]);
                mma8(o[2 * nn], pl0, pl2, b[0], b[1]);
                mma8(o[2 * nn + 1], ph0, ph2, b[2], b[3]);
                mma8(o[2 * nn + 1], pl0, pl2, b[2], b[3]);
            }
        }
        __syncwarp();  // every lane is done with this stage before it is refilled
    }
    cp_async_wait<0>();

    // merge the warps with the sink
    float *mer = reinterpret_cast<float *>(at_smem + AT_WARPS * 2 * AT_STAGE);
    float *mw = mer + warp * AT_G * (AT_HD + 2) + g * (AT_HD + 2);  // [m, l, O[64]] of head g
    if (t == 0) {
        mw[0] = mrun;
        mw[1] = nloc > 0 ? lrun : 0.0f;
    }
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
        mw[2 + nt * 8 + 2 * t] = o[nt][0];
        mw[2 + nt * 8 + 2 * t + 1] = o[nt][1];
    }
    __syncthreads();
    constexpr int WREC = AT_G * (AT_HD + 2);
    if (!FEW || nsp == 1) {
        for (int idx = threadIdx.x; idx < AT_G * AT_HD; idx += AT_WARPS * 32) {
            const int gg = idx / AT_HD, d = idx % AT_HD, h = kh * AT_G + gg;
            float M = a.sinks ? a.sinks[h] : -INFINITY;
#pragma unroll
            for (int w = 0; w < AT_WARPS; ++w) M = fmaxf(M, mer[w * WREC + gg * (AT_HD + 2)]);
            float L = a.sinks ? expf(__fsub_rn(a.sinks[h], M)) : 0.0f;
            float O = 0.0f;
#pragma unroll
            for (int w = 0; w < AT_WARPS; ++w) {
                const float *rec = mer + w * WREC + gg * (AT_HD + 2);
                if (rec[1] != 0.0f) {
                    const float f = expf(__fsub_rn(rec[0], M));
                    L = __fmaf_rn(rec[1], f, L);
                    O = __fmaf_rn(rec[2 + d], f, O);
                }
            }
            a.out[(int64_t)m * a.H * AT_HD + h * AT_HD + d] = __fdiv_rn(O, L);
        }
        return;
    }
    // this span's (max, sum, O) per head, without the sink
    const int stride = AT_HD + 2;
    for (int idx = threadIdx.x; idx < AT_G * AT_HD; idx += AT_WARPS * 32) {
        const int gg = idx / AT_HD, d = idx % AT_HD, h = kh * AT_G + gg;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < AT_WARPS; ++w) M = fmaxf(M, mer[w * WREC + gg * (AT_HD + 2)]);
        float L = 0.0f, O = 0.0f;
#pragma unroll
        for (int w = 0; w < AT_WARPS; ++w) {
            const float *rec = mer + w * WREC + gg * (AT_HD + 2);
            if (rec[1] != 0.0f) {
                const float f = expf(__fsub_rn(rec[0], M));
                L = __fmaf_rn(rec[1], f, L);
                O = __fmaf_rn(rec[2 + d], f, O);
            }
        }
        float *out = a.part + (((int64_t)m * a.H + h) * a.nsplit + sp) * stride;
        out[2 + d] = O;
        if (d == 0) {
            out[0] = M;
            out[1] = L;
        }
    }
    __threadfence();
    __syncthreads();
    __shared__ bool lastf;
    if (threadIdx.x == 0) {
        unsigned *c = a.counter + m * a.KVH + kh;
        lastf = atomicAdd(c, 1u) == (unsigned)(nsp - 1);
        if (lastf) *c = 0u;
    }
    __syncthreads();
    if (!lastf) return;
    __threadfence();
    // merge the spans with the sink (picchio.c:586-596)
    for (int idx = threadIdx.x; idx < AT_G * AT_HD; idx += AT_WARPS * 32) {
        const int gg = idx / AT_HD, d = idx % AT_HD, h = kh * AT_G + gg;
        const float *rec0 = a.part + (((int64_t)m * a.H + h) * a.nsplit) * stride;
        float M = a.sinks ? a.sinks[h] : -INFINITY;
        for (int k = 0; k < nsp; ++k) M = fmaxf(M, __ldcg(rec0 + k * stride));
        float L = a.sinks ? expf(__fsub_rn(a.sinks[h], M)) : 0.0f;
        float O = 0.0f;
        for (int k = 0; k < nsp; ++k) {
            const float l = __ldcg(rec0 + k * stride + 1);
            if (l != 0.0f) {
                const float f = expf(__fsub_rn(__ldcg(rec0 + k * stride), M));
                L = __fmaf_rn(l, f, L);
                O = __fmaf_rn(__ldcg(rec0 + k * stride + 2 + d), f, O);
            }
        }
        a.out[(int64_t)m * a.H * AT_HD + h * AT_HD + d] = __fdiv_rn(O, L);
    }
}

}  // namespace

bool attention_tc_ok(const AttnParams &a) {
    const char *v = getenv("PICCHIO_ATTN_TC");  // 0: the one-row kernel for every step
    const bool off = v && v[0] == '0';
    return !off && a.kv_bf16 && a.hd == AT_HD && a.H == a.KVH * AT_G;
}

cudaError_t attention_tc_configure() {
    cudaError_t e = cudaFuncSetAttribute(attn_tc_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, AT_SMEM);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(attn_tc_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, AT_SMEM);
    return e;
}

cudaError_t launch_attention_tc(const AttnParams &a, cudaStream_t st) {
    // few rows: the positions split over CTAs too, in spans of 512 (the
    // partial records hold a.nsplit spans of 256, so at most that many)
    if (a.M >= ATTN_TC_MIN_ROWS)
        return launch_k(attn_tc_kernel<false>, dim3(a.M, a.KVH), dim3(AT_WARPS * 32), AT_SMEM, st, a);
    const int nz = std::max(1, (a.nsplit + 1) / 2);
    return launch_k(attn_tc_kernel<true>, dim3(a.M, a.KVH, nz), dim3(AT_WARPS * 32), AT_SMEM, st, a);
}

}  // namespace pc
