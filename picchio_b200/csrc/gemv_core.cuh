// gemv_core.cuh - the dequant-fused GEMV that streams INT4/INT8 weight tiles from
// HBM: matmul_qt (quant.h:323-337) for up to 8 input rows per matrix, with
// the MoE and attention epilogues fused.
//
// One persistent CTA of 12 warps per SM; a CTA owns a contiguous range of
// 16-row tiles ("units").  The 12 warps form G groups: with few units per CTA
// one group splits every unit's K 12 ways (all warps busy on small
// matrices); with many, up to 12 one-warp groups stream whole units (no
// cross-warp reduction at all).  Per warp:
//  * weights stream from HBM through a per-warp ring of shared-memory step
//    slots filled with cp.async: per step (up to 4 T4 or 8 T8 k-blocks of one
//    unit) every lane copies its 16-byte A fragment of each block and its
//    rows' group scales, R - 1 steps ahead of the step it computes;
//  * the MMAs are s8 x s8 -> s32 m16n8k32: a nibble n becomes the signed byte
//    16 (n - 8) in one or two logic ops, INT8 weights need nothing;
//  * the input rows are scaled by a power of two, rounded to 22-bit integers
//    and split into three signed byte digits (the B operand, built once per
//    job in shared memory), so every group sum is exact in s32 and is scaled
//    into an fp32 accumulator (acc += group_sum * scale), the structure of
//    matmul_i4_gs (quant.h:259-319).
// Partials of a K-split unit are summed in a fixed order (deterministic
// results) through a ring of shared slots: only the unit's epilogue warp waits
// for them, and it fetched the epilogue's operands one epilogue earlier.
// Dense launches carry their job table in the kernel parameters and start
// streaming weights before waiting on the previous kernel (programmatic
// dependent launch).
#pragma once
#include <cuda_bf16.h>

#include "gemv.h"
#include "launch.cuh"
#include "ptx.cuh"

namespace pc {

namespace {


constexpr int NCONS = GEMV_CONSUMERS;
constexpr int NCT = NCONS * 32;

constexpr int OFF_JP = 0;                                        // int[MAX_JOBS + 1]
constexpr int OFF_TILES = 4224;                                  // const uint8_t *[MAX_JOBS]
constexpr int OFF_JOBS = OFF_TILES + 8 * GEMV_MAX_JOBS;          // GemvJob[INLINE]
constexpr int OFF_META = OFF_JOBS + 128 * GEMV_INLINE_JOBS;
constexpr int OFF_RED = OFF_META + 640;
constexpr int NRED = 4;  // reduction slots per group when one group holds all 12 warps

static_assert(OFF_TILES >= OFF_JP + 4 * (GEMV_MAX_JOBS + 1), "job prefix region");
static_assert(sizeof(GemvJob) <= 128, "inline job slot");

struct SMeta {
    float scale[2][GEMV_MAXR];  // 2^sh per input row (double-buffered by job parity)
    float inv[2][GEMV_MAXR];    // 2^-sh (x 1/16 for INT4)
    int njobs;
    float part[GEMV_CONSUMERS][GEMV_MAXR];  // per-warp max |x| while B is built
};
static_assert(sizeof(SMeta) <= 640, "meta region");

__host__ __device__ inline int off_B(int nt) { return (OFF_RED + NRED * nt * NCONS * 256 + 127) & ~127; }
__host__ __device__ inline int off_ring(int nt, int Ip) { return (off_B(nt) + nt * Ip * 8 + 127) & ~127; }
// The warps' ring-slot mbarriers follow the rings (8-byte aligned: a ring
// slot is a multiple of 64 bytes).
__host__ __device__ inline int off_mbar(int fmt, int nt, int Ip, int blk_bytes) {
    return off_ring(nt, Ip) + NCONS * gemv_ring_depth(fmt, nt) * gemv_step_blocks(fmt, nt) * blk_bytes;
}
// Shared memory of one CTA: fixed regions, the B operand, the warps' rings
// and their mbarriers.
__host__ __device__ inline int gemv_smem_need(int fmt, int nt, int Ip, int blk_bytes) {
    return off_mbar(fmt, nt, Ip, blk_bytes) + NCONS * gemv_ring_depth(fmt, nt) * 8;
}
// Bound on one wait for a ring slot's bulk copy (far above any real copy).
constexpr unsigned long long GEMV_WAIT_NS = 1000000000ull;
constexpr int GEMV_ERR_WAIT = 4;  // error word value when that wait gives up

__device__ __forceinline__ unsigned long long gemv_now() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// 1-D bulk copy global -> shared completing on bar (transaction bytes); no
// multicast.  Both addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void gemv_bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}
// A step copied by the lanes with cp.async (tiles that may sit in mapped
// host memory, streamed residency), arriving on bar.  Out of line: kept off
// the resident path's code, which is bound by instruction fetch in short
// launches (bs64 decode +1.2 %, bs1 +0.4 %).
__device__ __noinline__ void gemv_lanes_copy(uint8_t *dst, const uint8_t *src, int nb, int BB, int sbytes, int lane,
                                             uint64_t *bar) {
    for (int i = 0; i < nb; ++i) {
        cp_async16(dst + i * BB + lane * 16, src + (size_t)i * BB + lane * 16);
        if (lane * 16 < sbytes) cp_async16(dst + i * BB + 512 + lane * 16, src + (size_t)i * BB + 512 + lane * 16);
    }
    cp_async_mbar_arrive(bar);
}
// Bounded wait for phase `parity` of bar; false when the bound ran out.
__device__ __forceinline__ bool gemv_mbar_wait(uint64_t *bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = gemv_now();
    while (!mbar_try_wait(bar, parity))
        if (gemv_now() - t0 > GEMV_WAIT_NS) return false;
    return true;
}

// Signed digits of v (|v| <= 2^22): v = hi * 2^16 + mid * 2^8 + lo with
// lo, mid in [-128, 127] and |hi| <= 64.
__device__ __forceinline__ void digits3(int v, int &hi, int &mid, int &lo) {
    lo = ((v + 128) & 255) - 128;
    const int v1 = (v - lo) >> 8;
    mid = ((v1 + 128) & 255) - 128;
    hi = (v1 - mid) >> 8;
}

__device__ __forceinline__ uint32_t pack_s8x4(int a, int b, int c, int d) {
    return (uint32_t)(a & 255) | ((uint32_t)(b & 255) << 8) | ((uint32_t)(c & 255) << 16) | ((uint32_t)(d & 255) << 24);
}

__device__ __forceinline__ unsigned long long argmax_key(float v, int idx) {
    if (v != v) return 0ull;  // NaN never wins (picchio.c:1558 uses '>')
    if (v == 0.0f) v = 0.0f;  // -0 and +0 compare equal
    uint32_t u = __float_as_uint(v);
    uint32_t key = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)key << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)idx);
}

__device__ __forceinline__ float swiglu(float gate, float up, float limit, float alpha) {
    // picchio.c:1418-1423: gate = min(gate, lim); up = clamp(up, +-lim);
    // (up + 1) * gate * sigmoid(alpha * gate), sigmoid = 1 / (1 + expf(-x)).
    if (gate > limit) gate = limit;
    if (up > limit) up = limit;
    if (up < -limit) up = -limit;
    float sg = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-__fmul_rn(alpha, gate))));
    return __fmul_rn(__fmul_rn(__fadd_rn(up, 1.0f), gate), sg);
}

// Shift sh of an input row with max |x| = m: 22 - E where m = f 2^E, f in
// [0.5, 1) (frexpf), at most 126; 0 for a zero or non-finite row.  The
// exponent is read from the bits for normal m.
__device__ __forceinline__ int row_shift(float m) {
    if (!(m > 0.0f && m <= 3.4e38f)) return 0;
    const uint32_t b = __float_as_uint(m);
    int E;
    if (b >= 0x00800000u) E = (int)(b >> 23) - 126;
    else frexpf(m, &E);
    return min(126, 22 - E);
}
// 2^e for -126 <= e <= 127 (exact, what ldexpf(1, e) returns)
__device__ __forceinline__ float pow2i(int e) { return __int_as_float((e + 127) << 23); }

// Builds the input-row (B) operand of the s8 MMAs for input rows
// rows[0..n) in shared memory, once per job.  Row r is scaled by 2^sh, sh =
// 22 - (exponent of its max |x|), rounded to an integer v (|v| <= 2^22, the
// rounding error is below 2^-22 of the row's max) and split into three signed
// digits.  N-tile nt carries rows 2nt and 2nt + 1: MMA column n = 4 (r & 1) +
// d holds digit d (hi, mid, lo, zero) of row 2nt + (n >> 2).  Entry (nt,
// k-block, lane) is CPB pairs (b0, b1) of 4-digit words, one per 32-column
// MMA step of the block (CPB = 2 for T4 blocks, 1 for T8).
// Pass 1: every warp takes the max |x| of its twelfth of each row; pass 2:
// each thread rounds 8 values of one row for one lane column t and
// writes the 4 digit lanes of that row, four items per round so their loads
// overlap.
template <int NT, int CPB, int INV>
__device__ void fill_B(const GemvParams &p, const int *rows, int n, SMeta *meta, int mb, uint2 *Bsm,
                       int cw, int lane, int ctid) {
    const int nrows = min(n, NT * 2);
    const int nch = p.Ip / 32;          // 32-column MMA steps
    const int total = NT * nch * 8;     // items: (nt, step, row of the n-tile, t)
    const bool al4 = (p.ldx & 3) == 0;
    // Each item's 8 values, loaded all at once.
    auto load_item = [&](int idx, float (&v)[8], int &r) {
        const int t = idx & 3, rr = (idx >> 2) & 1, kc = (idx >> 3) % nch, nt = idx / (8 * nch);
        r = nt * 2 + rr;
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = 0.0f;
        if (idx < total && r < nrows) {
            const float *xr = p.x + (int64_t)rows[r] * p.ldx;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int k = kc * 32 + 16 * h + 4 * t;
                if (al4 && k + 3 < p.I) {
                    const float4 f = *reinterpret_cast<const float4 *>(xr + k);
                    v[4 * h + 0] = f.x;
                    v[4 * h + 1] = f.y;
                    v[4 * h + 2] = f.z;
                    v[4 * h + 3] = f.w;
                } else {
#pragma unroll
                    for (int j = 0; j < 4; ++j) v[4 * h + j] = k + j < p.I ? xr[k + j] : 0.0f;
                }
            }
        }
    };
    auto store_item = [&](int idx, const float (&v)[8], float sc) {
        const int t = idx & 3, rr = (idx >> 2) & 1, kc = (idx >> 3) % nch, nt = idx / (8 * nch);
        int hi[8], mi[8], lo[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) digits3(__float2int_rn(__fmul_rn(v[i], sc)), hi[i], mi[i], lo[i]);
        // lanes 4g + t, g = 4 rr + d
        uint2 *e = Bsm + ((int64_t)(nt * p.kblocks + kc / CPB) * 32 + 16 * rr + t) * CPB + kc % CPB;
        e[0 * 4 * CPB] = make_uint2(pack_s8x4(hi[0], hi[1], hi[2], hi[3]), pack_s8x4(hi[4], hi[5], hi[6], hi[7]));
        e[1 * 4 * CPB] = make_uint2(pack_s8x4(mi[0], mi[1], mi[2], mi[3]), pack_s8x4(mi[4], mi[5], mi[6], mi[7]));
        e[2 * 4 * CPB] = make_uint2(pack_s8x4(lo[0], lo[1], lo[2], lo[3]), pack_s8x4(lo[4], lo[5], lo[6], lo[7]));
        e[3 * 4 * CPB] = make_uint2(0u, 0u);
    };
    auto scale_of = [&](int r) {  // sh of row r from the per-warp maxima
        float m = 0.0f;
#pragma unroll
        for (int w = 0; w < NCONS; ++w) m = fmaxf(m, meta->part[w][r]);
        return row_shift(m);
    };
    constexpr int IPT = 4;  // items per thread for the one-pass form
    if (total <= IPT * NCT) {
        // one pass: load every item, take per-row maxima, then round from registers
        float v[IPT][8];
        int rq[IPT];
#pragma unroll
        for (int q = 0; q < IPT; ++q) load_item(ctid + q * NCT, v[q], rq[q]);
        float mr[2 * NT];
#pragma unroll
        for (int r = 0; r < 2 * NT; ++r) mr[r] = 0.0f;
#pragma unroll
        for (int q = 0; q < IPT; ++q) {
            float lm = 0.0f;
#pragma unroll
            for (int i = 0; i < 8; ++i) lm = fmaxf(lm, fabsf(v[q][i]));
#pragma unroll
            for (int r = 0; r < 2 * NT; ++r)
                if (rq[q] == r) mr[r] = fmaxf(mr[r], lm);
        }
#pragma unroll
        for (int r = 0; r < 2 * NT; ++r) {
            float m = mr[r];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            if (lane == 0) meta->part[cw][r] = m;
        }
        named_bar_sync(1, NCT);
        // every warp folds the NCONS per-warp maxima itself (lane w reads
        // warp w's): no second barrier, one shift per row
        int sh[2 * NT];
#pragma unroll
        for (int r = 0; r < 2 * NT; ++r) {
            float m = lane < NCONS ? meta->part[lane][r] : 0.0f;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            sh[r] = row_shift(m);
        }
#pragma unroll
        for (int r = 0; r < 2 * NT; ++r)
            if (ctid == r && r < nrows) {
                meta->scale[mb][r] = pow2i(sh[r]);
                // removes 2^sh and, for INT4, the factor 16 of the s8 nibble values
                meta->inv[mb][r] = ldexpf(1.0f, -sh[r] - INV);
            }
#pragma unroll
        for (int q = 0; q < IPT; ++q) {
            const int idx = ctid + q * NCT;
            float sc = 1.0f;
#pragma unroll
            for (int r = 0; r < 2 * NT; ++r)
                if (rq[q] == r && r < nrows) sc = pow2i(sh[r]);
            if (idx < total) store_item(idx, v[q], sc);
        }
        named_bar_sync(1, NCT);
        return;
    }
    // two passes (many input rows): every warp takes the max |x| of its twelfth of each row
    {
        const bool v4 = (p.ldx & 3) == 0 && (p.I & 3) == 0;
        const int n4 = v4 ? p.I >> 2 : p.I;
        const int k0 = n4 * cw / NCONS, k1 = n4 * (cw + 1) / NCONS;
        for (int r = 0; r < nrows; ++r) {
            const float *xr = p.x + (int64_t)rows[r] * p.ldx;
            float m = 0.0f;
            for (int k = k0 + lane; k < k1; k += 32) {
                if (v4) {
                    const float4 f = reinterpret_cast<const float4 *>(xr)[k];
                    m = fmaxf(m, fmaxf(fmaxf(fabsf(f.x), fabsf(f.y)), fmaxf(fabsf(f.z), fabsf(f.w))));
                } else {
                    m = fmaxf(m, fabsf(xr[k]));
                }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            if (lane == 0) meta->part[cw][r] = m;
        }
    }
    named_bar_sync(1, NCT);
    if (ctid < nrows) {
        const int sh = scale_of(ctid);
        meta->scale[mb][ctid] = pow2i(sh);
        meta->inv[mb][ctid] = ldexpf(1.0f, -sh - INV);
    }
    // pass 2: each thread rounds four items per round so their loads overlap
    for (int base = ctid; base < total; base += 4 * NCT) {
        float v[4][8];
        int rq[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) load_item(base + q * NCT, v[q], rq[q]);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int idx = base + q * NCT;
            if (idx < total) store_item(idx, v[q], rq[q] < nrows ? pow2i(scale_of(rq[q])) : 1.0f);
        }
    }
    named_bar_sync(1, NCT);
}

// One lane's weight bytes of one k-block: its 16-byte A fragment and the
// group scales of its two rows (gs32: 4 floats; gs64: 2 in s.x, s.y; gs16: 8
// in s, s2).  Fields a format does not use are never set and cost nothing.
struct BlkRegs {
    uint4 a, s, s2;
};

template <int FMT, int GS>
__device__ __forceinline__ void load_blk(BlkRegs &r, const uint8_t *blk, int lane) {
    const int g = lane >> 2;
    r.a = ldg_stream(blk + lane * 16);
    if (tf_4bit(FMT) && GS == 32) {
        r.s = ldg_stream(blk + 512 + g * 16);
    } else if (FMT == TF_T4 && GS == 64) {
        const uint2 v = ldg_stream2(blk + 512 + g * 8);
        r.s.x = v.x;
        r.s.y = v.y;
    } else if (FMT == TF_T4 && GS == 16) {
        r.s = ldg_stream(blk + 512 + g * 32);
        r.s2 = ldg_stream(blk + 512 + g * 32 + 16);
    }
}

// The grouped form: acc[0] (row g), acc[2] (row g + 8) += group scale *
// (wi * d_even + d_odd), the lane's two digit columns joined in s32 first
// (wi = 256 where they are (hi, mid), 1 where they are (lo, zero): below
// 2^28 in magnitude, exact), so a group costs two int-to-float conversions instead of four.
__device__ __forceinline__ void scale2(float (&acc)[4], const int (&d)[4], uint32_t s_g, uint32_t s_g8, int wi) {
    acc[0] = __fmaf_rn(__int2float_rn(d[0] * wi + d[1]), __uint_as_float(s_g), acc[0]);
    acc[2] = __fmaf_rn(__int2float_rn(d[2] * wi + d[3]), __uint_as_float(s_g8), acc[2]);
}

// The same from a block staged in shared memory.
template <int FMT, int GS>
__device__ __forceinline__ void load_blk_smem(BlkRegs &r, const uint8_t *blk, int lane) {
    const int g = lane >> 2;
    r.a = *reinterpret_cast<const uint4 *>(blk + lane * 16);
    if (tf_4bit(FMT) && GS == 32) {
        r.s = *reinterpret_cast<const uint4 *>(blk + 512 + g * 16);
    } else if (FMT == TF_T4 && GS == 64) {
        const uint2 v = *reinterpret_cast<const uint2 *>(blk + 512 + g * 8);
        r.s.x = v.x;
        r.s.y = v.y;
    } else if (FMT == TF_T4 && GS == 16) {
        r.s = *reinterpret_cast<const uint4 *>(blk + 512 + g * 32);
        r.s2 = *reinterpret_cast<const uint4 *>(blk + 512 + g * 32 + 16);
    }
}

// One T4 block (64 columns = two s8 MMA steps) of one lane.  Grouped scales:
// each group's sum is exact in s32 and is scaled into the fp32 accumulator
// acc, the structure of matmul_i4_gs (quant.h:259-319); per-row scale (GS 0):
// sums stay in the s32 accumulator ia.
// Four E2M1 codes (bits 0-15 of s, code j in bits 4j..4j+3) -> four signed
// bytes holding 2x their values: byte permutes into the magnitude table
// {0, 1, 2, 3, 4, 6, 8, 12} and its negation, then a permute picking, per
// byte, the one the code's sign bit names (so code 8, -0, gives 0).
__device__ __forceinline__ uint32_t e2m1x4_s8(uint32_t s) {
    const uint32_t idx = s & 0x7777u;
    const uint32_t mag = prmt(0x03020100u, 0x0C080604u, idx);
    const uint32_t neg = prmt(0xFDFEFF00u, 0xF4F8FAFCu, idx);
    return prmt(mag, neg, ((s >> 1) & 0x4444u) | 0x3210u);
}

// The A fragments of one 4-bit block for the two MMA steps: INT4 nibbles n
// become 16 (n - 8); MXFP4 codes become 2 x their E2M1 value.
template <int FMT>
__device__ __forceinline__ void a_frags4(const uint4 &a, uint32_t (&a0)[4], uint32_t (&a1)[4]) {
    if (FMT == TF_F4) {
        a0[0] = e2m1x4_s8(a.x); a0[1] = e2m1x4_s8(a.x >> 16); a0[2] = e2m1x4_s8(a.y); a0[3] = e2m1x4_s8(a.y >> 16);
        a1[0] = e2m1x4_s8(a.z); a1[1] = e2m1x4_s8(a.z >> 16); a1[2] = e2m1x4_s8(a.w); a1[3] = e2m1x4_s8(a.w >> 16);
    } else {
        a0[0] = nib_lo_s8(a.x); a0[1] = nib_hi_s8(a.x); a0[2] = nib_lo_s8(a.y); a0[3] = nib_hi_s8(a.y);
        a1[0] = nib_lo_s8(a.z); a1[1] = nib_hi_s8(a.z); a1[2] = nib_lo_s8(a.w); a1[3] = nib_hi_s8(a.w);
    }
}

template <int FMT, int NT, int GS>
__device__ __forceinline__ void block_t4(const BlkRegs &r, const uint4 (&B)[NT], float (&acc)[NT][4],
                                         int (&ia)[NT][4], int wi) {
    uint32_t a0[4], a1[4];
    a_frags4<FMT>(r.a, a0, a1);
    const int M[4] = {0, 0, 0, 0};
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        int d[4];
        if (GS == 32) {
            mma_s8_16832(d, a0, B[nt].x, B[nt].y, M);
            scale2(acc[nt], d, r.s.x, r.s.y, wi);
            mma_s8_16832(d, a1, B[nt].z, B[nt].w, M);
            scale2(acc[nt], d, r.s.z, r.s.w, wi);
        } else if (GS == 64) {
            mma_s8_16832(d, a0, B[nt].x, B[nt].y, M);
            mma_s8_16832(d, a1, B[nt].z, B[nt].w, d);
            scale2(acc[nt], d, r.s.x, r.s.y, wi);
        } else if (GS == 16) {  // one group per 16 columns: the other half of B is zero
            mma_s8_16832(d, a0, B[nt].x, 0u, M);
            scale2(acc[nt], d, r.s.x, r.s.y, wi);
            mma_s8_16832(d, a0, 0u, B[nt].y, M);
            scale2(acc[nt], d, r.s.z, r.s.w, wi);
            mma_s8_16832(d, a1, B[nt].z, 0u, M);
            scale2(acc[nt], d, r.s2.x, r.s2.y, wi);
            mma_s8_16832(d, a1, 0u, B[nt].w, M);
            scale2(acc[nt], d, r.s2.z, r.s2.w, wi);
        } else {
            mma_s8_16832(ia[nt], a0, B[nt].x, B[nt].y, ia[nt]);
            mma_s8_16832(ia[nt], a1, B[nt].z, B[nt].w, ia[nt]);
        }
    }
}

// One T8 block (32 columns = one s8 MMA step) of one lane; INT8 is always
// per-row scaled, so the sums stay in the s32 accumulator.
template <int NT>
__device__ __forceinline__ void block_t8(const BlkRegs &r, const uint2 (&B)[NT], int (&ia)[NT][4]) {
    const uint32_t a[4] = {r.a.x, r.a.y, r.a.z, r.a.w};
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) mma_s8_16832(ia[nt], a, B[nt].x, B[nt].y, ia[nt]);
}

// Per-lane epilogue operands of one row tile, fetched by the warp that will
// run that tile's epilogue NCONS tiles ahead of time, so their global-load
// latency never sits on the critical path.  Slot k covers input row 2k + (t >> 1).
template <int NT>
struct EpiPre {
    int rt, mb, O, seg, has_rs, has_b;
    float rs[2], b[2];
    int lrow[2];
    int jr[NT];  // job row whose B column is this slot's, or -1
    int out[NT], pos[NT], seq[NT];
    float cs[NT], sn[NT];
    float res[NT][2];  // residual values (EPI_STORE with residual)
};

template <int NT>
__device__ __forceinline__ void epi_prefetch(const GemvParams &p, const GemvJob &job, int rt, int mb, int lane,
                                             EpiPre<NT> &e) {
    const int g = lane >> 2, t = lane & 3;
    e.rt = rt;
    e.mb = mb;
    e.O = job.O;
    e.seg = job.seg;
    e.has_rs = job.rs != nullptr;
    e.has_b = job.bias != nullptr;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int o = tile_row_to_logical(p.perm, p.head_dim, rt, g + 8 * h);
        e.lrow[h] = o;
        const bool ok = o < job.O;
        e.rs[h] = (ok && job.rs) ? job.rs[o] : 1.0f;
        e.b[h] = (ok && job.bias) ? job.bias[o] : 0.0f;
    }
    const int nrows = min(job.nrows, NT * 2);
#pragma unroll
    for (int k = 0; k < NT; ++k) {
        const int col = k * 2 + (t >> 1);  // input row (B row) of this lane; odd t repeat even t
        int jr = -1;
        if (t & 1) {
        } else if (p.shared_rows > 0) {
            for (int r = 0; r < nrows; ++r)
                if (job.in_row[r] == col) jr = r;
        } else if (col < nrows) {
            jr = col;
        }
        e.jr[k] = jr;
        e.out[k] = jr >= 0 ? job.out_row[jr] : 0;
        e.pos[k] = 0;
        e.seq[k] = 0;
        e.cs[k] = 1.0f;
        e.sn[k] = 0.0f;
        e.res[k][0] = e.res[k][1] = 0.0f;
        if (p.epi == EPI_STORE && p.residual && jr >= 0) {
#pragma unroll
            for (int h = 0; h < 2; ++h)
                if (e.lrow[h] < job.O)
                    e.res[k][h] = (p.res_src ? p.res_src : p.y)[(int64_t)e.out[k] * p.ldy + e.lrow[h]];
        }
        if (p.epi == EPI_QKV && jr >= 0) {
            const int xrow = p.shared_rows > 0 ? col : job.in_row[jr];
            e.pos[k] = p.row_pos[xrow];
            e.seq[k] = p.row_seq[xrow];
            if (job.seg != 2) {
                const int half = p.head_dim >> 1, j = e.lrow[0] % p.head_dim;
                e.cs[k] = p.rope_cs[(int64_t)e.pos[k] * half + j];
                e.sn[k] = p.rope_sn[(int64_t)e.pos[k] * half + j];
            }
        }
    }
}

// Writes one lane's results of one row tile from the summed partials v.
template <int NT>
__device__ void epilogue(const GemvParams &p, const SMeta *meta, const EpiPre<NT> &e, float (&v)[NT][2],
                         int lane) {
    const int g = lane >> 2, t = lane & 3;
    const int rt = e.rt;
#pragma unroll
    for (int k = 0; k < NT; ++k) {
        float v0 = v[k][0], v1 = v[k][1];
        const bool live = e.jr[k] >= 0;
        if (live) {
            const float inv = meta->inv[e.mb][k * 2 + (t >> 1)];
            v0 = __fmul_rn(v0, inv);
            v1 = __fmul_rn(v1, inv);
        }
        if (p.epi == EPI_SWIGLU) {
            const int pr = rt * 8 + g;  // pair index
            if (!live || 2 * pr + 1 >= e.O) continue;
            float gate = v0, up = v1;
            if (e.has_rs) { gate = __fmul_rn(gate, e.rs[0]); up = __fmul_rn(up, e.rs[1]); }
            if (e.has_b) { gate = __fadd_rn(gate, e.b[0]); up = __fadd_rn(up, e.b[1]); }
            p.y[(int64_t)e.out[k] * p.ldy + pr] = swiglu(gate, up, p.swiglu_limit, p.swiglu_alpha);
        } else if (p.epi == EPI_QKV) {
            const int olo = e.lrow[0], ohi = e.lrow[1];
            if (!live || ohi >= e.O) continue;
            float lo = v0, hi = v1;
            if (e.has_rs) { lo = __fmul_rn(lo, e.rs[0]); hi = __fmul_rn(hi, e.rs[1]); }
            if (e.has_b) { lo = __fadd_rn(lo, e.b[0]); hi = __fadd_rn(hi, e.b[1]); }
            const int pos = e.pos[k];
            if (e.seg != 2) {
                // rope_apply (picchio.c:467-469) as the reference build rounds it:
                // a*cs - b*sn -> fma(a, cs, -(b*sn)); a*sn + b*cs -> fma(a, sn, b*cs).
                const float a = lo, b = hi, cs = e.cs[k], sn = e.sn[k];
                lo = __fmaf_rn(a, cs, -__fmul_rn(b, sn));
                hi = __fmaf_rn(a, sn, __fmul_rn(b, cs));
            }
            if (e.seg == 0) {
                float *q = p.qbuf + (int64_t)e.out[k] * p.ldq;
                q[olo] = lo;
                q[ohi] = hi;
            } else if (pos >= 0 && pos < p.kv_ctx) {  // kv_store drops pos >= max_pos (picchio.c:495)
                const int64_t base = (int64_t)e.seq[k] * p.kv_seq_stride + (int64_t)pos * p.kv_dim;
                void *cache = e.seg == 1 ? p.kcache : p.vcache;
                if (p.kv_bf16) {
                    __nv_bfloat16 *c = reinterpret_cast<__nv_bfloat16 *>(cache);
                    c[base + olo] = __float2bfloat16_rn(lo);
                    c[base + ohi] = __float2bfloat16_rn(hi);
                } else {
                    float *c = reinterpret_cast<float *>(cache);
                    c[base + olo] = lo;
                    c[base + ohi] = hi;
                }
            }
        } else {  // EPI_STORE, EPI_LOGITS
            unsigned long long best = 0ull;
#pragma unroll
            for (int hlf = 0; hlf < 2; ++hlf) {
                const int o = e.lrow[hlf];
                if (!live || o >= e.O) continue;
                float x = hlf ? v1 : v0;
                if (e.has_rs) x = __fmul_rn(x, e.rs[hlf]);
                if (e.has_b) x = __fadd_rn(x, e.b[hlf]);
                float *dst = p.y + (int64_t)e.out[k] * p.ldy + o;
                if (p.epi == EPI_STORE && p.residual) x = __fadd_rn(e.res[k][hlf], x);
                *dst = x;
                if (p.epi == EPI_LOGITS) {
                    const unsigned long long kk = argmax_key(x, o);
                    best = kk > best ? kk : best;
                }
            }
            if (p.epi == EPI_LOGITS) {
                // lanes with the same t hold the same input row: reduce over g (lane bits 2..4)
#pragma unroll
                for (int o = 4; o < 32; o <<= 1) {
                    const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
                    best = other > best ? other : best;
                }
                if (g == 0 && live && best) atomicMax(p.argmax + e.out[k], best);
            }
        }
    }
}

__device__ __forceinline__ int job_of(const int *jp, int u, int j) {
    while (u >= jp[j + 1]) ++j;
    return j;
}

constexpr int BAR_FILL = 1;  // named barrier 1: all threads (B refills); 2..15: group reductions

// FMT: TF_T4 / TF_F4 / TF_T8; NT: 1 or 2 N-tiles (<= 4 or <= 8 input rows); GS:
// INT4 group size (0 = per row).
// The GEMV work of one CTA (index cta of ncta) over the job list of p.  PDL:
// the launch is a programmatic dependent launch (gemv_kernel); MBX > 0
// overrides the blocks per ring step.
template <int FMT, int NT, int GS, bool PDL, int MBX = 0>
__device__ __forceinline__ void gemv_cta(const GemvParams &p, uint8_t *smem, int cta, int ncta) {
    constexpr int CPB = tf_4bit(FMT) ? 2 : 1;  // 32-column MMA steps per block
    // weight values in the MMA are 16 (n - 8) for INT4 and 2 x E2M1 for MXFP4:
    // the extra power of two the epilogue removes
    constexpr int INV = FMT == TF_T4 ? 4 : FMT == TF_F4 ? 1 : 0;
    constexpr int MB = MBX > 0 ? MBX : gemv_step_blocks(FMT, NT);  // blocks per step
    constexpr int R = gemv_ring_depth(FMT, NT);  // steps per warp ring (R - 1 in flight)
    int *jp = reinterpret_cast<int *>(smem + OFF_JP);
    const uint8_t **stiles = reinterpret_cast<const uint8_t **>(smem + OFF_TILES);
    GemvJob *sjobs = reinterpret_cast<GemvJob *>(smem + OFF_JOBS);
    SMeta *meta = reinterpret_cast<SMeta *>(smem + OFF_META);
    uint2 *Bsm = reinterpret_cast<uint2 *>(smem + off_B(NT));

    const int cw = threadIdx.x >> 5, lane = threadIdx.x & 31, ctid = threadIdx.x;
    const bool inl = p.n_inline > 0;

    if (inl) {  // job table from the launch parameters (static indices only)
        if (cw == 0) {
#pragma unroll
            for (int j = 0; j < GEMV_INLINE_JOBS; ++j)
                if (j < p.n_inline && lane == 0) {
                    sjobs[j] = p.ijobs[j];
                    stiles[j] = p.ijobs[j].tiles;
                }
        }
        if (ctid == 32) {
            int run = 0;
            jp[0] = 0;
#pragma unroll
            for (int j = 0; j < GEMV_INLINE_JOBS; ++j)
                if (j < p.n_inline) { run += p.ijobs[j].n_rt; jp[j + 1] = run; }
            meta->njobs = p.n_inline;
        }
    } else if (cw == 0) {  // prefix sum of row tiles over the device job table
        // A table written by the previous kernel needs the dependency wait.
        // One written two or more kernels back (jobs_early) is complete once
        // this grid runs: the kernel in between triggered this launch only
        // after its own wait, which returned when the writer had finished.
        // It is read through L2 (no line an older kernel left in L1).
        const bool early = p.jobs_early != 0;
        if (PDL && !p.static_jobs && !early) pdl_wait();
        int nj = early ? __ldcg(p.njobs) : *p.njobs;
        nj = nj < 0 ? 0 : (nj > GEMV_MAX_JOBS ? GEMV_MAX_JOBS : nj);
        int run = 0;
        for (int base = 0; base < nj; base += 32) {
            int v = 0;
            if (base + lane < nj) {
                const GemvJob *jb = p.jobs + base + lane;
                if (early) {
                    v = __ldcg(&jb->n_rt);
                    stiles[base + lane] = reinterpret_cast<const uint8_t *>(
                        __ldcg(reinterpret_cast<const unsigned long long *>(&jb->tiles)));
                } else {
                    v = jb->n_rt;
                    stiles[base + lane] = jb->tiles;
                }
            }
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int n = __shfl_up_sync(0xffffffffu, v, o);
                if (lane >= o) v += n;
            }
            if (base + lane < nj) jp[base + lane + 1] = run + v;
            run += __shfl_sync(0xffffffffu, v, 31);
        }
        if (lane == 0) {
            jp[0] = 0;
            meta->njobs = nj;
        }
    }
    __syncthreads();
    if (PDL) pdl_trigger();
    const GemvJob *jobs = inl ? sjobs : p.jobs;
    const int nj = meta->njobs;
    const int64_t U = jp[nj];
    const int u0 = (int)(U * cta / ncta), u1 = (int)(U * (cta + 1) / ncta);
    if (u0 >= u1) return;
    const int nunits = u1 - u0;
    const int BB = p.blk_bytes;
    const int j0 = job_of(jp, u0, 0);

    // G groups of wpu warps.  In every job segment of this CTA's range, group
    // gi takes units lo + gi, lo + gi + G, ...; warp wi of a group takes the
    // contiguous k-blocks [kb0, kb0 + nbw) of each of them.  Few units per CTA
    // -> one group splitting K 12 ways (all warps busy); many -> up to 12
    // groups of one warp, each streaming whole units with no reduction.
    const int G = nunits >= 24 ? 12 : nunits >= 12 ? 6 : nunits >= 8 ? 4 : nunits >= 6 ? 3 : nunits >= 4 ? 2 : 1;
    const int wpu = NCONS / G, gi = cw / wpu, wi = cw - gi * wpu;
    const int NS = G == 1 ? NRED : G == 2 ? 3 : G == 3 ? 2 : 1;  // reduction slots per group (2 barriers each)
    const int kb0 = p.kblocks * wi / wpu, nbw = p.kblocks * (wi + 1) / wpu - kb0;
    const int need = (p.kblocks + wpu - 1) / wpu;
    const int nch = (need + MB - 1) / MB;  // steps per unit
    auto step_blocks = [&](int c) { return max(0, min(MB, nbw - c * MB)); };

    // this group's unit sequence, across the job segments of [u0, u1)
    auto seg_lo = [&](int j) { return max(u0, jp[j]); };
    auto seg_hi = [&](int j) { return min(u1, jp[j + 1]); };
    auto first_from = [&](int j, int &u, int &jj) {
        for (; j < nj; ++j) {
            const int lo = seg_lo(j), hi = seg_hi(j);
            if (lo + gi < hi) { u = lo + gi; jj = j; return; }
            if (hi >= u1) break;
        }
        u = u1;
        jj = nj;
    };
    auto advance = [&](int &u, int &jj) {
        if (u + G < seg_hi(jj)) u += G;
        else first_from(jj + 1, u, jj);
    };
    int ntot = 0;  // this group's units
    for (int j = j0; j < nj; ++j) {
        const int lo = seg_lo(j), hi = seg_hi(j);
        if (lo + gi < hi) ntot += (hi - lo - gi + G - 1) / G;
        if (hi >= u1) break;
    }
    auto slice = [&](int u, int jj) {  // this warp's bytes of unit u
        return stiles[jj] + ((int64_t)(u - jp[jj]) * p.kblocks + kb0) * BB;
    };
    // HBM latency is covered by the warps' rings alone (R - 1 steps in flight
    // per warp).  Measured in the decode step: L2 prefetches of the next units
    // on top of them made every launch slower (their flood of requests
    // delays the latency-critical loads after the dependency wait: the input
    // row, the epilogue operands), the lm_head by 40 %.
    //
    // This warp's ring of R step slots in shared memory: a step's blocks are
    // contiguous in global memory, so lane 0 fetches each step with one bulk
    // copy (the TMA engine, not the load/store pipeline) completing on the
    // slot's mbarrier; step s lives in slot s % R; R - 1 steps are in flight
    // behind the one being computed.  Tiles that may sit in mapped host
    // memory (streamed residency) are copied by the lanes with cp.async
    // instead, each lane's copies arriving on the same mbarrier.
    uint8_t *myring = smem + off_ring(NT, p.Ip) + (size_t)cw * R * MB * BB;
    uint64_t *mybar = reinterpret_cast<uint64_t *>(smem + off_ring(NT, p.Ip) + (size_t)NCONS * R * MB * BB) + cw * R;
    const bool lanes_copy = p.host_tiles != 0;
    if (lane < R) mbar_init(mybar + lane, lanes_copy ? 32 : 1);
    fence_mbar_init();
    __syncwarp();
    const int sbytes = BB - 512;  // group-scale bytes per block (T4 with groups)
    int ld_u, ld_j, ld_c = 0, ld_seq = 0;
    first_from(j0, ld_u, ld_j);
    auto issue_step = [&]() {  // copies step (ld_u, ld_c), then moves the cursor on
        if (ld_u < u1) {
            const int nb = step_blocks(ld_c);
            uint64_t *bar = mybar + ld_seq % R;
            uint8_t *dst = myring + (size_t)(ld_seq % R) * MB * BB;
            const uint8_t *src = slice(ld_u, ld_j) + (size_t)ld_c * MB * BB;
            if (lanes_copy) {
                gemv_lanes_copy(dst, src, nb, BB, sbytes, lane, bar);
            } else if (lane == 0) {
                if (nb > 0) {
                    mbar_arrive_expect_tx(bar, (uint32_t)(nb * BB));
                    gemv_bulk_load(dst, src, (uint32_t)(nb * BB), bar);
                } else {
                    mbar_arrive(bar);  // an empty step (this warp's K share ended): completes at once
                }
            }
            if (++ld_c == nch) {
                ld_c = 0;
                advance(ld_u, ld_j);
            }
        }
        ++ld_seq;
    };
    // weights do not depend on earlier kernels: start streaming before waiting for them
    for (int i = 0; i < R - 1; ++i) issue_step();

    // inputs and outputs do
    if (PDL) pdl_wait();
    const bool shared = p.shared_rows > 0;
    // epilogue operands of this warp's next epilogue unit (the group's units
    // wi, wi + wpu, ...)
    EpiPre<NT> pre;
    int ep_u, ep_j;
    if (G == 1) {  // one group: its units are simply u0, u0 + 1, ...
        ep_u = min(u1, u0 + wi);
        ep_j = ep_u < u1 ? job_of(jp, ep_u, j0) : nj;
    } else {
        first_from(j0, ep_u, ep_j);
        for (int i = 0; i < wi; ++i) advance(ep_u, ep_j);
    }
    if (ep_u < u1) epi_prefetch<NT>(p, jobs[ep_j], ep_u - jp[ep_j], shared ? 0 : ((ep_j - j0) & 1), lane, pre);
    if (shared) {
        int rows[GEMV_MAXR];
#pragma unroll
        for (int r = 0; r < GEMV_MAXR; ++r) rows[r] = r;
        fill_B<NT, CPB, INV>(p, rows, p.shared_rows, meta, 0, Bsm, cw, lane, ctid);
    }
    int jfill = -1;
    float acc[NT][4];
    int ia[NT][4];
    const float W0 = (lane & 1) ? 1.0f : 65536.0f, W1 = (lane & 1) ? 0.0f : 256.0f;  // digit weights of my columns
    // grouped 4-bit scales: the two columns are joined as WI * first + second
    // per group (scale2), worth WJ each
    constexpr bool JOINED = tf_4bit(FMT) && GS != 0;
    const int WI = (lane & 1) ? 1 : 256;
    const float WJ = (lane & 1) ? 1.0f : 256.0f;
    // one step: issue the step R - 1 ahead, wait for this one, compute it
    int seq = 0;
    auto do_step = [&](int c) {
        issue_step();
        if (!gemv_mbar_wait(mybar + seq % R, (uint32_t)(seq / R) & 1u) && lane == 0 && p.err)
            atomicExch(p.err, GEMV_ERR_WAIT);
        const uint8_t *slot = myring + (size_t)(seq % R) * MB * BB;
        ++seq;
        const int nb = step_blocks(c);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int i = 0; i < 4; ++i) ia[nt][i] = 0;
        auto block = [&](int i) {
            const int kc = kb0 + c * MB + i;
            BlkRegs r;
            load_blk_smem<FMT, GS>(r, slot + i * BB, lane);
            if (tf_4bit(FMT)) {
                uint4 B[NT];
#pragma unroll
                for (int nt = 0; nt < NT; ++nt)
                    B[nt] = reinterpret_cast<const uint4 *>(Bsm)[(nt * p.kblocks + kc) * 32 + lane];
                block_t4<FMT, NT, GS>(r, B, acc, ia, WI);
            } else {
                uint2 B[NT];
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) B[nt] = Bsm[(nt * p.kblocks + kc) * 32 + lane];
                block_t8<NT>(r, B, ia);
            }
        };
        // A full step runs its blocks with no per-block bound check (the
        // check and its branch cost more than 1 % of the decode step); only
        // the last step of a warp's share of a unit can be partial.
        if (nb == MB) {
#pragma unroll
            for (int i = 0; i < MB; ++i) block(i);
        } else {
#pragma unroll 1
            for (int i = 0; i < nb; ++i) block(i);
        }
        __syncwarp();  // every lane is done with the slot before it is refilled
        if (FMT == TF_T8 || GS == 0) {  // per-row scale: the step's exact sums join the fp32 accumulator
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int i = 0; i < 4; ++i) acc[nt][i] = __fadd_rn(acc[nt][i], __int2float_rn(ia[nt][i]));
        }
    };
    int n = 0;         // this group's units done
    const int gbar = 2 + 2 * gi * NS;  // named barriers of this group: full/free per slot
    for (int j = j0; j < nj; ++j) {  // every warp visits every job segment, in order
        const int lo = seg_lo(j), hi = seg_hi(j);
        if (lo < hi && !shared) {
            const GemvJob &job = jobs[j];
            const int mb = (j - j0) & 1;
            // every warp has finished the epilogues of earlier jobs before meta and B change
            named_bar_sync(BAR_FILL, NCT);
            // Reuse the B operand when this job reads the same input rows as
            // the last job that filled it (decided from the read-only job
            // table, so every thread decides alike).
            bool same = jfill >= 0 && jobs[jfill].nrows == job.nrows;
            for (int r = 0; same && r < min(job.nrows, NT * 2); ++r) same = jobs[jfill].in_row[r] == job.in_row[r];
            if (same) {
                if (ctid < GEMV_MAXR) {
                    meta->scale[mb][ctid] = meta->scale[mb ^ 1][ctid];
                    meta->inv[mb][ctid] = meta->inv[mb ^ 1][ctid];
                }
                named_bar_sync(BAR_FILL, NCT);
            } else {
                fill_B<NT, CPB, INV>(p, job.in_row, job.nrows, meta, mb, Bsm, cw, lane, ctid);
                jfill = j;
            }
        }
        for (int u = lo + gi; u < hi; u += G, ++n) {
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int i = 0; i < 4; ++i) acc[nt][i] = 0.f;
            for (int c = 0; c < nch; ++c) do_step(c);
            // digits -> value: lanes 4g + 2m hold (hi, mid), lanes 4g + 2m + 1 (lo, 0) of input row 2nt + m
            float v[NT][2];
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                float vg = JOINED ? __fmul_rn(acc[nt][0], WJ) : __fmaf_rn(acc[nt][1], W1, __fmul_rn(acc[nt][0], W0));
                float vg8 = JOINED ? __fmul_rn(acc[nt][2], WJ) : __fmaf_rn(acc[nt][3], W1, __fmul_rn(acc[nt][2], W0));
                v[nt][0] = __fadd_rn(vg, __shfl_xor_sync(0xffffffffu, vg, 1));
                v[nt][1] = __fadd_rn(vg8, __shfl_xor_sync(0xffffffffu, vg8, 1));
            }
            bool mine = true;
            if (wpu > 1) {
                // reduction over the group's warps through NS shared slots:
                // only the unit's epilogue warp waits for the partials; the
                // others wait only when a slot is reused, for the epilogue
                // that read it NS units earlier.
                const int buf = n % NS, ew = n % wpu, nthr = wpu * 32;
                float(*slot)[32][NT * 2] =
                    reinterpret_cast<float(*)[32][NT * 2]>(smem + OFF_RED) + (gi * NS + buf) * wpu;
                if (n >= NS && wi != (n - NS) % wpu) named_bar_sync(gbar + 2 * buf + 1, nthr);
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    slot[wi][lane][nt * 2 + 0] = v[nt][0];
                    slot[wi][lane][nt * 2 + 1] = v[nt][1];
                }
                mine = wi == ew;
                if (!mine) {
                    named_bar_arrive(gbar + 2 * buf, nthr);
                } else {
                    named_bar_sync(gbar + 2 * buf, nthr);
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt) {
                        float v0 = 0.f, v1 = 0.f;
                        for (int w = 0; w < wpu; ++w) {
                            v0 = __fadd_rn(v0, slot[w][lane][nt * 2 + 0]);
                            v1 = __fadd_rn(v1, slot[w][lane][nt * 2 + 1]);
                        }
                        v[nt][0] = v0;
                        v[nt][1] = v1;
                    }
                    if (n + NS < ntot) named_bar_arrive(gbar + 2 * buf + 1, nthr);
                }
            }
            if (mine) {
                epilogue<NT>(p, meta, pre, v, lane);
                for (int i = 0; i < wpu; ++i) advance(ep_u, ep_j);
                if (ep_u < u1)
                    epi_prefetch<NT>(p, jobs[ep_j], ep_u - jp[ep_j], shared ? 0 : ((ep_j - j0) & 1), lane, pre);
            }
        }
        if (hi >= u1) break;
    }
}

}  // namespace

}  // namespace pc
