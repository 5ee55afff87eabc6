// gemv.cu - the dequant-fused GEMV that streams INT4/INT8 weight tiles from
// HBM: matmul_qt (quant.h:323-337) for up to 8 input rows per matrix, with
// the MoE and attention epilogues fused.
//
// One persistent CTA of 12 warps per SM.  A CTA owns a contiguous range of
// 16-row tiles ("units"); warp w owns a contiguous 1/12 of the k-blocks of
// every unit, so:
//  * each warp streams only its own bytes, straight into registers: per
//    step (up to 4 k-blocks of one unit) every lane loads its 16-byte A
//    fragment of each block and its rows' group scales, one step ahead of the
//    step it computes; HBM latency is covered by L2 prefetches of the warp's
//    slice several units ahead, which hold no registers or shared memory;
//  * the input-row fragments (f16 hi/lo pairs of x * 2^e, ~22 significant
//    bits) are built once per job in shared memory;
//  * per block it turns the nibbles (or bytes) into exact f16 values and
//    runs m16n8k16 tensor-core MMAs, taking partial sums per quantization
//    group and scaling them in fp32 (acc += group_sum * scale), the structure
//    of matmul_i4_gs (quant.h:259-319).
// At the end of a unit the 12 partials are summed in a fixed order
// (deterministic results) through a ring of shared buffers: only the unit's
// epilogue warp waits for them, and it prefetched the epilogue's operands 12
// units earlier.  Dense launches carry their job table in the kernel
// parameters and start streaming weights before waiting on the previous
// kernel (programmatic dependent launch).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>

#include "gemv.h"
#include "launch.cuh"
#include "ptx.cuh"

namespace pc {

namespace {

constexpr int NCONS = GEMV_CONSUMERS;
constexpr int NCT = NCONS * 32;
constexpr int PREFETCH_BYTES = 96 * 1024;  // weight bytes per SM requested ahead of use

constexpr int OFF_JP = 0;                                        // int[MAX_JOBS + 1]
constexpr int OFF_TILES = 4224;                                  // const uint8_t *[MAX_JOBS]
constexpr int OFF_JOBS = OFF_TILES + 8 * GEMV_MAX_JOBS;          // GemvJob[INLINE]
constexpr int OFF_META = OFF_JOBS + 128 * GEMV_INLINE_JOBS;
constexpr int OFF_RED = OFF_META + 256;
constexpr int NRED = 4;

static_assert(OFF_TILES >= OFF_JP + 4 * (GEMV_MAX_JOBS + 1), "job prefix region");
static_assert(sizeof(GemvJob) <= 128, "inline job slot");

struct SMeta {
    float scale[2][GEMV_MAXR];  // 2^e per B column (double-buffered by job parity)
    float inv[2][GEMV_MAXR];    // 2^-e
    int njobs;
};

__host__ __device__ inline int off_B(int nt) { return (OFF_RED + NRED * nt * NCONS * 256 + 127) & ~127; }
__host__ __device__ inline int off_end(int nt, int Ip) { return (off_B(nt) + nt * Ip * 16 + 127) & ~127; }

__device__ __forceinline__ uint32_t pack_h2(__half lo, __half hi) {
    return (uint32_t)__half_as_ushort(lo) | ((uint32_t)__half_as_ushort(hi) << 16);
}

__device__ __forceinline__ void split(float x, float sc, __half &hi, __half &lo) {
    const float v = __fmul_rn(x, sc);
    hi = __float2half_rn(v);
    lo = __float2half_rn(__fsub_rn(v, __half2float(hi)));
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

// Fills the f16 hi/lo B fragments for input rows rows[0..n) (B column c =
// rows[c]).  Pass 1: warp c takes row c's max |x| with 16-byte loads, all in
// flight; pass 2: each thread converts 8 values of one row for one lane
// column t into the hi lane (g = 2r) and the lo lane (g = 2r + 1) of one
// k-step pair, four entries per round so their loads overlap.
template <int NT>
__device__ void fill_B(const GemvParams &p, const int *rows, int n, SMeta *meta, int mb, uint4 *Bsm,
                       int cw, int lane, int ctid) {
    const int nrows = min(n, NT * 4);
    if (cw < nrows) {
        const float *xr = p.x + (int64_t)rows[cw] * p.ldx;
        float m = 0.0f;
        if ((p.ldx & 3) == 0 && (p.I & 3) == 0) {
            const float4 *x4 = reinterpret_cast<const float4 *>(xr);
            const int n4 = p.I >> 2;
            for (int k0 = lane; k0 < n4; k0 += 32 * 8) {
                float4 v[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) v[j] = k0 + 32 * j < n4 ? x4[k0 + 32 * j] : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    m = fmaxf(m, fmaxf(fmaxf(fabsf(v[j].x), fabsf(v[j].y)), fmaxf(fabsf(v[j].z), fabsf(v[j].w))));
            }
        } else {
            for (int k = lane; k < p.I; k += 32) m = fmaxf(m, fabsf(xr[k]));
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (lane == 0) {
            int e = 0;
            if (m > 0.0f && m <= 3.0e38f) {
                int E;
                frexpf(m, &E);
                e = 14 - E;
                e = max(-100, min(100, e));
            }
            meta->scale[mb][cw] = ldexpf(1.0f, e);
            meta->inv[mb][cw] = ldexpf(1.0f, -e);
        }
    }
    named_bar_sync(1, NCT);
    const int pairs = p.Ip / 32;
    const int total = NT * pairs * 16;
    const bool even = (p.ldx & 1) == 0;
    for (int base = ctid; base < total; base += 4 * NCT) {
        float v[4][8];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int idx = base + q * NCT;
            const int t = idx & 3, rr = (idx >> 2) & 3, pp = (idx >> 4) % pairs, nt = idx / (16 * pairs);
            const int r = nt * 4 + rr;
#pragma unroll
            for (int i = 0; i < 8; ++i) v[q][i] = 0.0f;
            if (idx < total && r < nrows) {
                const float *xr = p.x + (int64_t)rows[r] * p.ldx;
                const int k0 = pp * 32 + 2 * t;
#pragma unroll
                for (int h = 0; h < 4; ++h) {
                    const int k = k0 + 8 * h;
                    if (even && k + 1 < p.I) {
                        const float2 f = *reinterpret_cast<const float2 *>(xr + k);
                        v[q][2 * h] = f.x;
                        v[q][2 * h + 1] = f.y;
                    } else {
                        v[q][2 * h] = k < p.I ? xr[k] : 0.0f;
                        v[q][2 * h + 1] = k + 1 < p.I ? xr[k + 1] : 0.0f;
                    }
                }
            }
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int idx = base + q * NCT;
            if (idx >= total) continue;
            const int t = idx & 3, rr = (idx >> 2) & 3, pp = (idx >> 4) % pairs, nt = idx / (16 * pairs);
            const int r = nt * 4 + rr;
            const float sc = r < nrows ? meta->scale[mb][r] : 1.0f;
            __half h[8], l[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) split(v[q][i], sc, h[i], l[i]);
            uint4 *row = Bsm + (nt * pairs + pp) * 32;
            row[4 * (2 * rr) + t] =
                make_uint4(pack_h2(h[0], h[1]), pack_h2(h[2], h[3]), pack_h2(h[4], h[5]), pack_h2(h[6], h[7]));
            row[4 * (2 * rr + 1) + t] =
                make_uint4(pack_h2(l[0], l[1]), pack_h2(l[2], l[3]), pack_h2(l[4], l[5]), pack_h2(l[6], l[7]));
        }
    }
    named_bar_sync(1, NCT);
}

template <int NT>
__device__ __forceinline__ void mma_step(float (&d)[NT][4], const uint32_t (&a)[4], const uint4 (&B)[NT],
                                         bool second, bool fresh) {
    const float z[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        const uint32_t b0 = second ? B[nt].z : B[nt].x;
        const uint32_t b1 = second ? B[nt].w : B[nt].y;
        if (fresh)
            mma_f16_16816(d[nt], a, b0, b1, z);
        else
            mma_f16_16816(d[nt], a, b0, b1, d[nt]);
    }
}

template <int NT>
__device__ __forceinline__ void scale_acc(float (&acc)[NT][2], const float (&d)[NT][4], float s_lo, float s_hi) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        acc[nt][0] = __fmaf_rn(__fadd_rn(d[nt][0], d[nt][1]), s_lo, acc[nt][0]);
        acc[nt][1] = __fmaf_rn(__fadd_rn(d[nt][2], d[nt][3]), s_hi, acc[nt][1]);
    }
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
    if (FMT == TF_T4 && GS == 32) {
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

// One T4 block (64 columns) of one lane.  GS: group size (0 = per row, then
// the MMAs accumulate into dr and the row scale is applied in the epilogue).
template <int NT, int GS>
__device__ __forceinline__ void block_t4(const BlkRegs &r, const uint4 (&B0)[NT], const uint4 (&B1)[NT],
                                         float (&acc)[NT][2], float (&dr)[NT][4]) {
    const uint4 A = r.a;
    uint32_t a[4];
    float d[NT][4], e[NT][4];
    if (GS == 32) {
        const float s0 = __uint_as_float(r.s.x), s1 = __uint_as_float(r.s.y);
        const float s2 = __uint_as_float(r.s.z), s3 = __uint_as_float(r.s.w);
        dequant_i4_word(A.x, a); mma_step<NT>(d, a, B0, false, true);
        dequant_i4_word(A.z, a); mma_step<NT>(e, a, B1, false, true);
        dequant_i4_word(A.y, a); mma_step<NT>(d, a, B0, true, false);
        dequant_i4_word(A.w, a); mma_step<NT>(e, a, B1, true, false);
        scale_acc<NT>(acc, d, s0, s1);
        scale_acc<NT>(acc, e, s2, s3);
    } else if (GS == 64) {
        const float s0 = __uint_as_float(r.s.x), s1 = __uint_as_float(r.s.y);
        dequant_i4_word(A.x, a); mma_step<NT>(d, a, B0, false, true);
        dequant_i4_word(A.z, a); mma_step<NT>(e, a, B1, false, true);
        dequant_i4_word(A.y, a); mma_step<NT>(d, a, B0, true, false);
        dequant_i4_word(A.w, a); mma_step<NT>(e, a, B1, true, false);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int i = 0; i < 4; ++i) d[nt][i] = __fadd_rn(d[nt][i], e[nt][i]);
        scale_acc<NT>(acc, d, s0, s1);
    } else if (GS == 16) {
        dequant_i4_word(A.x, a); mma_step<NT>(d, a, B0, false, true);
        scale_acc<NT>(acc, d, __uint_as_float(r.s.x), __uint_as_float(r.s.y));
        dequant_i4_word(A.y, a); mma_step<NT>(e, a, B0, true, true);
        scale_acc<NT>(acc, e, __uint_as_float(r.s.z), __uint_as_float(r.s.w));
        dequant_i4_word(A.z, a); mma_step<NT>(d, a, B1, false, true);
        scale_acc<NT>(acc, d, __uint_as_float(r.s2.x), __uint_as_float(r.s2.y));
        dequant_i4_word(A.w, a); mma_step<NT>(e, a, B1, true, true);
        scale_acc<NT>(acc, e, __uint_as_float(r.s2.z), __uint_as_float(r.s2.w));
    } else {
        dequant_i4_word(A.x, a); mma_step<NT>(dr, a, B0, false, false);
        dequant_i4_word(A.y, a); mma_step<NT>(dr, a, B0, true, false);
        dequant_i4_word(A.z, a); mma_step<NT>(dr, a, B1, false, false);
        dequant_i4_word(A.w, a); mma_step<NT>(dr, a, B1, true, false);
    }
}

// One T8 block (32 columns) of one lane; INT8 is always per-row scaled.
template <int NT>
__device__ __forceinline__ void block_t8(const BlkRegs &r, const uint4 (&B0)[NT], float (&dr)[NT][4],
                                         float (&dr2)[NT][4]) {
    const uint4 A = r.a;
    uint32_t a[4], a2[4];
    dequant_i8_words(A.x, A.y, a);
    dequant_i8_words(A.z, A.w, a2);
    mma_step<NT>(dr, a, B0, false, false);
    mma_step<NT>(dr2, a2, B0, true, false);
}

// Per-lane epilogue operands of one row tile, fetched by the warp that will
// run that tile's epilogue NCONS tiles ahead of time, so their global-load
// latency never sits on the critical path.  Slot k covers B column k*4 + t.
template <int NT>
struct EpiPre {
    int rt, mb, O, seg, has_rs, has_b;
    float rs[2], b[2];
    int lrow[2];
    int jr[NT];  // job row whose B column is this slot's, or -1
    int out[NT], pos[NT], seq[NT];
    float cs[NT], sn[NT];
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
    const int nrows = min(job.nrows, NT * 4);
#pragma unroll
    for (int k = 0; k < NT; ++k) {
        const int col = k * 4 + t;
        int jr = -1;
        if (p.shared_rows > 0) {
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
            const float inv = meta->inv[e.mb][k * 4 + t];
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
                if (p.epi == EPI_STORE && p.residual) x = __fadd_rn(*dst, x);
                *dst = x;
                if (p.epi == EPI_LOGITS) {
                    const unsigned long long kk = argmax_key(x, o);
                    best = kk > best ? kk : best;
                }
            }
            if (p.epi == EPI_LOGITS) {
                // lanes with the same t hold the same column: reduce over g (lane bits 2..4)
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

constexpr int BAR_FILL = 1, BAR_FULL0 = 2, BAR_FREE0 = 6;

// FMT: TF_T4 / TF_T8; NT: 1 or 2 N-tiles (<= 4 or <= 8 input rows); GS:
// INT4 group size (0 = per row).
template <int FMT, int NT, int GS>
__global__ void __launch_bounds__(GEMV_THREADS, 1) gemv_kernel(const GemvParams p) {
    constexpr int BPB = FMT == TF_T4 ? 2 : 1;  // B fragment entries (k-step pairs) per block
    constexpr int MB = GEMV_STEP_BLOCKS;
    extern __shared__ __align__(128) uint8_t smem[];
    int *jp = reinterpret_cast<int *>(smem + OFF_JP);
    const uint8_t **stiles = reinterpret_cast<const uint8_t **>(smem + OFF_TILES);
    GemvJob *sjobs = reinterpret_cast<GemvJob *>(smem + OFF_JOBS);
    SMeta *meta = reinterpret_cast<SMeta *>(smem + OFF_META);
    float(*red)[NCONS][32][NT * 2] = reinterpret_cast<float(*)[NCONS][32][NT * 2]>(smem + OFF_RED);
    uint4 *Bsm = reinterpret_cast<uint4 *>(smem + off_B(NT));

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
        if (!p.static_jobs) pdl_wait();  // the job table comes from the previous kernel
        int nj = *p.njobs;
        nj = nj < 0 ? 0 : (nj > GEMV_MAX_JOBS ? GEMV_MAX_JOBS : nj);
        int run = 0;
        for (int base = 0; base < nj; base += 32) {
            int v = 0;
            if (base + lane < nj) {
                v = p.jobs[base + lane].n_rt;
                stiles[base + lane] = p.jobs[base + lane].tiles;
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
    pdl_trigger();
    const GemvJob *jobs = inl ? sjobs : p.jobs;
    const int nj = meta->njobs;
    const int64_t U = jp[nj];
    const int u0 = (int)(U * blockIdx.x / gridDim.x), u1 = (int)(U * (blockIdx.x + 1) / gridDim.x);
    if (u0 >= u1) return;
    const int nunits = u1 - u0;
    const int BB = p.blk_bytes;
    // This warp's contiguous k-block range of every unit, taken in nch steps
    // of at most MB blocks.
    const int kb0 = p.kblocks * cw / NCONS, nbw = p.kblocks * (cw + 1) / NCONS - kb0;
    const int nch = ((p.kblocks + NCONS - 1) / NCONS + MB - 1) / MB;
    const int nsteps = nunits * nch;
    const int PD = p.stages;  // L2 prefetch distance in units
    const int j0 = job_of(jp, u0, 0);
    auto step_blocks = [&](int c) { return max(0, min(MB, nbw - c * MB)); };
    auto slice = [&](int uc, int &jh) {  // this warp's bytes of unit uc
        const int u = u0 + uc;
        jh = job_of(jp, u, jh);
        return stiles[jh] + ((int64_t)(u - jp[jh]) * p.kblocks + kb0) * BB;
    };
    // HBM latency is covered by L2 prefetches PD units ahead (no registers or
    // shared memory held); L2 latency by loading the next step into
    // registers while this one is computed.
    int j_pf = j0, j_ld = j0;
    auto prefetch_unit = [&](int uc) {
        if (uc < nunits && nbw > 0) {
            const uintptr_t a0 = reinterpret_cast<uintptr_t>(slice(uc, j_pf));
            const uintptr_t a1 = a0 + (uintptr_t)nbw * BB;
            for (uintptr_t a = (a0 & ~(uintptr_t)127) + lane * 128; a < a1; a += 32 * 128)
                prefetch_l2(reinterpret_cast<const void *>(a));
        }
    };
    auto load_step = [&](BlkRegs(&f)[MB], int st) {
        if (st < nsteps) {
            const int uc = st / nch, c = st - uc * nch, nb = step_blocks(c);
            const uint8_t *src = slice(uc, j_ld) + (size_t)c * MB * BB;
#pragma unroll
            for (int i = 0; i < MB; ++i)
                if (i < nb) load_blk<FMT, GS>(f[i], src + i * BB, lane);
        }
    };
    // weights do not depend on earlier kernels: start streaming before waiting for them
    for (int uc = 0; uc < PD; ++uc) prefetch_unit(uc);
    BlkRegs cur[MB], nxt[MB];
    load_step(cur, 0);

    // inputs and outputs do
    pdl_wait();
    const int pairs = p.Ip / 32;
    const bool shared = p.shared_rows > 0;
    EpiPre<NT> pre;
    if (cw < nunits) {
        const int uf = u0 + cw, jf = job_of(jp, uf, j0);
        epi_prefetch<NT>(p, jobs[jf], uf - jp[jf], shared ? 0 : ((jf - j0) & 1), lane, pre);
    }
    if (shared) {
        int rows[GEMV_MAXR];
#pragma unroll
        for (int r = 0; r < GEMV_MAXR; ++r) rows[r] = r;
        fill_B<NT>(p, rows, p.shared_rows, meta, 0, Bsm, cw, lane, ctid);
    }
    int j = j0, jfill = -1;
    float acc[NT][2], acc2[NT][2], dr[NT][4], dr2[NT][4], dr3[NT][4], dr4[NT][4];
    for (int st = 0; st < nsteps; ++st) {
        const int uc = st / nch, c = st - uc * nch;
        const int u = u0 + uc;
        if (c == 0) {
            const int jn = job_of(jp, u, j);
            const bool changed = jn != j || uc == 0;
            j = jn;
            const GemvJob &job = jobs[j];
            if (changed && !shared) {
                const int mb = (j - j0) & 1;
                // every warp has finished its pending epilogue (which may still
                // read meta of the job before last) before meta is rewritten
                named_bar_sync(BAR_FILL, NCT);
                // Reuse the B fragments when this job reads the same input rows
                // as the last job that filled them (decided from the read-only
                // job table, so every thread decides alike).
                bool same = jfill >= 0 && jobs[jfill].nrows == job.nrows;
                for (int r = 0; same && r < min(job.nrows, NT * 4); ++r)
                    same = jobs[jfill].in_row[r] == job.in_row[r];
                if (same) {
                    if (ctid < GEMV_MAXR) {
                        meta->scale[mb][ctid] = meta->scale[mb ^ 1][ctid];
                        meta->inv[mb][ctid] = meta->inv[mb ^ 1][ctid];
                    }
                    named_bar_sync(BAR_FILL, NCT);
                } else {
                    fill_B<NT>(p, job.in_row, job.nrows, meta, mb, Bsm, cw, lane, ctid);
                    jfill = j;
                }
            }
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                acc[nt][0] = acc[nt][1] = acc2[nt][0] = acc2[nt][1] = 0.f;
#pragma unroll
                for (int i = 0; i < 4; ++i) dr[nt][i] = dr2[nt][i] = dr3[nt][i] = dr4[nt][i] = 0.f;
            }
            prefetch_unit(uc + PD);
        }
        load_step(nxt, st + 1);
        const int nb = step_blocks(c);
#pragma unroll
        for (int i = 0; i < MB; ++i) {
            if (i >= nb) break;
            const int kc = kb0 + c * MB + i;
            uint4 B0[NT], B1[NT];
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                B0[nt] = Bsm[(nt * pairs + kc * BPB) * 32 + lane];
                B1[nt] = Bsm[(nt * pairs + kc * BPB + BPB - 1) * 32 + lane];
            }
            if (FMT == TF_T4) {
                if (i & 1)
                    block_t4<NT, GS>(cur[i], B0, B1, acc2, dr2);
                else
                    block_t4<NT, GS>(cur[i], B0, B1, acc, dr);
            } else {
                if (i & 1)
                    block_t8<NT>(cur[i], B0, dr3, dr4);
                else
                    block_t8<NT>(cur[i], B0, dr, dr2);
            }
        }
        if (c == nch - 1) {
            float pa[NT][2];
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                if (FMT == TF_T8) {
                    pa[nt][0] = __fadd_rn(__fadd_rn(__fadd_rn(dr[nt][0], dr[nt][1]), __fadd_rn(dr2[nt][0], dr2[nt][1])),
                                          __fadd_rn(__fadd_rn(dr3[nt][0], dr3[nt][1]), __fadd_rn(dr4[nt][0], dr4[nt][1])));
                    pa[nt][1] = __fadd_rn(__fadd_rn(__fadd_rn(dr[nt][2], dr[nt][3]), __fadd_rn(dr2[nt][2], dr2[nt][3])),
                                          __fadd_rn(__fadd_rn(dr3[nt][2], dr3[nt][3]), __fadd_rn(dr4[nt][2], dr4[nt][3])));
                } else if (GS == 0) {
                    pa[nt][0] = __fadd_rn(__fadd_rn(dr[nt][0], dr[nt][1]), __fadd_rn(dr2[nt][0], dr2[nt][1]));
                    pa[nt][1] = __fadd_rn(__fadd_rn(dr[nt][2], dr[nt][3]), __fadd_rn(dr2[nt][2], dr2[nt][3]));
                } else {
                    pa[nt][0] = __fadd_rn(acc[nt][0], acc2[nt][0]);
                    pa[nt][1] = __fadd_rn(acc[nt][1], acc2[nt][1]);
                }
            }
            // cross-warp reduction through a ring of NRED buffers: only the unit's
            // epilogue warp waits for the partials; the others wait only when a
            // buffer is reused, for the epilogue that read it NRED units ago.
            const int buf = uc % NRED;
            const int ew = uc % NCONS;
            if (uc >= NRED && cw != (uc - NRED) % NCONS) named_bar_sync(BAR_FREE0 + buf, NCT);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                red[buf][cw][lane][nt * 2 + 0] = pa[nt][0];
                red[buf][cw][lane][nt * 2 + 1] = pa[nt][1];
            }
            if (cw != ew) {
                named_bar_arrive(BAR_FULL0 + buf, NCT);
            } else {
                named_bar_sync(BAR_FULL0 + buf, NCT);
                float v[NT][2];
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    float v0 = 0.f, v1 = 0.f;
#pragma unroll
                    for (int w = 0; w < NCONS; ++w) {
                        v0 = __fadd_rn(v0, red[buf][w][lane][nt * 2 + 0]);
                        v1 = __fadd_rn(v1, red[buf][w][lane][nt * 2 + 1]);
                    }
                    v[nt][0] = v0;
                    v[nt][1] = v1;
                }
                if (uc + NRED < nunits) named_bar_arrive(BAR_FREE0 + buf, NCT);
                epilogue<NT>(p, meta, pre, v, lane);
                const int uf = u + NCONS;
                if (uf < u1) {
                    const int jf = job_of(jp, uf, j);
                    epi_prefetch<NT>(p, jobs[jf], uf - jp[jf], shared ? 0 : ((jf - j0) & 1), lane, pre);
                }
            }
        }
#pragma unroll
        for (int i = 0; i < MB; ++i) cur[i] = nxt[i];
    }
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
    switch (p.gs) {
        case 32: return go<TF_T4, NT, 32>(p, grid, smem, st);
        case 64: return go<TF_T4, NT, 64>(p, grid, smem, st);
        case 16: return go<TF_T4, NT, 16>(p, grid, smem, st);
        case 0: return go<TF_T4, NT, 0>(p, grid, smem, st);
    }
    return cudaErrorInvalidValue;
}

}  // namespace

size_t gemv_smem_bytes(int nt, int Ip, int stages, int stage_bytes) {
    return (size_t)off_end(nt, Ip) + (size_t)stages * stage_bytes;
}

cudaError_t gemv_configure(int max_smem) {
    cudaError_t e = cudaSuccess;
#define PC_SET(F, N, G) if (e == cudaSuccess) e = set_smem<F, N, G>(max_smem)
    PC_SET(TF_T8, 1, 0); PC_SET(TF_T8, 2, 0);
    PC_SET(TF_T4, 1, 0); PC_SET(TF_T4, 2, 0);
    PC_SET(TF_T4, 1, 16); PC_SET(TF_T4, 2, 16);
    PC_SET(TF_T4, 1, 32); PC_SET(TF_T4, 2, 32);
    PC_SET(TF_T4, 1, 64); PC_SET(TF_T4, 2, 64);
#undef PC_SET
    return e;
}

// Launch plan: p.stages = L2 prefetch distance in units, enough that about
// PREFETCH_BYTES per SM are in flight (2..8 units); no staging buffers
// (p.stage_bytes = 0).  False if the input rows' fragments (nt * Ip * 16
// bytes) do not fit in shared memory.
bool gemv_plan(GemvParams &p, int nt, int max_smem) {
    if (off_end(nt, p.Ip) > max_smem) return false;
    const int unit_bytes = p.kblocks * p.blk_bytes;
    int pd = (PREFETCH_BYTES + unit_bytes - 1) / unit_bytes;
    p.stages = pd < 2 ? 2 : pd > 8 ? 8 : pd;
    p.stage_bytes = 0;
    return true;
}

cudaError_t gemv_launch(const GemvParams &p, int nt, int grid, cudaStream_t st) {
    const size_t smem = gemv_smem_bytes(nt, p.Ip, p.stages, p.stage_bytes);
    return nt == 1 ? go_nt<1>(p, grid, smem, st) : go_nt<2>(p, grid, smem, st);
}

}  // namespace pc
