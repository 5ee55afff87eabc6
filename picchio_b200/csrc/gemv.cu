// gemv.cu - the dequant-fused GEMV that streams INT4/INT8 weight tiles from
// HBM: matmul_qt (quant.h:323-337) for M <= 8 input rows per matrix, with
// the MoE and attention epilogues fused.
//
// One persistent CTA per SM.  Warp 0 is the producer: one lane walks this
// CTA's share of row tiles and issues cp.async.bulk copies of their bytes
// (whole 512/576/640/768-byte blocks, up to 16 KB per stage) into a ring of
// shared-memory stages, each guarded by a full/empty mbarrier pair.  Warps
// 1-8 consume: each takes every 8th block of a stage, turns the nibbles (or
// bytes) into exact f16 values in registers and runs m16n8k16 tensor-core
// MMAs against the input rows, which sit in shared memory as f16 hi/lo
// pairs (x * 2^e = hi + lo with a per-row power-of-two e, so hi + lo carries
// ~22 significant bits); MMA partials are taken per quantization group and
// scaled in fp32 (acc += group_sum * scale), the same structure as
// matmul_i4_gs (quant.h:259-319).  At the end of a row tile the eight warps'
// partials are summed in a fixed order (deterministic results) and one warp
// runs the epilogue.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "gemv.h"
#include "ptx.cuh"

namespace pc {

namespace {

constexpr int NCONS = GEMV_CONSUMERS;
constexpr int MAX_STAGES = 16;
constexpr uint32_t WAIT_LIMIT = 1u << 22;  // polls before a wait is declared stuck

constexpr int OFF_BAR = 0;
constexpr int OFF_JP = 256;
constexpr int OFF_META = OFF_JP + 4 * (GEMV_MAX_JOBS + 1) + 60;  // 4416
constexpr int META_BYTES = 256;
constexpr int OFF_RED = OFF_META + META_BYTES;                  // 4672

struct SMeta {
    float scale[2][GEMV_MAXR];  // 2^e per input row (double-buffered by job parity)
    float inv[2][GEMV_MAXR];    // 2^-e
    int njobs;
};

__host__ __device__ inline int off_B(int nt) { return (OFF_RED + nt * 4096 + 127) & ~127; }
__host__ __device__ inline int off_stage(int nt, int Ip) { return (off_B(nt) + nt * Ip * 16 + 127) & ~127; }

__device__ __forceinline__ uint32_t pack_h2(__half lo, __half hi) {
    return (uint32_t)__half_as_ushort(lo) | ((uint32_t)__half_as_ushort(hi) << 16);
}

__device__ __forceinline__ __half split_part(const float *xr, int k, int I, float sc, int part) {
    float v = (k < I) ? __fmul_rn(xr[k], sc) : 0.0f;
    __half h = __float2half_rn(v);
    if (part == 0) return h;
    return __float2half_rn(__fsub_rn(v, __half2float(h)));
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

// Fills the f16 hi/lo B fragments for the job's input rows.
template <int NT>
__device__ void fill_B(const GemvParams &p, const GemvJob &job, SMeta *meta, int mb, uint4 *Bsm,
                       int cw, int lane, int ctid) {
    const int nrows = min(job.nrows, NT * 4);
    if (cw < nrows) {
        const float *xr = p.x + (int64_t)job.in_row[cw] * p.ldx;
        float m = 0.0f;
        for (int k = lane; k < p.I; k += 32) m = fmaxf(m, fabsf(xr[k]));
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
    named_bar_sync(1, NCONS * 32);
    const int pairs = p.Ip / 32;
    const int total = NT * pairs * 32;
    for (int idx = ctid; idx < total; idx += NCONS * 32) {
        const int L = idx & 31, pp = (idx >> 5) % pairs, nt = idx / (32 * pairs);
        const int g = L >> 2, t = L & 3, r = nt * 4 + (g >> 1), part = g & 1;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (r < nrows) {
            const float *xr = p.x + (int64_t)job.in_row[r] * p.ldx;
            const float sc = meta->scale[mb][r];
            const int k0 = pp * 32 + 2 * t, k1 = k0 + 16;
            v.x = pack_h2(split_part(xr, k0, p.I, sc, part), split_part(xr, k0 + 1, p.I, sc, part));
            v.y = pack_h2(split_part(xr, k0 + 8, p.I, sc, part), split_part(xr, k0 + 9, p.I, sc, part));
            v.z = pack_h2(split_part(xr, k1, p.I, sc, part), split_part(xr, k1 + 1, p.I, sc, part));
            v.w = pack_h2(split_part(xr, k1 + 8, p.I, sc, part), split_part(xr, k1 + 9, p.I, sc, part));
        }
        Bsm[idx] = v;
    }
    named_bar_sync(1, NCONS * 32);
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

// One T4 block (64 columns) of one lane.
template <int NT>
__device__ __forceinline__ void block_t4(const uint8_t *blk, const uint4 *Bsm, int pairs, int kc, int gs,
                                         int lane, float (&acc)[NT][2], float (&dr)[NT][4]) {
    const int g = lane >> 2;
    const uint4 A = *reinterpret_cast<const uint4 *>(blk + lane * 16);
    uint4 B0[NT], B1[NT];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        B0[nt] = Bsm[(nt * pairs + kc * 2) * 32 + lane];
        B1[nt] = Bsm[(nt * pairs + kc * 2 + 1) * 32 + lane];
    }
    uint32_t a[4];
    float d[NT][4];
    if (gs == 32) {
        const float4 S = *reinterpret_cast<const float4 *>(blk + 512 + g * 16);
        dequant_i4_word(A.x, a); mma_step<NT>(d, a, B0, false, true);
        dequant_i4_word(A.y, a); mma_step<NT>(d, a, B0, true, false);
        scale_acc<NT>(acc, d, S.x, S.y);
        dequant_i4_word(A.z, a); mma_step<NT>(d, a, B1, false, true);
        dequant_i4_word(A.w, a); mma_step<NT>(d, a, B1, true, false);
        scale_acc<NT>(acc, d, S.z, S.w);
    } else if (gs == 64) {
        const float2 S = *reinterpret_cast<const float2 *>(blk + 512 + g * 8);
        dequant_i4_word(A.x, a); mma_step<NT>(d, a, B0, false, true);
        dequant_i4_word(A.y, a); mma_step<NT>(d, a, B0, true, false);
        dequant_i4_word(A.z, a); mma_step<NT>(d, a, B1, false, false);
        dequant_i4_word(A.w, a); mma_step<NT>(d, a, B1, true, false);
        scale_acc<NT>(acc, d, S.x, S.y);
    } else if (gs == 16) {
        const float4 S0 = *reinterpret_cast<const float4 *>(blk + 512 + g * 32);
        const float4 S1 = *reinterpret_cast<const float4 *>(blk + 512 + g * 32 + 16);
        dequant_i4_word(A.x, a); mma_step<NT>(d, a, B0, false, true); scale_acc<NT>(acc, d, S0.x, S0.y);
        dequant_i4_word(A.y, a); mma_step<NT>(d, a, B0, true, true);  scale_acc<NT>(acc, d, S0.z, S0.w);
        dequant_i4_word(A.z, a); mma_step<NT>(d, a, B1, false, true); scale_acc<NT>(acc, d, S1.x, S1.y);
        dequant_i4_word(A.w, a); mma_step<NT>(d, a, B1, true, true);  scale_acc<NT>(acc, d, S1.z, S1.w);
    } else {  // per-row scale: one running MMA sum, scaled in the epilogue
        dequant_i4_word(A.x, a); mma_step<NT>(dr, a, B0, false, false);
        dequant_i4_word(A.y, a); mma_step<NT>(dr, a, B0, true, false);
        dequant_i4_word(A.z, a); mma_step<NT>(dr, a, B1, false, false);
        dequant_i4_word(A.w, a); mma_step<NT>(dr, a, B1, true, false);
    }
}

// One T8 block (32 columns) of one lane; INT8 is always per-row scaled.
template <int NT>
__device__ __forceinline__ void block_t8(const uint8_t *blk, const uint4 *Bsm, int pairs, int kc, int lane,
                                         float (&dr)[NT][4]) {
    const uint4 A = *reinterpret_cast<const uint4 *>(blk + lane * 16);
    uint4 B0[NT];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) B0[nt] = Bsm[(nt * pairs + kc) * 32 + lane];
    uint32_t a[4];
    dequant_i8_words(A.x, A.y, a);
    mma_step<NT>(dr, a, B0, false, false);
    dequant_i8_words(A.z, A.w, a);
    mma_step<NT>(dr, a, B0, true, false);
}

// Writes one lane's results of one row tile.
template <int NT>
__device__ void epilogue(const GemvParams &p, const GemvJob &job, const SMeta *meta, int mb, int rt,
                         const float (*red)[32][NT * 2], int lane) {
    const int g = lane >> 2, t = lane & 3;
    const int nrows = min(job.nrows, NT * 4);
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        const int r = nt * 4 + t;
        float v0 = 0.f, v1 = 0.f;
#pragma unroll
        for (int w = 0; w < NCONS; ++w) {
            v0 = __fadd_rn(v0, red[w][lane][nt * 2 + 0]);
            v1 = __fadd_rn(v1, red[w][lane][nt * 2 + 1]);
        }
        const bool live = r < nrows;
        if (live) {
            const float inv = meta->inv[mb][r];
            v0 = __fmul_rn(v0, inv);
            v1 = __fmul_rn(v1, inv);
        }
        if (p.epi == EPI_SWIGLU) {
            if (!live) continue;
            const int pr = rt * 8 + g;  // pair index
            const int og = 2 * pr, ou = 2 * pr + 1;
            if (ou >= job.O) continue;
            float gate = v0, up = v1;
            if (job.rs) { gate = __fmul_rn(gate, job.rs[og]); up = __fmul_rn(up, job.rs[ou]); }
            if (job.bias) { gate = __fadd_rn(gate, job.bias[og]); up = __fadd_rn(up, job.bias[ou]); }
            p.y[(int64_t)job.out_row[r] * p.ldy + pr] = swiglu(gate, up, p.swiglu_limit, p.swiglu_alpha);
        } else if (p.epi == EPI_QKV) {
            if (!live) continue;
            const int hd = p.head_dim, half = hd >> 1, tph = hd / 16;
            const int h = rt / tph, j = (rt % tph) * 8 + g;
            const int olo = h * hd + j, ohi = olo + half;
            if (ohi >= job.O) continue;
            float lo = v0, hi = v1;
            if (job.rs) { lo = __fmul_rn(lo, job.rs[olo]); hi = __fmul_rn(hi, job.rs[ohi]); }
            if (job.bias) { lo = __fadd_rn(lo, job.bias[olo]); hi = __fadd_rn(hi, job.bias[ohi]); }
            const int in = job.in_row[r];
            const int pos = p.row_pos[in];
            if (job.seg != 2) {
                // rope_apply (picchio.c:467-469) as the reference build rounds it:
                // a*cs - b*sn -> fma(a, cs, -(b*sn)); a*sn + b*cs -> fma(a, sn, b*cs).
                const float cs = p.rope_cs[(int64_t)pos * half + j], sn = p.rope_sn[(int64_t)pos * half + j];
                const float a = lo, b = hi;
                lo = __fmaf_rn(a, cs, -__fmul_rn(b, sn));
                hi = __fmaf_rn(a, sn, __fmul_rn(b, cs));
            }
            if (job.seg == 0) {
                float *q = p.qbuf + (int64_t)job.out_row[r] * p.ldq;
                q[olo] = lo;
                q[ohi] = hi;
            } else if (pos >= 0 && pos < p.kv_ctx) {  // kv_store drops pos >= max_pos (picchio.c:495)
                const int64_t base = (int64_t)p.row_seq[in] * p.kv_seq_stride + (int64_t)pos * p.kv_dim;
                void *cache = job.seg == 1 ? p.kcache : p.vcache;
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
                const int o = tile_row_to_logical(p.perm, p.head_dim, rt, g + 8 * hlf);
                if (!live || o >= job.O) continue;
                float v = hlf ? v1 : v0;
                if (job.rs) v = __fmul_rn(v, job.rs[o]);
                if (job.bias) v = __fadd_rn(v, job.bias[o]);
                float *dst = p.y + (int64_t)job.out_row[r] * p.ldy + o;
                if (p.epi == EPI_STORE && p.residual) v = __fadd_rn(*dst, v);
                *dst = v;
                if (p.epi == EPI_LOGITS) {
                    const unsigned long long k = argmax_key(v, o);
                    best = k > best ? k : best;
                }
            }
            if (p.epi == EPI_LOGITS) {
                // lanes with the same t hold the same row: reduce over g (lane bits 2..4)
#pragma unroll
                for (int o = 4; o < 32; o <<= 1) {
                    const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
                    best = other > best ? other : best;
                }
                if (g == 0 && live && best) atomicMax(p.argmax + job.out_row[r], best);
            }
        }
    }
}

template <int FMT, int NT>
__global__ void __launch_bounds__(GEMV_THREADS, 1) gemv_kernel(const GemvParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + OFF_BAR);
    uint64_t *empty = full + MAX_STAGES;
    int *jp = reinterpret_cast<int *>(smem + OFF_JP);
    SMeta *meta = reinterpret_cast<SMeta *>(smem + OFF_META);
    float(*red)[NCONS][32][NT * 2] = reinterpret_cast<float(*)[NCONS][32][NT * 2]>(smem + OFF_RED);
    uint4 *Bsm = reinterpret_cast<uint4 *>(smem + off_B(NT));
    uint8_t *stages = smem + off_stage(NT, p.Ip);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int S = p.stages;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(full + s, 1);
            mbar_init(empty + s, NCONS);
        }
        fence_mbar_init();
    }
    if (warp == 0) {  // prefix sum of row tiles over jobs
        int nj = *p.njobs;
        nj = nj < 0 ? 0 : (nj > GEMV_MAX_JOBS ? GEMV_MAX_JOBS : nj);
        int run = 0;
        for (int base = 0; base < nj; base += 32) {
            int v = (base + lane < nj) ? p.jobs[base + lane].n_rt : 0;
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
    const int nj = meta->njobs;
    const int64_t U = jp[nj];
    const int u0 = (int)(U * blockIdx.x / gridDim.x), u1 = (int)(U * (blockIdx.x + 1) / gridDim.x);
    if (u0 >= u1) return;

    const int SB = p.stage_bytes / p.blk_bytes;  // blocks per stage
    const int nchunks = (p.kblocks + SB - 1) / SB;

    if (warp == 0) {
        if (lane == 0) {
            const uint64_t pol = l2_evict_first_policy();
            int j = 0, it = 0;
            for (int u = u0; u < u1; ++u) {
                while (u >= jp[j + 1]) ++j;
                const uint8_t *src = p.jobs[j].tiles + (int64_t)(u - jp[j]) * p.kblocks * p.blk_bytes;
                for (int c = 0; c < nchunks; ++c, ++it) {
                    const int nb = min(SB, p.kblocks - c * SB);
                    const int s = it % S, r = it / S;
                    if (r > 0 && !mbar_wait_bounded(empty + s, (r - 1) & 1, WAIT_LIMIT)) {
                        atomicExch(p.err, 1);
                        return;  // consumers time out on the stage that never fills
                    }
                    mbar_arrive_expect_tx(full + s, (uint32_t)(nb * p.blk_bytes));
                    bulk_g2s(stages + (size_t)s * p.stage_bytes, src + (size_t)c * SB * p.blk_bytes,
                             (uint32_t)(nb * p.blk_bytes), full + s, pol);
                }
            }
        }
        return;
    }

    // consumers
    const int cw = warp - 1, ctid = threadIdx.x - 32;
    const int pairs = p.Ip / 32;
    int j = -1, jord = -1, jfill = -1, it = 0;
    for (int u = u0, uc = 0; u < u1; ++u, ++uc) {
        bool changed = false;
        while (j < 0 || u >= jp[j + 1]) { ++j; changed = true; }
        const GemvJob &job = p.jobs[j];
        if (changed) {
            ++jord;
            const int mb = jord & 1;
            // Reuse the B fragments when this job reads the same input rows
            // as the last job that filled them (decided from the read-only
            // job table, so every consumer thread decides alike).
            bool same = jfill >= 0 && p.jobs[jfill].nrows == job.nrows;
            for (int r = 0; same && r < min(job.nrows, NT * 4); ++r)
                same = p.jobs[jfill].in_row[r] == job.in_row[r];
            if (same) {
                if (ctid < GEMV_MAXR) {
                    meta->scale[mb][ctid] = meta->scale[mb ^ 1][ctid];
                    meta->inv[mb][ctid] = meta->inv[mb ^ 1][ctid];
                }
                named_bar_sync(1, NCONS * 32);
            } else {
                fill_B<NT>(p, job, meta, mb, Bsm, cw, lane, ctid);
                jfill = j;
            }
        }
        const int rt = u - jp[j];
        float acc[NT][2], dr[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            acc[nt][0] = acc[nt][1] = 0.f;
            dr[nt][0] = dr[nt][1] = dr[nt][2] = dr[nt][3] = 0.f;
        }
        bool ok = true;
        for (int c = 0; c < nchunks; ++c, ++it) {
            const int s = it % S, r = it / S;
            if (!mbar_wait_bounded(full + s, r & 1, WAIT_LIMIT)) {
                if (lane == 0) atomicExch(p.err, 1);
                ok = false;
                break;
            }
            const uint8_t *st = stages + (size_t)s * p.stage_bytes;
            const int nb = min(SB, p.kblocks - c * SB);
            for (int b = cw; b < nb; b += NCONS) {
                const int kc = c * SB + b;
                if (FMT == TF_T4)
                    block_t4<NT>(st + (size_t)b * p.blk_bytes, Bsm, pairs, kc, p.gs, lane, acc, dr);
                else
                    block_t8<NT>(st + (size_t)b * p.blk_bytes, Bsm, pairs, kc, lane, dr);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(empty + s);
        }
        if (!ok) return;  // every consumer fails on the same stage
        if (FMT == TF_T8 || p.gs == 0) {
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                acc[nt][0] = __fadd_rn(dr[nt][0], dr[nt][1]);
                acc[nt][1] = __fadd_rn(dr[nt][2], dr[nt][3]);
            }
        }
        const int buf = uc & 1;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            red[buf][cw][lane][nt * 2 + 0] = acc[nt][0];
            red[buf][cw][lane][nt * 2 + 1] = acc[nt][1];
        }
        named_bar_sync(1, NCONS * 32);
        if (cw == uc % NCONS) epilogue<NT>(p, job, meta, jord & 1, rt, red[buf], lane);
    }
}

}  // namespace

size_t gemv_smem_bytes(int nt, int Ip, int stages, int stage_bytes) {
    return (size_t)off_stage(nt, Ip) + (size_t)stages * stage_bytes;
}

cudaError_t gemv_configure(int max_smem) {
    cudaError_t e;
    if ((e = cudaFuncSetAttribute(gemv_kernel<TF_T4, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem))) return e;
    if ((e = cudaFuncSetAttribute(gemv_kernel<TF_T4, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem))) return e;
    if ((e = cudaFuncSetAttribute(gemv_kernel<TF_T8, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem))) return e;
    return cudaFuncSetAttribute(gemv_kernel<TF_T8, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
}

// Picks the stage geometry for a launch; returns false if the input rows do
// not fit in shared memory next to two stages.
bool gemv_plan(GemvParams &p, int nt, int max_smem) {
    const int SB = 16384 / p.blk_bytes;
    p.stage_bytes = SB * p.blk_bytes;
    const int fixed = off_stage(nt, p.Ip);
    int S = (max_smem - fixed) / p.stage_bytes;
    if (S > MAX_STAGES) S = MAX_STAGES;
    // no more stages than a row tile has chunks times a few tiles
    const int nchunks = (p.kblocks + SB - 1) / SB;
    if (S > nchunks * 4) S = nchunks * 4 < 2 ? 2 : nchunks * 4;
    p.stages = S;
    return S >= 2;
}

cudaError_t gemv_launch(const GemvParams &p, int nt, int grid, cudaStream_t st) {
    const size_t smem = gemv_smem_bytes(nt, p.Ip, p.stages, p.stage_bytes);
    if (p.fmt == TF_T4) {
        if (nt == 1) gemv_kernel<TF_T4, 1><<<grid, GEMV_THREADS, smem, st>>>(p);
        else gemv_kernel<TF_T4, 2><<<grid, GEMV_THREADS, smem, st>>>(p);
    } else {
        if (nt == 1) gemv_kernel<TF_T8, 1><<<grid, GEMV_THREADS, smem, st>>>(p);
        else gemv_kernel<TF_T8, 2><<<grid, GEMV_THREADS, smem, st>>>(p);
    }
    return cudaGetLastError();
}

}  // namespace pc
