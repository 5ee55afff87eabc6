// tcgemm.cu - the INT8 dense projections (matmul_q8, quant.h:152-186) for a
// batch of 16..128 input rows on the tcgen05 tensor cores.
//
// The GEMV (gemv.cu) reads a weight matrix once per 8 input rows; a decode
// batch of 64 rows or a 64-token prefill chunk would stream q/k/v, o_proj and
// the lm_head eight times.  Here every weight byte is read once per launch:
//
//  * A (weights): a row-major INT8 copy of the matrix, rows in tile order,
//    loaded by TMA as 128-row x 128-column boxes in the 128-byte swizzle
//    layout the MMA reads directly (no dequantization: INT8 is the operand);
//  * B (input rows): each row scaled by 2^sh, rounded to an integer of at
//    most 22 bits and split into three signed byte digits (the GEMV's B
//    operand), written by tc_prep_kernel as three digit planes and loaded
//    by TMA likewise;
//  * D: three s32 accumulators in TMEM (one per digit plane), 128 rows x N
//    rows each.  Every product and sum is exact in s32, so a row's dot is
//    the exact integer hi * 2^16 + mid * 2^8 + lo (in 64 bits), rounded once
//    to fp32 and scaled by 2^-sh and the row scale: the per-row-scale
//    structure of matmul_q8 with a single rounding.
//
// Warp roles (192 threads): warp 0 issues the TMA loads (one elected lane,
// S stages in flight), warp 1 allocates TMEM and issues the MMAs (one lane),
// warps 2-5 are the epilogue, one thread per TMEM lane (= weight row).  A
// 128-row tile can be split over K between CTAs: each adds its exact 64-bit
// row sums into the tile's accumulator with integer atomics (exact in any
// order), and the last CTA of the tile (atomic ticket) runs the epilogue and
// clears the accumulator.  Every mbarrier wait is
// bounded (1 s); a timeout sets the error word and the CTA winds down.
#include "gemv_core.cuh"
#include "sm100.cuh"
#include "tcgemm.h"

namespace pc {

namespace {

constexpr unsigned long long TC_WAIT_NS = 1000ull * 1000 * 1000;

template <int N>
struct TcCfg {
    static constexpr int S = N <= 64 ? 4 : 3;    // pipeline stages
    static constexpr int A = 128 * 128;          // weight box bytes
    static constexpr int B = N * 128;            // one digit plane's box bytes
    static constexpr int STAGE = A + 3 * B;
    static constexpr int TCOLS = 3 * N <= 128 ? 128 : 3 * N <= 256 ? 256 : 512;  // TMEM columns
    static constexpr int SMEM = 1024 + S * STAGE + 256 + 12 * N;  // + barriers, + per-column operands
};

__device__ __forceinline__ void tc_fail(int *err, int code) {
    if (err) atomicCAS(err, 0, code);
}

// Epilogue of 16 columns (input rows c0..c0+15) of one weight row (this
// thread's TMEM lane): s[j] is the row's exact dot with input row c0 + j in
// units of 2^-sh.  Every global operand of the 16 columns is loaded before
// any is used; the per-column ones (2^-sh, position, sequence slot) come from
// shared memory.  All 32 lanes of the warp call this together (QKV pairs rows
// g and g + 8 of a 16-row tile through a shuffle; LOGITS reduces over rows).
__device__ __forceinline__ void tc_epi16(const TcParams &p, const TcSeg &sg, int c0, const long long (&s)[16], int o,
                                         bool rv, float rs, float bias, int tr16, int o_lo, const float *cinv,
                                         const int *cpos, const int *cseq) {
    float x[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        float v = __fmul_rn(__ll2float_rn(s[j]), cinv[c0 + j]);
        if (sg.rs) v = __fmul_rn(v, rs);
        if (sg.bias) v = __fadd_rn(v, bias);
        x[j] = v;
    }
    if (p.epi == EPI_QKV) {
        const bool is_lo = (tr16 & 8) == 0;
        const bool pair_ok = rv && __shfl_xor_sync(0xffffffffu, (int)rv, 8) != 0;
        float oth[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) oth[j] = __shfl_xor_sync(0xffffffffu, x[j], 8);
        if (!pair_ok) return;
        const int half = p.head_dim >> 1, jj = o_lo % p.head_dim;
        float cs[16], sn[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            cs[j] = 1.0f;
            sn[j] = 0.0f;
            const int n = c0 + j;
            if (sg.seg != 2 && n < p.M) {
                const int64_t at = (int64_t)cpos[n] * half + jj;
                cs[j] = p.rope_cs[at];
                sn[j] = p.rope_sn[at];
            }
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const int n = c0 + j;
            if (n >= p.M) continue;
            float lo = is_lo ? x[j] : oth[j], hi = is_lo ? oth[j] : x[j];
            if (sg.seg != 2) {
                // rope_apply (picchio.c:467-469) rounded as the reference build does
                const float a = lo, b = hi;
                lo = __fmaf_rn(a, cs[j], -__fmul_rn(b, sn[j]));
                hi = __fmaf_rn(a, sn[j], __fmul_rn(b, cs[j]));
            }
            const float val = is_lo ? lo : hi;
            const int pos = cpos[n];
            if (sg.seg == 0) {
                p.qbuf[(int64_t)n * p.ldq + o] = val;
            } else if (pos >= 0 && pos < p.kv_ctx) {  // kv_store drops pos >= max_pos (picchio.c:495)
                const int64_t at = (int64_t)cseq[n] * p.kv_seq_stride + (int64_t)pos * p.kv_dim + o;
                void *cache = sg.seg == 1 ? p.kcache : p.vcache;
                if (p.kv_bf16)
                    reinterpret_cast<__nv_bfloat16 *>(cache)[at] = __float2bfloat16_rn(val);
                else
                    reinterpret_cast<float *>(cache)[at] = val;
            }
        }
        return;
    }
    if (p.epi == EPI_LOGITS) {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const int n = c0 + j;
            const bool live = rv && n < p.M;
            unsigned long long key = 0ull;
            if (live) {
                p.y[(int64_t)n * p.ldy + o] = x[j];
                key = argmax_key(x[j], o);
            }
#pragma unroll
            for (int m = 16; m > 0; m >>= 1) {
                const unsigned long long ot = __shfl_xor_sync(0xffffffffu, key, m);
                key = ot > key ? ot : key;
            }
            if ((threadIdx.x & 31) == 0 && n < p.M && key) atomicMax(p.argmax + n, key);
        }
        return;
    }
    // EPI_STORE, optionally onto the residual
    if (!rv) return;
    if (p.residual) {
        const float *src = p.res_src ? p.res_src : p.y;
        float r[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) r[j] = c0 + j < p.M ? src[(int64_t)(c0 + j) * p.ldy + o] : 0.0f;
#pragma unroll
        for (int j = 0; j < 16; ++j) x[j] = __fadd_rn(r[j], x[j]);
    }
#pragma unroll
    for (int j = 0; j < 16; ++j)
        if (c0 + j < p.M) p.y[(int64_t)(c0 + j) * p.ldy + o] = x[j];
}

template <int N>
__global__ void __launch_bounds__(TC_THREADS, 1) tc_gemm_kernel(const __grid_constant__ TcParams p) {
    using C = TcCfg<N>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + C::S * C::STAGE);
    uint64_t *empty = full + C::S;
    uint64_t *accf = empty + C::S;
    uint32_t *tslot = reinterpret_cast<uint32_t *>(accf + 1);
    int *lastf = reinterpret_cast<int *>(tslot + 1);
    float *cinv = reinterpret_cast<float *>(smem + C::S * C::STAGE + 256);  // per-column operands
    int *cpos = reinterpret_cast<int *>(cinv + N);
    int *cseq = cpos + N;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tile = blockIdx.x / p.nsplit, split = blockIdx.x % p.nsplit;
    int si = 0;
    while (si + 1 < p.nseg && tile >= p.tile_base[si + 1]) ++si;
    const TcSeg &sg = p.segs[si];
    const int row0 = (tile - p.tile_base[si]) * 128;
    const int k0 = p.ksteps * split / p.nsplit, nk = p.ksteps * (split + 1) / p.nsplit - k0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(accf, 1);
        mbar_init_fence();
    }
    if (warp == 1) {
        tmem_alloc(tslot, C::TCOLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *tslot;
    pdl_trigger();

    if (warp == 0) {
        if (lane == 0) {  // TMA producer
            tma_prefetch_desc(&sg.amap);
            tma_prefetch_desc(&p.bmap);
            // weights do not depend on earlier kernels: the first stages' weight
            // boxes go out before waiting for them; the input digits after.
            const int pre = min(nk, C::S);
            for (int i = 0; i < pre; ++i) {
                mbar_arrive_expect_tx(&full[i], C::STAGE);
                tma_load_2d(smem + i * C::STAGE, &sg.amap, &full[i], (k0 + i) * 128, row0);
            }
            pdl_wait();
            bool ok = true;
            int issued = 0;
            for (int i = 0; i < nk; ++i) {
                const int s = i % C::S;
                uint8_t *st = smem + s * C::STAGE;
                if (i >= C::S) {
                    if (!mbar_wait(&empty[s], ((i / C::S) - 1) & 1, TC_WAIT_NS)) {
                        tc_fail(p.err, 3);
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&full[s], C::STAGE);
                    tma_load_2d(st, &sg.amap, &full[s], (k0 + i) * 128, row0);
                }
#pragma unroll
                for (int d = 0; d < 3; ++d)
                    tma_load_2d(st + C::A + d * C::B, &p.bmap, &full[s], (k0 + i) * 128, d * p.Mpad);
                issued = i + 1;
            }
            if (!ok) {
                // the stages in flight land before this CTA's shared memory is released
                issued = max(issued, pre);
                for (int j = max(0, issued - C::S); j < issued; ++j)
                    mbar_wait(&full[j % C::S], (j / C::S) & 1, TC_WAIT_NS);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {  // MMA issuer
            constexpr uint32_t idesc = idesc_i8(128, N);
            for (int i = 0; i < nk; ++i) {
                const int s = i % C::S;
                if (!mbar_wait(&full[s], (i / C::S) & 1, TC_WAIT_NS)) {
                    tc_fail(p.err, 3);
                    break;
                }
                tc_fence_after();
                uint8_t *st = smem + s * C::STAGE;
                const uint64_t ad = sw128_desc(st);
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
#pragma unroll
                    for (int d = 0; d < 3; ++d)
                        tc_mma_i8(tbase + d * N, ad + 2 * kk, sw128_desc(st + C::A + d * C::B) + 2 * kk, idesc,
                                  i > 0 || kk > 0);
                tc_commit(&empty[s]);
            }
            tc_commit(accf);  // fires once every MMA above has completed
        }
    } else {  // epilogue: warps 2..5, thread = TMEM lane = weight row of the tile
        pdl_wait();
        const int q = warp & 3, tr = 32 * q + lane, e = threadIdx.x - 64;
        const int prow = row0 + tr, rt = prow >> 4, tr16 = prow & 15;
        const int o = tile_row_to_logical(p.perm, p.head_dim, rt, tr16);
        const int o_lo = tile_row_to_logical(p.perm, p.head_dim, rt, tr16 & 7);
        const bool rv = prow < sg.Op && o < sg.O;
        const float rs = (rv && sg.rs) ? sg.rs[o] : 1.0f;
        const float bias = (rv && sg.bias) ? sg.bias[o] : 0.0f;
        if (e < N) {  // per-column operands, once per CTA
            cinv[e] = e < p.M ? p.inv[e] : 0.0f;
            cpos[e] = (p.epi == EPI_QKV && e < p.M) ? p.row_pos[e] : 0;
            cseq[e] = (p.epi == EPI_QKV && e < p.M) ? p.row_seq[e] : 0;
        }
        named_bar_sync(1, 128);
        if (!mbar_wait(accf, 0, TC_WAIT_NS)) tc_fail(p.err, 3);
        __syncwarp();
        tc_fence_after();
        const uint32_t tl = tbase + ((uint32_t)(32 * q) << 16);
        // split K: the tile's exact 64-bit sums, accumulated with integer
        // atomics (exact in any order) in [tile][N][128]
        unsigned long long *acc = reinterpret_cast<unsigned long long *>(p.part) + (size_t)tile * N * 128;
        for (int c0 = 0; c0 < N; c0 += 16) {
            uint32_t d0[16], d1[16], d2[16];
            tmem_ld16(tl + c0, d0);
            tmem_ld16(tl + N + c0, d1);
            tmem_ld16(tl + 2 * N + c0, d2);
            tmem_ld_wait();
            long long v[16];
#pragma unroll
            for (int j = 0; j < 16; ++j)
                v[j] = (long long)(int32_t)d0[j] * 65536 + (long long)(int32_t)d1[j] * 256 + (long long)(int32_t)d2[j];
            if (p.nsplit > 1) {
#pragma unroll
                for (int j = 0; j < 16; ++j) atomicAdd(acc + (size_t)(c0 + j) * 128 + tr, (unsigned long long)v[j]);
            } else {
                tc_epi16(p, sg, c0, v, o, rv, rs, bias, tr16, o_lo, cinv, cpos, cseq);
            }
        }
        if (p.nsplit > 1) {
            __threadfence();
            named_bar_sync(1, 128);
            if (e == 0) {
                const unsigned t = atomicAdd(p.ctr + tile, 1u);
                *lastf = t == (unsigned)(p.nsplit - 1);
                if (*lastf) p.ctr[tile] = 0u;
            }
            named_bar_sync(1, 128);
            if (*lastf) {
                __threadfence();
                for (int c0 = 0; c0 < N; c0 += 16) {
                    long long v[16];
#pragma unroll
                    for (int j = 0; j < 16; ++j) v[j] = (long long)__ldcg(acc + (size_t)(c0 + j) * 128 + tr);
#pragma unroll
                    for (int j = 0; j < 16; ++j) acc[(size_t)(c0 + j) * 128 + tr] = 0ull;  // ready for the next launch
                    tc_epi16(p, sg, c0, v, o, rv, rs, bias, tr16, o_lo, cinv, cpos, cseq);
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tbase, C::TCOLS);
    }
}

// One block per input row: max |x| -> sh, then the three digit planes.
__global__ void tc_prep_kernel(const float *x, int ldx, int I, int Kp, int Mpad, int8_t *dig, float *inv) {
    pdl_wait();
    pdl_trigger();
    __shared__ float red[8];
    const int m = blockIdx.x, tid = threadIdx.x;
    const float *xr = x + (int64_t)m * ldx;
    float mx = 0.0f;
    for (int i = tid; i < I; i += 256) mx = fmaxf(mx, fabsf(xr[i]));
    for (int s = 16; s > 0; s >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, s));
    if ((tid & 31) == 0) red[tid >> 5] = mx;
    __syncthreads();
    mx = red[0];
    for (int w = 1; w < 8; ++w) mx = fmaxf(mx, red[w]);
    int sh = 0;
    if (mx > 0.0f && mx <= 3.4e38f) {
        int E;
        frexpf(mx, &E);  // mx < 2^E
        sh = min(126, 22 - E);
    }
    const float sc = ldexpf(1.0f, sh);
    if (tid == 0) inv[m] = ldexpf(1.0f, -sh);
    const int64_t plane = (int64_t)Mpad * Kp;
    int8_t *d0 = dig + (int64_t)m * Kp;
    for (int c = tid * 4; c < Kp; c += 256 * 4) {
        uint32_t w[3] = {0u, 0u, 0u};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int v = c + j < I ? __float2int_rn(__fmul_rn(xr[c + j], sc)) : 0;
            int hi, mid, lo;
            digits3(v, hi, mid, lo);
            w[0] |= (uint32_t)(hi & 255) << (8 * j);
            w[1] |= (uint32_t)(mid & 255) << (8 * j);
            w[2] |= (uint32_t)(lo & 255) << (8 * j);
        }
#pragma unroll
        for (int d = 0; d < 3; ++d) *reinterpret_cast<uint32_t *>(d0 + d * plane + c) = w[d];
    }
}

// Row-major copy of a T8 tile matrix, rows in tile order.
__global__ void tc_copy_t8_kernel(const uint8_t *tiles, int kblocks, int Op, int Ip, int8_t *out) {
    const int64_t total = (int64_t)Op * Ip / 4;
    for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
         idx += (int64_t)gridDim.x * blockDim.x) {
        const int r = (int)(idx * 4 / Ip), c = (int)(idx * 4 % Ip);
        const int rt = r >> 4, tr = r & 15, g = tr & 7, rh = tr >> 3;
        const int kc = c / 32, cc = c % 32;  // cc is a multiple of 4: one whole word
        const int qw = 2 * (cc / 16) + rh, t = (cc % 16) / 4;
        const uint32_t w = *reinterpret_cast<const uint32_t *>(tiles + ((int64_t)rt * kblocks + kc) * 512 +
                                                               (4 * g + t) * 16 + qw * 4);
        *reinterpret_cast<uint32_t *>(out + (int64_t)r * Ip + c) = w;
    }
}

// ------------------------------------------------------------ expert GEMMs ----
// One CTA: 128 weight rows (8 row tiles) of one expert's matrix x that
// expert's pairs, TE_N at a time.  Warp 0 copies the raw INT4 blocks (1-D bulk
// copies, one per row tile and 64-column step) into a TE_RR-deep ring; warps
// 1-8 dequantize a step into the 128-byte-swizzled f16 A tile ((n - 8) *
// scale in fp32, as the reference dequantizes, then rounded to f16) and run
// the epilogue; warp 10 loads the pairs' f16 input rows with 2-D TMA; warp 9
// allocates TMEM and issues tcgen05.mma kind::f16 (K = 16) into one f32
// accumulator.  Two CTAs share an SM (102 KB of shared memory and 128 TMEM
// columns each), so one CTA's dequantization overlaps the other's waits and
// epilogue.  Every wait is bounded.
constexpr int TE_RR = 6;                 // raw ring depth (64-column steps)
constexpr int TE_S = 2;                  // f16 A / B stages
constexpr int TE_RAW = 8 * 768;          // raw slot: 8 blocks of at most 768 bytes (gs16)
constexpr int TE_A = 128 * 128;          // f16 A tile: 128 rows x 64 columns
constexpr int TE_B = TE_N * 128;         // f16 B tile: TE_N rows x 64 columns
constexpr int TE_DQ = 256;                // dequantizing (and epilogue) threads: warps 1-8
constexpr int TE_THREADS = 32 * (TE_DQ / 32 + 3);  // + raw producer, MMA, B producer
constexpr int TE_SMEM = 1024 + TE_S * (TE_A + TE_B) + TE_RR * TE_RAW + 512 + 4 * TE_N;

// byte offset of (row, 4-column group at col) in a 128-byte-swizzled K-major
// tile with 128-byte rows (col a multiple of 4)
__device__ __forceinline__ uint32_t sw128_off(int row, int col) {
    return (uint32_t)((row >> 3) * 1024 + (row & 7) * 128 + ((((col >> 3) ^ (row & 7)) << 4) | ((col & 7) * 2)));
}

// f16 arithmetic on packed pairs, rounded to nearest (the explicit rounding
// mode also keeps the two from being contracted into one fused operation).
__device__ __forceinline__ uint32_t h2_sub(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
__device__ __forceinline__ uint32_t h2_mul(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
__device__ __forceinline__ uint32_t h2_dup(float s) {
    uint32_t d;
    asm("cvt.rn.f16x2.f32 %0, %1, %1;" : "=r"(d) : "f"(s));
    return d;
}

// Dequantizes lane L's 16 bytes of one T4 block (rows g, g + 8; columns
// 32m + 16h + 4t + j) into the f16 tile at row tile r.  Byte j of word q holds
// column 32m + 16h + 4t + j (q = 2m + h): row g in its low nibble, row g + 8
// in its high nibble.  Each nibble n becomes the f16 1024 + n by one byte
// permute per pair (0x64 as the high byte), then (1024 + n) - 1032 = n - 8
// exactly, and one f16 multiply by the group scale rounded to f16: the
// MMA's f16 operand (n - 8) * scale, within one f16 rounding of the fp32
// product the reference forms, in under two instructions per weight.
template <int GS>
__device__ __forceinline__ void te_dequant_chunk(const uint8_t *blk, int L, int r, uint8_t *A) {
    const int g = L >> 2, t = L & 3;
    const uint4 w4 = *reinterpret_cast<const uint4 *>(blk + L * 16);
    const uint32_t w[4] = {w4.x, w4.y, w4.z, w4.w};
    uint32_t sc[4][2];  // [16-column group q][row half], as f16 pairs
    if (GS == 32) {
        const float4 s = *reinterpret_cast<const float4 *>(blk + 512 + g * 16);
        sc[0][0] = sc[1][0] = h2_dup(s.x); sc[0][1] = sc[1][1] = h2_dup(s.y);
        sc[2][0] = sc[3][0] = h2_dup(s.z); sc[2][1] = sc[3][1] = h2_dup(s.w);
    } else if (GS == 64) {
        const float2 s = *reinterpret_cast<const float2 *>(blk + 512 + g * 8);
        const uint32_t a = h2_dup(s.x), b = h2_dup(s.y);
#pragma unroll
        for (int q = 0; q < 4; ++q) { sc[q][0] = a; sc[q][1] = b; }
    } else if (GS == 16) {
        const float4 s0 = *reinterpret_cast<const float4 *>(blk + 512 + g * 32);
        const float4 s1 = *reinterpret_cast<const float4 *>(blk + 512 + g * 32 + 16);
        sc[0][0] = h2_dup(s0.x); sc[0][1] = h2_dup(s0.y); sc[1][0] = h2_dup(s0.z); sc[1][1] = h2_dup(s0.w);
        sc[2][0] = h2_dup(s1.x); sc[2][1] = h2_dup(s1.y); sc[3][0] = h2_dup(s1.z); sc[3][1] = h2_dup(s1.w);
    } else {  // per-row scale: applied in the epilogue
#pragma unroll
        for (int q = 0; q < 4; ++q) { sc[q][0] = 0x3C003C00u; sc[q][1] = 0x3C003C00u; }  // 1.0
    }
    constexpr uint32_t C1032 = 0x64086408u;  // the f16 pair (1032, 1032)
#pragma unroll
    for (int q = 0; q < 4; ++q) {  // word q = 2m + h
        const int col = 32 * (q >> 1) + 16 * (q & 1) + 4 * t;
#pragma unroll
        for (int rh = 0; rh < 2; ++rh) {
            const uint32_t nib = (w[q] >> (4 * rh)) & 0x0F0F0F0Fu;  // byte j = n of column j
            // columns (0, 1) and (2, 3) as the f16 pairs 1024 + n
            const uint32_t v01 = __byte_perm(nib, 0x64646464u, 0x4140), v23 = __byte_perm(nib, 0x64646464u, 0x4342);
            uint32_t h01 = h2_sub(v01, C1032), h23 = h2_sub(v23, C1032);
            if (GS != 0) {
                h01 = h2_mul(h01, sc[q][rh]);
                h23 = h2_mul(h23, sc[q][rh]);
            }
            const int row = r * 16 + g + 8 * rh;
            *reinterpret_cast<uint2 *>(A + sw128_off(row, col)) = make_uint2(h01, h23);
        }
    }
}

template <int GS>
__global__ void __launch_bounds__(TE_THREADS, 2) tc_exp_kernel(const __grid_constant__ TcExpParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t *Abuf = smem, *Bbuf = smem + TE_S * TE_A, *Raw = Bbuf + TE_S * TE_B;
    uint64_t *raw_full = reinterpret_cast<uint64_t *>(Raw + TE_RR * TE_RAW);
    uint64_t *raw_empty = raw_full + TE_RR;
    uint64_t *a_full = raw_empty + TE_RR;
    uint64_t *b_full = a_full + TE_S;
    uint64_t *st_empty = b_full + TE_S;
    uint64_t *accf = st_empty + TE_S;      // accumulator of column tile ct complete
    uint64_t *acce = accf + 1;             // ... and read out (TMEM free for the next)
    uint32_t *tslot = reinterpret_cast<uint32_t *>(acce + 1);
    int *cpair = reinterpret_cast<int *>(Raw + TE_RR * TE_RAW + 512);  // [TE_N] pair of each column
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int e = p.e_lo + blockIdx.y, rt0 = blockIdx.x * 8;

    pdl_wait();  // the pair lists come from the router, the rows from the gather
    pdl_trigger();
    const int pbeg = __ldcg(p.pair_start + e), npair = __ldcg(p.pair_start + e + 1) - pbeg;
    if (npair <= 0) return;  // uniform: no barrier or TMEM touched yet
    const int nct = (npair + TE_N - 1) / TE_N;  // column tiles, in turn
    const int nk = p.kblocks;
    const uint8_t *tiles = p.table + (int64_t)(e - p.e_lo) * p.stride + p.off_tiles;

    if (threadIdx.x == 0) {
        for (int i = 0; i < TE_RR; ++i) {
            mbar_init(&raw_full[i], 1);
            mbar_init(&raw_empty[i], TE_DQ);
        }
        for (int i = 0; i < TE_S; ++i) {
            mbar_init(&a_full[i], TE_DQ);
            mbar_init(&b_full[i], 1);
            mbar_init(&st_empty[i], 1);
        }
        mbar_init(accf, 1);
        mbar_init(acce, TE_DQ);
        mbar_init_fence();
    }
    constexpr int W_MMA = TE_DQ / 32 + 1, W_B = TE_DQ / 32 + 2;
    if (warp == W_MMA) {
        tmem_alloc(tslot, TE_N);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *tslot;
    const int nsteps = nct * nk;  // step ig = ct * nk + i

    if (warp == 0) {
        if (lane == 0) {  // raw INT4 blocks (re-read for every column tile)
            int issued = 0;
            for (int ig = 0; ig < nsteps; ++ig) {
                const int i = ig % nk, sl = ig % TE_RR;
                if (ig >= TE_RR && !mbar_wait(&raw_empty[sl], ((ig / TE_RR) - 1) & 1, TC_WAIT_NS)) {
                    tc_fail(p.err, 3);
                    break;
                }
                issued = ig + 1;
                int nb = 0;
                for (int r = 0; r < 8; ++r) nb += rt0 + r < p.n_rt;
                mbar_arrive_expect_tx(&raw_full[sl], (uint32_t)(nb * p.blk_bytes));
                for (int r = 0; r < 8; ++r)
                    if (rt0 + r < p.n_rt)
                        bulk_load(Raw + sl * TE_RAW + r * p.blk_bytes,
                                  tiles + ((int64_t)(rt0 + r) * nk + i) * p.blk_bytes, (uint32_t)p.blk_bytes,
                                  &raw_full[sl]);
            }
            // every copy issued has landed before the CTA can exit (already
            // true unless a wait above gave up)
            for (int j = max(0, issued - TE_RR); j < issued; ++j)
                mbar_wait(&raw_full[j % TE_RR], (j / TE_RR) & 1, TC_WAIT_NS);
        }
    } else if (warp == W_B) {
        if (lane == 0) {  // f16 input rows
            tma_prefetch_desc(&p.bmap);
            int issued = 0;
            for (int ig = 0; ig < nsteps; ++ig) {
                const int i = ig % nk, ct = ig / nk, s = ig % TE_S;
                if (ig >= TE_S && !mbar_wait(&st_empty[s], ((ig / TE_S) - 1) & 1, TC_WAIT_NS)) {
                    tc_fail(p.err, 3);
                    break;
                }
                issued = ig + 1;
                mbar_arrive_expect_tx(&b_full[s], TE_B);
                tma_load_2d(Bbuf + s * TE_B, &p.bmap, &b_full[s], i * 64, pbeg + ct * TE_N);
            }
            for (int j = max(0, issued - TE_S); j < issued; ++j)
                mbar_wait(&b_full[j % TE_S], (j / TE_S) & 1, TC_WAIT_NS);
        }
    } else if (warp == W_MMA) {
        if (lane == 0) {  // MMA issuer
            bool ok = true;
            for (int ct = 0; ct < nct && ok; ++ct) {
                // N: this tile's pairs rounded up to 16 (the B rows past them are
                // other experts' pairs or zero fill; their columns are not read)
                const uint32_t idesc = idesc_f16(128, min(TE_N, (npair - ct * TE_N + 15) & ~15));
                // the previous tile's accumulator has been read out
                if (ct > 0 && !mbar_wait(acce, (ct - 1) & 1, TC_WAIT_NS)) {
                    tc_fail(p.err, 3);
                    ok = false;
                    break;
                }
                tc_fence_after();
                for (int i = 0; i < nk; ++i) {
                    const int ig = ct * nk + i, s = ig % TE_S;
                    if (!mbar_wait(&a_full[s], (ig / TE_S) & 1, TC_WAIT_NS) ||
                        !mbar_wait(&b_full[s], (ig / TE_S) & 1, TC_WAIT_NS)) {
                        tc_fail(p.err, 3);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t ad = sw128_desc(Abuf + s * TE_A), bd = sw128_desc(Bbuf + s * TE_B);
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        tc_mma_f16(tbase, ad + 2 * kk, bd + 2 * kk, idesc, i > 0 || kk > 0);
                    tc_commit(&st_empty[s]);
                }
                tc_commit(accf);  // fires once every MMA above has completed
            }
            if (!ok) tc_commit(accf);
        }
    } else {  // warps 1-8: dequantize every step; the epilogue after each column tile
        const int td = threadIdx.x - 32;
        // epilogue: lane quarter q of TMEM (warp % 4), column half ch
        const int q = warp & 3, tr = 32 * q + lane, ch = (warp - 1) >> 2;
        const int rt = rt0 + (tr >> 4), t16 = tr & 15;
        const int o = tile_row_to_logical(p.perm, 0, rt, t16);
        const bool rv = rt < p.n_rt && o < p.O;
        const uint8_t *eb = p.table + (int64_t)(e - p.e_lo) * p.stride;
        const float rs = (rv && p.off_rs >= 0) ? reinterpret_cast<const float *>(eb + p.off_rs)[o] : 1.0f;
        const float bias = (rv && p.off_bias >= 0) ? reinterpret_cast<const float *>(eb + p.off_bias)[o] : 0.0f;
        const uint32_t tl = tbase + ((uint32_t)(32 * q) << 16);
        bool ok = true;
        for (int ct = 0; ct < nct; ++ct) {
            for (int i = 0; i < nk && ok; ++i) {
                const int ig = ct * nk + i, sl = ig % TE_RR, s = ig % TE_S;
                if (!mbar_wait(&raw_full[sl], (ig / TE_RR) & 1, TC_WAIT_NS) ||
                    (ig >= TE_S && !mbar_wait(&st_empty[s], ((ig / TE_S) - 1) & 1, TC_WAIT_NS))) {
                    tc_fail(p.err, 3);
                    ok = false;
                    break;
                }
                uint8_t *A = Abuf + s * TE_A;
#pragma unroll
                for (int k = 0; k < 256 / TE_DQ; ++k) {
                    const int c = td + TE_DQ * k, r = c >> 5, L = c & 31;
                    if (rt0 + r < p.n_rt) {
                        te_dequant_chunk<GS>(Raw + sl * TE_RAW + r * p.blk_bytes, L, r, A);
                    } else {  // rows past the matrix: zero
                        const int g = L >> 2, t = L & 3;
#pragma unroll
                        for (int w = 0; w < 4; ++w)
#pragma unroll
                            for (int rh = 0; rh < 2; ++rh)
                                *reinterpret_cast<uint2 *>(
                                    A + sw128_off(r * 16 + g + 8 * rh, 32 * (w >> 1) + 16 * (w & 1) + 4 * t)) =
                                    make_uint2(0u, 0u);
                    }
                }
                fence_async_smem();
                mbar_arrive(&a_full[s]);
                mbar_arrive(&raw_empty[sl]);
            }
            // epilogue of column tile ct: thread = TMEM lane = weight row of the tile
            const int c0 = ct * TE_N, ncols = min(TE_N, npair - c0);
            if (td < TE_N) cpair[td] = td < ncols ? __ldcg(p.pair_list + pbeg + c0 + td) : 0;
            named_bar_sync(1, TE_DQ);
            if (!mbar_wait(accf, ct & 1, TC_WAIT_NS)) {
                tc_fail(p.err, 3);
                ok = false;
            }
            __syncwarp();
            tc_fence_after();
            constexpr int CH = TE_N * 128 / TE_DQ;  // columns per warp (TE_DQ / 128 warps per lane quarter)
            for (int cc = ch * CH; cc < (ch + 1) * CH; cc += 16) {
                uint32_t d[16];
                tmem_ld16(tl + cc, d);
                tmem_ld_wait();
                float x[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    float v = __uint_as_float(d[j]);
                    if (p.off_rs >= 0) v = __fmul_rn(v, rs);
                    if (p.off_bias >= 0) v = __fadd_rn(v, bias);
                    x[j] = v;
                }
                if (p.epi == EPI_SWIGLU) {
                    // gate = tile row g (logical 2i), up = g + 8 (2i + 1): lanes l, l ^ 8
                    float up[16];
#pragma unroll
                    for (int j = 0; j < 16; ++j) up[j] = __shfl_xor_sync(0xffffffffu, x[j], 8);
                    if (ok && rv && t16 < 8 && (o + 1) < p.O) {
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            const int n = cc + j;
                            if (n < ncols)
                                p.y[(int64_t)cpair[n] * p.ldy + (o >> 1)] =
                                    swiglu(x[j], up[j], p.swiglu_limit, p.swiglu_alpha);
                        }
                    }
                } else if (ok && rv) {
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const int n = cc + j;
                        if (n < ncols) p.y[(int64_t)cpair[n] * p.ldy + o] = x[j];
                    }
                }
            }
            tc_fence_before();
            named_bar_sync(1, TE_DQ);  // every lane's reads done; cpair free
            mbar_arrive(acce);
            if (!ok) break;
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == W_MMA) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tbase, TE_N);
    }
}

// One block per sorted pair slot: that pair's input row to f16 (zero past I).
__global__ void tc_exp_gather_kernel(const float *x, int ldx, int I, int K, int by_pair, const int *pair_start,
                                     const int *pair_list, int E, int Kp, __half *xg) {
    pdl_wait();
    pdl_trigger();
    const int qi = blockIdx.x;
    if (qi >= __ldcg(pair_start + E)) return;
    const int pr = __ldcg(pair_list + qi);
    const float *src = x + (int64_t)(by_pair ? pr : pr / K) * ldx;
    __half2 *dst = reinterpret_cast<__half2 *>(xg + (int64_t)qi * Kp);
    for (int c = threadIdx.x * 2; c < Kp; c += blockDim.x * 2) {
        const float a = c < I ? src[c] : 0.0f, b = c + 1 < I ? src[c + 1] : 0.0f;
        dst[c >> 1] = __floats2half2_rn(a, b);
    }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = [] {
        void *f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return (EncodeTiledFn) nullptr;
        return reinterpret_cast<EncodeTiledFn>(f);
    }();
    return fn;
}

// 2-D int8 map [rows][cols] (row stride = cols bytes), box 128 columns x
// box_rows rows, 128-byte swizzle, zero fill outside.
cudaError_t make_map(CUtensorMap &m, void *base, int cols, int rows, int box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return cudaErrorNotSupported;
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)cols};
    const cuuint32_t box[2] = {128u, (cuuint32_t)box_rows};
    const cuuint32_t es[2] = {1u, 1u};
    const CUresult r = fn(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, base, dims, strides, box, es,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

template <int N>
cudaError_t tc_set() {
    return cudaFuncSetAttribute(tc_gemm_kernel<N>, cudaFuncAttributeMaxDynamicSharedMemorySize, TcCfg<N>::SMEM);
}

}  // namespace

bool tc_driver_ready() { return encode_fn() != nullptr; }

cudaError_t tc_configure() {
    cudaError_t e = tc_set<32>();
    if (e == cudaSuccess) e = tc_set<64>();
    if (e == cudaSuccess) e = tc_set<128>();
    return e;
}

cudaError_t tc_weight_from_tiles(const TileDesc &t, TcWeight &w, cudaStream_t st) {
    if (t.fmt != TF_T8 || (t.Ip % 32) != 0) return cudaErrorInvalidValue;
    w.O = t.O;
    w.Op = t.Op;
    w.Ip = t.Ip;
    w.rs = t.rs;
    cudaError_t e = cudaMalloc(&w.q, (size_t)t.Op * t.Ip);
    if (e != cudaSuccess) return e;
    const int64_t total = (int64_t)t.Op * t.Ip / 4;
    const int blocks = (int)std::min<int64_t>((total + 255) / 256, 65536);
    tc_copy_t8_kernel<<<blocks, 256, 0, st>>>(t.tiles, t.kblocks, t.Op, t.Ip, w.q);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    return make_map(w.map, w.q, t.Ip, t.Op, 128);
}

cudaError_t tc_state_init(TcState &s, int max_rows, int max_kp, size_t part_bytes, int max_tiles) {
    s.Mpad = (max_rows + 127) / 128 * 128;
    s.Kp = (max_kp + 127) / 128 * 128;
    cudaError_t e = cudaMalloc(&s.dig, (size_t)3 * s.Mpad * s.Kp);
    if (e == cudaSuccess) e = cudaMemset(s.dig, 0, (size_t)3 * s.Mpad * s.Kp);
    if (e == cudaSuccess) e = cudaMalloc(&s.inv, (size_t)s.Mpad * 4);
    if (e == cudaSuccess) e = cudaMemset(s.inv, 0, (size_t)s.Mpad * 4);
    s.part_bytes = part_bytes;
    if (e == cudaSuccess) e = cudaMalloc(&s.part, part_bytes);
    if (e == cudaSuccess) e = cudaMemset(s.part, 0, part_bytes);  // split-K accumulators start (and end) at 0
    s.ctr_n = max_tiles;
    if (e == cudaSuccess) e = cudaMalloc(&s.ctr, (size_t)max_tiles * 4);
    if (e == cudaSuccess) e = cudaMemset(s.ctr, 0, (size_t)max_tiles * 4);
    for (int i = 0; e == cudaSuccess && i < 3; ++i) e = make_map(s.bmap[i], s.dig, s.Kp, 3 * s.Mpad, 32 << i);
    return e;
}

cudaError_t tc_prep_rows(const TcState &s, const float *x, int ldx, int M, int I, cudaStream_t st) {
    if (M < 1 || M > s.Mpad || I > s.Kp) return cudaErrorInvalidValue;
    return launch_k(tc_prep_kernel, dim3(M), dim3(256), 0, st, x, ldx, I, s.Kp, s.Mpad, s.dig, s.inv);
}

// One wave: tiles x nsplit <= SMs (one CTA per SM), at least 4 K-steps per split.
int tc_nsplit(int tiles, int ksteps, int nsm) {
    return std::max(1, std::min(nsm / std::max(1, tiles), ksteps / 4));
}

size_t tc_part_bytes(int tiles, int nsplit, int M) {
    if (nsplit <= 1) return 0;
    const int N = M <= 32 ? 32 : M <= 64 ? 64 : 128;
    return (size_t)tiles * N * 128 * 8;
}

cudaError_t tc_exp_init(TcExpState &s, int max_pairs, int max_kp) {
    s.rows = max_pairs;
    s.Kp = (max_kp + 63) / 64 * 64;
    cudaError_t e = cudaMalloc(&s.xg, (size_t)s.rows * s.Kp * 2);
    if (e == cudaSuccess) e = cudaMemset(s.xg, 0, (size_t)s.rows * s.Kp * 2);
    if (e != cudaSuccess) return e;
    EncodeTiledFn fn = encode_fn();
    if (!fn) return cudaErrorNotSupported;
    const cuuint64_t dims[2] = {(cuuint64_t)s.Kp, (cuuint64_t)s.rows};
    const cuuint64_t strides[1] = {(cuuint64_t)s.Kp * 2};
    const cuuint32_t box[2] = {64u, (cuuint32_t)TE_N};
    const cuuint32_t es[2] = {1u, 1u};
    const CUresult r = fn(&s.bmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, s.xg, dims, strides, box, es,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
    for (int gs : {0, 16, 32, 64}) {
        cudaError_t a = cudaSuccess;
        if (gs == 0) a = cudaFuncSetAttribute(tc_exp_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, TE_SMEM);
        if (gs == 16) a = cudaFuncSetAttribute(tc_exp_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize, TE_SMEM);
        if (gs == 32) a = cudaFuncSetAttribute(tc_exp_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, TE_SMEM);
        if (gs == 64) a = cudaFuncSetAttribute(tc_exp_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, TE_SMEM);
        if (a != cudaSuccess) return a;
    }
    s.on = true;
    return cudaSuccess;
}

cudaError_t tc_exp_gather(const TcExpState &s, const float *x, int ldx, int I, int K, bool by_pair,
                          const int *pair_start, const int *pair_list, int E, int max_pairs, cudaStream_t st) {
    if (max_pairs > s.rows || I > s.Kp) return cudaErrorInvalidValue;
    return launch_k(tc_exp_gather_kernel, dim3(max_pairs), dim3(256), 0, st, x, ldx, I, K, (int)by_pair, pair_start,
                    pair_list, E, s.Kp, s.xg);
}

cudaError_t tc_exp_launch(const TcExpParams &p, int gs, int n_local, int max_pairs, cudaStream_t st) {
    if (p.blk_bytes > 768 || p.Ip % 64) return cudaErrorInvalidValue;
    (void)max_pairs;
    const dim3 grid((p.n_rt + 7) / 8, n_local);
    switch (gs) {
        case 0: return launch_k(tc_exp_kernel<0>, grid, dim3(TE_THREADS), TE_SMEM, st, p);
        case 16: return launch_k(tc_exp_kernel<16>, grid, dim3(TE_THREADS), TE_SMEM, st, p);
        case 32: return launch_k(tc_exp_kernel<32>, grid, dim3(TE_THREADS), TE_SMEM, st, p);
        case 64: return launch_k(tc_exp_kernel<64>, grid, dim3(TE_THREADS), TE_SMEM, st, p);
    }
    return cudaErrorInvalidValue;
}

cudaError_t tc_launch(TcParams &p, int M, cudaStream_t st) {
    if (M < 1 || M > TC_MAX_ROWS || p.nseg < 1 || p.nseg > TC_MAX_SEGS) return cudaErrorInvalidValue;
    const int items = p.tile_base[p.nseg] * p.nsplit;
    p.M = M;
    if (M <= 32) return launch_k(tc_gemm_kernel<32>, dim3(items), dim3(TC_THREADS), TcCfg<32>::SMEM, st, p);
    if (M <= 64) return launch_k(tc_gemm_kernel<64>, dim3(items), dim3(TC_THREADS), TcCfg<64>::SMEM, st, p);
    return launch_k(tc_gemm_kernel<128>, dim3(items), dim3(TC_THREADS), TcCfg<128>::SMEM, st, p);
}

}  // namespace pc
