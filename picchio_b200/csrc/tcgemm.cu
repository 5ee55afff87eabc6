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

cudaError_t tc_launch(TcParams &p, int M, cudaStream_t st) {
    if (M < 1 || M > TC_MAX_ROWS || p.nseg < 1 || p.nseg > TC_MAX_SEGS) return cudaErrorInvalidValue;
    const int items = p.tile_base[p.nseg] * p.nsplit;
    p.M = M;
    if (M <= 32) return launch_k(tc_gemm_kernel<32>, dim3(items), dim3(TC_THREADS), TcCfg<32>::SMEM, st, p);
    if (M <= 64) return launch_k(tc_gemm_kernel<64>, dim3(items), dim3(TC_THREADS), TcCfg<64>::SMEM, st, p);
    return launch_k(tc_gemm_kernel<128>, dim3(items), dim3(TC_THREADS), TcCfg<128>::SMEM, st, p);
}

}  // namespace pc
