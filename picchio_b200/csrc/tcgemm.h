// tcgemm.h - host interface of the tensor-core path for batches of input rows
// (tcgemm.cu): the INT8 dense projections (q/k/v, o_proj, lm_head) over
// 16..128 rows at once on tcgen05 s8 x s8 -> s32 MMAs.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "layout.h"

namespace pc {

constexpr int TC_MIN_ROWS = 16;   // batches of at least this many rows take the tensor-core path
constexpr int TC_MAX_ROWS = 128;  // rows per launch (MMA N)
constexpr int TC_MAX_SEGS = 3;    // weight matrices in one launch (q, k, v)
constexpr int TC_THREADS = 192;   // TMA warp, MMA warp, 4 epilogue warps

// One INT8 weight matrix, rows in tile order (row r of the copy is tile row
// r % 16 of row tile r / 16, i.e. logical row tile_row_to_logical(perm, hd,
// r / 16, r % 16)), plain row-major [Op][Ip] bytes, read by TMA.
struct TcWeight {
    int8_t *q = nullptr;
    int O = 0, Op = 0, Ip = 0;
    const float *rs = nullptr;  // per logical row scale
    CUtensorMap map;            // box 128 columns x 128 rows, 128-byte swizzle
};

struct TcSeg {
    CUtensorMap amap;
    const float *rs, *bias;
    int O, Op, seg;
};

// The kernel parameter (passed as a __grid_constant__ so the tensor maps
// stay in parameter space).
struct TcParams {
    TcSeg segs[TC_MAX_SEGS];
    int nseg;
    int tile_base[TC_MAX_SEGS + 1];  // first 128-row tile of each segment; [nseg] = total
    CUtensorMap bmap;                // input digits [3][Mpad][Kp] int8
    int Mpad;
    const float *inv;                // [M] 2^-sh of each input row
    int M, ksteps, nsplit;           // ksteps of 128 columns, split over nsplit CTAs per tile
    int32_t *part;                   // split-K accumulators, int64 [tiles][N][128], zero between launches
    unsigned *ctr;                   // per-tile tickets, zero between launches
    int *err;
    // epilogue (the GEMV's modes; input row m = output row m)
    int epi, perm, head_dim;
    float *y;
    int ldy, residual;
    const float *res_src;
    const float *rope_cs, *rope_sn;
    const int *row_pos, *row_seq;
    float *qbuf;
    int ldq;
    void *kcache, *vcache;
    int kv_bf16;
    int64_t kv_seq_stride;
    int kv_ctx, kv_dim;
    unsigned long long *argmax;
};

// Per-context state of the path.
struct TcState {
    bool on = false;
    int Mpad = 0, Kp = 0;
    int8_t *dig = nullptr;     // [3][Mpad][Kp]
    float *inv = nullptr;      // [Mpad]
    CUtensorMap bmap[3];       // digit planes, boxes of 32 / 64 / 128 rows
    int32_t *part = nullptr;
    size_t part_bytes = 0;
    unsigned *ctr = nullptr;
    int ctr_n = 0;
};

// ---- expert GEMMs on the tensor cores (many input rows per expert) --------
// One launch = one expert matrix (gate_up or down) of every resident expert
// over that expert's (token, k) pairs: INT4 tiles dequantized to f16 in
// shared memory ((n - 8) * scale rounded once), input rows gathered and
// rounded to f16, tcgen05 f16 x f16 -> f32 MMAs.
constexpr int TE_N = 128;            // pairs per CTA (MMA N)
constexpr int TE_MIN_PAIRS = 32;     // average pairs per expert from which run_moe uses this path

struct TcExpParams {
    const uint8_t *table;            // the layer's expert table
    int64_t stride;                  // bytes per expert
    int64_t off_tiles, off_rs, off_bias;  // within an expert; -1 = absent
    int kblocks, blk_bytes, n_rt, O, Ip;  // T4 tile geometry of this matrix
    int e_lo, e_hi;                  // resident experts (table slot = e - e_lo)
    const int *pair_start, *pair_list;  // from the router: pairs sorted by expert
    CUtensorMap bmap;                // gathered f16 input rows [pairs][Ip], box 64 x TE_N
    int epi, perm;                   // EPI_SWIGLU (gate_up, PERM_PAIR) or EPI_STORE (down)
    float *y;                        // output row = pair index
    int ldy;
    float swiglu_limit, swiglu_alpha;
    int *err;
};

struct TcExpState {
    bool on = false;
    int rows = 0, Kp = 0;            // capacity: pairs x padded input length
    __half *xg = nullptr;            // [rows][Kp]
    CUtensorMap bmap;
};

cudaError_t tc_exp_init(TcExpState &s, int max_pairs, int max_kp);
// Gathers the input row of every pair (down: row = pair index; otherwise row
// = pair / K) in expert order into s.xg, rounded to f16, zero past I.
cudaError_t tc_exp_gather(const TcExpState &s, const float *x, int ldx, int I, int K, bool by_pair,
                          const int *pair_start, const int *pair_list, int E, int max_pairs, cudaStream_t st);
cudaError_t tc_exp_launch(const TcExpParams &p, int gs, int n_local_experts, int max_pairs, cudaStream_t st);

// Resolves cuTensorMapEncodeTiled through the runtime (no link-time driver
// dependency); false when it is unavailable.
bool tc_driver_ready();
// Builds the row-major copy of a T8 tile matrix and its tensor map.
cudaError_t tc_weight_from_tiles(const TileDesc &t, TcWeight &w, cudaStream_t st);
cudaError_t tc_state_init(TcState &s, int max_rows, int max_kp, size_t part_bytes, int max_tiles);
// Input rows x[M][ldx] (I columns) -> three signed byte digits per value
// (x * 2^sh, rounded, |v| <= 2^22) and 2^-sh per row, as the GEMV's B
// operand is built.
cudaError_t tc_prep_rows(const TcState &s, const float *x, int ldx, int M, int I, cudaStream_t st);
// Split count and partial-sum bytes of a launch over the given weights.
int tc_nsplit(int tiles, int ksteps, int nsm);
size_t tc_part_bytes(int tiles, int nsplit, int M);
cudaError_t tc_configure();
cudaError_t tc_launch(TcParams &p, int M, cudaStream_t st);

}  // namespace pc
