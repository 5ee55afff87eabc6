// layout.h - device weight layouts and the job table of the dequant GEMV.
//
// Weights keep the reference's values exactly (quant.h:32-41: INT4 value =
// nibble - 8 times an fp32 group or row scale; INT8 value = q times an fp32
// row scale) but are stored in HBM in "tiles" shaped for the GEMV:
//
//  T4 (INT4): the matrix is cut into row tiles of 16 rows; a row tile is a
//   contiguous run of blocks, one block per 64 columns.  A block is 512 bytes
//   of nibbles - 32 lanes x 16 bytes, where lane L = 4g + t holds its A
//   fragments of the two m16n8k32 s8 MMA steps of the block: word 2m + h
//   has, in byte j, column 32m + 16h + 4t + j of row g (low nibble) and of
//   row g + 8 (high nibble) - then the group scales of the block:
//   float[8 g][64/gs groups][row g, row g+8].  Per-row scaled INT4
//   (block_size 0) has no scale bytes in the block and a separate float[O]
//   row-scale array instead.
//  T8 (INT8): same 16-row tiles, blocks of 32 columns = 512 bytes, one
//   m16n8k32 step: word 2h + r of lane 4g + t has columns 16h + 4t + j of
//   row g (r = 0) or g + 8 (r = 1); plus a float[O] row-scale array.
//  F4 (MXFP4, OCP microscaling: E2M1 codes with one scale per 32 columns):
//   the T4 block geometry with group size 32, but word q of a lane holds the
//   four 4-bit codes of row g in bits 0-15 (column 32m + 16h + 4t + j in
//   bits 4j..4j+3) and those of row g + 8 in bits 16-31, so that one
//   byte-permute turns 16 bits into four signed bytes (2 x the E2M1 value:
//   0, 1, 2, 3, 4, 6, 8, 12 with the code's sign); the scales are the
//   decoded E8M0 factors 2^(e - 127) as fp32.
//  F32: row-major float[O][I].
//
// A row tile is therefore one contiguous byte range in which every lane's
// 16 bytes of a block are its A fragment, loaded with one 16-byte load.
//
// Row permutations (the values are unchanged; only which logical row sits in
// which tile row):
//  PERM_PAIR: gate_up rows 2p (gate) and 2p+1 (up) land in tile rows g and
//   g+8 of tile p/8, so the SwiGLU of pair p is computed inside one lane.
//  PERM_HEAD: within each attention head, dims j and j + head_dim/2 land in
//   tile rows g and g+8, so the RoPE rotation of (j, j+half) is in one lane.
#pragma once
#include <cstdint>

namespace pc {

enum TileFmt { TF_F32 = 0, TF_T8 = 1, TF_T4 = 2, TF_F4 = 3 };
// 4-bit formats share the T4 block geometry (64 columns per block).
__host__ __device__ constexpr bool tf_4bit(int fmt) { return fmt == TF_T4 || fmt == TF_F4; }
enum RowPerm { PERM_NONE = 0, PERM_PAIR = 1, PERM_HEAD = 2 };

struct TileDesc {
    int fmt = TF_F32;
    int O = 0, I = 0;       // logical shape
    int Op = 0, Ip = 0;     // padded: Op % 16 == 0; Ip % 64 (T4, F4) or % 32 (T8)
    int gs = 0;             // T4 group size (16, 32, 64) or 0 = per-row scale; F4: 32
    int kblocks = 0;        // blocks per row tile
    int blk_bytes = 0;
    int64_t unit_bytes = 0; // bytes per row tile
    int perm = PERM_NONE;
    int head_dim = 0;       // PERM_HEAD
    uint8_t *tiles = nullptr;  // device, [Op/16][kblocks][blk_bytes]
    float *rs = nullptr;       // device, [Op] per-row scales (T8, or T4 with gs == 0)
    float *f32 = nullptr;      // device, [O][I] (F32)
};

__host__ __device__ inline int t4_blk_bytes(int gs) { return 512 + (gs > 0 ? (64 / gs) * 64 : 0); }

// Logical row held by tile row tr (0..15) of row tile rt.
__host__ __device__ inline int tile_row_to_logical(int perm, int head_dim, int rt, int tr) {
    if (perm == PERM_PAIR) {
        int p = rt * 8 + (tr & 7);
        return 2 * p + (tr >> 3);
    }
    if (perm == PERM_HEAD) {
        int tiles_per_head = head_dim / 16, half = head_dim / 2;
        int h = rt / tiles_per_head, ti = rt % tiles_per_head;
        int j = ti * 8 + (tr & 7) + ((tr >> 3) ? half : 0);
        return h * head_dim + j;
    }
    return rt * 16 + tr;
}

constexpr int GEMV_MAXR = 8;       // B rows (input vectors) per job
constexpr int GEMV_MAX_JOBS = 1024;
constexpr int GEMV_INLINE_JOBS = 6;

// One job = one weight matrix applied to up to 8 input rows.
struct GemvJob {
    const uint8_t *tiles;  // row tile 0 of the matrix
    const float *rs;       // per-row scale [Op] or null
    const float *bias;     // [O] in logical row order, or null
    int n_rt;              // row tiles
    int O;                 // logical rows (outputs beyond are dropped)
    int nrows;             // input rows used (<= 8)
    int seg;               // EPI_QKV: 0 q, 1 k, 2 v
    int in_row[GEMV_MAXR];
    int out_row[GEMV_MAXR];
};

enum GemvEpi {
    EPI_STORE = 0,   // y[out_row][o] (+)= acc * 2^-e (* rs) (+ bias)
    EPI_SWIGLU = 1,  // y[out_row][p] = clamped SwiGLU(gate 2p, up 2p+1)
    EPI_QKV = 2,     // q -> qbuf, k/v -> KV cache, RoPE on q/k
    EPI_LOGITS = 3,  // y[out_row][o] = logits, greedy argmax per row
};

struct GemvParams {
    const GemvJob *jobs;
    const int *njobs;       // device-resident job count
    int fmt;                // TF_T4 / TF_F4 / TF_T8 (must match the kernel instance)
    int gs;                 // T4 group size or 0
    int kblocks, blk_bytes;
    int I, Ip;              // input row length (logical, padded)
    int perm, head_dim;
    int epi;
    const float *x;         // input rows, stride ldx
    int ldx;
    float *y;               // output rows, stride ldy
    int ldy;
    int residual;           // EPI_STORE: accumulate into y
    const float *res_src;   // EPI_STORE with residual: read the residual here (same indexing as y), or null = y
    float swiglu_limit, swiglu_alpha;
    // EPI_QKV
    const float *rope_cs, *rope_sn;  // [ctx][half]
    const int *row_pos;     // per input row: position
    const int *row_seq;     // per input row: KV sequence slot
    float *qbuf;
    int ldq;
    void *kcache, *vcache;  // [seq][ctx][KVH*hd] for this layer
    int kv_bf16;
    int64_t kv_seq_stride;  // elements between sequences
    int kv_ctx;
    int kv_dim;
    // EPI_LOGITS
    unsigned long long *argmax;  // per output row: packed (value, ~index)
    int *err;               // device error word
    int stages;             // pipeline depth for this launch
    int stage_bytes;
    int static_jobs;        // 1: the job table does not depend on earlier kernels
    int jobs_early;         // 1: the job table was written two or more kernels back (the down GEMV
                            //    reads the router's): read through L2 before the dependency wait
    int host_tiles;         // 1: some tiles may sit in mapped host memory (streamed residency): the
                            //    weight rings use per-lane cp.async instead of bulk (TMA) copies
    // Shared input rows: > 0 means the B operand holds input rows
    // 0..shared_rows-1 for the whole launch (filled once per CTA) and a job's
    // in_row[r] is the B column of its row r.  0: per-job B (in_row = x row).
    int shared_rows;
    // Job table carried in the launch itself (n_inline > 0): no global reads
    // before the first weight copy.
    int n_inline;
    GemvJob ijobs[GEMV_INLINE_JOBS];
};

}  // namespace pc
