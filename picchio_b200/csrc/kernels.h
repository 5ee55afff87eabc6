// kernels.h - host interface of the small kernels around the GEMV
// (kernels.cu) and of the weight preparation kernels (weights.cu).
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

#include "layout.h"

namespace pc {

// ---- per-step kernels --------------------------------------------------

// embed_token (picchio.c:1472-1503) for M rows; tokens outside [0, V) -> 0.
cudaError_t launch_embed(int fmt, const void *table, const float *scales, int gs, int V, int D,
                         const int *tok, int M, float *h, cudaStream_t st);

// rmsnorm (quant.h:396-402) of M rows of length D.
cudaError_t launch_rmsnorm(const float *x, const float *w, float *out, int M, int D, float eps,
                           cudaStream_t st);

struct AttnParams {
    const float *q;        // [M][H*hd]
    float *out;            // [M][H*hd]
    const void *kc, *vc;   // layer base: [seq][ctx][KVH*hd]
    int kv_bf16;
    int64_t seq_stride;    // elements
    int ctx;               // KV capacity
    const float *sinks;    // [H] or null
    const int *row_pos, *row_seq;
    int M, H, KVH, hd;
    int window;            // sliding window size, or 0 for full attention
    float *part;           // scratch [M][H][nsplit][hd + 2]
    unsigned *counter;     // [M][KVH], zero, self-resetting
    int nsplit;            // splits over positions (each <= ATTN_SPLIT positions)
};
constexpr int ATTN_SPLIT = 256;
// gqa_attention's score / softmax-with-sink / P.V part (picchio.c:556-607).
cudaError_t launch_attention(const AttnParams &a, cudaStream_t st);
// The tensor-core form (attention_tc.cu) for a bf16 KV cache, head size 64
// and 8 query heads per KV head; launch_attention picks it when
// attention_tc_ok.  Below ATTN_TC_MIN_ROWS rows it also splits the positions
// over CTAs (spans of 512).
constexpr int ATTN_TC_MIN_ROWS = 16;
bool attention_tc_ok(const AttnParams &a);
cudaError_t attention_tc_configure();
cudaError_t launch_attention_tc(const AttnParams &a, cudaStream_t st);

constexpr int ROUTER_MAX_PAIRS = 4096;  // (row, k) pairs one router launch sorts by expert

struct RouterParams {
    const float *x;        // [M][D] normalized rows
    const float *R;        // [E][D]
    const float *bias;     // [E] or null
    int M, D, E, K;
    int bias_first;        // 1: prefill order (picchio.c:1838), 0: decode (picchio.c:1323)
    float *logits;         // [M][E]
    int *sel;              // [M][K]
    float *w;              // [M][K]
    unsigned *counter;     // zero, self-resetting tickets: [0] the launch, [1 + b] row block b (row-block form)
    const int *sel_in;     // optional given routing [M][K] (skips router + top-k)
    // optional fused input norm: x[m] = rmsnorm(h_in[m], ln_w, eps) computed
    // in every block (exactly as rmsnorm_kernel does), written to hn_out[m]
    // by the blocks with blockIdx.x == 0; r.x is then unused.  D % 4 == 0.
    const float *h_in, *ln_w;
    float eps;
    float *hn_out;
    const float *w_in;
    // job building for the expert GEMVs
    const uint8_t *table;  // this layer's expert table
    int64_t stride;        // bytes per expert
    int64_t off_gu, off_dn, off_gu_rs, off_dn_rs, off_gu_b, off_dn_b;  // -1 = absent
    int gu_rt, dn_rt, gu_O, dn_O;
    int e_lo, e_hi;        // experts resident here (expert parallelism)
    // optional (streamed residency): [E] address of each expert's bytes, an
    // HBM cache slot or its pinned host copy; null: table + (e - e_lo) * stride
    const uint8_t *const *emap;
    unsigned char *used;   // optional [E]: set to 1 for every expert a job reads
    GemvJob *jobs_gu, *jobs_dn;
    int per_job;           // (row, k) pairs per job, 1..GEMV_MAXR (0 = GEMV_MAXR)
    int *njobs;            // [2]: gate_up, down
    int *pair_local;       // [M*K] 1 if the pair's expert is resident here
    // optional: pairs sorted by expert (pair_list, ascending pair index within
    // an expert) and each expert's first entry (pair_start[E + 1]); resident
    // experts only
    int *pair_start, *pair_list;
};
// Router dot products (picchio.c:1316-1324), top-k with strict '>'
// (picchio.c:1330-1340), softmax over the k logits (picchio.c:1355), and the
// per-expert job tables of the two expert GEMVs.
cudaError_t launch_router(const RouterParams &r, cudaStream_t st);
// Kernel attributes (shared-memory limits) once per device.
cudaError_t kernels_configure();

// ---- expert-parallel combine exchange ------------------------------------
//
// Under expert parallelism every rank holds every token's hidden row (the
// dense part is replicated) and routes identically, so the dispatch side of
// the MoE all-to-all needs no transfer: a rank's expert launches read their
// (token, k) rows from its own copy.  The combine side moves bytes: each
// (token, k) output row is computed on the rank owning that expert and is
// needed by every rank.  ep_push writes this rank's rows straight into every
// rank's receive buffer over NVLink (peer mappings of the other ranks'
// exchange blocks) and then bumps, in every rank's flag array, this rank's
// entry to the exchange number; the combine waits for all entries to reach
// it before reading.  Receive buffers alternate with the exchange number, so
// a rank that runs ahead writes the buffer its peers are not reading.
constexpr int EP_MAX_RANKS = 8;
constexpr int EP_FLAG_BYTES = 256;            // flag array at the start of each exchange block
constexpr long long EP_WAIT_NS = 2000000000;  // bounded wait for the peers' rows (2 s)
constexpr int EP_ERR_WAIT = 3;                // error word value when that wait gives up

struct EpPushParams {
    const float *eo;        // [P][D] this rank's expert outputs (rows of its own pairs)
    const int *pair_local;  // [P] 1 where the pair's expert is on this rank
    int P, D, rank, n;
    char *blk[EP_MAX_RANKS];  // every rank's exchange block, mapped here
    int64_t rx_bytes;         // bytes of one receive buffer
    unsigned *state;          // this rank's [epoch, ticket]
};
cudaError_t launch_ep_push(const EpPushParams &p, int nsm, cudaStream_t st);

// What the combine needs to read the exchanged rows (n = 0: no exchange,
// eo is read as given).
struct EpWait {
    const char *blk;         // this rank's exchange block
    int64_t rx_bytes;
    const unsigned *state;   // this rank's epoch (the exchange to wait for)
    int n;                   // ranks
    int *err;                // error word: EP_ERR_WAIT when the wait gives up
};

// out[m][i] = sum over k (in k order) of w[m][k]*scale * eo[m*K+k][i]
// (picchio.c:1445-1454); h[m][i] += out[m][i] when h != null.  With ln_w
// (h required) hn[m] = rmsnorm(h[m] after the add, ln_w, eps), bit-equal to
// launch_rmsnorm on that row.  With ep (n > 0) the rows come from the
// exchange's receive buffer instead of eo, once every rank has pushed.
cudaError_t launch_combine(const float *eo, const float *w, const int *sel, float scale, int M, int K,
                           int D, float *out, float *h, cudaStream_t st, const float *ln_w = nullptr,
                           float eps = 0.0f, float *hn = nullptr, const EpWait *ep = nullptr);

// y[m][o] = W[o] . x[m] for fp32 weights (matmul_f32, quant.h:117-148),
// then (optional) + bias, and either stored, added to y (residual) or handed
// to the q/k/v epilogue.
struct F32GemvParams {
    const float *W;
    int O, I;
    const float *x;
    int ldx, M;
    const float *bias;
    float *y;
    int ldy, residual;
};
cudaError_t launch_gemv_f32(const F32GemvParams &p, cudaStream_t st);

// q/k/v post-processing for projections computed without the fused
// epilogue: bias, RoPE and KV store from raw rows [M][Oq + 2*Ok].
struct QkvPostParams {
    const float *raw;
    int M;
    const float *bq, *bk, *bv;
    int H, KVH, hd;
    const float *rope_cs, *rope_sn;
    const int *row_pos, *row_seq;
    float *q;
    void *kc, *vc;
    int kv_bf16;
    int64_t seq_stride;
    int ctx;
};
cudaError_t launch_qkv_post(const QkvPostParams &p, cudaStream_t st);

// Packed greedy argmax of fp32 logit rows (first maximum wins).
cudaError_t launch_argmax_rows(const float *logits, int M, int V, unsigned long long *packed, cudaStream_t st);

// On-device decode loop bookkeeping: gen[*step] = next[0]; ++*step; ++pos[0].
cudaError_t launch_gen_advance(const int *next, int *pos, int *gen, int *step, cudaStream_t st);

// Greedy ids from the packed argmax words (and re-arms them).
cudaError_t launch_argmax_finish(unsigned long long *packed, int n, int *ids, int *ids2,
                                 cudaStream_t st);

// ---- weight preparation (weights.cu) -------------------------------------

// Host-layout matrix on the device -> tiled layout of `dst` (which must have
// its geometry filled and its buffers allocated).
cudaError_t retile_t4(const uint8_t *q4, const float *scales, int src_block_size, TileDesc &dst,
                      cudaStream_t st);
cudaError_t retile_t8(const int8_t *q8, const float *scales, TileDesc &dst, cudaStream_t st);
// Inverse view for tests: the dequantized value of every weight, logical order.
cudaError_t dequant_tiles(const TileDesc &d, float *out, cudaStream_t st);

// Seeded random weights, N(mean, std) before quantization, generated on the
// device and quantized as convert.py does (INT4 amax/7 per group with a 1e-8
// floor, round half to even, clip [-8,7]; INT8 amax/127, clip [-127,127]).
cudaError_t gen_i4_rowmajor(uint8_t *q4, float *scales, int O, int I, int gs, uint64_t seed,
                            float std_, cudaStream_t st);
cudaError_t gen_i8_rowmajor(int8_t *q8, float *scales, int O, int I, uint64_t seed, float std_,
                            cudaStream_t st);
// The same N(0, std) weights as MXFP4 (OCP rule: shared exponent
// floor(log2 max|w|) - 2, E2M1 round-to-nearest-even, saturating), codes in
// the packed host layout and one decoded scale per 32 columns.  I % 32 == 0.
cudaError_t gen_f4_rowmajor(uint8_t *q4, float *scales, int O, int I, uint64_t seed, float std_,
                            cudaStream_t st);
cudaError_t gen_f32(float *dst, int64_t n, uint64_t seed, float mean, float std_, cudaStream_t st);
// N(0, 1) into n elements of a KV cache (fp32 or bf16) starting at element off.
cudaError_t gen_kv(void *base, int64_t off, int64_t n, int bf16, uint64_t seed, cudaStream_t st);

}  // namespace pc
