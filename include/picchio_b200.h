/* picchio_b200.h - C ABI of the B200 (sm_100a) implementation of picchio's
 * per-token MoE hot path.
 *
 * The reference (benmaster82/picchio) keeps its engine in one C translation
 * unit with static functions; the entry points below are the ones a C host
 * (picchio.c's main / service_loop, or any FFI) binds in place of them.  Each
 * declaration names the reference interface it replaces.
 *
 * Conventions
 *  - Every call returns a pc_status; nothing calls exit().  pc_last_error()
 *    gives a one-line description of the last failure on the calling thread.
 *  - One pc_ctx per GPU (per expert-parallel rank).  Calls on a context are
 *    ordered on the context's CUDA stream and return after the results they
 *    promise are on the host.  A context is not thread-safe (nor is the
 *    reference: it keeps its state in globals).
 *  - Pointers named *_dev are device pointers; all others are host memory.
 *    The context's stream does not wait for other streams: device inputs
 *    must be complete when the call is made (synchronize the stream that
 *    wrote them first).
 *  - Expert parallelism (ep_size > 1): every rank makes the same calls in
 *    the same order; each MoE block exchanges expert outputs between the
 *    ranks' GPUs, and a rank that stops calling makes the others' next MoE
 *    step fail with PC_ERR_TIMEOUT after about two seconds.
 *  - No torch types, no C++ types: plain pointers and sizes.
 */
#ifndef PICCHIO_B200_H
#define PICCHIO_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    PC_OK = 0,
    PC_ERR_INVALID_ARG = 1,    /* null pointer, bad size, bad option */
    PC_ERR_IO = 2,             /* model directory or file unreadable */
    PC_ERR_FORMAT = 3,         /* tensor dtype / shape / group size not supported */
    PC_ERR_MISSING_TENSOR = 4, /* a required tensor is absent (e.g. sinks, an expert) */
    PC_ERR_CUDA = 5,           /* a CUDA runtime call failed */
    PC_ERR_OOM = 6,            /* device or pinned-host allocation failed */
    PC_ERR_RANGE = 7,          /* token id, position or batch outside the context */
    PC_ERR_TIMEOUT = 8,        /* a bounded device-side wait gave up */
    PC_ERR_NCCL = 9,           /* NCCL unavailable or a collective failed */
    PC_ERR_STATE = 10          /* call not valid in the context's current state */
} pc_status;

typedef struct pc_ctx pc_ctx;
typedef struct pc_qt pc_qt;

/* Weight formats, as quant.h:32-41 numbers them (QT.fmt).  PC_FMT_MXFP4 is
 * the reference's fmt 3 (OCP MXFP4: E2M1 codes two per byte, low nibble =
 * even column, one scale per 32 columns), which the reference declares but
 * converts to INT4 at build time (quant.h:334-336, convert.py:391-447); here
 * it runs natively, value = E2M1(code) * scale as convert.py:129-178
 * dequantizes it. */
enum { PC_FMT_F32 = 0, PC_FMT_INT8 = 1, PC_FMT_INT4 = 2, PC_FMT_MXFP4 = 3 };

typedef struct {
    int device;        /* CUDA device ordinal */
    int ctx_len;       /* KV positions per sequence (env CTX; reference default 512) */
    int kv_bf16;       /* 1: bf16 KV cache; 0: fp32, the reference's precision */
    int max_batch;     /* sequences served by pc_decode_batch (>= 1) */
    int ep_rank;       /* expert-parallel rank (0 when ep_size <= 1) */
    int ep_size;       /* expert-parallel group size; <= 1 means one GPU */
    const void *nccl_id; /* 128-byte ncclUniqueId from rank 0 when ep_size > 1 (one GPU per rank) */
    int use_graphs;    /* 1: replay decode steps as CUDA graphs */
    int expert_residency; /* 0: whole expert table in HBM; 1: pinned host + HBM cache */
    int expert_cache_slots; /* per layer, when expert_residency == 1 */
    int prefill_chunk; /* positions per pc_prefill step without device sampling (default 64, the
                          reference's PREFILL_BATCH); larger chunks put the expert GEMMs on the
                          tensor cores (from 32 routed rows per expert); at most 4096 / topk */
} pc_opts;

/* Model shape (the fields cfg_load reads, picchio.c:349-425). */
typedef struct {
    int hidden;          /* D */
    int n_layers;
    int n_heads;
    int n_kv_heads;
    int head_dim;
    int n_experts;
    int topk;
    int intermediate;    /* intermediate_size; gate_up has 2x rows */
    int vocab;
    int ctx_len;         /* max_position_embeddings */
    int sliding_window;
    float eps;
    float theta;
    float swiglu_limit;
    float swiglu_alpha;
    float routed_scale;
    float rope_factor, rope_beta_fast, rope_beta_slow;
    int rope_original_ctx, rope_truncate;
    int group_size;      /* expert INT4 group size (0 = per-row scale) */
    int attn_format;     /* PC_FMT_* of q/k/v/o */
    int attn_group_size; /* group size when attn_format == PC_FMT_INT4 */
    int layer_type[256]; /* 0 sliding, 1 full (picchio.c:389-409) */
    int expert_format;   /* PC_FMT_INT4 (0 also means INT4) or PC_FMT_MXFP4 (group size 32): what
                            pc_init_synthetic generates; pc_init sets it from the experts it loads */
} pc_model_cfg;

/* Fills *o with the defaults (device 0, ctx 512, fp32 KV, batch 1, graphs on,
 * prefill chunks of 64). */
void pc_default_opts(pc_opts *o);

/* Status name and the calling thread's last error message. */
const char *pc_status_string(pc_status s);
const char *pc_last_error(void);

/* Loads config.json and the safetensors shards of `model_dir` the way
 * picchio's main does (picchio.c:2836-3000: cfg_load, shard discovery,
 * load_dense_weights picchio.c:2531-2650) and uploads every dense weight and
 * the whole expert table (replacing the disk-streamed LRU of
 * picchio.c:1000-1068, expert_load picchio.c:698-888) to HBM. */
pc_status pc_init(const char *model_dir, const pc_opts *opts, pc_ctx **out);

/* Same model family with seeded random weights generated on the device:
 * N(0, 0.02) quantized as the reference converter does (convert.py:45-126).
 * Used for shapes too large to write as files (GPT-OSS-20B/120B). */
pc_status pc_init_synthetic(const pc_model_cfg *cfg, uint64_t seed, const pc_opts *opts,
                            pc_ctx **out);

void pc_free(pc_ctx *ctx);

/* The configuration in use (after config.json parsing). */
pc_status pc_get_config(const pc_ctx *ctx, pc_model_cfg *cfg);

/* One decode step: replaces forward_token (picchio.c:1655-1756) with greedy
 * sampling (sample_logits at TEMPERATURE=0, picchio.c:1555-1560), or the
 * device draw when pc_set_sampling is on.  Writes the next id to *next_tok.
 * tok outside [0, vocab) embeds as zeros like embed_token
 * (picchio.c:1478-1481). */
pc_status pc_forward_token(pc_ctx *ctx, int tok, int pos, int *next_tok);

/* Prompt encoding: replaces prefill_tokens (picchio.c:1936-1975) in blocks
 * of 64 positions.  Returns the greedy id after the last position, or, with
 * device sampling on (pc_set_sampling), the id drawn there; like the
 * reference's forward_prefill, every block then draws (and records) one id.
 * The repetition history is seeded by the caller (pc_history_push), as
 * prefill_tokens seeds g_history before its blocks (picchio.c:1963-1967). */
pc_status pc_prefill(pc_ctx *ctx, const int *ids, int n, int pos_base, int *next_tok);

/* The same into KV slot `seq` of a batched-decode context (seq <
 * opts.max_batch), so that pc_decode_batch row `seq` continues that prompt.
 * The reference serves one sequence; this is prefill_tokens
 * (picchio.c:1936-1975) per slot.  Greedy only (device sampling follows
 * sequence 0). */
pc_status pc_prefill_seq(pc_ctx *ctx, int seq, const int *ids, int n, int pos_base, int *next_tok);

/* B independent sequences, one token each (sequence b uses KV slot b): the
 * batched-decode form of forward_token.  B <= opts.max_batch. */
pc_status pc_decode_batch(pc_ctx *ctx, const int *toks, const int *pos, int B, int *next);

/* Decode of n steps of one sequence without host round trips: the decode
 * loop of picchio's main (picchio.c:3212-3287), greedy (TEMPERATURE=0) or
 * with the device draw when pc_set_sampling is on.  Step i feeds the id of
 * step i-1 (tok for i = 0) at position pos + i; out_ids[i] receives its next
 * id.  *device_ms (optional) receives
 * the device time of the n steps, from CUDA events on the context stream. */
pc_status pc_generate(pc_ctx *ctx, int tok, int pos, int n, int *out_ids, float *device_ms);

/* Fills positions [0, n_pos) of sequence `seq`'s KV cache in every layer with
 * seeded N(0, 1) values, standing in for a prompt of n_pos tokens when only
 * the decode that follows is measured (no reference counterpart: the
 * reference fills its KV cache only through prefill_tokens). */
pc_status pc_kv_fill_synthetic(pc_ctx *ctx, int seq, int n_pos, uint64_t seed);

/* Copies the logits of the last step (row `row` of a batch) to the host. */
pc_status pc_get_logits(pc_ctx *ctx, int row, float *logits, int n);

/* Sampling settings of sample_logits (picchio.c:1540-1649; the globals
 * g_temperature, g_top_p, g_top_k, g_rep_penalty of picchio.c:1510-1513). */
typedef struct {
    float temperature; /* below 1e-6: argmax of the penalized logits */
    float top_p;       /* nucleus mass; active in (0, 1) */
    int top_k;         /* active in (0, vocab) */
    float rep_penalty; /* active above 1: ids in the history are penalized */
} pc_sampling;

/* Replaces the host-side sample_logits (picchio.c:1540-1649) with a device
 * draw for every later single-sequence step (pc_forward_token, pc_prefill,
 * pc_generate): the next id is drawn from the step's logits on the device,
 * recorded in the device history and returned, with no logits copy.  NULL
 * restores the default (plain argmax, no history).  Batched decode
 * (pc_decode_batch) stays greedy per row. */
pc_status pc_set_sampling(pc_ctx *ctx, const pc_sampling *s);

/* The xorshift64 generator state of the draws (g_rng, picchio.c:1520-1526). */
pc_status pc_set_rng(pc_ctx *ctx, uint64_t state);
pc_status pc_get_rng(pc_ctx *ctx, uint64_t *state);

/* The repetition-penalty history (g_history, picchio.c:1516-1517; at most
 * 4096 ids).  push appends ids in [0, vocab) and skips others, as
 * prefill_tokens seeds it with the prompt (picchio.c:1963-1967); get copies
 * up to cap ids and sets *n to the history length. */
pc_status pc_history_reset(pc_ctx *ctx);
pc_status pc_history_push(pc_ctx *ctx, const int *ids, int n);
pc_status pc_history_get(pc_ctx *ctx, int *ids, int cap, int *n);

/* One draw with the current settings from a device logits row of vocab
 * floats (sample_logits itself, picchio.c:1540): advances the generator and
 * appends the id to the history like the step's draw.  The logits are not
 * modified. */
pc_status pc_sample(pc_ctx *ctx, const float *logits_dev, int *id);

/* The MoE block of one layer on M rows: replaces moe_forward
 * (picchio.c:1309-1466): router + top-k + softmax, gate_up + bias + clamped
 * SwiGLU, down + bias, weighted combine.  x_dev [M][D] are the normalized
 * hidden states, out_dev [M][D] receives the MoE output (no residual). */
pc_status pc_moe_layer(pc_ctx *ctx, int layer, const float *x_dev, float *out_dev, int M);

/* The expert part of moe_forward with the routing given (sel_dev [M][K]
 * expert ids, w_dev [M][K] combine weights): expert_apply
 * (picchio.c:1769-1791) for every (row, k) and the combine in k order. */
pc_status pc_moe_experts(pc_ctx *ctx, int layer, const float *x_dev, const int *sel_dev,
                         const float *w_dev, int M, float *out_dev);

/* Router selections of the last step (decode step, batch, prefill chunk or
 * MoE call): expert ids [n_layers][rows][topk] in selection order, the
 * top-k of moe_forward (picchio.c:1326-1340) that the reference dumps as
 * layerN.top_indices.  *rows receives the step's row count; cap (ids) must
 * hold n_layers * rows * topk, else PC_ERR_RANGE.  Every expert-parallel rank
 * routes identically. */
pc_status pc_get_routing(pc_ctx *ctx, int *expert_ids, int cap, int *rows);

/* Stage tensors of the last pc_forward_token, under the names the reference's
 * ORACLE_DIR dump uses (picchio.c:204-249), e.g. "layer0.pre_moe_norm".
 * Requires pc_set_trace(ctx, 1) before the step. */
pc_status pc_set_trace(pc_ctx *ctx, int on);
pc_status pc_get_stage(pc_ctx *ctx, const char *name, float *out, int n);
pc_status pc_dump(pc_ctx *ctx, const char *dir);  /* writes <name>.npy like ORACLE_DIR */

/* Expert residency (opts.expert_residency).  0: every expert in one HBM
 * table.  1: the counterpart of the reference's expert cache (ESlot,
 * cache_load_batch, LRU; picchio.c:121-136, 1000-1068) for expert tables
 * larger than HBM: all experts in pinned, device-mapped host memory and
 * opts.expert_cache_slots experts per layer in HBM.  A step reads a
 * non-resident expert over the host link (never waits for the host); after
 * the step the experts it read move into HBM slots, least recently used
 * slot first.  Results are identical in both modes. */

/* Makes the given experts of a layer resident in HBM now, the counterpart of
 * cache_load_batch / prefetch_issue (picchio.c:1000-1068, 1180-1230); ids
 * of other ranks or -1 are skipped.  PC_OK without work in mode 0. */
pc_status pc_expert_prefetch(pc_ctx *ctx, int layer, const int *eids, int n);

/* Residency counters since pc_init (the reference's cache hit/miss stats):
 * experts read from HBM slots, experts read from the host, bytes copied
 * into slots.  Any pointer may be NULL.  All zero in mode 0. */
pc_status pc_expert_stats(pc_ctx *ctx, uint64_t *hits, uint64_t *misses, uint64_t *bytes_h2d);

/* ---- weight-level operator: matmul_qt (quant.h:323-337) ---------------- */

/* Uploads one QT weight in the reference's host layout (quant.h:32-41):
 * fmt PC_FMT_F32: data = float[O*I]; PC_FMT_INT8: data = int8[O*I], scales =
 * float[O]; PC_FMT_INT4: data = packed nibbles [O][ceil(I/2)] (low nibble =
 * even column, value = nibble - 8), scales = float[O] (block_size 0) or
 * float[O][ceil(I/gs)] (block_size = gs); PC_FMT_MXFP4: data = packed E2M1
 * codes in the same layout, block_size 32, scales = float[O][ceil(I/32)]
 * (the decoded E8M0 factors, 2^(e - 127)). */
pc_status pc_qt_create(int device, int fmt, int O, int I, int block_size, const void *data,
                       const float *scales, pc_qt **out);
/* y_dev[S][O] = x_dev[S][I] . W^T on `stream` (a cudaStream_t, NULL = default).
 * Up to 8 rows share one pass over the weights; when their padded input rows
 * do not fit one CTA's shared memory together (INT4 beyond ~4100 columns at
 * 3-8 rows), the rows run as jobs of two, each job streaming the weights. */
pc_status pc_qt_matmul(pc_qt *w, const float *x_dev, float *y_dev, int S, void *stream);
/* The same product as pc_qt_matmul, bit for bit, for callers that must not
 * allocate device memory during the call: code running under a memory budget
 * that forbids new allocations, or that cannot afford the implicit
 * synchronization cudaMalloc brings.  pc_qt_matmul allocates a job table the
 * first time it sees each row count S; this entry point allocates nothing, at
 * any call: its scratch (the GEMV job table and job count, ~1 KB) is a static
 * device array of this library that every GPU loading the library holds
 * until exit.  The first call on a device looks up that array's device
 * address (cudaGetSymbolAddress) - make that first call before any stream
 * capture that would include it.  Every call rewrites the whole table before
 * the GEMV reads it.
 * Limits: S <= PC_QT_NOALLOC_MAX_ROWS (PC_ERR_RANGE beyond); rows that
 * pc_qt_matmul would split into two-row jobs (see above) are refused with
 * PC_ERR_FORMAT; one scratch per
 * device, so calls that overlap in time (other streams or threads) race and
 * must be serialized by the caller.  This entry point has no counterpart in
 * the reference. */
#define PC_QT_NOALLOC_MAX_ROWS 64
pc_status pc_qt_matmul_noalloc(pc_qt *w, const float *x_dev, float *y_dev, int S, void *stream);
/* Waits for `stream`, then reports (PC_ERR_TIMEOUT) and clears a device-side
 * failure of earlier pc_qt_matmul calls on w, or of pc_qt_matmul_noalloc
 * calls on w's device: the GEMV's bounded wait for its weight copies giving
 * up.  Allocates nothing.  No counterpart in the reference (its matmul_qt
 * runs on the host and cannot fail this way). */
pc_status pc_qt_check(pc_qt *w, void *stream);
/* out_dev[O][I] = dequantized weights, (nibble-8)*scale in fp32. */
pc_status pc_qt_dequant(pc_qt *w, float *out_dev, void *stream);
void pc_qt_free(pc_qt *w);

/* ---- expert parallelism -------------------------------------------------- */

/* Writes a fresh 128-byte ncclUniqueId (rank 0 calls this and shares it). */
pc_status pc_nccl_unique_id(void *out128);

/* ---- diagnostics ---------------------------------------------------------- */

/* Returns PC_ERR_TIMEOUT if a device-side bounded wait has given up since the
 * last call (and clears the flag), else PC_OK. */
pc_status pc_check_device(pc_ctx *ctx);

/* Counts kernels this library launched on the context (for measurement). */
uint64_t pc_kernel_launches(const pc_ctx *ctx);

/* Smallest number of rows in one step (batch or prefill chunk) that runs the
 * INT8 dense projections on the tensor cores, or 0 when that path is off
 * (non-INT8 dense weights, no tensor-map encoder, or PICCHIO_TC=0). */
int pc_tensor_core_min_rows(const pc_ctx *ctx);

/* Kernel timing: between begin and end, every hot-path launch is bracketed by
 * CUDA events on the context stream.  With graphs enabled each step is
 * captured into a one-off graph (the events become graph nodes), so the
 * events time the device only, free of host launch gaps; kernels then do not
 * overlap one another across the events.  Without graphs the step is issued
 * launch by launch.
 * pc_profile_get returns the summed duration and launch count of one label
 * ("expert_gate_up", "expert_down", "qkv", "o_proj", "lm_head",
 * "attention", "router").  Replaces the reference's t_attn / t_moe / t_head
 * wall-clock accumulators (picchio.c:1686-1747). */
pc_status pc_profile_begin(pc_ctx *ctx);
pc_status pc_profile_end(pc_ctx *ctx);
pc_status pc_profile_get(pc_ctx *ctx, const char *label, double *total_ms, int *count);

#ifdef __cplusplus
}
#endif
#endif /* PICCHIO_B200_H */
