// context.h - the device-side model and per-step state behind a pc_ctx.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>
#include <map>
#include <string>
#include <vector>

#include "../../include/picchio_b200.h"
#include "kernels.h"
#include "layout.h"
#include "residency.h"
#include "sample.h"
#include "tcgemm.h"

namespace pc {

struct DenseMat {
    TileDesc t;
    float *bias = nullptr;
};

struct Layer {
    float *in_ln = nullptr, *post_ln = nullptr;
    DenseMat wq, wk, wv, wo;
    float *sinks = nullptr;
    float *router = nullptr, *router_bias = nullptr;
    int layer_type = 0;
    uint8_t *experts = nullptr;  // local expert table: [E_local][stride]
};

// Geometry shared by every expert: where each part sits inside one expert's
// bytes (offsets -1 = part absent).
struct ExpertGeom {
    TileDesc gu, dn;  // geometry only (tiles/rs pointers unused)
    int64_t stride = 0;
    int64_t off_gu = 0, off_dn = 0, off_gu_rs = -1, off_dn_rs = -1, off_gu_b = -1, off_dn_b = -1;
};

// Job tables of the dense projections for one step shape.
struct DenseJobs {
    GemvJob *d_jobs = nullptr;  // device
    int *d_counts = nullptr;    // device, one count per job list
    std::vector<int> qkv_off, o_off;  // per layer: offset into d_jobs / index into d_counts
    std::vector<int> qkv_cnt_idx, o_cnt_idx;
    int lm_off = 0, lm_cnt_idx = 0;
    std::vector<GemvJob> h_jobs;  // host copies, for launches that carry their jobs inline
    std::vector<int> h_counts;
};

struct StepGraph {
    cudaGraphExec_t exec = nullptr;
    uint64_t launches = 0;  // kernels of this library in one replay
};

}  // namespace pc

struct pc_ctx {
    pc_model_cfg cfg{};
    pc_opts opts{};
    int dev = 0, nsm = 148, max_smem = 0;
    cudaStream_t st = nullptr;
    bool own_stream = true;

    // embedding and head
    int emb_fmt = pc::TF_T8, emb_gs = 0;
    void *emb = nullptr;
    float *emb_s = nullptr;
    pc::DenseMat lm_head;
    float *final_norm = nullptr;
    std::vector<pc::Layer> L;
    pc::ExpertGeom eg;
    int e_lo = 0, e_hi = 0;  // resident experts

    // RoPE tables [rope_len][hd/2]
    float *rope_cs = nullptr, *rope_sn = nullptr;
    int rope_len = 0;

    // KV cache per layer: [nseq][kv_ctx][KVH*hd], fp32 or bf16
    std::vector<void *> kc, vc;
    int kv_ctx = 0, nseq = 1;
    int64_t seq_stride = 0;

    // per-step buffers, sized for maxm rows
    int maxm = 0;
    int *d_tok = nullptr, *d_pos = nullptr, *d_seq = nullptr, *d_next = nullptr;
    float *h = nullptr, *hn = nullptr, *qbuf = nullptr, *attn = nullptr, *tmp = nullptr;
    float *act = nullptr, *eo = nullptr, *moe_out = nullptr, *logits = nullptr, *raw = nullptr;
    float *rlogits = nullptr, *rw = nullptr;
    int *sel = nullptr;  // router selections of the last step, [layer][maxm][topk]
    int route_rows = 0;  // rows of the last step's selections (pc_get_routing)
    int *pair_local = nullptr, *njobs = nullptr;
    pc::GemvJob *jobs_gu = nullptr, *jobs_dn = nullptr;
    unsigned *router_ctr = nullptr, *attn_ctr = nullptr;
    float *attn_part = nullptr;
    int attn_max_split = 1;
    unsigned long long *argmax = nullptr;
    int *err = nullptr;
    int max_logit_rows = 1;
    pc::Sampler smp;  // device sample_logits (pc_set_sampling); off: argmax
    pc::Residency res;  // streamed experts (opts.expert_residency == 1)

    std::map<uint64_t, pc::DenseJobs> dense_jobs;
    std::map<uint64_t, pc::StepGraph> graphs;

    // pinned host staging for one step's inputs / outputs
    int *h_tok = nullptr, *h_pos = nullptr, *h_next = nullptr;

    // expert parallelism (ep.cpp): the NCCL communicator (set-up only) and
    // the combine exchange over peer memory.  ep_blk[q] is rank q's exchange
    // block (flags, then two receive buffers of maxm * topk * hidden floats),
    // mapped into this process; ep_blk[ep_rank] is this rank's own.
    void *nccl_comm = nullptr;
    int ep_n = 1, ep_rank = 0;
    char *ep_blk[pc::EP_MAX_RANKS] = {};
    int64_t ep_rx_bytes = 0;
    unsigned *ep_state = nullptr;  // [0] epoch (exchanges completed), [1] push ticket

    bool trace = false;
    std::map<std::string, std::vector<float>> stages;
    uint64_t launches = 0;

    int *d_seq_rows = nullptr;  // 0, 1, ..., maxm-1 (batched decode: row b -> sequence b)
    int *d_seq_zero = nullptr;  // all 0 (prefill: every row in sequence 0)
    int *d_seq_one = nullptr;   // all one slot (pc_prefill_seq into a slot other than 0)
    int *h_err = nullptr;       // pinned mirror of the device error word
    std::vector<void *> allocs; // device allocations owned by the context
    void *pinned = nullptr;     // pinned staging block

    // tensor-core path for batches of rows (tcgemm.cu): state, and the INT8
    // dense weights as row-major copies (per layer q, k, v, o; then lm_head)
    pc::TcState tc;
    std::vector<pc::TcWeight> tcw;
    // expert GEMMs on the tensor cores (tcgemm.cu): gathered f16 rows and the
    // router's expert-sorted pair lists
    pc::TcExpState tex;
    int *pair_start = nullptr, *pair_list = nullptr;

    // on-device greedy loop (pc_generate)
    int *d_gen = nullptr;       // ids produced by the loop
    int *d_step = nullptr;      // loop step counter
    int gen_cap = 0;

    // kernel timing with CUDA events (pc_profile_*)
    bool prof = false;
    struct ProfEv {
        std::string label;
        cudaEvent_t a, b;
    };
    std::vector<ProfEv> prof_evs;
    std::map<std::string, std::pair<double, int>> prof_acc;
};

namespace pc {
// Context helpers shared by load.cu and model.cu.
pc_status fail(pc_status s, const std::string &msg);
pc_status cuda_fail(cudaError_t e, const char *what);
pc_status dalloc(pc_ctx *c, size_t bytes, void **out);
// Host -> device copy on the context's stream, complete on return.  (A
// plain cudaMemcpy from pageable memory returns once the data is staged,
// with the transfer still in flight on the legacy default stream, which a
// kernel on the context's non-blocking stream does not wait for.)
pc_status upload(pc_ctx *c, void *dst, const void *src, size_t bytes);
void tile_geom(TileDesc &t, int fmt, int O, int I, int gs, int perm, int hd);
int64_t tile_bytes(const TileDesc &t);
pc_status load_model(pc_ctx *c, const std::string &dir);
pc_status synth_model(pc_ctx *c, uint64_t seed);
pc_status alloc_runtime(pc_ctx *c);
pc_status device_setup(int dev, int *nsm, int *max_smem);
}  // namespace pc

#define PC_CU(x)                                                   \
    do {                                                           \
        cudaError_t e_ = (x);                                      \
        if (e_ != cudaSuccess) return ::pc::cuda_fail(e_, #x);     \
    } while (0)
#define PC_TRY(x)                                                  \
    do {                                                           \
        pc_status s_ = (x);                                        \
        if (s_ != PC_OK) return s_;                                \
    } while (0)
