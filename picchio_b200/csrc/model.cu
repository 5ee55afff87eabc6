// model.cu - the forward step on the device and the C ABI (picchio_b200.h).
//
// One step processes M token rows (a decode batch, or a prefill chunk of one
// sequence), in the layer order of forward_token (picchio.c:1655-1756):
//   embed -> per layer { rmsnorm, q/k/v GEMV + bias + RoPE + KV store,
//   attention, o GEMV + bias + residual, rmsnorm, router + top-k + softmax,
//   gate_up GEMV + bias + SwiGLU, down GEMV + bias, weighted combine +
//   residual } -> rmsnorm -> lm_head GEMV + greedy argmax.
// Decode steps are captured once per shape in a CUDA graph and replayed.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "context.h"
#include "ep.h"
#include "gemv.h"
#include "host_io.h"
#include "kernels.h"

namespace pc {

thread_local std::string g_last_error;

pc_status fail(pc_status s, const std::string &msg) {
    g_last_error = msg;
    return s;
}

pc_status cuda_fail(cudaError_t e, const char *what) {
    return fail(e == cudaErrorMemoryAllocation ? PC_ERR_OOM : PC_ERR_CUDA,
                std::string(what) + ": " + cudaGetErrorString(e));
}

namespace {
std::mutex g_cfg_mu;
bool g_configured[64] = {false};
}  // namespace

pc_status device_setup(int dev, int *nsm, int *max_smem) {
    PC_CU(cudaSetDevice(dev));
    cudaDeviceProp prop;
    PC_CU(cudaGetDeviceProperties(&prop, dev));
    if (prop.major < 10) return fail(PC_ERR_CUDA, std::string("device ") + prop.name + " is not sm_100 (B200)");
    *nsm = prop.multiProcessorCount;
    *max_smem = (int)prop.sharedMemPerBlockOptin;
    std::lock_guard<std::mutex> lk(g_cfg_mu);
    if (dev >= 0 && dev < 64 && !g_configured[dev]) {
        PC_CU(gemv_configure(*max_smem));
        PC_CU(tc_configure());
        PC_CU(kernels_configure());
        PC_CU(attention_tc_configure());
        g_configured[dev] = true;
    }
    return PC_OK;
}

pc_status dalloc(pc_ctx *c, size_t bytes, void **out) {
    *out = nullptr;
    if (bytes == 0) bytes = 16;
    cudaError_t e = cudaMalloc(out, bytes);
    if (e != cudaSuccess) return fail(PC_ERR_OOM, "cudaMalloc(" + std::to_string(bytes) + "): " + cudaGetErrorString(e));
    // Zeroed on the context's stream and waited for: a plain cudaMemset runs
    // on the legacy default stream, which the context's non-blocking stream
    // does not wait for, so an upload or kernel on that stream could land
    // before the zeroing and be wiped by it.
    e = cudaMemsetAsync(*out, 0, bytes, c->st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->st);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemset");
    c->allocs.push_back(*out);
    return PC_OK;
}

pc_status upload(pc_ctx *c, void *dst, const void *src, size_t bytes) {
    if (bytes == 0) return PC_OK;
    cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, c->st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->st);
    if (e != cudaSuccess) return cuda_fail(e, "host-to-device copy");
    return PC_OK;
}

namespace {

pc_status configure_device(pc_ctx *c) { return device_setup(c->dev, &c->nsm, &c->max_smem); }

// CUDA events around one launch while profiling (pc_profile_begin/end).
struct Prof {
    pc_ctx *c;
    const char *label;
    cudaEvent_t a = nullptr, b = nullptr;
    unsigned flags = 0;
    Prof(pc_ctx *cc, const char *l) : c(cc), label(l) {
        if (!c->prof) return;
        cudaEventCreate(&a);
        cudaEventCreate(&b);
        // under stream capture the record must be an (external) graph node
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        cudaStreamIsCapturing(c->st, &cs);
        flags = cs == cudaStreamCaptureStatusActive ? cudaEventRecordExternal : cudaEventRecordDefault;
        cudaEventRecordWithFlags(a, c->st, flags);
    }
    ~Prof() {
        if (!a) return;
        cudaEventRecordWithFlags(b, c->st, flags);
        c->prof_evs.push_back({label, a, b});
    }
};

// Launch one GEMV over a device job list.
pc_status run_gemv(pc_ctx *c, GemvParams p, int rows_per_job, const char *label) {
    p.err = c->err;
    const int nt = gemv_nt_for_rows(p.shared_rows > 0 ? p.shared_rows : rows_per_job);
    if (!gemv_plan(p, nt, c->max_smem))
        return fail(PC_ERR_FORMAT, "GEMV input of " + std::to_string(p.Ip) + " columns does not fit in shared memory");
    Prof pr(c, label);
    PC_CU(gemv_launch(p, nt, c->nsm, c->st));
    ++c->launches;
    return PC_OK;
}

void params_for(GemvParams &p, const TileDesc &t, int epi) {
    p.fmt = t.fmt;
    p.gs = t.gs;
    p.kblocks = t.kblocks;
    p.blk_bytes = t.blk_bytes;
    p.I = t.I;
    p.Ip = t.Ip;
    p.perm = t.perm;
    p.head_dim = t.head_dim;
    p.epi = epi;
    p.static_jobs = 1;  // dense job tables are built on the host; MoE clears this
}

GemvJob make_job(const TileDesc &t, const float *bias, int seg, const int *in, const int *out, int n) {
    GemvJob j;
    memset(&j, 0, sizeof j);
    j.tiles = t.tiles;
    j.rs = t.rs;
    j.bias = bias;
    j.n_rt = t.Op / 16;
    j.O = t.O;
    j.nrows = n;
    j.seg = seg;
    for (int i = 0; i < n; ++i) { j.in_row[i] = in[i]; j.out_row[i] = out[i]; }
    return j;
}

// Job tables of the dense projections for M rows; lm_mode 0: logits for
// every row, 1: last row only, 2: none.
pc_status dense_jobs(pc_ctx *c, int M, int lm_mode, DenseJobs **out) {
    const uint64_t key = (uint64_t)M * 4 + lm_mode;
    auto it = c->dense_jobs.find(key);
    if (it != c->dense_jobs.end()) { *out = &it->second; return PC_OK; }
    DenseJobs dj;
    std::vector<GemvJob> jobs;
    std::vector<int> counts;
    const int ng = (M + GEMV_MAXR - 1) / GEMV_MAXR;
    std::vector<int> rows(M);
    for (int i = 0; i < M; ++i) rows[i] = i;
    for (auto &ly : c->L) {
        dj.qkv_off.push_back((int)jobs.size());
        dj.qkv_cnt_idx.push_back((int)counts.size());
        int n = 0;
        if (ly.wq.t.fmt != TF_F32) {
            for (int g = 0; g < ng; ++g) {
                const int r0 = g * GEMV_MAXR, nr = std::min(GEMV_MAXR, M - r0);
                jobs.push_back(make_job(ly.wq.t, ly.wq.bias, 0, &rows[r0], &rows[r0], nr));
                jobs.push_back(make_job(ly.wk.t, ly.wk.bias, 1, &rows[r0], &rows[r0], nr));
                jobs.push_back(make_job(ly.wv.t, ly.wv.bias, 2, &rows[r0], &rows[r0], nr));
                n += 3;
            }
        }
        counts.push_back(n);
        dj.o_off.push_back((int)jobs.size());
        dj.o_cnt_idx.push_back((int)counts.size());
        n = 0;
        if (ly.wo.t.fmt != TF_F32) {
            for (int g = 0; g < ng; ++g) {
                const int r0 = g * GEMV_MAXR, nr = std::min(GEMV_MAXR, M - r0);
                jobs.push_back(make_job(ly.wo.t, ly.wo.bias, 0, &rows[r0], &rows[r0], nr));
                ++n;
            }
        }
        counts.push_back(n);
    }
    dj.lm_off = (int)jobs.size();
    dj.lm_cnt_idx = (int)counts.size();
    int n = 0;
    if (lm_mode != 2 && c->lm_head.t.fmt != TF_F32) {
        if (lm_mode == 1) {
            const int in = M - 1, o = 0;
            jobs.push_back(make_job(c->lm_head.t, nullptr, 0, &in, &o, 1));
            n = 1;
        } else {
            for (int g = 0; g < ng; ++g) {
                const int r0 = g * GEMV_MAXR, nr = std::min(GEMV_MAXR, M - r0);
                jobs.push_back(make_job(c->lm_head.t, nullptr, 0, &rows[r0], &rows[r0], nr));
                ++n;
            }
        }
    }
    counts.push_back(n);
    if (jobs.empty()) jobs.push_back(GemvJob{});
    PC_TRY(dalloc(c, jobs.size() * sizeof(GemvJob), (void **)&dj.d_jobs));
    PC_TRY(dalloc(c, counts.size() * 4, (void **)&dj.d_counts));
    PC_TRY(upload(c, dj.d_jobs, jobs.data(), jobs.size() * sizeof(GemvJob)));
    PC_TRY(upload(c, dj.d_counts, counts.data(), counts.size() * 4));
    dj.h_jobs = jobs;
    dj.h_counts = counts;
    auto res = c->dense_jobs.emplace(key, dj);
    *out = &res.first->second;
    return PC_OK;
}

// Points a launch at job list `cnt_idx` (starting at `off`) of a dense table:
// carried inline in the launch when it is short, else read from the device.
void use_jobs(GemvParams &p, const DenseJobs *dj, int off, int cnt_idx) {
    const int n = dj->h_counts[cnt_idx];
    p.jobs = dj->d_jobs + off;
    p.njobs = dj->d_counts + cnt_idx;
    p.n_inline = 0;
    if (n > 0 && n <= GEMV_INLINE_JOBS) {
        p.n_inline = n;
        for (int j = 0; j < n; ++j) p.ijobs[j] = dj->h_jobs[off + j];
    }
}

// Launches with at most 8 input rows keep them all in the B operand.
int shared_rows_for(int rows) { return rows <= GEMV_MAXR ? rows : 0; }

bool use_tc(const pc_ctx *c, int M) { return c->tc.on && M >= TC_MIN_ROWS; }

pc_status run_tc_block(pc_ctx *c, const GemvParams &g, const TcWeight *const *w, const float *const *bias, int nseg,
                       int M, const char *label);

// The dense projection described by g (epilogue fields set as for the GEMV)
// over input rows 0..M-1 on the tensor cores, TC_MAX_ROWS rows per launch (a
// short last block included: the MMA tile is zero-padded, rows past it are
// not stored).
pc_status run_tc(pc_ctx *c, const GemvParams &g, const TcWeight *const *w, const float *const *bias, int nseg, int M,
                 const char *label) {
    for (int r0 = 0; r0 < M; r0 += TC_MAX_ROWS) {
        const int m = std::min(TC_MAX_ROWS, M - r0);
        GemvParams b = g;
        b.x = g.x + (size_t)r0 * g.ldx;
        b.y = g.y ? g.y + (size_t)r0 * g.ldy : nullptr;
        b.res_src = g.res_src ? g.res_src + (size_t)r0 * g.ldy : nullptr;
        b.row_pos = g.row_pos ? g.row_pos + r0 : nullptr;
        b.row_seq = g.row_seq ? g.row_seq + r0 : nullptr;
        b.qbuf = g.qbuf ? g.qbuf + (size_t)r0 * g.ldq : nullptr;
        b.argmax = g.argmax ? g.argmax + r0 : nullptr;
        PC_TRY(run_tc_block(c, b, w, bias, nseg, m, label));
    }
    return PC_OK;
}

// One launch of at most TC_MAX_ROWS rows: the rows' digit planes, then the
// tcgen05 GEMM over the nseg weight matrices (q, k, v or a single one).
pc_status run_tc_block(pc_ctx *c, const GemvParams &g, const TcWeight *const *w, const float *const *bias, int nseg,
                       int M, const char *label) {
    TcParams t;
    memset(&t, 0, sizeof t);
    int tiles = 0;
    for (int s = 0; s < nseg; ++s) {
        t.segs[s].amap = w[s]->map;
        t.segs[s].rs = w[s]->rs;
        t.segs[s].bias = bias[s];
        t.segs[s].O = w[s]->O;
        t.segs[s].Op = w[s]->Op;
        t.segs[s].seg = s;
        t.tile_base[s] = tiles;
        tiles += (w[s]->Op + 127) / 128;
    }
    t.nseg = nseg;
    t.tile_base[nseg] = tiles;
    t.ksteps = (w[0]->Ip + 127) / 128;
    t.nsplit = tc_nsplit(tiles, t.ksteps, c->nsm);
    if (tc_part_bytes(tiles, t.nsplit, M) > c->tc.part_bytes || tiles > c->tc.ctr_n) t.nsplit = 1;
    t.bmap = c->tc.bmap[M <= 32 ? 0 : M <= 64 ? 1 : 2];
    t.Mpad = c->tc.Mpad;
    t.inv = c->tc.inv;
    t.part = c->tc.part;
    t.ctr = c->tc.ctr;
    t.err = c->err;
    t.epi = g.epi;
    t.perm = g.perm;
    t.head_dim = g.head_dim;
    t.y = g.y;
    t.ldy = g.ldy;
    t.residual = g.residual;
    t.res_src = g.res_src;
    t.rope_cs = g.rope_cs;
    t.rope_sn = g.rope_sn;
    t.row_pos = g.row_pos;
    t.row_seq = g.row_seq;
    t.qbuf = g.qbuf;
    t.ldq = g.ldq;
    t.kcache = g.kcache;
    t.vcache = g.vcache;
    t.kv_bf16 = g.kv_bf16;
    t.kv_seq_stride = g.kv_seq_stride;
    t.kv_ctx = g.kv_ctx;
    t.kv_dim = g.kv_dim;
    t.argmax = g.argmax;
    Prof pr(c, label);
    PC_CU(tc_prep_rows(c->tc, g.x, g.ldx, M, g.I, c->st));
    PC_CU(tc_launch(t, M, c->st));
    c->launches += 2;
    return PC_OK;
}

void trace_row(pc_ctx *c, const std::string &name, const float *dev, int n) {
    if (!c->trace) return;
    std::vector<float> v(n);
    cudaStreamSynchronize(c->st);
    cudaMemcpy(v.data(), dev, (size_t)n * 4, cudaMemcpyDeviceToHost);
    c->stages[name] = std::move(v);
}

void trace_row_i(pc_ctx *c, const std::string &name, const int *dev, int n) {
    if (!c->trace) return;
    std::vector<int> v(n);
    cudaStreamSynchronize(c->st);
    cudaMemcpy(v.data(), dev, (size_t)n * 4, cudaMemcpyDeviceToHost);
    std::vector<float> f(v.begin(), v.end());
    c->stages[name] = std::move(f);
}

// Layer l's slice of the router selections ([maxm][topk] expert ids).
int *layer_sel(pc_ctx *c, int l) { return c->sel + (size_t)l * c->maxm * c->cfg.topk; }

// The MoE block of one layer for M rows whose normalized states are x:
// router (or given routing), gate_up + SwiGLU, down, combine.
// With next_ln set, the combine also writes c->hn = rmsnorm(h, next_ln): the
// next layer's input norm or the final norm, saving their launches.
// The expert half of run_moe on the tensor cores (after the router kernel
// wrote the expert-sorted pair lists): gate_up + SwiGLU, down, combine.
pc_status run_moe_tc(pc_ctx *c, int l, const float *x, int M, float *out, float *h, const float *next_ln) {
    const pc_model_cfg &k = c->cfg;
    const int K = k.topk, D = k.hidden, P = M * K;
    Layer &ly = c->L[l];
    const bool ep = c->nccl_comm != nullptr;
    TcExpParams t;
    memset(&t, 0, sizeof t);
    t.table = ly.experts;
    t.stride = c->eg.stride;
    t.e_lo = c->e_lo;
    t.e_hi = c->e_hi;
    t.pair_start = c->pair_start;
    t.pair_list = c->pair_list;
    t.bmap = c->tex.bmap;
    t.err = c->err;
    auto geom = [&](const TileDesc &g, int64_t off, int64_t off_rs, int64_t off_b) {
        t.off_tiles = off;
        t.off_rs = off_rs;
        t.off_bias = off_b;
        t.kblocks = g.kblocks;
        t.blk_bytes = g.blk_bytes;
        t.n_rt = g.Op / 16;
        t.O = g.O;
        t.Ip = g.Ip;
        t.perm = g.perm;
    };
    {
        Prof pr(c, "expert_gate_up");
        PC_CU(tc_exp_gather(c->tex, x, D, D, K, false, c->pair_start, c->pair_list, k.n_experts, P, c->st));
        geom(c->eg.gu, c->eg.off_gu, c->eg.off_gu_rs, c->eg.off_gu_b);
        t.epi = EPI_SWIGLU;
        t.y = c->act;
        t.ldy = k.intermediate;
        t.swiglu_limit = k.swiglu_limit;
        t.swiglu_alpha = k.swiglu_alpha;
        PC_CU(tc_exp_launch(t, c->eg.gu.gs, c->e_hi - c->e_lo, P, c->st));
    }
    {
        Prof pr(c, "expert_down");
        PC_CU(tc_exp_gather(c->tex, c->act, k.intermediate, k.intermediate, K, true, c->pair_start, c->pair_list,
                            k.n_experts, P, c->st));
        geom(c->eg.dn, c->eg.off_dn, c->eg.off_dn_rs, c->eg.off_dn_b);
        t.epi = EPI_STORE;
        t.y = c->eo;
        t.ldy = D;
        PC_CU(tc_exp_launch(t, c->eg.dn.gs, c->e_hi - c->e_lo, P, c->st));
    }
    c->launches += 4;
    EpWait ew{};
    if (ep) {
        Prof pr(c, "ep_exchange");
        PC_TRY(ep_exchange(c, P));
        ew = ep_wait_view(c);
    }
    {
        Prof pr(c, "combine");
        PC_CU(launch_combine(c->eo, c->rw, layer_sel(c, l), k.routed_scale, M, K, D, out, h, c->st, next_ln,
                             k.eps, c->hn, &ew));
    }
    ++c->launches;
    return PC_OK;
}

// With norm_ln set, x is rmsnorm(h, norm_ln), computed inside the router
// kernel (which also writes it to x, i.e. c->hn) instead of by a launch of
// its own.
pc_status run_moe(pc_ctx *c, int l, const float *x, int M, const int *sel_in, const float *w_in,
                  int bias_first, float *out, float *h, const float *next_ln = nullptr,
                  const float *norm_ln = nullptr) {
    const pc_model_cfg &k = c->cfg;
    const int K = k.topk, D = k.hidden;
    Layer &ly = c->L[l];
    RouterParams r{};
    r.x = x;
    r.R = ly.router;
    r.bias = ly.router_bias;
    r.M = M;
    r.D = D;
    r.E = k.n_experts;
    r.K = K;
    r.bias_first = bias_first;
    r.logits = c->rlogits;
    r.sel = layer_sel(c, l);
    c->route_rows = M;
    r.w = c->rw;
    r.counter = c->router_ctr;
    r.sel_in = sel_in;
    r.w_in = w_in;
    r.table = ly.experts;
    r.stride = c->eg.stride;
    r.off_gu = c->eg.off_gu;
    r.off_dn = c->eg.off_dn;
    r.off_gu_rs = c->eg.off_gu_rs;
    r.off_dn_rs = c->eg.off_dn_rs;
    r.off_gu_b = c->eg.off_gu_b;
    r.off_dn_b = c->eg.off_dn_b;
    r.gu_rt = c->eg.gu.Op / 16;
    r.dn_rt = c->eg.dn.Op / 16;
    r.gu_O = c->eg.gu.O;
    r.dn_O = c->eg.dn.O;
    r.e_lo = c->e_lo;
    r.e_hi = c->e_hi;
    r.emap = c->res.on ? c->res.emap + (size_t)l * k.n_experts : nullptr;
    r.used = c->res.on ? c->res.used + (size_t)l * k.n_experts : nullptr;
    r.jobs_gu = c->jobs_gu;
    r.jobs_dn = c->jobs_dn;
    // Many rows but few pairs per expert (batched decode, ~2 per expert):
    // jobs of at most 4 pairs keep the expert GEMVs on two N-tiles with
    // deeper weight rings than 8-pair jobs (an expert with more pairs is
    // streamed once per job).  Otherwise up to GEMV_MAXR pairs per job; with
    // M <= GEMV_MAXR the B operand holds all M token rows (shared_rows below).
    r.per_job = (M > GEMV_MAXR && (int64_t)M * K <= 3LL * k.n_experts) ? 4 : GEMV_MAXR;
    r.njobs = c->njobs;
    r.pair_local = c->pair_local;
    // many pairs per expert (large prefill chunks, the single-layer
    // microbench): expert GEMMs on the tensor cores, fed by the router's
    // expert-sorted pair lists
    const bool tc_exp = c->tex.on && !c->trace && (int64_t)M * K >= (int64_t)TE_MIN_PAIRS * k.n_experts;
    if (tc_exp) {
        r.pair_start = c->pair_start;
        r.pair_list = c->pair_list;
    }
    if (norm_ln) {
        r.h_in = h;
        r.ln_w = norm_ln;
        r.eps = k.eps;
        r.hn_out = const_cast<float *>(x);
    }
    {
        Prof pr(c, "router");
        PC_CU(launch_router(r, c->st));
    }
    ++c->launches;
    if (c->trace) {
        const int last = M - 1;
        trace_row(c, "layer" + std::to_string(l) + ".router_logits", c->rlogits + (size_t)last * k.n_experts, k.n_experts);
        trace_row_i(c, "layer" + std::to_string(l) + ".top_indices", layer_sel(c, l) + (size_t)last * K, K);
        trace_row(c, "layer" + std::to_string(l) + ".top_weights", c->rw + (size_t)last * K, K);
    }
    if (tc_exp) return run_moe_tc(c, l, x, M, out, h, next_ln);
    const int rows = std::min(M, r.per_job);
    GemvParams p{};
    params_for(p, c->eg.gu, EPI_SWIGLU);
    p.static_jobs = 0;  // written by the router kernel
    p.host_tiles = c->res.on ? 1 : 0;  // streamed residency: a job may read a pinned host copy
    p.jobs = c->jobs_gu;
    p.njobs = c->njobs;
    p.x = x;
    p.ldx = D;
    p.y = c->act;
    p.ldy = k.intermediate;
    p.swiglu_limit = k.swiglu_limit;
    p.swiglu_alpha = k.swiglu_alpha;
    p.shared_rows = shared_rows_for(M);  // B column = token row
    PC_TRY(run_gemv(c, p, rows, "expert_gate_up"));
    const bool ep = c->nccl_comm != nullptr;
    params_for(p, c->eg.dn, EPI_STORE);
    p.static_jobs = 0;
    p.jobs_early = 1;  // written by the router, two launches back: weights stream before the wait
    p.host_tiles = c->res.on ? 1 : 0;
    p.jobs = c->jobs_dn;
    p.njobs = c->njobs + 1;
    p.x = c->act;
    p.ldx = k.intermediate;
    p.y = c->eo;
    p.ldy = D;
    // B column = (token, k) pair when that keeps one N-tile; otherwise each
    // expert's job fills B with just its own rows
    p.shared_rows = gemv_nt_for_rows(M * K) == 1 ? M * K : 0;
    PC_TRY(run_gemv(c, p, rows, "expert_down"));
    EpWait ew{};
    if (ep) {
        Prof pr(c, "ep_exchange");
        PC_TRY(ep_exchange(c, M * K));
        ew = ep_wait_view(c);
    }
    if (c->trace) {
        const int last = M - 1;
        for (int kk = 0; kk < K; ++kk) {
            trace_row(c, "layer" + std::to_string(l) + ".expert" + std::to_string(kk) + ".activated",
                      c->act + ((size_t)last * K + kk) * k.intermediate, k.intermediate);
            trace_row(c, "layer" + std::to_string(l) + ".expert" + std::to_string(kk) + ".output",
                      c->eo + ((size_t)last * K + kk) * D, D);
        }
    }
    {
        Prof pr(c, "combine");
        PC_CU(launch_combine(c->eo, c->rw, layer_sel(c, l), k.routed_scale, M, K, D, out, h, c->st, next_ln,
                             k.eps, c->hn, &ew));
    }
    ++c->launches;
    return PC_OK;
}

// One full step over M rows already staged in d_tok / d_pos with sequence
// slots `seq`.  lm_mode as in dense_jobs; nsplit_full = attention splits for
// full-attention layers.
pc_status run_step(pc_ctx *c, int M, const int *seq, int lm_mode, int nsplit_full, DenseJobs *dj,
                   bool feedback = false) {
    const pc_model_cfg &k = c->cfg;
    const int D = k.hidden, H = k.n_heads, KVH = k.n_kv_heads, hd = k.head_dim;
    PC_CU(launch_embed(c->emb_fmt, c->emb, c->emb_s, c->emb_gs, k.vocab, D, c->d_tok, M, c->h, c->st));
    ++c->launches;
    const int last = M - 1;
    trace_row(c, "embedding", c->h + (size_t)last * D, D);
    for (int l = 0; l < k.n_layers; ++l) {
        Layer &ly = c->L[l];
        const std::string pre = "layer" + std::to_string(l) + ".";
        trace_row(c, pre + "input", c->h + (size_t)last * D, D);
        if (l == 0) {  // later layers get it from the previous combine
            PC_CU(launch_rmsnorm(c->h, ly.in_ln, c->hn, M, D, k.eps, c->st));
            ++c->launches;
        }
        trace_row(c, pre + "pre_attn_norm", c->hn + (size_t)last * D, D);
        void *kc = c->kc[l], *vc = c->vc[l];
        if (ly.wq.t.fmt != TF_F32) {
            GemvParams p{};
            params_for(p, ly.wq.t, EPI_QKV);
            use_jobs(p, dj, dj->qkv_off[l], dj->qkv_cnt_idx[l]);
            p.shared_rows = shared_rows_for(M);
            p.x = c->hn;
            p.ldx = D;
            p.rope_cs = c->rope_cs;
            p.rope_sn = c->rope_sn;
            p.row_pos = c->d_pos;
            p.row_seq = seq;
            p.qbuf = c->qbuf;
            p.ldq = H * hd;
            p.kcache = kc;
            p.vcache = vc;
            p.kv_bf16 = c->opts.kv_bf16;
            p.kv_seq_stride = c->seq_stride;
            p.kv_ctx = c->kv_ctx;
            p.kv_dim = KVH * hd;
            if (use_tc(c, M)) {
                const TcWeight *w[3] = {&c->tcw[4 * l], &c->tcw[4 * l + 1], &c->tcw[4 * l + 2]};
                const float *b[3] = {ly.wq.bias, ly.wk.bias, ly.wv.bias};
                PC_TRY(run_tc(c, p, w, b, 3, M, "qkv"));
            } else {
                PC_TRY(run_gemv(c, p, std::min(M, GEMV_MAXR), "qkv"));
            }
        } else {
            const int Oq = H * hd, Ok = KVH * hd, ldr = Oq + 2 * Ok;
            F32GemvParams f{};
            f.I = D; f.x = c->hn; f.ldx = D; f.M = M; f.ldy = ldr;
            f.W = ly.wq.t.f32; f.O = Oq; f.y = c->raw;
            PC_CU(launch_gemv_f32(f, c->st));
            f.W = ly.wk.t.f32; f.O = Ok; f.y = c->raw + Oq;
            PC_CU(launch_gemv_f32(f, c->st));
            f.W = ly.wv.t.f32; f.O = Ok; f.y = c->raw + Oq + Ok;
            PC_CU(launch_gemv_f32(f, c->st));
            QkvPostParams q{};
            q.raw = c->raw; q.M = M; q.bq = ly.wq.bias; q.bk = ly.wk.bias; q.bv = ly.wv.bias;
            q.H = H; q.KVH = KVH; q.hd = hd; q.rope_cs = c->rope_cs; q.rope_sn = c->rope_sn;
            q.row_pos = c->d_pos; q.row_seq = seq; q.q = c->qbuf; q.kc = kc; q.vc = vc;
            q.kv_bf16 = c->opts.kv_bf16; q.seq_stride = c->seq_stride; q.ctx = c->kv_ctx;
            PC_CU(launch_qkv_post(q, c->st));
            c->launches += 4;
        }
        trace_row(c, pre + "q_rope", c->qbuf + (size_t)last * H * hd, H * hd);
        AttnParams a{};
        a.q = c->qbuf; a.out = c->attn; a.kc = kc; a.vc = vc; a.kv_bf16 = c->opts.kv_bf16;
        a.seq_stride = c->seq_stride; a.ctx = c->kv_ctx; a.sinks = ly.sinks; a.row_pos = c->d_pos;
        a.row_seq = seq; a.M = M; a.H = H; a.KVH = KVH; a.hd = hd;
        a.window = ly.layer_type == 0 ? k.sliding_window : 0;
        a.part = c->attn_part; a.counter = c->attn_ctr;
        a.nsplit = a.window > 0 ? std::max(1, std::min(c->attn_max_split, (a.window + ATTN_SPLIT - 1) / ATTN_SPLIT))
                                : nsplit_full;
        {
            Prof pr(c, "attention");
            PC_CU(launch_attention(a, c->st));
        }
        ++c->launches;
        trace_row(c, pre + "attn_concat", c->attn + (size_t)last * H * hd, H * hd);
        // o projection: + bias, + residual (picchio.c:615-616, 1691)
        float *ydst = c->trace ? c->tmp : c->h;
        if (ly.wo.t.fmt != TF_F32) {
            GemvParams p{};
            params_for(p, ly.wo.t, EPI_STORE);
            use_jobs(p, dj, dj->o_off[l], dj->o_cnt_idx[l]);
            p.shared_rows = shared_rows_for(M);
            p.x = c->attn;
            p.ldx = H * hd;
            p.y = ydst;
            p.ldy = D;
            p.residual = c->trace ? 0 : 1;
            if (use_tc(c, M)) {
                const TcWeight *w[1] = {&c->tcw[4 * l + 3]};
                const float *b[1] = {ly.wo.bias};
                PC_TRY(run_tc(c, p, w, b, 1, M, "o_proj"));
            } else {
                PC_TRY(run_gemv(c, p, std::min(M, GEMV_MAXR), "o_proj"));
            }
        } else {
            F32GemvParams f{};
            f.W = ly.wo.t.f32; f.O = D; f.I = H * hd; f.x = c->attn; f.ldx = H * hd; f.M = M;
            f.bias = ly.wo.bias; f.y = ydst; f.ldy = D; f.residual = c->trace ? 0 : 1;
            PC_CU(launch_gemv_f32(f, c->st));
            ++c->launches;
        }
        if (c->trace) {
            trace_row(c, pre + "attn_out", c->tmp + (size_t)last * D, D);
            // residual add exactly as the fused epilogue does it (one fp32 add)
            std::vector<float> hh((size_t)M * D), aa((size_t)M * D);
            cudaStreamSynchronize(c->st);
            cudaMemcpy(hh.data(), c->h, hh.size() * 4, cudaMemcpyDeviceToHost);
            cudaMemcpy(aa.data(), c->tmp, aa.size() * 4, cudaMemcpyDeviceToHost);
            for (size_t i = 0; i < hh.size(); ++i) hh[i] = hh[i] + aa[i];
            PC_TRY(upload(c, c->h, hh.data(), hh.size() * 4));
        }
        trace_row(c, pre + "post_attn_residual", c->h + (size_t)last * D, D);
        // the post-attention norm runs inside the router kernel, except when
        // tracing (its output is recorded before the router runs)
        const bool fuse_norm = !c->trace && (D & 3) == 0 && D <= 4096;
        if (!fuse_norm) {
            PC_CU(launch_rmsnorm(c->h, ly.post_ln, c->hn, M, D, k.eps, c->st));
            ++c->launches;
        }
        trace_row(c, pre + "pre_moe_norm", c->hn + (size_t)last * D, D);
        const float *next_ln = l + 1 < k.n_layers ? c->L[l + 1].in_ln : c->final_norm;
        PC_TRY(run_moe(c, l, c->hn, M, nullptr, nullptr, 0, c->trace ? c->moe_out : nullptr, c->h, next_ln,
                       fuse_norm ? ly.post_ln : nullptr));
        trace_row(c, pre + "moe_out", c->moe_out + (size_t)last * D, D);
        trace_row(c, pre + "output", c->h + (size_t)last * D, D);
    }
    if (k.n_layers == 0) {  // otherwise the last combine wrote it
        PC_CU(launch_rmsnorm(c->h, c->final_norm, c->hn, M, D, k.eps, c->st));
        ++c->launches;
    }
    trace_row(c, "final_norm", c->hn + (size_t)last * D, D);
    if (lm_mode == 2) return PC_OK;
    const int nlog = lm_mode == 1 ? 1 : M;
    if (c->lm_head.t.fmt != TF_F32) {
        GemvParams p{};
        params_for(p, c->lm_head.t, EPI_LOGITS);
        use_jobs(p, dj, dj->lm_off, dj->lm_cnt_idx);
        p.shared_rows = shared_rows_for(M);
        p.x = c->hn;
        p.ldx = D;
        p.y = c->logits;
        p.ldy = k.vocab;
        p.argmax = c->argmax;
        if (nlog == M && use_tc(c, M)) {
            const TcWeight *w[1] = {&c->tcw.back()};
            const float *b[1] = {nullptr};
            PC_TRY(run_tc(c, p, w, b, 1, M, "lm_head"));
        } else {
            PC_TRY(run_gemv(c, p, std::min(M, GEMV_MAXR), "lm_head"));
        }
    } else {
        F32GemvParams f{};
        f.W = c->lm_head.t.f32; f.O = k.vocab; f.I = D; f.x = c->hn + (size_t)(lm_mode == 1 ? M - 1 : 0) * D;
        f.ldx = D; f.M = nlog; f.y = c->logits; f.ldy = k.vocab;
        PC_CU(launch_gemv_f32(f, c->st));
        PC_CU(launch_argmax_rows(c->logits, nlog, k.vocab, c->argmax, c->st));
        c->launches += 2;
    }
    trace_row(c, "logits", c->logits + (size_t)(nlog - 1) * k.vocab, k.vocab);
    PC_CU(launch_argmax_finish(c->argmax, nlog, c->d_next, feedback ? c->d_tok : nullptr, c->st));
    ++c->launches;
    if (c->smp.on && nlog == 1) {  // sample_logits on the device: overwrites the argmax id
        int n = 0;
        PC_CU(sampler_launch(c->smp, c->logits, c->d_next, feedback ? c->d_tok : nullptr, c->err, c->st, n));
        c->launches += n;
    }
    if (feedback) {  // on-device loop: record the id, advance the position
        PC_CU(launch_gen_advance(c->d_next, c->d_pos, c->d_gen, c->d_step, c->st));
    }
    ++c->launches;
    return PC_OK;
}

int split_bucket(const pc_ctx *c, int max_pos) {
    int n = (std::min(max_pos, c->kv_ctx - 1) + 1 + ATTN_SPLIT - 1) / ATTN_SPLIT;
    int b = 1;
    while (b < n) b <<= 1;
    return std::min(b, c->attn_max_split);
}

pc_status check_err(pc_ctx *c) {
    if (*c->h_err) {
        const int v = *c->h_err;
        *c->h_err = 0;
        cudaMemsetAsync(c->err, 0, 4, c->st);
        if (v == SAMPLE_ERR_CANDIDATES)
            return fail(PC_ERR_RANGE, "sampling: more than " + std::to_string(SAMPLE_SORT_CAP) +
                                          " top-p candidates (values tied at the top-k threshold)");
        return fail(PC_ERR_TIMEOUT, "a device-side bounded wait gave up");
    }
    return PC_OK;
}

// Graph-key bits of the sampler configuration (its launches are part of the
// captured step).
uint64_t sampler_key(const pc_ctx *c) { return c->smp.on ? (c->smp.big ? 2ull : 1ull) << 56 : 0ull; }

// Runs `body` on the context stream: captured once into a CUDA graph under
// `key` and replayed afterwards, unless graphs are off or the step is traced
// or profiled (those need host work between kernels).
template <typename F>
pc_status run_graph(pc_ctx *c, uint64_t key, F &&body) {
    if (c->prof && c->opts.use_graphs && !c->trace) {
        // profiled step: a one-off graph, so that the events around each
        // launch (graph nodes) time the device without host launch gaps
        cudaGraph_t g = nullptr;
        PC_CU(cudaStreamBeginCapture(c->st, cudaStreamCaptureModeThreadLocal));
        pc_status s = body();
        cudaError_t e = cudaStreamEndCapture(c->st, &g);
        if (s != PC_OK) { if (g) cudaGraphDestroy(g); return s; }
        if (e != cudaSuccess) return cuda_fail(e, "cudaStreamEndCapture");
        cudaGraphExec_t ex = nullptr;
        e = cudaGraphInstantiate(&ex, g, 0);
        cudaGraphDestroy(g);
        if (e != cudaSuccess) return cuda_fail(e, "cudaGraphInstantiate");
        e = cudaGraphLaunch(ex, c->st);
        if (e == cudaSuccess) e = cudaStreamSynchronize(c->st);
        cudaGraphExecDestroy(ex);
        if (e != cudaSuccess) return cuda_fail(e, "profiled step");
        return PC_OK;
    }
    if (!c->opts.use_graphs || c->trace || c->prof) return body();
    auto it = c->graphs.find(key);
    if (it == c->graphs.end()) {
        cudaGraph_t g = nullptr;
        const uint64_t before = c->launches;
        PC_CU(cudaStreamBeginCapture(c->st, cudaStreamCaptureModeThreadLocal));
        pc_status s = body();
        cudaError_t e = cudaStreamEndCapture(c->st, &g);
        const uint64_t per_step = c->launches - before;
        c->launches = before;  // counted per replay below
        if (s != PC_OK) { if (g) cudaGraphDestroy(g); return s; }
        if (e != cudaSuccess) return cuda_fail(e, "cudaStreamEndCapture");
        cudaGraphExec_t ex = nullptr;
        e = cudaGraphInstantiate(&ex, g, 0);
        cudaGraphDestroy(g);
        if (e != cudaSuccess) return cuda_fail(e, "cudaGraphInstantiate");
        it = c->graphs.emplace(key, StepGraph{ex, per_step}).first;
    }
    PC_CU(cudaGraphLaunch(it->second.exec, c->st));
    c->launches += it->second.launches;
    return PC_OK;
}

// Decode-shaped step (tokens/positions in h_tok/h_pos, M rows, KV slot =
// row for batches, 0 for a single sequence): graph replay when enabled.
pc_status decode_step(pc_ctx *c, int M, int *next) {
    int maxp = 0;
    for (int i = 0; i < M; ++i) maxp = std::max(maxp, c->h_pos[i]);
    const int ns = split_bucket(c, maxp);
    const int *seq = c->d_seq_rows;
    DenseJobs *dj = nullptr;
    PC_TRY(dense_jobs(c, M, 0, &dj));  // before any capture: it allocates
    auto body = [&]() -> pc_status {
        PC_CU(cudaMemcpyAsync(c->d_tok, c->h_tok, (size_t)M * 4, cudaMemcpyHostToDevice, c->st));
        PC_CU(cudaMemcpyAsync(c->d_pos, c->h_pos, (size_t)M * 4, cudaMemcpyHostToDevice, c->st));
        PC_TRY(run_step(c, M, seq, 0, ns, dj));
        PC_CU(cudaMemcpyAsync(c->h_next, c->d_next, (size_t)(M) * 4, cudaMemcpyDeviceToHost, c->st));
        PC_CU(cudaMemcpyAsync(c->h_err, c->err, 4, cudaMemcpyDeviceToHost, c->st));
        return PC_OK;
    };
    PC_TRY(run_graph(c, ((uint64_t)M << 20) | (uint64_t)ns | sampler_key(c), body));
    PC_CU(cudaStreamSynchronize(c->st));
    PC_TRY(check_err(c));
    PC_TRY(res_after_step(c));
    for (int i = 0; i < M; ++i) next[i] = c->h_next[i];
    return PC_OK;
}

// Greedy decode of one sequence entirely on the device: each step's argmax
// becomes the next step's token without a host round trip (the decode loop
// of picchio.c:3212-3287 at TEMPERATURE=0).
pc_status generate(pc_ctx *c, int tok, int pos, int n, int *out, float *device_ms) {
    const int ns = split_bucket(c, pos + n - 1);
    DenseJobs *dj = nullptr;
    PC_TRY(dense_jobs(c, 1, 0, &dj));
    auto body = [&]() -> pc_status { return run_step(c, 1, c->d_seq_rows, 0, ns, dj, true); };
    c->h_tok[0] = tok;
    c->h_pos[0] = pos;
    PC_CU(cudaMemcpyAsync(c->d_tok, c->h_tok, 4, cudaMemcpyHostToDevice, c->st));
    PC_CU(cudaMemcpyAsync(c->d_pos, c->h_pos, 4, cudaMemcpyHostToDevice, c->st));
    PC_CU(cudaMemsetAsync(c->d_step, 0, 4, c->st));
    cudaEvent_t e0, e1;
    PC_CU(cudaEventCreate(&e0));
    PC_CU(cudaEventCreate(&e1));
    PC_CU(cudaEventRecord(e0, c->st));
    for (int i = 0; i < n; ++i) PC_TRY(run_graph(c, (1ull << 62) | (uint64_t)ns | sampler_key(c), body));
    PC_CU(cudaEventRecord(e1, c->st));
    PC_CU(cudaMemcpyAsync(out, c->d_gen, (size_t)n * 4, cudaMemcpyDeviceToHost, c->st));
    PC_CU(cudaMemcpyAsync(c->h_err, c->err, 4, cudaMemcpyDeviceToHost, c->st));
    PC_CU(cudaStreamSynchronize(c->st));
    float ms = 0.0f;
    cudaEventElapsedTime(&ms, e0, e1);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    if (device_ms) *device_ms = ms;
    PC_TRY(check_err(c));
    return res_after_step(c);
}

pc_status check_ctx(pc_ctx *c) {
    if (!c) return fail(PC_ERR_INVALID_ARG, "null context");
    cudaError_t e = cudaSetDevice(c->dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
    return PC_OK;
}

pc_status make_ctx(const pc_opts *opts, pc_ctx **out) {
    if (!out) return fail(PC_ERR_INVALID_ARG, "null output pointer");
    *out = nullptr;
    pc_ctx *c = new pc_ctx();
    if (opts) c->opts = *opts;
    else pc_default_opts(&c->opts);
    if (c->opts.expert_residency != 0 && c->opts.expert_residency != 1) {
        delete c;
        return fail(PC_ERR_INVALID_ARG, "expert_residency must be 0 (HBM table) or 1 (pinned host + HBM slots)");
    }
    c->dev = c->opts.device;
    pc_status s = configure_device(c);
    if (s != PC_OK) { delete c; return s; }
    cudaError_t e = cudaStreamCreateWithFlags(&c->st, cudaStreamNonBlocking);
    if (e != cudaSuccess) { delete c; return cuda_fail(e, "cudaStreamCreate"); }
    *out = c;
    return PC_OK;
}

// The tensor-core paths (tcgemm.cu): for INT4 experts, the gathered-row
// buffer and pair lists of the expert GEMMs; for INT8 dense projections,
// their row-major copies and the shared digit / partial-sum buffers (batches
// of 16..128 rows).  Off without the driver's tensor-map encoder or with
// PICCHIO_TC=0.
pc_status tc_setup(pc_ctx *c) {
    const char *v = getenv("PICCHIO_TC");
    if ((v && v[0] == '0') || !tc_driver_ready() || c->L.empty()) return PC_OK;
    // expert GEMMs (INT4 experts resident in HBM)
    if (!c->res.on && c->eg.gu.fmt == TF_T4 && c->eg.dn.fmt == TF_T4 && c->eg.gu.blk_bytes <= 768 && c->eg.dn.blk_bytes <= 768 &&
        c->eg.gu.Ip % 64 == 0 && c->eg.dn.Ip % 64 == 0) {
        const int pairs = c->maxm * c->cfg.topk;
        PC_TRY(dalloc(c, (size_t)(c->cfg.n_experts + 1) * 4, (void **)&c->pair_start));
        PC_TRY(dalloc(c, (size_t)pairs * 4, (void **)&c->pair_list));
        const cudaError_t e = tc_exp_init(c->tex, pairs, std::max(c->eg.gu.Ip, c->eg.dn.Ip));
        if (c->tex.xg) c->allocs.push_back(c->tex.xg);
        if (e != cudaSuccess) return cuda_fail(e, "tc_exp_init");
    }
    // dense projections (INT8)
    bool ok = c->lm_head.t.fmt == TF_T8;
    for (auto &ly : c->L)
        ok = ok && ly.wq.t.fmt == TF_T8 && ly.wk.t.fmt == TF_T8 && ly.wv.t.fmt == TF_T8 && ly.wo.t.fmt == TF_T8 &&
             ly.wk.t.perm == ly.wq.t.perm && ly.wv.t.perm == ly.wq.t.perm;
    if (!ok) return PC_OK;
    const int rows = std::min(c->maxm, TC_MAX_ROWS);
    size_t part = 16;
    int max_tiles = 1, max_kp = 0;
    auto need = [&](std::initializer_list<const TileDesc *> ts) {
        int tiles = 0, ip = 0;
        for (const TileDesc *t : ts) { tiles += (t->Op + 127) / 128; ip = t->Ip; }
        const int ks = (ip + 127) / 128;
        part = std::max(part, tc_part_bytes(tiles, tc_nsplit(tiles, ks, c->nsm), rows));
        max_tiles = std::max(max_tiles, tiles);
        max_kp = std::max(max_kp, ip);
    };
    need({&c->L[0].wq.t, &c->L[0].wk.t, &c->L[0].wv.t});
    need({&c->L[0].wo.t});
    need({&c->lm_head.t});
    c->tcw.assign(4 * c->L.size() + 1, TcWeight{});
    for (size_t l = 0; l < c->L.size(); ++l) {
        const TileDesc *ts[4] = {&c->L[l].wq.t, &c->L[l].wk.t, &c->L[l].wv.t, &c->L[l].wo.t};
        for (int i = 0; i < 4; ++i) {
            TcWeight &w = c->tcw[4 * l + i];
            cudaError_t e = tc_weight_from_tiles(*ts[i], w, c->st);
            if (w.q) c->allocs.push_back(w.q);
            if (e != cudaSuccess) return cuda_fail(e, "tc_weight_from_tiles");
        }
    }
    TcWeight &lm = c->tcw.back();
    cudaError_t e = tc_weight_from_tiles(c->lm_head.t, lm, c->st);
    if (lm.q) c->allocs.push_back(lm.q);
    if (e != cudaSuccess) return cuda_fail(e, "tc_weight_from_tiles");
    e = tc_state_init(c->tc, rows, max_kp, part, max_tiles);
    for (void *p : {(void *)c->tc.dig, (void *)c->tc.inv, (void *)c->tc.part, (void *)c->tc.ctr})
        if (p) c->allocs.push_back(p);
    if (e != cudaSuccess) return cuda_fail(e, "tc_state_init");
    PC_CU(cudaStreamSynchronize(c->st));
    c->tc.on = true;
    return PC_OK;
}

pc_status finish_init(pc_ctx *c) {
    if (c->opts.ep_size > 1) PC_TRY(ep_init(c));
    PC_TRY(tc_setup(c));
    // Allocations are zeroed with cudaMemset, on the legacy default stream:
    // the context's non-blocking stream does not wait for it, so every
    // zeroing (and upload) must be complete before the first step runs.
    PC_CU(cudaDeviceSynchronize());
    return PC_OK;
}

void expert_range(pc_ctx *c) {
    const int E = c->cfg.n_experts;
    const int n = c->opts.ep_size > 1 ? c->opts.ep_size : 1, r = c->opts.ep_size > 1 ? c->opts.ep_rank : 0;
    c->e_lo = (int)((int64_t)E * r / n);
    c->e_hi = (int)((int64_t)E * (r + 1) / n);
}

}  // namespace
}  // namespace pc

using namespace pc;

extern "C" {

void pc_default_opts(pc_opts *o) {
    if (!o) return;
    memset(o, 0, sizeof *o);
    o->device = 0;
    o->ctx_len = 512;
    o->kv_bf16 = 0;
    o->max_batch = 1;
    o->ep_size = 1;
    o->use_graphs = 1;
    o->prefill_chunk = 64;
}

const char *pc_status_string(pc_status s) {
    switch (s) {
        case PC_OK: return "PC_OK";
        case PC_ERR_INVALID_ARG: return "PC_ERR_INVALID_ARG";
        case PC_ERR_IO: return "PC_ERR_IO";
        case PC_ERR_FORMAT: return "PC_ERR_FORMAT";
        case PC_ERR_MISSING_TENSOR: return "PC_ERR_MISSING_TENSOR";
        case PC_ERR_CUDA: return "PC_ERR_CUDA";
        case PC_ERR_OOM: return "PC_ERR_OOM";
        case PC_ERR_RANGE: return "PC_ERR_RANGE";
        case PC_ERR_TIMEOUT: return "PC_ERR_TIMEOUT";
        case PC_ERR_NCCL: return "PC_ERR_NCCL";
        case PC_ERR_STATE: return "PC_ERR_STATE";
    }
    return "PC_ERR_UNKNOWN";
}

const char *pc_last_error(void) { return g_last_error.c_str(); }

pc_status pc_init(const char *model_dir, const pc_opts *opts, pc_ctx **out) {
    if (!model_dir) return fail(PC_ERR_INVALID_ARG, "null model_dir");
    pc_ctx *c = nullptr;
    PC_TRY(make_ctx(opts, &c));
    std::string err;
    // the expert range needs the config first
    pc_status s = PC_OK;
    if (!load_config(model_dir, &c->cfg, &err)) s = fail(PC_ERR_IO, err);
    else expert_range(c);
    if (s == PC_OK) s = load_model(c, model_dir);
    if (s == PC_OK) s = finish_init(c);
    if (s != PC_OK) { pc_free(c); return s; }
    *out = c;
    return PC_OK;
}

pc_status pc_init_synthetic(const pc_model_cfg *cfg, uint64_t seed, const pc_opts *opts, pc_ctx **out) {
    if (!cfg) return fail(PC_ERR_INVALID_ARG, "null cfg");
    pc_ctx *c = nullptr;
    PC_TRY(make_ctx(opts, &c));
    c->cfg = *cfg;
    if (c->cfg.swiglu_alpha == 0.0f) c->cfg.swiglu_alpha = 1.702f;
    if (c->cfg.routed_scale == 0.0f) c->cfg.routed_scale = 1.0f;
    if (c->cfg.eps == 0.0f) c->cfg.eps = 1e-5f;
    if (c->cfg.theta == 0.0f) c->cfg.theta = 150000.0f;
    if (c->cfg.swiglu_limit == 0.0f) c->cfg.swiglu_limit = 7.0f;
    if (c->cfg.ctx_len == 0) c->cfg.ctx_len = 131072;
    if (c->cfg.rope_factor == 0.0f) c->cfg.rope_factor = 1.0f;
    expert_range(c);
    pc_status s = synth_model(c, seed);
    if (s == PC_OK) s = finish_init(c);
    if (s != PC_OK) { pc_free(c); return s; }
    *out = c;
    return PC_OK;
}

void pc_free(pc_ctx *c) {
    if (!c) return;
    cudaSetDevice(c->dev);
    if (c->st) cudaStreamSynchronize(c->st);
    for (auto &g : c->graphs) cudaGraphExecDestroy(g.second.exec);
    c->graphs.clear();
    ep_destroy(c);
    sampler_free(c->smp);
    res_free(c);
    for (void *p : c->allocs) cudaFree(p);
    if (c->pinned) cudaFreeHost(c->pinned);
    if (c->st) cudaStreamDestroy(c->st);
    delete c;
}

pc_status pc_get_config(const pc_ctx *c, pc_model_cfg *cfg) {
    if (!c || !cfg) return fail(PC_ERR_INVALID_ARG, "null argument");
    *cfg = c->cfg;
    return PC_OK;
}

pc_status pc_forward_token(pc_ctx *c, int tok, int pos, int *next_tok) {
    PC_TRY(check_ctx(c));
    if (!next_tok) return fail(PC_ERR_INVALID_ARG, "null next_tok");
    if (pos < 0 || pos >= c->kv_ctx) return fail(PC_ERR_RANGE, "position " + std::to_string(pos) + " outside the KV capacity " + std::to_string(c->kv_ctx));
    c->h_tok[0] = tok;
    c->h_pos[0] = pos;
    c->stages.clear();
    return decode_step(c, 1, next_tok);
}

pc_status pc_decode_batch(pc_ctx *c, const int *toks, const int *pos, int B, int *next) {
    PC_TRY(check_ctx(c));
    if (!toks || !pos || !next) return fail(PC_ERR_INVALID_ARG, "null argument");
    if (B < 1 || B > c->nseq || B > 256) return fail(PC_ERR_RANGE, "batch " + std::to_string(B) + " outside [1, max_batch]");
    for (int i = 0; i < B; ++i) {
        if (pos[i] < 0 || pos[i] >= c->kv_ctx) return fail(PC_ERR_RANGE, "position outside the KV capacity");
        c->h_tok[i] = toks[i];
        c->h_pos[i] = pos[i];
    }
    c->stages.clear();
    return decode_step(c, B, next);
}

pc_status pc_prefill(pc_ctx *c, const int *ids, int n, int pos_base, int *next_tok) {
    return pc_prefill_seq(c, 0, ids, n, pos_base, next_tok);
}

pc_status pc_prefill_seq(pc_ctx *c, int seq, const int *ids, int n, int pos_base, int *next_tok) {
    PC_TRY(check_ctx(c));
    if (!ids || !next_tok || n < 1) return fail(PC_ERR_INVALID_ARG, "empty prompt");
    if (pos_base < 0 || pos_base + n > c->kv_ctx) return fail(PC_ERR_RANGE, "prompt does not fit the KV capacity");
    if (seq < 0 || seq >= c->nseq) return fail(PC_ERR_RANGE, "sequence slot outside [0, max_batch)");
    if (seq != 0 && c->smp.on) return fail(PC_ERR_STATE, "device sampling serves sequence 0 only");
    const int *seq_rows = c->d_seq_zero;  // every row of the step in slot seq
    if (seq != 0) {
        std::vector<int> sv(c->maxm, seq);
        PC_CU(cudaMemcpyAsync(c->d_seq_one, sv.data(), sv.size() * 4, cudaMemcpyHostToDevice, c->st));
        PC_CU(cudaStreamSynchronize(c->st));
        seq_rows = c->d_seq_one;
    }
    // with device sampling the blocks are the reference's 64 positions (each
    // draws); otherwise opts.prefill_chunk positions per step
    const int chunk = std::min(c->maxm, c->smp.on ? 64 : std::max(1, c->opts.prefill_chunk));
    std::vector<int> tok(chunk), ps(chunk);
    c->stages.clear();
    for (int off = 0; off < n; off += chunk) {
        const int m = std::min(chunk, n - off);
        for (int i = 0; i < m; ++i) { tok[i] = ids[off + i]; ps[i] = pos_base + off + i; }
        PC_CU(cudaMemcpyAsync(c->d_tok, tok.data(), (size_t)m * 4, cudaMemcpyHostToDevice, c->st));
        PC_CU(cudaMemcpyAsync(c->d_pos, ps.data(), (size_t)m * 4, cudaMemcpyHostToDevice, c->st));
        // with device sampling every block draws, as every forward_prefill
        // block of the reference does (picchio.c:1920-1926, 1970-1973)
        const bool lm = off + m >= n || c->smp.on;
        DenseJobs *dj = nullptr;
        PC_TRY(dense_jobs(c, m, lm ? 1 : 2, &dj));
        PC_TRY(run_step(c, m, seq_rows, lm ? 1 : 2, split_bucket(c, ps[m - 1]), dj));
        PC_CU(cudaStreamSynchronize(c->st));
        PC_TRY(res_after_step(c));
    }
    PC_CU(cudaMemcpy(c->h_next, c->d_next, 4, cudaMemcpyDeviceToHost));
    PC_CU(cudaMemcpy(c->h_err, c->err, 4, cudaMemcpyDeviceToHost));
    PC_TRY(check_err(c));
    *next_tok = c->h_next[0];
    return PC_OK;
}

pc_status pc_get_logits(pc_ctx *c, int row, float *logits, int n) {
    PC_TRY(check_ctx(c));
    if (!logits || row < 0 || row >= c->max_logit_rows || n > c->cfg.vocab) return fail(PC_ERR_INVALID_ARG, "bad logits request");
    PC_CU(cudaStreamSynchronize(c->st));
    PC_CU(cudaMemcpy(logits, c->logits + (size_t)row * c->cfg.vocab, (size_t)n * 4, cudaMemcpyDeviceToHost));
    return PC_OK;
}

pc_status pc_set_sampling(pc_ctx *c, const pc_sampling *s) {
    PC_TRY(check_ctx(c));
    if (!s) {
        c->smp.on = false;
        return PC_OK;
    }
    if (!(s->temperature >= 0.0f) || !(s->top_p == s->top_p) || !(s->rep_penalty == s->rep_penalty))
        return fail(PC_ERR_INVALID_ARG, "sampling settings must be numbers, temperature >= 0");
    const int V = c->cfg.vocab;
    PC_CU(sampler_init(c->smp, V));
    SampleParams p{};
    p.temperature = s->temperature;
    p.top_p = s->top_p;
    p.rep = s->rep_penalty;
    p.inv_temp = s->temperature < 1e-6f ? 1.0f : 1.0f / s->temperature;  // picchio.c:1564
    p.top_k = s->top_k;
    PC_CU(cudaMemcpyAsync(&c->smp.state->p, &p, sizeof p, cudaMemcpyHostToDevice, c->st));
    PC_CU(cudaStreamSynchronize(c->st));
    const bool top_p = s->top_p < 1.0f && s->top_p > 0.0f;
    const bool small_k = s->top_k > 0 && s->top_k < V && s->top_k <= SAMPLE_TOPK_SMALL;
    c->smp.big = top_p && !small_k;
    c->smp.on = true;
    return PC_OK;
}

pc_status pc_set_rng(pc_ctx *c, uint64_t state) {
    PC_TRY(check_ctx(c));
    PC_CU(sampler_init(c->smp, c->cfg.vocab));
    const unsigned long long v = state;
    PC_CU(cudaMemcpyAsync(&c->smp.state->rng, &v, sizeof v, cudaMemcpyHostToDevice, c->st));
    PC_CU(cudaStreamSynchronize(c->st));
    return PC_OK;
}

pc_status pc_get_rng(pc_ctx *c, uint64_t *state) {
    PC_TRY(check_ctx(c));
    if (!state) return fail(PC_ERR_INVALID_ARG, "null state");
    PC_CU(sampler_init(c->smp, c->cfg.vocab));
    unsigned long long v = 0;
    PC_CU(cudaStreamSynchronize(c->st));
    PC_CU(cudaMemcpy(&v, &c->smp.state->rng, sizeof v, cudaMemcpyDeviceToHost));
    *state = v;
    return PC_OK;
}

pc_status pc_history_reset(pc_ctx *c) {
    PC_TRY(check_ctx(c));
    PC_CU(sampler_init(c->smp, c->cfg.vocab));
    PC_CU(cudaMemsetAsync(&c->smp.state->hist_len, 0, sizeof(int), c->st));
    PC_CU(cudaStreamSynchronize(c->st));
    return PC_OK;
}

pc_status pc_history_push(pc_ctx *c, const int *ids, int n) {
    PC_TRY(check_ctx(c));
    if (n < 0 || (n > 0 && !ids)) return fail(PC_ERR_INVALID_ARG, "bad history ids");
    PC_CU(sampler_init(c->smp, c->cfg.vocab));
    PC_CU(cudaStreamSynchronize(c->st));
    int len = 0;
    PC_CU(cudaMemcpy(&len, &c->smp.state->hist_len, sizeof len, cudaMemcpyDeviceToHost));
    std::vector<int> keep;  // ids outside the vocabulary take no slot (picchio.c:1964-1966)
    for (int i = 0; i < n && len + (int)keep.size() < SAMPLE_HIST_CAP; ++i)
        if (ids[i] >= 0 && ids[i] < c->cfg.vocab) keep.push_back(ids[i]);
    if (keep.empty()) return PC_OK;
    PC_TRY(upload(c, c->smp.hist + len, keep.data(), keep.size() * sizeof(int)));
    len += (int)keep.size();
    PC_TRY(upload(c, &c->smp.state->hist_len, &len, sizeof len));
    return PC_OK;
}

pc_status pc_history_get(pc_ctx *c, int *ids, int cap, int *n) {
    PC_TRY(check_ctx(c));
    if (!n || cap < 0 || (cap > 0 && !ids)) return fail(PC_ERR_INVALID_ARG, "bad history request");
    PC_CU(sampler_init(c->smp, c->cfg.vocab));
    PC_CU(cudaStreamSynchronize(c->st));
    int len = 0;
    PC_CU(cudaMemcpy(&len, &c->smp.state->hist_len, sizeof len, cudaMemcpyDeviceToHost));
    *n = len;
    if (cap > 0 && len > 0) PC_CU(cudaMemcpy(ids, c->smp.hist, (size_t)std::min(cap, len) * sizeof(int), cudaMemcpyDeviceToHost));
    return PC_OK;
}

pc_status pc_sample(pc_ctx *c, const float *logits_dev, int *id) {
    PC_TRY(check_ctx(c));
    if (!logits_dev || !id) return fail(PC_ERR_INVALID_ARG, "null argument");
    if (!c->smp.on) return fail(PC_ERR_STATE, "no sampling settings (pc_set_sampling)");
    int launches = 0;
    PC_CU(sampler_launch(c->smp, logits_dev, c->d_next, nullptr, c->err, c->st, launches));
    c->launches += launches;
    PC_CU(cudaMemcpyAsync(c->h_next, c->d_next, 4, cudaMemcpyDeviceToHost, c->st));
    PC_CU(cudaMemcpyAsync(c->h_err, c->err, 4, cudaMemcpyDeviceToHost, c->st));
    PC_CU(cudaStreamSynchronize(c->st));
    PC_TRY(check_err(c));
    *id = c->h_next[0];
    return PC_OK;
}

// run_moe over M rows in chunks whose (row, k) pairs fit one router job table.
pc_status run_moe_rows(pc_ctx *c, int layer, const float *x, int M, const int *sel, const float *w, float *out) {
    const int K = c->cfg.topk, D = c->cfg.hidden;
    // chunks whose pairs fit one router launch: the expert-sorted lists of the
    // tensor-core path hold more than the GEMV's job table
    const bool tc = c->tex.on && (int64_t)M * K >= (int64_t)TE_MIN_PAIRS * c->cfg.n_experts;
    const int chunk = std::max(1, (tc ? ROUTER_MAX_PAIRS : GEMV_MAX_JOBS) / K);
    for (int off = 0; off < M;) {
        int m = std::min(chunk, M - off);
        if ((int64_t)m * K < (int64_t)TE_MIN_PAIRS * c->cfg.n_experts) m = std::min(m, std::max(1, GEMV_MAX_JOBS / K));
        PC_TRY(run_moe(c, layer, x + (size_t)off * D, m, sel ? sel + (size_t)off * K : nullptr,
                       w ? w + (size_t)off * K : nullptr, 0, out + (size_t)off * D, nullptr));
        off += m;
    }
    return PC_OK;
}

pc_status pc_moe_layer(pc_ctx *c, int layer, const float *x_dev, float *out_dev, int M) {
    PC_TRY(check_ctx(c));
    if (layer < 0 || layer >= c->cfg.n_layers || !x_dev || !out_dev) return fail(PC_ERR_INVALID_ARG, "bad moe_layer arguments");
    if (M < 1 || M > c->maxm) return fail(PC_ERR_RANGE, "M outside [1, " + std::to_string(c->maxm) + "]");
    PC_TRY(run_moe_rows(c, layer, x_dev, M, nullptr, nullptr, out_dev));
    PC_CU(cudaMemcpyAsync(c->h_err, c->err, 4, cudaMemcpyDeviceToHost, c->st));
    PC_CU(cudaStreamSynchronize(c->st));
    PC_TRY(check_err(c));
    return res_after_step(c);
}

pc_status pc_moe_experts(pc_ctx *c, int layer, const float *x_dev, const int *sel_dev, const float *w_dev, int M,
                         float *out_dev) {
    PC_TRY(check_ctx(c));
    if (layer < 0 || layer >= c->cfg.n_layers || !x_dev || !out_dev || !sel_dev || !w_dev)
        return fail(PC_ERR_INVALID_ARG, "bad moe_experts arguments");
    if (M < 1 || M > c->maxm) return fail(PC_ERR_RANGE, "M outside [1, " + std::to_string(c->maxm) + "]");
    PC_TRY(run_moe_rows(c, layer, x_dev, M, sel_dev, w_dev, out_dev));
    PC_CU(cudaMemcpyAsync(c->h_err, c->err, 4, cudaMemcpyDeviceToHost, c->st));
    PC_CU(cudaStreamSynchronize(c->st));
    PC_TRY(check_err(c));
    return res_after_step(c);
}

pc_status pc_get_routing(pc_ctx *c, int *expert_ids, int cap, int *rows) {
    PC_TRY(check_ctx(c));
    if (!rows || cap < 0 || (cap > 0 && !expert_ids)) return fail(PC_ERR_INVALID_ARG, "bad pc_get_routing arguments");
    const int L = c->cfg.n_layers, M = c->route_rows, K = c->cfg.topk;
    *rows = M;
    if ((int64_t)L * M * K > cap) return fail(PC_ERR_RANGE, "pc_get_routing needs n_layers * rows * topk ids");
    PC_CU(cudaStreamSynchronize(c->st));
    for (int l = 0; l < L && M > 0; ++l)
        PC_CU(cudaMemcpy(expert_ids + (size_t)l * M * K, layer_sel(c, l), (size_t)M * K * 4, cudaMemcpyDeviceToHost));
    return PC_OK;
}

pc_status pc_set_trace(pc_ctx *c, int on) {
    if (!c) return fail(PC_ERR_INVALID_ARG, "null context");
    c->trace = on != 0;
    return PC_OK;
}

pc_status pc_get_stage(pc_ctx *c, const char *name, float *out, int n) {
    if (!c || !name || !out) return fail(PC_ERR_INVALID_ARG, "null argument");
    auto it = c->stages.find(name);
    if (it == c->stages.end()) return fail(PC_ERR_STATE, std::string("no stage named ") + name);
    if (n != (int)it->second.size()) return fail(PC_ERR_INVALID_ARG, "stage size is " + std::to_string(it->second.size()));
    memcpy(out, it->second.data(), (size_t)n * 4);
    return PC_OK;
}

pc_status pc_dump(pc_ctx *c, const char *dir) {
    if (!c || !dir) return fail(PC_ERR_INVALID_ARG, "null argument");
    for (auto &kv : c->stages) {
        // same .npy header as oracle_dump (picchio.c:206-242): '<f4', shape (1, 1, n)
        std::string path = std::string(dir) + "/" + kv.first + ".npy";
        FILE *f = fopen(path.c_str(), "wb");
        if (!f) return fail(PC_ERR_IO, "cannot write " + path);
        char header[512];
        int hl = snprintf(header, sizeof header, "{'descr': '<f4', 'fortran_order': False, 'shape': (1, 1, %zu), }",
                          kv.second.size());
        int padded = hl + 1;
        while ((10 + padded) % 16) ++padded;
        memset(header + hl, ' ', (size_t)(padded - hl));
        header[padded - 1] = '\n';
        const unsigned char magic[8] = {0x93, 'N', 'U', 'M', 'P', 'Y', 1, 0};
        uint16_t hlen = (uint16_t)padded;
        fwrite(magic, 1, 8, f);
        fwrite(&hlen, 2, 1, f);
        fwrite(header, 1, (size_t)padded, f);
        fwrite(kv.second.data(), 4, kv.second.size(), f);
        fclose(f);
    }
    return PC_OK;
}

pc_status pc_expert_prefetch(pc_ctx *c, int layer, const int *eids, int n) {
    if (!c) return fail(PC_ERR_INVALID_ARG, "null context");
    if (layer < 0 || layer >= c->cfg.n_layers || n < 0 || (n > 0 && !eids))
        return fail(PC_ERR_INVALID_ARG, "bad pc_expert_prefetch arguments");
    PC_TRY(check_ctx(c));
    return res_prefetch(c, layer, eids, n);  // no-op when the whole table is in HBM
}

pc_status pc_expert_stats(pc_ctx *c, uint64_t *hits, uint64_t *misses, uint64_t *bytes_h2d) {
    if (!c) return fail(PC_ERR_INVALID_ARG, "null context");
    if (hits) *hits = c->res.hits;
    if (misses) *misses = c->res.misses;
    if (bytes_h2d) *bytes_h2d = c->res.bytes;
    return PC_OK;
}

pc_status pc_check_device(pc_ctx *c) {
    PC_TRY(check_ctx(c));
    PC_CU(cudaStreamSynchronize(c->st));
    PC_CU(cudaMemcpy(c->h_err, c->err, 4, cudaMemcpyDeviceToHost));
    return check_err(c);
}

uint64_t pc_kernel_launches(const pc_ctx *c) { return c ? c->launches : 0; }

int pc_tensor_core_min_rows(const pc_ctx *c) { return (c && c->tc.on) ? TC_MIN_ROWS : 0; }

pc_status pc_generate(pc_ctx *c, int tok, int pos, int n, int *out_ids, float *device_ms) {
    PC_TRY(check_ctx(c));
    if (!out_ids || n < 1) return fail(PC_ERR_INVALID_ARG, "bad pc_generate arguments");
    if (pos < 0 || pos + n > c->kv_ctx) return fail(PC_ERR_RANGE, "decode does not fit the KV capacity");
    c->stages.clear();
    return generate(c, tok, pos, n, out_ids, device_ms);
}

pc_status pc_kv_fill_synthetic(pc_ctx *c, int seq, int n_pos, uint64_t seed) {
    PC_TRY(check_ctx(c));
    if (seq < 0 || seq >= c->nseq || n_pos < 0 || n_pos > c->kv_ctx) return fail(PC_ERR_RANGE, "bad KV range");
    const int64_t n = (int64_t)n_pos * c->cfg.n_kv_heads * c->cfg.head_dim;
    for (int l = 0; l < c->cfg.n_layers; ++l) {
        for (int kv = 0; kv < 2; ++kv) {
            void *base = kv ? c->vc[l] : c->kc[l];
            const int64_t off = (int64_t)seq * c->seq_stride;
            PC_CU(gen_kv(base, off, n, c->opts.kv_bf16, seed ^ (0x1000ull * l + kv), c->st));
        }
    }
    PC_CU(cudaStreamSynchronize(c->st));
    return PC_OK;
}

pc_status pc_profile_begin(pc_ctx *c) {
    if (!c) return fail(PC_ERR_INVALID_ARG, "null context");
    for (auto &e : c->prof_evs) { cudaEventDestroy(e.a); cudaEventDestroy(e.b); }
    c->prof_evs.clear();
    c->prof_acc.clear();
    c->prof = true;
    return PC_OK;
}

pc_status pc_profile_end(pc_ctx *c) {
    PC_TRY(check_ctx(c));
    PC_CU(cudaStreamSynchronize(c->st));
    for (auto &e : c->prof_evs) {
        float ms = 0.0f;
        cudaEventElapsedTime(&ms, e.a, e.b);
        auto &acc = c->prof_acc[e.label];
        acc.first += ms;
        acc.second += 1;
        cudaEventDestroy(e.a);
        cudaEventDestroy(e.b);
    }
    c->prof_evs.clear();
    c->prof = false;
    return PC_OK;
}

pc_status pc_profile_get(pc_ctx *c, const char *label, double *total_ms, int *count) {
    if (!c || !label || !total_ms || !count) return fail(PC_ERR_INVALID_ARG, "null argument");
    auto it = c->prof_acc.find(label);
    *total_ms = it == c->prof_acc.end() ? 0.0 : it->second.first;
    *count = it == c->prof_acc.end() ? 0 : it->second.second;
    return PC_OK;
}

}  // extern "C"
