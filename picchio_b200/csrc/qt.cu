// qt.cu - the weight-level operator of the C ABI: one QT matrix uploaded
// from the reference's host layout (quant.h:32-41) and applied with the
// streaming GEMV, matmul_qt (quant.h:323-337).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "context.h"
#include "gemv.h"
#include "kernels.h"
#include "launch.cuh"

struct pc_qt {
    int dev = 0, nsm = 148, max_smem = 0;
    pc::TileDesc t;
    std::vector<void *> allocs;
    std::map<int, std::pair<pc::GemvJob *, int *>> jobs;  // per row count S
    int *err = nullptr;
};

namespace {

using namespace pc;

pc_status qalloc(pc_qt *w, size_t bytes, void **out) {
    cudaError_t e = cudaMalloc(out, bytes ? bytes : 16);
    if (e != cudaSuccess) return fail(PC_ERR_OOM, std::string("cudaMalloc: ") + cudaGetErrorString(e));
    w->allocs.push_back(*out);
    return cudaMemset(*out, 0, bytes ? bytes : 16) == cudaSuccess ? PC_OK : fail(PC_ERR_CUDA, "cudaMemset");
}

// Device job table for S input rows, `per` rows per job (cached per pair).
pc_status jobs_for(pc_qt *w, int S, int per, std::pair<GemvJob *, int *> &out) {
    const int key = S * 16 + per;
    auto it = w->jobs.find(key);
    if (it != w->jobs.end()) { out = it->second; return PC_OK; }
    std::vector<GemvJob> jobs;
    for (int r0 = 0; r0 < S; r0 += per) {
        GemvJob j;
        memset(&j, 0, sizeof j);
        j.tiles = w->t.tiles;
        j.rs = w->t.rs;
        j.n_rt = w->t.Op / 16;
        j.O = w->t.O;
        j.nrows = std::min(per, S - r0);
        for (int i = 0; i < j.nrows; ++i) j.in_row[i] = j.out_row[i] = r0 + i;
        jobs.push_back(j);
    }
    GemvJob *dj = nullptr;
    int *dc = nullptr;
    PC_TRY(qalloc(w, jobs.size() * sizeof(GemvJob), (void **)&dj));
    PC_TRY(qalloc(w, 4, (void **)&dc));
    const int n = (int)jobs.size();
    PC_CU(cudaMemcpy(dj, jobs.data(), jobs.size() * sizeof(GemvJob), cudaMemcpyHostToDevice));
    PC_CU(cudaMemcpy(dc, &n, 4, cudaMemcpyHostToDevice));
    // a pageable copy can still be in flight on the legacy stream when
    // cudaMemcpy returns; the caller's stream need not wait for that stream
    PC_CU(cudaDeviceSynchronize());
    out = {dj, dc};
    w->jobs[key] = out;
    return PC_OK;
}

}  // namespace

// ---- pc_qt_matmul_noalloc: the same product, for callers that cannot allocate
//
// Scratch lives in one file-scope device array per device: the GEMV job
// table (up to PC_QT_NOALLOC_MAX_ROWS input rows = 8 jobs of 8 rows) and its
// job count.  Its address is taken once per device with cudaGetSymbolAddress;
// every call rewrites the job count and table with a one-warp kernel before
// the GEMV reads them, so nothing in it has to start at zero.  Nothing is
// allocated, so two calls that overlap (different streams or threads) race on
// it.  The GEMV's only device-side failure is a bounded wait for a weight
// copy giving up; it records that in an error word kept in the same scratch
// (sticky until pc_qt_check reads and clears it).  Launch failures come back
// from the launch itself.

namespace {

constexpr int NOALLOC_MAX_JOBS = PC_QT_NOALLOC_MAX_ROWS / GEMV_MAXR;

struct NoallocScratch {
    GemvJob jobs[NOALLOC_MAX_JOBS];
    int njobs;
    int err;  // nonzero: a GEMV wait gave up (cleared by pc_qt_check)
};

__device__ __align__(256) unsigned char g_noalloc_scratch[sizeof(NoallocScratch)];

constexpr int NOALLOC_MAX_DEVICES = 64;
std::mutex g_noalloc_mu;
NoallocScratch *g_noalloc_ptr[NOALLOC_MAX_DEVICES] = {};

// Once per device (the current one): the device address of the scratch
// array.  The host-side name g_noalloc_scratch is not a device address.
pc_status noalloc_scratch(int dev, NoallocScratch **out) {
    if (dev < 0 || dev >= NOALLOC_MAX_DEVICES) return fail(PC_ERR_INVALID_ARG, "device ordinal out of range");
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        void *p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(noalloc scratch)");
        g_noalloc_ptr[dev] = static_cast<NoallocScratch *>(p);
    }
    *out = g_noalloc_ptr[dev];
    return PC_OK;
}

// One thread per job: the job table pc_qt_matmul builds on the host, rows
// 8j..8j+7 of x into the same rows of y.
__global__ void noalloc_jobs_kernel(NoallocScratch *s, const uint8_t *tiles, const float *rs, int n_rt, int O,
                                    int S) {
    const int nj = (S + GEMV_MAXR - 1) / GEMV_MAXR, j = threadIdx.x;
    if (j == 0) s->njobs = nj;
    if (j >= nj) return;
    GemvJob g;
    memset(&g, 0, sizeof g);
    g.tiles = tiles;
    g.rs = rs;
    g.n_rt = n_rt;
    g.O = O;
    g.nrows = min(GEMV_MAXR, S - j * GEMV_MAXR);
    for (int i = 0; i < g.nrows; ++i) g.in_row[i] = g.out_row[i] = j * GEMV_MAXR + i;
    s->jobs[j] = g;
}

}  // namespace

extern "C" {

pc_status pc_qt_create(int device, int fmt, int O, int I, int block_size, const void *data, const float *scales,
                       pc_qt **out) {
    if (!out || !data || O <= 0 || I <= 0) return fail(PC_ERR_INVALID_ARG, "bad pc_qt_create arguments");
    if (fmt != PC_FMT_F32 && !scales) return fail(PC_ERR_INVALID_ARG, "quantized weights need scales");
    if (fmt == PC_FMT_INT4 && block_size != 0 && block_size != 16 && block_size != 32 && block_size != 64)
        return fail(PC_ERR_FORMAT, "INT4 block size must be 0, 16, 32 or 64");
    if (fmt == PC_FMT_MXFP4 && block_size != 32) return fail(PC_ERR_FORMAT, "MXFP4 blocks are 32 columns");
    pc_qt *w = new pc_qt();
    w->dev = device;
    pc_status s = device_setup(device, &w->nsm, &w->max_smem);
    if (s != PC_OK) { delete w; return s; }
    auto done = [&](pc_status st) { if (st != PC_OK) pc_qt_free(w); else *out = w; return st; };
    s = qalloc(w, 4, (void **)&w->err);
    if (s != PC_OK) return done(s);
    if (fmt == PC_FMT_F32) {
        tile_geom(w->t, TF_F32, O, I, 0, PERM_NONE, 0);
        if ((s = qalloc(w, (size_t)O * I * 4, (void **)&w->t.f32)) != PC_OK) return done(s);
        if (cudaMemcpy(w->t.f32, data, (size_t)O * I * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
            cudaDeviceSynchronize() != cudaSuccess)
            return done(fail(PC_ERR_CUDA, "upload"));
        return done(PC_OK);
    }
    // INT4 and MXFP4 share the host layout: two 4-bit values per byte, low
    // nibble = even column; MXFP4 scales are one float per 32 columns
    const bool i4 = fmt == PC_FMT_INT4 || fmt == PC_FMT_MXFP4;
    if (!i4 && fmt != PC_FMT_INT8) return done(fail(PC_ERR_FORMAT, "unknown format"));
    tile_geom(w->t, fmt == PC_FMT_MXFP4 ? TF_F4 : i4 ? TF_T4 : TF_T8, O, I, i4 ? block_size : 0, PERM_NONE, 0);
    if ((s = qalloc(w, (size_t)tile_bytes(w->t), (void **)&w->t.tiles)) != PC_OK) return done(s);
    if (!i4 || block_size == 0)
        if ((s = qalloc(w, (size_t)w->t.Op * 4, (void **)&w->t.rs)) != PC_OK) return done(s);
    const int64_t qbytes = i4 ? (int64_t)O * ((I + 1) / 2) : (int64_t)O * I;
    const int64_t ns = (i4 && block_size) ? (int64_t)O * ((I + block_size - 1) / block_size) : O;
    void *dq = nullptr, *ds = nullptr;
    if (cudaMalloc(&dq, qbytes) != cudaSuccess || cudaMalloc(&ds, ns * 4) != cudaSuccess)
        return done(fail(PC_ERR_OOM, "staging"));
    cudaMemcpy(dq, data, qbytes, cudaMemcpyHostToDevice);
    cudaMemcpy(ds, scales, ns * 4, cudaMemcpyHostToDevice);
    cudaError_t e = i4 ? retile_t4((const uint8_t *)dq, (const float *)ds, block_size, w->t, 0)
                       : retile_t8((const int8_t *)dq, (const float *)ds, w->t, 0);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    cudaFree(dq);
    cudaFree(ds);
    if (e != cudaSuccess) return done(cuda_fail(e, "retile"));
    return done(PC_OK);
}

pc_status pc_qt_matmul(pc_qt *w, const float *x_dev, float *y_dev, int S, void *stream) {
    if (!w || !x_dev || !y_dev || S < 1) return fail(PC_ERR_INVALID_ARG, "bad pc_qt_matmul arguments");
    PC_CU(cudaSetDevice(w->dev));
    cudaStream_t st = (cudaStream_t)stream;
    if (w->t.fmt == TF_F32) {
        F32GemvParams f{};
        f.W = w->t.f32; f.O = w->t.O; f.I = w->t.I; f.x = x_dev; f.ldx = w->t.I; f.M = S;
        f.y = y_dev; f.ldy = w->t.O;
        PC_CU(launch_gemv_f32(f, st));
        return PC_OK;
    }
    // The B operand of all rows (up to 8, four N-tiles) and the weight rings
    // must fit in one CTA's shared memory; a long input row that does not fit
    // with the N-tiles its row count needs runs as jobs of two rows on one
    // N-tile (the weights are then streamed once per job).
    int nt = gemv_nt_for_rows(std::min(S, GEMV_MAXR));
    int per = GEMV_MAXR;
    if (nt > 1 && gemv_smem_bytes(w->t.fmt, nt, w->t.Ip, w->t.blk_bytes) > (size_t)w->max_smem) {
        nt = 1;
        per = 2;
    }
    std::pair<GemvJob *, int *> j;
    PC_TRY(jobs_for(w, S, per, j));
    GemvParams p{};
    p.jobs = j.first;
    p.njobs = j.second;
    p.fmt = w->t.fmt;
    p.gs = w->t.gs;
    p.kblocks = w->t.kblocks;
    p.blk_bytes = w->t.blk_bytes;
    p.I = w->t.I;
    p.Ip = w->t.Ip;
    p.perm = PERM_NONE;
    p.epi = EPI_STORE;
    p.static_jobs = 1;
    if (S <= per) {  // one job, carried in the launch; all rows in the B operand
        GemvJob jb;
        memset(&jb, 0, sizeof jb);
        jb.tiles = w->t.tiles;
        jb.rs = w->t.rs;
        jb.n_rt = w->t.Op / 16;
        jb.O = w->t.O;
        jb.nrows = S;
        for (int i = 0; i < S; ++i) jb.in_row[i] = jb.out_row[i] = i;
        p.n_inline = 1;
        p.ijobs[0] = jb;
        p.shared_rows = S;
    }
    p.x = x_dev;
    p.ldx = w->t.I;
    p.y = y_dev;
    p.ldy = w->t.O;
    p.err = w->err;
    if (!gemv_plan(p, nt, w->max_smem)) return fail(PC_ERR_FORMAT, "input rows do not fit in shared memory");
    PC_CU(gemv_launch(p, nt, w->nsm, st));
    return PC_OK;
}

pc_status pc_qt_matmul_noalloc(pc_qt *w, const float *x_dev, float *y_dev, int S, void *stream) {
    if (!w || !x_dev || !y_dev || S < 1) return fail(PC_ERR_INVALID_ARG, "bad pc_qt_matmul_noalloc arguments");
    if (S > PC_QT_NOALLOC_MAX_ROWS)
        return fail(PC_ERR_RANGE, "pc_qt_matmul_noalloc takes at most " + std::to_string(PC_QT_NOALLOC_MAX_ROWS) +
                                      " input rows");
    PC_CU(cudaSetDevice(w->dev));
    cudaStream_t st = (cudaStream_t)stream;
    if (w->t.fmt == TF_F32) {  // the fp32 kernel uses no scratch
        F32GemvParams f{};
        f.W = w->t.f32; f.O = w->t.O; f.I = w->t.I; f.x = x_dev; f.ldx = w->t.I; f.M = S;
        f.y = y_dev; f.ldy = w->t.O;
        PC_CU(launch_gemv_f32(f, st));
        return PC_OK;
    }
    NoallocScratch *s = nullptr;
    PC_TRY(noalloc_scratch(w->dev, &s));
    noalloc_jobs_kernel<<<1, 32, 0, st>>>(s, w->t.tiles, w->t.rs, w->t.Op / 16, w->t.O, S);
    PC_CU(cudaGetLastError());
    GemvParams p{};
    p.jobs = s->jobs;
    p.njobs = &s->njobs;
    p.static_jobs = 0;  // the table is written by the kernel just launched
    p.fmt = w->t.fmt;
    p.gs = w->t.gs;
    p.kblocks = w->t.kblocks;
    p.blk_bytes = w->t.blk_bytes;
    p.I = w->t.I;
    p.Ip = w->t.Ip;
    p.perm = PERM_NONE;
    p.epi = EPI_STORE;
    p.x = x_dev;
    p.ldx = w->t.I;
    p.y = y_dev;
    p.ldy = w->t.O;
    p.err = &s->err;
    const int nt = gemv_nt_for_rows(std::min(S, GEMV_MAXR));
    if (!gemv_plan(p, nt, w->max_smem)) return fail(PC_ERR_FORMAT, "input rows do not fit in shared memory");
    PC_CU(gemv_launch(p, nt, w->nsm, st));
    return PC_OK;
}

pc_status pc_qt_check(pc_qt *w, void *stream) {
    if (!w) return fail(PC_ERR_INVALID_ARG, "null weight");
    PC_CU(cudaSetDevice(w->dev));
    PC_CU(cudaStreamSynchronize((cudaStream_t)stream));
    int e1 = 0, e2 = 0;
    const int zero = 0;
    PC_CU(cudaMemcpy(&e1, w->err, 4, cudaMemcpyDeviceToHost));
    if (e1) PC_CU(cudaMemcpy(w->err, &zero, 4, cudaMemcpyHostToDevice));  // completed below
    NoallocScratch *sc = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_noalloc_mu);
        if (w->dev >= 0 && w->dev < NOALLOC_MAX_DEVICES) sc = g_noalloc_ptr[w->dev];
    }
    if (sc) {
        PC_CU(cudaMemcpy(&e2, &sc->err, 4, cudaMemcpyDeviceToHost));
        if (e2) PC_CU(cudaMemcpy(&sc->err, &zero, 4, cudaMemcpyHostToDevice));
    }
    if (e1 || e2) {
        PC_CU(cudaDeviceSynchronize());  // the clearing copies have landed before any later product
        return fail(PC_ERR_TIMEOUT, "a GEMV wait for its weight copies gave up");
    }
    return PC_OK;
}

pc_status pc_qt_dequant(pc_qt *w, float *out_dev, void *stream) {
    if (!w || !out_dev) return fail(PC_ERR_INVALID_ARG, "bad pc_qt_dequant arguments");
    PC_CU(cudaSetDevice(w->dev));
    if (w->t.fmt == TF_F32) {
        PC_CU(cudaMemcpyAsync(out_dev, w->t.f32, (size_t)w->t.O * w->t.I * 4, cudaMemcpyDeviceToDevice,
                              (cudaStream_t)stream));
        return PC_OK;
    }
    PC_CU(dequant_tiles(w->t, out_dev, (cudaStream_t)stream));
    return PC_OK;
}

void pc_qt_free(pc_qt *w) {
    if (!w) return;
    cudaSetDevice(w->dev);
    cudaDeviceSynchronize();
    for (void *p : w->allocs) cudaFree(p);
    delete w;
}

}  // extern "C"
