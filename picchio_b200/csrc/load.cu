// load.cu - from a model container (or a seed) to the device-resident model:
// dense weights as load_dense_weights does it (picchio.c:2531-2650), every
// expert as expert_load does it (picchio.c:698-888) but into one HBM table
// per layer instead of a disk-fed LRU, RoPE tables, KV cache, step buffers.
#include <cuda_bf16.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <vector>

#include "context.h"
#include "host_io.h"
#include "kernels.h"

namespace pc {

namespace {

int round_up(int v, int m) { return (v + m - 1) / m * m; }
int64_t align256(int64_t v) { return (v + 255) & ~int64_t(255); }

// load_f32_tensor (picchio.c:2385-2437): F32 as is, BF16 as the high half of
// an F32, F16 with subnormals flushed to zero.
bool read_as_f32(const StDB &db, const StTensor &t, std::vector<float> &out) {
    const int64_t n = t.numel();
    out.resize(n);
    if (t.dtype == ST_F32) return db.read(t, out.data(), n * 4);
    if (t.dtype == ST_BF16 || t.dtype == ST_F16) {
        std::vector<uint16_t> tmp(n);
        if (!db.read(t, tmp.data(), n * 2)) return false;
        for (int64_t i = 0; i < n; ++i) {
            uint32_t f;
            if (t.dtype == ST_BF16) {
                f = (uint32_t)tmp[i] << 16;
            } else {
                const uint16_t h = tmp[i];
                const uint32_t sign = (uint32_t)(h & 0x8000) << 16, ex = (h >> 10) & 0x1F, man = h & 0x3FF;
                if (ex == 0) f = sign;
                else if (ex == 31) f = sign | 0x7F800000u | (man << 13);
                else f = sign | ((ex + 112) << 23) | (man << 13);
            }
            memcpy(&out[i], &f, 4);
        }
        return true;
    }
    return false;
}

// quantize_rows_i4 (quant.h:364-392).
void quantize_rows_i4_host(const float *w, uint8_t *q4, float *scale, int O, int I) {
    const int rb = (I + 1) / 2;
    for (int o = 0; o < O; ++o) {
        const float *wr = w + (int64_t)o * I;
        float amax = 0;
        for (int i = 0; i < I; ++i) { const float a = fabsf(wr[i]); if (a > amax) amax = a; }
        float s = amax / 7.f;
        if (s < 1e-8f) s = 1e-8f;
        scale[o] = s;
        uint8_t *qr = q4 + (int64_t)o * rb;
        for (int i = 0; i < I; i += 2) {
            int v0 = (int)lrintf(wr[i] / s);
            v0 = v0 > 7 ? 7 : (v0 < -8 ? -8 : v0);
            int v1 = 0;
            if (i + 1 < I) {
                v1 = (int)lrintf(wr[i + 1] / s);
                v1 = v1 > 7 ? 7 : (v1 < -8 ? -8 : v1);
            }
            qr[i >> 1] = (uint8_t)((v0 + 8) | ((v1 + 8) << 4));
        }
    }
}

// Host layout INT4 / INT8 -> tiles on the device.
pc_status place_t4(pc_ctx *c, const uint8_t *q4, const float *scales, int64_t n_scales, int bs,
                   TileDesc &t) {
    const int O = t.O, I = t.I;
    const int64_t qbytes = (int64_t)O * ((I + 1) / 2);
    void *dq = nullptr, *ds = nullptr;
    PC_CU(cudaMalloc(&dq, qbytes));
    PC_CU(cudaMalloc(&ds, n_scales * 4));
    PC_CU(cudaMemcpyAsync(dq, q4, qbytes, cudaMemcpyHostToDevice, c->st));
    PC_CU(cudaMemcpyAsync(ds, scales, n_scales * 4, cudaMemcpyHostToDevice, c->st));
    PC_CU(retile_t4((const uint8_t *)dq, (const float *)ds, bs, t, c->st));
    PC_CU(cudaStreamSynchronize(c->st));
    cudaFree(dq);
    cudaFree(ds);
    return PC_OK;
}

pc_status place_t8(pc_ctx *c, const int8_t *q8, const float *scales, TileDesc &t) {
    const int64_t qbytes = (int64_t)t.O * t.I;
    void *dq = nullptr, *ds = nullptr;
    PC_CU(cudaMalloc(&dq, qbytes));
    PC_CU(cudaMalloc(&ds, (int64_t)t.O * 4));
    PC_CU(cudaMemcpyAsync(dq, q8, qbytes, cudaMemcpyHostToDevice, c->st));
    PC_CU(cudaMemcpyAsync(ds, scales, (int64_t)t.O * 4, cudaMemcpyHostToDevice, c->st));
    PC_CU(retile_t8((const int8_t *)dq, (const float *)ds, t, c->st));
    PC_CU(cudaStreamSynchronize(c->st));
    cudaFree(dq);
    cudaFree(ds);
    return PC_OK;
}

pc_status alloc_tiles(pc_ctx *c, TileDesc &t) {
    if (t.fmt == TF_F32) return dalloc(c, (size_t)t.O * t.I * 4, (void **)&t.f32);
    PC_TRY(dalloc(c, (size_t)tile_bytes(t), (void **)&t.tiles));
    if (t.fmt == TF_T8 || t.gs == 0) PC_TRY(dalloc(c, (size_t)t.Op * 4, (void **)&t.rs));
    return PC_OK;
}

// Block size rule of load_qt_i4 / expert_load (picchio.c:2461-2467, 780-785).
pc_status infer_block(const std::string &name, int64_t n_scale, int O, int I, int *bs) {
    if (n_scale > O) {
        int b = (int)((int64_t)O * I / n_scale);
        if (b <= 0) b = 64;
        *bs = b;
    } else {
        *bs = 0;
        if (n_scale != O) return fail(PC_ERR_FORMAT, name + ": " + std::to_string(n_scale) + " scales for " + std::to_string(O) + " rows");
    }
    if (*bs != 0 && *bs != 16 && *bs != 32 && *bs != 64)
        return fail(PC_ERR_FORMAT, name + ": INT4 group size " + std::to_string(*bs) + " not supported (16, 32, 64 or per-row)");
    return PC_OK;
}

// load_qt_i4 (picchio.c:2441-2527) for one dense projection / head.
pc_status load_dense(pc_ctx *c, const StDB &db, const std::string &name, int O, int I, int perm, int hd,
                     TileDesc &t) {
    const StTensor *st = db.find(name);
    if (!st) return fail(PC_ERR_MISSING_TENSOR, "tensor not found: " + name);
    if (st->dtype == ST_U8) {
        const int64_t rb = (I + 1) / 2;
        std::vector<uint8_t> q((size_t)(O * rb));
        if (!db.read(*st, q.data(), (int64_t)O * rb)) return fail(PC_ERR_IO, "short read: " + name);
        std::vector<float> s;
        int bs = 0;
        const StTensor *ts = db.find(name + ".qs");
        if (ts) {
            if (!read_as_f32(db, *ts, s)) return fail(PC_ERR_FORMAT, "bad scales: " + name + ".qs");
            PC_TRY(infer_block(name, (int64_t)s.size(), O, I, &bs));
        } else {
            s.assign(O, 1.0f);
        }
        tile_geom(t, TF_T4, O, I, bs, perm, hd);
        PC_TRY(alloc_tiles(c, t));
        return place_t4(c, q.data(), s.data(), (int64_t)s.size(), bs, t);
    }
    if (st->dtype == ST_I8) {
        std::vector<int8_t> q((size_t)O * I);
        if (!db.read(*st, q.data(), (int64_t)O * I)) return fail(PC_ERR_IO, "short read: " + name);
        const StTensor *ts = db.find(name + ".qs");
        if (!ts) return fail(PC_ERR_MISSING_TENSOR, "missing INT8 scales: " + name + ".qs");
        std::vector<float> s;
        if (!read_as_f32(db, *ts, s) || (int64_t)s.size() != O)
            return fail(PC_ERR_FORMAT, name + ".qs: expected " + std::to_string(O) + " scales");
        tile_geom(t, TF_T8, O, I, 0, perm, hd);
        PC_TRY(alloc_tiles(c, t));
        return place_t8(c, q.data(), s.data(), t);
    }
    std::vector<float> f;
    if (!read_as_f32(db, *st, f)) return fail(PC_ERR_FORMAT, name + ": unsupported dtype");
    if ((int64_t)f.size() < (int64_t)O * I) return fail(PC_ERR_FORMAT, name + ": too few elements");
    if (st->dtype == ST_F32) {  // kept F32 (picchio.c:2513-2517)
        tile_geom(t, TF_F32, O, I, 0, PERM_NONE, hd);
        PC_TRY(alloc_tiles(c, t));
        PC_TRY(upload(c, t.f32, f.data(), (size_t)O * I * 4));
        return PC_OK;
    }
    // BF16 / F16 -> per-row INT4 (picchio.c:2519-2526)
    std::vector<uint8_t> q((size_t)O * ((I + 1) / 2));
    std::vector<float> s(O);
    quantize_rows_i4_host(f.data(), q.data(), s.data(), O, I);
    tile_geom(t, TF_T4, O, I, 0, perm, hd);
    PC_TRY(alloc_tiles(c, t));
    return place_t4(c, q.data(), s.data(), O, 0, t);
}

pc_status load_vec(pc_ctx *c, const StDB &db, const std::string &name, int64_t n, float **dev, bool required,
                   float fill) {
    std::vector<float> v;
    const StTensor *st = db.find(name);
    if (st) {
        if (!read_as_f32(db, *st, v)) return fail(PC_ERR_FORMAT, name + ": unsupported dtype");
        if ((int64_t)v.size() < n) return fail(PC_ERR_FORMAT, name + ": too few elements");
    } else {
        if (required) return fail(PC_ERR_MISSING_TENSOR, "tensor not found: " + name);
        if (std::isnan(fill)) { *dev = nullptr; return PC_OK; }
        v.assign(n, fill);
    }
    PC_TRY(dalloc(c, (size_t)n * 4, (void **)dev));
    PC_TRY(upload(c, *dev, v.data(), (size_t)n * 4));
    return PC_OK;
}

// load_expert_bias (picchio.c:634-696): per-expert F32, aggregated [E, n]
// F32, or the legacy aggregated INT4 + .qs form (gs 64).
pc_status expert_bias(const StDB &db, int layer, int eid, const char *suffix, int E, int n,
                      std::vector<float> &out, bool *present) {
    char nm[300];
    snprintf(nm, sizeof nm, "model.layers.%d.mlp.experts.%d.%s", layer, eid, suffix);
    const StTensor *t = db.find(nm);
    bool aggregated = false;
    if (!t) {
        snprintf(nm, sizeof nm, "model.layers.%d.mlp.experts.%s", layer, suffix);
        t = db.find(nm);
        aggregated = t != nullptr;
    }
    *present = false;
    out.assign(n, 0.0f);
    if (!t) return PC_OK;
    const StTensor *ts = db.find(std::string(nm) + ".qs");
    const bool full_f32 = t->dtype == ST_F32 && t->numel() == (int64_t)E * n;
    if (aggregated && ts && !full_f32) {
        const int packed_n = (n + 1) / 2, groups = (n + 63) / 64;
        std::vector<uint8_t> packed(packed_n);
        std::vector<float> sc(groups);
        if (t->dtype == ST_F32) {
            std::vector<float> stored(packed_n);
            if (!db.read(*t, stored.data(), (int64_t)packed_n * 4, (int64_t)eid * packed_n * 4)) return fail(PC_ERR_IO, nm);
            for (int i = 0; i < packed_n; ++i) packed[i] = (uint8_t)lrintf(stored[i]);
        } else if (t->dtype == ST_U8) {
            if (!db.read(*t, packed.data(), packed_n, (int64_t)eid * packed_n)) return fail(PC_ERR_IO, nm);
        } else {
            return PC_OK;
        }
        if (!db.read(*ts, sc.data(), (int64_t)groups * 4, (int64_t)eid * groups * 4)) return fail(PC_ERR_IO, nm);
        for (int i = 0; i < n; ++i) {
            const uint8_t b = packed[i >> 1];
            const int q = (i & 1) ? (int)(b >> 4) - 8 : (int)(b & 0x0F) - 8;
            out[i] = q * sc[i / 64];
        }
        *present = true;
        return PC_OK;
    }
    if (t->dtype != ST_F32) return PC_OK;
    const int64_t off = aggregated ? (int64_t)eid * n * 4 : 0;
    if (!db.read(*t, out.data(), (int64_t)n * 4, off)) return fail(PC_ERR_IO, std::string("short read: ") + nm);
    *present = true;
    return PC_OK;
}

struct ExpertMat {
    std::vector<uint8_t> q;
    std::vector<float> s;
    int bs = 0;
    int fmt = TF_T4;  // TF_T4 (INT4) or TF_F4 (MXFP4)
};

// Expert e of the checkpoint's own MXFP4 form (the layout convert.py:400-431
// reads before requantizing): `<which>_blocks` U8 [E][O][I/32][16] (two E2M1
// codes per byte, low nibble = even column) and `<which>_scales` U8
// [E][O][I/32] (E8M0: factor 2^(e - 127)).  Kept as MXFP4 (the reference's
// fmt 3) instead of converted to INT4.
pc_status expert_matrix_mxfp4(const StDB &db, int layer, int eid, const char *which, int O, int I, ExpertMat &m,
                              bool *found) {
    char bn[300], sn[300];
    snprintf(bn, sizeof bn, "model.layers.%d.mlp.experts.%s_blocks", layer, which);
    snprintf(sn, sizeof sn, "model.layers.%d.mlp.experts.%s_scales", layer, which);
    const StTensor *tb = db.find(bn), *ts = db.find(sn);
    *found = tb && ts;
    if (!*found) return PC_OK;
    if (tb->dtype != ST_U8 || ts->dtype != ST_U8) return fail(PC_ERR_FORMAT, std::string(bn) + ": MXFP4 blocks and scales must be U8");
    if (I % 32) return fail(PC_ERR_FORMAT, std::string(bn) + ": MXFP4 rows must be a multiple of 32 columns");
    const int64_t rb = I / 2, nb = I / 32;
    if (tb->nbytes() < (int64_t)(eid + 1) * O * rb || ts->nbytes() < (int64_t)(eid + 1) * O * nb)
        return fail(PC_ERR_FORMAT, std::string(bn) + ": fewer experts or smaller rows than the config");
    m.q.resize((size_t)(O * rb));
    if (!db.read(*tb, m.q.data(), (int64_t)O * rb, (int64_t)eid * O * rb)) return fail(PC_ERR_IO, std::string("short read: ") + bn);
    std::vector<uint8_t> e8((size_t)(O * nb));
    if (!db.read(*ts, e8.data(), (int64_t)O * nb, (int64_t)eid * O * nb)) return fail(PC_ERR_IO, std::string("short read: ") + sn);
    m.s.resize(e8.size());
    for (size_t i = 0; i < e8.size(); ++i) m.s[i] = ldexpf(1.0f, (int)e8[i] - 127);  // decode_e8m0, convert.py:129-134
    m.bs = 32;
    m.fmt = TF_F4;
    return PC_OK;
}

// The weight half of expert_load (picchio.c:712-866) for one matrix.
pc_status expert_matrix(const StDB &db, int layer, int eid, const char *which, int O, int I, ExpertMat &m) {
    bool mx = false;
    PC_TRY(expert_matrix_mxfp4(db, layer, eid, which, O, I, m, &mx));
    if (mx) return PC_OK;
    char nm[300];
    const char *fmts[3] = {"model.layers.%d.mlp.experts.%s.%d", "model.layers.%d.mlp.experts.%d.%s",
                           "model.layers.%d.mlp.experts.%d.%s.weight"};
    const StTensor *t = nullptr;
    snprintf(nm, sizeof nm, fmts[0], layer, which, eid);
    t = db.find(nm);
    if (!t) { snprintf(nm, sizeof nm, "model.layers.%d.mlp.experts.%d.%s", layer, eid, which); t = db.find(nm); }
    if (!t) { snprintf(nm, sizeof nm, "model.layers.%d.mlp.experts.%d.%s.weight", layer, eid, which); t = db.find(nm); }
    if (!t) return fail(PC_ERR_MISSING_TENSOR, std::string("expert tensor not found: layer ") + std::to_string(layer) + " expert " + std::to_string(eid) + " " + which);
    if (t->dtype != ST_U8)
        return fail(PC_ERR_FORMAT, std::string(nm) + ": expert weights must be packed INT4 (U8); F32/BF16 experts are not supported on the device path");
    const int64_t rb = (I + 1) / 2;
    m.q.resize((size_t)(O * rb));
    if (!db.read(*t, m.q.data(), (int64_t)O * rb)) return fail(PC_ERR_IO, std::string("short read: ") + nm);
    char sn[340];
    snprintf(sn, sizeof sn, "model.layers.%d.mlp.experts.%s.%d.qs", layer, which, eid);
    const StTensor *ts = db.find(sn);
    if (!ts) { snprintf(sn, sizeof sn, "model.layers.%d.mlp.experts.%d.%s.qs", layer, eid, which); ts = db.find(sn); }
    if (ts) {
        if (!read_as_f32(db, *ts, m.s)) return fail(PC_ERR_FORMAT, std::string("bad scales: ") + sn);
        return infer_block(nm, (int64_t)m.s.size(), O, I, &m.bs);
    }
    m.s.assign(O, 1.0f);
    m.bs = 0;
    (void)fmts;
    return PC_OK;
}

pc_status expert_geometry(pc_ctx *c, int gs_gu, int gs_dn, int fmt) {
    const pc_model_cfg &k = c->cfg;
    ExpertGeom &g = c->eg;
    tile_geom(g.gu, fmt, 2 * k.intermediate, k.hidden, gs_gu, PERM_PAIR, 0);
    tile_geom(g.dn, fmt, k.hidden, k.intermediate, gs_dn, PERM_NONE, 0);
    int64_t off = 0;
    g.off_gu = off; off = align256(off + tile_bytes(g.gu));
    g.off_dn = off; off = align256(off + tile_bytes(g.dn));
    g.off_gu_rs = -1; g.off_dn_rs = -1;
    if (gs_gu == 0) { g.off_gu_rs = off; off = align256(off + (int64_t)g.gu.Op * 4); }
    if (gs_dn == 0) { g.off_dn_rs = off; off = align256(off + (int64_t)g.dn.Op * 4); }
    g.off_gu_b = off; off = align256(off + (int64_t)2 * k.intermediate * 4);
    g.off_dn_b = off; off = align256(off + (int64_t)k.hidden * 4);
    g.stride = off;
    return PC_OK;
}

// Where one expert's matrices live inside the table.
void expert_views(const pc_ctx *c, uint8_t *base, TileDesc &gu, TileDesc &dn) {
    gu = c->eg.gu;
    dn = c->eg.dn;
    gu.tiles = base + c->eg.off_gu;
    dn.tiles = base + c->eg.off_dn;
    gu.rs = c->eg.off_gu_rs >= 0 ? reinterpret_cast<float *>(base + c->eg.off_gu_rs) : nullptr;
    dn.rs = c->eg.off_dn_rs >= 0 ? reinterpret_cast<float *>(base + c->eg.off_dn_rs) : nullptr;
}

pc_status check_shapes(const pc_model_cfg &k) {
    if (k.hidden <= 0 || k.n_heads <= 0 || k.n_kv_heads <= 0 || k.head_dim <= 0 || k.n_experts <= 0 ||
        k.topk <= 0 || k.intermediate <= 0 || k.vocab <= 0)
        return fail(PC_ERR_FORMAT, "config: non-positive dimension");
    if (k.n_heads % k.n_kv_heads) return fail(PC_ERR_FORMAT, "config: heads not a multiple of kv heads");
    if (k.head_dim != 16 && k.head_dim != 32 && k.head_dim != 64)
        return fail(PC_ERR_FORMAT, "config: head_dim must be 16, 32 or 64");
    if (k.n_heads / k.n_kv_heads > 8) return fail(PC_ERR_FORMAT, "config: more than 8 query heads per kv head");
    if (k.n_experts > 256 || k.topk > 16 || k.topk > k.n_experts) return fail(PC_ERR_FORMAT, "config: experts <= 256, top-k <= 16");
    if (k.intermediate % 8) return fail(PC_ERR_FORMAT, "config: intermediate_size must be a multiple of 8");
    return PC_OK;
}

uint64_t seed_of(uint64_t seed, uint64_t a, uint64_t b = 0, uint64_t cc = 0) {
    uint64_t z = seed ^ (a * 0x9E3779B97F4A7C15ull) ^ (b * 0xC2B2AE3D27D4EB4Full) ^ (cc * 0x165667B19E3779F9ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

pc_status rope_tables(pc_ctx *c) {
    // yarn_inv_freq + rope_apply angle/cos/sin (picchio.c:431-466), on the host
    // with the reference's float expressions.
    const pc_model_cfg &k = c->cfg;
    const int dim = k.head_dim, half = dim / 2;
    std::vector<float> inv(half);
    const float attn_factor = k.rope_factor > 1.0f ? 0.1f * logf(k.rope_factor) + 1.0f : 1.0f;
    for (int j = 0; j < half; ++j) {
        const float pos_freq = powf(k.theta, 2.0f * j / dim);
        const float extrap = 1.0f / pos_freq;
        if (k.rope_factor <= 1.0f) { inv[j] = extrap; continue; }
        float low = dim * logf(k.rope_original_ctx / (k.rope_beta_fast * 2.0f * (float)M_PI)) / (2.0f * logf(k.theta));
        float high = dim * logf(k.rope_original_ctx / (k.rope_beta_slow * 2.0f * (float)M_PI)) / (2.0f * logf(k.theta));
        if (k.rope_truncate) { low = floorf(low); high = ceilf(high); }
        if (low < 0) low = 0;
        if (high > dim - 1) high = (float)(dim - 1);
        if (low == high) high += 0.001f;
        float ramp = (j - low) / (high - low);
        if (ramp < 0) ramp = 0;
        if (ramp > 1) ramp = 1;
        const float ef = 1.0f - ramp;
        const float interp = extrap / k.rope_factor;
        inv[j] = interp * (1.0f - ef) + extrap * ef;
    }
    c->rope_len = c->kv_ctx;
    std::vector<float> cs((size_t)c->rope_len * half), sn((size_t)c->rope_len * half);
    for (int p = 0; p < c->rope_len; ++p)
        for (int j = 0; j < half; ++j) {
            const float ang = p * inv[j];
            cs[(size_t)p * half + j] = cosf(ang) * attn_factor;
            sn[(size_t)p * half + j] = sinf(ang) * attn_factor;
        }
    PC_TRY(dalloc(c, cs.size() * 4, (void **)&c->rope_cs));
    PC_TRY(dalloc(c, sn.size() * 4, (void **)&c->rope_sn));
    PC_TRY(upload(c, c->rope_cs, cs.data(), cs.size() * 4));
    PC_TRY(upload(c, c->rope_sn, sn.data(), sn.size() * 4));
    return PC_OK;
}

}  // namespace

void tile_geom(TileDesc &t, int fmt, int O, int I, int gs, int perm, int hd) {
    t = TileDesc{};
    t.fmt = fmt;
    t.O = O;
    t.I = I;
    t.gs = fmt == TF_T4 ? gs : fmt == TF_F4 ? 32 : 0;
    t.perm = perm;
    t.head_dim = hd;
    t.Op = round_up(O, 16);
    if (tf_4bit(fmt)) {
        t.Ip = round_up(I, 64);
        t.kblocks = t.Ip / 64;
        t.blk_bytes = t4_blk_bytes(t.gs);
    } else if (fmt == TF_T8) {
        t.Ip = round_up(I, 32);
        t.kblocks = t.Ip / 32;
        t.blk_bytes = 512;
    } else {
        t.Ip = I;
    }
    t.unit_bytes = (int64_t)t.kblocks * t.blk_bytes;
}

int64_t tile_bytes(const TileDesc &t) { return (int64_t)(t.Op / 16) * t.unit_bytes; }

pc_status alloc_runtime(pc_ctx *c) {
    const pc_model_cfg &k = c->cfg;
    const int D = k.hidden, H = k.n_heads, KVH = k.n_kv_heads, hd = k.head_dim, K = k.topk;
    c->nseq = c->opts.max_batch > 0 ? c->opts.max_batch : 1;
    c->kv_ctx = c->opts.ctx_len > 0 ? c->opts.ctx_len : 512;
    if (c->kv_ctx > k.ctx_len) c->kv_ctx = k.ctx_len;  // picchio.c:2935
    c->maxm = std::max({c->nseq, 64, c->opts.prefill_chunk});
    if ((int64_t)c->maxm * k.topk > ROUTER_MAX_PAIRS)
        return fail(PC_ERR_RANGE, "max_batch / prefill_chunk above " + std::to_string(ROUTER_MAX_PAIRS / k.topk) +
                                      " rows (" + std::to_string(ROUTER_MAX_PAIRS) + " routed pairs per step)");
    const int M = c->maxm;
    PC_TRY(rope_tables(c));
    const int kvd = KVH * hd;
    c->seq_stride = (int64_t)c->kv_ctx * kvd;
    const size_t esz = c->opts.kv_bf16 ? 2 : 4;
    c->kc.resize(k.n_layers);
    c->vc.resize(k.n_layers);
    for (int l = 0; l < k.n_layers; ++l) {
        PC_TRY(dalloc(c, (size_t)c->nseq * c->seq_stride * esz, &c->kc[l]));
        PC_TRY(dalloc(c, (size_t)c->nseq * c->seq_stride * esz, &c->vc[l]));
    }
    PC_TRY(dalloc(c, M * 4, (void **)&c->d_tok));
    PC_TRY(dalloc(c, M * 4, (void **)&c->d_pos));
    PC_TRY(dalloc(c, (M + 1) * 4, (void **)&c->d_next));
    c->err = c->d_next + M;
    PC_TRY(dalloc(c, M * 4, (void **)&c->d_seq_rows));
    PC_TRY(dalloc(c, M * 4, (void **)&c->d_seq_zero));
    PC_TRY(dalloc(c, M * 4, (void **)&c->d_seq_one));
    std::vector<int> rows(M);
    for (int i = 0; i < M; ++i) rows[i] = i < c->nseq ? i : 0;
    PC_TRY(upload(c, c->d_seq_rows, rows.data(), M * 4));
    PC_TRY(dalloc(c, (size_t)M * D * 4, (void **)&c->h));
    PC_TRY(dalloc(c, (size_t)M * D * 4, (void **)&c->hn));
    PC_TRY(dalloc(c, (size_t)M * D * 4, (void **)&c->tmp));
    PC_TRY(dalloc(c, (size_t)M * H * hd * 4, (void **)&c->qbuf));
    PC_TRY(dalloc(c, (size_t)M * H * hd * 4, (void **)&c->attn));
    PC_TRY(dalloc(c, (size_t)M * (H * hd + 2 * kvd) * 4, (void **)&c->raw));
    PC_TRY(dalloc(c, (size_t)M * K * k.intermediate * 4, (void **)&c->act));
    PC_TRY(dalloc(c, (size_t)M * K * D * 4, (void **)&c->eo));
    PC_TRY(dalloc(c, (size_t)M * D * 4, (void **)&c->moe_out));
    c->max_logit_rows = c->nseq;
    PC_TRY(dalloc(c, (size_t)c->max_logit_rows * k.vocab * 4, (void **)&c->logits));
    PC_TRY(dalloc(c, (size_t)M * k.n_experts * 4, (void **)&c->rlogits));
    PC_TRY(dalloc(c, (size_t)std::max(1, k.n_layers) * M * K * 4, (void **)&c->sel));  // [layer][row][k]
    PC_TRY(dalloc(c, (size_t)M * K * 4, (void **)&c->rw));
    PC_TRY(dalloc(c, (size_t)M * K * 4, (void **)&c->pair_local));
    PC_TRY(dalloc(c, 16, (void **)&c->njobs));
    PC_TRY(dalloc(c, sizeof(GemvJob) * GEMV_MAX_JOBS, (void **)&c->jobs_gu));
    PC_TRY(dalloc(c, sizeof(GemvJob) * GEMV_MAX_JOBS, (void **)&c->jobs_dn));
    // router tickets: [0] the whole launch, [1 + b] row block b of the row-block form
    PC_TRY(dalloc(c, (size_t)(M + 4) * 4, (void **)&c->router_ctr));
    PC_CU(cudaMemset(c->router_ctr, 0, (size_t)(M + 4) * 4));
    PC_TRY(dalloc(c, (size_t)M * KVH * 4, (void **)&c->attn_ctr));
    c->attn_max_split = (c->kv_ctx + 255) / 256;
    if (c->attn_max_split > 64)  // the decode attention merges at most 64 spans of 256 positions
        return fail(PC_ERR_RANGE, "ctx_len above 16384 positions is not supported");
    PC_TRY(dalloc(c, (size_t)M * H * c->attn_max_split * (hd + 2) * 4, (void **)&c->attn_part));
    PC_TRY(dalloc(c, (size_t)M * 8, (void **)&c->argmax));
    c->gen_cap = c->kv_ctx;
    PC_TRY(dalloc(c, (size_t)c->gen_cap * 4, (void **)&c->d_gen));
    PC_TRY(dalloc(c, 16, (void **)&c->d_step));
    PC_CU(cudaMallocHost(&c->pinned, 4096));
    c->h_tok = (int *)c->pinned;
    c->h_pos = c->h_tok + 256;
    c->h_next = c->h_pos + 256;
    c->h_err = c->h_next + 256;
    return PC_OK;
}

pc_status load_model(pc_ctx *c, const std::string &dir) {
    std::string err;
    if (!load_config(dir, &c->cfg, &err)) return fail(PC_ERR_IO, err);
    pc_model_cfg &k = c->cfg;
    PC_TRY(check_shapes(k));
    StDB db;
    if (!open_model_dir(db, dir, &err)) return fail(PC_ERR_IO, err);
    const int D = k.hidden, H = k.n_heads, KVH = k.n_kv_heads, hd = k.head_dim, E = k.n_experts;
    const int I2 = 2 * k.intermediate;

    // embedding: kept in the host row layout for the row gather
    {
        const std::string nm = "model.embed_tokens.weight";
        const StTensor *t = db.find(nm);
        if (!t) return fail(PC_ERR_MISSING_TENSOR, "tensor not found: " + nm);
        if (t->dtype == ST_I8) {
            std::vector<int8_t> q((size_t)k.vocab * D);
            if (!db.read(*t, q.data(), (int64_t)k.vocab * D)) return fail(PC_ERR_IO, "short read: " + nm);
            const StTensor *ts = db.find(nm + ".qs");
            std::vector<float> s;
            if (!ts || !read_as_f32(db, *ts, s) || (int64_t)s.size() != k.vocab)
                return fail(PC_ERR_MISSING_TENSOR, "missing INT8 scales: " + nm + ".qs");
            c->emb_fmt = TF_T8;
            PC_TRY(dalloc(c, q.size(), &c->emb));
            PC_TRY(dalloc(c, s.size() * 4, (void **)&c->emb_s));
            PC_TRY(upload(c, c->emb, q.data(), q.size()));
            PC_TRY(upload(c, c->emb_s, s.data(), s.size() * 4));
        } else if (t->dtype == ST_U8) {
            const int64_t rb = (D + 1) / 2;
            std::vector<uint8_t> q((size_t)(k.vocab * rb));
            if (!db.read(*t, q.data(), (int64_t)k.vocab * rb)) return fail(PC_ERR_IO, "short read: " + nm);
            std::vector<float> s;
            const StTensor *ts = db.find(nm + ".qs");
            int bs = 0;
            if (ts) {
                if (!read_as_f32(db, *ts, s)) return fail(PC_ERR_FORMAT, nm + ".qs");
                if ((int64_t)s.size() > k.vocab) {
                    bs = (int)((int64_t)k.vocab * D / (int64_t)s.size());
                    if (bs <= 0) bs = 64;
                }
            } else {
                s.assign(k.vocab, 1.0f);
            }
            c->emb_fmt = TF_T4;
            c->emb_gs = bs;
            PC_TRY(dalloc(c, q.size(), &c->emb));
            PC_TRY(dalloc(c, s.size() * 4, (void **)&c->emb_s));
            PC_TRY(upload(c, c->emb, q.data(), q.size()));
            PC_TRY(upload(c, c->emb_s, s.data(), s.size() * 4));
        } else {
            std::vector<float> f;
            if (!read_as_f32(db, *t, f)) return fail(PC_ERR_FORMAT, nm + ": unsupported dtype");
            if (t->dtype == ST_F32) {
                c->emb_fmt = TF_F32;
                PC_TRY(dalloc(c, f.size() * 4, &c->emb));
                PC_TRY(upload(c, c->emb, f.data(), f.size() * 4));
            } else {
                std::vector<uint8_t> q((size_t)k.vocab * ((D + 1) / 2));
                std::vector<float> s(k.vocab);
                quantize_rows_i4_host(f.data(), q.data(), s.data(), k.vocab, D);
                c->emb_fmt = TF_T4;
                c->emb_gs = 0;
                PC_TRY(dalloc(c, q.size(), &c->emb));
                PC_TRY(dalloc(c, s.size() * 4, (void **)&c->emb_s));
                PC_TRY(upload(c, c->emb, q.data(), q.size()));
                PC_TRY(upload(c, c->emb_s, s.data(), s.size() * 4));
            }
        }
    }
    PC_TRY(load_dense(c, db, "lm_head.weight", k.vocab, D, PERM_NONE, 0, c->lm_head.t));
    PC_TRY(load_vec(c, db, "model.norm.weight", D, &c->final_norm, false, 1.0f));

    c->L.resize(k.n_layers);
    char nm[300];
    for (int l = 0; l < k.n_layers; ++l) {
        Layer &ly = c->L[l];
        ly.layer_type = k.layer_type[l];
        auto P = [&](const char *s) { snprintf(nm, sizeof nm, "model.layers.%d.%s", l, s); return std::string(nm); };
        PC_TRY(load_vec(c, db, P("input_layernorm.weight"), D, &ly.in_ln, false, 1.0f));
        PC_TRY(load_vec(c, db, P("post_attention_layernorm.weight"), D, &ly.post_ln, false, 1.0f));
        PC_TRY(load_dense(c, db, P("self_attn.q_proj.weight"), H * hd, D, PERM_HEAD, hd, ly.wq.t));
        PC_TRY(load_dense(c, db, P("self_attn.k_proj.weight"), KVH * hd, D, PERM_HEAD, hd, ly.wk.t));
        PC_TRY(load_dense(c, db, P("self_attn.v_proj.weight"), KVH * hd, D, PERM_HEAD, hd, ly.wv.t));
        PC_TRY(load_dense(c, db, P("self_attn.o_proj.weight"), D, H * hd, PERM_NONE, 0, ly.wo.t));
        const float NONE = NAN;
        PC_TRY(load_vec(c, db, P("self_attn.q_proj.bias"), H * hd, &ly.wq.bias, false, NONE));
        PC_TRY(load_vec(c, db, P("self_attn.k_proj.bias"), KVH * hd, &ly.wk.bias, false, NONE));
        PC_TRY(load_vec(c, db, P("self_attn.v_proj.bias"), KVH * hd, &ly.wv.bias, false, NONE));
        PC_TRY(load_vec(c, db, P("self_attn.o_proj.bias"), D, &ly.wo.bias, false, NONE));
        PC_TRY(load_vec(c, db, P("self_attn.sinks"), H, &ly.sinks, true, NONE));  // picchio.c:2621-2626
        if (db.find(P("mlp.router.weight")))
            PC_TRY(load_vec(c, db, P("mlp.router.weight"), (int64_t)E * D, &ly.router, true, NONE));
        else
            PC_TRY(load_vec(c, db, P("block_sparse_moe.gate.weight"), (int64_t)E * D, &ly.router, true, NONE));
        PC_TRY(load_vec(c, db, P("mlp.router.bias"), E, &ly.router_bias, false, NONE));
    }

    // experts: one HBM table per layer
    std::vector<uint8_t> stage;
    void *dtmp = nullptr;
    bool geom = false;
    for (int l = 0; l < k.n_layers; ++l) {
        for (int e = c->e_lo; e < c->e_hi; ++e) {
            ExpertMat gu, dn;
            PC_TRY(expert_matrix(db, l, e, "gate_up_proj", I2, D, gu));
            PC_TRY(expert_matrix(db, l, e, "down_proj", D, k.intermediate, dn));
            if (gu.fmt != dn.fmt) return fail(PC_ERR_FORMAT, "gate_up and down experts in different formats");
            if (!geom) {
                PC_TRY(expert_geometry(c, gu.bs, dn.bs, gu.fmt));
                k.expert_format = gu.fmt == TF_F4 ? PC_FMT_MXFP4 : PC_FMT_INT4;
                if (c->opts.expert_residency == 1) PC_TRY(res_init(c));
                geom = true;
                const int64_t raw = (int64_t)I2 * ((D + 1) / 2) + (int64_t)gu.s.size() * 4 +
                                    (int64_t)D * ((k.intermediate + 1) / 2) + (int64_t)dn.s.size() * 4 + 1024;
                PC_CU(cudaMalloc(&dtmp, raw));
            }
            if (gu.bs != c->eg.gu.gs || dn.bs != c->eg.dn.gs || gu.fmt != c->eg.gu.fmt)
                return fail(PC_ERR_FORMAT, "experts with different formats or group sizes in one model");
            if (!c->L[l].experts)
                PC_TRY(dalloc(c, (size_t)(c->e_hi - c->e_lo) * c->eg.stride, (void **)&c->L[l].experts));
            // streamed residency: assembled in a staging expert, then stored on the host
            uint8_t *base = c->res.on ? c->res.stage : c->L[l].experts + (int64_t)(e - c->e_lo) * c->eg.stride;
            TileDesc tg, td;
            expert_views(c, base, tg, td);
            uint8_t *d = (uint8_t *)dtmp;
            const int64_t a = (int64_t)gu.q.size(), b = (int64_t)gu.s.size() * 4, cc = (int64_t)dn.q.size();
            PC_TRY(upload(c, d, gu.q.data(), a));
            PC_TRY(upload(c, d + align256(a), gu.s.data(), b));
            PC_CU(retile_t4(d, (const float *)(d + align256(a)), gu.bs, tg, c->st));
            PC_CU(cudaStreamSynchronize(c->st));
            PC_TRY(upload(c, d, dn.q.data(), cc));
            PC_TRY(upload(c, d + align256(cc), dn.s.data(), dn.s.size() * 4));
            PC_CU(retile_t4(d, (const float *)(d + align256(cc)), dn.bs, td, c->st));
            PC_CU(cudaStreamSynchronize(c->st));
            std::vector<float> bgu, bdn;
            bool has;
            PC_TRY(expert_bias(db, l, e, "gate_up_proj_bias", E, I2, bgu, &has));
            PC_TRY(expert_bias(db, l, e, "down_proj_bias", E, D, bdn, &has));
            PC_TRY(upload(c, base + c->eg.off_gu_b, bgu.data(), bgu.size() * 4));
            PC_TRY(upload(c, base + c->eg.off_dn_b, bdn.data(), bdn.size() * 4));
            if (c->res.on) PC_TRY(res_store(c, l, e));
        }
    }
    if (c->res.on) PC_TRY(res_finish_load(c));
    if (dtmp) cudaFree(dtmp);
    (void)stage;
    return alloc_runtime(c);
}

pc_status synth_model(pc_ctx *c, uint64_t seed) {
    pc_model_cfg &k = c->cfg;
    PC_TRY(check_shapes(k));
    const int D = k.hidden, H = k.n_heads, KVH = k.n_kv_heads, hd = k.head_dim, E = k.n_experts;
    const int I2 = 2 * k.intermediate, V = k.vocab;
    cudaStream_t st = c->st;
    // scratch for the row-major matrix being generated and its scales: the
    // largest of every matrix generated below (embedding / lm_head, q and o
    // projections, expert gate_up and down), scales for gs >= 8
    const int64_t big = std::max({(int64_t)V * D, (int64_t)I2 * D, (int64_t)H * hd * D,
                                  (int64_t)D * k.intermediate});
    const int64_t max_rows = std::max({(int64_t)V, (int64_t)I2, (int64_t)H * hd, (int64_t)D});
    const int64_t max_cols = std::max({(int64_t)D, (int64_t)H * hd, (int64_t)k.intermediate});
    const int64_t soff = align256(big);
    int64_t tmpb = soff + max_rows * (max_cols / 8 + 2) * 4 + 4096;
    uint8_t *tmp = nullptr;
    PC_CU(cudaMalloc(&tmp, tmpb));
    float *tmps = reinterpret_cast<float *>(tmp + soff);
    uint64_t tag = 0;
    auto dense = [&](int O, int I, int perm, int hdim, TileDesc &t, int fmt, int gs) -> pc_status {
        ++tag;
        if (fmt == PC_FMT_F32) {
            tile_geom(t, TF_F32, O, I, 0, PERM_NONE, hdim);
            PC_TRY(alloc_tiles(c, t));
            PC_CU(gen_f32(t.f32, (int64_t)O * I, seed_of(seed, tag), 0.0f, 0.02f, st));
            return PC_OK;
        }
        if (fmt == PC_FMT_INT8) {
            tile_geom(t, TF_T8, O, I, 0, perm, hdim);
            PC_TRY(alloc_tiles(c, t));
            PC_CU(gen_i8_rowmajor((int8_t *)tmp, tmps, O, I, seed_of(seed, tag), 0.02f, st));
            PC_CU(retile_t8((const int8_t *)tmp, tmps, t, st));
        } else {
            tile_geom(t, TF_T4, O, I, gs, perm, hdim);
            PC_TRY(alloc_tiles(c, t));
            PC_CU(gen_i4_rowmajor(tmp, tmps, O, I, gs, seed_of(seed, tag), 0.02f, st));
            PC_CU(retile_t4(tmp, tmps, gs, t, st));
        }
        PC_CU(cudaStreamSynchronize(st));
        return PC_OK;
    };
    auto vec = [&](int64_t n, float mean, float sd, float **dst) -> pc_status {
        ++tag;
        PC_TRY(dalloc(c, (size_t)n * 4, (void **)dst));
        PC_CU(gen_f32(*dst, n, seed_of(seed, tag), mean, sd, st));
        return PC_OK;
    };
    // embedding (INT8 rows) and head
    ++tag;
    PC_TRY(dalloc(c, (size_t)V * D, &c->emb));
    PC_TRY(dalloc(c, (size_t)V * 4, (void **)&c->emb_s));
    PC_CU(gen_i8_rowmajor((int8_t *)c->emb, c->emb_s, V, D, seed_of(seed, tag), 0.02f, st));
    c->emb_fmt = TF_T8;
    PC_TRY(dense(V, D, PERM_NONE, 0, c->lm_head.t, PC_FMT_INT8, 0));
    PC_TRY(vec(D, 1.0f, 0.05f, &c->final_norm));
    c->L.resize(k.n_layers);
    for (int l = 0; l < k.n_layers; ++l) {
        Layer &ly = c->L[l];
        ly.layer_type = k.layer_type[l];
        PC_TRY(vec(D, 1.0f, 0.05f, &ly.in_ln));
        PC_TRY(vec(D, 1.0f, 0.05f, &ly.post_ln));
        PC_TRY(dense(H * hd, D, PERM_HEAD, hd, ly.wq.t, k.attn_format, k.attn_group_size));
        PC_TRY(dense(KVH * hd, D, PERM_HEAD, hd, ly.wk.t, k.attn_format, k.attn_group_size));
        PC_TRY(dense(KVH * hd, D, PERM_HEAD, hd, ly.wv.t, k.attn_format, k.attn_group_size));
        PC_TRY(dense(D, H * hd, PERM_NONE, 0, ly.wo.t, k.attn_format, k.attn_group_size));
        PC_TRY(vec(H * hd, 0.0f, 0.01f, &ly.wq.bias));
        PC_TRY(vec(KVH * hd, 0.0f, 0.01f, &ly.wk.bias));
        PC_TRY(vec(KVH * hd, 0.0f, 0.01f, &ly.wv.bias));
        PC_TRY(vec(D, 0.0f, 0.01f, &ly.wo.bias));
        PC_TRY(vec(H, 0.0f, 0.5f, &ly.sinks));
        PC_TRY(vec((int64_t)E * D, 0.0f, 0.1f, &ly.router));
        PC_TRY(vec(E, 0.0f, 0.01f, &ly.router_bias));
    }
    const bool f4 = k.expert_format == PC_FMT_MXFP4;
    if (f4) k.group_size = 32;
    PC_TRY(expert_geometry(c, k.group_size, k.group_size, f4 ? TF_F4 : TF_T4));
    if (c->opts.expert_residency == 1) PC_TRY(res_init(c));
    for (int l = 0; l < k.n_layers; ++l) {
        if (!c->res.on) PC_TRY(dalloc(c, (size_t)(c->e_hi - c->e_lo) * c->eg.stride, (void **)&c->L[l].experts));
        for (int e = c->e_lo; e < c->e_hi; ++e) {
            uint8_t *base = c->res.on ? c->res.stage : c->L[l].experts + (int64_t)(e - c->e_lo) * c->eg.stride;
            TileDesc tg, td;
            expert_views(c, base, tg, td);
            if (f4) PC_CU(gen_f4_rowmajor(tmp, tmps, I2, D, seed_of(seed, 1000 + l, e, 1), 0.02f, st));
            else PC_CU(gen_i4_rowmajor(tmp, tmps, I2, D, k.group_size, seed_of(seed, 1000 + l, e, 1), 0.02f, st));
            PC_CU(retile_t4(tmp, tmps, k.group_size, tg, st));
            if (f4) PC_CU(gen_f4_rowmajor(tmp, tmps, D, k.intermediate, seed_of(seed, 1000 + l, e, 2), 0.02f, st));
            else PC_CU(gen_i4_rowmajor(tmp, tmps, D, k.intermediate, k.group_size, seed_of(seed, 1000 + l, e, 2), 0.02f, st));
            PC_CU(retile_t4(tmp, tmps, k.group_size, td, st));
            PC_CU(gen_f32(reinterpret_cast<float *>(base + c->eg.off_gu_b), I2, seed_of(seed, 1000 + l, e, 3), 0.0f, 0.01f, st));
            PC_CU(gen_f32(reinterpret_cast<float *>(base + c->eg.off_dn_b), D, seed_of(seed, 1000 + l, e, 4), 0.0f, 0.01f, st));
            if (c->res.on) PC_TRY(res_store(c, l, e));
        }
        PC_CU(cudaStreamSynchronize(st));
    }
    if (c->res.on) PC_TRY(res_finish_load(c));
    cudaFree(tmp);
    return alloc_runtime(c);
}

}  // namespace pc
