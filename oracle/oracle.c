/* oracle.c - CPU restatement of picchio's per-token MoE hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in picchio_b200/ links, loads or calls
 * this file; only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
 * leg use it, and only as the checker.
 *
 * Every function restates one piece of the reference (benmaster82/picchio)
 * and names the file:line it follows.  The arithmetic is written to reproduce
 * the reference's fp32 results bit for bit as the reference is built
 * (gcc -O3 with AVX2+FMA): where the reference sums 8 AVX2 lanes and folds
 * them with hsum256, the lane structure and the fold order are restated in
 * plain C.  Which multiply-adds the reference's build fuses is not uniform
 * (explicit _mm256_fmadd_ps, the scalar tails and the loops gcc vectorizes
 * fuse; the per-group `a += ga * sc`, the attention score dot and the router
 * dot do not); each statement below writes out the fused form (fmaf) or the
 * unfused one as the compiled reference does it.  This file is compiled with -ffp-contract=off so that only
 * the explicit fmaf() calls fuse.  The tests pin these bit-exact claims
 * against the reference compiled from its own sources (oracle/_ref/).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define OR_API __attribute__((visibility("default")))

/* hsum256 (quant.h:86-95): ((l0+l4)+(l2+l6)) + ((l1+l5)+(l3+l7)). */
static float hsum8(const float l[8]) {
    float s0 = l[0] + l[4], s1 = l[1] + l[5], s2 = l[2] + l[6], s3 = l[3] + l[7];
    return (s0 + s2) + (s1 + s3);
}

static inline float nib(const uint8_t *w, int i) {
    uint8_t b = w[i >> 1];
    return (float)((int)((i & 1) ? (b >> 4) : (b & 0xF)) - 8);
}

/* matmul_f32, quant.h:117-148 (AVX2 branch + scalar tail). */
OR_API void or_matmul_f32(float *y, const float *x, const float *W, int S, int I, int O) {
    for (int o = 0; o < O; o++) {
        const float *w = W + (int64_t)o * I;
        for (int s = 0; s < S; s++) {
            const float *xs = x + (int64_t)s * I;
            float l[8] = {0};
            int i = 0;
            for (; i + 8 <= I; i += 8)
                for (int j = 0; j < 8; j++) l[j] = fmaf(xs[i + j], w[i + j], l[j]);
            float a = hsum8(l);
            for (; i < I; i++) a = fmaf(xs[i], w[i], a);
            y[(int64_t)s * O + o] = a;
        }
    }
}

/* matmul_q8, quant.h:152-186. */
OR_API void or_matmul_q8(float *y, const float *x, const int8_t *q, const float *scale,
                         int S, int I, int O) {
    for (int o = 0; o < O; o++) {
        const int8_t *w = q + (int64_t)o * I;
        float sc = scale[o];
        for (int s = 0; s < S; s++) {
            const float *xs = x + (int64_t)s * I;
            float l[8] = {0};
            int i = 0;
            for (; i + 8 <= I; i += 8)
                for (int j = 0; j < 8; j++) l[j] = fmaf(xs[i + j], (float)w[i + j], l[j]);
            float a = hsum8(l);
            for (; i < I; i++) a = fmaf(xs[i], (float)w[i], a);
            y[(int64_t)s * O + o] = a * sc;
        }
    }
}

/* matmul_i4 (per-row scale), quant.h:191-253. */
OR_API void or_matmul_i4(float *y, const float *x, const uint8_t *q4, const float *scale,
                         int S, int I, int O) {
    int rb = (I + 1) / 2;
    for (int o = 0; o < O; o++) {
        const uint8_t *w = q4 + (int64_t)o * rb;
        float sc = scale[o];
        for (int s = 0; s < S; s++) {
            const float *xs = x + (int64_t)s * I;
            float l[8] = {0};
            int i = 0;
            for (; i + 16 <= I; i += 16) {
                for (int j = 0; j < 8; j++) l[j] = fmaf(xs[i + j], nib(w, i + j), l[j]);
                for (int j = 0; j < 8; j++) l[j] = fmaf(xs[i + 8 + j], nib(w, i + 8 + j), l[j]);
            }
            float a = hsum8(l);
            for (; i + 1 < I; i += 2)
                a = a + fmaf(xs[i], nib(w, i), xs[i + 1] * nib(w, i + 1));
            if (i < I) a = fmaf(xs[i], nib(w, i), a);
            y[(int64_t)s * O + o] = a * sc;
        }
    }
}

/* matmul_i4_gs (group-scaled), quant.h:259-319 (AVX2 branch). */
OR_API void or_matmul_i4_gs(float *y, const float *x, const uint8_t *q4, const float *scale,
                            int S, int I, int O, int gs) {
    int rb = (I + 1) / 2;
    int ng = (I + gs - 1) / gs;
    for (int o = 0; o < O; o++) {
        const uint8_t *w = q4 + (int64_t)o * rb;
        const float *sc = scale + (int64_t)o * ng;
        for (int s = 0; s < S; s++) {
            const float *xs = x + (int64_t)s * I;
            float a = 0;
            for (int g = 0; g < ng; g++) {
                int g0 = g * gs, g1 = g0 + gs;
                if (g1 > I) g1 = I;
                float l[8] = {0};
                int gi = g0;
                for (; gi + 16 <= g1; gi += 16) {
                    for (int j = 0; j < 8; j++) l[j] = fmaf(xs[gi + j], nib(w, gi + j), l[j]);
                    for (int j = 0; j < 8; j++) l[j] = fmaf(xs[gi + 8 + j], nib(w, gi + 8 + j), l[j]);
                }
                float ga = hsum8(l);
                for (; gi < g1; gi += 2) {
                    ga = fmaf(xs[gi], nib(w, gi), ga);
                    if (gi + 1 < g1) ga = fmaf(xs[gi + 1], nib(w, gi + 1), ga);
                }
                a = a + ga * sc[g];
            }
            y[(int64_t)s * O + o] = a;
        }
    }
}

/* Dequantization as the reference defines it for one weight:
 * value = (float)((int)nibble - 8) * scale, one fp32 multiply
 * (quant.h:201-204 nibble convention; picchio.c:680-682 dequant form). */
OR_API void or_dequant_i4(float *out, const uint8_t *q4, const float *scale,
                          int O, int I, int gs) {
    int rb = (I + 1) / 2;
    int ng = gs > 0 ? (I + gs - 1) / gs : 1;
    for (int o = 0; o < O; o++)
        for (int i = 0; i < I; i++) {
            float s = gs > 0 ? scale[(int64_t)o * ng + i / gs] : scale[o];
            out[(int64_t)o * I + i] = nib(q4 + (int64_t)o * rb, i) * s;
        }
}

/* INT8 per-row dequant, as embed_token does it (picchio.c:1488-1491). */
OR_API void or_dequant_i8(float *out, const int8_t *q, const float *scale, int O, int I) {
    for (int o = 0; o < O; o++)
        for (int i = 0; i < I; i++)
            out[(int64_t)o * I + i] = (float)q[(int64_t)o * I + i] * scale[o];
}

/* quantize_rows_i4, quant.h:364-392 (per-row INT4 quantizer). */
OR_API void or_quantize_rows_i4(const float *w, uint8_t *q4, float *scale, int O, int I) {
    int rb = (I + 1) / 2;
    for (int o = 0; o < O; o++) {
        const float *wr = w + (int64_t)o * I;
        float amax = 0;
        for (int i = 0; i < I; i++) { float a = fabsf(wr[i]); if (a > amax) amax = a; }
        float s = amax / 7.f;
        if (s < 1e-8f) s = 1e-8f;
        scale[o] = s;
        uint8_t *qr = q4 + (int64_t)o * rb;
        for (int i = 0; i < I; i += 2) {
            int v0 = (int)lrintf(wr[i] / s);
            if (v0 > 7) v0 = 7;
            if (v0 < -8) v0 = -8;
            int v1 = 0;
            if (i + 1 < I) {
                v1 = (int)lrintf(wr[i + 1] / s);
                if (v1 > 7) v1 = 7;
                if (v1 < -8) v1 = -8;
            }
            qr[i >> 1] = (uint8_t)((v0 + 8) | ((v1 + 8) << 4));
        }
    }
}

/* rmsnorm, quant.h:396-402: double sum of squares, fp32 rescale. */
OR_API void or_rmsnorm(float *out, const float *x, const float *w, int D, float eps) {
    double ms = 0;
    for (int i = 0; i < D; i++) ms += (double)x[i] * x[i];
    float r = 1.f / sqrtf((float)(ms / D) + eps);
    for (int i = 0; i < D; i++) out[i] = x[i] * r * w[i];
}

/* softmax, quant.h:406-412. */
OR_API void or_softmax(float *x, int n) {
    float m = -1e30f;
    for (int i = 0; i < n; i++) if (x[i] > m) m = x[i];
    float s = 0;
    for (int i = 0; i < n; i++) { x[i] = expf(x[i] - m); s += x[i]; }
    for (int i = 0; i < n; i++) x[i] /= s;
}

/* Router logits + top-k + softmax weights.
 * Decode (picchio.c:1316-1355): dot accumulated from 0, bias added last.
 * Prefill (picchio.c:1837-1855): dot starts at the bias.
 * Top-k: K rounds of strict-'>' argmax over unselected experts, so ties go to
 * the lowest index; the weights are softmax over the K raw logits. */
OR_API void or_router_topk(const float *x, const float *R, const float *bias, int E, int D,
                           int K, int bias_first, float *logits, int *sel, float *wts) {
    for (int e = 0; e < E; e++) {
        const float *rw = R + (int64_t)e * D;
        float dot = (bias_first && bias) ? bias[e] : 0.0f;
        for (int i = 0; i < D; i++) dot = dot + x[i] * rw[i];
        if (!bias_first && bias) dot += bias[e];
        logits[e] = dot;
    }
    for (int k = 0; k < K; k++) {
        int best = -1;
        float bs = -1e30f;
        for (int e = 0; e < E; e++) {
            int already = 0;
            for (int j = 0; j < k; j++) if (sel[j] == e) { already = 1; break; }
            if (!already && logits[e] > bs) { bs = logits[e]; best = e; }
        }
        sel[k] = best;
        wts[k] = bs;
    }
    or_softmax(wts, K);
}

static inline float sigm(float v) { return 1.f / (1.f + expf(-v)); }   /* quant.h:417 */

/* Clamped SwiGLU over interleaved (gate, up) pairs, picchio.c:1416-1424.
 * act[i] = (clamp(up,+-lim)+1) * min(gate,lim) * sigmoid(alpha*min(gate,lim)). */
OR_API void or_swiglu(float *act, const float *gu, int I2, float limit, float alpha) {
    for (int i = 0; i < I2 / 2; i++) {
        float gate = gu[2 * i], up = gu[2 * i + 1];
        if (gate > limit) gate = limit;
        if (up > limit) up = limit;
        if (up < -limit) up = -limit;
        act[i] = (up + 1.0f) * gate * sigm(alpha * gate);
    }
}

/* yarn_inv_freq, picchio.c:431-453. */
OR_API float or_yarn_inv_freq(int head_dim, float theta, float factor, float beta_fast,
                              float beta_slow, int orig_ctx, int truncate, int j) {
    int dim = head_dim;
    float pos_freq = powf(theta, 2.0f * j / dim);
    float extrap = 1.0f / pos_freq;
    if (factor <= 1.0f) return extrap;
    float low = dim * logf(orig_ctx / (beta_fast * 2.0f * (float)M_PI)) / (2.0f * logf(theta));
    float high = dim * logf(orig_ctx / (beta_slow * 2.0f * (float)M_PI)) / (2.0f * logf(theta));
    if (truncate) { low = floorf(low); high = ceilf(high); }
    if (low < 0) low = 0;
    if (high > dim - 1) high = (float)(dim - 1);
    if (low == high) high += 0.001f;
    float ramp = (j - low) / (high - low);
    if (ramp < 0) ramp = 0;
    if (ramp > 1) ramp = 1;
    float ef = 1.0f - ramp;
    float interp = extrap / factor;
    return interp * (1.0f - ef) + extrap * ef;
}

/* cos/sin table for one position, as rope_apply forms them (picchio.c:462-466):
 * ang = pos * inv_freq[j] (fp32), cos/sin scaled by the YaRN attention factor. */
OR_API void or_rope_cs(const float *inv_freq, int half, int pos, float attn_factor,
                       float *cs, float *sn) {
    for (int j = 0; j < half; j++) {
        float ang = pos * inv_freq[j];
        cs[j] = cosf(ang) * attn_factor;
        sn[j] = sinf(ang) * attn_factor;
    }
}

/* RoPE rotation of one head vector, non-interleaved halves (picchio.c:467-469).
 * gcc contracts a*cs - b*sn into fma(a, cs, -(b*sn)) and a*sn + b*cs into
 * fma(a, sn, b*cs); the tests pin this against the compiled reference. */
OR_API void or_rope_rotate(float *v, int head_dim, const float *cs, const float *sn) {
    int half = head_dim / 2;
    for (int j = 0; j < half; j++) {
        float a = v[j], b = v[j + half];
        v[j] = fmaf(a, cs[j], -(b * sn[j]));
        v[j + half] = fmaf(a, sn[j], b * cs[j]);
    }
}

/* GQA decode attention for one position with sinks and window
 * (picchio.c:556-607).  Kc/Vc: [n_pos_alloc][KVH*hd] fp32; q: [H*hd];
 * out: [H*hd].  start/end are inclusive positions. */
OR_API void or_attention(float *out, const float *q, const float *Kc, const float *Vc,
                         const float *sinks, int H, int KVH, int hd, int start, int end) {
    int kv_dim = KVH * hd, group = H / KVH;
    int n_pos = end - start + 1;
    if (n_pos <= 0) n_pos = 1;
    float *sc = (float *)calloc((size_t)n_pos, sizeof(float));
    float scale = 1.0f / sqrtf((float)hd);
    memset(out, 0, sizeof(float) * (size_t)H * hd);
    for (int h = 0; h < H; h++) {
        int kh = h / group;
        const float *qh = q + h * hd;
        for (int t = start; t <= end; t++) {
            const float *kt = Kc + (int64_t)t * kv_dim + kh * hd;
            float dot = 0;
            /* The reference build keeps this dot as separate multiply and
             * add (pinned against oracle/_ref); the P.V update below fuses. */
            for (int i = 0; i < hd; i++) dot = dot + qh[i] * kt[i];
            sc[t - start] = dot * scale;
        }
        float mx = sinks ? sinks[h] : -INFINITY;
        for (int i = 0; i < n_pos; i++) if (sc[i] > mx) mx = sc[i];
        float sum = sinks ? expf(sinks[h] - mx) : 0.0f;
        for (int i = 0; i < n_pos; i++) { sc[i] = expf(sc[i] - mx); sum += sc[i]; }
        for (int i = 0; i < n_pos; i++) sc[i] /= sum;
        float *oh = out + h * hd;
        for (int t = start; t <= end; t++) {
            const float *vt = Vc + (int64_t)t * kv_dim + kh * hd;
            float w = sc[t - start];
            for (int i = 0; i < hd; i++) oh[i] = fmaf(w, vt[i], oh[i]);
        }
    }
    free(sc);
}

/* Weighted expert accumulate, picchio.c:1453-1454: out[i] += w * eo[i]. */
OR_API void or_axpy(float *out, const float *eo, float w, int n) {
    for (int i = 0; i < n; i++) out[i] = fmaf(w, eo[i], out[i]);
}

/* Greedy pick, picchio.c:1555-1560: first maximum wins. */
OR_API int or_argmax(const float *logits, int n) {
    int best = 0;
    for (int i = 1; i < n; i++) if (logits[i] > logits[best]) best = i;
    return best;
}

/* ------------------------------------------------------------ sampling ---- */
/* sample_logits (picchio.c:1540-1649) with the sampler's globals passed in:
 * repetition penalty over the history (1542-1552), temperature (1555-1565),
 * top-k with the k-th largest value as threshold and ties kept (1571-1581),
 * softmax with expf (1584-1591), top-p over the probabilities above 1e-10
 * sorted descending (1594-1627), then the draw from the xorshift64 generator
 * (1520-1526, 1631-1647).  The reference leaves the order of EQUAL
 * probabilities in its top-p sort to qsort; this restatement orders them by
 * id, as the device sampler does.  logits are modified in place like the
 * reference's; the history (at most 4096 ids) and the generator state are
 * read and updated through the pointers. */
typedef struct { float p; int id; } or_cand;

static int or_desc_f(const void *a, const void *b) {
    const float x = *(const float *)a, y = *(const float *)b;
    return (x < y) - (x > y);
}

static int or_desc_cand(const void *a, const void *b) {
    const or_cand *x = (const or_cand *)a, *y = (const or_cand *)b;
    if (x->p != y->p) return x->p < y->p ? 1 : -1;
    return (x->id > y->id) - (x->id < y->id);
}

static int or_keep(int *hist, int *hist_len, int id) {
    if (*hist_len < 4096) hist[(*hist_len)++] = id;
    return id;
}

OR_API int or_sample(float *lg, int V, float temperature, float top_p, int top_k, float rep,
                     int *hist, int *hist_len, uint64_t *rng) {
    if (rep > 1.0f)
        for (int h = 0; h < *hist_len; ++h) {
            const int t = hist[h];
            if (t >= 0 && t < V) lg[t] = lg[t] > 0 ? lg[t] / rep : lg[t] * rep;
        }
    if (temperature < 1e-6f) {
        int best = 0;
        for (int i = 1; i < V; ++i)
            if (lg[i] > lg[best]) best = i;
        return or_keep(hist, hist_len, best);
    }
    const float inv = 1.0f / temperature;
    for (int i = 0; i < V; ++i) lg[i] *= inv;
    if (top_k > 0 && top_k < V) {
        float *sorted = (float *)malloc((size_t)V * sizeof(float));
        memcpy(sorted, lg, (size_t)V * sizeof(float));
        qsort(sorted, (size_t)V, sizeof(float), or_desc_f);
        const float th = sorted[top_k - 1];
        free(sorted);
        for (int i = 0; i < V; ++i)
            if (lg[i] < th) lg[i] = -1e30f;
    }
    float mx = -1e30f;
    for (int i = 0; i < V; ++i)
        if (lg[i] > mx) mx = lg[i];
    float sum = 0.0f;
    for (int i = 0; i < V; ++i) {
        lg[i] = expf(lg[i] - mx);
        sum += lg[i];
    }
    for (int i = 0; i < V; ++i) lg[i] /= sum;
    if (top_p < 1.0f && top_p > 0.0f) {
        int n = 0;
        for (int i = 0; i < V; ++i) n += lg[i] > 1e-10f;
        if (n > 1) {
            or_cand *c = (or_cand *)malloc((size_t)n * sizeof(or_cand));
            n = 0;
            for (int i = 0; i < V; ++i)
                if (lg[i] > 1e-10f) {
                    c[n].p = lg[i];
                    c[n].id = i;
                    ++n;
                }
            qsort(c, (size_t)n, sizeof(or_cand), or_desc_cand);
            float cum = 0.0f;
            int cut = n;
            for (int j = 0; j < n; ++j) {
                cum += c[j].p;
                if (cum >= top_p) {
                    cut = j + 1;
                    break;
                }
            }
            for (int j = cut; j < n; ++j) lg[c[j].id] = 0.0f;
            float s2 = 0.0f;
            for (int i = 0; i < V; ++i) s2 += lg[i];
            if (s2 > 0)
                for (int i = 0; i < V; ++i) lg[i] /= s2;
            free(c);
        }
    }
    uint64_t s = *rng;
    s ^= s << 13;
    s ^= s >> 7;
    s ^= s << 17;
    *rng = s;
    const float r = (float)(s >> 33) / (float)(1ULL << 31);
    float cum = 0.0f;
    for (int i = 0; i < V; ++i) {
        cum += lg[i];
        if (cum >= r) return or_keep(hist, hist_len, i);
    }
    for (int i = V - 1; i >= 0; --i)
        if (lg[i] > 0) return or_keep(hist, hist_len, i);
    return 0;
}
