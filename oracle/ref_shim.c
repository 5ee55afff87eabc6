/* ref_shim.c - exposes the reference's own static functions to the tests.
 *
 * TEST INFRASTRUCTURE ONLY.  This file holds no arithmetic of its own: it
 * compiles the unmodified reference translation unit (picchio.c, which
 * includes quant.h) from the reference tree named on the compiler command
 * line (-I <reference>) and adds thin extern wrappers around the static
 * functions the parity tests call.  The result, oracle/_ref/libpicchio_ref.so,
 * is the reference itself run here; oracle/oracle.c is checked against it.
 */
#define main picchio_reference_main
#include "picchio.c"
#undef main

#define REF_API __attribute__((visibility("default")))

/* quant.h:323 matmul_qt for each format. */
REF_API void ref_matmul_f32(float *y, const float *x, const float *W, int S, int I, int O) {
    matmul_f32(y, x, W, S, I, O);
}
REF_API void ref_matmul_q8(float *y, const float *x, const int8_t *q, const float *s,
                           int S, int I, int O) {
    matmul_q8(y, x, q, s, S, I, O);
}
REF_API void ref_matmul_i4(float *y, const float *x, const uint8_t *q4, const float *s,
                           int S, int I, int O) {
    matmul_i4(y, x, q4, s, S, I, O);
}
REF_API void ref_matmul_i4_gs(float *y, const float *x, const uint8_t *q4, const float *s,
                              int S, int I, int O, int gs) {
    matmul_i4_gs(y, x, q4, s, S, I, O, gs);
}
REF_API void ref_quantize_rows_i4(const float *w, uint8_t *q4, float *s, int O, int I) {
    quantize_rows_i4(w, q4, s, O, I);
}
REF_API void ref_rmsnorm(float *out, const float *x, const float *w, int D, float eps) {
    rmsnorm(out, x, w, D, eps);
}
REF_API void ref_softmax(float *x, int n) { softmax(x, n); }
REF_API float ref_sigmoidf(float x) { return sigmoidf(x); }

/* picchio.c:455 rope_apply on one q block and one k block. */
REF_API void ref_rope_apply(float *q, float *k, int pos, int head_dim, int nq, int nkv,
                            float theta, float factor, float beta_fast, float beta_slow,
                            int orig_ctx, int truncate) {
    Cfg c;
    memset(&c, 0, sizeof(c));
    c.head_dim = head_dim;
    c.theta = theta;
    c.rope_factor = factor;
    c.rope_beta_fast = beta_fast;
    c.rope_beta_slow = beta_slow;
    c.rope_original_ctx = orig_ctx;
    c.rope_truncate = truncate;
    c.rope_attn_factor = factor > 1.0f ? 0.1f * logf(factor) + 1.0f : 1.0f;
    rope_apply(q, k, pos, head_dim, nq, nkv, &c);
}

REF_API float ref_yarn_inv_freq(int head_dim, float theta, float factor, float beta_fast,
                                float beta_slow, int orig_ctx, int truncate, int j) {
    Cfg c;
    memset(&c, 0, sizeof(c));
    c.head_dim = head_dim;
    c.theta = theta;
    c.rope_factor = factor;
    c.rope_beta_fast = beta_fast;
    c.rope_beta_slow = beta_slow;
    c.rope_original_ctx = orig_ctx;
    c.rope_truncate = truncate;
    return yarn_inv_freq(&c, j);
}

/* expert_apply (picchio.c:1769-1791) on one expert given as buffers in the
 * reference's host layout: gate_up + bias + clamped SwiGLU + down + bias,
 * dst += w * out. */
REF_API void ref_expert_apply(const uint8_t *gu_q, const float *gu_s, int gu_bs, const float *gu_b,
                              const uint8_t *dn_q, const float *dn_s, int dn_bs, const float *dn_b,
                              int D, int I2, const float *x, float *dst, float w, float limit) {
    Cfg c;
    memset(&c, 0, sizeof(c));
    c.hidden = D;
    c.moe_inter = I2;
    c.swiglu_limit = limit;
    c.swiglu_alpha = 1.702f;
    ESlot es;
    memset(&es, 0, sizeof(es));
    es.gu.fmt = 2; es.gu.O = I2; es.gu.I = D; es.gu.q4 = (uint8_t *)gu_q; es.gu.s = (float *)gu_s;
    es.gu.block_size = gu_bs;
    es.d.fmt = 2; es.d.O = D; es.d.I = I2 / 2; es.d.q4 = (uint8_t *)dn_q; es.d.s = (float *)dn_s;
    es.d.block_size = dn_bs;
    es.gu_bias = (float *)gu_b;
    es.d_bias = (float *)dn_b;
    expert_apply(&es, x, dst, w, &c);
}

/* gqa_attention (picchio.c:504-623) for one layer with INT8 projections and
 * an fp32 KV cache of max_pos positions: projections, bias, RoPE, KV store,
 * scores with sinks and window, P.V, output projection. */
REF_API void ref_gqa_attention(const int8_t *wq, const float *sq, const int8_t *wk, const float *sk,
                               const int8_t *wv, const float *sv, const int8_t *wo, const float *so,
                               const float *bq, const float *bk, const float *bv, const float *bo,
                               const float *sinks, float *Kc, float *Vc, int max_pos, int layer_type,
                               int window, int pos, const float *x, float *out, int D, int H, int KVH,
                               int hd, float theta) {
    Cfg c;
    memset(&c, 0, sizeof(c));
    c.hidden = D; c.n_heads = H; c.n_kv_heads = KVH; c.head_dim = hd; c.sliding_window = window;
    c.theta = theta; c.rope_factor = 1.0f; c.rope_attn_factor = 1.0f;
    Layer ly;
    memset(&ly, 0, sizeof(ly));
    ly.wq.fmt = 1; ly.wq.O = H * hd; ly.wq.I = D; ly.wq.q8 = (int8_t *)wq; ly.wq.s = (float *)sq;
    ly.wk.fmt = 1; ly.wk.O = KVH * hd; ly.wk.I = D; ly.wk.q8 = (int8_t *)wk; ly.wk.s = (float *)sk;
    ly.wv.fmt = 1; ly.wv.O = KVH * hd; ly.wv.I = D; ly.wv.q8 = (int8_t *)wv; ly.wv.s = (float *)sv;
    ly.wo.fmt = 1; ly.wo.O = D; ly.wo.I = H * hd; ly.wo.q8 = (int8_t *)wo; ly.wo.s = (float *)so;
    ly.bq = (float *)bq; ly.bk = (float *)bk; ly.bv = (float *)bv; ly.bo = (float *)bo;
    ly.sinks = (float *)sinks;
    ly.layer_type = layer_type;
    float *Kp[1] = {Kc}, *Vp[1] = {Vc};
    KVCache kv;
    kv.K = Kp; kv.V = Vp; kv.max_pos = max_pos; kv.cur_pos = 0;
    gqa_attention(out, x, &ly, &kv, 0, pos, &c);
}

/* sample_logits (picchio.c:1540) with its globals (g_temperature, g_top_p,
 * g_top_k, g_rep_penalty, g_history, g_history_len, g_rng) loaded from the
 * arguments before the call and stored back after it. */
REF_API int ref_sample_logits(float *logits, int vocab, float temperature, float top_p, int top_k,
                              float rep, int *history, int *history_len, uint64_t *rng) {
    g_temperature = temperature;
    g_top_p = top_p;
    g_top_k = top_k;
    g_rep_penalty = rep;
    g_history_len = *history_len;
    memcpy(g_history, history, (size_t)g_history_len * sizeof(int));
    g_rng = *rng;
    const int id = sample_logits(logits, vocab);
    *history_len = g_history_len;
    memcpy(history, g_history, (size_t)g_history_len * sizeof(int));
    *rng = g_rng;
    return id;
}

/* The OpenMP team size of the reference's parallel loops (#pragma omp
 * parallel for in quant.h's matmuls): set before timing, whatever
 * OMP_NUM_THREADS said when the runtime started, and read back. */
#include <omp.h>
REF_API void ref_set_threads(int n) { omp_set_num_threads(n); }
REF_API int ref_max_threads(void) { return omp_get_max_threads(); }
