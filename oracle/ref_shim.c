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
