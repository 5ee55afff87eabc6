/* picchio_gpu.c - the picchio command-line engine on the B200 C ABI.
 *
 * Same interface as the reference binary (picchio.c:2801-3310): MODEL or
 * argv[1], MAX or argv[2], CTX, INPUT_FILE (decimal token ids), INPUT / RAW
 * ids, OUTPUT=ids, TEMPERATURE / TOPP / TOPK / REP / SEED sampling, SERVICE=1
 * line protocol (picchio.c:2700-2795: READY / TURN / TOKEN / DONE / ERROR /
 * RESET / SHUTDOWN).  Extra: KV_BF16=1 selects the bf16 KV cache, DEVICE
 * the CUDA ordinal.  There is no tokenizer here: prompts are token ids, as
 * the reference takes them when it has no tokenizer.json.
 *
 * Greedy decoding without a repetition penalty takes the next id from the
 * device argmax; any other setting draws it on the device (pc_set_sampling:
 * the reference's sample_logits, picchio.c:1520-1649, with the generator
 * state and the repetition history kept in device memory).
 */
#include <limits.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include "picchio_b200.h"

#define TOK_RETURN 200002
#define TOK_CALL 200012

/* the reference's defaults (picchio.c:1510-1520) */
static float g_temperature = 1.0f, g_top_p = 0.95f, g_rep = 1.1f;
static int g_top_k = 50;
static uint64_t g_seed = 1234567890123456789ULL;

/* Device sampling is needed unless decoding is greedy without a penalty
 * (then sample_logits is the plain argmax, picchio.c:1555-1560, and the
 * history it records is never read). */
static pc_model_cfg g_cfg;

static pc_status apply_sampling(pc_ctx *ctx) {
    if (g_temperature < 1e-6f && !(g_rep > 1.0f)) return pc_set_sampling(ctx, NULL);
    pc_sampling s;
    s.temperature = g_temperature;
    s.top_p = g_top_p;
    s.top_k = g_top_k;
    s.rep_penalty = g_rep;
    return pc_set_sampling(ctx, &s);
}

static int die(const char *what, pc_status s) {
    fprintf(stderr, "error: %s: %s (%s)\n", what, pc_status_string(s), pc_last_error());
    return 1;
}

static int read_ids(const char *path, int max_tokens, int **out) {
    FILE *f = fopen(path, "rb");
    if (!f) { fprintf(stderr, "error: cannot open INPUT_FILE=%s\n", path); return -1; }
    int cap = 256, n = 0;
    int *ids = (int *)malloc((size_t)cap * sizeof(int));
    long v;
    int rc;
    while ((rc = fscanf(f, "%ld", &v)) == 1) {
        if (v < 0 || v > INT_MAX || n >= max_tokens) {
            fprintf(stderr, "error: invalid ID or prompt beyond %d tokens in %s\n", max_tokens, path);
            free(ids); fclose(f); return -1;
        }
        if (n == cap) { cap *= 2; ids = (int *)realloc(ids, (size_t)cap * sizeof(int)); }
        ids[n++] = (int)v;
    }
    fclose(f);
    if (rc != EOF) { fprintf(stderr, "error: non-numeric content in INPUT_FILE=%s\n", path); free(ids); return -1; }
    if (n == 0) { fprintf(stderr, "error: empty INPUT_FILE: %s\n", path); free(ids); return -1; }
    *out = ids;
    return n;
}

/* service_loop (picchio.c:2700-2795) */
static int service(pc_ctx *ctx, int cap) {
    int pos = 0;
    printf("READY %d %d %d %d\n", cap, g_cfg.vocab, TOK_RETURN, TOK_CALL);
    fflush(stdout);
    char cmd[32];
    while (scanf("%31s", cmd) == 1) {
        if (!strcmp(cmd, "SHUTDOWN")) break;
        if (!strcmp(cmd, "RESET")) {
            pos = 0;
            pc_status rs = pc_history_reset(ctx);
            if (rs != PC_OK) return die("history reset", rs);
            printf("DONE RESET 0 0\n");
            fflush(stdout);
            continue;
        }
        if (strcmp(cmd, "TURN")) { printf("ERROR BAD_COMMAND 1 unknown command\n"); fflush(stdout); return 1; }
        long max_new = 0, keep = 0, n_ids = 0, t_topk = 0;
        float t_temp = 0, t_topp = 0;
        if (scanf("%ld %ld %f %f %ld %ld", &max_new, &keep, &t_temp, &t_topp, &t_topk, &n_ids) != 6) {
            printf("ERROR BAD_HEADER 1 unreadable TURN header\n");
            fflush(stdout);
            return 1;
        }
        if (t_temp < 0) t_temp = 0;
        if (t_temp > 5) t_temp = 5;
        if (t_topp <= 0 || t_topp > 1) t_topp = 1;
        if (t_topk < 0) t_topk = 0;
        g_temperature = t_temp;
        g_top_p = t_topp;
        g_top_k = (int)t_topk;
        pc_status ss = apply_sampling(ctx);
        if (ss != PC_OK) return die("sampling settings", ss);
        if (max_new < 0 || keep < 0 || keep > pos || n_ids <= 0 || keep + n_ids > cap || n_ids > cap) {
            printf("ERROR BAD_RANGE 0 keep/n_ids out of bounds (pos=%d cap=%d)\n", pos, cap);
            fflush(stdout);
            for (long i = 0; i < n_ids; i++) { long s; if (scanf("%ld", &s) != 1) return 1; }
            continue;
        }
        int *ids = (int *)malloc((size_t)n_ids * sizeof(int));
        int valid = 1;
        for (long i = 0; i < n_ids; i++) {
            long v;
            if (scanf("%ld", &v) != 1) { free(ids); return 1; }
            if (v < 0 || v >= g_cfg.vocab) valid = 0;
            ids[i] = (int)v;
        }
        if (!valid) { free(ids); printf("ERROR BAD_TOKEN 0 ID out of vocabulary\n"); fflush(stdout); continue; }
        pos = (int)keep;  /* prefix reuse: later positions are overwritten */
        int next;
        pc_status s = PC_OK;
        /* prefill_tokens seeds the history with a multi-token prompt (picchio.c:1963-1967) */
        if (g_rep > 1.0f && n_ids > 1) s = pc_history_push(ctx, ids, (int)n_ids);
        if (s == PC_OK) s = pc_prefill(ctx, ids, (int)n_ids, pos, &next);
        free(ids);
        if (s != PC_OK) return die("prefill", s);
        pos += (int)n_ids;
        const char *reason = "MAX_TOKENS";
        int produced = 0, tok = next;
        for (;;) {
            if (produced >= max_new) { reason = "MAX_TOKENS"; break; }
            if (pos >= cap) { reason = "CONTEXT_FULL"; break; }
            printf("TOKEN %d\n", tok);
            fflush(stdout);
            produced++;
            int following;
            s = pc_forward_token(ctx, tok, pos, &following);
            if (s != PC_OK) return die("forward", s);
            pos++;
            if (tok == TOK_RETURN) { reason = "RETURN"; break; }
            if (tok == TOK_CALL) { reason = "CALL"; break; }
            tok = (following < 0 || following >= g_cfg.vocab) ? 0 : following;
        }
        printf("DONE %s %d %d\n", reason, produced, pos);
        fflush(stdout);
    }
    return 0;
}

static double now_s(void) {
    struct timespec t;
    clock_gettime(CLOCK_MONOTONIC, &t);
    return t.tv_sec + t.tv_nsec * 1e-9;
}

int main(int argc, char **argv) {
    const char *model = getenv("MODEL");
    if (!model) {
        if (argc > 1) model = argv[1];
        else { fprintf(stderr, "Usage: MODEL=/path/to/model ./picchio-gpu [max_tokens]\n"); return 1; }
    }
    int max_tokens = 128;
    const char *v;
    if ((v = getenv("MAX"))) max_tokens = atoi(v);
    else if (argc > 2) max_tokens = atoi(argv[2]);
    pc_opts o;
    pc_default_opts(&o);
    if ((v = getenv("CTX"))) o.ctx_len = atoi(v);
    if ((v = getenv("KV_BF16"))) o.kv_bf16 = atoi(v) != 0;
    if ((v = getenv("DEVICE"))) o.device = atoi(v);
    if ((v = getenv("TEMPERATURE"))) g_temperature = (float)atof(v);
    if ((v = getenv("TOPP"))) g_top_p = (float)atof(v);
    if ((v = getenv("TOPK"))) g_top_k = atoi(v);
    if ((v = getenv("REP"))) g_rep = (float)atof(v);
    if ((v = getenv("SEED"))) g_seed = (uint64_t)atoll(v);
    else g_seed = (uint64_t)time(NULL);

    pc_ctx *ctx = NULL;
    double t0 = now_s();
    pc_status s = pc_init(model, &o, &ctx);
    if (s != PC_OK) return die("pc_init", s);
    pc_get_config(ctx, &g_cfg);
    if ((s = pc_set_rng(ctx, g_seed)) != PC_OK || (s = apply_sampling(ctx)) != PC_OK)
        return die("sampling setup", s);
    fprintf(stderr, "loaded %s in %.1f s: D=%d L=%d E=%d top%d vocab=%d ctx=%d\n", model, now_s() - t0,
            g_cfg.hidden, g_cfg.n_layers, g_cfg.n_experts, g_cfg.topk, g_cfg.vocab, o.ctx_len);

    if ((v = getenv("SERVICE")) && atoi(v)) {
        int rc = service(ctx, o.ctx_len);
        pc_free(ctx);
        return rc;
    }

    int *prompt = NULL, n_prompt = 0;
    const char *input_file = getenv("INPUT_FILE");
    if (input_file && *input_file) {
        n_prompt = read_ids(input_file, g_cfg.ctx_len, &prompt);
        if (n_prompt < 0) { pc_free(ctx); return 1; }
    } else {
        const char *p = getenv("INPUT");
        if (!p) p = getenv("PROMPT");
        char line[65536] = "";
        if (!p) { if (fgets(line, sizeof line, stdin)) p = line; }
        prompt = (int *)malloc(8192 * sizeof(int));
        while (p && *p && n_prompt < 8192) {
            while (*p == ' ' || *p == '\n' || *p == '\r') p++;
            if (!*p) break;
            char *e;
            long id = strtol(p, &e, 10);
            if (e == p) break;
            prompt[n_prompt++] = (int)id;
            p = e;
        }
    }
    if (n_prompt == 0) { fprintf(stderr, "error: empty prompt\n"); pc_free(ctx); return 1; }
    for (int i = 0; i < n_prompt; i++)
        if (prompt[i] < 0 || prompt[i] >= g_cfg.vocab) {
            fprintf(stderr, "error: token ID out of vocabulary at position %d: %d\n", i, prompt[i]);
            pc_free(ctx);
            return 1;
        }
    if (g_rep > 1.0f && n_prompt > 1 && (s = pc_history_push(ctx, prompt, n_prompt)) != PC_OK)  /* picchio.c:1963-1967 */
        return die("history", s);
    int output_ids = (v = getenv("OUTPUT")) && !strcmp(v, "ids");

    double tp = now_s();
    int tok;
    s = pc_prefill(ctx, prompt, n_prompt, 0, &tok);
    if (s != PC_OK) return die("prefill", s);
    fprintf(stderr, "prefill %d tokens in %.3f s\n", n_prompt, now_s() - tp);
    double tg = now_s();
    int pos = n_prompt, emitted = 0;
    for (int i = 0; i < max_tokens; i++) {
        if (output_ids) { printf("%d\n", tok); fflush(stdout); }
        if (tok == TOK_RETURN || tok == TOK_CALL) break;
        if (!output_ids) { printf("[%d]", tok); fflush(stdout); }
        if (pos >= o.ctx_len) { fprintf(stderr, "context full (%d)\n", o.ctx_len); break; }
        int next;
        s = pc_forward_token(ctx, tok, pos, &next);
        if (s != PC_OK) return die("forward", s);
        tok = next;
        pos++;
        emitted++;
    }
    printf("\n");
    double dt = now_s() - tg;
    if (emitted > 0) fprintf(stderr, "generated %d tokens in %.3f s (%.1f tok/s)\n", emitted, dt, emitted / dt);
    free(prompt);
    pc_free(ctx);
    return 0;
}
