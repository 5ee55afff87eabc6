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
 * Greedy decoding (TEMPERATURE=0) takes the next id from the device argmax;
 * other settings copy the logits back and sample on the host with the
 * reference's procedure (picchio.c:1520-1649).
 */
#include <limits.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <math.h>
#include <time.h>

#include "picchio_b200.h"

#define TOK_RETURN 200002
#define TOK_CALL 200012

static float g_temperature = 1.0f, g_top_p = 0.95f, g_rep = 1.1f;
static int g_top_k = 50;
static int g_history[4096];
static int g_history_len = 0;
static uint64_t g_rng = 1234567890123456789ULL;

static float rng_float(void) { /* xorshift64, picchio.c:1521-1526 */
    g_rng ^= g_rng << 13;
    g_rng ^= g_rng >> 7;
    g_rng ^= g_rng << 17;
    return (float)(g_rng >> 33) / (float)(1ULL << 31);
}

typedef struct { float v; int i; } IV;
static int cmp_iv(const void *a, const void *b) {
    float x = ((const IV *)a)->v, y = ((const IV *)b)->v;
    return (x < y) - (x > y);
}
static int cmp_f(const void *a, const void *b) {
    float x = *(const float *)a, y = *(const float *)b;
    return (x < y) - (x > y);
}

/* sample_logits (picchio.c:1540-1649) for TEMPERATURE > 0. */
static int sample_host(float *lg, int V) {
    if (g_rep > 1.0f)
        for (int i = 0; i < g_history_len; i++) {
            int t = g_history[i];
            if (t >= 0 && t < V) lg[t] = lg[t] > 0 ? lg[t] / g_rep : lg[t] * g_rep;
        }
    if (g_temperature < 1e-6f) {
        int best = 0;
        for (int i = 1; i < V; i++) if (lg[i] > lg[best]) best = i;
        if (g_history_len < 4096) g_history[g_history_len++] = best;
        return best;
    }
    float inv = 1.0f / g_temperature;
    for (int i = 0; i < V; i++) lg[i] *= inv;
    if (g_top_k > 0 && g_top_k < V) {
        float *s = (float *)malloc((size_t)V * sizeof(float));
        if (s) {
            memcpy(s, lg, (size_t)V * sizeof(float));
            qsort(s, V, sizeof(float), cmp_f);
            float th = s[g_top_k - 1];
            free(s);
            for (int i = 0; i < V; i++) if (lg[i] < th) lg[i] = -1e30f;
        }
    }
    float mx = -1e30f;
    for (int i = 0; i < V; i++) if (lg[i] > mx) mx = lg[i];
    float sum = 0;
    for (int i = 0; i < V; i++) { lg[i] = expf(lg[i] - mx); sum += lg[i]; }
    for (int i = 0; i < V; i++) lg[i] /= sum;
    if (g_top_p < 1.0f && g_top_p > 0.0f) {
        int n = 0;
        for (int i = 0; i < V; i++) if (lg[i] > 1e-10f) n++;
        if (n > 1) {
            IV *so = (IV *)malloc((size_t)n * sizeof(IV));
            int k = 0;
            for (int i = 0; i < V; i++) if (lg[i] > 1e-10f) { so[k].v = lg[i]; so[k].i = i; k++; }
            qsort(so, n, sizeof(IV), cmp_iv);
            float cum = 0;
            int cut = n;
            for (int i = 0; i < n; i++) { cum += so[i].v; if (cum >= g_top_p) { cut = i + 1; break; } }
            for (int i = cut; i < n; i++) lg[so[i].i] = 0.0f;
            sum = 0;
            for (int i = 0; i < V; i++) sum += lg[i];
            if (sum > 0) for (int i = 0; i < V; i++) lg[i] /= sum;
            free(so);
        }
    }
    float r = rng_float(), cum = 0;
    for (int i = 0; i < V; i++) {
        cum += lg[i];
        if (cum >= r) { if (g_history_len < 4096) g_history[g_history_len++] = i; return i; }
    }
    for (int i = V - 1; i >= 0; i--)
        if (lg[i] > 0) { if (g_history_len < 4096) g_history[g_history_len++] = i; return i; }
    return 0;
}

static pc_model_cfg g_cfg;
static float *g_logits = NULL;

static int need_host_sampling(void) { return !(g_temperature < 1e-6f) || g_rep > 1.0f; }

/* Picks the next id after a forward: device argmax when greedy without a
 * repetition penalty, else the host sampler on the copied logits. */
static int choose(pc_ctx *ctx, int device_pick) {
    if (!need_host_sampling()) {
        if (g_history_len < 4096) g_history[g_history_len++] = device_pick;
        return device_pick;
    }
    if (pc_get_logits(ctx, 0, g_logits, g_cfg.vocab) != PC_OK) return device_pick;
    return sample_host(g_logits, g_cfg.vocab);
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
            g_history_len = 0;
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
        pc_status s = pc_prefill(ctx, ids, (int)n_ids, pos, &next);
        free(ids);
        if (s != PC_OK) return die("prefill", s);
        next = choose(ctx, next);
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
            following = choose(ctx, following);
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
    if ((v = getenv("SEED"))) g_rng = (uint64_t)atoll(v);
    else g_rng = (uint64_t)time(NULL);

    pc_ctx *ctx = NULL;
    double t0 = now_s();
    pc_status s = pc_init(model, &o, &ctx);
    if (s != PC_OK) return die("pc_init", s);
    pc_get_config(ctx, &g_cfg);
    g_logits = (float *)malloc((size_t)g_cfg.vocab * sizeof(float));
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
    if (g_rep > 1.0f)
        for (int i = 0; i < n_prompt && g_history_len < 4096; i++) g_history[g_history_len++] = prompt[i];
    int output_ids = (v = getenv("OUTPUT")) && !strcmp(v, "ids");

    double tp = now_s();
    int tok;
    s = pc_prefill(ctx, prompt, n_prompt, 0, &tok);
    if (s != PC_OK) return die("prefill", s);
    tok = choose(ctx, tok);
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
        tok = choose(ctx, next);
        pos++;
        emitted++;
    }
    printf("\n");
    double dt = now_s() - tg;
    if (emitted > 0) fprintf(stderr, "generated %d tokens in %.3f s (%.1f tok/s)\n", emitted, dt, emitted / dt);
    free(prompt);
    free(g_logits);
    pc_free(ctx);
    return 0;
}
