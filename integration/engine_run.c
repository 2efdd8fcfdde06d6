/*
 * engine_run.c — drives an engine library through its public API (the
 * reference's src/waste.h): opens a container, evaluates a prompt (one call
 * with every prompt token, which the engine runs as a chunked prefill
 * through moe_chunk), then greedy decode steps (one token each, moe_layer),
 * and writes each call's logits to a file.
 *
 *   engine_run <engine.so> <container dir> <out.bin> <decode steps> <tok>...
 *
 * The engine library is opened with dlopen, so the same driver runs the
 * unmodified reference engine and the one built by this directory's
 * Makefile with the CUDA backend. out.bin: int32 evals, int32 vocab, then
 * per eval int32 argmax and vocab floats. The engine's build info (which
 * names the backend it selected) is printed on stdout.
 *
 * With ENGINE_RUN_STATE=<path> the conversation state goes through a
 * snapshot half way: after the prompt and steps/2 decode steps the state is
 * saved (waste_state_save), the context reset (waste_state_reset) and the
 * prompt evaluated again (one extra eval, which must repeat eval 0), then
 * the snapshot loaded (waste_state_load) and the remaining steps decoded
 * from where the save left off.
 *
 * Each eval's wall-clock time is printed ("eval <e>: next token <t> (<ms>
 * ms)"), the time to open the container ("open: <ms> ms") and, with
 * WASTE_PROFILE=1, the engine's own phase times per eval over the evals
 * after the first three ("prof <phase>: ...").
 */
#include "waste.h"

#include <dlfcn.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <time.h>

static double now_ms(void)
{
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return ts.tv_sec * 1e3 + ts.tv_nsec * 1e-6;
}

typedef void (*cfg_init_fn)(waste_cfg *);
typedef waste_status (*open_fn)(const char *, const waste_cfg *, waste_ctx **);
typedef waste_status (*eval_fn)(waste_ctx *, const int32_t *, size_t, const float **, size_t *);
typedef void (*close_fn)(waste_ctx *);
typedef const char *(*str_fn)(void);
typedef const char *(*detail_fn)(const waste_ctx *);
typedef waste_status (*state_fn)(waste_ctx *, const char *);
typedef void (*reset_fn)(waste_ctx *);

static int argmax(const float *v, size_t n)
{
    size_t b = 0;
    for (size_t i = 1; i < n; i++)
        if (v[i] > v[b]) b = i;
    return (int)b;
}

int main(int argc, char **argv)
{
    if (argc < 6) {
        fprintf(stderr, "usage: %s engine.so container out.bin steps tok...\n", argv[0]);
        return 2;
    }
    void *h = dlopen(argv[1], RTLD_NOW | RTLD_LOCAL);
    if (!h) { fprintf(stderr, "dlopen: %s\n", dlerror()); return 2; }
    cfg_init_fn cfg_init = (cfg_init_fn)dlsym(h, "waste_cfg_init");
    open_fn wopen = (open_fn)dlsym(h, "waste_open");
    eval_fn weval = (eval_fn)dlsym(h, "waste_eval");
    close_fn wclose = (close_fn)dlsym(h, "waste_close");
    str_fn info = (str_fn)dlsym(h, "waste_build_info");
    detail_fn detail = (detail_fn)dlsym(h, "waste_error_detail");
    if (!cfg_init || !wopen || !weval || !wclose || !info) {
        fprintf(stderr, "engine library lacks the waste.h entry points\n");
        return 2;
    }
    const int steps = atoi(argv[4]);
    const int np = argc - 5;
    int32_t *prompt = (int32_t *)malloc((size_t)np * sizeof(int32_t));
    for (int i = 0; i < np; i++) prompt[i] = atoi(argv[5 + i]);

    waste_cfg cfg;
    cfg_init(&cfg);
    cfg.ctx_tokens = 256;
    cfg.n_threads = 0;
    waste_ctx *ctx = NULL;
    const double t_open = now_ms();
    waste_status st = wopen(argv[2], &cfg, &ctx);
    if (st != WASTE_OK) { fprintf(stderr, "waste_open: %d\n", (int)st); return 1; }
    printf("build: %s\n", info());
    printf("open: %.1f ms\n", now_ms() - t_open);

    FILE *out = fopen(argv[3], "wb");
    if (!out) { perror("out"); return 1; }
    const char *snap = getenv("ENGINE_RUN_STATE");
    state_fn ssave = (state_fn)dlsym(h, "waste_state_save");
    state_fn sload = (state_fn)dlsym(h, "waste_state_load");
    reset_fn sreset = (reset_fn)dlsym(h, "waste_state_reset");
    if (snap && (!ssave || !sload || !sreset)) {
        fprintf(stderr, "engine library lacks the state entry points\n");
        return 2;
    }
    const int half = snap ? steps / 2 : -1;     /* decode steps before the snapshot */
    const int32_t nev = 1 + steps + (snap ? 1 : 0);
    int32_t vocab32 = 0;
    fwrite(&nev, 4, 1, out);
    fwrite(&vocab32, 4, 1, out);           /* patched below */
    const float *lg = NULL;
    size_t vocab = 0;
    int32_t tok = 0, tok_saved = 0;
    /* the profile is reported over the decode evals after the first two */
    const double *prof = (const double *)dlsym(h, "waste_prof");
    const uint64_t *prof_n = (const uint64_t *)dlsym(h, "waste_prof_n");
    double prof0[16] = {0};
    uint64_t prof0_n[16] = {0};
    const int prof_from = nev > 4 ? 3 : 0;
    for (int e = 0; e < nev; e++) {
        if (prof && prof_n && e == prof_from)
            for (int i = 0; i < 16; i++) { prof0[i] = prof[i]; prof0_n[i] = prof_n[i]; }
        const int again = snap && e == 1 + half;   /* the prompt after the reset */
        if (again) {
            tok_saved = tok;
            if (ssave(ctx, snap) != WASTE_OK) { fprintf(stderr, "state save failed\n"); return 1; }
            sreset(ctx);
        }
        if (snap && e == 2 + half) {
            if (sload(ctx, snap) != WASTE_OK) { fprintf(stderr, "state load failed\n"); return 1; }
            tok = tok_saved;
        }
        const double t0 = now_ms();
        st = (e == 0 || again) ? weval(ctx, prompt, (size_t)np, &lg, &vocab)
                               : weval(ctx, &tok, 1, &lg, &vocab);
        const double dt = now_ms() - t0;
        if (st != WASTE_OK) {
            fprintf(stderr, "waste_eval %d: %d (%s)\n", e, (int)st,
                    detail && detail(ctx) ? detail(ctx) : "");
            return 1;
        }
        tok = argmax(lg, vocab);
        fwrite(&tok, 4, 1, out);
        fwrite(lg, sizeof(float), vocab, out);
        printf("eval %d: next token %d (%.3f ms)\n", e, tok, dt);
    }
    /* the CUDA backend's own count of its kernel launches, when the engine
     * links it (a dependency of the patched engine library) */
    uint64_t (*launches)(void) = (uint64_t (*)(void))dlsym(h, "waste_cuda_launch_count");
    if (launches) printf("cuda launches: %llu\n", (unsigned long long)launches());
    /* the engine's own phase timers (WASTE_PROFILE=1), per eval over the
     * evals from prof_from on */
    if (prof && prof_n && getenv("WASTE_PROFILE")) {
        static const char *names[] = { "lutb", "kda", "mla", "moe", "expert_read",
                                       "expert_mm", "head", "lut_apply", "matmul" };
        const int ne = nev - prof_from;
        for (int i = 0; i < 9; i++)
            if (prof_n[i] > prof0_n[i])
                printf("prof %s: %.3f ms per eval in %llu calls (evals %d..%d)\n", names[i],
                       (prof[i] - prof0[i]) * 1e3 / ne,
                       (unsigned long long)(prof_n[i] - prof0_n[i]), prof_from, nev - 1);
    }
    vocab32 = (int32_t)vocab;
    fseek(out, 4, SEEK_SET);
    fwrite(&vocab32, 4, 1, out);
    fclose(out);
    wclose(ctx);
    free(prompt);
    return 0;
}
