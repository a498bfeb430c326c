/*
 * ref_decode_bench.c - times the reference engine's own decode step
 * (dsv4_forward_token, src/dsv4/dsv4_model.c:8388) on the host cores, for
 * the CPU baseline of the whole-model decode benchmark.
 *
 *   ref_decode_bench <checkpoint dir> <warmup tokens> <timed tokens> <threads>
 *
 * Greedy decode from token 1 at position 0; after the warm-up every expert
 * the route touches is resident in the engine's RAM cache (the cache is
 * sized for all of them), so the timed tokens measure compute from RAM, not
 * disk streaming. Prints one line:
 *   RESULT layers <n> tokens <k> total_s <t> head_s <h> embed_s <e>
 * with the engine's own profile accumulators (DSV4_PROFILE), so a caller can
 * split the per-layer cost from the vocab head and extrapolate to a deeper
 * model of the same layer shape.
 *
 * TEST/BENCH INFRASTRUCTURE ONLY: built by oracle/Makefile from the
 * reference's sources; the product library never links it.
 */
#include <stdio.h>
#include <stdlib.h>
#include <time.h>

#include "dsv4.h"
#include "dsv4_internal.h"

static double now_s(void)
{
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return (double)ts.tv_sec + 1e-9 * (double)ts.tv_nsec;
}

static int argmax(const float *v, int n)
{
    int best = 0;
    for (int i = 1; i < n; i++)
        if (v[i] > v[best]) best = i;
    return best;
}

int main(int argc, char **argv)
{
    if (argc < 5) {
        fprintf(stderr, "usage: %s <dir> <warmup> <timed> <threads>\n", argv[0]);
        return 2;
    }
    const int warm = atoi(argv[2]), timed = atoi(argv[3]), threads = atoi(argv[4]);
    setenv("DSV4_PROFILE", "1", 1);
    DSV4Options opt = {0};
    opt.max_context = warm + timed + 8;
    opt.threads = threads;
    opt.expert_cache_bytes = 300ull * (13369344ull + 4 * 4096ull);
    DSV4Model *m = dsv4_model_open(argv[1], &opt);
    if (!m) { fprintf(stderr, "FAIL: model open\n"); return 1; }
    const int vocab = dsv4_model_config(m)->vocab;
    float *logits = (float *)malloc(sizeof(float) * (size_t)vocab);
    int tok = 1, pos = 0;
    for (int i = 0; i < warm; i++, pos++) {
        if (dsv4_forward_token(m, tok, pos, logits) != 0) return 1;
        tok = argmax(logits, vocab);
    }
    const double h0 = m->time_head, e0 = m->time_embed;
    const double t0 = now_s();
    for (int i = 0; i < timed; i++, pos++) {
        if (dsv4_forward_token(m, tok, pos, logits) != 0) return 1;
        tok = argmax(logits, vocab);
    }
    const double t1 = now_s();
    printf("RESULT layers %d tokens %d total_s %.6f head_s %.6f embed_s %.6f\n",
           dsv4_model_config(m)->n_layers, timed, t1 - t0, m->time_head - h0,
           m->time_embed - e0);
    dsv4_model_close(m);
    free(logits);
    return 0;
}
