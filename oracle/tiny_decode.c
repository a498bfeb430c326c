/*
 * tiny_decode.c - greedy decode through the reference engine's public API
 * (include/dsv4/dsv4.h: dsv4_model_open :152, dsv4_prefill :166,
 * dsv4_forward_token :161), for the tiny-model parity checks.
 *
 *   tiny_decode <checkpoint dir> <n_generate> <prompt id> [<prompt id> ...]
 *
 * TINY_DECODE_THREADS sets the engine's thread count (default 2).
 *
 * Prefills the prompt layer-major, then decodes n_generate tokens greedily
 * (argmax, lowest id on ties, as the reference CLI's argmax_logits,
 * src/cli/dsv4_run.c:355). Prints one line per generated position,
 * "POS <position> TOK <token> LOGITS <hex float> ...", every logit as %a so
 * two runs can be compared bit for bit.
 *
 * TEST INFRASTRUCTURE ONLY: it links the reference engine compiled from its
 * own sources (oracle/Makefile). Run plainly it is the reference; run with
 * libdsv4_cuda.so preloaded, the engine's kernel calls resolve to the GPU
 * drop-ins instead.
 */
#include <stdio.h>
#include <stdlib.h>

#include "dsv4.h"

static int argmax(const float *v, int n)
{
    int best = 0;
    for (int i = 1; i < n; i++)
        if (v[i] > v[best]) best = i;
    return best;
}

static void emit(int pos, int tok, const float *logits, int vocab)
{
    printf("POS %d TOK %d LOGITS", pos, tok);
    for (int i = 0; i < vocab; i++) printf(" %a", (double)logits[i]);
    printf("\n");
}

int main(int argc, char **argv)
{
    if (argc < 4) {
        fprintf(stderr, "usage: %s <dir> <n_generate> <prompt ids...>\n", argv[0]);
        return 2;
    }
    const int n_gen = atoi(argv[2]);
    const int n_prompt = argc - 3;
    int *ids = (int *)malloc(sizeof(int) * (size_t)n_prompt);
    for (int i = 0; i < n_prompt; i++) ids[i] = atoi(argv[3 + i]);

    DSV4Options opt = {0};
    opt.max_context = n_prompt + n_gen + 8;
    const char *th = getenv("TINY_DECODE_THREADS");
    opt.threads = th && atoi(th) > 0 ? atoi(th) : 2;
    opt.expert_cache_bytes = 64ull * (13369344ull + 4 * 4096ull);
    DSV4Model *m = dsv4_model_open(argv[1], &opt);
    if (!m) { fprintf(stderr, "FAIL: model open\n"); return 1; }
    const DSV4Config *cfg = dsv4_model_config(m);
    const int vocab = cfg->vocab;
    float *logits = (float *)malloc(sizeof(float) * (size_t)vocab);

    if (dsv4_prefill(m, ids, n_prompt, 0, logits) != 0) {
        fprintf(stderr, "FAIL: prefill\n");
        return 1;
    }
    int pos = n_prompt;
    for (int g = 0; g < n_gen; g++) {
        const int tok = argmax(logits, vocab);
        emit(pos, tok, logits, vocab);
        if (g + 1 == n_gen) break;
        if (dsv4_forward_token(m, tok, pos, logits) != 0) {
            fprintf(stderr, "FAIL: forward at %d\n", pos);
            return 1;
        }
        pos++;
    }
    fflush(stdout);
    dsv4_model_close(m);
    free(logits);
    free(ids);
    return 0;
}
