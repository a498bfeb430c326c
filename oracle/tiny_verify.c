/*
 * tiny_verify.c - the reference engine's batched speculative verify:
 * dsv4_prefill_capture with all_logits (src/dsv4/dsv4_model.c:8434-8529,
 * declared in src/dsv4/dsv4_internal.h:296), for the verify parity checks.
 *
 *   tiny_verify <checkpoint dir> <start> <n_rows> <id> ...   (start + n_rows ids)
 *
 * TINY_DECODE_THREADS sets the engine's thread count (default 2).
 *
 * Prefills ids[0 .. start) with dsv4_prefill (include/dsv4/dsv4.h:166), then
 * runs ids[start .. start + n_rows) through one dsv4_prefill_capture call
 * (the rows layer-major, every row's logits) and prints one line per row,
 * "ROW <r> POS <position> LOGITS <hex float> ...", every logit as %a so two
 * runs can be compared bit for bit.
 *
 * TEST INFRASTRUCTURE ONLY: it links the reference engine compiled from its
 * own sources (oracle/Makefile).
 */
#include <stdio.h>
#include <stdlib.h>

#include "dsv4.h"
#include "dsv4_internal.h"

int main(int argc, char **argv)
{
    if (argc < 5) {
        fprintf(stderr, "usage: %s <dir> <start> <n_rows> <ids...>\n", argv[0]);
        return 2;
    }
    const int start = atoi(argv[2]);
    const int n_rows = atoi(argv[3]);
    const int n_ids = argc - 4;
    if (start < 1 || n_rows < 1 || n_ids != start + n_rows) {
        fprintf(stderr, "need start >= 1, n_rows >= 1 and start + n_rows ids\n");
        return 2;
    }
    int *ids = (int *)malloc(sizeof(int) * (size_t)n_ids);
    for (int i = 0; i < n_ids; i++) ids[i] = atoi(argv[4 + i]);

    DSV4Options opt = {0};
    opt.max_context = n_ids + 8;
    const char *th = getenv("TINY_DECODE_THREADS");
    opt.threads = th && atoi(th) > 0 ? atoi(th) : 2;
    opt.expert_cache_bytes = 64ull * (13369344ull + 4 * 4096ull);
    DSV4Model *m = dsv4_model_open(argv[1], &opt);
    if (!m) { fprintf(stderr, "FAIL: model open\n"); return 1; }
    const int vocab = dsv4_model_config(m)->vocab;
    float *logits = (float *)malloc(sizeof(float) * (size_t)vocab * (size_t)n_rows);

    if (dsv4_prefill(m, ids, start, 0, logits) != 0) {
        fprintf(stderr, "FAIL: prefill\n");
        return 1;
    }
    if (dsv4_prefill_capture(m, ids + start, n_rows, start, NULL, logits, 0, NULL, NULL) != 0) {
        fprintf(stderr, "FAIL: prefill_capture\n");
        return 1;
    }
    for (int r = 0; r < n_rows; r++) {
        printf("ROW %d POS %d LOGITS", r, start + r);
        const float *row = logits + (size_t)r * vocab;
        for (int i = 0; i < vocab; i++) printf(" %a", (double)row[i]);
        printf("\n");
    }
    fflush(stdout);
    dsv4_model_close(m);
    free(logits);
    free(ids);
    return 0;
}
