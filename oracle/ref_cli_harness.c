/* ref_cli_harness.c - exposes the reference CLI's static sampling and
 * speculative-acceptance helpers (src/cli/dsv4_run.c) for parity tests.
 * Test infrastructure only: compiled by oracle/Makefile into
 * oracle/_ref/libdsv4_refcli.so from the reference sources where they lie;
 * the CLI's main() is renamed so the file links as a library. */
#define main dsv4_cli_main_unused
#include "dsv4_run.c"
#undef main

#define REF_API __attribute__((visibility("default")))

/* rng_next (src/cli/dsv4_run.c:248-254) on caller-held state. */
REF_API uint64_t ref_rng_next(uint64_t *state)
{
    rng_state = *state;
    uint64_t v = rng_next();
    *state = rng_state;
    return v;
}

/* argmax_logits (src/cli/dsv4_run.c:355). */
REF_API int ref_argmax_logits(const float *logits, int vocab)
{
    return argmax_logits(logits, vocab);
}

/* sample_top_p (src/cli/dsv4_run.c:308-353) on caller-held rng state. */
REF_API int ref_sample_top_p(const float *logits, int vocab, double temperature,
                             double top_p, uint64_t *state)
{
    SampleItem *items = (SampleItem *)malloc((size_t)vocab * sizeof(SampleItem));
    if (!items) return -1;
    rng_state = *state;
    int r = sample_top_p(logits, vocab, temperature, top_p, items);
    *state = rng_state;
    free(items);
    return r;
}

/* ngram_draft (src/cli/dsv4_run.c:262-305). */
REF_API int ref_ngram_draft(const int *history, int n_history, int cap, int min_match,
                            int allow_overlap, int periodic_extend, int *out)
{
    return ngram_draft(history, n_history, cap, min_match, allow_overlap,
                       periodic_extend, out);
}
