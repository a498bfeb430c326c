/*
 * dsv4_oracle.h - CPU restatement of the DeepSeek-V4-Flash decode hot-path
 * numerics of the reference C engine (deepseek-v4-flash-0731-in-c).
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker for the CUDA path:
 * only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg load
 * it. The product (libdsv4_cuda.so) never links or calls it.
 *
 * Every routine restates one reference routine (cited file:line inside
 * dsv4_oracle.c) with the same operation order, the same fmaf / separate
 * multiply-add choices and the same BF16 rounding points, compiled with
 * -ffp-contract=off, so its results are bit-identical to the reference's
 * scalar path. Parity of this restatement is pinned two ways:
 *   - against the reference itself, compiled from its own sources into
 *     oracle/_ref/ (tests/test_oracle_vs_ref.py), and
 *   - against the reference's own known-answer values and benchmark
 *     checksums (tests/test_oracle_golden.py, tests/golden/).
 */
#ifndef DSV4_ORACLE_H
#define DSV4_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- scalar codecs ---- */
uint16_t orc_f32_to_bf16(float f);
float orc_bf16r(float f);
float orc_e4m3(uint8_t code);
float orc_e8m0(uint8_t code);
float orc_round_e4m3(float v);

/* ---- activation quantisation ---- */
void orc_quant_fp8_codes(float *qx, float *qscale, const float *x, int n);
void orc_act_quant_inplace(float *x, int n, int group, int mode);

/* ---- GEMVs (row-major weights, reference layouts) ---- */
void orc_gemv_bf16(float *y, const float *x, const uint16_t *W, int in, int out,
                   int round_out);
void orc_gemv_bf16_batch(float *const *y, const float *const *x, int batch,
                         const uint16_t *W, int in, int out, int round_out);
void orc_gemv_fp8_q(float *y, const float *qx, const float *qscale,
                    const uint8_t *W, const uint8_t *wscale_code, int in,
                    int out, int round_out);
void orc_gemv_fp8_batch_q(float *const *y, const float *const *qx,
                          const float *const *qscale, int batch,
                          const uint8_t *W, const uint8_t *wscale_code,
                          int in, int out, int round_out);
void orc_gemv_fp8_pair_q(float *y0, float *y1, const float *qx,
                         const float *qscale, const uint8_t *W0,
                         const uint8_t *S0, const uint8_t *W1,
                         const uint8_t *S1, int in, int out);
void orc_gemv_fp4_q(float *y, const float *qx, const float *qscale,
                    const uint8_t *W, const uint8_t *wscale_code, int in,
                    int rows);
void orc_gemv_fp4_batch_q(float *const *y, const float *const *qx,
                          const float *const *qscale, int batch,
                          const uint8_t *W, const uint8_t *wscale_code,
                          int in, int rows);
void orc_gemv_fp4_pair_q(float *y0, float *y1, const float *qx,
                         const float *qscale, const uint8_t *W0,
                         const uint8_t *S0, const uint8_t *W1,
                         const uint8_t *S1, int in, int rows);

/* ---- MoE pieces ---- */
float orc_sqrt_softplus(float z);
/* Router as moe_forward runs it: BF16 gate GEMV with fmaf chains, ids sorted
 * ascending, weights carried. tid2eid != NULL selects the hash path. */
void orc_router_moe(int *idx, float *wt, float *score_out, const float *x,
                    const uint16_t *gate, const float *bias,
                    const int64_t *tid2eid, int token_id, int hidden,
                    int n_experts, int topk, float route_scale);
/* The public dsv4_router() twin (separate multiply and add, 1/sum weights). */
void orc_router_public(int *idx, float *wt, const float *x,
                       const uint16_t *gate, const float *bias,
                       const int64_t *tid2eid, int token_id, int hidden,
                       int n_experts, int topk, int hash_layer,
                       float route_scale);
void orc_swiglu_quant(float *y, float *qy, float *qscale, const float *gate,
                      const float *up, int n, int limit, float route_weight);

/* Expert weight bundle: routed experts are FP4 (w1 gate, w3 up: [mi][hid/2]
 * with [mi][hid/32] E8M0; w2 down: [hid][mi/2] with [hid][mi/32]). */
typedef struct {
    const uint8_t *w1, *s1, *w3, *s3, *w2, *s2;
} OrcFp4Expert;
/* Shared expert in FP8 E4M3 with [128x128] E8M0 blocks. */
typedef struct {
    const uint8_t *w1, *s1, *w3, *s3, *w2, *s2;
} OrcFp8Expert;

void orc_expert_forward_fp4(float *out, const float *qx, const float *qsc,
                            const OrcFp4Expert *e, int hid, int mi, int limit,
                            float weight);
void orc_shared_forward_fp8(float *out, const float *qx, const float *qsc,
                            const OrcFp8Expert *e, int hid, int mi, int limit);

/* One MoE layer for one token (moe_forward). Routed expert e uses
 * w1 + e*w1_stride etc. (contiguous [E] arrays). shared_fp8 selects the
 * reference's FP8 shared expert; otherwise shared_fp4 (FP4, same layout as a
 * routed expert, weight 1.0). idx_out/wt_out (topk each) may be NULL. */
typedef struct {
    int hidden, moe_inter, n_experts, topk, swiglu_limit;
    float route_scale;
    const uint16_t *gate_w;     /* [E][H] BF16 */
    const float *bias;          /* [E] or NULL */
    const int64_t *tid2eid;     /* [vocab][topk] or NULL */
    const uint8_t *w1, *s1, *w3, *s3, *w2, *s2;   /* routed, expert-major */
    int has_shared, shared_fp8;
    OrcFp8Expert shared8;
    OrcFp4Expert shared4;
} OrcMoeLayer;

void orc_moe_forward(float *out, int *idx_out, float *wt_out,
                     const OrcMoeLayer *L, const float *x, int token_id);

/* ---- attention ---- */
void orc_sparse_attn(float *o, const float *q, const float *kv,
                     const float *attn_sink, const int *topk_idx,
                     int topk_total, int H, int d, float scale);
/* Inverse RoPE on the last 2n dims of each head
 * (dsv4_rope_apply_buf_inv, src/dsv4/dsv4_model.c:1569-1580). */
void orc_rope_inv(float *x, int heads, int head_dim, const float *cosv,
                  const float *sinv, int n);

/* ---- helpers for tests ---- */
/* ---- speculative acceptance (src/cli/dsv4_run.c) ---- */
uint64_t orc_rng_next(uint64_t *state);                       /* :248-254 */
int orc_argmax_logits(const float *logits, int vocab);        /* :355 */
int orc_sample_top_p(const float *logits, int vocab, double temperature,
                     double top_p, uint64_t *state);          /* :308-353 */
/* The verify-step acceptance of :951-1043 for one proposal of `proposed`
 * draft tokens against logits [(proposed + 1)][vocab]: emits the accepted
 * drafts and the correction or bonus token (or stops after eos_id). Returns
 * the number of emitted tokens; *n_commit = positions to keep (the
 * reference's snapshot commit length), *n_accepted, *n_samples = uniforms
 * consumed (T > 0). */
int orc_accept_chain(const int *proposal, int proposed, const float *logits, int vocab,
                     double temperature, double top_p, uint64_t *state, int eos_id,
                     int *tokens, int *n_commit, int *n_accepted, int *n_samples);

uint64_t orc_xorshift_fill_u8(uint8_t *dst, int64_t n, uint64_t state,
                              int mod);
uint64_t orc_xorshift_next_many(uint64_t *dst, int64_t n, uint64_t state);

#ifdef __cplusplus
}
#endif
#endif
