/*
 * ref_harness.c - exposes the reference engine's file-static hot-path
 * routines so tests and the CPU baseline can call the reference itself.
 *
 * TEST INFRASTRUCTURE ONLY. Built by oracle/Makefile into oracle/_ref/
 * straight from the reference's own sources (this TU #includes
 * src/dsv4/dsv4_model.c where it lies); nothing of the reference is copied.
 * The product library never links this.
 */
#include "dsv4_model.c"

#define REF_API __attribute__((visibility("default")))

/* A zeroed model with just the fields the compute routines read. */
static void ref_model_init(DSV4Model *m, int hid, int mi, int ne, int topk,
                           int limit)
{
    memset(m, 0, sizeof(*m));
    m->cfg.hidden = hid;
    m->cfg.moe_inter = mi;
    m->cfg.n_experts = ne;
    m->cfg.topk = topk;
    m->cfg.swiglu_limit = (float)limit;
    const size_t stride = (size_t)4 * mi + (mi + 127) / 128;
    m->expert_work = (float *)calloc((size_t)(DSV4_MAX_TOPK + 2) * stride,
                                     sizeof(float));
}

static void ref_model_fini(DSV4Model *m) { free(m->expert_work); }

/* sparse_attn (src/dsv4/dsv4_model.c:5767), OpenMP over heads. */
REF_API void ref_sparse_attn(float *o, const float *q, const float *kv,
                             const float *sink, const int *idx, int n, int H,
                             int d, float scale)
{
    DSV4Model m;
    memset(&m, 0, sizeof(m));
    sparse_attn(&m, o, q, kv, sink, idx, n, H, d, scale);
}

/* routed_swiglu_quant (src/dsv4/dsv4_model.c:6239). */
REF_API void ref_routed_swiglu_quant(float *y, float *qy, float *qscale,
                                     const float *gate, const float *up,
                                     int n, int limit, float route_weight)
{
    routed_swiglu_quant(y, qy, qscale, gate, up, n, limit, route_weight);
}

REF_API float ref_sqrt_softplus(float z) { return sqrt_softplus(z); }

REF_API void ref_sqrt_softplus_many(const float *z, float *s, int n)
{
    for (int i = 0; i < n; i++) s[i] = sqrt_softplus(z[i]);
}

/* Expert slot layout used by the reference's cache (dsv4_internal.h:13-16,
 * :33-37): scale run [w1][w2][w3], weight run [w1][w2][w3]. */
REF_API void ref_expert_slot_pack(uint8_t *scales, uint8_t *weights,
                                  const uint8_t *w1, const uint8_t *s1,
                                  const uint8_t *w2, const uint8_t *s2,
                                  const uint8_t *w3, const uint8_t *s3,
                                  int hid, int mi)
{
    const size_t w13 = (size_t)mi * ((hid + 1) / 2), w2n = (size_t)hid * ((mi + 1) / 2);
    const size_t s13 = (size_t)mi * ((hid + 31) / 32), s2n = (size_t)hid * ((mi + 31) / 32);
    memcpy(weights, w1, w13);
    memcpy(weights + w13, w2, w2n);
    memcpy(weights + w13 + w2n, w3, w13);
    memcpy(scales, s1, s13);
    memcpy(scales + s13, s2, s2n);
    memcpy(scales + s13 + s2n, s3, s13);
}

/* expert_forward (src/dsv4/dsv4_model.c:6338) on a packed slot. */
REF_API void ref_expert_forward(float *out, const float *qx, const float *qsc,
                                const uint8_t *slot_scales,
                                const uint8_t *slot_weights, int hid, int mi,
                                int limit, float weight)
{
    DSV4Model m;
    ref_model_init(&m, hid, mi, 1, 1, limit);
    DSV4ExpertSlot s;
    memset(&s, 0, sizeof(s));
    s.scales = (uint8_t *)slot_scales;
    s.weights = (uint8_t *)slot_weights;
    DSV4ExpertWork work;
    bind_expert_work(&m, &work, 0);
    expert_forward(&m, &s, qx, qsc, &work, weight, 0, 0, out);
    ref_model_fini(&m);
}

/* shared_expert_forward (src/dsv4/dsv4_model.c:6399), FP8 weights. */
REF_API void ref_shared_expert_forward(float *out, const float *qx,
                                       const float *qsc, const uint8_t *w1,
                                       const uint8_t *s1, const uint8_t *w3,
                                       const uint8_t *s3, const uint8_t *w2,
                                       const uint8_t *s2, int hid, int mi,
                                       int limit)
{
    DSV4Model m;
    ref_model_init(&m, hid, mi, 1, 1, limit);
    DSV4LayerW w;
    memset(&w, 0, sizeof(w));
    w.sh1 = w1; w.sh1_s = s1; w.sh3 = w3; w.sh3_s = s3; w.sh2 = w2; w.sh2_s = s2;
    DSV4ExpertWork work;
    bind_expert_work(&m, &work, 0);
    shared_expert_forward(&m, &w, qx, qsc, &work, 0, out);
    ref_model_fini(&m);
}

/* One token through one MoE layer with every expert resident: the compute
 * sequence of moe_forward (src/dsv4/dsv4_model.c:6599-6807) with the
 * disk-cache plumbing (expert_batch_begin and friends) left out. Routing
 * glue is restated; every kernel called is the reference's own. */
REF_API void ref_moe_forward(float *out, int *idx_out, float *wt_out,
                             const float *x, int token_id,
                             const uint16_t *gate_w, const float *bias,
                             const int64_t *tid2eid,
                             const uint8_t *const *slot_scales,
                             const uint8_t *const *slot_weights,
                             const uint8_t *sh1, const uint8_t *sh1_s,
                             const uint8_t *sh3, const uint8_t *sh3_s,
                             const uint8_t *sh2, const uint8_t *sh2_s,
                             int hid, int mi, int ne, int topk, int limit,
                             float route_scale)
{
    DSV4Model m;
    ref_model_init(&m, hid, mi, ne, topk, limit);
    float *score = (float *)malloc((size_t)ne * sizeof(float));
    float *choice = (float *)malloc((size_t)ne * sizeof(float));
    float *qx = (float *)malloc((size_t)hid * sizeof(float));
    float *qsc = (float *)malloc((size_t)((hid + 127) / 128) * sizeof(float));
    float *routed = (float *)malloc((size_t)topk * hid * sizeof(float));
    float *shared = (float *)calloc((size_t)hid, sizeof(float));
    int idx[DSV4_MAX_TOPK], order[DSV4_MAX_TOPK];
    float wt[DSV4_MAX_TOPK];

    dsv4_gemv_bf16(score, x, gate_w, hid, ne, 0);
    for (int e = 0; e < ne; e++) score[e] = sqrt_softplus(score[e]);
    for (int e = 0; e < ne; e++) choice[e] = score[e] + (bias ? bias[e] : 0.0f);
    if (tid2eid) {
        for (int k = 0; k < topk; k++) idx[k] = order[k] = (int)tid2eid[(size_t)token_id * topk + k];
    } else {
        for (int k = 0; k < topk; k++) {
            int best = -1;
            float bv = -INFINITY;
            for (int e = 0; e < ne; e++) {
                int used = 0;
                for (int t = 0; t < k; t++) if (order[t] == e) { used = 1; break; }
                if (!used && choice[e] > bv) { bv = choice[e]; best = e; }
            }
            order[k] = idx[k] = best;
        }
    }
    float sum = 0.0f;
    for (int k = 0; k < topk; k++) sum += score[idx[k]];
    if (sum > 0.0f) {
        float rs = route_scale / sum;
        for (int k = 0; k < topk; k++) wt[k] = score[idx[k]] * rs;
    } else {
        for (int k = 0; k < topk; k++) wt[k] = 0.0f;
    }
    for (int i = 0; i < topk; i++)
        for (int j = i + 1; j < topk; j++)
            if (idx[j] < idx[i]) {
                int ti = idx[i]; idx[i] = idx[j]; idx[j] = ti;
                float tw = wt[i]; wt[i] = wt[j]; wt[j] = tw;
            }

    dsv4_quant_fp8_codes(qx, qsc, x, hid);
    DSV4ExpertWork work;
    bind_expert_work(&m, &work, 0);
    for (int k = 0; k < topk; k++) {
        DSV4ExpertSlot s;
        memset(&s, 0, sizeof(s));
        s.scales = (uint8_t *)slot_scales[idx[k]];
        s.weights = (uint8_t *)slot_weights[idx[k]];
        expert_forward(&m, &s, qx, qsc, &work, wt[k], idx[k], 0,
                       routed + (size_t)k * hid);
    }
    if (sh1) {
        DSV4LayerW w;
        memset(&w, 0, sizeof(w));
        w.sh1 = sh1; w.sh1_s = sh1_s; w.sh3 = sh3; w.sh3_s = sh3_s;
        w.sh2 = sh2; w.sh2_s = sh2_s;
        shared_expert_forward(&m, &w, qx, qsc, &work, 0, shared);
    }
    float *acc = (float *)calloc((size_t)hid, sizeof(float));
    for (int k = 0; k < topk; k++)
        for (int i = 0; i < hid; i++) acc[i] += routed[(size_t)k * hid + i];
    for (int i = 0; i < hid; i++) acc[i] += shared[i];
    round_bf16_vec(acc, hid);
    memcpy(out, acc, (size_t)hid * sizeof(float));
    if (idx_out) memcpy(idx_out, idx, (size_t)topk * sizeof(int));
    if (wt_out) memcpy(wt_out, wt, (size_t)topk * sizeof(float));
    free(acc); free(score); free(choice); free(qx); free(qsc); free(routed);
    free(shared);
    ref_model_fini(&m);
}

REF_API int ref_omp_max_threads(void)
{
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* Threads of the next OpenMP teams (launchers such as torchrun pre-set
 * OMP_NUM_THREADS=1 in the environment); returns the new maximum. */
REF_API int ref_omp_set_threads(int n)
{
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
    return omp_get_max_threads();
#else
    (void)n;
    return 1;
#endif
}

/* dsv4_rope_apply_buf_inv (src/dsv4/dsv4_model.c:1569). */
REF_API void ref_rope_inv(float *x, int heads, int head_dim, float *cosv,
                          float *sinv, int n)
{
    DSV4RopeFreq f;
    f.cosv = cosv;
    f.sinv = sinv;
    f.n = n;
    dsv4_rope_apply_buf_inv(x, heads, head_dim, &f);
}
