/*
 * dsv4_oracle.c - CPU restatement of the reference engine's decode hot-path
 * numerics. TEST INFRASTRUCTURE ONLY (the checker; see dsv4_oracle.h).
 *
 * Build with -ffp-contract=off: the reference is compiled that way
 * (GNUmakefile:48), so a*b+c is two roundings unless fmaf() is written.
 * Citations are file:line inside the reference project.
 */
#include "dsv4_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#define ORC_FP8_BLOCK 128   /* src/dsv4/dsv4_internal.h:28 */
#define ORC_FP4_GROUP 32    /* src/dsv4/dsv4_internal.h:29 */
#define ORC_MAX_TOPK 32     /* include/dsv4/dsv4.h:54 */

/* ------------------------------------------------------------ codecs -- */

/* src/dsv4/dsv4_ops.c:35 - round to nearest even by the carry trick. */
uint16_t orc_f32_to_bf16(float f)
{
    uint32_t u;
    memcpy(&u, &f, 4);
    u += 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

static float bf16_widen(uint16_t h)
{
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* src/dsv4/dsv4_internal.h:254 (f32bf) */
float orc_bf16r(float f) { return bf16_widen(orc_f32_to_bf16(f)); }

/* src/dsv4/dsv4_ops.c:47 */
float orc_e4m3(uint8_t code)
{
    int exp = (code >> 3) & 15, man = code & 7;
    float mag;
    if (exp == 0)
        mag = ldexpf((float)man, -9);
    else if (exp == 15 && man == 7)
        mag = NAN;
    else
        mag = ldexpf((float)(8 + man), exp - 10);
    return (code & 0x80) ? -mag : mag;
}

/* src/dsv4/dsv4_ops.c:63 - code 255 is NaN (the header's "+inf" is stale). */
float orc_e8m0(uint8_t code)
{
    if (code == 255) return NAN;
    return ldexpf(1.0f, (int)code - 127);
}

/* src/dsv4/dsv4_ops.c:81 */
static float rne_half(float x)
{
    float lo = floorf(x);
    float frac = x - lo;
    if (frac > 0.5f) return lo + 1.0f;
    if (frac < 0.5f) return lo;
    return (fmodf(lo, 2.0f) == 0.0f) ? lo : lo + 1.0f;
}

/* src/dsv4/dsv4_ops.c:92 */
float orc_round_e4m3(float v)
{
    if (v == 0.0f) return 0.0f;
    float av = fabsf(v);
    float sgn = v < 0 ? -1.0f : 1.0f;
    int e;
    float m = frexpf(av, &e);
    if (e >= -5) {
        float mr = rne_half(m * 16.0f) / 16.0f;
        if (mr >= 1.0f) { mr = 0.5f; e++; }
        if (e - 1 > 8) return sgn * 448.0f;
        return sgn * mr * ldexpf(1.0f, e);
    }
    return sgn * (rne_half(av * 512.0f) / 512.0f);
}

/* ceil(log2(amax/448)) as used by every activation quantiser
 * (src/dsv4/dsv4_model.c:5591-5596). */
static float pow2_scale_448(float amax)
{
    if (amax < 1e-4f) amax = 1e-4f;
    float r = amax * (1.0f / 448.0f);
    int e;
    float m = frexpf(r, &e);
    if (m == 0.5f) e--;
    return ldexpf(1.0f, e);
}

/* ------------------------------------------------------------- quant -- */

/* src/dsv4/dsv4_model.c:5580 (dsv4_quant_fp8_codes); identical arithmetic to
 * the public dsv4_quant_fp8_act (src/dsv4/dsv4_ops.c:122). */
void orc_quant_fp8_codes(float *qx, float *qscale, const float *x, int n)
{
    for (int g = 0; g * ORC_FP8_BLOCK < n; g++) {
        int base = g * ORC_FP8_BLOCK;
        int len = n - base < ORC_FP8_BLOCK ? n - base : ORC_FP8_BLOCK;
        float amax = 0.0f;
        for (int i = 0; i < len; i++) {
            float a = fabsf(x[base + i]);
            if (a > amax) amax = a;
        }
        float scale = pow2_scale_448(amax);
        qscale[g] = scale;
        float inv = 1.0f / scale;
        for (int i = 0; i < len; i++) {
            float q = x[base + i] * inv;
            if (q > 448.0f) q = 448.0f;
            else if (q < -448.0f) q = -448.0f;
            qx[base + i] = orc_round_e4m3(q);
        }
    }
}

/* src/dsv4/dsv4_model.c:1386 (dsv4_act_quant_inplace). mode 0 = BF16
 * storage, 1 = E4M3 re-round, 2 = raw dequant. */
void orc_act_quant_inplace(float *x, int n, int group, int mode)
{
    for (int g = 0; g * group < n; g++) {
        int base = g * group;
        int len = n - base < group ? n - base : group;
        float amax = 0.0f;
        for (int i = 0; i < len; i++) {
            float a = fabsf(x[base + i]);
            if (a > amax) amax = a;
        }
        float scale = pow2_scale_448(amax);
        float inv = 1.0f / scale;
        for (int i = 0; i < len; i++) {
            float q = x[base + i] * inv;
            if (q > 448.0f) q = 448.0f;
            else if (q < -448.0f) q = -448.0f;
            float dq = orc_round_e4m3(q) * scale;
            if (mode == 2) x[base + i] = dq;
            else if (mode == 1) x[base + i] = orc_round_e4m3(dq);
            else x[base + i] = orc_bf16r(dq);
        }
    }
}

/* ------------------------------------------------------------- GEMVs -- */

/* src/dsv4/dsv4_model.c:299-302: one fmaf chain per row, columns in order. */
void orc_gemv_bf16(float *y, const float *x, const uint16_t *W, int in, int out,
                   int round_out)
{
    for (int r = 0; r < out; r++) {
        const uint16_t *row = W + (size_t)r * in;
        float acc = 0.0f;
        for (int c = 0; c < in; c++) acc = fmaf(bf16_widen(row[c]), x[c], acc);
        y[r] = round_out ? orc_bf16r(acc) : acc;
    }
}

/* src/dsv4/dsv4_model.c:308 - every token keeps the single-token chain. */
void orc_gemv_bf16_batch(float *const *y, const float *const *x, int batch,
                         const uint16_t *W, int in, int out, int round_out)
{
    for (int t = 0; t < batch; t++) orc_gemv_bf16(y[t], x[t], W, in, out, round_out);
}

/* src/dsv4/dsv4_model.c:657-672: 128-column fmaf partial, then
 * acc = fmaf(partial, qscale*ws, acc); a NaN block scale skips the block. */
void orc_gemv_fp8_q(float *y, const float *qx, const float *qscale,
                    const uint8_t *W, const uint8_t *wscale_code, int in,
                    int out, int round_out)
{
    const int cblocks = (in + ORC_FP8_BLOCK - 1) / ORC_FP8_BLOCK;
    for (int r = 0; r < out; r++) {
        const uint8_t *row = W + (size_t)r * in;
        const uint8_t *srow = wscale_code + (size_t)(r / ORC_FP8_BLOCK) * cblocks;
        float acc = 0.0f;
        for (int cb = 0; cb < cblocks; cb++) {
            int c1 = (cb + 1) * ORC_FP8_BLOCK < in ? (cb + 1) * ORC_FP8_BLOCK : in;
            float partial = 0.0f;
            for (int c = cb * ORC_FP8_BLOCK; c < c1; c++)
                partial = fmaf(orc_e4m3(row[c]), qx[c], partial);
            float ws = orc_e8m0(srow[cb]);
            if (!isnan(ws)) acc = fmaf(partial, qscale[cb] * ws, acc);
        }
        y[r] = round_out ? orc_bf16r(acc) : acc;
    }
}

/* src/dsv4/dsv4_model.c:678 */
void orc_gemv_fp8_batch_q(float *const *y, const float *const *qx,
                          const float *const *qscale, int batch,
                          const uint8_t *W, const uint8_t *wscale_code,
                          int in, int out, int round_out)
{
    for (int t = 0; t < batch; t++)
        orc_gemv_fp8_q(y[t], qx[t], qscale[t], W, wscale_code, in, out, round_out);
}

/* src/dsv4/dsv4_model.c:809 - both outputs BF16-rounded. */
void orc_gemv_fp8_pair_q(float *y0, float *y1, const float *qx,
                         const float *qscale, const uint8_t *W0,
                         const uint8_t *S0, const uint8_t *W1,
                         const uint8_t *S1, int in, int out)
{
    orc_gemv_fp8_q(y0, qx, qscale, W0, S0, in, out, 1);
    orc_gemv_fp8_q(y1, qx, qscale, W1, S1, in, out, 1);
}

static const float k_e2m1[16] = {
    0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f,
    -0.0f, -0.5f, -1.0f, -1.5f, -2.0f, -3.0f, -4.0f, -6.0f
};

/* src/dsv4/dsv4_model.c:1055-1073: 32-column fmaf partial (low nibble
 * first), acc = fmaf(partial, qscale[c0/128]*ws, acc), BF16 output. */
void orc_gemv_fp4_q(float *y, const float *qx, const float *qscale,
                    const uint8_t *W, const uint8_t *wscale_code, int in,
                    int rows)
{
    const int pcols = (in + 1) / 2;
    const int gcols = (in + ORC_FP4_GROUP - 1) / ORC_FP4_GROUP;
    for (int r = 0; r < rows; r++) {
        const uint8_t *row = W + (size_t)r * pcols;
        float acc = 0.0f;
        for (int g = 0; g < gcols; g++) {
            int c0 = g * ORC_FP4_GROUP;
            int c1 = c0 + ORC_FP4_GROUP < in ? c0 + ORC_FP4_GROUP : in;
            float partial = 0.0f;
            for (int c = c0; c < c1; c++) {
                uint8_t b = row[c >> 1];
                partial = fmaf(k_e2m1[(c & 1) ? (b >> 4) : (b & 15)], qx[c], partial);
            }
            float ws = orc_e8m0(wscale_code[(size_t)r * gcols + g]);
            if (!isnan(ws)) acc = fmaf(partial, qscale[c0 / 128] * ws, acc);
        }
        y[r] = orc_bf16r(acc);
    }
}

/* src/dsv4/dsv4_model.c:1080 */
void orc_gemv_fp4_batch_q(float *const *y, const float *const *qx,
                          const float *const *qscale, int batch,
                          const uint8_t *W, const uint8_t *wscale_code,
                          int in, int rows)
{
    for (int t = 0; t < batch; t++)
        orc_gemv_fp4_q(y[t], qx[t], qscale[t], W, wscale_code, in, rows);
}

/* src/dsv4/dsv4_model.c:1220 */
void orc_gemv_fp4_pair_q(float *y0, float *y1, const float *qx,
                         const float *qscale, const uint8_t *W0,
                         const uint8_t *S0, const uint8_t *W1,
                         const uint8_t *S1, int in, int rows)
{
    orc_gemv_fp4_q(y0, qx, qscale, W0, S0, in, rows);
    orc_gemv_fp4_q(y1, qx, qscale, W1, S1, in, rows);
}

/* --------------------------------------------------------------- MoE -- */

/* src/dsv4/dsv4_model.c:5827 */
float orc_sqrt_softplus(float z)
{
    if (z > 20.0f) return sqrtf(z);
    return sqrtf(log1pf(expf(z)));
}

/* Strict ">" over ascending ids from -inf; a tie keeps the lower id
 * (src/dsv4/dsv4_model.c:6636-6646). */
static void select_topk(int *order, const float *choice, int n, int k)
{
    for (int j = 0; j < k; j++) {
        int best = -1;
        float bv = -INFINITY;
        for (int e = 0; e < n; e++) {
            int used = 0;
            for (int t = 0; t < j; t++) if (order[t] == e) { used = 1; break; }
            if (!used && choice[e] > bv) { bv = choice[e]; best = e; }
        }
        order[j] = best;
    }
}

/* Exchange sort by ascending id, carrying weights
 * (src/dsv4/dsv4_model.c:6669-6676). */
static void sort_by_id(int *idx, float *wt, int k)
{
    for (int i = 0; i < k; i++)
        for (int j = i + 1; j < k; j++)
            if (idx[j] < idx[i]) {
                int ti = idx[i]; idx[i] = idx[j]; idx[j] = ti;
                float tw = wt[i]; wt[i] = wt[j]; wt[j] = tw;
            }
}

/* Router exactly as moe_forward runs it: src/dsv4/dsv4_model.c:6615-6676. */
void orc_router_moe(int *idx, float *wt, float *score_out, const float *x,
                    const uint16_t *gate, const float *bias,
                    const int64_t *tid2eid, int token_id, int hidden,
                    int n_experts, int topk, float route_scale)
{
    float *score = (float *)malloc((size_t)n_experts * sizeof(float));
    float *choice = (float *)malloc((size_t)n_experts * sizeof(float));
    orc_gemv_bf16(score, x, gate, hidden, n_experts, 0);
    for (int e = 0; e < n_experts; e++) score[e] = orc_sqrt_softplus(score[e]);
    for (int e = 0; e < n_experts; e++)
        choice[e] = score[e] + (bias ? bias[e] : 0.0f);
    if (tid2eid) {
        for (int k = 0; k < topk; k++)
            idx[k] = (int)tid2eid[(size_t)token_id * topk + k];
    } else {
        select_topk(idx, choice, n_experts, topk);
    }
    float sum = 0.0f;
    for (int k = 0; k < topk; k++) sum += score[idx[k]];
    if (sum > 0.0f) {
        float rs = route_scale / sum;
        for (int k = 0; k < topk; k++) wt[k] = score[idx[k]] * rs;
    } else {
        for (int k = 0; k < topk; k++) wt[k] = 0.0f;
    }
    sort_by_id(idx, wt, topk);
    if (score_out) memcpy(score_out, score, (size_t)n_experts * sizeof(float));
    free(score);
    free(choice);
}

/* Public dsv4_router: src/dsv4/dsv4_ops.c:473-545. The dot product is a
 * separate multiply then add (no fmaf), and the weights are
 * score * (1/sum) * route_scale. */
void orc_router_public(int *idx, float *wt, const float *x,
                       const uint16_t *gate, const float *bias,
                       const int64_t *tid2eid, int token_id, int hidden,
                       int n_experts, int topk, int hash_layer,
                       float route_scale)
{
    float *score = (float *)calloc((size_t)n_experts, sizeof(float));
    float *choice = (float *)calloc((size_t)n_experts, sizeof(float));
    int order[ORC_MAX_TOPK];
    if (hash_layer) {
        for (int k = 0; k < topk; k++) {
            int e = (int)tid2eid[(size_t)token_id * topk + k];
            order[k] = e;
            const uint16_t *row = gate + (size_t)e * hidden;
            float z = 0.0f;
            for (int i = 0; i < hidden; i++) {
                float p = bf16_widen(row[i]) * x[i];
                z = z + p;
            }
            score[e] = orc_sqrt_softplus(z);
        }
    } else {
        for (int e = 0; e < n_experts; e++) {
            const uint16_t *row = gate + (size_t)e * hidden;
            float z = 0.0f;
            for (int i = 0; i < hidden; i++) {
                float p = bf16_widen(row[i]) * x[i];
                z = z + p;
            }
            score[e] = orc_sqrt_softplus(z);
            choice[e] = score[e] + (bias ? bias[e] : 0.0f);
        }
        select_topk(order, choice, n_experts, topk);
    }
    float sum = 0.0f;
    for (int k = 0; k < topk; k++) sum += score[order[k]];
    float inv = sum > 0.0f ? 1.0f / sum : 0.0f;
    for (int k = 0; k < topk; k++) wt[k] = score[order[k]] * inv * route_scale;
    sort_by_id(order, wt, topk);
    for (int k = 0; k < topk; k++) idx[k] = order[k];
    free(score);
    free(choice);
}

/* Fused SwiGLU + BF16 + FP8 quant: src/dsv4/dsv4_model.c:6257-6286. The
 * shared expert's unfused form (:6416-6426) is this with route_weight 1. */
void orc_swiglu_quant(float *y, float *qy, float *qscale, const float *gate,
                      const float *up, int n, int limit, float route_weight)
{
    const float L = (float)limit;
    for (int base = 0; base < n; base += ORC_FP8_BLOCK) {
        int len = n - base < ORC_FP8_BLOCK ? n - base : ORC_FP8_BLOCK;
        float amax = 0.0f;
        for (int i = 0; i < len; i++) {
            float g = gate[base + i], u = up[base + i];
            if (u > L) u = L;
            else if (u < -L) u = -L;
            if (g > L) g = L;
            float silu = g / (1.0f + expf(-g));
            float v = orc_bf16r(silu * u * route_weight);
            y[base + i] = v;
            if (fabsf(v) > amax) amax = fabsf(v);
        }
        float scale = pow2_scale_448(amax);
        qscale[base / ORC_FP8_BLOCK] = scale;
        float inv = 1.0f / scale;
        for (int i = 0; i < len; i++) {
            float q = y[base + i] * inv;
            if (q > 448.0f) q = 448.0f;
            else if (q < -448.0f) q = -448.0f;
            qy[base + i] = orc_round_e4m3(q);
        }
    }
}

/* src/dsv4/dsv4_model.c:6289-6345 (expert_forward_l1 + _l2). */
void orc_expert_forward_fp4(float *out, const float *qx, const float *qsc,
                            const OrcFp4Expert *e, int hid, int mi, int limit,
                            float weight)
{
    float *gate = (float *)malloc((size_t)mi * sizeof(float));
    float *up = (float *)malloc((size_t)mi * sizeof(float));
    float *y = (float *)malloc((size_t)mi * sizeof(float));
    float *qy = (float *)malloc((size_t)mi * sizeof(float));
    float *qys = (float *)malloc((size_t)((mi + 127) / 128) * sizeof(float));
    orc_gemv_fp4_pair_q(gate, up, qx, qsc, e->w1, e->s1, e->w3, e->s3, hid, mi);
    orc_swiglu_quant(y, qy, qys, gate, up, mi, limit, weight);
    orc_gemv_fp4_q(out, qy, qys, e->w2, e->s2, mi, hid);
    free(gate); free(up); free(y); free(qy); free(qys);
}

/* src/dsv4/dsv4_model.c:6399-6433 (shared_expert_forward). */
void orc_shared_forward_fp8(float *out, const float *qx, const float *qsc,
                            const OrcFp8Expert *e, int hid, int mi, int limit)
{
    float *gate = (float *)malloc((size_t)mi * sizeof(float));
    float *up = (float *)malloc((size_t)mi * sizeof(float));
    float *y = (float *)malloc((size_t)mi * sizeof(float));
    float *qy = (float *)malloc((size_t)mi * sizeof(float));
    float *qys = (float *)malloc((size_t)((mi + 127) / 128) * sizeof(float));
    orc_gemv_fp8_pair_q(gate, up, qx, qsc, e->w1, e->s1, e->w3, e->s3, hid, mi);
    orc_swiglu_quant(y, qy, qys, gate, up, mi, limit, 1.0f);
    orc_gemv_fp8_q(out, qy, qys, e->w2, e->s2, mi, hid, 1);
    free(gate); free(up); free(y); free(qy); free(qys);
}

/* One token through one MoE layer: src/dsv4/dsv4_model.c:6599-6807. Routed
 * outputs are summed in ascending expert-id order, then the shared output,
 * then one BF16 rounding (:6795-6805). */
void orc_moe_forward(float *out, int *idx_out, float *wt_out,
                     const OrcMoeLayer *L, const float *x, int token_id)
{
    const int hid = L->hidden, mi = L->moe_inter, topk = L->topk;
    int idx[ORC_MAX_TOPK];
    float wt[ORC_MAX_TOPK];
    orc_router_moe(idx, wt, NULL, x, L->gate_w, L->bias, L->tid2eid, token_id,
                   hid, L->n_experts, topk, L->route_scale);
    float *qx = (float *)malloc((size_t)hid * sizeof(float));
    float *qsc = (float *)malloc((size_t)((hid + 127) / 128) * sizeof(float));
    float *routed = (float *)malloc((size_t)topk * hid * sizeof(float));
    float *shared = (float *)calloc((size_t)hid, sizeof(float));
    orc_quant_fp8_codes(qx, qsc, x, hid);
    const size_t w13 = (size_t)mi * ((hid + 1) / 2), s13 = (size_t)mi * ((hid + 31) / 32);
    const size_t w2 = (size_t)hid * ((mi + 1) / 2), s2 = (size_t)hid * ((mi + 31) / 32);
    for (int k = 0; k < topk; k++) {
        const int e = idx[k];
        OrcFp4Expert ex = {
            L->w1 + (size_t)e * w13, L->s1 + (size_t)e * s13,
            L->w3 + (size_t)e * w13, L->s3 + (size_t)e * s13,
            L->w2 + (size_t)e * w2, L->s2 + (size_t)e * s2,
        };
        orc_expert_forward_fp4(routed + (size_t)k * hid, qx, qsc, &ex, hid, mi,
                               L->swiglu_limit, wt[k]);
    }
    if (L->has_shared) {
        if (L->shared_fp8)
            orc_shared_forward_fp8(shared, qx, qsc, &L->shared8, hid, mi,
                                   L->swiglu_limit);
        else
            orc_expert_forward_fp4(shared, qx, qsc, &L->shared4, hid, mi,
                                   L->swiglu_limit, 1.0f);
    }
    for (int i = 0; i < hid; i++) {
        float acc = 0.0f;
        for (int k = 0; k < topk; k++) acc += routed[(size_t)k * hid + i];
        if (L->has_shared) acc += shared[i];
        out[i] = orc_bf16r(acc);
    }
    if (idx_out) memcpy(idx_out, idx, (size_t)topk * sizeof(int));
    if (wt_out) memcpy(wt_out, wt, (size_t)topk * sizeof(float));
    free(qx); free(qsc); free(routed); free(shared);
}

/* --------------------------------------------------------- attention -- */

/* src/dsv4/dsv4_model.c:5767-5822. Per head: fmaf dot over all d dims,
 * times scale; max; den = expf(sink-m) + sum expf(s-m) in fp32; value weight
 * is the BF16-rounded expf; o = bf16(sum w*kv / den). idx < 0 is padding. */
void orc_sparse_attn(float *o, const float *q, const float *kv,
                     const float *attn_sink, const int *topk_idx,
                     int topk_total, int H, int d, float scale)
{
    const size_t n = (size_t)(topk_total > 0 ? topk_total : 1);
    float *s = (float *)malloc(n * sizeof(float));
    float *w = (float *)malloc(n * sizeof(float));
    for (int h = 0; h < H; h++) {
        const float *qh = q + (size_t)h * d;
        float mx = -INFINITY;
        for (int t = 0; t < topk_total; t++) {
            int id = topk_idx[t];
            float v = -INFINITY;
            if (id >= 0) {
                const float *kp = kv + (size_t)id * d;
                float dot = 0.0f;
                for (int i = 0; i < d; i++) dot = fmaf(qh[i], kp[i], dot);
                v = dot * scale;
            }
            s[t] = v;
            if (v > mx) mx = v;
        }
        float den = expf(attn_sink[h] - mx);
        for (int t = 0; t < topk_total; t++) {
            if (s[t] != -INFINITY) {
                float e = expf(s[t] - mx);
                w[t] = orc_bf16r(e);
                den += e;
            } else {
                w[t] = 0.0f;
            }
        }
        float *oh = o + (size_t)h * d;
        for (int i = 0; i < d; i++) oh[i] = 0.0f;
        for (int t = 0; t < topk_total; t++) {
            int id = topk_idx[t];
            if (id < 0) continue;
            const float *kp = kv + (size_t)id * d;
            for (int i = 0; i < d; i++) oh[i] = fmaf(w[t], kp[i], oh[i]);
        }
        for (int i = 0; i < d; i++) oh[i] = orc_bf16r(oh[i] / den);
    }
    free(s);
    free(w);
}

/* ----------------------------------------------------------- helpers -- */

/* xorshift64 (13, 7, 17) as in benchmarks/bench_dsv4_kernels.c:25-32.
 * mod == 0 stores the low byte; otherwise x % mod. Returns the new state. */
uint64_t orc_xorshift_fill_u8(uint8_t *dst, int64_t n, uint64_t state, int mod)
{
    for (int64_t i = 0; i < n; i++) {
        state ^= state << 13;
        state ^= state >> 7;
        state ^= state << 17;
        dst[i] = mod ? (uint8_t)(state % (uint64_t)mod) : (uint8_t)state;
    }
    return state;
}

/* Raw xorshift64 outputs, for generators that derive floats from them. */
uint64_t orc_xorshift_next_many(uint64_t *dst, int64_t n, uint64_t state)
{
    for (int64_t i = 0; i < n; i++) {
        state ^= state << 13;
        state ^= state >> 7;
        state ^= state << 17;
        dst[i] = state;
    }
    return state;
}

/* dsv4_rope_apply_buf_inv (src/dsv4/dsv4_model.c:1569-1580): pairs
 * (x0, x1) -> (bf16(x0 c + x1 s), bf16(-x0 s + x1 c)), no contraction. */
void orc_rope_inv(float *x, int heads, int head_dim, const float *cosv,
                  const float *sinv, int n)
{
    const int start = head_dim - 2 * n;
    for (int h = 0; h < heads; h++) {
        float *p = x + (size_t)h * head_dim + start;
        for (int i = 0; i < n; i++) {
            const float x0 = p[2 * i], x1 = p[2 * i + 1];
            const float c = cosv[i], s = sinv[i];
            const float a = x0 * c, b = x1 * s;
            const float e = -x0 * s, f = x1 * c;
            p[2 * i] = orc_bf16r(a + b);
            p[2 * i + 1] = orc_bf16r(e + f);
        }
    }
}

/* ------------------------------------------- speculative acceptance -- */

/* xorshift64 13/7/17 (src/cli/dsv4_run.c:248-254). */
uint64_t orc_rng_next(uint64_t *state)
{
    uint64_t x = *state;
    x ^= x << 13;
    x ^= x >> 7;
    x ^= x << 17;
    *state = x;
    return x;
}

/* First index of the maximum under strict ">" (src/cli/dsv4_run.c:355). */
int orc_argmax_logits(const float *logits, int vocab)
{
    int best = 0;
    for (int v = 1; v < vocab; v++)
        if (logits[v] > logits[best]) best = v;
    return best;
}

typedef struct { double w; int id; } OrcItem;

static int orc_item_desc(const void *ap, const void *bp)
{
    const OrcItem *a = (const OrcItem *)ap, *b = (const OrcItem *)bp;
    if (a->w > b->w) return -1;
    if (a->w < b->w) return 1;
    return (a->id > b->id) - (a->id < b->id);
}

/* Temperature softmax in double, a 53-bit uniform, optional nucleus cut
 * (src/cli/dsv4_run.c:308-353, comparator :80-87). */
int orc_sample_top_p(const float *logits, int vocab, double temperature,
                     double top_p, uint64_t *state)
{
    OrcItem *it = (OrcItem *)malloc((size_t)vocab * sizeof(OrcItem));
    double mx = logits[0];
    for (int v = 1; v < vocab; v++)
        if (logits[v] > mx) mx = logits[v];
    double total = 0.0;
    const double inv_t = temperature > 1e-5 ? 1.0 / temperature : 1e5;
    for (int v = 0; v < vocab; v++) {
        it[v].w = exp(((double)logits[v] - mx) * inv_t);
        it[v].id = v;
        total += it[v].w;
    }
    const double u = (double)(orc_rng_next(state) >> 11) * (1.0 / 9007199254740992.0);
    int r;
    if (top_p == 1.0) {
        const double target = u * total;
        double cum = 0.0;
        r = it[vocab - 1].id;
        for (int i = 0; i < vocab; i++) {
            cum += it[i].w;
            if (target < cum) { r = it[i].id; break; }
        }
    } else {
        qsort(it, (size_t)vocab, sizeof(*it), orc_item_desc);
        double kept = 0.0;
        int keep = vocab;
        const double thr = total * top_p;
        for (int i = 0; i < vocab; i++) {
            kept += it[i].w;
            if (kept >= thr) { keep = i + 1; break; }
        }
        const double target = u * kept;
        double cum = 0.0;
        r = it[keep - 1].id;
        for (int i = 0; i < keep; i++) {
            cum += it[i].w;
            if (target < cum) { r = it[i].id; break; }
        }
    }
    free(it);
    return r;
}

int orc_accept_chain(const int *proposal, int proposed, const float *logits, int vocab,
                     double temperature, double top_p, uint64_t *state, int eos_id,
                     int *tokens, int *n_commit, int *n_accepted, int *n_samples)
{
    int accepted = 0, correction = -1, samples = 0;
    while (accepted < proposed) {
        const float *row = logits + (size_t)accepted * vocab;
        int target;
        if (temperature == 0.0) target = orc_argmax_logits(row, vocab);
        else { target = orc_sample_top_p(row, vocab, temperature, top_p, state); samples++; }
        if (proposal[accepted] != target) { correction = target; break; }
        accepted++;
        if (target == eos_id) break;
    }
    int eos_at = -1;
    for (int i = 0; i < accepted; i++)
        if (proposal[i] == eos_id) { eos_at = i; break; }
    int n = 0;
    if (eos_at >= 0) {
        for (int i = 0; i <= eos_at; i++) tokens[n++] = proposal[i];
        *n_commit = eos_at + 1;
    } else if (accepted < proposed) {
        for (int i = 0; i < accepted; i++) tokens[n++] = proposal[i];
        tokens[n++] = correction;
        *n_commit = accepted + 1;
    } else {
        const float *row = logits + (size_t)proposed * vocab;
        int bonus;
        if (temperature == 0.0) bonus = orc_argmax_logits(row, vocab);
        else { bonus = orc_sample_top_p(row, vocab, temperature, top_p, state); samples++; }
        for (int i = 0; i < proposed; i++) tokens[n++] = proposal[i];
        tokens[n++] = bonus;
        *n_commit = proposed + 1;
    }
    *n_accepted = accepted;
    *n_samples = samples;
    return n;
}
