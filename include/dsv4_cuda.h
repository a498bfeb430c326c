/*
 * dsv4_cuda.h - C ABI of libdsv4_cuda.so, the B200 (sm_100a) implementation
 * of the DeepSeek-V4-Flash decode hot path of deepseek-v4-flash-0731-in-c.
 *
 * Three layers, all plain C types (no torch, no C++ in the signatures):
 *
 *  1. Drop-in kernel symbols. Same names, signatures, argument meaning and
 *     error behaviour as the reference's kernel ABI, host pointers in and
 *     out; each call stages its operands through device memory and returns
 *     bit-identical results. A host program links (or LD_PRELOADs) this
 *     library in place of the reference's definitions. Every one is also
 *     exported with a dsv4cuda_ prefix so both can live in one process.
 *  2. Device-resident entry points (dsv4cuda_*): device pointers and a CUDA
 *     stream, int status (0 = ok, negative = error), never abort.
 *  3. Lifecycle and error reporting.
 *
 * Each drop-in declaration cites the reference interface it replaces as
 * path:line inside the reference project.
 */
#ifndef DSV4_CUDA_H
#define DSV4_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------ 1. drop-in kernel ABI --
 * Host pointers. Activations are floats on the E4M3 grid (qx) with one
 * power-of-two scale per 128 columns (qscale); weight scales are E8M0 codes.
 * A batch above 33 prints the reference's message and exits(1), as the
 * reference does; a CUDA failure prints "dsv4_cuda: ..." and exits(1) unless
 * dsv4cuda_set_abort_on_error(0) was called (then the error is recorded and
 * the outputs are left unspecified).
 */

/* src/dsv4/dsv4_internal.h:257 (defined src/dsv4/dsv4_model.c:266) */
void dsv4_gemv_bf16(float *y, const float *x, const uint16_t *W, int in, int out,
                    int round_out);
/* src/dsv4/dsv4_internal.h:259 (src/dsv4/dsv4_model.c:308) */
void dsv4_gemv_bf16_batch(float *const *y, const float *const *x, int batch,
                          const uint16_t *W, int in, int out, int round_out);
/* src/dsv4/dsv4_internal.h:263 (src/dsv4/dsv4_model.c:571) */
void dsv4_gemv_fp8_q(float *y, const float *qx, const float *qscale,
                     const uint8_t *W, const uint8_t *wscale_code,
                     int in, int out, int round_out);
/* src/dsv4/dsv4_internal.h:266 (src/dsv4/dsv4_model.c:678) */
void dsv4_gemv_fp8_batch_q(float *const *y, const float *const *qx,
                           const float *const *qscale, int batch,
                           const uint8_t *W, const uint8_t *wscale_code,
                           int in, int out, int round_out);
/* src/dsv4/dsv4_internal.h:270 (src/dsv4/dsv4_model.c:809) */
void dsv4_gemv_fp8_pair_q(float *y0, float *y1, const float *qx,
                          const float *qscale, const uint8_t *W0,
                          const uint8_t *S0, const uint8_t *W1,
                          const uint8_t *S1, int in, int out);
/* src/dsv4/dsv4_internal.h:276 (src/dsv4/dsv4_model.c:967) */
void dsv4_gemv_fp4_q(float *y, const float *qx, const float *qscale,
                     const uint8_t *W, const uint8_t *wscale_code,
                     int in, int rows);
/* src/dsv4/dsv4_internal.h:279 (src/dsv4/dsv4_model.c:1080) */
void dsv4_gemv_fp4_batch_q(float *const *y, const float *const *qx,
                           const float *const *qscale, int batch,
                           const uint8_t *W, const uint8_t *wscale_code,
                           int in, int rows);
/* src/dsv4/dsv4_internal.h:283 (src/dsv4/dsv4_model.c:1220) */
void dsv4_gemv_fp4_pair_q(float *y0, float *y1, const float *qx,
                          const float *qscale, const uint8_t *W0,
                          const uint8_t *S0, const uint8_t *W1,
                          const uint8_t *S1, int in, int rows);
/* src/dsv4/dsv4_internal.h:327 (src/dsv4/dsv4_model.c:5580) */
void dsv4_quant_fp8_codes(float *qx, float *qscale, const float *x, int n);
/* include/dsv4/dsv4.h:195 (src/dsv4/dsv4_ops.c:122) - same arithmetic */
void dsv4_quant_fp8_act(float *out, float *scales, const float *x, int n);
/* include/dsv4/dsv4.h:251 (src/dsv4/dsv4_ops.c:473). `gate` is declared
 * float* like the reference but read as a BF16 [n_experts][hidden] matrix,
 * as the reference does (src/dsv4/dsv4_ops.c:494, :502). */
void dsv4_router(int *idx, float *wt, const float *x, const float *gate,
                 const float *bias, const int64_t *tid2eid, int token_id,
                 int hidden, int n_experts, int topk, int hash_layer,
                 float route_scale, float rms_eps);

/* routed_swiglu_quant (src/dsv4/dsv4_model.c:6239, file-static there):
 * clamp, SiLU, x route_weight, BF16 into y, then per-128 FP8 quant into qy
 * (E4M3-grid floats) and qscale. Host pointers, like the drop-ins above. */
void dsv4cuda_routed_swiglu_quant(float *y, float *qy, float *qscale, const float *gate,
                                  const float *up, int n, int limit, float route_weight);

/* Prefixed aliases of the nine model-path kernels above. */
void dsv4cuda_gemv_bf16(float *y, const float *x, const uint16_t *W, int in,
                        int out, int round_out);
void dsv4cuda_gemv_bf16_batch(float *const *y, const float *const *x, int batch,
                              const uint16_t *W, int in, int out, int round_out);
void dsv4cuda_gemv_fp8_q(float *y, const float *qx, const float *qscale,
                         const uint8_t *W, const uint8_t *wscale_code, int in,
                         int out, int round_out);
void dsv4cuda_gemv_fp8_batch_q(float *const *y, const float *const *qx,
                               const float *const *qscale, int batch,
                               const uint8_t *W, const uint8_t *wscale_code,
                               int in, int out, int round_out);
void dsv4cuda_gemv_fp8_pair_q(float *y0, float *y1, const float *qx,
                              const float *qscale, const uint8_t *W0,
                              const uint8_t *S0, const uint8_t *W1,
                              const uint8_t *S1, int in, int out);
void dsv4cuda_gemv_fp4_q(float *y, const float *qx, const float *qscale,
                         const uint8_t *W, const uint8_t *wscale_code, int in,
                         int rows);
void dsv4cuda_gemv_fp4_batch_q(float *const *y, const float *const *qx,
                               const float *const *qscale, int batch,
                               const uint8_t *W, const uint8_t *wscale_code,
                               int in, int rows);
void dsv4cuda_gemv_fp4_pair_q(float *y0, float *y1, const float *qx,
                              const float *qscale, const uint8_t *W0,
                              const uint8_t *S0, const uint8_t *W1,
                              const uint8_t *S1, int in, int rows);
void dsv4cuda_quant_fp8_codes(float *qx, float *qscale, const float *x, int n);

/* ---------------------------------------------------- 3. lifecycle -- */

/* Select the CUDA device for the calling thread's drop-in calls and create
 * its stream and staging buffers. Optional: the first call on a thread does
 * it for the current device. Returns 0 or a negative error. */
int dsv4cuda_init(int device);
/* Release the calling thread's stream and staging buffers. */
void dsv4cuda_shutdown(void);
/* Last error recorded on the calling thread ("" if none). */
const char *dsv4cuda_last_error(void);
/* Device-side error flags of the current device (synchronous): bit 0 = a
 * GEMV kernel gave up waiting on a shared-memory barrier, bit 1 = the
 * attention kernel did (bounded waits; the results of that launch are
 * invalid), bit 2 = an attention key index >= kv_rows was skipped.
 * clear != 0 resets them. */
int dsv4cuda_device_error(unsigned int *flags, int clear);
/* Drop-in calls served since the library loaded, per kernel family:
 * counts[0] FP4 GEMVs, [1] FP8 GEMVs, [2] BF16 GEMVs, [3] activation quant,
 * [4] router, [5] SwiGLU quant (the first n of them). Returns the number of
 * families. With DSV4CUDA_DROPIN_REPORT=1 in the environment the library
 * prints the counts to stderr at exit, so a host program that preloads it
 * can show which of its kernel calls ran on the GPU. */
int dsv4cuda_dropin_calls(unsigned long long *counts, int n);
/* 1 (default): a drop-in call that hits a CUDA error exits(1) like the
 * reference's fatal paths; 0: record the error and return. Returns the
 * previous mode. */
int dsv4cuda_set_abort_on_error(int abort_on_error);

/* ------------------------------------ 2. device-resident MoE layer -- */

/* Shared expert formats. */
#define DSV4CUDA_SHARED_NONE 0
#define DSV4CUDA_SHARED_FP8 1 /* the reference's [128x128]-block FP8 expert */
#define DSV4CUDA_SHARED_FP4 2 /* same layout as a routed FP4 expert */

typedef struct {
    int hidden;        /* H  */
    int moe_inter;     /* I  */
    int n_experts;     /* E  */
    int topk;          /* k <= 32 */
    int swiglu_limit;  /* (int)cfg.swiglu_limit, as the reference casts it */
    float route_scale;
    int shared_kind;   /* DSV4CUDA_SHARED_* */
    int hash_vocab;    /* rows of tid2eid for a hash layer, else 0 */
} dsv4cuda_moe_config;

/* Weights in the reference's layouts. Routed experts are expert-major:
 * w1/w3 [E][I][H/2] packed E2M1 (low nibble first) with s1/s3 [E][I][H/32]
 * E8M0; w2 [E][H][I/2] with s2 [E][H][I/32]. gate_w [E][H] BF16; bias [E]
 * f32 or NULL; tid2eid [hash_vocab][topk] int64 or NULL. Shared FP8:
 * sh1/sh3 [I][H] E4M3 with [ceil(I/128)][ceil(H/128)] E8M0, sh2 [H][I]
 * with [ceil(H/128)][ceil(I/128)]; shared FP4: routed layout without [E]. */
typedef struct {
    const uint16_t *gate_w;
    const float *bias;
    const int64_t *tid2eid;
    const uint8_t *w1, *s1, *w3, *s3, *w2, *s2;
    const uint8_t *sh1, *sh1s, *sh3, *sh3s, *sh2, *sh2s;
} dsv4cuda_moe_weights;

typedef struct dsv4cuda_moe_layer dsv4cuda_moe_layer;

/* Replaces the per-layer weight binding + expert cache feeding moe_forward
 * (src/dsv4/dsv4_model.c:1793-2056, :3642): copies every weight of the layer
 * from host memory into HBM once. max_tokens bounds one forward's batch. */
int dsv4cuda_moe_create(dsv4cuda_moe_layer **out, const dsv4cuda_moe_config *cfg,
                        const dsv4cuda_moe_weights *host_weights, int max_tokens);
/* Same, adopting weights that already live in device memory (not copied,
 * not freed by destroy). */
int dsv4cuda_moe_create_device(dsv4cuda_moe_layer **out,
                               const dsv4cuda_moe_config *cfg,
                               const dsv4cuda_moe_weights *device_weights,
                               int max_tokens);
void dsv4cuda_moe_destroy(dsv4cuda_moe_layer *L);

/* moe_forward / moe_forward_batch (src/dsv4/dsv4_model.c:6599, :6812): x
 * [n][H] device fp32 (BF16-valued) -> out [n][H] device, per token
 * identical to the reference's single-token result. token_ids (device,
 * [n]) is read only by hash layers and may be NULL otherwise. stream is a
 * cudaStream_t (NULL = default stream). Asynchronous. */
int dsv4cuda_moe_forward(dsv4cuda_moe_layer *L, const float *x, const int *token_ids,
                         int n_tokens, float *out, void *stream);
/* The same call with HOST buffers: copies x/token_ids in, runs, copies out
 * and synchronises (the reference-facing end-to-end path). */
int dsv4cuda_moe_forward_host(dsv4cuda_moe_layer *L, const float *x,
                              const int *token_ids, int n_tokens, float *out);
/* Routing of the last forward on L: idx/wt [n][topk] (ids ascending), host
 * buffers; synchronises. Returns the number of tokens (since the layer was
 * created) whose top-k needed the exact fp32 logit replay of a near tie,
 * or a negative error. */
int dsv4cuda_moe_last_routes(dsv4cuda_moe_layer *L, int n_tokens, int *idx, float *wt);
/* The router's score sqrt(softplus(z)) (src/dsv4/dsv4_model.c:5827) exactly
 * as the device selection evaluates it: scores[i] for z[i], DEVICE pointers,
 * async on stream. For checking the device score against the host libm's. */
int dsv4cuda_router_scores(const float *z, float *scores, int n, void *stream);
/* Router alone (device x), writing host idx/wt. public_router selects the
 * public dsv4_router() numerics instead of moe_forward's. */
int dsv4cuda_moe_route(dsv4cuda_moe_layer *L, const float *x, const int *token_ids,
                       int n_tokens, int public_router, int *idx, float *wt);
/* Expert-GEMV timing for roofline measurement: between _begin and _end,
 * every dsv4cuda_moe_forward on L records CUDA events around its routed
 * gate/up and down GEMV launches (not inside graph capture). _end waits for
 * them and returns the number of timed forwards and the summed milliseconds
 * of the two launches. */
int dsv4cuda_moe_timing_begin(dsv4cuda_moe_layer *L);
int dsv4cuda_moe_timing_end(dsv4cuda_moe_layer *L, int *n_forwards, float *gateup_ms,
                            float *down_ms);
/* Reads event group `index` (0 = the first forward since _begin) without
 * ending the timing: for forwards captured into a CUDA graph, whose event
 * nodes are re-recorded by every replay. */
int dsv4cuda_moe_timing_read(dsv4cuda_moe_layer *L, int index, float *gateup_ms, float *down_ms,
                             float *logits_ms, float *select_ms);
/* Same, also returning the summed router logit and selection milliseconds. */
int dsv4cuda_moe_timing_end2(dsv4cuda_moe_layer *L, int *n_forwards, float *gateup_ms,
                             float *down_ms, float *logits_ms, float *select_ms);
/* Allocation-free MoE layer forward. No counterpart in the reference (the
 * reference is a CPU engine); this is for callers that cannot allocate GPU
 * memory while they run a layer - inside a stream capture, under an engine
 * that owns every device allocation through its own pool, or with a fixed
 * memory footprint. Same computation and results as dsv4cuda_moe_forward,
 * but the caller supplies the config, DEVICE weight pointers (layouts as in
 * dsv4cuda_moe_weights), x [n][H], token_ids (hash layers) and out [n][H];
 * the working memory is a 4 MiB array inside this library, present on
 * every GPU that loads it until the process exits. No device memory is
 * allocated or freed (no cudaMalloc/cudaFree, no stream or event creation,
 * no allocating library routine); the device error word lives in the same
 * array and the TMA descriptors are encoded on every call, not cached.
 * Returns -1 with a message (dsv4cuda_last_error) when n_tokens needs more
 * than the 4 MiB (up to 9 tokens fit at hidden 7168 / inter 2048 /
 * 256 experts / top-8). The first call on each device looks up the array's
 * device address for that device (make that first call before any stream
 * capture). Every call on a device shares the one array and starts by
 * resetting the parts that must begin at zero; calls that overlap on the
 * GPU (different streams, no ordering between them) race on it. Runs on
 * `stream` only (the shared expert is not overlapped on a side stream). */
int dsv4cuda_moe_forward_noalloc(const dsv4cuda_moe_config *cfg,
                                 const dsv4cuda_moe_weights *device_weights,
                                 const float *x, const int *token_ids, int n_tokens,
                                 float *out, void *stream);
/* Device bytes the layer holds (weights it owns + workspace). */
size_t dsv4cuda_moe_device_bytes(const dsv4cuda_moe_layer *L);

/* ---- Expert parallelism (no counterpart in the reference, which runs every
 * expert on one host; expert parallel over G GPUs, attention replicated).
 * Device g creates its layer with the full router (gate_w/bias/tid2eid for
 * all n_experts) but routed weights only for experts [expert_lo, expert_hi)
 * (w1..s2 expert-major over those experts). Per step:
 *   dsv4cuda_moe_forward_local   router (identical on every device), this
 *                                device's experts, shared expert; the
 *                                [n][topk][H] fp32 slots of experts held
 *                                elsewhere are zero;
 *   sum dsv4cuda_moe_routed_slots over the devices (e.g. ncclAllReduce,
 *                                ncclFloat32, ncclSum, n*topk*H elements);
 *                                every slot has one non-zero contributor, so
 *                                the sum is exact;
 *   dsv4cuda_moe_combine         the ascending-id ordered combine
 *                                (src/dsv4/dsv4_model.c:6795-6805), whose
 *                                accumulator starts at +0 like the
 *                                reference's, so the output is bit-identical
 *                                to the single-device layer. */
int dsv4cuda_moe_create_device_ep(dsv4cuda_moe_layer **out, const dsv4cuda_moe_config *cfg,
                                  const dsv4cuda_moe_weights *device_weights, int max_tokens,
                                  int expert_lo, int expert_hi);
int dsv4cuda_moe_forward_local(dsv4cuda_moe_layer *L, const float *x, const int *token_ids,
                               int n_tokens, void *stream);
/* Device pointer of the routed slots [max_tokens][topk][H] fp32. */
float *dsv4cuda_moe_routed_slots(dsv4cuda_moe_layer *L);
int dsv4cuda_moe_combine(dsv4cuda_moe_layer *L, int n_tokens, float *out, void *stream);

/* Expert parallelism without a collective: the slot exchange runs over peer
 * memory (NVLink P2P) inside two kernels of the forward.
 *   dsv4cuda_moe_ep_buffer_bytes  size of one rank's exchange buffer
 *                                 (flags, counters, 2 x [max_tokens*topk][H]
 *                                 fp32 slots);
 *   dsv4cuda_moe_ep_attach        bufs[r] = rank r's exchange buffer as
 *                                 mapped in this process (bufs[rank] is this
 *                                 rank's own, e.g. from dsv4cuda_ipc_alloc;
 *                                 the others from dsv4cuda_ipc_open); zeroes
 *                                 this rank's buffer, so every rank attaches
 *                                 before any rank runs a forward;
 *   dsv4cuda_moe_forward_ep       router + local experts + shared expert,
 *                                 then this rank's slots are written into
 *                                 every rank's buffer and a step epoch into
 *                                 each peer's flags, then the ordered combine
 *                                 waits (bounded: a peer that never arrives
 *                                 sets bit 3 of the device error word) for
 *                                 every peer's epoch. Output bit-identical to
 *                                 the single-device layer; no host sync, so
 *                                 the call can be captured in a CUDA graph.
 * Ranks may also be emulated in one process on one device (bufs in the same
 * memory) when every rank's forward is issued before any rank waits, i.e.
 * in stream order on one stream. */
size_t dsv4cuda_moe_ep_buffer_bytes(const dsv4cuda_moe_layer *L);
int dsv4cuda_moe_ep_attach(dsv4cuda_moe_layer *L, int rank, int world, void *const *bufs);
int dsv4cuda_moe_forward_ep(dsv4cuda_moe_layer *L, const float *x, const int *token_ids,
                            int n_tokens, float *out, void *stream);
/* Token-parallel expert parallelism (each rank brings its own tokens, as
 * with data-parallel attention): the n_local rows of x_local are gathered
 * into every rank over peer memory, every rank routes all world * n_local
 * tokens (identically) and runs its experts for them, each slot goes only
 * to its token's owner, and each rank combines its own n_local tokens into
 * out_local. Requires world * n_local <= max_tokens; not for hash-routed
 * layers. Output rows bit-identical to the single-device layer on the same
 * tokens. */
int dsv4cuda_moe_forward_ep_tokens(dsv4cuda_moe_layer *L, const float *x_local, int n_local,
                                   float *out_local, void *stream);
/* Its three stages (gather; wait + route + local experts + push; wait +
 * combine), for callers that interleave ranks in one process. */
int dsv4cuda_moe_ep_tokens_gather(dsv4cuda_moe_layer *L, const float *x_local, int n_local,
                                  void *stream);
int dsv4cuda_moe_ep_tokens_compute(dsv4cuda_moe_layer *L, int n_local, void *stream);
int dsv4cuda_moe_ep_tokens_combine(dsv4cuda_moe_layer *L, int n_local, float *out_local,
                                   void *stream);
/* The exchange's two halves, separately (dsv4cuda_moe_forward_local first). */
int dsv4cuda_moe_ep_push(dsv4cuda_moe_layer *L, int n_tokens, void *stream);
int dsv4cuda_moe_ep_combine(dsv4cuda_moe_layer *L, int n_tokens, float *out, void *stream);

/* Device memory shared across processes (CUDA IPC): handle = 64 bytes. */
int dsv4cuda_ipc_alloc(size_t bytes, void **ptr, unsigned char *handle);
int dsv4cuda_ipc_open(const unsigned char *handle, void **ptr);
int dsv4cuda_ipc_close(void *ptr);
int dsv4cuda_ipc_free(void *ptr);

/* ---------------------------------------------------------------------
 * Latent KV cache and decode attention.
 *
 * The reference keeps each layer's latent cache as fp32 rows
 * (kv_cache [win + max_comp][head_dim], src/dsv4/dsv4_model.c:2416) whose
 * non-RoPE dims hold bf16(e4m3 * 2^k) with one power-of-two scale per 64 dims
 * (dsv4_act_quant_inplace group 64 mode 0, :1386, applied at :5300) and whose
 * RoPE dims hold BF16 (:1555). dsv4cuda_kv_cache stores exactly those values
 * as E4M3 codes + E8M0 scale codes + BF16, losslessly (DEVICE pointers):
 *   codes  [rows][nope]      scales [rows][8]      rope [rows][rope_dim] */
typedef struct {
    uint8_t *codes;
    uint8_t *scales;
    uint16_t *rope;
    int nope;          /* head_dim - rope_dim; multiple of 64, <= 512 */
    int rope_dim;
    long long rows;
} dsv4cuda_kv_cache;

/* Quantise n latents kv [n][nope + rope_dim] (fp32, BF16-valued: the
 * reference's kvn after kv_norm and RoPE) into cache rows rows[n]; the
 * reference's dsv4_act_quant_inplace + memcpy into the ring slot
 * (src/dsv4/dsv4_model.c:5300-5304). Device pointers, async on `stream`. */
int dsv4cuda_kv_write(const dsv4cuda_kv_cache *cache, const float *kv, const long long *rows,
                      int n, void *stream);
/* Decode cache rows rows[n] to fp32 [n][nope + rope_dim], the exact values
 * the reference would hold in its kv_cache. */
int dsv4cuda_kv_read(const dsv4cuda_kv_cache *cache, const long long *rows, int n, float *out,
                     void *stream);

typedef struct {
    int batch;            /* independent queries (decode batch) */
    int heads;            /* H */
    int head_dim;         /* d (512 for DSV4: 448 + 64 RoPE) */
    int n_keys;           /* topk_total: indices per query */
    float scale;          /* d^-1/2 */
    int rope_dim;         /* inverse RoPE on the last rope_dim dims */
    long long kv_batch_stride;  /* cache rows between consecutive queries' caches */
    long long kv_rows;    /* valid rows per query (indices must be < kv_rows) */
} dsv4cuda_attn_shape;

/* Device scratch bytes dsv4cuda_sparse_attn needs for `shape`. */
size_t dsv4cuda_attn_workspace_bytes(const dsv4cuda_attn_shape *shape, int use_cache);

/* Replaces sparse_attn (src/dsv4/dsv4_model.c:5767-5822) followed by
 * dsv4_rope_apply_buf_inv (:5373) for `batch` queries at once. DEVICE
 * pointers: q [batch][H][d] (BF16-valued fp32), either kv (fp32 rows, the
 * reference layout, row = b * kv_batch_stride + idx) or cache (kv == NULL),
 * sink [H], idx [batch][n_keys] (-1 = padding, as topk_idx), rope_cos /
 * rope_sin [batch][rope_dim/2] (NULL: no inverse RoPE), out [batch][H][d]
 * (BF16-valued). workspace may be NULL (the library keeps a per-thread
 * buffer, allocating when it grows). d = 512 with H <= 128 runs the
 * tensor-core kernel; other shapes run SIMT kernels. Results agree with the
 * reference within the tolerance stated in the tests (BF16 weights and
 * outputs; summation order differs). Index >= kv_rows sets device-error
 * bit 2 and the key is skipped. */
int dsv4cuda_sparse_attn(float *out, const float *q, const float *kv,
                         const dsv4cuda_kv_cache *cache, const float *sink, const int *idx,
                         const float *rope_cos, const float *rope_sin,
                         const dsv4cuda_attn_shape *shape, void *workspace,
                         size_t workspace_bytes, void *stream);

/* Host-pointer form with the reference's sparse_attn arguments
 * (o, q, kv, attn_sink, topk_idx, topk_total, H, d, scale;
 * src/dsv4/dsv4_model.c:5767): stages to the GPU, runs, copies o back. */
void dsv4cuda_sparse_attn_host(float *o, const float *q, const float *kv, const float *attn_sink,
                               const int *topk_idx, int topk_total, int H, int d, float scale);

/* Attention kernel timing for roofline measurement (CUDA events around the
 * main attention kernel of every dsv4cuda_sparse_attn call on this thread
 * between _begin and _end; not inside graph capture). */
int dsv4cuda_attn_timing_begin(void);
int dsv4cuda_attn_timing_end(int *n_calls, float *main_ms);

/* ---------------------------------------------------------------------
 * Speculative-decoding acceptance (the reference runs it on the host in
 * its CLI: rng_next src/cli/dsv4_run.c:248, sample_top_p :308, argmax_logits
 * :355, the verify loop :951-1043; EOS is token 1 there, eos_id here).
 *
 * Host forms (host pointers), the same arithmetic in the same order: */
uint64_t dsv4cuda_rng_next(uint64_t *state);
int dsv4cuda_argmax_logits(const float *logits, int vocab);
int dsv4cuda_sample_top_p(const float *logits, int vocab, double temperature, double top_p,
                          uint64_t *rng_state);
/* One verify step: proposal[proposed] drafts against logits
 * [(proposed + 1)][vocab]; temperature 0 = greedy. Writes the emitted tokens
 * (accepted drafts then the correction or bonus, or up to an accepted EOS)
 * and returns their count; *n_commit = verified positions to keep (the
 * snapshot commit length), *n_accepted, *n_samples = uniforms drawn. */
int dsv4cuda_accept_chain(const int *proposal, int proposed, const float *logits, int vocab,
                          double temperature, double top_p, uint64_t *rng_state, int eos_id,
                          int *tokens, int *n_commit, int *n_accepted, int *n_samples);

/* Device forms (DEVICE pointers, async on stream): logits stay in HBM.
 * dsv4cuda_argmax_rows: out[r] = argmax_logits(row r), bit-exact.
 * dsv4cuda_sample_rows: top_p = 1 sampling with uniforms[r] =
 *   (rng_next() >> 11) * 2^-53 drawn in row order; the softmax sums are
 *   formed in parallel, so a target within a few ulps of a running sum may
 *   select the neighbouring token (use the host form for exact replay or
 *   top_p < 1).
 * dsv4cuda_accept_device: row targets of the proposed + 1 rows, then the
 *   chain; result holds 2 * proposed + 6 ints: [0] emitted, [1] n_commit,
 *   [2] n_accepted, [3] uniforms consumed (advance the host rng by this),
 *   [4 ..] emitted tokens. */
int dsv4cuda_argmax_rows(const float *logits, int rows, int vocab, int *out, void *stream);
int dsv4cuda_sample_rows(const float *logits, int rows, int vocab, double temperature,
                         const double *uniforms, int *out, void *stream);
int dsv4cuda_accept_device(const int *proposal, int proposed, const float *logits, int vocab,
                           double temperature, const double *uniforms, int eos_id, int *result,
                           void *stream);

/* ---------------------------------------------------------------------
 * Speculative transaction on the latent KV ring (dsv4_context_snapshot_take
 * / _restore / _commit_prefix, src/dsv4/dsv4_model.c:2842-3056), device
 * memory. Each registered cache holds a window ring at rows
 * [ring_base, ring_base + window) (position p -> row ring_base + p % window);
 * state buffers (e.g. the hyper-connection residual state) are saved at
 * take and captured after each verified position. Per verify step:
 *   take(start, n)            save the ring rows positions start..start+n-1
 *                             will overwrite, and the states (n <= window,
 *                             n <= max_positions <= 64);
 *   capture_state(step)       after position start+step: copy the states;
 *   commit_prefix(k)          keep positions < k, put the saved rows back
 *                             for the others, states = capture of step k-1;
 *   restore()                 undo the whole step. */
typedef struct dsv4cuda_snapshot dsv4cuda_snapshot;
int dsv4cuda_snapshot_create(dsv4cuda_snapshot **out, int max_positions, int n_caches,
                             const dsv4cuda_kv_cache *caches, const long long *ring_base,
                             const int *windows, int n_states, float *const *states,
                             const size_t *state_elems);
int dsv4cuda_snapshot_take(dsv4cuda_snapshot *s, int start_position, int n_positions,
                           void *stream);
int dsv4cuda_snapshot_capture_state(dsv4cuda_snapshot *s, int step, void *stream);
int dsv4cuda_snapshot_commit_prefix(dsv4cuda_snapshot *s, int n_positions, void *stream);
int dsv4cuda_snapshot_restore(dsv4cuda_snapshot *s, void *stream);
void dsv4cuda_snapshot_destroy(dsv4cuda_snapshot *s);

/* ---------------------------------------------------------------------
 * Verify step over a draft tree (a chain: parents = -1, 0, 1, ...), the
 * batched verify of dsv4_prefill_capture (src/dsv4/dsv4_model.c:8434) with
 * an ancestor mask. Node j is at position committed + depth(j) and sees the
 * window window_topk (:5073) gives that position, where positions >=
 * committed are its ancestors and itself, held in scratch rows
 * scratch_row + node. Writes idx [n_nodes][row_len] (host, -1 padded) for
 * dsv4cuda_sparse_attn with batch = n_nodes and kv_batch_stride = 0, and
 * returns the longest row. */
int dsv4cuda_tree_attn_indices(const int *parents, int n_nodes, int committed, int window,
                               long long ring_base, long long scratch_row, int *idx,
                               int row_len);
/* Copy cache rows src_rows[i] -> dst_rows[i] (host arrays, n <= 64): moves
 * the accepted path's scratch rows into their ring slots. */
int dsv4cuda_kv_copy_rows(const dsv4cuda_kv_cache *cache, const long long *src_rows,
                          const long long *dst_rows, int n, void *stream);

/* ---------------------------------------------------------------------
 * Whole-model decode on the device: dsv4_forward_token
 * (src/dsv4/dsv4_model.c:8388, public API include/dsv4/dsv4.h:161) with
 * every weight resident in HBM. Layers of compress ratio 0 attend to the
 * sliding window; ratio-4 and ratio-128 layers also run the compressor
 * (and for ratio 4 the indexer and its top-k) and attend to the window plus
 * the selected compressed rows, in the reference's order. One call per token: embedding, per
 * layer hyper-connection pre, RMSNorm, attention (FP8 projections, norms,
 * RoPE, FP8 latent ring, sparse attention over the window, inverse RoPE,
 * grouped wo_a, wo_b), HC post, HC pre, RMSNorm, MoE layer, HC post; then
 * the HC head, final RMSNorm, BF16 vocab head and argmax. All weight
 * pointers are DEVICE pointers in the checkpoint's layouts. */
typedef struct {
    int hidden, n_layers, vocab;
    int n_heads, head_dim, rope_dim, q_lora, o_groups, o_lora, window;
    int hc_mult, hc_iters;        /* hc_mult <= 4 */
    float rms_eps, hc_eps, rope_theta;
    int max_context;              /* positions 0 .. max_context - 1 */
    dsv4cuda_moe_config moe;      /* moe.hidden == hidden */
    /* 1: the hyper-connection mixes run the reference's sequential fp32
     * fmaf chains (hc_mult * hidden long; one thread per mix row) and the
     * step reproduces dsv4_forward_token bit for bit up to the host libm's
     * last-ulp expf differences; 0: the mixes are summed in double in
     * parallel (fast, within the chains' rounding of the reference). */
    int hc_exact;
    /* Layers of compress ratio 4 / 128 (dsv4cuda_layer_weights.compress_ratio):
     * the indexer's heads, head dim and top-k, and the RoPE of compressed
     * layers (YaRN, rope_freqs_fill src/dsv4/dsv4_model.c:1475-1503). Unused
     * when every layer has ratio 0. */
    int index_heads, index_dim, index_topk;
    float compress_rope_theta, rope_factor, beta_fast, beta_slow;
    int original_position;
} dsv4cuda_decoder_config;

typedef struct {
    const uint16_t *embed;        /* [vocab][hidden] BF16 */
    const uint16_t *head;         /* [vocab][hidden] BF16 */
    const uint16_t *norm;         /* [hidden] BF16 final RMSNorm gain */
    const float *hc_head_fn;      /* [hc_mult][hc_mult * hidden] */
    const float *hc_head_base;    /* [hc_mult] */
    const float *hc_head_scale;   /* [1] */
} dsv4cuda_model_weights;

typedef struct {
    const uint16_t *attn_norm, *ffn_norm;                    /* [hidden] BF16 */
    const float *hc_attn_fn, *hc_attn_scale, *hc_attn_base;  /* [(2+m)m][m*hidden], [3], [(2+m)m] */
    const float *hc_ffn_fn, *hc_ffn_scale, *hc_ffn_base;
    const float *attn_sink;                                  /* [n_heads] */
    const uint8_t *wq_a, *wq_a_s;     /* FP8 [q_lora][hidden] + [128x128] E8M0 */
    const uint16_t *q_norm;           /* [q_lora] */
    const uint8_t *wq_b, *wq_b_s;     /* FP8 [n_heads*head_dim][q_lora] */
    const uint8_t *wkv, *wkv_s;       /* FP8 [head_dim][hidden] */
    const uint16_t *kv_norm;          /* [head_dim] */
    const uint16_t *wo_a;             /* BF16 [o_groups*o_lora][n_heads*head_dim/o_groups], or NULL: */
    const uint8_t *wo_a_fp8, *wo_a_fp8_s;  /* the checkpoint's FP8 form, decoded to BF16 at create
                                              as the reference does at load (:1927-1936) */
    const uint8_t *wo_b, *wo_b_s;     /* FP8 [hidden][o_groups*o_lora] */
    dsv4cuda_moe_weights moe;         /* expert-major routed FP4 + shared expert */
    /* compress ratio 0 (sliding window only), 4 (compressor with overlapping
     * blocks + indexer top-k) or 128 (compressor, every compressed row
     * attended): compressor_update / indexer_forward, src/dsv4/dsv4_model.c:
     * 5100-5236, :5685-5760. coff = 2 for ratio 4, else 1. */
    int compress_ratio;
    const uint16_t *comp_wkv, *comp_wgate;      /* BF16 [coff*head_dim][hidden] */
    const float *comp_ape;                      /* [ratio][coff*head_dim] */
    const uint16_t *comp_norm;                  /* [head_dim] BF16 */
    const uint8_t *idx_wq_b, *idx_wq_b_s;       /* FP8 [index_heads*index_dim][q_lora] */
    const uint16_t *idx_weights_proj;           /* BF16 [index_heads][hidden] */
    const uint16_t *idx_comp_wkv, *idx_comp_wgate;  /* BF16 [2*index_dim][hidden] */
    const float *idx_ape;                       /* [4][2*index_dim] */
    const uint16_t *idx_comp_norm;              /* [index_dim] BF16 */
} dsv4cuda_layer_weights;

typedef struct dsv4cuda_decoder dsv4cuda_decoder;

/* Builds a decoder over the given device weights (not copied; wo_a is
 * decoded into a decoder-owned BF16 copy when only its FP8 form is given)
 * and allocates the per-layer FP8 latent rings (window rows each), the
 * RoPE tables of every position and the step buffers. Returns 0 or -1
 * (dsv4cuda_decoder_last_error). */
int dsv4cuda_decoder_create(dsv4cuda_decoder **out, const dsv4cuda_decoder_config *cfg,
                            const dsv4cuda_model_weights *model,
                            const dsv4cuda_layer_weights *layers);
void dsv4cuda_decoder_destroy(dsv4cuda_decoder *D);
const char *dsv4cuda_decoder_last_error(void);
/* Expert parallelism: layers[i] (n == n_layers) is an EP-attached MoE layer
 * (dsv4cuda_moe_create_device_ep + dsv4cuda_moe_ep_attach, max_tokens >=
 * world) that layer i's MoE block runs through, token-parallel: each rank's
 * decoder brings its own token, the tokens of all ranks are routed
 * together, every rank computes its own experts and each slot returns to
 * its token's owner over peer memory (dsv4cuda_moe_forward_ep_tokens). All
 * ranks step in lockstep. n == 0 returns to the local MoE weights. */
int dsv4cuda_decoder_set_moe_layers(dsv4cuda_decoder *D, dsv4cuda_moe_layer *const *layers, int n);
/* replicated = 1: every rank decodes the same token (batch-1 decode over
 * the ranks' experts, dsv4cuda_moe_forward_ep: each rank routes the token,
 * computes its own experts' slots and exchanges them); 0 (default): the
 * token-parallel exchange above. */
int dsv4cuda_decoder_set_ep_replicated(dsv4cuda_decoder *D, int replicated);
/* Clears the latent rings (dsv4_model_reset_context). Async on stream. */
int dsv4cuda_decoder_reset(dsv4cuda_decoder *D, void *stream);
/* dsv4_forward_token: host token/position in, host logits[vocab] (may be
 * NULL) and the greedy next token (argmax, lowest id on ties; may be NULL)
 * out; synchronous. */
int dsv4cuda_decoder_forward_token(dsv4cuda_decoder *D, int token, int position, float *logits,
                                   int *next_token);
/* The same step reading token and position from the decoder's own device
 * slots (dsv4cuda_decoder_token_slot / _position_slot) and leaving logits and
 * argmax in device memory (dsv4cuda_decoder_logits / _argmax): no host
 * synchronisation, so a captured CUDA graph of it replays for any position. */
int dsv4cuda_decoder_step(dsv4cuda_decoder *D, void *stream);
/* Copies device token/position into the slots, then steps. */
int dsv4cuda_decoder_step_device(dsv4cuda_decoder *D, const int *token, const int *position,
                                 void *stream);
/* Number of kernels one step launches (counted from a captured graph of
 * one step, which is not run), or -1. */
int dsv4cuda_decoder_step_kernels(dsv4cuda_decoder *D);
/* Waits for the device, then copies the last step's logits[vocab] and
 * argmax to host memory (either may be NULL). */
int dsv4cuda_decoder_read(dsv4cuda_decoder *D, float *logits, int *next_token);
/* Layer `layer`'s latent ring (window rows; position p at row p % window),
 * e.g. to register it with dsv4cuda_snapshot_create for a verify step. */
int dsv4cuda_decoder_cache(dsv4cuda_decoder *D, int layer, dsv4cuda_kv_cache *out);
int *dsv4cuda_decoder_token_slot(dsv4cuda_decoder *D);
int *dsv4cuda_decoder_position_slot(dsv4cuda_decoder *D);
float *dsv4cuda_decoder_logits(dsv4cuda_decoder *D);
int *dsv4cuda_decoder_argmax(dsv4cuda_decoder *D);

/* Speculative verify on the decoder: dsv4_prefill_capture with all_logits
 * (src/dsv4/dsv4_model.c:8434-8529, include/dsv4/dsv4_internal.h:296),
 * i.e. n_rows tokens [pending, d1 .. dk] at positions start .. start +
 * n_rows - 1 through every layer layer-major (forward_loaded_layer_batch
 * :7577): each projection and expert GEMV streams its weights once for all
 * rows, each row attends to the window of its own position (the earlier
 * rows' latents included), and every row's logits come out
 * (compute_logits_batch :7784). The rows' latents go to scratch rows beside
 * each layer's ring, which is left untouched: nothing needs undoing when
 * drafts are rejected, and a commit moves the kept rows into the ring
 * (the reference's snapshot take / commit_prefix, :2842-3056, reduced to a
 * row copy because these layers keep no other per-position state).
 * Layers with the local MoE weights only (no expert parallelism). */
#define DSV4CUDA_VERIFY_MAX_ROWS 8
/* Host form: tokens[n_rows] and start_position in; all_logits
 * [n_rows][vocab] and argmax[n_rows] (either may be NULL) out; synchronous. */
int dsv4cuda_decoder_verify(dsv4cuda_decoder *D, const int *tokens, int n_rows,
                            int start_position, float *all_logits, int *argmax);
/* Device form: rows from dsv4cuda_decoder_verify_tokens, row 0's position
 * from dsv4cuda_decoder_verify_start; logits and argmax stay in device memory
 * (dsv4cuda_decoder_verify_logits / _argmax). Async, graph-capturable. */
int dsv4cuda_decoder_verify_device(dsv4cuda_decoder *D, int n_rows, void *stream);
/* Keep rows 0 .. n_keep - 1 of the last verify (positions start .. start +
 * n_keep - 1): their latents move into the ring. Synchronous on stream. */
int dsv4cuda_decoder_commit(dsv4cuda_decoder *D, int n_keep, void *stream);
/* Greedy acceptance on the device (the reference CLI's chain at temperature
 * 0, src/cli/dsv4_run.c:951-1043): accepts drafts while they equal the
 * previous row's argmax, commits the pending row and the accepted drafts,
 * makes the bonus token the next pending row and advances the start; the
 * totals of tokens emitted, drafts accepted and steps accumulate in
 * dsv4cuda_decoder_verify_stats. Async, graph-capturable. */
int dsv4cuda_decoder_accept_greedy(dsv4cuda_decoder *D, int n_rows, void *stream);
/* Uniform random drafts for rows 1 .. n_rows - 1 (the reference CLI's
 * xorshift64 rng_next modulo the vocabulary, a decoder-owned seed).
 * Async, graph-capturable. */
int dsv4cuda_decoder_draft_random(dsv4cuda_decoder *D, int n_rows, void *stream);
/* Waits for the device, then reads the totals (stats3: tokens emitted,
 * drafts accepted, verify steps) and the pending token / its position that
 * accept_greedy left for the next step. */
int dsv4cuda_decoder_verify_stats(dsv4cuda_decoder *D, long long *stats3);
int dsv4cuda_decoder_verify_pending(dsv4cuda_decoder *D, int *token, int *position);
int *dsv4cuda_decoder_verify_tokens(dsv4cuda_decoder *D);
int *dsv4cuda_decoder_verify_start(dsv4cuda_decoder *D);
float *dsv4cuda_decoder_verify_logits(dsv4cuda_decoder *D);
int *dsv4cuda_decoder_verify_argmax(dsv4cuda_decoder *D);

#ifdef __cplusplus
}
#endif

#endif /* DSV4_CUDA_H */
