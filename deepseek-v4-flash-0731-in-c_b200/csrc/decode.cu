// decode.cu - the whole DeepSeek-V4-Flash decode step on the device:
// dsv4_forward_token (src/dsv4/dsv4_model.c:8388) for layers whose attention
// is the sliding window (compress ratio 0), with every weight resident in HBM.
//
// Per token: embedding row -> per layer [hyper-connection pre (HC mixes,
// Sinkhorn split, weighted reduce) -> RMSNorm -> attention (FP8 projections,
// q/kv norms, RoPE, FP8 latent ring, sparse_attn over the window, inverse
// RoPE, grouped BF16 wo_a, FP8 wo_b) -> HC post -> HC pre -> RMSNorm -> MoE
// layer -> HC post] -> HC head + final RMSNorm -> BF16 vocab head -> argmax.
// Token id and position are read from device memory, so one CUDA graph of a
// whole step replays for every position.
//
// Numerics against the reference. Exact (same operations in the same order):
// the embedding, every GEMV (FP8, BF16, the MoE layer's FP4), activation
// quantisation, RMSNorm (its double sum of squares is exact for BF16-valued
// inputs of ordinary range, so a parallel sum gives the same double), the
// weighted HC reduce and HC post (fmaf chains of length hc_mult), the q-head
// norm and RoPE (host-computed cos/sin tables from the reference's formula;
// products and sums rounded separately, as the reference's
// -ffp-contract=off build does), the KV quantisation and window indexing.
// Within tolerance: the HC mixes (the reference's 16384-long fp32 fmaf chain
// is summed in double here), the Sinkhorn split and HC head sigmoid (expf)
// and the attention (tensor-core sums, BF16 weights against a running max).
#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "attn.cuh"
#include "bulk.cuh"
#include "dsv4_common.cuh"
#include "gemv.cuh"
#include "launch.cuh"
#include "moe.cuh"
#include "sample.cuh"
#include "../../include/dsv4_cuda.h"

#define DSV4_API extern "C" __attribute__((visibility("default")))

namespace dsv4 {
namespace {

constexpr int kMixMax = 24;      // HC mix rows a partial kernel carries: (2 + 4) * 4
constexpr int kHcMultMax = 8;    // the reference keeps pre[8]
constexpr int kMixThreads = 128;

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Sum of one double per thread over the block (any block size <= 1024); the
// result is returned to every thread. Exact whenever the double sums are
// (the only use: squares of BF16-valued floats).
__device__ double block_sum_d(double v, double* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum_d(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  double t = 0.0;
  const int nw = (blockDim.x + 31) >> 5;
  for (int w = 0; w < nw; ++w) t += red[w];
  return t;
}

__device__ __forceinline__ float rms_factor(double ss, int n, float eps) {
  // 1.0f / sqrtf((float)(ss / n) + eps)  (src/dsv4/dsv4_model.c:4937-4939)
  return 1.0f / sqrtf(__fadd_rn(static_cast<float>(ss / n), eps));
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  return (__float_as_uint(bf16_round(lo)) >> 16) | (__float_as_uint(bf16_round(hi)) & 0xFFFF0000u);
}

// ------------------------------------------------------------ kernels ----

// embed_token (src/dsv4/dsv4_model.c:7478): every HC copy gets the BF16 row.
// Row blockIdx.y of a verify step embeds token[blockIdx.y] into its own state.
__global__ void embed_kernel(const uint16_t* embed, const int* token, int vocab, int hid, int mult,
                             float* state) {
  pdl_wait();
  pdl_trigger();
  int t = token[blockIdx.y];
  if (t < 0 || t >= vocab) t = 0;
  state += static_cast<size_t>(blockIdx.y) * mult * hid;
  const uint16_t* row = embed + static_cast<size_t>(t) * hid;
  for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < hid; j += gridDim.x * blockDim.x) {
    const float v = bf16_widen(row[j]);
    for (int k = 0; k < mult; ++k) state[static_cast<size_t>(k) * hid + j] = v;
  }
}

// Per-position set-up shared by every layer of a step: the window's key list
// (window_topk with padding, src/dsv4/dsv4_model.c:5073), the ring row the
// new latent goes to (pos % win, :5304) and the RoPE cos/sin of the position.
__global__ void position_kernel(const int* pos_ptr, int win, int half, int max_pos,
                                const float* cos_tab, const float* sin_tab, int* idx,
                                long long* row, float* cosv, float* sinv, const float* cos_tab_c,
                                const float* sin_tab_c, float* cosv_c, float* sinv_c) {
  pdl_wait();
  pdl_trigger();
  int pos = *pos_ptr;
  if (pos < 0) pos = 0;
  if (pos >= max_pos) pos = max_pos - 1;
  for (int i = threadIdx.x; i < win; i += blockDim.x) {
    if (pos >= win - 1) idx[i] = (pos % win + 1 + i) % win;
    else idx[i] = i <= pos ? i : -1;
  }
  for (int i = threadIdx.x; i < half; i += blockDim.x) {
    cosv[i] = cos_tab[static_cast<size_t>(pos) * half + i];
    sinv[i] = sin_tab[static_cast<size_t>(pos) * half + i];
    if (cosv_c) {  // the compressed layers' table (YaRN)
      cosv_c[i] = cos_tab_c[static_cast<size_t>(pos) * half + i];
      sinv_c[i] = sin_tab_c[static_cast<size_t>(pos) * half + i];
    }
  }
  if (threadIdx.x == 0) *row = pos % win;
}

// The verify step's per-row set-up (dsv4_prefill_capture's rows at positions
// start + r, src/dsv4/dsv4_model.c:8434): row r's window lists the same
// positions in the same order as window_topk gives position start + r
// (:5073), but the positions start .. start + r are the verify rows' own
// latents, held in the scratch cache rows win + (position - start) until a
// commit moves the accepted ones into the ring; the ring itself is not
// written, so a rejected draft leaves nothing to undo. CTA r = row r.
__global__ void verify_position_kernel(const int* start_ptr, int win, int half, int max_pos,
                                       const float* cos_tab, const float* sin_tab, int* idx,
                                       long long* row, float* cosv, float* sinv) {
  pdl_wait();
  pdl_trigger();
  const int r = blockIdx.x;
  const int start = *start_ptr;
  int pos = start + r;
  if (pos < 0) pos = 0;
  if (pos >= max_pos) pos = max_pos - 1;
  for (int i = threadIdx.x; i < win; i += blockDim.x) {
    const int q = pos >= win - 1 ? pos - win + 1 + i : (i <= pos ? i : -1);
    idx[static_cast<size_t>(r) * win + i] = q < 0 ? -1 : (q >= start ? win + (q - start) : q % win);
  }
  for (int i = threadIdx.x; i < half; i += blockDim.x) {
    cosv[static_cast<size_t>(r) * half + i] = cos_tab[static_cast<size_t>(pos) * half + i];
    sinv[static_cast<size_t>(r) * half + i] = sin_tab[static_cast<size_t>(pos) * half + i];
  }
  if (threadIdx.x == 0) row[r] = win + r;
}

// HC mixes, partial sums: CTA b covers columns [b * kMixThreads, ...) of the
// flattened state (n = mult * hid): part[b] = {sum x^2, fn_0 . x, ...} in
// double (fp32 x fp32 products are exact in double).
__global__ void __launch_bounds__(kMixThreads) hc_mix_partial_kernel(const float* fn, int rows,
                                                                     const float* state, int n,
                                                                     double* part) {
  __shared__ double red[kMixThreads / 32][kMixMax + 1];
  pdl_wait();
  pdl_trigger();
  const int c = blockIdx.x * kMixThreads + threadIdx.x;
  double acc[kMixMax + 1];
#pragma unroll
  for (int j = 0; j <= kMixMax; ++j) acc[j] = 0.0;
  if (c < n) {
    const double x = state[c];
    acc[0] = x * x;
#pragma unroll
    for (int j = 0; j < kMixMax; ++j)
      if (j < rows) acc[1 + j] = static_cast<double>(fn[static_cast<size_t>(j) * n + c]) * x;
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int j = 0; j <= kMixMax; ++j) {
    const double v = warp_sum_d(acc[j]);
    if (lane == 0) red[warp][j] = v;
  }
  __syncthreads();
  if (threadIdx.x <= rows) {
    double t = 0.0;
    for (int w = 0; w < kMixThreads / 32; ++w) t += red[w][threadIdx.x];
    part[static_cast<size_t>(blockIdx.x) * (kMixMax + 1) + threadIdx.x] = t;
  }
}

// HC mixes in the reference's own order (hc_pre_scratch, src/dsv4/dsv4_model.c:
// 7133-7141): lane j < rows runs row j's fp32 fmaf chain over the whole
// state, lane 31 the double sum of squares; written as one "partial block".
// Sequential by construction (n fmaf per chain): the decoder's exact mode.
__global__ void hc_mix_exact_kernel(const float* fn, int rows, const float* state, int n,
                                    double* part) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x;
  if (lane < rows) {
    const float* row = fn + static_cast<size_t>(lane) * n;
    float acc = 0.0f;
    int i = 0;
    for (; i + 4 <= n; i += 4) {
      const float4 w4 = *reinterpret_cast<const float4*>(row + i);
      const float4 s4 = *reinterpret_cast<const float4*>(state + i);
      acc = fmaf(w4.x, s4.x, acc);
      acc = fmaf(w4.y, s4.y, acc);
      acc = fmaf(w4.z, s4.z, acc);
      acc = fmaf(w4.w, s4.w, acc);
    }
    for (; i < n; ++i) acc = fmaf(row[i], state[i], acc);
    part[1 + lane] = static_cast<double>(acc);
  } else if (lane == 31) {
    double ss = 0.0;
    for (int i = 0; i < n; ++i) ss += static_cast<double>(state[i]) * state[i];
    part[0] = ss;
  }
}

__device__ __forceinline__ float sigmoid_stable(float x) {
  // src/dsv4/dsv4_ops.c:398-405
  if (x >= 0.0f) {
    const float e = expf_r1(-x);
    return 1.0f / (1.0f + e);
  }
  const float e = expf_r1(x);
  return e / (1.0f + e);
}

// mixes * scale + base, rounded after the product (no contraction)
__device__ __forceinline__ float mul_add(float a, float b, float c) {
  return __fadd_rn(__fmul_rn(a, b), c);
}

// dsv4_hc_split (src/dsv4/dsv4_ops.c:412-460) on one warp for a compile-time
// M: lane l < M*M holds comb[l / M][l % M]; each row or column sum is formed
// by every lane from shuffled values in the reference's sequential order
// (unrolled, so a sum costs one round of independent shuffles), and every
// division is the lane's own IEEE division, as in the reference's loops.
template <int M>
__device__ void hc_split_warp(const float* mixes, const float* scale3, const float* base,
                              int iters, float eps, float* pre_out, float* post_out,
                              float* comb_out) {
  const int lane = threadIdx.x & 31;
  const int li = lane < M * M ? lane : 0;
  const int ri = li / M, cj = li % M;
  if (lane < M) {
    pre_out[lane] = sigmoid_stable(mul_add(mixes[lane], scale3[0], base[lane])) + eps;
    post_out[lane] = 2.0f * sigmoid_stable(mul_add(mixes[M + lane], scale3[1], base[M + lane]));
  }
  float c = mul_add(mixes[2 * M + li], scale3[2], base[2 * M + li]);
  float v[M];
  {  // softmax rows
#pragma unroll
    for (int j = 0; j < M; ++j) v[j] = __shfl_sync(0xffffffffu, c, ri * M + j);
    float mx = v[0];
#pragma unroll
    for (int j = 1; j < M; ++j) mx = v[j] > mx ? v[j] : mx;
    const float e = expf_r1(c - mx);
#pragma unroll
    for (int j = 0; j < M; ++j) v[j] = __shfl_sync(0xffffffffu, e, ri * M + j);
    float sum = 0.0f;
#pragma unroll
    for (int j = 0; j < M; ++j) sum += v[j];
    c = e / sum + eps;
  }
  auto col_norm = [&]() {
#pragma unroll
    for (int i = 0; i < M; ++i) v[i] = __shfl_sync(0xffffffffu, c, i * M + cj);
    float sum = 0.0f;
#pragma unroll
    for (int i = 0; i < M; ++i) sum += v[i];
    c /= (sum + eps);
  };
  auto row_norm = [&]() {
#pragma unroll
    for (int j = 0; j < M; ++j) v[j] = __shfl_sync(0xffffffffu, c, ri * M + j);
    float sum = 0.0f;
#pragma unroll
    for (int j = 0; j < M; ++j) sum += v[j];
    c /= (sum + eps);
  };
  col_norm();
  for (int it = 0; it < iters - 1; ++it) {
    row_norm();
    col_norm();
  }
  if (lane < M * M) comb_out[lane] = c;
}

struct HcReduceArgs {
  const double* part;
  int nblk, rows;        // partial blocks; mix rows
  int head;              // 0: layer HC (Sinkhorn split), 1: model head (sigmoid pre)
  const float* scale;    // [3] (layer) or [1] (head)
  const float* base;     // [rows]
  int mult, hid, iters;
  float hc_eps, rms_eps;
  const float* state;    // [mult][hid]
  const uint16_t* norm;  // RMSNorm gain [hid] (BF16)
  float* post;           // [mult] (layer only)
  float* comb;           // [mult * mult] (layer only)
  float* out;            // [hid]: rmsnorm(bf16(pre . state))
};

// hc_pre_scratch (src/dsv4/dsv4_model.c:7123-7153) or model_head (:7190-7216)
// from the partial sums, followed by rmsnorm_bf16 with the gain (:4934).
constexpr int kHcThreads = 1024;
__global__ void __launch_bounds__(kHcThreads) hc_reduce_kernel(const HcReduceArgs a) {
  __shared__ double tot[kMixMax + 1];
  __shared__ float mixes[kMixMax];
  __shared__ float pre_s[kHcMultMax], post_s[kHcMultMax], comb_s[kHcMultMax * kHcMultMax];
  __shared__ double red[kHcThreads / 32];
  pdl_wait();
  pdl_trigger();
  const int n = a.mult * a.hid;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // partial sums: warp w reduces value w over the blocks (a fixed order, so
  // the result is the same on every run)
  for (int j = warp; j <= a.rows; j += kHcThreads / 32) {
    double t = 0.0;
    for (int b = lane; b < a.nblk; b += 32) t += a.part[static_cast<size_t>(b) * (kMixMax + 1) + j];
    t = warp_sum_d(t);
    if (lane == 0) tot[j] = t;
  }
  __syncthreads();
  const float rs = rms_factor(tot[0], n, a.rms_eps);
  if (static_cast<int>(threadIdx.x) < a.rows) mixes[threadIdx.x] = static_cast<float>(tot[1 + threadIdx.x]) * rs;
  __syncthreads();
  if (warp == 0) {
    if (a.head) {
      if (lane < a.mult)
        pre_s[lane] =
            1.0f / (1.0f + expf_r1(-mul_add(mixes[lane], a.scale[0], a.base[lane]))) + a.hc_eps;
    } else {
      switch (a.mult) {
        case 1: hc_split_warp<1>(mixes, a.scale, a.base, a.iters, a.hc_eps, pre_s, post_s, comb_s); break;
        case 2: hc_split_warp<2>(mixes, a.scale, a.base, a.iters, a.hc_eps, pre_s, post_s, comb_s); break;
        case 3: hc_split_warp<3>(mixes, a.scale, a.base, a.iters, a.hc_eps, pre_s, post_s, comb_s); break;
        default: hc_split_warp<4>(mixes, a.scale, a.base, a.iters, a.hc_eps, pre_s, post_s, comb_s); break;
      }
      __syncwarp();
      if (lane < a.mult) a.post[lane] = post_s[lane];
      if (lane < a.mult * a.mult) a.comb[lane] = comb_s[lane];
    }
  }
  __syncthreads();
  // bin = bf16(pre . state), held in registers across the norm's reduction
  constexpr int kPer = 8;  // hid <= kPer * kHcThreads
  float v[kPer];
  double ss = 0.0;
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    const int j = threadIdx.x + k * kHcThreads;
    v[k] = 0.0f;
    if (j < a.hid) {
      float acc = 0.0f;
      for (int i = 0; i < a.mult; ++i)
        acc = fmaf(pre_s[i], a.state[static_cast<size_t>(i) * a.hid + j], acc);
      v[k] = bf16_round(acc);
      ss += static_cast<double>(v[k]) * v[k];
    }
  }
  ss = block_sum_d(ss, red);
  const float r = rms_factor(ss, a.hid, a.rms_eps);
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    const int j = threadIdx.x + k * kHcThreads;
    if (j < a.hid) a.out[j] = bf16_round(__fmul_rn(__fmul_rn(v[k], r), bf16_widen(a.norm[j])));
  }
}

// Sums 32 doubles over a warp with 31 shuffles instead of 160: at each
// level a lane keeps half of its values and trades the other half with its
// partner, so lane l ends with the warp's sum of value l. A fixed butterfly,
// so the same bits on every run.
__device__ __forceinline__ double warp_transpose_sum32(double (&v)[32]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int s = 16; s >= 1; s >>= 1) {
    const bool upper = (lane & s) != 0;
#pragma unroll
    for (int k = 0; k < s; ++k) {
      const double send = upper ? v[k] : v[k + s];
      const double keep = upper ? v[k + s] : v[k];
      v[k] = keep + __shfl_xor_sync(0xffffffffu, send, s);
    }
  }
  return v[0];
}

// One hyper-connection boundary in one launch (the fast mode's path):
// hc_post of the branch that just finished (src/dsv4/dsv4_model.c:7165-7177;
// skipped when branch is null), then hc_pre of the next one (:7123-7153, or
// the model head :7190-7216): the HC mixes of the new state, the pre
// weights (sigmoid of the first mult mixes), the weighted reduce, RMSNorm
// with the gain (:4934) and, when xq is set, the per-128 FP8 quantisation of
// the result (dsv4_quant_fp8_codes, :5580) for the projections that read it.
// The mixes are written out; the Sinkhorn split of the post and comb mixes
// (hc_sinkhorn_kernel) is only needed by the next boundary's post step and
// runs beside the branch.
// Thread = one column of the state (all mult rows): the post update needs
// only the column, so it is done in place; the column's mix partials are
// summed over the CTA into part[cta][32]; the last CTA to arrive (a ticket
// counter it resets) sums the CTAs' partials in CTA order and finishes the
// step. Weights (the mix rows, the norm gain, scale and base) are loaded
// before the wait on the previous kernel.
struct HcFusedArgs {
  float* state;                 // [mult][hid], updated in place
  const float* branch;          // [hid] or null (no post step)
  const float* post_in;         // [mult] from the previous boundary's split
  const float* comb_in;         // [mult][mult]
  const float* fn;              // [rows][mult * hid]
  int rows;                     // (2 + mult) * mult, or mult for the head
  int head;
  const float* scale;           // [3] (layer) or [1] (head)
  const float* base;            // [rows]
  int hid;
  float hc_eps, rms_eps;
  const uint16_t* norm;         // RMSNorm gain [hid] (BF16)
  float* mix_out;               // [rows] the mixes (for the split)
  float* out;                   // [hid]
  __half* xq;                   // optional FP8-grid quant of out [hid]
  float* xs;                    // [hid / 128] its scales
  double* part;                 // [gridDim.x][32]
  unsigned int* ticket;         // zero between launches
  // verify steps (gridDim.y rows): row r's buffers follow row 0's at these
  // strides - state mult*hid, branch/out hid, post kHcMultMax, comb
  // kHcMultMax^2, mix kMixMax, xq xq_ld (xs xq_ld / 128), part part_rs,
  // ticket 1
  int xq_ld;
  size_t part_rs;
};

template <int M>
__device__ __forceinline__ HcFusedArgs hc_row(HcFusedArgs a, int r) {
  if (r == 0) return a;
  const size_t hid = static_cast<size_t>(a.hid);
  a.state += r * M * hid;
  if (a.branch) a.branch += r * hid;
  a.post_in += r * kHcMultMax;
  a.comb_in += r * kHcMultMax * kHcMultMax;
  a.mix_out += r * kMixMax;
  a.out += r * hid;
  if (a.xq) {
    a.xq += static_cast<size_t>(r) * a.xq_ld;
    a.xs += static_cast<size_t>(r) * (a.xq_ld / 128);
  }
  a.part += r * a.part_rs;
  a.ticket += r;
  return a;
}

constexpr int kHcfThreads = 256;
constexpr int kHcfMaxCtas = 128;  // hid <= 8192 at 64 columns per CTA
constexpr int kHcfPer = 8;        // tail chunks of 4 columns per thread: hid <= 8 * 256 * 4

// Unit u of a boundary: the state columns [u COLS, (u + 1) COLS), thread =
// (row m, column). hc_unit_load: the unit's mix weights (before the wait on
// the previous work) and the gain row toward L2; hc_unit_run: the post step
// in place and the unit's mix partials, summed over the CTA into part[u].
template <int M>
__device__ __forceinline__ void hc_unit_load(const HcFusedArgs& a, int u, float (&f)[(2 + M) * M]) {
  constexpr int R = (2 + M) * M;
  constexpr int COLS = kHcfThreads / M;
  const int tid = threadIdx.x;
  const int m = tid / COLS, ic = tid - m * COLS;
  const int i = u * COLS + ic;
  const bool col = m < M && i < a.hid;
  const size_t n = static_cast<size_t>(M) * a.hid;
  const size_t e_mi = col ? static_cast<size_t>(m) * a.hid + i : 0;
#pragma unroll
  for (int j = 0; j < R; ++j) f[j] = (col && j < a.rows) ? __ldg(a.fn + j * n + e_mi) : 0.f;
  for (int o = tid * 128; o < a.hid * 2; o += static_cast<int>(blockDim.x) * 128)
    asm volatile("prefetch.global.L2 [%0];" ::"l"(reinterpret_cast<const char*>(a.norm) + o));
}

template <int M>
__device__ __forceinline__ void hc_unit_run(const HcFusedArgs& a, int u, const float (&f)[(2 + M) * M],
                                            double (*red)[32]) {
  constexpr int R = (2 + M) * M;
  constexpr int COLS = kHcfThreads / M;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int m = tid / COLS, ic = tid - m * COLS;
  const int i = u * COLS + ic;
  const bool col = m < M && i < a.hid;
  const size_t e_mi = col ? static_cast<size_t>(m) * a.hid + i : 0;
  float v = 0.f;
  if (a.branch) {
    float old[M];
#pragma unroll
    for (int k = 0; k < M; ++k) old[k] = col ? a.state[static_cast<size_t>(k) * a.hid + i] : 0.f;
    __syncthreads();  // the CTA's columns are read whole before any row is rewritten
    if (col) {
      float y = __fmul_rn(a.post_in[m], a.branch[i]);
#pragma unroll
      for (int k = 0; k < M; ++k) y = fmaf(a.comb_in[m * M + k], old[k], y);
      v = bf16_round(y);
      a.state[e_mi] = v;
    }
  } else if (col) {
    v = a.state[e_mi];
  }
  double p[32];
  p[0] = static_cast<double>(v) * v;
#pragma unroll
  for (int j = 0; j < 31; ++j) p[1 + j] = j < R ? static_cast<double>(f[j]) * v : 0.0;
  red[warp][lane] = warp_transpose_sum32(p);
  __syncthreads();
  if (tid < 32) {
    double t = 0.0;
#pragma unroll
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) t += red[w][tid];
    a.part[static_cast<size_t>(u) * 32 + tid] = t;
  }
}

// The boundary's tail on one CTA once every unit's partials are written:
// the mixes (summed in unit order), the pre weights, the bin, RMSNorm,
// the optional quant. pall: n_units * 32 doubles of shared memory.
template <int M>
__device__ void hc_tail(const HcFusedArgs& a, int n_units, double* pall) {
  __shared__ double tot[32];
  __shared__ double red2[32];
  __shared__ float pre_s[kHcMultMax];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nt = blockDim.x;  // columns are dealt 4 per thread, nt threads per chunk
  const size_t n = static_cast<size_t>(M) * a.hid;
  const float sc0 = __ldg(a.scale);
  const float bs = lane < M ? __ldg(a.base + lane) : 0.f;
  uint16_t g4[kHcfPer][4];
#pragma unroll
  for (int k = 0; k < kHcfPer; ++k) {
    const int c0 = (k * nt + tid) * 4;
#pragma unroll
    for (int e = 0; e < 4; ++e) g4[k][e] = c0 < a.hid ? __ldg(a.norm + c0 + e) : uint16_t(0);
  }
  // the state's first four chunks, every CTA's partials: all loads in flight
  // together; the partials are then summed in CTA order
  float4 sv[4][M];
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
    const int cc = (kk * nt + tid) * 4;
#pragma unroll
    for (int mm = 0; mm < M; ++mm)
      sv[kk][mm] = cc < a.hid ? __ldcg(reinterpret_cast<const float4*>(a.state + static_cast<size_t>(mm) * a.hid + cc))
                              : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  for (int e = tid; e < n_units * 32; e += nt) pall[e] = __ldcg(a.part + e);
  __syncthreads();
  if (tid < 32) {
    double t = 0.0;
    for (int b = 0; b < n_units; ++b) t += pall[b * 32 + tid];
    tot[tid] = t;
  }
  __syncthreads();
  const float rs = rms_factor(tot[0], static_cast<int>(n), a.rms_eps);
  if (warp == 0) {
    const float mix = lane < a.rows ? static_cast<float>(tot[1 + lane]) * rs : 0.f;
    if (lane < a.rows) a.mix_out[lane] = mix;
    if (lane < M) {
      const float z = mul_add(mix, sc0, bs);
      // the head's pre (src/dsv4/dsv4_model.c:7203-7206) or the layer's
      // (dsv4_hc_split, src/dsv4/dsv4_ops.c:418)
      pre_s[lane] = (a.head ? 1.0f / (1.0f + expf_r1(-z)) : sigmoid_stable(z)) + a.hc_eps;
    }
  }
  __syncthreads();
  // bin = bf16(pre . state) over 4 consecutive columns per chunk, the norm
  float y[kHcfPer][4];
  double ss = 0.0;
#pragma unroll
  for (int k = 0; k < kHcfPer; ++k) {
    const int c0 = (k * nt + tid) * 4;
    if (k > 0 && k % 4 == 0 && k * nt * 4 < a.hid) {
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const int cc = ((k + kk) * nt + tid) * 4;
#pragma unroll
        for (int mm = 0; mm < M; ++mm)
          sv[kk][mm] = cc < a.hid ? __ldcg(reinterpret_cast<const float4*>(a.state + static_cast<size_t>(mm) * a.hid + cc))
                                  : make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) y[k][e] = 0.f;
    if (c0 < a.hid) {
      const float4* s = sv[k % 4];
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int mm = 0; mm < M; ++mm) {
        acc[0] = fmaf(pre_s[mm], s[mm].x, acc[0]);
        acc[1] = fmaf(pre_s[mm], s[mm].y, acc[1]);
        acc[2] = fmaf(pre_s[mm], s[mm].z, acc[2]);
        acc[3] = fmaf(pre_s[mm], s[mm].w, acc[3]);
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        y[k][e] = bf16_round(acc[e]);
        ss += static_cast<double>(y[k][e]) * y[k][e];
      }
    }
  }
  ss = block_sum_d(ss, red2);
  const float r = rms_factor(ss, a.hid, a.rms_eps);
#pragma unroll
  for (int k = 0; k < kHcfPer; ++k) {
    const int c0 = (k * nt + tid) * 4;
    if (k * nt * 4 >= a.hid) break;  // uniform over the CTA
    const float gn[4] = {bf16_widen(g4[k][0]), bf16_widen(g4[k][1]), bf16_widen(g4[k][2]),
                         bf16_widen(g4[k][3])};
    float o[4];
    float amax = 0.f;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      o[e] = c0 < a.hid ? bf16_round(__fmul_rn(__fmul_rn(y[k][e], r), gn[e])) : 0.f;
      amax = fmaxf(amax, fabsf(o[e]));
    }
    if (c0 < a.hid) *reinterpret_cast<float4*>(a.out + c0) = make_float4(o[0], o[1], o[2], o[3]);
    if (a.xq) {
      // this warp's 32 x 4 columns are one 128-column quantisation block
      amax = warp_max(amax);
      const float scale = pow2_scale_448(amax);
      const float inv = 1.0f / scale;
      if (c0 < a.hid) {
        if (lane == 0) a.xs[c0 / 128] = scale;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float q = o[e] * inv;
          q = q > 448.f ? 448.f : (q < -448.f ? -448.f : q);
          a.xq[c0 + e] = e4m3_round_f16(q);
        }
      }
    }
  }
}

template <int M>
__global__ void __launch_bounds__(kHcfThreads) hc_fused_kernel(const HcFusedArgs a0) {
  const HcFusedArgs a = hc_row<M>(a0, blockIdx.y);
  __shared__ double red[kHcfThreads / 32][32];
  __shared__ double pall[kHcfMaxCtas * 32];
  __shared__ int last;
  pdl_trigger();
  float f[(2 + M) * M];
  hc_unit_load<M>(a, blockIdx.x, f);
  pdl_wait();
  hc_unit_run<M>(a, blockIdx.x, f, red);
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    last = atomicAdd(a.ticket, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  if (threadIdx.x == 0) *a.ticket = 0u;
  hc_tail<M>(a, gridDim.x, pall);
}

// The Sinkhorn split of a layer boundary's mixes (dsv4_hc_split,
// src/dsv4/dsv4_ops.c:412-460) into the post weights and the comb matrix
// the next boundary's post step applies. One warp.
// CTA r splits row r's mixes (verify steps: one CTA per row, the hc_row
// strides).
template <int M>
__global__ void hc_sinkhorn_kernel(const float* mix, const float* scale, const float* base, int iters,
                                   float eps, float* post, float* comb) {
  __shared__ float pre_s[kHcMultMax], post_s[kHcMultMax], comb_s[kHcMultMax * kHcMultMax];
  mix += blockIdx.x * kMixMax;
  post += blockIdx.x * kHcMultMax;
  comb += blockIdx.x * kHcMultMax * kHcMultMax;
  hc_split_warp<M>(mix, scale, base, iters, eps, pre_s, post_s, comb_s);
  __syncwarp();
  const int lane = threadIdx.x;
  if (lane < M) post[lane] = post_s[lane];
  if (lane < M * M) comb[lane] = comb_s[lane];
}

// rmsnorm_bf16 with a gain (src/dsv4/dsv4_model.c:4934), optionally followed
// by dsv4_rope_apply_buf on the last 2 * half dims (:1547-1558), kept in
// shared memory and handed straight to its consumer in the same launch: the
// per-128 FP8 quantisation of the q latent for wq_b (xq set), or the KV
// write of the kv latent into its ring row (kv_quant_group per 64 dims, the
// RoPE dims as BF16; cache.codes set). One CTA.
struct NormTailArgs {
  const float* x;
  int n;
  const uint16_t* w;
  float eps;
  int half;
  const float* cosv;
  const float* sinv;
  __half* xq;             // optional: FP8-grid quant of the result
  float* xs;
  Fp8KvCache cache;       // optional (codes != null): KV write at *row
  const long long* row;
  // with the KV write: the window's rows as BF16, win[t] = the cached value
  // of ring row idx[t] (zeros for padding); CTA 0 provides the new row,
  // CTAs 1.. decode the others from the cache (null: no staging)
  uint16_t* win;          // [n_win][nope + rope]
  const int* idx;         // [n_win]
  int n_win;
  // verify steps (gridDim.y rows): row r reads x + r x_rs, quantises into
  // xq + r xq_ld (xs + r xq_ld / 128), takes cos/sin + r cs_rs, writes
  // ring row row[r] and stages into win + r n_win d from idx + r n_win
  int x_rs, xq_ld, cs_rs;
};

__device__ __forceinline__ NormTailArgs norm_row(NormTailArgs a, int r) {
  if (r == 0) return a;
  a.x += static_cast<size_t>(r) * a.x_rs;
  if (a.xq) {
    a.xq += static_cast<size_t>(r) * a.xq_ld;
    a.xs += static_cast<size_t>(r) * (a.xq_ld / 128);
  }
  if (a.cosv) {
    a.cosv += static_cast<size_t>(r) * a.cs_rs;
    a.sinv += static_cast<size_t>(r) * a.cs_rs;
  }
  if (a.row) a.row += r;
  if (a.idx) a.idx += static_cast<size_t>(r) * a.n_win;
  if (a.win) a.win += static_cast<size_t>(r) * a.n_win * (a.cache.nope + a.cache.rope_dim);
  return a;
}

// Rows [t0, t1) of the window into win (warp = row, lane = 16 dims), all
// but the ring row `skip` (being rewritten by CTA 0; kNoSkipRow: none).
// Padding keys (idx -1) are staged as zeros.
constexpr long long kNoSkipRow = -2;
__device__ void stage_window_rows(const NormTailArgs& a, long long skip, int cta, int n_cta) {
  const Fp8KvCache& c = a.cache;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int d = c.nope + c.rope_dim, pieces = d / 16, np16 = c.nope / 16;
  for (int t = cta * nw + warp; t < a.n_win; t += n_cta * nw) {
    const int r = a.idx[t];
    if (r == skip || lane >= pieces) continue;
    const bool live = r >= 0 && r < c.rows;
    uint4 o0 = make_uint4(0u, 0u, 0u, 0u), o1 = o0;
    if (live && lane < np16) {
      const uint4 raw = *reinterpret_cast<const uint4*>(c.codes + static_cast<size_t>(r) * c.nope + 16 * lane);
      const float sc = e8m0_decode(c.scales[static_cast<size_t>(r) * kKvScaleSlots + lane / 4]);
      const uint32_t cw[4] = {raw.x, raw.y, raw.z, raw.w};
      uint32_t o[8];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        uint32_t h01, h23;
        asm("{ .reg .b16 lo, hi; mov.b32 {lo, hi}, %2; cvt.rn.f16x2.e4m3x2 %0, lo;"
            " cvt.rn.f16x2.e4m3x2 %1, hi; }"
            : "=r"(h01), "=r"(h23) : "r"(cw[k]));
        const __half2 p01 = *reinterpret_cast<const __half2*>(&h01);
        const __half2 p23 = *reinterpret_cast<const __half2*>(&h23);
        o[2 * k] = pack_bf16x2(__fmul_rn(__low2float(p01), sc), __fmul_rn(__high2float(p01), sc));
        o[2 * k + 1] = pack_bf16x2(__fmul_rn(__low2float(p23), sc), __fmul_rn(__high2float(p23), sc));
      }
      o0 = make_uint4(o[0], o[1], o[2], o[3]);
      o1 = make_uint4(o[4], o[5], o[6], o[7]);
    } else if (live) {
      const uint16_t* rp = c.rope + static_cast<size_t>(r) * c.rope_dim + 16 * (lane - np16);
      o0 = *reinterpret_cast<const uint4*>(rp);
      o1 = *reinterpret_cast<const uint4*>(rp + 8);
    }
    uint4* dst = reinterpret_cast<uint4*>(a.win + static_cast<size_t>(t) * d + 16 * lane);
    dst[0] = o0;
    dst[1] = o1;
  }
}

// One norm CTA (any multiple of 32 threads); ys: a.n floats of shared memory. The gain is
// loaded before `wait` runs (the PDL wait of a standalone launch).
template <class Wait>
__device__ void norm_tail_run(const NormTailArgs& a, float* ys, Wait wait) {
  __shared__ double red[32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // up to kPer values per thread in registers, all loads in flight at once
  // (the gain before the wait: it is a weight); longer rows in rounds
  constexpr int kPer = 4;
  const int step = blockDim.x * kPer;
  float g[kPer];
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    const int i = tid + k * blockDim.x;
    g[k] = i < a.n ? bf16_widen(a.w[i]) : 0.f;
  }
  wait();
  double ss = 0.0;
  for (int i0 = 0; i0 < a.n; i0 += step) {
    float v[kPer];
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      const int i = i0 + tid + k * blockDim.x;
      v[k] = i < a.n ? a.x[i] : 0.f;
    }
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      const int i = i0 + tid + k * blockDim.x;
      if (i < a.n) {
        ss += static_cast<double>(v[k]) * v[k];
        ys[i] = v[k];
      }
    }
  }
  ss = block_sum_d(ss, red);
  const float r = rms_factor(ss, a.n, a.eps);
  for (int i0 = 0; i0 < a.n; i0 += step) {
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      const int i = i0 + tid + k * blockDim.x;
      if (i < a.n)
        ys[i] = bf16_round(__fmul_rn(__fmul_rn(ys[i], r), i0 == 0 ? g[k] : bf16_widen(a.w[i])));
    }
  }
  __syncthreads();
  if (a.half > 0) {
    const int start = a.n - 2 * a.half;
    for (int i = tid; i < a.half; i += blockDim.x) {
      const float x0 = ys[start + 2 * i], x1 = ys[start + 2 * i + 1];
      const float c = a.cosv[i], s = a.sinv[i];
      ys[start + 2 * i] = bf16_round(__fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s)));
      ys[start + 2 * i + 1] = bf16_round(__fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c)));
    }
    __syncthreads();
  }
  if (a.xq) {
    for (int b = warp; b < (a.n + 127) / 128; b += blockDim.x >> 5) {
      const int len = min(128, a.n - b * 128);
      float v[4];
      float amax = 0.f;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int i = lane + 32 * k;
        v[k] = i < len ? ys[b * 128 + i] : 0.f;
        amax = fmaxf(amax, fabsf(v[k]));
      }
      amax = warp_max(amax);
      const float scale = pow2_scale_448(amax);
      const float inv = 1.0f / scale;
      if (lane == 0) a.xs[b] = scale;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int i = lane + 32 * k;
        if (i >= len) continue;
        float q = v[k] * inv;
        q = q > 448.f ? 448.f : (q < -448.f ? -448.f : q);
        a.xq[b * 128 + i] = e4m3_round_f16(q);
      }
    }
  }
  if (a.cache.codes) {
    const long long rr = *a.row;
    if (rr < 0 || rr >= a.cache.rows) return;
    __shared__ int tw_s;  // the new row's window slot
    if (tid == 0) tw_s = -1;
    __syncthreads();
    if (a.win)
      for (int t = tid; t < a.n_win; t += blockDim.x)
        if (a.idx[t] == rr) tw_s = t;
    __syncthreads();
    const int tw = tw_s;
    const int d = a.cache.nope + a.cache.rope_dim;
    for (int g = warp; g < a.cache.nope / 64; g += blockDim.x >> 5) {
      kv_quant_group(a.cache, rr, g, ys[g * 64 + lane], ys[g * 64 + 32 + lane], lane);
      if (tw >= 0) {
        // the cached value of what was just written: bf16(e4m3 * 2^k)
        __syncwarp();
        const uint8_t* cd = a.cache.codes + rr * a.cache.nope + g * 64;
        const float sc = e8m0_decode(a.cache.scales[rr * kKvScaleSlots + g]);
        uint16_t* wr = a.win + static_cast<size_t>(tw) * d + g * 64;
        wr[lane] = static_cast<uint16_t>(__float_as_uint(bf16_round(__fmul_rn(e4m3_decode(cd[lane]), sc))) >> 16);
        wr[32 + lane] =
            static_cast<uint16_t>(__float_as_uint(bf16_round(__fmul_rn(e4m3_decode(cd[32 + lane]), sc))) >> 16);
      }
    }
    for (int i = tid; i < a.cache.rope_dim; i += blockDim.x) {
      const uint16_t b = static_cast<uint16_t>(__float_as_uint(bf16_round(ys[a.cache.nope + i])) >> 16);
      a.cache.rope[rr * a.cache.rope_dim + i] = b;
      if (tw >= 0) a.win[static_cast<size_t>(tw) * d + a.cache.nope + i] = b;
    }
  }
}

// CTA 0 runs `a0`; CTA 1 runs `a1` when a1.x is set (two independent
// norms in one launch); the remaining CTAs stage a0's window. blockIdx.y
// selects the row of a verify step (norm_row).
__global__ void __launch_bounds__(256) norm_tail_kernel(const NormTailArgs a0, const NormTailArgs a1) {
  extern __shared__ float ys[];  // [n]
  pdl_trigger();
  const int n_norm = a1.x ? 2 : 1;
  if (static_cast<int>(blockIdx.x) >= n_norm) {
    pdl_wait();
    const NormTailArgs a = norm_row(a0, blockIdx.y);
    stage_window_rows(a, *a.row, blockIdx.x - n_norm, gridDim.x - n_norm);
    return;
  }
  norm_tail_run(norm_row(blockIdx.x == 0 ? a0 : a1, blockIdx.y), ys, [] { pdl_wait(); });
}

// A verify step's window staging, after every row's latent is in the cache
// (the rows' windows include the other verify rows' scratch rows):
// blockIdx.y = row, the CTAs along x share its window.
__global__ void __launch_bounds__(256) stage_rows_kernel(const NormTailArgs a0) {
  pdl_wait();
  pdl_trigger();
  stage_window_rows(norm_row(a0, blockIdx.y), kNoSkipRow, blockIdx.x, gridDim.x);
}

// Per-head RMS of q and its RoPE (src/dsv4/dsv4_model.c:5283-5291), one CTA
// per head; q is updated in place.
__global__ void __launch_bounds__(128) q_head_kernel(float* q, int d, float eps, int half,
                                                     const float* cosv, const float* sinv) {
  __shared__ double red[4];
  __shared__ float qs[512];
  pdl_trigger();
  pdl_wait();
  float* qh = q + static_cast<size_t>(blockIdx.x) * d;
  // d <= 512: four values per thread, loaded together
  float v[4];
  double ss = 0.0;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int i = threadIdx.x + 128 * k;
    v[k] = i < d ? qh[i] : 0.f;
  }
#pragma unroll
  for (int k = 0; k < 4; ++k) ss += static_cast<double>(v[k]) * v[k];
  ss = block_sum_d(ss, red);
  const float rr = rms_factor(ss, d, eps);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int i = threadIdx.x + 128 * k;
    if (i < d) qs[i] = bf16_round(__fmul_rn(v[k], rr));
  }
  __syncthreads();
  const int start = d - 2 * half;
  for (int i = threadIdx.x; i < half; i += blockDim.x) {
    const float x0 = qs[start + 2 * i], x1 = qs[start + 2 * i + 1];
    const float c = cosv[i], s = sinv[i];
    qs[start + 2 * i] = bf16_round(__fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s)));
    qs[start + 2 * i + 1] = bf16_round(__fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c)));
  }
  __syncthreads();
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int i = threadIdx.x + 128 * k;
    if (i < d) qh[i] = qs[i];
  }
}

// ---- exact-order attention over the sliding window ----
// sparse_attn (src/dsv4/dsv4_model.c:5767-5822) step for step: per (head,
// key) the 512-long fmaf dot in dimension order times the scale; per head
// the max, the denominator expf(sink - m) + sum expf(s - m) added in key
// order, the BF16 weights; per (head, dim) the fmaf chain over the keys in
// key order, divided by the denominator and rounded to BF16; then the
// inverse RoPE of :5373. The expf is the once-rounded one (dsv4_common.cuh).
// Used for the decode step's window of at most a few hundred keys, where it
// is also faster than the tensor-core kernel built for long contexts.
struct WinAttnArgs {
  const float* q;             // [H][d], BF16-valued
  Fp8KvCache cache;
  const int* idx;             // [n], -1 = padding
  const float* sink;          // [H]
  const float* cosv;          // [rope_dim / 2] of the position
  const float* sinv;
  int H, d, n, rope_dim;
  float scale;
  float* kvdec;               // scratch [n][d]: the keys' cached values
  float* kvt;                 // scratch [d][n]: the same, transposed
  float* s;                   // scratch [H][n] scores
  float* w;                   // scratch [H][n] BF16 weights
  float* den;                 // scratch [H] denominators
  float* out;                 // [H][d]
  // win_head_kernel only: q arrives before its per-head RMS and RoPE
  // (q_head_kernel's step, done by the head's CTA) when q_raw is set
  int q_raw;
  float q_eps;
  // win_head_kernel on a verify step (gridDim.y rows): row r's q, out at
  // + r H d, idx + r n, cos/sin + r rope_dim / 2, staged window + r n d
};

__device__ __forceinline__ float cache_value(const Fp8KvCache& c, long long r, int i) {
  // the reference's cached value: bf16(e4m3 * 2^k) on the non-RoPE dims
  if (i < c.nope)
    return bf16_round(__fmul_rn(e4m3_decode(c.codes[r * c.nope + i]),
                                e8m0_decode(c.scales[r * kKvScaleSlots + i / 64])));
  return bf16_widen(c.rope[r * c.rope_dim + (i - c.nope)]);
}

// The window's cached rows, decoded once into kvdec [n][d] and its transpose
// kvt [d][n] (each read coalesced by one of the next kernels). Padding keys get
// zeros (their BF16 weight is 0 too, so a chain term 0 * 0 adds +0 and
// leaves the chain's value as the reference's skip does: the chains start
// at +0 and never hold -0).
__global__ void win_decode_kernel(const WinAttnArgs a) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x;
  const int r = a.idx[t];
  const bool live = r >= 0 && r < a.cache.rows;
  for (int i = threadIdx.x; i < a.d; i += blockDim.x) {
    const float v = live ? cache_value(a.cache, r, i) : 0.0f;
    a.kvdec[static_cast<size_t>(t) * a.d + i] = v;
    a.kvt[static_cast<size_t>(i) * a.n + t] = v;
  }
}

// Scores: CTA = kWinHeads heads (warps) x 32 keys (lanes). The keys' cached
// columns [d][32] are staged in shared memory from the transposed copy (lane
// t reads word t of each row: distinct banks), the heads' q rows beside
// them; each thread runs its (head, key) dot as one fmaf chain in dimension
// order, times the scale.
constexpr int kWinHeads = 8, kWinKeys = 32;
__global__ void __launch_bounds__(kWinHeads * 32) win_scores_kernel(const WinAttnArgs a) {
  extern __shared__ __align__(16) float sm[];  // q [kWinHeads][d], k [d][kWinKeys]
  pdl_wait();
  pdl_trigger();
  const int h0 = blockIdx.x * kWinHeads, t0 = blockIdx.y * kWinKeys;
  float* qs = sm;
  float* ks = sm + kWinHeads * a.d;
  const int d4 = a.d / 4;
  for (int e = threadIdx.x; e < kWinHeads * d4; e += blockDim.x) {
    const int hh = e / d4, i4 = e - hh * d4;
    const int h = h0 + hh;
    reinterpret_cast<float4*>(qs)[e] =
        h < a.H ? reinterpret_cast<const float4*>(a.q + static_cast<size_t>(h) * a.d)[i4]
                : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  for (int e = threadIdx.x; e < a.d * (kWinKeys / 4); e += blockDim.x) {
    const int i = e / (kWinKeys / 4), t4 = e - i * (kWinKeys / 4);
    const int t = t0 + 4 * t4;  // n is a multiple of 4: a group is all in or all out
    reinterpret_cast<float4*>(ks)[e] =
        t < a.n ? *reinterpret_cast<const float4*>(a.kvt + static_cast<size_t>(i) * a.n + t)
                : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  __syncthreads();
  const int lane = threadIdx.x & 31, hw = threadIdx.x >> 5;
  const int h = h0 + hw, t = t0 + lane;
  if (h >= a.H || t >= a.n) return;
  float st = -INFINITY;
  const int r = a.idx[t];
  if (r >= 0 && r < a.cache.rows) {
    const float* q = qs + hw * a.d;
    float dot = 0.0f;
#pragma unroll 16
    for (int i = 0; i < a.d; ++i) dot = fmaf(q[i], ks[i * kWinKeys + lane], dot);
    st = __fmul_rn(dot, a.scale);
  }
  a.s[static_cast<size_t>(h) * a.n + t] = st;
}

// CTA h: the head's max, exponentials, BF16 weights and the denominator
// summed in key order by thread 0.
__global__ void __launch_bounds__(256) win_softmax_kernel(const WinAttnArgs a) {
  extern __shared__ float ex[];
  __shared__ float red[8];
  pdl_wait();
  pdl_trigger();
  const int h = blockIdx.x;
  const float* sh = a.s + static_cast<size_t>(h) * a.n;
  float mxl = -INFINITY;
  for (int t = threadIdx.x; t < a.n; t += blockDim.x) mxl = fmaxf(mxl, sh[t]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mxl = fmaxf(mxl, __shfl_xor_sync(0xffffffffu, mxl, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mxl;
  __syncthreads();
  float mx = red[0];
  for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w) mx = fmaxf(mx, red[w]);
  for (int t = threadIdx.x; t < a.n; t += blockDim.x) {
    const float st = sh[t];
    const bool live = st != -INFINITY;
    const float e = live ? expf_r1(st - mx) : 0.0f;
    ex[t] = e;
    a.w[static_cast<size_t>(h) * a.n + t] = live ? bf16_round(e) : 0.0f;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float sum = expf_r1(a.sink[h] - mx);
    for (int t = 0; t < a.n; ++t)
      if (sh[t] != -INFINITY) sum += ex[t];
    a.den[h] = sum;
  }
}

// CTA (h, 128-dim block), thread = dimension pair: the two value chains
// over the keys in key order, the division, BF16, and the inverse RoPE of
// the pair when it lies in the RoPE dims.
__global__ void __launch_bounds__(64) win_values_kernel(const WinAttnArgs a) {
  extern __shared__ float ws[];  // w_h [n]
  pdl_wait();
  pdl_trigger();
  const int h = blockIdx.x;
  for (int t = threadIdx.x; t < a.n; t += blockDim.x) ws[t] = a.w[static_cast<size_t>(h) * a.n + t];
  __syncthreads();
  const int pairs = a.d / 2;
  for (int p = blockIdx.y * 64 + threadIdx.x; p < min(pairs, (blockIdx.y + 1) * 64);
       p += blockDim.x) {
    const int i = 2 * p;
    float o0 = 0.0f, o1 = 0.0f;
    // 32 keys' rows requested ahead of their fmaf (the chains wait on L2)
#pragma unroll 32
    for (int t = 0; t < a.n; ++t) {
      const float2 kv = *reinterpret_cast<const float2*>(a.kvdec + static_cast<size_t>(t) * a.d + i);
      o0 = fmaf(ws[t], kv.x, o0);
      o1 = fmaf(ws[t], kv.y, o1);
    }
    const float den = a.den[h];
    float x0 = bf16_round(o0 / den), x1 = bf16_round(o1 / den);
    const int start = a.d - a.rope_dim;
    if (a.cosv && i >= start) {
      const int k = (i - start) / 2;
      const float c = a.cosv[k], sn = a.sinv[k];
      const float y0 = bf16_round(__fadd_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn)));
      const float y1 = bf16_round(__fadd_rn(__fmul_rn(-x0, sn), __fmul_rn(x1, c)));
      x0 = y0;
      x1 = y1;
    }
    float* oh = a.out + static_cast<size_t>(h) * a.d;
    oh[i] = x0;
    oh[i + 1] = x1;
  }
}

// The softmax and value pass for long key lists (a compressed layer's
// window + compressed rows), one launch: CTA (head, 256-dim block). Each
// CTA takes its head's max over the scores, the exponentials (ex) and
// their BF16 weights into shared memory, as win_softmax_kernel; then thread
// = dimension pair, the two value chains over the keys in key order with
// the keys' rows streamed through shared memory in chunks of kValKeys
// (coalesced loads; the next chunk held in registers while this one is
// consumed). Warp 0 adds the denominator expf(sink - m) + ex[0] + ex[1] ...
// in key order beside its chains (a dead key's ex is +0, which leaves the
// sum as the reference's skip does: the sum starts positive or +0).
constexpr int kValKeys = 32;
constexpr int kValThreads = 128;  // 256 dims per CTA
size_t win_values_long_smem(int n) {
  return sizeof(float) * (2 * ((static_cast<size_t>(n) + 3) & ~static_cast<size_t>(3)) +
                          kValKeys * 2 * kValThreads);
}
__global__ void __launch_bounds__(kValThreads) win_values_long_kernel(const WinAttnArgs a) {
  extern __shared__ __align__(16) float vsm[];  // ws [n4] | ex [n4] | rows [kValKeys][256]
  __shared__ float red[kValThreads / 32];
  pdl_wait();
  pdl_trigger();
  const int h = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int n = a.n, d = a.d, n4 = (n + 3) & ~3;
  const int cols = 2 * kValThreads;
  const int col0 = blockIdx.y * cols;
  float* ws = vsm;
  float* ex = vsm + n4;
  float* rows = ex + n4;
  const float* sh = a.s + static_cast<size_t>(h) * n;
  float mxl = -INFINITY;
  for (int t = tid; t < n; t += kValThreads) mxl = fmaxf(mxl, sh[t]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mxl = fmaxf(mxl, __shfl_xor_sync(0xffffffffu, mxl, o));
  if (lane == 0) red[warp] = mxl;
  __syncthreads();
  float mx = red[0];
#pragma unroll
  for (int w = 1; w < kValThreads / 32; ++w) mx = fmaxf(mx, red[w]);
  for (int t = tid; t < n; t += kValThreads) {
    const float st = sh[t];
    const bool live = st != -INFINITY;
    const float e = live ? expf_r1(st - mx) : 0.0f;
    ex[t] = e;
    ws[t] = live ? bf16_round(e) : 0.0f;
  }
  // each thread moves kValKeys * cols / 4 / kValThreads float4 per chunk
  constexpr int kPer = kValKeys * 2 * kValThreads / 4 / kValThreads;  // 16
  float4 buf[kPer];
  auto fetch = [&](int c0) {
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      const int e = k * kValThreads + tid;      // float4 index within the chunk
      const int t = e / (cols / 4), c4 = e - t * (cols / 4);
      const int col = col0 + 4 * c4;
      buf[k] = (c0 + t < n && col < d)
                   ? *reinterpret_cast<const float4*>(a.kvdec + static_cast<size_t>(c0 + t) * d + col)
                   : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  };
  fetch(0);
  const int p = col0 / 2 + tid;  // this thread's dimension pair
  const bool live = 2 * p < d;
  float o0 = 0.0f, o1 = 0.0f;
  float den = expf_r1(a.sink[h] - mx);
  for (int c0 = 0; c0 < n; c0 += kValKeys) {
    __syncthreads();  // the previous chunk is consumed (and ws, ex are in)
#pragma unroll
    for (int k = 0; k < kPer; ++k)
      reinterpret_cast<float4*>(rows)[k * kValThreads + tid] = buf[k];
    __syncthreads();
    if (c0 + kValKeys < n) fetch(c0 + kValKeys);
    const int nk = min(kValKeys, n - c0);
    if (warp == 0) {
#pragma unroll 8
      for (int t = 0; t < nk; ++t) {
        const float2 kv = reinterpret_cast<const float2*>(rows + t * cols)[tid];
        const float wt = ws[c0 + t];
        o0 = fmaf(wt, kv.x, o0);
        o1 = fmaf(wt, kv.y, o1);
        den = __fadd_rn(den, ex[c0 + t]);
      }
    } else {
#pragma unroll 8
      for (int t = 0; t < nk; ++t) {
        const float2 kv = reinterpret_cast<const float2*>(rows + t * cols)[tid];
        const float wt = ws[c0 + t];
        o0 = fmaf(wt, kv.x, o0);
        o1 = fmaf(wt, kv.y, o1);
      }
    }
  }
  if (warp == 0 && lane == 0) red[0] = den;
  __syncthreads();
  den = red[0];
  if (blockIdx.y == 0 && tid == 0) a.den[h] = den;
  if (!live) return;
  const int i = 2 * p;
  float x0 = bf16_round(o0 / den), x1 = bf16_round(o1 / den);
  const int start = d - a.rope_dim;
  if (a.cosv && i >= start) {
    const int k = (i - start) / 2;
    const float c = a.cosv[k], sn = a.sinv[k];
    const float y0 = bf16_round(__fadd_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn)));
    const float y1 = bf16_round(__fadd_rn(__fmul_rn(-x0, sn), __fmul_rn(x1, c)));
    x0 = y0;
    x1 = y1;
  }
  float* oh = a.out + static_cast<size_t>(h) * d;
  oh[i] = x0;
  oh[i + 1] = x1;
}

// 16-byte global -> shared copies that bypass the registers (cp.async,
// L2 only), and the wait for every copy this thread issued.
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  const unsigned sa = static_cast<unsigned>(__cvta_generic_to_shared(dst));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(sa), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

// Scores for long key lists (a compressed layer's window + compressed
// rows): CTA = kWinHeads heads (warps) x kWinKeys keys (lanes), as
// win_scores_kernel, with the heads' q rows and the keys' decoded rows
// (kvdec [n][d], rows padded to d + 4 floats: a quarter-warp's 16-byte reads
// of 8 rows hit distinct banks) copied to shared memory by cp.async, all in
// flight together. Each thread runs its (head, key) dot as one fmaf chain in
// dimension order, four dimensions per pair of shared-memory reads, times
// the scale. Needs d % 4 == 0.
size_t win_scores_rows_smem(int d) {
  return sizeof(float) * (static_cast<size_t>(kWinHeads) * d + static_cast<size_t>(kWinKeys) * (d + 4));
}
__global__ void __launch_bounds__(kWinHeads * 32) win_scores_rows_kernel(const WinAttnArgs a) {
  extern __shared__ __align__(16) float rsm[];  // q [kWinHeads][d] | k [kWinKeys][d + 4]
  pdl_wait();
  pdl_trigger();
  const int h0 = blockIdx.x * kWinHeads, t0 = blockIdx.y * kWinKeys;
  const int d = a.d, kd = d + 4, d4 = d / 4;
  float* qs = rsm;
  float* ks = rsm + kWinHeads * d;
  const int nh = min(kWinHeads, a.H - h0), nk = min(kWinKeys, a.n - t0);
  for (int e = threadIdx.x; e < nh * d4; e += blockDim.x) {
    const int hh = e / d4, i4 = e - hh * d4;
    cp_async16(qs + hh * d + 4 * i4, a.q + static_cast<size_t>(h0 + hh) * d + 4 * i4);
  }
  for (int e = threadIdx.x; e < nk * d4; e += blockDim.x) {
    const int tl = e / d4, i4 = e - tl * d4;
    cp_async16(ks + tl * kd + 4 * i4, a.kvdec + static_cast<size_t>(t0 + tl) * d + 4 * i4);
  }
  cp_async_wait_all();
  __syncthreads();
  const int lane = threadIdx.x & 31, hw = threadIdx.x >> 5;
  const int h = h0 + hw, t = t0 + lane;
  if (hw >= nh || lane >= nk) return;
  float st = -INFINITY;
  const int r = a.idx[t];
  if (r >= 0 && r < a.cache.rows) {
    const float4* q4 = reinterpret_cast<const float4*>(qs + hw * d);
    const float4* k4 = reinterpret_cast<const float4*>(ks + lane * kd);
    float dot = 0.0f;
#pragma unroll 8
    for (int i = 0; i < d4; ++i) {
      const float4 qv = q4[i], kv = k4[i];
      dot = fmaf(qv.x, kv.x, dot);
      dot = fmaf(qv.y, kv.y, dot);
      dot = fmaf(qv.z, kv.z, dot);
      dot = fmaf(qv.w, kv.w, dot);
    }
    st = __fmul_rn(dot, a.scale);
  }
  a.s[static_cast<size_t>(h) * a.n + t] = st;
}

// The same softmax and value pass with several heads per CTA, for key lists
// that fit shared memory: CTA (kVhHeads heads, kVhCols dims). The keys'
// kVhCols-column slice of kvdec [n][d] is copied to shared memory once
// (cp.async, every copy in flight together) and serves the CTA's heads, so
// L2 delivers each key row slice once per head group instead of once per
// head; the heads' scores [kVhHeads][n] come in beside them. Then warp w
// takes heads w, w + 4, ...: the max, the exponentials (ex) and the BF16
// weights (ws), as win_softmax_kernel.
// Then thread = (head, dimension pair): the two value chains over the keys
// in key order and the head's denominator expf(sink - m) + ex[0] + ... in
// key order (a dead key's ex is +0, which leaves the sum unchanged, as the
// reference's skip does), the division, BF16, the inverse RoPE.
constexpr int kVhHeads = 8, kVhCols = 32;
constexpr int kVhThreads = kVhHeads * kVhCols / 2;  // 128
size_t win_values_mh_smem(int n) {
  const size_t n4 = (static_cast<size_t>(n) + 3) & ~static_cast<size_t>(3);
  return sizeof(float) * (n4 * kVhCols + 2 * kVhHeads * (n4 + 1) + kVhHeads * n4);
}
__global__ void __launch_bounds__(kVhThreads) win_values_mh_kernel(const WinAttnArgs a) {
  // kv [n4][kVhCols] | sc [kVhHeads][n4] | ws [kVhHeads][n4 + 1] | ex [kVhHeads][n4 + 1]
  extern __shared__ __align__(16) float msm[];
  __shared__ float mxs[kVhHeads];
  pdl_wait();
  pdl_trigger();
  const int n = a.n, d = a.d, n4 = (n + 3) & ~3, ns = n4 + 1;
  const int h0 = blockIdx.x * kVhHeads, col0 = blockIdx.y * kVhCols;
  const int nh = min(kVhHeads, a.H - h0);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float* kv = msm;
  float* sc = kv + static_cast<size_t>(n4) * kVhCols;
  float* ws = sc + kVhHeads * n4;
  float* ex = ws + kVhHeads * ns;
  // the scores rows first (n is a multiple of 4: every row starts 16-byte
  // aligned), then the key slice: the softmax waits for the first group only
  for (int e = tid; e < nh * (n / 4); e += kVhThreads) {
    const int hh = e / (n / 4), t4 = e - hh * (n / 4);
    cp_async16(sc + hh * n4 + 4 * t4, a.s + static_cast<size_t>(h0 + hh) * n + 4 * t4);
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
  for (int e = tid; e < n * (kVhCols / 4); e += kVhThreads) {
    const int t = e / (kVhCols / 4), c4 = e - t * (kVhCols / 4);
    cp_async16(kv + t * kVhCols + 4 * c4, a.kvdec + static_cast<size_t>(t) * d + col0 + 4 * c4);
  }
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 1;" ::: "memory");
  __syncthreads();
  for (int hh = warp; hh < nh; hh += kVhThreads / 32) {
    const float* sh = sc + hh * n4;
    float mx = -INFINITY;
    for (int t = lane; t < n; t += 32) mx = fmaxf(mx, sh[t]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    for (int t = lane; t < n; t += 32) {
      const float st = sh[t];
      const bool live = st != -INFINITY;
      const float e = live ? expf_r1(st - mx) : 0.0f;
      ex[hh * ns + t] = e;
      ws[hh * ns + t] = live ? bf16_round(e) : 0.0f;
    }
    if (lane == 0) mxs[hh] = mx;
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  __syncthreads();
  const int hh = tid / (kVhCols / 2), p = tid - hh * (kVhCols / 2);
  const int h = h0 + hh;
  if (h >= a.H) return;
  const float* wr = ws + hh * ns;
  const float* er = ex + hh * ns;
  float o0 = 0.0f, o1 = 0.0f;
  float den = expf_r1(a.sink[h] - mxs[hh]);
#pragma unroll 4
  for (int t = 0; t < n; ++t) {
    const float2 v = *reinterpret_cast<const float2*>(kv + t * kVhCols + 2 * p);
    const float wt = wr[t];
    o0 = fmaf(wt, v.x, o0);
    o1 = fmaf(wt, v.y, o1);
    den = __fadd_rn(den, er[t]);
  }
  if (blockIdx.y == 0 && p == 0) a.den[h] = den;
  const int i = col0 + 2 * p;
  float x0 = bf16_round(o0 / den), x1 = bf16_round(o1 / den);
  const int start = d - a.rope_dim;
  if (a.cosv && i >= start) {
    const int k = (i - start) / 2;
    const float c = a.cosv[k], sn = a.sinv[k];
    const float y0 = bf16_round(__fadd_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn)));
    const float y1 = bf16_round(__fadd_rn(__fmul_rn(-x0, sn), __fmul_rn(x1, c)));
    x0 = y0;
    x1 = y1;
  }
  float* oh = a.out + static_cast<size_t>(h) * d;
  oh[i] = x0;
  oh[i + 1] = x1;
}

__device__ __forceinline__ void bf16x8_to_f32(const uint4 u, float (&f)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    f[2 * k] = __uint_as_float(w[k] << 16);
    f[2 * k + 1] = __uint_as_float(w[k] & 0xFFFF0000u);
  }
}

// The same attention for one head per CTA over the window staged as BF16
// rows (NormTailArgs::win): each row lands in shared memory by one bulk
// copy (rows padded by 8 elements so 16-byte reads of consecutive keys are
// conflict-free); thread = key for the scores (the dimension-order chain),
// warp 0 for the softmax, thread = dimension pairs for the values (the
// key-order chains), then the division, BF16 and the inverse RoPE.
constexpr int kWhThreads = 128;

__host__ __device__ inline size_t win_head_smem(int n, int d) {
  return static_cast<size_t>(n) * (d + 8) * 2 + static_cast<size_t>(d) * 4 +
         static_cast<size_t>(3) * n * 4 + 16;
}

template <class Wait>
__device__ void win_head_run(const WinAttnArgs& a, const uint16_t* win, unsigned int* err, int h,
                             unsigned char* wsm, Wait wait) {
  __shared__ uint64_t bar;
  __shared__ float den_s;
  const int n = a.n, d = a.d, ldk = d + 8;
  uint16_t* ks = reinterpret_cast<uint16_t*>(wsm);                                // [n][d + 8]
  float* qs = reinterpret_cast<float*>(wsm + static_cast<size_t>(n) * ldk * 2);   // [d]
  float* ss = qs + d;                                                              // [n]
  float* ws = ss + n;                                                              // [n]
  int* sidx = reinterpret_cast<int*>(ws + n);                                      // [n]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nth = blockDim.x;  // any multiple of 32 up to 1024
  if (tid == 0) {
    mbar_init(&bar, 1);
    mbar_fence_init();
  }
  __syncthreads();
  wait();
  const uint32_t row_bytes = static_cast<uint32_t>(d) * 2;
  if (tid == 0) mbar_arrive_expect_tx(&bar, row_bytes * static_cast<uint32_t>(n));
  __syncthreads();
  for (int t = tid; t < n; t += nth) {
    bulk_g2s(ks + static_cast<size_t>(t) * ldk, win + static_cast<size_t>(t) * d, row_bytes, &bar);
    sidx[t] = a.idx[t];
  }
  for (int i = tid; i < d / 4; i += nth)
    reinterpret_cast<float4*>(qs)[i] = reinterpret_cast<const float4*>(a.q + static_cast<size_t>(h) * d)[i];
  if (a.q_raw) {
    // the head's RMS and RoPE (src/dsv4/dsv4_model.c:5283-5291), as
    // q_head_kernel computes them
    __shared__ double qred[32];
    __syncthreads();
    double ss = 0.0;
    for (int i = tid; i < d; i += nth) ss += static_cast<double>(qs[i]) * qs[i];
    ss = block_sum_d(ss, qred);
    const float rr = rms_factor(ss, d, a.q_eps);
    for (int i = tid; i < d; i += nth) qs[i] = bf16_round(__fmul_rn(qs[i], rr));
    __syncthreads();
    const int half = a.rope_dim / 2, start = d - a.rope_dim;
    for (int i = tid; i < half; i += nth) {
      const float x0 = qs[start + 2 * i], x1 = qs[start + 2 * i + 1];
      const float c = a.cosv[i], sn = a.sinv[i];
      qs[start + 2 * i] = bf16_round(__fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn)));
      qs[start + 2 * i + 1] = bf16_round(__fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c)));
    }
  }
  bool ok = mbar_wait(&bar, 0, err);
  if (!__syncthreads_and(ok)) {
    if (!ok) mbar_wait(&bar, 0, err);  // the copies in flight land before the CTA exits
    return;
  }
  // scores
  for (int t = tid; t < n; t += nth) {
    const int r = sidx[t];
    float st = -INFINITY;
    if (r >= 0 && r < a.cache.rows) {
      const uint16_t* kr = ks + static_cast<size_t>(t) * ldk;
      float dot = 0.0f;
#pragma unroll 4
      for (int i = 0; i < d; i += 8) {
        float kf[8];
        bf16x8_to_f32(*reinterpret_cast<const uint4*>(kr + i), kf);
        const float4 q0 = *reinterpret_cast<const float4*>(qs + i);
        const float4 q1 = *reinterpret_cast<const float4*>(qs + i + 4);
        dot = fmaf(q0.x, kf[0], dot);
        dot = fmaf(q0.y, kf[1], dot);
        dot = fmaf(q0.z, kf[2], dot);
        dot = fmaf(q0.w, kf[3], dot);
        dot = fmaf(q1.x, kf[4], dot);
        dot = fmaf(q1.y, kf[5], dot);
        dot = fmaf(q1.z, kf[6], dot);
        dot = fmaf(q1.w, kf[7], dot);
      }
      st = __fmul_rn(dot, a.scale);
    }
    ss[t] = st;
  }
  __syncthreads();
  if (warp == 0) {
    float mx = -INFINITY;
    for (int t = lane; t < n; t += 32) mx = fmaxf(mx, ss[t]);
    mx = warp_max(mx);
    for (int t = lane; t < n; t += 32) {
      const float st = ss[t];
      ws[t] = st != -INFINITY ? expf_r1(st - mx) : 0.0f;
    }
    __syncwarp();
    if (lane == 0) {
      float sum = expf_r1(a.sink[h] - mx);
      for (int t = 0; t < n; ++t)
        if (ss[t] != -INFINITY) sum += ws[t];
      den_s = sum;
    }
    __syncwarp();
    for (int t = lane; t < n; t += 32) ws[t] = bf16_round(ws[t]);
  }
  __syncthreads();
  const float den = den_s;
  const int start = d - a.rope_dim;
  for (int p0 = tid; p0 < d / 2; p0 += 2 * nth) {
    // two dimension pairs per pass: four independent key-order chains
    const int p1 = p0 + nth;
    const bool has1 = p1 < d / 2;
    float o[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
#pragma unroll 4
    for (int t = 0; t < n; ++t) {
      const float wt = ws[t];
      const uint16_t* vr = ks + static_cast<size_t>(t) * ldk;
      const uint32_t v0 = *reinterpret_cast<const uint32_t*>(vr + 2 * p0);
      const uint32_t v1 = has1 ? *reinterpret_cast<const uint32_t*>(vr + 2 * p1) : 0u;
      o[0][0] = fmaf(wt, __uint_as_float(v0 << 16), o[0][0]);
      o[0][1] = fmaf(wt, __uint_as_float(v0 & 0xFFFF0000u), o[0][1]);
      o[1][0] = fmaf(wt, __uint_as_float(v1 << 16), o[1][0]);
      o[1][1] = fmaf(wt, __uint_as_float(v1 & 0xFFFF0000u), o[1][1]);
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      if (u == 1 && !has1) break;
      const int i = 2 * (u ? p1 : p0);
      float x0 = bf16_round(o[u][0] / den), x1 = bf16_round(o[u][1] / den);
      if (a.cosv && i >= start) {
        const int k = (i - start) / 2;
        const float cs = a.cosv[k], sn = a.sinv[k];
        const float y0 = bf16_round(__fadd_rn(__fmul_rn(x0, cs), __fmul_rn(x1, sn)));
        const float y1 = bf16_round(__fadd_rn(__fmul_rn(-x0, sn), __fmul_rn(x1, cs)));
        x0 = y0;
        x1 = y1;
      }
      *reinterpret_cast<float2*>(a.out + static_cast<size_t>(h) * d + i) = make_float2(x0, x1);
    }
  }
}

__global__ void __launch_bounds__(kWhThreads) win_head_kernel(const WinAttnArgs a0, const uint16_t* win,
                                                              unsigned int* err) {
  extern __shared__ __align__(16) unsigned char wsm[];
  pdl_trigger();
  const size_t r = blockIdx.y;
  const size_t hd = static_cast<size_t>(a0.H) * a0.d;
  WinAttnArgs a = a0;
  a.q = a0.q + r * hd;
  a.out = a0.out + r * hd;
  a.idx = a0.idx + r * a0.n;
  a.cosv = a0.cosv + r * (a0.rope_dim / 2);
  a.sinv = a0.sinv + r * (a0.rope_dim / 2);
  win_head_run(a, win + r * a0.n * a0.d, err, blockIdx.x, wsm, [] { pdl_wait(); });
}

// Greedy token: argmax_logits (src/cli/dsv4_run.c:355; first maximum, strict
// >) in two stages - each CTA finds its chunk's first maximum, then one warp
// takes the chunks' results in chunk order with the same strict >. For
// finite logits this is the sequential scan's answer.
constexpr int kArgmaxCtas = 148;
// blockIdx.y = row of a verify step's logits [rows][n] (its chunk results
// at + row gridDim.x).
__global__ void __launch_bounds__(256) argmax_chunks_kernel(const float* x, int n, float* cv,
                                                            int* ci) {
  __shared__ float sv[8];
  __shared__ int si[8];
  pdl_wait();
  pdl_trigger();
  x += static_cast<size_t>(blockIdx.y) * n;
  cv += blockIdx.y * gridDim.x;
  ci += blockIdx.y * gridDim.x;
  const int chunk = (n + gridDim.x - 1) / gridDim.x;
  const int b = blockIdx.x * chunk, e = min(n, b + chunk);
  float bv = -INFINITY;
  int bi = 0x7FFFFFFF;
  for (int i = b + threadIdx.x; i < e; i += blockDim.x) {
    const float v = x[i];
    if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
  }
  if ((threadIdx.x & 31) == 0) { sv[threadIdx.x >> 5] = bv; si[threadIdx.x >> 5] = bi; }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w)
      if (sv[w] > bv || (sv[w] == bv && si[w] < bi)) { bv = sv[w]; bi = si[w]; }
    cv[blockIdx.x] = bv;
    ci[blockIdx.x] = bi < e ? bi : b;
  }
}

// CTA r: row r's chunks.
__global__ void argmax_final_kernel(const float* cv, const int* ci, int chunks, int* out) {
  pdl_wait();
  pdl_trigger();
  if (threadIdx.x != 0) return;
  cv += blockIdx.x * chunks;
  ci += blockIdx.x * chunks;
  out += blockIdx.x;
  int best = 0;
  for (int c = 1; c < chunks; ++c)
    if (cv[c] > cv[best]) best = c;
  *out = ci[best];
}

// hc_post (src/dsv4/dsv4_model.c:7165-7177): thread = column j of the state.
__global__ void hc_post_kernel(float* state, const float* branch, const float* post,
                               const float* comb, int mult, int hid) {
  pdl_wait();
  pdl_trigger();
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= hid) return;
  float col[kHcMultMax];
  for (int k = 0; k < mult; ++k) col[k] = state[static_cast<size_t>(k) * hid + j];
  const float b = branch[j];
  for (int i = 0; i < mult; ++i) {
    float y = __fmul_rn(post[i], b);
    for (int k = 0; k < mult; ++k) y = fmaf(comb[i * mult + k], col[k], y);
    state[static_cast<size_t>(i) * hid + j] = bf16_round(y);
  }
}

__global__ void fill_f32_kernel(float* p, size_t n, float v) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x)
    p[i] = v;
}

// wo_a decode at load (src/dsv4/dsv4_model.c:1927-1936): BF16 of the E4M3
// code times its [128x128] block's E8M0 scale.
__global__ void fp8_to_bf16_kernel(const uint8_t* codes, const uint8_t* scales, int rows, int cols,
                                   uint16_t* out) {
  const int scols = (cols + 127) / 128;
  const size_t n = static_cast<size_t>(rows) * cols;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int r = static_cast<int>(i / cols), c = static_cast<int>(i % cols);
    const float v = __fmul_rn(e4m3_decode(codes[i]),
                              e8m0_decode(scales[static_cast<size_t>(r / 128) * scols + c / 128]));
    out[i] = static_cast<uint16_t>(__float_as_uint(bf16_round(v)) >> 16);
  }
}

// ---- compressed attention state (compress ratio 4 / 128 layers) ----

// 2^ceil(log2(r)) for a positive normal r, frexp's rule as the reference
// writes it (m == 0.5 -> one binade down).
__device__ __forceinline__ float pow2_ceil(float r) {
  const uint32_t u = __float_as_uint(r);
  int e = static_cast<int>((u >> 23) & 0xFFu) - 126;
  if ((u & 0x7FFFFFu) == 0u) e -= 1;
  return __uint_as_float(static_cast<uint32_t>(e + 127) << 23);
}

// dsv4_hadamard_inplace (src/dsv4/dsv4_model.c:1454-1468) on x[0..n) in
// shared memory, n a power of two: the butterfly stages (each pair's sum and
// difference in fp32), then x * (1 / sqrtf(n)) rounded to BF16. Every
// thread of the CTA calls it.
__device__ void hadamard_smem(float* x, int n) {
  for (int len = 1; len < n; len <<= 1) {
    __syncthreads();
    for (int k = threadIdx.x; k < n / 2; k += blockDim.x) {
      const int i = (k / len) * 2 * len + (k % len);
      const float a = x[i], b = x[i + len];
      x[i] = __fadd_rn(a, b);
      x[i + len] = __fsub_rn(a, b);
    }
  }
  __syncthreads();
  const float inv = 1.0f / sqrtf(static_cast<float>(n));
  for (int i = threadIdx.x; i < n; i += blockDim.x) x[i] = bf16_round(__fmul_rn(x[i], inv));
  __syncthreads();
}

// dsv4_fp4_act_quant_inplace (:1417-1452, mode 0) on x[0..n) in shared
// memory: per 32 values the power-of-two scale of amax / 6 (floor 6 *
// 2^-126), each value to the nearest E2M1 magnitude (ties to the even
// code, the reference's scan), times the scale, BF16. Warp = group.
__device__ void fp4_quant_smem(float* x, int n) {
  const float mags[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  for (int g = warp; g * 32 < n; g += nw) {
    const int i = g * 32 + lane;
    const float v = i < n ? x[i] : 0.0f;
    float amax = warp_max(fabsf(v));
    const float floor6 = 6.0f * __uint_as_float(1u << 23);  // 6 * 2^-126
    if (amax < floor6) amax = floor6;
    const float scale = pow2_ceil(__fmul_rn(amax, 1.0f / 6.0f));
    const float inv = 1.0f / scale;
    if (i < n) {
      float q = __fmul_rn(v, inv);
      q = q > 6.0f ? 6.0f : (q < -6.0f ? -6.0f : q);
      const float aq = fabsf(q);
      int idx = 0;
      float best = aq;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float dd = fabsf(__fsub_rn(aq, mags[k]));
        if (dd < best) { best = dd; idx = k; }
        else if (dd == best && (k & 1) == 0) idx = k;
      }
      x[i] = bf16_round(__fmul_rn(q < 0.0f ? -mags[idx] : mags[idx], scale));
    }
  }
  __syncthreads();
}

// compressor_update (src/dsv4/dsv4_model.c:5100-5236) for one token, after
// its two BF16 projections kv, sc [coff * d] (fp32, as the reference keeps
// them): score += ape[pos % ratio], both into the state slot; at a block's
// last position the block's rows are pooled per channel (softmax of the
// scores over the rows, fmaf-weighted sum of the kv rows in row order),
// rounded to BF16, RMSNorm with the gain, RoPE of the compressed table at
// the block's first position, then the FP8 QAT of the KV cache (the row goes
// to cache row row0 + count) or, for the indexer (rotate), Hadamard + FP4
// QAT (the row goes to out[count][d]). One CTA per step (any multiple of 32
// threads).
struct CompStepArgs {
  const float* kv;        // [coff * d]
  const float* sc;        // [coff * d]
  const float* ape;       // [ratio][coff * d]
  float* kvs;             // state [coff * ratio][coff * d], zeros at reset
  float* scs;             // state, -inf at reset
  const uint16_t* norm;   // [d] BF16 gain
  int d, ratio, coff, rotate, rope_dim;
  float eps;
  const int* pos;
  int* count;
  int max_count;
  const float* cos_tab;   // compressed-layer RoPE [max_pos][rope_dim / 2]
  const float* sin_tab;
  int max_pos;
  Fp8KvCache cache;       // main compressor: the cache and its first compressed row
  long long row0;
  float* out;             // indexer: [max_count][d]
  unsigned int* err;
};

// CTA i runs step a[i]: a compress-ratio-4 layer's main compressor and its
// indexer's compressor in one launch (independent state, rows and outputs).
// With list set (a ratio-128 layer, one step), CTA 0 then writes the layer's
// attention key list: the window's list, every compressed row in order
// (row0 + i, i < the count after the step; src/dsv4/dsv4_model.c:5330-5336),
// -1 padding to n_list.
struct CompStepPair {
  CompStepArgs a[2];
  const int* win_idx;
  int win;
  int* list;
  int n_list;
};
__device__ void comp_step_body(const CompStepArgs& a, float* csm, double* red);
__global__ void comp_step_kernel(const __grid_constant__ CompStepPair p) {
  extern __shared__ float csm[];  // [d]
  __shared__ double red[32];
  pdl_trigger();
  pdl_wait();
  const CompStepArgs& a = p.a[blockIdx.x];
  comp_step_body(a, csm, red);
  if (!p.list) return;
  __syncthreads();  // the count the step wrote is visible to the CTA
  const int k = *a.count;
  for (int i = threadIdx.x; i < p.win; i += blockDim.x) p.list[i] = p.win_idx[i];
  for (int i = threadIdx.x; i < p.n_list - p.win; i += blockDim.x)
    p.list[p.win + i] = i < k ? static_cast<int>(a.row0 + i) : -1;
}
__device__ void comp_step_body(const CompStepArgs& a, float* csm, double* red) {
  const int tid = threadIdx.x, nt = blockDim.x, lane = tid & 31, warp = tid >> 5;
  const int pos = *a.pos;
  const int cd = a.coff * a.d;
  const int r = pos % a.ratio;
  const int slot = r + (a.coff == 2 ? a.ratio : 0);
  for (int i = tid; i < cd; i += nt) {
    a.kvs[static_cast<size_t>(slot) * cd + i] = a.kv[i];
    a.scs[static_cast<size_t>(slot) * cd + i] = __fadd_rn(a.sc[i], a.ape[static_cast<size_t>(r) * cd + i]);
  }
  if ((pos + 1) % a.ratio != 0) return;  // uniform over the CTA
  __syncthreads();
  const int rows = a.ratio * a.coff;
  for (int ch = tid; ch < a.d; ch += nt) {
    // row i of the block: the previous block's first half, then this
    // block's second half (coff 2), or this block (coff 1)
    auto at = [&](int i) {
      return static_cast<size_t>(i) * cd + ((a.coff == 2 && i >= a.ratio) ? a.d : 0) + ch;
    };
    float mx = a.scs[at(0)];
    for (int i = 1; i < rows; ++i) {
      const float b = a.scs[at(i)];
      if (b > mx) mx = b;
    }
    float sum = 0.0f;
    for (int i = 0; i < rows; ++i) sum = __fadd_rn(sum, expf_r1(__fsub_rn(a.scs[at(i)], mx)));
    const float inv = 1.0f / sum;
    float acc = 0.0f;
    for (int i = 0; i < rows; ++i)
      acc = fmaf(__fmul_rn(expf_r1(__fsub_rn(a.scs[at(i)], mx)), inv), a.kvs[at(i)], acc);
    csm[ch] = bf16_round(acc);
  }
  __syncthreads();
  if (a.coff == 2) {
    // kv_state[:ratio] = kv_state[ratio:] (the halves do not overlap)
    for (int i = tid; i < a.ratio * cd; i += nt) {
      a.kvs[i] = a.kvs[static_cast<size_t>(a.ratio) * cd + i];
      a.scs[i] = a.scs[static_cast<size_t>(a.ratio) * cd + i];
    }
  }
  // RMSNorm with the gain (rmsnorm_bf16, :4934)
  double ss = 0.0;
  for (int ch = tid; ch < a.d; ch += nt) ss += static_cast<double>(csm[ch]) * csm[ch];
  ss = block_sum_d(ss, red);
  const float rr = rms_factor(ss, a.d, a.eps);
  for (int ch = tid; ch < a.d; ch += nt)
    csm[ch] = bf16_round(__fmul_rn(__fmul_rn(csm[ch], rr), bf16_widen(a.norm[ch])));
  __syncthreads();
  // RoPE at the block start (dsv4_rope_apply_buf, :1547-1558)
  if (a.d >= a.rope_dim) {
    int blk = pos + 1 - a.ratio;
    if (blk < 0) blk = 0;
    if (blk >= a.max_pos) blk = a.max_pos - 1;
    const int half = a.rope_dim / 2, start = a.d - a.rope_dim;
    for (int i = tid; i < half; i += nt) {
      const float x0 = csm[start + 2 * i], x1 = csm[start + 2 * i + 1];
      const float c = a.cos_tab[static_cast<size_t>(blk) * half + i];
      const float sn = a.sin_tab[static_cast<size_t>(blk) * half + i];
      csm[start + 2 * i] = bf16_round(__fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn)));
      csm[start + 2 * i + 1] = bf16_round(__fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c)));
    }
  }
  __syncthreads();
  const int cnt = *a.count;
  if (cnt >= a.max_count) {
    if (tid == 0) atomicOr(a.err, 16u);  // more compressed rows than the decoder holds
    return;
  }
  if (a.rotate) {
    hadamard_smem(csm, a.d);
    fp4_quant_smem(csm, a.d);
    for (int ch = tid; ch < a.d; ch += nt) a.out[static_cast<size_t>(cnt) * a.d + ch] = csm[ch];
  } else {
    const long long row = a.row0 + cnt;
    for (int g = warp; g < a.cache.nope / 64; g += nt >> 5)
      kv_quant_group(a.cache, row, g, csm[g * 64 + lane], csm[g * 64 + 32 + lane], lane);
    for (int i = tid; i < a.cache.rope_dim; i += nt)
      a.cache.rope[row * a.cache.rope_dim + i] =
          static_cast<uint16_t>(__float_as_uint(bf16_round(csm[a.cache.nope + i])) >> 16);
  }
  __syncthreads();
  if (tid == 0) *a.count = cnt + 1;
}

// The indexer's query of one head (indexer_forward, :5699-5712) built by
// one warp in registers: lane holds values lane * V .. lane * V + V - 1 of
// the head's id = 32 V. The RoPE of the compressed table at the position on
// the last rope_dim dims (pairs inside a lane, or across a lane pair for
// V = 1), the Hadamard butterflies stage by stage (partners inside a lane
// while the stride is below V, else by shuffle), x / sqrt(id) to BF16, and
// the FP4 QAT per 32 values (32 / V lanes per group): the reference's
// operations per element. The result goes to out[0 .. id).
template <int V>
__device__ __forceinline__ void idx_query_warp(const float* src, float* out, int id, int rope_dim,
                                               const float* cosv, const float* sinv, int lane) {
  float x[V];
#pragma unroll
  for (int r = 0; r < V; ++r) x[r] = src[lane * V + r];
  const int start = id - rope_dim;
  if constexpr (V >= 2) {
#pragma unroll
    for (int r = 0; r < V; r += 2) {
      const int j = lane * V + r;
      if (j >= start) {
        const int i = (j - start) >> 1;
        const float x0 = x[r], x1 = x[r + 1], c = cosv[i], sn = sinv[i];
        x[r] = bf16_round(__fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn)));
        x[r + 1] = bf16_round(__fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c)));
      }
    }
  } else {
    const float other = __shfl_xor_sync(0xffffffffu, x[0], 1);
    if (lane >= start) {
      const int i = (lane - start) >> 1;
      const bool odd = lane & 1;
      const float x0 = odd ? other : x[0], x1 = odd ? x[0] : other;
      const float c = cosv[i], sn = sinv[i];
      x[0] = odd ? bf16_round(__fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c)))
                 : bf16_round(__fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn)));
    }
  }
#pragma unroll
  for (int len = 1; len < V; len <<= 1)
#pragma unroll
    for (int r = 0; r < V; ++r)
      if ((r & len) == 0) {
        const float u = x[r], v = x[r + len];
        x[r] = __fadd_rn(u, v);
        x[r + len] = __fsub_rn(u, v);
      }
  for (int lm = 1; lm < 32; lm <<= 1) {  // lane stride lm = len / V
    const bool upper = (lane & lm) != 0;
#pragma unroll
    for (int r = 0; r < V; ++r) {
      const float o = __shfl_xor_sync(0xffffffffu, x[r], lm);
      x[r] = upper ? __fsub_rn(o, x[r]) : __fadd_rn(x[r], o);
    }
  }
  const float inv = 1.0f / sqrtf(static_cast<float>(id));
  float amax = 0.0f;
#pragma unroll
  for (int r = 0; r < V; ++r) {
    x[r] = bf16_round(__fmul_rn(x[r], inv));
    amax = fmaxf(amax, fabsf(x[r]));
  }
#pragma unroll
  for (int o = 1; o < 32 / V; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float floor6 = 6.0f * __uint_as_float(1u << 23);  // 6 * 2^-126
  if (amax < floor6) amax = floor6;
  const float scale = pow2_ceil(__fmul_rn(amax, 1.0f / 6.0f));
  const float rs = 1.0f / scale;
  const float mags[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};
#pragma unroll
  for (int r = 0; r < V; ++r) {
    float qv = __fmul_rn(x[r], rs);
    qv = qv > 6.0f ? 6.0f : (qv < -6.0f ? -6.0f : qv);
    const float aq = fabsf(qv);
    int idx = 0;
    float best = aq;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float dd = fabsf(__fsub_rn(aq, mags[k]));
      if (dd < best) { best = dd; idx = k; }
      else if (dd == best && (k & 1) == 0) idx = k;
    }
    out[lane * V + r] = bf16_round(__fmul_rn(qv < 0.0f ? -mags[idx] : mags[idx], scale));
  }
}

// Index scores (indexer_forward, :5699-5747), one launch. Each CTA first
// builds the indexer's query from the BF16 output of idx_wq_b (a warp per
// head, idx_query_warp) into shared memory, rows padded to id + 1 floats so
// a warp's heads sit on distinct banks. Then score[t] = sum over heads h in
// order of fmaf(relu(q_h . k_t), w_h, acc), the dot one fmaf chain over the
// head's dims; w_h = bf16(bf16(proj_h) * (id^-1/2 * ih^-1/2)). CTA = kIdxT
// compressed rows x ih heads (thread = (row, head) dot), the CTA's keys in
// shared memory beside the query, t < min(count, (pos+1)/4). id = 32 V with
// V in {1, 2, 4, 8}.
// 8 rows: 512-thread CTAs at 64 heads (a 1024-thread CTA, which needs an
// SM's registers nearly to itself, was measured slower to start in the chain)
constexpr int kIdxT = 8;
__global__ void idx_score_kernel(const float* q, const float* keys, const float* wproj, int ih,
                                 int id, int rope_dim, const float* cosv, const float* sinv,
                                 const int* count, const int* pos, float* score) {
  extern __shared__ float ism[];
  const int ld = id + 1;
  float* qs = ism;                   // [ih][id + 1]
  float* kt = qs + ih * ld;          // [kIdxT][id]
  float* dots = kt + kIdxT * id;     // [kIdxT][ih]
  float* wh = dots + kIdxT * ih;     // [ih]
  pdl_trigger();
  pdl_wait();
  int nt = *count;
  const int maxc = (*pos + 1) / 4;
  if (nt > maxc) nt = maxc;
  const int t0 = blockIdx.x * kIdxT;
  if (t0 >= nt) return;  // uniform over the CTA
  const int tid = threadIdx.x, nth = blockDim.x;
  const int lane = tid & 31, warp = tid >> 5, nw = nth >> 5;
  for (int i = tid; i < kIdxT * id; i += nth) {
    const int tl = i / id;
    kt[i] = t0 + tl < nt ? keys[static_cast<size_t>(t0) * id + i] : 0.0f;
  }
  const float s = __fmul_rn(1.0f / sqrtf(static_cast<float>(id)), 1.0f / sqrtf(static_cast<float>(ih)));
  // wproj: the BF16 GEMV's fp32 sums; the reference rounds them to BF16
  // (round_out = 1) before the scale
  for (int k = tid; k < ih; k += nth) wh[k] = bf16_round(__fmul_rn(bf16_round(wproj[k]), s));
  {
    const int sh = __ffs(id) - 1;  // id is a power of two
#pragma unroll 4
    for (int i = tid; i < ih * id; i += nth) qs[(i >> sh) * ld + (i & (id - 1))] = q[i];
  }
  __syncthreads();
  for (int h = warp; h < ih; h += nw) {
    const float* src = qs + h * ld;
    float* dst = qs + h * ld;
    switch (id >> 5) {
      case 1: idx_query_warp<1>(src, dst, id, rope_dim, cosv, sinv, lane); break;
      case 2: idx_query_warp<2>(src, dst, id, rope_dim, cosv, sinv, lane); break;
      case 4: idx_query_warp<4>(src, dst, id, rope_dim, cosv, sinv, lane); break;
      default: idx_query_warp<8>(src, dst, id, rope_dim, cosv, sinv, lane); break;
    }
  }
  __syncthreads();
  const int tl = tid / ih, h = tid % ih;
  const int t = t0 + tl;
  if (tl < kIdxT && t < nt) {
    const float* kr = kt + tl * id;
    const float* qh = qs + h * ld;
    float dot = 0.0f;
#pragma unroll 8
    for (int dd = 0; dd < id; ++dd) dot = fmaf(qh[dd], kr[dd], dot);
    if (dot < 0.0f) dot = 0.0f;
    dots[tl * ih + h] = dot;
  }
  __syncthreads();
  if (h == 0 && tl < kIdxT && t < nt) {
    float acc = 0.0f;
#pragma unroll 8
    for (int k = 0; k < ih; ++k) acc = fmaf(dots[tl * ih + k], wh[k], acc);
    score[t] = acc;
  }
}

// The attention key list of a compress-ratio-4 layer: the window's list (as
// the window-only layers use it, -1 padded), then the indexer's top-k of the
// compressed rows (dsv4_indexer_select_topk, :5636-5679: score descending,
// lower index first, k = min(index_topk, n)), then -1 padding to n_max. Rows
// are row0 + compressed index. (A ratio-128 layer lists every compressed row
// in order, :5330-5336, written by its compressor-step launch.) One CTA of
// kListThreads; the selection sorts the n scores with a bitonic network
// over the next power of two >= n: while that fits the CTA, one key per
// thread in registers (partners within a warp by shuffle, farther ones
// through a double-buffered shared array, one barrier per stage); beyond
// it, in shared memory over n2 (a power of two >= the most compressed rows).
// The order is a strict total order on the keys (indices are distinct), so
// both forms give the order.
constexpr int kListThreads = 1024;
size_t comp_list_smem(int n2) {
  return sizeof(float) * std::max(2 * n2, 4 * kListThreads);
}
__device__ __forceinline__ bool topk_before(float sa, int ia, float sb, int ib) {
  // real before padding (-1); higher score first; lower index first
  if (ib < 0) return ia >= 0;
  if (ia < 0) return false;
  if (sa > sb) return true;
  if (sa < sb) return false;
  return ia < ib;
}
__global__ void __launch_bounds__(kListThreads)
comp_list_kernel(const int* win_idx, int win, const float* score, const int* count, const int* pos,
                 int topk, long long row0, int n2, int n_max, int* out) {
  extern __shared__ unsigned char lsm[];
  pdl_trigger();
  pdl_wait();
  const int tid = threadIdx.x, nt = blockDim.x;
  for (int i = tid; i < win; i += nt) out[i] = win_idx[i];
  int n = *count;
  const int maxc = (*pos + 1) / 4;
  if (n > maxc) n = maxc;
  const int k = topk < n ? topk : n;
  int m2 = 32;
  while (m2 < n) m2 <<= 1;
  if (m2 <= nt) {
    float* bs = reinterpret_cast<float*>(lsm);        // [2][nt]
    int* bi = reinterpret_cast<int*>(bs + 2 * nt);     // [2][nt]
    float sv = tid < n ? score[tid] : 0.0f;
    int iv = tid < n ? tid : -1;
    int stage = 0;
    for (int size = 2; size <= m2; size <<= 1)
      for (int stride = size >> 1; stride > 0; stride >>= 1) {
        float so;
        int io;
        if (stride >= 32) {
          float* ws_ = bs + (stage & 1) * nt;
          int* wi_ = bi + (stage & 1) * nt;
          ws_[tid] = sv;
          wi_[tid] = iv;
          __syncthreads();
          so = ws_[tid ^ stride];
          io = wi_[tid ^ stride];
          ++stage;
        } else {
          so = __shfl_xor_sync(0xffffffffu, sv, stride);
          io = __shfl_xor_sync(0xffffffffu, iv, stride);
        }
        if (tid < m2) {
          const bool up = (tid & size) == 0, lower = (tid & stride) == 0;
          const bool mine_first = topk_before(sv, iv, so, io);
          if (lower == up ? !mine_first : mine_first) {
            sv = so;
            iv = io;
          }
        }
      }
    for (int i = tid; i < n_max - win; i += nt)
      out[win + i] = i < k ? static_cast<int>(row0 + (i == tid ? iv : 0)) : -1;
    return;
  }
  float* ks = reinterpret_cast<float*>(lsm);
  int* ki = reinterpret_cast<int*>(ks + n2);
  for (int i = tid; i < n2; i += nt) {
    ks[i] = i < n ? score[i] : 0.0f;
    ki[i] = i < n ? i : -1;  // -1: padding, after every real row
  }
  for (int size = 2; size <= n2; size <<= 1)
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      __syncthreads();
      for (int i = tid; i < n2; i += nt) {
        const int j = i ^ stride;
        if (j > i) {
          const bool up = (i & size) == 0;
          const bool swap = up ? topk_before(ks[j], ki[j], ks[i], ki[i])
                               : topk_before(ks[i], ki[i], ks[j], ki[j]);
          if (swap) {
            const float tf = ks[i]; ks[i] = ks[j]; ks[j] = tf;
            const int ti = ki[i]; ki[i] = ki[j]; ki[j] = ti;
          }
        }
      }
    }
  __syncthreads();
  for (int i = tid; i < n_max - win; i += nt)
    out[win + i] = i < k ? static_cast<int>(row0 + ki[i]) : -1;
}

// Greedy acceptance of a verify step (the reference CLI's chain,
// src/cli/dsv4_run.c:951-1043 at temperature 0): rows [pending, d1 .. dk]
// with targets argmax[r]; d(a+1) is accepted while it equals argmax[a].
// Emits the accepted drafts and the bonus argmax[a] (a + 1 tokens), keeps
// rows 0 .. a (the commit), and sets the next step up on the device: the
// bonus becomes the pending row, the start advances by a + 1. stats[0] +=
// tokens emitted, stats[1] += drafts accepted, stats[2] += verify steps.
__global__ void verify_accept_kernel(int* tok, const int* argmax, int n, int* start, int* from,
                                     int* count, long long* stats) {
  pdl_wait();
  pdl_trigger();
  if (threadIdx.x != 0) return;
  int a = 0;
  while (a < n - 1 && tok[a + 1] == argmax[a]) ++a;
  const int s0 = *start;
  *from = s0;
  *count = a + 1;
  *start = s0 + a + 1;
  tok[0] = argmax[a];
  stats[0] += a + 1;
  stats[1] += a;
  stats[2] += 1;
}

// Commit of a verify step: the first *count rows' latents move from their
// scratch rows (win + j) into the ring rows of their positions
// ((*from + j) % win), in every layer's cache. CTA (layer, j).
__global__ void verify_commit_kernel(const Fp8KvCache* caches, int win, const int* from,
                                     const int* count) {
  pdl_wait();
  pdl_trigger();
  const int j = blockIdx.y;
  if (j >= *count) return;
  const Fp8KvCache c = caches[blockIdx.x];
  const long long src = win + j, dst = (*from + j) % win;
  for (int i = threadIdx.x; i < c.nope; i += blockDim.x)
    c.codes[dst * c.nope + i] = c.codes[src * c.nope + i];
  for (int i = threadIdx.x; i < kKvScaleSlots; i += blockDim.x)
    c.scales[dst * kKvScaleSlots + i] = c.scales[src * kKvScaleSlots + i];
  for (int i = threadIdx.x; i < c.rope_dim; i += blockDim.x)
    c.rope[dst * c.rope_dim + i] = c.rope[src * c.rope_dim + i];
}

// Uniform random draft ids for rows 1 .. n - 1 (the verify benchmark's
// drafts): xorshift64 (the reference CLI's rng_next, src/cli/dsv4_run.c:
// 248-254) modulo the vocabulary, one state advanced in row order.
__global__ void draft_random_kernel(unsigned long long* state, int* tok, int n, int vocab) {
  pdl_wait();
  pdl_trigger();
  if (threadIdx.x != 0) return;
  unsigned long long x = *state;
  for (int r = 1; r < n; ++r) {
    x ^= x << 13;
    x ^= x >> 7;
    x ^= x << 17;
    tok[r] = static_cast<int>(x % static_cast<unsigned long long>(vocab));
  }
  *state = x;
}

// ------------------------------------------------------- host side ----

struct Layer {
  dsv4cuda_layer_weights w;
  MoeConfig mc;
  MoeWeights mw;
  Fp8KvCache cache;
  uint16_t* wo_a = nullptr;  // BF16, decoded at create when given as FP8
  // compress ratio 4 / 128: the compressor's state, its rows in the cache
  // (from comp_row0) and, for ratio 4, the indexer's state and rows
  int ratio = 0, coff = 1;
  float *kvs = nullptr, *scs = nullptr;
  int* count = nullptr;
  int max_count = 0;
  long long comp_row0 = 0;
  float *idx_kvs = nullptr, *idx_scs = nullptr, *idx_rows = nullptr;
  int* idx_count = nullptr;
  int n_keys = 0;                 // its attention list: window + compressed rows
  // the BF16 projections of the layer input, stacked: compressor wkv and
  // wgate, then (ratio 4) the indexer compressor's wkv, wgate and the
  // indexer weights
  uint16_t* comp_w = nullptr;
  int comp_rows = 0;
};

}  // namespace
}  // namespace dsv4

struct dsv4cuda_decoder {
  dsv4cuda_decoder_config cfg{};
  dsv4cuda_model_weights g{};
  std::vector<dsv4::Layer> layers;
  // expert parallelism: per layer an EP-attached MoE layer (token-parallel
  // exchange over peer memory); empty = every expert on this device
  std::vector<dsv4cuda_moe_layer*> ep;
  bool ep_replicated = false;  // every rank decodes the same token (batch-1 strong scaling)
  std::vector<void*> owned;  // device allocations to free
  // per-step buffers
  int* d_token = nullptr;
  int* d_pos = nullptr;
  float* state = nullptr;     // [mult][hid]
  double* part = nullptr;     // [nblk][kMixMax + 1]
  unsigned int* hc_ticket = nullptr;  // last-CTA counter of hc_fused_kernel
  float* mix = nullptr;       // [kMixMax] the last boundary's mixes
  cudaStream_t hc_side = nullptr;      // the Sinkhorn split's stream
  cudaEvent_t hc_fork = nullptr, hc_join = nullptr;
  int nblk = 0;
  float *post = nullptr, *comb = nullptr;
  float* x = nullptr;         // [hid] normed branch input
  __half* xq = nullptr;       // [ld] FP8-grid activations (f16)
  float* xs = nullptr;        // [ld / 128] scales
  float* qr = nullptr;        // [q_lora]
  float* qn = nullptr;        // [q_lora]
  float* q = nullptr;         // [H][d]
  float* kv = nullptr;        // [d]
  float* o = nullptr;         // [H][d]
  float* kvdec = nullptr;     // [window][d] the window's cached values
  float* kvt = nullptr;       // [d][window] transposed
  float* fp8_part = nullptr;  // split-K FP8 GEMV partials [in / 128][rows]
  unsigned int* tile_cnt = nullptr;  // split-K row-tile counters (zero between launches)
  size_t win_smem = 0;        // dynamic shared memory of win_scores_kernel
  bool win_staged = false;    // the window attention runs as win_head_kernel
  uint16_t* kvwin = nullptr;  // [window][head_dim] the window's rows as BF16
  float* att_s = nullptr;     // [H][window] scores
  float* att_w = nullptr;     // [H][window] BF16 weights
  float* att_den = nullptr;   // [H]
  float* oall = nullptr;      // [G][o_lora]
  float* branch = nullptr;    // [hid]
  float* logits = nullptr;    // [vocab]
  int* argmax = nullptr;      // [1]
  float* am_v = nullptr;      // per-chunk maxima of the argmax
  int* am_i = nullptr;
  int* idx = nullptr;         // [window]
  long long* row = nullptr;   // [1]
  float *cosv = nullptr, *sinv = nullptr;      // [rope/2] of the current position
  float *cos_tab = nullptr, *sin_tab = nullptr;  // [max_context][rope/2]
  // compressed layers: their RoPE (YaRN table), scratch of the compressor
  // and indexer, the key list and its staged rows
  bool any_comp = false;
  int n_max = 0;                   // keys of the longest list
  size_t vmh_smem = 0;             // win_values_mh_kernel's shared memory limit (0: not used)
  int comp_rows_max = 0;           // rows of the largest stacked projection
  float *cosv_c = nullptr, *sinv_c = nullptr;
  float *cos_tab_c = nullptr, *sin_tab_c = nullptr;
  float* comp_proj = nullptr;      // the stacked projections' outputs
  cudaStream_t comp_side = nullptr;    // they run beside the q / kv path
  cudaEvent_t comp_fork = nullptr, comp_join = nullptr;
  float* idx_q = nullptr;          // [index_heads * index_dim]
  float* idx_score = nullptr;      // [most compressed rows]
  int idx_n2 = 0;                  // its sort width (a power of two)
  int* idx_full = nullptr;         // [n_max]
  float *c_kvdec = nullptr, *c_kvt = nullptr;    // [n_max][head_dim], transposed
  float *c_att_s = nullptr, *c_att_w = nullptr;  // [n_heads][n_max]
  dsv4::GemvItem* item1 = nullptr;   // one (x row 0 -> y row 0) item
  dsv4::GemvItem* items_g = nullptr; // o_groups items (group g: matrix g, rows g)
  int* n_one = nullptr;
  int* n_groups = nullptr;
  dsv4::MoeWorkspace moe_ws{};
  int ld = 0;                 // activation row stride (multiple of 512)
  cudaGraphExec_t graph = nullptr;  // forward_token's captured step
  cudaStream_t graph_stream = nullptr;
  bool stepped = false;
  std::string err;
  // speculative verify (dsv4cuda_decoder_verify*): up to
  // DSV4CUDA_VERIFY_MAX_ROWS rows per step, each row's buffers at the
  // single-token size apart
  struct Verify {
    int* tok = nullptr;            // [V] row tokens: pending, then drafts
    int* start = nullptr;          // [1] position of row 0
    int* from = nullptr;           // [1] the last accepted step's start
    int* count = nullptr;          // [1] its rows to commit
    long long* stats = nullptr;    // [3] emitted, accepted, steps
    unsigned long long* rng = nullptr;  // [1] draft generator state
    float* state = nullptr;        // [V][mult][hid]
    double* part = nullptr;        // [V][part_rs]
    size_t part_rs = 0;
    unsigned int* ticket = nullptr;  // [V]
    float* mix = nullptr;          // [V][kMixMax]
    float *post = nullptr, *comb = nullptr;  // [V][kHcMultMax], [V][kHcMultMax^2]
    float* x = nullptr;            // [V][hid]
    __half* xq = nullptr;          // [V][ld]
    float* xs = nullptr;           // [V][ld / 128]
    float *qr = nullptr, *q = nullptr, *kv = nullptr, *o = nullptr;  // [V][q_lora], [V][H d], [V][d], [V][H d]
    float *oall = nullptr, *branch = nullptr;  // [V][G o_lora], [V][hid]
    uint16_t* kvwin = nullptr;     // [V][window][d]
    int* idx = nullptr;            // [V][window]
    long long* row = nullptr;      // [V]
    float *cosv = nullptr, *sinv = nullptr;  // [V][rope / 2]
    float* logits = nullptr;       // [V][vocab]
    int* argmax = nullptr;         // [V]
    float* am_v = nullptr;         // [V][kArgmaxCtas]
    int* am_i = nullptr;
    dsv4::GemvItem* items = nullptr;    // [V]: item n - 1 maps rows 0 .. n - 1
    dsv4::GemvItem* items_g = nullptr;  // [V][G]: the grouped wo_a's items for n rows
    int* n_one = nullptr;
    int* n_groups = nullptr;
    dsv4::Fp8KvCache* caches = nullptr;  // [n_layers] for the commit kernel
    float* mt_part = nullptr;      // the multi-token FP8 GEMVs' block partials
    size_t mt_part_floats = 0;
    dsv4::MoeWorkspace moe_ws{};
  } v;
};

namespace {

thread_local std::string t_dec_error;

int fail(const char* fmt, ...) __attribute__((format(printf, 1, 2)));
int fail(const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_dec_error = buf;
  return -1;
}

template <class T>
T* dalloc(dsv4cuda_decoder* D, size_t count) {
  void* p = nullptr;
  if (cudaMalloc(&p, std::max<size_t>(count * sizeof(T), 256)) != cudaSuccess) return nullptr;
  cudaMemset(p, 0, std::max<size_t>(count * sizeof(T), 256));
  D->owned.push_back(p);
  return static_cast<T*>(p);
}

// RoPE cos/sin of every position for a non-compressed layer, computed on the
// host by the reference's formula (rope_freqs_fill, src/dsv4/dsv4_model.c:
// 1475-1503 with yarn = 0: layers of compress ratio 0 use the plain table),
// with the host libm, as the reference does.
void rope_tables(const dsv4cuda_decoder_config& c, std::vector<float>& cs, std::vector<float>& sn) {
  const int half = c.rope_dim / 2;
  cs.resize(static_cast<size_t>(c.max_context) * half);
  sn.resize(cs.size());
  std::vector<float> inv(half);
  for (int i = 0; i < half; ++i) {
    volatile float expo = static_cast<float>(2 * i) / static_cast<float>(c.rope_dim);
    inv[i] = 1.0f / powf(c.rope_theta, expo);
  }
  for (int p = 0; p < c.max_context; ++p)
    for (int i = 0; i < half; ++i) {
      volatile float angle = static_cast<float>(p) * inv[i];
      cs[static_cast<size_t>(p) * half + i] = cosf(angle);
      sn[static_cast<size_t>(p) * half + i] = sinf(angle);
    }
}

// The compressed layers' RoPE table: rope_freqs_fill (src/dsv4/dsv4_model.c:
// 1475-1503) with YaRN on and compress_rope_theta, host libm as the
// reference.
void rope_tables_yarn(const dsv4cuda_decoder_config& c, std::vector<float>& cs,
                      std::vector<float>& sn) {
  const int half = c.rope_dim / 2;
  cs.resize(static_cast<size_t>(c.max_context) * half);
  sn.resize(cs.size());
  const float theta = c.compress_rope_theta;
  const float rd = static_cast<float>(c.rope_dim);
  const float pi = static_cast<float>(M_PI);
  volatile float lnum = logf(static_cast<float>(c.original_position) / (c.beta_fast * 2.0f * pi));
  volatile float lden = 2.0f * logf(theta);
  float low = floorf(rd * lnum / lden);
  volatile float hnum = logf(static_cast<float>(c.original_position) / (c.beta_slow * 2.0f * pi));
  float high = ceilf(rd * hnum / lden);
  if (low < 0) low = 0;
  if (high > rd - 1.0f) high = rd - 1.0f;
  if (high == low) high += 0.001f;
  std::vector<float> inv(half);
  for (int i = 0; i < half; ++i) {
    volatile float expo = static_cast<float>(2 * i) / rd;
    volatile float base = 1.0f / powf(theta, expo);
    float ramp = (static_cast<float>(i) - low) / (high - low);
    if (ramp < 0.0f) ramp = 0.0f;
    if (ramp > 1.0f) ramp = 1.0f;
    volatile float interp = base / c.rope_factor;
    volatile float a = interp * ramp;
    volatile float b = base * (1.0f - ramp);
    inv[i] = a + b;
  }
  for (int p = 0; p < c.max_context; ++p)
    for (int i = 0; i < half; ++i) {
      volatile float angle = static_cast<float>(p) * inv[i];
      cs[static_cast<size_t>(p) * half + i] = cosf(angle);
      sn[static_cast<size_t>(p) * half + i] = sinf(angle);
    }
}

#define DEC_CHECK(expr)                             \
  do {                                              \
    cudaError_t e__ = (expr);                       \
    if (e__ != cudaSuccess) return e__;             \
  } while (0)

// xf set: the fp32 activations, quantised inside the split-K kernel (into
// x / xs) or by a quant launch first when that kernel cannot take them.
cudaError_t fp8_gemv(const uint8_t* W, const uint8_t* S, int in, int rows, const __half* x,
                     const float* xs, int ld, float* y, const dsv4::GemvItem* item, const int* n_one,
                     float* part, unsigned int* cnt, cudaStream_t st, const float* xf = nullptr) {
  if (xf) {
    dsv4::Fp8GemvArgs q{};
    q.W[0] = W;
    q.S[0] = S;
    q.in = in;
    q.rows = rows;
    q.round_out = 1;
    q.act = dsv4::QAct{x, xs, ld, nullptr};
    q.Y[0] = y;
    q.items = item;
    q.n_items = n_one;
    q.max_items = 1;
    q.xf = xf;
    const cudaError_t e = dsv4::launch_fp8_gemv_splitk(q, part, st, cnt);
    if (e != cudaErrorNotSupported) return e;
    DEC_CHECK(dsv4::launch_quant_fp8(xf, in, in, 1, const_cast<__half*>(x), const_cast<float*>(xs), ld, st));
  }
  dsv4::Fp8GemvArgs a{};
  a.W[0] = W;
  a.S[0] = S;
  a.in = in;
  a.rows = rows;
  a.round_out = 1;
  a.act = dsv4::QAct{x, xs, ld, nullptr};
  a.Y[0] = y;
  a.items = item;
  a.n_items = n_one;
  a.max_items = 1;
  cudaError_t e = dsv4::launch_fp8_gemv_splitk(a, part, st, cnt);
  return e == cudaErrorNotSupported ? dsv4::launch_fp8_gemv(a, false, 1, st) : e;
}

// Two projections of the same activations (wq_a and wkv) in one split-K
// launch pair when their shapes allow, else one after the other.
cudaError_t fp8_gemv2(const uint8_t* W0, const uint8_t* S0, int rows0, float* y0,
                      const uint8_t* W1, const uint8_t* S1, int rows1, float* y1, int in,
                      const __half* x, const float* xs, int ld, const dsv4::GemvItem* item,
                      const int* n_one, float* part, unsigned int* cnt, cudaStream_t st) {
  dsv4::Fp8GemvArgs a{};
  a.W[0] = W0;
  a.S[0] = S0;
  a.W[1] = W1;
  a.S[1] = S1;
  a.in = in;
  a.rows = rows0;
  a.rows1 = rows1;
  a.round_out = 1;
  a.act = dsv4::QAct{x, xs, ld, nullptr};
  a.Y[0] = y0;
  a.Y[1] = y1;
  a.items = item;
  a.n_items = n_one;
  a.max_items = 1;
  cudaError_t e = dsv4::launch_fp8_gemv_splitk(a, part, st, cnt);
  if (e != cudaErrorNotSupported) return e;
  DEC_CHECK(fp8_gemv(W0, S0, in, rows0, x, xs, ld, y0, item, n_one, part, cnt, st));
  return fp8_gemv(W1, S1, in, rows1, x, xs, ld, y1, item, n_one, part, cnt, st);
}


// The buffers one hyper-connection boundary works on: the single-token
// step's, or a verify step's n rows (row r's buffers at the hc_row strides).
struct HcRows {
  float* state;
  double* part;
  size_t part_rs;
  unsigned int* ticket;
  float* mix;
  float* post;
  float* comb;
  float* x;
  const float* branch;
  int n;
};

HcRows hc_single(dsv4cuda_decoder* D) {
  return HcRows{D->state, D->part, 0, D->hc_ticket, D->mix, D->post, D->comb, D->x, D->branch, 1};
}

HcRows hc_verify(dsv4cuda_decoder* D, int n) {
  auto& v = D->v;
  return HcRows{v.state, v.part, v.part_rs, v.ticket, v.mix, v.post, v.comb, v.x, v.branch, n};
}

// The exact mode's hc_pre of row r (one launch pair per row).
cudaError_t hc_pre(dsv4cuda_decoder* D, const HcRows& R, int r, const float* fn, const float* scale,
                   const float* base, const uint16_t* norm, int head, cudaStream_t st) {
  const auto& c = D->cfg;
  const int n = c.hc_mult * c.hidden;
  const int rows = head ? c.hc_mult : (2 + c.hc_mult) * c.hc_mult;
  const float* state = R.state + static_cast<size_t>(r) * n;
  double* part = R.part + r * R.part_rs;
  if (c.hc_exact)
    DEC_CHECK(dsv4::launch_pdl(dsv4::hc_mix_exact_kernel, dim3(1), dim3(32), 0, st, fn, rows, state,
                               n, part));
  else
    DEC_CHECK(dsv4::launch_pdl(dsv4::hc_mix_partial_kernel, dim3(D->nblk), dim3(dsv4::kMixThreads),
                               0, st, fn, rows, state, n, part));
  dsv4::HcReduceArgs a{};
  a.part = part;
  a.nblk = c.hc_exact ? 1 : D->nblk;
  a.rows = rows;
  a.head = head;
  a.scale = scale;
  a.base = base;
  a.mult = c.hc_mult;
  a.hid = c.hidden;
  a.iters = c.hc_iters;
  a.hc_eps = c.hc_eps;
  a.rms_eps = c.rms_eps;
  a.state = state;
  a.norm = norm;
  a.post = R.post + r * dsv4::kHcMultMax;
  a.comb = R.comb + r * dsv4::kHcMultMax * dsv4::kHcMultMax;
  a.out = R.x + static_cast<size_t>(r) * c.hidden;
  return dsv4::launch_pdl(dsv4::hc_reduce_kernel, dim3(1), dim3(dsv4::kHcThreads), 0, st, a);
}

cudaError_t hc_post(dsv4cuda_decoder* D, const HcRows& R, int r, cudaStream_t st) {
  const int hid = D->cfg.hidden;
  return dsv4::launch_pdl(dsv4::hc_post_kernel, dim3((hid + 255) / 256), dim3(256), 0, st,
                          R.state + static_cast<size_t>(r) * D->cfg.hc_mult * hid,
                          R.branch + static_cast<size_t>(r) * hid,
                          static_cast<const float*>(R.post + r * dsv4::kHcMultMax),
                          static_cast<const float*>(R.comb + r * dsv4::kHcMultMax * dsv4::kHcMultMax),
                          D->cfg.hc_mult, hid);
}

// One hyper-connection boundary over R's rows: hc_post of R.branch (when
// `post`), then hc_pre of the next branch into R.x, and when xq is set its
// FP8 quant into xq / xs (row r at + r xq_ld). The fast mode runs it as one
// launch (CTA row blockIdx.y = row), with a layer boundary's Sinkhorn split
// forked onto D->hc_side (joined by hc_join before the next boundary); the
// exact mode keeps the sequential mix chains in launches of their own.
cudaError_t hc_boundary(dsv4cuda_decoder* D, const HcRows& R, bool post, const float* fn,
                        const float* scale, const float* base, const uint16_t* norm, int head,
                        __half* xq, float* xs, int xq_ld, cudaStream_t st) {
  const auto& c = D->cfg;
  if (c.hc_exact) {
    for (int r = 0; r < R.n; ++r) {
      if (post) DEC_CHECK(hc_post(D, R, r, st));
      DEC_CHECK(hc_pre(D, R, r, fn, scale, base, norm, head, st));
    }
    return xq ? dsv4::launch_quant_fp8(R.x, c.hidden, c.hidden, R.n, xq, xs, xq_ld, st)
              : cudaSuccess;
  }
  dsv4::HcFusedArgs a{};
  a.state = R.state;
  a.branch = post ? R.branch : nullptr;
  a.post_in = R.post;
  a.comb_in = R.comb;
  a.fn = fn;
  a.rows = head ? c.hc_mult : (2 + c.hc_mult) * c.hc_mult;
  a.head = head;
  a.scale = scale;
  a.base = base;
  a.hid = c.hidden;
  a.hc_eps = c.hc_eps;
  a.rms_eps = c.rms_eps;
  a.norm = norm;
  a.mix_out = R.mix;
  a.out = R.x;
  a.xq = xq;
  a.xs = xs;
  a.part = R.part;
  a.ticket = R.ticket;
  a.xq_ld = xq_ld;
  a.part_rs = R.part_rs;
  const int cols = dsv4::kHcfThreads / c.hc_mult;
  const dim3 grid((c.hidden + cols - 1) / cols, R.n), block(dsv4::kHcfThreads);
  cudaError_t e;
  switch (c.hc_mult) {
    case 1: e = dsv4::launch_pdl(dsv4::hc_fused_kernel<1>, grid, block, 0, st, a); break;
    case 2: e = dsv4::launch_pdl(dsv4::hc_fused_kernel<2>, grid, block, 0, st, a); break;
    case 3: e = dsv4::launch_pdl(dsv4::hc_fused_kernel<3>, grid, block, 0, st, a); break;
    default: e = dsv4::launch_pdl(dsv4::hc_fused_kernel<4>, grid, block, 0, st, a); break;
  }
  if (e != cudaSuccess || head) return e;
  // the split of the post / comb mixes beside the branch
  DEC_CHECK(cudaEventRecord(D->hc_fork, st));
  DEC_CHECK(cudaStreamWaitEvent(D->hc_side, D->hc_fork, 0));
  const float* mx = R.mix;
  switch (c.hc_mult) {
    case 1: dsv4::hc_sinkhorn_kernel<1><<<R.n, 32, 0, D->hc_side>>>(mx, scale, base, c.hc_iters, c.hc_eps, R.post, R.comb); break;
    case 2: dsv4::hc_sinkhorn_kernel<2><<<R.n, 32, 0, D->hc_side>>>(mx, scale, base, c.hc_iters, c.hc_eps, R.post, R.comb); break;
    case 3: dsv4::hc_sinkhorn_kernel<3><<<R.n, 32, 0, D->hc_side>>>(mx, scale, base, c.hc_iters, c.hc_eps, R.post, R.comb); break;
    default: dsv4::hc_sinkhorn_kernel<4><<<R.n, 32, 0, D->hc_side>>>(mx, scale, base, c.hc_iters, c.hc_eps, R.post, R.comb); break;
  }
  DEC_CHECK(cudaGetLastError());
  return cudaEventRecord(D->hc_join, D->hc_side);
}

// Makes `st` wait for the last forked split (fast mode; a no-op otherwise).
cudaError_t hc_join(dsv4cuda_decoder* D, cudaStream_t st) {
  return D->cfg.hc_exact ? cudaSuccess : cudaStreamWaitEvent(st, D->hc_join, 0);
}

// attention_forward_impl for a compress-ratio-0 layer (src/dsv4/dsv4_model.c:
// 5241-5429): writes the branch output [hid] into D->branch.
// D->x arrives with its FP8 quant in D->xq / D->xs.
cudaError_t attention_comp(dsv4cuda_decoder* D, dsv4::Layer& L, cudaStream_t st);

cudaError_t attention(dsv4cuda_decoder* D, dsv4::Layer& L, cudaStream_t st) {
  if (L.ratio) return attention_comp(D, L, st);
  const auto& c = D->cfg;
  const auto& w = L.w;
  const int H = c.n_heads, d = c.head_dim, ql = c.q_lora, half = c.rope_dim / 2;
  const int G = c.o_groups, ol = c.o_lora, hid = c.hidden;
  // wq_a and wkv on quant(x); kv: kv_norm -> RoPE -> FP8 latent into the
  // ring row of the position; q: q_norm -> quant -> wq_b -> per-head RMS + RoPE
  DEC_CHECK(fp8_gemv2(w.wq_a, w.wq_a_s, ql, D->qr, w.wkv, w.wkv_s, d, D->kv, hid, D->xq, D->xs,
                      D->ld, D->item1, D->n_one, D->fp8_part, D->tile_cnt, st));
  dsv4::NormTailArgs kt{};
  kt.x = D->kv;
  kt.n = d;
  kt.w = w.kv_norm;
  kt.eps = c.rms_eps;
  kt.half = half;
  kt.cosv = D->cosv;
  kt.sinv = D->sinv;
  kt.cache = L.cache;
  kt.row = D->row;
  if (D->win_staged) {
    kt.win = D->kvwin;
    kt.idx = D->idx;
    kt.n_win = c.window;
  }
  dsv4::NormTailArgs qt{};
  qt.x = D->qr;
  qt.n = ql;
  qt.w = w.q_norm;
  qt.eps = c.rms_eps;
  qt.xq = D->xq;
  qt.xs = D->xs;
  // one launch: CTA 0 writes the new latent, CTA 1 normalises and quantises
  // the q latent for wq_b, and with staging CTAs 2.. (eight rows each)
  // decode the rest of the window
  const int stage_ctas = D->win_staged ? (c.window + 7) / 8 : 0;
  DEC_CHECK(dsv4::launch_pdl(dsv4::norm_tail_kernel, dim3(2 + stage_ctas), dim3(256),
                             sizeof(float) * std::max(d, ql), st, kt, qt));
  DEC_CHECK(fp8_gemv(w.wq_b, w.wq_b_s, ql, H * d, D->xq, D->xs, D->ld, D->q, D->item1, D->n_one, D->fp8_part, D->tile_cnt, st));
  // the per-head RMS + RoPE of q: inside the attention CTAs when staged
  if (!D->win_staged)
    DEC_CHECK(dsv4::launch_pdl(dsv4::q_head_kernel, dim3(H), dim3(128), 0, st, D->q, d, c.rms_eps,
                               half, static_cast<const float*>(D->cosv),
                               static_cast<const float*>(D->sinv)));
  // sparse_attn over the window, inverse RoPE (exact order)
  dsv4::WinAttnArgs wa{};
  wa.q = D->q;
  wa.cache = L.cache;
  wa.idx = D->idx;
  wa.sink = w.attn_sink;
  wa.cosv = D->cosv;
  wa.sinv = D->sinv;
  wa.H = H;
  wa.d = d;
  wa.n = c.window;
  wa.rope_dim = c.rope_dim;
  wa.scale = 1.0f / sqrtf(static_cast<float>(d));
  wa.kvdec = D->kvdec;
  wa.kvt = D->kvt;
  wa.s = D->att_s;
  wa.w = D->att_w;
  wa.den = D->att_den;
  wa.out = D->o;
  // the attention boundary's split (consumed by the FFN boundary) joins here,
  // long after it finished
  DEC_CHECK(hc_join(D, st));
  if (D->win_staged) {
    wa.q_raw = 1;
    wa.q_eps = c.rms_eps;
    DEC_CHECK(dsv4::launch_pdl(dsv4::win_head_kernel, dim3(H), dim3(dsv4::kWhThreads),
                               dsv4::win_head_smem(c.window, d), st, wa,
                               static_cast<const uint16_t*>(D->kvwin), dsv4::device_error_word()));
  } else {
    DEC_CHECK(dsv4::launch_pdl(dsv4::win_decode_kernel, dim3(c.window), dim3(128), 0, st, wa));
    DEC_CHECK(dsv4::launch_pdl(
        dsv4::win_scores_kernel,
        dim3((H + dsv4::kWinHeads - 1) / dsv4::kWinHeads, (c.window + dsv4::kWinKeys - 1) / dsv4::kWinKeys),
        dim3(dsv4::kWinHeads * 32), D->win_smem, st, wa));
    DEC_CHECK(dsv4::launch_pdl(dsv4::win_softmax_kernel, dim3(H), dim3(256),
                               sizeof(float) * c.window, st, wa));
    DEC_CHECK(dsv4::launch_pdl(dsv4::win_values_kernel, dim3(H, (d / 2 + 63) / 64), dim3(64),
                               sizeof(float) * c.window, st, wa));
  }
  // grouped BF16 wo_a, then quant -> FP8 wo_b
  dsv4::Bf16GemvArgs ga{};
  ga.W = L.wo_a;
  ga.w_stride = static_cast<size_t>(ol) * (H * d / G);
  ga.in = H * d / G;
  ga.rows = ol;
  ga.round_out = 1;
  ga.x = D->o;
  ga.ldx = H * d / G;
  ga.Y = D->oall;
  ga.items = D->items_g;
  ga.n_items = D->n_groups;
  ga.max_items = G;
  ga.static_items = 1;
  DEC_CHECK(dsv4::launch_bf16_gemv(ga, 1, st));
  return fp8_gemv(w.wo_b, w.wo_b_s, G * ol, hid, D->xq, D->xs, D->ld, D->branch, D->item1,
                  D->n_one, D->fp8_part, D->tile_cnt, st, D->oall);
}

size_t idx_score_smem(const dsv4cuda_decoder_config& c) {
  return sizeof(float) * (static_cast<size_t>(c.index_dim + 1) * c.index_heads +
                          static_cast<size_t>(dsv4::kIdxT) * c.index_dim +
                          static_cast<size_t>(dsv4::kIdxT) * c.index_heads + c.index_heads);
}

// A BF16 projection of the layer input D->x (one token) into y.
cudaError_t bf16_x(dsv4cuda_decoder* D, const uint16_t* W, int rows, int round_out, float* y,
                   cudaStream_t st) {
  dsv4::Bf16GemvArgs a{};
  a.W = W;
  a.in = D->cfg.hidden;
  a.rows = rows;
  a.round_out = round_out;
  a.x = D->x;
  a.ldx = D->cfg.hidden;
  a.Y = y;
  a.items = D->item1;
  a.n_items = D->n_one;
  a.max_items = 1;
  a.static_items = 1;
  return dsv4::launch_bf16_gemv(a, 1, st);
}

dsv4::CompStepArgs comp_args(dsv4cuda_decoder* D, dsv4::Layer& L, bool indexer, const float* ape,
                             const uint16_t* norm, const float* kv, const float* sc) {
  const auto& c = D->cfg;
  dsv4::CompStepArgs a{};
  a.kv = kv;
  a.sc = sc;
  a.ape = ape;
  a.norm = norm;
  a.rope_dim = c.rope_dim;
  a.eps = c.rms_eps;
  a.pos = D->d_pos;
  a.max_count = L.max_count;
  a.cos_tab = D->cos_tab_c;
  a.sin_tab = D->sin_tab_c;
  a.max_pos = c.max_context;
  a.err = dsv4::device_error_word();
  if (indexer) {
    a.kvs = L.idx_kvs;
    a.scs = L.idx_scs;
    a.d = c.index_dim;
    a.ratio = 4;
    a.coff = 2;
    a.rotate = 1;
    a.count = L.idx_count;
    a.out = L.idx_rows;
  } else {
    a.kvs = L.kvs;
    a.scs = L.scs;
    a.d = c.head_dim;
    a.ratio = L.ratio;
    a.coff = L.coff;
    a.count = L.count;
    a.cache = L.cache;
    a.row0 = L.comp_row0;
  }
  return a;
}

// One launch of n (1 or 2) compressor steps, CTA i = step i; the block
// fits the widest. With list: a ratio-128 layer's key list after its step.
cudaError_t comp_steps(const dsv4::CompStepArgs* a, int n, cudaStream_t st,
                       const int* win_idx = nullptr, int win = 0, int* list = nullptr,
                       int n_list = 0) {
  dsv4::CompStepPair p{};
  p.win_idx = win_idx;
  p.win = win;
  p.list = list;
  p.n_list = n_list;
  int d = 0;
  for (int i = 0; i < n; ++i) {
    p.a[i] = a[i];
    d = std::max(d, a[i].d);
  }
  const int threads = std::min(1024, std::max(32, (d + 31) / 32 * 32));
  return dsv4::launch_pdl(dsv4::comp_step_kernel, dim3(n), dim3(threads), sizeof(float) * d, st, p);
}

// attention_forward_impl for a compress-ratio-4 or -128 layer (src/dsv4/
// dsv4_model.c:5241-5429): the window layer's projections (the q / kv RoPE
// from the compressed table), then compressor_update (:5319), for ratio 4
// indexer_forward (:5685: its query, its own compressor, the scores and the
// top-k), the key list window + compressed rows, sparse_attn over it and the
// output projections. D->x arrives with its FP8 quant in D->xq / D->xs.
cudaError_t attention_comp(dsv4cuda_decoder* D, dsv4::Layer& L, cudaStream_t st) {
  const auto& c = D->cfg;
  const auto& w = L.w;
  const int H = c.n_heads, d = c.head_dim, ql = c.q_lora, half = c.rope_dim / 2;
  const int G = c.o_groups, ol = c.o_lora, hid = c.hidden;
  // the stacked BF16 projections of x (compressor, indexer compressor,
  // indexer weights) beside the q / kv path
  DEC_CHECK(cudaEventRecord(D->comp_fork, st));
  DEC_CHECK(cudaStreamWaitEvent(D->comp_side, D->comp_fork, 0));
  DEC_CHECK(bf16_x(D, L.comp_w, L.comp_rows, 0, D->comp_proj, D->comp_side));
  DEC_CHECK(cudaEventRecord(D->comp_join, D->comp_side));
  const float* p_kv = D->comp_proj;
  const float* p_sc = p_kv + L.coff * d;
  const float* p_ikv = p_sc + L.coff * d;
  const float* p_isc = p_ikv + 2 * c.index_dim;
  const float* p_iw = p_isc + 2 * c.index_dim;
  DEC_CHECK(fp8_gemv2(w.wq_a, w.wq_a_s, ql, D->qr, w.wkv, w.wkv_s, d, D->kv, hid, D->xq, D->xs,
                      D->ld, D->item1, D->n_one, D->fp8_part, D->tile_cnt, st));
  dsv4::NormTailArgs kt{};
  kt.x = D->kv;
  kt.n = d;
  kt.w = w.kv_norm;
  kt.eps = c.rms_eps;
  kt.half = half;
  kt.cosv = D->cosv_c;
  kt.sinv = D->sinv_c;
  kt.cache = L.cache;
  kt.row = D->row;
  dsv4::NormTailArgs qt{};
  qt.x = D->qr;
  qt.n = ql;
  qt.w = w.q_norm;
  qt.eps = c.rms_eps;
  qt.xq = D->xq;
  qt.xs = D->xs;
  DEC_CHECK(dsv4::launch_pdl(dsv4::norm_tail_kernel, dim3(2), dim3(256),
                             sizeof(float) * std::max(d, ql), st, kt, qt));
  // wq_b, and for ratio 4 the indexer's query projection of the same
  // quantised q latent, in one split-K launch
  if (L.ratio == 4)
    DEC_CHECK(fp8_gemv2(w.wq_b, w.wq_b_s, H * d, D->q, w.idx_wq_b, w.idx_wq_b_s,
                        c.index_heads * c.index_dim, D->idx_q, ql, D->xq, D->xs, D->ld, D->item1,
                        D->n_one, D->fp8_part, D->tile_cnt, st));
  else
    DEC_CHECK(fp8_gemv(w.wq_b, w.wq_b_s, ql, H * d, D->xq, D->xs, D->ld, D->q, D->item1, D->n_one,
                       D->fp8_part, D->tile_cnt, st));
  // the per-head RMS + RoPE of q needs only wq_b: it runs while the side
  // stream's compressor projections finish
  DEC_CHECK(dsv4::launch_pdl(dsv4::q_head_kernel, dim3(H), dim3(128), 0, st, D->q, d, c.rms_eps,
                             half, static_cast<const float*>(D->cosv_c),
                             static_cast<const float*>(D->sinv_c)));
  DEC_CHECK(cudaStreamWaitEvent(st, D->comp_join, 0));
  {
    // the main compressor's step (its row into the cache) and, for ratio 4,
    // the indexer's compressor step (its row into the indexer's keys)
    dsv4::CompStepArgs ca[2] = {comp_args(D, L, false, w.comp_ape, w.comp_norm, p_kv, p_sc), {}};
    if (L.ratio == 4) {
      ca[1] = comp_args(D, L, true, w.idx_ape, w.idx_comp_norm, p_ikv, p_isc);
      DEC_CHECK(comp_steps(ca, 2, st));
    } else {  // ratio 128: every compressed row is a key; the list in the same launch
      DEC_CHECK(comp_steps(ca, 1, st, D->idx, c.window, D->idx_full, L.n_keys));
    }
  }
  const int* win_idx = D->idx;
  if (L.ratio == 4) {
    const int ih = c.index_heads, id = c.index_dim;
    DEC_CHECK(dsv4::launch_pdl(dsv4::idx_score_kernel,
                               dim3((L.max_count + dsv4::kIdxT - 1) / dsv4::kIdxT),
                               dim3(dsv4::kIdxT * ih), idx_score_smem(c), st,
                               static_cast<const float*>(D->idx_q),
                               static_cast<const float*>(L.idx_rows), p_iw, ih, id, c.rope_dim,
                               static_cast<const float*>(D->cosv_c),
                               static_cast<const float*>(D->sinv_c),
                               static_cast<const int*>(L.idx_count),
                               static_cast<const int*>(D->d_pos), D->idx_score));
    DEC_CHECK(dsv4::launch_pdl(dsv4::comp_list_kernel, dim3(1), dim3(dsv4::kListThreads),
                               dsv4::comp_list_smem(D->idx_n2), st, win_idx, c.window,
                               static_cast<const float*>(D->idx_score),
                               static_cast<const int*>(L.idx_count),
                               static_cast<const int*>(D->d_pos), c.index_topk, L.comp_row0,
                               D->idx_n2, L.n_keys, D->idx_full));
  }
  // sparse_attn over the list with the inverse RoPE, in the reference's
  // order: the rows decoded, every (head, key) score, per head the softmax
  // and the key-order denominator, per (head, dimension pair) the key-order
  // value chains (q's per-head RMS + RoPE ran before the side stream's join)
  dsv4::WinAttnArgs wa{};
  wa.q = D->q;
  wa.cache = L.cache;
  wa.idx = D->idx_full;
  wa.sink = w.attn_sink;
  wa.cosv = D->cosv_c;
  wa.sinv = D->sinv_c;
  wa.H = H;
  wa.d = d;
  wa.n = L.n_keys;
  wa.rope_dim = c.rope_dim;
  wa.scale = 1.0f / sqrtf(static_cast<float>(d));
  wa.kvdec = D->c_kvdec;
  wa.kvt = D->c_kvt;
  wa.s = D->c_att_s;
  wa.w = D->c_att_w;
  wa.den = D->att_den;
  wa.out = D->o;
  DEC_CHECK(hc_join(D, st));
  DEC_CHECK(dsv4::launch_pdl(dsv4::win_decode_kernel, dim3(L.n_keys), dim3(128), 0, st, wa));
  DEC_CHECK(dsv4::launch_pdl(
      dsv4::win_scores_rows_kernel,
      dim3((H + dsv4::kWinHeads - 1) / dsv4::kWinHeads, (L.n_keys + dsv4::kWinKeys - 1) / dsv4::kWinKeys),
      dim3(dsv4::kWinHeads * 32), dsv4::win_scores_rows_smem(d), st, wa));
  if (D->vmh_smem && dsv4::win_values_mh_smem(L.n_keys) <= D->vmh_smem)
    DEC_CHECK(dsv4::launch_pdl(dsv4::win_values_mh_kernel,
                               dim3((H + dsv4::kVhHeads - 1) / dsv4::kVhHeads, d / dsv4::kVhCols),
                               dim3(dsv4::kVhThreads), dsv4::win_values_mh_smem(L.n_keys), st, wa));
  else
    DEC_CHECK(dsv4::launch_pdl(
        dsv4::win_values_long_kernel, dim3(H, (d + 2 * dsv4::kValThreads - 1) / (2 * dsv4::kValThreads)),
        dim3(dsv4::kValThreads), dsv4::win_values_long_smem(L.n_keys), st, wa));
  dsv4::Bf16GemvArgs ga{};
  ga.W = L.wo_a;
  ga.w_stride = static_cast<size_t>(ol) * (H * d / G);
  ga.in = H * d / G;
  ga.rows = ol;
  ga.round_out = 1;
  ga.x = D->o;
  ga.ldx = H * d / G;
  ga.Y = D->oall;
  ga.items = D->items_g;
  ga.n_items = D->n_groups;
  ga.max_items = G;
  ga.static_items = 1;
  DEC_CHECK(dsv4::launch_bf16_gemv(ga, 1, st));
  return fp8_gemv(w.wo_b, w.wo_b_s, G * ol, hid, D->xq, D->xs, D->ld, D->branch, D->item1,
                  D->n_one, D->fp8_part, D->tile_cnt, st, D->oall);
}

// One decode step from device token/position into logits + argmax.
cudaError_t step(dsv4cuda_decoder* D, cudaStream_t st) {
  const auto& c = D->cfg;
  const int hid = c.hidden, half = c.rope_dim / 2;
  DEC_CHECK(dsv4::launch_pdl(dsv4::embed_kernel, dim3((hid + 255) / 256), dim3(256), 0, st,
                             D->g.embed, static_cast<const int*>(D->d_token), c.vocab, hid,
                             c.hc_mult, D->state));
  DEC_CHECK(dsv4::launch_pdl(dsv4::position_kernel, dim3(1), dim3(128), 0, st,
                             static_cast<const int*>(D->d_pos), c.window, half, c.max_context,
                             static_cast<const float*>(D->cos_tab),
                             static_cast<const float*>(D->sin_tab), D->idx, D->row, D->cosv,
                             D->sinv, static_cast<const float*>(D->cos_tab_c),
                             static_cast<const float*>(D->sin_tab_c), D->cosv_c, D->sinv_c));
  dsv4::MoeExecOptions opt;
  opt.x_quantized = true;
  if (!c.hc_exact) opt.join = D->hc_join;  // the FFN boundary's split, before the combine
  for (size_t li = 0; li < D->layers.size(); ++li) {
    auto& L = D->layers[li];
    const auto& w = L.w;
    DEC_CHECK(hc_boundary(D, hc_single(D), li > 0, w.hc_attn_fn, w.hc_attn_scale, w.hc_attn_base,
                          w.attn_norm, 0, D->xq, D->xs, D->ld, st));
    DEC_CHECK(attention(D, L, st));
    // the MoE layer's input quant comes out of the boundary kernel (its
    // shared-expert item for the one token was written at create)
    const bool local = D->ep.empty();
    DEC_CHECK(hc_boundary(D, hc_single(D), true, w.hc_ffn_fn, w.hc_ffn_scale, w.hc_ffn_base,
                          w.ffn_norm, 0, local ? D->moe_ws.xq : nullptr,
                          local ? D->moe_ws.xs : nullptr, c.hidden, st));
    if (!local) {
      const int rc = D->ep_replicated
                         ? dsv4cuda_moe_forward_ep(D->ep[li], D->x, D->d_token, 1, D->branch, st)
                         : dsv4cuda_moe_forward_ep_tokens(D->ep[li], D->x, 1, D->branch, st);
      if (rc != 0) return cudaErrorLaunchFailure;
      DEC_CHECK(hc_join(D, st));
    } else {
      DEC_CHECK(dsv4::moe_forward(L.mc, L.mw, D->moe_ws, D->x, D->d_token, 1, D->branch, st, opt));
    }
  }
  // the last layer's hc_post, model_head + head_logits (src/dsv4/dsv4_model.c:
  // 7755-7760), argmax
  DEC_CHECK(hc_boundary(D, hc_single(D), true, D->g.hc_head_fn, D->g.hc_head_scale,
                        D->g.hc_head_base, D->g.norm, 1, nullptr, nullptr, 0, st));
  dsv4::Bf16GemvArgs ha{};
  ha.W = D->g.head;
  ha.in = hid;
  ha.rows = c.vocab;
  ha.round_out = 0;
  ha.x = D->x;
  ha.ldx = hid;
  ha.Y = D->logits;
  ha.items = D->item1;
  ha.n_items = D->n_one;
  ha.max_items = 1;
  ha.static_items = 1;
  DEC_CHECK(dsv4::launch_bf16_gemv(ha, 1, st));
  const int chunks = std::min(dsv4::kArgmaxCtas, c.vocab);
  DEC_CHECK(dsv4::launch_pdl(dsv4::argmax_chunks_kernel, dim3(chunks), dim3(256), 0, st,
                             static_cast<const float*>(D->logits), c.vocab, D->am_v, D->am_i));
  return dsv4::launch_pdl(dsv4::argmax_final_kernel, dim3(1), dim3(32), 0, st,
                          static_cast<const float*>(D->am_v), static_cast<const int*>(D->am_i),
                          chunks, D->argmax);
}

// The compressor / indexer state of every compressed layer to its start:
// kv state zeros, score state -inf, no compressed rows (as the reference's
// layer run state, src/dsv4/dsv4_model.c:2423-2432, 2693-2700).
cudaError_t comp_reset(dsv4cuda_decoder* D, cudaStream_t st) {
  const auto& c = D->cfg;
  for (auto& L : D->layers) {
    if (!L.ratio) continue;
    const size_t nst = static_cast<size_t>(L.coff) * L.ratio * L.coff * c.head_dim;
    DEC_CHECK(cudaMemsetAsync(L.kvs, 0, nst * sizeof(float), st));
    dsv4::fill_f32_kernel<<<64, 256, 0, st>>>(L.scs, nst, -INFINITY);
    DEC_CHECK(cudaGetLastError());
    DEC_CHECK(cudaMemsetAsync(L.count, 0, sizeof(int), st));
    if (L.ratio == 4) {
      const size_t nidx = 16 * static_cast<size_t>(c.index_dim);
      DEC_CHECK(cudaMemsetAsync(L.idx_kvs, 0, nidx * sizeof(float), st));
      dsv4::fill_f32_kernel<<<16, 256, 0, st>>>(L.idx_scs, nidx, -INFINITY);
      DEC_CHECK(cudaGetLastError());
      DEC_CHECK(cudaMemsetAsync(L.idx_count, 0, sizeof(int), st));
    }
  }
  return cudaSuccess;
}

// Buffers shared by the compressed layers, the YaRN RoPE table, the kernels'
// shared-memory limits, and every layer's state at its start. D->err says
// what failed.
bool comp_alloc(dsv4cuda_decoder* D) {
  const auto& c = D->cfg;
  const int half = c.rope_dim / 2;
  if (c.index_heads <= 0 || c.index_dim < 32 || c.index_dim > 256 ||
      (c.index_dim & (c.index_dim - 1)) || c.index_dim < c.rope_dim ||
      c.index_heads * dsv4::kIdxT > 1024 ||
      c.index_topk <= 0 || c.compress_rope_theta <= 0.f || c.rope_factor <= 0.f ||
      c.original_position <= 0 || D->idx_n2 > 8192 ||
      idx_score_smem(c) > 200 * 1024) {
    D->err = "index heads / dim (a power of two in [32, 256], >= rope_dim) / top-k or the YaRN "
             "parameters out of range, or max_context too long for the top-k sort";
    return false;
  }
  bool ok = true;
  auto chk = [&](const void* p) { ok = ok && p != nullptr; };
  chk(D->cosv_c = dalloc<float>(D, half));
  chk(D->sinv_c = dalloc<float>(D, half));
  chk(D->cos_tab_c = dalloc<float>(D, static_cast<size_t>(c.max_context) * half));
  chk(D->sin_tab_c = dalloc<float>(D, static_cast<size_t>(c.max_context) * half));
  chk(D->comp_proj = dalloc<float>(D, D->comp_rows_max));
  chk(D->idx_q = dalloc<float>(D, static_cast<size_t>(c.index_heads) * c.index_dim));
  chk(D->idx_score = dalloc<float>(D, std::max(D->idx_n2, 1)));
  chk(D->idx_full = dalloc<int>(D, D->n_max));
  chk(D->c_kvdec = dalloc<float>(D, static_cast<size_t>(D->n_max) * c.head_dim));
  chk(D->c_kvt = dalloc<float>(D, static_cast<size_t>(D->n_max) * c.head_dim));
  chk(D->c_att_s = dalloc<float>(D, static_cast<size_t>(D->n_max) * c.n_heads));
  chk(D->c_att_w = dalloc<float>(D, static_cast<size_t>(D->n_max) * c.n_heads));
  if (!ok) {
    D->err = "out of device memory";
    return false;
  }
  // the multi-head value pass while its shared-memory slice of the longest
  // list fits 200 KB (the longer lists of ratio-128 layers at long contexts
  // take win_values_long_kernel)
  if (c.head_dim % dsv4::kVhCols == 0)
    D->vmh_smem = std::min<size_t>(dsv4::win_values_mh_smem(D->n_max), 200 * 1024);
  if (cudaStreamCreateWithFlags(&D->comp_side, cudaStreamNonBlocking) != cudaSuccess ||
      cudaEventCreateWithFlags(&D->comp_fork, cudaEventDisableTiming) != cudaSuccess ||
      cudaEventCreateWithFlags(&D->comp_join, cudaEventDisableTiming) != cudaSuccess) {
    D->err = "stream / event creation failed";
    return false;
  }
  std::vector<float> cs, sn;
  rope_tables_yarn(c, cs, sn);
  if (cudaMemcpy(D->cos_tab_c, cs.data(), cs.size() * sizeof(float), cudaMemcpyHostToDevice) != cudaSuccess ||
      cudaMemcpy(D->sin_tab_c, sn.data(), sn.size() * sizeof(float), cudaMemcpyHostToDevice) != cudaSuccess ||
      dsv4::set_max_dynamic_smem(reinterpret_cast<const void*>(dsv4::win_scores_kernel),
                                 static_cast<int>(sizeof(float) * (dsv4::kWinHeads + dsv4::kWinKeys) *
                                                  c.head_dim)) != cudaSuccess ||
      dsv4::set_max_dynamic_smem(reinterpret_cast<const void*>(dsv4::comp_list_kernel),
                                 static_cast<int>(dsv4::comp_list_smem(D->idx_n2))) != cudaSuccess ||
      dsv4::set_max_dynamic_smem(reinterpret_cast<const void*>(dsv4::idx_score_kernel),
                                 static_cast<int>(idx_score_smem(c))) != cudaSuccess ||
      dsv4::set_max_dynamic_smem(reinterpret_cast<const void*>(dsv4::win_scores_rows_kernel),
                                 static_cast<int>(dsv4::win_scores_rows_smem(c.head_dim))) != cudaSuccess ||
      dsv4::set_max_dynamic_smem(reinterpret_cast<const void*>(dsv4::win_values_long_kernel),
                                 static_cast<int>(dsv4::win_values_long_smem(D->n_max))) != cudaSuccess ||
      (D->vmh_smem && dsv4::set_max_dynamic_smem(reinterpret_cast<const void*>(dsv4::win_values_mh_kernel),
                                                 static_cast<int>(D->vmh_smem)) != cudaSuccess) ||
      comp_reset(D, nullptr) != cudaSuccess) {
    D->err = "set-up failed";
    return false;
  }
  return true;
}

// The verify step's buffers (DSV4CUDA_VERIFY_MAX_ROWS rows), its GEMV items
// for every row count, the layer caches for the commit kernel and a MoE
// workspace for that many tokens. Called by create after the layers exist.
bool verify_alloc(dsv4cuda_decoder* D) {
  const auto& c = D->cfg;
  auto& v = D->v;
  constexpr int V = DSV4CUDA_VERIFY_MAX_ROWS;
  const int H = c.n_heads, d = c.head_dim, half = c.rope_dim / 2, G = c.o_groups;
  const size_t hid = c.hidden, hd = static_cast<size_t>(H) * d;
  bool ok = true;
  auto chk = [&](const void* p) { ok = ok && p != nullptr; };
  chk(v.tok = dalloc<int>(D, V));
  chk(v.start = dalloc<int>(D, 1));
  chk(v.from = dalloc<int>(D, 1));
  chk(v.count = dalloc<int>(D, 1));
  chk(v.stats = dalloc<long long>(D, 3));
  chk(v.rng = dalloc<unsigned long long>(D, 1));
  chk(v.state = dalloc<float>(D, V * c.hc_mult * hid));
  v.part_rs = std::max(static_cast<size_t>(D->nblk) * (dsv4::kMixMax + 1),
                       static_cast<size_t>(dsv4::kHcfMaxCtas) * 32);
  chk(v.part = dalloc<double>(D, V * v.part_rs));
  chk(v.ticket = dalloc<unsigned int>(D, V));
  chk(v.mix = dalloc<float>(D, V * dsv4::kMixMax));
  chk(v.post = dalloc<float>(D, V * dsv4::kHcMultMax));
  chk(v.comb = dalloc<float>(D, V * dsv4::kHcMultMax * dsv4::kHcMultMax));
  chk(v.x = dalloc<float>(D, V * hid));
  chk(v.xq = dalloc<__half>(D, static_cast<size_t>(V) * D->ld));
  chk(v.xs = dalloc<float>(D, static_cast<size_t>(V) * D->ld / 128));
  chk(v.qr = dalloc<float>(D, static_cast<size_t>(V) * c.q_lora));
  chk(v.q = dalloc<float>(D, V * hd));
  chk(v.kv = dalloc<float>(D, static_cast<size_t>(V) * d));
  chk(v.o = dalloc<float>(D, V * hd));
  chk(v.oall = dalloc<float>(D, static_cast<size_t>(V) * G * c.o_lora));
  chk(v.branch = dalloc<float>(D, V * hid));
  if (D->win_staged) chk(v.kvwin = dalloc<uint16_t>(D, static_cast<size_t>(V) * c.window * d));
  chk(v.idx = dalloc<int>(D, static_cast<size_t>(V) * c.window));
  chk(v.row = dalloc<long long>(D, V));
  chk(v.cosv = dalloc<float>(D, static_cast<size_t>(V) * half));
  chk(v.sinv = dalloc<float>(D, static_cast<size_t>(V) * half));
  chk(v.logits = dalloc<float>(D, static_cast<size_t>(V) * c.vocab));
  chk(v.argmax = dalloc<int>(D, V));
  chk(v.am_v = dalloc<float>(D, static_cast<size_t>(V) * dsv4::kArgmaxCtas));
  chk(v.am_i = dalloc<int>(D, static_cast<size_t>(V) * dsv4::kArgmaxCtas));
  chk(v.items = dalloc<dsv4::GemvItem>(D, V));
  chk(v.items_g = dalloc<dsv4::GemvItem>(D, static_cast<size_t>(V) * G));
  chk(v.n_one = dalloc<int>(D, 1));
  chk(v.n_groups = dalloc<int>(D, 1));
  chk(v.caches = dalloc<dsv4::Fp8KvCache>(D, D->layers.size()));
  {
    // [V][in / 128][rows] for the largest projection (wq_a + wkv, wq_b, wo_b)
    const size_t ql = c.q_lora, go = static_cast<size_t>(G) * c.o_lora;
    v.mt_part_floats = V * std::max(std::max(hid / 128 * (ql + d), ql / 128 * hd), go / 128 * hid);
    chk(v.mt_part = dalloc<float>(D, v.mt_part_floats));
  }
  if (!ok) return false;
  std::vector<dsv4::GemvItem> it(V), itg(static_cast<size_t>(V) * G);
  for (int n = 1; n <= V; ++n) {
    auto& a = it[n - 1];
    a = dsv4::GemvItem{};
    a.mat = 0;
    a.ntok = n;
    for (int t = 0; t < n; ++t) a.tok[t] = dsv4::TokMap{t, t};
    for (int g = 0; g < G; ++g) {
      auto& b = itg[static_cast<size_t>(n - 1) * G + g];
      b = dsv4::GemvItem{};
      b.mat = g;
      b.ntok = n;
      for (int t = 0; t < n; ++t) b.tok[t] = dsv4::TokMap{t * G + g, t * G + g};
    }
  }
  std::vector<dsv4::Fp8KvCache> caches;
  for (const auto& L : D->layers) caches.push_back(L.cache);
  const int one = 1;
  const unsigned long long seed = 0x9E3779B97F4A7C15ull;
  if (cudaMemcpy(v.items, it.data(), sizeof(dsv4::GemvItem) * it.size(), cudaMemcpyHostToDevice) != cudaSuccess ||
      cudaMemcpy(v.items_g, itg.data(), sizeof(dsv4::GemvItem) * itg.size(), cudaMemcpyHostToDevice) != cudaSuccess ||
      cudaMemcpy(v.n_one, &one, sizeof(int), cudaMemcpyHostToDevice) != cudaSuccess ||
      cudaMemcpy(v.n_groups, &G, sizeof(int), cudaMemcpyHostToDevice) != cudaSuccess ||
      cudaMemcpy(v.rng, &seed, sizeof(seed), cudaMemcpyHostToDevice) != cudaSuccess ||
      cudaMemcpy(v.caches, caches.data(), sizeof(dsv4::Fp8KvCache) * caches.size(),
                 cudaMemcpyHostToDevice) != cudaSuccess)
    return false;
  dsv4::MoeConfig mc = D->layers[0].mc;
  mc.hash_vocab = 0;
  char* base = dalloc<char>(D, dsv4::moe_workspace_bytes(mc, V));
  if (!base) return false;
  dsv4::moe_workspace_carve(&v.moe_ws, mc, V, base);
  return true;
}

// A BF16 GEMV over a verify step's n rows: the (row, token)-lane kernel, or
// the item kernel when the shape does not fit it.
cudaError_t bf16_rows(const dsv4::Bf16GemvArgs& a, int n, cudaStream_t st) {
  const cudaError_t e = n > 1 ? dsv4::launch_bf16_gemv_mt(a, n, st) : cudaErrorNotSupported;
  return e == cudaErrorNotSupported ? dsv4::launch_bf16_gemv(a, n, st) : e;
}

// attention_forward_batch_projected (src/dsv4/dsv4_model.c:5449-5572) for a
// verify step's n rows: every projection one GEMV over the n rows (the
// weights stream once), each row's latent into its scratch cache row, then
// every row's sparse_attn over its own window (which holds the earlier
// verify rows' latents, as the reference's row-by-row pass sees them).
// v.x arrives with its FP8 quant in v.xq / v.xs; the branch goes to v.branch.
cudaError_t verify_attention(dsv4cuda_decoder* D, dsv4::Layer& L, int n, cudaStream_t st) {
  const auto& c = D->cfg;
  auto& v = D->v;
  const auto& w = L.w;
  const int H = c.n_heads, d = c.head_dim, ql = c.q_lora, half = c.rope_dim / 2;
  const int G = c.o_groups, ol = c.o_lora, hid = c.hidden;
  // one matrix (or two on the same input) over the n rows: the split-K
  // multi-token kernels, else the item GEMVs
  auto gemv8 = [&](const uint8_t* W, const uint8_t* S, int in, int rows, float* y,
                   const uint8_t* W1 = nullptr, const uint8_t* S1 = nullptr, int rows1 = 0,
                   float* y1 = nullptr) -> cudaError_t {
    dsv4::Fp8GemvArgs a{};
    a.W[0] = W;
    a.S[0] = S;
    a.W[1] = W1;
    a.S[1] = S1;
    a.rows1 = rows1;
    a.Y[1] = y1;
    a.in = in;
    a.rows = rows;
    a.round_out = 1;
    a.act = dsv4::QAct{v.xq, v.xs, D->ld, nullptr};
    a.Y[0] = y;
    a.items = v.items + (n - 1);
    a.n_items = v.n_one;
    a.max_items = 1;
    if (dsv4::fp8_gemv_mt_part_floats(a, n) <= v.mt_part_floats) {
      const cudaError_t e = dsv4::launch_fp8_gemv_mt(a, n, v.mt_part, st);
      if (e != cudaErrorNotSupported) return e;
    }
    if (W1) return cudaErrorNotSupported;
    return dsv4::launch_fp8_gemv(a, false, n, st);
  };
  if (gemv8(w.wq_a, w.wq_a_s, hid, ql, v.qr, w.wkv, w.wkv_s, d, v.kv) == cudaErrorNotSupported) {
    DEC_CHECK(gemv8(w.wq_a, w.wq_a_s, hid, ql, v.qr));
    DEC_CHECK(gemv8(w.wkv, w.wkv_s, hid, d, v.kv));
  }
  // per row: kv_norm + RoPE + KV write into the scratch row; q_norm + quant
  dsv4::NormTailArgs kt{};
  kt.x = v.kv;
  kt.n = d;
  kt.w = w.kv_norm;
  kt.eps = c.rms_eps;
  kt.half = half;
  kt.cosv = v.cosv;
  kt.sinv = v.sinv;
  kt.cache = L.cache;
  kt.row = v.row;
  kt.x_rs = d;
  kt.cs_rs = half;
  dsv4::NormTailArgs qt{};
  qt.x = v.qr;
  qt.n = ql;
  qt.w = w.q_norm;
  qt.eps = c.rms_eps;
  qt.xq = v.xq;
  qt.xs = v.xs;
  qt.x_rs = ql;
  qt.xq_ld = D->ld;
  DEC_CHECK(dsv4::launch_pdl(dsv4::norm_tail_kernel, dim3(2, n), dim3(256),
                             sizeof(float) * std::max(d, ql), st, kt, qt));
  // every row's window as BF16, now that all the rows' latents are cached
  dsv4::NormTailArgs sa = kt;
  sa.win = v.kvwin;
  sa.idx = v.idx;
  sa.n_win = c.window;
  DEC_CHECK(dsv4::launch_pdl(dsv4::stage_rows_kernel, dim3((c.window + 7) / 8, n), dim3(256), 0,
                             st, sa));
  DEC_CHECK(gemv8(w.wq_b, w.wq_b_s, ql, H * d, v.q));
  dsv4::WinAttnArgs wa{};
  wa.q = v.q;
  wa.cache = L.cache;
  wa.idx = v.idx;
  wa.sink = w.attn_sink;
  wa.cosv = v.cosv;
  wa.sinv = v.sinv;
  wa.H = H;
  wa.d = d;
  wa.n = c.window;
  wa.rope_dim = c.rope_dim;
  wa.scale = 1.0f / sqrtf(static_cast<float>(d));
  wa.out = v.o;
  wa.q_raw = 1;
  wa.q_eps = c.rms_eps;
  DEC_CHECK(hc_join(D, st));
  DEC_CHECK(dsv4::launch_pdl(dsv4::win_head_kernel, dim3(H, n), dim3(dsv4::kWhThreads),
                             dsv4::win_head_smem(c.window, d), st, wa,
                             static_cast<const uint16_t*>(v.kvwin), dsv4::device_error_word()));
  // grouped BF16 wo_a over the rows, quant, FP8 wo_b
  dsv4::Bf16GemvArgs ga{};
  ga.W = L.wo_a;
  ga.w_stride = static_cast<size_t>(ol) * (H * d / G);
  ga.in = H * d / G;
  ga.rows = ol;
  ga.round_out = 1;
  ga.x = v.o;
  ga.ldx = H * d / G;
  ga.Y = v.oall;
  ga.items = v.items_g + static_cast<size_t>(n - 1) * G;
  ga.n_items = v.n_groups;
  ga.max_items = G;
  ga.static_items = 1;
  DEC_CHECK(bf16_rows(ga, n, st));
  DEC_CHECK(dsv4::launch_quant_fp8(v.oall, G * ol, G * ol, n, v.xq, v.xs, D->ld, st));
  return gemv8(w.wo_b, w.wo_b_s, G * ol, hid, v.branch);
}

// dsv4_prefill_capture with all_logits (src/dsv4/dsv4_model.c:8434-8529):
// rows v.tok[0 .. n) at positions *v.start + r through every layer
// layer-major (forward_loaded_layer_batch, :7577-7753), then the HC head,
// the vocab head of every row (compute_logits_batch, :7784) and each row's
// argmax. The ring is not written; the rows' latents wait in the scratch
// rows for a commit.
cudaError_t verify(dsv4cuda_decoder* D, int n, cudaStream_t st) {
  const auto& c = D->cfg;
  auto& v = D->v;
  const int hid = c.hidden, half = c.rope_dim / 2;
  DEC_CHECK(dsv4::launch_pdl(dsv4::embed_kernel, dim3((hid + 255) / 256, n), dim3(256), 0, st,
                             D->g.embed, static_cast<const int*>(v.tok), c.vocab, hid, c.hc_mult,
                             v.state));
  DEC_CHECK(dsv4::launch_pdl(dsv4::verify_position_kernel, dim3(n), dim3(128), 0, st,
                             static_cast<const int*>(v.start), c.window, half, c.max_context,
                             static_cast<const float*>(D->cos_tab),
                             static_cast<const float*>(D->sin_tab), v.idx, v.row, v.cosv, v.sinv));
  const HcRows R = hc_verify(D, n);
  dsv4::MoeExecOptions opt;
  if (!c.hc_exact) opt.join = D->hc_join;  // the FFN boundary's split, before the combine
  opt.mt_part = v.mt_part;  // the shared expert over the rows, split-K
  opt.mt_part_floats = v.mt_part_floats;
  for (size_t li = 0; li < D->layers.size(); ++li) {
    auto& L = D->layers[li];
    const auto& w = L.w;
    DEC_CHECK(hc_boundary(D, R, li > 0, w.hc_attn_fn, w.hc_attn_scale, w.hc_attn_base,
                          w.attn_norm, 0, v.xq, v.xs, D->ld, st));
    DEC_CHECK(verify_attention(D, L, n, st));
    DEC_CHECK(hc_boundary(D, R, true, w.hc_ffn_fn, w.hc_ffn_scale, w.hc_ffn_base, w.ffn_norm, 0,
                          nullptr, nullptr, 0, st));
    DEC_CHECK(dsv4::moe_forward(L.mc, L.mw, v.moe_ws, v.x, v.tok, n, v.branch, st, opt));
  }
  DEC_CHECK(hc_boundary(D, R, true, D->g.hc_head_fn, D->g.hc_head_scale, D->g.hc_head_base,
                        D->g.norm, 1, nullptr, nullptr, 0, st));
  dsv4::Bf16GemvArgs ha{};
  ha.W = D->g.head;
  ha.in = hid;
  ha.rows = c.vocab;
  ha.round_out = 0;
  ha.x = v.x;
  ha.ldx = hid;
  ha.Y = v.logits;
  ha.items = v.items + (n - 1);
  ha.n_items = v.n_one;
  ha.max_items = 1;
  ha.static_items = 1;
  DEC_CHECK(bf16_rows(ha, n, st));
  const int chunks = std::min(dsv4::kArgmaxCtas, c.vocab);
  DEC_CHECK(dsv4::launch_pdl(dsv4::argmax_chunks_kernel, dim3(chunks, n), dim3(256), 0, st,
                             static_cast<const float*>(v.logits), c.vocab, v.am_v, v.am_i));
  return dsv4::launch_pdl(dsv4::argmax_final_kernel, dim3(n), dim3(32), 0, st,
                          static_cast<const float*>(v.am_v), static_cast<const int*>(v.am_i),
                          chunks, v.argmax);
}

cudaError_t verify_commit(dsv4cuda_decoder* D, const int* from, cudaStream_t st) {
  return dsv4::launch_pdl(dsv4::verify_commit_kernel,
                          dim3(static_cast<unsigned>(D->layers.size()), DSV4CUDA_VERIFY_MAX_ROWS),
                          dim3(128), 0, st, static_cast<const dsv4::Fp8KvCache*>(D->v.caches),
                          D->cfg.window, from, static_cast<const int*>(D->v.count));
}

const char* verify_unsupported(const dsv4cuda_decoder* D, int n) {
  if (n < 1 || n > DSV4CUDA_VERIFY_MAX_ROWS) return "n_rows must be 1 .. DSV4CUDA_VERIFY_MAX_ROWS";
  if (!D->ep.empty()) return "the verify step runs the local MoE layers (no expert parallelism)";
  if (D->any_comp) return "layers of compress ratio 4 / 128 decode one token at a time";
  if (!D->win_staged || !D->v.kvwin) return "the window does not fit the one-launch attention";
  return nullptr;
}

bool cfg_ok(const dsv4cuda_decoder_config* c) {
  return c && c->hidden > 0 && c->hidden % 128 == 0 && c->n_layers > 0 && c->vocab > 0 &&
         c->n_heads > 0 && c->head_dim > 0 && c->head_dim % 4 == 0 && c->rope_dim > 0 && c->rope_dim % 2 == 0 &&
         c->rope_dim <= c->head_dim && (c->head_dim - c->rope_dim) % 64 == 0 &&
         (c->head_dim - c->rope_dim) / 64 <= dsv4::kKvScaleSlots && c->q_lora > 0 &&
         c->o_groups > 0 && (c->n_heads * c->head_dim) % c->o_groups == 0 && c->o_lora > 0 &&
         c->window > 0 && c->window % 4 == 0 && c->hc_mult > 0 && c->hc_mult <= 4 &&
         c->hc_iters > 0 &&
         c->hidden <= 8 * dsv4::kHcThreads && c->head_dim <= 512 &&
         c->max_context > 0 && c->moe.hidden == c->hidden;
}

}  // namespace

DSV4_API const char* dsv4cuda_decoder_last_error(void) { return t_dec_error.c_str(); }

DSV4_API int dsv4cuda_decoder_create(dsv4cuda_decoder** out, const dsv4cuda_decoder_config* cfg,
                                     const dsv4cuda_model_weights* g,
                                     const dsv4cuda_layer_weights* layers) {
  if (!out || !cfg_ok(cfg) || !g || !layers || !g->embed || !g->head || !g->norm ||
      !g->hc_head_fn || !g->hc_head_base || !g->hc_head_scale)
    return fail("dsv4cuda_decoder_create: bad arguments (hc_mult <= 4, head_dim - rope_dim a "
                "multiple of 64 up to 512, hidden a multiple of 128)");
  auto* D = new dsv4cuda_decoder();
  D->cfg = *cfg;
  D->g = *g;
  const auto& c = D->cfg;
  const int H = c.n_heads, d = c.head_dim, half = c.rope_dim / 2;
  const int maxv = std::max(std::max(c.hidden, c.q_lora), std::max(c.o_groups * c.o_lora, H * d));
  D->ld = (maxv + 511) / 512 * 512;
  const int n = c.hc_mult * c.hidden;
  D->nblk = (n + dsv4::kMixThreads - 1) / dsv4::kMixThreads;
  bool ok = true;
  auto chk = [&](const void* p) { ok = ok && p != nullptr; };
  chk(D->d_token = dalloc<int>(D, 1));
  chk(D->d_pos = dalloc<int>(D, 1));
  chk(D->state = dalloc<float>(D, n));
  chk(D->part = dalloc<double>(D, std::max(static_cast<size_t>(D->nblk) * (dsv4::kMixMax + 1),
                                           static_cast<size_t>(dsv4::kHcfMaxCtas) * 32)));
  chk(D->hc_ticket = dalloc<unsigned int>(D, 1));
  chk(D->mix = dalloc<float>(D, dsv4::kMixMax));
  if (ok && (cudaStreamCreateWithFlags(&D->hc_side, cudaStreamNonBlocking) != cudaSuccess ||
             cudaEventCreateWithFlags(&D->hc_fork, cudaEventDisableTiming) != cudaSuccess ||
             cudaEventCreateWithFlags(&D->hc_join, cudaEventDisableTiming) != cudaSuccess))
    ok = false;
  chk(D->post = dalloc<float>(D, dsv4::kHcMultMax));
  chk(D->comb = dalloc<float>(D, dsv4::kHcMultMax * dsv4::kHcMultMax));
  chk(D->x = dalloc<float>(D, c.hidden));
  chk(D->xq = dalloc<__half>(D, D->ld));
  chk(D->xs = dalloc<float>(D, D->ld / 128));
  chk(D->qr = dalloc<float>(D, c.q_lora));
  chk(D->qn = dalloc<float>(D, c.q_lora));
  chk(D->q = dalloc<float>(D, static_cast<size_t>(H) * d));
  chk(D->kv = dalloc<float>(D, d));
  chk(D->o = dalloc<float>(D, static_cast<size_t>(H) * d));
  chk(D->oall = dalloc<float>(D, static_cast<size_t>(c.o_groups) * c.o_lora));
  chk(D->kvdec = dalloc<float>(D, static_cast<size_t>(c.window) * d));
  chk(D->kvt = dalloc<float>(D, static_cast<size_t>(c.window) * d));
  {
    const size_t hid = c.hidden, ql = c.q_lora;
    // wq_b's rows, with the indexer's query projection stacked after them
    const size_t hd = static_cast<size_t>(H) * d +
                      static_cast<size_t>(std::max(0, c.index_heads)) * std::max(0, c.index_dim);
    const size_t go = static_cast<size_t>(c.o_groups) * c.o_lora;
    const size_t np = std::max(std::max((hid + 127) / 128 * (ql + d), (ql + 127) / 128 * hd),
                               (go + 127) / 128 * hid);
    chk(D->fp8_part = dalloc<float>(D, np));
    const size_t maxr = std::max(std::max(ql + d, hd), std::max(hid, go));
    chk(D->tile_cnt = dalloc<unsigned int>(D, maxr / 32 + 1));
  }
  chk(D->att_s = dalloc<float>(D, static_cast<size_t>(H) * c.window));
  chk(D->att_w = dalloc<float>(D, static_cast<size_t>(H) * c.window));
  chk(D->att_den = dalloc<float>(D, H));
  chk(D->branch = dalloc<float>(D, c.hidden));
  chk(D->logits = dalloc<float>(D, c.vocab));
  chk(D->argmax = dalloc<int>(D, 1));
  chk(D->am_v = dalloc<float>(D, dsv4::kArgmaxCtas));
  chk(D->am_i = dalloc<int>(D, dsv4::kArgmaxCtas));
  chk(D->idx = dalloc<int>(D, c.window));
  chk(D->row = dalloc<long long>(D, 1));
  chk(D->cosv = dalloc<float>(D, half));
  chk(D->sinv = dalloc<float>(D, half));
  chk(D->cos_tab = dalloc<float>(D, static_cast<size_t>(c.max_context) * half));
  chk(D->sin_tab = dalloc<float>(D, static_cast<size_t>(c.max_context) * half));
  chk(D->item1 = dalloc<dsv4::GemvItem>(D, 1));
  chk(D->items_g = dalloc<dsv4::GemvItem>(D, c.o_groups));
  chk(D->n_one = dalloc<int>(D, 1));
  chk(D->n_groups = dalloc<int>(D, 1));
  if (!ok) {
    dsv4cuda_decoder_destroy(D);
    return fail("dsv4cuda_decoder_create: out of device memory");
  }
  {
    std::vector<float> cs, sn;
    rope_tables(c, cs, sn);
    cudaMemcpy(D->cos_tab, cs.data(), cs.size() * sizeof(float), cudaMemcpyHostToDevice);
    cudaMemcpy(D->sin_tab, sn.data(), sn.size() * sizeof(float), cudaMemcpyHostToDevice);
    std::vector<dsv4::GemvItem> items(c.o_groups);
    for (int gi = 0; gi < c.o_groups; ++gi) {
      items[gi] = dsv4::GemvItem{};
      items[gi].mat = gi;
      items[gi].ntok = 1;
      for (int t = 0; t < dsv4::kItemTok; ++t) items[gi].tok[t] = dsv4::TokMap{gi, gi};
    }
    dsv4::GemvItem one{};
    one.mat = 0;
    one.ntok = 1;
    const int n1 = 1, ng = c.o_groups;
    cudaMemcpy(D->item1, &one, sizeof(one), cudaMemcpyHostToDevice);
    cudaMemcpy(D->items_g, items.data(), sizeof(dsv4::GemvItem) * items.size(),
               cudaMemcpyHostToDevice);
    cudaMemcpy(D->n_one, &n1, sizeof(int), cudaMemcpyHostToDevice);
    cudaMemcpy(D->n_groups, &ng, sizeof(int), cudaMemcpyHostToDevice);
  }
  D->win_smem = sizeof(float) * (dsv4::kWinHeads + dsv4::kWinKeys) * static_cast<size_t>(d);
  if (D->win_smem > 48 * 1024 &&
      dsv4::set_max_dynamic_smem(reinterpret_cast<const void*>(dsv4::win_scores_kernel),
                                 static_cast<int>(D->win_smem)) != cudaSuccess) {
    dsv4cuda_decoder_destroy(D);
    return fail("dsv4cuda_decoder_create: head_dim %d needs too much shared memory", d);
  }
  {
    // the one-launch window attention holds the window's rows in shared
    // memory; larger windows keep the four-launch form
    const size_t wsm = dsv4::win_head_smem(c.window, d);
    D->win_staged = d % 16 == 0 && c.rope_dim % 16 == 0 && wsm <= 220 * 1024 &&
                    dsv4::set_max_dynamic_smem(reinterpret_cast<const void*>(dsv4::win_head_kernel),
                                               220 * 1024) == cudaSuccess;
    if (D->win_staged && !(D->kvwin = dalloc<uint16_t>(D, static_cast<size_t>(c.window) * d))) {
      dsv4cuda_decoder_destroy(D);
      return fail("dsv4cuda_decoder_create: out of device memory");
    }
  }
  // per layer: the FP8 latent ring, wo_a as BF16, the MoE layer's view
  const int nope = d - c.rope_dim;
  for (int li = 0; li < c.n_layers; ++li) {
    dsv4::Layer L;
    L.w = layers[li];
    const auto& w = L.w;
    if (!w.attn_norm || !w.ffn_norm || !w.hc_attn_fn || !w.hc_ffn_fn || !w.wq_a || !w.wq_b ||
        !w.wkv || !w.wo_b || !w.q_norm || !w.kv_norm || !w.attn_sink ||
        (!w.wo_a && !(w.wo_a_fp8 && w.wo_a_fp8_s)) || !w.moe.gate_w || !w.moe.w1) {
      dsv4cuda_decoder_destroy(D);
      return fail("dsv4cuda_decoder_create: layer %d misses a weight", li);
    }
    L.cache.nope = nope;
    L.cache.rope_dim = c.rope_dim;
    // rows [0, window): the ring; [window, window + V): a verify step's rows;
    // then a compressed layer's compressed rows
    L.ratio = w.compress_ratio;
    if (L.ratio != 0 && L.ratio != 4 && L.ratio != 128) {
      dsv4cuda_decoder_destroy(D);
      return fail("dsv4cuda_decoder_create: layer %d: compress ratio %d (0, 4 or 128)", li, L.ratio);
    }
    if (L.ratio && (!w.comp_wkv || !w.comp_wgate || !w.comp_ape || !w.comp_norm ||
                    (L.ratio == 4 && (!w.idx_wq_b || !w.idx_wq_b_s || !w.idx_weights_proj ||
                                      !w.idx_comp_wkv || !w.idx_comp_wgate || !w.idx_ape ||
                                      !w.idx_comp_norm)))) {
      dsv4cuda_decoder_destroy(D);
      return fail("dsv4cuda_decoder_create: layer %d misses a compressor / indexer weight", li);
    }
    L.coff = L.ratio == 4 ? 2 : 1;
    L.max_count = L.ratio ? c.max_context / L.ratio + 1 : 0;
    L.comp_row0 = static_cast<long long>(c.window) + DSV4CUDA_VERIFY_MAX_ROWS;
    const size_t crows = static_cast<size_t>(c.window) + DSV4CUDA_VERIFY_MAX_ROWS + L.max_count;
    L.cache.rows = static_cast<long long>(crows);
    L.cache.codes = dalloc<uint8_t>(D, crows * nope);
    L.cache.scales = dalloc<uint8_t>(D, crows * dsv4::kKvScaleSlots);
    L.cache.rope = dalloc<uint16_t>(D, crows * c.rope_dim);
    const int rows = c.o_groups * c.o_lora, cols = H * d / c.o_groups;
    if (w.wo_a) {
      L.wo_a = const_cast<uint16_t*>(w.wo_a);
    } else {
      L.wo_a = dalloc<uint16_t>(D, static_cast<size_t>(rows) * cols);
      if (L.wo_a)
        dsv4::fp8_to_bf16_kernel<<<1024, 256>>>(w.wo_a_fp8, w.wo_a_fp8_s, rows, cols, L.wo_a);
    }
    if (L.ratio) {
      const size_t cd = static_cast<size_t>(L.coff) * d, nst = static_cast<size_t>(L.coff) * L.ratio * cd;
      L.kvs = dalloc<float>(D, nst);
      L.scs = dalloc<float>(D, nst);
      L.count = dalloc<int>(D, 1);
      bool okc = L.kvs && L.scs && L.count;
      if (L.ratio == 4) {
        const size_t icd = 2 * static_cast<size_t>(c.index_dim);
        L.idx_kvs = dalloc<float>(D, 8 * icd);
        L.idx_scs = dalloc<float>(D, 8 * icd);
        L.idx_rows = dalloc<float>(D, static_cast<size_t>(L.max_count) * c.index_dim);
        L.idx_count = dalloc<int>(D, 1);
        okc = okc && L.idx_kvs && L.idx_scs && L.idx_rows && L.idx_count;
      }
      if (!okc) {
        dsv4cuda_decoder_destroy(D);
        return fail("dsv4cuda_decoder_create: out of device memory (layer %d state)", li);
      }
      D->any_comp = true;
      const int keys = L.ratio == 4 ? std::min(c.index_topk, L.max_count) : L.max_count;
      L.n_keys = (c.window + keys + 3) / 4 * 4;  // the scores kernel takes keys in fours
      D->n_max = std::max(D->n_max, L.n_keys);
      {
        const size_t H = c.hidden;
        std::vector<std::pair<const uint16_t*, int>> parts = {{w.comp_wkv, L.coff * d},
                                                              {w.comp_wgate, L.coff * d}};
        if (L.ratio == 4) {
          parts.push_back({w.idx_comp_wkv, 2 * c.index_dim});
          parts.push_back({w.idx_comp_wgate, 2 * c.index_dim});
          parts.push_back({w.idx_weights_proj, c.index_heads});
        }
        for (const auto& pr : parts) L.comp_rows += pr.second;
        L.comp_w = dalloc<uint16_t>(D, static_cast<size_t>(L.comp_rows) * H);
        size_t off = 0;
        for (const auto& pr : parts) {
          if (L.comp_w && cudaMemcpy(L.comp_w + off, pr.first, static_cast<size_t>(pr.second) * H * 2,
                                     cudaMemcpyDeviceToDevice) != cudaSuccess)
            L.comp_w = nullptr;
          off += static_cast<size_t>(pr.second) * H;
        }
        if (!L.comp_w) {
          dsv4cuda_decoder_destroy(D);
          return fail("dsv4cuda_decoder_create: out of device memory (layer %d projections)", li);
        }
        D->comp_rows_max = std::max(D->comp_rows_max, L.comp_rows);
      }
      if (L.ratio == 4) {
        int n2 = 1;
        while (n2 < L.max_count) n2 <<= 1;
        D->idx_n2 = std::max(D->idx_n2, n2);
      }
    }
    if (!L.cache.codes || !L.cache.scales || !L.cache.rope || !L.wo_a) {
      dsv4cuda_decoder_destroy(D);
      return fail("dsv4cuda_decoder_create: out of device memory (layer %d)", li);
    }
    L.mc = dsv4::MoeConfig{};
    L.mc.hidden = c.moe.hidden;
    L.mc.moe_inter = c.moe.moe_inter;
    L.mc.n_experts = c.moe.n_experts;
    L.mc.topk = c.moe.topk;
    L.mc.swiglu_limit = c.moe.swiglu_limit;
    L.mc.route_scale = c.moe.route_scale;
    L.mc.shared_kind = c.moe.shared_kind;
    L.mc.hash_vocab = w.moe.tid2eid ? c.moe.hash_vocab : 0;
    const auto& m = w.moe;
    L.mw = dsv4::MoeWeights{m.gate_w, m.bias, m.tid2eid, m.w1, m.s1, m.w3, m.s3, m.w2, m.s2,
                            m.sh1, m.sh1s, m.sh3, m.sh3s, m.sh2, m.sh2s};
    D->layers.push_back(L);
  }
  if (!verify_alloc(D)) {
    dsv4cuda_decoder_destroy(D);
    return fail("dsv4cuda_decoder_create: out of device memory (verify buffers)");
  }
  if (D->any_comp && !comp_alloc(D)) {
    dsv4cuda_decoder_destroy(D);
    return fail("dsv4cuda_decoder_create: compressed layers: %s", D->err.c_str());
  }
  // one MoE workspace serves every layer (their forwards run in stream order)
  {
    dsv4::MoeConfig mc = D->layers[0].mc;
    mc.hash_vocab = 0;
    const size_t wsb = dsv4::moe_workspace_bytes(mc, 1);
    char* base = dalloc<char>(D, wsb);
    if (!base) {
      dsv4cuda_decoder_destroy(D);
      return fail("dsv4cuda_decoder_create: out of device memory (MoE workspace)");
    }
    dsv4::moe_workspace_carve(&D->moe_ws, mc, 1, base);
    // the one token's shared-expert item, written once: the steps hand the
    // MoE layer an input that is already quantised
    dsv4::GemvItem sh{};
    sh.mat = 0;
    sh.ntok = 1;
    const int one = 1;
    cudaMemcpy(D->moe_ws.items_sh, &sh, sizeof(sh), cudaMemcpyHostToDevice);
    cudaMemcpy(D->moe_ws.counters + 3, &one, sizeof(int), cudaMemcpyHostToDevice);
  }
  const cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    dsv4cuda_decoder_destroy(D);
    return fail("dsv4cuda_decoder_create: %s", cudaGetErrorString(e));
  }
  *out = D;
  return 0;
}

DSV4_API void dsv4cuda_decoder_destroy(dsv4cuda_decoder* D) {
  if (!D) return;
  if (D->graph) cudaGraphExecDestroy(D->graph);
  if (D->graph_stream) cudaStreamDestroy(D->graph_stream);
  if (D->hc_side) cudaStreamDestroy(D->hc_side);
  if (D->hc_fork) cudaEventDestroy(D->hc_fork);
  if (D->hc_join) cudaEventDestroy(D->hc_join);
  if (D->comp_side) cudaStreamDestroy(D->comp_side);
  if (D->comp_fork) cudaEventDestroy(D->comp_fork);
  if (D->comp_join) cudaEventDestroy(D->comp_join);
  for (void* p : D->owned) cudaFree(p);
  delete D;
}

DSV4_API int dsv4cuda_decoder_set_moe_layers(dsv4cuda_decoder* D, dsv4cuda_moe_layer* const* layers,
                                             int n) {
  if (!D || n < 0 || (n > 0 && (!layers || n != static_cast<int>(D->layers.size()))))
    return fail("dsv4cuda_decoder_set_moe_layers: give one MoE layer per decoder layer, or none");
  D->ep.assign(layers, layers + n);
  for (auto* L : D->ep)
    if (!L) return fail("dsv4cuda_decoder_set_moe_layers: null layer");
  if (D->graph) {  // the captured step called the previous MoE path
    cudaGraphExecDestroy(D->graph);
    D->graph = nullptr;
  }
  return 0;
}

DSV4_API int dsv4cuda_decoder_set_ep_replicated(dsv4cuda_decoder* D, int replicated) {
  if (!D) return fail("dsv4cuda_decoder_set_ep_replicated: null decoder");
  D->ep_replicated = replicated != 0;
  if (D->graph) {  // the captured step called the other exchange
    cudaGraphExecDestroy(D->graph);
    D->graph = nullptr;
  }
  return 0;
}

DSV4_API int dsv4cuda_decoder_reset(dsv4cuda_decoder* D, void* stream) {
  if (!D) return fail("dsv4cuda_decoder_reset: null decoder");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const auto& c = D->cfg;
  for (auto& L : D->layers) {
    const size_t rows = static_cast<size_t>(L.cache.rows);
    cudaMemsetAsync(L.cache.codes, 0, rows * L.cache.nope, st);
    cudaMemsetAsync(L.cache.scales, 0, rows * dsv4::kKvScaleSlots, st);
    cudaMemsetAsync(L.cache.rope, 0, rows * c.rope_dim * 2, st);
  }
  if (D->any_comp) comp_reset(D, st);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : fail("dsv4cuda_decoder_reset: %s", cudaGetErrorString(e));
}

DSV4_API int dsv4cuda_decoder_step_device(dsv4cuda_decoder* D, const int* token, const int* position,
                                          void* stream) {
  if (!D || !token || !position) return fail("dsv4cuda_decoder_step_device: bad arguments");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyAsync(D->d_token, token, sizeof(int), cudaMemcpyDeviceToDevice, st);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(D->d_pos, position, sizeof(int), cudaMemcpyDeviceToDevice, st);
  if (e == cudaSuccess) e = step(D, st);
  return e == cudaSuccess ? 0 : fail("dsv4cuda_decoder_step_device: %s", cudaGetErrorString(e));
}

// The host-argument step: the first call runs the step's launches directly
// (every kernel's one-time set-up happens there), the second captures them
// into a CUDA graph that this and every later call replays.
DSV4_API int dsv4cuda_decoder_forward_token(dsv4cuda_decoder* D, int token, int position,
                                            float* logits, int* next_token) {
  if (!D) return fail("dsv4cuda_decoder_forward_token: null decoder");
  if (token < 0 || token >= D->cfg.vocab || position < 0 || position >= D->cfg.max_context)
    return fail("dsv4cuda_decoder_forward_token: token or position out of range");
  cudaError_t e = cudaSuccess;
  if (!D->graph_stream) e = cudaStreamCreateWithFlags(&D->graph_stream, cudaStreamNonBlocking);
  cudaStream_t st = D->graph_stream;
  if (e == cudaSuccess) e = cudaMemcpyAsync(D->d_token, &token, sizeof(int), cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(D->d_pos, &position, sizeof(int), cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess) {
    if (D->graph) {
      e = cudaGraphLaunch(D->graph, st);
    } else if (!D->stepped) {
      e = step(D, st);
      D->stepped = true;
    } else {
      cudaGraph_t g = nullptr;
      e = cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal);
      if (e == cudaSuccess) {
        const cudaError_t es = step(D, st);
        e = cudaStreamEndCapture(st, &g);
        if (e == cudaSuccess) e = es;
      }
      if (e == cudaSuccess) e = cudaGraphInstantiate(&D->graph, g, 0);
      if (g) cudaGraphDestroy(g);
      if (e == cudaSuccess) e = cudaGraphLaunch(D->graph, st);
    }
  }
  if (e == cudaSuccess && logits)
    e = cudaMemcpyAsync(logits, D->logits, sizeof(float) * D->cfg.vocab, cudaMemcpyDeviceToHost,
                        st);
  if (e == cudaSuccess && next_token)
    e = cudaMemcpyAsync(next_token, D->argmax, sizeof(int), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  return e == cudaSuccess ? 0 : fail("dsv4cuda_decoder_forward_token: %s", cudaGetErrorString(e));
}

// Kernels one step launches: a step captured into a graph (not run), its
// kernel nodes counted (the MoE layers' side-stream kernels included).
DSV4_API int dsv4cuda_decoder_step_kernels(dsv4cuda_decoder* D) {
  if (!D) return fail("dsv4cuda_decoder_step_kernels: null decoder");
  cudaStream_t st = nullptr;
  cudaError_t e = cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking);
  cudaGraph_t g = nullptr;
  if (e == cudaSuccess) e = cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal);
  if (e == cudaSuccess) {
    const cudaError_t es = step(D, st);
    e = cudaStreamEndCapture(st, &g);
    if (e == cudaSuccess) e = es;
  }
  int kernels = 0;
  size_t n = 0;
  if (e == cudaSuccess) e = cudaGraphGetNodes(g, nullptr, &n);
  if (e == cudaSuccess && n) {
    std::vector<cudaGraphNode_t> nodes(n);
    e = cudaGraphGetNodes(g, nodes.data(), &n);
    for (size_t i = 0; e == cudaSuccess && i < n; ++i) {
      cudaGraphNodeType t;
      e = cudaGraphNodeGetType(nodes[i], &t);
      if (e == cudaSuccess && t == cudaGraphNodeTypeKernel) ++kernels;
    }
  }
  if (g) cudaGraphDestroy(g);
  if (st) cudaStreamDestroy(st);
  return e == cudaSuccess ? kernels : fail("dsv4cuda_decoder_step_kernels: %s", cudaGetErrorString(e));
}

DSV4_API int dsv4cuda_decoder_read(dsv4cuda_decoder* D, float* logits, int* next_token) {
  if (!D) return fail("dsv4cuda_decoder_read: null decoder");
  cudaError_t e = cudaDeviceSynchronize();
  if (e == cudaSuccess && logits)
    e = cudaMemcpy(logits, D->logits, sizeof(float) * D->cfg.vocab, cudaMemcpyDeviceToHost);
  if (e == cudaSuccess && next_token)
    e = cudaMemcpy(next_token, D->argmax, sizeof(int), cudaMemcpyDeviceToHost);
  return e == cudaSuccess ? 0 : fail("dsv4cuda_decoder_read: %s", cudaGetErrorString(e));
}

DSV4_API int dsv4cuda_decoder_cache(dsv4cuda_decoder* D, int layer, dsv4cuda_kv_cache* out) {
  if (!D || !out || layer < 0 || layer >= static_cast<int>(D->layers.size()))
    return fail("dsv4cuda_decoder_cache: bad arguments");
  const dsv4::Fp8KvCache& c = D->layers[layer].cache;
  out->codes = c.codes;
  out->scales = c.scales;
  out->rope = c.rope;
  out->nope = c.nope;
  out->rope_dim = c.rope_dim;
  out->rows = D->cfg.window;  // the ring (a verify step's scratch rows follow it)
  return 0;
}

DSV4_API float* dsv4cuda_decoder_logits(dsv4cuda_decoder* D) { return D ? D->logits : nullptr; }
DSV4_API int* dsv4cuda_decoder_argmax(dsv4cuda_decoder* D) { return D ? D->argmax : nullptr; }
DSV4_API int* dsv4cuda_decoder_token_slot(dsv4cuda_decoder* D) { return D ? D->d_token : nullptr; }
DSV4_API int* dsv4cuda_decoder_position_slot(dsv4cuda_decoder* D) { return D ? D->d_pos : nullptr; }
DSV4_API int dsv4cuda_decoder_step(dsv4cuda_decoder* D, void* stream) {
  if (!D) return fail("dsv4cuda_decoder_step: null decoder");
  const cudaError_t e = step(D, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? 0 : fail("dsv4cuda_decoder_step: %s", cudaGetErrorString(e));
}

DSV4_API int dsv4cuda_decoder_verify_device(dsv4cuda_decoder* D, int n_rows, void* stream) {
  if (!D) return fail("dsv4cuda_decoder_verify_device: null decoder");
  if (const char* why = verify_unsupported(D, n_rows))
    return fail("dsv4cuda_decoder_verify_device: %s", why);
  const cudaError_t e = verify(D, n_rows, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? 0 : fail("dsv4cuda_decoder_verify_device: %s", cudaGetErrorString(e));
}

DSV4_API int dsv4cuda_decoder_verify(dsv4cuda_decoder* D, const int* tokens, int n_rows,
                                     int start_position, float* all_logits, int* argmax) {
  if (!D || !tokens) return fail("dsv4cuda_decoder_verify: bad arguments");
  if (const char* why = verify_unsupported(D, n_rows))
    return fail("dsv4cuda_decoder_verify: %s", why);
  if (start_position < 0 || start_position + n_rows > D->cfg.max_context)
    return fail("dsv4cuda_decoder_verify: positions out of range");
  for (int r = 0; r < n_rows; ++r)
    if (tokens[r] < 0 || tokens[r] >= D->cfg.vocab)
      return fail("dsv4cuda_decoder_verify: token out of range");
  cudaError_t e = cudaSuccess;
  if (!D->graph_stream) e = cudaStreamCreateWithFlags(&D->graph_stream, cudaStreamNonBlocking);
  cudaStream_t st = D->graph_stream;
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(D->v.tok, tokens, sizeof(int) * n_rows, cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(D->v.start, &start_position, sizeof(int), cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess) e = verify(D, n_rows, st);
  if (e == cudaSuccess && all_logits)
    e = cudaMemcpyAsync(all_logits, D->v.logits, sizeof(float) * n_rows * D->cfg.vocab,
                        cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess && argmax)
    e = cudaMemcpyAsync(argmax, D->v.argmax, sizeof(int) * n_rows, cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  return e == cudaSuccess ? 0 : fail("dsv4cuda_decoder_verify: %s", cudaGetErrorString(e));
}

DSV4_API int dsv4cuda_decoder_commit(dsv4cuda_decoder* D, int n_keep, void* stream) {
  if (!D || n_keep < 0 || n_keep > DSV4CUDA_VERIFY_MAX_ROWS)
    return fail("dsv4cuda_decoder_commit: bad arguments");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyAsync(D->v.count, &n_keep, sizeof(int), cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess) e = verify_commit(D, D->v.start, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  return e == cudaSuccess ? 0 : fail("dsv4cuda_decoder_commit: %s", cudaGetErrorString(e));
}

DSV4_API int dsv4cuda_decoder_accept_greedy(dsv4cuda_decoder* D, int n_rows, void* stream) {
  if (!D || n_rows < 1 || n_rows > DSV4CUDA_VERIFY_MAX_ROWS)
    return fail("dsv4cuda_decoder_accept_greedy: bad arguments");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto& v = D->v;
  cudaError_t e = dsv4::launch_pdl(dsv4::verify_accept_kernel, dim3(1), dim3(32), 0, st, v.tok,
                                   static_cast<const int*>(v.argmax), n_rows, v.start, v.from,
                                   v.count, v.stats);
  if (e == cudaSuccess) e = verify_commit(D, v.from, st);
  return e == cudaSuccess ? 0 : fail("dsv4cuda_decoder_accept_greedy: %s", cudaGetErrorString(e));
}

DSV4_API int dsv4cuda_decoder_draft_random(dsv4cuda_decoder* D, int n_rows, void* stream) {
  if (!D || n_rows < 1 || n_rows > DSV4CUDA_VERIFY_MAX_ROWS)
    return fail("dsv4cuda_decoder_draft_random: bad arguments");
  const cudaError_t e = dsv4::launch_pdl(dsv4::draft_random_kernel, dim3(1), dim3(32), 0,
                                         static_cast<cudaStream_t>(stream), D->v.rng, D->v.tok,
                                         n_rows, D->cfg.vocab);
  return e == cudaSuccess ? 0 : fail("dsv4cuda_decoder_draft_random: %s", cudaGetErrorString(e));
}

DSV4_API int dsv4cuda_decoder_verify_stats(dsv4cuda_decoder* D, long long* stats3) {
  if (!D || !stats3) return fail("dsv4cuda_decoder_verify_stats: bad arguments");
  cudaError_t e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMemcpy(stats3, D->v.stats, 3 * sizeof(long long), cudaMemcpyDeviceToHost);
  return e == cudaSuccess ? 0 : fail("dsv4cuda_decoder_verify_stats: %s", cudaGetErrorString(e));
}

DSV4_API int dsv4cuda_decoder_verify_pending(dsv4cuda_decoder* D, int* token, int* position) {
  if (!D || !token || !position) return fail("dsv4cuda_decoder_verify_pending: bad arguments");
  cudaError_t e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMemcpy(token, D->v.tok, sizeof(int), cudaMemcpyDeviceToHost);
  if (e == cudaSuccess) e = cudaMemcpy(position, D->v.start, sizeof(int), cudaMemcpyDeviceToHost);
  return e == cudaSuccess ? 0 : fail("dsv4cuda_decoder_verify_pending: %s", cudaGetErrorString(e));
}

DSV4_API int* dsv4cuda_decoder_verify_tokens(dsv4cuda_decoder* D) { return D ? D->v.tok : nullptr; }
DSV4_API int* dsv4cuda_decoder_verify_start(dsv4cuda_decoder* D) { return D ? D->v.start : nullptr; }
DSV4_API float* dsv4cuda_decoder_verify_logits(dsv4cuda_decoder* D) { return D ? D->v.logits : nullptr; }
DSV4_API int* dsv4cuda_decoder_verify_argmax(dsv4cuda_decoder* D) { return D ? D->v.argmax : nullptr; }
