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

// ------------------------------------------------------------ kernels ----

// embed_token (src/dsv4/dsv4_model.c:7478): every HC copy gets the BF16 row.
__global__ void embed_kernel(const uint16_t* embed, const int* token, int vocab, int hid, int mult,
                             float* state) {
  pdl_wait();
  pdl_trigger();
  int t = *token;
  if (t < 0 || t >= vocab) t = 0;
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
                                long long* row, float* cosv, float* sinv) {
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
  }
  if (threadIdx.x == 0) *row = pos % win;
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

// rmsnorm_bf16 with a gain (src/dsv4/dsv4_model.c:4934), optionally followed
// by dsv4_rope_apply_buf on the last 2 * half dims (:1547-1558). One CTA.
__global__ void __launch_bounds__(256) rmsnorm_rope_kernel(const float* x, int n, const uint16_t* w,
                                                           float eps, int half, const float* cosv,
                                                           const float* sinv, float* y) {
  __shared__ double red[8];
  pdl_wait();
  pdl_trigger();
  double ss = 0.0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) ss += static_cast<double>(x[i]) * x[i];
  ss = block_sum_d(ss, red);
  const float r = rms_factor(ss, n, eps);
  for (int i = threadIdx.x; i < n; i += blockDim.x)
    y[i] = bf16_round(__fmul_rn(__fmul_rn(x[i], r), bf16_widen(w[i])));
  if (half <= 0) return;
  __syncthreads();
  const int start = n - 2 * half;
  for (int i = threadIdx.x; i < half; i += blockDim.x) {
    const float x0 = y[start + 2 * i], x1 = y[start + 2 * i + 1];
    const float c = cosv[i], s = sinv[i];
    y[start + 2 * i] = bf16_round(__fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s)));
    y[start + 2 * i + 1] = bf16_round(__fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c)));
  }
}

// Per-head RMS of q and its RoPE (src/dsv4/dsv4_model.c:5283-5291), one CTA
// per head; q is updated in place.
__global__ void __launch_bounds__(128) q_head_kernel(float* q, int d, float eps, int half,
                                                     const float* cosv, const float* sinv) {
  __shared__ double red[4];
  pdl_wait();
  pdl_trigger();
  float* qh = q + static_cast<size_t>(blockIdx.x) * d;
  double ss = 0.0;
  for (int i = threadIdx.x; i < d; i += blockDim.x) ss += static_cast<double>(qh[i]) * qh[i];
  ss = block_sum_d(ss, red);
  const float rr = rms_factor(ss, d, eps);
  for (int i = threadIdx.x; i < d; i += blockDim.x) qh[i] = bf16_round(__fmul_rn(qh[i], rr));
  __syncthreads();
  const int start = d - 2 * half;
  for (int i = threadIdx.x; i < half; i += blockDim.x) {
    const float x0 = qh[start + 2 * i], x1 = qh[start + 2 * i + 1];
    const float c = cosv[i], s = sinv[i];
    qh[start + 2 * i] = bf16_round(__fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s)));
    qh[start + 2 * i + 1] = bf16_round(__fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c)));
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
#pragma unroll 8
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

// Greedy token: argmax_logits (src/cli/dsv4_run.c:355; first maximum, strict
// >) in two stages - each CTA finds its chunk's first maximum, then one warp
// takes the chunks' results in chunk order with the same strict >. For
// finite logits this is the sequential scan's answer.
constexpr int kArgmaxCtas = 148;
__global__ void __launch_bounds__(256) argmax_chunks_kernel(const float* x, int n, float* cv,
                                                            int* ci) {
  __shared__ float sv[8];
  __shared__ int si[8];
  pdl_wait();
  pdl_trigger();
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

__global__ void argmax_final_kernel(const float* cv, const int* ci, int chunks, int* out) {
  pdl_wait();
  pdl_trigger();
  if (threadIdx.x != 0) return;
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

// ------------------------------------------------------- host side ----

struct Layer {
  dsv4cuda_layer_weights w;
  MoeConfig mc;
  MoeWeights mw;
  Fp8KvCache cache;
  uint16_t* wo_a = nullptr;  // BF16, decoded at create when given as FP8
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
  std::vector<void*> owned;  // device allocations to free
  // per-step buffers
  int* d_token = nullptr;
  int* d_pos = nullptr;
  float* state = nullptr;     // [mult][hid]
  double* part = nullptr;     // [nblk][kMixMax + 1]
  int nblk = 0;
  float *post = nullptr, *comb = nullptr;
  float* x = nullptr;         // [hid] normed branch input
  __half* xq = nullptr;       // [ld] FP8-grid activations (f16)
  float* xs = nullptr;        // [ld / 128] scales
  float* qr = nullptr;        // [q_lora]
  float* qn = nullptr;        // [q_lora]
  float* q = nullptr;         // [H][d]
  float* kv = nullptr;        // [d]
  float* kvn = nullptr;       // [d]
  float* o = nullptr;         // [H][d]
  float* kvdec = nullptr;     // [window][d] the window's cached values
  float* kvt = nullptr;       // [d][window] transposed
  float* fp8_part = nullptr;  // split-K FP8 GEMV partials [in / 128][rows]
  size_t win_smem = 0;        // dynamic shared memory of win_scores_kernel
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

cudaError_t fp8_gemv(const uint8_t* W, const uint8_t* S, int in, int rows, const __half* x,
                     const float* xs, int ld, float* y, const dsv4::GemvItem* item, const int* n_one,
                     float* part, cudaStream_t st) {
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
  const cudaError_t e = dsv4::launch_fp8_gemv_splitk(a, part, st);
  return e == cudaErrorNotSupported ? dsv4::launch_fp8_gemv(a, false, 1, st) : e;
}

cudaError_t quant(dsv4cuda_decoder* D, const float* x, int n, cudaStream_t st) {
  return dsv4::launch_quant_fp8(x, n, n, 1, D->xq, D->xs, D->ld, st);
}

#define DEC_CHECK(expr)                             \
  do {                                              \
    cudaError_t e__ = (expr);                       \
    if (e__ != cudaSuccess) return e__;             \
  } while (0)


cudaError_t hc_pre(dsv4cuda_decoder* D, const float* fn, const float* scale, const float* base,
                   const uint16_t* norm, int head, cudaStream_t st) {
  const auto& c = D->cfg;
  const int n = c.hc_mult * c.hidden;
  const int rows = head ? c.hc_mult : (2 + c.hc_mult) * c.hc_mult;
  if (c.hc_exact)
    DEC_CHECK(dsv4::launch_pdl(dsv4::hc_mix_exact_kernel, dim3(1), dim3(32), 0, st, fn, rows,
                               static_cast<const float*>(D->state), n, D->part));
  else
    DEC_CHECK(dsv4::launch_pdl(dsv4::hc_mix_partial_kernel, dim3(D->nblk), dim3(dsv4::kMixThreads),
                               0, st, fn, rows, static_cast<const float*>(D->state), n, D->part));
  dsv4::HcReduceArgs a{};
  a.part = D->part;
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
  a.state = D->state;
  a.norm = norm;
  a.post = D->post;
  a.comb = D->comb;
  a.out = D->x;
  return dsv4::launch_pdl(dsv4::hc_reduce_kernel, dim3(1), dim3(dsv4::kHcThreads), 0, st, a);
}

cudaError_t hc_post(dsv4cuda_decoder* D, cudaStream_t st) {
  const int hid = D->cfg.hidden;
  return dsv4::launch_pdl(dsv4::hc_post_kernel, dim3((hid + 255) / 256), dim3(256), 0, st,
                          D->state, static_cast<const float*>(D->branch),
                          static_cast<const float*>(D->post), static_cast<const float*>(D->comb),
                          D->cfg.hc_mult, hid);
}

// attention_forward_impl for a compress-ratio-0 layer (src/dsv4/dsv4_model.c:
// 5241-5429): writes the branch output [hid] into D->branch.
cudaError_t attention(dsv4cuda_decoder* D, dsv4::Layer& L, cudaStream_t st) {
  const auto& c = D->cfg;
  const auto& w = L.w;
  const int H = c.n_heads, d = c.head_dim, ql = c.q_lora, half = c.rope_dim / 2;
  const int G = c.o_groups, ol = c.o_lora, hid = c.hidden;
  // q: quant(x) -> wq_a -> q_norm -> quant -> wq_b -> per-head RMS + RoPE
  DEC_CHECK(quant(D, D->x, hid, st));
  DEC_CHECK(fp8_gemv(w.wq_a, w.wq_a_s, hid, ql, D->xq, D->xs, D->ld, D->qr, D->item1, D->n_one, D->fp8_part, st));
  DEC_CHECK(dsv4::launch_pdl(dsv4::rmsnorm_rope_kernel, dim3(1), dim3(256), 0, st,
                             static_cast<const float*>(D->qr), ql, w.q_norm, c.rms_eps, 0,
                             static_cast<const float*>(nullptr), static_cast<const float*>(nullptr),
                             D->qn));
  // wkv reads quant(x) too: run it before the activation buffer is reused
  DEC_CHECK(fp8_gemv(w.wkv, w.wkv_s, hid, d, D->xq, D->xs, D->ld, D->kv, D->item1, D->n_one, D->fp8_part, st));
  DEC_CHECK(quant(D, D->qn, ql, st));
  DEC_CHECK(fp8_gemv(w.wq_b, w.wq_b_s, ql, H * d, D->xq, D->xs, D->ld, D->q, D->item1, D->n_one, D->fp8_part, st));
  DEC_CHECK(dsv4::launch_pdl(dsv4::q_head_kernel, dim3(H), dim3(128), 0, st, D->q, d, c.rms_eps,
                             half, static_cast<const float*>(D->cosv),
                             static_cast<const float*>(D->sinv)));
  // kv: kv_norm -> RoPE -> FP8 latent into the ring row of the position
  DEC_CHECK(dsv4::launch_pdl(dsv4::rmsnorm_rope_kernel, dim3(1), dim3(256), 0, st,
                             static_cast<const float*>(D->kv), d, w.kv_norm, c.rms_eps, half,
                             static_cast<const float*>(D->cosv), static_cast<const float*>(D->sinv),
                             D->kvn));
  DEC_CHECK(dsv4::kv_cache_write(L.cache, D->kvn, D->row, 1, st));
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
  DEC_CHECK(dsv4::launch_pdl(dsv4::win_decode_kernel, dim3(c.window), dim3(128), 0, st, wa));
  DEC_CHECK(dsv4::launch_pdl(
      dsv4::win_scores_kernel,
      dim3((H + dsv4::kWinHeads - 1) / dsv4::kWinHeads, (c.window + dsv4::kWinKeys - 1) / dsv4::kWinKeys),
      dim3(dsv4::kWinHeads * 32), D->win_smem, st, wa));
  DEC_CHECK(dsv4::launch_pdl(dsv4::win_softmax_kernel, dim3(H), dim3(256),
                             sizeof(float) * c.window, st, wa));
  DEC_CHECK(dsv4::launch_pdl(dsv4::win_values_kernel, dim3(H, (d / 2 + 63) / 64), dim3(64),
                             sizeof(float) * c.window, st, wa));
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
  DEC_CHECK(dsv4::launch_bf16_gemv(ga, 1, st));
  DEC_CHECK(quant(D, D->oall, G * ol, st));
  return fp8_gemv(w.wo_b, w.wo_b_s, G * ol, hid, D->xq, D->xs, D->ld, D->branch, D->item1,
                  D->n_one, D->fp8_part, st);
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
                             D->sinv));
  dsv4::MoeExecOptions opt;
  for (size_t li = 0; li < D->layers.size(); ++li) {
    auto& L = D->layers[li];
    const auto& w = L.w;
    DEC_CHECK(hc_pre(D, w.hc_attn_fn, w.hc_attn_scale, w.hc_attn_base, w.attn_norm, 0, st));
    DEC_CHECK(attention(D, L, st));
    DEC_CHECK(hc_post(D, st));
    DEC_CHECK(hc_pre(D, w.hc_ffn_fn, w.hc_ffn_scale, w.hc_ffn_base, w.ffn_norm, 0, st));
    if (!D->ep.empty()) {
      if (dsv4cuda_moe_forward_ep_tokens(D->ep[li], D->x, 1, D->branch, st) != 0)
        return cudaErrorLaunchFailure;
    } else {
      DEC_CHECK(dsv4::moe_forward(L.mc, L.mw, D->moe_ws, D->x, D->d_token, 1, D->branch, st, opt));
    }
    DEC_CHECK(hc_post(D, st));
  }
  // model_head + head_logits (src/dsv4/dsv4_model.c:7755-7760), argmax
  DEC_CHECK(hc_pre(D, D->g.hc_head_fn, D->g.hc_head_scale, D->g.hc_head_base, D->g.norm, 1, st));
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
  DEC_CHECK(dsv4::launch_bf16_gemv(ha, 1, st));
  const int chunks = std::min(dsv4::kArgmaxCtas, c.vocab);
  DEC_CHECK(dsv4::launch_pdl(dsv4::argmax_chunks_kernel, dim3(chunks), dim3(256), 0, st,
                             static_cast<const float*>(D->logits), c.vocab, D->am_v, D->am_i));
  return dsv4::launch_pdl(dsv4::argmax_final_kernel, dim3(1), dim3(32), 0, st,
                          static_cast<const float*>(D->am_v), static_cast<const int*>(D->am_i),
                          chunks, D->argmax);
}

bool cfg_ok(const dsv4cuda_decoder_config* c) {
  return c && c->hidden > 0 && c->hidden % 128 == 0 && c->n_layers > 0 && c->vocab > 0 &&
         c->n_heads > 0 && c->head_dim > 0 && c->head_dim % 4 == 0 && c->rope_dim > 0 && c->rope_dim % 2 == 0 &&
         c->rope_dim <= c->head_dim && (c->head_dim - c->rope_dim) % 64 == 0 &&
         (c->head_dim - c->rope_dim) / 64 <= dsv4::kKvScaleSlots && c->q_lora > 0 &&
         c->o_groups > 0 && (c->n_heads * c->head_dim) % c->o_groups == 0 && c->o_lora > 0 &&
         c->window > 0 && c->window % 4 == 0 && c->hc_mult > 0 && c->hc_mult <= 4 &&
         c->hc_iters > 0 &&
         c->hidden <= 8 * dsv4::kHcThreads &&
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
  chk(D->part = dalloc<double>(D, static_cast<size_t>(D->nblk) * (dsv4::kMixMax + 1)));
  chk(D->post = dalloc<float>(D, dsv4::kHcMultMax));
  chk(D->comb = dalloc<float>(D, dsv4::kHcMultMax * dsv4::kHcMultMax));
  chk(D->x = dalloc<float>(D, c.hidden));
  chk(D->xq = dalloc<__half>(D, D->ld));
  chk(D->xs = dalloc<float>(D, D->ld / 128));
  chk(D->qr = dalloc<float>(D, c.q_lora));
  chk(D->qn = dalloc<float>(D, c.q_lora));
  chk(D->q = dalloc<float>(D, static_cast<size_t>(H) * d));
  chk(D->kv = dalloc<float>(D, d));
  chk(D->kvn = dalloc<float>(D, d));
  chk(D->o = dalloc<float>(D, static_cast<size_t>(H) * d));
  chk(D->oall = dalloc<float>(D, static_cast<size_t>(c.o_groups) * c.o_lora));
  chk(D->kvdec = dalloc<float>(D, static_cast<size_t>(c.window) * d));
  chk(D->kvt = dalloc<float>(D, static_cast<size_t>(c.window) * d));
  {
    const size_t hid = c.hidden, ql = c.q_lora, hd = static_cast<size_t>(H) * d;
    const size_t go = static_cast<size_t>(c.o_groups) * c.o_lora;
    const size_t np = std::max(std::max((hid + 127) / 128 * ql, (ql + 127) / 128 * hd),
                               std::max((hid + 127) / 128 * d, (go + 127) / 128 * hid));
    chk(D->fp8_part = dalloc<float>(D, np));
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
    L.cache.rows = c.window;
    L.cache.codes = dalloc<uint8_t>(D, static_cast<size_t>(c.window) * nope);
    L.cache.scales = dalloc<uint8_t>(D, static_cast<size_t>(c.window) * dsv4::kKvScaleSlots);
    L.cache.rope = dalloc<uint16_t>(D, static_cast<size_t>(c.window) * c.rope_dim);
    const int rows = c.o_groups * c.o_lora, cols = H * d / c.o_groups;
    if (w.wo_a) {
      L.wo_a = const_cast<uint16_t*>(w.wo_a);
    } else {
      L.wo_a = dalloc<uint16_t>(D, static_cast<size_t>(rows) * cols);
      if (L.wo_a)
        dsv4::fp8_to_bf16_kernel<<<1024, 256>>>(w.wo_a_fp8, w.wo_a_fp8_s, rows, cols, L.wo_a);
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

DSV4_API int dsv4cuda_decoder_reset(dsv4cuda_decoder* D, void* stream) {
  if (!D) return fail("dsv4cuda_decoder_reset: null decoder");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const auto& c = D->cfg;
  for (auto& L : D->layers) {
    cudaMemsetAsync(L.cache.codes, 0, static_cast<size_t>(c.window) * L.cache.nope, st);
    cudaMemsetAsync(L.cache.scales, 0, static_cast<size_t>(c.window) * dsv4::kKvScaleSlots, st);
    cudaMemsetAsync(L.cache.rope, 0, static_cast<size_t>(c.window) * c.rope_dim * 2, st);
  }
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
  out->rows = c.rows;
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
