// moe.cu - device-resident MoE layer: router with exact expert selection,
// token->expert permutation, grouped FP4 expert GEMVs, shared expert and the
// ascending-id ordered combine.
//
// Router (src/dsv4/dsv4_model.c:6615-6676). The reference's logit z is one
// sequential fp32 fmaf chain over the hidden dimension; replaying that chain
// costs hidden x 4 cycles of latency (~15 us at 7168), so the router instead
//   1. computes the exact dot product in fp64 (bf16 x fp32 products are exact
//      in fp64) together with a rigorous bound on how far the reference's
//      fp32 chain can drift from it: |z_ref - z| <= u * sum_i |s_i| (u=2^-24,
//      s_i the prefix sums; a warp scan supplies them);
//   2. selects the top-k with the reference's rule (score + bias, strict >,
//      lower id wins ties) and checks that every selected expert's lower
//      bound clears every unselected expert's upper bound;
//   3. when the check fails (a near tie), replays the reference's fp32 chain
//      exactly for the experts inside the ambiguous band and selects again.
// The selected SET therefore equals the reference's; combine weights come
// from sqrt(softplus) of the rounded logit and agree to ~1e-6 relative
// (transcendentals differ from glibc in the last ulp).
#include <algorithm>
#include <mutex>

#include "dsv4_common.cuh"
#include "moe.cuh"

namespace dsv4 {

namespace {

constexpr double kU = 5.9604644775390625e-08;  // 2^-24, fp32 unit roundoff
constexpr int kSelThreads = 256;

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// sqrt(softplus(z)) in the reference's fp32 operation order
// (src/dsv4/dsv4_model.c:5827).
__device__ __forceinline__ float sqrt_softplus_f(float z) {
  if (z > 20.0f) return sqrtf(z);
  return sqrtf(log1pf(expf(z)));
}
__device__ __forceinline__ double sqrt_softplus_d(double z) {
  if (z > 20.0) return sqrt(z);
  return sqrt(log1p(exp(z)));
}

// One warp per (token, expert): exact fp64 logit and the reference-error bound.
__global__ void router_logits_kernel(const float* __restrict__ x, int H,
                                     const uint16_t* __restrict__ gate, int E,
                                     double* __restrict__ zd, double* __restrict__ zb,
                                     int public_router) {
  const int lane = threadIdx.x & 31;
  const int e = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int t = blockIdx.y;
  if (e >= E) return;
  const float* xr = x + static_cast<size_t>(t) * H;
  const uint16_t* g = gate + static_cast<size_t>(e) * H;
  const int seg = (H + 31) / 32;
  const int c0 = min(lane * seg, H), c1 = min(c0 + seg, H);
  double local = 0.0;
  for (int c = c0; c < c1; ++c)
    local += static_cast<double>(bf16_widen(g[c])) * static_cast<double>(xr[c]);
  double incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  double run = __shfl_up_sync(0xffffffffu, incl, 1);
  if (lane == 0) run = 0.0;
  double sabs = 0.0, pabs = 0.0;
  for (int c = c0; c < c1; ++c) {
    const double p = static_cast<double>(bf16_widen(g[c])) * static_cast<double>(xr[c]);
    run += p;
    sabs += fabs(run);
    pabs += fabs(p);
  }
  const double total = __shfl_sync(0xffffffffu, incl, 31);
  sabs = warp_sum_d(sabs);
  pabs = warp_sum_d(pabs);
  if (lane == 0) {
    const size_t o = static_cast<size_t>(t) * E + e;
    zd[o] = total;
    // fused chain: each step rounds its result (<= u|s_i|); the public
    // router also rounds every product (<= u|p_i|). fp64 summation error and
    // subnormal steps are covered by the last two terms.
    const double b = kU * (sabs + (public_router ? pabs : 0.0));
    zb[o] = b * 1.01 + 1e-12 * pabs + 1e-40 * H;
  }
}

struct SelectArgs {
  const float* x;
  int H, E, topk;
  const uint16_t* gate;
  const float* bias;
  const int64_t* tid2eid;
  int hash_vocab;
  const int* token_ids;
  const double* zd;
  const double* zb;
  float route_scale;
  int public_router;
  int* idx;
  float* wt;
  int* counters;
};

struct Cand {
  float v;
  int id;
};
__device__ __forceinline__ bool better(const Cand& a, const Cand& b) {
  // strict ">" scan from -inf over ascending ids: larger value first, lower
  // id on equal values; -inf and NaN never win (src/dsv4/dsv4_model.c:6636).
  if (a.id < 0) return false;
  if (b.id < 0) return true;
  if (a.v > b.v) return true;
  if (a.v < b.v) return false;
  return a.id < b.id;
}

__device__ Cand block_best(Cand c, Cand* red) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    Cand n;
    n.v = __shfl_xor_sync(0xffffffffu, c.v, o);
    n.id = __shfl_xor_sync(0xffffffffu, c.id, o);
    if (better(n, c)) c = n;
  }
  if (lane == 0) red[w] = c;
  __syncthreads();
  Cand r = red[0];
  for (int i = 1; i < static_cast<int>(blockDim.x >> 5); ++i)
    if (better(red[i], r)) r = red[i];
  __syncthreads();
  return r;
}

// Top-k by the reference rule over `val`; writes order[0..k).
__device__ void select_topk(const float* val, int E, int k, unsigned char* used, int* order,
                            Cand* red) {
  for (int j = 0; j < k; ++j) {
    Cand c{0.f, -1};
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
      const float v = val[e];
      if (used[e] || !(v > -INFINITY)) continue;  // excludes -inf and NaN
      const Cand n{v, e};
      if (better(n, c)) c = n;
    }
    const Cand b = block_best(c, red);
    if (threadIdx.x == 0) {
      order[j] = b.id;
      if (b.id >= 0) used[b.id] = 1;
    }
    __syncthreads();
  }
}

// One CTA per token: scores, selection (with exact fallback), weights, sort.
__global__ void __launch_bounds__(kSelThreads) router_select_kernel(const SelectArgs a) {
  extern __shared__ unsigned char smem[];
  const int E = a.E;
  float* choice = reinterpret_cast<float*>(smem);
  float* score = choice + E;
  double* lo = reinterpret_cast<double*>(score + E + (E & 1));
  double* hi = lo + E;
  unsigned char* used = reinterpret_cast<unsigned char*>(hi + E);
  __shared__ Cand red[kSelThreads / 32];
  __shared__ int order[kMaxTopk];
  __shared__ float band[2];
  __shared__ int n_cand;
  const int t = blockIdx.x;
  const int tok = a.token_ids ? a.token_ids[t] : 0;
  const bool hash = a.tid2eid != nullptr;

  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    const size_t o = static_cast<size_t>(t) * E + e;
    const double z = a.zd[o];
    const float b = a.bias ? a.bias[e] : 0.0f;
    const float s = sqrt_softplus_f(static_cast<float>(z));
    score[e] = s;
    choice[e] = s + b;
    const double sm = sqrt_softplus_d(z);
    const double rad = 0.5 * a.zb[o] + 1e-6 * (fabs(sm) + fabs(static_cast<double>(b))) + 1e-37;
    lo[e] = sm + b - rad;
    hi[e] = sm + b + rad;
    used[e] = 0;
  }
  if (threadIdx.x == 0) n_cand = 0;
  __syncthreads();

  if (hash) {
    if (threadIdx.x == 0) {
      const int tk = (tok >= 0 && tok < a.hash_vocab) ? tok : 0;
      for (int k = 0; k < a.topk; ++k) {
        const int64_t e = a.tid2eid[static_cast<size_t>(tk) * a.topk + k];
        order[k] = (e >= 0 && e < E) ? static_cast<int>(e) : -1;
      }
    }
    __syncthreads();
  } else {
    select_topk(choice, E, a.topk, used, order, red);
    // margin check: min lower bound of the selected vs max upper bound of the rest
    double mlo = INFINITY, mhi = -INFINITY;
    bool nan_seen = false;
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
      if (isnan(lo[e]) || isnan(hi[e])) nan_seen = true;
      if (used[e]) mlo = fmin(mlo, lo[e]);
      else mhi = fmax(mhi, hi[e]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      mlo = fmin(mlo, __shfl_xor_sync(0xffffffffu, mlo, o));
      mhi = fmax(mhi, __shfl_xor_sync(0xffffffffu, mhi, o));
    }
    const int any_nan = __syncthreads_or(nan_seen ? 1 : 0);
    __shared__ double wlo[kSelThreads / 32], whi[kSelThreads / 32];
    if ((threadIdx.x & 31) == 0) { wlo[threadIdx.x >> 5] = mlo; whi[threadIdx.x >> 5] = mhi; }
    __syncthreads();
    if (threadIdx.x == 0) {
      double l = wlo[0], h = whi[0];
      for (int i = 1; i < kSelThreads / 32; ++i) { l = fmin(l, wlo[i]); h = fmax(h, whi[i]); }
      band[0] = static_cast<float>(l);
      band[1] = static_cast<float>(h);
      // the band is used only to pick candidates; keep it in double precision
      wlo[0] = l;
      whi[0] = h;
    }
    __syncthreads();
    const double blo = wlo[0], bhi = whi[0];
    const bool safe = !any_nan && (blo > bhi);
    if (!safe) {
      // replay the reference's fp32 logit chain for every expert in the band
      const float* xr = a.x + static_cast<size_t>(t) * a.H;
      for (int e = threadIdx.x; e < E; e += blockDim.x) {
        const bool cand = any_nan || (hi[e] >= blo && lo[e] <= bhi);
        if (!cand) continue;
        atomicAdd(&n_cand, 1);
        const uint16_t* g = a.gate + static_cast<size_t>(e) * a.H;
        float z = 0.0f;
        if (a.public_router) {
          for (int c = 0; c < a.H; ++c) {
            const float p = __fmul_rn(bf16_widen(g[c]), xr[c]);
            z = __fadd_rn(z, p);
          }
        } else {
          for (int c = 0; c < a.H; ++c) z = fmaf(bf16_widen(g[c]), xr[c], z);
        }
        const float s = sqrt_softplus_f(z);
        score[e] = s;
        choice[e] = s + (a.bias ? a.bias[e] : 0.0f);
      }
      for (int e = threadIdx.x; e < E; e += blockDim.x) used[e] = 0;
      __syncthreads();
      select_topk(choice, E, a.topk, used, order, red);
      if (threadIdx.x == 0) atomicAdd(&a.counters[2], 1);
    }
  }

  if (threadIdx.x == 0) {
    const int K = a.topk;
    int id[kMaxTopk];
    float w[kMaxTopk];
    float sum = 0.0f;
    for (int k = 0; k < K; ++k) {
      id[k] = order[k];
      sum += id[k] >= 0 ? score[id[k]] : 0.0f;
    }
    if (a.public_router) {
      // dsv4_router (src/dsv4/dsv4_ops.c:528-531)
      const float inv = sum > 0.0f ? 1.0f / sum : 0.0f;
      for (int k = 0; k < K; ++k) w[k] = (id[k] >= 0 ? score[id[k]] : 0.f) * inv * a.route_scale;
    } else if (sum > 0.0f) {
      // moe_forward (src/dsv4/dsv4_model.c:6651-6658)
      const float rs = a.route_scale / sum;
      for (int k = 0; k < K; ++k) w[k] = (id[k] >= 0 ? score[id[k]] : 0.f) * rs;
    } else {
      for (int k = 0; k < K; ++k) w[k] = 0.0f;
    }
    // the reference's exchange sort by ascending id, carrying weights (:6669)
    for (int i = 0; i < K; ++i)
      for (int j = i + 1; j < K; ++j)
        if (id[j] < id[i]) {
          const int ti = id[i]; id[i] = id[j]; id[j] = ti;
          const float tw = w[i]; w[i] = w[j]; w[j] = tw;
        }
    for (int k = 0; k < K; ++k) {
      a.idx[static_cast<size_t>(t) * K + k] = id[k];
      a.wt[static_cast<size_t>(t) * K + k] = w[k];
    }
  }
}

// Per-forward setup that depends on the token count: shared-expert items.
__global__ void moe_prep_kernel(GemvItem* items_sh, int n_tokens, int* counters) {
  const int j = threadIdx.x + blockIdx.x * blockDim.x;
  const int n_items = (n_tokens + kItemTok - 1) / kItemTok;
  if (j == 0) counters[3] = n_items;
  if (j < n_items) {
    GemvItem it;
    it.mat = 0;
    it.ntok = min(kItemTok, n_tokens - j * kItemTok);
    for (int i = 0; i < kItemTok; ++i) {
      const int t = min(j * kItemTok + i, n_tokens - 1);
      it.tok[i].x = t;
      it.tok[i].y = t;
    }
    items_sh[j] = it;
  }
}

// Token->expert permutation (moe_forward_batch grouping,
// src/dsv4/dsv4_model.c:6925-6926 and expert_forward_batch_routes :6486):
// unique experts ascending; each expert's routes in token order, packed into
// items of <= kItemTok routes. Route (t,k) owns slot t*topk+k.
__global__ void moe_plan_kernel(const int* idx, int n_tokens, int topk, int E,
                                GemvItem* items_gu, GemvItem* items_dn, int* counters) {
  extern __shared__ int cnt[];  // [E] item count per expert, then exclusive offsets
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int n = 0;
    for (int r = 0; r < n_tokens * topk; ++r) n += (idx[r] == e);
    cnt[e] = (n + kItemTok - 1) / kItemTok;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int run = 0;
    for (int e = 0; e < E; ++e) {
      const int c = cnt[e];
      cnt[e] = run;
      run += c;
    }
    counters[0] = run;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int item = cnt[e];
    GemvItem gu, dn;
    gu.mat = dn.mat = e;
    gu.ntok = dn.ntok = 0;
    for (int t = 0; t < n_tokens; ++t) {
      for (int k = 0; k < topk; ++k) {
        const int slot = t * topk + k;
        if (idx[slot] != e) continue;
        gu.tok[gu.ntok].x = t;
        gu.tok[gu.ntok].y = slot;
        dn.tok[dn.ntok].x = slot;
        dn.tok[dn.ntok].y = slot;
        gu.ntok++;
        dn.ntok++;
        if (gu.ntok == kItemTok) {
          items_gu[item] = gu;
          items_dn[item] = dn;
          ++item;
          gu.ntok = dn.ntok = 0;
        }
      }
    }
    if (gu.ntok > 0) {
      for (int i = gu.ntok; i < kItemTok; ++i) { gu.tok[i] = gu.tok[0]; dn.tok[i] = dn.tok[0]; }
      items_gu[item] = gu;
      items_dn[item] = dn;
    }
  }
}

// out[t] = bf16( sum_k routed[t*topk+k] (ascending id order) + shared[t] )
// (src/dsv4/dsv4_model.c:6795-6805, :7096-7112).
__global__ void moe_combine_kernel(const float* __restrict__ routed, const float* __restrict__ shared,
                                   const int* __restrict__ idx, int n_tokens, int topk, int H,
                                   float* __restrict__ out) {
  const size_t n = static_cast<size_t>(n_tokens) * H;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int t = static_cast<int>(i / H);
    const int c = static_cast<int>(i % H);
    float acc = 0.0f;
    for (int k = 0; k < topk; ++k) {
      const int slot = t * topk + k;
      if (idx[slot] >= 0) acc += routed[static_cast<size_t>(slot) * H + c];
    }
    if (shared) acc += shared[i];
    out[i] = bf16_round(acc);
  }
}

size_t align256(size_t b) { return (b + 255) & ~static_cast<size_t>(255); }

struct SideStream {
  cudaStream_t s = nullptr;
  cudaEvent_t fork = nullptr, join = nullptr;
};

SideStream& side_stream() {
  static thread_local SideStream ss;
  if (!ss.s) {
    cudaStreamCreateWithFlags(&ss.s, cudaStreamNonBlocking);
    cudaEventCreateWithFlags(&ss.fork, cudaEventDisableTiming);
    cudaEventCreateWithFlags(&ss.join, cudaEventDisableTiming);
  }
  return ss;
}

int nt_bucket(int n) { return n <= 1 ? 1 : n <= 2 ? 2 : n <= 4 ? 4 : 8; }

}  // namespace

size_t moe_workspace_bytes(const MoeConfig& c, int M) {
  const size_t H = c.hidden, I = c.moe_inter, E = c.n_experts, K = c.topk;
  const size_t R = static_cast<size_t>(M) * K;
  size_t b = 0;
  b += align256(M * H * sizeof(__half));
  b += align256(M * (H / 128 + 1) * sizeof(float));
  b += 2 * align256(M * E * sizeof(double));
  b += align256(R * sizeof(int)) + align256(R * sizeof(float));
  b += 2 * align256(R * sizeof(GemvItem));
  b += align256(((M + kItemTok - 1) / kItemTok) * sizeof(GemvItem));
  b += align256(8 * sizeof(int));
  b += 2 * align256(R * I * sizeof(float));
  b += align256(R * I * sizeof(__half)) + align256(R * (I / 128 + 1) * sizeof(float));
  b += align256(R * H * sizeof(float));
  b += 2 * align256(M * I * sizeof(float));
  b += align256(M * I * sizeof(__half)) + align256(M * (I / 128 + 1) * sizeof(float));
  b += align256(M * H * sizeof(float));
  return b;
}

void moe_workspace_carve(MoeWorkspace* ws, const MoeConfig& c, int M, void* base) {
  const size_t H = c.hidden, I = c.moe_inter, E = c.n_experts, K = c.topk;
  const size_t R = static_cast<size_t>(M) * K;
  char* p = static_cast<char*>(base);
  auto take = [&](size_t bytes) {
    void* r = p;
    p += align256(bytes);
    return r;
  };
  ws->max_tokens = M;
  ws->xq = static_cast<__half*>(take(M * H * sizeof(__half)));
  ws->xs = static_cast<float*>(take(M * (H / 128 + 1) * sizeof(float)));
  ws->zd = static_cast<double*>(take(M * E * sizeof(double)));
  ws->zb = static_cast<double*>(take(M * E * sizeof(double)));
  ws->idx = static_cast<int*>(take(R * sizeof(int)));
  ws->wt = static_cast<float*>(take(R * sizeof(float)));
  ws->items_gu = static_cast<GemvItem*>(take(R * sizeof(GemvItem)));
  ws->items_dn = static_cast<GemvItem*>(take(R * sizeof(GemvItem)));
  ws->items_sh = static_cast<GemvItem*>(take(((M + kItemTok - 1) / kItemTok) * sizeof(GemvItem)));
  ws->counters = static_cast<int*>(take(8 * sizeof(int)));
  ws->gate = static_cast<float*>(take(R * I * sizeof(float)));
  ws->up = static_cast<float*>(take(R * I * sizeof(float)));
  ws->qy = static_cast<__half*>(take(R * I * sizeof(__half)));
  ws->qys = static_cast<float*>(take(R * (I / 128 + 1) * sizeof(float)));
  ws->routed = static_cast<float*>(take(R * H * sizeof(float)));
  ws->sh_gate = static_cast<float*>(take(M * I * sizeof(float)));
  ws->sh_up = static_cast<float*>(take(M * I * sizeof(float)));
  ws->sh_qy = static_cast<__half*>(take(M * I * sizeof(__half)));
  ws->sh_qys = static_cast<float*>(take(M * (I / 128 + 1) * sizeof(float)));
  ws->shared = static_cast<float*>(take(M * H * sizeof(float)));
  ws->bytes = static_cast<size_t>(p - static_cast<char*>(base));
}

static cudaError_t route_impl(const MoeConfig& c, const MoeWeights& w, const MoeWorkspace& ws,
                              const float* x, const int* token_ids, int M, int public_router,
                              cudaStream_t st) {
  const int E = c.n_experts;
  dim3 lg((E + 7) / 8, M);
  router_logits_kernel<<<lg, 256, 0, st>>>(x, c.hidden, w.gate_w, E, ws.zd, ws.zb,
                                           public_router);
  SelectArgs sa;
  sa.x = x;
  sa.H = c.hidden;
  sa.E = E;
  sa.topk = c.topk;
  sa.gate = w.gate_w;
  sa.bias = w.bias;
  sa.tid2eid = w.tid2eid;
  sa.hash_vocab = c.hash_vocab;
  sa.token_ids = token_ids;
  sa.zd = ws.zd;
  sa.zb = ws.zb;
  sa.route_scale = c.route_scale;
  sa.public_router = public_router;
  sa.idx = ws.idx;
  sa.wt = ws.wt;
  sa.counters = ws.counters;
  const size_t smem = static_cast<size_t>(E) * (4 + 4 + 8 + 8 + 1) + 16;
  router_select_kernel<<<M, kSelThreads, smem, st>>>(sa);
  return cudaGetLastError();
}

cudaError_t moe_route(const MoeConfig& c, const MoeWeights& w, const MoeWorkspace& ws,
                      const float* x, const int* token_ids, int M, int public_router,
                      cudaStream_t st) {
  if (M <= 0) return cudaSuccess;
  if (M > ws.max_tokens || c.topk > kMaxTopk) return cudaErrorInvalidValue;
  return route_impl(c, w, ws, x, token_ids, M, public_router, st);
}

cudaError_t moe_forward(const MoeConfig& c, const MoeWeights& w, const MoeWorkspace& ws,
                        const float* x, const int* token_ids, int M, float* out,
                        cudaStream_t st) {
  if (M <= 0) return cudaSuccess;
  if (M > ws.max_tokens || c.topk > kMaxTopk || c.n_experts <= 0) return cudaErrorInvalidValue;
  const int H = c.hidden, I = c.moe_inter, K = c.topk, E = c.n_experts;
  const int R = M * K;
  cudaError_t err;

  moe_prep_kernel<<<(M + kItemTok * 128 - 1) / (kItemTok * 128), 128, 0, st>>>(ws.items_sh, M,
                                                                              ws.counters);
  if ((err = launch_quant_fp8(x, H, H, M, ws.xq, ws.xs, H, st)) != cudaSuccess) return err;
  const QAct act{ws.xq, ws.xs, H, nullptr};

  SideStream& side = side_stream();
  const bool has_shared = c.shared_kind != kSharedNone && w.sh1 != nullptr;
  if (has_shared) {
    cudaEventRecord(side.fork, st);
    cudaStreamWaitEvent(side.s, side.fork, 0);
    const int nt = nt_bucket(std::min(M, kItemTok));
    const int sh_items = (M + kItemTok - 1) / kItemTok;
    const QAct sact{ws.sh_qy, ws.sh_qys, I, nullptr};
    if (c.shared_kind == kSharedFp8) {
      Fp8GemvArgs g{};
      g.W[0] = w.sh1; g.S[0] = w.sh1s; g.W[1] = w.sh3; g.S[1] = w.sh3s;
      g.in = H; g.rows = I; g.round_out = 1; g.act = act;
      g.Y[0] = ws.sh_gate; g.Y[1] = ws.sh_up;
      g.items = ws.items_sh; g.n_items = ws.counters + 3; g.max_items = sh_items;
      if ((err = launch_fp8_gemv(g, true, nt, side.s)) != cudaSuccess) return err;
      if ((err = launch_swiglu_quant(ws.sh_gate, ws.sh_up, I, M, nullptr, c.swiglu_limit,
                                     ws.sh_qy, ws.sh_qys, nullptr, side.s)) != cudaSuccess)
        return err;
      Fp8GemvArgs d{};
      d.W[0] = w.sh2; d.S[0] = w.sh2s;
      d.in = I; d.rows = H; d.round_out = 1; d.act = sact;
      d.Y[0] = ws.shared;
      d.items = ws.items_sh; d.n_items = ws.counters + 3; d.max_items = sh_items;
      if ((err = launch_fp8_gemv(d, false, nt, side.s)) != cudaSuccess) return err;
    } else {
      Fp4GemvArgs g{};
      g.W[0] = w.sh1; g.S[0] = w.sh1s; g.W[1] = w.sh3; g.S[1] = w.sh3s;
      g.in = H; g.rows = I; g.act = act;
      g.Y[0] = ws.sh_gate; g.Y[1] = ws.sh_up;
      g.items = ws.items_sh; g.n_items = ws.counters + 3; g.max_items = sh_items;
      if ((err = launch_fp4_gemv(g, true, nt, side.s)) != cudaSuccess) return err;
      if ((err = launch_swiglu_quant(ws.sh_gate, ws.sh_up, I, M, nullptr, c.swiglu_limit,
                                     ws.sh_qy, ws.sh_qys, nullptr, side.s)) != cudaSuccess)
        return err;
      Fp4GemvArgs d{};
      d.W[0] = w.sh2; d.S[0] = w.sh2s;
      d.in = I; d.rows = H; d.act = sact;
      d.Y[0] = ws.shared;
      d.items = ws.items_sh; d.n_items = ws.counters + 3; d.max_items = sh_items;
      if ((err = launch_fp4_gemv(d, false, nt, side.s)) != cudaSuccess) return err;
    }
    cudaEventRecord(side.join, side.s);
  }

  if ((err = route_impl(c, w, ws, x, token_ids, M, 0, st)) != cudaSuccess) return err;
  moe_plan_kernel<<<1, 256, E * sizeof(int), st>>>(ws.idx, M, K, E, ws.items_gu, ws.items_dn,
                                                   ws.counters);

  const int nt = nt_bucket(std::min(M, kItemTok));
  const size_t w13 = static_cast<size_t>(I) * (H / 2), s13 = static_cast<size_t>(I) * (H / 32);
  const size_t w2 = static_cast<size_t>(H) * (I / 2), s2 = static_cast<size_t>(H) * (I / 32);
  Fp4GemvArgs gu{};
  gu.W[0] = w.w1; gu.S[0] = w.s1; gu.W[1] = w.w3; gu.S[1] = w.s3;
  gu.w_stride = w13; gu.s_stride = s13;
  gu.in = H; gu.rows = I; gu.act = act;
  gu.Y[0] = ws.gate; gu.Y[1] = ws.up;
  gu.items = ws.items_gu; gu.n_items = ws.counters; gu.max_items = R;
  if (ws.timing) cudaEventRecord(ws.timing[0], st);
  if ((err = launch_fp4_gemv(gu, true, nt, st)) != cudaSuccess) return err;
  if (ws.timing) cudaEventRecord(ws.timing[1], st);
  if ((err = launch_swiglu_quant(ws.gate, ws.up, I, R, ws.wt, c.swiglu_limit, ws.qy, ws.qys,
                                 nullptr, st)) != cudaSuccess)
    return err;
  Fp4GemvArgs dn{};
  dn.W[0] = w.w2; dn.S[0] = w.s2;
  dn.w_stride = w2; dn.s_stride = s2;
  dn.in = I; dn.rows = H; dn.act = QAct{ws.qy, ws.qys, I, nullptr};
  dn.Y[0] = ws.routed;
  dn.items = ws.items_dn; dn.n_items = ws.counters; dn.max_items = R;
  if (ws.timing) cudaEventRecord(ws.timing[2], st);
  if ((err = launch_fp4_gemv(dn, false, nt, st)) != cudaSuccess) return err;
  if (ws.timing) cudaEventRecord(ws.timing[3], st);

  if (has_shared) cudaStreamWaitEvent(st, side.join, 0);
  const size_t n = static_cast<size_t>(M) * H;
  const int grid = static_cast<int>(std::min<size_t>((n + 255) / 256, 2048));
  moe_combine_kernel<<<grid, 256, 0, st>>>(ws.routed, has_shared ? ws.shared : nullptr, ws.idx,
                                           M, K, H, out);
  return cudaGetLastError();
}

}  // namespace dsv4
