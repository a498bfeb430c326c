// moe.cu - device-resident MoE layer: router with exact expert selection,
// token->expert permutation, grouped FP4 expert GEMVs, shared expert and the
// ascending-id ordered combine.
//
// Router (src/dsv4/dsv4_model.c:6615-6676). The reference's logit z is one
// sequential fp32 fmaf chain over the hidden dimension; replaying that chain
// costs hidden x 4 cycles of latency (~15 us at 7168), so the router instead
//   1. computes the dot product in fp32 with a warp prefix scan, together
//      with a rigorous bound on how far the reference's sequential fp32
//      chain can be from it: the chain's own roundings, u * sum_i |s_i|
//      (u = 2^-24, s_i its prefix sums), plus the scan's rounding error;
//   2. selects the top-k with the reference's rule (score + bias, strict >,
//      lower id wins ties) and checks that every selected expert's lower
//      bound clears every unselected expert's upper bound;
//   3. when the check fails (a near tie), replays the reference's fp32 chain
//      exactly for the experts inside the ambiguous band and selects again.
// The selected SET therefore equals the reference's unless two candidates'
// scores sit within the last-ulp difference between this device's
// sqrt(softplus) and the host libm's; combine weights come from the same
// scores in the reference's order and agree to ~1e-6 relative.
#include <algorithm>
#include <mutex>

#include "dsv4_common.cuh"
#include "moe.cuh"
#include "launch.cuh"

namespace dsv4 {

namespace {

constexpr double kU = 5.9604644775390625e-08;  // 2^-24, fp32 unit roundoff

// sqrt(softplus(z)) in the reference's fp32 operation order
// (src/dsv4/dsv4_model.c:5827), each transcendental rounded once from
// double precision (dsv4_common.cuh states how close that is to the host's
// libm).
__device__ __forceinline__ float sqrt_softplus_f(float z) {
  if (z > 20.0f) return sqrtf(z);
  return sqrtf(log1pf_r1(expf_r1(z)));
}

__global__ void router_scores_kernel(const float* z, float* s, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) s[i] = sqrt_softplus_f(z[i]);
}

// ------------------------------------------------------------- router ----
constexpr int kLogitWarps = 4;    // warps per expert in router_logits_kernel
constexpr int kSelThreads = 256;  // threads per token in router_select_kernel

struct RouterArgs {
  const float* x;            // [M][H] fp32 (BF16-valued)
  int H, M, E, topk;
  const uint16_t* gate;      // [E][H] BF16
  const float* bias;         // [E] or null
  const int64_t* tid2eid;    // [hash_vocab][topk] or null
  int hash_vocab;
  const int* token_ids;      // [M] (hash layers)
  float route_scale;
  int public_router;
  double* zd;                // [M][E] logits
  double* zb;                // [M][E] bound on |z_ref - zd|
  __half* xq;                // [M][H] activation quant (skipped when null)
  float* xs;                 // [M][ceil(H/128)]
  int* idx;                  // [M][topk]
  float* wt;                 // [M][topk]
  GemvItem* items_gu;        // plan outputs (skipped when null): multi-token items
  GemvItem* items_dn;
  GemvItem* items_gu1;       // single-token items
  GemvItem* items_dn1;
  GemvItem* items_sh;
  int* counters;             // [0] multi items, [1] CTA ticket, [2] tie fallbacks,
                             // [3] shared items, [4] single items
  int elo, ehi;              // experts computed on this device (plan only)
  int sh_t0, sh_n;           // tokens the shared expert runs for
};

// The reference's fp32 logit chain, replayed exactly (near-tie path):
// moe_forward uses fmaf (src/dsv4/dsv4_model.c:299-302); the public
// dsv4_router rounds the product and the sum separately (dsv4_ops.c:504).
// Both the gate row and x are staged in shared memory, so the replay runs
// at the FMA chain's latency.
__device__ float exact_logit(const uint16_t* g, const float* xs, int H, int pub) {
  float z = 0.0f;
  if ((H & 7) == 0) {
    const int n8 = H >> 3;
    for (int i = 0; i < n8; i += 4) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int c8 = i + j;
        if (c8 < n8) {
          const uint4 gv = reinterpret_cast<const uint4*>(g)[c8];
          const float4 x0 = reinterpret_cast<const float4*>(xs)[2 * c8];
          const float4 x1 = reinterpret_cast<const float4*>(xs)[2 * c8 + 1];
          const float w[8] = {__uint_as_float(gv.x << 16), __uint_as_float(gv.x & 0xFFFF0000u),
                              __uint_as_float(gv.y << 16), __uint_as_float(gv.y & 0xFFFF0000u),
                              __uint_as_float(gv.z << 16), __uint_as_float(gv.z & 0xFFFF0000u),
                              __uint_as_float(gv.w << 16), __uint_as_float(gv.w & 0xFFFF0000u)};
          const float xv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
          for (int k = 0; k < 8; ++k)
            z = pub ? __fadd_rn(z, __fmul_rn(w[k], xv[k])) : fmaf(w[k], xv[k], z);
        }
      }
    }
  } else {
    for (int c = 0; c < H; ++c)
      z = pub ? __fadd_rn(z, __fmul_rn(bf16_widen(g[c]), xs[c])) : fmaf(bf16_widen(g[c]), xs[c], z);
  }
  return z;
}

// One warp's pass over its chunks [c_begin, c_end) of 256 columns (lane l
// takes 8 consecutive columns of each): running prefix sums t_i in column
// order starting from `offset`. Returns the segment total (from 0) and adds
// sum|offset + t_i| to *sabs and sum|fl(w x)| to *pabs when requested.
__device__ float warp_segment(const uint16_t* g, const float* xr, int H, int c_begin, int c_end,
                              float offset, float* sabs, float* pabs) {
  const int lane = threadIdx.x & 31;
  const bool vec = (H & 7) == 0;
  float carry = 0.0f, sa = 0.0f, pa = 0.0f;
  constexpr int CG = 4;  // chunks whose loads and scans are in flight together
  for (int c0 = c_begin; c0 < c_end; c0 += CG) {
    float q[CG][8], tot[CG];
#pragma unroll
    for (int j = 0; j < CG; ++j) {
      const int col = (c0 + j) * 256 + lane * 8;
      float run = 0.0f;
      const bool live = c0 + j < c_end;
      if (live && vec && col + 8 <= H) {
        const uint4 gv = __ldg(reinterpret_cast<const uint4*>(g + col));
        const float4 x0 = __ldg(reinterpret_cast<const float4*>(xr + col));
        const float4 x1 = __ldg(reinterpret_cast<const float4*>(xr + col + 4));
        const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w};
        const float xv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float w = __uint_as_float((k & 1) ? (gw[k >> 1] & 0xFFFF0000u) : (gw[k >> 1] << 16));
          const float p = w * xv[k];
          run += p;
          q[j][k] = run;
          pa += fabsf(p);
        }
      } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const int c = col + k;
          const float p = (live && c < H) ? bf16_widen(g[c]) * xr[c] : 0.0f;
          run += p;
          q[j][k] = run;
          pa += fabsf(p);
        }
      }
      tot[j] = run;
    }
    float incl[CG];
#pragma unroll
    for (int j = 0; j < CG; ++j) incl[j] = tot[j];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
#pragma unroll
      for (int j = 0; j < CG; ++j) {
        const float v = __shfl_up_sync(0xffffffffu, incl[j], o);
        if (lane >= o) incl[j] += v;
      }
    }
#pragma unroll
    for (int j = 0; j < CG; ++j) {
      if (sabs) {
        const float base = offset + (carry + (incl[j] - tot[j]));
#pragma unroll
        for (int k = 0; k < 8; ++k) sa += fabsf(base + q[j][k]);
      }
      carry += __shfl_sync(0xffffffffu, incl[j], 31);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    sa += __shfl_xor_sync(0xffffffffu, sa, o);
    pa += __shfl_xor_sync(0xffffffffu, pa, o);
  }
  if (sabs) *sabs = sa;
  if (pabs) *pabs = pa;
  return carry;
}

// warp_segment in one pass over memory for segments of at most kSegCache
// full 256-column chunks: the products' running sums stay in registers while
// the block exchanges the segment totals, then sabs is formed with the same
// expressions as warp_segment's second pass (identical t_i, so the same
// bound holds).
constexpr int kSegCache = 8;
struct SegState {
  float q[kSegCache][8];
  float part[kSegCache];  // carry + (incl - tot): lane's offset inside the segment
  float total, pabs;
};

__device__ __forceinline__ void warp_segment_load(const uint16_t* g, const float* xr, int c_begin, int c_end,
                                  SegState& st) {
  const int lane = threadIdx.x & 31;
  float tot[kSegCache];
  float pa = 0.0f;
  // every chunk's gate and activation vectors are requested before the
  // first is used, so the segment costs one memory round trip
  uint4 gvs[kSegCache];
  float4 x0s[kSegCache], x1s[kSegCache];
#pragma unroll
  for (int j = 0; j < kSegCache; ++j) {
    if (c_begin + j < c_end) {
      const int col = (c_begin + j) * 256 + lane * 8;
      gvs[j] = __ldg(reinterpret_cast<const uint4*>(g + col));
      x0s[j] = __ldg(reinterpret_cast<const float4*>(xr + col));
      x1s[j] = __ldg(reinterpret_cast<const float4*>(xr + col + 4));
    }
  }
#pragma unroll
  for (int j = 0; j < kSegCache; ++j) {
    float run = 0.0f;
    if (c_begin + j < c_end) {
      const uint4 gv = gvs[j];
      const float4 x0 = x0s[j];
      const float4 x1 = x1s[j];
      const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w};
      const float xv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float w = __uint_as_float((k & 1) ? (gw[k >> 1] & 0xFFFF0000u) : (gw[k >> 1] << 16));
        const float pr = w * xv[k];
        run += pr;
        st.q[j][k] = run;
        pa += fabsf(pr);
      }
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k) st.q[j][k] = 0.0f;
    }
    tot[j] = run;
  }
  float incl[kSegCache];
#pragma unroll
  for (int j = 0; j < kSegCache; ++j) incl[j] = tot[j];
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
#pragma unroll
    for (int j = 0; j < kSegCache; ++j) {
      const float v = __shfl_up_sync(0xffffffffu, incl[j], o);
      if (lane >= o) incl[j] += v;
    }
  }
  float carry = 0.0f;
#pragma unroll
  for (int j = 0; j < kSegCache; ++j) {
    st.part[j] = carry + (incl[j] - tot[j]);
    if (c_begin + j < c_end) carry += __shfl_sync(0xffffffffu, incl[j], 31);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) pa += __shfl_xor_sync(0xffffffffu, pa, o);
  st.total = carry;
  st.pabs = pa;
}

__device__ __forceinline__ float warp_segment_abs(const SegState& st, int c_begin, int c_end, float offset) {
  float sa = 0.0f;
#pragma unroll
  for (int j = 0; j < kSegCache; ++j) {
    if (c_begin + j < c_end) {
      const float base = offset + st.part[j];
#pragma unroll
      for (int k = 0; k < 8; ++k) sa += fabsf(base + st.q[j][k]);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sa += __shfl_xor_sync(0xffffffffu, sa, o);
  return sa;
}

// Launch 1, grid (E, M) x 4 warps: activation quant (spread over all warps)
// and one router logit per CTA, in fp32, with a rigorous bound on how far
// the reference's sequential chain can be from it. The row is split over 4
// warps; pass 1 gives each warp's segment total, pass 2 (L2-resident data)
// re-walks the segment from its exact offset to sum |t_i|. Notation: p_i
// exact products, q_i = fl(p_i), P = sum |q_i|, s_i exact prefix sums, t_i
// the computed ones (depth d: 8 in-lane + 5 scan + the segment's chunk
// carries + 3 offset/base adds + 4 for the cross-warp sums), zc the computed
// total. Then |zc - z| <= (d + 1) u P, |s_i - t_i| <= (d + 1) u P and
// |z_ref - z| <= u sum_i |s_i| (+ u P for the public router's rounded
// products), so
//   zb = u sum|t_i| + (d + 1) u P (1 + n u) (+ u P)   (x 1.01 for the fp32
// evaluation of the bound itself).
__device__ void write_shared_items(const RouterArgs& a);

// FP8 (E4M3 grid, power-of-two per-128 scale) quant of every token row of x
// into xq/xs, one (row, 128-column block) per warp task; gw/nw = this warp's
// index and the warp count over the launch.
__device__ void quant_rows(const RouterArgs& a, int gw, int nw) {
  const int lane = threadIdx.x & 31;
  const int nb = (a.H + 127) / 128;
  for (int task = gw; task < a.M * nb; task += nw) {
    const int r = task / nb, b = task % nb;
    const float* xr = a.x + static_cast<size_t>(r) * a.H + b * 128;
    const int len = min(128, a.H - b * 128);
    float v[4];
    float amax = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int i = lane + 32 * k;
      v[k] = i < len ? xr[i] : 0.f;
      amax = fmaxf(amax, fabsf(v[k]));
    }
    amax = warp_max(amax);
    const float scale = pow2_scale_448(amax);
    const float inv = 1.0f / scale;
    if (lane == 0) a.xs[static_cast<size_t>(r) * nb + b] = scale;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int i = lane + 32 * k;
      if (i < len) {
        float q = v[k] * inv;
        q = q > 448.f ? 448.f : (q < -448.f ? -448.f : q);
        a.xq[static_cast<size_t>(r) * a.H + b * 128 + i] = e4m3_round_f16(q);
      }
    }
  }
}

__global__ void __launch_bounds__(kLogitWarps * 32) router_logits_kernel(const RouterArgs a) {
  __shared__ float seg_tot[kLogitWarps], seg_abs[kLogitWarps], seg_p[kLogitWarps];
  pdl_trigger();
  {
    // the expert's gate row toward L2 while the previous kernel finishes
    const char* gr = reinterpret_cast<const char*>(a.gate + static_cast<size_t>(blockIdx.x) * a.H);
    for (int o = threadIdx.x * 128; o < a.H * 2; o += blockDim.x * 128)
      asm volatile("prefetch.global.L2 [%0];" ::"l"(gr + o));
  }
  pdl_wait();  // x comes from the previous kernel
  if (a.items_sh && blockIdx.x == 0 && blockIdx.y == 0) write_shared_items(a);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int e = blockIdx.x, t = blockIdx.y;
  if (a.xq) quant_rows(a, (blockIdx.y * gridDim.x + blockIdx.x) * kLogitWarps + warp,
                      gridDim.x * gridDim.y * kLogitWarps);
  const uint16_t* g = a.gate + static_cast<size_t>(e) * a.H;
  const float* xr = a.x + static_cast<size_t>(t) * a.H;
  const int nch = (a.H + 255) / 256;
  const int per = (nch + kLogitWarps - 1) / kLogitWarps;
  const int cb = min(nch, warp * per), ce = min(nch, cb + per);
  const bool cached = (a.H % 256 == 0) && per <= kSegCache;
  SegState seg;
  float pw = 0.0f, tw;
  if (cached) {
    warp_segment_load(g, xr, cb, ce, seg);
    tw = seg.total;
    pw = seg.pabs;
  } else {
    tw = warp_segment(g, xr, a.H, cb, ce, 0.0f, nullptr, &pw);
  }
  if (lane == 0) {
    seg_tot[warp] = tw;
    seg_p[warp] = pw;
  }
  __syncthreads();
  float off = 0.0f;
  for (int w = 0; w < warp; ++w) off += seg_tot[w];
  float aw = 0.0f;
  if (cached) aw = warp_segment_abs(seg, cb, ce, off);
  else warp_segment(g, xr, a.H, cb, ce, off, &aw, nullptr);
  if (lane == 0) seg_abs[warp] = aw;
  __syncthreads();
  if (threadIdx.x == 0) {
    float z = 0.0f, sabs = 0.0f, P = 0.0f;
    for (int w = 0; w < kLogitWarps; ++w) {
      z += seg_tot[w];
      sabs += seg_abs[w];
      P += seg_p[w];
    }
    const double u = kU, n = static_cast<double>(a.H);
    const double d = 20.0 + static_cast<double>(per);
    const size_t o = static_cast<size_t>(t) * a.E + e;
    a.zd[o] = static_cast<double>(z);
    a.zb[o] = 1.01 * (u * static_cast<double>(sabs) +
                      (d + 1.0) * u * static_cast<double>(P) * (1.0 + n * u) +
                      (a.public_router ? u * static_cast<double>(P) : 0.0)) + 1e-40 * n;
  }
}

// Orderable key of a selection value: a larger value gives a larger key;
// -inf and NaN give 0 and are never selected (the reference's strict ">"
// scan starts from -inf, src/dsv4/dsv4_model.c:6636); -0 compares equal to
// +0 as it does in the reference.
__device__ __forceinline__ uint32_t sel_key(float v) {
  if (!(v > -INFINITY)) return 0u;
  if (v == 0.0f) v = 0.0f;
  const uint32_t b = __float_as_uint(v);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// Top-k by the reference rule (largest value, lowest id among equal values),
// order[] in selection order, used[] marks the picks. Warp 0 does the work
// with warp reductions (no block barrier per pick); every thread calls it.
__device__ void warp_topk(const float* val, unsigned char* used, int E, int k, int* order) {
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    for (int e = lane; e < E; e += 32) used[e] = 0;
    __syncwarp();
    for (int j = 0; j < k; ++j) {
      uint32_t bk = 0u;
      int bid = 0x7FFFFFFF;
      for (int e = lane; e < E; e += 32) {  // ascending ids: ">" keeps the lower id
        if (used[e]) continue;
        const uint32_t key = sel_key(val[e]);
        if (key > bk) { bk = key; bid = e; }
      }
      const uint32_t mk = __reduce_max_sync(0xffffffffu, bk);
      const int id = static_cast<int>(__reduce_min_sync(
          0xffffffffu, static_cast<unsigned>((bk == mk) ? bid : 0x7FFFFFFF)));
      const int pick = mk == 0u ? -1 : id;
      if (lane == 0) {
        order[j] = pick;
        if (pick >= 0) used[pick] = 1;
      }
      __syncwarp();
    }
  }
  __syncthreads();
}

// Exclusive prefix sum of one int per thread over the block (blockDim.x a
// multiple of 32, <= 1024); *total receives the sum. Uses wsum[33]
// (wsum[32] holds the total).
__device__ int block_excl_scan(int v, int* wsum, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  if (lane == 31) wsum[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int w = lane < nw ? wsum[lane] : 0;
    int wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += t;
    }
    if (lane < nw) wsum[lane] = wi - w;  // exclusive warp offsets
    if (lane == 31) wsum[32] = wi;       // lane 31 holds the block total
  }
  __syncthreads();
  const int r = wsum[warp] + incl - v;
  *total = wsum[32];
  __syncthreads();
  return r;
}

// In-place exclusive scan of arr[0..E) by the whole block; the total goes
// to *total (shared memory) for every thread.
__device__ void plan_excl_scan(int* arr, int E, int* total) {
  if (E <= static_cast<int>(blockDim.x)) {
    __shared__ int wsum[33];
    int t = 0;
    const int v = static_cast<int>(threadIdx.x) < E ? arr[threadIdx.x] : 0;
    const int off = block_excl_scan(v, wsum, &t);
    if (static_cast<int>(threadIdx.x) < E) arr[threadIdx.x] = off;
    if (threadIdx.x == 0) *total = t;
  } else if (threadIdx.x < 32) {
    // one warp: 32-element tiles with a carry
    int carry = 0;
    for (int b0 = 0; b0 < E; b0 += 32) {
      const int e = b0 + threadIdx.x;
      const int v = e < E ? arr[e] : 0;
      int incl = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int tt = __shfl_up_sync(0xffffffffu, incl, o);
        if (static_cast<int>(threadIdx.x) >= o) incl += tt;
      }
      if (e < E) arr[e] = carry + incl - v;
      carry += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (threadIdx.x == 0) *total = carry;
  }
  __syncthreads();
}

// Token->expert permutation (moe_forward_batch grouping,
// src/dsv4/dsv4_model.c:6925-6926, expert_forward_batch_routes :6486): unique
// experts ascending; each expert's routes in token order. An expert with one
// route becomes a single-token item (items_gu1/dn1, counters[4]); one with
// more becomes items of <= kItemTok routes (items_gu/dn, counters[0]), so the
// single-token items run on the one-token GEMV kernel. Route (t,k) owns slot
// t*topk+k. One CTA; idx staged in shared memory.
__device__ void block_plan(const RouterArgs& a, int* cnt, int* cnt1, int* ids) {
  const int E = a.E, K = a.topk, R = a.M * a.topk;
  __shared__ int n_multi, n_single;
  for (int r = threadIdx.x; r < R; r += blockDim.x) ids[r] = a.idx[r];
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int n = 0;
    if (e >= a.elo && e < a.ehi)
      for (int r = 0; r < R; ++r) n += (ids[r] == e);
    cnt[e] = n >= 2 ? (n + kItemTok - 1) / kItemTok : 0;
    cnt1[e] = n == 1 ? 1 : 0;
  }
  __syncthreads();
  plan_excl_scan(cnt, E, &n_multi);
  plan_excl_scan(cnt1, E, &n_single);
  if (threadIdx.x == 0) {
    a.counters[0] = n_multi;
    a.counters[4] = n_single;
  }
  for (int e = a.elo + threadIdx.x; e < a.ehi; e += blockDim.x) {
    int n = 0;
    for (int r = 0; r < R; ++r) n += (ids[r] == e);
    if (n == 0) continue;
    GemvItem gu, dn;
    gu.mat = dn.mat = e - a.elo;  // index into this device's expert weights
    gu.ntok = dn.ntok = 0;
    GemvItem* out_gu = n == 1 ? a.items_gu1 : a.items_gu;
    GemvItem* out_dn = n == 1 ? a.items_dn1 : a.items_dn;
    int item = n == 1 ? cnt1[e] : cnt[e];
    for (int r = 0; r < R; ++r) {
      if (ids[r] != e) continue;
      gu.tok[gu.ntok].x = r / K;
      gu.tok[gu.ntok].y = r;
      dn.tok[dn.ntok].x = r;
      dn.tok[dn.ntok].y = r;
      gu.ntok++;
      dn.ntok++;
      if (gu.ntok == kItemTok) {
        out_gu[item] = gu;
        out_dn[item] = dn;
        ++item;
        gu.ntok = dn.ntok = 0;
      }
    }
    if (gu.ntok > 0) {
      for (int i = gu.ntok; i < kItemTok; ++i) { gu.tok[i] = gu.tok[0]; dn.tok[i] = dn.tok[0]; }
      out_gu[item] = gu;
      out_dn[item] = dn;
    }
  }
}

// The activation quant and the shared-expert items as a launch of their
// own, ahead of the logits, so the shared expert (which needs only these)
// starts while the router is still running.
__global__ void __launch_bounds__(kLogitWarps * 32) act_quant_kernel(const RouterArgs a) {
  pdl_wait();  // x comes from the previous kernel
  pdl_trigger();
  if (a.items_sh && blockIdx.x == 0) write_shared_items(a);
  quant_rows(a, blockIdx.x * kLogitWarps + (threadIdx.x >> 5), gridDim.x * kLogitWarps);
}

// Shared-expert items (every token, in groups of kItemTok); they depend on M
// only, so the logit kernel writes them and the shared expert can start
// before the selection finishes.
__device__ void write_shared_items(const RouterArgs& a) {
  const int nsh = (a.sh_n + kItemTok - 1) / kItemTok;
  for (int j = threadIdx.x; j < nsh; j += blockDim.x) {
    GemvItem it;
    it.mat = 0;
    it.ntok = min(kItemTok, a.sh_n - j * kItemTok);
    for (int i = 0; i < kItemTok; ++i) {
      const int tt = a.sh_t0 + min(j * kItemTok + i, a.sh_n - 1);
      it.tok[i].x = tt;
      it.tok[i].y = tt;
    }
    a.items_sh[j] = it;
  }
  if (threadIdx.x == 0) a.counters[3] = nsh;
}

constexpr int kReplayRows = 4;  // candidate gate rows staged per replay round

struct SelectSmem {
  float* x;       // [H] token activation (exact replay)
  uint16_t* g;    // [kReplayRows][H] candidate gate rows (exact replay)
  int* cand;      // [E] candidate list
  double* lo;     // [E]
  double* hi;     // [E]
  float* choice;  // [E]
  float* score;   // [E]
  int* cnt;       // [E] plan (multi-token items)
  int* cnt1;      // [E] plan (single-token items)
  int* ids;       // [R] plan
  unsigned char* used;  // [E]
};

__host__ __device__ inline size_t select_smem_bytes(int H, int E, int R, SelectSmem* sm,
                                                    unsigned char* base) {
  size_t off = 0;
  auto take = [&](size_t bytes) {
    unsigned char* p = base + off;
    off += (bytes + 15) & ~static_cast<size_t>(15);
    return p;
  };
  unsigned char* px = take(static_cast<size_t>(H) * 4);
  unsigned char* pg = take(static_cast<size_t>(kReplayRows) * H * 2);
  unsigned char* pk = take(static_cast<size_t>(E) * 4);
  unsigned char* plo = take(static_cast<size_t>(E) * 8);
  unsigned char* phi = take(static_cast<size_t>(E) * 8);
  unsigned char* pc = take(static_cast<size_t>(E) * 4);
  unsigned char* ps = take(static_cast<size_t>(E) * 4);
  unsigned char* pn = take(static_cast<size_t>(E) * 4);
  unsigned char* pn1 = take(static_cast<size_t>(E) * 4);
  unsigned char* pi = take(static_cast<size_t>(R) * 4);
  unsigned char* pu = take(static_cast<size_t>(E));
  if (sm) {
    sm->x = reinterpret_cast<float*>(px);
    sm->g = reinterpret_cast<uint16_t*>(pg);
    sm->cand = reinterpret_cast<int*>(pk);
    sm->lo = reinterpret_cast<double*>(plo);
    sm->hi = reinterpret_cast<double*>(phi);
    sm->choice = reinterpret_cast<float*>(pc);
    sm->score = reinterpret_cast<float*>(ps);
    sm->cnt = reinterpret_cast<int*>(pn);
    sm->cnt1 = reinterpret_cast<int*>(pn1);
    sm->ids = reinterpret_cast<int*>(pi);
    sm->used = pu;
  }
  return off;
}

// Launch 2, one CTA per token: selection with the reference's rule and the
// margin check (exact replay of the band on a near tie), combine weights and
// the id sort (src/dsv4/dsv4_model.c:6615-6676; public twin
// src/dsv4/dsv4_ops.c:473-545); the last CTA to finish builds the plan.
__global__ void __launch_bounds__(kSelThreads) router_select_kernel(const RouterArgs a) {
  extern __shared__ __align__(16) unsigned char ssm[];
  __shared__ double rlo[kSelThreads / 32], rhi[kSelThreads / 32];
  __shared__ int order[kMaxTopk];
  __shared__ int is_last, n_cand;
  SelectSmem sm;
  select_smem_bytes(a.H, a.E, a.M * a.topk, &sm, ssm);
  pdl_wait();  // the logits and bounds come from router_logits_kernel
  pdl_trigger();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int t = blockIdx.x;
  const int E = a.E;
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    const size_t o = static_cast<size_t>(t) * E + e;
    const double z = a.zd[o];
    const float b = a.bias ? a.bias[e] : 0.0f;
    const float s = sqrt_softplus_f(static_cast<float>(z));
    sm.score[e] = s;
    sm.choice[e] = s + b;
    // |d sqrt(softplus)/dz| <= 0.5 (|z - z_ref| <= zb, plus the rounding of
    // z to fp32); 1e-6 relative covers the few-ulp differences of expf,
    // log1pf, sqrtf and the bias add between glibc and CUDA.
    const double rad = 0.5 * (a.zb[o] + kU * fabs(z)) +
                       1e-6 * (fabs(static_cast<double>(s)) + fabs(static_cast<double>(b))) + 1e-37;
    sm.lo[e] = static_cast<double>(s) + b - rad;
    sm.hi[e] = static_cast<double>(s) + b + rad;
  }
  __syncthreads();
  if (a.tid2eid) {
    if (threadIdx.x == 0) {
      const int tok = a.token_ids ? a.token_ids[t] : 0;
      const int tk = (tok >= 0 && tok < a.hash_vocab) ? tok : 0;
      for (int k = 0; k < a.topk; ++k) {
        const int64_t e = a.tid2eid[static_cast<size_t>(tk) * a.topk + k];
        order[k] = (e >= 0 && e < E) ? static_cast<int>(e) : -1;
      }
    }
    __syncthreads();
  } else {
    __shared__ int s_replay, s_nan;
    __shared__ double s_mlo, s_mhi;
    if (E <= 8 * 32) {
      // warp 0 holds every expert's choice and interval in registers (lane l:
      // experts l + 32 i): top-k and the margin check without block barriers
      if (warp == 0) {
        float cv[8];
        double lo[8], hi[8];
        bool nan_seen = false;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int e = lane + 32 * i;
          const bool in = e < E;
          cv[i] = in ? sm.choice[e] : -INFINITY;
          lo[i] = in ? sm.lo[e] : INFINITY;
          hi[i] = in ? sm.hi[e] : -INFINITY;
          if (in && (isnan(lo[i]) || isnan(hi[i]))) nan_seen = true;
        }
        uint32_t used = 0u;  // bit i: expert lane + 32 i was picked
        for (int j = 0; j < a.topk; ++j) {
          uint32_t bk = 0u;
          int bi = 0x7FFFFFFF;
#pragma unroll
          for (int i = 0; i < 8; ++i) {  // ascending ids within the lane
            const uint32_t key = ((used >> i) & 1u) ? 0u : sel_key(cv[i]);
            if (key > bk) { bk = key; bi = lane + 32 * i; }
          }
          const uint32_t mk = __reduce_max_sync(0xffffffffu, bk);
          const int id = static_cast<int>(__reduce_min_sync(
              0xffffffffu, static_cast<unsigned>((bk == mk) ? bi : 0x7FFFFFFF)));
          const int pick = mk == 0u ? -1 : id;
          if (pick >= 0 && (pick & 31) == lane) used |= 1u << (pick >> 5);
          if (lane == 0) order[j] = pick;
        }
        double mlo = INFINITY, mhi = -INFINITY;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          if ((used >> i) & 1u) mlo = fmin(mlo, lo[i]);
          else mhi = fmax(mhi, hi[i]);
          const int e = lane + 32 * i;
          if (e < E) sm.used[e] = static_cast<unsigned char>((used >> i) & 1u);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          mlo = fmin(mlo, __shfl_xor_sync(0xffffffffu, mlo, o));
          mhi = fmax(mhi, __shfl_xor_sync(0xffffffffu, mhi, o));
        }
        const bool any_nan = __any_sync(0xffffffffu, nan_seen);
        if (lane == 0) {
          s_nan = any_nan ? 1 : 0;
          s_replay = (any_nan || !(mlo > mhi)) ? 1 : 0;
          s_mlo = mlo;
          s_mhi = mhi;
        }
      }
      __syncthreads();
    } else {
      warp_topk(sm.choice, sm.used, E, a.topk, order);
      double mlo = INFINITY, mhi = -INFINITY;
      int nan_seen = 0;
      for (int e = threadIdx.x; e < E; e += blockDim.x) {
        if (isnan(sm.lo[e]) || isnan(sm.hi[e])) nan_seen = 1;
        if (sm.used[e]) mlo = fmin(mlo, sm.lo[e]);
        else mhi = fmax(mhi, sm.hi[e]);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        mlo = fmin(mlo, __shfl_xor_sync(0xffffffffu, mlo, o));
        mhi = fmax(mhi, __shfl_xor_sync(0xffffffffu, mhi, o));
      }
      if (lane == 0) { rlo[warp] = mlo; rhi[warp] = mhi; }
      const int any_nan = __syncthreads_or(nan_seen);
      if (threadIdx.x == 0) {
        for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w) {
          mlo = fmin(mlo, rlo[w]);
          mhi = fmax(mhi, rhi[w]);
        }
        s_nan = any_nan;
        s_replay = (any_nan || !(mlo > mhi)) ? 1 : 0;
        s_mlo = mlo;
        s_mhi = mhi;
      }
      __syncthreads();
    }
    if (s_replay) {
      // near tie: replay the reference's fp32 chain for every expert whose
      // interval reaches into the ambiguous band, then select again
      const int any_nan = s_nan;
      const double mlo = s_mlo, mhi = s_mhi;
      const float* xr = a.x + static_cast<size_t>(t) * a.H;
      if (threadIdx.x == 0) n_cand = 0;
      for (int i = threadIdx.x; i < a.H; i += blockDim.x) sm.x[i] = xr[i];
      __syncthreads();
      for (int e = threadIdx.x; e < E; e += blockDim.x)
        if (any_nan || (sm.hi[e] >= mlo && sm.lo[e] <= mhi)) sm.cand[atomicAdd(&n_cand, 1)] = e;
      __syncthreads();
      const int nc = n_cand;
      for (int c0 = 0; c0 < nc; c0 += kReplayRows) {
        const int rows = min(kReplayRows, nc - c0);
        // stage the round's gate rows (coalesced, all threads)
        for (int r = 0; r < rows; ++r) {
          const uint16_t* src = a.gate + static_cast<size_t>(sm.cand[c0 + r]) * a.H;
          uint16_t* dst = sm.g + static_cast<size_t>(r) * a.H;
          for (int i = threadIdx.x; i < a.H; i += blockDim.x) dst[i] = src[i];
        }
        __syncthreads();
        if (static_cast<int>(threadIdx.x) < rows) {
          const int e = sm.cand[c0 + threadIdx.x];
          const float z = exact_logit(sm.g + static_cast<size_t>(threadIdx.x) * a.H, sm.x, a.H,
                                      a.public_router);
          const float s = sqrt_softplus_f(z);
          sm.score[e] = s;
          sm.choice[e] = s + (a.bias ? a.bias[e] : 0.0f);
        }
        __syncthreads();
      }
      warp_topk(sm.choice, sm.used, E, a.topk, order);
      if (threadIdx.x == 0) atomicAdd(&a.counters[2], 1);
    }
  }
  if (threadIdx.x < 32) {
    // warp 0, lane k = k-th pick: weights from the scores summed in pick
    // order (src/dsv4/dsv4_model.c:6651-6658; public twin
    // src/dsv4/dsv4_ops.c:528-531), then the ascending-id exchange sort of
    // :6669-6676 restated as a stable rank (equal ids keep their order)
    const int K = a.topk, k = lane;
    const int id = k < K ? order[k] : 0x7FFFFFFF;
    const float sc = (k < K && id >= 0) ? sm.score[id] : 0.0f;
    float sum = 0.0f;
    for (int j = 0; j < K; ++j) sum += __shfl_sync(0xffffffffu, sc, j);
    float w;
    if (a.public_router) {
      const float inv = sum > 0.0f ? 1.0f / sum : 0.0f;
      w = sc * inv * a.route_scale;
    } else {
      w = sum > 0.0f ? sc * (a.route_scale / sum) : 0.0f;
    }
    int rank = 0;
    for (int j = 0; j < K; ++j) {
      const int o = __shfl_sync(0xffffffffu, id, j);
      rank += (o < id) || (o == id && j < k);
    }
    if (k < K) {
      a.idx[static_cast<size_t>(t) * K + rank] = id;
      a.wt[static_cast<size_t>(t) * K + rank] = w;
    }
    if (a.items_gu && gridDim.x == 1 && !a.tid2eid) {
      // single token, distinct picks: one item per local route, in
      // ascending id order (what block_plan produces for M = 1)
      if (k < K) order[rank] = id;
      __syncwarp();
      const int e = k < K ? order[k] : -1;
      const bool local = e >= a.elo && e < a.ehi;
      const unsigned m = __ballot_sync(0xffffffffu, local);
      if (local) {
        const int item = __popc(m & ((1u << k) - 1u));
        GemvItem gu, dn;
        gu.mat = dn.mat = e - a.elo;
        gu.ntok = dn.ntok = 1;
#pragma unroll
        for (int i = 0; i < kItemTok; ++i) {
          gu.tok[i].x = 0;
          gu.tok[i].y = k;
          dn.tok[i].x = k;
          dn.tok[i].y = k;
        }
        a.items_gu1[item] = gu;
        a.items_dn1[item] = dn;
      }
      if (lane == 0) {
        a.counters[4] = __popc(m);
        a.counters[0] = 0;
      }
    }
  }
  if (!a.items_gu || (gridDim.x == 1 && !a.tid2eid)) return;  // no plan, or planned above
  if (gridDim.x == 1) {
    // one token: this CTA wrote every route itself
    __syncthreads();
  } else {
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) is_last = atomicAdd(&a.counters[1], 1) == static_cast<int>(gridDim.x) - 1;
    __syncthreads();
    if (!is_last) return;
    __threadfence();
  }
  block_plan(a, sm.cnt, sm.cnt1, sm.ids);
  if (threadIdx.x == 0 && gridDim.x > 1) a.counters[1] = 0;  // ticket ready for the next launch
}

// out[t] = bf16( sum_k routed[t*topk+k] (ascending id order) + shared[t] )
// (src/dsv4/dsv4_model.c:6795-6805, :7096-7112).
__global__ void moe_combine_kernel(const float* __restrict__ routed, const float* __restrict__ shared,
                                   const int* __restrict__ idx, int n_tokens, int topk, int H,
                                   float* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const size_t n = static_cast<size_t>(n_tokens) * H;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int t = static_cast<int>(i / H);
    const int c = static_cast<int>(i % H);
    float acc = sum_routes(idx + t * topk, routed + static_cast<size_t>(t) * topk * H + c, H,
                           topk);
    if (shared) acc += shared[i];
    out[i] = bf16_round(acc);
  }
}

size_t align256(size_t b) { return (b + 255) & ~static_cast<size_t>(255); }

// Timing events are recorded as external event nodes when the stream is
// being captured, so a replayed graph records them too.
void record_timing(cudaEvent_t ev, cudaStream_t st) {
  cudaEventRecordWithFlags(ev, st, cudaEventRecordExternal);
}

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
  b += 4 * align256(R * sizeof(GemvItem));
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
  ws->items_gu1 = static_cast<GemvItem*>(take(R * sizeof(GemvItem)));
  ws->items_dn1 = static_cast<GemvItem*>(take(R * sizeof(GemvItem)));
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

static RouterArgs make_router_args(const MoeConfig& c, const MoeWeights& w, const MoeWorkspace& ws,
                            const float* x, const int* token_ids, int M, int public_router,
                            bool plan) {
  RouterArgs a{};
  a.x = x;
  a.H = c.hidden;
  a.M = M;
  a.E = c.n_experts;
  a.topk = c.topk;
  a.gate = w.gate_w;
  a.bias = w.bias;
  a.tid2eid = w.tid2eid;
  a.hash_vocab = c.hash_vocab;
  a.token_ids = token_ids;
  a.route_scale = c.route_scale;
  a.public_router = public_router;
  a.zd = ws.zd;
  a.zb = ws.zb;
  a.idx = ws.idx;
  a.wt = ws.wt;
  a.counters = ws.counters;
  a.elo = c.expert_lo;
  a.ehi = moe_local_hi(c);
  a.sh_t0 = 0;
  a.sh_n = M;
  if (plan) {
    a.xq = ws.xq;
    a.xs = ws.xs;
    a.items_gu = ws.items_gu;
    a.items_dn = ws.items_dn;
    a.items_gu1 = ws.items_gu1;
    a.items_dn1 = ws.items_dn1;
    a.items_sh = ws.items_sh;
  }
  return a;
}

// Launch 1 of the router: logits, bounds, activation quant, shared items.
cudaError_t route_logits(const RouterArgs& a, const MoeConfig& c, const MoeWorkspace& ws, int M,
                         bool plan, cudaStream_t st, bool mark_start = true) {
  if (plan && ws.timing && mark_start) record_timing(ws.timing[4], st);
  {
    cudaError_t e = launch_pdl(router_logits_kernel, dim3(c.n_experts, M), dim3(kLogitWarps * 32),
                               0, st, a);
    if (e != cudaSuccess) return e;
  }
  if (plan && ws.timing) record_timing(ws.timing[5], st);
  return cudaSuccess;
}

// Launch 2: selection, weights and the expert plan.
cudaError_t route_select(const RouterArgs& a, const MoeConfig& c, const MoeWorkspace& ws, int M,
                         bool plan, cudaStream_t st) {
  const size_t smem = select_smem_bytes(c.hidden, c.n_experts, M * c.topk, nullptr, nullptr);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(router_select_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
  }
  {
    cudaError_t e = launch_pdl(router_select_kernel, dim3(M), dim3(kSelThreads), smem, st, a);
    if (e != cudaSuccess) return e;
  }
  if (plan && ws.timing) record_timing(ws.timing[6], st);
  return cudaGetLastError();
}

cudaError_t route_impl(const MoeConfig& c, const MoeWeights& w, const MoeWorkspace& ws,
                       const float* x, const int* token_ids, int M, int public_router, bool plan,
                       cudaStream_t st) {
  const RouterArgs a = make_router_args(c, w, ws, x, token_ids, M, public_router, plan);
  cudaError_t e = route_logits(a, c, ws, M, plan, st);
  return e != cudaSuccess ? e : route_select(a, c, ws, M, plan, st);
}

cudaError_t moe_route(const MoeConfig& c, const MoeWeights& w, const MoeWorkspace& ws,
                      const float* x, const int* token_ids, int M, int public_router,
                      cudaStream_t st) {
  if (M <= 0) return cudaSuccess;
  if (M > ws.max_tokens || c.topk > kMaxTopk) return cudaErrorInvalidValue;
  return route_impl(c, w, ws, x, token_ids, M, public_router, false, st);
}

cudaError_t moe_forward_local(const MoeConfig& c, const MoeWeights& w, const MoeWorkspace& ws,
                              const float* x, const int* token_ids, int M, cudaStream_t st,
                              const MoeExecOptions& opt) {
  if (M <= 0) return cudaSuccess;
  if (M > ws.max_tokens || c.topk > kMaxTopk || c.n_experts <= 0) return cudaErrorInvalidValue;
  if (c.expert_lo < 0 || c.expert_lo >= moe_local_hi(c) || moe_local_hi(c) > c.n_experts)
    return cudaErrorInvalidValue;
  const int H = c.hidden, I = c.moe_inter, K = c.topk;
  const int R = M * K;
  const int n_local = moe_local_hi(c) - c.expert_lo;
  cudaError_t err;
  // slots of experts computed elsewhere stay zero for the cross-device sum
  if (moe_is_partial(c) &&
      (err = cudaMemsetAsync(ws.routed, 0, sizeof(float) * R * H, st)) != cudaSuccess)
    return err;

  // router launch 1: activation quant + logits (+ the shared-expert items)
  const int sh_t0 = opt.shared_n < 0 ? 0 : opt.shared_t0;
  const int sh_n = opt.shared_n < 0 ? M : opt.shared_n;
  if (sh_t0 < 0 || sh_n < 1 || sh_t0 + sh_n > M) return cudaErrorInvalidValue;
  RouterArgs ra = make_router_args(c, w, ws, x, token_ids, M, 0, true);
  ra.sh_t0 = sh_t0;
  ra.sh_n = sh_n;
  const QAct act{ws.xq, ws.xs, H, nullptr};

  const bool has_shared = c.shared_kind != kSharedNone && w.sh1 != nullptr;
  // the shared expert overlaps the router and the routed path on a side
  // stream, or runs first on `st` when the caller asked for a single stream
  SideStream* side = nullptr;
  if (has_shared && !opt.single_stream) side = &side_stream();
  const cudaStream_t sst = side ? side->s : st;
  // With a side stream the activation quant runs as its own launch and the
  // shared expert forks right after it, ahead of the logits; otherwise the
  // logit kernel does the quant on the side.
  const bool early = side != nullptr;
  RouterArgs rl = ra;  // the logit launch's arguments
  if (opt.x_quantized) {
    rl.xq = nullptr;
    rl.xs = nullptr;
    rl.items_sh = nullptr;
  }
  if (early) {
    if (ws.timing) record_timing(ws.timing[4], st);  // the router's time includes the quant
    if (!opt.x_quantized) {
      const int nb = (H + 127) / 128;
      const int grid = std::max(1, std::min((M * nb + kLogitWarps - 1) / kLogitWarps, 1024));
      if ((err = launch_pdl(act_quant_kernel, dim3(grid), dim3(kLogitWarps * 32), 0, st, ra)) !=
          cudaSuccess)
        return err;
    }
    rl.xq = nullptr;
    rl.xs = nullptr;
    rl.items_sh = nullptr;
  } else if ((err = route_logits(rl, c, ws, M, true, st)) != cudaSuccess) {
    return err;
  }
  if (has_shared) {
    if (side) {
      cudaEventRecord(side->fork, st);
      cudaStreamWaitEvent(side->s, side->fork, 0);
    }
    const int nt = nt_bucket(std::min(sh_n, kItemTok));
    const int sh_items = (sh_n + kItemTok - 1) / kItemTok;
    const QAct sact{ws.sh_qy, ws.sh_qys, I, nullptr};
    const size_t so = static_cast<size_t>(sh_t0) * I;  // first shared row
    const size_t sq = static_cast<size_t>(sh_t0) * ((I + 127) / 128);
    // two or more tokens with scratch: the split-K multi-token kernels (the
    // items' one-warp-per-32-rows form leaves most SMs idle at this size)
    bool shared_done = false;
    if (c.shared_kind == kSharedFp8 && opt.mt_part && sh_n >= 2 && sh_n <= kItemTok) {
      Fp8GemvArgs g{};
      g.W[0] = w.sh1; g.S[0] = w.sh1s; g.W[1] = w.sh3; g.S[1] = w.sh3s; g.rows1 = I;
      g.in = H; g.rows = I; g.round_out = 1; g.act = act;
      g.Y[0] = ws.sh_gate; g.Y[1] = ws.sh_up;
      g.items = ws.items_sh; g.n_items = ws.counters + 3; g.max_items = 1;
      Fp8GemvArgs d{};
      d.W[0] = w.sh2; d.S[0] = w.sh2s;
      d.in = I; d.rows = H; d.round_out = 1; d.act = sact;
      d.Y[0] = ws.shared;
      d.items = ws.items_sh; d.n_items = ws.counters + 3; d.max_items = 1;
      if (fp8_gemv_mt_part_floats(g, sh_n) <= opt.mt_part_floats &&
          fp8_gemv_mt_part_floats(d, sh_n) <= opt.mt_part_floats) {
        err = launch_fp8_gemv_mt(g, sh_n, opt.mt_part, sst);
        if (err == cudaSuccess)
          err = launch_swiglu_quant(ws.sh_gate + so, ws.sh_up + so, I, sh_n, nullptr,
                                    c.swiglu_limit, ws.sh_qy + so, ws.sh_qys + sq, nullptr, sst);
        if (err == cudaSuccess) err = launch_fp8_gemv_mt(d, sh_n, opt.mt_part, sst);
        if (err != cudaSuccess && err != cudaErrorNotSupported) return err;
        shared_done = err == cudaSuccess;
      }
    }
    if (shared_done) {
    } else if (c.shared_kind == kSharedFp8) {
      Fp8GemvArgs g{};
      g.W[0] = w.sh1; g.S[0] = w.sh1s; g.W[1] = w.sh3; g.S[1] = w.sh3s;
      g.in = H; g.rows = I; g.round_out = 1; g.act = act;
      g.Y[0] = ws.sh_gate; g.Y[1] = ws.sh_up;
      g.items = ws.items_sh; g.n_items = ws.counters + 3; g.max_items = sh_items;
      g.beside = side != nullptr;
      g.err = opt.err;
      if ((err = launch_fp8_gemv(g, true, nt, sst, opt.map_cache)) != cudaSuccess) return err;
      if ((err = launch_swiglu_quant(ws.sh_gate + so, ws.sh_up + so, I, sh_n, nullptr,
                                     c.swiglu_limit, ws.sh_qy + so, ws.sh_qys + sq, nullptr,
                                     sst)) != cudaSuccess)
        return err;
      Fp8GemvArgs d{};
      d.W[0] = w.sh2; d.S[0] = w.sh2s;
      d.in = I; d.rows = H; d.round_out = 1; d.act = sact;
      d.Y[0] = ws.shared;
      d.items = ws.items_sh; d.n_items = ws.counters + 3; d.max_items = sh_items;
      d.beside = side != nullptr;
      d.err = opt.err;
      if ((err = launch_fp8_gemv(d, false, nt, sst, opt.map_cache)) != cudaSuccess) return err;
    } else {
      Fp4GemvArgs g{};
      g.W[0] = w.sh1; g.S[0] = w.sh1s; g.W[1] = w.sh3; g.S[1] = w.sh3s;
      g.in = H; g.rows = I; g.act = act;
      g.Y[0] = ws.sh_gate; g.Y[1] = ws.sh_up;
      g.items = ws.items_sh; g.n_items = ws.counters + 3; g.max_items = sh_items; g.err = opt.err;
      if ((err = launch_fp4_gemv(g, true, nt, sst, opt.map_cache)) != cudaSuccess) return err;
      if ((err = launch_swiglu_quant(ws.sh_gate + so, ws.sh_up + so, I, sh_n, nullptr,
                                     c.swiglu_limit, ws.sh_qy + so, ws.sh_qys + sq, nullptr,
                                     sst)) != cudaSuccess)
        return err;
      Fp4GemvArgs d{};
      d.W[0] = w.sh2; d.S[0] = w.sh2s;
      d.in = I; d.rows = H; d.act = sact;
      d.Y[0] = ws.shared;
      d.items = ws.items_sh; d.n_items = ws.counters + 3; d.max_items = sh_items; d.err = opt.err;
      if ((err = launch_fp4_gemv(d, false, nt, sst, opt.map_cache)) != cudaSuccess) return err;
    }
    if (side) cudaEventRecord(side->join, side->s);
  }
  if (early && (err = route_logits(rl, c, ws, M, true, st, false)) != cudaSuccess) return err;

  // router launch 2: selection and the routed expert plan (overlaps the
  // shared expert on the side stream)
  if ((err = route_select(ra, c, ws, M, true, st)) != cudaSuccess) return err;

  // single-token items on the one-token kernel; items of two or more routes
  // (only possible when M >= 2) on the kernel for their token count
  const int nt = nt_bucket(std::min(M, kItemTok));
  const int R_multi = R / 2;  // each multi item holds at least two routes
  const size_t w13 = static_cast<size_t>(I) * (H / 2), s13 = static_cast<size_t>(I) * (H / 32);
  const size_t w2 = static_cast<size_t>(H) * (I / 2), s2 = static_cast<size_t>(H) * (I / 32);
  Fp4GemvArgs gu{};
  gu.W[0] = w.w1; gu.S[0] = w.s1; gu.W[1] = w.w3; gu.S[1] = w.s3;
  gu.w_stride = w13; gu.s_stride = s13;
  gu.in = H; gu.rows = I; gu.act = act;
  gu.Y[0] = ws.gate; gu.Y[1] = ws.up;
  gu.items = ws.items_gu1; gu.n_items = ws.counters + 4; gu.max_items = R; gu.n_mats = n_local;
  gu.err = opt.err;
  if (ws.timing) record_timing(ws.timing[0], st);
  if ((err = launch_fp4_gemv(gu, true, 1, st, opt.map_cache)) != cudaSuccess) return err;
  if (M >= 2) {
    Fp4GemvArgs gm = gu;
    gm.items = ws.items_gu; gm.n_items = ws.counters; gm.max_items = R_multi;
    if ((err = launch_fp4_gemv(gm, true, nt, st, opt.map_cache)) != cudaSuccess) return err;
  }
  if (ws.timing) record_timing(ws.timing[1], st);
  if ((err = launch_swiglu_quant(ws.gate, ws.up, I, R, ws.wt, c.swiglu_limit, ws.qy, ws.qys,
                                 nullptr, st)) != cudaSuccess)
    return err;
  Fp4GemvArgs dn{};
  dn.W[0] = w.w2; dn.S[0] = w.s2;
  dn.w_stride = w2; dn.s_stride = s2;
  dn.in = I; dn.rows = H; dn.act = QAct{ws.qy, ws.qys, I, nullptr};
  dn.Y[0] = ws.routed;
  dn.items = ws.items_dn1; dn.n_items = ws.counters + 4; dn.max_items = R; dn.n_mats = n_local;
  dn.err = opt.err;
  if (ws.timing) record_timing(ws.timing[2], st);
  if ((err = launch_fp4_gemv(dn, false, 1, st, opt.map_cache)) != cudaSuccess) return err;
  if (M >= 2) {
    Fp4GemvArgs dm = dn;
    dm.items = ws.items_dn; dm.n_items = ws.counters; dm.max_items = R_multi;
    if ((err = launch_fp4_gemv(dm, false, nt, st, opt.map_cache)) != cudaSuccess) return err;
  }
  if (ws.timing) record_timing(ws.timing[3], st);

  if (side) cudaStreamWaitEvent(st, side->join, 0);
  if (opt.join) cudaStreamWaitEvent(st, opt.join, 0);
  return cudaGetLastError();
}

cudaError_t router_scores(const float* z, float* s, int n, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  router_scores_kernel<<<(n + 255) / 256, 256, 0, st>>>(z, s, n);
  return cudaGetLastError();
}

cudaError_t moe_combine(const MoeConfig& c, const MoeWorkspace& ws, int M, float* out,
                        bool has_shared, cudaStream_t st) {
  if (M <= 0) return cudaSuccess;
  const int H = c.hidden, K = c.topk;
  const size_t n = static_cast<size_t>(M) * H;
  const int grid = static_cast<int>(std::min<size_t>((n + 255) / 256, 2048));
  return launch_pdl(moe_combine_kernel, dim3(grid), dim3(256), 0, st,
                    static_cast<const float*>(ws.routed),
                    static_cast<const float*>(has_shared ? ws.shared : nullptr),
                    static_cast<const int*>(ws.idx), M, K, H, out);
}

cudaError_t moe_forward(const MoeConfig& c, const MoeWeights& w, const MoeWorkspace& ws,
                        const float* x, const int* token_ids, int M, float* out,
                        cudaStream_t st, const MoeExecOptions& opt) {
  cudaError_t err = moe_forward_local(c, w, ws, x, token_ids, M, st, opt);
  if (err != cudaSuccess) return err;
  return moe_combine(c, ws, M, out, c.shared_kind != kSharedNone && w.sh1 != nullptr, st);
}

}  // namespace dsv4
