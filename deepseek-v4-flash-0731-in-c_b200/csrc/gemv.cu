// gemv.cu - exact-order GEMV kernels for the decode hot path.
//
// Every kernel reproduces the reference's accumulation order bit for bit:
//   FP4 (dsv4_gemv_fp4_q, src/dsv4/dsv4_model.c:1055-1073): per row, each
//     32-column group is a sequential fmaf chain (low nibble first); the
//     group partials enter acc = fmaf(partial, qscale[c/128]*ws, acc) in
//     column order; a NaN E8M0 scale skips its group; BF16 output.
//   FP8 (dsv4_gemv_fp8_q, :657-672): the same with 128-column blocks and
//     [128x128] block scales; optional BF16 output.
//   BF16 (dsv4_gemv_bf16, :299-302): one fmaf chain over all columns.
//
// Layout of the work: one output row is owned by LPR lanes of a warp (LPR in
// {1,2,4}); each lane streams 32-byte chunks of its row with 256-bit loads
// (every DRAM sector is read exactly once), computes the group partials of
// its chunks, and the row's leader lane folds the partials into the
// accumulator in column order via warp shuffles. Products of an E2M1 or
// E4M3 weight with an E4M3-grid activation are exact in f16 operands, so
// the multiply-add uses the sm_100 mixed fma.rn.f32.f16 (one rounding, same
// as fmaf on the widened values). Activations are read through L1 (every
// lane of a warp reads the same few lines); weights bypass L1.
#include <algorithm>

#include "dsv4_common.cuh"
#include "gemv.cuh"

namespace dsv4 {

namespace {

__device__ __forceinline__ int load_n_items(const int* p, int max_items) {
  const int n = *p;
  return n < max_items ? n : max_items;
}

__device__ __forceinline__ U8x32 ldg32_l1(const void* p) {
  U8x32 r;
  asm volatile("ld.global.nc.v8.u32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r.w[0]), "=r"(r.w[1]), "=r"(r.w[2]), "=r"(r.w[3]),
                 "=r"(r.w[4]), "=r"(r.w[5]), "=r"(r.w[6]), "=r"(r.w[7])
               : "l"(p));
  return r;
}

// Sequential 32-column FP4 partial: 16 packed bytes (4 words) of weights
// against 16 f16x2 activation words, columns in order.
__device__ __forceinline__ float fp4_partial16(const uint32_t* w4, const uint32_t* x16) {
  float p = 0.0f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint32_t h0, h1, h2, h3;
    asm("{ .reg .b8 b0, b1, b2, b3; mov.b32 {b0, b1, b2, b3}, %4;"
        " cvt.rn.f16x2.e2m1x2 %0, b0; cvt.rn.f16x2.e2m1x2 %1, b1;"
        " cvt.rn.f16x2.e2m1x2 %2, b2; cvt.rn.f16x2.e2m1x2 %3, b3; }"
        : "=r"(h0), "=r"(h1), "=r"(h2), "=r"(h3) : "r"(w4[i]));
    p = fma_h_lo(h0, x16[4 * i + 0], p);
    p = fma_h_hi(h0, x16[4 * i + 0], p);
    p = fma_h_lo(h1, x16[4 * i + 1], p);
    p = fma_h_hi(h1, x16[4 * i + 1], p);
    p = fma_h_lo(h2, x16[4 * i + 2], p);
    p = fma_h_hi(h2, x16[4 * i + 2], p);
    p = fma_h_lo(h3, x16[4 * i + 3], p);
    p = fma_h_hi(h3, x16[4 * i + 3], p);
  }
  return p;
}

// Sequential FP8 partial over 32 columns (8 words of codes, 16 f16x2 words).
__device__ __forceinline__ float fp8_chain32(const uint32_t* w8, const uint32_t* x16, float p) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    uint32_t h0, h1;
    asm("{ .reg .b16 lo, hi; mov.b32 {lo, hi}, %2; cvt.rn.f16x2.e4m3x2 %0, lo;"
        " cvt.rn.f16x2.e4m3x2 %1, hi; }"
        : "=r"(h0), "=r"(h1) : "r"(w8[i]));
    p = fma_h_lo(h0, x16[2 * i + 0], p);
    p = fma_h_hi(h0, x16[2 * i + 0], p);
    p = fma_h_lo(h1, x16[2 * i + 1], p);
    p = fma_h_hi(h1, x16[2 * i + 1], p);
  }
  return p;
}

// ---------------------------------------------------------------- FP4 ----
// Grid: one warp per (item, block of 32/LPR rows). NT = max tokens per item.
template <int LPR, int NT, bool PAIR>
__global__ void __launch_bounds__(128) fp4_gemv_kernel(const Fp4GemvArgs a) {
  constexpr int RPW = 32 / LPR;
  const int lane = threadIdx.x & 31;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int rblocks = (a.rows + RPW - 1) / RPW;
  const int item_idx = gw / rblocks;
  if (item_idx >= load_n_items(a.n_items, a.max_items)) return;
  const GemvItem& it = a.items[item_idx];
  const int ntok = it.ntok;
  const int sub = lane % LPR;
  const int row = (gw % rblocks) * RPW + lane / LPR;
  const bool row_ok = row < a.rows;
  const int rowc = row_ok ? row : a.rows - 1;
  const int G = a.in >> 5;                  // groups per row
  const int NP = G / (2 * LPR);             // 32-byte chunks per lane
  const size_t rb = static_cast<size_t>(a.in) >> 1;
  const uint8_t* wp0 = a.W[0] + it.mat * a.w_stride + rowc * rb + sub * 32;
  const uint8_t* sp0 = a.S[0] + it.mat * a.s_stride + static_cast<size_t>(rowc) * G + sub * 2;
  const uint8_t* wp1 = nullptr;
  const uint8_t* sp1 = nullptr;
  if (PAIR) {
    wp1 = a.W[1] + it.mat * a.w_stride + rowc * rb + sub * 32;
    sp1 = a.S[1] + it.mat * a.s_stride + static_cast<size_t>(rowc) * G + sub * 2;
  }
  const __half* xr[NT];
  const float* xsr[NT];
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    const int xi = t < ntok ? it.tok[t].x : it.tok[0].x;
    xr[t] = a.act.x + static_cast<size_t>(xi) * a.act.ld + sub * 64;
    xsr[t] = a.act.s + static_cast<size_t>(xi) * ((a.act.ld + 127) >> 7);
  }
  float acc0[NT], acc1[NT];
#pragma unroll
  for (int t = 0; t < NT; ++t) { acc0[t] = 0.0f; acc1[t] = 0.0f; }

  constexpr int PF = PAIR ? 2 : 4;
  U8x32 buf0[PF], buf1[PF];
#pragma unroll
  for (int j = 0; j < PF; ++j) {
    if (j < NP) {
      buf0[j] = ldg32(wp0 + static_cast<size_t>(j) * LPR * 32);
      if (PAIR) buf1[j] = ldg32(wp1 + static_cast<size_t>(j) * LPR * 32);
    }
  }
  for (int p0 = 0; p0 < NP; p0 += PF) {
#pragma unroll
    for (int j = 0; j < PF; ++j) {
      const int p = p0 + j;
      if (p < NP) {
        const U8x32 cw0 = buf0[j];
        U8x32 cw1;
        if (PAIR) cw1 = buf1[j];
        if (p + PF < NP) {
          buf0[j] = ldg32(wp0 + static_cast<size_t>(p + PF) * LPR * 32);
          if (PAIR) buf1[j] = ldg32(wp1 + static_cast<size_t>(p + PF) * LPR * 32);
        }
        const int col0 = (p * LPR + sub) * 64;  // first column of this chunk
        const uint32_t sc0 = *reinterpret_cast<const uint16_t*>(sp0 + p * LPR * 2);
        const float wsa0 = e8m0_decode(sc0 & 0xFFu), wsb0 = e8m0_decode(sc0 >> 8);
        float wsa1 = 0.f, wsb1 = 0.f;
        if (PAIR) {
          const uint32_t sc1 = *reinterpret_cast<const uint16_t*>(sp1 + p * LPR * 2);
          wsa1 = e8m0_decode(sc1 & 0xFFu);
          wsb1 = e8m0_decode(sc1 >> 8);
        }
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          if (t < ntok) {
            uint32_t xw[32];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const U8x32 v = ldg32_l1(xr[t] + static_cast<size_t>(p) * LPR * 64 + q * 16);
#pragma unroll
              for (int k = 0; k < 8; ++k) xw[q * 8 + k] = v.w[k];
            }
            const float qs = xsr[t][col0 >> 7];
            float pa0 = fp4_partial16(&cw0.w[0], &xw[0]);
            float pb0 = fp4_partial16(&cw0.w[4], &xw[16]);
            float sa0 = qs * wsa0, sb0 = qs * wsb0;
            if (isnan(wsa0)) { pa0 = 0.f; sa0 = 0.f; }
            if (isnan(wsb0)) { pb0 = 0.f; sb0 = 0.f; }
            float pa1 = 0.f, pb1 = 0.f, sa1 = 0.f, sb1 = 0.f;
            if (PAIR) {
              pa1 = fp4_partial16(&cw1.w[0], &xw[0]);
              pb1 = fp4_partial16(&cw1.w[4], &xw[16]);
              sa1 = qs * wsa1;
              sb1 = qs * wsb1;
              if (isnan(wsa1)) { pa1 = 0.f; sa1 = 0.f; }
              if (isnan(wsb1)) { pb1 = 0.f; sb1 = 0.f; }
            }
            if (LPR == 1) {
              acc0[t] = fmaf(pa0, sa0, acc0[t]);
              acc0[t] = fmaf(pb0, sb0, acc0[t]);
              if (PAIR) {
                acc1[t] = fmaf(pa1, sa1, acc1[t]);
                acc1[t] = fmaf(pb1, sb1, acc1[t]);
              }
            } else {
              const int base = lane - sub;
#pragma unroll
              for (int s = 0; s < LPR; ++s) {
                const float qa = __shfl_sync(0xffffffffu, pa0, base + s);
                const float qsa = __shfl_sync(0xffffffffu, sa0, base + s);
                const float qb = __shfl_sync(0xffffffffu, pb0, base + s);
                const float qsb = __shfl_sync(0xffffffffu, sb0, base + s);
                acc0[t] = fmaf(qa, qsa, acc0[t]);
                acc0[t] = fmaf(qb, qsb, acc0[t]);
                if (PAIR) {
                  const float ra = __shfl_sync(0xffffffffu, pa1, base + s);
                  const float rsa = __shfl_sync(0xffffffffu, sa1, base + s);
                  const float rb2 = __shfl_sync(0xffffffffu, pb1, base + s);
                  const float rsb = __shfl_sync(0xffffffffu, sb1, base + s);
                  acc1[t] = fmaf(ra, rsa, acc1[t]);
                  acc1[t] = fmaf(rb2, rsb, acc1[t]);
                }
              }
            }
          }
        }
      }
    }
  }
  if (sub == 0 && row_ok) {
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      if (t < ntok) {
        const size_t yo = static_cast<size_t>(it.tok[t].y) * a.rows + row;
        a.Y[0][yo] = bf16_round(acc0[t]);
        if (PAIR) a.Y[1][yo] = bf16_round(acc1[t]);
      }
    }
  }
}

// Scalar fallback for shapes the vector kernel does not cover (in not a
// multiple of 64, unaligned pointers): one thread per (item token, row).
__global__ void fp4_gemv_scalar_kernel(const Fp4GemvArgs a, int pair_idx) {
  const int n_items = load_n_items(a.n_items, a.max_items);
  const long long total = static_cast<long long>(n_items) * kItemTok * a.rows;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int row = static_cast<int>(i % a.rows);
    const int t = static_cast<int>((i / a.rows) % kItemTok);
    const int item = static_cast<int>(i / (static_cast<long long>(a.rows) * kItemTok));
    const GemvItem& it = a.items[item];
    if (t >= it.ntok) continue;
    const int pc = (a.in + 1) / 2, gc = (a.in + 31) / 32;
    const uint8_t* w = a.W[pair_idx] + it.mat * a.w_stride + static_cast<size_t>(row) * pc;
    const uint8_t* s = a.S[pair_idx] + it.mat * a.s_stride + static_cast<size_t>(row) * gc;
    const __half* x = a.act.x + static_cast<size_t>(it.tok[t].x) * a.act.ld;
    const float* xs = a.act.s + static_cast<size_t>(it.tok[t].x) * ((a.act.ld + 127) >> 7);
    float acc = 0.0f;
    for (int g = 0; g < gc; ++g) {
      const int c0 = g * 32, c1 = min(c0 + 32, a.in);
      float part = 0.0f;
      for (int c = c0; c < c1; ++c) {
        const uint32_t b = w[c >> 1];
        const uint32_t nib = (c & 1) ? (b >> 4) : (b & 15u);
        const float xv = a.act.x32 ? a.act.x32[static_cast<size_t>(it.tok[t].x) * a.act.ld + c]
                                   : __half2float(x[c]);
        part = fmaf(e2m1_decode(nib), xv, part);
      }
      const float ws = e8m0_decode(s[g]);
      if (!isnan(ws)) acc = fmaf(part, xs[c0 / 128] * ws, acc);
    }
    a.Y[pair_idx][static_cast<size_t>(it.tok[t].y) * a.rows + row] = bf16_round(acc);
  }
}

// ---------------------------------------------------------------- FP8 ----
template <int LPR, int NT, bool PAIR>
__global__ void __launch_bounds__(128) fp8_gemv_kernel(const Fp8GemvArgs a) {
  constexpr int RPW = 32 / LPR;
  const int lane = threadIdx.x & 31;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int rblocks = (a.rows + RPW - 1) / RPW;
  const int item_idx = gw / rblocks;
  if (item_idx >= load_n_items(a.n_items, a.max_items)) return;
  const GemvItem& it = a.items[item_idx];
  const int ntok = it.ntok;
  const int sub = lane % LPR;
  const int row = (gw % rblocks) * RPW + lane / LPR;
  const bool row_ok = row < a.rows;
  const int rowc = row_ok ? row : a.rows - 1;
  const int CB = a.in >> 7;           // 128-column blocks per row
  const int NB = CB / LPR;            // blocks per lane
  const uint8_t* wp0 = a.W[0] + it.mat * a.w_stride + static_cast<size_t>(rowc) * a.in + sub * 128;
  const uint8_t* sp0 = a.S[0] + it.mat * a.s_stride + static_cast<size_t>(rowc >> 7) * CB + sub;
  const uint8_t* wp1 = nullptr;
  const uint8_t* sp1 = nullptr;
  if (PAIR) {
    wp1 = a.W[1] + it.mat * a.w_stride + static_cast<size_t>(rowc) * a.in + sub * 128;
    sp1 = a.S[1] + it.mat * a.s_stride + static_cast<size_t>(rowc >> 7) * CB + sub;
  }
  const __half* xr[NT];
  const float* xsr[NT];
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    const int xi = t < ntok ? it.tok[t].x : it.tok[0].x;
    xr[t] = a.act.x + static_cast<size_t>(xi) * a.act.ld + sub * 128;
    xsr[t] = a.act.s + static_cast<size_t>(xi) * ((a.act.ld + 127) >> 7) + sub;
  }
  float acc0[NT], acc1[NT];
#pragma unroll
  for (int t = 0; t < NT; ++t) { acc0[t] = 0.f; acc1[t] = 0.f; }

  for (int b = 0; b < NB; ++b) {
    // the lane's 128-byte block: 4 x 32-byte loads, issued together
    U8x32 w0[4], w1[4];
    const size_t off = static_cast<size_t>(b) * LPR * 128;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      w0[q] = ldg32(wp0 + off + q * 32);
      if (PAIR) w1[q] = ldg32(wp1 + off + q * 32);
    }
    const float ws0 = e8m0_decode(sp0[b * LPR]);
    const float ws1 = PAIR ? e8m0_decode(sp1[b * LPR]) : 0.f;
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      if (t < ntok) {
        float p0 = 0.f, p1 = 0.f;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint32_t xw[16];
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const U8x32 v = ldg32_l1(xr[t] + off + q * 32 + h * 16);
#pragma unroll
            for (int k = 0; k < 8; ++k) xw[h * 8 + k] = v.w[k];
          }
          p0 = fp8_chain32(w0[q].w, xw, p0);
          if (PAIR) p1 = fp8_chain32(w1[q].w, xw, p1);
        }
        const float qs = xsr[t][b * LPR];
        float s0 = qs * ws0, s1 = qs * ws1;
        if (isnan(ws0)) { p0 = 0.f; s0 = 0.f; }
        if (PAIR && isnan(ws1)) { p1 = 0.f; s1 = 0.f; }
        if (LPR == 1) {
          acc0[t] = fmaf(p0, s0, acc0[t]);
          if (PAIR) acc1[t] = fmaf(p1, s1, acc1[t]);
        } else {
          const int base = lane - sub;
#pragma unroll
          for (int s = 0; s < LPR; ++s) {
            const float q0 = __shfl_sync(0xffffffffu, p0, base + s);
            const float r0 = __shfl_sync(0xffffffffu, s0, base + s);
            acc0[t] = fmaf(q0, r0, acc0[t]);
            if (PAIR) {
              const float q1 = __shfl_sync(0xffffffffu, p1, base + s);
              const float r1 = __shfl_sync(0xffffffffu, s1, base + s);
              acc1[t] = fmaf(q1, r1, acc1[t]);
            }
          }
        }
      }
    }
  }
  if (sub == 0 && row_ok) {
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      if (t < ntok) {
        const size_t yo = static_cast<size_t>(it.tok[t].y) * a.rows + row;
        a.Y[0][yo] = a.round_out ? bf16_round(acc0[t]) : acc0[t];
        if (PAIR) a.Y[1][yo] = a.round_out ? bf16_round(acc1[t]) : acc1[t];
      }
    }
  }
}

__global__ void fp8_gemv_scalar_kernel(const Fp8GemvArgs a, int pair_idx) {
  const int n_items = load_n_items(a.n_items, a.max_items);
  const long long total = static_cast<long long>(n_items) * kItemTok * a.rows;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int row = static_cast<int>(i % a.rows);
    const int t = static_cast<int>((i / a.rows) % kItemTok);
    const int item = static_cast<int>(i / (static_cast<long long>(a.rows) * kItemTok));
    const GemvItem& it = a.items[item];
    if (t >= it.ntok) continue;
    const int cb = (a.in + 127) / 128;
    const uint8_t* w = a.W[pair_idx] + it.mat * a.w_stride + static_cast<size_t>(row) * a.in;
    const uint8_t* s = a.S[pair_idx] + it.mat * a.s_stride + static_cast<size_t>(row / 128) * cb;
    const __half* x = a.act.x + static_cast<size_t>(it.tok[t].x) * a.act.ld;
    const float* xs = a.act.s + static_cast<size_t>(it.tok[t].x) * ((a.act.ld + 127) >> 7);
    float acc = 0.0f;
    for (int b = 0; b < cb; ++b) {
      const int c1 = min((b + 1) * 128, a.in);
      float part = 0.0f;
      for (int c = b * 128; c < c1; ++c) {
        const float xv = a.act.x32 ? a.act.x32[static_cast<size_t>(it.tok[t].x) * a.act.ld + c]
                                   : __half2float(x[c]);
        part = fmaf(e4m3_decode(w[c]), xv, part);
      }
      const float ws = e8m0_decode(s[b]);
      if (!isnan(ws)) acc = fmaf(part, xs[b] * ws, acc);
    }
    a.Y[pair_idx][static_cast<size_t>(it.tok[t].y) * a.rows + row] =
        a.round_out ? bf16_round(acc) : acc;
  }
}

// --------------------------------------------------------------- BF16 ----
// One lane per row, one fmaf chain over all columns (no partial structure to
// split, so LPR is 1). 32-byte loads carry 16 columns.
template <int NT>
__global__ void __launch_bounds__(128) bf16_gemv_kernel(const Bf16GemvArgs a) {
  const int lane = threadIdx.x & 31;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int rblocks = (a.rows + 31) / 32;
  const int item_idx = gw / rblocks;
  if (item_idx >= load_n_items(a.n_items, a.max_items)) return;
  const GemvItem& it = a.items[item_idx];
  const int ntok = it.ntok;
  const int row = (gw % rblocks) * 32 + lane;
  const bool row_ok = row < a.rows;
  const int rowc = row_ok ? row : a.rows - 1;
  const uint16_t* wp = a.W + static_cast<size_t>(rowc) * a.in;
  const float* xr[NT];
#pragma unroll
  for (int t = 0; t < NT; ++t)
    xr[t] = a.x + static_cast<size_t>(t < ntok ? it.tok[t].x : it.tok[0].x) * a.ldx;
  float acc[NT];
#pragma unroll
  for (int t = 0; t < NT; ++t) acc[t] = 0.f;
  const int NC = a.in >> 4;  // 16-column chunks
  constexpr int PF = 4;
  U8x32 buf[PF];
#pragma unroll
  for (int j = 0; j < PF; ++j)
    if (j < NC) buf[j] = ldg32(wp + j * 16);
  for (int c0 = 0; c0 < NC; c0 += PF) {
#pragma unroll
    for (int j = 0; j < PF; ++j) {
      const int c = c0 + j;
      if (c < NC) {
        const U8x32 w = buf[j];
        if (c + PF < NC) buf[j] = ldg32(wp + (c + PF) * 16);
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          if (t < ntok) {
            const U8x32 x0 = ldg32_l1(xr[t] + c * 16);
            const U8x32 x1 = ldg32_l1(xr[t] + c * 16 + 8);
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              const float xa = __uint_as_float(k < 4 ? x0.w[2 * k] : x1.w[2 * k - 8]);
              const float xb = __uint_as_float(k < 4 ? x0.w[2 * k + 1] : x1.w[2 * k - 7]);
              acc[t] = fmaf(__uint_as_float(w.w[k] << 16), xa, acc[t]);
              acc[t] = fmaf(__uint_as_float(w.w[k] & 0xFFFF0000u), xb, acc[t]);
            }
          }
        }
      }
    }
  }
  if (row_ok) {
#pragma unroll
    for (int t = 0; t < NT; ++t)
      if (t < ntok) {
        const size_t yo = static_cast<size_t>(it.tok[t].y) * a.rows + row;
        a.Y[yo] = a.round_out ? bf16_round(acc[t]) : acc[t];
      }
  }
}

__global__ void bf16_gemv_scalar_kernel(const Bf16GemvArgs a) {
  const int n_items = load_n_items(a.n_items, a.max_items);
  const long long total = static_cast<long long>(n_items) * kItemTok * a.rows;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int row = static_cast<int>(i % a.rows);
    const int t = static_cast<int>((i / a.rows) % kItemTok);
    const int item = static_cast<int>(i / (static_cast<long long>(a.rows) * kItemTok));
    const GemvItem& it = a.items[item];
    if (t >= it.ntok) continue;
    const uint16_t* w = a.W + static_cast<size_t>(row) * a.in;
    const float* x = a.x + static_cast<size_t>(it.tok[t].x) * a.ldx;
    float acc = 0.0f;
    for (int c = 0; c < a.in; ++c) acc = fmaf(bf16_widen(w[c]), x[c], acc);
    a.Y[static_cast<size_t>(it.tok[t].y) * a.rows + row] = a.round_out ? bf16_round(acc) : acc;
  }
}

// ---------------------------------------------------------- quantisers ----
// One warp per 128-column block: amax, power-of-two scale, E4M3 rounding
// (dsv4_quant_fp8_codes, src/dsv4/dsv4_model.c:5580-5606).
__global__ void quant_fp8_kernel(const float* x, int ldx, int n, int rows, __half* qx,
                                 float* qs, int ld_out, float* qx32) {
  const int lane = threadIdx.x & 31;
  const int nb = (n + 127) / 128;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (gw >= nb * rows) return;
  const int r = gw / nb, b = gw % nb;
  const float* xr = x + static_cast<size_t>(r) * ldx + b * 128;
  const int len = min(128, n - b * 128);
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
  if (lane == 0) qs[static_cast<size_t>(r) * ((ld_out + 127) >> 7) + b] = scale;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int i = lane + 32 * k;
    if (i < len) {
      float q = v[k] * inv;
      q = q > 448.f ? 448.f : (q < -448.f ? -448.f : q);
      const float g = round_e4m3(q);
      if (qx) qx[static_cast<size_t>(r) * ld_out + b * 128 + i] = __float2half_rn(g);
      if (qx32) qx32[static_cast<size_t>(r) * ld_out + b * 128 + i] = g;
    }
  }
}

// Fused SwiGLU + route weight + BF16 + FP8 quant
// (routed_swiglu_quant, src/dsv4/dsv4_model.c:6257-6286).
__global__ void swiglu_quant_kernel(const float* gate, const float* up, int n, int rows,
                                    const float* weight, int limit, __half* qy, float* qs,
                                    float* ybf) {
  const int lane = threadIdx.x & 31;
  const int nb = (n + 127) / 128;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (gw >= nb * rows) return;
  const int r = gw / nb, b = gw % nb;
  const int len = min(128, n - b * 128);
  const float L = static_cast<float>(limit);
  const float w = weight ? weight[r] : 1.0f;
  float v[4];
  float amax = 0.f;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int i = lane + 32 * k;
    v[k] = 0.f;
    if (i < len) {
      const size_t o = static_cast<size_t>(r) * n + b * 128 + i;
      float g = gate[o], u = up[o];
      if (u > L) u = L;
      else if (u < -L) u = -L;
      if (g > L) g = L;
      const float silu = g / (1.0f + expf(-g));
      v[k] = bf16_round(silu * u * w);
      amax = fmaxf(amax, fabsf(v[k]));
    }
  }
  amax = warp_max(amax);
  const float scale = pow2_scale_448(amax);
  const float inv = 1.0f / scale;
  if (lane == 0) qs[static_cast<size_t>(r) * nb + b] = scale;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int i = lane + 32 * k;
    if (i < len) {
      const size_t o = static_cast<size_t>(r) * n + b * 128 + i;
      float q = v[k] * inv;
      q = q > 448.f ? 448.f : (q < -448.f ? -448.f : q);
      qy[o] = __float2half_rn(round_e4m3(q));
      if (ybf) ybf[o] = v[k];
    }
  }
}

__global__ void f32_to_f16_kernel(const float* x, __half* y, size_t n) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x)
    y[i] = __float2half_rn(x[i]);
}

int blocks_for_warps(long long warps) {
  return static_cast<int>((warps * 32 + 127) / 128);
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

template <int LPR, bool PAIR>
cudaError_t fp4_dispatch_nt(const Fp4GemvArgs& a, int nt, cudaStream_t st) {
  const int rblocks = (a.rows + 32 / LPR - 1) / (32 / LPR);
  const int grid = blocks_for_warps(static_cast<long long>(a.max_items) * rblocks);
  if (grid <= 0) return cudaSuccess;
  switch (nt) {
    case 1: fp4_gemv_kernel<LPR, 1, PAIR><<<grid, 128, 0, st>>>(a); break;
    case 2: fp4_gemv_kernel<LPR, 2, PAIR><<<grid, 128, 0, st>>>(a); break;
    case 3:
    case 4: fp4_gemv_kernel<LPR, 4, PAIR><<<grid, 128, 0, st>>>(a); break;
    default: fp4_gemv_kernel<LPR, 8, PAIR><<<grid, 128, 0, st>>>(a); break;
  }
  return cudaGetLastError();
}

template <int LPR, bool PAIR>
cudaError_t fp8_dispatch_nt(const Fp8GemvArgs& a, int nt, cudaStream_t st) {
  const int rblocks = (a.rows + 32 / LPR - 1) / (32 / LPR);
  const int grid = blocks_for_warps(static_cast<long long>(a.max_items) * rblocks);
  if (grid <= 0) return cudaSuccess;
  switch (nt) {
    case 1: fp8_gemv_kernel<LPR, 1, PAIR><<<grid, 128, 0, st>>>(a); break;
    case 2: fp8_gemv_kernel<LPR, 2, PAIR><<<grid, 128, 0, st>>>(a); break;
    case 3:
    case 4: fp8_gemv_kernel<LPR, 4, PAIR><<<grid, 128, 0, st>>>(a); break;
    default: fp8_gemv_kernel<LPR, 8, PAIR><<<grid, 128, 0, st>>>(a); break;
  }
  return cudaGetLastError();
}

int sm_count() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

// Lanes per row: split rows over more lanes when there are too few warps to
// fill the GPU (the item count is an upper bound when it lives on device).
int pick_lpr(long long rows_total, int chunks_per_row) {
  const long long want_warps = 12LL * sm_count();
  int lpr = 1;
  while (lpr < 4 && (rows_total * lpr) / 32 < want_warps && chunks_per_row % (4 * lpr) == 0)
    lpr *= 2;
  return lpr;
}

}  // namespace

cudaError_t launch_fp4_gemv(const Fp4GemvArgs& a, bool pair, int item_tokens, cudaStream_t st) {
  if (a.rows <= 0 || a.max_items <= 0) return cudaSuccess;
  const bool vec_ok = !a.act.x32 && (a.in % 64 == 0) && aligned(a.W[0], 32) && (a.w_stride % 32 == 0) &&
                      (a.s_stride % 2 == 0) && aligned(a.S[0], 2) &&
                      aligned(a.act.x, 32) && (a.act.ld % 128 == 0) &&
                      (!pair || (aligned(a.W[1], 32) && aligned(a.S[1], 2)));
  if (!vec_ok) {
    const long long work = static_cast<long long>(a.max_items) * kItemTok * a.rows;
    const int grid = static_cast<int>(std::min<long long>((work + 255) / 256, 65535));
    for (int p = 0; p < (pair ? 2 : 1); ++p)
      fp4_gemv_scalar_kernel<<<grid, 256, 0, st>>>(a, p);
    return cudaGetLastError();
  }
  const int G = a.in / 32;
  const int lpr = pick_lpr(static_cast<long long>(a.max_items) * a.rows * (pair ? 2 : 1), G);
  if (pair) {
    if (lpr == 4) return fp4_dispatch_nt<4, true>(a, item_tokens, st);
    if (lpr == 2) return fp4_dispatch_nt<2, true>(a, item_tokens, st);
    return fp4_dispatch_nt<1, true>(a, item_tokens, st);
  }
  if (lpr == 4) return fp4_dispatch_nt<4, false>(a, item_tokens, st);
  if (lpr == 2) return fp4_dispatch_nt<2, false>(a, item_tokens, st);
  return fp4_dispatch_nt<1, false>(a, item_tokens, st);
}

cudaError_t launch_fp8_gemv(const Fp8GemvArgs& a, bool pair, int item_tokens, cudaStream_t st) {
  if (a.rows <= 0 || a.max_items <= 0) return cudaSuccess;
  const bool vec_ok = !a.act.x32 && (a.in % 128 == 0) && aligned(a.W[0], 32) && (a.w_stride % 32 == 0) &&
                      aligned(a.act.x, 32) && (a.act.ld % 128 == 0) &&
                      (!pair || aligned(a.W[1], 32));
  if (!vec_ok) {
    const long long work = static_cast<long long>(a.max_items) * kItemTok * a.rows;
    const int grid = static_cast<int>(std::min<long long>((work + 255) / 256, 65535));
    for (int p = 0; p < (pair ? 2 : 1); ++p)
      fp8_gemv_scalar_kernel<<<grid, 256, 0, st>>>(a, p);
    return cudaGetLastError();
  }
  const int CB = a.in / 128;
  int lpr = pick_lpr(static_cast<long long>(a.max_items) * a.rows * (pair ? 2 : 1), 2 * CB);
  while (lpr > 1 && CB % lpr != 0) lpr /= 2;
  if (pair) {
    if (lpr == 4) return fp8_dispatch_nt<4, true>(a, item_tokens, st);
    if (lpr == 2) return fp8_dispatch_nt<2, true>(a, item_tokens, st);
    return fp8_dispatch_nt<1, true>(a, item_tokens, st);
  }
  if (lpr == 4) return fp8_dispatch_nt<4, false>(a, item_tokens, st);
  if (lpr == 2) return fp8_dispatch_nt<2, false>(a, item_tokens, st);
  return fp8_dispatch_nt<1, false>(a, item_tokens, st);
}

cudaError_t launch_bf16_gemv(const Bf16GemvArgs& a, int item_tokens, cudaStream_t st) {
  if (a.rows <= 0 || a.max_items <= 0) return cudaSuccess;
  const bool vec_ok = (a.in % 16 == 0) && aligned(a.W, 32) && aligned(a.x, 32) &&
                      (a.ldx % 8 == 0);
  if (!vec_ok) {
    const long long work = static_cast<long long>(a.max_items) * kItemTok * a.rows;
    const int grid = static_cast<int>(std::min<long long>((work + 255) / 256, 65535));
    bf16_gemv_scalar_kernel<<<grid, 256, 0, st>>>(a);
    return cudaGetLastError();
  }
  const int rblocks = (a.rows + 31) / 32;
  const int grid = blocks_for_warps(static_cast<long long>(a.max_items) * rblocks);
  switch (item_tokens) {
    case 1: bf16_gemv_kernel<1><<<grid, 128, 0, st>>>(a); break;
    case 2: bf16_gemv_kernel<2><<<grid, 128, 0, st>>>(a); break;
    case 3:
    case 4: bf16_gemv_kernel<4><<<grid, 128, 0, st>>>(a); break;
    default: bf16_gemv_kernel<8><<<grid, 128, 0, st>>>(a); break;
  }
  return cudaGetLastError();
}

cudaError_t launch_quant_fp8(const float* x, int ldx, int n, int rows, __half* qx, float* qs,
                             int ld_out, cudaStream_t st) {
  const long long warps = static_cast<long long>(rows) * ((n + 127) / 128);
  if (warps <= 0) return cudaSuccess;
  quant_fp8_kernel<<<blocks_for_warps(warps), 128, 0, st>>>(x, ldx, n, rows, qx, qs, ld_out,
                                                            nullptr);
  return cudaGetLastError();
}

cudaError_t launch_quant_fp8_f32(const float* x, int n, float* qx, float* qs, cudaStream_t st) {
  const long long warps = (n + 127) / 128;
  if (warps <= 0) return cudaSuccess;
  // ld_out = n rounded up to 128 keeps the per-row scale stride consistent.
  const int ld = (n + 127) / 128 * 128;
  quant_fp8_kernel<<<blocks_for_warps(warps), 128, 0, st>>>(x, n, n, 1, nullptr, qs, ld, qx);
  return cudaGetLastError();
}

cudaError_t launch_swiglu_quant(const float* gate, const float* up, int n, int rows,
                                const float* weight, int limit, __half* qy, float* qs,
                                float* y_bf16, cudaStream_t st) {
  const long long warps = static_cast<long long>(rows) * ((n + 127) / 128);
  if (warps <= 0) return cudaSuccess;
  swiglu_quant_kernel<<<blocks_for_warps(warps), 128, 0, st>>>(gate, up, n, rows, weight,
                                                               limit, qy, qs, y_bf16);
  return cudaGetLastError();
}

cudaError_t launch_f32_to_f16(const float* x, __half* y, size_t n, cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  const int grid = static_cast<int>(std::min<size_t>((n + 255) / 256, 4096));
  f32_to_f16_kernel<<<grid, 256, 0, st>>>(x, y, n);
  return cudaGetLastError();
}

}  // namespace dsv4
