// dsv4_common.cuh - device-side numeric codecs shared by every kernel.
//
// The reference engine's numerical contract (BF16 at module boundaries, FP32
// accumulation, explicit fmaf chains) is restated here with integer/bit
// operations so that each decode and rounding is bit-identical to the
// reference's scalar C code (src/dsv4/dsv4_ops.c:35-120). No fast-math: the
// library is compiled without --use_fast_math, so fmaf/mul/add/div/sqrt are
// IEEE round-to-nearest with denormals preserved.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_fp16.h>

namespace dsv4 {

constexpr int kFp8Block = 128;  // FP8 weight/activation block (dsv4_internal.h:28)
constexpr int kFp4Group = 32;   // FP4 scale group (dsv4_internal.h:29)
constexpr int kMaxTopk = 32;    // DSV4_MAX_TOPK (dsv4.h:54)
constexpr int kMaxBatch = kMaxTopk + 1;  // batch GEMV limit (dsv4_model.c:316)

// f32 -> bf16 -> f32, round to nearest even by the carry trick
// (src/dsv4/dsv4_ops.c:35 + dsv4_internal.h:254).
__device__ __forceinline__ float bf16_round(float f) {
  uint32_t u = __float_as_uint(f);
  u += 0x7FFFu + ((u >> 16) & 1u);
  return __uint_as_float(u & 0xFFFF0000u);
}

// expf / log1pf evaluated in double precision and rounded once to fp32
// (correctly rounded except in the rarest hard cases). The host engine's
// libm is not correctly rounded either, so neither form matches it on every
// input; the once-rounded form is the closer one: an exhaustive comparison
// with glibc 2.39 over every fp32 z in [-104, 89] disagrees on 7.6e-5 of
// the inputs for expf, 3.5e-3 for log1pf and 7.6e-3 for
// sqrtf(log1pf(expf(z))), each by one ulp.
__device__ __forceinline__ float expf_r1(float x) { return static_cast<float>(exp(static_cast<double>(x))); }
__device__ __forceinline__ float log1pf_r1(float x) {
  return static_cast<float>(log1p(static_cast<double>(x)));
}

__device__ __forceinline__ float bf16_widen(uint16_t h) {
  return __uint_as_float(static_cast<uint32_t>(h) << 16);
}

// E8M0 scale: 2^(code-127); code 255 is NaN (src/dsv4/dsv4_ops.c:63). Code 0
// is the subnormal 2^-127.
__device__ __forceinline__ float e8m0_decode(uint32_t code) {
  if (code == 255u) return __uint_as_float(0x7FC00000u);
  if (code == 0u) return __uint_as_float(0x00400000u);
  return __uint_as_float(code << 23);
}

// E4M3 (OCP e4m3fn) -> f32, exact (src/dsv4/dsv4_ops.c:47).
__device__ __forceinline__ float e4m3_decode(uint32_t code) {
  const uint32_t sign = (code & 0x80u) << 24;
  const uint32_t mag = code & 0x7Fu;
  float v;
  if (mag == 0x7Fu) {
    v = __uint_as_float(0x7FC00000u);
  } else if (mag < 8u) {
    v = static_cast<float>(mag) * (1.0f / 512.0f);
  } else {
    v = __uint_as_float((mag << 20) + (120u << 23));
  }
  return __uint_as_float(__float_as_uint(v) | sign);
}

// One E2M1 nibble -> f32 (bit 3 is the sign; magnitudes 0,.5,1,1.5,2,3,4,6).
__device__ __forceinline__ float e2m1_decode(uint32_t nib) {
  // magnitude bits m (3 bits) placed as a tiny float and scaled by 2^126:
  // m<2 gives the subnormal 0 / 0.5, m>=2 gives 2^(e-1)*(1+m0/2).
  const float mag = __uint_as_float((nib & 7u) << 22) * 8.5070592e37f;  // 2^126
  return (nib & 8u) ? -mag : mag;
}

// Two packed E2M1 nibbles (low nibble first) -> f16x2, exact.
__device__ __forceinline__ uint32_t e2m1x2_to_f16x2(uint32_t byte) {
  uint32_t out;
  asm("{ .reg .b8 t, u; .reg .b16 h; cvt.u16.u32 h, %1; mov.b16 {t, u}, h;"
      " cvt.rn.f16x2.e2m1x2 %0, t; }"
      : "=r"(out) : "r"(byte));
  return out;
}

// Two packed E4M3 codes (low byte first) -> f16x2, exact.
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint32_t two) {
  uint32_t out;
  asm("{ .reg .b16 h; cvt.u16.u32 h, %1; cvt.rn.f16x2.e4m3x2 %0, h; }"
      : "=r"(out) : "r"(two));
  return out;
}

// acc = fma(a, b, acc) with a, b f16 halves widened exactly to f32; one
// rounding, i.e. identical to fmaf((float)a, (float)b, acc).
// Sum over routes k = 0..topk-1 of vals[k * stride] for the routes with
// ids[k] >= 0, added in route order (the reference's combine order,
// src/dsv4/dsv4_model.c:6795-6805); eight routes' loads are issued together
// so their latencies overlap. Every vals[k * stride] must be readable.
__device__ __forceinline__ float sum_routes(const int* ids, const float* vals, size_t stride,
                                            int topk) {
  float acc = 0.0f;
  for (int k0 = 0; k0 < topk; k0 += 8) {
    int id[8];
    float v[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      id[k] = -1;
      v[k] = 0.0f;
      if (k0 + k < topk) {
        id[k] = ids[k0 + k];
        v[k] = vals[static_cast<size_t>(k0 + k) * stride];
      }
    }
#pragma unroll
    for (int k = 0; k < 8; ++k)
      if (id[k] >= 0) acc += v[k];
  }
  return acc;
}

__device__ __forceinline__ float fma_h_lo(uint32_t a2, uint32_t b2, float acc) {
  asm("{ .reg .b16 al, ah, bl, bh; mov.b32 {al, ah}, %1; mov.b32 {bl, bh}, %2;"
      " fma.rn.f32.f16 %0, al, bl, %0; }"
      : "+f"(acc) : "r"(a2), "r"(b2));
  return acc;
}
__device__ __forceinline__ float fma_h_hi(uint32_t a2, uint32_t b2, float acc) {
  asm("{ .reg .b16 al, ah, bl, bh; mov.b32 {al, ah}, %1; mov.b32 {bl, bh}, %2;"
      " fma.rn.f32.f16 %0, ah, bh, %0; }"
      : "+f"(acc) : "r"(a2), "r"(b2));
  return acc;
}

// 32-byte read-only global load (sm_100 256-bit LDG).
struct alignas(32) U8x32 {
  uint32_t w[8];
};
__device__ __forceinline__ U8x32 ldg32(const void* p) {
  U8x32 r;
  asm volatile("ld.global.nc.L1::no_allocate.v8.u32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r.w[0]), "=r"(r.w[1]), "=r"(r.w[2]), "=r"(r.w[3]),
                 "=r"(r.w[4]), "=r"(r.w[5]), "=r"(r.w[6]), "=r"(r.w[7])
               : "l"(p));
  return r;
}

// 32-byte global load that may stay in L1 (activations every lane reads).
__device__ __forceinline__ U8x32 ldg32_l1(const void* p) {
  U8x32 r;
  asm volatile("ld.global.nc.v8.u32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r.w[0]), "=r"(r.w[1]), "=r"(r.w[2]), "=r"(r.w[3]),
                 "=r"(r.w[4]), "=r"(r.w[5]), "=r"(r.w[6]), "=r"(r.w[7])
               : "l"(p));
  return r;
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

// ceil(log2(amax/448)) power-of-two activation scale with the 1e-4 amax
// floor (src/dsv4/dsv4_model.c:5591-5596); returns 2^e.
__device__ __forceinline__ float pow2_scale_448(float amax) {
  if (amax < 1e-4f) amax = 1e-4f;
  const float r = amax * (1.0f / 448.0f);
  const uint32_t u = __float_as_uint(r);
  // r is a normal positive float here (r >= 2.2e-7).
  int e = static_cast<int>((u >> 23) & 0xFFu) - 126;  // frexp exponent
  if ((u & 0x7FFFFFu) == 0u) e -= 1;                   // exact power of two
  return __uint_as_float(static_cast<uint32_t>(e + 127) << 23);
}

// Round to the nearest E4M3 grid value, restating dsv4_round_e4m3
// (src/dsv4/dsv4_ops.c:81-109) exactly: RNE on the 3-bit mantissa for the
// normal range, RNE on the 2^-9 grid below it, and the 448 overflow rule.
__device__ __forceinline__ float round_half_even(float x) {
  const float lo = floorf(x);
  const float frac = x - lo;
  if (frac > 0.5f) return lo + 1.0f;
  if (frac < 0.5f) return lo;
  return (fmodf(lo, 2.0f) == 0.0f) ? lo : lo + 1.0f;
}
__device__ __forceinline__ float round_e4m3(float v) {
  if (v == 0.0f) return 0.0f;
  const float av = fabsf(v);
  const float sgn = v < 0.0f ? -1.0f : 1.0f;
  int e;
  const float m = frexpf(av, &e);
  if (e >= -5) {
    float mr = round_half_even(m * 16.0f) / 16.0f;
    if (mr >= 1.0f) { mr = 0.5f; e++; }
    if (e - 1 > 8) return sgn * 448.0f;
    return sgn * mr * ldexpf(1.0f, e);
  }
  return sgn * (round_half_even(av * 512.0f) / 512.0f);
}

// Round to the nearest E4M3 value (|q| <= 448, finite; callers clamp) and
// return it as an f16 (exact). The hardware conversion is round-to-nearest-
// even on the 3-bit mantissa and on the 2^-9 subnormal grid, which is what
// dsv4_round_e4m3 (src/dsv4/dsv4_ops.c:92-109) computes for this range; the
// reference maps an exact zero (either sign) to +0, so do we.
__device__ __forceinline__ __half e4m3_round_f16(float q) {
  uint32_t h2;
  asm("{ .reg .b16 t; cvt.rn.satfinite.e4m3x2.f32 t, %1, %1; cvt.rn.f16x2.e4m3x2 %0, t; }"
      : "=r"(h2) : "f"(q));
  const unsigned short h = static_cast<unsigned short>(h2 & 0xFFFFu);
  return __ushort_as_half(q == 0.0f ? static_cast<unsigned short>(0) : h);
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

}  // namespace dsv4

