// attn.cuh - latent-KV decode attention (sparse_attn) and the FP8 latent cache.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

#ifdef __CUDACC__
#include "dsv4_common.cuh"
#endif

namespace dsv4 {

// Lossless FP8 layout of one cached latent. The reference stores each
// latent as fp32 holding bf16(e4m3 * 2^k) on the non-RoPE dims, one
// power-of-two scale per 64 dims (dsv4_act_quant_inplace, group 64, mode 0,
// src/dsv4/dsv4_model.c:1386, applied at :5300), and BF16 on the RoPE dims
// (dsv4_rope_apply_buf rounds, :1555). Every such value is exactly an E4M3
// code times an E8M0 power of two, so per position the cache keeps nope
// codes, nope/64 scale codes (padded to 8 bytes) and rope BF16 values:
// 448 + 8 + 128 = 584 bytes at DSV4 sizes (583 of them carry information).
struct Fp8KvCache {
  uint8_t* codes = nullptr;    // [rows][nope]   E4M3
  uint8_t* scales = nullptr;   // [rows][8]      E8M0, one per 64 dims
  uint16_t* rope = nullptr;    // [rows][rope]   BF16
  int nope = 448;
  int rope_dim = 64;
  long long rows = 0;          // allocated positions (all batch elements)
};

constexpr int kKvScaleSlots = 8;

#ifdef __CUDACC__
// One 64-dim group g of a latent into cache row r, dsv4_act_quant_inplace
// (group 64, mode 0; src/dsv4/dsv4_model.c:1386-1417): lane l of a whole warp
// holds dims g*64 + l (a) and g*64 + 32 + l (b).
__device__ __forceinline__ void kv_quant_group(const Fp8KvCache& c, long long r, int g, float a,
                                               float b, int lane) {
  const float amax = warp_max(fmaxf(fabsf(a), fabsf(b)));
  const float scale = pow2_scale_448(amax);
  const float inv = 1.0f / scale;  // exact: scale is a normal power of two
  uint8_t code[2];
  const float v[2] = {a, b};
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    float q = v[k] * inv;
    q = fminf(fmaxf(q, -448.0f), 448.0f);
    unsigned short t;
    asm("{ .reg .b16 h; cvt.rn.satfinite.e4m3x2.f32 h, %1, %1; mov.b16 %0, h; }"
        : "=h"(t) : "f"(q));
    code[k] = (q == 0.0f) ? 0 : static_cast<uint8_t>(t & 0xFF);
  }
  uint8_t* dst = c.codes + r * c.nope + g * 64;
  dst[lane] = code[0];
  dst[32 + lane] = code[1];
  if (lane == 0)
    c.scales[r * kKvScaleSlots + g] = static_cast<uint8_t>((__float_as_uint(scale) >> 23) & 0xFF);
}
#endif

// Quantise fp32 latents [n][nope + rope] (BF16-valued) into cache rows
// row[n]: the reference's KV write (memcpy into the ring slot,
// src/dsv4/dsv4_model.c:5304, of the vector quantised at :5300).
cudaError_t kv_cache_write(const Fp8KvCache& c, const float* kv, const long long* row, int n,
                           cudaStream_t st);
// Decode cache rows back to fp32 [n][nope + rope] (the reference layout).
cudaError_t kv_cache_read(const Fp8KvCache& c, const long long* row, int n, float* out,
                          cudaStream_t st);

struct AttnProblem {
  const float* q = nullptr;        // [B][H][d], BF16-valued
  const float* kv = nullptr;       // fp32 rows [.][d] (reference layout) or null
  Fp8KvCache cache;                // used when kv == null (d = nope + rope)
  long long kv_batch_stride = 0;   // rows between consecutive batch elements
  long long kv_rows = 0;           // valid rows per batch element (index bound)
  const int* idx = nullptr;        // [B][n], -1 = padding
  const float* sink = nullptr;     // [H]
  const float* rope_cos = nullptr; // [B][rope/2] or null (no inverse RoPE)
  const float* rope_sin = nullptr;
  int rope_dim = 64;               // inverse RoPE on the last rope_dim dims
  float* out = nullptr;            // [B][H][d], BF16-valued
  int B = 1, H = 128, d = 512, n = 0;
  float scale = 0.0f;
  unsigned int* err = nullptr;     // device error word
};

// Bytes of scratch attn_forward needs (0-size problems need none).
size_t attn_workspace_bytes(const AttnProblem& p);
// True when the tensor-core kernel serves this shape (d = 512 with a
// 448 + 64 split, H <= 128); other shapes run the general SIMT kernels.
bool attn_uses_tensor_cores(const AttnProblem& p);
// Number of key splits the tensor-core path uses (1 for the SIMT path).
int attn_splits(const AttnProblem& p);

// out = sparse_attn(q, kv, sink, idx) for B independent queries
// (src/dsv4/dsv4_model.c:5767-5822), then the inverse RoPE of :5373 when
// rope_cos/rope_sin are given. `ws` holds attn_workspace_bytes(p) bytes.
cudaError_t attn_forward(const AttnProblem& p, void* ws, cudaStream_t st,
                         cudaEvent_t main_begin = nullptr, cudaEvent_t main_end = nullptr);

}  // namespace dsv4
