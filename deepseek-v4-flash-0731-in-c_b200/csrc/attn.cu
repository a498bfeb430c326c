// attn.cu - latent-KV decode attention (sparse_attn) and the FP8 latent
// cache on sm_100a.
//
// Reference: sparse_attn, src/dsv4/dsv4_model.c:5767-5822. Per head h:
//   s_t  = (fmaf-chain dot(q_h, kv_t)) * scale        (-inf for idx < 0)
//   m    = max_t s_t
//   den  = expf(sink_h - m) + sum_t expf(s_t - m)     (raw expf)
//   w_t  = bf16(expf(s_t - m))
//   o_h  = bf16(sum_t w_t * kv_t / den)
// followed by the inverse RoPE of the last rope dims (:5373, :1569).
//
// Tensor-core path (d = 512 = 448 + 64, H <= 128): split-KV flash decoding.
// One CTA per (batch element, key split, output half): the 128 heads are the
// MMA's M, so S = Q K^T lands in TMEM with one head per TMEM lane and the
// softmax needs no cross-thread reduction. Each CTA computes the full S tile
// (K = 512) and accumulates O for its 256 output dims in TMEM
// (tcgen05.mma kind::f16, BF16 operands, FP32 accumulators). The latent
// tile is dequantised once into a 128-byte-swizzled BF16 tile that serves
// as the K-major B operand of Q K^T and, unchanged, as the MN-major B
// operand of P V. The softmax keeps a running max per head and rescales
// the head's O row in TMEM when it grows; P = bf16(exp(s - m_run)) is the
// BF16 operand, the denominator sums raw expf as the reference does. A
// combine kernel merges the splits (m, den, O partials), divides, rounds to
// BF16 and applies the inverse RoPE.
//
// General path (other shapes): SIMT kernels in the reference's order.
#include <cmath>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "attn.cuh"
#include "bulk.cuh"
#include "dsv4_common.cuh"
#include "launch.cuh"

namespace dsv4 {
namespace {

constexpr unsigned kErrWait = 2u;    // an mbarrier wait in the attention kernel timed out
constexpr unsigned kErrIndex = 4u;   // a key index beyond the cache rows

// ============================================================ FP8 cache ==

// One block per position; warp w < nope/64 quantises group w exactly like
// dsv4_act_quant_inplace(group 64, mode 0) (src/dsv4/dsv4_model.c:1386-1417),
// the remaining warps copy the RoPE dims as BF16.
__global__ void kv_write_kernel(Fp8KvCache c, const float* __restrict__ kv,
                                const long long* __restrict__ row, int n) {
  const int p = blockIdx.x;
  if (p >= n) return;
  const int d = c.nope + c.rope_dim;
  const long long r = row[p];
  if (r < 0 || r >= c.rows) return;
  const float* x = kv + static_cast<size_t>(p) * d;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int groups = c.nope / 64;
  for (int g = warp; g < groups; g += blockDim.x >> 5)
    kv_quant_group(c, r, g, x[g * 64 + lane], x[g * 64 + 32 + lane], lane);
  for (int i = threadIdx.x; i < c.rope_dim; i += blockDim.x) {
    const float v = bf16_round(x[c.nope + i]);
    c.rope[r * c.rope_dim + i] = static_cast<uint16_t>(__float_as_uint(v) >> 16);
  }
}

__device__ __forceinline__ float kv_cache_value(const Fp8KvCache& c, long long r, int i) {
  if (i < c.nope) {
    const float v = e4m3_decode(c.codes[r * c.nope + i]) *
                    e8m0_decode(c.scales[r * kKvScaleSlots + i / 64]);
    return bf16_round(v);
  }
  return bf16_widen(c.rope[r * c.rope_dim + (i - c.nope)]);
}

__global__ void kv_read_kernel(Fp8KvCache c, const long long* __restrict__ row, int n,
                               float* __restrict__ out) {
  const int p = blockIdx.x;
  const int d = c.nope + c.rope_dim;
  const long long r = row[p];
  for (int i = threadIdx.x; i < d; i += blockDim.x)
    out[static_cast<size_t>(p) * d + i] =
        (r >= 0 && r < c.rows) ? kv_cache_value(c, r, i) : 0.0f;
}

// ============================================================ SIMT path ==

struct SimtArgs {
  AttnProblem p;
  float* scores;  // [B][H][n]
};

__device__ __forceinline__ float key_value(const AttnProblem& p, long long r, int i) {
  return p.kv ? p.kv[r * p.d + i] : kv_cache_value(p.cache, r, i);
}

__device__ __forceinline__ float block_reduce(float v, bool is_max, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float u = __shfl_xor_sync(0xffffffffu, v, o);
    v = is_max ? fmaxf(v, u) : v + u;
  }
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float r = red[0];
  for (int w = 1; w < nw; ++w) r = is_max ? fmaxf(r, red[w]) : r + red[w];
  return r;
}

// Inverse RoPE on one pair (src/dsv4/dsv4_model.c:1569-1580, contraction off).
__device__ __forceinline__ void rope_inv_pair(float& x0, float& x1, float c, float s) {
  const float y0 = __fadd_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
  const float y1 = __fadd_rn(__fmul_rn(-x0, s), __fmul_rn(x1, c));
  x0 = bf16_round(y0);
  x1 = bf16_round(y1);
}

// One block per (head, batch element); the dot products and the value sums
// run in the reference's order (fmaf over dims, then over keys).
__global__ void __launch_bounds__(256) attn_simt_kernel(SimtArgs a) {
  extern __shared__ float sm[];
  const AttnProblem& p = a.p;
  const int h = blockIdx.x, b = blockIdx.y;
  float* qs = sm;             // [d]
  float* os = sm + p.d;       // [d]
  float* red = os + p.d;      // [32]
  const float* q = p.q + (static_cast<size_t>(b) * p.H + h) * p.d;
  for (int i = threadIdx.x; i < p.d; i += blockDim.x) qs[i] = q[i];
  __syncthreads();
  float* sc = a.scores + (static_cast<size_t>(b) * p.H + h) * p.n;
  const int* idx = p.idx + static_cast<size_t>(b) * p.n;
  const long long base = static_cast<long long>(b) * p.kv_batch_stride;
  float mx = -INFINITY;
  for (int t = threadIdx.x; t < p.n; t += blockDim.x) {
    const int pos = idx[t];
    float s = -INFINITY;
    if (pos >= 0 && pos < p.kv_rows) {
      float dot = 0.0f;
      for (int i = 0; i < p.d; ++i) dot = fmaf(qs[i], key_value(p, base + pos, i), dot);
      s = dot * p.scale;
    } else if (pos >= 0 && p.err) {
      atomicOr(p.err, kErrIndex);
    }
    sc[t] = s;
    mx = fmaxf(mx, s);
  }
  mx = block_reduce(mx, true, red);
  float part = 0.0f;
  for (int t = threadIdx.x; t < p.n; t += blockDim.x) {
    const float s = sc[t];
    float w = 0.0f;
    if (s != -INFINITY) {
      const float e = expf(s - mx);
      part += e;
      w = bf16_round(e);
    }
    sc[t] = w;
  }
  const float den = expf(p.sink[h] - mx) + block_reduce(part, false, red);
  __syncthreads();
  for (int i = threadIdx.x; i < p.d; i += blockDim.x) {
    float acc = 0.0f;
    for (int t = 0; t < p.n; ++t) {
      const int pos = idx[t];
      if (pos < 0 || pos >= p.kv_rows) continue;
      acc = fmaf(sc[t], key_value(p, base + pos, i), acc);
    }
    os[i] = bf16_round(acc / den);
  }
  __syncthreads();
  const int rd = p.rope_dim, r0 = p.d - rd;
  if (p.rope_cos) {
    for (int i = threadIdx.x; i < rd / 2; i += blockDim.x) {
      float x0 = os[r0 + 2 * i], x1 = os[r0 + 2 * i + 1];
      rope_inv_pair(x0, x1, p.rope_cos[b * (rd / 2) + i], p.rope_sin[b * (rd / 2) + i]);
      os[r0 + 2 * i] = x0;
      os[r0 + 2 * i + 1] = x1;
    }
    __syncthreads();
  }
  float* o = p.out + (static_cast<size_t>(b) * p.H + h) * p.d;
  for (int i = threadIdx.x; i < p.d; i += blockDim.x) o[i] = os[i];
}

// ===================================================== tensor-core path ==

constexpr int kTcD = 512;
constexpr int kTcNope = 448;
constexpr int kTcRope = 64;
constexpr int kTcM = 128;       // heads (MMA M), zero-padded above H
constexpr int kTcKeys = 64;     // keys per tile: N of Q K^T, K of P V
constexpr int kTcHalf = 256;    // output dims per CTA: N of P V
constexpr int kTcOwnStages = 3;  // ring of the tile's own-half dims (the V of P V)
constexpr int kTcProdWarps = 8;
constexpr int kTcMmaWarp = 4 + kTcProdWarps;
constexpr int kTcThreads = 32 * (kTcMmaWarp + 1);  // 416: softmax 0-3, producers 4-11, MMA 12
constexpr float kTcLazyMargin = 8.0f;  // log2 units: the running max moves only past this margin
constexpr uint32_t kQBlock = kTcM * 128;                // one 64-dim column block of Q (16 KB)
constexpr uint32_t kKBlock = kTcKeys * 128;             // one 64-dim column block of a tile (8 KB)
constexpr uint32_t kQSmemBytes = 4 * kQBlock;           // Q dims 256-511 (64 KB)
constexpr uint32_t kHalfTile = 4 * kKBlock;             // 256 dims of a tile (32 KB)
constexpr uint32_t kPBytes = kTcM * kTcKeys * 2;        // 16384
constexpr uint32_t kOffQ = 0;
constexpr uint32_t kOffOwn = kOffQ + kQSmemBytes;
constexpr uint32_t kOffOther = kOffOwn + kTcOwnStages * kHalfTile;
constexpr uint32_t kOffP = kOffOther + kHalfTile;
constexpr uint32_t kOffBar = kOffP + 2 * kPBytes;       // 229376
constexpr uint32_t kTcSmem = kOffBar + 256 + 1024;      // + barriers + alignment slack
constexpr uint32_t kTmemCols = 512;  // O: cols 0-255, S: 256-383, Q dims 0-255 (A operand): 384-511
constexpr uint32_t kTmemS = 256;
constexpr uint32_t kTmemQ = 384;
constexpr float kLog2e = 1.4426950408889634f;

static_assert(kTcSmem <= 232448, "attention tile exceeds the 227 KB shared-memory limit");

struct TcArgs {
  const float* q;
  const float* kv;
  Fp8KvCache cache;
  long long kv_bstride, kv_rows;
  const int* idx;
  int B, H, n;
  float scale;
  int splits, keys_per_split;
  float* m_part;    // [B][splits][H] running max of the scores, log2 units
  float* den_part;  // [B][splits][H]
  float* o_part;    // [B][splits][H][512]
  unsigned* err;
};

// Byte offset of the 16-byte chunk (row, dc) in a 128-byte-swizzled tile
// whose 64-dim column blocks are `rows` rows tall (dc = dim / 8).
__device__ __forceinline__ uint32_t sw128_off(int row, int dc, int rows) {
  return static_cast<uint32_t>((dc >> 3) * rows * 128 + (row >> 3) * 1024 + (row & 7) * 128 +
                               (((dc & 7) ^ (row & 7)) << 4));
}

// UMMA shared-memory descriptor, 128-byte swizzle (layout type 2), sm_100
// version bit; addresses and offsets in 16-byte units.
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) |
         (static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16) |
         (static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}

// Instruction descriptor of kind::f16: FP32 accumulate, BF16 A and B.
__host__ __device__ constexpr uint32_t umma_idesc_bf16(int m, int n, bool b_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((b_mn_major ? 1u : 0u) << 16) |
         (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(m >> 4) << 24);
}

// MMA issue, warp-converged: every lane of the MMA warp executes these, one
// elected lane (the same one each time) issues. A rolled single-lane issue
// loop runs several times slower than the tensor pipe. The _ts form takes
// A (M x 16, BF16 pairs packed along K) from TMEM.
__device__ __forceinline__ void umma_bf16_e(uint32_t d_tmem, uint64_t a, uint64_t b,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p, e;\n setp.ne.b32 p, %4, 0;\n elect.sync _|e, 0xffffffff;\n"
      " @e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void umma_bf16_ts_e(uint32_t d_tmem, uint32_t a_tmem, uint64_t b,
                                               uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p, e;\n setp.ne.b32 p, %4, 0;\n elect.sync _|e, 0xffffffff;\n"
      " @e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void umma_commit_e(uint64_t* bar) {
  asm volatile(
      "{\n .reg .pred e;\n elect.sync _|e, 0xffffffff;\n"
      " @e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n}\n" ::"r"(
          smem_addr(bar))
      : "memory");
}

// 2^x on the MUFU unit (ex2.approx.ftz: relative error ~2^-22, 2^-inf = +0).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

#define DSV4_R32(X)                                                                          \
  X(0), X(1), X(2), X(3), X(4), X(5), X(6), X(7), X(8), X(9), X(10), X(11), X(12), X(13),  \
      X(14), X(15), X(16), X(17), X(18), X(19), X(20), X(21), X(22), X(23), X(24), X(25),  \
      X(26), X(27), X(28), X(29), X(30), X(31)
#define DSV4_OUT(i) "=r"(r[i])
#define DSV4_INOUT(i) "+r"(r[i])
#define DSV4_IN(i) "r"(r[i])

// 32 consecutive TMEM columns of this thread's lane (32x32b shape).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : DSV4_R32(DSV4_OUT)
      : "r"(taddr));
  // The wait names the registers so no use is scheduled before it.
  asm volatile("tcgen05.wait::ld.sync.aligned;" : DSV4_R32(DSV4_INOUT)::"memory");
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,"
      "%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(
          taddr),
      DSV4_R32(DSV4_IN)
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Bounded wait that also gives up once another role has aborted.
__device__ __forceinline__ bool tc_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                        unsigned* err) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_timer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (*abort_flag) return false;
    if (global_timer_ns() - t0 > kWaitLimitNs) {
      if (err) atomicOr(err, kErrWait);
      *abort_flag = 1;
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

// Four E4M3 codes (low byte first) times a power of two -> 2 x bf16x2; exact.
__device__ __forceinline__ uint2 e4m3x4_to_bf16(uint32_t w, float sc) {
  const uint32_t h01 = e4m3x2_to_f16x2(w & 0xFFFFu), h23 = e4m3x2_to_f16x2(w >> 16);
  const float2 f01 = __half22float2(*reinterpret_cast<const __half2*>(&h01));
  const float2 f23 = __half22float2(*reinterpret_cast<const __half2*>(&h23));
  return make_uint2(pack_bf16x2(f01.x * sc, f01.y * sc), pack_bf16x2(f23.x * sc, f23.y * sc));
}

// Four E4M3 codes times 2^(c - 127) -> 2 x bf16x2 on the integer and FMA
// pipes. Each code's 7 magnitude bits placed at BF16 bits 4-10 read as a
// BF16 number equal to the E4M3 value times 2^-120 (subnormal codes become
// BF16 subnormals, zero stays zero), the sign goes to bit 15, and one BF16
// multiply by k2 = 2^(c - 7) (exponent field c + 120) in both halves scales
// exactly. Valid for 10 <= c <= 134 (every product a normal BF16) and codes
// other than 0x7F/0xFF (NaN); the caller checks.
__device__ __forceinline__ uint2 e4m3x4_to_bf16_mul(uint32_t w, uint32_t k2) {
  const uint32_t m = w & 0x7F7F7F7Fu;
  uint32_t t0, t1, s0, s1, r0, r1;
  asm("prmt.b32 %0, %1, 0, 0x4140;" : "=r"(t0) : "r"(m));  // [b0, 0, b1, 0]
  asm("prmt.b32 %0, %1, 0, 0x4342;" : "=r"(t1) : "r"(m));  // [b2, 0, b3, 0]
  asm("prmt.b32 %0, %1, 0, 0x9484;" : "=r"(s0) : "r"(w));  // sign bytes of b0, b1
  asm("prmt.b32 %0, %1, 0, 0xB4A4;" : "=r"(s1) : "r"(w));  // sign bytes of b2, b3
  const uint32_t v0 = (t0 << 4) | (s0 & 0x80008000u), v1 = (t1 << 4) | (s1 & 0x80008000u);
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(r0) : "r"(v0), "r"(k2));
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(r1) : "r"(v1), "r"(k2));
  return make_uint2(r0, r1);
}

// Nonzero iff a byte of w is an E4M3 NaN code (0x7F or 0xFF).
__device__ __forceinline__ uint32_t e4m3_nan_bytes(uint32_t w) {
  return ((w & 0x7F7F7F7Fu) + 0x01010101u) & 0x80808080u;
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

struct TcBars {
  // A tile's dims split in two: "own" = this CTA's output half (also the V
  // of P V), held in a 3-slot ring, and "other" = the rest, in one slot.
  // full_*: that part of a tile is written; empty_other: Q K^T has read
  // the other part; empty_own: P V has read the own part.
  uint64_t full_own[kTcOwnStages], empty_own[kTcOwnStages], full_other, empty_other;
  uint64_t s_full[2], p_full[2], pv_done[2], fin;
  // validity bits of tile j's keys in slot j & 3, written by the first
  // own-quarter producers (tile j + 4 only after P V of tile j + 1, so after
  // the softmax of tile j has read slot j & 3)
  unsigned long long key_mask[4];
  uint32_t tmem_base;
  int abort_flag;
};
static_assert(sizeof(TcBars) <= 256, "barrier block exceeds its reservation");

// One CTA per (batch element, key split, output half): the 128 heads are
// the MMA's M, S = Q K^T (K = all 512 dims) lands in TMEM with one head per
// lane, and the CTA accumulates O for its 256 output dims. The two CTAs of
// a (batch element, split) read the same latent rows (the second read hits
// L2) and compute the same S and P, so no data moves between CTAs. Q K^T
// takes dims 0-255 of Q from TMEM and dims 256-511 from shared memory.
// Roles:
//   warps 0-3   softmax, thread = head = TMEM lane
//   warps 4-11  tile producers: 64 keys x 4 quarters of 128 dims
//   warp 12     TMEM allocation and MMA issue (one thread)
__global__ void __launch_bounds__(kTcThreads, 1) attn_tc_kernel(const __grid_constant__ TcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_s = smem_addr(smem_raw);
  const uint32_t pad = ((raw_s + 1023u) & ~1023u) - raw_s;
  uint8_t* smem = smem_raw + pad;
  const uint32_t sbase = raw_s + pad;
  const uint32_t q_s = sbase + kOffQ, own_s = sbase + kOffOwn, other_s = sbase + kOffOther;
  const uint32_t p_s = sbase + kOffP;
  TcBars* bars = reinterpret_cast<TcBars*>(smem + kOffBar);
  volatile int* abort_flag = &bars->abort_flag;

  const int half = blockIdx.x & 1, split = blockIdx.x >> 1, b = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int k0 = split * a.keys_per_split;
  const int k_end = min(a.n, k0 + a.keys_per_split);
  const int T = k_end > k0 ? (k_end - k0 + kTcKeys - 1) / kTcKeys : 0;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kTcOwnStages; ++i) {
      mbar_init(&bars->full_own[i], 16 * kTcProdWarps);
      mbar_init(&bars->empty_own[i], 1);
    }
    mbar_init(&bars->full_other, 16 * kTcProdWarps);
    mbar_init(&bars->empty_other, 1);
    for (int i = 0; i < 4; ++i) bars->key_mask[i] = 0;
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->s_full[i], 1);
      mbar_init(&bars->p_full[i], 128);
      mbar_init(&bars->pv_done[i], 1);
    }
    mbar_init(&bars->fin, 1);
    bars->abort_flag = 0;
    mbar_fence_init();
  }
  pdl_wait();  // q, the cache rows and the indices come from earlier kernels
  pdl_trigger();
  if (warp == kTcMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_addr(&bars->tmem_base)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  } else {
    // Q dims 256-511: fp32 (BF16-valued) -> BF16, K-major 128-byte swizzled,
    // rows >= H zero
    const float* qb = a.q + static_cast<size_t>(b) * a.H * kTcD + kTcHalf;
    for (int c = threadIdx.x; c < kTcM * (kTcHalf / 8); c += 32 * kTcMmaWarp) {
      const int row = c >> 5, dc = c & 31;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (row < a.H) {
        const float4* src = reinterpret_cast<const float4*>(qb + row * kTcD + dc * 8);
        const float4 x0 = src[0], x1 = src[1];
        v = make_uint4(pack_bf16x2(x0.x, x0.y), pack_bf16x2(x0.z, x0.w), pack_bf16x2(x1.x, x1.y),
                       pack_bf16x2(x1.z, x1.w));
      }
      st_shared_v4(q_s + sw128_off(row, dc, kTcM), v);
    }
    fence_async_smem();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  if (warp < 4) {
    // Q dims 0-255 of row h -> BF16 pairs in TMEM lane h, columns kTmemQ..
    const int h = threadIdx.x;
    const float4* src = reinterpret_cast<const float4*>(
        a.q + (static_cast<size_t>(b) * a.H + (h < a.H ? h : 0)) * kTcD);
#pragma unroll 1
    for (int c32 = 0; c32 < kTcHalf / 2; c32 += 32) {
      uint32_t r[32];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float4 x = h < a.H ? src[c32 / 2 + i] : make_float4(0.f, 0.f, 0.f, 0.f);
        r[2 * i] = pack_bf16x2(x.x, x.y);
        r[2 * i + 1] = pack_bf16x2(x.z, x.w);
      }
      tmem_st32(tmem + (static_cast<uint32_t>(warp * 32) << 16) + kTmemQ + c32, r);
    }
    tmem_st_wait();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  if (warp == kTcMmaWarp) {
    // ------------------------------------------------------------ MMA issue
    // The whole warp waits and runs the unrolled issue code; one elected
    // lane issues. Descriptor addresses advance in 16-byte units.
    constexpr uint32_t idesc_qk = umma_idesc_bf16(kTcM, kTcKeys, false);
    constexpr uint32_t idesc_pv = umma_idesc_bf16(kTcM, kTcHalf, true);
    const uint64_t q_desc = umma_desc(q_s, 16, 1024);
    // O += P V for tile jj, V = its own-half slot read MN-major
    auto issue_pv = [&](int jj, int slot) -> bool {
      const int sb = jj & 1;
      const bool w = tc_wait(&bars->p_full[sb], (jj >> 1) & 1, abort_flag, a.err);
      if (!__all_sync(0xffffffffu, w)) return false;
      tc_fence_after();
      const uint64_t ad = umma_desc(p_s + sb * kPBytes, 16, 1024);
      const uint64_t bd = umma_desc(own_s + slot * kHalfTile, kKBlock, 1024);
#pragma unroll
      for (int kk = 0; kk < kTcKeys / 16; ++kk)
        umma_bf16_e(tmem, ad + kk * 2, bd + kk * 128, idesc_pv, (jj > 0 || kk > 0) ? 1u : 0u);
      umma_commit_e(&bars->pv_done[sb]);
      umma_commit_e(&bars->empty_own[slot]);
      return true;
    };
    // Q K^T over 256 dims of a half-tile (column block kk / 4, 32 bytes into
    // its swizzle row): Q dims 0-255 come from TMEM, 256-511 from shared
    // memory. Fully unrolled with compile-time offsets: the issue rate of
    // this warp bounds the MMA rate.
    auto qk_tmem_a = [&](uint32_t s_col, uint64_t k_desc, bool first) {
#pragma unroll
      for (int kk = 0; kk < kTcHalf / 16; ++kk)
        umma_bf16_ts_e(s_col, tmem + kTmemQ + kk * 8,
                       k_desc + ((kk >> 2) * kKBlock + (kk & 3) * 32) / 16, idesc_qk,
                       (first && kk == 0) ? 0u : 1u);
    };
    auto qk_smem_a = [&](uint32_t s_col, uint64_t k_desc, bool first) {
#pragma unroll
      for (int kk = 0; kk < kTcHalf / 16; ++kk)
        umma_bf16_e(s_col, q_desc + ((kk >> 2) * kQBlock + (kk & 3) * 32) / 16,
                    k_desc + ((kk >> 2) * kKBlock + (kk & 3) * 32) / 16, idesc_qk,
                    (first && kk == 0) ? 0u : 1u);
    };
    const uint64_t other_desc = umma_desc(other_s, 16, 1024);
    bool ok = true;
    int slot = 0, prev_slot = 0;
    uint32_t ph = 0;
    for (int j = 0; j < T && ok; ++j) {
      const uint32_t s_col = tmem + kTmemS + (j & 1) * kTcKeys;
      // the other half of the dims first (its single slot is released as
      // soon as these MMAs complete), then the own half
      bool w = tc_wait(&bars->full_other, j & 1, abort_flag, a.err);
      if (!__all_sync(0xffffffffu, w)) { ok = false; break; }
      tc_fence_after();
      if (half == 0)
        qk_smem_a(s_col, other_desc, true);
      else
        qk_tmem_a(s_col, other_desc, true);
      umma_commit_e(&bars->empty_other);
      w = tc_wait(&bars->full_own[slot], ph, abort_flag, a.err);
      if (!__all_sync(0xffffffffu, w)) { ok = false; break; }
      tc_fence_after();
      const uint64_t own_desc = umma_desc(own_s + slot * kHalfTile, 16, 1024);
      if (half == 0)
        qk_tmem_a(s_col, own_desc, false);
      else
        qk_smem_a(s_col, own_desc, false);
      umma_commit_e(&bars->s_full[j & 1]);
      // P V of the previous tile runs while the softmax works on this one
      if (j > 0 && !issue_pv(j - 1, prev_slot)) { ok = false; break; }
      prev_slot = slot;
      if (++slot == kTcOwnStages) { slot = 0; ph ^= 1u; }
    }
    if (ok && T > 0) issue_pv(T - 1, prev_slot);
    umma_commit_e(&bars->fin);
    mbar_wait(&bars->fin, 0, a.err);
    __syncwarp();
  } else if (warp >= 4) {
    // ------------------------------------------------- latent tile producer
    // Thread (r, q) owns key r of every tile and dims [128 q, 128 q + 128)
    // (column blocks 2q, 2q + 1): FP8 codes with scale slots 2q, 2q + 1, or
    // for q 3 the codes 384-447 (slot 6) and the 64 BF16 RoPE dims; a warp
    // holds one quarter q for 32 keys. The quarters of this CTA's output half
    // go to the own ring and wait for P V to release a slot, the others to
    // the other slot and wait only for Q K^T. The indices of tile j + 3 are
    // read and the rows of tile j + 2 bulk-prefetched into L2 while tile j
    // is converted; the registers of tile j + 1 are loaded right after tile
    // j is handed over.
    const int c = threadIdx.x - 128;
    const int r = c & (kTcKeys - 1), q = c / kTcKeys;
    const bool own = (q >> 1) == half;
    const int* idxb = a.idx + static_cast<size_t>(b) * a.n;
    const long long rbase = static_cast<long long>(b) * a.kv_bstride;
    auto load_idx = [&](int j) -> long long {
      const int key = k0 + j * kTcKeys + r;
      return (j < T && key < k_end) ? static_cast<long long>(idxb[key]) : -1;
    };
    auto in_range = [&](long long pos) { return pos >= 0 && pos < a.kv_rows; };
    auto prefetch_rows = [&](long long pos) {
      if (!in_range(pos)) return;
      const long long row = rbase + pos;
      if (a.kv) {
        bulk_prefetch_l2(a.kv + row * kTcD + q * 128, 512);
      } else if (q == 0) {
        bulk_prefetch_l2(a.cache.codes + row * kTcNope, kTcNope);
      } else if (q == 1) {
        bulk_prefetch_l2(a.cache.rope + row * kTcRope, kTcRope * 2);
      } else if (q == 2) {
        const long long r2 = row & ~1ll;  // the 16-byte pair of scale rows holding this one
        if (r2 + 1 < a.cache.rows) bulk_prefetch_l2(a.cache.scales + r2 * kKvScaleSlots, 16);
      }
    };
    // q < 3: 8 x 16 codes; q == 3: 4 x 16 codes then 8 x 8 RoPE BF16 values
    uint4 raw[12];
    uint32_t sc2 = 0;  // scale codes of the thread's two column blocks
    auto load_raw = [&](long long pos) {
      if (!in_range(pos) || a.kv) return;
      const long long row = rbase + pos;
      const uint4* cp = reinterpret_cast<const uint4*>(a.cache.codes + row * kTcNope + q * 128);
      const uint4* rp = reinterpret_cast<const uint4*>(a.cache.rope + row * kTcRope);
#pragma unroll
      for (int u = 0; u < 12; ++u) {
        if (q < 3) {
          if (u < 8) raw[u] = __ldg(cp + u);
        } else {
          raw[u] = u < 4 ? __ldg(cp + u) : __ldg(rp + (u - 4));
        }
      }
      sc2 = *reinterpret_cast<const uint16_t*>(a.cache.scales + row * kKvScaleSlots + 2 * q);
    };
    if (c == 0 && T > 0) {
      // the split's key indices into L2 up front (whole 16-byte blocks
      // inside the array): the per-tile index loads then miss only to L2
      const uintptr_t lo = reinterpret_cast<uintptr_t>(idxb + k0);
      const uintptr_t hi = reinterpret_cast<uintptr_t>(idxb + k_end);
      for (uintptr_t p0 = (lo + 15) & ~static_cast<uintptr_t>(15); p0 + 16 <= hi; p0 += 16384) {
        const uintptr_t p1 = p0 + 16384 < hi ? p0 + 16384 : (hi & ~static_cast<uintptr_t>(15));
        bulk_prefetch_l2(reinterpret_cast<const void*>(p0), static_cast<uint32_t>(p1 - p0));
      }
    }
    long long p_cur = load_idx(0), p_nxt = load_idx(1), p_n2 = load_idx(2);
    prefetch_rows(p_cur);
    prefetch_rows(p_nxt);
    load_raw(p_cur);
    int slot = 0;
    uint32_t ph = 0;
    const int qb = (q & 1) * 16;  // the quarter's first 16-byte chunk in its half-tile
    for (int j = 0; j < T; ++j) {
      const long long p_n3 = load_idx(j + 3);
      if (p_cur >= a.kv_rows && a.err) atomicOr(a.err, kErrIndex);
      const bool valid = in_range(p_cur);
      const long long row = rbase + p_cur;
      const bool w = own ? tc_wait(&bars->empty_own[slot], ph ^ 1u, abort_flag, a.err)
                         : tc_wait(&bars->empty_other, (j & 1) ^ 1, abort_flag, a.err);
      if (!w) break;
      const uint32_t tile = own ? own_s + slot * kHalfTile : other_s;
      if (!valid) {
#pragma unroll
        for (int dc = 0; dc < 16; ++dc)
          st_shared_v4(tile + sw128_off(r, qb + dc, kTcKeys), make_uint4(0, 0, 0, 0));
      } else if (a.kv) {
        const float4* src = reinterpret_cast<const float4*>(a.kv + row * kTcD + q * 128);
#pragma unroll 4
        for (int dc = 0; dc < 16; ++dc) {
          const float4 x0 = __ldg(src + 2 * dc), x1 = __ldg(src + 2 * dc + 1);
          st_shared_v4(tile + sw128_off(r, qb + dc, kTcKeys),
                       make_uint4(pack_bf16x2(x0.x, x0.y), pack_bf16x2(x0.z, x0.w),
                                  pack_bf16x2(x1.x, x1.y), pack_bf16x2(x1.z, x1.w)));
        }
      } else {
        // the integer path unless a scale is out of its range or a code is NaN
        uint32_t nan = 0;
#pragma unroll
        for (int u = 0; u < 8; ++u)
          if (q < 3 || u < 4)
            nan |= e4m3_nan_bytes(raw[u].x) | e4m3_nan_bytes(raw[u].y) |
                   e4m3_nan_bytes(raw[u].z) | e4m3_nan_bytes(raw[u].w);
        const uint32_t c0 = sc2 & 0xFFu, c1 = q < 3 ? (sc2 >> 8) & 0xFFu : c0;
        if (nan == 0 && c0 >= 10 && c0 <= 134 && c1 >= 10 && c1 <= 134) {
          const uint32_t k0s = (c0 + 120) * 0x00800080u, k1s = (c1 + 120) * 0x00800080u;
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            if (q < 3 || u < 4) {
              const uint32_t k2 = u < 4 ? k0s : k1s;
              const uint2 lo = e4m3x4_to_bf16_mul(raw[u].x, k2),
                          hi = e4m3x4_to_bf16_mul(raw[u].y, k2);
              const uint2 lo2 = e4m3x4_to_bf16_mul(raw[u].z, k2),
                          hi2 = e4m3x4_to_bf16_mul(raw[u].w, k2);
              st_shared_v4(tile + sw128_off(r, qb + 2 * u, kTcKeys),
                           make_uint4(lo.x, lo.y, hi.x, hi.y));
              st_shared_v4(tile + sw128_off(r, qb + 2 * u + 1, kTcKeys),
                           make_uint4(lo2.x, lo2.y, hi2.x, hi2.y));
            }
          }
        } else {
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            if (q < 3 || u < 4) {
              const float sc = e8m0_decode((sc2 >> (8 * (u >> 2))) & 0xFFu);
              const uint2 lo = e4m3x4_to_bf16(raw[u].x, sc), hi = e4m3x4_to_bf16(raw[u].y, sc);
              const uint2 lo2 = e4m3x4_to_bf16(raw[u].z, sc), hi2 = e4m3x4_to_bf16(raw[u].w, sc);
              st_shared_v4(tile + sw128_off(r, qb + 2 * u, kTcKeys),
                           make_uint4(lo.x, lo.y, hi.x, hi.y));
              st_shared_v4(tile + sw128_off(r, qb + 2 * u + 1, kTcKeys),
                           make_uint4(lo2.x, lo2.y, hi2.x, hi2.y));
            }
          }
        }
        if (q == 3) {
#pragma unroll
          for (int u = 0; u < 8; ++u)
            st_shared_v4(tile + sw128_off(r, 24 + u, kTcKeys), raw[4 + u]);
        }
      }
      // validity mask of the tile's keys (bit r), written by the warps of the
      // first own quarter
      const uint32_t vb = __ballot_sync(0xffffffffu, valid);
      if (q == 2 * half && lane == 0)
        reinterpret_cast<volatile uint32_t*>(&bars->key_mask[j & 3])[r >> 5] = vb;
      __syncwarp();
      fence_async_smem();
      mbar_arrive(own ? &bars->full_own[slot] : &bars->full_other);
      prefetch_rows(p_n2);
      load_raw(p_nxt);
      p_cur = p_nxt;
      p_nxt = p_n2;
      p_n2 = p_n3;
      if (++slot == kTcOwnStages) { slot = 0; ph ^= 1u; }
    }
  } else {
    // --------------------------------------------------------------- softmax
    const int h = threadIdx.x;  // head = TMEM lane
    const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
    // scores in log2 units: t = dot * scale * log2(e), weights 2^(t - m)
    const float sc2 = a.scale * kLog2e;
    float m_run = -INFINITY, den = 0.0f;
    bool ok = true;
    int kst = 0;
    uint32_t kph = 0;
    for (int j = 0; j < T; ++j) {
      const int sb = j & 1;
      // full_own (its producers wrote the key mask) cannot run a phase
      // ahead: tile j + 3's own part waits for P V of tile j
      bool w = tc_wait(&bars->s_full[sb], (j >> 1) & 1, abort_flag, a.err);
      w = w && tc_wait(&bars->full_own[kst], kph, abort_flag, a.err);
      if (!__all_sync(0xffffffffu, w)) { ok = false; break; }
      tc_fence_after();
      const unsigned long long mask =
          *reinterpret_cast<volatile unsigned long long*>(&bars->key_mask[j & 3]);
      float s[kTcKeys];
      float tmax = -INFINITY;
#pragma unroll
      for (int c32 = 0; c32 < kTcKeys; c32 += 32) {
        uint32_t r[32];
        tmem_ld32(tmem + lane_base + kTmemS + sb * kTcKeys + c32, r);
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int k = c32 + i;
          s[k] = ((mask >> k) & 1ull) ? __uint_as_float(r[i]) * sc2 : -INFINITY;
          tmax = fmaxf(tmax, s[k]);
        }
      }
      // lazy running max: it moves only when a score exceeds it by the
      // margin (then O and den are rescaled), so the weights stay <= 2^8
      float m_use = m_run, alpha = 1.0f;
      bool resc = false;
      if (tmax != -INFINITY) {
        if (m_run == -INFINITY) {
          m_use = tmax;
        } else if (tmax > m_run + kTcLazyMargin) {
          m_use = tmax;
          alpha = ex2_approx(m_run - tmax);
          resc = true;
        }
      }
      den *= alpha;
      uint32_t pw[kTcKeys / 2];
      float part[4] = {0.f, 0.f, 0.f, 0.f};
      const float m_sub = m_use == -INFINITY ? 0.0f : m_use;  // a masked tile: 2^-inf = 0
#pragma unroll
      for (int i = 0; i < kTcKeys; i += 2) {
        // MUFU exp2: relative error ~2^-22, far below the BF16 rounding the
        // weights get
        const float e0 = ex2_approx(s[i] - m_sub);
        const float e1 = ex2_approx(s[i + 1] - m_sub);
        part[(i >> 1) & 3] += e0 + e1;
        pw[i / 2] = pack_bf16x2(e0, e1);
      }
      den += (part[0] + part[1]) + (part[2] + part[3]);
      m_run = m_use;
      // P buffer sb was last read by P V of tile j - 2
      if (j >= 2) {
        const bool wp = tc_wait(&bars->pv_done[sb], ((j - 2) >> 1) & 1, abort_flag, a.err);
        if (!__all_sync(0xffffffffu, wp)) { ok = false; break; }
      }
      if (__any_sync(0xffffffffu, resc)) {
        // O holds tiles < j once P V of tile j - 1 is done (j >= 1 here: a
        // finite running max comes from an earlier tile)
        const bool wv = tc_wait(&bars->pv_done[(j - 1) & 1], ((j - 1) >> 1) & 1, abort_flag, a.err);
        if (!__all_sync(0xffffffffu, wv)) { ok = false; break; }
        tc_fence_after();
#pragma unroll 1
        for (int cb = 0; cb < kTcHalf; cb += 32) {
          uint32_t o[32];
          tmem_ld32(tmem + lane_base + cb, o);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st32(tmem + lane_base + cb, o);
        }
        tmem_st_wait();
      }
      const uint32_t prow = p_s + sb * kPBytes + (h >> 3) * 1024 + (h & 7) * 128;
#pragma unroll
      for (int c8 = 0; c8 < 8; ++c8)
        st_shared_v4(prow + ((c8 ^ (h & 7)) << 4),
                     make_uint4(pw[4 * c8], pw[4 * c8 + 1], pw[4 * c8 + 2], pw[4 * c8 + 3]));
      fence_async_smem();
      tc_fence_before();
      mbar_arrive(&bars->p_full[sb]);
      if (++kst == kTcOwnStages) { kst = 0; kph ^= 1u; }
    }
    // epilogue: O partial row, m and den
    const size_t prow = (static_cast<size_t>(b) * a.splits + split) * a.H + h;
    bool have = ok && T > 0;
    if (have) {
      const bool wv = tc_wait(&bars->pv_done[(T - 1) & 1], ((T - 1) >> 1) & 1, abort_flag, a.err);
      have = __all_sync(0xffffffffu, wv);
    }
    if (have) {
      tc_fence_after();
      for (int cb = 0; cb < kTcHalf; cb += 32) {
        uint32_t o[32];
        tmem_ld32(tmem + lane_base + cb, o);
        if (h < a.H) {
          float4* dst = reinterpret_cast<float4*>(a.o_part + prow * kTcD + half * kTcHalf + cb);
#pragma unroll
          for (int i = 0; i < 8; ++i)
            dst[i] = make_float4(__uint_as_float(o[4 * i]), __uint_as_float(o[4 * i + 1]),
                                 __uint_as_float(o[4 * i + 2]), __uint_as_float(o[4 * i + 3]));
        }
      }
    } else if (h < a.H) {
      float4* dst = reinterpret_cast<float4*>(a.o_part + prow * kTcD + half * kTcHalf);
      for (int i = 0; i < kTcHalf / 4; ++i) dst[i] = make_float4(0.f, 0.f, 0.f, 0.f);
      m_run = -INFINITY;
      den = 0.0f;
    }
    if (half == 0 && h < a.H) {
      a.m_part[prow] = m_run;
      a.den_part[prow] = den;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kTcMmaWarp)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTmemCols)
                 : "memory");
}

// Merge the splits of one (head, batch element): 128 threads x 4 dims.
__global__ void __launch_bounds__(128) attn_combine_kernel(AttnProblem p, int splits,
                                                           const float* __restrict__ m_part,
                                                           const float* __restrict__ den_part,
                                                           const float* __restrict__ o_part) {
  const int h = blockIdx.x, b = blockIdx.y;
  extern __shared__ float wsm[];  // [splits]
  __shared__ float s_den;
  pdl_wait();  // the partials come from attn_tc_kernel
  pdl_trigger();
  if (threadIdx.x < 32) {
    // warp 0: the splits' maxima and weighted denominators, lanes striding
    // over the splits, then warp reductions
    const int lane = threadIdx.x;
    // a lane's splits (lane, lane + 32, ...) four at a time: their maxima
    // and denominators are loaded together
    constexpr int kPer = 4;
    float M = -INFINITY;
    float den = 0.0f;
    if (splits <= 32 * kPer) {
      float mv[kPer], dv[kPer];
#pragma unroll
      for (int k = 0; k < kPer; ++k) {
        const int s = lane + 32 * k;
        const size_t i = (static_cast<size_t>(b) * splits + s) * p.H + h;
        mv[k] = s < splits ? m_part[i] : -INFINITY;
        dv[k] = s < splits ? den_part[i] : 0.0f;
      }
#pragma unroll
      for (int k = 0; k < kPer; ++k) M = fmaxf(M, mv[k]);
      M = warp_max(M);
#pragma unroll
      for (int k = 0; k < kPer; ++k) {
        const int s = lane + 32 * k;
        if (s < splits) {
          const float w = (mv[k] == -INFINITY) ? 0.0f : exp2f(mv[k] - M);
          wsm[s] = w;
          den += dv[k] * w;
        }
      }
    } else {
      for (int s = lane; s < splits; s += 32)
        M = fmaxf(M, m_part[(static_cast<size_t>(b) * splits + s) * p.H + h]);
      M = warp_max(M);
      for (int s = lane; s < splits; s += 32) {
        const size_t i = (static_cast<size_t>(b) * splits + s) * p.H + h;
        const float w = (m_part[i] == -INFINITY) ? 0.0f : exp2f(m_part[i] - M);
        wsm[s] = w;
        den += den_part[i] * w;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) den += __shfl_xor_sync(0xffffffffu, den, o);
    if (lane == 0) s_den = den + exp2f(p.sink[h] * kLog2e - M);
  }
  __syncthreads();
  const float den = s_den;
  const int d0 = threadIdx.x * 4;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  const float* ob = o_part + (static_cast<size_t>(b) * splits * p.H + h) * kTcD + d0;
  const size_t sstride = static_cast<size_t>(p.H) * kTcD;  // floats between splits
  // kBatch splits' partial rows are loaded together (independent L2 reads in
  // flight), then added in split order; an empty split (w == 0) adds nothing
  constexpr int kBatch = 16;
  for (int s = 0; s < splits; s += kBatch) {
    float4 v[kBatch];
#pragma unroll
    for (int k = 0; k < kBatch; ++k)
      if (s + k < splits)
        v[k] = *reinterpret_cast<const float4*>(ob + static_cast<size_t>(s + k) * sstride);
#pragma unroll
    for (int k = 0; k < kBatch; ++k) {
      const float w = s + k < splits ? wsm[s + k] : 0.0f;
      if (w != 0.0f) {
        acc[0] += v[k].x * w;
        acc[1] += v[k].y * w;
        acc[2] += v[k].z * w;
        acc[3] += v[k].w * w;
      }
    }
  }
  float o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) o[i] = bf16_round(acc[i] / den);
  const int r0 = kTcD - p.rope_dim;
  if (p.rope_cos && d0 >= r0) {
    const int pi = (d0 - r0) / 2;
    const float* cs = p.rope_cos + b * (p.rope_dim / 2);
    const float* sn = p.rope_sin + b * (p.rope_dim / 2);
    rope_inv_pair(o[0], o[1], cs[pi], sn[pi]);
    rope_inv_pair(o[2], o[3], cs[pi + 1], sn[pi + 1]);
  }
  *reinterpret_cast<float4*>(p.out + (static_cast<size_t>(b) * p.H + h) * kTcD + d0) =
      make_float4(o[0], o[1], o[2], o[3]);
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

// m and den partials first, then the O partials from a 256-byte boundary
// (the kernels move O partials as float4).
size_t tc_o_part_offset(size_t rows) { return (2 * rows + 63) & ~static_cast<size_t>(63); }

struct TcPlan {
  int splits, keys_per_split;
};

TcPlan tc_plan(const AttnProblem& p) {
  const int tiles = (p.n + kTcKeys - 1) / kTcKeys;
  if (tiles == 0) return {1, kTcKeys};
  int per_b = sm_count() / (2 * p.B);
  if (per_b < 1) per_b = 1;
  // at least kMinSplitTiles tiles per split: fewer CTAs pay the Q load and
  // TMEM setup, and the combine reads fewer partials
  constexpr int kMinSplitTiles = 2;
  const int max_splits = (tiles + kMinSplitTiles - 1) / kMinSplitTiles;
  if (per_b > max_splits) per_b = max_splits;
  int splits = per_b < tiles ? per_b : tiles;
  const int tiles_per = (tiles + splits - 1) / splits;
  splits = (tiles + tiles_per - 1) / tiles_per;
  return {splits, tiles_per * kTcKeys};
}

}  // namespace

bool attn_uses_tensor_cores(const AttnProblem& p) {
  if (p.d != kTcD || p.H < 1 || p.H > kTcM) return false;
  if (!p.kv && (p.cache.nope != kTcNope || p.cache.rope_dim != kTcRope)) return false;
  // the combine kernel's threads own 4 dims each: RoPE pairs must not straddle
  if (p.rope_cos && (p.rope_dim % 4 != 0)) return false;
  return true;
}

int attn_splits(const AttnProblem& p) {
  return attn_uses_tensor_cores(p) ? tc_plan(p).splits : 1;
}

size_t attn_workspace_bytes(const AttnProblem& p) {
  if (attn_uses_tensor_cores(p)) {
    const size_t rows = static_cast<size_t>(p.B) * tc_plan(p).splits * p.H;
    return tc_o_part_offset(rows) * sizeof(float) + rows * kTcD * sizeof(float) + 256;
  }
  return static_cast<size_t>(p.B) * p.H * (p.n > 0 ? p.n : 1) * sizeof(float) + 256;
}

cudaError_t kv_cache_write(const Fp8KvCache& c, const float* kv, const long long* row, int n,
                           cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  if (c.nope % 64 != 0 || c.nope / 64 > kKvScaleSlots) return cudaErrorInvalidValue;
  kv_write_kernel<<<n, 256, 0, st>>>(c, kv, row, n);
  return cudaGetLastError();
}

cudaError_t kv_cache_read(const Fp8KvCache& c, const long long* row, int n, float* out,
                          cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  kv_read_kernel<<<n, 256, 0, st>>>(c, row, n, out);
  return cudaGetLastError();
}

cudaError_t attn_forward(const AttnProblem& p, void* ws, cudaStream_t st, cudaEvent_t main_begin,
                         cudaEvent_t main_end) {
  if (p.B <= 0 || p.H <= 0) return cudaSuccess;
  if (p.d <= 0 || p.n < 0 || p.rope_dim < 0 || p.rope_dim > p.d || (p.rope_dim & 1))
    return cudaErrorInvalidValue;
  if (!p.kv && (p.cache.nope + p.cache.rope_dim != p.d || p.cache.nope % 64 != 0))
    return cudaErrorInvalidValue;
  if (attn_uses_tensor_cores(p)) {
    const TcPlan plan = tc_plan(p);
    float* base = reinterpret_cast<float*>(ws);
    const size_t rows = static_cast<size_t>(p.B) * plan.splits * p.H;
    TcArgs a;
    a.q = p.q;
    a.kv = p.kv;
    a.cache = p.cache;
    a.kv_bstride = p.kv_batch_stride;
    a.kv_rows = p.kv_rows;
    a.idx = p.idx;
    a.B = p.B;
    a.H = p.H;
    a.n = p.n;
    a.scale = p.scale;
    a.splits = plan.splits;
    a.keys_per_split = plan.keys_per_split;
    a.m_part = base;
    a.den_part = base + rows;
    a.o_part = base + tc_o_part_offset(rows);
    a.err = p.err;
    static bool attr_set[64] = {};  // per device
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !attr_set[dev]) {
      cudaError_t e = cudaFuncSetAttribute(attn_tc_kernel,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmem);
      if (e != cudaSuccess) return e;
      if (dev >= 0 && dev < 64) attr_set[dev] = true;
    }
    if (main_begin) cudaEventRecord(main_begin, st);
    cudaError_t e = launch_pdl(attn_tc_kernel, dim3(2 * plan.splits, p.B), dim3(kTcThreads),
                               kTcSmem, st, a);
    if (e != cudaSuccess) return e;
    if (main_end) cudaEventRecord(main_end, st);
    e = launch_pdl(attn_combine_kernel, dim3(p.H, p.B), dim3(128), plan.splits * sizeof(float), st,
                   p, plan.splits, static_cast<const float*>(a.m_part),
                   static_cast<const float*>(a.den_part), static_cast<const float*>(a.o_part));
    return e != cudaSuccess ? e : cudaGetLastError();
  }
  SimtArgs a;
  a.p = p;
  a.scores = reinterpret_cast<float*>(ws);
  const size_t smem = (2 * static_cast<size_t>(p.d) + 32) * sizeof(float);
  if (smem > 48 * 1024) return cudaErrorInvalidValue;
  if (main_begin) cudaEventRecord(main_begin, st);
  attn_simt_kernel<<<dim3(p.H, p.B), 256, smem, st>>>(a);
  if (main_end) cudaEventRecord(main_end, st);
  return cudaGetLastError();
}

}  // namespace dsv4
