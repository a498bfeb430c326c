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
#include <mutex>
#include <utility>
#include <vector>

#include <cudaTypedefs.h>

#include "bulk.cuh"
#include "dsv4_common.cuh"
#include "gemv.cuh"
#include "gemv_dev.cuh"
#include "launch.cuh"

namespace dsv4 {

namespace {
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}
struct MapKey {
  const void* base;
  uint64_t row_bytes, rows;
  uint32_t box_bytes, box_rows;
  bool sw;
  bool operator==(const MapKey& o) const {
    return base == o.base && row_bytes == o.row_bytes && rows == o.rows &&
           box_bytes == o.box_bytes && box_rows == o.box_rows && sw == o.sw;
  }
};
}  // namespace

bool make_tma_map_u8(CUtensorMap* out, const void* base, uint64_t row_bytes, uint64_t rows,
                     uint32_t box_bytes, uint32_t box_rows, bool swizzle128, bool use_cache) {
  static std::mutex mu;
  static std::vector<std::pair<MapKey, CUtensorMap>> cache;
  const MapKey key{base, row_bytes, rows, box_bytes, box_rows, swizzle128};
  if (use_cache) {
    std::lock_guard<std::mutex> lock(mu);
    for (const auto& e : cache)
      if (e.first == key) { *out = e.second; return true; }
  }
  auto fn = encode_fn();
  if (!fn || reinterpret_cast<uintptr_t>(base) % 16 != 0 || row_bytes % 16 != 0 ||
      box_bytes % 16 != 0 || rows == 0)
    return false;
  const cuuint64_t dims[2] = {row_bytes, rows};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {box_bytes, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  CUtensorMap m;
  if (fn(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
         CU_TENSOR_MAP_INTERLEAVE_NONE,
         swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return false;
  *out = m;
  if (!use_cache) return true;
  std::lock_guard<std::mutex> lock(mu);
  if (cache.size() > 4096) cache.clear();
  cache.emplace_back(key, m);
  *out = m;
  return true;
}

unsigned int* device_error_word() {
  static unsigned int* words[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  if (!words[dev]) {
    unsigned int* w = nullptr;
    if (cudaMalloc(&w, sizeof(unsigned int)) != cudaSuccess) return nullptr;
    cudaMemset(w, 0, sizeof(unsigned int));
    words[dev] = w;
  }
  return words[dev];
}

namespace {


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


// ---------------------------------------------------------------- FP4 ----
// E8M0 decode table with the NaN code (255) mapped to 0. FP4 group partials
// are always finite (E2M1 x E4M3-grid products), so fmaf(p, qs*0, acc) ==
// acc: exactly the reference's "skip a NaN-scaled group" (the accumulator
// starts at +0 and can never become -0).
__device__ __forceinline__ void fill_e8m0_skip_table(float* tbl) {
  for (int i = threadIdx.x; i < 256; i += blockDim.x) tbl[i] = i == 255 ? 0.0f : e8m0_decode(i);
}

// Grid: one warp per (item, block of 32/LPR rows); LPR lanes share a row.
// NT = max tokens per item; PAIR streams W[0] and W[1] (gate and up) with
// one activation.
template <int LPR, int NT, bool PAIR>
__global__ void __launch_bounds__(128, NT <= 2 ? 4 : 3) fp4_gemv_kernel(const Fp4GemvArgs a) {
  constexpr int RPW = 32 / LPR;
  constexpr int PF = PAIR ? 3 : 4;  // 32-byte chunks in flight per stream
  __shared__ float e8m0_tbl[256];
  fill_e8m0_skip_table(e8m0_tbl);
  __syncthreads();
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
  const int G = a.in >> 5;                  // 32-column groups per row
  const int NP = G / (2 * LPR);             // 32-byte chunks per lane
  const size_t rb = static_cast<size_t>(a.in) >> 1;
  const uint8_t* wp0 = a.W[0] + it.mat * a.w_stride + rowc * rb + sub * 32;
  const uint8_t* sp0 = a.S[0] + it.mat * a.s_stride + static_cast<size_t>(rowc) * G + sub * 2;
  const uint8_t* wp1 = PAIR ? a.W[1] + it.mat * a.w_stride + rowc * rb + sub * 32 : nullptr;
  const uint8_t* sp1 = PAIR ? a.S[1] + it.mat * a.s_stride + static_cast<size_t>(rowc) * G + sub * 2
                            : nullptr;
  const int sld = (a.act.ld + 127) >> 7;
  const __half* xr[NT];
  const float* xsr[NT];
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    const int xi = (NT == 1 || t < ntok) ? it.tok[t].x : it.tok[0].x;
    xr[t] = a.act.x + static_cast<size_t>(xi) * a.act.ld + sub * 64;
    xsr[t] = a.act.s + static_cast<size_t>(xi) * sld;
  }
  float acc0[NT], acc1[NT];
#pragma unroll
  for (int t = 0; t < NT; ++t) { acc0[t] = 0.0f; acc1[t] = 0.0f; }
  const int base_lane = lane - sub;
  constexpr size_t kStep = static_cast<size_t>(LPR) * 32;  // bytes between a lane's chunks

  auto process = [&](const U8x32& cw0, const U8x32& cw1, int p) {
    const int col0 = (p * LPR + sub) * 64;
    const uint32_t sc0 = *reinterpret_cast<const uint16_t*>(sp0 + p * LPR * 2);
    const float wa0 = e8m0_tbl[sc0 & 0xFFu], wb0 = e8m0_tbl[sc0 >> 8];
    float wa1 = 0.f, wb1 = 0.f;
    if (PAIR) {
      const uint32_t sc1 = *reinterpret_cast<const uint16_t*>(sp1 + p * LPR * 2);
      wa1 = e8m0_tbl[sc1 & 0xFFu];
      wb1 = e8m0_tbl[sc1 >> 8];
    }
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      if (NT == 1 || t < ntok) {
        const __half* xp = xr[t] + static_cast<size_t>(p) * LPR * 64;
        const float qs = xsr[t][col0 >> 7];
        float pa0, pb0, pa1 = 0.f, pb1 = 0.f;
        {
          uint32_t xw[16];
          const U8x32 v0 = ldg32_l1(xp), v1 = ldg32_l1(xp + 16);
#pragma unroll
          for (int k = 0; k < 8; ++k) { xw[k] = v0.w[k]; xw[8 + k] = v1.w[k]; }
          pa0 = fp4_partial16(&cw0.w[0], xw);
          if (PAIR) pa1 = fp4_partial16(&cw1.w[0], xw);
        }
        {
          uint32_t xw[16];
          const U8x32 v0 = ldg32_l1(xp + 32), v1 = ldg32_l1(xp + 48);
#pragma unroll
          for (int k = 0; k < 8; ++k) { xw[k] = v0.w[k]; xw[8 + k] = v1.w[k]; }
          pb0 = fp4_partial16(&cw0.w[4], xw);
          if (PAIR) pb1 = fp4_partial16(&cw1.w[4], xw);
        }
        const float sa0 = qs * wa0, sb0 = qs * wb0;
        float sa1 = 0.f, sb1 = 0.f;
        if (PAIR) {
          sa1 = qs * wa1;
          sb1 = qs * wb1;
        }
        if (LPR == 1) {
          acc0[t] = fmaf(pb0, sb0, fmaf(pa0, sa0, acc0[t]));
          if (PAIR) acc1[t] = fmaf(pb1, sb1, fmaf(pa1, sa1, acc1[t]));
        } else {
#pragma unroll
          for (int s = 0; s < LPR; ++s) {
            const float qa = __shfl_sync(0xffffffffu, pa0, base_lane + s);
            const float ra = __shfl_sync(0xffffffffu, sa0, base_lane + s);
            const float qb = __shfl_sync(0xffffffffu, pb0, base_lane + s);
            const float rb2 = __shfl_sync(0xffffffffu, sb0, base_lane + s);
            acc0[t] = fmaf(qb, rb2, fmaf(qa, ra, acc0[t]));
            if (PAIR) {
              const float ua = __shfl_sync(0xffffffffu, pa1, base_lane + s);
              const float va = __shfl_sync(0xffffffffu, sa1, base_lane + s);
              const float ub = __shfl_sync(0xffffffffu, pb1, base_lane + s);
              const float vb = __shfl_sync(0xffffffffu, sb1, base_lane + s);
              acc1[t] = fmaf(ub, vb, fmaf(ua, va, acc1[t]));
            }
          }
        }
      }
    }
  };

  U8x32 buf0[PF], buf1[PF];
#pragma unroll
  for (int j = 0; j < PF; ++j) {
    if (j < NP) {
      buf0[j] = ldg32(wp0 + j * kStep);
      if (PAIR) buf1[j] = ldg32(wp1 + j * kStep);
    }
  }
  int p = 0;
  for (; p + PF <= NP; p += PF) {
#pragma unroll
    for (int j = 0; j < PF; ++j) {
      const U8x32 c0 = buf0[j];
      U8x32 c1;
      if (PAIR) c1 = buf1[j];
      if (p + j + PF < NP) {
        buf0[j] = ldg32(wp0 + (p + j + PF) * kStep);
        if (PAIR) buf1[j] = ldg32(wp1 + (p + j + PF) * kStep);
      }
      process(c0, c1, p + j);
    }
  }
#pragma unroll
  for (int j = 0; j < PF; ++j)
    if (p + j < NP) process(buf0[j], buf1[j], p + j);

  if (sub == 0 && row_ok) {
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      if (NT == 1 || t < ntok) {
        const size_t yo = static_cast<size_t>(it.tok[t].y) * a.rows + row;
        a.Y[0][yo] = bf16_round(acc0[t]);
        if (PAIR) a.Y[1][yo] = bf16_round(acc1[t]);
      }
    }
  }
}

// -------------------------------------------------------- FP4 stream ----
// Streaming form of the FP4 GEMV for in % 512 == 0. Each warp owns a tile of
// 32 rows (lane = row) and walks it in 512-column chunks. Per chunk, one
// elected lane issues three 2-D TMA box loads (two [32 rows x 128 B] weight
// boxes with the 128-byte swizzle, one [32 x 16 B] box of E8M0 codes) and
// one 1-D bulk copy per token of the activation slice into a per-warp ring of
// kStages shared-memory stages, completed on an mbarrier each. The swizzle
// makes the lane-per-row 16-byte shared loads conflict-free, and every lane
// folds its own row's 32-column partials in column order - the reference's
// accumulation order - with no cross-lane traffic.
constexpr int kSCols = 512;                  // FP4 columns per stage row
constexpr int kSRowBytes = kSCols / 2;       // 256
constexpr int kSGroups = kSCols / 32;        // 16 E8M0 codes per stage row
constexpr int kStages = 2;
constexpr size_t kSplitkSmemCap = 227 * 1024 - 2048;  // dynamic bytes beside the static tables

template <int NT>
struct StreamLayout {
  static constexpr int kW = 32 * kSRowBytes;      // two swizzled [32][128] boxes
  static constexpr int kS = 32 * kSGroups;        // [32][16] codes
  static constexpr int kA = NT * kSCols * 2;      // activations (f16)
  static constexpr int kQ = NT * 16;              // activation scales of the chunk (4 x f32)
  static constexpr int kStage = (kW + kS + kA + kQ + 1023) / 1024 * 1024;  // 1 KB aligned
  static constexpr int kWarpBytes = kStages * kStage;
};

struct Fp4Maps {
  CUtensorMap w[2];  // [rows_total][in/2] bytes, box [32][128], 128B swizzle
  CUtensorMap s[2];  // [rows_total][in/32] codes, box [32][16]
};

// Four 32-column partials with four interleaved (independent) chains: one
// warp keeps four FMAs in flight per four-cycle FMA latency.
__device__ __forceinline__ void fp4_partial16x4(const uint32_t (*w)[4], const uint32_t (*x)[16],
                                                float* p) {
#pragma unroll
  for (int c = 0; c < 4; ++c) p[c] = 0.0f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint32_t h[4][4];
#pragma unroll
    for (int c = 0; c < 4; ++c)
      asm("{ .reg .b8 c0, c1, c2, c3; mov.b32 {c0, c1, c2, c3}, %4;"
          " cvt.rn.f16x2.e2m1x2 %0, c0; cvt.rn.f16x2.e2m1x2 %1, c1;"
          " cvt.rn.f16x2.e2m1x2 %2, c2; cvt.rn.f16x2.e2m1x2 %3, c3; }"
          : "=r"(h[c][0]), "=r"(h[c][1]), "=r"(h[c][2]), "=r"(h[c][3]) : "r"(w[c][i]));
#pragma unroll
    for (int k = 0; k < 4; ++k) {
#pragma unroll
      for (int c = 0; c < 4; ++c) p[c] = fma_h_lo(h[c][k], x[c][4 * i + k], p[c]);
#pragma unroll
      for (int c = 0; c < 4; ++c) p[c] = fma_h_hi(h[c][k], x[c][4 * i + k], p[c]);
    }
  }
}

template <int NT, int WARPS>
__global__ void __launch_bounds__(WARPS * 32, 1)
    fp4_stream_kernel(const __grid_constant__ Fp4Maps maps, const Fp4GemvArgs a, int pair) {
  using L = StreamLayout<NT>;
  extern __shared__ __align__(1024) unsigned char smem[];
  __shared__ float e8m0_tbl[256];
  __shared__ uint64_t bars_all[WARPS][kStages];
  fill_e8m0_skip_table(e8m0_tbl);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // swizzled boxes need 1 KB aligned destinations: the launch adds 1 KB of
  // slack and the base is rounded up here
  unsigned char* const sbase =
      smem + ((1024u - (smem_addr(smem) & 1023u)) & 1023u);
  unsigned char* wbase = sbase + warp * L::kWarpBytes;
  uint64_t* bars = bars_all[warp];
  if (lane == 0) {
#pragma unroll
    for (int s = 0; s < kStages; ++s) mbar_init(&bars[s], 1);
    mbar_fence_init();
    if (warp == 0) {
      tma_prefetch_desc(&maps.w[0]);
      tma_prefetch_desc(&maps.s[0]);
      if (pair) {
        tma_prefetch_desc(&maps.w[1]);
        tma_prefetch_desc(&maps.s[1]);
      }
    }
  }
  __syncthreads();
  pdl_wait();  // the item list and activations come from the previous kernels
  pdl_trigger();

  const int n_items = load_n_items(a.n_items, a.max_items);
  const int V = pair ? 2 : 1;
  const int rblocks = (a.rows + 31) / 32;
  const long long tiles = static_cast<long long>(n_items) * V * rblocks;
  const int CPT = a.in / kSCols;  // chunks per tile
  const long long nwarps = static_cast<long long>(gridDim.x) * WARPS;
  // consecutive tiles go to consecutive CTAs first: equal work per SM
  const long long first = static_cast<long long>(warp) * gridDim.x + blockIdx.x;
  const long long my_tiles = tiles > first ? (tiles - first + nwarps - 1) / nwarps : 0;
  const long long jobs = my_tiles * CPT;
  const int sld = (a.act.ld + 127) >> 7;

  // Job j = (my tile j / CPT, chunk j % CPT). The consumer and the issuer
  // (kStages jobs ahead) each walk their own cursor; a tile's item, matrix
  // and row block are decoded with 32-bit arithmetic once per tile.
  struct Cursor {
    int chunk = 0, tile_n = 0, item = 0, v = 0, rb = 0, mat = 0, ntok = 0;
    int tx[NT], ty[NT];  // the item's token rows (x) and output rows (y)
  };
  const int per_item = V * rblocks;
  const long long my_tile_count = my_tiles;
  auto decode = [&](Cursor& c) {
    if (c.tile_n >= my_tile_count) return;  // past the last job
    const int tile = static_cast<int>(first + static_cast<long long>(c.tile_n) * nwarps);
    c.item = tile / per_item;
    const int rem = tile - c.item * per_item;
    c.v = rem / rblocks;
    c.rb = rem - c.v * rblocks;
    const GemvItem& it = a.items[c.item];
    c.mat = it.mat;
    c.ntok = it.ntok;
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      const int tt = (NT == 1 || t < c.ntok) ? t : 0;
      c.tx[t] = it.tok[tt].x;
      c.ty[t] = it.tok[tt].y;
    }
  };
  auto advance = [&](Cursor& c) {
    if (++c.chunk == CPT) {
      c.chunk = 0;
      ++c.tile_n;
      decode(c);
    }
  };
  Cursor ic;  // issue cursor
  decode(ic);
  int stage_i = 0;
  auto issue = [&]() {
    if (lane == 0) {
      const int ntok = ic.ntok;
      unsigned char* st = wbase + stage_i * L::kStage;
      mbar_arrive_expect_tx(&bars[stage_i],
                            static_cast<uint32_t>(L::kW + L::kS + ntok * (kSCols * 2 + 16)));
      const int y = ic.mat * a.rows + ic.rb * 32;
      const CUtensorMap* wm = ic.v ? &maps.w[1] : &maps.w[0];
      const CUtensorMap* sm = ic.v ? &maps.s[1] : &maps.s[0];
      tma_load_2d(st, wm, ic.chunk * kSRowBytes, y, &bars[stage_i]);
      tma_load_2d(st + L::kW / 2, wm, ic.chunk * kSRowBytes + 128, y, &bars[stage_i]);
      tma_load_2d(st + L::kW, sm, ic.chunk * kSGroups, y, &bars[stage_i]);
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        if (NT == 1 || t < ntok) {
          bulk_g2s(st + L::kW + L::kS + t * kSCols * 2,
                   a.act.x + static_cast<size_t>(ic.tx[t]) * a.act.ld + ic.chunk * kSCols,
                   kSCols * 2, &bars[stage_i]);
          bulk_g2s(st + L::kW + L::kS + L::kA + t * 16,
                   a.act.s + static_cast<size_t>(ic.tx[t]) * sld + ic.chunk * 4, 16,
                   &bars[stage_i]);
        }
      }
    }
    advance(ic);
    stage_i = stage_i + 1 == kStages ? 0 : stage_i + 1;
  };

  float acc[NT];
#pragma unroll
  for (int t = 0; t < NT; ++t) acc[t] = 0.0f;

  for (long long j = 0; j < jobs && j < kStages; ++j) issue();
  __syncwarp();
  bool ok = true;
  long long j = 0;
  Cursor cc;  // consumer cursor
  decode(cc);
  int s = 0;
  uint32_t phase = 0;
  for (; j < jobs; ++j) {
    if (!mbar_wait(&bars[s], phase, a.err)) { ok = false; break; }
    const int chunk = cc.chunk;
    const int v = cc.v, rb = cc.rb;
    const int ntok = cc.ntok;
    const unsigned char* st = wbase + s * L::kStage;
    const unsigned char* wrow = st + lane * 128;
    const int sw = lane & 7;
    const uint4 codes = *reinterpret_cast<const uint4*>(st + L::kW + lane * kSGroups);
    const uint32_t cw[4] = {codes.x, codes.y, codes.z, codes.w};
    float qs[NT][4];
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      const float4 q4 = *reinterpret_cast<const float4*>(
          st + L::kW + L::kS + L::kA + ((NT == 1 || t < ntok) ? t : 0) * 16);
      qs[t][0] = q4.x; qs[t][1] = q4.y; qs[t][2] = q4.z; qs[t][3] = q4.w;
    }
#pragma unroll
    for (int g = 0; g < kSGroups; g += 4) {
      // group g lives in box g/8, 16-byte chunk (g%8) xor (row%8)
      uint32_t w4[4][4];
      float sc[4];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int gc = g + c;
        const uint4 wv = *reinterpret_cast<const uint4*>(wrow + (gc >> 3) * (L::kW / 2) +
                                                         (((gc & 7) ^ sw) << 4));
        w4[c][0] = wv.x; w4[c][1] = wv.y; w4[c][2] = wv.z; w4[c][3] = wv.w;
        sc[c] = e8m0_tbl[(cw[gc >> 2] >> (8 * (gc & 3))) & 0xFFu];
      }
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        if (NT == 1 || t < ntok) {
          const uint4* xg = reinterpret_cast<const uint4*>(st + L::kW + L::kS + t * kSCols * 2 + g * 64);
          uint32_t x4[4][16];
#pragma unroll
          for (int c = 0; c < 4; ++c)
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const uint4 u = xg[4 * c + q];
              x4[c][4 * q] = u.x; x4[c][4 * q + 1] = u.y; x4[c][4 * q + 2] = u.z; x4[c][4 * q + 3] = u.w;
            }
          float p[4];
          fp4_partial16x4(w4, x4, p);
          // group g + c's 128-column activation block is (g + c) / 4 = g / 4
#pragma unroll
          for (int c = 0; c < 4; ++c) acc[t] = fmaf(p[c], qs[t][g >> 2] * sc[c], acc[t]);
        }
      }
    }
    if (chunk == CPT - 1) {
      const int row = rb * 32 + lane;
      if (row < a.rows) {
        float* Yv = v ? a.Y[1] : a.Y[0];
#pragma unroll
        for (int t = 0; t < NT; ++t)
          if (NT == 1 || t < ntok)
            Yv[static_cast<size_t>(cc.ty[t]) * a.rows + row] = bf16_round(acc[t]);
      }
#pragma unroll
      for (int t = 0; t < NT; ++t) acc[t] = 0.0f;
    }
    __syncwarp();
    if (j + kStages < jobs) issue();
    __syncwarp();
    advance(cc);
    if (++s == kStages) {
      s = 0;
      phase ^= 1u;
    }
  }
  if (!ok) {
    // drain this warp's copies still in flight (the failed stage's
    // included) before the CTA exits
    mbar_wait(&bars[s], phase, a.err);
    uint32_t ph = phase;
    int k = s;
    for (long long q = j + 1; q < jobs && q < j + kStages; ++q) {
      if (++k == kStages) { k = 0; ph ^= 1u; }
      mbar_wait(&bars[k], ph, a.err);
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
  const uint16_t* wp = a.W + static_cast<size_t>(it.mat) * a.w_stride + static_cast<size_t>(rowc) * a.in;
  const float* xr[NT];
#pragma unroll
  for (int t = 0; t < NT; ++t)
    xr[t] = a.x + static_cast<size_t>(t < ntok ? it.tok[t].x : it.tok[0].x) * a.ldx;
  float acc[NT];
#pragma unroll
  for (int t = 0; t < NT; ++t) acc[t] = 0.f;
  const int NC = a.in >> 4;  // 16-column chunks
  constexpr int PF = NT == 1 ? 8 : 4;  // 32-byte chunks in flight per lane
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
    const uint16_t* w = a.W + static_cast<size_t>(it.mat) * a.w_stride + static_cast<size_t>(row) * a.in;
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
      const __half g = e4m3_round_f16(q);
      if (qx) qx[static_cast<size_t>(r) * ld_out + b * 128 + i] = g;
      if (qx32) qx32[static_cast<size_t>(r) * ld_out + b * 128 + i] = __half2float(g);
    }
  }
}

// Fused SwiGLU + route weight + BF16 + FP8 quant
// (routed_swiglu_quant, src/dsv4/dsv4_model.c:6257-6286).
__global__ void swiglu_quant_kernel(const float* gate, const float* up, int n, int rows,
                                    const float* weight, int limit, __half* qy, float* qs,
                                    float* ybf) {
  pdl_wait();
  pdl_trigger();
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
      const float silu = g / (1.0f + expf_r1(-g));
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
      qy[o] = e4m3_round_f16(q);
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

// Lanes per row: the largest split (1, 2 or 4 lanes per row) whose warp
// count still fits one resident wave (16 warps per SM at <=128 registers),
// so every row block streams concurrently and no tail wave is left.
int pick_lpr(long long rows_total, int chunks_per_row) {
  const long long wave = 16LL * sm_count();
  int lpr = 1;
  while (lpr < 4 && (rows_total * lpr * 2) / 32 <= wave && chunks_per_row % (4 * lpr) == 0)
    lpr *= 2;
  return lpr;
}

template <int NT, int WARPS>
cudaError_t launch_stream_nt(const Fp4Maps& maps, const Fp4GemvArgs& a, bool pair,
                             cudaStream_t st) {
  const size_t smem = static_cast<size_t>(WARPS) * StreamLayout<NT>::kWarpBytes + 1024;
  {
    cudaError_t e = set_max_dynamic_smem(reinterpret_cast<const void*>(fp4_stream_kernel<NT, WARPS>),
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
  }
  const long long tiles = static_cast<long long>(a.max_items) * (pair ? 2 : 1) *
                          ((a.rows + 31) / 32);
  const int grid = static_cast<int>(std::max<long long>(
      1, std::min<long long>(sm_count(), (tiles + WARPS - 1) / WARPS)));
  Fp4GemvArgs b = a;
  if (!b.err) b.err = device_error_word();
  return launch_pdl(fp4_stream_kernel<NT, WARPS>, dim3(grid), dim3(WARPS * 32), smem, st, maps, b,
                    pair ? 1 : 0);
}


// Tensor maps over every matrix of the launch: rows_total = rows of all
// matrices an item index can select (max mat + 1 experts).
bool fp4_maps(Fp4Maps* m, const Fp4GemvArgs& a, bool pair, long long n_mats, bool cache) {
  const uint64_t rows_total = static_cast<uint64_t>(n_mats) * a.rows;
  for (int v = 0; v < (pair ? 2 : 1); ++v) {
    if (!make_tma_map_u8(&m->w[v], a.W[v], static_cast<uint64_t>(a.in) / 2, rows_total, 128, 32,
                         true, cache))
      return false;
    if (!make_tma_map_u8(&m->s[v], a.S[v], static_cast<uint64_t>(a.in) / 32, rows_total, 16, 32,
                         false, cache))
      return false;
  }
  if (!pair) {
    m->w[1] = m->w[0];
    m->s[1] = m->s[0];
  }
  return true;
}

// -------------------------------------------------------- FP8 stream ----
// Streaming form of the FP8 GEMV (the shared expert, dense projections) for
// one matrix or a pair: in % 512 == 0, at most 64 128-column blocks. Each
// warp owns a tile of 32 rows (lane = row) and walks it in 512-column chunks
// (four 128-column blocks): one elected lane loads four [32 rows x 128 B]
// 128-byte-swizzled TMA boxes, the chunk's activations and their scales into
// a per-warp ring of kF8Stages stages. Each lane runs the four blocks'
// 128-long fmaf chains interleaved and folds them in column order
// (dsv4_model.c:571-676). The tile's 32 rows share one row of
// [128 x 128]-block E8M0 codes, held one per lane and fetched by shuffle.
constexpr int kF8Cols = 512;
constexpr int kF8Blocks = kF8Cols / 128;  // 128-column scale blocks per chunk
constexpr int kF8Stages = 4;

template <int NT>
struct F8Layout {
  static constexpr int kW = kF8Blocks * 32 * 128;  // one swizzled [32][128 B] box per block
  static constexpr int kA = NT * kF8Cols * 2;      // activations (f16)
  static constexpr int kQ = NT * 16;               // 4 activation scales covering the chunk
  static constexpr int kStage = (kW + kA + kQ + 1023) / 1024 * 1024;
  static constexpr int kWarpBytes = kF8Stages * kStage;
};

struct Fp8Maps {
  CUtensorMap w[2];  // [rows][in] bytes, box [32][128], 128B swizzle
};

// 32-value pieces of four independent 128-long chains (one per block).
__device__ __forceinline__ void fp8_step32x4(const uint32_t (*w)[8], const uint32_t (*x)[16],
                                             float* p) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    uint32_t h[4][2];
#pragma unroll
    for (int c = 0; c < 4; ++c)
      asm("{ .reg .b16 lo, hi; mov.b32 {lo, hi}, %2; cvt.rn.f16x2.e4m3x2 %0, lo;"
          " cvt.rn.f16x2.e4m3x2 %1, hi; }"
          : "=r"(h[c][0]), "=r"(h[c][1]) : "r"(w[c][i]));
#pragma unroll
    for (int c = 0; c < 4; ++c) p[c] = fma_h_lo(h[c][0], x[c][2 * i], p[c]);
#pragma unroll
    for (int c = 0; c < 4; ++c) p[c] = fma_h_hi(h[c][0], x[c][2 * i], p[c]);
#pragma unroll
    for (int c = 0; c < 4; ++c) p[c] = fma_h_lo(h[c][1], x[c][2 * i + 1], p[c]);
#pragma unroll
    for (int c = 0; c < 4; ++c) p[c] = fma_h_hi(h[c][1], x[c][2 * i + 1], p[c]);
  }
}

template <int NT, int WARPS>
__global__ void __launch_bounds__(WARPS * 32, 1)
    fp8_stream_kernel(const __grid_constant__ Fp8Maps maps, const Fp8GemvArgs a, int pair,
                      unsigned int* err) {
  using L = F8Layout<NT>;
  extern __shared__ __align__(1024) unsigned char smem[];
  __shared__ float e8m0_tbl[256];
  __shared__ uint64_t bars_all[WARPS][kF8Stages];
  fill_e8m0_skip_table(e8m0_tbl);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  unsigned char* const sbase = smem + ((1024u - (smem_addr(smem) & 1023u)) & 1023u);
  unsigned char* wbase = sbase + warp * L::kWarpBytes;
  uint64_t* bars = bars_all[warp];
  if (lane == 0) {
#pragma unroll
    for (int s = 0; s < kF8Stages; ++s) mbar_init(&bars[s], 1);
    mbar_fence_init();
    if (warp == 0) {
      tma_prefetch_desc(&maps.w[0]);
      if (pair) tma_prefetch_desc(&maps.w[1]);
    }
  }
  __syncthreads();
  pdl_wait();
  pdl_trigger();

  const int n_items = load_n_items(a.n_items, a.max_items);
  const int V = pair ? 2 : 1;
  const int rblocks = a.rows / 32;
  const int per_item = V * rblocks;
  const long long tiles = static_cast<long long>(n_items) * per_item;
  const int CPT = a.in / kF8Cols;
  const int CB = a.in / 128;
  const long long nwarps = static_cast<long long>(gridDim.x) * WARPS;
  const long long first = static_cast<long long>(warp) * gridDim.x + blockIdx.x;
  const long long my_tiles = tiles > first ? (tiles - first + nwarps - 1) / nwarps : 0;
  const long long jobs = my_tiles * CPT;
  const int sld = (a.act.ld + 127) >> 7;

  struct Cursor {
    int chunk = 0, tile_n = 0, item = 0, v = 0, rb = 0, ntok = 0;
    int tx[NT], ty[NT];
  };
  auto decode = [&](Cursor& c) {
    if (c.tile_n >= my_tiles) return;
    const int tile = static_cast<int>(first + static_cast<long long>(c.tile_n) * nwarps);
    c.item = tile / per_item;
    const int rem = tile - c.item * per_item;
    c.v = rem / rblocks;
    c.rb = rem - c.v * rblocks;
    const GemvItem& it = a.items[c.item];
    c.ntok = it.ntok;
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      const int tt = (NT == 1 || t < c.ntok) ? t : 0;
      c.tx[t] = it.tok[tt].x;
      c.ty[t] = it.tok[tt].y;
    }
  };
  auto advance = [&](Cursor& c) {
    if (++c.chunk == CPT) {
      c.chunk = 0;
      ++c.tile_n;
      decode(c);
    }
  };
  Cursor ic;
  decode(ic);
  int stage_i = 0;
  auto issue = [&]() {
    if (lane == 0) {
      unsigned char* st = wbase + stage_i * L::kStage;
      mbar_arrive_expect_tx(&bars[stage_i],
                            static_cast<uint32_t>(L::kW + ic.ntok * (kF8Cols * 2 + 16)));
      const CUtensorMap* wm = ic.v ? &maps.w[1] : &maps.w[0];
      const int y = ic.rb * 32;
#pragma unroll
      for (int q = 0; q < kF8Blocks; ++q)
        tma_load_2d(st + q * (32 * 128), wm, ic.chunk * kF8Cols + q * 128, y, &bars[stage_i]);
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        if (NT == 1 || t < ic.ntok) {
          bulk_g2s(st + L::kW + t * kF8Cols * 2,
                   a.act.x + static_cast<size_t>(ic.tx[t]) * a.act.ld + ic.chunk * kF8Cols,
                   kF8Cols * 2, &bars[stage_i]);
          // the chunk's four activation scales (blocks 4c .. 4c + 3)
          bulk_g2s(st + L::kW + L::kA + t * 16,
                   a.act.s + static_cast<size_t>(ic.tx[t]) * sld + ic.chunk * 4, 16,
                   &bars[stage_i]);
        }
      }
    }
    advance(ic);
    stage_i = stage_i + 1 == kF8Stages ? 0 : stage_i + 1;
  };

  float acc[NT];
#pragma unroll
  for (int t = 0; t < NT; ++t) acc[t] = 0.0f;
  for (long long j = 0; j < jobs && j < kF8Stages; ++j) issue();
  __syncwarp();
  Cursor cc;
  decode(cc);
  // the tile's row of block scale codes: lane l holds blocks l and l + 32
  uint32_t code_lo = 0, code_hi = 0;
  int codes_tile = -1, codes_v = -1;
  bool ok = true;
  long long j = 0;
  int s = 0;
  uint32_t phase = 0;
  for (; j < jobs; ++j) {
    if (cc.tile_n != codes_tile || cc.v != codes_v) {
      const uint8_t* srow = a.S[cc.v] + static_cast<size_t>(cc.rb * 32 / 128) * CB;
      code_lo = lane < CB ? srow[lane] : 255u;
      code_hi = lane + 32 < CB ? srow[lane + 32] : 255u;
      codes_tile = cc.tile_n;
      codes_v = cc.v;
    }
    if (!mbar_wait(&bars[s], phase, err)) { ok = false; break; }
    const int chunk = cc.chunk;
    const int ntok = cc.ntok;
    const unsigned char* st = wbase + s * L::kStage;
    const unsigned char* wrow = st + lane * 128;
    const int sw = lane & 7;
    uint32_t cb[kF8Blocks];
    float wsb[kF8Blocks];
#pragma unroll
    for (int q = 0; q < kF8Blocks; ++q) {
      const int bq = kF8Blocks * chunk + q;
      cb[q] = __shfl_sync(0xffffffffu, bq < 32 ? code_lo : code_hi, bq & 31);
      wsb[q] = e8m0_tbl[cb[q]];
    }
    float pp[NT][kF8Blocks];
#pragma unroll
    for (int t = 0; t < NT; ++t)
#pragma unroll
      for (int q = 0; q < kF8Blocks; ++q) pp[t][q] = 0.f;
#pragma unroll
    for (int pc = 0; pc < 4; ++pc) {  // 32-column pieces of the four blocks
      uint32_t w8[kF8Blocks][8];
#pragma unroll
      for (int q = 0; q < kF8Blocks; ++q)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int ca = 2 * pc + h;  // 16-byte chunk index within the 128-byte block row
          const uint4 v = *reinterpret_cast<const uint4*>(wrow + q * (32 * 128) + ((ca ^ sw) << 4));
          w8[q][4 * h] = v.x; w8[q][4 * h + 1] = v.y; w8[q][4 * h + 2] = v.z; w8[q][4 * h + 3] = v.w;
        }
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        if (NT == 1 || t < ntok) {
          uint32_t x16[kF8Blocks][16];
#pragma unroll
          for (int q = 0; q < kF8Blocks; ++q) {
            const uint4* xq = reinterpret_cast<const uint4*>(st + L::kW + t * kF8Cols * 2 +
                                                             q * 256 + pc * 64);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const uint4 u = xq[k];
              x16[q][4 * k] = u.x; x16[q][4 * k + 1] = u.y; x16[q][4 * k + 2] = u.z;
              x16[q][4 * k + 3] = u.w;
            }
          }
          fp8_step32x4(w8, x16, pp[t]);
        }
      }
    }
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      if (NT == 1 || t < ntok) {
        const float* qv = reinterpret_cast<const float*>(st + L::kW + L::kA + t * 16);
#pragma unroll
        for (int q = 0; q < kF8Blocks; ++q)
          // a NaN block scale (code 255) skips the block, as the reference does
          if (cb[q] != 255u) acc[t] = fmaf(pp[t][q], qv[q] * wsb[q], acc[t]);
      }
    }
    if (chunk == CPT - 1) {
      const int row = cc.rb * 32 + lane;
      float* Yv = cc.v ? a.Y[1] : a.Y[0];
#pragma unroll
      for (int t = 0; t < NT; ++t)
        if (NT == 1 || t < ntok)
          Yv[static_cast<size_t>(cc.ty[t]) * a.rows + row] =
              a.round_out ? bf16_round(acc[t]) : acc[t];
#pragma unroll
      for (int t = 0; t < NT; ++t) acc[t] = 0.0f;
    }
    __syncwarp();
    if (j + kF8Stages < jobs) issue();
    __syncwarp();
    advance(cc);
    if (++s == kF8Stages) {
      s = 0;
      phase ^= 1u;
    }
  }
  if (!ok) {
    // the copies still in flight (the failed stage's included) land first
    mbar_wait(&bars[s], phase, err);
    uint32_t ph = phase;
    int k = s;
    for (long long q = j + 1; q < jobs && q < j + kF8Stages; ++q) {
      if (++k == kF8Stages) { k = 0; ph ^= 1u; }
      mbar_wait(&bars[k], ph, err);
    }
  }
}

template <int NT, int WARPS>
cudaError_t launch_fp8_stream_nt(const Fp8Maps& maps, const Fp8GemvArgs& a, bool pair,
                                 cudaStream_t st) {
  const size_t smem = static_cast<size_t>(WARPS) * F8Layout<NT>::kWarpBytes + 1024;
  {
    cudaError_t e = set_max_dynamic_smem(reinterpret_cast<const void*>(fp8_stream_kernel<NT, WARPS>),
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
  }
  const long long tiles = static_cast<long long>(a.max_items) * (pair ? 2 : 1) * (a.rows / 32);
  const int grid = static_cast<int>(std::max<long long>(
      1, std::min<long long>(sm_count(), (tiles + WARPS - 1) / WARPS)));
  unsigned int* err = a.err ? a.err : device_error_word();
  return launch_pdl(fp8_stream_kernel<NT, WARPS>, dim3(grid), dim3(WARPS * 32), smem, st, maps, a,
                    pair ? 1 : 0, err);
}

// Returns cudaErrorNotSupported when the shape or alignment does not fit
// the streaming kernel (the caller then uses the LDG kernel).
cudaError_t launch_fp8_stream(const Fp8GemvArgs& a, bool pair, int nt, cudaStream_t st,
                              bool map_cache) {
  const int CB = a.in / 128;
  if (a.in % kF8Cols != 0 || CB > 64 || a.rows % 32 != 0 || a.act.ld % 512 != 0 ||
      a.act.x32 || !aligned(a.W[0], 16) || !aligned(a.act.x, 16) || !aligned(a.act.s, 16) ||
      (pair && !aligned(a.W[1], 16)))
    return cudaErrorNotSupported;
  // the item list names one matrix (or pair): every item's mat must be 0
  Fp8Maps maps;
  for (int v = 0; v < (pair ? 2 : 1); ++v)
    if (!make_tma_map_u8(&maps.w[v], a.W[v], static_cast<uint64_t>(a.in), a.rows, 128, 32, true,
                         map_cache))
      return cudaErrorNotSupported;
  if (!pair) maps.w[1] = maps.w[0];
  // Few tiles (one expert): spread them one or two warps per SM, so the
  // per-lane fmaf chains of each tile get a whole SM's issue slots; a launch
  // beside other kernels packs two warps per CTA and leaves SMs to them.
  const long long tiles = static_cast<long long>(a.max_items) * (pair ? 2 : 1) * (a.rows / 32);
  const bool two = a.beside || tiles > sm_count();
  switch (nt) {
    case 1: return two ? launch_fp8_stream_nt<1, 2>(maps, a, pair, st)
                       : launch_fp8_stream_nt<1, 1>(maps, a, pair, st);
    case 2: return two ? launch_fp8_stream_nt<2, 2>(maps, a, pair, st)
                       : launch_fp8_stream_nt<2, 1>(maps, a, pair, st);
    case 3:
    case 4: return two ? launch_fp8_stream_nt<4, 2>(maps, a, pair, st)
                       : launch_fp8_stream_nt<4, 1>(maps, a, pair, st);
    default: return two ? launch_fp8_stream_nt<8, 2>(maps, a, pair, st)
                        : launch_fp8_stream_nt<8, 1>(maps, a, pair, st);
  }
}

// ------------------------------------------------- FP4 split-K stream ----
// Single-token form of the FP4 GEMV with the columns of every 32-row tile
// split over a CTA's CW compute warps. Warp w streams chunks
// [w CPT / CW, (w + 1) CPT / CW) of each of the CTA's tiles through its own
// two-stage TMA ring (as fp4_stream_kernel does) and writes the 32-column
// group partials and the rows' E8M0 codes to shared memory; a fold warp then
// folds each row's partials in column order - the reference's sequential
// fmaf fold - and writes the row. Two partial buffers let the compute warps
// fill tile k + 1 while tile k is folded. With the tile's columns spread
// over the CTA, a launch with few tiles (one expert per GPU under expert
// parallelism, or a down projection's last wave) still keeps every SM busy.
template <int CW>
__global__ void __launch_bounds__((CW + 1) * 32, 1)
    fp4_splitk_kernel(const __grid_constant__ Fp4Maps maps, const Fp4GemvArgs a, int pair) {
  using L = StreamLayout<1>;
  extern __shared__ __align__(1024) unsigned char smem[];
  __shared__ float e8m0_tbl[256];
  __shared__ uint64_t sbar[CW][kStages];
  __shared__ uint64_t full_bar[2], empty_bar[2];
  __shared__ float qsb[64];
  __shared__ int abort_flag;
  fill_e8m0_skip_table(e8m0_tbl);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  unsigned char* const sbase = smem + ((1024u - (smem_addr(smem) & 1023u)) & 1023u);
  const int G = a.in / 32, CPT = a.in / kSCols;
  float* pbuf = reinterpret_cast<float*>(sbase + CW * L::kWarpBytes);  // [2][G][32]
  uint4* cbuf = reinterpret_cast<uint4*>(pbuf + 2 * G * 32);          // [2][CPT][32]
  if (threadIdx.x == 0) {
    for (int w = 0; w < CW; ++w)
      for (int s = 0; s < kStages; ++s) mbar_init(&sbar[w][s], 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&full_bar[s], CW);
      mbar_init(&empty_bar[s], 1);
    }
    abort_flag = 0;
    mbar_fence_init();
    tma_prefetch_desc(&maps.w[0]);
    tma_prefetch_desc(&maps.s[0]);
    if (pair) {
      tma_prefetch_desc(&maps.w[1]);
      tma_prefetch_desc(&maps.s[1]);
    }
  }
  __syncthreads();
  pdl_wait();
  pdl_trigger();
  volatile int* abort_v = &abort_flag;
  auto wait_bar = [&](uint64_t* bar, uint32_t parity) -> bool {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = global_timer_ns();
    while (!mbar_try_wait(bar, parity)) {
      if (*abort_v) return false;
      if (global_timer_ns() - t0 > kWaitLimitNs) {
        if (a.err) atomicOr(a.err, 1u);
        *abort_v = 1;
        return false;
      }
    }
    return true;
  };

  const int n_items = load_n_items(a.n_items, a.max_items);
  const int V = pair ? 2 : 1;
  const int rblocks = (a.rows + 31) / 32;
  const int per_item = V * rblocks;
  const int tiles = n_items * per_item;
  const int n_my = tiles > static_cast<int>(blockIdx.x)
                       ? (tiles - static_cast<int>(blockIdx.x) + gridDim.x - 1) / gridDim.x : 0;
  const int sld = (a.act.ld + 127) >> 7;
  struct TileInfo {
    int item, v, rb, mat, tx, ty;
  };
  auto tile_info = [&](int k) {
    TileInfo ti;
    const int tile = static_cast<int>(blockIdx.x) + k * static_cast<int>(gridDim.x);
    ti.item = tile / per_item;
    const int rem = tile - ti.item * per_item;
    ti.v = rem / rblocks;
    ti.rb = rem - ti.v * rblocks;
    const GemvItem& it = a.items[ti.item];
    ti.mat = it.mat;
    ti.tx = it.tok[0].x;
    ti.ty = it.tok[0].y;
    return ti;
  };

  if (warp < CW) {
    // ------------------------------------------------------ compute warp
    const int c_lo = (warp * CPT) / CW, c_hi = ((warp + 1) * CPT) / CW;
    const int n_seg = c_hi - c_lo;
    const int jobs = n_my * n_seg;
    unsigned char* wbase = sbase + warp * L::kWarpBytes;
    uint64_t* bars = sbar[warp];
    // issue cursor
    int i_k = 0, i_c = c_lo, stage_i = 0;
    TileInfo i_ti{};
    if (jobs > 0) i_ti = tile_info(0);
    auto issue = [&]() {
      if (lane == 0) {
        unsigned char* st = wbase + stage_i * L::kStage;
        mbar_arrive_expect_tx(&bars[stage_i], static_cast<uint32_t>(L::kW + L::kS + kSCols * 2));
        const int y = i_ti.mat * a.rows + i_ti.rb * 32;
        const CUtensorMap* wm = i_ti.v ? &maps.w[1] : &maps.w[0];
        const CUtensorMap* sm = i_ti.v ? &maps.s[1] : &maps.s[0];
        tma_load_2d(st, wm, i_c * kSRowBytes, y, &bars[stage_i]);
        tma_load_2d(st + L::kW / 2, wm, i_c * kSRowBytes + 128, y, &bars[stage_i]);
        tma_load_2d(st + L::kW, sm, i_c * kSGroups, y, &bars[stage_i]);
        bulk_g2s(st + L::kW + L::kS,
                 a.act.x + static_cast<size_t>(i_ti.tx) * a.act.ld + i_c * kSCols, kSCols * 2,
                 &bars[stage_i]);
      }
      if (++i_c == c_hi) {
        i_c = c_lo;
        if (++i_k < n_my) i_ti = tile_info(i_k);
      }
      stage_i = stage_i + 1 == kStages ? 0 : stage_i + 1;
    };
    for (int j = 0; j < jobs && j < kStages; ++j) issue();
    __syncwarp();
    int k = 0, c = c_lo, s = 0;
    uint32_t phase = 0;
    int j = 0;
    bool ok = true;
    for (; j < jobs; ++j) {
      const int slot = k & 1;
      if (c == c_lo && k >= 2 && !wait_bar(&empty_bar[slot], ((k - 2) >> 1) & 1)) { ok = false; break; }
      if (!wait_bar(&bars[s], phase)) { ok = false; break; }
      const unsigned char* st = wbase + s * L::kStage;
      const unsigned char* wrow = st + lane * 128;
      const int sw = lane & 7;
      cbuf[(slot * CPT + c) * 32 + lane] = *reinterpret_cast<const uint4*>(st + L::kW + lane * kSGroups);
      float* pout = pbuf + (static_cast<size_t>(slot) * G + c * kSGroups) * 32 + lane;
      const unsigned char* xt = st + L::kW + L::kS;
#pragma unroll
      for (int g = 0; g < kSGroups; g += 4) {
        uint32_t w4[4][4];
        uint32_t x4[4][16];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int gq = g + q;
          const uint4 wv = *reinterpret_cast<const uint4*>(wrow + (gq >> 3) * (L::kW / 2) +
                                                           (((gq & 7) ^ sw) << 4));
          w4[q][0] = wv.x; w4[q][1] = wv.y; w4[q][2] = wv.z; w4[q][3] = wv.w;
          const uint4* xg = reinterpret_cast<const uint4*>(xt + gq * 64);
#pragma unroll
          for (int r = 0; r < 4; ++r) {
            const uint4 u = xg[r];
            x4[q][4 * r] = u.x; x4[q][4 * r + 1] = u.y; x4[q][4 * r + 2] = u.z; x4[q][4 * r + 3] = u.w;
          }
        }
        float p[4];
        fp4_partial16x4(w4, x4, p);
#pragma unroll
        for (int q = 0; q < 4; ++q) pout[(g + q) * 32] = p[q];
      }
      __syncwarp();
      if (c + 1 == c_hi && lane == 0) mbar_arrive(&full_bar[slot]);
      if (j + kStages < jobs) issue();
      __syncwarp();
      if (++c == c_hi) {
        c = c_lo;
        ++k;
      }
      if (++s == kStages) {
        s = 0;
        phase ^= 1u;
      }
    }
    if (!ok) {
      // the copies still in flight (the failed stage's included) land first
      mbar_wait(&bars[s], phase, a.err);
      uint32_t ph = phase;
      int q = s;
      for (int jj = j + 1; jj < jobs && jj < j + kStages; ++jj) {
        if (++q == kStages) { q = 0; ph ^= 1u; }
        mbar_wait(&bars[q], ph, a.err);
      }
    }
  } else {
    // --------------------------------------------------------- fold warp
    for (int k = 0; k < n_my; ++k) {
      const int slot = k & 1;
      const TileInfo ti = tile_info(k);
      const float* qrow = a.act.s + static_cast<size_t>(ti.tx) * sld;
      for (int b = lane; b < G / 4; b += 32) qsb[b] = qrow[b];
      if (!wait_bar(&full_bar[slot], (k >> 1) & 1)) break;
      __syncwarp();
      const float* pin = pbuf + static_cast<size_t>(slot) * G * 32 + lane;
      const unsigned char* cb = reinterpret_cast<const unsigned char*>(cbuf + slot * CPT * 32);
      float acc = 0.0f;
      for (int c = 0; c < CPT; ++c) {
        const uint4 codes = *reinterpret_cast<const uint4*>(cb + (c * 32 + lane) * 16);
        const uint32_t cw[4] = {codes.x, codes.y, codes.z, codes.w};
#pragma unroll
        for (int g = 0; g < kSGroups; ++g) {
          const int gg = c * kSGroups + g;
          const float sc = e8m0_tbl[(cw[g >> 2] >> (8 * (g & 3))) & 0xFFu];
          acc = fmaf(pin[gg * 32], qsb[gg >> 2] * sc, acc);
        }
      }
      const int row = ti.rb * 32 + lane;
      if (row < a.rows) {
        float* Yv = ti.v ? a.Y[1] : a.Y[0];
        Yv[static_cast<size_t>(ti.ty) * a.rows + row] = bf16_round(acc);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty_bar[slot]);
    }
  }
}

template <int CW>
cudaError_t launch_splitk_cw(const Fp4Maps& maps, const Fp4GemvArgs& a, bool pair,
                             cudaStream_t st) {
  const int G = a.in / 32, CPT = a.in / kSCols;
  const size_t smem = static_cast<size_t>(CW) * StreamLayout<1>::kWarpBytes +
                      2 * static_cast<size_t>(G) * 32 * sizeof(float) +
                      2 * static_cast<size_t>(CPT) * 32 * 16 + 1024;
  {
    cudaError_t e = set_max_dynamic_smem(reinterpret_cast<const void*>(fp4_splitk_kernel<CW>),
                                         static_cast<int>(kSplitkSmemCap));
    if (e != cudaSuccess) return e;
  }
  if (smem > kSplitkSmemCap) return cudaErrorNotSupported;
  const long long tiles = static_cast<long long>(a.max_items) * (pair ? 2 : 1) * ((a.rows + 31) / 32);
  const int per_sm = smem * 2 + 4096 <= 232448 ? 2 : 1;
  const int grid = static_cast<int>(std::max<long long>(
      1, std::min<long long>(static_cast<long long>(sm_count()) * per_sm, tiles)));
  Fp4GemvArgs b = a;
  if (!b.err) b.err = device_error_word();
  return launch_pdl(fp4_splitk_kernel<CW>, dim3(grid), dim3((CW + 1) * 32), smem, st, maps, b,
                    pair ? 1 : 0);
}

cudaError_t launch_fp4_stream(const Fp4GemvArgs& a, bool pair, int nt, cudaStream_t st,
                              bool map_cache) {
  Fp4Maps maps;
  // matrices are w_stride apart; n_mats must cover every `mat` an item names
  const long long n_mats = a.n_mats > 0 ? a.n_mats : 1;
  if (!fp4_maps(&maps, a, pair, n_mats, map_cache)) return cudaErrorInvalidValue;
  const long long tiles = static_cast<long long>(a.max_items) * (pair ? 2 : 1) * ((a.rows + 31) / 32);
  // single matrices up to six tiles per SM (down projections), pairs below
  // four (a pair's two chains per tile fill an SM on their own)
  if (nt == 1 && a.in / 32 <= 256 && tiles <= (pair ? 4LL : 6LL) * sm_count() &&
      (pair ? tiles < 4LL * sm_count() : true)) {
    // one token per item and few tiles (one to four experts, e.g. a GPU's
    // share under expert parallelism): split every tile's columns over a
    // CTA's warps so the launch still covers every SM
    const int CPT = a.in / kSCols;
    cudaError_t e = cudaErrorNotSupported;
    if (CPT >= 7) e = launch_splitk_cw<7>(maps, a, pair, st);
    else if (CPT >= 4) e = launch_splitk_cw<4>(maps, a, pair, st);
    else if (CPT >= 2) e = launch_splitk_cw<2>(maps, a, pair, st);
    if (e != cudaErrorNotSupported) return e;
  }
  switch (nt) {
    case 1: return launch_stream_nt<1, 8>(maps, a, pair, st);
    case 2: return launch_stream_nt<2, 8>(maps, a, pair, st);
    case 3:
    case 4: return launch_stream_nt<4, 8>(maps, a, pair, st);
    default: return launch_stream_nt<8, 6>(maps, a, pair, st);
  }
}

}  // namespace

cudaError_t launch_fp4_gemv(const Fp4GemvArgs& a, bool pair, int item_tokens, cudaStream_t st,
                            bool map_cache) {
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
  // the streaming kernel needs 512-column chunks, matrices stacked at their
  // natural pitch (so one tensor map covers them) and 16-byte alignment
  const bool stacked = (a.n_mats <= 1) ||
                       (a.w_stride == static_cast<size_t>(a.rows) * (a.in / 2) &&
                        a.s_stride == static_cast<size_t>(a.rows) * (a.in / 32));
  if (a.in % kSCols == 0 && stacked && aligned(a.W[0], 16) && aligned(a.S[0], 16) &&
      a.act.ld % kSCols == 0 && aligned(a.act.x, 16) && aligned(a.act.s, 16) &&
      (!pair || (aligned(a.W[1], 16) && aligned(a.S[1], 16)))) {
    cudaError_t e = launch_fp4_stream(a, pair, item_tokens, st, map_cache);
    if (e != cudaErrorInvalidValue) return e;  // else: map rejected, use the LDG kernel
  }
  const int G = a.in / 32;
  const int lpr = pick_lpr(static_cast<long long>(a.max_items) * a.rows, G);
  if (pair) {
    if (lpr == 4) return fp4_dispatch_nt<4, true>(a, item_tokens, st);
    if (lpr == 2) return fp4_dispatch_nt<2, true>(a, item_tokens, st);
    return fp4_dispatch_nt<1, true>(a, item_tokens, st);
  }
  if (lpr == 4) return fp4_dispatch_nt<4, false>(a, item_tokens, st);
  if (lpr == 2) return fp4_dispatch_nt<2, false>(a, item_tokens, st);
  return fp4_dispatch_nt<1, false>(a, item_tokens, st);
}

cudaError_t launch_fp8_gemv(const Fp8GemvArgs& a, bool pair, int item_tokens, cudaStream_t st,
                            bool map_cache) {
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
  {
    cudaError_t e = launch_fp8_stream(a, pair, item_tokens, st, map_cache);
    if (e != cudaErrorNotSupported) return e;
  }
  const int CB = a.in / 128;
  int lpr = pick_lpr(static_cast<long long>(a.max_items) * a.rows, 2 * CB);
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

// ------------------------------------------------------ FP8 split-K ----
// One-token FP8 GEMV with every 128-column block's partial computed
// independently (the decode step's projections, whose few row tiles leave
// most SMs idle when a warp walks a whole row): kernel A gives each warp 32
// rows (lane = row) x `bps` consecutive blocks and writes the blocks'
// sequential fmaf partials to part[block][row]; kernel B folds each row's
// partials in block order, acc = fmaf(partial, qscale * ws, acc) with
// NaN-scaled blocks skipped, as dsv4_gemv_fp8_q does
// (src/dsv4/dsv4_model.c:657-672). Same operations in the same order as the
// other FP8 kernels, so the same bits.
__global__ void __launch_bounds__(128) fp8_partials_kernel(const Fp8GemvArgs a, int bps,
                                                           float* part, unsigned int* tile_cnt) {
  __shared__ __align__(16) __half xsm[4][kPartMaxBps * 128];  // per warp: its quantised blocks
  pdl_trigger();
  const Fp8Unit u = fp8_unit(a, bps, (blockIdx.x * blockDim.x + threadIdx.x) >> 5);
  U8x32 w[4];
  if (u.valid) fp8_unit_preload(u, w);
  pdl_wait();
  if (u.valid) fp8_unit_run(a, bps, part, tile_cnt, u, w, xsm[threadIdx.x >> 5]);
}

__global__ void __launch_bounds__(128) fp8_fold_kernel(const Fp8GemvArgs a, const float* part) {
  pdl_trigger();
  pdl_wait();
  const int total = a.rows + a.rows1;
  const int row = blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= total) return;
  const int mat = row >= a.rows;
  const int lrow = mat ? row - a.rows : row;
  const int CB = a.in / 128;
  const GemvItem& it = a.items[0];
  const float* qs = a.act.s + static_cast<size_t>(it.tok[0].x) * (a.act.ld / 128);
  const uint8_t* sr = a.S[mat] + static_cast<size_t>(lrow / 128) * ((a.in + 127) / 128);
  float acc = 0.0f;
  for (int b0 = 0; b0 < CB; b0 += 8) {
    float pv[8], sv[8];
    uint32_t code[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int b = b0 + j < CB ? b0 + j : CB - 1;
      pv[j] = part[static_cast<size_t>(b) * total + row];
      sv[j] = qs[b];
      code[j] = sr[b];
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (b0 + j >= CB) break;
      const float ws = e8m0_decode(code[j]);
      if (!isnan(ws)) acc = fmaf(pv[j], sv[j] * ws, acc);
    }
  }
  const int rows_m = mat ? a.rows1 : a.rows;
  a.Y[mat][static_cast<size_t>(it.tok[0].y) * rows_m + lrow] = a.round_out ? bf16_round(acc) : acc;
}

// ------------------------------------------------------- BF16 stream ----
// Streaming BF16 GEMV for one-token items (the decode step's grouped wo_a and
// vocab head). A warp owns 32 rows (lane = row) and walks them in 256-column
// chunks through a ring of STAGES shared-memory stages: per chunk one lane
// issues four 2-D TMA boxes of [32 rows x 128 B] with the 128-byte swizzle
// (the matrix read 128 contiguous bytes per row at a time; the swizzle makes
// the lanes' 16-byte reads conflict-free) and a bulk copy of the chunk's
// fp32 activations, completed on the stage's mbarrier (bounded wait). Each
// lane runs its row's fmaf chain in column order, the reference's order, so
// the result is the LDG kernel's bit for bit.

template <int WARPS, int STAGES>
__global__ void __launch_bounds__(WARPS * 32, 1)
    bf16_stream_kernel(const __grid_constant__ CUtensorMap wmap, const Bf16GemvArgs a,
                       unsigned int* err) {
  extern __shared__ __align__(1024) unsigned char smem[];
  __shared__ uint64_t bars_all[WARPS][STAGES];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  unsigned char* const sbase = smem + ((1024u - (smem_addr(smem) & 1023u)) & 1023u);
  uint64_t* bars = bars_all[warp];
  if (lane == 0) {
#pragma unroll
    for (int q = 0; q < STAGES; ++q) mbar_init(&bars[q], 1);
    mbar_fence_init();
    if (warp == 0) tma_prefetch_desc(&wmap);
  }
  __syncthreads();
  pdl_trigger();
  bf16_stream_warp<STAGES>(&wmap, a, static_cast<long long>(warp) * gridDim.x + blockIdx.x,
                           static_cast<long long>(gridDim.x) * WARPS,
                           sbase + static_cast<size_t>(warp) * STAGES * kBStage, bars, err,
                           [] { pdl_wait(); });
}


int device_sm_count() { return sm_count(); }

int fp8_splitk_bps(const Fp8GemvArgs& a) {
  const int total = a.rows + a.rows1;
  if (total <= 0 || total % 32 != 0 || a.in % 128 != 0) return 0;
  const int CB = a.in / 128, tiles = total / 32;
  // about 16 warps per SM, at least one block per warp
  const long long target = 16LL * sm_count();
  int bps = static_cast<int>(std::max<long long>(1, (static_cast<long long>(tiles) * CB + target - 1) / target));
  bps = std::min(bps, CB);
  return a.xf && bps > kPartMaxBps ? 0 : bps;
}

cudaError_t launch_fp8_gemv_splitk(const Fp8GemvArgs& a, float* part, cudaStream_t st,
                                   unsigned int* tile_cnt) {
  if (a.rows <= 0) return cudaSuccess;
  if (a.rows % 32 != 0 || a.in % 128 != 0 || !aligned(a.W[0], 32) || !aligned(a.act.x, 32) ||
      a.act.ld % 128 != 0 || a.act.x32 || a.max_items != 1 || a.rows1 < 0 || a.rows1 % 32 != 0 ||
      (a.rows1 > 0 && !aligned(a.W[1], 32)))
    return cudaErrorNotSupported;
  const int total = a.rows + a.rows1;
  const int CB = a.in / 128, tiles = total / 32;
  if (a.xf && (!tile_cnt || a.rows1 != 0)) return cudaErrorNotSupported;
  const int bps = fp8_splitk_bps(a);
  if (bps <= 0) return cudaErrorNotSupported;
  const int nseg = (CB + bps - 1) / bps;
  const long long warps = static_cast<long long>(tiles) * nseg;
  cudaError_t e = launch_pdl(fp8_partials_kernel, dim3(static_cast<unsigned>((warps + 3) / 4)),
                             dim3(128), 0, st, a, bps, part, tile_cnt);
  if (e != cudaSuccess || tile_cnt) return e;
  return launch_pdl(fp8_fold_kernel, dim3((total + 127) / 128), dim3(128), 0, st, a,
                    static_cast<const float*>(part));
}

cudaError_t launch_bf16_gemv(const Bf16GemvArgs& a, int item_tokens, cudaStream_t st) {
  if (a.rows <= 0 || a.max_items <= 0) return cudaSuccess;
  // few row tiles (grouped projections): the streaming kernel keeps more
  // bytes in flight per warp; many tiles (the vocab head): the LDG kernel's
  // full occupancy does better
  // the streaming kernel when the matrices are stacked at their natural pitch
  // (one tensor map covers every item's matrix)
  const long long n_mats = a.w_stride ? a.max_items : 1;
  if (item_tokens == 1 && a.rows % 32 == 0 && a.in % kBCols == 0 && aligned(a.W, 16) &&
      (a.w_stride == 0 || a.w_stride == static_cast<size_t>(a.rows) * a.in) && aligned(a.x, 16) &&
      a.ldx % 4 == 0) {
    CUtensorMap wmap;
    if (make_tma_map_u8(&wmap, a.W, static_cast<uint64_t>(a.in) * 2,
                        static_cast<uint64_t>(n_mats) * a.rows, 128, 32, true)) {
      const long long tiles = static_cast<long long>(a.max_items) * (a.rows / 32);
      // few tiles (grouped wo_a): two warps per SM, each with a deep ring
      // (a warp's 32 fmaf chains are latency-bound, so its copies must run
      // far ahead); many tiles (the vocab head): four warps, three stages
      auto run = [&](auto kern, int warps, int stages) -> cudaError_t {
        const size_t smem = static_cast<size_t>(warps) * stages * kBStage + 1024;
        cudaError_t e = set_max_dynamic_smem(reinterpret_cast<const void*>(kern), static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        const int grid = static_cast<int>(std::max<long long>(
            1, std::min<long long>(sm_count(), (tiles + warps - 1) / warps)));
        return launch_pdl(kern, dim3(grid), dim3(warps * 32), smem, st, wmap, a, device_error_word());
      };
      if (tiles <= 2LL * sm_count()) return run(bf16_stream_kernel<2, 6>, 2, 6);
      return run(bf16_stream_kernel<4, 3>, 4, 3);
    }
  }
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
  return launch_pdl(swiglu_quant_kernel, dim3(blocks_for_warps(warps)), dim3(128), 0, st, gate,
                    up, n, rows, weight, limit, qy, qs, y_bf16);
}

cudaError_t launch_f32_to_f16(const float* x, __half* y, size_t n, cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  const int grid = static_cast<int>(std::min<size_t>((n + 255) / 256, 4096));
  f32_to_f16_kernel<<<grid, 256, 0, st>>>(x, y, n);
  return cudaGetLastError();
}

// ------------------------------------------- multi-token (verify rows) ----
// The verify step's projections run 2..8 token rows through one matrix. The
// one-token kernels keep a warp per 32 output rows, which leaves most SMs
// idle when there are few row tiles and the per-byte work is several
// tokens' FMAs. These two forms spread the work the other way while keeping
// each output's reference order.
//
// FP8 (dsv4_gemv_fp8_batch_q, src/dsv4/dsv4_model.c:678): every 128-column
// block's partial is an independent sequential chain, so a warp takes 32
// rows x `bps` blocks, converts each block's weights to f16 once, and runs
// the block's chain for every token (part[t][block][row]); the fold then
// sums each (token, row) over the blocks in block order,
// acc = fmaf(partial, qscale * ws, acc), NaN-scaled blocks skipped. W[1] /
// rows1 is an optional second matrix on the same input (wq_a beside wkv).
template <int NT>
__global__ void __launch_bounds__(128) fp8_mt_partials_kernel(const Fp8GemvArgs a, int ntok,
                                                              int bps, float* part) {
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const long long gw = (blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x) >> 5;
  const int CB = a.in / 128, total = a.rows + a.rows1;
  const int nseg = (CB + bps - 1) / bps;
  if (gw >= static_cast<long long>(total / 32) * nseg) return;
  const int tile = static_cast<int>(gw / nseg), seg = static_cast<int>(gw % nseg);
  const int row = tile * 32 + lane;
  const int mat = row >= a.rows;
  const uint8_t* wr = a.W[mat] + static_cast<size_t>(mat ? row - a.rows : row) * a.in;
  const int b0 = seg * bps, b1 = min(CB, b0 + bps);
  U8x32 w[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) w[k] = ldg32(wr + static_cast<size_t>(b0) * 128 + 32 * k);
  pdl_wait();
  const GemvItem& it = a.items[0];
  for (int b = b0; b < b1; ++b) {
    uint32_t wh[64];  // the block's 128 codes as f16 pairs, in column order
#pragma unroll
    for (int k = 0; k < 4; ++k)
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        wh[k * 16 + 2 * i] = e4m3x2_to_f16x2(w[k].w[i] & 0xFFFFu);
        wh[k * 16 + 2 * i + 1] = e4m3x2_to_f16x2(w[k].w[i] >> 16);
      }
    if (b + 1 < b1) {
#pragma unroll
      for (int k = 0; k < 4; ++k) w[k] = ldg32(wr + static_cast<size_t>(b + 1) * 128 + 32 * k);
    }
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      if (t >= ntok) break;
      const __half* xr = a.act.x + static_cast<size_t>(it.tok[t].x) * a.act.ld + b * 128;
      float p = 0.0f;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const U8x32 x0 = ldg32_l1(xr + 32 * k);
        const U8x32 x1 = ldg32_l1(xr + 32 * k + 16);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const uint32_t xv = i < 8 ? x0.w[i] : x1.w[i - 8];
          p = fma_h_lo(wh[k * 16 + i], xv, p);
          p = fma_h_hi(wh[k * 16 + i], xv, p);
        }
      }
      part[(static_cast<size_t>(t) * CB + b) * total + row] = p;
    }
  }
}

__global__ void __launch_bounds__(128) fp8_mt_fold_kernel(const Fp8GemvArgs a, int ntok,
                                                          const float* part) {
  pdl_trigger();
  pdl_wait();
  const int total = a.rows + a.rows1;
  const long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  if (i >= static_cast<long long>(ntok) * total) return;
  const int t = static_cast<int>(i / total), row = static_cast<int>(i % total);
  const int mat = row >= a.rows;
  const int lrow = mat ? row - a.rows : row;
  const int CB = a.in / 128;
  const GemvItem& it = a.items[0];
  const float* qs = a.act.s + static_cast<size_t>(it.tok[t].x) * (a.act.ld / 128);
  const uint8_t* sr = a.S[mat] + static_cast<size_t>(lrow / 128) * ((a.in + 127) / 128);
  const float* pp = part + static_cast<size_t>(t) * CB * total + row;
  float acc = 0.0f;
  for (int b0 = 0; b0 < CB; b0 += 8) {
    float pv[8], sv[8];
    uint32_t code[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int b = b0 + j < CB ? b0 + j : CB - 1;
      pv[j] = pp[static_cast<size_t>(b) * total];
      sv[j] = qs[b];
      code[j] = sr[b];
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (b0 + j >= CB) break;
      const float ws = e8m0_decode(code[j]);
      if (!isnan(ws)) acc = fmaf(pv[j], sv[j] * ws, acc);
    }
  }
  const int rows_m = mat ? a.rows1 : a.rows;
  a.Y[mat][static_cast<size_t>(it.tok[t].y) * rows_m + lrow] = a.round_out ? bf16_round(acc) : acc;
}

// BF16 (dsv4_gemv_bf16_batch, :308; the grouped wo_a :371): one fmaf chain
// per (row, token) over all columns in column order, so the columns cannot
// be split. The streaming form of the one-token kernel (a warp owns 32 rows,
// lane = row, 256-column chunks of four swizzled [32 rows x 128 B] TMA
// boxes through a ring of shared-memory stages) with the chunk's
// activations of every token beside the weights: each weight is widened
// once and feeds NT independent chains, which also hide the FMA latency.
template <int NT>
__host__ __device__ constexpr int bf16_mt_stage() { return kBW + NT * kBCols * 4; }

template <int STAGES, int NT>
__device__ void bf16_stream_mt_warp(const CUtensorMap* wmapp, const Bf16GemvArgs& a, int ntok,
                                    long long first, long long nwarps, unsigned char* wbase,
                                    uint64_t* bars, unsigned int* err) {
  constexpr int kStage = bf16_mt_stage<NT>();
  const CUtensorMap& wmap = *wmapp;
  const int lane = threadIdx.x & 31;
  const int n_items = load_n_items(a.n_items, a.max_items);
  const int rblocks = a.rows / 32;
  const long long tiles = static_cast<long long>(n_items) * rblocks;
  const int CPT = a.in / kBCols;
  const long long my_tiles = tiles > first ? (tiles - first + nwarps - 1) / nwarps : 0;
  const long long jobs = my_tiles * CPT;
  const uint32_t bytes = kBW + static_cast<uint32_t>(ntok) * kBCols * 4;
  auto issue = [&](long long j, int q) {
    if (lane != 0) return;
    const long long tile = first + (j / CPT) * nwarps;
    const int chunk = static_cast<int>(j % CPT);
    const int item = static_cast<int>(tile / rblocks);
    const int rb = static_cast<int>(tile - static_cast<long long>(item) * rblocks);
    const GemvItem& it = a.items[item];
    unsigned char* st = wbase + q * kStage;
    mbar_arrive_expect_tx(&bars[q], bytes);
    const int y = it.mat * a.rows + rb * 32;
#pragma unroll
    for (int k = 0; k < 4; ++k) tma_load_2d(st + k * 4096, &wmap, chunk * 512 + k * 128, y, &bars[q]);
    for (int t = 0; t < ntok; ++t)
      bulk_g2s(st + kBW + t * kBCols * 4,
               a.x + static_cast<size_t>(it.tok[t].x) * a.ldx + chunk * kBCols, kBCols * 4, &bars[q]);
  };
  for (long long j = 0; j < jobs && j < STAGES; ++j) issue(j, static_cast<int>(j));
  __syncwarp();
  float acc[NT];
#pragma unroll
  for (int t = 0; t < NT; ++t) acc[t] = 0.0f;
  int q = 0;
  uint32_t phase = 0;
  long long j = 0;
  bool ok = true;
  const int sw = lane & 7;
  for (; j < jobs; ++j) {
    if (!mbar_wait(&bars[q], phase, err)) { ok = false; break; }
    const unsigned char* st = wbase + q * kStage;
    const float4* xs = reinterpret_cast<const float4*>(st + kBW);
#pragma unroll 4
    for (int p = 0; p < 32; ++p) {
      const uint4 w8 = *reinterpret_cast<const uint4*>(st + (p >> 3) * 4096 + lane * 128 +
                                                       (((p & 7) ^ sw) << 4));
      const float wf[8] = {__uint_as_float(w8.x << 16), __uint_as_float(w8.x & 0xFFFF0000u),
                           __uint_as_float(w8.y << 16), __uint_as_float(w8.y & 0xFFFF0000u),
                           __uint_as_float(w8.z << 16), __uint_as_float(w8.z & 0xFFFF0000u),
                           __uint_as_float(w8.w << 16), __uint_as_float(w8.w & 0xFFFF0000u)};
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        const float4 x0 = xs[t * (kBCols / 4) + 2 * p], x1 = xs[t * (kBCols / 4) + 2 * p + 1];
        acc[t] = fmaf(wf[0], x0.x, acc[t]);
        acc[t] = fmaf(wf[1], x0.y, acc[t]);
        acc[t] = fmaf(wf[2], x0.z, acc[t]);
        acc[t] = fmaf(wf[3], x0.w, acc[t]);
        acc[t] = fmaf(wf[4], x1.x, acc[t]);
        acc[t] = fmaf(wf[5], x1.y, acc[t]);
        acc[t] = fmaf(wf[6], x1.z, acc[t]);
        acc[t] = fmaf(wf[7], x1.w, acc[t]);
      }
    }
    if (j % CPT == CPT - 1) {
      const long long tile = first + (j / CPT) * nwarps;
      const int item = static_cast<int>(tile / rblocks);
      const int rb = static_cast<int>(tile - static_cast<long long>(item) * rblocks);
      const GemvItem& it = a.items[item];
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        if (t < ntok)
          a.Y[static_cast<size_t>(it.tok[t].y) * a.rows + rb * 32 + lane] =
              a.round_out ? bf16_round(acc[t]) : acc[t];
        acc[t] = 0.0f;
      }
    }
    __syncwarp();  // every lane is done with stage q before it is refilled
    if (j + STAGES < jobs) issue(j + STAGES, q);
    __syncwarp();
    if (++q == STAGES) {
      q = 0;
      phase ^= 1u;
    }
  }
  if (!ok) {
    // drain this warp's copies still in flight before the CTA exits
    mbar_wait(&bars[q], phase, err);
    uint32_t ph = phase;
    int k = q;
    for (long long r = j + 1; r < jobs && r < j + STAGES; ++r) {
      if (++k == STAGES) { k = 0; ph ^= 1u; }
      mbar_wait(&bars[k], ph, err);
    }
  }
}

template <int WARPS, int STAGES, int NT>
__global__ void __launch_bounds__(WARPS * 32, 1)
    bf16_stream_mt_kernel(const __grid_constant__ CUtensorMap wmap, const Bf16GemvArgs a, int ntok,
                          unsigned int* err) {
  extern __shared__ __align__(1024) unsigned char smem[];
  __shared__ uint64_t bars_all[WARPS][STAGES];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  unsigned char* const sbase = smem + ((1024u - (smem_addr(smem) & 1023u)) & 1023u);
  uint64_t* bars = bars_all[warp];
  if (lane == 0) {
#pragma unroll
    for (int q = 0; q < STAGES; ++q) mbar_init(&bars[q], 1);
    mbar_fence_init();
    if (warp == 0) tma_prefetch_desc(&wmap);
  }
  __syncthreads();
  pdl_trigger();
  pdl_wait();
  bf16_stream_mt_warp<STAGES, NT>(&wmap, a, ntok, static_cast<long long>(warp) * gridDim.x + blockIdx.x,
                                  static_cast<long long>(gridDim.x) * WARPS,
                                  sbase + static_cast<size_t>(warp) * STAGES * bf16_mt_stage<NT>(),
                                  bars, err);
}

int fp8_mt_bps(const Fp8GemvArgs& a) {
  const int total = a.rows + a.rows1, CB = a.in / 128;
  const long long target = 16LL * sm_count();
  const long long units = static_cast<long long>(total / 32) * CB;
  return static_cast<int>(std::min<long long>(CB, std::max<long long>(1, (units + target - 1) / target)));
}

size_t fp8_gemv_mt_part_floats(const Fp8GemvArgs& a, int ntok) {
  return static_cast<size_t>(ntok) * (a.in / 128) * (a.rows + a.rows1);
}

cudaError_t launch_fp8_gemv_mt(const Fp8GemvArgs& a, int ntok, float* part, cudaStream_t st) {
  if (ntok < 1 || ntok > kItemTok || a.rows <= 0) return cudaErrorInvalidValue;
  if (a.rows % 32 != 0 || a.rows1 % 32 != 0 || a.in % 128 != 0 || a.act.ld % 128 != 0 ||
      a.act.x32 || !aligned(a.W[0], 32) || !aligned(a.act.x, 32) ||
      (a.rows1 > 0 && !aligned(a.W[1], 32)))
    return cudaErrorNotSupported;
  const int bps = fp8_mt_bps(a);
  const int CB = a.in / 128, total = a.rows + a.rows1;
  const long long warps = static_cast<long long>(total / 32) * ((CB + bps - 1) / bps);
  const dim3 grid(static_cast<unsigned>((warps + 3) / 4));
  cudaError_t e;
  if (ntok <= 2) e = launch_pdl(fp8_mt_partials_kernel<2>, grid, dim3(128), 0, st, a, ntok, bps, part);
  else if (ntok <= 4) e = launch_pdl(fp8_mt_partials_kernel<4>, grid, dim3(128), 0, st, a, ntok, bps, part);
  else if (ntok <= 6) e = launch_pdl(fp8_mt_partials_kernel<6>, grid, dim3(128), 0, st, a, ntok, bps, part);
  else e = launch_pdl(fp8_mt_partials_kernel<8>, grid, dim3(128), 0, st, a, ntok, bps, part);
  if (e != cudaSuccess) return e;
  const long long n = static_cast<long long>(ntok) * total;
  return launch_pdl(fp8_mt_fold_kernel, dim3(static_cast<unsigned>((n + 127) / 128)), dim3(128), 0,
                    st, a, ntok, static_cast<const float*>(part));
}

cudaError_t launch_bf16_gemv_mt(const Bf16GemvArgs& a, int ntok, cudaStream_t st) {
  if (ntok < 1 || ntok > kItemTok || a.rows <= 0 || a.max_items <= 0) return cudaErrorInvalidValue;
  const long long n_mats = a.w_stride ? a.max_items : 1;
  if (a.rows % 32 != 0 || a.in % kBCols != 0 || !aligned(a.W, 16) || !aligned(a.x, 16) ||
      a.ldx % 4 != 0 || (a.w_stride != 0 && a.w_stride != static_cast<size_t>(a.rows) * a.in))
    return cudaErrorNotSupported;
  CUtensorMap wmap;
  if (!make_tma_map_u8(&wmap, a.W, static_cast<uint64_t>(a.in) * 2,
                       static_cast<uint64_t>(n_mats) * a.rows, 128, 32, true))
    return cudaErrorNotSupported;
  const long long tiles = static_cast<long long>(a.max_items) * (a.rows / 32);
  auto run = [&](auto kern, int warps, int stages, int stage_bytes) -> cudaError_t {
    const size_t smem = static_cast<size_t>(warps) * stages * stage_bytes + 1024;
    cudaError_t e = set_max_dynamic_smem(reinterpret_cast<const void*>(kern), static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    const int grid = static_cast<int>(std::max<long long>(
        1, std::min<long long>(sm_count(), (tiles + warps - 1) / warps)));
    return launch_pdl(kern, dim3(grid), dim3(warps * 32), smem, st, wmap, a, ntok,
                      device_error_word());
  };
  // few tiles (grouped wo_a): two warps per SM with a deep ring; many tiles
  // (the vocab head): four warps, two stages
  const bool few = tiles <= 2LL * sm_count();
  if (ntok <= 2)
    return few ? run(bf16_stream_mt_kernel<2, 4, 2>, 2, 4, bf16_mt_stage<2>())
               : run(bf16_stream_mt_kernel<4, 2, 2>, 4, 2, bf16_mt_stage<2>());
  if (ntok <= 4)
    return few ? run(bf16_stream_mt_kernel<2, 4, 4>, 2, 4, bf16_mt_stage<4>())
               : run(bf16_stream_mt_kernel<4, 2, 4>, 4, 2, bf16_mt_stage<4>());
  if (ntok <= 6)
    return few ? run(bf16_stream_mt_kernel<2, 4, 6>, 2, 4, bf16_mt_stage<6>())
               : run(bf16_stream_mt_kernel<4, 2, 6>, 4, 2, bf16_mt_stage<6>());
  return few ? run(bf16_stream_mt_kernel<2, 4, 8>, 2, 4, bf16_mt_stage<8>())
             : run(bf16_stream_mt_kernel<4, 2, 8>, 4, 2, bf16_mt_stage<8>());
}

}  // namespace dsv4
