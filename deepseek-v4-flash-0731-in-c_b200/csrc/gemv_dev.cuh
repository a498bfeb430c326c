// gemv_dev.cuh - device-side pieces of the one-token split-K FP8 GEMV and
// the streaming BF16 GEMV, as device functions of one unit of work (a
// warp's rows) that a kernel calls for the units it owns.
//
// A unit is one warp's share of the GEMV: 32 rows (lane = row) of a tile of
// the stacked rows [W[0]: rows | W[1]: rows1] times `bps` consecutive
// 128-column blocks. The unit's blocks' sequential fmaf partials go to
// part[block][row]; the warp finishing a tile's last segment folds its rows
// in block order, acc = fmaf(partial, qscale * ws, acc) with NaN-scaled
// blocks skipped, as dsv4_gemv_fp8_q does (src/dsv4/dsv4_model.c:657-672).
#pragma once
#include <cstdint>
#include <cuda_fp16.h>

#include "bulk.cuh"
#include "dsv4_common.cuh"
#include "gemv.cuh"

namespace dsv4 {

constexpr int kPartMaxBps = 8;  // blocks per unit when the kernel quantises its input

// The fold of a row tile in block order from every segment's partials
// (fp8_fold_kernel's arithmetic, for the warp that finishes the tile).
__device__ __forceinline__ float fp8_fold_tile(const Fp8GemvArgs& a, const float* part, int total,
                                               int row, int CB) {
  const int mat = row >= a.rows;
  const int lrow = mat ? row - a.rows : row;
  const GemvItem& it = a.items[0];
  const float* qs = a.act.s + static_cast<size_t>(it.tok[0].x) * (a.act.ld / 128);
  const uint8_t* sr = a.S[mat] + static_cast<size_t>(lrow / 128) * ((a.in + 127) / 128);
  float acc = 0.0f;
  for (int b0 = 0; b0 < CB; b0 += 16) {
    float pv[16], sv[16];
    uint32_t code[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int b = b0 + j < CB ? b0 + j : CB - 1;
      pv[j] = __ldcg(part + static_cast<size_t>(b) * total + row);
      sv[j] = qs[b];
      code[j] = sr[b];
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      if (b0 + j >= CB) break;
      const float ws = e8m0_decode(code[j]);
      if (!isnan(ws)) acc = fmaf(pv[j], sv[j] * ws, acc);
    }
  }
  return acc;
}

struct Fp8Unit {
  bool valid;
  int tile, seg, nseg, b0, b1, row, mat;
  const uint8_t* wr;  // the lane's row
};

__device__ __forceinline__ Fp8Unit fp8_unit(const Fp8GemvArgs& a, int bps, long long gw) {
  Fp8Unit u{};
  const int CB = a.in / 128;
  u.nseg = (CB + bps - 1) / bps;
  const int tiles = (a.rows + a.rows1) / 32;
  u.valid = gw < static_cast<long long>(tiles) * u.nseg;
  if (!u.valid) return u;
  u.tile = static_cast<int>(gw / u.nseg);
  u.seg = static_cast<int>(gw % u.nseg);
  u.row = u.tile * 32 + (threadIdx.x & 31);
  u.mat = u.row >= a.rows;
  u.wr = a.W[u.mat] + static_cast<size_t>(u.mat ? u.row - a.rows : u.row) * a.in;
  u.b0 = u.seg * bps;
  u.b1 = min(CB, (u.seg + 1) * bps);
  return u;
}

// The unit's weights do not depend on earlier work: its first block into
// registers and the rest toward L2.
__device__ __forceinline__ void fp8_unit_preload(const Fp8Unit& u, U8x32 (&w)[4]) {
#pragma unroll
  for (int k = 0; k < 4; ++k) w[k] = ldg32(u.wr + u.b0 * 128 + 32 * k);
  for (int b = u.b0 + 1; b < u.b1; ++b) asm volatile("prefetch.global.L2 [%0];" ::"l"(u.wr + b * 128));
}

// The rest of the unit once its inputs are ready; xsm: the warp's
// kPartMaxBps * 128 halves of shared memory (used when a.xf is set).
__device__ __forceinline__ void fp8_unit_run(const Fp8GemvArgs& a, int bps, float* part,
                                             unsigned int* tile_cnt, const Fp8Unit& u,
                                             U8x32 (&w)[4], __half* xsm) {
  const int lane = threadIdx.x & 31;
  const int CB = a.in / 128;
  const int total = a.rows + a.rows1;
  const int b0 = u.b0, b1 = u.b1, row = u.row, mat = u.mat;
  const uint8_t* wr = u.wr;
  const GemvItem& it = a.items[0];
  const __half* xr = a.act.x + static_cast<size_t>(it.tok[0].x) * a.act.ld;
  if (a.xf) {
    // the activation quant of this unit's blocks (quant_fp8_kernel's
    // arithmetic); every unit covering a block writes the same scale
    const float* xf = a.xf + static_cast<size_t>(it.tok[0].x) * a.act.ld;
    float* qs = const_cast<float*>(a.act.s) + static_cast<size_t>(it.tok[0].x) * (a.act.ld / 128);
    for (int b = b0; b < b1; ++b) {
      float v[4];
      float amax = 0.f;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        v[k] = xf[b * 128 + lane + 32 * k];
        amax = fmaxf(amax, fabsf(v[k]));
      }
      amax = warp_max(amax);
      const float scale = pow2_scale_448(amax);
      const float inv = 1.0f / scale;
      if (lane == 0) qs[b] = scale;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        float q = v[k] * inv;
        q = q > 448.f ? 448.f : (q < -448.f ? -448.f : q);
        xsm[(b - b0) * 128 + lane + 32 * k] = e4m3_round_f16(q);
      }
    }
    __syncwarp();
  }
  for (int b = b0; b < b1; ++b) {
    // the next block's weights are requested before this block's chain runs
    U8x32 wn[4];
    if (b + 1 < b1) {
#pragma unroll
      for (int k = 0; k < 4; ++k) wn[k] = ldg32(wr + (b + 1) * 128 + 32 * k);
    }
    float p = 0.0f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      uint32_t x16[16];
      if (a.xf) {
        const uint4* xs4 = reinterpret_cast<const uint4*>(&xsm[(b - b0) * 128 + 32 * k]);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint4 v = xs4[q];
          x16[4 * q] = v.x; x16[4 * q + 1] = v.y; x16[4 * q + 2] = v.z; x16[4 * q + 3] = v.w;
        }
      } else {
        const U8x32 x0 = ldg32_l1(xr + b * 128 + 32 * k);
        const U8x32 x1 = ldg32_l1(xr + b * 128 + 32 * k + 16);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          x16[q] = x0.w[q];
          x16[8 + q] = x1.w[q];
        }
      }
      p = fp8_chain32(w[k].w, x16, p);
    }
    if (b + 1 < b1) {
#pragma unroll
      for (int k = 0; k < 4; ++k) w[k] = wn[k];
    }
    part[static_cast<size_t>(b) * total + row] = p;
  }
  if (!tile_cnt) return;
  // the last of the tile's segments to finish folds the tile
  __threadfence();
  __syncwarp();
  unsigned int prev = 0;
  if (lane == 0) prev = atomicAdd(tile_cnt + u.tile, 1u);
  prev = __shfl_sync(0xffffffffu, prev, 0);
  if (prev != static_cast<unsigned>(u.nseg - 1)) return;
  __threadfence();
  if (lane == 0) tile_cnt[u.tile] = 0u;  // zero again for the next launch
  const float acc = fp8_fold_tile(a, part, total, row, CB);
  const int rows_m = mat ? a.rows1 : a.rows;
  a.Y[mat][static_cast<size_t>(it.tok[0].y) * rows_m + (mat ? row - a.rows : row)] =
      a.round_out ? bf16_round(acc) : acc;
}

__device__ __forceinline__ int load_n_items(const int* p, int max_items) {
  const int n = *p;
  return n < max_items ? n : max_items;
}

// ------------------------------------------------------- BF16 stream ----
// One warp of the streaming BF16 GEMV for one-token items (the decode
// step's grouped wo_a and vocab head): the warp owns 32 rows (lane = row)
// of tiles first, first + nwarps, ... and walks them in 256-column chunks
// through a ring of STAGES shared-memory stages at wbase (kBStage bytes
// each, 1024-byte aligned; bars: STAGES initialised mbarriers). Per chunk
// lane 0 issues four 2-D TMA boxes of [32 rows x 128 B] with the 128-byte
// swizzle (the swizzle makes the lanes' 16-byte reads conflict-free) and a
// bulk copy of the chunk's fp32 activations, completed on the stage's
// mbarrier (bounded wait). Each lane runs its row's fmaf chain in column
// order, the reference's order, so the result is the LDG kernel's bit for
// bit. `wait` is called before the first read of data earlier work
// produced (after the first weight boxes when the items are fixed).
constexpr int kBCols = 256;
constexpr int kBW = 32 * kBCols * 2;             // four swizzled [32][128 B] boxes
constexpr int kBStage = kBW + kBCols * 4;        // + the activation chunk

template <int STAGES, class Wait>
__device__ void bf16_stream_warp(const CUtensorMap* wmapp, const Bf16GemvArgs& a, long long first,
                                 long long nwarps, unsigned char* wbase, uint64_t* bars,
                                 unsigned int* err, Wait wait) {
  const CUtensorMap& wmap = *wmapp;
  const int lane = threadIdx.x & 31;
  if (!a.static_items) wait();
  const int n_items = load_n_items(a.n_items, a.max_items);
  const int rblocks = a.rows / 32;
  const long long tiles = static_cast<long long>(n_items) * rblocks;
  const int CPT = a.in / kBCols;
  const long long my_tiles = tiles > first ? (tiles - first + nwarps - 1) / nwarps : 0;
  const long long jobs = my_tiles * CPT;
  // a job's weight boxes and its activation chunk land on one mbarrier; the
  // weights of the first stages may be requested before the wait
  auto issue_w = [&](long long j, int q) {
    if (lane != 0) return;
    const long long tile = first + (j / CPT) * nwarps;
    const int chunk = static_cast<int>(j % CPT);
    const int item = static_cast<int>(tile / rblocks);
    const int rb = static_cast<int>(tile - static_cast<long long>(item) * rblocks);
    const GemvItem& it = a.items[item];
    unsigned char* st = wbase + q * kBStage;
    mbar_arrive_expect_tx(&bars[q], kBStage);
    const int y = it.mat * a.rows + rb * 32;
#pragma unroll
    for (int k = 0; k < 4; ++k) tma_load_2d(st + k * 4096, &wmap, chunk * 512 + k * 128, y, &bars[q]);
  };
  auto issue_x = [&](long long j, int q) {
    if (lane != 0) return;
    const long long tile = first + (j / CPT) * nwarps;
    const int chunk = static_cast<int>(j % CPT);
    const int item = static_cast<int>(tile / rblocks);
    const GemvItem& it = a.items[item];
    unsigned char* st = wbase + q * kBStage;
    bulk_g2s(st + kBW, a.x + static_cast<size_t>(it.tok[0].x) * a.ldx + chunk * kBCols, kBCols * 4,
             &bars[q]);
  };
  auto issue = [&](long long j, int q) {
    issue_w(j, q);
    issue_x(j, q);
  };
  for (long long j = 0; j < jobs && j < STAGES; ++j) issue_w(j, static_cast<int>(j));
  if (a.static_items) wait();
  for (long long j = 0; j < jobs && j < STAGES; ++j) issue_x(j, static_cast<int>(j));
  __syncwarp();
  float acc = 0.0f;
  int q = 0;
  uint32_t phase = 0;
  long long j = 0;
  bool ok = true;
  const int sw = lane & 7;
  for (; j < jobs; ++j) {
    if (!mbar_wait(&bars[q], phase, err)) { ok = false; break; }
    const unsigned char* st = wbase + q * kBStage;
    const float4* xs = reinterpret_cast<const float4*>(st + kBW);
    // 32 pieces of 8 columns (4 boxes x 8 swizzled 16-byte chunks), the
    // operands of piece p + 2 loaded while piece p's eight fmaf run, so the
    // chain never waits on shared memory
    auto wld = [&](int p) {
      return *reinterpret_cast<const uint4*>(st + (p >> 3) * 4096 + lane * 128 + (((p & 7) ^ sw) << 4));
    };
    uint4 wq[3];
    float4 xq0[3], xq1[3];
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      wq[p] = wld(p);
      xq0[p] = xs[2 * p];
      xq1[p] = xs[2 * p + 1];
    }
#pragma unroll
    for (int p = 0; p < 32; ++p) {
      if (p + 2 < 32) {
        wq[(p + 2) % 3] = wld(p + 2);
        xq0[(p + 2) % 3] = xs[2 * (p + 2)];
        xq1[(p + 2) % 3] = xs[2 * (p + 2) + 1];
      }
      const uint4 w8 = wq[p % 3];
      const float4 x0 = xq0[p % 3], x1 = xq1[p % 3];
      acc = fmaf(__uint_as_float(w8.x << 16), x0.x, acc);
      acc = fmaf(__uint_as_float(w8.x & 0xFFFF0000u), x0.y, acc);
      acc = fmaf(__uint_as_float(w8.y << 16), x0.z, acc);
      acc = fmaf(__uint_as_float(w8.y & 0xFFFF0000u), x0.w, acc);
      acc = fmaf(__uint_as_float(w8.z << 16), x1.x, acc);
      acc = fmaf(__uint_as_float(w8.z & 0xFFFF0000u), x1.y, acc);
      acc = fmaf(__uint_as_float(w8.w << 16), x1.z, acc);
      acc = fmaf(__uint_as_float(w8.w & 0xFFFF0000u), x1.w, acc);
    }
    if (j % CPT == CPT - 1) {
      const long long tile = first + (j / CPT) * nwarps;
      const int item = static_cast<int>(tile / rblocks);
      const int rb = static_cast<int>(tile - static_cast<long long>(item) * rblocks);
      a.Y[static_cast<size_t>(a.items[item].tok[0].y) * a.rows + rb * 32 + lane] =
          a.round_out ? bf16_round(acc) : acc;
      acc = 0.0f;
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
    // drain this warp's copies still in flight (the failed stage's
    // included) before the CTA exits
    mbar_wait(&bars[q], phase, err);
    uint32_t ph = phase;
    int k = q;
    for (long long r = j + 1; r < jobs && r < j + STAGES; ++r) {
      if (++k == STAGES) { k = 0; ph ^= 1u; }
      mbar_wait(&bars[k], ph, err);
    }
  }
}

}  // namespace dsv4
