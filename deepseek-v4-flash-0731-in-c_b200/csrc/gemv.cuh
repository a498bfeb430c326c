// gemv.cuh - work descriptors and launchers for the exact-order GEMV family
// (FP4 E2M1, FP8 E4M3, BF16 weights), the activation quantiser and the
// fused SwiGLU quantiser.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace dsv4 {

constexpr int kItemTok = 8;  // tokens one GEMV work item carries

// One (matrix, token set) unit of GEMV work. `mat` selects the matrix
// (W + mat * mat_stride); tok[i].x indexes the activation rows, tok[i].y the
// output rows.
struct TokMap {
  int x, y;
};
struct GemvItem {
  int mat;
  int ntok;
  TokMap tok[kItemTok];
};

// Quantised activation in device memory: E4M3-grid values stored as f16
// (exact), one power-of-two scale per 128 columns.
struct QAct {
  const __half* x;   // [rows][ld]
  const float* s;    // [rows][ld / 128]
  int ld;
  const float* x32;  // optional fp32 copy [rows][ld]: set when a caller's
                     // activation is not exactly representable in f16
};

struct Fp4GemvArgs {
  const uint8_t* W[2];     // packed E2M1 [rows][in/2] per matrix; W[1] for pairs
  const uint8_t* S[2];     // E8M0 [rows][in/32]
  size_t w_stride, s_stride;  // bytes between consecutive matrices (experts)
  int in, rows;
  QAct act;
  float* Y[2];             // [out rows][rows] outputs (BF16-valued floats)
  const GemvItem* items;
  const int* n_items;      // device count (<= max_items)
  int max_items;
  unsigned int* err;       // device error word (null: the library's default)
  long long n_mats;        // matrices addressable by items (w_stride apart); 0 = 1
};

struct Fp8GemvArgs {
  const uint8_t* W[2];     // E4M3 [rows][in]
  const uint8_t* S[2];     // E8M0 [ceil(rows/128)][ceil(in/128)]
  size_t w_stride, s_stride;
  int in, rows;
  int round_out;
  QAct act;
  float* Y[2];
  const GemvItem* items;
  const int* n_items;
  int max_items;
  // 1: the launch runs beside other kernels (the shared expert beside the
  // router and the routed experts): two warps per CTA on half as many SMs
  int beside = 0;
  unsigned int* err = nullptr;  // device error word (null: the library's default)
  // split-K kernels only: a second matrix W[1] / S[1] of rows1 rows (same
  // input) whose outputs go to Y[1]; one launch computes both
  int rows1 = 0;
  // split-K kernel with in-kernel folds only: fp32 activations [*][act.ld]
  // that the kernel quantises itself (act.x unused, act.s receives the
  // per-128 scales)
  const float* xf = nullptr;
};

struct Bf16GemvArgs {
  const uint16_t* W;       // [rows][in]; an item's matrix is W + mat * w_stride
  size_t w_stride;         // elements between matrices (grouped projections)
  int in, rows;
  int round_out;
  const float* x;          // [*][ldx] fp32 activations
  int ldx;
  float* Y;                // [*][rows]
  const GemvItem* items;
  const int* n_items;
  int max_items;
  // 1: items / n_items are fixed before the launch (not written by the
  // previous kernel), so the streaming kernel starts its weight copies
  // before waiting on that kernel
  int static_items = 0;
};

cudaError_t launch_fp4_gemv(const Fp4GemvArgs& a, bool pair, int item_tokens,
                            cudaStream_t st, bool map_cache = true);
cudaError_t launch_fp8_gemv(const Fp8GemvArgs& a, bool pair, int item_tokens,
                            cudaStream_t st, bool map_cache = true);
cudaError_t launch_bf16_gemv(const Bf16GemvArgs& a, int item_tokens,
                             cudaStream_t st);
// One-token, one-item FP8 GEMV split over 128-column blocks (more warps for
// matrices with few row tiles); part holds in/128 * rows floats of scratch.
// cudaErrorNotSupported when the shape or alignment does not fit.
// Blocks per split-K unit for `a` (0: the split-K form does not apply).
int fp8_splitk_bps(const Fp8GemvArgs& a);
// Streaming multiprocessors of the current device.
int device_sm_count();

// tile_cnt (zeroed, rows / 32 counters): the last segment of each row tile
// folds it in the same launch; null: a separate fold launch.
cudaError_t launch_fp8_gemv_splitk(const Fp8GemvArgs& a, float* part, cudaStream_t st,
                                   unsigned int* tile_cnt = nullptr);

// Multi-token forms for 1..kItemTok token rows through one matrix (the
// verify step), each output in the reference's order. FP8: split over
// 128-column blocks, items[0] names the tokens, W[1] / rows1 an optional
// second matrix on the same input; part holds fp8_gemv_mt_part_floats
// floats. BF16: one lane per (row, token) chain; items as launch_bf16_gemv.
// cudaErrorNotSupported when the shape or alignment does not fit.
size_t fp8_gemv_mt_part_floats(const Fp8GemvArgs& a, int ntok);
cudaError_t launch_fp8_gemv_mt(const Fp8GemvArgs& a, int ntok, float* part, cudaStream_t st);
cudaError_t launch_bf16_gemv_mt(const Bf16GemvArgs& a, int ntok, cudaStream_t st);

// x [rows][n] fp32 -> E4M3 grid (f16) + per-128 scales (dsv4_quant_fp8_codes).
cudaError_t launch_quant_fp8(const float* x, int ldx, int n, int rows, __half* qx,
                             float* qs, int ld_out, cudaStream_t st);
// Same, but also writes the quantised values back as fp32 (drop-in API).
cudaError_t launch_quant_fp8_f32(const float* x, int n, float* qx, float* qs,
                                 cudaStream_t st);

// gate/up [rows][n] -> SwiGLU * weight -> BF16 -> FP8 quant (routed_swiglu_quant).
// weight == nullptr means 1.0 for every row (shared expert).
cudaError_t launch_swiglu_quant(const float* gate, const float* up, int n, int rows,
                                const float* weight, int limit, __half* qy, float* qs,
                                float* y_bf16, cudaStream_t st);

// fp32 activations on the E4M3 grid -> f16 (exact), for host-supplied qx.
cudaError_t launch_f32_to_f16(const float* x, __half* y, size_t n, cudaStream_t st);

}  // namespace dsv4
