// moe.cuh - device-resident MoE layer (router, expert permute, grouped
// expert GEMVs, ordered combine).
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "gemv.cuh"

namespace dsv4 {

enum SharedKind { kSharedNone = 0, kSharedFp8 = 1, kSharedFp4 = 2 };

struct MoeConfig {
  int hidden, moe_inter, n_experts, topk, swiglu_limit;
  float route_scale;
  int shared_kind;   // SharedKind
  int hash_vocab;    // rows of tid2eid (0 = not a hash layer)
  // Expert parallelism: this device computes experts [expert_lo, expert_hi)
  // and its routed weights hold only those (local index e - expert_lo);
  // expert_hi == 0 means every expert.
  int expert_lo = 0, expert_hi = 0;
};

inline int moe_local_hi(const MoeConfig& c) { return c.expert_hi > 0 ? c.expert_hi : c.n_experts; }
inline bool moe_is_partial(const MoeConfig& c) {
  return c.expert_lo != 0 || moe_local_hi(c) != c.n_experts;
}

// Device pointers of one layer's weights (reference layouts, expert-major).
struct MoeWeights {
  const uint16_t* gate_w;   // [E][H] BF16
  const float* bias;        // [E] or null
  const int64_t* tid2eid;   // [hash_vocab][topk] or null
  const uint8_t *w1, *s1, *w3, *s3, *w2, *s2;     // routed FP4
  const uint8_t *sh1, *sh1s, *sh3, *sh3s, *sh2, *sh2s;  // shared (FP8 or FP4)
};

// Scratch for one forward of up to max_tokens tokens. All device memory.
struct MoeWorkspace {
  int max_tokens = 0;
  __half* xq = nullptr;      // [M][H]
  float* xs = nullptr;       // [M][H/128]
  double* zd = nullptr;      // [M][E] exact router logits
  double* zb = nullptr;      // [M][E] bound of the reference's rounding error
  int* idx = nullptr;        // [M][topk] ascending ids
  float* wt = nullptr;       // [M][topk]
  GemvItem* items_gu = nullptr;   // [M*topk] items of two or more routes
  GemvItem* items_dn = nullptr;   // [M*topk]
  GemvItem* items_gu1 = nullptr;  // [M*topk] single-route items
  GemvItem* items_dn1 = nullptr;  // [M*topk]
  GemvItem* items_sh = nullptr;   // [ceil(M/8)] (static)
  int* counters = nullptr;   // [0]=multi items, [1]=done CTAs, [2]=tie fallbacks,
                             // [3]=n_shared_items, [4]=single items
  float* gate = nullptr;     // [M*topk][I]
  float* up = nullptr;       // [M*topk][I]
  __half* qy = nullptr;      // [M*topk][I]
  float* qys = nullptr;      // [M*topk][I/128]
  float* routed = nullptr;   // [M*topk][H]
  float* sh_gate = nullptr;  // [M][I]
  float* sh_up = nullptr;    // [M][I]
  __half* sh_qy = nullptr;   // [M][I]
  float* sh_qys = nullptr;   // [M][I/128]
  float* shared = nullptr;   // [M][H]
  size_t bytes = 0;
  // Optional timing: when set, events are recorded on the forward stream
  // around the routed expert GEMV launches ([0..1] gate/up, [2..3] down) and
  // the router ([4] before the logits, [5] after them, [6] after selection).
  cudaEvent_t* timing = nullptr;
};

// Bytes a workspace for `max_tokens` needs (256-byte aligned pieces).
size_t moe_workspace_bytes(const MoeConfig& c, int max_tokens);
// Carve a workspace out of `base` (>= moe_workspace_bytes bytes).
void moe_workspace_carve(MoeWorkspace* ws, const MoeConfig& c, int max_tokens, void* base);

// One MoE layer for n_tokens tokens: x [n][H] fp32 (BF16-valued) -> out [n][H]
// (BF16-valued), per-token results identical to moe_forward
// (src/dsv4/dsv4_model.c:6599) / moe_forward_batch (:6812).
// exact_router: 1 = the reference's fused fmaf logits (moe_forward),
// 2 = the public dsv4_router's separate multiply/add logits.
// Execution options. The defaults are what the library's own entry points
// use; the allocation-free entry point runs everything on the caller's
// stream, encodes tensor maps without the host-side cache and passes its own
// device error word.
struct MoeExecOptions {
  bool single_stream = false;  // shared expert on `st` instead of a side stream
  bool map_cache = true;       // cache TMA descriptors by argument
  unsigned int* err = nullptr; // device error word (null: the library's)
  // shared expert only for tokens [shared_t0, shared_t0 + shared_n) (-1: all);
  // token-parallel expert parallelism computes it for this rank's tokens
  int shared_t0 = 0;
  int shared_n = -1;
  // ws.xq / ws.xs already hold x's FP8 quant (written by the caller's last
  // kernel), and ws.items_sh / ws.counters[3] the shared expert's items for
  // these tokens: no quant launch ahead of the router
  bool x_quantized = false;
  // an event `st` also waits on before the combine (work forked by the
  // caller that must finish before the layer's output is consumed)
  cudaEvent_t join = nullptr;
  // scratch for the multi-token split-K FP8 kernels (mt_part_floats
  // floats): with it, an FP8 shared expert over two or more tokens runs
  // split over its 128-column blocks (the verify step's rows)
  float* mt_part = nullptr;
  size_t mt_part_floats = 0;
};

cudaError_t moe_forward(const MoeConfig& c, const MoeWeights& w, const MoeWorkspace& ws,
                        const float* x, const int* token_ids, int n_tokens, float* out,
                        cudaStream_t st, const MoeExecOptions& opt = MoeExecOptions());

// The two halves of moe_forward, for expert parallelism: moe_forward_local
// runs the router, this device's routed experts (ws.routed slots [n][topk][H]
// of other devices' experts are zero) and the shared expert; after the
// caller has summed ws.routed over the devices (x + 0 is exact),
// moe_combine forms out. moe_forward = moe_forward_local + moe_combine.
cudaError_t moe_forward_local(const MoeConfig& c, const MoeWeights& w, const MoeWorkspace& ws,
                              const float* x, const int* token_ids, int n_tokens,
                              cudaStream_t st, const MoeExecOptions& opt = MoeExecOptions());
cudaError_t moe_combine(const MoeConfig& c, const MoeWorkspace& ws, int n_tokens, float* out,
                        bool has_shared, cudaStream_t st);

// The router's score function sqrt(softplus(z)) as the selection evaluates
// it, elementwise over n device floats.
cudaError_t router_scores(const float* z, float* s, int n, cudaStream_t st);

// Router only: idx/wt [n][topk] (ids ascending), same numerics as above.
cudaError_t moe_route(const MoeConfig& c, const MoeWeights& w, const MoeWorkspace& ws,
                      const float* x, const int* token_ids, int n_tokens, int public_router,
                      cudaStream_t st);

}  // namespace dsv4
