// capi.cu - the C ABI of libdsv4_cuda.so (declared in include/dsv4_cuda.h).
//
// Drop-in kernel symbols stage host operands through per-thread device
// buffers on a per-thread stream (the reference may call its kernels from
// several OpenMP threads, src/dsv4/dsv4_model.c:6703-6725), run the exact
// kernels and copy the results back before returning, like the reference's
// synchronous kernels.
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>
#include <atomic>
#include <mutex>

#include <cuda_fp16.h>

#include "bulk.cuh"
#include "dsv4_common.cuh"
#include "gemv.cuh"
#include "moe.cuh"
#include "attn.cuh"
#include "sample.cuh"
#include "snapshot.cuh"
#include "ep.cuh"
#include "../../include/dsv4_cuda.h"

#define DSV4_API extern "C" __attribute__((visibility("default")))

namespace {

std::atomic<int> g_abort{1};
thread_local std::string t_last_error;

// Drop-in calls served, per kernel family (the order of
// dsv4cuda_dropin_calls): FP4 GEMVs, FP8 GEMVs, BF16 GEMVs, activation
// quant, router, SwiGLU quant.
constexpr int kDropinKinds = 6;
std::atomic<unsigned long long> g_dropin_calls[kDropinKinds];

void dropin_report() {
  fprintf(stderr, "dsv4_cuda drop-in calls: fp4=%llu fp8=%llu bf16=%llu quant=%llu router=%llu "
                  "swiglu=%llu\n",
          g_dropin_calls[0].load(), g_dropin_calls[1].load(), g_dropin_calls[2].load(),
          g_dropin_calls[3].load(), g_dropin_calls[4].load(), g_dropin_calls[5].load());
}

// DSV4CUDA_DROPIN_REPORT=1 in the environment: print the counts at exit, so
// a host program that preloads the library can show which of its kernel
// calls the GPU served.
struct DropinReportAtExit {
  DropinReportAtExit() {
    const char* v = getenv("DSV4CUDA_DROPIN_REPORT");
    if (v && v[0] && v[0] != '0') atexit(dropin_report);
  }
} g_dropin_report_at_exit;

struct ThreadState {
  int device = -1;
  cudaStream_t stream = nullptr;
  char* dbuf = nullptr;
  size_t dcap = 0;
  int* counter = nullptr;  // device int used as "n_items" for host-built lists
};
thread_local ThreadState t_state;

void record_error(const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
}

// Drop-in fatal path: the reference exits on its own fatal errors.
void fatal_or_record(const char* what, cudaError_t e) {
  record_error("%s: %s", what, cudaGetErrorString(e));
  if (g_abort.load()) {
    fprintf(stderr, "dsv4_cuda: %s\n", t_last_error.c_str());
    exit(1);
  }
}

int ensure_thread_state() {
  if (t_state.stream) return 0;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) { record_error("cudaGetDevice: %s", cudaGetErrorString(e)); return -1; }
  e = cudaStreamCreateWithFlags(&t_state.stream, cudaStreamNonBlocking);
  if (e != cudaSuccess) { record_error("stream: %s", cudaGetErrorString(e)); return -1; }
  e = cudaMalloc(&t_state.counter, sizeof(int) * 4);
  if (e != cudaSuccess) { record_error("cudaMalloc: %s", cudaGetErrorString(e)); return -1; }
  t_state.device = dev;
  return 0;
}

// Grow-only per-thread device staging buffer.
char* staging(size_t bytes) {
  if (bytes > t_state.dcap) {
    if (t_state.dbuf) cudaFree(t_state.dbuf);
    t_state.dbuf = nullptr;
    t_state.dcap = 0;
    const size_t cap = bytes + bytes / 4 + 4096;
    if (cudaMalloc(&t_state.dbuf, cap) != cudaSuccess) return nullptr;
    t_state.dcap = cap;
  }
  return t_state.dbuf;
}

size_t al(size_t b) { return (b + 255) & ~static_cast<size_t>(255); }

// Carves 256-byte aligned pieces out of the staging buffer.
struct Carver {
  char* base;
  size_t off = 0;
  template <class T>
  T* take(size_t count) {
    T* p = reinterpret_cast<T*>(base + off);
    off += al(count * sizeof(T));
    return p;
  }
};

bool f16_exact(float v) {
  const __half h = __float2half_rn(v);
  const float back = __half2float(h);
  return back == v || (v != v && back != back);
}

// Host item list for a batch of `batch` tokens against one matrix.
std::vector<dsv4::GemvItem> batch_items(int batch) {
  std::vector<dsv4::GemvItem> items((batch + dsv4::kItemTok - 1) / dsv4::kItemTok);
  for (size_t j = 0; j < items.size(); ++j) {
    dsv4::GemvItem& it = items[j];
    it.mat = 0;
    it.ntok = std::min<int>(dsv4::kItemTok, batch - static_cast<int>(j) * dsv4::kItemTok);
    for (int i = 0; i < dsv4::kItemTok; ++i) {
      const int t = std::min<int>(static_cast<int>(j) * dsv4::kItemTok + i, batch - 1);
      it.tok[i].x = t;
      it.tok[i].y = t;
    }
  }
  return items;
}

int nt_bucket(int n) { return n <= 1 ? 1 : n <= 2 ? 2 : n <= 4 ? 4 : 8; }

void batch_limit(const char* kind, int batch) {
  if (batch > dsv4::kMaxBatch) {
    // src/dsv4/dsv4_model.c:316-320 / :689-693 / :1094-1098
    fprintf(stderr, "dsv4: %s batch %d exceeds %d\n", kind, batch, dsv4::kMaxBatch);
    exit(1);
  }
}

#define STAGE_CHECK(expr, what)                      \
  do {                                               \
    cudaError_t e__ = (expr);                        \
    if (e__ != cudaSuccess) {                        \
      fatal_or_record(what, e__);                    \
      return;                                        \
    }                                                \
  } while (0)

// Upload activations for `batch` tokens: f16 copy (plus an fp32 copy when any
// value is not exactly representable in f16) and scales.
struct StagedAct {
  dsv4::QAct act;
};

void fp4_or_fp8_gemv(bool fp4, float* const* y0, float* const* y1, const float* const* qx,
                     const float* const* qscale, int batch, const uint8_t* W0, const uint8_t* S0,
                     const uint8_t* W1, const uint8_t* S1, int in, int rows, int round_out) {
  g_dropin_calls[fp4 ? 0 : 1].fetch_add(1, std::memory_order_relaxed);
  if (batch <= 0 || rows <= 0) return;
  if (ensure_thread_state() != 0) { fatal_or_record("init", cudaErrorInitializationError); return; }
  cudaStream_t st = t_state.stream;
  const bool pair = W1 != nullptr;
  const size_t wbytes = fp4 ? static_cast<size_t>(rows) * ((in + 1) / 2)
                            : static_cast<size_t>(rows) * in;
  const size_t sbytes = fp4 ? static_cast<size_t>(rows) * ((in + 31) / 32)
                            : static_cast<size_t>((rows + 127) / 128) * ((in + 127) / 128);
  const int ld = (in + 127) / 128 * 128;
  const int nsc = ld / 128;
  bool exact16 = true;
  for (int t = 0; t < batch && exact16; ++t)
    for (int c = 0; c < in; ++c)
      if (!f16_exact(qx[t][c])) { exact16 = false; break; }
  const std::vector<dsv4::GemvItem> items = batch_items(batch);
  const size_t need = al(wbytes) * (pair ? 2 : 1) + al(sbytes) * (pair ? 2 : 1) +
                      al(sizeof(float) * batch * ld) * 2 + al(sizeof(__half) * batch * ld) +
                      al(sizeof(float) * batch * nsc) + al(sizeof(float) * batch * rows) * 2 +
                      al(sizeof(dsv4::GemvItem) * items.size()) + 1024;
  char* base = staging(need);
  if (!base) { fatal_or_record("staging cudaMalloc", cudaErrorMemoryAllocation); return; }
  Carver cv{base};
  uint8_t* dW0 = cv.take<uint8_t>(wbytes);
  uint8_t* dS0 = cv.take<uint8_t>(sbytes);
  uint8_t* dW1 = pair ? cv.take<uint8_t>(wbytes) : nullptr;
  uint8_t* dS1 = pair ? cv.take<uint8_t>(sbytes) : nullptr;
  float* dx32 = cv.take<float>(static_cast<size_t>(batch) * ld);
  __half* dx16 = cv.take<__half>(static_cast<size_t>(batch) * ld);
  float* dqs = cv.take<float>(static_cast<size_t>(batch) * nsc);
  float* dy0 = cv.take<float>(static_cast<size_t>(batch) * rows);
  float* dy1 = cv.take<float>(static_cast<size_t>(batch) * rows);
  dsv4::GemvItem* ditems = cv.take<dsv4::GemvItem>(items.size());

  STAGE_CHECK(cudaMemcpyAsync(dW0, W0, wbytes, cudaMemcpyHostToDevice, st), "copy W");
  STAGE_CHECK(cudaMemcpyAsync(dS0, S0, sbytes, cudaMemcpyHostToDevice, st), "copy S");
  if (pair) {
    STAGE_CHECK(cudaMemcpyAsync(dW1, W1, wbytes, cudaMemcpyHostToDevice, st), "copy W1");
    STAGE_CHECK(cudaMemcpyAsync(dS1, S1, sbytes, cudaMemcpyHostToDevice, st), "copy S1");
  }
  STAGE_CHECK(cudaMemsetAsync(dx32, 0, sizeof(float) * batch * ld, st), "memset");
  for (int t = 0; t < batch; ++t) {
    STAGE_CHECK(cudaMemcpyAsync(dx32 + static_cast<size_t>(t) * ld, qx[t], sizeof(float) * in,
                                cudaMemcpyHostToDevice, st), "copy qx");
    STAGE_CHECK(cudaMemcpyAsync(dqs + static_cast<size_t>(t) * nsc, qscale[t],
                                sizeof(float) * ((in + 127) / 128), cudaMemcpyHostToDevice, st),
                "copy qscale");
  }
  STAGE_CHECK(cudaMemcpyAsync(ditems, items.data(), sizeof(dsv4::GemvItem) * items.size(),
                              cudaMemcpyHostToDevice, st), "copy items");
  const int nitems = static_cast<int>(items.size());
  STAGE_CHECK(cudaMemcpyAsync(t_state.counter, &nitems, sizeof(int), cudaMemcpyHostToDevice, st),
              "copy count");
  STAGE_CHECK(dsv4::launch_f32_to_f16(dx32, dx16, static_cast<size_t>(batch) * ld, st), "cvt");
  const dsv4::QAct act{dx16, dqs, ld, exact16 ? nullptr : dx32};
  const int nt = nt_bucket(std::min(batch, dsv4::kItemTok));
  if (fp4) {
    dsv4::Fp4GemvArgs a{};
    a.W[0] = dW0; a.S[0] = dS0; a.W[1] = dW1; a.S[1] = dS1;
    a.in = in; a.rows = rows; a.act = act;
    a.Y[0] = dy0; a.Y[1] = dy1;
    a.items = ditems; a.n_items = t_state.counter; a.max_items = nitems;
    STAGE_CHECK(dsv4::launch_fp4_gemv(a, pair, nt, st), "fp4 gemv");
  } else {
    dsv4::Fp8GemvArgs a{};
    a.W[0] = dW0; a.S[0] = dS0; a.W[1] = dW1; a.S[1] = dS1;
    a.in = in; a.rows = rows; a.round_out = round_out; a.act = act;
    a.Y[0] = dy0; a.Y[1] = dy1;
    a.items = ditems; a.n_items = t_state.counter; a.max_items = nitems;
    STAGE_CHECK(dsv4::launch_fp8_gemv(a, pair, nt, st), "fp8 gemv");
  }
  for (int t = 0; t < batch; ++t) {
    STAGE_CHECK(cudaMemcpyAsync(y0[t], dy0 + static_cast<size_t>(t) * rows, sizeof(float) * rows,
                                cudaMemcpyDeviceToHost, st), "copy y");
    if (pair)
      STAGE_CHECK(cudaMemcpyAsync(y1[t], dy1 + static_cast<size_t>(t) * rows,
                                  sizeof(float) * rows, cudaMemcpyDeviceToHost, st), "copy y1");
  }
  STAGE_CHECK(cudaStreamSynchronize(st), "sync");
}

void bf16_gemv(float* const* y, const float* const* x, int batch, const uint16_t* W, int in,
               int out, int round_out) {
  g_dropin_calls[2].fetch_add(1, std::memory_order_relaxed);
  if (batch <= 0 || out <= 0) return;
  if (ensure_thread_state() != 0) { fatal_or_record("init", cudaErrorInitializationError); return; }
  cudaStream_t st = t_state.stream;
  const size_t wbytes = static_cast<size_t>(out) * in * sizeof(uint16_t);
  const int ld = (in + 7) / 8 * 8;
  const std::vector<dsv4::GemvItem> items = batch_items(batch);
  const size_t need = al(wbytes) + al(sizeof(float) * batch * ld) +
                      al(sizeof(float) * batch * out) + al(sizeof(dsv4::GemvItem) * items.size()) +
                      1024;
  char* base = staging(need);
  if (!base) { fatal_or_record("staging cudaMalloc", cudaErrorMemoryAllocation); return; }
  Carver cv{base};
  uint16_t* dW = cv.take<uint16_t>(static_cast<size_t>(out) * in);
  float* dx = cv.take<float>(static_cast<size_t>(batch) * ld);
  float* dy = cv.take<float>(static_cast<size_t>(batch) * out);
  dsv4::GemvItem* ditems = cv.take<dsv4::GemvItem>(items.size());
  STAGE_CHECK(cudaMemcpyAsync(dW, W, wbytes, cudaMemcpyHostToDevice, st), "copy W");
  for (int t = 0; t < batch; ++t)
    STAGE_CHECK(cudaMemcpyAsync(dx + static_cast<size_t>(t) * ld, x[t], sizeof(float) * in,
                                cudaMemcpyHostToDevice, st), "copy x");
  STAGE_CHECK(cudaMemcpyAsync(ditems, items.data(), sizeof(dsv4::GemvItem) * items.size(),
                              cudaMemcpyHostToDevice, st), "copy items");
  const int nitems = static_cast<int>(items.size());
  STAGE_CHECK(cudaMemcpyAsync(t_state.counter, &nitems, sizeof(int), cudaMemcpyHostToDevice, st),
              "copy count");
  dsv4::Bf16GemvArgs a{};
  a.W = dW; a.in = in; a.rows = out; a.round_out = round_out;
  a.x = dx; a.ldx = ld; a.Y = dy;
  a.items = ditems; a.n_items = t_state.counter; a.max_items = nitems;
  STAGE_CHECK(dsv4::launch_bf16_gemv(a, nt_bucket(std::min(batch, dsv4::kItemTok)), st),
              "bf16 gemv");
  for (int t = 0; t < batch; ++t)
    STAGE_CHECK(cudaMemcpyAsync(y[t], dy + static_cast<size_t>(t) * out, sizeof(float) * out,
                                cudaMemcpyDeviceToHost, st), "copy y");
  STAGE_CHECK(cudaStreamSynchronize(st), "sync");
}

void quant_codes(float* qx, float* qscale, const float* x, int n) {
  g_dropin_calls[3].fetch_add(1, std::memory_order_relaxed);
  if (n <= 0) return;
  if (ensure_thread_state() != 0) { fatal_or_record("init", cudaErrorInitializationError); return; }
  cudaStream_t st = t_state.stream;
  const int nb = (n + 127) / 128;
  char* base = staging(al(sizeof(float) * n) * 2 + al(sizeof(float) * nb) + 1024);
  if (!base) { fatal_or_record("staging cudaMalloc", cudaErrorMemoryAllocation); return; }
  Carver cv{base};
  float* dx = cv.take<float>(n);
  float* dq = cv.take<float>(n);
  float* ds = cv.take<float>(nb);
  STAGE_CHECK(cudaMemcpyAsync(dx, x, sizeof(float) * n, cudaMemcpyHostToDevice, st), "copy x");
  STAGE_CHECK(dsv4::launch_quant_fp8_f32(dx, n, dq, ds, st), "quant");
  STAGE_CHECK(cudaMemcpyAsync(qx, dq, sizeof(float) * n, cudaMemcpyDeviceToHost, st), "copy qx");
  STAGE_CHECK(cudaMemcpyAsync(qscale, ds, sizeof(float) * nb, cudaMemcpyDeviceToHost, st),
              "copy qs");
  STAGE_CHECK(cudaStreamSynchronize(st), "sync");
}

}  // namespace

// ---------------------------------------------------------------- layer --
struct dsv4cuda_moe_layer {
  dsv4::MoeConfig cfg{};
  dsv4::MoeWeights w{};
  dsv4::MoeWorkspace ws{};
  void* owned = nullptr;      // weights copied in by dsv4cuda_moe_create
  size_t owned_bytes = 0;
  void* ws_mem = nullptr;
  size_t ws_bytes = 0;
  float* d_x = nullptr;       // host-path staging
  float* d_out = nullptr;
  int* d_tok = nullptr;
  int max_tokens = 0;
  // expert-GEMV timing (dsv4cuda_moe_timing_*): event quadruples per forward
  std::vector<cudaEvent_t> events;
  int timed = 0;
  bool timing = false;
  // dsv4cuda_moe_forward_host: the forward of n tokens (d_x -> d_out)
  // captured once into a CUDA graph per n and replayed after that
  std::vector<cudaGraphExec_t> host_graphs;
  // expert-parallel exchange over peer memory (dsv4cuda_moe_ep_attach)
  dsv4::EpExchange ep{};
  bool ep_attached = false;
};

namespace {

struct LayerSizes {
  size_t gate, bias, tid, w13, s13, w2, s2, sh13, sh13s, sh2, sh2s;
};

LayerSizes layer_sizes(const dsv4::MoeConfig& c) {
  const size_t H = c.hidden, I = c.moe_inter, E = c.n_experts, K = c.topk;
  LayerSizes s{};
  s.gate = E * H * 2;
  s.bias = E * 4;
  s.tid = static_cast<size_t>(c.hash_vocab) * K * 8;
  s.w13 = E * I * (H / 2);
  s.s13 = E * I * (H / 32);
  s.w2 = E * H * (I / 2);
  s.s2 = E * H * (I / 32);
  if (c.shared_kind == dsv4::kSharedFp8) {
    s.sh13 = I * H;
    s.sh13s = ((I + 127) / 128) * ((H + 127) / 128);
    s.sh2 = H * I;
    s.sh2s = ((H + 127) / 128) * ((I + 127) / 128);
  } else if (c.shared_kind == dsv4::kSharedFp4) {
    s.sh13 = I * (H / 2);
    s.sh13s = I * (H / 32);
    s.sh2 = H * (I / 2);
    s.sh2s = H * (I / 32);
  }
  return s;
}

int validate_cfg(const dsv4cuda_moe_config* c) {
  if (!c || c->hidden <= 0 || c->moe_inter <= 0 || c->n_experts <= 0 || c->topk <= 0 ||
      c->topk > dsv4::kMaxTopk || c->topk > c->n_experts || c->hidden % 32 != 0 ||
      c->moe_inter % 32 != 0 || c->shared_kind < 0 || c->shared_kind > 2 || c->hash_vocab < 0) {
    record_error("invalid dsv4cuda_moe_config");
    return -1;
  }
  return 0;
}

int layer_finish(dsv4cuda_moe_layer* L, int max_tokens) {
  L->max_tokens = max_tokens;
  L->ws_bytes = dsv4::moe_workspace_bytes(L->cfg, max_tokens) +
                al(sizeof(float) * max_tokens * L->cfg.hidden) * 2 + al(sizeof(int) * max_tokens);
  cudaError_t e = cudaMalloc(&L->ws_mem, L->ws_bytes);
  if (e != cudaSuccess) { record_error("workspace cudaMalloc: %s", cudaGetErrorString(e)); return -1; }
  cudaMemset(L->ws_mem, 0, L->ws_bytes);
  dsv4::moe_workspace_carve(&L->ws, L->cfg, max_tokens, L->ws_mem);
  char* p = static_cast<char*>(L->ws_mem) + L->ws.bytes;
  L->d_x = reinterpret_cast<float*>(p);
  p += al(sizeof(float) * max_tokens * L->cfg.hidden);
  L->d_out = reinterpret_cast<float*>(p);
  p += al(sizeof(float) * max_tokens * L->cfg.hidden);
  L->d_tok = reinterpret_cast<int*>(p);
  return 0;
}

// While timing is on, the forward records its phase events into a fresh
// group of 8 events of the layer.
int timed_workspace(dsv4cuda_moe_layer* L, dsv4::MoeWorkspace* ws) {
  if (!L->timing) return 0;
  const size_t need = static_cast<size_t>(L->timed + 1) * 8;
  while (L->events.size() < need) {
    cudaEvent_t ev;
    if (cudaEventCreate(&ev) != cudaSuccess) { record_error("cudaEventCreate"); return -1; }
    L->events.push_back(ev);
  }
  ws->timing = &L->events[static_cast<size_t>(L->timed) * 8];
  L->timed++;
  return 0;
}

dsv4::MoeConfig to_cfg(const dsv4cuda_moe_config* c) {
  dsv4::MoeConfig m{};
  m.hidden = c->hidden;
  m.moe_inter = c->moe_inter;
  m.n_experts = c->n_experts;
  m.topk = c->topk;
  m.swiglu_limit = c->swiglu_limit;
  m.route_scale = c->route_scale;
  m.shared_kind = c->shared_kind;
  m.hash_vocab = c->hash_vocab;
  return m;
}

}  // namespace

// ================================================================ exports ==

DSV4_API void dsv4cuda_shutdown(void) {
  if (t_state.dbuf) cudaFree(t_state.dbuf);
  if (t_state.counter) cudaFree(t_state.counter);
  if (t_state.stream) cudaStreamDestroy(t_state.stream);
  t_state = ThreadState();
}

DSV4_API int dsv4cuda_init(int device) {
  if (t_state.stream && t_state.device != device) dsv4cuda_shutdown();
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) { record_error("cudaSetDevice(%d): %s", device, cudaGetErrorString(e)); return -1; }
  return ensure_thread_state();
}

DSV4_API const char* dsv4cuda_last_error(void) { return t_last_error.c_str(); }

DSV4_API int dsv4cuda_device_error(unsigned int* flags, int clear) {
  unsigned int* w = dsv4::device_error_word();
  if (!w) { record_error("device error word unavailable"); return -1; }
  unsigned int v = 0;
  cudaError_t e = cudaMemcpy(&v, w, sizeof(v), cudaMemcpyDeviceToHost);
  if (e == cudaSuccess && clear) e = cudaMemset(w, 0, sizeof(v));
  if (e != cudaSuccess) { record_error("device error word: %s", cudaGetErrorString(e)); return -1; }
  if (flags) *flags = v;
  return 0;
}

DSV4_API int dsv4cuda_dropin_calls(unsigned long long* counts, int n) {
  const int k = n < kDropinKinds ? n : kDropinKinds;
  for (int i = 0; i < k; ++i) counts[i] = g_dropin_calls[i].load();
  return kDropinKinds;
}

DSV4_API int dsv4cuda_set_abort_on_error(int abort_on_error) {
  return g_abort.exchange(abort_on_error ? 1 : 0);
}


// ---- drop-in kernels
DSV4_API void dsv4cuda_gemv_fp4_q(float* y, const float* qx, const float* qscale, const uint8_t* W,
                                  const uint8_t* wscale_code, int in, int rows) {
  float* ys[1] = {y};
  const float* xs[1] = {qx};
  const float* ss[1] = {qscale};
  fp4_or_fp8_gemv(true, ys, nullptr, xs, ss, 1, W, wscale_code, nullptr, nullptr, in, rows, 1);
}
DSV4_API void dsv4cuda_gemv_fp4_batch_q(float* const* y, const float* const* qx,
                                        const float* const* qscale, int batch, const uint8_t* W,
                                        const uint8_t* wscale_code, int in, int rows) {
  if (batch <= 0) return;
  batch_limit("FP4", batch);
  fp4_or_fp8_gemv(true, y, nullptr, qx, qscale, batch, W, wscale_code, nullptr, nullptr, in, rows,
                  1);
}
DSV4_API void dsv4cuda_gemv_fp4_pair_q(float* y0, float* y1, const float* qx, const float* qscale,
                                       const uint8_t* W0, const uint8_t* S0, const uint8_t* W1,
                                       const uint8_t* S1, int in, int rows) {
  float* a[1] = {y0};
  float* b[1] = {y1};
  const float* xs[1] = {qx};
  const float* ss[1] = {qscale};
  fp4_or_fp8_gemv(true, a, b, xs, ss, 1, W0, S0, W1, S1, in, rows, 1);
}
DSV4_API void dsv4cuda_gemv_fp8_q(float* y, const float* qx, const float* qscale, const uint8_t* W,
                                  const uint8_t* wscale_code, int in, int out, int round_out) {
  float* ys[1] = {y};
  const float* xs[1] = {qx};
  const float* ss[1] = {qscale};
  fp4_or_fp8_gemv(false, ys, nullptr, xs, ss, 1, W, wscale_code, nullptr, nullptr, in, out,
                  round_out);
}
DSV4_API void dsv4cuda_gemv_fp8_batch_q(float* const* y, const float* const* qx,
                                        const float* const* qscale, int batch, const uint8_t* W,
                                        const uint8_t* wscale_code, int in, int out,
                                        int round_out) {
  if (batch <= 0) return;
  batch_limit("FP8", batch);
  fp4_or_fp8_gemv(false, y, nullptr, qx, qscale, batch, W, wscale_code, nullptr, nullptr, in, out,
                  round_out);
}
DSV4_API void dsv4cuda_gemv_fp8_pair_q(float* y0, float* y1, const float* qx, const float* qscale,
                                       const uint8_t* W0, const uint8_t* S0, const uint8_t* W1,
                                       const uint8_t* S1, int in, int out) {
  float* a[1] = {y0};
  float* b[1] = {y1};
  const float* xs[1] = {qx};
  const float* ss[1] = {qscale};
  fp4_or_fp8_gemv(false, a, b, xs, ss, 1, W0, S0, W1, S1, in, out, 1);
}
DSV4_API void dsv4cuda_gemv_bf16(float* y, const float* x, const uint16_t* W, int in, int out,
                                 int round_out) {
  float* ys[1] = {y};
  const float* xs[1] = {x};
  bf16_gemv(ys, xs, 1, W, in, out, round_out);
}
DSV4_API void dsv4cuda_gemv_bf16_batch(float* const* y, const float* const* x, int batch,
                                       const uint16_t* W, int in, int out, int round_out) {
  if (batch <= 0) return;
  batch_limit("BF16", batch);
  bf16_gemv(y, x, batch, W, in, out, round_out);
}
DSV4_API void dsv4cuda_quant_fp8_codes(float* qx, float* qscale, const float* x, int n) {
  quant_codes(qx, qscale, x, n);
}

// Unprefixed drop-in names: identical signatures to the reference.
DSV4_API void dsv4_gemv_fp4_q(float* y, const float* qx, const float* qscale, const uint8_t* W,
                              const uint8_t* s, int in, int rows) {
  dsv4cuda_gemv_fp4_q(y, qx, qscale, W, s, in, rows);
}
DSV4_API void dsv4_gemv_fp4_batch_q(float* const* y, const float* const* qx,
                                    const float* const* qscale, int batch, const uint8_t* W,
                                    const uint8_t* s, int in, int rows) {
  dsv4cuda_gemv_fp4_batch_q(y, qx, qscale, batch, W, s, in, rows);
}
DSV4_API void dsv4_gemv_fp4_pair_q(float* y0, float* y1, const float* qx, const float* qscale,
                                   const uint8_t* W0, const uint8_t* S0, const uint8_t* W1,
                                   const uint8_t* S1, int in, int rows) {
  dsv4cuda_gemv_fp4_pair_q(y0, y1, qx, qscale, W0, S0, W1, S1, in, rows);
}
DSV4_API void dsv4_gemv_fp8_q(float* y, const float* qx, const float* qscale, const uint8_t* W,
                              const uint8_t* s, int in, int out, int round_out) {
  dsv4cuda_gemv_fp8_q(y, qx, qscale, W, s, in, out, round_out);
}
DSV4_API void dsv4_gemv_fp8_batch_q(float* const* y, const float* const* qx,
                                    const float* const* qscale, int batch, const uint8_t* W,
                                    const uint8_t* s, int in, int out, int round_out) {
  dsv4cuda_gemv_fp8_batch_q(y, qx, qscale, batch, W, s, in, out, round_out);
}
DSV4_API void dsv4_gemv_fp8_pair_q(float* y0, float* y1, const float* qx, const float* qscale,
                                   const uint8_t* W0, const uint8_t* S0, const uint8_t* W1,
                                   const uint8_t* S1, int in, int out) {
  dsv4cuda_gemv_fp8_pair_q(y0, y1, qx, qscale, W0, S0, W1, S1, in, out);
}
DSV4_API void dsv4_gemv_bf16(float* y, const float* x, const uint16_t* W, int in, int out,
                             int round_out) {
  dsv4cuda_gemv_bf16(y, x, W, in, out, round_out);
}
DSV4_API void dsv4_gemv_bf16_batch(float* const* y, const float* const* x, int batch,
                                   const uint16_t* W, int in, int out, int round_out) {
  dsv4cuda_gemv_bf16_batch(y, x, batch, W, in, out, round_out);
}
DSV4_API void dsv4_quant_fp8_codes(float* qx, float* qscale, const float* x, int n) {
  quant_codes(qx, qscale, x, n);
}
DSV4_API void dsv4_quant_fp8_act(float* out, float* scales, const float* x, int n) {
  quant_codes(out, scales, x, n);
}

// routed_swiglu_quant (src/dsv4/dsv4_model.c:6239, file-static in the
// reference): host pointers staged through the thread's device buffers.
DSV4_API void dsv4cuda_routed_swiglu_quant(float* y, float* qy, float* qscale, const float* gate,
                                           const float* up, int n, int limit,
                                           float route_weight) {
  g_dropin_calls[5].fetch_add(1, std::memory_order_relaxed);
  if (n <= 0) return;
  if (ensure_thread_state() != 0) { fatal_or_record("init", cudaErrorInitializationError); return; }
  cudaStream_t st = t_state.stream;
  const int nb = (n + 127) / 128;
  const size_t need = al(sizeof(float) * n) * 3 + al(sizeof(__half) * n) +
                      al(sizeof(float) * nb) + al(sizeof(float)) + 1024;
  char* base = staging(need);
  if (!base) { fatal_or_record("staging cudaMalloc", cudaErrorMemoryAllocation); return; }
  Carver cv{base};
  float* dg = cv.take<float>(n);
  float* du = cv.take<float>(n);
  float* dy = cv.take<float>(n);
  __half* dq = cv.take<__half>(n);
  float* ds = cv.take<float>(nb);
  float* dw = cv.take<float>(1);
  STAGE_CHECK(cudaMemcpyAsync(dg, gate, sizeof(float) * n, cudaMemcpyHostToDevice, st), "copy gate");
  STAGE_CHECK(cudaMemcpyAsync(du, up, sizeof(float) * n, cudaMemcpyHostToDevice, st), "copy up");
  STAGE_CHECK(cudaMemcpyAsync(dw, &route_weight, sizeof(float), cudaMemcpyHostToDevice, st),
              "copy weight");
  STAGE_CHECK(dsv4::launch_swiglu_quant(dg, du, n, 1, dw, limit, dq, ds, dy, st), "swiglu");
  std::vector<__half> hq(static_cast<size_t>(n));
  STAGE_CHECK(cudaMemcpyAsync(y, dy, sizeof(float) * n, cudaMemcpyDeviceToHost, st), "copy y");
  STAGE_CHECK(cudaMemcpyAsync(hq.data(), dq, sizeof(__half) * n, cudaMemcpyDeviceToHost, st),
              "copy qy");
  STAGE_CHECK(cudaMemcpyAsync(qscale, ds, sizeof(float) * nb, cudaMemcpyDeviceToHost, st),
              "copy qscale");
  STAGE_CHECK(cudaStreamSynchronize(st), "sync");
  for (int i = 0; i < n; ++i) qy[i] = __half2float(hq[static_cast<size_t>(i)]);
}

DSV4_API int dsv4cuda_router_scores(const float* z, float* scores, int n, void* stream) {
  if (n < 0 || (n > 0 && (!z || !scores))) {
    record_error("dsv4cuda_router_scores: bad arguments");
    return -1;
  }
  const cudaError_t e = dsv4::router_scores(z, scores, n, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    record_error("dsv4cuda_router_scores: %s", cudaGetErrorString(e));
    return -1;
  }
  return 0;
}

// Public dsv4_router (src/dsv4/dsv4_ops.c:473): stages the BF16 gate, runs
// the device router with the public numerics (separate multiply and add,
// 1/sum weights) for one token.
DSV4_API void dsv4_router(int* idx, float* wt, const float* x, const float* gate,
                          const float* bias, const int64_t* tid2eid, int token_id, int hidden,
                          int n_experts, int topk, int hash_layer, float route_scale,
                          float rms_eps) {
  g_dropin_calls[4].fetch_add(1, std::memory_order_relaxed);
  (void)rms_eps;
  if (topk <= 0) return;
  if (ensure_thread_state() != 0) { fatal_or_record("init", cudaErrorInitializationError); return; }
  cudaStream_t st = t_state.stream;
  dsv4::MoeConfig c{};
  c.hidden = hidden;
  c.moe_inter = 128;
  c.n_experts = n_experts;
  c.topk = topk;
  c.route_scale = route_scale;
  c.hash_vocab = hash_layer ? 1 : 0;
  // router-only workspace pieces: zd, zb, idx, wt, counters
  const size_t gbytes = static_cast<size_t>(n_experts) * hidden * 2;
  const size_t need = al(gbytes) + al(sizeof(float) * n_experts) + al(sizeof(float) * hidden) +
                      al(8 * topk) + 2 * al(sizeof(double) * n_experts) + al(sizeof(int) * topk) +
                      al(sizeof(float) * topk) + al(8 * sizeof(int)) + al(sizeof(int)) + 1024;
  char* base = staging(need);
  if (!base) { fatal_or_record("staging cudaMalloc", cudaErrorMemoryAllocation); return; }
  Carver cv{base};
  uint16_t* dg = cv.take<uint16_t>(static_cast<size_t>(n_experts) * hidden);
  float* db = cv.take<float>(n_experts);
  float* dx = cv.take<float>(hidden);
  int64_t* dt = cv.take<int64_t>(topk);
  dsv4::MoeWorkspace ws{};
  ws.max_tokens = 1;
  ws.zd = cv.take<double>(n_experts);
  ws.zb = cv.take<double>(n_experts);
  ws.idx = cv.take<int>(topk);
  ws.wt = cv.take<float>(topk);
  ws.counters = cv.take<int>(8);
  int* dtok = cv.take<int>(1);
  STAGE_CHECK(cudaMemcpyAsync(dg, gate, gbytes, cudaMemcpyHostToDevice, st), "copy gate");
  if (bias)
    STAGE_CHECK(cudaMemcpyAsync(db, bias, sizeof(float) * n_experts, cudaMemcpyHostToDevice, st),
                "copy bias");
  STAGE_CHECK(cudaMemcpyAsync(dx, x, sizeof(float) * hidden, cudaMemcpyHostToDevice, st), "copy x");
  const int zero = 0;
  if (hash_layer)
    STAGE_CHECK(cudaMemcpyAsync(dt, tid2eid + static_cast<size_t>(token_id) * topk,
                                sizeof(int64_t) * topk, cudaMemcpyHostToDevice, st), "copy tid2eid");
  STAGE_CHECK(cudaMemcpyAsync(dtok, &zero, sizeof(int), cudaMemcpyHostToDevice, st), "copy tok");
  STAGE_CHECK(cudaMemsetAsync(ws.counters, 0, 8 * sizeof(int), st), "memset");
  dsv4::MoeWeights w{};
  w.gate_w = dg;
  w.bias = bias ? db : nullptr;
  w.tid2eid = hash_layer ? dt : nullptr;
  STAGE_CHECK(dsv4::moe_route(c, w, ws, dx, dtok, 1, 1, st), "router");
  STAGE_CHECK(cudaMemcpyAsync(idx, ws.idx, sizeof(int) * topk, cudaMemcpyDeviceToHost, st), "copy idx");
  STAGE_CHECK(cudaMemcpyAsync(wt, ws.wt, sizeof(float) * topk, cudaMemcpyDeviceToHost, st), "copy wt");
  STAGE_CHECK(cudaStreamSynchronize(st), "sync");
}

// ---- MoE layer
DSV4_API int dsv4cuda_moe_create(dsv4cuda_moe_layer** out, const dsv4cuda_moe_config* cfg,
                                 const dsv4cuda_moe_weights* hw, int max_tokens) {
  if (!out || !hw || max_tokens <= 0) { record_error("dsv4cuda_moe_create: bad arguments"); return -1; }
  *out = nullptr;
  if (validate_cfg(cfg) != 0) return -1;
  if (!hw->gate_w || !hw->w1 || !hw->s1 || !hw->w3 || !hw->s3 || !hw->w2 || !hw->s2 ||
      (cfg->shared_kind != 0 && (!hw->sh1 || !hw->sh1s || !hw->sh3 || !hw->sh3s || !hw->sh2 ||
                                 !hw->sh2s)) ||
      (cfg->hash_vocab > 0 && !hw->tid2eid)) {
    record_error("dsv4cuda_moe_create: missing weight pointer");
    return -1;
  }
  dsv4cuda_moe_layer* L = new dsv4cuda_moe_layer();
  L->cfg = to_cfg(cfg);
  const LayerSizes s = layer_sizes(L->cfg);
  const size_t total = al(s.gate) + al(s.bias) + al(s.tid) + 2 * al(s.w13) + 2 * al(s.s13) +
                       al(s.w2) + al(s.s2) + 2 * al(s.sh13) + 2 * al(s.sh13s) + al(s.sh2) +
                       al(s.sh2s);
  cudaError_t e = cudaMalloc(&L->owned, total);
  if (e != cudaSuccess) {
    record_error("weights cudaMalloc(%zu): %s", total, cudaGetErrorString(e));
    delete L;
    return -1;
  }
  L->owned_bytes = total;
  char* p = static_cast<char*>(L->owned);
  auto put = [&](const void* src, size_t bytes) -> const void* {
    if (!src || bytes == 0) return nullptr;
    void* dst = p;
    p += al(bytes);
    if (cudaMemcpy(dst, src, bytes, cudaMemcpyHostToDevice) != cudaSuccess) e = cudaErrorUnknown;
    return dst;
  };
  L->w.gate_w = static_cast<const uint16_t*>(put(hw->gate_w, s.gate));
  L->w.bias = static_cast<const float*>(put(hw->bias, s.bias));
  L->w.tid2eid = cfg->hash_vocab > 0 ? static_cast<const int64_t*>(put(hw->tid2eid, s.tid)) : nullptr;
  L->w.w1 = static_cast<const uint8_t*>(put(hw->w1, s.w13));
  L->w.s1 = static_cast<const uint8_t*>(put(hw->s1, s.s13));
  L->w.w3 = static_cast<const uint8_t*>(put(hw->w3, s.w13));
  L->w.s3 = static_cast<const uint8_t*>(put(hw->s3, s.s13));
  L->w.w2 = static_cast<const uint8_t*>(put(hw->w2, s.w2));
  L->w.s2 = static_cast<const uint8_t*>(put(hw->s2, s.s2));
  if (cfg->shared_kind != 0) {
    L->w.sh1 = static_cast<const uint8_t*>(put(hw->sh1, s.sh13));
    L->w.sh1s = static_cast<const uint8_t*>(put(hw->sh1s, s.sh13s));
    L->w.sh3 = static_cast<const uint8_t*>(put(hw->sh3, s.sh13));
    L->w.sh3s = static_cast<const uint8_t*>(put(hw->sh3s, s.sh13s));
    L->w.sh2 = static_cast<const uint8_t*>(put(hw->sh2, s.sh2));
    L->w.sh2s = static_cast<const uint8_t*>(put(hw->sh2s, s.sh2s));
  }
  if (e != cudaSuccess || layer_finish(L, max_tokens) != 0) {
    if (e != cudaSuccess) record_error("weight upload failed");
    dsv4cuda_moe_destroy(L);
    return -1;
  }
  *out = L;
  return 0;
}

DSV4_API int dsv4cuda_moe_create_device(dsv4cuda_moe_layer** out, const dsv4cuda_moe_config* cfg,
                                        const dsv4cuda_moe_weights* dw, int max_tokens) {
  if (!out || !dw || max_tokens <= 0) { record_error("dsv4cuda_moe_create_device: bad arguments"); return -1; }
  *out = nullptr;
  if (validate_cfg(cfg) != 0) return -1;
  dsv4cuda_moe_layer* L = new dsv4cuda_moe_layer();
  L->cfg = to_cfg(cfg);
  L->w.gate_w = dw->gate_w;
  L->w.bias = dw->bias;
  L->w.tid2eid = dw->tid2eid;
  L->w.w1 = dw->w1; L->w.s1 = dw->s1; L->w.w3 = dw->w3; L->w.s3 = dw->s3;
  L->w.w2 = dw->w2; L->w.s2 = dw->s2;
  L->w.sh1 = dw->sh1; L->w.sh1s = dw->sh1s; L->w.sh3 = dw->sh3; L->w.sh3s = dw->sh3s;
  L->w.sh2 = dw->sh2; L->w.sh2s = dw->sh2s;
  if (layer_finish(L, max_tokens) != 0) {
    dsv4cuda_moe_destroy(L);
    return -1;
  }
  *out = L;
  return 0;
}

DSV4_API int dsv4cuda_moe_create_device_ep(dsv4cuda_moe_layer** out,
                                           const dsv4cuda_moe_config* cfg,
                                           const dsv4cuda_moe_weights* dw, int max_tokens,
                                           int expert_lo, int expert_hi) {
  if (!cfg || expert_lo < 0 || expert_hi <= expert_lo || expert_hi > cfg->n_experts) {
    record_error("dsv4cuda_moe_create_device_ep: expert range [%d, %d) outside [0, %d)",
                 expert_lo, expert_hi, cfg ? cfg->n_experts : 0);
    return -1;
  }
  if (dsv4cuda_moe_create_device(out, cfg, dw, max_tokens) != 0) return -1;
  (*out)->cfg.expert_lo = expert_lo;
  (*out)->cfg.expert_hi = expert_hi;
  return 0;
}

DSV4_API int dsv4cuda_moe_forward_local(dsv4cuda_moe_layer* L, const float* x,
                                        const int* token_ids, int n_tokens, void* stream) {
  if (!L || !x || n_tokens < 0 || n_tokens > L->max_tokens) {
    record_error("dsv4cuda_moe_forward_local: bad arguments");
    return -1;
  }
  if (L->cfg.hash_vocab > 0 && !token_ids) { record_error("hash layer needs token_ids"); return -1; }
  dsv4::MoeWorkspace ws = L->ws;
  if (timed_workspace(L, &ws) != 0) return -1;
  cudaError_t e = dsv4::moe_forward_local(L->cfg, L->w, ws, x, token_ids, n_tokens,
                                          static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) { record_error("moe_forward_local: %s", cudaGetErrorString(e)); return -1; }
  return 0;
}

namespace {
// moe_forward_local with the shared expert restricted to tokens [t0, t0 + n)
int forward_local_shared_range(dsv4cuda_moe_layer* L, const float* x, int n_tokens, int t0, int n,
                               void* stream) {
  dsv4::MoeWorkspace ws = L->ws;
  if (timed_workspace(L, &ws) != 0) return -1;
  dsv4::MoeExecOptions opt;
  opt.shared_t0 = t0;
  opt.shared_n = n;
  cudaError_t e = dsv4::moe_forward_local(L->cfg, L->w, ws, x, nullptr, n_tokens,
                                          static_cast<cudaStream_t>(stream), opt);
  if (e != cudaSuccess) { record_error("moe_forward_local: %s", cudaGetErrorString(e)); return -1; }
  return 0;
}
}  // namespace

DSV4_API float* dsv4cuda_moe_routed_slots(dsv4cuda_moe_layer* L) { return L ? L->ws.routed : nullptr; }

DSV4_API size_t dsv4cuda_moe_ep_buffer_bytes(const dsv4cuda_moe_layer* L) {
  return L ? dsv4::ep_exchange_bytes(L->max_tokens * L->cfg.topk, L->max_tokens, L->cfg.hidden)
           : 0;
}

DSV4_API int dsv4cuda_moe_ep_attach(dsv4cuda_moe_layer* L, int rank, int world, void* const* bufs) {
  if (!L || !bufs || world < 1 || world > dsv4::kEpMaxRanks || rank < 0 || rank >= world) {
    record_error("dsv4cuda_moe_ep_attach: bad arguments");
    return -1;
  }
  for (int r = 0; r < world; ++r) {
    if (!bufs[r] || (reinterpret_cast<uintptr_t>(bufs[r]) & 255) != 0) {
      record_error("dsv4cuda_moe_ep_attach: buffer %d missing or not 256-byte aligned", r);
      return -1;
    }
  }
  if (L->cfg.hidden % 4 != 0) {
    record_error("dsv4cuda_moe_ep_attach: hidden %% 4 != 0");
    return -1;
  }
  cudaError_t e = cudaMemset(bufs[rank], 0, dsv4cuda_moe_ep_buffer_bytes(L));
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) { record_error("ep_attach memset: %s", cudaGetErrorString(e)); return -1; }
  L->ep = dsv4::ep_exchange_make(bufs, rank, world, L->max_tokens * L->cfg.topk, L->max_tokens,
                                 L->cfg.hidden);
  L->ep_attached = true;
  return 0;
}

DSV4_API int dsv4cuda_moe_ep_push(dsv4cuda_moe_layer* L, int n_tokens, void* stream) {
  if (!L || !L->ep_attached || n_tokens < 0 || n_tokens > L->max_tokens) {
    record_error("dsv4cuda_moe_ep_push: bad arguments or no exchange attached");
    return -1;
  }
  cudaError_t e = dsv4::ep_push(L->ep, L->ws.routed, L->ws.idx, n_tokens * L->cfg.topk,
                                L->cfg.hidden, L->cfg.expert_lo, dsv4::moe_local_hi(L->cfg),
                                static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) { record_error("ep_push: %s", cudaGetErrorString(e)); return -1; }
  return 0;
}

DSV4_API int dsv4cuda_moe_ep_combine(dsv4cuda_moe_layer* L, int n_tokens, float* out, void* stream) {
  if (!L || !L->ep_attached || !out || n_tokens < 0 || n_tokens > L->max_tokens) {
    record_error("dsv4cuda_moe_ep_combine: bad arguments or no exchange attached");
    return -1;
  }
  const bool has_shared = L->cfg.shared_kind != dsv4::kSharedNone && L->w.sh1 != nullptr;
  cudaError_t e = dsv4::ep_combine(L->ep, has_shared ? L->ws.shared : nullptr, L->ws.idx,
                                   n_tokens, L->cfg.topk, L->cfg.hidden, out,
                                   dsv4::device_error_word(), static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) { record_error("ep_combine: %s", cudaGetErrorString(e)); return -1; }
  return 0;
}

DSV4_API int dsv4cuda_moe_forward_ep(dsv4cuda_moe_layer* L, const float* x, const int* token_ids,
                                     int n_tokens, float* out, void* stream) {
  if (!L || !L->ep_attached) {
    record_error("dsv4cuda_moe_forward_ep: no exchange attached");
    return -1;
  }
  if (dsv4cuda_moe_forward_local(L, x, token_ids, n_tokens, stream) != 0) return -1;
  if (dsv4cuda_moe_ep_push(L, n_tokens, stream) != 0) return -1;
  return dsv4cuda_moe_ep_combine(L, n_tokens, out, stream);
}

namespace {
int ep_tokens_check(dsv4cuda_moe_layer* L, int n_local, const char* what) {
  if (!L || !L->ep_attached || n_local <= 0 || n_local * L->ep.world > L->max_tokens) {
    record_error("%s: bad arguments (world * n_local must fit max_tokens) or no exchange "
                 "attached", what);
    return -1;
  }
  if (L->cfg.hash_vocab > 0) {
    record_error("%s: hash-routed layers need token ids; not supported", what);
    return -1;
  }
  return 0;
}
}  // namespace

DSV4_API int dsv4cuda_moe_ep_tokens_gather(dsv4cuda_moe_layer* L, const float* x_local,
                                           int n_local, void* stream) {
  if (ep_tokens_check(L, n_local, "dsv4cuda_moe_ep_tokens_gather") != 0 || !x_local) return -1;
  cudaError_t e = dsv4::ep_gather(L->ep, x_local, n_local, L->cfg.hidden,
                                  static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) { record_error("ep_gather: %s", cudaGetErrorString(e)); return -1; }
  return 0;
}

DSV4_API int dsv4cuda_moe_ep_tokens_compute(dsv4cuda_moe_layer* L, int n_local, void* stream) {
  if (ep_tokens_check(L, n_local, "dsv4cuda_moe_ep_tokens_compute") != 0) return -1;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = dsv4::ep_gather_wait(L->ep, dsv4::device_error_word(), st);
  if (e != cudaSuccess) { record_error("ep_gather_wait: %s", cudaGetErrorString(e)); return -1; }
  // every rank routes all tokens; the shared expert runs for this rank's
  // tokens only (rows rank * n_local of the shared output)
  if (forward_local_shared_range(L, L->ep.tokens[L->ep.rank], n_local * L->ep.world,
                                 L->ep.rank * n_local, n_local, stream) != 0)
    return -1;
  e = dsv4::ep_push_owner(L->ep, L->ws.routed, L->ws.idx, n_local, L->cfg.topk, L->cfg.hidden,
                          L->cfg.expert_lo, dsv4::moe_local_hi(L->cfg), st);
  if (e != cudaSuccess) { record_error("ep_push_owner: %s", cudaGetErrorString(e)); return -1; }
  return 0;
}

DSV4_API int dsv4cuda_moe_ep_tokens_combine(dsv4cuda_moe_layer* L, int n_local, float* out_local,
                                            void* stream) {
  if (ep_tokens_check(L, n_local, "dsv4cuda_moe_ep_tokens_combine") != 0 || !out_local) return -1;
  const bool has_shared = L->cfg.shared_kind != dsv4::kSharedNone && L->w.sh1 != nullptr;
  cudaError_t e = dsv4::ep_combine_owner(L->ep, has_shared ? L->ws.shared : nullptr, L->ws.idx,
                                         n_local, L->cfg.topk, L->cfg.hidden, out_local,
                                         dsv4::device_error_word(),
                                         static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) { record_error("ep_combine_owner: %s", cudaGetErrorString(e)); return -1; }
  return 0;
}

DSV4_API int dsv4cuda_moe_forward_ep_tokens(dsv4cuda_moe_layer* L, const float* x_local,
                                            int n_local, float* out_local, void* stream) {
  if (dsv4cuda_moe_ep_tokens_gather(L, x_local, n_local, stream) != 0) return -1;
  if (dsv4cuda_moe_ep_tokens_compute(L, n_local, stream) != 0) return -1;
  return dsv4cuda_moe_ep_tokens_combine(L, n_local, out_local, stream);
}

DSV4_API int dsv4cuda_ipc_alloc(size_t bytes, void** ptr, unsigned char* handle) {
  if (!ptr || !handle || bytes == 0) { record_error("dsv4cuda_ipc_alloc: bad arguments"); return -1; }
  *ptr = nullptr;
  cudaError_t e = cudaMalloc(ptr, bytes);
  if (e != cudaSuccess) { record_error("ipc cudaMalloc: %s", cudaGetErrorString(e)); return -1; }
  cudaIpcMemHandle_t h;
  e = cudaIpcGetMemHandle(&h, *ptr);
  if (e != cudaSuccess) {
    cudaFree(*ptr);
    *ptr = nullptr;
    record_error("cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
    return -1;
  }
  std::memcpy(handle, &h, sizeof(h));
  return 0;
}

DSV4_API int dsv4cuda_ipc_open(const unsigned char* handle, void** ptr) {
  if (!ptr || !handle) { record_error("dsv4cuda_ipc_open: bad arguments"); return -1; }
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) { record_error("cudaIpcOpenMemHandle: %s", cudaGetErrorString(e)); return -1; }
  return 0;
}

DSV4_API int dsv4cuda_ipc_close(void* ptr) {
  cudaError_t e = cudaIpcCloseMemHandle(ptr);
  if (e != cudaSuccess) { record_error("cudaIpcCloseMemHandle: %s", cudaGetErrorString(e)); return -1; }
  return 0;
}

DSV4_API int dsv4cuda_ipc_free(void* ptr) {
  cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess) { record_error("ipc cudaFree: %s", cudaGetErrorString(e)); return -1; }
  return 0;
}

DSV4_API int dsv4cuda_moe_combine(dsv4cuda_moe_layer* L, int n_tokens, float* out, void* stream) {
  if (!L || !out || n_tokens < 0 || n_tokens > L->max_tokens) {
    record_error("dsv4cuda_moe_combine: bad arguments");
    return -1;
  }
  cudaError_t e = dsv4::moe_combine(L->cfg, L->ws, n_tokens, out,
                                    L->cfg.shared_kind != 0 && L->w.sh1 != nullptr,
                                    static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) { record_error("moe_combine: %s", cudaGetErrorString(e)); return -1; }
  return 0;
}

DSV4_API void dsv4cuda_moe_destroy(dsv4cuda_moe_layer* L) {
  if (!L) return;
  for (cudaGraphExec_t g : L->host_graphs)
    if (g) cudaGraphExecDestroy(g);
  for (cudaEvent_t e : L->events) cudaEventDestroy(e);
  if (L->owned) cudaFree(L->owned);
  if (L->ws_mem) cudaFree(L->ws_mem);
  delete L;
}

DSV4_API size_t dsv4cuda_moe_device_bytes(const dsv4cuda_moe_layer* L) {
  return L ? L->owned_bytes + L->ws_bytes : 0;
}


DSV4_API int dsv4cuda_moe_forward(dsv4cuda_moe_layer* L, const float* x, const int* token_ids,
                                  int n_tokens, float* out, void* stream) {
  if (!L || !x || !out || n_tokens < 0) { record_error("dsv4cuda_moe_forward: bad arguments"); return -1; }
  if (n_tokens > L->max_tokens) {
    record_error("dsv4cuda_moe_forward: %d tokens exceed max_tokens %d", n_tokens, L->max_tokens);
    return -1;
  }
  if (L->cfg.hash_vocab > 0 && !token_ids) { record_error("hash layer needs token_ids"); return -1; }
  dsv4::MoeWorkspace ws = L->ws;
  if (timed_workspace(L, &ws) != 0) return -1;
  cudaError_t e = dsv4::moe_forward(L->cfg, L->w, ws, x, token_ids, n_tokens, out,
                                    static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) { record_error("moe_forward: %s", cudaGetErrorString(e)); return -1; }
  return 0;
}

DSV4_API int dsv4cuda_moe_timing_begin(dsv4cuda_moe_layer* L) {
  if (!L) return -1;
  L->timing = true;
  L->timed = 0;
  return 0;
}

DSV4_API int dsv4cuda_moe_timing_end2(dsv4cuda_moe_layer* L, int* n_forwards, float* gateup_ms,
                                      float* down_ms, float* logits_ms, float* select_ms) {
  if (!L) return -1;
  L->timing = false;
  float gu = 0.f, dn = 0.f, lg = 0.f, sl = 0.f;
  for (int i = 0; i < L->timed; ++i) {
    float a = 0.f, b = 0.f, c = 0.f, d = 0.f;
    cudaEvent_t* ev = &L->events[static_cast<size_t>(i) * 8];
    if (cudaEventSynchronize(ev[3]) != cudaSuccess ||
        cudaEventElapsedTime(&a, ev[0], ev[1]) != cudaSuccess ||
        cudaEventElapsedTime(&b, ev[2], ev[3]) != cudaSuccess ||
        cudaEventElapsedTime(&c, ev[4], ev[5]) != cudaSuccess ||
        cudaEventElapsedTime(&d, ev[5], ev[6]) != cudaSuccess) {
      record_error("timing events failed");
      return -1;
    }
    gu += a;
    dn += b;
    lg += c;
    sl += d;
  }
  if (n_forwards) *n_forwards = L->timed;
  if (gateup_ms) *gateup_ms = gu;
  if (down_ms) *down_ms = dn;
  if (logits_ms) *logits_ms = lg;
  if (select_ms) *select_ms = sl;
  L->timed = 0;
  return 0;
}

DSV4_API int dsv4cuda_moe_timing_read(dsv4cuda_moe_layer* L, int index, float* gateup_ms,
                                      float* down_ms, float* logits_ms, float* select_ms) {
  if (!L || index < 0 || index >= L->timed) { record_error("dsv4cuda_moe_timing_read: bad index"); return -1; }
  cudaEvent_t* ev = &L->events[static_cast<size_t>(index) * 8];
  float a = 0.f, b = 0.f, c = 0.f, d = 0.f;
  if (cudaEventSynchronize(ev[3]) != cudaSuccess ||
      cudaEventElapsedTime(&a, ev[0], ev[1]) != cudaSuccess ||
      cudaEventElapsedTime(&b, ev[2], ev[3]) != cudaSuccess ||
      cudaEventElapsedTime(&c, ev[4], ev[5]) != cudaSuccess ||
      cudaEventElapsedTime(&d, ev[5], ev[6]) != cudaSuccess) {
    record_error("timing events failed");
    return -1;
  }
  if (gateup_ms) *gateup_ms = a;
  if (down_ms) *down_ms = b;
  if (logits_ms) *logits_ms = c;
  if (select_ms) *select_ms = d;
  return 0;
}

DSV4_API int dsv4cuda_moe_timing_end(dsv4cuda_moe_layer* L, int* n_forwards, float* gateup_ms,
                                     float* down_ms) {
  return dsv4cuda_moe_timing_end2(L, n_forwards, gateup_ms, down_ms, nullptr, nullptr);
}

DSV4_API int dsv4cuda_moe_forward_host(dsv4cuda_moe_layer* L, const float* x, const int* token_ids,
                                       int n_tokens, float* out) {
  if (!L || !x || !out || n_tokens < 0 || n_tokens > L->max_tokens) {
    record_error("dsv4cuda_moe_forward_host: bad arguments");
    return -1;
  }
  if (ensure_thread_state() != 0) return -1;
  cudaStream_t st = t_state.stream;
  const size_t bytes = sizeof(float) * n_tokens * L->cfg.hidden;
  cudaError_t e = cudaMemcpyAsync(L->d_x, x, bytes, cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess && token_ids)
    e = cudaMemcpyAsync(L->d_tok, token_ids, sizeof(int) * n_tokens, cudaMemcpyHostToDevice, st);
  if (e != cudaSuccess) { record_error("H2D: %s", cudaGetErrorString(e)); return -1; }
  const int* dtok = L->cfg.hash_vocab > 0 ? L->d_tok : nullptr;
  if (L->host_graphs.size() < static_cast<size_t>(L->max_tokens) + 1)
    L->host_graphs.assign(static_cast<size_t>(L->max_tokens) + 1, nullptr);
  cudaGraphExec_t& ge = L->host_graphs[n_tokens];
  if (ge && !L->timing) {
    e = cudaGraphLaunch(ge, st);
    if (e != cudaSuccess) { record_error("graph launch: %s", cudaGetErrorString(e)); return -1; }
  } else {
    if (dsv4cuda_moe_forward(L, L->d_x, dtok, n_tokens, L->d_out, st) != 0) return -1;
    if (!L->timing && n_tokens > 0) {
      // capture this token count's forward for the next calls (the first,
      // ungraphed call has set up kernel attributes, streams and maps)
      cudaGraph_t g = nullptr;
      e = cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal);
      int rc = 0;
      if (e == cudaSuccess) {
        rc = dsv4cuda_moe_forward(L, L->d_x, dtok, n_tokens, L->d_out, st);
        e = cudaStreamEndCapture(st, &g);
      }
      if (e == cudaSuccess && rc == 0 && g) e = cudaGraphInstantiate(&ge, g, 0);
      if (g) cudaGraphDestroy(g);
      if (e != cudaSuccess || rc != 0) {
        ge = nullptr;  // keep running ungraphed
        cudaGetLastError();
      }
    }
  }
  e = cudaMemcpyAsync(out, L->d_out, bytes, cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) { record_error("D2H: %s", cudaGetErrorString(e)); return -1; }
  return 0;
}

DSV4_API int dsv4cuda_moe_last_routes(dsv4cuda_moe_layer* L, int n_tokens, int* idx, float* wt) {
  if (!L || n_tokens < 0 || n_tokens > L->max_tokens) { record_error("bad arguments"); return -1; }
  cudaError_t e = cudaDeviceSynchronize();
  const size_t n = static_cast<size_t>(n_tokens) * L->cfg.topk;
  if (e == cudaSuccess && idx) e = cudaMemcpy(idx, L->ws.idx, n * sizeof(int), cudaMemcpyDeviceToHost);
  if (e == cudaSuccess && wt) e = cudaMemcpy(wt, L->ws.wt, n * sizeof(float), cudaMemcpyDeviceToHost);
  int counters[4] = {0, 0, 0, 0};
  if (e == cudaSuccess) e = cudaMemcpy(counters, L->ws.counters, sizeof(counters), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) { record_error("routes: %s", cudaGetErrorString(e)); return -1; }
  return counters[2];
}

DSV4_API int dsv4cuda_moe_route(dsv4cuda_moe_layer* L, const float* x, const int* token_ids,
                                int n_tokens, int public_router, int* idx, float* wt) {
  if (!L || !x || n_tokens <= 0 || n_tokens > L->max_tokens) { record_error("bad arguments"); return -1; }
  cudaError_t e = dsv4::moe_route(L->cfg, L->w, L->ws, x, token_ids, n_tokens, public_router, 0);
  if (e != cudaSuccess) { record_error("route: %s", cudaGetErrorString(e)); return -1; }
  return dsv4cuda_moe_last_routes(L, n_tokens, idx, wt);
}

// ===================================================== allocation-free ==
//
// Some callers cannot allocate device memory at the moment they run a MoE
// layer: code inside a region where the runtime's allocator must not be
// called (a stream being captured into a CUDA graph, where cudaMalloc would
// break the capture), engines whose device memory is handed out entirely by
// their own pool and forbid any other allocation, or hosts that have to run
// with a fixed, pre-reserved memory footprint. For them,
// dsv4cuda_moe_forward_noalloc runs the same MoE layer without calling
// cudaMalloc, cudaFree or any allocating routine: its working memory is the
// file-scope array below, which exists once on every GPU that loads this
// library and stays there until the process exits.
namespace {

constexpr size_t kNoAllocScratchBytes = 4u << 20;  // 4 MiB per device
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_base[kMaxDevices] = {};  // device address of the array, per device

}  // namespace

DSV4_API int dsv4cuda_moe_forward_noalloc(const dsv4cuda_moe_config* cfg,
                                          const dsv4cuda_moe_weights* dw, const float* x,
                                          const int* token_ids, int n_tokens, float* out,
                                          void* stream) {
  if (!cfg || !dw || !x || !out || n_tokens <= 0) {
    record_error("dsv4cuda_moe_forward_noalloc: bad arguments");
    return -1;
  }
  if (validate_cfg(cfg) != 0) return -1;
  if (!dw->gate_w || !dw->w1 || !dw->s1 || !dw->w3 || !dw->s3 || !dw->w2 || !dw->s2 ||
      (cfg->shared_kind != 0 && (!dw->sh1 || !dw->sh1s || !dw->sh3 || !dw->sh3s || !dw->sh2 ||
                                 !dw->sh2s)) ||
      (cfg->hash_vocab > 0 && (!dw->tid2eid || !token_ids))) {
    record_error("dsv4cuda_moe_forward_noalloc: missing weight pointer or token ids");
    return -1;
  }
  const dsv4::MoeConfig c = to_cfg(cfg);
  const size_t ws_bytes = dsv4::moe_workspace_bytes(c, n_tokens);
  const size_t need = ws_bytes + 256;  // + the device error word
  if (need > kNoAllocScratchBytes) {
    record_error("dsv4cuda_moe_forward_noalloc: %d tokens need %zu bytes of working memory; "
                 "the allocation-free path has %zu (use dsv4cuda_moe_forward)",
                 n_tokens, need, kNoAllocScratchBytes);
    return -1;
  }
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    record_error("dsv4cuda_moe_forward_noalloc: no usable current device");
    return -1;
  }
  void* base = nullptr;
  {
    // one-time set-up per device, with that device current: the host-side
    // name of the array is not a device address, so ask the runtime for it
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_base[dev]) {
      void* p = nullptr;
      e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
      if (e != cudaSuccess || !p) {
        record_error("dsv4cuda_moe_forward_noalloc: cudaGetSymbolAddress: %s",
                     cudaGetErrorString(e));
        return -1;
      }
      g_noalloc_base[dev] = p;
    }
    base = g_noalloc_base[dev];
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  dsv4::MoeWorkspace ws{};
  dsv4::moe_workspace_carve(&ws, c, n_tokens, base);
  unsigned int* err_word = reinterpret_cast<unsigned int*>(static_cast<char*>(base) + ws_bytes);
  // the array keeps the previous call's contents: reset what must start at
  // zero (router counters, including the CTA ticket, and the error word)
  e = cudaMemsetAsync(ws.counters, 0, 8 * sizeof(int), st);
  if (e == cudaSuccess) e = cudaMemsetAsync(err_word, 0, sizeof(unsigned int), st);
  if (e != cudaSuccess) {
    record_error("dsv4cuda_moe_forward_noalloc: %s", cudaGetErrorString(e));
    return -1;
  }
  dsv4::MoeWeights w{};
  w.gate_w = dw->gate_w;
  w.bias = dw->bias;
  w.tid2eid = dw->tid2eid;
  w.w1 = dw->w1; w.s1 = dw->s1; w.w3 = dw->w3; w.s3 = dw->s3; w.w2 = dw->w2; w.s2 = dw->s2;
  w.sh1 = dw->sh1; w.sh1s = dw->sh1s; w.sh3 = dw->sh3; w.sh3s = dw->sh3s;
  w.sh2 = dw->sh2; w.sh2s = dw->sh2s;
  dsv4::MoeExecOptions opt;
  opt.single_stream = true;
  opt.map_cache = false;
  opt.err = err_word;
  e = dsv4::moe_forward(c, w, ws, x, token_ids, n_tokens, out, st, opt);
  if (e != cudaSuccess) {
    record_error("dsv4cuda_moe_forward_noalloc: %s", cudaGetErrorString(e));
    return -1;
  }
  return 0;
}

// ============================================================ attention ==

namespace {

struct AttnThreadState {
  char* ws = nullptr;
  size_t cap = 0;
  bool timing = false;
  std::vector<cudaEvent_t> events;  // pairs around the main kernel
  int timed = 0;
};
thread_local AttnThreadState t_attn;

dsv4::Fp8KvCache to_cache(const dsv4cuda_kv_cache* c) {
  dsv4::Fp8KvCache k;
  k.codes = c->codes;
  k.scales = c->scales;
  k.rope = c->rope;
  k.nope = c->nope;
  k.rope_dim = c->rope_dim;
  k.rows = c->rows;
  return k;
}

bool cache_ok(const dsv4cuda_kv_cache* c) {
  return c && c->codes && c->scales && c->rope && c->nope > 0 && c->nope % 64 == 0 &&
         c->nope / 64 <= dsv4::kKvScaleSlots && c->rope_dim >= 0 && c->rows > 0;
}

dsv4::AttnProblem make_problem(const dsv4cuda_attn_shape* s, const float* q, const float* kv,
                               const dsv4cuda_kv_cache* cache, const float* sink, const int* idx,
                               const float* rc, const float* rs, float* out) {
  dsv4::AttnProblem p;
  p.q = q;
  p.kv = kv;
  if (!kv && cache) p.cache = to_cache(cache);
  p.kv_batch_stride = s->kv_batch_stride;
  p.kv_rows = s->kv_rows;
  p.idx = idx;
  p.sink = sink;
  p.rope_cos = rc;
  p.rope_sin = rs;
  p.rope_dim = s->rope_dim;
  p.out = out;
  p.B = s->batch;
  p.H = s->heads;
  p.d = s->head_dim;
  p.n = s->n_keys;
  p.scale = s->scale;
  p.err = dsv4::device_error_word();
  return p;
}

}  // namespace

DSV4_API int dsv4cuda_kv_write(const dsv4cuda_kv_cache* cache, const float* kv,
                               const long long* rows, int n, void* stream) {
  if (!cache_ok(cache) || (n > 0 && (!kv || !rows)) || n < 0 ||
      reinterpret_cast<uintptr_t>(cache->codes) % 16 || reinterpret_cast<uintptr_t>(cache->rope) % 16 ||
      reinterpret_cast<uintptr_t>(cache->scales) % 8) {
    record_error("dsv4cuda_kv_write: bad arguments (cache codes/rope 16-byte aligned, scales 8)");
    return -1;
  }
  cudaError_t e = dsv4::kv_cache_write(to_cache(cache), kv, rows, n,
                                       static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) { record_error("dsv4cuda_kv_write: %s", cudaGetErrorString(e)); return -1; }
  return 0;
}

DSV4_API int dsv4cuda_kv_read(const dsv4cuda_kv_cache* cache, const long long* rows, int n,
                              float* out, void* stream) {
  if (!cache_ok(cache) || (n > 0 && (!out || !rows)) || n < 0) {
    record_error("dsv4cuda_kv_read: bad arguments");
    return -1;
  }
  cudaError_t e = dsv4::kv_cache_read(to_cache(cache), rows, n, out,
                                      static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) { record_error("dsv4cuda_kv_read: %s", cudaGetErrorString(e)); return -1; }
  return 0;
}

DSV4_API size_t dsv4cuda_attn_workspace_bytes(const dsv4cuda_attn_shape* shape, int use_cache) {
  if (!shape) return 0;
  dsv4::AttnProblem p = make_problem(shape, nullptr, use_cache ? nullptr : reinterpret_cast<const float*>(1),
                                     nullptr, nullptr, nullptr, nullptr, nullptr, nullptr);
  if (use_cache) {
    p.cache.nope = shape->head_dim - shape->rope_dim;
    p.cache.rope_dim = shape->rope_dim;
  }
  return dsv4::attn_workspace_bytes(p);
}

DSV4_API int dsv4cuda_sparse_attn(float* out, const float* q, const float* kv,
                                  const dsv4cuda_kv_cache* cache, const float* sink,
                                  const int* idx, const float* rope_cos, const float* rope_sin,
                                  const dsv4cuda_attn_shape* shape, void* workspace,
                                  size_t workspace_bytes, void* stream) {
  if (!shape || !out || !q || !sink || (!kv && !cache_ok(cache)) ||
      (shape->n_keys > 0 && !idx) || shape->batch < 0 || shape->heads <= 0 ||
      shape->head_dim <= 0 || shape->n_keys < 0 || ((rope_cos == nullptr) != (rope_sin == nullptr))) {
    record_error("dsv4cuda_sparse_attn: bad arguments");
    return -1;
  }
  if (!kv && cache->nope + cache->rope_dim != shape->head_dim) {
    record_error("dsv4cuda_sparse_attn: cache nope + rope_dim != head_dim");
    return -1;
  }
  if (!kv && shape->batch > 0 &&
      (shape->kv_rows < 0 || shape->kv_batch_stride < 0 ||
       static_cast<long long>(shape->batch - 1) * shape->kv_batch_stride + shape->kv_rows >
           cache->rows)) {
    record_error("dsv4cuda_sparse_attn: batch regions exceed the cache's %lld rows", cache->rows);
    return -1;
  }
  auto misaligned = [](const void* ptr, uintptr_t a) {
    return ptr && (reinterpret_cast<uintptr_t>(ptr) % a) != 0;
  };
  // the kernels move q, kv, out, the cache codes and rope values in 16-byte vectors
  if (misaligned(q, 16) || misaligned(out, 16) || misaligned(kv, 16) || misaligned(workspace, 16) ||
      (!kv && (misaligned(cache->codes, 16) || misaligned(cache->rope, 16) ||
               misaligned(cache->scales, 8)))) {
    record_error("dsv4cuda_sparse_attn: q, out, kv, workspace, cache codes and rope must be "
                 "16-byte aligned (cache scales 8-byte)");
    return -1;
  }
  dsv4::AttnProblem p = make_problem(shape, q, kv, cache, sink, idx, rope_cos, rope_sin, out);
  const size_t need = dsv4::attn_workspace_bytes(p);
  void* ws = workspace;
  if (!ws) {
    if (need > t_attn.cap) {
      if (t_attn.ws) cudaFree(t_attn.ws);
      t_attn.ws = nullptr;
      t_attn.cap = 0;
      if (cudaMalloc(&t_attn.ws, need) != cudaSuccess) {
        record_error("dsv4cuda_sparse_attn: cannot allocate %zu bytes of workspace", need);
        return -1;
      }
      t_attn.cap = need;
    }
    ws = t_attn.ws;
  } else if (workspace_bytes < need) {
    record_error("dsv4cuda_sparse_attn: workspace of %zu bytes, need %zu", workspace_bytes, need);
    return -1;
  }
  cudaEvent_t eb = nullptr, ee = nullptr;
  if (t_attn.timing) {
    const size_t i = static_cast<size_t>(t_attn.timed) * 2;
    while (t_attn.events.size() < i + 2) {
      cudaEvent_t ev;
      if (cudaEventCreate(&ev) != cudaSuccess) { record_error("event create failed"); return -1; }
      t_attn.events.push_back(ev);
    }
    eb = t_attn.events[i];
    ee = t_attn.events[i + 1];
    ++t_attn.timed;
  }
  cudaError_t e = dsv4::attn_forward(p, ws, static_cast<cudaStream_t>(stream), eb, ee);
  if (e != cudaSuccess) {
    record_error("dsv4cuda_sparse_attn: %s", cudaGetErrorString(e));
    return -1;
  }
  return 0;
}

DSV4_API int dsv4cuda_attn_timing_begin(void) {
  t_attn.timing = true;
  t_attn.timed = 0;
  return 0;
}

DSV4_API int dsv4cuda_attn_timing_end(int* n_calls, float* main_ms) {
  t_attn.timing = false;
  float total = 0.f;
  for (int i = 0; i < t_attn.timed; ++i) {
    float ms = 0.f;
    if (cudaEventSynchronize(t_attn.events[2 * i + 1]) != cudaSuccess ||
        cudaEventElapsedTime(&ms, t_attn.events[2 * i], t_attn.events[2 * i + 1]) != cudaSuccess) {
      record_error("attention timing events failed");
      return -1;
    }
    total += ms;
  }
  if (n_calls) *n_calls = t_attn.timed;
  if (main_ms) *main_ms = total;
  t_attn.timed = 0;
  return 0;
}

DSV4_API void dsv4cuda_sparse_attn_host(float* o, const float* q, const float* kv,
                                        const float* attn_sink, const int* topk_idx,
                                        int topk_total, int H, int d, float scale) {
  if (H <= 0 || d <= 0) return;
  if (ensure_thread_state() != 0) { fatal_or_record("init", cudaErrorInitializationError); return; }
  cudaStream_t st = t_state.stream;
  const int n = topk_total > 0 ? topk_total : 0;
  long long rows = 0;
  for (int t = 0; t < n; ++t) rows = std::max<long long>(rows, static_cast<long long>(topk_idx[t]) + 1);
  dsv4cuda_attn_shape s{};
  s.batch = 1;
  s.heads = H;
  s.head_dim = d;
  s.n_keys = n;
  s.scale = scale;
  s.rope_dim = 0;
  s.kv_batch_stride = 0;
  s.kv_rows = rows;
  const size_t qb = sizeof(float) * H * d, kb = sizeof(float) * static_cast<size_t>(rows) * d;
  char* base = staging(al(qb) * 2 + al(kb) + al(sizeof(float) * H) + al(sizeof(int) * (n + 1)) + 256);
  if (!base) { fatal_or_record("staging cudaMalloc", cudaErrorMemoryAllocation); return; }
  Carver cv{base};
  float* dq = cv.take<float>(static_cast<size_t>(H) * d);
  float* dout = cv.take<float>(static_cast<size_t>(H) * d);
  float* dkv = cv.take<float>(static_cast<size_t>(rows) * d + 1);
  float* dsink = cv.take<float>(H);
  int* didx = cv.take<int>(n + 1);
  STAGE_CHECK(cudaMemcpyAsync(dq, q, qb, cudaMemcpyHostToDevice, st), "copy q");
  if (kb) STAGE_CHECK(cudaMemcpyAsync(dkv, kv, kb, cudaMemcpyHostToDevice, st), "copy kv");
  STAGE_CHECK(cudaMemcpyAsync(dsink, attn_sink, sizeof(float) * H, cudaMemcpyHostToDevice, st),
              "copy sink");
  if (n) STAGE_CHECK(cudaMemcpyAsync(didx, topk_idx, sizeof(int) * n, cudaMemcpyHostToDevice, st),
                     "copy idx");
  if (dsv4cuda_sparse_attn(dout, dq, dkv, nullptr, dsink, didx, nullptr, nullptr, &s, nullptr, 0,
                           st) != 0) {
    fatal_or_record("sparse_attn", cudaErrorInvalidValue);
    return;
  }
  STAGE_CHECK(cudaMemcpyAsync(o, dout, qb, cudaMemcpyDeviceToHost, st), "copy o");
  STAGE_CHECK(cudaStreamSynchronize(st), "sync");
}

// ============================================== speculative acceptance ==

DSV4_API uint64_t dsv4cuda_rng_next(uint64_t* state) { return dsv4::rng_next_host(state); }

DSV4_API int dsv4cuda_argmax_logits(const float* logits, int vocab) {
  return vocab > 0 ? dsv4::argmax_host(logits, vocab) : 0;
}

DSV4_API int dsv4cuda_sample_top_p(const float* logits, int vocab, double temperature,
                                   double top_p, uint64_t* rng_state) {
  if (!logits || !rng_state || vocab <= 0) return -1;
  return dsv4::sample_top_p_host(logits, vocab, temperature, top_p, rng_state);
}

DSV4_API int dsv4cuda_accept_chain(const int* proposal, int proposed, const float* logits,
                                   int vocab, double temperature, double top_p,
                                   uint64_t* rng_state, int eos_id, int* tokens, int* n_commit,
                                   int* n_accepted, int* n_samples) {
  if (proposed < 0 || vocab <= 0 || !logits || !tokens || !n_commit || !n_accepted ||
      !n_samples || (proposed > 0 && !proposal) || (temperature != 0.0 && !rng_state)) {
    record_error("dsv4cuda_accept_chain: bad arguments");
    return -1;
  }
  return dsv4::accept_chain_host(proposal, proposed, logits, vocab, temperature, top_p,
                                 rng_state, eos_id, tokens, n_commit, n_accepted, n_samples);
}

DSV4_API int dsv4cuda_argmax_rows(const float* logits, int rows, int vocab, int* out,
                                  void* stream) {
  if (!logits || !out || rows < 0 || vocab <= 0) {
    record_error("dsv4cuda_argmax_rows: bad arguments");
    return -1;
  }
  cudaError_t e = dsv4::argmax_rows(logits, rows, vocab, out, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) { record_error("argmax_rows: %s", cudaGetErrorString(e)); return -1; }
  return 0;
}

DSV4_API int dsv4cuda_sample_rows(const float* logits, int rows, int vocab, double temperature,
                                  const double* uniforms, int* out, void* stream) {
  if (!logits || !out || !uniforms || rows < 0 || vocab <= 0 || !(temperature > 0.0)) {
    record_error("dsv4cuda_sample_rows: bad arguments");
    return -1;
  }
  cudaError_t e = dsv4::sample_rows(logits, rows, vocab, temperature, uniforms, out,
                                    static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) { record_error("sample_rows: %s", cudaGetErrorString(e)); return -1; }
  return 0;
}

DSV4_API int dsv4cuda_accept_device(const int* proposal, int proposed, const float* logits,
                                    int vocab, double temperature, const double* uniforms,
                                    int eos_id, int* result, void* stream) {
  if (!logits || !result || proposed < 0 || vocab <= 0 || (proposed > 0 && !proposal) ||
      (temperature != 0.0 && (!uniforms || !(temperature > 0.0)))) {
    record_error("dsv4cuda_accept_device: bad arguments");
    return -1;
  }
  cudaError_t e = dsv4::accept_device(proposal, proposed, logits, vocab, temperature, uniforms,
                                      eos_id, result, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) { record_error("accept_device: %s", cudaGetErrorString(e)); return -1; }
  return 0;
}

// ==================================================== KV-ring snapshot ==
//
// dsv4_context_snapshot_take / _restore / _commit_prefix
// (src/dsv4/dsv4_model.c:2842-3056) for the latent caches and the state
// buffers a caller registers (device memory, async on the given stream).

struct dsv4cuda_snapshot {
  int max_positions = 0;
  std::vector<dsv4::Fp8KvCache> caches;
  std::vector<long long> ring_base;   // first cache row of each ring
  std::vector<int> windows;
  std::vector<float*> states;
  std::vector<size_t> state_elems;
  void* mem = nullptr;
  std::vector<uint8_t*> pre_rows;     // per cache [max_positions][row bytes]
  std::vector<float*> pre_state;      // per state [elems]
  std::vector<float*> post_state;     // per state [max_positions][elems]
  std::vector<char> captured;         // per step
  int start = 0, n = 0;
  bool ready = false;
};

namespace {

dsv4::SnapRows ring_rows(const dsv4cuda_snapshot* s, size_t c, int first, int last) {
  dsv4::SnapRows r{};
  r.n = 0;
  for (int p = first; p < last; ++p)
    r.row[r.n++] = s->ring_base[c] + (s->start + p) % s->windows[c];
  return r;
}

}  // namespace

DSV4_API int dsv4cuda_snapshot_create(dsv4cuda_snapshot** out, int max_positions, int n_caches,
                                      const dsv4cuda_kv_cache* caches,
                                      const long long* ring_base, const int* windows,
                                      int n_states, float* const* states,
                                      const size_t* state_elems) {
  if (!out || max_positions <= 0 || max_positions > dsv4::kMaxSnapPositions || n_caches < 0 ||
      n_states < 0 || (n_caches > 0 && (!caches || !windows)) ||
      (n_states > 0 && (!states || !state_elems))) {
    record_error("dsv4cuda_snapshot_create: bad arguments (max_positions <= %d)",
                 dsv4::kMaxSnapPositions);
    return -1;
  }
  *out = nullptr;
  dsv4cuda_snapshot* s = new dsv4cuda_snapshot();
  s->max_positions = max_positions;
  size_t bytes = 0;
  for (int c = 0; c < n_caches; ++c) {
    if (!cache_ok(&caches[c]) || windows[c] < max_positions) {
      record_error("dsv4cuda_snapshot_create: cache %d invalid or window < max_positions", c);
      delete s;
      return -1;
    }
    s->caches.push_back(to_cache(&caches[c]));
    s->ring_base.push_back(ring_base ? ring_base[c] : 0);
    s->windows.push_back(windows[c]);
    bytes += al(static_cast<size_t>(max_positions) * dsv4::kv_row_bytes(s->caches.back()));
  }
  for (int i = 0; i < n_states; ++i) {
    s->states.push_back(states[i]);
    s->state_elems.push_back(state_elems[i]);
    bytes += al(state_elems[i] * sizeof(float)) * (1 + static_cast<size_t>(max_positions));
  }
  if (bytes && cudaMalloc(&s->mem, bytes) != cudaSuccess) {
    record_error("dsv4cuda_snapshot_create: cannot allocate %zu bytes", bytes);
    delete s;
    return -1;
  }
  char* p = static_cast<char*>(s->mem);
  for (size_t c = 0; c < s->caches.size(); ++c) {
    s->pre_rows.push_back(reinterpret_cast<uint8_t*>(p));
    p += al(static_cast<size_t>(max_positions) * dsv4::kv_row_bytes(s->caches[c]));
  }
  for (size_t i = 0; i < s->states.size(); ++i) {
    s->pre_state.push_back(reinterpret_cast<float*>(p));
    p += al(s->state_elems[i] * sizeof(float));
    s->post_state.push_back(reinterpret_cast<float*>(p));
    p += al(s->state_elems[i] * sizeof(float)) * max_positions;
  }
  s->captured.assign(max_positions, 0);
  *out = s;
  return 0;
}

DSV4_API void dsv4cuda_snapshot_destroy(dsv4cuda_snapshot* s) {
  if (!s) return;
  if (s->mem) cudaFree(s->mem);
  delete s;
}

DSV4_API int dsv4cuda_snapshot_take(dsv4cuda_snapshot* s, int start_position, int n_positions,
                                    void* stream) {
  if (!s || start_position < 0 || n_positions <= 0 || n_positions > s->max_positions) {
    record_error("dsv4cuda_snapshot_take: bad arguments");
    return -1;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  s->start = start_position;
  s->n = n_positions;
  for (size_t c = 0; c < s->caches.size(); ++c) {
    cudaError_t e = dsv4::kv_rows_save(s->caches[c], ring_rows(s, c, 0, n_positions),
                                       s->pre_rows[c], st);
    if (e != cudaSuccess) { record_error("snapshot take: %s", cudaGetErrorString(e)); return -1; }
  }
  for (size_t i = 0; i < s->states.size(); ++i) {
    cudaError_t e = cudaMemcpyAsync(s->pre_state[i], s->states[i], s->state_elems[i] * sizeof(float),
                                    cudaMemcpyDeviceToDevice, st);
    if (e != cudaSuccess) { record_error("snapshot take: %s", cudaGetErrorString(e)); return -1; }
  }
  std::fill(s->captured.begin(), s->captured.end(), 0);
  s->ready = true;
  return 0;
}

DSV4_API int dsv4cuda_snapshot_capture_state(dsv4cuda_snapshot* s, int step, void* stream) {
  if (!s || !s->ready || step < 0 || step >= s->n) {
    record_error("dsv4cuda_snapshot_capture_state: bad arguments");
    return -1;
  }
  for (size_t i = 0; i < s->states.size(); ++i) {
    cudaError_t e = cudaMemcpyAsync(s->post_state[i] + static_cast<size_t>(step) * s->state_elems[i],
                                    s->states[i], s->state_elems[i] * sizeof(float),
                                    cudaMemcpyDeviceToDevice, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) { record_error("capture: %s", cudaGetErrorString(e)); return -1; }
  }
  s->captured[step] = 1;
  return 0;
}

DSV4_API int dsv4cuda_snapshot_commit_prefix(dsv4cuda_snapshot* s, int n_positions,
                                             void* stream) {
  if (!s || !s->ready || n_positions <= 0 || n_positions > s->n ||
      (!s->states.empty() && !s->captured[n_positions - 1])) {
    record_error("dsv4cuda_snapshot_commit_prefix: bad arguments or state of step %d not captured",
                 n_positions - 1);
    return -1;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  for (size_t c = 0; c < s->caches.size(); ++c) {
    const int rb = dsv4::kv_row_bytes(s->caches[c]);
    cudaError_t e = dsv4::kv_rows_load(s->caches[c], ring_rows(s, c, n_positions, s->n),
                                       s->pre_rows[c] + static_cast<size_t>(n_positions) * rb, st);
    if (e != cudaSuccess) { record_error("commit: %s", cudaGetErrorString(e)); return -1; }
  }
  for (size_t i = 0; i < s->states.size(); ++i) {
    cudaError_t e = cudaMemcpyAsync(
        s->states[i], s->post_state[i] + static_cast<size_t>(n_positions - 1) * s->state_elems[i],
        s->state_elems[i] * sizeof(float), cudaMemcpyDeviceToDevice, st);
    if (e != cudaSuccess) { record_error("commit: %s", cudaGetErrorString(e)); return -1; }
  }
  s->ready = false;
  return 0;
}

DSV4_API int dsv4cuda_snapshot_restore(dsv4cuda_snapshot* s, void* stream) {
  if (!s || !s->ready) { record_error("dsv4cuda_snapshot_restore: no snapshot taken"); return -1; }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  for (size_t c = 0; c < s->caches.size(); ++c) {
    cudaError_t e = dsv4::kv_rows_load(s->caches[c], ring_rows(s, c, 0, s->n), s->pre_rows[c], st);
    if (e != cudaSuccess) { record_error("restore: %s", cudaGetErrorString(e)); return -1; }
  }
  for (size_t i = 0; i < s->states.size(); ++i) {
    cudaError_t e = cudaMemcpyAsync(s->states[i], s->pre_state[i], s->state_elems[i] * sizeof(float),
                                    cudaMemcpyDeviceToDevice, st);
    if (e != cudaSuccess) { record_error("restore: %s", cudaGetErrorString(e)); return -1; }
  }
  s->ready = false;
  return 0;
}

// ======================================================== tree verify ==
//
// A verify step over a draft tree (a chain is the tree with parents
// -1, 0, 1, ...). Node j sits at position committed + depth(j); it attends
// to the window the reference's window_topk (src/dsv4/dsv4_model.c:5073)
// gives that position, except that positions >= committed are the node's
// own ancestors (and itself), whose latents live in scratch rows
// scratch_row + ancestor (siblings share a position, so they cannot share a
// ring slot). After acceptance, dsv4cuda_kv_copy_rows moves the accepted
// path's scratch rows into their ring slots.

DSV4_API int dsv4cuda_tree_attn_indices(const int* parents, int n_nodes, int committed,
                                        int window, long long ring_base, long long scratch_row,
                                        int* idx, int row_len) {
  if (!parents || !idx || n_nodes <= 0 || n_nodes > dsv4::kMaxSnapPositions || committed < 0 ||
      window <= 0 || row_len <= 0) {
    record_error("dsv4cuda_tree_attn_indices: bad arguments");
    return -1;
  }
  std::vector<int> depth(n_nodes, 0);
  for (int j = 0; j < n_nodes; ++j) {
    const int p = parents[j];
    if (p >= j || p < -1) {
      record_error("dsv4cuda_tree_attn_indices: parents[%d] = %d (parents must precede children)", j, p);
      return -1;
    }
    depth[j] = p < 0 ? 0 : depth[p] + 1;
  }
  int longest = 0;
  for (int j = 0; j < n_nodes; ++j) {
    const int pos = committed + depth[j];
    const int first = std::max(0, pos - window + 1);  // oldest position in the window
    int* out = idx + static_cast<size_t>(j) * row_len;
    int n = 0;
    for (int q = first; q < committed; ++q) {
      if (n >= row_len) { record_error("row_len %d too small", row_len); return -1; }
      out[n++] = static_cast<int>(ring_base + q % window);
    }
    // ancestors root..j (positions committed..pos)
    int chain[dsv4::kMaxSnapPositions];
    int c = 0;
    for (int a = j; a >= 0; a = parents[a]) chain[c++] = a;
    for (int i = c - 1; i >= 0; --i) {
      if (committed + depth[chain[i]] < first) continue;  // fell out of the window
      if (n >= row_len) { record_error("row_len %d too small", row_len); return -1; }
      out[n++] = static_cast<int>(scratch_row + chain[i]);
    }
    longest = std::max(longest, n);
    for (int i = n; i < row_len; ++i) out[i] = -1;
  }
  return longest;
}

DSV4_API int dsv4cuda_kv_copy_rows(const dsv4cuda_kv_cache* cache, const long long* src_rows,
                                   const long long* dst_rows, int n, void* stream) {
  if (!cache_ok(cache) || n < 0 || n > dsv4::kMaxSnapPositions || (n > 0 && (!src_rows || !dst_rows))) {
    record_error("dsv4cuda_kv_copy_rows: bad arguments (n <= %d)", dsv4::kMaxSnapPositions);
    return -1;
  }
  dsv4::SnapRows s{}, d{};
  s.n = d.n = n;
  for (int i = 0; i < n; ++i) {
    s.row[i] = src_rows[i];
    d.row[i] = dst_rows[i];
  }
  cudaError_t e = dsv4::kv_rows_move(to_cache(cache), s, d, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) { record_error("kv_copy_rows: %s", cudaGetErrorString(e)); return -1; }
  return 0;
}
