// ep.cu - expert-parallel slot exchange over peer memory (see ep.cuh).
//
// Reference: the combine of moe_forward (src/dsv4/dsv4_model.c:6795-6805)
// sums the routed outputs in ascending expert order and adds the shared
// expert; expert parallelism has no reference counterpart (one host).
#include <algorithm>

#include "bulk.cuh"
#include "dsv4_common.cuh"
#include "ep.cuh"
#include "launch.cuh"

namespace dsv4 {
namespace {

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Bounded wait of thread r < world (r != rank) for flag array f's entry r to
// reach epoch e; clears *ok on timeout.
__device__ __forceinline__ void wait_peer_epochs(const EpExchange& x, const unsigned* f,
                                                 unsigned e, unsigned* err, int* ok) {
  const int r = threadIdx.x;
  if (r >= x.world || r == x.rank) return;
  const unsigned* p = f + r;
  if (static_cast<int>(ld_acquire_sys(p) - e) >= 0) return;
  const unsigned long long t0 = global_timer_ns();
  while (static_cast<int>(ld_acquire_sys(p) - e) < 0) {
    if (global_timer_ns() - t0 > kWaitLimitNs) {
      if (err) atomicOr(err, kErrEpWait);
      *ok = 0;
      return;
    }
  }
}

// Last-CTA publication of epoch e into flag arrays `which` (0 = slot flags,
// 1 = token flags) of every peer; `bump` also stores e as this rank's epoch.
__device__ __forceinline__ void publish_epoch(const EpExchange& x, unsigned e, int which,
                                              bool bump) {
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x != 0) return;
  const unsigned prev = atomicAdd(&x.ctr[1], 1u);
  if (prev != gridDim.x - 1) return;
  __threadfence_system();
  x.ctr[1] = 0;
  if (bump) x.ctr[0] = e;
  for (int r = 0; r < x.world; ++r)
    if (r != x.rank) st_release_sys((which ? x.gflags[r] : x.flags[r]) + x.rank, e);
}

// One CTA per slot (grid-stride): copy the slot's H floats to every rank.
// The last CTA to finish publishes the epoch: every CTA fences its stores at
// system scope before counting itself done, the last one fences again and
// release-stores the epoch into each peer's flag array.
__global__ void __launch_bounds__(256) ep_push_kernel(EpExchange x, const float* __restrict__ routed,
                                                      const int* __restrict__ idx, int n_slots,
                                                      int H, int lo, int hi) {
  pdl_wait();
  pdl_trigger();
  const unsigned e = *reinterpret_cast<volatile unsigned*>(&x.ctr[0]) + 1u;
  const size_t half = (e & 1u) ? x.half_floats : 0;
  for (int slot = blockIdx.x; slot < n_slots; slot += gridDim.x) {
    const int ex = idx[slot];
    if (ex < lo || ex >= hi) continue;
    const float4* src = reinterpret_cast<const float4*>(routed + static_cast<size_t>(slot) * H);
    for (int r = 0; r < x.world; ++r) {
      float4* dst = reinterpret_cast<float4*>(x.slots[r] + half + static_cast<size_t>(slot) * H);
      for (int i = threadIdx.x; i < H / 4; i += blockDim.x) dst[i] = src[i];
    }
  }
  publish_epoch(x, e, 0, true);
}

// Thread r < world waits for rank r's epoch (bounded); then the combine of
// moe_combine_kernel over the current half.
__global__ void __launch_bounds__(256) ep_combine_kernel(EpExchange x, const float* __restrict__ shared,
                                                         const int* __restrict__ idx, int n_tokens,
                                                         int topk, int H, float* __restrict__ out,
                                                         unsigned* err) {
  pdl_wait();
  pdl_trigger();
  __shared__ int s_ok;
  const unsigned e = *reinterpret_cast<volatile unsigned*>(&x.ctr[0]);
  if (threadIdx.x == 0) s_ok = 1;
  __syncthreads();
  wait_peer_epochs(x, x.flags[x.rank], e, err, &s_ok);
  __syncthreads();
  if (!s_ok) return;
  const float* slots = x.slots[x.rank] + ((e & 1u) ? x.half_floats : 0);
  const size_t n = static_cast<size_t>(n_tokens) * H;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int t = static_cast<int>(i / H);
    const int c = static_cast<int>(i % H);
    float acc = sum_routes(idx + t * topk, slots + static_cast<size_t>(t) * topk * H + c, H,
                           topk);
    if (shared) acc += shared[i];
    out[i] = bf16_round(acc);
  }
}

// This rank's n_local token rows into every rank's token buffer.
__global__ void __launch_bounds__(256) ep_gather_kernel(EpExchange x, const float* __restrict__ xl,
                                                        int n_local, int H) {
  pdl_wait();
  pdl_trigger();
  const unsigned e = *reinterpret_cast<volatile unsigned*>(&x.ctr[0]) + 1u;
  const size_t n4 = static_cast<size_t>(n_local) * H / 4;
  const float4* src = reinterpret_cast<const float4*>(xl);
  const size_t off = static_cast<size_t>(x.rank) * n_local * H / 4;
  for (int r = 0; r < x.world; ++r) {
    float4* dst = reinterpret_cast<float4*>(x.tokens[r]) + off;
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n4;
         i += static_cast<size_t>(gridDim.x) * blockDim.x)
      dst[i] = src[i];
  }
  publish_epoch(x, e, 1, true);
}

__global__ void ep_gather_wait_kernel(EpExchange x, unsigned* err) {
  pdl_wait();
  pdl_trigger();
  __shared__ int s_ok;
  if (threadIdx.x == 0) s_ok = 1;
  __syncthreads();
  const unsigned e = *reinterpret_cast<volatile unsigned*>(&x.ctr[0]);
  wait_peer_epochs(x, x.gflags[x.rank], e, err, &s_ok);
}

// Slots of local experts to the token's owner only.
__global__ void __launch_bounds__(256) ep_push_owner_kernel(EpExchange x, const float* __restrict__ routed,
                                                            const int* __restrict__ idx,
                                                            int n_local, int topk, int H, int lo,
                                                            int hi) {
  pdl_wait();
  pdl_trigger();
  const unsigned e = *reinterpret_cast<volatile unsigned*>(&x.ctr[0]);
  const size_t half = (e & 1u) ? x.half_floats : 0;
  const int n_slots = x.world * n_local * topk;
  for (int slot = blockIdx.x; slot < n_slots; slot += gridDim.x) {
    const int ex = idx[slot];
    if (ex < lo || ex >= hi) continue;
    const int t = slot / topk, k = slot - t * topk;
    const int owner = t / n_local, tl = t - owner * n_local;
    const float4* src = reinterpret_cast<const float4*>(routed + static_cast<size_t>(slot) * H);
    float4* dst = reinterpret_cast<float4*>(x.slots[owner] + half +
                                            static_cast<size_t>(tl * topk + k) * H);
    for (int i = threadIdx.x; i < H / 4; i += blockDim.x) dst[i] = src[i];
  }
  publish_epoch(x, e, 0, false);
}

__global__ void __launch_bounds__(256) ep_combine_owner_kernel(EpExchange x, const float* __restrict__ shared,
                                                               const int* __restrict__ idx,
                                                               int n_local, int topk, int H,
                                                               float* __restrict__ out,
                                                               unsigned* err) {
  pdl_wait();
  pdl_trigger();
  __shared__ int s_ok;
  const unsigned e = *reinterpret_cast<volatile unsigned*>(&x.ctr[0]);
  if (threadIdx.x == 0) s_ok = 1;
  __syncthreads();
  wait_peer_epochs(x, x.flags[x.rank], e, err, &s_ok);
  __syncthreads();
  if (!s_ok) return;
  const float* slots = x.slots[x.rank] + ((e & 1u) ? x.half_floats : 0);
  const int t0 = x.rank * n_local;
  const size_t n = static_cast<size_t>(n_local) * H;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int tl = static_cast<int>(i / H);
    const int c = static_cast<int>(i % H);
    float acc = sum_routes(idx + (t0 + tl) * topk,
                           slots + static_cast<size_t>(tl) * topk * H + c, H, topk);
    if (shared) acc += shared[static_cast<size_t>(t0) * H + i];
    out[i] = bf16_round(acc);
  }
}

}  // namespace

size_t ep_exchange_bytes(int slot_cap, int tok_cap, int H) {
  return 512 + (2 * static_cast<size_t>(slot_cap) + tok_cap) * H * sizeof(float);
}

EpExchange ep_exchange_make(void* const* bufs, int rank, int world, int slot_cap, int tok_cap,
                            int H) {
  EpExchange x;
  for (int r = 0; r < kEpMaxRanks; ++r) {
    x.slots[r] = nullptr;
    x.tokens[r] = nullptr;
    x.flags[r] = nullptr;
    x.gflags[r] = nullptr;
  }
  for (int r = 0; r < world; ++r) {
    char* b = static_cast<char*>(bufs[r]);
    x.flags[r] = reinterpret_cast<unsigned*>(b);
    x.gflags[r] = reinterpret_cast<unsigned*>(b + 64);
    x.slots[r] = reinterpret_cast<float*>(b + 512);
    x.tokens[r] = x.slots[r] + 2 * static_cast<size_t>(slot_cap) * H;
  }
  (void)tok_cap;
  x.ctr = reinterpret_cast<unsigned*>(static_cast<char*>(bufs[rank]) + 256);
  x.rank = rank;
  x.world = world;
  x.half_floats = static_cast<size_t>(slot_cap) * H;
  return x;
}

cudaError_t ep_gather(const EpExchange& x, const float* x_local, int n_local, int H,
                      cudaStream_t st) {
  if (n_local <= 0 || H % 4 != 0) return cudaErrorInvalidValue;
  const size_t n4 = static_cast<size_t>(n_local) * H / 4;
  const int grid = static_cast<int>(std::min<size_t>((n4 + 255) / 256, 148));
  return launch_pdl(ep_gather_kernel, dim3(grid), dim3(256), 0, st, x, x_local, n_local, H);
}

cudaError_t ep_gather_wait(const EpExchange& x, unsigned* err, cudaStream_t st) {
  return launch_pdl(ep_gather_wait_kernel, dim3(1), dim3(32), 0, st, x, err);
}

cudaError_t ep_push_owner(const EpExchange& x, const float* routed, const int* idx, int n_local,
                          int topk, int H, int lo, int hi, cudaStream_t st) {
  if (n_local <= 0 || H % 4 != 0) return cudaErrorInvalidValue;
  const int grid = std::min(x.world * n_local * topk, 148);
  return launch_pdl(ep_push_owner_kernel, dim3(grid), dim3(256), 0, st, x, routed, idx, n_local,
                    topk, H, lo, hi);
}

cudaError_t ep_combine_owner(const EpExchange& x, const float* shared, const int* idx,
                             int n_local, int topk, int H, float* out, unsigned* err,
                             cudaStream_t st) {
  if (n_local <= 0) return cudaSuccess;
  const size_t n = static_cast<size_t>(n_local) * H;
  const int grid = static_cast<int>(std::min<size_t>((n + 255) / 256, 2048));
  return launch_pdl(ep_combine_owner_kernel, dim3(grid), dim3(256), 0, st, x, shared, idx,
                    n_local, topk, H, out, err);
}

cudaError_t ep_push(const EpExchange& x, const float* routed, const int* idx, int n_slots, int H,
                    int lo, int hi, cudaStream_t st) {
  if (n_slots <= 0) return cudaSuccess;
  if (H % 4 != 0) return cudaErrorInvalidValue;
  const int grid = std::min(n_slots, 148);
  return launch_pdl(ep_push_kernel, dim3(grid), dim3(256), 0, st, x, routed, idx, n_slots, H, lo,
                    hi);
}

cudaError_t ep_combine(const EpExchange& x, const float* shared, const int* idx, int n_tokens,
                       int topk, int H, float* out, unsigned* err, cudaStream_t st) {
  if (n_tokens <= 0) return cudaSuccess;
  const size_t n = static_cast<size_t>(n_tokens) * H;
  const int grid = static_cast<int>(std::min<size_t>((n + 255) / 256, 2048));
  return launch_pdl(ep_combine_kernel, dim3(grid), dim3(256), 0, st, x, shared, idx, n_tokens,
                    topk, H, out, err);
}

}  // namespace dsv4
