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
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned prev = atomicAdd(&x.ctr[1], 1u);
    if (prev == gridDim.x - 1) {
      __threadfence_system();
      x.ctr[1] = 0;
      x.ctr[0] = e;
      for (int r = 0; r < x.world; ++r)
        if (r != x.rank) st_release_sys(x.flags[r] + x.rank, e);
    }
  }
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
  const int r = threadIdx.x;
  if (r < x.world && r != x.rank) {
    const unsigned* f = x.flags[x.rank] + r;
    if (static_cast<int>(ld_acquire_sys(f) - e) < 0) {
      const unsigned long long t0 = global_timer_ns();
      while (static_cast<int>(ld_acquire_sys(f) - e) < 0) {
        if (global_timer_ns() - t0 > kWaitLimitNs) {
          if (err) atomicOr(err, kErrEpWait);
          s_ok = 0;
          break;
        }
      }
    }
  }
  __syncthreads();
  if (!s_ok) return;
  const float* slots = x.slots[x.rank] + ((e & 1u) ? x.half_floats : 0);
  const size_t n = static_cast<size_t>(n_tokens) * H;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int t = static_cast<int>(i / H);
    const int c = static_cast<int>(i % H);
    float acc = 0.0f;
    for (int k = 0; k < topk; ++k) {
      const int slot = t * topk + k;
      if (idx[slot] >= 0) acc += slots[static_cast<size_t>(slot) * H + c];
    }
    if (shared) acc += shared[i];
    out[i] = bf16_round(acc);
  }
}

}  // namespace

size_t ep_exchange_bytes(int slot_cap, int H) {
  return 512 + 2 * static_cast<size_t>(slot_cap) * H * sizeof(float);
}

EpExchange ep_exchange_make(void* const* bufs, int rank, int world, int slot_cap, int H) {
  EpExchange x;
  for (int r = 0; r < kEpMaxRanks; ++r) {
    x.slots[r] = nullptr;
    x.flags[r] = nullptr;
  }
  for (int r = 0; r < world; ++r) {
    char* b = static_cast<char*>(bufs[r]);
    x.flags[r] = reinterpret_cast<unsigned*>(b);
    x.slots[r] = reinterpret_cast<float*>(b + 512);
  }
  x.ctr = reinterpret_cast<unsigned*>(static_cast<char*>(bufs[rank]) + 256);
  x.rank = rank;
  x.world = world;
  x.half_floats = static_cast<size_t>(slot_cap) * H;
  return x;
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
