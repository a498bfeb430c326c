// bulk.cuh - sm_100a bulk-copy (TMA engine) and mbarrier primitives.
//
// Every copy lands in the issuing CTA's own shared memory, its completion
// counted on an mbarrier in that CTA's shared memory. Every wait is bounded by %globaltimer; on timeout the kernel sets
// the device error word (read by dsv4cuda_device_error()) instead of hanging.
#pragma once
#include <cstdint>

namespace dsv4 {

// Device error word (one per device, allocated by the library; bit 0 = an
// mbarrier wait timed out). Returns the calling device's word.
unsigned int* device_error_word();

constexpr unsigned long long kWaitLimitNs = 200ull * 1000 * 1000;  // 200 ms

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long global_timer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
               : "memory");
}

// Makes initialised mbarriers visible to the async (bulk-copy) proxy.
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;"
      " selp.u32 %0, 1, 0, p; }"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait; false (and bit 0 of *err set) after kWaitLimitNs.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned int* err) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_timer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_timer_ns() - t0 > kWaitLimitNs) {
      if (err) atomicOr(err, 1u);
      return false;
    }
  }
  return true;
}

// Bulk prefetch of [src, src + bytes) into L2 (TMA engine, no completion
// tracking); src 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// global -> shared bulk copy; bytes and both addresses multiples of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

}  // namespace dsv4

#include <cuda.h>

namespace dsv4 {

// 2-D tiled TMA load of one box into this CTA's shared memory only,
// completion counted on `bar`. x is the inner (byte) coordinate
// and must be a multiple of 16 bytes; the tensor map lives in kernel
// parameter space (__grid_constant__).
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Host: encodes a 2-D uint8 tensor map over `rows` rows of `row_bytes`
// bytes (row pitch = row_bytes) with a box of box_bytes x box_rows;
// swizzle128 selects the 128-byte swizzle (box_bytes must be <= 128).
// Results are cached by their arguments unless use_cache is false. Returns false if the encoding is
// rejected (unaligned base or pitch).
bool make_tma_map_u8(CUtensorMap* out, const void* base, uint64_t row_bytes, uint64_t rows,
                     uint32_t box_bytes, uint32_t box_rows, bool swizzle128,
                     bool use_cache = true);

}  // namespace dsv4
